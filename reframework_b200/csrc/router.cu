// K1 — router: logits GEMM, then softmax + top-k + renormalisation per token.
//
// Restates FusedMoE.route (reframework/moe/moe_layer.py:320-344) and
// torch_fused_topk (reframework/moe/fused.py:32-46) for the GPU:
//   logits = x . gate^T (fp32 accumulate, optionally rounded to the layer
//   dtype and/or biased), p = softmax(logits) in fp32, top-k of p (descending,
//   ties to the lower expert id), w = p / sum(top-k p) when renormalising.
//
// Two launches.  The logits come from one of:
//   the tensor cores (gemm_tc.cu, dense fp32-output mode) when x and the gate
//       share a 16-bit dtype and a shared gate, if any, is the row right after
//       the gate's E rows: one tile per (128 tokens, 256-wide slice of H), each
//       slice's logits a fixed sequence of MMAs written as fp32 partials of
//       round_up(E', 4) columns (independent of T; a decode batch still gets a
//       CTA per slice);
//   router_logits_kernel  otherwise (fp32 layers): a tiled CUDA-core GEMM.
//       A block computes a tile of TT tokens x ET experts over one 256-wide
//       slice of H (the slices give parallelism when there are few tokens);
//       x and gate chunks are staged
//       in shared memory as fp32, so each gate element is read once per tile
//       of TT tokens instead of once per token.  Each output is a sequential
//       fp32 FMA chain over its slice; slices go to a partials buffer.  The
//       slicing depends on H only, so a token's logits are the same bits
//       whatever T is (a token-sharded expert-parallel layer routes exactly
//       like the single-GPU layer).
//   router_topk_kernel    one warp per token: sums the slice partials in slice
//       order (deterministic), applies rounding / bias, softmax, top-k,
//       renormalisation or the entropy-adaptive rule, writes weights and ids.
// The shared-expert gate (sigmoid(x . w_s)) is one more "expert" column.
#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int THREADS = 256;
constexpr int SLICE = 256;     // H elements per slice: fixed, so the sum order never depends on T
constexpr int KMAX = 16;

__device__ __forceinline__ float round_dt(int dtype, float v) {
  if (dtype == RF_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == RF_F16) return __half2float(__float2half_rn(v));
  return v;
}

struct LogitsArgs {
  const void *x;
  const void *gate;
  const void *shared_gate;
  float *partial;  // [slices][T][Ec]
  int64_t T;
  int H, E, Ec;    // Ec = E (+1 with a shared gate)
};

// 8 consecutive elements of T held raw in registers (16 B, or 32 B for fp32).
template <typename T> struct Raw8 {
  uint4 v[sizeof(T) == 4 ? 2 : 1];
};

template <typename T>
__device__ __forceinline__ void fetch8(const T *p, bool ok, Raw8<T> &r) {
  const uint4 *q = reinterpret_cast<const uint4 *>(p);
#pragma unroll
  for (int i = 0; i < (int)(sizeof(r.v) / sizeof(uint4)); ++i)
    r.v[i] = ok ? __ldg(q + i) : make_uint4(0u, 0u, 0u, 0u);
}

template <typename T>
__device__ __forceinline__ void unpack8(const Raw8<T> &r, float *f) {
  if constexpr (sizeof(T) == 4) {
    rf::unpack16<float>(r.v[0], f);
    rf::unpack16<float>(r.v[1], f + 4);
  } else {
    rf::unpack16<T>(r.v[0], f);
  }
}

// Column of token `tok` in k-row `k` of the staged x chunk.  Groups of four
// tokens are XOR-swizzled by the 8-row band of k, so the transposing stores
// of a warp (8 tokens x 4 bands) land in 32 distinct banks while the float4 /
// float2 / scalar reads of the multiply stay conflict-free.
__device__ __forceinline__ int xcol(int k, int tok) {
  return (((tok >> 2) ^ (((k >> 3) & 3) << 1)) << 2) | (tok & 3);
}

// Block = TT tokens x ET experts x one SLICE of H.  Thread (tg, eg) owns the
// TM tokens tg*TM.. and the 8 experts eg*4..eg*4+3, ET/2+eg*4..ET/2+eg*4+3
// (a register tile: per k, one x read and two float4 gate reads feed 8*TM
// FMAs).  The chunk k0+KC is fetched into registers while chunk k0 is
// multiplied from shared memory; KC = 64 for the narrow tile used with few
// tokens (fewer, larger round trips), 32 otherwise.  Each output is one fp32
// FMA chain over its slice in ascending k, whatever the tile shape, KC or T
// (a chunk past the slice end adds exact zeros).
template <typename TX, typename TG, int ET, int TM, int KC>
__global__ void __launch_bounds__(THREADS) router_logits_kernel(LogitsArgs a) {
  constexpr int EGRP = ET / 8;
  constexpr int TT = TM * THREADS / EGRP;  // tokens per tile
  static_assert(TT % 32 == 0 && TT <= 256, "token tile");
  constexpr int PIECES = KC / 8;
  constexpr int XV = (TT * PIECES + THREADS - 1) / THREADS;
  constexpr int GV = (ET * PIECES + THREADS - 1) / THREADS;
  __shared__ __align__(16) float xs[KC][TT];
  __shared__ __align__(16) float gs[KC][ET];
  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * TT;
  const int e0 = blockIdx.y * ET;
  const int z = blockIdx.z;
  const int k_begin = z * SLICE;
  const int k_end = min(a.H, k_begin + SLICE);
  const TX *x = reinterpret_cast<const TX *>(a.x);
  const TG *gate = reinterpret_cast<const TG *>(a.gate);
  const TG *sgate = reinterpret_cast<const TG *>(a.shared_gate);
  const int eg = tid % EGRP, tg = tid / EGRP;
  Raw8<TX> rx[XV];
  Raw8<TG> rg[GV];

  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < XV; ++i) {
      const int v = tid + i * THREADS;
      const int tok = v / PIECES, k = k0 + (v % PIECES) * 8;
      const int64_t t = t0 + tok;
      const bool ok = v < TT * PIECES && t < a.T && k < k_end;
      fetch8<TX>(ok ? x + t * a.H + k : x, ok, rx[i]);
    }
#pragma unroll
    for (int i = 0; i < GV; ++i) {
      const int v = tid + i * THREADS;
      const int e = e0 + v / PIECES, k = k0 + (v % PIECES) * 8;
      const bool ok = v < ET * PIECES && e < a.Ec && k < k_end;
      const TG *row = (e < a.E) ? gate + (int64_t)e * a.H : sgate;
      fetch8<TG>(ok ? row + k : gate, ok, rg[i]);
    }
  };
  auto stage = [&]() {
#pragma unroll
    for (int i = 0; i < XV; ++i) {
      const int v = tid + i * THREADS;
      if (v < TT * PIECES) {
        float f[8];
        unpack8<TX>(rx[i], f);
        const int tok = v / PIECES, kb = (v % PIECES) * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) xs[kb + j][xcol(kb + j, tok)] = f[j];
      }
    }
#pragma unroll
    for (int i = 0; i < GV; ++i) {
      const int v = tid + i * THREADS;
      if (v < ET * PIECES) {
        float f[8];
        unpack8<TG>(rg[i], f);
        const int er = v / PIECES, kb = (v % PIECES) * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) gs[kb + j][er] = f[j];
      }
    }
  };

  float acc[TM][8];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  fetch(k_begin);
  for (int k0 = k_begin; k0 < k_end; k0 += KC) {
    stage();
    __syncthreads();
    if (k0 + KC < k_end) fetch(k0 + KC);
#pragma unroll 4
    for (int k = 0; k < KC; ++k) {
      float xv[TM];
      const float *xr = &xs[k][xcol(k, tg * TM)];
      if constexpr (TM == 4) {
        const float4 q = *reinterpret_cast<const float4 *>(xr);
        xv[0] = q.x; xv[1] = q.y; xv[2] = q.z; xv[3] = q.w;
      } else if constexpr (TM == 2) {
        const float2 q = *reinterpret_cast<const float2 *>(xr);
        xv[0] = q.x; xv[1] = q.y;
      } else {
        xv[0] = *xr;
      }
      const float4 ga = *reinterpret_cast<const float4 *>(&gs[k][eg * 4]);
      const float4 gb = *reinterpret_cast<const float4 *>(&gs[k][ET / 2 + eg * 4]);
      const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(xv[i], gv[j], acc[i][j]);
    }
    __syncthreads();
  }
  float *out = a.partial + (int64_t)z * a.T * a.Ec;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t t = t0 + tg * TM + i;
    if (t >= a.T) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + (j < 4 ? eg * 4 + j : ET / 2 + eg * 4 + (j - 4));
      if (e < a.Ec) out[t * a.Ec + e] = acc[i][j];
    }
  }
}

struct TopkArgs {
  const float *partial;  // [splits][T][ld] fp32 partial logits (columns E.. include the shared gate)
  const void *x_logits;  // gate == NULL: x holds the [T,E] logits
  int x_dtype;
  const float *bias;
  float *shared_scale;
  float *topk_w;
  int32_t *ids32;
  int64_t *ids64;
  float *logits_out;
  int64_t T;
  int E, Ec, K, ksplit;
  int64_t ld;            // row stride of partial (>= Ec)
  int has_shared;
  int renormalize, round_dtype, entropy_k_min;
};

template <typename TX>
__device__ __forceinline__ float load_logit(const TopkArgs &a, int64_t t, int e) {
  return rf::Cvt<TX>::to_f(reinterpret_cast<const TX *>(a.x_logits)[t * a.E + e]);
}

constexpr int TK_WARPS = 8;

// 0 + p[0] + p[stride] + ... in slice order, eight loads in flight at a time.
__device__ __forceinline__ float sum_slices(const float *p, int64_t stride, int n) {
  float v = 0.f;
  int z = 0;
  for (; z + 8 <= n; z += 8) {
    float q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = p[(int64_t)(z + i) * stride];
#pragma unroll
    for (int i = 0; i < 8; ++i) v += q[i];
  }
  for (; z < n; ++z) v += p[(int64_t)z * stride];
  return v;
}

template <typename TX>
__global__ void __launch_bounds__(TK_WARPS * 32) router_topk_kernel(TopkArgs a) {
  extern __shared__ float s_lg[];  // [TK_WARPS][E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *lg = s_lg + warp * a.E;
  const int64_t nwarps = (int64_t)gridDim.x * TK_WARPS;
  for (int64_t t = (int64_t)blockIdx.x * TK_WARPS + warp; t < a.T; t += nwarps) {
    // ---- logits: slice partials summed in slice order, rounding, bias
    float m = -INFINITY;
    for (int e = lane; e < a.E; e += 32) {
      float v;
      if (a.partial) {
        v = sum_slices(a.partial + t * a.ld + e, a.T * a.ld, a.ksplit);
      } else {
        v = load_logit<TX>(a, t, e);
      }
      if (a.round_dtype >= 0) v = round_dt(a.round_dtype, v);
      if (a.bias) {
        v += a.bias[e];
        if (a.round_dtype >= 0) v = round_dt(a.round_dtype, v);
      }
      lg[e] = v;
      if (a.logits_out) a.logits_out[t * a.E + e] = v;
      m = fmaxf(m, v);
    }
    if (a.has_shared && lane == 0) {
      const float z = sum_slices(a.partial + t * a.ld + a.E, a.T * a.ld, a.ksplit);
      a.shared_scale[t] = 1.0f / (1.0f + expf(-z));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncwarp();
    // ---- softmax statistics
    float s = 0.f;
    for (int e = lane; e < a.E; e += 32) s += expf(lg[e] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.0f / s;
    float ent = 0.f;
    for (int e = lane; e < a.E; e += 32) {
      const float p = expf(lg[e] - m) * inv;
      lg[e] = p;
      if (a.entropy_k_min > 0) ent -= p * logf(fmaxf(p, 1e-9f));
    }
    if (a.entropy_k_min > 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ent += __shfl_xor_sync(0xffffffffu, ent, o);
    }
    __syncwarp();
    // ---- top-k by probability, ties to the lower id; lane k keeps choice k
    float my_p = 0.f;
    int my_i = 0;
    float psum = 0.f;
    for (int k = 0; k < a.K; ++k) {
      float best = -1.f;
      int bi = 0x7fffffff;
      for (int e = lane; e < a.E; e += 32) {
        const float p = lg[e];
        if (p > best) { best = p; bi = e; }  // ascending ids per lane: strict '>' keeps the lowest
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
      if (bi < 0 || bi >= a.E) {  // only reachable with NaN logits
        rf_report(RF_DEV_BAD_EXPERT_ID);
        bi = 0;
        best = 0.f;
      }
      if (lane == k) { my_p = best; my_i = bi; }
      psum += best;
      __syncwarp();
      if (lane == (bi & 31)) lg[bi] = -2.f;  // taken
      __syncwarp();
    }
    // ---- weights
    float w = my_p;
    if (a.entropy_k_min > 0) {
      const float hn = ent / logf((float)a.E);
      int kd = (int)rintf((float)a.entropy_k_min + (float)(a.K - a.entropy_k_min) * hn);
      kd = min(max(kd, a.entropy_k_min), a.K);
      float kept = (lane < kd) ? my_p : 0.f;
      float sum = 0.f;  // in choice order k = 0..K-1
      for (int k = 0; k < a.K; ++k) sum += __shfl_sync(0xffffffffu, kept, k);
      w = kept / fmaxf(sum, 1e-9f);
    } else if (a.renormalize) {
      float sum = 0.f;
      for (int k = 0; k < a.K; ++k) sum += __shfl_sync(0xffffffffu, my_p, k);
      w = my_p / sum;
    }
    (void)psum;
    if (lane < a.K) {
      a.topk_w[t * a.K + lane] = w;
      if (a.ids32) a.ids32[t * a.K + lane] = my_i;
      if (a.ids64) a.ids64[t * a.K + lane] = my_i;
    }
    __syncwarp();
  }
}

struct Plan {
  int64_t ttiles;
  int et, tm, etiles, slices;
};

// The tiling depends on T; the slices (and so every sum's order) only on H.
Plan make_plan(int64_t T, int H, int Ec) {
  Plan p;
  p.et = Ec <= 8 ? 8 : Ec <= 16 ? 16 : Ec <= 32 ? 32 : 64;
  p.tm = p.et == 8 ? 1 : p.et == 16 ? 2 : 4;
  p.etiles = (Ec + p.et - 1) / p.et;
  p.slices = (H + SLICE - 1) / SLICE;
  if (p.et == 64) {  // few tokens: narrower token tiles for more blocks
    const int64_t tiles = (T + 127) / 128 * p.etiles * p.slices;
    if (tiles < 2 * rf::num_sms()) p.tm = 1;
  }
  const int tt = p.tm * THREADS / (p.et / 8);
  p.ttiles = (T + tt - 1) / tt;
  return p;
}

template <typename TX, typename TG>
void launch_logits(const LogitsArgs &a, const Plan &p, cudaStream_t st) {
  dim3 grid((unsigned)p.ttiles, p.etiles, p.slices);
  if (p.et == 8) router_logits_kernel<TX, TG, 8, 1, 32><<<grid, THREADS, 0, st>>>(a);
  else if (p.et == 16) router_logits_kernel<TX, TG, 16, 2, 32><<<grid, THREADS, 0, st>>>(a);
  else if (p.et == 32) router_logits_kernel<TX, TG, 32, 4, 32><<<grid, THREADS, 0, st>>>(a);
  else if (p.tm == 4) router_logits_kernel<TX, TG, 64, 4, 32><<<grid, THREADS, 0, st>>>(a);
  else router_logits_kernel<TX, TG, 64, 1, 64><<<grid, THREADS, 0, st>>>(a);
}

template <typename TX>
void launch_logits_tg(const LogitsArgs &a, const Plan &p, int gate_dtype, cudaStream_t st) {
  switch (gate_dtype) {
    case RF_F32: launch_logits<TX, float>(a, p, st); break;
    case RF_F16: launch_logits<TX, __half>(a, p, st); break;
    default: launch_logits<TX, __nv_bfloat16>(a, p, st); break;
  }
}

}  // namespace

extern "C" size_t rf_moe_router_workspace_size(int64_t T, int64_t H, int64_t E, int has_shared_gate) {
  if (T <= 0 || H <= 0 || E <= 0) return 256;
  const int64_t Ec = E + (has_shared_gate ? 1 : 0);
  const size_t slices = (size_t)((H + SLICE - 1) / SLICE);
  // per-slice partials: [slices][T][Ec] on CUDA cores, [slices][T][round_up(Ec, 4)]
  // on the tensor cores
  return slices * (size_t)T * (size_t)((Ec + 3) / 4 * 4) * sizeof(float) + 256;
}

extern "C" int rf_moe_router_topk(const void *x, int x_dtype, const void *gate, int gate_dtype,
                                  const float *bias, int64_t T, int64_t H, int64_t E, int64_t K,
                                  int renormalize, int round_dtype, int entropy_k_min,
                                  const void *shared_gate, float *shared_scale,
                                  float *topk_weights, int32_t *topk_ids32, int64_t *topk_ids64,
                                  float *logits, void *workspace, size_t workspace_bytes,
                                  rf_stream_t stream) {
  RF_CHECK_ARG(rf::valid_dtype(x_dtype) && rf::valid_dtype(gate_dtype),
               "rf_moe_router_topk: unknown dtype");
  RF_CHECK_ARG(round_dtype < 0 || rf::valid_dtype(round_dtype), "rf_moe_router_topk: bad round_dtype");
  RF_CHECK_ARG(T >= 0 && H > 0 && E > 0, "rf_moe_router_topk: sizes must be positive");
  RF_CHECK_ARG(E <= 1024, "rf_moe_router_topk: at most 1024 experts");
  RF_CHECK_ARG(K >= 1 && K <= E && K <= KMAX, "rf_moe_router_topk: need 1 <= K <= min(E, 16)");
  RF_CHECK_ARG(!gate || H % 8 == 0, "rf_moe_router_topk: hidden size must be a multiple of 8");
  RF_CHECK_ARG(gate || (H == E && !shared_gate),
               "rf_moe_router_topk: without a gate, x holds the [T,E] logits (H == E)");
  RF_CHECK_ARG(entropy_k_min <= K, "rf_moe_router_topk: entropy_k_min > K");
  // an empty batch (T == 0) has empty, possibly null, outputs and returns at once
  RF_CHECK_ARG(T == 0 || (topk_weights && (topk_ids32 || topk_ids64)), "rf_moe_router_topk: missing outputs");
  RF_CHECK_ARG(T == 0 || x, "rf_moe_router_topk: null input");
  RF_CHECK_ARG(T == 0 || !shared_gate || shared_scale, "rf_moe_router_topk: shared_gate needs shared_scale");
  RF_CHECK_ARG((!gate || ((uintptr_t)x % 16) == 0) && ((uintptr_t)gate % 16) == 0 &&
                   ((uintptr_t)shared_gate % 16) == 0,
               "rf_moe_router_topk: x / gate must be 16-byte aligned");
  if (T == 0) return RF_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int Ec = (int)E + (shared_gate ? 1 : 0);
  TopkArgs b;
  b.partial = nullptr;
  b.x_logits = x;
  b.x_dtype = x_dtype;
  b.bias = bias;
  b.shared_scale = shared_scale;
  b.topk_w = topk_weights;
  b.ids32 = topk_ids32;
  b.ids64 = topk_ids64;
  b.logits_out = logits;
  b.T = T;
  b.E = (int)E;
  b.Ec = Ec;
  b.K = (int)K;
  b.ksplit = 1;
  b.ld = Ec;
  b.has_shared = shared_gate ? 1 : 0;
  b.renormalize = renormalize;
  b.round_dtype = round_dtype;
  b.entropy_k_min = entropy_k_min;
  if (gate) {
    const Plan p = make_plan(T, (int)H, Ec);
    const size_t need = (size_t)p.slices * (size_t)T * (size_t)Ec * sizeof(float);
    RF_CHECK_ARG(workspace && workspace_bytes >= need && ((uintptr_t)workspace % 16) == 0,
                 "rf_moe_router_topk: workspace too small (see rf_moe_router_workspace_size)");
    RF_CHECK_ARG(p.ttiles <= 0x7fffffff && p.slices <= 65535, "rf_moe_router_topk: too many tokens");
    // Tensor cores when x and the gate share a 16-bit dtype and the shared
    // gate (if any) is the row right after the gate's E rows: one tile per
    // (128 tokens, slice of H), each slice a fixed MMA sequence, partials
    // [slices][T][ld] summed in slice order by the top-k pass (the same bits
    // whatever T is; few tokens still get one CTA per slice).  Otherwise the
    // CUDA-core slices.
    const size_t esz = (size_t)rf::dtype_size(gate_dtype);
    const bool adjacent = !shared_gate ||
                          (const char *)shared_gate == (const char *)gate + (size_t)E * (size_t)H * esz;
    const int64_t ld = (Ec + 3) / 4 * 4;
    int rc = -1;
    if (x_dtype == gate_dtype && adjacent &&
        workspace_bytes >= (size_t)p.slices * (size_t)T * (size_t)ld * sizeof(float))
      rc = rf::tc_dense_f32(x, gate, reinterpret_cast<float *>(workspace), T, Ec, H, ld, x_dtype, st, SLICE);
    if (rc > 0) return rc;
    if (rc == 0) {
      b.partial = reinterpret_cast<const float *>(workspace);
      b.ksplit = p.slices;
      b.ld = ld;
    } else {
      LogitsArgs a{x, gate, shared_gate, reinterpret_cast<float *>(workspace), T, (int)H, (int)E, Ec};
      switch (x_dtype) {
        case RF_F32: launch_logits_tg<float>(a, p, gate_dtype, st); break;
        case RF_F16: launch_logits_tg<__half>(a, p, gate_dtype, st); break;
        default: launch_logits_tg<__nv_bfloat16>(a, p, gate_dtype, st); break;
      }
      rc = rf::check_launch("rf_moe_router_topk(logits)");
      if (rc) return rc;
      b.partial = a.partial;
      b.ksplit = p.slices;
      b.ld = Ec;
    }
  }
  int64_t blocks = (T + TK_WARPS - 1) / TK_WARPS;
  const int64_t cap = (int64_t)rf::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  const int smem = TK_WARPS * (int)E * (int)sizeof(float);
  switch (x_dtype) {
    case RF_F32: router_topk_kernel<float><<<(int)blocks, TK_WARPS * 32, smem, st>>>(b); break;
    case RF_F16: router_topk_kernel<__half><<<(int)blocks, TK_WARPS * 32, smem, st>>>(b); break;
    default: router_topk_kernel<__nv_bfloat16><<<(int)blocks, TK_WARPS * 32, smem, st>>>(b); break;
  }
  return rf::check_launch("rf_moe_router_topk(topk)");
}
