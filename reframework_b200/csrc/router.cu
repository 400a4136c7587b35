// K1 — router GEMV + softmax + top-k + renormalisation, one warp per token.
//
// Restates FusedMoE.route (reframework/moe/moe_layer.py:320-344) and
// torch_fused_topk (reframework/moe/fused.py:32-46) for the GPU:
//   logits = x . gate^T (fp32 accumulate, optionally rounded to the layer
//   dtype and/or biased), p = softmax(logits) in fp32, top-k of p (descending,
//   ties to the lower expert id), w = p / sum(top-k p) when renormalising.
// The op is HBM-bound on x (T*H elements read once); the gate rows are
// re-read from L1/L2 by every warp.
#include "common.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int WARPS = 8;
constexpr int EC = 8;       // experts accumulated per pass over the x row
constexpr int VEC = 8;      // elements per vector (16 B of a 16-bit type)
constexpr int XV = 8;       // vectors per lane per chunk: chunk = 2048 elements
constexpr int KMAX = 16;

template <typename T>
__device__ __forceinline__ void load8(const T *p, float *f) {
  const uint4 *q = reinterpret_cast<const uint4 *>(p);
  if constexpr (sizeof(T) == 4) {
    uint4 a = __ldg(q), b = __ldg(q + 1);
    rf::unpack16<float>(a, f);
    rf::unpack16<float>(b, f + 4);
  } else {
    uint4 a = __ldg(q);
    rf::unpack16<T>(a, f);
  }
}

__device__ __forceinline__ float round_to(int dtype, float v) {
  if (dtype == RF_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == RF_F16) return __half2float(__float2half_rn(v));
  return v;
}

struct RouterArgs {
  const void *x;
  const void *gate;
  const float *bias;
  const void *shared_gate;
  float *shared_scale;
  float *topk_w;
  int32_t *ids32;
  int64_t *ids64;
  float *logits_out;
  int64_t T;
  int H, E, K;
  int renormalize, round_dtype, entropy_k_min;
};

template <typename TX, typename TG>
__global__ void __launch_bounds__(WARPS * 32) router_kernel(RouterArgs a) {
  extern __shared__ float s_logits[];  // [WARPS][E + 1]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *lg = s_logits + warp * (a.E + 1);
  const int R = a.E + (a.shared_gate ? 1 : 0);
  const TX *x = reinterpret_cast<const TX *>(a.x);
  const TG *gate = reinterpret_cast<const TG *>(a.gate);
  const TG *sgate = reinterpret_cast<const TG *>(a.shared_gate);
  const int64_t nwarps = (int64_t)gridDim.x * WARPS;

  for (int64_t t = (int64_t)blockIdx.x * WARPS + warp; t < a.T; t += nwarps) {
    const TX *xr = x + t * a.H;
    if (!gate) {  // x already holds the logits (H == E)
      for (int e = lane; e < a.E; e += 32) lg[e] = rf::Cvt<TX>::to_f(xr[e]);
    }
    // ---- logits.  The x row is consumed in chunks of 32 lanes x XV vectors
    // of 8 elements, all loads of a chunk issued before any arithmetic (the
    // row is the HBM traffic; the gate rows come from L1).  Each lane keeps a
    // fixed-order fp32 partial sum per expert; a butterfly reduces them.
    for (int g0 = 0; gate && g0 < R; g0 += EC) {
      float acc[EC];
#pragma unroll
      for (int j = 0; j < EC; ++j) acc[j] = 0.f;
      for (int h0 = 0; h0 < a.H; h0 += 32 * VEC * XV) {
        float xf[XV][VEC];
#pragma unroll
        for (int v = 0; v < XV; ++v) {
          const int h = h0 + (v * 32 + lane) * VEC;
          if (h < a.H) load8<TX>(xr + h, xf[v]);
          else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) xf[v][i] = 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < EC; ++j) {
          const int e = g0 + j;
          if (e < R) {
            const TG *row = (e < a.E) ? gate + (int64_t)e * a.H : sgate;
            float s = acc[j];
#pragma unroll
            for (int v = 0; v < XV; ++v) {
              const int h = h0 + (v * 32 + lane) * VEC;
              if (h < a.H) {
                float gf[VEC];
                load8<TG>(row + h, gf);
#pragma unroll
                for (int i = 0; i < VEC; ++i) s = fmaf(xf[v][i], gf[i], s);
              }
            }
            acc[j] = s;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < EC; ++j) {
        if (g0 + j < R) {  // warp-uniform
          float v = acc[j];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0) lg[g0 + j] = v;
        }
      }
    }
    __syncwarp();
    // ---- rounding / bias, softmax statistics
    float m = -INFINITY;
    for (int e = lane; e < a.E; e += 32) {
      float v = lg[e];
      if (a.round_dtype >= 0) v = round_to(a.round_dtype, v);
      if (a.bias) {
        v += a.bias[e];
        if (a.round_dtype >= 0) v = round_to(a.round_dtype, v);
      }
      lg[e] = v;
      if (a.logits_out) a.logits_out[t * a.E + e] = v;
      m = fmaxf(m, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncwarp();
    float s = 0.f;
    for (int e = lane; e < a.E; e += 32) s += expf(lg[e] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.0f / s;
    float ent = 0.f;
    for (int e = lane; e < a.E; e += 32) {
      const float p = expf(lg[e] - m) * inv;
      lg[e] = p;  // probabilities from here on
      if (a.entropy_k_min > 0) ent -= p * logf(fmaxf(p, 1e-9f));
    }
    if (a.entropy_k_min > 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ent += __shfl_xor_sync(0xffffffffu, ent, o);
    }
    __syncwarp();
    // ---- top-k by probability, ties to the lower id
    float pk[KMAX];
    int ik[KMAX];
    for (int k = 0; k < a.K; ++k) {
      float best = -1.f;
      int bi = 0x7fffffff;
      for (int e = lane; e < a.E; e += 32) {
        const float p = lg[e];
        if (p > best) { best = p; bi = e; }   // lanes scan ascending ids: strict '>' keeps the lowest
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
      pk[k] = best;
      ik[k] = bi;
      __syncwarp();
      if (lane == (bi & 31)) lg[bi] = -2.f;  // taken
      __syncwarp();
    }
    // ---- weights
    float w[KMAX];
    if (a.entropy_k_min > 0) {
      const float hn = ent / logf((float)a.E);
      int kd = (int)rintf((float)a.entropy_k_min + (float)(a.K - a.entropy_k_min) * hn);
      kd = min(max(kd, a.entropy_k_min), a.K);
      float sum = 0.f;
      for (int k = 0; k < a.K; ++k) { w[k] = k < kd ? pk[k] : 0.f; sum += w[k]; }
      const float d = fmaxf(sum, 1e-9f);
      for (int k = 0; k < a.K; ++k) w[k] = w[k] / d;
    } else if (a.renormalize) {
      float sum = 0.f;
      for (int k = 0; k < a.K; ++k) sum += pk[k];
      for (int k = 0; k < a.K; ++k) w[k] = pk[k] / sum;
    } else {
      for (int k = 0; k < a.K; ++k) w[k] = pk[k];
    }
    if (lane < a.K) {
      float wv = 0.f;
      int iv = 0;
      for (int k = 0; k < a.K; ++k)
        if (k == lane) { wv = w[k]; iv = ik[k]; }
      a.topk_w[t * a.K + lane] = wv;
      if (a.ids32) a.ids32[t * a.K + lane] = iv;
      if (a.ids64) a.ids64[t * a.K + lane] = iv;
    }
    if (a.shared_gate && lane == 0) {
      const float z = lg[a.E] ;  // shared-gate logit was left untouched above
      a.shared_scale[t] = 1.0f / (1.0f + expf(-z));
    }
    __syncwarp();
  }
}

template <typename TX>
int launch_router_tg(const RouterArgs &a, int gate_dtype, cudaStream_t st) {
  const int smem = WARPS * (a.E + 1) * (int)sizeof(float);
  int64_t blocks = (a.T + WARPS - 1) / WARPS;
  const int64_t cap = (int64_t)rf::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  switch (gate_dtype) {
    case RF_F32: router_kernel<TX, float><<<(int)blocks, WARPS * 32, smem, st>>>(a); break;
    case RF_F16: router_kernel<TX, __half><<<(int)blocks, WARPS * 32, smem, st>>>(a); break;
    default: router_kernel<TX, __nv_bfloat16><<<(int)blocks, WARPS * 32, smem, st>>>(a); break;
  }
  return rf::check_launch("rf_moe_router_topk");
}

}  // namespace

extern "C" int rf_moe_router_topk(const void *x, int x_dtype, const void *gate, int gate_dtype,
                                  const float *bias, int64_t T, int64_t H, int64_t E, int64_t K,
                                  int renormalize, int round_dtype, int entropy_k_min,
                                  const void *shared_gate, float *shared_scale,
                                  float *topk_weights, int32_t *topk_ids32, int64_t *topk_ids64,
                                  float *logits, rf_stream_t stream) {
  RF_CHECK_ARG(rf::valid_dtype(x_dtype) && rf::valid_dtype(gate_dtype),
               "rf_moe_router_topk: unknown dtype");
  RF_CHECK_ARG(round_dtype < 0 || rf::valid_dtype(round_dtype), "rf_moe_router_topk: bad round_dtype");
  RF_CHECK_ARG(T >= 0 && H > 0 && E > 0, "rf_moe_router_topk: sizes must be positive");
  RF_CHECK_ARG(E <= 1024, "rf_moe_router_topk: at most 1024 experts");
  RF_CHECK_ARG(K >= 1 && K <= E && K <= KMAX, "rf_moe_router_topk: need 1 <= K <= min(E, 16)");
  RF_CHECK_ARG(!gate || H % VEC == 0, "rf_moe_router_topk: hidden size must be a multiple of 8");
  RF_CHECK_ARG(gate || (H == E && !shared_gate),
               "rf_moe_router_topk: without a gate, x holds the [T,E] logits (H == E)");
  RF_CHECK_ARG(entropy_k_min <= K, "rf_moe_router_topk: entropy_k_min > K");
  RF_CHECK_ARG(topk_weights && (topk_ids32 || topk_ids64), "rf_moe_router_topk: missing outputs");
  RF_CHECK_ARG(T == 0 || x, "rf_moe_router_topk: null input");
  RF_CHECK_ARG(!shared_gate || shared_scale, "rf_moe_router_topk: shared_gate needs shared_scale");
  RF_CHECK_ARG((!gate || ((uintptr_t)x % 16) == 0) && ((uintptr_t)gate % 16) == 0 &&
                   ((uintptr_t)shared_gate % 16) == 0,
               "rf_moe_router_topk: x / gate must be 16-byte aligned");
  if (T == 0) return RF_OK;
  RouterArgs a;
  a.x = x; a.gate = gate; a.bias = bias; a.shared_gate = shared_gate; a.shared_scale = shared_scale;
  a.topk_w = topk_weights; a.ids32 = topk_ids32; a.ids64 = topk_ids64; a.logits_out = logits;
  a.T = T; a.H = (int)H; a.E = (int)E; a.K = (int)K;
  a.renormalize = renormalize; a.round_dtype = round_dtype; a.entropy_k_min = entropy_k_min;
  cudaStream_t st = (cudaStream_t)stream;
  switch (x_dtype) {
    case RF_F32: return launch_router_tg<float>(a, gate_dtype, st);
    case RF_F16: return launch_router_tg<__half>(a, gate_dtype, st);
    default: return launch_router_tg<__nv_bfloat16>(a, gate_dtype, st);
  }
}
