// The expert split's int8 half: the routed experts that are not resident this
// step run on symmetric int8 copies of their weights (the reference's
// CPU/GPU split, reframework/moe/moe_layer.py:523-627, computes them on the
// host with torch._int_mm; here their int8 copies cross PCIe, half the bytes
// of the 16-bit weights, and run on the GPU).  Arithmetic restated from
// reframework/moe/fused.py:140-197 (slot (t, k) belongs to token t):
//   per listed expert e, over its rows of the permuted layout:
//     xs = max|x| / 127 (fp32), xq = round(x / xs) clamped to +-127   (int8_quantize)
//     gu = float(xq . w1q[e]^T) * (xs * s1[e])    exact int32 sums     (int8_grouped_gemm, gated)
//     inter = act(gu[:, :I]) * gu[:, I:] in fp32, block max|inter|
//     iq = round(inter / is) with is = max|inter| / 127               (int8_quantize)
//     y = float(iq . w2q[e]^T) * (is * s2[e]) * w (routing weight)    (int8_grouped_gemm, down)
//   out[t] = (sum of the resident experts' rows, reference rounding in the
//             layer dtype) + (sum of the int8 rows in fp32), rounded once  (split_combine)
// The int8 GEMMs accumulate exactly in int32 (tcgen05.mma kind::i8 on the
// tensor cores, gemm_tc.cu; dp4a on CUDA cores for shapes TMA cannot
// describe), so they equal torch._int_mm bit for bit; the activation uses IEEE fp32 division with
// CUDA's expf / erff / tanhf, within an ulp or two of torch's CPU kernels.
// The work is bound by the PCIe copy of the int8 weights, not by these kernels.
#include <string>

#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int QBLOCKS = 32;  // row blocks per listed expert in the quantize kernels

struct Groups {              // listed experts and their rows in the permuted layout
  const int32_t *offsets;    // [E] first row of each expert
  const int32_t *counts;     // [E] rows of each expert
  const int32_t *groups;     // [n] listed expert ids
  int n, E;
};

__device__ __forceinline__ bool group_rows(const Groups &g, int i, int64_t &r0, int64_t &cnt) {
  const int e = g.groups[i];
  if (e < 0 || e >= g.E) {
    rf_report(RF_DEV_BAD_EXPERT_ID);
    return false;
  }
  r0 = g.offsets[e];
  cnt = g.counts[e];
  return true;
}

__device__ __forceinline__ float block_max(float m) {
  __shared__ float s_red[32];
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) s_red[w] = m;
  __syncthreads();
  if (w == 0) {
    m = l < (int)(blockDim.x >> 5) ? s_red[l] : 0.f;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  }
  return m;  // valid in thread 0
}

// max|src| over each listed expert's rows (non-negative floats order like
// their bit patterns, so an integer atomicMax is exact and order-free)
template <typename T>
__global__ void __launch_bounds__(256) amax_kernel(const T *src, int64_t cols, const Groups g, float *amax) {
  int64_t r0, cnt;
  if (!group_rows(g, blockIdx.x, r0, cnt)) return;
  float m = 0.f;
  for (int64_t r = blockIdx.y; r < cnt; r += gridDim.y) {
    const T *row = src + (r0 + r) * cols;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(rf::Cvt<T>::to_f(row[c])));
  }
  m = block_max(m);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<int *>(amax) + blockIdx.x, __float_as_int(m));
}

// codes = round-half-even(x / scale) clamped to +-127 with scale = amax / 127
// in fp32; a block whose amax is <= 0 gets scale 1 and zero codes
// (offload_cache.py:58-72)
template <typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T *src, int64_t cols, const Groups g, const float *amax,
                                                       float *scales, int8_t *q) {
  int64_t r0, cnt;
  if (!group_rows(g, blockIdx.x, r0, cnt)) return;
  const float a = amax[blockIdx.x];
  const bool zero = a <= 0.f;
  const float scale = zero ? 1.0f : __fdiv_rn(a, 127.0f);
  if (blockIdx.y == 0 && threadIdx.x == 0) scales[blockIdx.x] = scale;
  for (int64_t r = blockIdx.y; r < cnt; r += gridDim.y) {
    const T *row = src + (r0 + r) * cols;
    int8_t *qr = q + (r0 + r) * cols;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      float v = zero ? 0.f : rintf(__fdiv_rn(rf::Cvt<T>::to_f(row[c]), scale));
      v = fminf(fmaxf(v, -127.f), 127.f);
      qr[c] = (int8_t)(int)v;
    }
  }
}

}  // namespace

extern "C" int rf_moe_int8_quantize(const void *src, int32_t src_dtype, const int32_t *offsets, const int32_t *counts,
                                    const int32_t *groups, int32_t n_groups, int32_t E, int64_t rows_capacity,
                                    int64_t cols, float *amax, int32_t compute_amax, float *scales, int8_t *q,
                                    rf_stream_t stream) {
  RF_CHECK_ARG(rf::valid_dtype(src_dtype), "rf_moe_int8_quantize: unknown dtype");
  RF_CHECK_ARG(n_groups >= 0 && n_groups <= 65535 && E >= 1 && rows_capacity >= 0 && cols >= 1,
               "rf_moe_int8_quantize: bad sizes");
  if (n_groups == 0 || rows_capacity == 0) return RF_OK;
  RF_CHECK_ARG(src && offsets && counts && groups && amax && scales && q, "rf_moe_int8_quantize: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  Groups g{offsets, counts, groups, n_groups, E};
  const dim3 grid((unsigned)n_groups, QBLOCKS);
  if (compute_amax) {
    if (cudaMemsetAsync(amax, 0, sizeof(float) * (size_t)n_groups, st) != cudaSuccess)
      return rf::check_launch("rf_moe_int8_quantize (amax reset)");
    if (src_dtype == RF_F32)
      amax_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float *>(src), cols, g, amax);
    else if (src_dtype == RF_BF16)
      amax_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16 *>(src), cols, g, amax);
    else
      amax_kernel<__half><<<grid, 256, 0, st>>>(reinterpret_cast<const __half *>(src), cols, g, amax);
    const int rc = rf::check_launch("rf_moe_int8_quantize (amax)");
    if (rc != RF_OK) return rc;
  }
  if (src_dtype == RF_F32)
    quantize_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float *>(src), cols, g, amax, scales, q);
  else if (src_dtype == RF_BF16)
    quantize_kernel<__nv_bfloat16>
        <<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16 *>(src), cols, g, amax, scales, q);
  else
    quantize_kernel<__half><<<grid, 256, 0, st>>>(reinterpret_cast<const __half *>(src), cols, g, amax, scales, q);
  return rf::check_launch("rf_moe_int8_quantize");
}

namespace {

constexpr int GBM = 64, GBN = 64, GBK = 64;  // rows x output columns x int8 depth of a tile
constexpr int KW = GBK / 4;                  // int32 words per tile row
constexpr int KWP = KW + 1;                  // padded: column reads hit distinct banks
constexpr int MAX_G = 1024;

struct GemmArgs {
  const int8_t *a;          // [rows_capacity, Kdim] codes of the permuted rows
  const int8_t *w;          // [num_slots, (gated ? 2N : N), Kdim] weight codes
  Groups g;
  const int32_t *slot;      // [E] expert -> weight slot
  int num_slots;
  int64_t Kdim, N;
  const float *a_scales;    // [n] per listed expert
  const float *w_scales;    // scale of expert e at w_scales[e * w_stride]
  int64_t w_stride;
  int act;
  float *out;               // gated: inter [rows_capacity, N]; down: y [rows_capacity, N]
  float *amax_out;          // gated: [n] max|inter| per listed expert (zeroed by the host)
  const float *row_w;       // down: routing weight of each slot (t*K + k)
  const int32_t *src_slot;  // down: slot of each permuted row
};

using rf::act_ieee;

template <bool GATED>
__global__ void __launch_bounds__(256) int8_gemm_kernel(const GemmArgs p) {
  __shared__ int32_t sA[GBM][KWP];
  __shared__ int32_t sB[GATED ? 2 : 1][GBN][KWP];
  __shared__ int s_prefix[MAX_G + 1];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int G = p.g.n;
  const int ntn = (int)((p.N + GBN - 1) / GBN);
  if (tid == 0) {  // tiles per listed expert -> prefix
    int acc = 0;
    s_prefix[0] = 0;
    for (int i = 0; i < G; ++i) {
      const int e = p.g.groups[i];
      const int cnt = (e >= 0 && e < p.g.E) ? p.g.counts[e] : 0;
      acc += ((cnt + GBM - 1) / GBM) * ntn;
      s_prefix[i + 1] = acc;
    }
  }
  __syncthreads();
  const int total = s_prefix[G];
  const int lr = tid >> 2, lc = (tid & 3) * 16;  // this thread's 16 bytes of a tile
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    int lo = 0, hi = G - 1;  // last listed expert whose first tile is <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_prefix[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    const int gi = lo, e = p.g.groups[gi];
    const int s = p.slot ? p.slot[e] : e;
    const bool ok = s >= 0 && s < p.num_slots;  // block-uniform
    if (!ok) {
      if (tid == 0) rf_report(RF_DEV_BAD_EXPERT_ID);
      continue;
    }
    const int64_t cnt = p.g.counts[e];
    const int mt = (int)((cnt + GBM - 1) / GBM);
    const int local = t - s_prefix[gi];
    const int nb = local / mt, mb = local - nb * mt;
    const int64_t row0 = (int64_t)p.g.offsets[e] + (int64_t)mb * GBM;
    const int rows = (int)min((int64_t)GBM, cnt - (int64_t)mb * GBM);
    const int64_t n0 = (int64_t)nb * GBN;
    const int8_t *W = p.w + (int64_t)s * (GATED ? 2 : 1) * p.N * p.Kdim;
    int acc[4][4], accu[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = accu[i][j] = 0;
    for (int64_t k0 = 0; k0 < p.Kdim; k0 += GBK) {
      __syncthreads();  // the previous tile's reads are done
      int4 va = make_int4(0, 0, 0, 0), vb = make_int4(0, 0, 0, 0), vu = make_int4(0, 0, 0, 0);
      const bool kin = k0 + lc < p.Kdim;
      if (kin && lr < rows) va = *reinterpret_cast<const int4 *>(p.a + (row0 + lr) * p.Kdim + k0 + lc);
      if (kin && n0 + lr < p.N) {
        vb = *reinterpret_cast<const int4 *>(W + (n0 + lr) * p.Kdim + k0 + lc);
        if (GATED) vu = *reinterpret_cast<const int4 *>(W + (p.N + n0 + lr) * p.Kdim + k0 + lc);
      }
      const int w0 = (tid & 3) * 4;
      sA[lr][w0] = va.x; sA[lr][w0 + 1] = va.y; sA[lr][w0 + 2] = va.z; sA[lr][w0 + 3] = va.w;
      sB[0][lr][w0] = vb.x; sB[0][lr][w0 + 1] = vb.y; sB[0][lr][w0 + 2] = vb.z; sB[0][lr][w0 + 3] = vb.w;
      if (GATED) {
        sB[GATED ? 1 : 0][lr][w0] = vu.x; sB[GATED ? 1 : 0][lr][w0 + 1] = vu.y;
        sB[GATED ? 1 : 0][lr][w0 + 2] = vu.z; sB[GATED ? 1 : 0][lr][w0 + 3] = vu.w;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < KW; ++kk) {
        int a[4], b[4], u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = sA[ty * 4 + i][kk];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          b[j] = sB[0][tx * 4 + j][kk];
          u[j] = GATED ? sB[GATED ? 1 : 0][tx * 4 + j][kk] : 0;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[i][j] = __dp4a(a[i], b[j], acc[i][j]);
            if (GATED) accu[i][j] = __dp4a(a[i], u[j], accu[i][j]);
          }
      }
    }
    // epilogue: exact int32 sums -> fp32 with the reference's scale products
    const float dq = __fmul_rn(p.a_scales[gi], p.w_scales[(int64_t)e * p.w_stride]);
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      if (r >= rows) continue;
      float* orow = p.out + (row0 + r) * p.N;
      const float rw = GATED ? 0.f : p.row_w[p.src_slot[row0 + r]];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + tx * 4 + j;
        if (n >= p.N) continue;
        if (GATED) {
          const float gf = __fmul_rn(__int2float_rn(acc[i][j]), dq);
          const float uf = __fmul_rn(__int2float_rn(accu[i][j]), dq);
          const float v = __fmul_rn(act_ieee(p.act, gf), uf);
          orow[n] = v;
          m = fmaxf(m, fabsf(v));
        } else {
          orow[n] = __fmul_rn(__fmul_rn(__int2float_rn(acc[i][j]), dq), rw);
        }
      }
    }
    if (GATED) {
      m = block_max(m);
      if (tid == 0) atomicMax(reinterpret_cast<int *>(p.amax_out) + gi, __float_as_int(m));
    }
  }
}

}  // namespace

extern "C" int rf_moe_int8_grouped_gemm(const int8_t *a, const int8_t *w, const int32_t *offsets,
                                        const int32_t *counts, const int32_t *groups, const int32_t *slot,
                                        int32_t n_groups, int32_t E, int32_t num_slots, int64_t rows_capacity,
                                        int64_t Kdim, int64_t N, const float *a_scales, const float *w_scales,
                                        int64_t w_scale_stride, int32_t gated, int32_t act, float *out,
                                        float *amax_out, const float *row_weights, const int32_t *src_slot,
                                        rf_stream_t stream) {
  RF_CHECK_ARG(n_groups >= 0 && n_groups <= MAX_G && E >= 1 && num_slots >= 1 && rows_capacity >= 0 && N >= 1 &&
                   Kdim >= 16 && Kdim % 16 == 0 && Kdim < (1 << 30) && N < (1 << 30) && w_scale_stride >= 1,
               "rf_moe_int8_grouped_gemm: bad sizes (Kdim a multiple of 16, at most 1024 listed experts)");
  RF_CHECK_ARG(act == RF_ACT_SILU || act == RF_ACT_GELU || act == RF_ACT_GELU_TANH,
               "rf_moe_int8_grouped_gemm: unknown activation");
  if (n_groups == 0 || rows_capacity == 0) return RF_OK;
  RF_CHECK_ARG(a && w && offsets && counts && groups && a_scales && w_scales && out,
               "rf_moe_int8_grouped_gemm: null pointer");
  RF_CHECK_ARG(!gated || amax_out, "rf_moe_int8_grouped_gemm: the gated GEMM needs amax_out");
  RF_CHECK_ARG(gated || (row_weights && src_slot), "rf_moe_int8_grouped_gemm: the down GEMM needs row weights");
  RF_CHECK_ARG((uintptr_t)a % 16 == 0 && (uintptr_t)w % 16 == 0, "rf_moe_int8_grouped_gemm: 16-byte alignment");
  cudaStream_t st = (cudaStream_t)stream;
  GemmArgs p;
  p.a = a;
  p.w = w;
  p.g = Groups{offsets, counts, groups, n_groups, E};
  p.slot = slot;
  p.num_slots = num_slots;
  p.Kdim = Kdim;
  p.N = N;
  p.a_scales = a_scales;
  p.w_scales = w_scales;
  p.w_stride = w_scale_stride;
  p.act = act;
  p.out = out;
  p.amax_out = amax_out;
  p.row_w = row_weights;
  p.src_slot = src_slot;
  const int grid = rf::num_sms() * 4;
  if (gated && cudaMemsetAsync(amax_out, 0, sizeof(float) * (size_t)n_groups, st) != cudaSuccess)
    return rf::check_launch("rf_moe_int8_grouped_gemm (amax reset)");
  // the tensor cores (kind::i8) when the shape allows; the dp4a kernel below otherwise
  const int tc = rf::tc_int8_grouped_gemm(a, w, offsets, counts, groups, slot, n_groups, E, num_slots, rows_capacity,
                                          Kdim, N, a_scales, w_scales, w_scale_stride, gated != 0, act, out, amax_out,
                                          row_weights, src_slot, st);
  if (tc >= 0) return tc;
  if (gated) {
    int8_gemm_kernel<true><<<grid, 256, 0, st>>>(p);
  } else {
    int8_gemm_kernel<false><<<grid, 256, 0, st>>>(p);
  }
  return rf::check_launch("rf_moe_int8_grouped_gemm");
}

namespace {

constexpr int KMAX = 16;

// out[t] = round_T( float(hit sum) + miss sum ): per token, in ascending
// permuted row (= ascending expert) order, the resident experts' rows as the
// reference's layer-dtype half does it (each y * round_T(w) rounded to T, added
// and rounded to T; fused.py:89-137) and the int8 rows (already weighted, fp32)
// added in fp32 (fused.py:194-196); the two halves meet in fp32
// (moe_layer.py:604-605).
template <typename T>
__global__ void __launch_bounds__(256) split_combine_kernel(const T *y_hit, const float *y_int8,
                                                            const int32_t *row_of_slot, const int32_t *ids,
                                                            const uint8_t *is_miss, const float *w, int64_t T_,
                                                            int K, int64_t H, int E, T *out) {
  __shared__ int s_row[KMAX];
  __shared__ int s_miss[KMAX];
  __shared__ float s_w[KMAX];
  __shared__ int s_n;
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int k = 0; k < K; ++k) {
      const int32_t r = row_of_slot[t * K + k];
      const int32_t e = ids[t * K + k];
      if (r < 0) continue;
      if (e < 0 || e >= E) {
        rf_report(RF_DEV_BAD_EXPERT_ID);
        continue;
      }
      int i = n++;  // insertion by row
      while (i > 0 && s_row[i - 1] > r) {
        s_row[i] = s_row[i - 1];
        s_miss[i] = s_miss[i - 1];
        s_w[i] = s_w[i - 1];
        --i;
      }
      s_row[i] = r;
      s_miss[i] = is_miss[e] ? 1 : 0;
      s_w[i] = w[t * K + k];
    }
    s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
    float acc_h = 0.f, acc8 = 0.f;
    for (int i = 0; i < n; ++i) {
      const int64_t r = s_row[i];
      if (s_miss[i]) {
        acc8 = __fadd_rn(acc8, y_int8[r * H + h]);
      } else {
        const float prod = rf::round_to<T>(__fmul_rn(rf::Cvt<T>::to_f(y_hit[r * H + h]), rf::round_to<T>(s_w[i])));
        acc_h = rf::round_to<T>(__fadd_rn(acc_h, prod));
      }
    }
    out[t * H + h] = rf::Cvt<T>::from_f(__fadd_rn(acc_h, acc8));
  }
}

}  // namespace

extern "C" int rf_moe_split_combine(const void *y_hit, const float *y_int8, const int32_t *row_of_slot,
                                    const int32_t *ids, const uint8_t *is_miss, const float *topk_weights, int64_t T,
                                    int32_t K, int64_t H, int32_t E, int32_t dtype, void *out, rf_stream_t stream) {
  RF_CHECK_ARG(rf::valid_dtype(dtype), "rf_moe_split_combine: unknown dtype");
  RF_CHECK_ARG(T >= 0 && K >= 1 && K <= KMAX && H >= 1 && E >= 1, "rf_moe_split_combine: bad sizes (K <= 16)");
  if (T == 0) return RF_OK;
  RF_CHECK_ARG(y_hit && y_int8 && row_of_slot && ids && is_miss && topk_weights && out,
               "rf_moe_split_combine: null pointer");
  RF_CHECK_ARG(T < ((int64_t)1 << 31), "rf_moe_split_combine: too many tokens");
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)T);
  if (dtype == RF_F32)
    split_combine_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float *>(y_hit), y_int8, row_of_slot,
                                                      ids, is_miss, topk_weights, T, K, H, E,
                                                      reinterpret_cast<float *>(out));
  else if (dtype == RF_BF16)
    split_combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16 *>(y_hit), y_int8, row_of_slot, ids, is_miss, topk_weights, T, K, H, E,
        reinterpret_cast<__nv_bfloat16 *>(out));
  else
    split_combine_kernel<__half><<<grid, 256, 0, st>>>(reinterpret_cast<const __half *>(y_hit), y_int8, row_of_slot,
                                                       ids, is_miss, topk_weights, T, K, H, E,
                                                       reinterpret_cast<__half *>(out));
  return rf::check_launch("rf_moe_split_combine");
}
