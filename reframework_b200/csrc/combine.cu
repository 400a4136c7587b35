// K5 — weighted combine of the expert outputs back into token order.
//
// Restates reframework/moe/fused.py:79,84-86 as a gather: each token reads its
// K expert rows (located through row_of_slot) and sums them; the optional
// shared-expert output and residual are added.  No atomics: deterministic.
//
// Two summation modes:
//   RF_COMBINE_REFERENCE  the reference's rounding points: the routing weight
//       is cast to the output dtype (fused.py:79), each weighted row is
//       rounded (`y * w`, fused.py:84) and the rows are accumulated in the
//       output dtype in ascending expert order (the order of the per-expert
//       `index_add_` loop, fused.py:76-86).  Rows of the permuted layout are
//       expert-major, so ascending row index is ascending expert id.  The
//       shared output (times its gate) and the residual are then added with
//       one rounding each.  For fp32 this is plain fp32 arithmetic in that
//       order.
//   RF_COMBINE_FP32  fp32 accumulation of every term, one rounding at the end.
// HBM-bound: reads T*K*H + T*H (+ T*H per optional input), writes T*H elements.
#include "common.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int CT = 128;  // threads per block; a block handles one token row at a time
constexpr int KMAX = 16;

struct CombineArgs {
  const void *y;
  const int32_t *row_of_slot;
  const float *w;
  const void *shared_y;
  const float *shared_scale;
  const void *residual;
  void *out;
  int64_t T;
  int K, H;
  int accumulate;
  int mode;
};

template <typename T>
__device__ __forceinline__ void store16(T *p, const float *f);
template <> __device__ __forceinline__ void store16<float>(float *p, const float *f) {
  *reinterpret_cast<uint4 *>(p) =
      make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}
template <> __device__ __forceinline__ void store16<__nv_bfloat16>(__nv_bfloat16 *p, const float *f) {
  *reinterpret_cast<uint4 *>(p) = make_uint4(rf::pack2<__nv_bfloat16>(f[0], f[1]), rf::pack2<__nv_bfloat16>(f[2], f[3]),
                                             rf::pack2<__nv_bfloat16>(f[4], f[5]), rf::pack2<__nv_bfloat16>(f[6], f[7]));
}
template <> __device__ __forceinline__ void store16<__half>(__half *p, const float *f) {
  *reinterpret_cast<uint4 *>(p) = make_uint4(rf::pack2<__half>(f[0], f[1]), rf::pack2<__half>(f[2], f[3]),
                                             rf::pack2<__half>(f[4], f[5]), rf::pack2<__half>(f[6], f[7]));
}

template <typename T, bool REF>
__global__ void __launch_bounds__(CT) combine_kernel(CombineArgs a) {
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  __shared__ int s_row[KMAX];
  __shared__ float s_w[KMAX];
  __shared__ int s_n;
  const T *y = reinterpret_cast<const T *>(a.y);
  const T *sy = reinterpret_cast<const T *>(a.shared_y);
  const T *res = reinterpret_cast<const T *>(a.residual);
  T *out = reinterpret_cast<T *>(a.out);
  const int nv = a.H / V;
  for (int64_t t = blockIdx.x; t < a.T; t += gridDim.x) {
    if (threadIdx.x == 0) {
      // valid slots, sorted by row (= by expert id) for the reference order
      int n = 0;
      for (int k = 0; k < a.K; ++k) {
        const int r = a.row_of_slot[t * a.K + k];
        if (r < 0) continue;
        float wk = a.w[t * a.K + k];
        if (REF) wk = rf::round_to<T>(wk);
        int j = n++;
        while (REF && j > 0 && s_row[j - 1] > r) {
          s_row[j] = s_row[j - 1];
          s_w[j] = s_w[j - 1];
          --j;
        }
        s_row[j] = r;
        s_w[j] = wk;
      }
      s_n = n;
    }
    __syncthreads();
    const int n = s_n;
    const float sscale = (sy && a.shared_scale) ? a.shared_scale[t] : 1.0f;
    for (int v = threadIdx.x; v < nv; v += CT) {
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      for (int k = 0; k < n; ++k) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(y + (int64_t)s_row[k] * a.H) + v);
        float f[V];
        rf::unpack16<T>(q, f);
        const float wk = s_w[k];
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (REF) acc[i] = rf::round_to<T>(__fadd_rn(acc[i], rf::round_to<T>(__fmul_rn(f[i], wk))));
          else acc[i] = fmaf(wk, f[i], acc[i]);
        }
      }
      if (sy) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(sy + t * a.H) + v);
        float f[V];
        rf::unpack16<T>(q, f);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (REF) acc[i] = rf::round_to<T>(__fadd_rn(acc[i], rf::round_to<T>(__fmul_rn(f[i], sscale))));
          else acc[i] = fmaf(sscale, f[i], acc[i]);
        }
      }
      if (res) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(res + t * a.H) + v);
        float f[V];
        rf::unpack16<T>(q, f);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = REF ? rf::round_to<T>(__fadd_rn(acc[i], f[i])) : acc[i] + f[i];
      }
      T *o = out + t * a.H + (int64_t)v * V;
      if (a.accumulate) {
        const uint4 q = *reinterpret_cast<const uint4 *>(o);
        float f[V];
        rf::unpack16<T>(q, f);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], f[i]);
      }
      store16<T>(o, acc);
    }
    __syncthreads();
  }
}

template <typename T>
void launch_t(const CombineArgs &a, int blocks, cudaStream_t st) {
  if (a.mode == RF_COMBINE_REFERENCE) combine_kernel<T, true><<<blocks, CT, 0, st>>>(a);
  else combine_kernel<T, false><<<blocks, CT, 0, st>>>(a);
}

}  // namespace

extern "C" int rf_moe_combine(const void *y, const int32_t *row_of_slot, const float *topk_weights,
                              int64_t T, int64_t K, int64_t H, int dtype, const void *shared_y,
                              const float *shared_scale, const void *residual, int accumulate, int mode,
                              void *out, rf_stream_t stream) {
  RF_CHECK_ARG(rf::valid_dtype(dtype), "rf_moe_combine: unknown dtype");
  RF_CHECK_ARG(mode == RF_COMBINE_REFERENCE || mode == RF_COMBINE_FP32, "rf_moe_combine: unknown mode");
  RF_CHECK_ARG(T >= 0 && K >= 1 && K <= KMAX && H > 0, "rf_moe_combine: bad sizes (K <= 16)");
  RF_CHECK_ARG((H * (int64_t)rf::dtype_size(dtype)) % 16 == 0,
               "rf_moe_combine: H * element size must be a multiple of 16 bytes");
  RF_CHECK_ARG(T == 0 || (y && row_of_slot && topk_weights && out), "rf_moe_combine: null pointer");
  RF_CHECK_ARG((uintptr_t)y % 16 == 0 && (uintptr_t)out % 16 == 0 && (uintptr_t)shared_y % 16 == 0 &&
                   (uintptr_t)residual % 16 == 0,
               "rf_moe_combine: buffers must be 16-byte aligned");
  if (T == 0) return RF_OK;
  CombineArgs a{y, row_of_slot, topk_weights, shared_y, shared_scale, residual, out, T, (int)K, (int)H,
                accumulate, mode};
  int64_t blocks = T;
  const int64_t cap = (int64_t)rf::num_sms() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case RF_F32: launch_t<float>(a, (int)blocks, st); break;
    case RF_F16: launch_t<__half>(a, (int)blocks, st); break;
    default: launch_t<__nv_bfloat16>(a, (int)blocks, st); break;
  }
  return rf::check_launch("rf_moe_combine");
}
