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
  // fused RMSNorm (norm_out != NULL): `out` receives the new residual row
  // r = combine + residual and norm_out = r / sqrt(mean(r^2) + eps) * w (+ b)
  void *norm_out;
  const float *norm_w;
  const float *norm_b;
  float eps;
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

// One block per token (grid-stride).  Warp 0's lanes read the K slots of the
// next token while this one is combined (the read is off the critical path)
// and rank the valid ones with shuffles (by row in reference mode, by slot
// otherwise) into a shared list.  Each thread owns up to VPT 16-byte vectors
// of the row and, KB listed slots at a time, issues all their loads before
// accumulating.
//
// Reference mode, 16-bit types: the weighted rows are accumulated with packed
// bf16x2 / half2 instructions that round each product and each sum once to
// the storage type (__hmul2_rn / __hadd2_rn, never contracted into an FMA).
// A product of two 16-bit values is exact in fp32, so this equals rounding the
// fp32 product, and a sum of two 16-bit values rounds to the same 16-bit value
// whether or not it passes through fp32 first: the same bits as the scalar
// fp32-then-round formulation, at one instruction per element.
constexpr int KB = 4;   // slots whose loads are issued together
constexpr int VPT = 2;  // vectors per thread per pass

template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ T2 splat(float w) { return __float2bfloat162_rn(w); }
};
template <> struct Pair<__half> {
  using T2 = __half2;
  static __device__ __forceinline__ T2 splat(float w) { return __float2half2_rn(w); }
};

template <typename T>
__device__ __forceinline__ uint32_t mul_add2(uint32_t acc, uint32_t y, typename Pair<T>::T2 w2) {
  using T2 = typename Pair<T>::T2;
  const T2 a = *reinterpret_cast<const T2 *>(&acc);
  const T2 b = *reinterpret_cast<const T2 *>(&y);
  const T2 r = __hadd2_rn(a, __hmul2_rn(b, w2));
  return *reinterpret_cast<const uint32_t *>(&r);
}

template <typename T, bool REF, bool NORM>
__global__ void __launch_bounds__(CT) combine_kernel(CombineArgs a) {
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr bool PACKED = REF && sizeof(T) == 2;
  __shared__ int s_row[KMAX];
  __shared__ float s_w[KMAX];
  __shared__ int s_n;
  __shared__ float s_red[CT / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T *y = reinterpret_cast<const T *>(a.y);
  const T *sy = reinterpret_cast<const T *>(a.shared_y);
  const T *res = reinterpret_cast<const T *>(a.residual);
  T *out = reinterpret_cast<T *>(a.out);
  const int nv = a.H / V;
  int r_next = -1;
  float w_next = 0.f;
  if (warp == 0 && lane < a.K && (int64_t)blockIdx.x < a.T) {
    r_next = a.row_of_slot[(int64_t)blockIdx.x * a.K + lane];
    w_next = a.w[(int64_t)blockIdx.x * a.K + lane];
  }
  for (int64_t t = blockIdx.x; t < a.T; t += gridDim.x) {
    if (warp == 0) {
      const int r = lane < a.K ? r_next : -1;
      float wk = w_next;
      const int64_t tn = t + gridDim.x;
      if (lane < a.K && tn < a.T) {
        r_next = a.row_of_slot[tn * a.K + lane];
        w_next = a.w[tn * a.K + lane];
      }
      if (REF) wk = rf::round_to<T>(wk);
      const bool valid = r >= 0;
      int rank = 0;
      for (int j = 0; j < a.K; ++j) {
        const int rj = __shfl_sync(0xffffffffu, r, j);
        if (rj >= 0 && (REF ? rj < r : j < lane)) ++rank;
      }
      const int n = __popc(__ballot_sync(0xffffffffu, valid));
      if (valid) {
        s_row[rank] = r;
        s_w[rank] = wk;
      }
      if (lane == 0) s_n = n;
    }
    __syncthreads();
    const int n = s_n;
    const float sscale = (sy && a.shared_scale) ? a.shared_scale[t] : 1.0f;
    float ss = 0.f;  // NORM: sum of squares of the stored residual row (this thread's part)
    for (int v0 = threadIdx.x; v0 < nv; v0 += CT * VPT) {
      float acc[VPT][V];
      uint32_t pacc[VPT][4];
#pragma unroll
      for (int u = 0; u < VPT; ++u) {
#pragma unroll
        for (int i = 0; i < V; ++i) acc[u][i] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) pacc[u][i] = 0u;
      }
      for (int k0 = 0; k0 < n; k0 += KB) {
        uint4 q[KB][VPT];
#pragma unroll
        for (int j = 0; j < KB; ++j) {
          const bool kj = k0 + j < n;
          const uint4 *yr = reinterpret_cast<const uint4 *>(y + (int64_t)(kj ? s_row[k0 + j] : 0) * a.H);
#pragma unroll
          for (int u = 0; u < VPT; ++u) {
            const int v = v0 + u * CT;
            q[j][u] = (kj && v < nv) ? __ldg(yr + v) : make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int j = 0; j < KB; ++j) {
          if (k0 + j >= n) break;
          const float w = s_w[k0 + j];
          if constexpr (PACKED) {
            const typename Pair<T>::T2 w2 = Pair<T>::splat(w);
#pragma unroll
            for (int u = 0; u < VPT; ++u) {
              pacc[u][0] = mul_add2<T>(pacc[u][0], q[j][u].x, w2);
              pacc[u][1] = mul_add2<T>(pacc[u][1], q[j][u].y, w2);
              pacc[u][2] = mul_add2<T>(pacc[u][2], q[j][u].z, w2);
              pacc[u][3] = mul_add2<T>(pacc[u][3], q[j][u].w, w2);
            }
          } else {
#pragma unroll
            for (int u = 0; u < VPT; ++u) {
              float f[V];
              rf::unpack16<T>(q[j][u], f);
#pragma unroll
              for (int i = 0; i < V; ++i) {
                if (REF) acc[u][i] = rf::round_to<T>(__fadd_rn(acc[u][i], rf::round_to<T>(__fmul_rn(f[i], w))));
                else acc[u][i] = fmaf(w, f[i], acc[u][i]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) {
        const int v = v0 + u * CT;
        if (v >= nv) continue;
        float *ac = acc[u];
        if constexpr (PACKED) rf::unpack16<T>(make_uint4(pacc[u][0], pacc[u][1], pacc[u][2], pacc[u][3]), ac);
        if (sy) {
          const uint4 q = __ldg(reinterpret_cast<const uint4 *>(sy + t * a.H) + v);
          float f[V];
          rf::unpack16<T>(q, f);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            if (REF) ac[i] = rf::round_to<T>(__fadd_rn(ac[i], rf::round_to<T>(__fmul_rn(f[i], sscale))));
            else ac[i] = fmaf(sscale, f[i], ac[i]);
          }
        }
        if (res) {
          const uint4 q = __ldg(reinterpret_cast<const uint4 *>(res + t * a.H) + v);
          float f[V];
          rf::unpack16<T>(q, f);
#pragma unroll
          for (int i = 0; i < V; ++i) ac[i] = REF ? rf::round_to<T>(__fadd_rn(ac[i], f[i])) : ac[i] + f[i];
        }
        T *o = out + t * a.H + (int64_t)v * V;
        if (a.accumulate) {
          const uint4 q = *reinterpret_cast<const uint4 *>(o);
          float f[V];
          rf::unpack16<T>(q, f);
#pragma unroll
          for (int i = 0; i < V; ++i) ac[i] = __fadd_rn(ac[i], f[i]);
        }
        store16<T>(o, ac);
        if constexpr (NORM) {
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const float r = rf::round_to<T>(ac[i]);  // the value stored above
            ss = fmaf(r, r, ss);
          }
        }
      }
    }
    if constexpr (NORM) {
      // norm.py:27-35 on the stored row: x32 * (mean(x32^2) + eps).sqrt().reciprocal() * w (+ b)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < CT / 32; ++w) tot += s_red[w];
      const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)a.H), a.eps));
      T *nout = reinterpret_cast<T *>(a.norm_out);
      for (int v0 = threadIdx.x; v0 < nv; v0 += CT * VPT) {
#pragma unroll
        for (int u = 0; u < VPT; ++u) {
          const int v = v0 + u * CT;
          if (v >= nv) continue;
          // this thread stored these vectors of `out` in the first sweep
          const uint4 q = *reinterpret_cast<const uint4 *>(out + t * a.H + (int64_t)v * V);
          float f[V];
          rf::unpack16<T>(q, f);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const int col = v * V + i;
            float z = __fmul_rn(__fmul_rn(f[i], inv), a.norm_w[col]);
            if (a.norm_b) z = __fadd_rn(z, a.norm_b[col]);
            f[i] = z;
          }
          store16<T>(nout + t * a.H + (int64_t)v * V, f);
        }
      }
    }
    __syncthreads();
  }
}

template <typename T>
void launch_t(const CombineArgs &a, int blocks, cudaStream_t st) {
  if (a.norm_out) {
    if (a.mode == RF_COMBINE_REFERENCE) combine_kernel<T, true, true><<<blocks, CT, 0, st>>>(a);
    else combine_kernel<T, false, true><<<blocks, CT, 0, st>>>(a);
    return;
  }
  if (a.mode == RF_COMBINE_REFERENCE) combine_kernel<T, true, false><<<blocks, CT, 0, st>>>(a);
  else combine_kernel<T, false, false><<<blocks, CT, 0, st>>>(a);
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
                accumulate, mode, nullptr, nullptr, nullptr, 0.f};
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

extern "C" int rf_moe_combine_rmsnorm(const void *y, const int32_t *row_of_slot, const float *topk_weights,
                                      int64_t T, int64_t K, int64_t H, int dtype, const void *shared_y,
                                      const float *shared_scale, const void *residual, int mode,
                                      const float *norm_weight, const float *norm_bias, float eps,
                                      void *residual_out, void *normed_out, rf_stream_t stream) {
  RF_CHECK_ARG(rf::valid_dtype(dtype), "rf_moe_combine_rmsnorm: unknown dtype");
  RF_CHECK_ARG(mode == RF_COMBINE_REFERENCE || mode == RF_COMBINE_FP32, "rf_moe_combine_rmsnorm: unknown mode");
  RF_CHECK_ARG(T >= 0 && K >= 1 && K <= KMAX && H > 0 && H < ((int64_t)1 << 30),
               "rf_moe_combine_rmsnorm: bad sizes (K <= 16)");
  RF_CHECK_ARG((H * (int64_t)rf::dtype_size(dtype)) % 16 == 0,
               "rf_moe_combine_rmsnorm: H * element size must be a multiple of 16 bytes");
  RF_CHECK_ARG(eps >= 0.f, "rf_moe_combine_rmsnorm: eps must be >= 0");
  RF_CHECK_ARG(T == 0 || (y && row_of_slot && topk_weights && residual_out && normed_out && norm_weight),
               "rf_moe_combine_rmsnorm: null pointer");
  RF_CHECK_ARG((uintptr_t)y % 16 == 0 && (uintptr_t)residual_out % 16 == 0 && (uintptr_t)normed_out % 16 == 0 &&
                   (uintptr_t)shared_y % 16 == 0 && (uintptr_t)residual % 16 == 0,
               "rf_moe_combine_rmsnorm: buffers must be 16-byte aligned");
  RF_CHECK_ARG(T == 0 || normed_out != residual_out, "rf_moe_combine_rmsnorm: the two outputs must not alias");
  if (T == 0) return RF_OK;
  CombineArgs a{y, row_of_slot, topk_weights, shared_y, shared_scale, residual, residual_out, T, (int)K, (int)H,
                0, mode, normed_out, norm_weight, norm_bias, eps};
  int64_t blocks = T;
  const int64_t cap = (int64_t)rf::num_sms() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case RF_F32: launch_t<float>(a, (int)blocks, st); break;
    case RF_F16: launch_t<__half>(a, (int)blocks, st); break;
    default: launch_t<__nv_bfloat16>(a, (int)blocks, st); break;
  }
  return rf::check_launch("rf_moe_combine_rmsnorm");
}
