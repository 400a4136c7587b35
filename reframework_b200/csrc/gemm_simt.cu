// Grouped expert GEMMs on CUDA cores (FFMA, fp32 accumulation).
//
// Used for the fp32 layer dtype — the tensor-core kinds available on sm_100a
// round fp32 inputs to tf32, which misses a 1e-4 relative tolerance — and for
// 16-bit shapes the TMA path cannot describe (rows not a multiple of 16 B).
// Same contract as the tensor-core kernels: per listed expert e, rows
// [offsets[e], offsets[e] + counts[e]) of `a` times the expert's weights.
// 64x64 output tile per block, 16-deep k-steps through shared memory, each
// thread 4x4 outputs (x2 for the gated kernel, which keeps gate and up tiles).
#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

template <typename T, bool GATED>
__global__ void __launch_bounds__(NT) simt_grouped_gemm(rf::GroupedGemmArgs p) {
  __shared__ float sA[BK][BM + 4];
  __shared__ float sG[BK][BN + 4];
  __shared__ float sU[GATED ? BK : 1][GATED ? BN + 4 : 1];
  const int g = blockIdx.y;
  const int e = p.groups ? p.groups[g] : g;
  if (e < 0 || e >= p.E) {
    if (threadIdx.x == 0) rf_report(RF_DEV_BAD_EXPERT_ID);
    return;
  }
  const int cnt = p.counts[e];
  const int m0 = blockIdx.z * BM;
  if (m0 >= cnt) return;
  const int64_t row0 = (int64_t)p.offsets[e] + m0;
  const int rows = min(BM, cnt - m0);
  const int s = p.slot ? p.slot[e] : e;
  if (s < 0 || s >= p.num_slots) {
    if (threadIdx.x == 0) rf_report(RF_DEV_BAD_EXPERT_ID);
    return;
  }
  const int n0 = blockIdx.x * BN;
  const T *A = reinterpret_cast<const T *>(p.a);
  const int64_t wstride = (int64_t)(GATED ? 2 : 1) * p.N * p.Kdim;
  const T *W = reinterpret_cast<const T *>(p.w) + (int64_t)s * wstride;
  const T *Wu = W + (int64_t)p.N * p.Kdim;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float accg[4][4] = {}, accu[4][4] = {};
  for (int k0 = 0; k0 < p.Kdim; k0 += BK) {
#pragma unroll
    for (int i = 0; i < (BM * BK) / NT; ++i) {
      const int idx = threadIdx.x + i * NT;
      const int r = idx / BK, kk = idx % BK;
      float v = 0.f;
      if (r < rows && k0 + kk < p.Kdim) v = rf::Cvt<T>::to_f(A[(row0 + r) * p.Kdim + k0 + kk]);
      sA[kk][r] = v;
      const int n = r;
      float gv = 0.f, uv = 0.f;
      if (n0 + n < p.N && k0 + kk < p.Kdim) {
        gv = rf::Cvt<T>::to_f(W[(int64_t)(n0 + n) * p.Kdim + k0 + kk]);
        if (GATED) uv = rf::Cvt<T>::to_f(Wu[(int64_t)(n0 + n) * p.Kdim + k0 + kk]);
      }
      sG[kk][n] = gv;
      if (GATED) sU[kk][n] = uv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[4], gv[4], uv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        av[i] = sA[kk][ty * 4 + i];
        gv[i] = sG[kk][tx * 4 + i];
        if (GATED) uv[i] = sU[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          accg[i][j] = fmaf(av[i], gv[j], accg[i][j]);
          if (GATED) accu[i][j] = fmaf(av[i], uv[j], accu[i][j]);
        }
    }
    __syncthreads();
  }
  T *out = reinterpret_cast<T *>(p.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty * 4 + i;
    if (r >= rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tx * 4 + j;
      if (c >= p.N) continue;
      const float v = GATED ? rf::gated_elem<T>(p.act, accg[i][j], accu[i][j]) : accg[i][j];
      out[(row0 + r) * p.N + c] = rf::Cvt<T>::from_f(v);
    }
  }
}

template <bool GATED>
int launch_t(const rf::GroupedGemmArgs &p, cudaStream_t st) {
  const int64_t mt = (p.rows_capacity + BM - 1) / BM;
  if (mt > 65535 || p.n_groups > 65535)
    return rf::fail(RF_ERR_UNSUPPORTED, "CUDA-core grouped GEMM: too many rows or groups");
  dim3 grid((p.N + BN - 1) / BN, p.n_groups, (unsigned)mt);
  switch (p.dtype) {
    case RF_F32: simt_grouped_gemm<float, GATED><<<grid, NT, 0, st>>>(p); break;
    case RF_F16: simt_grouped_gemm<__half, GATED><<<grid, NT, 0, st>>>(p); break;
    default: simt_grouped_gemm<__nv_bfloat16, GATED><<<grid, NT, 0, st>>>(p); break;
  }
  return rf::check_launch("CUDA-core grouped GEMM");
}

}  // namespace

namespace rf {
int launch_simt_grouped_gemm(const GroupedGemmArgs &g, bool gated, cudaStream_t st) {
  if (g.n_groups == 0 || g.rows_capacity == 0) return RF_OK;
  return gated ? launch_t<true>(g, st) : launch_t<false>(g, st);
}
}  // namespace rf
