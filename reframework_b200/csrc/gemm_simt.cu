// Grouped expert GEMMs on CUDA cores (FFMA, fp32 accumulation).
//
// Used for the fp32 layer dtype — the tensor-core kinds available on sm_100a
// round fp32 inputs to tf32, which misses a 1e-4 relative tolerance — and for
// 16-bit shapes the TMA path cannot describe (rows not a multiple of 16 B).
// Same contract as the tensor-core kernels: per listed expert e, rows
// [offsets[e], offsets[e] + counts[e]) of `a` times the expert's weights.
// 64x64 output tile per block, 32-deep k-chunks through shared memory (16-byte
// vector loads, the next chunk fetched into registers while the current one is
// multiplied), each thread 4x4 outputs (x2 for the gated kernel, which keeps
// gate and up tiles).
#include <algorithm>
#include <mutex>
#include <string>
#include <type_traits>

#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int BM = 64, BN = 64, BK = 32, NT = 256;

// Staging of one BK-deep chunk: the A tile (BM rows) and the weight tile(s)
// (BN rows, x2 for the gated kernel) are read with 16-byte vectors along k
// (VEC) or element by element, held raw in registers while the previous chunk
// is multiplied, then stored transposed into shared memory.
template <typename T, bool VEC>
struct Stage {
  static constexpr int E16 = 16 / sizeof(T);            // elements per 16-byte vector
  static constexpr int PER = VEC ? E16 : 1;             // elements per load
  static constexpr int LOADS = (BM * BK) / (NT * PER);  // loads per thread per tile
  using Raw = typename std::conditional<VEC, uint4, float>::type;
  Raw v[LOADS];
  // element (r, kk) of load i of this thread
  static __device__ __forceinline__ void coord(int i, int &r, int &kk) {
    const int idx = threadIdx.x + i * NT;
    r = idx / (BK / PER);
    kk = (idx % (BK / PER)) * PER;
  }
  __device__ __forceinline__ void fetch(const T *base, int64_t ld, int rows, int kbeg, int kdim) {
#pragma unroll
    for (int i = 0; i < LOADS; ++i) {
      int r, kk;
      coord(i, r, kk);
      const int k = kbeg + kk;
      if constexpr (VEC) {
        v[i] = (r < rows && k < kdim) ? __ldg(reinterpret_cast<const uint4 *>(base + r * ld + k))
                                      : make_uint4(0u, 0u, 0u, 0u);
      } else {
        v[i] = (r < rows && k < kdim) ? rf::Cvt<T>::to_f(base[r * ld + k]) : 0.f;
      }
    }
  }
  __device__ __forceinline__ void store(float (*dst)[BM + 1]) const {
#pragma unroll
    for (int i = 0; i < LOADS; ++i) {
      int r, kk;
      coord(i, r, kk);
      if constexpr (VEC) {
        float f[8];
        rf::unpack16<T>(v[i], f);
#pragma unroll
        for (int j = 0; j < PER; ++j) dst[kk + j][r] = f[j];
      } else {
        dst[kk][r] = v[i];
      }
    }
  }
};

// One BM x BN output tile of one expert per block; thread (ty, tx) owns a
// 4 x 4 patch (x2 for gated: gate and up).  Each output is one fp32 FMA chain
// in ascending k.
template <typename T, bool GATED, bool VEC>
__global__ void __launch_bounds__(NT) simt_grouped_gemm(rf::GroupedGemmArgs p) {
  __shared__ float sA[BK][BM + 1];
  __shared__ float sG[BK][BN + 1];
  __shared__ float sU[GATED ? BK : 1][GATED ? BN + 1 : 1];
  static_assert(BM == BN, "staging assumes square tiles");
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
  const int ncols = min(BN, p.N - n0);
  const T *A = reinterpret_cast<const T *>(p.a) + row0 * p.Kdim;
  const int64_t wstride = (int64_t)(GATED ? 2 : 1) * p.N * p.Kdim;
  const T *W = reinterpret_cast<const T *>(p.w) + (int64_t)s * wstride + (int64_t)n0 * p.Kdim;
  const T *Wu = W + (int64_t)p.N * p.Kdim;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float accg[4][4] = {}, accu[4][4] = {};
  Stage<T, VEC> ra, rg, ru;
  ra.fetch(A, p.Kdim, rows, 0, p.Kdim);
  rg.fetch(W, p.Kdim, ncols, 0, p.Kdim);
  if constexpr (GATED) ru.fetch(Wu, p.Kdim, ncols, 0, p.Kdim);
  for (int k0 = 0; k0 < p.Kdim; k0 += BK) {
    ra.store(sA);
    rg.store(sG);
    if constexpr (GATED) ru.store(sU);
    __syncthreads();
    if (k0 + BK < p.Kdim) {
      ra.fetch(A, p.Kdim, rows, k0 + BK, p.Kdim);
      rg.fetch(W, p.Kdim, ncols, k0 + BK, p.Kdim);
      if constexpr (GATED) ru.fetch(Wu, p.Kdim, ncols, k0 + BK, p.Kdim);
    }
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
      float v = GATED ? rf::gated_elem<T>(p.act, accg[i][j], accu[i][j]) : accg[i][j];
      if (!GATED && p.addend)  // a second shared expert adds onto the first: both rounded, summed
        v = rf::Cvt<T>::to_f(reinterpret_cast<const T *>(p.addend)[(row0 + r) * p.N + c]) + rf::round_to<T>(v);
      out[(row0 + r) * p.N + c] = rf::Cvt<T>::from_f(v);
    }
  }
}

// Skinny variant for experts with few rows (decode-sized groups): a block
// covers SN output columns for every row of the expert, SR rows at a time.
// Each warp owns 8 columns and all SR rows: lane (c, rg) = (lane % 8, lane / 8)
// computes column c for the RPT rows rg, rg + 4, rg + 8, ... (interleaved, so the
// four row groups read different banks).  A 3- (gated) or 4-stage (down) cp.async ring streams
// 32-deep k-chunks of the SN weight rows (x2 gated) and of the expert's
// activation rows into shared memory, both kept k-contiguous ([col][k],
// [row][k], padded rows); the multiply reads 16-byte vectors along k.  In one
// warp a weight vector is shared by the 4 row groups and an activation vector
// by the 8 columns (broadcast reads), so per 16-byte step a warp issues
// (1 + gated) + RPT loads for 32 * RPT * (1 + gated) * vector-width FMAs.
// Small blocks (SN = 32, 128 threads, ~41 KB of ring for fp32, at most 102
// registers a thread) give a fine grid: five blocks per SM and a short last
// wave.  Each output is the same
// ascending-k fp32 FMA chain as in the tiled kernel, so the two kernels give
// the same bits.
constexpr int SN = 32, SR = 32, SK = 32;
// ring depth: 3 for the gated kernel (five 41 KB blocks per SM for fp32, one
// wave for C1-sized launches), 4 for the down kernel
template <bool GATED> constexpr int skinny_stages() { return GATED ? 3 : 4; }
constexpr int RPT = 8;                      // rows per thread
constexpr int SRG = SR / RPT;               // row groups (4) = lanes per column
constexpr int SCW = 32 / SRG;               // columns per warp (8)
constexpr int SNT = (SN / SCW) * 32;        // threads per block (128)
static_assert(SRG * RPT == SR && SCW * SRG == 32 && RPT == 8, "skinny lane layout (the NR dispatch covers 1..8)");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
struct SkinnyCfg {
  static constexpr int E16 = 16 / (int)sizeof(T);   // elements per 16-byte vector
  static constexpr int KV = SK / E16;               // vectors per row per chunk
  static constexpr int LD = SK + E16;               // padded row length (elements), 16-byte multiple
  static constexpr int ROW_BYTES = LD * (int)sizeof(T);
};

// The multiply of one staged chunk for NR rows per thread (NR block-uniform:
// rows past the expert's are computed on stale shared memory and never stored),
// branch-free so the compiler interleaves the NR * (1 + gated) FMA chains.
template <typename T, bool GATED, int NR>
__device__ __forceinline__ void skinny_chunk(const uint8_t *wg, const uint8_t *wu, const uint8_t *xs,
                                             float *accg, float *accu) {
  using C = SkinnyCfg<T>;
  // vectors of step kv + 1 are loaded while step kv multiplies (shared-memory
  // latency hidden inside the warp)
  uint4 vg[2], vu[2], vx[2][NR];
  auto load = [&](int kv, int b) {
    vg[b] = *reinterpret_cast<const uint4 *>(wg + kv * 16);
    if constexpr (GATED) vu[b] = *reinterpret_cast<const uint4 *>(wu + kv * 16);
#pragma unroll
    for (int r = 0; r < NR; ++r) vx[b][r] = *reinterpret_cast<const uint4 *>(xs + r * SRG * C::ROW_BYTES + kv * 16);
  };
  load(0, 0);
#pragma unroll
  for (int kv = 0; kv < C::KV; ++kv) {
    const int b = kv & 1;
    if (kv + 1 < C::KV) load(kv + 1, b ^ 1);
    float fg[8], fu[8];
    rf::unpack16<T>(vg[b], fg);
    if constexpr (GATED) rf::unpack16<T>(vu[b], fu);
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float fx[8];
      rf::unpack16<T>(vx[b][r], fx);
#pragma unroll
      for (int j = 0; j < C::E16; ++j) {
        accg[r] = fmaf(fx[j], fg[j], accg[r]);
        if constexpr (GATED) accu[r] = fmaf(fx[j], fu[j], accu[r]);
      }
    }
  }
}

template <typename T, bool GATED>
__global__ void __launch_bounds__(SNT, GATED ? 5 : 1) simt_skinny_gemm(rf::GroupedGemmArgs p) {
  using C = SkinnyCfg<T>;
  constexpr int NW = GATED ? 2 : 1;
  constexpr int STAGE_BYTES = (NW * SN + SR) * C::ROW_BYTES;
  constexpr int SSTAGES = skinny_stages<GATED>();
  constexpr int MAXC = ((NW * SN + SR) * C::KV + SNT - 1) / SNT;  // 16-byte copies per thread per chunk
  extern __shared__ __align__(16) uint8_t s_raw[];
  const int g = blockIdx.y;
  const int e = p.groups ? p.groups[g] : g;
  if (e < 0 || e >= p.E) {
    if (threadIdx.x == 0) rf_report(RF_DEV_BAD_EXPERT_ID);
    return;
  }
  const int cnt = p.counts[e];
  if (cnt <= 0) return;
  const int s = p.slot ? p.slot[e] : e;
  if (s < 0 || s >= p.num_slots) {
    if (threadIdx.x == 0) rf_report(RF_DEV_BAD_EXPERT_ID);
    return;
  }
  const int n0 = blockIdx.x * SN;
  const int lane = threadIdx.x & 31;
  const int c = (threadIdx.x >> 5) * SCW + (lane % SCW), rg = lane / SCW;
  const int64_t wstride = (int64_t)NW * p.N * p.Kdim;
  const T *W = reinterpret_cast<const T *>(p.w) + (int64_t)s * wstride;
  T *out = reinterpret_cast<T *>(p.out);
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(s_raw);
  const int nchunks = (p.Kdim + SK - 1) / SK;
  for (int m0 = 0; m0 < cnt; m0 += SR) {
    const int rows = min(SR, cnt - m0);
    const int nr = (rows + SRG - 1) / SRG;  // rows per thread, the same in the whole block
    const T *A = reinterpret_cast<const T *>(p.a) + ((int64_t)p.offsets[e] + m0) * p.Kdim;
    // this thread's copies of every chunk: rows [0, NW*SN) weights, then the
    // activation rows; the source moves by SK elements per chunk
    const T *csrc[MAXC];
    uint32_t cdst[MAXC];
    int ck[MAXC];  // the copy's first k inside a chunk, or -1 (no copy)
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int v = threadIdx.x + i * SNT;
      const int row = v / C::KV, kv = v % C::KV;
      ck[i] = -1;
      csrc[i] = W;
      cdst[i] = (uint32_t)(row * C::ROW_BYTES + kv * 16);
      if (row < NW * SN) {
        const int m = row / SN, n = n0 + row % SN;
        if (n < p.N) {
          ck[i] = kv * C::E16;
          csrc[i] = W + ((int64_t)m * p.N + n) * p.Kdim + ck[i];
        }
      } else if (row - NW * SN < rows) {
        ck[i] = kv * C::E16;
        csrc[i] = A + (int64_t)(row - NW * SN) * p.Kdim + ck[i];
      }
    }
    auto issue = [&](int q) {
      if (q < nchunks) {
        const int k0 = q * SK;
        const uint32_t st = sbase + (uint32_t)((q % SSTAGES) * STAGE_BYTES);
#pragma unroll
        for (int i = 0; i < MAXC; ++i)
          if (ck[i] >= 0) {
            const bool ok = k0 + ck[i] < p.Kdim;
            cp_async16(st + cdst[i], ok ? csrc[i] + k0 : csrc[i], ok);
          }
      }
      cp_async_commit();  // one group per chunk slot, empty past the end
    };
    float accg[RPT], accu[GATED ? RPT : 1];
#pragma unroll
    for (int r = 0; r < RPT; ++r) accg[r] = 0.f;
#pragma unroll
    for (int r = 0; r < (GATED ? RPT : 1); ++r) accu[r] = 0.f;
#pragma unroll
    for (int q = 0; q < SSTAGES - 1; ++q) issue(q);
    for (int q = 0; q < nchunks; ++q) {
      cp_async_wait<SSTAGES - 2>();
      __syncthreads();  // chunk q landed for every thread; slot (q-1) % SSTAGES is free
      issue(q + SSTAGES - 1);
      const uint8_t *st = s_raw + (q % SSTAGES) * STAGE_BYTES;
      const uint8_t *wg = st + c * C::ROW_BYTES;
      const uint8_t *wu = st + (SN + c) * C::ROW_BYTES;
      const uint8_t *xs = st + (NW * SN + rg) * C::ROW_BYTES;
      switch (nr) {  // block-uniform
        case 1: skinny_chunk<T, GATED, 1>(wg, wu, xs, accg, accu); break;
        case 2: skinny_chunk<T, GATED, 2>(wg, wu, xs, accg, accu); break;
        case 3: skinny_chunk<T, GATED, 3>(wg, wu, xs, accg, accu); break;
        case 4: skinny_chunk<T, GATED, 4>(wg, wu, xs, accg, accu); break;
        case 5: skinny_chunk<T, GATED, 5>(wg, wu, xs, accg, accu); break;
        case 6: skinny_chunk<T, GATED, 6>(wg, wu, xs, accg, accu); break;
        case 7: skinny_chunk<T, GATED, 7>(wg, wu, xs, accg, accu); break;
        default: skinny_chunk<T, GATED, 8>(wg, wu, xs, accg, accu); break;
      }
    }
    cp_async_wait<0>();
    __syncthreads();  // the ring is reused by the next row chunk
    const int n = n0 + c;
    if (n < p.N) {
      T *ocol = out + ((int64_t)p.offsets[e] + m0) * p.N + n;
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int row = rg + r * SRG;
        if (row >= rows) break;
        float v = GATED ? rf::gated_elem<T>(p.act, accg[r], accu[GATED ? r : 0]) : accg[r];
        if (!GATED && p.addend)
          v = rf::Cvt<T>::to_f(reinterpret_cast<const T *>(p.addend)[(ocol - out) + (int64_t)row * p.N]) +
              rf::round_to<T>(v);
        ocol[(int64_t)row * p.N] = rf::Cvt<T>::from_f(v);
      }
    }
  }
}

template <typename T, bool GATED>
int launch_skinny(const rf::GroupedGemmArgs &p, cudaStream_t st) {
  constexpr int NW = GATED ? 2 : 1;
  constexpr size_t smem = (size_t)skinny_stages<GATED>() * (NW * SN + SR) * SkinnyCfg<T>::ROW_BYTES;
  auto kern = simt_skinny_gemm<T, GATED>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    if (smem > 48 * 1024)
      attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr_err != cudaSuccess)
    return rf::fail(RF_ERR_CUDA, std::string("CUDA-core grouped GEMM (skinny): ") + cudaGetErrorString(attr_err));
  dim3 grid((p.N + SN - 1) / SN, p.n_groups);
  kern<<<grid, SNT, smem, st>>>(p);
  return rf::check_launch("CUDA-core grouped GEMM (skinny)");
}

template <bool GATED>
int launch_t(const rf::GroupedGemmArgs &p, cudaStream_t st) {
  const int64_t mt = (p.rows_capacity + BM - 1) / BM;
  if (mt > 65535 || p.n_groups > 65535)
    return rf::fail(RF_ERR_UNSUPPORTED, "CUDA-core grouped GEMM: too many rows or groups");
  dim3 grid((p.N + BN - 1) / BN, p.n_groups, (unsigned)mt);
  // 16-byte vector loads need every row start (and so Kdim * element size)
  // and both base pointers 16-byte aligned
  const bool vec = ((int64_t)p.Kdim * rf::dtype_size(p.dtype)) % 16 == 0 && (uintptr_t)p.a % 16 == 0 &&
                   (uintptr_t)p.w % 16 == 0;
  // few rows per expert (estimated from the row capacity the caller sized for
  // the permute's padding): the skinny kernel
  const int64_t groups = p.n_groups > 0 ? p.n_groups : 1;
  int64_t pairs = p.rows_capacity - groups * 127;
  if (pairs < 1) pairs = std::min<int64_t>(p.rows_capacity, groups);
  if (vec && pairs < groups * 32 && p.N <= 65535 * (int64_t)SN) {
    switch (p.dtype) {
      case RF_F32: return launch_skinny<float, GATED>(p, st);
      case RF_F16: return launch_skinny<__half, GATED>(p, st);
      default: return launch_skinny<__nv_bfloat16, GATED>(p, st);
    }
  }
  switch (p.dtype) {
    case RF_F32:
      if (vec) simt_grouped_gemm<float, GATED, true><<<grid, NT, 0, st>>>(p);
      else simt_grouped_gemm<float, GATED, false><<<grid, NT, 0, st>>>(p);
      break;
    case RF_F16:
      if (vec) simt_grouped_gemm<__half, GATED, true><<<grid, NT, 0, st>>>(p);
      else simt_grouped_gemm<__half, GATED, false><<<grid, NT, 0, st>>>(p);
      break;
    default:
      if (vec) simt_grouped_gemm<__nv_bfloat16, GATED, true><<<grid, NT, 0, st>>>(p);
      else simt_grouped_gemm<__nv_bfloat16, GATED, false><<<grid, NT, 0, st>>>(p);
      break;
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
