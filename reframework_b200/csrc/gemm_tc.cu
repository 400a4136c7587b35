// K3/K4 — grouped expert GEMMs on the sm_100a tensor cores (tcgen05).
//
// Restates the per-expert matmuls of reframework/moe/fused.py:81-83
// (`x @ w1[e].t()`, gated activation, `inter @ w2[e].t()`) as two persistent
// grouped GEMMs over all experts at once:
//   gated: h[r, j] = act(a[r] . w1[s, j]) * (a[r] . w1[s, I + j])
//   down:  y[r, n] = h[r] . w2[s, n]
// for the rows r of every listed expert (s = the expert's weight slot).
//
// Design (one CTA per SM, 320 threads, warp-specialised):
//   warp 0      TMA producer: per 64-deep k-block loads the 128-row A tile
//               and the 256-row B tile (gated: 128 gate rows + the matching
//               128 up rows, so one accumulator holds both halves) into a
//               4-stage shared-memory ring (128-byte swizzle, this CTA only).
//   warp 1      allocates 512 TMEM columns and issues tcgen05.mma (M=128,
//               N=256, K=16, bf16/fp16 in, fp32 accumulate) from one thread;
//               two accumulators (2 x 256 columns) let the epilogue of tile i
//               overlap the main loop of tile i+1.
//   warps 2-9   epilogue: tcgen05.ld of their 32-lane TMEM quadrant (two
//               warps per quadrant, each taking half of the columns), gated
//               activation (compiled per activation), rounding, 16-byte
//               global stores of the valid rows.
// Tiles: per listed expert ceil(count/128) m-blocks x n-blocks, ordered
// n-major / m-minor inside an expert so concurrently running CTAs share the
// weight tile through L2; CTAs stride over the tile list.  The tile table is
// built on the device from expert_counts, so no host synchronisation.
// Every mbarrier wait is bounded (2 s): on expiry the CTA sets the device
// error word, stops issuing, waits for its own in-flight MMAs and copies and
// releases TMEM before returning.
// REMOTE (down GEMM of the expert-parallel layer): the epilogue stores each
// output row straight into the return buffer of the rank that sent the token
// (NVLink peer stores, overlapping the next tile's MMAs), and the last CTA
// raises that exchange's completion flags; see rf::RemoteOut.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();
#include "tc_ptx.cuh"

namespace {

constexpr int BM = 128, BK = 64;
#ifndef RF_EPI_WARPS
#define RF_EPI_WARPS 8
#endif
#ifndef RF_EPI_SLEEP_NS
#define RF_EPI_SLEEP_NS 256
#endif
constexpr int EPI_WARPS = RF_EPI_WARPS;  // 4 or 8: one or two per TMEM lane quadrant
constexpr int EPI_SPLIT = EPI_WARPS / 4;  // warps sharing a quadrant's columns
static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
constexpr int NTHREADS = 32 * (2 + EPI_WARPS);
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int BM_SMALL = 32;          // A rows loaded for a tile with at most 32 valid rows
constexpr int MAX_GROUPS = 1024;

// Per tile width BN (the MMA's N: 256, 128 or 64).  Narrower tiles give more
// tiles (better balance over 148 SMs when there are few rows, as in decode)
// and, with the same ~192 KB ring, deeper pipelines; wider tiles read less
// per FLOP.  TMEM holds two BN-column fp32 accumulators.
template <int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 6 : 8;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int NUM_BARS = 2 * STAGES + 5;  // full, empty, tmem full x2, tmem empty x2, drain
  static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + NUM_BARS * 8 + 16 +
                                       (size_t)(MAX_GROUPS + 1) * 4 + (size_t)3 * MAX_GROUPS * 4;
  static_assert(BN == 256 || BN == 128 || BN == 64, "tile width");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

struct TcArgs {
  const int32_t *offsets, *counts, *slot, *groups;  // offsets == counts == NULL: one dense group
  int n_groups, E, num_slots;
  int dense_rows; // rows of the dense group
  // dense fp32-output mode: K cut into k_slices fixed slices of kb_per_slice
  // k-blocks, one tile each, slice j's sums written at out + j * slice_stride
  // (0 or 1 = no slicing)
  int k_slices, kb_per_slice;
  int64_t slice_stride;
  int Kdim;       // reduction length
  int N;          // output columns
  int n_tiles_n;  // n-blocks per expert
  void *out;
  int64_t out_ld; // output row stride (elements)
  int act;
  // gather mode: A row r of the permuted layout is row gather_src[r] / gather_div
  // of the tensor behind the A map (the token's activation row); -1 = pad row
  const int32_t *gather_src;
  int gather_div;
  const void *addend;  // down only: out = round(addend + round(acc)); may be NULL or out
  // int8 mode (T = int8_t, kind::i8, exact int32 sums; the expert split):
  // dequantize with a_scales[listed position] * w_scales[expert * w_stride];
  // gated: fp32 act(g) * u, per-listed-expert max |.| into i8_amax; down:
  // times the routing weight row_w[src_slot[row]]; fp32 output rows
  const float *i8_as, *i8_ws;
  int64_t i8_wstride;
  float *i8_amax;
  const float *i8_rw;
  const int32_t *i8_src;
};

// Instruction descriptor of kind::f16: fp32 accumulator, A/B K-major,
// M = 128, N = BN; operand format 0 = f16, 1 = bf16 (A and B always equal).
template <typename T, int BN>
__host__ __device__ constexpr uint32_t instr_desc() {
  if constexpr (std::is_same<T, int8_t>::value)  // kind::i8: s32 accumulator, signed 8-bit A and B
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  return (1u << 4) | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7) |
         ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

struct NoRemote {};

__device__ __forceinline__ void st_release_sys_u32(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// OUTF32 (down kernel only): the accumulator is stored as fp32, unrounded.
// GATHER: A rows are fetched from the token rows with TMA gather4 (no
// expert-ordered activation copy in HBM).
// REMOTE (down kernel only): rows go to the peers' return buffers (ro).
template <typename T, bool GATED, int ACT, int BN_, bool OUTF32 = false, bool GATHER = false,
          bool REMOTE = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_grouped_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA32,
                    const __grid_constant__ CUtensorMap tmB, const TcArgs p,
                    const __grid_constant__ std::conditional_t<REMOTE, rf::RemoteOut, NoRemote> ro) {
  static_assert(!REMOTE || (!GATED && !OUTF32 && !GATHER), "remote stores: plain down GEMM only");
  constexpr bool I8 = std::is_same<T, int8_t>::value;
  static_assert(!I8 || (!OUTF32 && !GATHER && !REMOTE), "int8 mode: grouped gated / down only");
  constexpr int BKE = I8 ? 2 * BK : BK;  // k-block depth in elements: 128 bytes of a row either way
  using C = Cfg<BN_>;
  constexpr int BN = C::BN, STAGES = C::STAGES, B_BYTES = C::B_BYTES, STAGE_BYTES = C::STAGE_BYTES;
  constexpr int NUM_BARS = C::NUM_BARS;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + STAGES * B_BYTES);
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + NUM_BARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int *tile_prefix = reinterpret_cast<int *>(tmem_holder + 4);  // [G+1]
  int *g_row0 = tile_prefix + MAX_GROUPS + 1;                      // [G]
  int *g_cnt = g_row0 + MAX_GROUPS;                                // [G]
  int *g_slot = g_cnt + MAX_GROUPS;                                // [G]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.n_groups;
  const uint32_t bar0 = smem_u32(bars);
#define FULL(s) (bar0 + 8u * (uint32_t)(s))
#define EMPTY(s) (bar0 + 8u * (uint32_t)(STAGES + (s)))
#define TFULL(a) (bar0 + 8u * (uint32_t)(2 * STAGES + (a)))
#define TEMPTY(a) (bar0 + 8u * (uint32_t)(2 * STAGES + 2 + (a)))
  const uint32_t DRAIN = bar0 + 8u * (uint32_t)(2 * STAGES + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(FULL(s), 1);
      mbar_init(EMPTY(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(TFULL(a), 1);
      mbar_init(TEMPTY(a), EPI_WARPS);  // one arrival per epilogue warp
    }
    mbar_init(DRAIN, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA32) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
  }
  // per-group table: first row, row count, weight slot, tile count
  for (int g = threadIdx.x; g < G; g += NTHREADS) {
    int e = p.groups ? p.groups[g] : g;
    int tiles = 0, row0 = 0, cnt = 0, s = 0;
    if (e >= 0 && e < p.E) {
      s = p.slot ? p.slot[e] : e;
      if (s >= 0 && s < p.num_slots) {
        row0 = p.offsets ? p.offsets[e] : 0;
        cnt = p.counts ? p.counts[e] : p.dense_rows;
        tiles = ((cnt + BM - 1) / BM) * p.n_tiles_n;
      } else {
        rf_report(RF_DEV_BAD_EXPERT_ID);
      }
    } else {
      rf_report(RF_DEV_BAD_EXPERT_ID);
    }
    g_row0[g] = row0;
    g_cnt[g] = tiles ? cnt : 0;
    g_slot[g] = s;
    tile_prefix[g + 1] = tiles;
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  if (warp == 2) {  // inclusive scan of tile counts -> tile_prefix
    int carry = 0;
    for (int c = 0; c < G; c += 32) {
      int v = (c + lane < G) ? tile_prefix[c + lane + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (c + lane < G) tile_prefix[c + lane + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) tile_prefix[0] = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int base_total = tile_prefix[G];
  const int nsl = p.k_slices > 1 ? p.k_slices : 1;
  const int total = base_total * nsl;
  const int num_kb = (p.Kdim + BKE - 1) / BKE;
  const int kps = nsl > 1 ? p.kb_per_slice : num_kb;
  // tile t -> (tile of the group table, its k-block range, output offset)
  auto kspan = [&](int t, int &tt, int &kb0, int &kb1, int64_t &obase) {
    const int sl = nsl > 1 ? t / base_total : 0;
    tt = t - sl * base_total;
    kb0 = sl * kps;
    kb1 = min(num_kb, kb0 + kps);
    obase = (int64_t)sl * p.slice_stride;
  };

  // tile -> (group, n-block, m-block); groups with zero tiles are skipped by
  // taking the last group whose prefix is <= t
  int gi = 0;  // group of the tile decode() last looked at
  auto decode = [&](int t, int &row0, int &rows, int &nb, int &s) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile_prefix[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    const int cnt = g_cnt[lo];
    const int mt = (cnt + BM - 1) / BM;
    const int local = t - tile_prefix[lo];
    nb = local / mt;
    const int mb = local - nb * mt;
    row0 = g_row0[lo] + mb * BM;
    rows = min(BM, cnt - mb * BM);
    s = g_slot[lo];
    gi = lo;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // lane 0 waits for a free stage, posts the expected bytes and issues the
    // B (and, without gather, the A) copies; in gather mode lane i then
    // fetches A rows 4i..4i+3 of the tile with one gather4
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    // without gather only lane 0 works (no per-k-block warp shuffle)
    for (int t = blockIdx.x; t < total && ok && (GATHER || lane == 0); t += gridDim.x) {
      int row0, rows, nb, s, tt, kb0, kb1;
      int64_t obase;
      kspan(t, tt, kb0, kb1, obase);
      decode(tt, row0, rows, nb, s);
      int src[4] = {0, 0, 0, 0};
      int groups4 = 0;
      if (GATHER) {
        groups4 = (rows + 3) >> 2;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = 4 * lane + j;
          const int sl = r < rows ? p.gather_src[row0 + r] : -1;
          src[j] = sl >= 0 ? sl / p.gather_div : 0;  // pad rows read token 0; never stored
        }
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        int go = 1;
        if (lane == 0) go = mbar_wait(EMPTY(stage), phase ^ 1u, abort_flag) ? 1 : 0;
        if constexpr (GATHER) go = __shfl_sync(0xffffffffu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        const uint32_t a_dst = smem_u32(sA + stage * A_BYTES);
        const uint32_t b_dst = smem_u32(sB + stage * B_BYTES);
        if (lane == 0) {
          // a tile of at most 32 valid rows loads only those rows; the MMA
          // still reads 128 (rows past the tile's count are never stored)
          const bool small = rows <= BM_SMALL;
          const uint32_t a_bytes =
              GATHER ? (uint32_t)groups4 * 512u : (small ? (uint32_t)(A_BYTES / (BM / BM_SMALL)) : (uint32_t)A_BYTES);
          mbar_expect_tx(FULL(stage), a_bytes + (uint32_t)B_BYTES);
          if (!GATHER) tma_load_2d(a_dst, small ? &tmA32 : &tmA, FULL(stage), kb * BKE, row0);
          if (GATED) {
            tma_load_3d(b_dst, &tmB, FULL(stage), kb * BKE, nb * (BN / 2), 2 * s);
            tma_load_3d(b_dst + B_BYTES / 2, &tmB, FULL(stage), kb * BKE, nb * (BN / 2), 2 * s + 1);
          } else {
            tma_load_3d(b_dst, &tmB, FULL(stage), kb * BKE, nb * BN, s);
          }
        }
        if (GATHER) {
          __syncwarp();
          if (lane < groups4)
            tma_gather4(a_dst + (uint32_t)lane * 512u, &tmA, FULL(stage), kb * BK, src[0], src[1], src[2], src[3]);
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && lane == 0) {
      // let the copies already issued land before the CTA can exit
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int j = first; j < issued; ++j)
        mbar_wait_teardown(FULL(j % STAGES), (uint32_t)((j / STAGES) & 1));
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = instr_desc<T, BN>();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        int tt, kb0, kb1;
        int64_t obase;
        kspan(t, tt, kb0, kb1, obase);
        const int acc = it & 1;
        const uint32_t aph = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait(TEMPTY(acc), aph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(FULL(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 32-byte steps: K = 16 (16-bit) or 32 (int8) per MMA
            if constexpr (I8)
              tc_mma_i8(d, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), IDESC, (kb != kb0 || k) ? 1u : 0u);
            else
              tc_mma(d, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), IDESC, (kb != kb0 || k) ? 1u : 0u);
          }
          tc_commit(EMPTY(stage));  // frees the stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) tc_commit(TFULL(acc));
      }
      // no MMA may still be running when TMEM is released
      tc_commit(DRAIN);
      mbar_wait_teardown(DRAIN, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;             // TMEM lane quadrant this warp may access
    const int part = (warp - 2) >> 2;    // which share of the columns it stores
    const int r = wq * 32 + lane;
    T *out = reinterpret_cast<T *>(p.out);
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      int row0, rows, nb, s, tt, kb0, kb1;
      int64_t obase;
      kspan(t, tt, kb0, kb1, obase);
      decode(tt, row0, rows, nb, s);
      const int acc = it & 1;
      const uint32_t aph = (uint32_t)((it >> 1) & 1);
      // one lane waits, the warp re-converges on the broadcast before the
      // warp-collective (.sync.aligned) TMEM loads
      int ok = 1;
      if (lane == 0) ok = mbar_wait(TFULL(acc), aph, abort_flag, RF_EPI_SLEEP_NS) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(wq * 32) << 16) + (uint32_t)(acc * BN);
      const bool row_ok = r < rows;
      T *orow = out + (int64_t)(row0 + r) * p.out_ld;
      if constexpr (REMOTE) {
        if (row_ok) {  // source rank of local row k of slot s, and its row there
          const int64_t k = (int64_t)(row0 + r) - g_row0[s];
          const int64_t *cj = ro.cj + (int64_t)s * (ro.R + 1);
          int lo = 0, hi = ro.R - 1;
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (cj[mid] <= k) lo = mid;
            else hi = mid - 1;
          }
          orow = reinterpret_cast<T *>(ro.dst[lo]) + (ro.ps[(int64_t)lo * ro.S + s] + (k - cj[lo])) * p.out_ld;
        }
      }
      if constexpr (I8) {
        const int e = p.groups ? p.groups[gi] : gi;
        const float dq = __fmul_rn(p.i8_as[gi], p.i8_ws[(int64_t)e * p.i8_wstride]);
        float *orowf = reinterpret_cast<float *>(p.out) + (int64_t)(row0 + r) * p.out_ld;
        const float rw = (!GATED && row_ok) ? p.i8_rw[p.i8_src[row0 + r]] : 0.f;
        float m = 0.f;
        const int n0 = GATED ? nb * (BN / 2) : nb * BN;
#pragma unroll 1
        for (int c = part * 32; c < (GATED ? BN / 2 : BN); c += 32 * EPI_SPLIT) {
          uint32_t g[32], u[32];
          tmem_ld32(tb + c, g);
          if (GATED) tmem_ld32(tb + BN / 2 + c, u);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const int col = n0 + c + 4 * v;
              if (col >= p.N) continue;
              float o[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float gf = __fmul_rn(__int2float_rn((int)g[4 * v + i]), dq);
                if (GATED) {
                  const float uf = __fmul_rn(__int2float_rn((int)u[4 * v + i]), dq);
                  o[i] = __fmul_rn(rf::act_ieee(ACT, gf), uf);
                  m = fmaxf(m, fabsf(o[i]));
                } else {
                  o[i] = __fmul_rn(gf, rw);
                }
              }
              *reinterpret_cast<float4 *>(orowf + col) = make_float4(o[0], o[1], o[2], o[3]);
            }
          }
        }
        if (GATED) {  // per listed expert max |inter| (non-negative floats order like their bits)
#pragma unroll
          for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0 && m > 0.f) atomicMax(reinterpret_cast<int *>(p.i8_amax) + gi, __float_as_int(m));
        }
      } else if (GATED) {
        const int n0 = nb * (BN / 2);
#pragma unroll 1
        for (int c = part * 32; c < BN / 2; c += 32 * EPI_SPLIT) {
          uint32_t g[32], u[32];
          tmem_ld32(tb + c, g);
          tmem_ld32(tb + BN / 2 + c, u);
          tmem_ld_wait();
          if (row_ok) {
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float h0 = rf::gated_elem_t<T, ACT>(__uint_as_float(g[2 * j]), __uint_as_float(u[2 * j]));
              const float h1 =
                  rf::gated_elem_t<T, ACT>(__uint_as_float(g[2 * j + 1]), __uint_as_float(u[2 * j + 1]));
              pk[j] = rf::pack2<T>(h0, h1);
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = n0 + c + 8 * v;
              if (col < p.N)
                *reinterpret_cast<uint4 *>(orow + col) =
                    make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
            }
          }
        }
      } else if (OUTF32) {
        // fp32 rows of out_ld (a multiple of 4) columns; columns in
        // [N, out_ld) hold the zero products of the out-of-range weight rows
        const int n0 = nb * BN;
        float *orowf = reinterpret_cast<float *>(p.out) + obase + (int64_t)(row0 + r) * p.out_ld;
#pragma unroll 1
        for (int c = part * 32; c < BN; c += 32 * EPI_SPLIT) {
          uint32_t v32[32];
          tmem_ld32(tb + c, v32);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const int col = n0 + c + 4 * v;
              if (col < p.out_ld)
                *reinterpret_cast<uint4 *>(orowf + col) =
                    make_uint4(v32[4 * v], v32[4 * v + 1], v32[4 * v + 2], v32[4 * v + 3]);
            }
          }
        }
      } else {
        const int n0 = nb * BN;
#pragma unroll 1
        for (int c = part * 32; c < BN; c += 32 * EPI_SPLIT) {
          uint32_t v32[32];
          tmem_ld32(tb + c, v32);
          tmem_ld_wait();
          if (row_ok) {
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
              pk[j] = rf::pack2<T>(__uint_as_float(v32[2 * j]), __uint_as_float(v32[2 * j + 1]));
            if (!REMOTE && p.addend) {  // a second shared expert adds onto the first
              const T *arow = reinterpret_cast<const T *>(p.addend) + (int64_t)(row0 + r) * p.out_ld;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const int col = n0 + c + 8 * v;
                if (col >= p.N) continue;
                float yf[8], af[8];
                rf::unpack16<T>(make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]), yf);
                rf::unpack16<T>(*reinterpret_cast<const uint4 *>(arow + col), af);
#pragma unroll
                for (int i = 0; i < 4; ++i) pk[4 * v + i] = rf::pack2<T>(af[2 * i] + yf[2 * i], af[2 * i + 1] + yf[2 * i + 1]);
              }
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = n0 + c + 8 * v;
              if (col < p.N)
                *reinterpret_cast<uint4 *>(orow + col) =
                    make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(TEMPTY(acc));
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if constexpr (REMOTE) {
    if (threadIdx.x == 0) {
      __threadfence_system();  // this CTA's peer stores, visible to every GPU, before the count
      const uint32_t prev = atomicAdd(ro.done, 1u);
      if (prev == gridDim.x - 1) {  // last CTA: every row of the launch has landed
        __threadfence_system();
        for (int d = 0; d < ro.R; ++d) st_release_sys_u32(ro.flag[d], ro.epoch);
        *ro.done = 0u;
      }
    }
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
}

// ----------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 0 = auto (CTA-pair tensor-core kernel where it applies), 1 = CUDA cores only,
// 2/3/4 = single-CTA tensor-core kernel with BN 256/128/64, 5 = CTA pairs
int g_gemm_impl = 0;

bool encode(CUtensorMap *m, int dtype, int rank, const void *base, const cuuint64_t *dims,
            const cuuint64_t *strides, const cuuint32_t *box) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};  // element strides, one per dimension (rank <= 5)
  const CUtensorMapDataType dt = dtype == RF_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dtype == RF_F16  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_UINT8;  // int8 codes: plain bytes
  CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, bool GATED, int ACT, int BN, bool GATHER = false, bool REMOTE = false>
int launch_tc_t(const rf::GroupedGemmArgs &g, const CUtensorMap &ma, const CUtensorMap &ma32,
                const CUtensorMap &mb, cudaStream_t st) {
  using C = Cfg<BN>;
  auto kern = tc_grouped_gemm<T, GATED, ACT, BN, false, GATHER, REMOTE>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess)
    return rf::fail(RF_ERR_CUDA, std::string("tensor-core GEMM: ") + cudaGetErrorString(attr_err));
  TcArgs p;
  p.offsets = g.offsets;
  p.counts = g.counts;
  p.slot = g.slot;
  p.groups = g.groups;
  p.n_groups = g.n_groups;
  p.E = g.E;
  p.num_slots = g.num_slots;
  p.Kdim = g.Kdim;
  p.N = g.N;
  p.n_tiles_n = GATED ? (g.N + BN / 2 - 1) / (BN / 2) : (g.N + BN - 1) / BN;
  p.out = g.out;
  p.out_ld = g.N;
  p.dense_rows = 0;
  p.k_slices = 1;
  p.kb_per_slice = 0;
  p.slice_stride = 0;
  p.act = g.act;
  p.gather_src = g.gather_src;
  p.gather_div = g.gather_div;
  p.addend = GATED ? nullptr : g.addend;
  if constexpr (REMOTE) {
    kern<<<rf::num_sms(), NTHREADS, C::SMEM_BYTES, st>>>(ma, ma32, mb, p, *g.remote);
    return rf::check_launch("tensor-core down GEMM with peer stores");
  } else {
    kern<<<rf::num_sms(), NTHREADS, C::SMEM_BYTES, st>>>(ma, ma32, mb, p, NoRemote{});
    return rf::check_launch(GATED ? "tensor-core gated GEMM" : "tensor-core down GEMM");
  }
}

template <typename T, int BN>
int launch_tc_bn(const rf::GroupedGemmArgs &g, bool gated, const CUtensorMap &ma, const CUtensorMap &ma32,
                 const CUtensorMap &mb, cudaStream_t st) {
  if (!gated) {
    if (g.remote) return launch_tc_t<T, false, 0, BN, false, true>(g, ma, ma32, mb, st);
    return launch_tc_t<T, false, 0, BN>(g, ma, ma32, mb, st);
  }
  if (g.gather_src) {
    if (g.act == RF_ACT_SILU) return launch_tc_t<T, true, RF_ACT_SILU, BN, true>(g, ma, ma32, mb, st);
    if (g.act == RF_ACT_GELU) return launch_tc_t<T, true, RF_ACT_GELU, BN, true>(g, ma, ma32, mb, st);
    return launch_tc_t<T, true, RF_ACT_GELU_TANH, BN, true>(g, ma, ma32, mb, st);
  }
  if (g.act == RF_ACT_SILU) return launch_tc_t<T, true, RF_ACT_SILU, BN>(g, ma, ma32, mb, st);
  if (g.act == RF_ACT_GELU) return launch_tc_t<T, true, RF_ACT_GELU, BN>(g, ma, ma32, mb, st);
  return launch_tc_t<T, true, RF_ACT_GELU_TANH, BN>(g, ma, ma32, mb, st);
}

template <typename T>
int launch_tc_dt(const rf::GroupedGemmArgs &g, bool gated, int bn, const CUtensorMap &ma,
                 const CUtensorMap &ma32, const CUtensorMap &mb, cudaStream_t st) {
  if (bn == 256) return launch_tc_bn<T, 256>(g, gated, ma, ma32, mb, st);
  if (bn == 128) return launch_tc_bn<T, 128>(g, gated, ma, ma32, mb, st);
  return launch_tc_bn<T, 64>(g, gated, ma, ma32, mb, st);
}

// Tile width of one launch.  The per-expert row counts live on the device,
// so the host estimates the routed pairs from the row capacity minus the
// permute's padding allowance.  With many rows per group the widest tile
// wins clearly (measured on B200: narrower tiles read more bytes per FLOP and
// the kernel is then bound by L2->SM bandwidth); with few rows per group
// (decode) the launch streams weights and twice the tiles balance better over
// the SMs, so N = 128.
int pick_bn(const rf::GroupedGemmArgs &g, bool gated) {
  (void)gated;
  if (g_gemm_impl >= 2 && g_gemm_impl <= 4) return g_gemm_impl == 2 ? 256 : g_gemm_impl == 3 ? 128 : 64;
  const int64_t groups = std::max(1, g.n_groups);
  int64_t pairs = g.rows_capacity - groups * (BM - 1);
  if (pairs < 1) pairs = std::min<int64_t>(g.rows_capacity, groups);
  return pairs < groups * 64 ? 128 : 256;
}

// Returns 1 if the tensor-core path took the call (status in *rc), 0 if the
// shape or dtype is outside what it handles (the CUDA-core kernel runs then).
int try_tc(const rf::GroupedGemmArgs &g, bool gated, cudaStream_t st, int *rc) {
  if (g_gemm_impl == 1) return 0;
  if (g_gemm_impl == 0 || g_gemm_impl == 5) {
    const int prc = rf::launch_pair_grouped_gemm(g, gated, st);
    if (prc >= 0) {
      *rc = prc;
      return 1;
    }
  }
  if (g.dtype != RF_BF16 && g.dtype != RF_F16) return 0;
  if (g.Kdim % 8 || g.N % 8 || g.n_groups > MAX_GROUPS) return 0;
  if ((uintptr_t)g.a % 16 || (uintptr_t)g.w % 16 || (uintptr_t)g.out % 16) return 0;
  *rc = RF_OK;
  if (!encode_fn()) {
    *rc = rf::fail(RF_ERR_CUDA, "tensor-core GEMM: cuTensorMapEncodeTiled is unavailable");
    return 1;
  }
  const int bn = pick_bn(g, gated);
  CUtensorMap ma, ma32, mb;
  bool ok;
  if (g.gather_src) {
    // token rows, fetched four at a time (box: 64 columns x 1 row)
    const cuuint64_t dA[2] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.a_rows};
    const cuuint64_t sAs[1] = {(cuuint64_t)g.Kdim * 2};
    const cuuint32_t bA1[2] = {BK, 1};
    ok = encode(&ma, g.dtype, 2, g.a, dA, sAs, bA1);
    ma32 = ma;
  } else {
    const cuuint64_t dA[2] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.rows_capacity};
    const cuuint64_t sAs[1] = {(cuuint64_t)g.Kdim * 2};
    const cuuint32_t bA[2] = {BK, BM};
    const cuuint32_t bA32[2] = {BK, BM_SMALL};
    ok = encode(&ma, g.dtype, 2, g.a, dA, sAs, bA) && encode(&ma32, g.dtype, 2, g.a, dA, sAs, bA32);
  }
  if (gated) {
    // w1 [S, 2N, K] viewed as [2S][N][K]: half 0 = gate rows, half 1 = up rows
    const cuuint64_t dB[3] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.N, (cuuint64_t)(2 * g.num_slots)};
    const cuuint64_t sB[2] = {(cuuint64_t)g.Kdim * 2, (cuuint64_t)g.N * g.Kdim * 2};
    const cuuint32_t bB[3] = {BK, (cuuint32_t)(bn / 2), 1};
    ok = ok && encode(&mb, g.dtype, 3, g.w, dB, sB, bB);
  } else {
    const cuuint64_t dB[3] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.N, (cuuint64_t)g.num_slots};
    const cuuint64_t sB[2] = {(cuuint64_t)g.Kdim * 2, (cuuint64_t)g.N * g.Kdim * 2};
    const cuuint32_t bB[3] = {BK, (cuuint32_t)bn, 1};
    ok = ok && encode(&mb, g.dtype, 3, g.w, dB, sB, bB);
  }
  if (!ok) {
    *rc = rf::fail(RF_ERR_CUDA, "tensor-core GEMM: cuTensorMapEncodeTiled rejected the operands");
    return 1;
  }
  if (g.dtype == RF_BF16)
    *rc = launch_tc_dt<__nv_bfloat16>(g, gated, bn, ma, ma32, mb, st);
  else
    *rc = launch_tc_dt<__half>(g, gated, bn, ma, ma32, mb, st);
  return 1;
}

template <typename T, int BN>
int launch_dense(const CUtensorMap &ma, const CUtensorMap &ma32, const CUtensorMap &mb, const TcArgs &p,
                 int64_t M, cudaStream_t st) {
  using C = Cfg<BN>;
  auto kern = tc_grouped_gemm<T, false, 0, BN, true>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess)
    return rf::fail(RF_ERR_CUDA, std::string("tensor-core GEMM: ") + cudaGetErrorString(attr_err));
  const int64_t tiles = (M + BM - 1) / BM * p.n_tiles_n * std::max(1, p.k_slices);
  const int grid = (int)std::min<int64_t>(tiles, rf::num_sms());
  kern<<<grid, NTHREADS, C::SMEM_BYTES, st>>>(ma, ma32, mb, p, NoRemote{});
  return rf::check_launch("tensor-core dense GEMM (fp32 out)");
}

}  // namespace

namespace rf {
bool tma_encode(CUtensorMap *m, int dtype, int rank, const void *base, const cuuint64_t *dims,
                const cuuint64_t *strides, const cuuint32_t *box) {
  return encode(m, dtype, rank, base, dims, strides, box);
}
int gemm_impl() { return g_gemm_impl; }

// out[m, n] = sum_k a[m, k] * w[n, k] for m < M, n < N, fp32 accumulation
// on the tensor cores, stored unrounded as fp32 rows of ld_out (a multiple of
// 4, >= N) columns.  a [M, K] and w [N, K] are 16-bit of the same dtype.
// Returns -1 when the tensor-core path does not take the shape (the caller
// then runs its CUDA-core code), else a status.  Each output is one fixed
// sequence of MMAs over k, independent of M and of the other rows.
int tc_dense_f32(const void *a, const void *w, float *out, int64_t M, int64_t N, int64_t Kdim,
                 int64_t ld_out, int dtype, cudaStream_t st, int64_t slice_k) {
  if (g_gemm_impl == 1) return -1;
  if (dtype != RF_BF16 && dtype != RF_F16) return -1;
  if (M <= 0 || N <= 0 || Kdim % 8 || ld_out % 4 || ld_out < N || M >= ((int64_t)1 << 31) ||
      Kdim >= (1 << 30) || N >= (1 << 30))
    return -1;
  if ((uintptr_t)a % 16 || (uintptr_t)w % 16 || (uintptr_t)out % 16) return -1;
  if (!encode_fn()) return rf::fail(RF_ERR_CUDA, "tensor-core GEMM: cuTensorMapEncodeTiled is unavailable");
  const int bn = N <= 64 ? 64 : N <= 128 ? 128 : 256;
  CUtensorMap ma, ma32, mb;
  const cuuint64_t dA[2] = {(cuuint64_t)Kdim, (cuuint64_t)M};
  const cuuint64_t sAs[1] = {(cuuint64_t)Kdim * 2};
  const cuuint32_t bA[2] = {BK, BM};
  const cuuint32_t bA32[2] = {BK, BM_SMALL};
  const cuuint64_t dB[3] = {(cuuint64_t)Kdim, (cuuint64_t)N, 1};
  const cuuint64_t sB[2] = {(cuuint64_t)Kdim * 2, (cuuint64_t)N * Kdim * 2};
  const cuuint32_t bB[3] = {BK, (cuuint32_t)bn, 1};
  if (!(encode(&ma, dtype, 2, a, dA, sAs, bA) && encode(&ma32, dtype, 2, a, dA, sAs, bA32) &&
        encode(&mb, dtype, 3, w, dB, sB, bB)))
    return rf::fail(RF_ERR_CUDA, "tensor-core GEMM: cuTensorMapEncodeTiled rejected the operands");
  TcArgs p{};
  p.n_groups = 1;
  p.E = 1;
  p.num_slots = 1;
  p.dense_rows = (int)M;
  p.Kdim = (int)Kdim;
  p.N = (int)N;
  p.n_tiles_n = (int)((N + bn - 1) / bn);
  p.out = out;
  p.out_ld = ld_out;
  p.act = 0;
  if (slice_k > 0) {  // fixed slices of K, each a tile of its own; sums at out + j * M * ld_out
    if (slice_k % BK) return -1;
    p.kb_per_slice = (int)(slice_k / BK);
    p.k_slices = (int)((Kdim + slice_k - 1) / slice_k);
    p.slice_stride = M * ld_out;
  }
  if (dtype == RF_BF16) {
    if (bn == 64) return launch_dense<__nv_bfloat16, 64>(ma, ma32, mb, p, M, st);
    if (bn == 128) return launch_dense<__nv_bfloat16, 128>(ma, ma32, mb, p, M, st);
    return launch_dense<__nv_bfloat16, 256>(ma, ma32, mb, p, M, st);
  }
  if (bn == 64) return launch_dense<__half, 64>(ma, ma32, mb, p, M, st);
  if (bn == 128) return launch_dense<__half, 128>(ma, ma32, mb, p, M, st);
  return launch_dense<__half, 256>(ma, ma32, mb, p, M, st);
}

// The int8 grouped GEMMs of the expert split on the tensor cores
// (tcgen05.mma kind::i8, exact int32 sums), same contract as the CUDA-core
// kernel of int8_split.cu; -1 when the shape is not handled here.
int tc_int8_grouped_gemm(const int8_t *a, const int8_t *w, const int32_t *offsets, const int32_t *counts,
                         const int32_t *groups, const int32_t *slot, int n_groups, int E, int num_slots,
                         int64_t rows_capacity, int64_t Kdim, int64_t N, const float *a_scales,
                         const float *w_scales, int64_t w_stride, bool gated, int act, float *out, float *amax,
                         const float *row_w, const int32_t *src_slot, cudaStream_t st) {
  if (g_gemm_impl == 1) return -1;
  if (Kdim % 16 || N % 8 || n_groups < 1 || n_groups > MAX_GROUPS || rows_capacity < 1 ||
      rows_capacity >= ((int64_t)1 << 31) || Kdim >= (1 << 30) || N >= (1 << 30))
    return -1;
  if ((uintptr_t)a % 16 || (uintptr_t)w % 16 || (uintptr_t)out % 16) return -1;
  if (!encode_fn()) return -1;
  constexpr int I8D = -1;  // encode(): any code other than the 16-bit ones maps to 8-bit bytes
  const int64_t groups_est = std::max(1, n_groups);
  const int bn = rows_capacity - groups_est * (BM - 1) < groups_est * 64 ? 128 : 256;
  CUtensorMap ma, ma32, mb;
  const cuuint64_t dA[2] = {(cuuint64_t)Kdim, (cuuint64_t)rows_capacity};
  const cuuint64_t sAs[1] = {(cuuint64_t)Kdim};
  const cuuint32_t bA[2] = {2 * BK, BM};
  const cuuint32_t bA32[2] = {2 * BK, BM_SMALL};
  bool ok = encode(&ma, I8D, 2, a, dA, sAs, bA) && encode(&ma32, I8D, 2, a, dA, sAs, bA32);
  if (gated) {
    const cuuint64_t dB[3] = {(cuuint64_t)Kdim, (cuuint64_t)N, (cuuint64_t)(2 * num_slots)};
    const cuuint64_t sB[2] = {(cuuint64_t)Kdim, (cuuint64_t)N * Kdim};
    const cuuint32_t bB[3] = {2 * BK, (cuuint32_t)(bn / 2), 1};
    ok = ok && encode(&mb, I8D, 3, w, dB, sB, bB);
  } else {
    const cuuint64_t dB[3] = {(cuuint64_t)Kdim, (cuuint64_t)N, (cuuint64_t)num_slots};
    const cuuint64_t sB[2] = {(cuuint64_t)Kdim, (cuuint64_t)N * Kdim};
    const cuuint32_t bB[3] = {2 * BK, (cuuint32_t)bn, 1};
    ok = ok && encode(&mb, I8D, 3, w, dB, sB, bB);
  }
  if (!ok) return -1;
  TcArgs p{};
  p.offsets = offsets;
  p.counts = counts;
  p.slot = slot;
  p.groups = groups;
  p.n_groups = n_groups;
  p.E = E;
  p.num_slots = num_slots;
  p.Kdim = (int)Kdim;
  p.N = (int)N;
  p.n_tiles_n = gated ? (int)((N + bn / 2 - 1) / (bn / 2)) : (int)((N + bn - 1) / bn);
  p.out = out;
  p.out_ld = N;
  p.act = act;
  p.i8_as = a_scales;
  p.i8_ws = w_scales;
  p.i8_wstride = w_stride;
  p.i8_amax = amax;
  p.i8_rw = row_w;
  p.i8_src = src_slot;
  auto go = [&](auto kern, size_t smem) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return rf::fail(RF_ERR_CUDA, std::string("int8 tensor-core GEMM: ") + cudaGetErrorString(e));
    kern<<<rf::num_sms(), NTHREADS, smem, st>>>(ma, ma32, mb, p, NoRemote{});
    return rf::check_launch(gated ? "int8 tensor-core gated GEMM" : "int8 tensor-core down GEMM");
  };
  if (bn == 256) {
    if (!gated) return go(tc_grouped_gemm<int8_t, false, 0, 256>, Cfg<256>::SMEM_BYTES);
    if (act == RF_ACT_SILU) return go(tc_grouped_gemm<int8_t, true, RF_ACT_SILU, 256>, Cfg<256>::SMEM_BYTES);
    if (act == RF_ACT_GELU) return go(tc_grouped_gemm<int8_t, true, RF_ACT_GELU, 256>, Cfg<256>::SMEM_BYTES);
    return go(tc_grouped_gemm<int8_t, true, RF_ACT_GELU_TANH, 256>, Cfg<256>::SMEM_BYTES);
  }
  if (!gated) return go(tc_grouped_gemm<int8_t, false, 0, 128>, Cfg<128>::SMEM_BYTES);
  if (act == RF_ACT_SILU) return go(tc_grouped_gemm<int8_t, true, RF_ACT_SILU, 128>, Cfg<128>::SMEM_BYTES);
  if (act == RF_ACT_GELU) return go(tc_grouped_gemm<int8_t, true, RF_ACT_GELU, 128>, Cfg<128>::SMEM_BYTES);
  return go(tc_grouped_gemm<int8_t, true, RF_ACT_GELU_TANH, 128>, Cfg<128>::SMEM_BYTES);
}

int tc_down_remote(const GroupedGemmArgs &g, cudaStream_t st) {
  if (!g.remote || g.slot || g.groups || g.gather_src) return -1;
  if (g.rows_capacity <= 0 || g.n_groups < 1 || g.remote->R < 1 || g.remote->R > REMOTE_MAX_RANKS) return -1;
  int rc = RF_OK;
  if (!try_tc(g, false, st, &rc)) return -1;
  return rc;
}
}  // namespace rf

namespace {

int grouped_gemm(const void *a, const void *w, void *out, const int32_t *offsets,
                 const int32_t *counts, const int32_t *slot, const int32_t *groups,
                 int64_t n_groups, int64_t E, int64_t num_slots, int64_t rows_capacity,
                 int64_t Kdim, int64_t N, int dtype, int act, bool gated, rf_stream_t stream,
                 const char *name, const void *addend = nullptr) {
  const std::string nm(name);
  RF_CHECK_ARG(rf::valid_dtype(dtype), nm + ": unknown dtype");
  RF_CHECK_ARG(act == RF_ACT_SILU || act == RF_ACT_GELU || act == RF_ACT_GELU_TANH,
               nm + ": unknown activation");
  RF_CHECK_ARG(E >= 1 && E <= 65535 && num_slots >= 1 && rows_capacity >= 0 && Kdim >= 1 && N >= 1,
               nm + ": bad sizes");
  RF_CHECK_ARG(Kdim < (1 << 30) && N < (1 << 30) && rows_capacity < ((int64_t)1 << 31),
               nm + ": sizes exceed int32");
  // no rows (an empty batch): the row buffers may be empty, possibly null
  RF_CHECK_ARG((rows_capacity == 0 || (a && out)) && w && offsets && counts, nm + ": null pointer");
  const int64_t G = groups ? n_groups : E;
  RF_CHECK_ARG(G >= 0 && G <= 65535, nm + ": bad group count");
  if (G == 0 || rows_capacity == 0) return RF_OK;
  rf::GroupedGemmArgs g;
  g.a = a;
  g.w = w;
  g.out = out;
  g.offsets = offsets;
  g.counts = counts;
  g.slot = slot;
  g.groups = groups;
  g.n_groups = (int)G;
  g.E = (int)E;
  g.num_slots = (int)num_slots;
  g.rows_capacity = rows_capacity;
  g.Kdim = (int)Kdim;
  g.N = (int)N;
  g.dtype = dtype;
  g.act = act;
  g.addend = addend;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = RF_OK;
  if (try_tc(g, gated, st, &rc)) return rc;
  return rf::launch_simt_grouped_gemm(g, gated, st);
}

}  // namespace

extern "C" int rf_moe_set_gemm_impl(int impl) {
  if (impl < 0 || impl > 5) return rf::fail(RF_ERR_ARG, "rf_moe_set_gemm_impl: 0 to 5");
  g_gemm_impl = impl;
  return RF_OK;
}

extern "C" int rf_moe_grouped_gemm_gated(const void *a, const void *w1, void *h,
                                         const int32_t *expert_offsets,
                                         const int32_t *expert_counts, const int32_t *expert_slot,
                                         const int32_t *groups, int64_t n_groups, int64_t E,
                                         int64_t num_slots, int64_t rows_capacity, int64_t H,
                                         int64_t I, int dtype, int activation, rf_stream_t stream) {
  return grouped_gemm(a, w1, h, expert_offsets, expert_counts, expert_slot, groups, n_groups, E,
                      num_slots, rows_capacity, H, I, dtype, activation, true, stream,
                      "rf_moe_grouped_gemm_gated");
}

extern "C" int rf_moe_grouped_gemm_gated_gather(const void *x, int64_t x_rows, const int32_t *src_slot,
                                                int64_t topk, const void *w1, void *h,
                                                const int32_t *expert_offsets, const int32_t *expert_counts,
                                                const int32_t *expert_slot, const int32_t *groups,
                                                int64_t n_groups, int64_t E, int64_t num_slots,
                                                int64_t rows_capacity, int64_t H, int64_t I, int dtype,
                                                int activation, rf_stream_t stream) {
  const char *nm = "rf_moe_grouped_gemm_gated_gather";
  RF_CHECK_ARG(rf::valid_dtype(dtype), std::string(nm) + ": unknown dtype");
  RF_CHECK_ARG(activation == RF_ACT_SILU || activation == RF_ACT_GELU || activation == RF_ACT_GELU_TANH,
               std::string(nm) + ": unknown activation");
  RF_CHECK_ARG(x_rows >= 1 && x_rows < ((int64_t)1 << 31) && topk >= 1, std::string(nm) + ": bad sizes");
  RF_CHECK_ARG(E >= 1 && E <= 65535 && num_slots >= 1 && rows_capacity >= 0 && H >= 1 && I >= 1 &&
                   H < (1 << 30) && I < (1 << 30) && rows_capacity < ((int64_t)1 << 31),
               std::string(nm) + ": bad sizes");
  RF_CHECK_ARG(x && src_slot && w1 && h && expert_offsets && expert_counts, std::string(nm) + ": null pointer");
  const int64_t G = groups ? n_groups : E;
  RF_CHECK_ARG(G >= 0 && G <= 65535, std::string(nm) + ": bad group count");
  if (G == 0 || rows_capacity == 0) return RF_OK;
  rf::GroupedGemmArgs g;
  g.a = x;
  g.w = w1;
  g.out = h;
  g.offsets = expert_offsets;
  g.counts = expert_counts;
  g.slot = expert_slot;
  g.groups = groups;
  g.n_groups = (int)G;
  g.E = (int)E;
  g.num_slots = (int)num_slots;
  g.rows_capacity = rows_capacity;
  g.Kdim = (int)H;
  g.N = (int)I;
  g.dtype = dtype;
  g.act = activation;
  g.gather_src = src_slot;
  g.gather_div = (int)topk;
  g.a_rows = x_rows;
  int rc = RF_OK;
  if (try_tc(g, true, (cudaStream_t)stream, &rc)) return rc;
  return rf::fail(RF_ERR_UNSUPPORTED, std::string(nm) +
                                          ": needs the tensor-core path (16-bit dtype, 16-byte aligned "
                                          "rows); gather the rows with rf_moe_permute instead");
}

extern "C" int rf_moe_grouped_gemm_down(const void *h, const void *w2, void *y,
                                        const int32_t *expert_offsets, const int32_t *expert_counts,
                                        const int32_t *expert_slot, const int32_t *groups,
                                        int64_t n_groups, int64_t E, int64_t num_slots,
                                        int64_t rows_capacity, int64_t H, int64_t I, int dtype,
                                        rf_stream_t stream) {
  return grouped_gemm(h, w2, y, expert_offsets, expert_counts, expert_slot, groups, n_groups, E,
                      num_slots, rows_capacity, I, H, dtype, RF_ACT_SILU, false, stream,
                      "rf_moe_grouped_gemm_down");
}

extern "C" int rf_moe_grouped_gemm_down_add(const void *h, const void *w2, void *y, const void *addend,
                                            const int32_t *expert_offsets, const int32_t *expert_counts,
                                            const int32_t *expert_slot, const int32_t *groups,
                                            int64_t n_groups, int64_t E, int64_t num_slots,
                                            int64_t rows_capacity, int64_t H, int64_t I, int dtype,
                                            rf_stream_t stream) {
  RF_CHECK_ARG(addend || rows_capacity == 0, "rf_moe_grouped_gemm_down_add: null addend");
  return grouped_gemm(h, w2, y, expert_offsets, expert_counts, expert_slot, groups, n_groups, E,
                      num_slots, rows_capacity, I, H, dtype, RF_ACT_SILU, false, stream,
                      "rf_moe_grouped_gemm_down_add", addend);
}
