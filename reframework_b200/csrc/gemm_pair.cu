// K3/K4 on CTA pairs — grouped expert GEMMs with tcgen05.mma.cta_group::2.
//
// The same math as gemm_tc.cu (reframework/moe/fused.py:81-83):
//   gated: h[r, j] = act(a[r] . w1[s, j]) * (a[r] . w1[s, I + j])
//   down:  y[r, n] = h[r] . w2[s, n]
// with the operands swapped: WEIGHT rows are the MMA's M side and TOKEN rows
// its N side.  The two CTAs of a cluster form a pair: each holds 128 weight
// rows (M = 256 per pair) and half of the tile's token rows (N/2), and one
// thread of the first CTA issues the pair's MMAs over both CTAs' shared memory
// and accumulates into both CTAs' TMEM.  Why this shape on B200:
//   * per 64-deep k-block a CTA loads 16 KB of weights and at most 16 KB of
//     tokens for the MMA work a single-CTA 128 x 256 tile does with 48 KB, so
//     the L2 -> shared-memory traffic per FLOP drops by a third;
//   * a tile's token count is rounded up to 16 (N = 16..256), not to a
//     128-row M tile, so an expert's last tile computes at most 15 pad rows
//     (C2's skewed routing wastes 6-9 % of the MMA work on 128-row tiles);
//   * decode (a few tokens per expert) becomes N = 16 tiles that stream the
//     weights, instead of 128-row tiles that are almost all padding.
// Gated tiles: a CTA's 128 weight rows are 64 gate rows and the matching 64
// up rows (two TMA boxes), so a pair covers 128 features; the epilogue pairs
// TMEM lane i (gate) with lane 64 + i (up) through shared memory.  Down tiles:
// 128 rows of w2 per CTA, 256 output columns per pair.
//
// Roles (one cluster of 2 CTAs per SM pair, persistent, 320 threads):
//   warp 0      TMA producer (both CTAs): this CTA's weight rows and token
//               rows into a 3-stage ring of 128-deep k-blocks (128-byte swizzle, each
//               CTA copying only its own operands); the copies of both CTAs
//               complete on the first CTA's stage barrier (.cta_group::2),
//               which expects the bytes of both.
//   warp 1      first CTA: allocates 512 TMEM columns for the pair and issues
//               the MMAs (two 256-column accumulators).
//   warps 2-9   epilogue (both CTAs): tcgen05.ld of a 32-lane quadrant, values
//               rounded to the layer dtype and staged in shared memory as
//               [token][row], then 16-byte stores of whole token rows.
// Tiles: per group n_fb feature blocks x ceil(count / 256) token blocks,
// token-fastest so concurrently running pairs share a weight block in L2.
// A pair's first tile is its cluster index; later tiles are claimed
// dynamically (one global atomic counter per launch, the next tile claimed
// while the current one loads), so a pair that starts late, because another
// kernel still held its SMs, takes fewer tiles instead of stretching the
// launch by its whole static share.  The first CTA's producer claims for the
// pair and publishes each index through a small ring in both CTAs' shared
// memory (full / empty barriers; read by the MMA issuer, the second producer
// and one epilogue warp per CTA; the second CTA waits with cluster-scope
// acquire).
// Each mbarrier wait is bounded (2 s): on expiry the CTA flags the device
// error word and both CTAs of the pair stop, let their copies in flight land
// (a bounded pause: the second CTA's copies signal the first CTA's barrier, so
// neither CTA can count them), drain their MMAs, meet at a cluster barrier and
// release TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();
#include "tc_ptx.cuh"

namespace {

// Ring: 3 stages of two 64-deep sub-blocks (64 KB per CTA per stage).  Measured
// on B200 at C2's shapes: the same 192 KB as 6 stages of one sub-block but one
// barrier wait and one stage release per 8 MMAs instead of per 4, which was
// worth 6 % on the gated GEMM (4, 5 or 6 single sub-block stages made no
// difference: the loop is bound by per-stage work, not by copy latency).
#ifndef RF_PAIR_KSUB
#define RF_PAIR_KSUB 2
#endif
#ifndef RF_PAIR_STAGES
#define RF_PAIR_STAGES 3
#endif
#ifndef RF_PAIR_EPI_SLEEP_NS
#define RF_PAIR_EPI_SLEEP_NS 256
#endif
constexpr int PBK = 64;                        // TMA box / swizzle atom depth (elements)
constexpr int P_KSUB = RF_PAIR_KSUB;           // 64-deep sub-blocks per ring stage
constexpr int P_AROWS = 128;                   // weight rows per CTA
constexpr int P_TOK = 256;                     // token rows per tile (max N)
constexpr int P_A_SUB = P_AROWS * PBK * 2;     // 16 KB per sub-block
constexpr int P_B_SUB = (P_TOK / 2) * PBK * 2; // 16 KB: at most N/2 = 128 token rows per CTA
constexpr int P_A_BYTES = P_KSUB * P_A_SUB;
constexpr int P_B_BYTES = P_KSUB * P_B_SUB;
constexpr int P_STAGES = RF_PAIR_STAGES;
constexpr int P_EPI_WARPS = 8;
constexpr int P_THREADS = 32 * (2 + P_EPI_WARPS);
constexpr int P_CHUNK = 32;                    // token columns per epilogue round
constexpr int P_STG_BYTES = P_CHUNK * P_AROWS * 2;  // [32 tokens][128 rows] 16-bit
constexpr int P_MAX_GROUPS = 512;
constexpr int P_TQ = 8;                        // tile-index ring slots
// Readers that release a ring slot: the MMA issuer and the second CTA's
// producer (neither stores to global memory, so their release arrives are
// cheap).  The epilogue reads each index too but does not arrive: it cannot
// fall more than 2 tiles behind the MMA issuer (two TMEM accumulators), which
// itself is at most P_STAGES stages behind the producer, so with P_TQ > 6 a
// slot is never rewritten before the epilogue has read it.
constexpr int P_TQ_READERS = 2;
constexpr int P_NUM_BARS = 2 * P_STAGES + 5 + 2 * P_TQ;  // full, empty, tmem full x2, tmem empty x2, drain, tile ring
constexpr int P_SCHED_SLOTS = 64;              // launches in flight with their own tile counter
constexpr uint64_t P_ABORT_DRAIN_NS = 1000000;  // pause for copies in flight after an abort (1 ms)
constexpr uint32_t P_TMEM_COLS = 512;
constexpr int P_N_BOXES = 5;                   // token boxes of 8, 16, 32, 64, 128 rows
constexpr unsigned P_EPI_SLEEP_NS = RF_PAIR_EPI_SLEEP_NS;  // epilogue polls of the accumulator barrier
constexpr size_t P_SMEM_BYTES = 1024 + (size_t)P_STAGES * (P_A_BYTES + P_B_BYTES) + 2 * P_STG_BYTES +
                                P_NUM_BARS * 8 + 16 + (size_t)(P_MAX_GROUPS + 1) * 4 +
                                (size_t)3 * P_MAX_GROUPS * 4 + (P_TQ + 2) * 4;
static_assert(P_SMEM_BYTES <= 227 * 1024, "shared memory");

struct PairArgs {
  const int32_t *offsets, *counts, *slot, *groups;
  int n_groups, E, num_slots;
  int Kdim;  // reduction length
  int N;     // output columns (I gated, H down)
  int n_fb;  // feature blocks per group (128 features per pair gated, 256 down)
  void *out;
  const void *addend;  // down only: out = round(addend + round(acc)); may be NULL or out
  int sched;           // this launch's tile counter (g_pair_sched row)
};

// Per-launch tile counters.  Every pair claims until it draws an index past
// the last tile, so a launch makes exactly npairs + max(0, total - npairs)
// claims; the pair that drew the last of them puts the counter back to zero
// when it finishes (after a wait timeout the counter may be left nonzero: the
// device error word then reports RF_DEV_WAIT_TIMEOUT).  The host hands
// consecutive launches consecutive counters, so up to P_SCHED_SLOTS launches
// may be in flight at once (several streams, graphs) without sharing one.
__device__ int g_pair_sched[P_SCHED_SLOTS];

// Token-row maps of one launch: the same 2-D tensor with boxes of 8 << i rows.
struct TokMaps {
  CUtensorMap m[P_N_BOXES];
};

// ------------------------------------------------------------ pair PTX
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t ncluster_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// The shared::cluster address of `addr` (this CTA's shared window) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Tile loads whose completion is counted on barrier `bar` of either CTA of the
// pair (shared::cluster address); the destination is this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at shared::cluster address `bar` (this CTA's or the
// other CTA's) once all MMAs this thread issued so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 32 TMEM lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// try_wait with cluster-scope acquire: the phase was completed by the other
// CTA of the pair, which wrote the data it guards into this CTA's memory.
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe: has the phase of `parity` completed?
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Named barrier over the epilogue warps that also ANDs a predicate.
__device__ __forceinline__ bool epi_vote_and(int ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(ok), "n"(32 * P_EPI_WARPS)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * P_EPI_WARPS) : "memory");
}

// Kind::f16 instruction descriptor: fp32 accumulator, A and B K-major and of
// the same 16-bit type, M = 256 (the pair); N is or-ed in per tile.
template <typename T>
__host__ __device__ constexpr uint32_t pair_idesc_base() {
  return (1u << 4) | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7) |
         ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10) | ((uint32_t)(256 >> 4) << 24);
}

struct PairNoRemote {};

__device__ __forceinline__ void st_release_sys_pair(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// REMOTE (down GEMM of the expert-parallel layer, groups = this rank's local
// slots): each output row goes to its token's rank over NVLink, at that
// rank's permuted row (rf::RemoteOut), and the launch's last CTA raises the
// return flags in every rank.
template <typename T, bool GATED, int ACT, bool REMOTE = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    tc_pair_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ TokMaps tmX, const PairArgs p,
                 const __grid_constant__ std::conditional_t<REMOTE, rf::RemoteOut, PairNoRemote> ro) {
  static_assert(!REMOTE || !GATED, "remote stores: down GEMM only");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *sA = smem;
  uint8_t *sB = sA + P_STAGES * P_A_BYTES;
  uint8_t *sS = sB + P_STAGES * P_B_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sS + 2 * P_STG_BYTES);
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + P_NUM_BARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int *tile_prefix = reinterpret_cast<int *>(tmem_holder + 4);  // [G+1]
  int *g_row0 = tile_prefix + P_MAX_GROUPS + 1;                   // [G]
  int *g_cnt = g_row0 + P_MAX_GROUPS;                             // [G]
  int *g_slot = g_cnt + P_MAX_GROUPS;                             // [G]
  volatile int *tq = g_slot + P_MAX_GROUPS;                       // [P_TQ] claimed tile indices
  volatile int *epi_t = tq + P_TQ;                                // [2] the epilogue's current tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the pair's MMAs
  const int G = p.n_groups;
  // a pair's first tile is its cluster index; later tiles are claimed
  // (counter value c -> tile npairs + c) and pass through the ring
  const int pair = (int)cluster_id_x(), npairs = (int)ncluster_x();
  const uint32_t bar0 = smem_u32(bars);
#define FULL(s) (bar0 + 8u * (uint32_t)(s))
#define EMPTY(s) (bar0 + 8u * (uint32_t)(P_STAGES + (s)))
#define TFULL(a) (bar0 + 8u * (uint32_t)(2 * P_STAGES + (a)))
#define TEMPTY(a) (bar0 + 8u * (uint32_t)(2 * P_STAGES + 2 + (a)))
  const uint32_t DRAIN = bar0 + 8u * (uint32_t)(2 * P_STAGES + 4);
#define TQF(i) (bar0 + 8u * (uint32_t)(2 * P_STAGES + 5 + (i)))
#define TQE(i) (bar0 + 8u * (uint32_t)(2 * P_STAGES + 5 + P_TQ + (i)))
  const uint32_t peer_abort = mapa_shared(smem_u32((const void *)abort_flag), rank ^ 1u);

  // bounded wait; on expiry both CTAs of the pair are told to stop
  auto pwait = [&](uint32_t bar, uint32_t parity, unsigned sleep_ns, bool cluster_acq = false) -> bool {
    auto probe = [&]() { return cluster_acq ? mbar_try_cluster(bar, parity) : mbar_try(bar, parity); };
    if (probe()) return true;
    const uint64_t t0 = rf::globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      if (sleep_ns) __nanosleep(sleep_ns);
      if (probe()) return true;
      if ((it & 63) == 0) {
        if (*abort_flag) return false;
        if (rf::globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
          *abort_flag = 1;
          st_cluster_u32(peer_abort, 1u);
          rf_report(RF_DEV_WAIT_TIMEOUT);
          return false;
        }
      }
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(FULL(s), 1);  // the first CTA's: its producer's arrival + both CTAs' bytes
      mbar_init(EMPTY(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(TFULL(a), 1);
      mbar_init(TEMPTY(a), 2 * P_EPI_WARPS);  // every epilogue warp of both CTAs
    }
    mbar_init(DRAIN, 1);
    epi_t[0] = epi_t[1] = 0;
    for (int i = 0; i < P_TQ; ++i) {
      mbar_init(TQF(i), 1);             // the first CTA's producer publishes
      mbar_init(TQE(i), P_TQ_READERS);  // used in the first CTA only
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmW) : "memory");
    for (int i = 0; i < P_N_BOXES; ++i) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX.m[i]) : "memory");
  }
  for (int g = threadIdx.x; g < G; g += P_THREADS) {
    const int e = p.groups ? p.groups[g] : g;
    int tiles = 0, row0 = 0, cnt = 0, s = 0;
    if (e >= 0 && e < p.E) {
      s = p.slot ? p.slot[e] : e;
      if (s >= 0 && s < p.num_slots) {
        row0 = p.offsets[e];
        cnt = p.counts[e];
        tiles = cnt > 0 ? ((cnt + P_TOK - 1) / P_TOK) * p.n_fb : 0;
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
    tmem_alloc_pair(smem_u32(tmem_holder), P_TMEM_COLS);
    tmem_relinquish_pair();
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
  // barrier inits and the TMEM address visible to both CTAs of the pair
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total = tile_prefix[G];
  const int num_kb = (p.Kdim + PBK * P_KSUB - 1) / (PBK * P_KSUB);  // ring stages per tile

  // tile -> (first token row, token count, feature block, weight slot)
  auto decode = [&](int t, int &row0, int &ntok, int &fb, int &s) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile_prefix[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    const int cnt = g_cnt[lo];
    const int ntb = (cnt + P_TOK - 1) / P_TOK;
    const int local = t - tile_prefix[lo];
    fb = local / ntb;
    const int tb = local - fb * ntb;
    row0 = g_row0[lo] + tb * P_TOK;
    ntok = min(P_TOK, cnt - tb * P_TOK);
    s = g_slot[lo];
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(FULL(0), 0);  // the first CTA's stage barriers
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int *claim = &g_pair_sched[p.sched];
      const int last_claim = npairs + max(0, total - npairs) - 1;
      auto draw = [&]() { return npairs + atomicAdd(claim, 1); };  // the result is used a tile later
      const uint32_t tq_peer = mapa_shared(smem_u32((const void *)tq), 1);
      const uint32_t tqf_peer = mapa_shared(TQF(0), 1);
      const uint32_t tqe_lead = mapa_shared(TQE(0), 0);
      // the first CTA publishes each iteration's tile during the iteration
      // before, so the second CTA's producer never waits for it at a tile
      // boundary
      int t_lead = pair;                                            // this iteration's tile
      int t_next = rank == 0 ? draw() : 0;  // the next one's (claimed)
      for (int it = 0; ok; ++it) {
        int t;
        if (rank == 0) {
          t = t_lead;
          if (t >= total) break;  // the sentinel went out one iteration earlier (or t is the first tile)
        } else if (it == 0) {
          t = pair;
          if (t >= total) break;
        } else {
          const int slot = (it - 1) % P_TQ;
          if (!pwait(TQF(slot), (uint32_t)(((it - 1) / P_TQ) & 1), 0, true)) {
            ok = false;
            break;
          }
          t = tq[slot];
          mbar_arrive_cluster(tqe_lead + 8u * (uint32_t)slot);
          if (t >= total) break;
        }
        int row0, ntok, fb, s;
        decode(t, row0, ntok, fb, s);
        const int half = ((ntok + 15) & ~15) >> 1;  // token rows per CTA: N/2, a multiple of 8
        int bi = 0;
        while ((8 << bi) < half) ++bi;
        const uint32_t bytes = (uint32_t)P_KSUB * ((uint32_t)P_A_SUB + (uint32_t)(8 << bi) * (PBK * 2));  // per CTA
        const int xrow = row0 + (rank ? half : 0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!pwait(EMPTY(stage), phase ^ 1u, 0)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = smem_u32(sA + stage * P_A_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * P_B_BYTES);
          const uint32_t full = full0 + 8u * (uint32_t)stage;
          if (rank == 0) mbar_expect_tx(FULL(stage), 2u * bytes);  // both CTAs load the same box sizes
#pragma unroll
          for (int j = 0; j < P_KSUB; ++j) {
            const int k0 = (kb * P_KSUB + j) * PBK;
            const uint32_t aj = a_dst + (uint32_t)(j * P_A_SUB), bj = b_dst + (uint32_t)(j * P_B_SUB);
            if (GATED) {
              const int f = fb * 128 + (int)rank * 64;
              tma_load_3d_pair(aj, &tmW, full, k0, f, 2 * s);
              tma_load_3d_pair(aj + P_A_SUB / 2, &tmW, full, k0, f, 2 * s + 1);
            } else {
              tma_load_3d_pair(aj, &tmW, full, k0, fb * 256 + (int)rank * 128, s);
            }
            tma_load_2d_pair(bj, &tmX.m[bi], full, k0, xrow);
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (rank == 0 && kb == min(P_STAGES - 1, num_kb - 1)) {
            // once this tile's first stages are in flight (the claim issued
            // a tile earlier, or at kernel start, has returned by then):
            // publish the next iteration's tile (ring slot it % P_TQ) and
            // claim the one after
            const int slot = it % P_TQ;
            if (!pwait(TQE(slot), (uint32_t)(((it / P_TQ) & 1) ^ 1), 0)) {
              ok = false;
              break;
            }
            tq[slot] = t_next;
            st_cluster_u32(tq_peer + 4u * (uint32_t)slot, (uint32_t)t_next);
            mbar_arrive(TQF(slot));
            mbar_arrive_cluster(tqf_peer + 8u * (uint32_t)slot);
            t_lead = t_next;
            if (t_next < total) t_next = draw();  // its latency overlaps this tile
          }
        }
      }
      // a pair's last draw is past the last tile; the draw that was the
      // launch's last claim puts the counter back to zero for the next launch
      if (rank == 0 && t_next - npairs == last_claim) atomicExch(claim, 0);
      if (!ok) {  // let the copies in flight land before this CTA can exit (bounded pause)
        const uint64_t t0 = rf::globaltimer_ns();
        while (rf::globaltimer_ns() - t0 < P_ABORT_DRAIN_NS) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------- MMA issuer
      const uint32_t IDESC = pair_idesc_base<T>();
      const uint32_t peer_bars = mapa_shared(bar0, 1);  // the second CTA's barriers
      int stage = 0, it = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool ready = false;  // the stage about to be consumed was seen complete by the early probe
      for (;; ++it) {
        int t = pair;
        if (it > 0) {
          const int slot = (it - 1) % P_TQ;
          if (!pwait(TQF(slot), (uint32_t)(((it - 1) / P_TQ) & 1), 0)) break;
          t = tq[slot];
          mbar_arrive(TQE(slot));
        }
        if (t >= total) break;
        int row0, ntok, fb, s;
        decode(t, row0, ntok, fb, s);
        const uint32_t idesc = IDESC | ((uint32_t)(((ntok + 15) & ~15) >> 3) << 17);
        const int acc = it & 1;
        const uint32_t aph = (uint32_t)((it >> 1) & 1);
        if (!pwait(TEMPTY(acc), aph ^ 1u, 0)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * 256);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!ready && !pwait(FULL(stage), phase, 0)) {
            ok = false;
            break;
          }
          // probe the next stage now, so that check overlaps this stage's MMA issue
          ready = stage + 1 == P_STAGES ? mbar_test(FULL(0), phase ^ 1u) : mbar_test(FULL(stage + 1), phase);
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * P_A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * P_B_BYTES);
#pragma unroll
          for (int j = 0; j < P_KSUB; ++j)
#pragma unroll
            for (int k = 0; k < PBK / 16; ++k)
              tc_mma_pair(d, sw128_desc(a0 + j * P_A_SUB + k * 32), sw128_desc(b0 + j * P_B_SUB + k * 32), idesc,
                          (kb | j | k) ? 1u : 0u);
          tc_commit_pair(EMPTY(stage));  // frees the stage in both CTAs once read
          tc_commit_pair(peer_bars + (EMPTY(stage) - bar0));
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(TFULL(acc));
        tc_commit_pair(peer_bars + (TFULL(acc) - bar0));
      }
      // no MMA may still be running when either CTA releases TMEM or exits
      tc_commit_pair(DRAIN);
      mbar_wait_teardown(DRAIN, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;           // TMEM lane quadrant of this warp
    const int part = (warp - 2) >> 2;  // which 16 of a round's 32 token columns it loads
    const int etid = threadIdx.x - 64;
    const uint32_t tempty0 = mapa_shared(TEMPTY(0), 0);
    T *out = reinterpret_cast<T *>(p.out);
    int it = 0, round = 0;
    for (;; ++it) {
      // the first epilogue warp reads the ring for all eight (one reader per CTA)
      int tok_ok = 1;
      if (it > 0 && warp == 2 && lane == 0) {
        const int slot = (it - 1) % P_TQ;
        tok_ok = pwait(TQF(slot), (uint32_t)(((it - 1) / P_TQ) & 1), P_EPI_SLEEP_NS, true) ? 1 : 0;
        if (tok_ok) epi_t[it & 1] = tq[slot];
      }
      tok_ok = __shfl_sync(0xffffffffu, tok_ok, 0);
      if (!epi_vote_and(tok_ok)) break;  // every epilogue warp takes the same branch
      const int t = it > 0 ? epi_t[it & 1] : pair;
      if (t >= total) break;             // the same index in every warp
      int row0, ntok, fb, s;
      decode(t, row0, ntok, fb, s);
      const int np = (ntok + 15) & ~15;
      const int acc = it & 1;
      const uint32_t aph = (uint32_t)((it >> 1) & 1);
      int ok = 1;
      if (lane == 0) ok = pwait(TFULL(acc), aph, P_EPI_SLEEP_NS) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!epi_vote_and(ok)) break;  // every epilogue warp takes the same branch
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(wq * 32) << 16) + (uint32_t)(acc * 256);
      const int nrounds = (np + P_CHUNK - 1) / P_CHUNK;
      for (int ch = 0; ch < nrounds; ++ch, ++round) {
        const int c = ch * P_CHUNK;
        const int w = min(P_CHUNK, np - c);  // 16 or 32
        T *stg = reinterpret_cast<T *>(sS + (round & 1) * P_STG_BYTES);
        if (16 * part < w) {
          uint32_t v[16];
          tmem_ld16(tb + (uint32_t)(c + 16 * part), v);
          tmem_ld_wait();
          T *col = stg + (16 * part) * P_AROWS + wq * 32 + lane;
#pragma unroll
          for (int j = 0; j < 16; ++j) col[j * P_AROWS] = rf::Cvt<T>::from_f(__uint_as_float(v[j]));
        }
        if (ch == nrounds - 1) {  // the accumulator is free for the pair's next tile
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * (uint32_t)acc);
        }
        epi_sync();
        const int j = etid >> 3;
        const int tok = c + j;
        if (j < w && tok < ntok) {
          const T *srow = stg + j * P_AROWS;
          T *orow = out + (int64_t)(row0 + tok) * p.N;
          if constexpr (GATED) {
            const int k8 = (etid & 7) * 8;
            const int f = fb * 128 + (int)rank * 64 + k8;
            if (f < p.N) {
              float gf[8], uf[8];
              rf::unpack16<T>(*reinterpret_cast<const uint4 *>(srow + k8), gf);
              rf::unpack16<T>(*reinterpret_cast<const uint4 *>(srow + 64 + k8), uf);
              uint32_t pk[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                pk[i] = rf::pack2<T>(rf::gated_elem_t<T, ACT>(gf[2 * i], uf[2 * i]),
                                     rf::gated_elem_t<T, ACT>(gf[2 * i + 1], uf[2 * i + 1]));
              *reinterpret_cast<uint4 *>(orow + f) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          } else {
            const int k16 = (etid & 7) * 16;
            const int f = fb * 256 + (int)rank * 128 + k16;
            const T *arow = p.addend ? reinterpret_cast<const T *>(p.addend) + (int64_t)(row0 + tok) * p.N : nullptr;
            if constexpr (REMOTE) {  // source rank of local row k of slot s, and the row there
              const int64_t k = (int64_t)(row0 + tok) - g_row0[s];
              const int64_t *cj = ro.cj + (int64_t)s * (ro.R + 1);
              int lo = 0, hi = ro.R - 1;
              while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (cj[mid] <= k) lo = mid;
                else hi = mid - 1;
              }
              orow = reinterpret_cast<T *>(ro.dst[lo]) + (ro.ps[(int64_t)lo * ro.S + s] + (k - cj[lo])) * p.N;
            }
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              if (f + 8 * v >= p.N) break;
              uint4 val = *reinterpret_cast<const uint4 *>(srow + k16 + 8 * v);
              if (arow) {  // a second shared expert adds onto the first: both rounded, summed, rounded
                float yf[8], af[8];
                rf::unpack16<T>(val, yf);
                rf::unpack16<T>(*reinterpret_cast<const uint4 *>(arow + f + 8 * v), af);
                val = make_uint4(rf::pack2<T>(af[0] + yf[0], af[1] + yf[1]), rf::pack2<T>(af[2] + yf[2], af[3] + yf[3]),
                                 rf::pack2<T>(af[4] + yf[4], af[5] + yf[5]), rf::pack2<T>(af[6] + yf[6], af[7] + yf[7]));
              }
              *reinterpret_cast<uint4 *>(orow + f + 8 * v) = val;
            }
          }
        }
      }
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA of the pair leaves while the other may still reach into it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, P_TMEM_COLS);
  }
  if constexpr (REMOTE) {
    if (threadIdx.x == 0) {
      __threadfence_system();  // this CTA's peer stores, visible to every GPU, before the count
      const uint32_t prev = atomicAdd(ro.done, 1u);
      if (prev == gridDim.x - 1) {  // last CTA: every row of the launch has landed
        __threadfence_system();
        for (int d = 0; d < ro.R; ++d) st_release_sys_pair(ro.flag[d], ro.epoch);
        *ro.done = 0u;
      }
    }
  }
#undef TQF
#undef TQE
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
}

template <typename T, bool GATED, int ACT, bool REMOTE = false>
int launch_pair_t(const CUtensorMap &mw, const TokMaps &mx, const PairArgs &p, cudaStream_t st,
                  const rf::RemoteOut *remote = nullptr) {
  auto kern = tc_pair_gemm<T, GATED, ACT, REMOTE>;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  static int clusters = 0;
  std::call_once(once, [&] {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM_BYTES);
    if (err != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * std::max(1, rf::num_sms() / 2), 1, 1);
    cfg.blockDim = dim3(P_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    err = cudaOccupancyMaxActiveClusters(&clusters, (void *)kern, &cfg);
  });
  if (err != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (clusters < 1) return -1;
  if constexpr (REMOTE) {
    kern<<<2 * clusters, P_THREADS, P_SMEM_BYTES, st>>>(mw, mx, p, *remote);
  } else {
    kern<<<2 * clusters, P_THREADS, P_SMEM_BYTES, st>>>(mw, mx, p, PairNoRemote{});
  }
  return rf::check_launch(REMOTE ? "tensor-core down GEMM with peer stores (CTA pairs)"
                                 : GATED ? "tensor-core gated GEMM (CTA pairs)" : "tensor-core down GEMM (CTA pairs)");
}

template <typename T>
int launch_pair_dt(const rf::GroupedGemmArgs &g, bool gated, const CUtensorMap &mw, const TokMaps &mx,
                   const PairArgs &p, cudaStream_t st) {
  if (!gated && g.remote) return launch_pair_t<T, false, 0, true>(mw, mx, p, st, g.remote);
  if (!gated) return launch_pair_t<T, false, 0>(mw, mx, p, st);
  if (g.act == RF_ACT_SILU) return launch_pair_t<T, true, RF_ACT_SILU>(mw, mx, p, st);
  if (g.act == RF_ACT_GELU) return launch_pair_t<T, true, RF_ACT_GELU>(mw, mx, p, st);
  return launch_pair_t<T, true, RF_ACT_GELU_TANH>(mw, mx, p, st);
}

}  // namespace

namespace rf {

int launch_pair_grouped_gemm(const GroupedGemmArgs &g, bool gated, cudaStream_t st) {
  if (g.dtype != RF_BF16 && g.dtype != RF_F16) return -1;
  if (g.gather_src) return -1;
  if (g.remote && (gated || g.slot || g.groups || g.addend || g.remote->R < 1 || g.remote->R > rf::REMOTE_MAX_RANKS))
    return -1;
  if (g.Kdim % 8 || g.N % 8 || g.n_groups < 1 || g.n_groups > P_MAX_GROUPS || g.rows_capacity < 1) return -1;
  if ((uintptr_t)g.a % 16 || (uintptr_t)g.w % 16 || (uintptr_t)g.out % 16) return -1;
  if (!g.offsets || !g.counts) return -1;
  CUtensorMap mw;
  TokMaps mx;
  const cuuint64_t dX[2] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.rows_capacity};
  const cuuint64_t sX[1] = {(cuuint64_t)g.Kdim * 2};
  for (int i = 0; i < P_N_BOXES; ++i) {
    const cuuint32_t bX[2] = {PBK, (cuuint32_t)(8 << i)};
    if (!tma_encode(&mx.m[i], g.dtype, 2, g.a, dX, sX, bX)) return -1;
  }
  if (gated) {
    // w1 [S, 2N, K] viewed as [2S][N][K]: half 0 = gate rows, half 1 = up rows
    const cuuint64_t dW[3] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.N, (cuuint64_t)(2 * g.num_slots)};
    const cuuint64_t sW[2] = {(cuuint64_t)g.Kdim * 2, (cuuint64_t)g.N * g.Kdim * 2};
    const cuuint32_t bW[3] = {PBK, 64, 1};
    if (!tma_encode(&mw, g.dtype, 3, g.w, dW, sW, bW)) return -1;
  } else {
    const cuuint64_t dW[3] = {(cuuint64_t)g.Kdim, (cuuint64_t)g.N, (cuuint64_t)g.num_slots};
    const cuuint64_t sW[2] = {(cuuint64_t)g.Kdim * 2, (cuuint64_t)g.N * g.Kdim * 2};
    const cuuint32_t bW[3] = {PBK, 128, 1};
    if (!tma_encode(&mw, g.dtype, 3, g.w, dW, sW, bW)) return -1;
  }
  PairArgs p;
  p.offsets = g.offsets;
  p.counts = g.counts;
  p.slot = g.slot;
  p.groups = g.groups;
  p.n_groups = g.n_groups;
  p.E = g.E;
  p.num_slots = g.num_slots;
  p.Kdim = g.Kdim;
  p.N = g.N;
  p.n_fb = gated ? (g.N + 127) / 128 : (g.N + 255) / 256;
  p.out = g.out;
  p.addend = gated ? nullptr : g.addend;
  static std::atomic<unsigned> next_sched{0};
  p.sched = (int)(next_sched.fetch_add(1u) % (unsigned)P_SCHED_SLOTS);
  if (g.dtype == RF_BF16) return launch_pair_dt<__nv_bfloat16>(g, gated, mw, mx, p, st);
  return launch_pair_dt<__half>(g, gated, mw, mx, p, st);
}

}  // namespace rf
