// Expert-parallel row exchange over NVLink peer memory (replaces the two NCCL
// all-to-alls of reframework/parallel/dist.py:194-206 as used by the
// token-dispatch EP layer).
//
// Every rank owns a receive buffer, a return buffer and a small control block
// (flag words), allocated here and mapped into the peers' address spaces with
// CUDA IPC.  A step then needs no collective for the rows themselves:
//   rf_moe_ep_push_rows  one kernel: each warp copies rows of this rank (read
//       through up to two index maps, so the permute's gather and the send
//       reorder are folded in) straight into the destination rank's buffer at
//       that rank's receive offset, with 16-byte NVLink stores.  The last block
//       to finish fences at system scope and raises this rank's flag word in
//       every peer's control block to the step's epoch (st.release.sys).
//   rf_moe_ep_wait       one block: waits (ld.acquire.sys, bounded by 2 s of
//       globaltimer) until every source's flag holds the epoch; on timeout it
//       sets the device error word and returns instead of hanging.
//   rf_moe_ep_counts_push / rf_moe_ep_counts_collect  the per-step exchange
//       of the [R][E] routed-row counts the planner needs (the counts
//       all-gather), as the same one-sided stores: each rank writes its row
//       into every rank's table and raises a flag; each rank waits (bounded)
//       for all R flags and copies its table out.
// Ordering: a rank pushes into a peer's receive buffer for step n+1 only after
// that peer's return push of step n reached it, and the peer issues that push
// after it finished reading its receive buffer, so no buffer is overwritten
// while it is read (the same argument holds for the return buffers).
#include <cstring>
#include <string>

#include "common.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int MAX_RANKS = 64;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

struct PushArgs {
  const uint8_t *src;
  int64_t row_bytes;
  const int32_t *idx1;  // row i reads j = idx1 ? idx1[i] : i
  const int32_t *idx2;  // then source row idx2 ? idx2[j] / div : j
  int64_t div;
  int R, me;
  int32_t epoch;
  uint32_t *done;       // this rank's block counter (zero between launches)
  int64_t chunk_off[MAX_RANKS + 1];  // rows [chunk_off[d], chunk_off[d+1]) go to rank d
  int64_t dst_row0[MAX_RANKS];       // ... starting at this row of rank d's buffer
  uint8_t *dst[MAX_RANKS];           // rank d's buffer
  int32_t *flag[MAX_RANKS];          // rank d's flag word for this rank
};

__device__ __forceinline__ void st_release_sys(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t *p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) push_rows_kernel(const __grid_constant__ PushArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t n = a.chunk_off[a.R];
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  const int64_t vecs = a.row_bytes / 16;
  // rows for all destinations interleaved, ranks staggered (see rf::scatter_pos)
  const int64_t stride = n == 0 ? 1 : rf::scatter_stride(n);
  const int64_t offset = n == 0 ? 0 : (int64_t)a.me * (n / a.R);
  for (int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); w < n; w += nwarps) {
    const int64_t i = rf::scatter_pos(w, n, stride, offset);
    // destination rank: the chunk holding row i (binary search, R <= 64)
    int lo = 0, hi = a.R - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.chunk_off[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    const int d = lo;
    const int64_t j = a.idx1 ? (int64_t)a.idx1[i] : i;
    const int64_t srow = a.idx2 ? (int64_t)a.idx2[j] / a.div : j;
    const uint4 *s = reinterpret_cast<const uint4 *>(a.src + srow * a.row_bytes);
    uint4 *t = reinterpret_cast<uint4 *>(a.dst[d] + (a.dst_row0[d] + (i - a.chunk_off[d])) * a.row_bytes);
    int64_t v = lane;
    for (; v + 96 < vecs; v += 128) {
      const uint4 q0 = __ldg(s + v), q1 = __ldg(s + v + 32), q2 = __ldg(s + v + 64), q3 = __ldg(s + v + 96);
      t[v] = q0;
      t[v + 32] = q1;
      t[v + 64] = q2;
      t[v + 96] = q3;
    }
    for (; v < vecs; v += 32) t[v] = __ldg(s + v);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this block's stores, seen by every GPU, before the count
    const uint32_t prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {  // last block: every row of this launch has landed
      __threadfence_system();
      for (int d = 0; d < a.R; ++d) st_release_sys(a.flag[d], a.epoch);
      *a.done = 0u;
    }
  }
}

__global__ void wait_flags_kernel(const int32_t *flags, int R, int32_t epoch) {
  const int r = threadIdx.x;
  if (r >= R) return;
  if (ld_acquire_sys(flags + r) == epoch) return;
  const uint64_t t0 = rf::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(64);
    if (ld_acquire_sys(flags + r) == epoch) return;
    if ((it & 255) == 0 && rf::globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
      rf_report(RF_DEV_WAIT_TIMEOUT);
      return;
    }
  }
}

// One block: this rank's expert counts row into row `me` of every rank's
// counts table (NVLink stores into the peers' control blocks), then, once all
// of them are visible system-wide, this rank's counts flag in every rank.
struct CountsPushArgs {
  const int32_t *counts;  // [E] this rank's routed rows per expert
  int R, me, E;
  int32_t epoch;
  int32_t *dst[MAX_RANKS];   // rank d's counts table [R][E] for this step
  int32_t *flag[MAX_RANKS];  // rank d's counts flag word for this rank
};

__global__ void __launch_bounds__(256) counts_push_kernel(const __grid_constant__ CountsPushArgs a) {
  for (int d = 0; d < a.R; ++d)
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.dst[d][(int64_t)a.me * a.E + e] = a.counts[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // every row stored above, seen by every GPU, before the flags
    for (int d = 0; d < a.R; ++d) st_release_sys(a.flag[d], a.epoch);
  }
}

// One block: warp w takes source rows w, w + 8, ...: every lane waits
// (acquire, bounded) for that source's flag, then the lanes copy the row.
__global__ void __launch_bounds__(256) counts_collect_kernel(const int32_t *flags, const int32_t *table, int R,
                                                             int E, int32_t epoch, int32_t *out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < R; r += 8) {
    bool ok = ld_acquire_sys(flags + r) == epoch;
    if (!ok) {
      const uint64_t t0 = rf::globaltimer_ns();
      for (uint32_t it = 1; !ok; ++it) {
        __nanosleep(64);
        ok = ld_acquire_sys(flags + r) == epoch;
        if (!ok && (it & 255) == 0 && rf::globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
      }
    }
    if (!ok) {
      if (lane == 0) rf_report(RF_DEV_WAIT_TIMEOUT);
      for (int e = lane; e < E; e += 32) out[(int64_t)r * E + e] = 0;
      continue;
    }
    for (int e = lane; e < E; e += 32) out[(int64_t)r * E + e] = table[(int64_t)r * E + e];
  }
}

}  // namespace

extern "C" int rf_moe_peer_alloc(size_t bytes, void **ptr, void *handle) {
  RF_CHECK_ARG(bytes > 0 && ptr && handle, "rf_moe_peer_alloc: bad arguments");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return rf::fail(RF_ERR_CUDA, std::string("rf_moe_peer_alloc: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return rf::fail(RF_ERR_CUDA, std::string("rf_moe_peer_alloc: ") + cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return RF_OK;
}

extern "C" int rf_moe_peer_open(const void *handle, void **ptr) {
  RF_CHECK_ARG(handle && ptr, "rf_moe_peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return rf::fail(RF_ERR_CUDA, std::string("rf_moe_peer_open: ") + cudaGetErrorString(e));
  *ptr = p;
  return RF_OK;
}

extern "C" int rf_moe_peer_close(void *ptr) {
  if (!ptr) return RF_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return rf::fail(RF_ERR_CUDA, std::string("rf_moe_peer_close: ") + cudaGetErrorString(e));
  return RF_OK;
}

extern "C" int rf_moe_peer_free(void *ptr) {
  if (!ptr) return RF_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return rf::fail(RF_ERR_CUDA, std::string("rf_moe_peer_free: ") + cudaGetErrorString(e));
  return RF_OK;
}

extern "C" int rf_moe_ep_push_rows(const void *src, int64_t row_bytes, const int32_t *idx1, const int32_t *idx2,
                                   int64_t div, int32_t R, int32_t me, const int64_t *chunk_off,
                                   const int64_t *dst_row0, void *const *dst, int32_t *const *flag, int32_t epoch,
                                   uint32_t *done, rf_stream_t stream) {
  RF_CHECK_ARG(R >= 1 && R <= MAX_RANKS && me >= 0 && me < R, "rf_moe_ep_push_rows: 1 <= R <= 64, 0 <= me < R");
  RF_CHECK_ARG(row_bytes > 0 && row_bytes % 16 == 0 && div >= 1, "rf_moe_ep_push_rows: row_bytes % 16 / div");
  RF_CHECK_ARG(chunk_off && dst_row0 && dst && flag && done, "rf_moe_ep_push_rows: null pointer");
  RF_CHECK_ARG(chunk_off[0] == 0, "rf_moe_ep_push_rows: chunk_off[0] must be 0");
  PushArgs a;
  a.src = reinterpret_cast<const uint8_t *>(src);
  a.row_bytes = row_bytes;
  a.idx1 = idx1;
  a.idx2 = idx2;
  a.div = div;
  a.R = R;
  a.me = me;
  a.epoch = epoch;
  a.done = done;
  for (int d = 0; d <= R; ++d) {
    RF_CHECK_ARG(d == 0 || chunk_off[d] >= chunk_off[d - 1], "rf_moe_ep_push_rows: chunk_off not ascending");
    a.chunk_off[d] = chunk_off[d];
  }
  for (int d = 0; d < R; ++d) {
    RF_CHECK_ARG(flag[d] && (dst[d] || chunk_off[d + 1] == chunk_off[d]) && dst_row0[d] >= 0,
                 "rf_moe_ep_push_rows: missing peer buffer or flag");
    a.dst_row0[d] = dst_row0[d];
    a.dst[d] = reinterpret_cast<uint8_t *>(dst[d]);
    a.flag[d] = flag[d];
  }
  const int64_t n = chunk_off[R];
  RF_CHECK_ARG(n == 0 || src, "rf_moe_ep_push_rows: null source");
  RF_CHECK_ARG((uintptr_t)src % 16 == 0, "rf_moe_ep_push_rows: source must be 16-byte aligned");
  int64_t blocks = (n + 7) / 8;
  const int64_t cap = (int64_t)rf::num_sms() * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;  // the flags are raised even when nothing is sent
  push_rows_kernel<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(a);
  return rf::check_launch("rf_moe_ep_push_rows");
}

extern "C" int rf_moe_ep_wait(const int32_t *flags, int32_t R, int32_t epoch, rf_stream_t stream) {
  RF_CHECK_ARG(flags && R >= 1 && R <= MAX_RANKS, "rf_moe_ep_wait: bad arguments");
  wait_flags_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(flags, R, epoch);
  return rf::check_launch("rf_moe_ep_wait");
}

extern "C" int rf_moe_ep_counts_push(const int32_t *counts, int32_t E, int32_t R, int32_t me, int32_t *const *dst,
                                     int32_t *const *flag, int32_t epoch, rf_stream_t stream) {
  RF_CHECK_ARG(R >= 1 && R <= MAX_RANKS && me >= 0 && me < R && E >= 1 && E <= 65535,
               "rf_moe_ep_counts_push: 1 <= R <= 64, 0 <= me < R, 1 <= E <= 65535");
  RF_CHECK_ARG(counts && dst && flag, "rf_moe_ep_counts_push: null pointer");
  CountsPushArgs a;
  a.counts = counts;
  a.R = R;
  a.me = me;
  a.E = E;
  a.epoch = epoch;
  for (int d = 0; d < R; ++d) {
    RF_CHECK_ARG(dst[d] && flag[d], "rf_moe_ep_counts_push: missing peer table or flag");
    a.dst[d] = dst[d];
    a.flag[d] = flag[d];
  }
  counts_push_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(a);
  return rf::check_launch("rf_moe_ep_counts_push");
}

extern "C" int rf_moe_ep_counts_collect(const int32_t *flags, const int32_t *table, int32_t R, int32_t E,
                                        int32_t epoch, int32_t *out, rf_stream_t stream) {
  RF_CHECK_ARG(flags && table && out && R >= 1 && R <= MAX_RANKS && E >= 1 && E <= 65535,
               "rf_moe_ep_counts_collect: bad arguments");
  counts_collect_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(flags, table, R, E, epoch, out);
  return rf::check_launch("rf_moe_ep_counts_collect");
}
