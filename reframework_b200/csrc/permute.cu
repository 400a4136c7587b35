// K2 — stable counting-sort permute of the (token, slot) pairs by expert, and
// the row gather that builds the expert-contiguous activation buffer.
//
// Restates the grouping of reframework/moe/fused.py:71-80 (bincount, then per
// active expert the rows `flat_expert == e` in ascending flat index t*K+k, and
// `hidden_states[tok]`).  Up to three launches:
//   1. permute_hist     per-block expert histograms of the flat ids (only
//                       with more than one block: a single block, as in
//                       decode, counts its own pairs)
//   2. permute_scatter  per-expert totals -> padded exclusive scan (offsets),
//                       then a stable in-block ranking (warp match + per-warp
//                       running cursors) that assigns every pair its row
//   3. gather_rows      x_perm[row] = x[src_slot[row] / K] (zero on pad rows),
//                       one warp per row with 16-byte vector copies
// The first two kernels touch only 4-byte ids; the gather is the HBM-bound part
// (reads and writes T*K*H elements).  A decode-sized call with the gather (one
// block of pairs, at most 256 experts) runs as one launch instead,
// permute_gather_single: every block ranks the pairs itself and then copies
// its share of the rows.
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int PT = 256;        // threads per block (8 warps)
constexpr int PW = PT / 32;
constexpr int CHUNK = 1024;    // pairs per block
constexpr int SUB = CHUNK / PW;  // pairs per warp

__global__ void __launch_bounds__(PT) permute_hist(const int32_t *ids, int64_t n, int E,
                                                   int32_t *block_counts) {
  extern __shared__ int s_hist[];
  for (int e = threadIdx.x; e < E; e += PT) s_hist[e] = 0;
  __syncthreads();
  const int64_t b0 = (int64_t)blockIdx.x * CHUNK;
  const int64_t b1 = min(n, b0 + CHUNK);
  for (int64_t i = b0 + threadIdx.x; i < b1; i += PT) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&s_hist[e], 1);
    else rf_report(RF_DEV_BAD_EXPERT_ID);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += PT) block_counts[(int64_t)blockIdx.x * E + e] = s_hist[e];
}

// Block-wide exclusive scan of v[0..E) in place (E <= 1024, PT threads);
// returns the total.  Uses s_tmp[PW] scratch.
__device__ int block_exclusive_scan(int *v, int E, int *s_tmp) {
  const int per = (E + PT - 1) / PT;
  const int beg = threadIdx.x * per;
  const int end = min(E, beg + per);
  int local = 0;
  for (int i = beg; i < end; ++i) local += v[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) s_tmp[warp] = inc;
  __syncthreads();
  int warp_base = 0, total = 0;
  for (int w = 0; w < PW; ++w) {
    if (w < warp) warp_base += s_tmp[w];
    total += s_tmp[w];
  }
  int run = warp_base + inc - local;
  __syncthreads();
  for (int i = beg; i < end; ++i) {
    const int c = v[i];
    v[i] = run;
    run += c;
  }
  __syncthreads();
  return total;
}

// One block per CHUNK pairs; warp w owns pairs [w0, w1) of the block and
// keeps their ids in registers (PER_LANE per lane) for both passes.
// single != 0 (one block in the grid, the decode case): the block's own warp
// histograms give the expert totals and block_counts is not read, so the
// permute_hist launch is skipped.
constexpr int PER_LANE = SUB / 32;

__global__ void __launch_bounds__(PT) permute_scatter(const int32_t *ids, int64_t n, int E, int align,
                                                      const int32_t *block_counts, int nblk,
                                                      int single, int32_t *offsets_out,
                                                      int32_t *counts_out, int32_t *row_of_slot,
                                                      int32_t *src_slot) {
  extern __shared__ int smem[];
  int *s_tot = smem;                 // [E]   expert totals, later the block's first row per expert
  int *s_off = s_tot + E;            // [E]   padded exclusive offsets
  int *s_before = s_off + E;         // [E]   pairs of earlier blocks per expert
  int *s_wc = s_before + E;          // [PW][E] per-warp counts, then per-warp cursors
  int *s_tmp = s_wc + PW * E;        // [PW]
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t w0 = (int64_t)b * CHUNK + (int64_t)warp * SUB;
  const int64_t w1 = min(n, w0 + SUB);

  // 0. this warp's ids, loaded once (invalid ids become -1 and are reported)
  int my_e[PER_LANE];
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int64_t i = w0 + j * 32 + lane;
    int e = -1;
    if (i < w1) {
      e = ids[i];
      if (e < 0 || e >= E) {
        if (single) rf_report(RF_DEV_BAD_EXPERT_ID);
        e = -1;
      }
    }
    my_e[j] = e;
  }
  for (int i = threadIdx.x; i < PW * E; i += PT) s_wc[i] = 0;
  __syncthreads();
  // 1. per-warp histograms of this block's chunk
  int *wc = s_wc + warp * E;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int e = my_e[j];
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    if (lane == __ffs(grp) - 1 && e >= 0) wc[e] += __popc(grp);
    __syncwarp();
  }
  __syncthreads();
  // 2. per-expert totals and this block's base within each expert
  for (int e = threadIdx.x; e < E; e += PT) {
    int tot = 0, before = 0;
    if (single) {
      for (int w = 0; w < PW; ++w) tot += s_wc[w * E + e];
    } else {
      for (int bb = 0; bb < nblk; ++bb) {
        const int c = block_counts[(int64_t)bb * E + e];
        if (bb < b) before += c;
        tot += c;
      }
    }
    s_tot[e] = tot;
    s_off[e] = (tot + align - 1) / align * align;
    s_before[e] = before;
  }
  __syncthreads();
  const int used = block_exclusive_scan(s_off, E, s_tmp);
  if (b == 0) {
    for (int e = threadIdx.x; e < E; e += PT) {
      offsets_out[e] = s_off[e];
      counts_out[e] = s_tot[e];
    }
    if (threadIdx.x == 0) offsets_out[E] = used;
  }
  // pad rows of the experts owned (e % nblk == b) by this block, one expert
  // per warp at a time
  for (int e = b + warp * nblk; e < E; e += nblk * PW) {
    const int p0 = s_off[e] + s_tot[e];
    const int p1 = s_off[e] + (s_tot[e] + align - 1) / align * align;
    for (int r = p0 + lane; r < p1; r += 32) src_slot[r] = -1;
  }
  // 3. exclusive prefix over warps, seeded with the block's first row
  for (int e = threadIdx.x; e < E; e += PT) {
    int run = s_off[e] + s_before[e];
    for (int w = 0; w < PW; ++w) {
      const int c = s_wc[w * E + e];
      s_wc[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  // 4. stable scatter: rank inside each 32-pair group, groups in order
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int64_t i = w0 + j * 32 + lane;
    const int e = my_e[j];
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(grp) - 1;
    int row = -1;
    if (e >= 0) row = wc[e] + __popc(grp & lt);
    __syncwarp();
    if (lane == leader && e >= 0) wc[e] += __popc(grp);
    __syncwarp();
    if (i < w1) {
      row_of_slot[i] = row;
      if (row >= 0) src_slot[row] = (int32_t)i;
    }
  }
}

template <int UNROLL>
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint8_t *src, const int32_t *index,
                                                          int64_t index_div, int64_t n_max,
                                                          const int32_t *n_dev, int64_t row_bytes,
                                                          uint8_t *dst) {
  const int64_t n = n_dev ? min((int64_t)*n_dev, n_max) : n_max;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * 8;
  const int64_t vecs = row_bytes / 16;
  for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < n; r += warps) {
    const int32_t s = index[r];
    uint4 *d = reinterpret_cast<uint4 *>(dst + r * row_bytes);
    if (s < 0) {
      for (int64_t v = lane; v < vecs; v += 32) d[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint4 *q = reinterpret_cast<const uint4 *>(src + (int64_t)(s / index_div) * row_bytes);
    int64_t v = lane;
    for (; v + 32 * (UNROLL - 1) < vecs; v += 32 * UNROLL) {
      uint4 t[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) t[u] = __ldg(q + v + 32 * u);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) d[v + 32 * u] = t[u];
    }
    for (; v < vecs; v += 32) d[v] = __ldg(q + v);
  }
}

// Decode-sized permute with the gather in the same launch (at most CHUNK
// pairs, at most FUSED_MAX_E experts).  Every block ranks all the pairs in its
// own shared memory (a few hundred ids: the single-block permute_scatter
// algorithm, same stable order), block 0 writes the permutation, and then all
// blocks copy rows: row r of expert e (found by a binary search of the padded
// offsets) is x[pair / K] for its pair, or zeros on pad rows.  This replaces
// the scatter + gather pair of launches when a decode step's permute is
// latency-bound.
constexpr int FUSED_MAX_E = 256;

__global__ void __launch_bounds__(PT) permute_gather_single(const int32_t *ids, int64_t n, int E, int align,
                                                            int64_t K, const uint8_t *x, int64_t row_bytes,
                                                            int32_t *offsets_out, int32_t *counts_out,
                                                            int32_t *row_of_slot, int32_t *src_slot,
                                                            uint8_t *x_perm) {
  __shared__ int s_tot[FUSED_MAX_E];      // expert totals
  __shared__ int s_off[FUSED_MAX_E + 1];  // padded exclusive offsets; [E] = rows used
  __shared__ int s_cb[FUSED_MAX_E];       // exclusive prefix of the totals (compact row base)
  __shared__ int s_wc[PW * FUSED_MAX_E];  // per-warp counts, then per-warp cursors
  __shared__ int s_tmp[PW];
  __shared__ int s_src[CHUNK];            // pair of each real row, in compact row order
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool lead = blockIdx.x == 0;
  const int64_t w0 = (int64_t)warp * SUB;
  const int64_t w1 = min(n, w0 + SUB);
  int my_e[PER_LANE];
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int64_t i = w0 + j * 32 + lane;
    int e = -1;
    if (i < w1) {
      e = ids[i];
      if (e < 0 || e >= E) {
        if (lead) rf_report(RF_DEV_BAD_EXPERT_ID);
        e = -1;
      }
    }
    my_e[j] = e;
  }
  for (int i = threadIdx.x; i < PW * E; i += PT) s_wc[i] = 0;
  __syncthreads();
  int *wc = s_wc + warp * E;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int e = my_e[j];
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    if (lane == __ffs(grp) - 1 && e >= 0) wc[e] += __popc(grp);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += PT) {
    int tot = 0;
    for (int w = 0; w < PW; ++w) tot += s_wc[w * E + e];
    s_tot[e] = tot;
    s_cb[e] = tot;
    s_off[e] = (tot + align - 1) / align * align;
  }
  __syncthreads();
  const int used = block_exclusive_scan(s_off, E, s_tmp);
  block_exclusive_scan(s_cb, E, s_tmp);
  if (threadIdx.x == 0) s_off[E] = used;
  if (lead) {
    for (int e = threadIdx.x; e < E; e += PT) {
      offsets_out[e] = s_off[e];
      counts_out[e] = s_tot[e];
    }
    if (threadIdx.x == 0) offsets_out[E] = used;
    for (int e = warp; e < E; e += PW) {  // pad rows of every expert
      const int p0 = s_off[e] + s_tot[e];
      const int p1 = s_off[e] + (s_tot[e] + align - 1) / align * align;
      for (int r = p0 + lane; r < p1; r += 32) src_slot[r] = -1;
    }
  }
  for (int e = threadIdx.x; e < E; e += PT) {
    int run = s_off[e];
    for (int w = 0; w < PW; ++w) {
      const int c = s_wc[w * E + e];
      s_wc[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int64_t i = w0 + j * 32 + lane;
    const int e = my_e[j];
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(grp) - 1;
    int row = -1;
    if (e >= 0) row = wc[e] + __popc(grp & lt);
    __syncwarp();
    if (lane == leader && e >= 0) wc[e] += __popc(grp);
    __syncwarp();
    if (i < w1) {
      if (row >= 0) s_src[s_cb[e] + (row - s_off[e])] = (int)i;
      if (lead) {
        row_of_slot[i] = row;
        if (row >= 0) src_slot[row] = (int32_t)i;
      }
    }
  }
  __syncthreads();
  // the gather: one warp per row, 16-byte vectors
  const int64_t vecs = row_bytes / 16;
  const int64_t warps = (int64_t)gridDim.x * PW;
  for (int64_t r = (int64_t)blockIdx.x * PW + warp; r < used; r += warps) {
    int lo = 0, hi = E - 1;  // the last expert whose segment starts at or before r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_off[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int64_t jrow = r - s_off[lo];
    uint4 *d = reinterpret_cast<uint4 *>(x_perm + r * row_bytes);
    if (jrow >= s_tot[lo]) {
      for (int64_t v = lane; v < vecs; v += 32) d[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint4 *q = reinterpret_cast<const uint4 *>(x + (int64_t)(s_src[s_cb[lo] + jrow] / K) * row_bytes);
    int64_t v = lane;
    for (; v + 96 < vecs; v += 128) {
      uint4 t[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) t[u] = __ldg(q + v + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) d[v + 32 * u] = t[u];
    }
    for (; v < vecs; v += 32) d[v] = __ldg(q + v);
  }
}

int launch_gather(const void *src, const int32_t *index, int64_t index_div, int64_t n_max,
                  const int32_t *n_dev, int64_t row_bytes, void *dst, cudaStream_t st) {
  if (n_max <= 0) return RF_OK;
  int64_t blocks = (n_max + 7) / 8;
  const int64_t cap = (int64_t)rf::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  gather_rows_kernel<4><<<(int)blocks, 256, 0, st>>>((const uint8_t *)src, index, index_div, n_max,
                                                      n_dev, row_bytes, (uint8_t *)dst);
  return rf::check_launch("rf_moe_gather_rows");
}

// hist (several blocks only) + scatter + optional gather.  block_counts holds
// ceil(n/CHUNK) * E words when there is more than one block.
int launch_permute(const int32_t *topk_ids, int64_t n, int64_t K, int64_t E, int64_t align,
                   const void *x, int dtype, int64_t H, int32_t *expert_offsets,
                   int32_t *expert_counts, int32_t *row_of_slot, int32_t *src_slot, void *x_perm,
                   int32_t *block_counts, cudaStream_t st, const char *name) {
  const std::string nm(name);
  if (n == 0) {
    // no pairs: every expert is empty
    cudaError_t e1 = cudaMemsetAsync(expert_offsets, 0, (E + 1) * 4, st);
    cudaError_t e2 = cudaMemsetAsync(expert_counts, 0, E * 4, st);
    if (e1 != cudaSuccess || e2 != cudaSuccess) return rf::fail(RF_ERR_CUDA, nm + ": memset failed");
    return RF_OK;
  }
  const int nblk = (int)((n + CHUNK - 1) / CHUNK);
  if (nblk == 1 && x_perm && E <= FUSED_MAX_E) {
    // decode-sized: rank and gather in one launch (grid sized for the padded
    // rows, at most two blocks per SM; every block ranks the pairs itself)
    const int64_t rows_cap = n + E * (align - 1);
    const int64_t blocks = std::min<int64_t>((rows_cap + PW - 1) / PW, (int64_t)rf::num_sms() * 2);
    permute_gather_single<<<(int)blocks, PT, 0, st>>>(topk_ids, n, (int)E, (int)align, K,
                                                       (const uint8_t *)x, H * (int64_t)rf::dtype_size(dtype),
                                                       expert_offsets, expert_counts, row_of_slot, src_slot,
                                                       (uint8_t *)x_perm);
    return rf::check_launch((nm + "(rank+gather)").c_str());
  }
  if (nblk > 1) {
    // permute_hist writes every one of the nblk*E words the scatter reads
    permute_hist<<<nblk, PT, E * sizeof(int), st>>>(topk_ids, n, (int)E, block_counts);
    int rc = rf::check_launch((nm + "(hist)").c_str());
    if (rc) return rc;
  }
  const size_t smem = (size_t)(3 * E + PW * E + PW) * sizeof(int);
  permute_scatter<<<nblk, PT, smem, st>>>(topk_ids, n, (int)E, (int)align, block_counts, nblk,
                                          nblk == 1 ? 1 : 0, expert_offsets, expert_counts,
                                          row_of_slot, src_slot);
  int rc = rf::check_launch((nm + "(scatter)").c_str());
  if (rc) return rc;
  if (x_perm) {
    const int64_t rows_cap = n + E * (align - 1);
    return launch_gather(x, src_slot, K, rows_cap, expert_offsets + E,
                         H * (int64_t)rf::dtype_size(dtype), x_perm, st);
  }
  return RF_OK;
}

}  // namespace

extern "C" size_t rf_moe_permute_workspace_size(int64_t n_pairs, int64_t num_experts) {
  const int64_t nblk = n_pairs > 0 ? (n_pairs + CHUNK - 1) / CHUNK : 1;
  return (size_t)(nblk * num_experts * 4 + 256);
}

extern "C" int rf_moe_gather_rows(const void *src, const int32_t *index, int64_t index_div,
                                  int64_t n_rows_max, const int32_t *n_rows_dev, int64_t row_bytes,
                                  void *dst, rf_stream_t stream) {
  RF_CHECK_ARG(row_bytes > 0 && row_bytes % 16 == 0, "rf_moe_gather_rows: row_bytes % 16 != 0");
  RF_CHECK_ARG(index_div >= 1, "rf_moe_gather_rows: index_div must be >= 1");
  RF_CHECK_ARG(n_rows_max == 0 || (src && index && dst), "rf_moe_gather_rows: null pointer");
  RF_CHECK_ARG((uintptr_t)src % 16 == 0 && (uintptr_t)dst % 16 == 0,
               "rf_moe_gather_rows: src/dst must be 16-byte aligned");
  return launch_gather(src, index, index_div, n_rows_max, n_rows_dev, row_bytes, dst,
                       (cudaStream_t)stream);
}

extern "C" int rf_moe_permute(const int32_t *topk_ids, int64_t T, int64_t K, int64_t E,
                              int64_t align, const void *x, int dtype, int64_t H,
                              int32_t *expert_offsets, int32_t *expert_counts,
                              int32_t *row_of_slot, int32_t *src_slot, void *x_perm,
                              void *workspace, size_t workspace_bytes, rf_stream_t stream) {
  RF_CHECK_ARG(T >= 0 && K >= 1 && E >= 1 && E <= 1024, "rf_moe_permute: bad sizes (E <= 1024)");
  RF_CHECK_ARG(align == 1 || align == 64 || align == 128 || align == 256,
               "rf_moe_permute: align must be 1, 64, 128 or 256");
  const int64_t n = T * K;
  RF_CHECK_ARG(n + E * (align - 1) < (int64_t)1 << 31, "rf_moe_permute: too many rows for int32");
  RF_CHECK_ARG(expert_offsets && expert_counts && (n == 0 || (row_of_slot && src_slot)),
               "rf_moe_permute: null output");
  RF_CHECK_ARG(workspace_bytes >= rf_moe_permute_workspace_size(n, E) && workspace,
               "rf_moe_permute: workspace too small");
  RF_CHECK_ARG(!x_perm || n == 0 || (x && rf::valid_dtype(dtype) && H > 0 &&
                                      (H * (int64_t)rf::dtype_size(dtype)) % 16 == 0),
               "rf_moe_permute: gather needs x, a dtype and H*elsize % 16 == 0");
  return launch_permute(topk_ids, n, K, E, align, x, dtype, H, expert_offsets, expert_counts,
                        row_of_slot, src_slot, x_perm, reinterpret_cast<int32_t *>(workspace),
                        (cudaStream_t)stream, "rf_moe_permute");
}

// ---------------------------------------------------------------------------
// rf_moe_permute_noalloc — the same permute for callers that cannot allocate
// device memory.  Its only scratch (the per-block expert histograms) lives in
// this file-scope device array instead of a caller workspace.  Every GPU that
// loads the library holds the array until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocScratchWords = 1 << 16;  // 65,536 int32 = 256 KiB per device
static __device__ __align__(256) int32_t g_noalloc_block_counts[kNoAllocScratchWords];

// Device address of g_noalloc_block_counts, fetched once per device.  In host
// code the array's name is only a host-side handle, so the kernels must be
// given this address instead.  The cache is keyed by device ordinal and lives
// as long as the process: after cudaDeviceReset the module may load at
// another address, so the header tells callers not to use this entry point
// past a reset.
int noalloc_scratch(int32_t **out) {
  static std::mutex mu;
  static std::vector<int32_t *> addr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return rf::fail(RF_ERR_CUDA, std::string("rf_moe_permute_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if ((int)addr.size() <= dev) addr.resize(dev + 1, nullptr);
  if (!addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_block_counts);
    if (e != cudaSuccess || !p)
      return rf::fail(RF_ERR_CUDA, std::string("rf_moe_permute_noalloc: cudaGetSymbolAddress: ") +
                                       cudaGetErrorString(e));
    addr[dev] = static_cast<int32_t *>(p);
  }
  *out = addr[dev];
  return RF_OK;
}

}  // namespace

extern "C" int rf_moe_permute_noalloc(const int32_t *topk_ids, int64_t T, int64_t K, int64_t E,
                                      int64_t align, const void *x, int dtype, int64_t H,
                                      int32_t *expert_offsets, int32_t *expert_counts,
                                      int32_t *row_of_slot, int32_t *src_slot, void *x_perm,
                                      rf_stream_t stream) {
  RF_CHECK_ARG(T >= 0 && K >= 1 && E >= 1 && E <= 1024, "rf_moe_permute_noalloc: bad sizes (E <= 1024)");
  RF_CHECK_ARG(align == 1 || align == 64 || align == 128 || align == 256,
               "rf_moe_permute_noalloc: align must be 1, 64, 128 or 256");
  const int64_t n = T * K;
  RF_CHECK_ARG(n + E * (align - 1) < (int64_t)1 << 31, "rf_moe_permute_noalloc: too many rows for int32");
  const int64_t nblk = n > 0 ? (n + CHUNK - 1) / CHUNK : 1;
  if (nblk * E > kNoAllocScratchWords)
    return rf::fail(RF_ERR_ARG,
                    "rf_moe_permute_noalloc: ceil(T*K/" + std::to_string(CHUNK) + ") * E = " +
                        std::to_string(nblk * E) + " histogram words exceeds the fixed scratch of " +
                        std::to_string(kNoAllocScratchWords) + "; use rf_moe_permute with a workspace");
  RF_CHECK_ARG(expert_offsets && expert_counts && (n == 0 || (row_of_slot && src_slot)),
               "rf_moe_permute_noalloc: null output");
  RF_CHECK_ARG(!x_perm || n == 0 || (x && rf::valid_dtype(dtype) && H > 0 &&
                                      (H * (int64_t)rf::dtype_size(dtype)) % 16 == 0),
               "rf_moe_permute_noalloc: gather needs x, a dtype and H*elsize % 16 == 0");
  int32_t *block_counts = nullptr;
  int rc = noalloc_scratch(&block_counts);
  if (rc) return rc;
  return launch_permute(topk_ids, n, K, E, align, x, dtype, H, expert_offsets, expert_counts,
                        row_of_slot, src_slot, x_perm, block_counts, (cudaStream_t)stream,
                        "rf_moe_permute_noalloc");
}
