/*
 * rf_moe.h — C ABI of the B200 (sm_100a) MoE-layer forward.
 *
 * One entry point per stage of the MoE layer.  Every call takes raw device
 * pointers owned by the caller (the library never allocates or frees tensor
 * memory), int64 sizes, and a CUDA stream; it enqueues work on that stream and
 * returns an rf_status.  No call synchronises the stream, and no C++
 * exception crosses this boundary.  rf_moe_last_error() returns the message
 * of the calling thread's most recent failure.
 *
 * An empty batch is valid: with T == 0 (or no rows, for the grouped GEMMs) the
 * router, permute, grouped GEMMs and combines accept null pointers for the
 * zero-size token and row buffers (what a zero-row tensor hands over) and
 * return RF_OK; the permute still writes its (all-zero) offsets and counts.
 *
 * Row layout shared by the stages: the T*K (token, slot) pairs are grouped by
 * expert ("permuted rows").  Expert e owns rows
 *     [expert_offsets[e], expert_offsets[e] + expert_counts[e])
 * and every expert_offsets[e] is a multiple of the `align` given to
 * rf_moe_permute (128 for the grouped GEMMs, 1 for a compact layout).
 * Within an expert, rows are in ascending flat order t*K+k — the order of the
 * reference's per-expert boolean selection.  Pad rows (between an expert's
 * last row and the next expert's first) hold src_slot = -1 and zero inputs.
 * A buffer of permuted rows needs rf_moe_rows_capacity(T*K, E, align) rows.
 *
 * Reference interfaces replaced (paths relative to the Reframework root):
 *   rf_moe_router_topk      reframework/moe/moe_layer.py:320-344 (FusedMoE.route)
 *                           reframework/moe/fused.py:32-46 (torch_fused_topk)
 *   rf_moe_permute          reframework/moe/fused.py:71-80 (bincount + per-expert
 *                           select + hidden_states[tok] gather)
 *   rf_moe_gather_rows      reframework/moe/fused.py:80 (hidden_states[tok]);
 *                           reframework/parallel/dist.py:194-206 (all_to_all
 *                           chunk packing, for EP dispatch/combine)
 *   rf_moe_grouped_gemm_gated  reframework/moe/fused.py:81-82 (x @ w1[e].t(),
 *                           gated_act_and_mul) + reframework/layers/activation.py:15-59
 *   rf_moe_grouped_gemm_gated_gather  the same with fused.py:80 (hidden_states[tok])
 *                           folded into the operand load
 *   rf_moe_grouped_gemm_down   reframework/moe/fused.py:83 (inter @ w2[e].t())
 *   rf_moe_grouped_gemm_down_add  the same plus a rounded add: the shared
 *                           experts' sum (reframework/layers/mlp.py:35-39 each)
 *   rf_moe_combine          reframework/moe/fused.py:84-86 (y * w, index_add_)
 *                           + reframework/layers/norm.py:43-53 (residual add, opt-in)
 *   rf_moe_combine_rmsnorm  the same + the next RMSNorm (norm.py:27-53)
 *   rf_moe_ep_push_rows / rf_moe_ep_wait  reframework/parallel/dist.py:194-206
 *                           (EP dispatch / return all-to-all) as NVLink stores
 *   rf_moe_ep_counts_push / _collect  the per-step counts all-gather
 *                           (dist.py:186-191) as NVLink stores
 *   rf_moe_ep_plan / rf_moe_ep_pair_rows  the split of that exchange, replacing
 *                           the replicate-and-all-reduce forward of
 *                           reframework/parallel/ep.py:119-150
 *   rf_moe_ep_devplan, rf_moe_ep_devplan_host, _push, _regroup,
 *                           _regroup_remote  the same plan
 *                           and exchange driven from the GPU (no host sync)
 *   rf_moe_ep_devplan_down_return  reframework/moe/fused.py:83 on the expert's
 *                           rank + the return all-to-all (dist.py:194-206) in
 *                           one kernel
 *   rf_moe_peer_alloc / _open / _close / _free  buffers mapped by every peer
 *                           (no reference counterpart)
 *   rf_moe_int8_quantize, rf_moe_int8_grouped_gemm, rf_moe_split_combine
 *                           the int8 half of the CPU/GPU expert split
 *                           (reframework/moe/fused.py:89-197,
 *                           moe_layer.py:523-627, offload_cache.py:58-72)
 */
#ifndef RF_MOE_H
#define RF_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *rf_stream_t; /* a cudaStream_t; NULL = legacy default stream */

typedef enum {
  RF_F32 = 0,
  RF_F16 = 1,
  RF_BF16 = 2
} rf_dtype;

typedef enum {
  RF_ACT_SILU = 0,      /* silu(gate) * up            (activation.py:15-24) */
  RF_ACT_GELU = 1,      /* gelu(gate) * up, erf form  (activation.py:27-35) */
  RF_ACT_GELU_TANH = 2  /* gelu_tanh(gate) * up       (activation.py:38-46) */
} rf_activation;

typedef enum {
  RF_OK = 0,
  RF_ERR_ARG = 1,          /* invalid argument (message says which) */
  RF_ERR_UNSUPPORTED = 2,  /* valid but not implemented for these sizes/dtypes */
  RF_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  RF_ERR_DEVICE = 4        /* a kernel reported an error (see rf_moe_device_status) */
} rf_status;

/* Device-side error codes reported by rf_moe_device_status. */
#define RF_DEV_OK 0
#define RF_DEV_BAD_EXPERT_ID 1   /* a routed id was outside [0, E) */
#define RF_DEV_WAIT_TIMEOUT 2    /* a pipeline wait ran out of time and gave up */
#define RF_DEV_PLAN_OVERFLOW 3   /* an expert-parallel plan needed more rows than its buffers hold */

/* Message of the calling thread's last failed call ("" if none). */
const char *rf_moe_last_error(void);

/* ABI version (major*100 + minor). */
int rf_moe_version(void);

/* Reads and clears the device-side error word of the current device
 * (synchronises the device).  *code gets one of RF_DEV_*. */
int rf_moe_device_status(int *code);

/* Rows needed for the permuted layout of n_pairs = T*K pairs over E experts. */
int64_t rf_moe_rows_capacity(int64_t n_pairs, int64_t num_experts, int64_t align);

/* Workspace bytes rf_moe_permute needs (caller-allocated device memory). */
size_t rf_moe_permute_workspace_size(int64_t n_pairs, int64_t num_experts);

/*
 * Workspace bytes rf_moe_router_topk needs with a gate of H columns over E
 * experts (+1 column when a shared-expert gate is given): fp32 partial logits
 * of ceil(H/256) slices of the hidden dimension.
 */
size_t rf_moe_router_workspace_size(int64_t T, int64_t H, int64_t E, int has_shared_gate);

/*
 * K1 — router.  For each token t:
 *   logit[e] = sum_h x[t,h] * gate[e,h]   (fp32 accumulation in a fixed order
 *              that depends on H only: a sequential chain over each 256-wide
 *              slice of h, then the slice sums in slice order; the result for
 *              a token does not depend on T or on the other tokens)
 *   if round_dtype >= 0: logit rounded to that dtype (the reference runs the
 *                        router GEMM in the layer dtype, moe_layer.py:324)
 *   if bias:             logit += bias[e]  (fp32 router with load bias)
 *   p = softmax(logit) in fp32; top-k by p (descending, ties -> lower id);
 *   weights = p / sum(top-k p) when renormalize, else p.
 * entropy_k_min > 0 selects the entropy-adaptive branch of moe_layer.py:327-342
 * (slots past k_dyn get weight 0; weights always renormalised).
 * shared_gate (optional, [H] in gate_dtype) also writes
 *   shared_scale[t] = sigmoid(sum_h x[t,h] * shared_gate[h]).
 * Outputs: topk_weights [T,K] fp32; topk_ids32 [T,K] and/or topk_ids64 [T,K]
 * (either may be NULL, not both); logits [T,E] fp32 (NULL to skip).
 * Requires 1 <= K <= min(E, 16), E <= 1024, H % 8 == 0.
 * gate == NULL means x already holds the [T,E] logits (H must equal E): the
 * call is then torch_fused_topk alone and needs no workspace.
 * workspace: rf_moe_router_workspace_size(T, H, E, shared_gate != NULL)
 * bytes of device memory, 16-byte aligned.
 */
int rf_moe_router_topk(const void *x, int x_dtype, const void *gate, int gate_dtype,
                       const float *bias, int64_t T, int64_t H, int64_t E, int64_t K,
                       int renormalize, int round_dtype, int entropy_k_min,
                       const void *shared_gate, float *shared_scale,
                       float *topk_weights, int32_t *topk_ids32, int64_t *topk_ids64,
                       float *logits, void *workspace, size_t workspace_bytes,
                       rf_stream_t stream);

/*
 * K2 — counting-sort permute of the T*K pairs by expert (stable), plus the
 * gather of the activation rows.  Inputs: topk_ids [T,K] int32.
 * Outputs (device):
 *   expert_offsets [E+1] int32   first row of each expert (multiple of align);
 *                                expert_offsets[E] = rows used
 *   expert_counts  [E]   int32
 *   row_of_slot    [T*K] int32   permuted row of pair t*K+k (-1 if its id was invalid)
 *   src_slot       [rows_capacity] int32  pair t*K+k feeding each row, -1 for pads
 *   x_perm         [rows_capacity, H] (optional; NULL skips the gather):
 *                  x_perm[row] = x[src_slot[row] / K], zero on pad rows
 * workspace: rf_moe_permute_workspace_size(T*K, E) bytes.
 * align is one of 1, 64, 128, 256; E <= 1024.
 */
int rf_moe_permute(const int32_t *topk_ids, int64_t T, int64_t K, int64_t E, int64_t align,
                   const void *x, int dtype, int64_t H,
                   int32_t *expert_offsets, int32_t *expert_counts, int32_t *row_of_slot,
                   int32_t *src_slot, void *x_perm, void *workspace, size_t workspace_bytes,
                   rf_stream_t stream);

/*
 * rf_moe_permute without a workspace argument: it allocates nothing and uses
 * no caller scratch.  There is no counterpart in the reference.
 *
 * For callers that cannot allocate device memory at the point where they
 * permute: for example a host that plans every device buffer at start-up and
 * forbids later allocations (cudaMalloc may also synchronise the device, which
 * a latency-bound serving loop cannot afford), or a plugin whose host owns the
 * memory pool and only hands it input and output buffers.  The caller still
 * passes every input and output; the kernels' scratch (per-block expert
 * histograms) is a file-scope device array of 65,536 int32 words (256 KiB)
 * that every GPU which loads the library holds until the process exits.
 *
 * Limit: ceil(T*K / 1024) * E <= 65536 (e.g. T*K <= 1,048,576 pairs with 64
 * experts); larger calls fail with RF_ERR_ARG and a message — use
 * rf_moe_permute with a workspace for them.  Outputs and their meaning are
 * those of rf_moe_permute.
 *
 * The first call on a device looks up the array's device address for that
 * device (cudaGetSymbolAddress, with that device current); make that first
 * call before any stream capture.  The address is kept per device ordinal
 * for the life of the process: it does not survive cudaDeviceReset (or any
 * other teardown of the device's primary context), after which this entry
 * point must not be called again in that process.  The address is kept per device ordinal
 * for the life of the process: it does not survive cudaDeviceReset (or any
 * other teardown of the device's primary context), after which this entry
 * point must not be called again in that process.  All calls share the one array, which keeps
 * the last call's contents (nothing in it needs to start at zero: each call
 * overwrites the words it reads), so calls that overlap on the same GPU —
 * from two streams at once, for instance — race; order them on one stream or
 * with events.
 */
int rf_moe_permute_noalloc(const int32_t *topk_ids, int64_t T, int64_t K, int64_t E, int64_t align,
                           const void *x, int dtype, int64_t H,
                           int32_t *expert_offsets, int32_t *expert_counts, int32_t *row_of_slot,
                           int32_t *src_slot, void *x_perm, rf_stream_t stream);

/*
 * Row gather: dst[r] = src[index[r] / index_div] for r < n_rows (n_rows read
 * from *n_rows_dev when non-NULL, else n_rows_max), zero rows where index < 0.
 * Rows are `row_bytes` long (a multiple of 16); src/dst 16-byte aligned.
 */
int rf_moe_gather_rows(const void *src, const int32_t *index, int64_t index_div,
                       int64_t n_rows_max, const int32_t *n_rows_dev, int64_t row_bytes,
                       void *dst, rf_stream_t stream);

/*
 * K3 — grouped GEMM with the gated activation fused into the epilogue:
 *   for every expert e in the group list and every row r of expert e:
 *     h[r, j] = act(sum_k a[r,k] * w1[s,j,k]) * (sum_k a[r,k] * w1[s,I+j,k])
 *   with s = expert_slot ? expert_slot[e] : e, j in [0, I).
 * a [rows_capacity, H], w1 [num_slots, 2I, H] (rows 0..I-1 gate, I..2I-1 up),
 * h [rows_capacity, I]; all in `dtype`; fp32 accumulation.  For 16-bit dtypes
 * the epilogue keeps the reference's rounding points: both sums are rounded
 * to `dtype`, act() of the rounded gate is rounded to `dtype`, and the product
 * is rounded on store.  bf16/fp16 run on tcgen05 tensor cores (TMA-fed, TMEM
 * accumulators) when H % 8 == 0 and I % 8 == 0; fp32 (and other shapes) run
 * on CUDA cores.  Segments may start at any row.
 * groups: expert ids to compute (NULL = all E experts, n_groups ignored).
 */
int rf_moe_grouped_gemm_gated(const void *a, const void *w1, void *h,
                              const int32_t *expert_offsets, const int32_t *expert_counts,
                              const int32_t *expert_slot, const int32_t *groups, int64_t n_groups,
                              int64_t E, int64_t num_slots, int64_t rows_capacity,
                              int64_t H, int64_t I, int dtype, int activation,
                              rf_stream_t stream);

/*
 * K3 with the row gather fused into the operand load: the same h as
 * rf_moe_grouped_gemm_gated computes from a = x_perm, but row r of the
 * permuted layout is read straight from the token rows,
 *   a[r] = x[src_slot[r] / topk]      (src_slot from rf_moe_permute; pad rows,
 *                                       src_slot = -1, are never stored)
 * with TMA tile::gather4 (four token rows per copy), so the expert-ordered
 * activation copy (T*K rows) is neither written nor read.  x [x_rows, H].
 * Tensor cores only (bf16/fp16, H % 8 == 0, I % 8 == 0, 16-byte aligned
 * pointers); otherwise returns RF_ERR_UNSUPPORTED and the caller gathers with
 * rf_moe_permute(..., x_perm) and calls rf_moe_grouped_gemm_gated.
 * Replaces reframework/moe/fused.py:80-82 (hidden_states[tok] @ w1[e].t() +
 * gated_act_and_mul).
 */
int rf_moe_grouped_gemm_gated_gather(const void *x, int64_t x_rows, const int32_t *src_slot,
                                     int64_t topk, const void *w1, void *h,
                                     const int32_t *expert_offsets, const int32_t *expert_counts,
                                     const int32_t *expert_slot, const int32_t *groups,
                                     int64_t n_groups, int64_t E, int64_t num_slots,
                                     int64_t rows_capacity, int64_t H, int64_t I, int dtype,
                                     int activation, rf_stream_t stream);

/*
 * Selects the grouped-GEMM implementation for subsequent calls of this
 * process: 0 = automatic (tensor cores whenever the shape allows, tile width
 * chosen per launch), 1 = CUDA cores only (used by tests to cross-check the
 * two implementations), 2 / 3 / 4 = single-CTA tensor-core kernel with tile
 * width N = 256 / 128 / 64, 5 = the CTA-pair tensor-core kernel (weights on
 * the MMA's M side; the automatic choice for 16-bit layers).
 * No reference counterpart (the reference has a single torch matmul path).
 */
int rf_moe_set_gemm_impl(int impl);

/*
 * K4 — grouped down-projection GEMM:
 *   y[r, n] = sum_j h[r,j] * w2[s,n,j]      for rows r of each listed expert
 * h [rows_capacity, I], w2 [num_slots, H, I], y [rows_capacity, H].
 * Same dtype / group / slot rules as K3.
 */
int rf_moe_grouped_gemm_down(const void *h, const void *w2, void *y,
                             const int32_t *expert_offsets, const int32_t *expert_counts,
                             const int32_t *expert_slot, const int32_t *groups, int64_t n_groups,
                             int64_t E, int64_t num_slots, int64_t rows_capacity,
                             int64_t H, int64_t I, int dtype, rf_stream_t stream);

/*
 * K4 with an addend: y[r, n] = round(addend[r, n] + round(sum_j h[r,j] *
 * w2[s,n,j])) in the layer dtype (addend has y's layout and may be y).  The
 * layer sums its shared experts with it in the reference harness's order:
 * each expert's output rounded, then added in the layer dtype
 * (sum_s MLP_s(x), reframework/layers/mlp.py:35-39 per shared expert).
 */
int rf_moe_grouped_gemm_down_add(const void *h, const void *w2, void *y, const void *addend,
                                 const int32_t *expert_offsets, const int32_t *expert_counts,
                                 const int32_t *expert_slot, const int32_t *groups, int64_t n_groups,
                                 int64_t E, int64_t num_slots, int64_t rows_capacity,
                                 int64_t H, int64_t I, int dtype, rf_stream_t stream);

/*
 * Expert-parallel exchange plan for one rank (host function, no GPU work).
 * Replaces the reference's replicate-and-all-reduce combine
 * (reframework/parallel/ep.py:120-150) with a token all-to-all; this computes
 * that all-to-all's bookkeeping.
 *   counts       [R, E] rows each rank routes to each expert this step
 *   slot_experts experts held per rank, rank r's at
 *                [slot_offsets[r], slot_offsets[r+1]) (primaries, then replicas)
 * Replicated experts' rows are split over their holders by water-filling
 * (`rounds` passes) so the ranks' row counts even out; holders take
 * consecutive runs of an expert's rows in rank order.
 * Outputs: send_splits[R], recv_splits[R] (rows), and in `packed` (int32):
 *   gather_index  GEMM row -> received row (-1 on pad rows), slot segments
 *                 aligned to `align`
 *   inverse_index received row -> GEMM row
 *   local_offsets [S+1], local_counts [S] of this rank's S slots
 *   send_index    send position -> permuted row, and pos_of_row (its
 *                 inverse) — both empty when the send order is the identity
 * layout[15]: {off, len} of the six arrays at [0..11], then rows_capacity,
 * send_is_identity, needed packed size.  Fails with RF_ERR_ARG (and fills
 * layout) when packed_capacity is too small.
 */
int rf_moe_ep_plan(const int32_t *counts, int32_t R, int32_t E, int32_t rank,
                   const int32_t *slot_experts, const int32_t *slot_offsets, int32_t align,
                   int32_t rounds, int64_t *send_splits, int64_t *recv_splits,
                   int32_t *packed, int64_t packed_capacity, int64_t *layout);

/*
 * M[s * R + d] = rows rank s sends to rank d this step: the all-to-all matrix
 * of the split rf_moe_ep_plan computes (same arguments).  With it every rank
 * knows where its rows land in every peer's receive buffer.
 */
int rf_moe_ep_pair_rows(const int32_t *counts, int32_t R, int32_t E, const int32_t *slot_experts,
                        const int32_t *slot_offsets, int32_t rounds, int64_t *pair_rows);

/*
 * Peer-visible device memory (CUDA IPC): rf_moe_peer_alloc allocates `bytes`
 * (zeroed) and writes a 64-byte handle; a process on another GPU of the node
 * maps it with rf_moe_peer_open and unmaps with rf_moe_peer_close; the owner
 * releases it with rf_moe_peer_free (after every peer closed it).
 */
int rf_moe_peer_alloc(size_t bytes, void **ptr, void *handle);
int rf_moe_peer_open(const void *handle, void **ptr);
int rf_moe_peer_close(void *ptr);
int rf_moe_peer_free(void *ptr);

/*
 * EP row exchange over NVLink peer memory — replaces the dispatch and return
 * all-to-alls (reframework/parallel/dist.py:194-206) of the token-dispatch EP
 * layer with one-sided stores:
 *   for each of this rank's rows i in [chunk_off[d], chunk_off[d+1]):
 *     j   = idx1 ? idx1[i] : i;   row = idx2 ? idx2[j] / div : j
 *     dst[d][dst_row0[d] + i - chunk_off[d]] = src[row]      (row_bytes each)
 *   then *flag[d] = epoch for every d (release, system scope) once all rows of
 *   the launch are visible.  dst/flag: R device pointers (peer mappings or
 *   this rank's own buffers), passed by value (R <= 64); done: a zeroed
 *   uint32 of this rank.
 * rf_moe_ep_wait: stream-ordered wait until flags[0..R) all equal epoch
 * (bounded: after 2 s it sets RF_DEV_WAIT_TIMEOUT and returns).
 */
int rf_moe_ep_push_rows(const void *src, int64_t row_bytes, const int32_t *idx1, const int32_t *idx2,
                        int64_t div, int32_t R, int32_t me, const int64_t *chunk_off,
                        const int64_t *dst_row0, void *const *dst, int32_t *const *flag, int32_t epoch,
                        uint32_t *done, rf_stream_t stream);
int rf_moe_ep_wait(const int32_t *flags, int32_t R, int32_t epoch, rf_stream_t stream);

/*
 * The counts all-gather of the expert-parallel step (reframework/parallel/
 * dist.py:186-191 as the token-dispatch layer uses it: every rank needs every
 * rank's routed rows per expert) as one-sided NVLink stores.
 * rf_moe_ep_counts_push: counts [E] (this rank's) into row `me` of every
 *   rank's table, dst[d] = rank d's [R][E] int32 table for this step (peer
 *   mappings or this rank's own), then flag[d] = rank d's counts flag word for
 *   this rank is set to epoch (st.release.sys) once the rows are visible.
 * rf_moe_ep_counts_collect: stream-ordered wait (bounded, 2 s) until
 *   flags[0..R) all equal epoch, then out [R][E] = table.  A source whose flag
 *   never arrives gets a zero row and sets RF_DEV_WAIT_TIMEOUT.
 * Callers alternate two tables (by step parity) so that a rank one step ahead
 * never writes the table a slower rank is reading.
 */
int rf_moe_ep_counts_push(const int32_t *counts, int32_t E, int32_t R, int32_t me, int32_t *const *dst,
                          int32_t *const *flag, int32_t epoch, rf_stream_t stream);
int rf_moe_ep_counts_collect(const int32_t *flags, const int32_t *table, int32_t R, int32_t E, int32_t epoch,
                             int32_t *out, rf_stream_t stream);

/*
 * The same exchange planned on the device (no host synchronisation per step).
 * rf_moe_ep_devplan runs the split of rf_moe_ep_plan on the GPU from the
 * all-gathered counts [R][E] (device) and the placement (slot_experts /
 * slot_offsets, device copies of the host arrays; S = this rank's slot count,
 * n_slots = all slots) into `workspace` (rf_moe_ep_devplan_workspace_size
 * bytes): small tables — send pieces, per-peer offsets, the receive table and
 * the slot-major GEMM segments.  recv_capacity / back_capacity are the rows of
 * every rank's receive / return buffer and rows_capacity those of this rank's
 * GEMM rows; a plan exceeding them is flagged (device error word) and moves
 * no rows (the buffer check is global, so every rank's plan fails with it).
 *   rf_moe_ep_devplan_push     dir 0: this rank's routed token rows (src = x,
 *                              src_slot from rf_moe_permute, div = K; both may
 *                              be NULL when this rank has no tokens) into the
 *                              experts' ranks' receive buffers; dir 1: the GEMM
 *                              output rows back into the tokens' ranks' return
 *                              buffers, each at its permuted row there (the
 *                              token rank's rf_moe_permute layout, align 1), so
 *                              rf_moe_combine reads the return buffer through
 *                              that permute's row_of_slot; then flags as
 *                              rf_moe_ep_push_rows.  For a dispatch that
 *                              overlaps the exchange with the GEMM of this
 *                              rank's own rows: dir 2 is dir 0 without the
 *                              rows this rank routes to itself (flags as
 *                              dir 0); dir 3 copies just those rows straight
 *                              into their slot-major GEMM rows (dst[me] = xl;
 *                              no flags, `flag`/`done` unused but non-NULL)
 *   rf_moe_ep_devplan_regroup  receive buffer -> slot-major GEMM rows
 *   rf_moe_ep_devplan_regroup_remote  the same for the rows of the other
 *                              sources only (after dir 2 + dir 3)
 *   rf_moe_ep_devplan_down_return  dir 1 fused into the down GEMM: the
 *                              tensor-core epilogue stores every row of
 *                              h[rows_capacity, I] . w2[j][H, I]^T straight
 *                              into its token rank's return buffer (same rows
 *                              as the GEMM + dir-1 push), then flags as
 *                              rf_moe_ep_push_rows; RF_ERR_UNSUPPORTED when the
 *                              tensor-core path does not take the dtype/shape
 * rf_moe_ep_devplan_layout: byte offsets inside the workspace of
 *   [0] int32 segment offsets [S+1], [1] int32 segment counts [S] (grouped
 *   GEMM arguments), [2] int32 overflow, [3] int64 recv_total, [4] int64 n_send,
 *   [5] workspace bytes, [6] int64 send_off [R+1], [7] int64 dst_row0 [R],
 *   [8] int64 recv_off [R+1], [9] int64 back_row0 [R], [10] int32 identity,
 *   [11] int64 rows used, [12] int64 cs [R][S+1] (rows from source s for the
 *   slots below j), [13] int64 cj [S][R+1] (rows of slot j from the sources
 *   below s), [14] int64 pstart [R][S] (source s's permuted row of its first
 *   row for slot j), [15] int64 piece_pos [n_pieces+1], [16] int64 piece_src
 *   [n_pieces] (send positions [piece_pos[k], piece_pos[k+1]) carry permuted
 *   rows from piece_src[k]), [17] int32 n_pieces, [18] int32 [S] offsets then
 *   [S] counts: this rank's own rows of each local slot (the grouped-GEMM
 *   groups of the dir-3 rows), [19] int32 [2S] offsets then [2S] counts: the
 *   other sources' rows of each slot, those below this rank then those above
 *   (groups 2j and 2j+1 use slot j's weights), [20] int32 piece_slot
 *   [n_pieces] (the destination rank's local slot of each send piece).  `out` holds
 *   RF_EP_DEVPLAN_LAYOUT_N entries.
 */
#define RF_EP_DEVPLAN_LAYOUT_N 21
size_t rf_moe_ep_devplan_workspace_size(int32_t R, int32_t E, int32_t S, int32_t n_slots);
int rf_moe_ep_devplan_layout(int32_t R, int32_t E, int32_t S, int32_t n_slots, int64_t *out);
int rf_moe_ep_devplan(const int32_t *counts, const int32_t *slot_experts, const int32_t *slot_offsets,
                      int32_t R, int32_t E, int32_t me, int32_t S, int32_t n_slots, int32_t align,
                      int32_t rounds, int64_t recv_capacity, int64_t back_capacity, int64_t rows_capacity,
                      void *workspace, size_t ws_bytes, rf_stream_t stream);
/* The planner of rf_moe_ep_devplan (the same source) run on the host over host
 * buffers, for checks on the CPU: *status gets the RF_DEV_* code the kernel
 * would have reported (0 = a valid plan). */
int rf_moe_ep_devplan_host(const int32_t *counts, const int32_t *slot_experts, const int32_t *slot_offsets,
                           int32_t R, int32_t E, int32_t me, int32_t S, int32_t n_slots, int32_t align,
                           int32_t rounds, int64_t recv_capacity, int64_t back_capacity, int64_t rows_capacity,
                           void *workspace, size_t ws_bytes, int32_t *status);
int rf_moe_ep_devplan_push(const void *workspace, int32_t R, int32_t E, int32_t S, int32_t n_slots,
                           int32_t dir, const void *src, const int32_t *src_slot, int64_t div,
                           int64_t row_bytes, void *const *dst, int32_t *const *flag, int32_t epoch,
                           uint32_t *done, rf_stream_t stream);
int rf_moe_ep_devplan_regroup(const void *workspace, int32_t R, int32_t E, int32_t S, int32_t n_slots,
                              const void *recv, void *xl, int64_t row_bytes, rf_stream_t stream);
int rf_moe_ep_devplan_regroup_remote(const void *workspace, int32_t R, int32_t E, int32_t S, int32_t n_slots,
                                     const void *recv, void *xl, int64_t row_bytes, rf_stream_t stream);
int rf_moe_ep_devplan_down_return(const void *workspace, int32_t R, int32_t E, int32_t S, int32_t n_slots,
                                  const void *h, const void *w2, int64_t rows_capacity, int64_t H, int64_t I,
                                  int32_t dtype, void *const *dst, int32_t *const *flag, int32_t epoch,
                                  uint32_t *done, rf_stream_t stream);

/*
 * Expert split, int8 half (fused.py:140-197 with slot (t, k) -> token t;
 * offload_cache.py:58-72 for the quantizer).  The listed experts (groups[n],
 * expert ids) own rows [offsets[e], offsets[e] + counts[e]) of the permuted
 * layout.
 *   rf_moe_int8_quantize  per listed expert: scale = max|src| / 127 over its
 *       rows (fp32; 1 when that max is <= 0), q = round-half-even(src / scale)
 *       clamped to +-127; scales[n] receive the scales.  compute_amax = 0
 *       takes amax[n] as given (the gated GEMM's max|inter|).
 *   rf_moe_int8_grouped_gemm  exact int32 sums of a[rows] . w[slot[e]]^T
 *       (w int8 [num_slots, gated ? 2N : N, Kdim], Kdim % 16 == 0), scaled by
 *       a_scales[i] * w_scales[e * w_scale_stride] in fp32.  gated: out[r, n] =
 *       act(g) * u in fp32 with g / u the first / second N rows' sums, and
 *       amax_out[i] = max|out| over the expert's rows.  down: out[r, n] =
 *       scaled sum * row_weights[src_slot[r]].
 *   rf_moe_split_combine  out[t] = round(float(sum over the token's resident
 *       experts of round(y_hit * round(w)), accumulated in the layer dtype) +
 *       sum over its int8 experts of y_int8 (fp32)), both in ascending expert
 *       order; is_miss[E] marks the int8 experts, ids [T*K] the slot experts.
 */
int rf_moe_int8_quantize(const void *src, int32_t src_dtype, const int32_t *offsets, const int32_t *counts,
                         const int32_t *groups, int32_t n_groups, int32_t E, int64_t rows_capacity, int64_t cols,
                         float *amax, int32_t compute_amax, float *scales, int8_t *q, rf_stream_t stream);
int rf_moe_int8_grouped_gemm(const int8_t *a, const int8_t *w, const int32_t *offsets, const int32_t *counts,
                             const int32_t *groups, const int32_t *slot, int32_t n_groups, int32_t E,
                             int32_t num_slots, int64_t rows_capacity, int64_t Kdim, int64_t N,
                             const float *a_scales, const float *w_scales, int64_t w_scale_stride, int32_t gated,
                             int32_t act, float *out, float *amax_out, const float *row_weights,
                             const int32_t *src_slot, rf_stream_t stream);
int rf_moe_split_combine(const void *y_hit, const float *y_int8, const int32_t *row_of_slot, const int32_t *ids,
                         const uint8_t *is_miss, const float *topk_weights, int64_t T, int32_t K, int64_t H,
                         int32_t E, int32_t dtype, void *out, rf_stream_t stream);

/* Summation modes of rf_moe_combine. */
#define RF_COMBINE_REFERENCE 0  /* the reference's rounding points and order */
#define RF_COMBINE_FP32 1       /* fp32 accumulation, one rounding */

/*
 * K5 — weighted combine:
 *   out[t] = sum_k topk_weights[t,k] * y[row_of_slot[t*K+k]]     (rows < 0 skipped)
 *          + (shared_y ? (shared_scale ? shared_scale[t] : 1) * shared_y[t] : 0)
 *          + (residual ? residual[t] : 0)
 *          + (accumulate ? out[t] : 0)
 * y [rows, H], shared_y/residual/out [T, H], all in `dtype`.
 * mode RF_COMBINE_REFERENCE rounds like the reference's fused_experts: the
 * weight is cast to `dtype`, every weighted row is rounded to `dtype`, and the
 * rows are accumulated in `dtype` in ascending expert order (ascending row of
 * the expert-major permuted layout); the shared and residual terms are added
 * with one rounding each.  RF_COMBINE_FP32 accumulates everything in fp32 and
 * rounds once.
 */
int rf_moe_combine(const void *y, const int32_t *row_of_slot, const float *topk_weights,
                   int64_t T, int64_t K, int64_t H, int dtype,
                   const void *shared_y, const float *shared_scale, const void *residual,
                   int accumulate, int mode, void *out, rf_stream_t stream);

/*
 * K5 with the decoder's next RMSNorm fused into its epilogue
 * (reframework/layers/norm.py:43-53, RMSNorm.forward_add_residual):
 *   residual_out[t] = combine(t) + residual[t]   (as rf_moe_combine, in `dtype`;
 *                                                  residual may be NULL)
 *   normed_out[t]   = r * (mean(r^2) + eps).sqrt().reciprocal() * norm_weight
 *                     (+ norm_bias)              with r = residual_out[t] in fp32,
 *                                                  each step rounded to fp32 as in
 *                                                  norm.py:27-35, stored in `dtype`
 * norm_weight / norm_bias: fp32 [H] (bias may be NULL).  The row mean is one
 * fixed-order block reduction per token.  The outputs must not alias.
 */
int rf_moe_combine_rmsnorm(const void *y, const int32_t *row_of_slot, const float *topk_weights,
                           int64_t T, int64_t K, int64_t H, int dtype,
                           const void *shared_y, const float *shared_scale, const void *residual,
                           int mode, const float *norm_weight, const float *norm_bias, float eps,
                           void *residual_out, void *normed_out, rf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RF_MOE_H */
