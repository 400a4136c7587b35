// Expert-parallel exchange planned on the device: no host synchronisation in
// the EP forward.
//
// rf_moe_ep_plan (ep_plan.cu) derives every rank's split from the global
// [R, E] counts on the host, which costs a device->host copy, host work and an
// upload each step.  The planner kernel below runs the same deterministic
// integer algorithm on the GPU from the all-gathered counts (one block: the
// water-filling and sorts are tiny and run in thread 0; the table loops are
// spread over the block) and writes small tables instead of per-row maps:
//   * send pieces: send positions [pos_k, pos_{k+1}) carry permuted rows
//     [src_k, ...) — the send order, grouped by destination rank;
//   * per-destination send bounds and the first row of this rank's chunk in
//     every destination's receive buffer; per-source receive bounds;
//   * the receive table c[s][j] (rows from source s for local slot j) with its
//     prefix sums, the aligned slot-major segments of the local GEMM rows, and
//     p[s][j], the source's permuted row of the first of those rows.
// The row kernels (push, regroup, return) locate each row with a binary
// search in those tables.  The return push writes every result row at its
// permuted (expert-major) row in the source's return buffer, so the combine
// reads the rows through the permute's own row_of_slot and sums each token's
// rows in ascending expert order, whichever rank computed them.  Bit-for-bit
// the same split as the host planner: tests compare the two.
#include <cstddef>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gemm.cuh"

RF_DEVICE_ERROR_WORD();

namespace {

constexpr int MAXR = 64;
constexpr int MAXS = 1024;   // slots (experts + replicas) one rank holds
constexpr int MAXP = 4096;   // send pieces of one rank

}  // namespace

// Fixed-size part of the device plan (tables sized by R and S follow it in
// the same buffer: cs_prefix [R][S+1], cj_prefix [S][R+1], pstart [R][S],
// int64 each).
struct RfEpDevPlan {
  int64_t send_off[MAXR + 1];   // this rank's rows for destination d: send positions [send_off[d], send_off[d+1])
  int64_t dst_row0[MAXR];       // ... landing at this row of d's receive buffer
  int64_t recv_off[MAXR + 1];   // rows from source s: receive rows [recv_off[s], recv_off[s+1])
  int64_t back_row0[MAXR];      // rows of s's earlier destinations (the host plan's return offset)
  int64_t piece_pos[MAXP + 1];  // send pieces (send order)
  int64_t piece_src[MAXP];
  int32_t piece_slot[MAXP];     // the destination rank's local slot of each piece
  int32_t loff32[MAXS + 1];     // int32 copies of loff / lcount for the grouped GEMMs
  int32_t lcount32[MAXS];
  int64_t loff[MAXS + 1];       // local slot segments (aligned) and their row counts
  int64_t lcount[MAXS];
  int64_t n_send, recv_total, rows_used;
  int32_t R, E, S, me, n_pieces, identity, overflow, pad_;
};

namespace {

__host__ __device__ void waterfill_dev(int64_t n, const int64_t *base, int m, int64_t *out, int *order, int64_t *loads,
                              int64_t *give) {
  for (int i = 0; i < m; ++i) order[i] = i;
  for (int i = 1; i < m; ++i) {  // stable insertion sort by base
    const int v = order[i];
    int j = i;
    while (j > 0 && base[order[j - 1]] > base[v]) {
      order[j] = order[j - 1];
      --j;
    }
    order[j] = v;
  }
  for (int i = 0; i < m; ++i) loads[i] = base[order[i]];
  int k = m;
  auto prefix = [&](int kk) {
    int64_t s = 0;
    for (int i = 0; i < kk; ++i) s += loads[i];
    return s;
  };
  while (k > 1 && n + prefix(k) <= loads[k - 1] * (int64_t)k) --k;
  const int64_t level = (n + prefix(k)) / k;
  int64_t used = 0;
  for (int i = 0; i < m; ++i) give[i] = 0;
  for (int i = 0; i < k; ++i) {
    give[i] = level - loads[i] > 0 ? level - loads[i] : 0;
    used += give[i];
  }
  int64_t rem = n - used;
  for (int i = 0; rem > 0; ++i, --rem) give[i % k] += 1;
  for (int pos = 0; pos < m; ++pos) out[order[pos]] = give[pos];
}

#ifdef __CUDA_ARCH__
// waterfill_dev on one warp, one lane per holder (m <= 32 holders): lane i
// passes base[i] and gets out[i].  The same integer steps, each lane working
// at its own sorted position: its stable rank r (ties keep lane order) and the
// sum of the sorted loads up to and including it, P(r + 1), come from one
// pass of shuffles; k = the largest k' in [2, m] with n + P(k') > loads[k'-1]
// * k' (else 1: where the scalar loop's descent from m stops), then the level
// and the remainder for the first sorted positions.
__device__ int64_t waterfill_warp(int64_t n, int64_t b, int m) {
  const unsigned full = 0xffffffffu;
  const int lane = (int)(threadIdx.x & 31);
  const bool act = lane < m;
  int rank = 0;
  int64_t upto = 0;  // P(rank + 1)
  for (int j = 0; j < m; ++j) {
    const int64_t bj = __shfl_sync(full, b, j);
    const bool before = (bj < b) || (bj == b && j < lane);
    rank += before;
    if (before || j == lane) upto += bj;
  }
  const bool stays = act && rank >= 1 && !(n + upto <= b * (int64_t)(rank + 1));
  const int k = max(1, (int)__reduce_max_sync(full, stays ? (unsigned)(rank + 1) : 0u));
  const unsigned at = __ballot_sync(full, act && rank == k - 1);  // the lane at sorted position k - 1
  const int64_t Pk = __shfl_sync(full, upto, __ffs(at) - 1);
  const int64_t level = (n + Pk) / k;
  int64_t give = 0;
  if (act && rank < k) give = level - b > 0 ? level - b : 0;
  int64_t used = give;
  for (int o = 16; o > 0; o >>= 1) used += __shfl_xor_sync(full, used, o);
  const int64_t rem = n - used;
  if (act && rank < k && rem > 0) give += rem / k + (rank < rem % k ? 1 : 0);
  return give;
}
#endif

struct PlanScratch {  // global scratch of the planner (E x R tables)
  int64_t *quota, *lo, *sbase, *total, *load;
  int32_t *repl;
};

}  // namespace

namespace {

struct PlannerArgs {
  const int32_t *counts;        // [R][E]
  const int32_t *slot_experts;  // [total slots]
  const int32_t *slot_offsets;  // [R+1]
  int R, E, me, S, n_slots, align, rounds;  // S: this rank's slot count as the host laid out the workspace
  int64_t recv_capacity, back_capacity;  // every rank's receive / return buffer rows
  int64_t rows_capacity;                 // this rank's slot-major GEMM rows
  RfEpDevPlan *plan;
  int64_t *cs_prefix;           // [R][S+1]
  int64_t *cj_prefix;           // [S][R+1]
  int64_t *pstart;              // [R][S]: permuted row in source s of its first row for slot j
  int64_t *cpre;                // [R][E+1]: rows of source s routed to experts below e
  // GEMM groups of the overlapped dispatch (int32): this rank's own rows of
  // each local slot, [S] offsets then [S] counts; the other sources' rows,
  // [2S] offsets then [2S] counts (rows before and after this rank's, per slot)
  int32_t *loc, *rem;
  PlanScratch sc;               // quota/lo/sbase [E*R], total [E], load [R], repl [E]
  int64_t *M;                   // [R][R]
  int32_t *hoff, *hlist;        // holders CSR: [E+1], [total slots]
  // the first thread's running sums of this rank's receive side (shared
  // memory when the planner runs there): per local slot the rows so far, the
  // rows from sources below this rank and up to it, and the segment starts
  // ([S], [S], [S], [S+1]); the tables above are only written from these
  int64_t *tail;
};

__host__ __device__ int64_t piece_dev(const PlannerArgs &a, int e, int src, int h, int64_t *offset) {
  const int R = a.R;
  const int64_t qlo = a.sc.lo[(int64_t)e * R + h], qhi = qlo + a.sc.quota[(int64_t)e * R + h];
  const int64_t slo = a.sc.sbase[(int64_t)e * R + src], shi = slo + a.counts[(int64_t)src * a.E + e];
  const int64_t lo = qlo > slo ? qlo : slo, hi = qhi < shi ? qhi : shi;
  if (offset) *offset = lo - slo;
  return hi - lo > 0 ? hi - lo : 0;
}

// A failed plan moves no row and gives the GEMMs empty segments.
__host__ __device__ void clear_plan(RfEpDevPlan *P, int S) {
  for (int j = 0; j <= S; ++j) {
    P->loff[j] = 0;
    P->loff32[j] = 0;
  }
  for (int j = 0; j < S; ++j) {
    P->lcount[j] = 0;
    P->lcount32[j] = 0;
  }
  P->n_send = P->recv_total = P->rows_used = 0;
  P->n_pieces = 0;
  P->overflow = 1;
}

// A failed plan also gives the overlapped dispatch's GEMM groups no rows.
__host__ __device__ void clear_groups(const PlannerArgs &a) {
  for (int j = 0; j < 2 * a.S; ++j) a.loc[j] = 0;
  for (int j = 0; j < 4 * a.S; ++j) a.rem[j] = 0;
}

// Runs the planner body: one block on the device (threads meet at barriers and
// share `bad` in shared memory), one thread on the host (the same code, for
// checks on the CPU; errors are recorded instead of setting the error word).
struct PlanExec {
  int *bad;
  int code = 0;
  __host__ __device__ int tid() const {
#ifdef __CUDA_ARCH__
    return (int)threadIdx.x;
#else
    return 0;
#endif
  }
  __host__ __device__ int nthreads() const {
#ifdef __CUDA_ARCH__
    return (int)blockDim.x;
#else
    return 1;
#endif
  }
  __host__ __device__ void sync() const {
#ifdef __CUDA_ARCH__
    __syncthreads();
#endif
  }
  __host__ __device__ void report(int c) {
#ifdef __CUDA_ARCH__
    rf_report(c);
#else
    if (!code) code = c;
#endif
  }
};

__host__ __device__ void planner_body(const PlannerArgs &a, PlanExec &x) {
  const int R = a.R, E = a.E, me = a.me;
  RfEpDevPlan *P = a.plan;
  int &s_bad = *x.bad;
  int64_t *quota = a.sc.quota, *lo = a.sc.lo, *sbase = a.sc.sbase, *total = a.sc.total, *load = a.sc.load;
  const int T0 = x.tid(), NT = x.nthreads();
  if (T0 == 0) {
    s_bad = 0;
    // the placement: offsets from 0 to n_slots, ascending, this rank's count as laid out
    if (a.slot_offsets[0] != 0 || a.slot_offsets[R] != a.n_slots) s_bad = 1;
    for (int r = 0; r < R; ++r)
      if (a.slot_offsets[r + 1] < a.slot_offsets[r]) s_bad = 1;
    if (!s_bad && a.slot_offsets[me + 1] - a.slot_offsets[me] != a.S) s_bad = 1;
  }
  x.sync();
  // per expert (one thread each): holder count, routed total, bad counts
  for (int s = T0; s < a.n_slots && !s_bad; s += NT)
    if (a.slot_experts[s] < 0 || a.slot_experts[s] >= E) s_bad = 1;
  for (int e = T0; e < E; e += NT) {
    int k = 0;
    for (int s = 0; s < a.n_slots && !s_bad; ++s) k += a.slot_experts[s] == e;
    a.hoff[e + 1] = k;
    int64_t t = 0;
    for (int r = 0; r < R; ++r) {
      const int32_t c = a.counts[(int64_t)r * E + e];
      if (c < 0) s_bad = 1;
      t += c;
    }
    total[e] = t;
  }
  x.sync();
  if (T0 == 0) {
    a.hoff[0] = 0;
    for (int e = 0; e < E; ++e) a.hoff[e + 1] += a.hoff[e];
  }
  x.sync();
  // holders of every expert, in rank order (CSR); no rank holds an expert
  // twice; every routed expert has a holder; the initial quotas
  for (int e = T0; e < E && !s_bad; e += NT) {
    int h = a.hoff[e];
    for (int r = 0; r < R; ++r)
      for (int s = a.slot_offsets[r]; s < a.slot_offsets[r + 1]; ++s)
        if (a.slot_experts[s] == e) a.hlist[h++] = r;
    const int h0 = a.hoff[e], k = a.hoff[e + 1] - h0;
    for (int i = h0 + 1; i < h0 + k; ++i)
      if (a.hlist[i] == a.hlist[i - 1]) s_bad = 1;
    if (k == 0 && total[e] != 0) s_bad = 1;
    for (int r = 0; r < R; ++r) quota[(int64_t)e * R + r] = 0;
    if (k == 1) quota[(int64_t)e * R + a.hlist[h0]] = total[e];
    for (int i = 0; k > 1 && i < k; ++i) quota[(int64_t)e * R + a.hlist[h0 + i]] = total[e] / k + (i < total[e] % k ? 1 : 0);
  }
  x.sync();
  for (int r = T0; r < R && !s_bad; r += NT) {
    int64_t l = 0;
    for (int e = 0; e < E; ++e) l += quota[(int64_t)e * R + r];
    load[r] = l;
  }
  x.sync();
#ifdef __CUDA_ARCH__
  if (T0 < 32 && !s_bad) {
    // the replicated experts, stable-sorted by total (descending), then the
    // water-filled split of each, in that order, for `rounds` passes: warp 0,
    // the first lane for the bookkeeping, one lane per holder for the split
    const unsigned full = 0xffffffffu;
    int nrep = 0;
    if (T0 == 0) {
      for (int e = 0; e < E; ++e)
        if (a.hoff[e + 1] - a.hoff[e] > 1) a.sc.repl[nrep++] = e;
      for (int i = 1; i < nrep; ++i) {
        const int v = a.sc.repl[i];
        int j = i;
        while (j > 0 && total[a.sc.repl[j - 1]] < total[v]) {
          a.sc.repl[j] = a.sc.repl[j - 1];
          --j;
        }
        a.sc.repl[j] = v;
      }
    }
    nrep = __shfl_sync(full, nrep, 0);
    __syncwarp();
    for (int it = 0; it < a.rounds; ++it) {
      int changed = 0, stop = 0;
      for (int ri = 0; ri < nrep; ++ri) {
        const int e = a.sc.repl[ri], h0 = a.hoff[e], k = a.hoff[e + 1] - h0;
        if (k > MAXR) {
          if (T0 == 0) s_bad = 1;
          stop = 1;
          break;
        }
        if (k <= 32) {
          const int h = T0 < k ? a.hlist[h0 + T0] : 0;
          const int64_t b = T0 < k ? load[h] - quota[(int64_t)e * R + h] : 0;
          const int64_t q_new = waterfill_warp(total[e], b, k);
          int ch = 0;
          if (T0 < k) {
            int64_t &q = quota[(int64_t)e * R + h];
            if (q != q_new) {
              load[h] += q_new - q;
              q = q_new;
              ch = 1;
            }
          }
          changed |= __any_sync(full, ch);
        } else {  // more than 32 holders: the scalar split on the first lane
          int ch = 0;
          if (T0 == 0) {
            int64_t base[MAXR], nq[MAXR], loads[MAXR], give[MAXR];
            int order[MAXR];
            for (int i = 0; i < k; ++i) base[i] = load[a.hlist[h0 + i]] - quota[(int64_t)e * R + a.hlist[h0 + i]];
            waterfill_dev(total[e], base, k, nq, order, loads, give);
            for (int i = 0; i < k; ++i) {
              int64_t &q = quota[(int64_t)e * R + a.hlist[h0 + i]];
              if (q != nq[i]) {
                load[a.hlist[h0 + i]] += nq[i] - q;
                q = nq[i];
                ch = 1;
              }
            }
          }
          changed |= __shfl_sync(full, ch, 0);
        }
        __syncwarp();  // this expert's quotas and loads, seen by every lane
      }
      if (stop || !changed) break;
    }
  }
#else
  if (T0 == 0 && !s_bad) {
    // the replicated experts, stable-sorted by total (descending), then the
    // water-filled split of each, in that order, for `rounds` passes
    int nrep = 0;
    for (int e = 0; e < E; ++e)
      if (a.hoff[e + 1] - a.hoff[e] > 1) a.sc.repl[nrep++] = e;
    for (int i = 1; i < nrep; ++i) {
      const int v = a.sc.repl[i];
      int j = i;
      while (j > 0 && total[a.sc.repl[j - 1]] < total[v]) {
        a.sc.repl[j] = a.sc.repl[j - 1];
        --j;
      }
      a.sc.repl[j] = v;
    }
    int64_t base[MAXR], nq[MAXR], loads[MAXR], give[MAXR];
    int order[MAXR];
    for (int it = 0; it < a.rounds && !s_bad; ++it) {
      bool changed = false;
      for (int ri = 0; ri < nrep; ++ri) {
        const int e = a.sc.repl[ri], h0 = a.hoff[e], k = a.hoff[e + 1] - h0;
        if (k > MAXR) {
          s_bad = 1;
          break;
        }
        for (int i = 0; i < k; ++i) base[i] = load[a.hlist[h0 + i]] - quota[(int64_t)e * R + a.hlist[h0 + i]];
        waterfill_dev(total[e], base, k, nq, order, loads, give);
        for (int i = 0; i < k; ++i) {
          int64_t &q = quota[(int64_t)e * R + a.hlist[h0 + i]];
          if (q != nq[i]) {
            load[a.hlist[h0 + i]] += nq[i] - q;
            q = nq[i];
            changed = true;
          }
        }
      }
      if (!changed) break;
    }
  }
#endif
  x.sync();
  // runs: holder h of expert e covers global rows [lo, lo + quota) (rank order)
  for (int e = T0; e < E && !s_bad; e += NT) {
    int64_t acc = 0, src = 0;
    for (int r = 0; r < R; ++r) {
      lo[(int64_t)e * R + r] = acc;
      acc += quota[(int64_t)e * R + r];
      sbase[(int64_t)e * R + r] = src;
      src += a.counts[(int64_t)r * E + e];
    }
  }
  x.sync();
  if (s_bad) {
    if (x.tid() == 0) {
      clear_plan(P, a.S);
      clear_groups(a);
      x.report(RF_DEV_BAD_EXPERT_ID);
    }
    return;
  }
  // the all-to-all matrix M[s][d], one (s, d) pair per thread, and every
  // source's expert-major row starts (its permuted layout, align 1)
  for (int t = x.tid(); t < R * R; t += x.nthreads()) {
    const int s = t / R, d = t % R;
    int64_t n = 0;
    for (int sl = a.slot_offsets[d]; sl < a.slot_offsets[d + 1]; ++sl) n += piece_dev(a, a.slot_experts[sl], s, d, nullptr);
    a.M[t] = n;
  }
  for (int s = x.tid(); s < R; s += x.nthreads()) {
    int64_t *c = a.cpre + (int64_t)s * (E + 1);
    c[0] = 0;
    for (int e = 0; e < E; ++e) c[e + 1] = c[e] + a.counts[(int64_t)s * E + e];
  }
  x.sync();
  // every rank's buffers (the same check on every rank: all plans fail together)
  if (x.tid() == 0) {
    for (int d = 0; d < R; ++d) {
      int64_t in = 0;
      for (int s = 0; s < R; ++s) in += a.M[(int64_t)s * R + d];
      if (in > a.recv_capacity || a.cpre[(int64_t)d * (E + 1) + E] > a.back_capacity) s_bad = 1;
    }
  }
  x.sync();
  if (s_bad) {
    if (x.tid() == 0) {
      clear_plan(P, a.S);
      clear_groups(a);
      x.report(RF_DEV_PLAN_OVERFLOW);
    }
    return;
  }
  if (x.tid() != 0) return;
  // ---- this rank's tables
  int bad = 0;
  P->R = R;
  P->E = E;
  P->me = me;
  const int s0 = a.slot_offsets[me], S = a.slot_offsets[me + 1] - s0;
  if (S > MAXS || R > MAXR) bad = 1;
  P->S = S;
  // send side: pieces in destination order, each destination's slots in order
  int64_t pos = 0;
  int np = 0, identity = 1;
  P->send_off[0] = 0;
  for (int d = 0; d < R && !bad; ++d) {
    for (int sl = a.slot_offsets[d]; sl < a.slot_offsets[d + 1]; ++sl) {
      const int e = a.slot_experts[sl];
      int64_t off = 0;
      const int64_t ln = piece_dev(a, e, me, d, &off);
      if (ln > 0) {
        if (np >= MAXP) {
          bad = 1;
          break;
        }
        const int64_t start = a.cpre[(int64_t)me * (E + 1) + e] + off;  // its first permuted row
        if (start != pos) identity = 0;
        P->piece_pos[np] = pos;
        P->piece_src[np] = start;
        P->piece_slot[np] = sl - a.slot_offsets[d];
        ++np;
        pos += ln;
      }
    }
    P->send_off[d + 1] = pos;
  }
  P->piece_pos[np] = pos;
  P->n_pieces = np;
  P->identity = identity;
  P->n_send = pos;
  // offsets inside the peers' buffers
  for (int d = 0; d < R; ++d) {
    int64_t below = 0, back = 0;
    for (int s = 0; s < me; ++s) below += a.M[(int64_t)s * R + d];  // earlier sources' rows to d
    P->dst_row0[d] = below;
    for (int dd = 0; dd < me; ++dd) back += a.M[(int64_t)d * R + dd];  // d's rows to lower ranks
    P->back_row0[d] = back;
  }
  // receive side: c[s][j], source bounds, slot segments and both prefix tables
  // (running values kept in the scratch `tail`, never read back from the plan)
  int64_t *lc = a.tail, *cjm = a.tail + S, *cjm1 = a.tail + 2 * S, *lof = a.tail + 3 * S;
  P->recv_off[0] = 0;
  for (int j = 0; j < S; ++j) lc[j] = cjm[j] = cjm1[j] = 0;
  int64_t roff = 0;
  for (int s = 0; s < R && !bad; ++s) {
    int64_t run = 0;
    for (int j = 0; j < S; ++j) {
      a.cs_prefix[(int64_t)s * (S + 1) + j] = run;
      const int e = a.slot_experts[s0 + j];
      int64_t off = 0;
      const int64_t c = piece_dev(a, e, s, me, &off);
      a.pstart[(int64_t)s * S + j] = c > 0 ? a.cpre[(int64_t)s * (E + 1) + e] + off : 0;
      a.cj_prefix[(int64_t)j * (R + 1) + s] = lc[j];
      if (s == me) cjm[j] = lc[j];
      if (s == me + 1) cjm1[j] = lc[j];
      lc[j] += c;
      run += c;
    }
    a.cs_prefix[(int64_t)s * (S + 1) + S] = run;
    roff += run;
    P->recv_off[s + 1] = roff;
  }
  for (int j = 0; j < S; ++j) {
    a.cj_prefix[(int64_t)j * (R + 1) + R] = lc[j];
    if (me + 1 == R) cjm1[j] = lc[j];
  }
  int64_t rows = 0;
  lof[0] = 0;
  for (int j = 0; j < S; ++j) {
    rows += (lc[j] + a.align - 1) / a.align * a.align;
    lof[j + 1] = rows;
  }
  for (int j = 0; j <= S; ++j) {
    P->loff[j] = lof[j];
    P->loff32[j] = (int32_t)lof[j];
  }
  for (int j = 0; j < S; ++j) {
    P->lcount[j] = lc[j];
    P->lcount32[j] = (int32_t)lc[j];
  }
  P->recv_total = roff;
  P->rows_used = rows;
  if (roff > a.recv_capacity || rows > a.rows_capacity) bad = 1;
  P->overflow = bad;
  if (bad) {
    clear_plan(P, S);
    clear_groups(a);
    x.report(RF_DEV_PLAN_OVERFLOW);
  } else {
    for (int j = 0; j < S; ++j) {
      a.loc[j] = (int32_t)(lof[j] + cjm[j]);
      a.loc[S + j] = (int32_t)(cjm1[j] - cjm[j]);
      a.rem[2 * j] = (int32_t)lof[j];
      a.rem[2 * j + 1] = (int32_t)(lof[j] + cjm1[j]);
      a.rem[2 * S + 2 * j] = (int32_t)cjm[j];
      a.rem[2 * S + 2 * j + 1] = (int32_t)(lc[j] - cjm1[j]);
    }
  }
}

__global__ void __launch_bounds__(256) ep_planner_kernel(const PlannerArgs a) {
  __shared__ int s_bad;
  PlanExec x{&s_bad};
  planner_body(a, x);
}

// Shared-memory layout of the planner's inputs and scratch (the planner is
// one block whose first thread walks these tables sequentially: from shared
// memory each access costs a few cycles instead of a global round trip).
struct SmemPlan {
  size_t counts, sexp, soff, hoff, hlist, quota, lo, sbase, total, load, repl, M, cpre, tail, bytes;
};
__host__ __device__ inline SmemPlan smem_plan_layout(int R, int E, int n_slots) {
  SmemPlan L;
  size_t o = 0;
  auto take = [&](size_t n) {
    const size_t at = o;
    o = (o + n + 15) / 16 * 16;
    return at;
  };
  L.quota = take((size_t)E * R * 8);
  L.lo = take((size_t)E * R * 8);
  L.sbase = take((size_t)E * R * 8);
  L.total = take((size_t)E * 8);
  L.load = take((size_t)R * 8);
  L.M = take((size_t)R * R * 8);
  L.cpre = take((size_t)R * (E + 1) * 8);
  L.tail = take((size_t)(4 * (n_slots > 0 ? n_slots : 1) + 1) * 8);
  L.counts = take((size_t)R * E * 4);
  L.sexp = take((size_t)(n_slots > 0 ? n_slots : 1) * 4);
  L.soff = take((size_t)(R + 1) * 4);
  L.hoff = take((size_t)(E + 1) * 4);
  L.hlist = take((size_t)(n_slots > 0 ? n_slots : 1) * 4);
  L.repl = take((size_t)E * 4);
  L.bytes = o;
  return L;
}
constexpr size_t PLAN_SMEM_MAX = 200 * 1024;

// The planner with its inputs copied to, and its scratch in, shared memory
// (when they fit in PLAN_SMEM_MAX); the outputs other kernels read (the plan,
// the prefix tables, the GEMM groups) stay in the workspace.
__global__ void __launch_bounds__(256) ep_planner_smem_kernel(const PlannerArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ int s_bad;
  const SmemPlan L = smem_plan_layout(a.R, a.E, a.n_slots);
  PlannerArgs b = a;
  int32_t *counts = reinterpret_cast<int32_t *>(sm + L.counts);
  int32_t *sexp = reinterpret_cast<int32_t *>(sm + L.sexp);
  int32_t *soff = reinterpret_cast<int32_t *>(sm + L.soff);
  for (int i = threadIdx.x; i < a.R * a.E; i += blockDim.x) counts[i] = a.counts[i];
  for (int i = threadIdx.x; i < a.n_slots; i += blockDim.x) sexp[i] = a.slot_experts[i];
  for (int i = threadIdx.x; i <= a.R; i += blockDim.x) soff[i] = a.slot_offsets[i];
  __syncthreads();
  b.counts = counts;
  b.slot_experts = sexp;
  b.slot_offsets = soff;
  b.hoff = reinterpret_cast<int32_t *>(sm + L.hoff);
  b.hlist = reinterpret_cast<int32_t *>(sm + L.hlist);
  b.sc.quota = reinterpret_cast<int64_t *>(sm + L.quota);
  b.sc.lo = reinterpret_cast<int64_t *>(sm + L.lo);
  b.sc.sbase = reinterpret_cast<int64_t *>(sm + L.sbase);
  b.sc.total = reinterpret_cast<int64_t *>(sm + L.total);
  b.sc.load = reinterpret_cast<int64_t *>(sm + L.load);
  b.sc.repl = reinterpret_cast<int32_t *>(sm + L.repl);
  b.M = reinterpret_cast<int64_t *>(sm + L.M);
  b.cpre = reinterpret_cast<int64_t *>(sm + L.cpre);
  b.tail = reinterpret_cast<int64_t *>(sm + L.tail);
  PlanExec x{&s_bad};
  planner_body(b, x);
}

}  // namespace

namespace {

// One 16-byte-aligned workspace per EP layer: the plan, its two prefix tables
// and the planner's scratch.
struct Layout {
  size_t plan, cs, cj, ps, cpre, quota, lo, sbase, total, load, repl, M, hoff, hlist, loc, rem, tail, bytes;
};

size_t up16(size_t v) { return (v + 15) / 16 * 16; }

Layout layout_of(int64_t R, int64_t E, int64_t S, int64_t nslots) {
  Layout L;
  size_t o = 0;
  L.plan = o; o = up16(o + sizeof(RfEpDevPlan));
  L.cs = o; o = up16(o + (size_t)R * (S + 1) * 8);
  L.cj = o; o = up16(o + (size_t)S * (R + 1) * 8);
  L.ps = o; o = up16(o + (size_t)R * (S > 0 ? S : 1) * 8);
  L.cpre = o; o = up16(o + (size_t)R * (E + 1) * 8);
  L.quota = o; o = up16(o + (size_t)E * R * 8);
  L.lo = o; o = up16(o + (size_t)E * R * 8);
  L.sbase = o; o = up16(o + (size_t)E * R * 8);
  L.total = o; o = up16(o + (size_t)E * 8);
  L.load = o; o = up16(o + (size_t)R * 8);
  L.repl = o; o = up16(o + (size_t)E * 4);
  L.M = o; o = up16(o + (size_t)R * R * 8);
  L.hoff = o; o = up16(o + (size_t)(E + 1) * 4);
  L.hlist = o; o = up16(o + (size_t)(nslots > 0 ? nslots : 1) * 4);
  L.loc = o; o = up16(o + (size_t)2 * (S > 0 ? S : 1) * 4);
  L.rem = o; o = up16(o + (size_t)4 * (S > 0 ? S : 1) * 4);
  L.tail = o; o = up16(o + (size_t)(4 * S + 1) * 8);
  L.bytes = o;
  return L;
}

// largest k in [0, n) with a[k] <= v (a ascending, a[0] <= v)
__device__ __forceinline__ int find_le(const int64_t *a, int n, int64_t v) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void copy_row(uint4 *t, const uint4 *s, int64_t vecs, int lane) {
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

__device__ __forceinline__ void st_release_sys_dp(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct PlanPushArgs {
  const RfEpDevPlan *plan;
  const int64_t *cs, *cj, *ps;  // prefix tables and permuted row starts of the plan
  const uint8_t *src;
  const int32_t *src_slot;      // dispatch: permuted row -> pair index (t*K+k)
  int64_t div, row_bytes;
  int R, S, ret;                // ret (mode): 0 dispatch, 1 return, 2 dispatch to the other ranks only,
                                // 3 this rank's own dispatch rows straight into its GEMM rows (dst[me])
  int32_t epoch;
  uint32_t *done;
  uint8_t *dst[MAXR];
  int32_t *flag[MAXR];
};

// Dispatch (ret = 0): send positions i -> token rows, into the destinations'
// receive buffers.  Return (ret = 1): receive rows q -> their local GEMM rows
// of `src` (= y), into the sources' return buffers at the source's permuted
// row of each.  Either way the last block
// raises this rank's flag in every peer, also when the plan overflowed (then
// no row is written and the device error word is already set).
__global__ void __launch_bounds__(256) plan_push_kernel(const __grid_constant__ PlanPushArgs a) {
  const RfEpDevPlan *P = a.plan;
  const int lane = threadIdx.x & 31;
  const int R = a.R, S = a.S;
  const int64_t vecs = a.row_bytes / 16;
  const int mode = a.ret, ok = !P->overflow, me = ok ? P->me : 0;  // a failed plan leaves `me` unset
  // send positions of this rank's own rows: mode 2 skips them, mode 3 moves only them
  const int64_t own0 = ok ? P->send_off[me] : 0, own = ok ? P->send_off[me + 1] - own0 : 0;
  const int64_t n = !ok ? 0 : mode == 1 ? P->recv_total : mode == 2 ? P->n_send - own : mode == 3 ? own : P->n_send;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  // copies to other ranks interleave all destinations (see rf::scatter_pos)
  const int64_t stride = mode == 3 || n == 0 ? 1 : rf::scatter_stride(n);
  const int64_t offset = n == 0 ? 0 : (int64_t)me * (n / (R > 0 ? R : 1));
  for (int64_t t0 = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); t0 < n; t0 += nwarps) {
    const int64_t t = mode == 3 ? t0 : rf::scatter_pos(t0, n, stride, offset);
    const int64_t i = mode == 3 ? own0 + t : (mode == 2 && t >= own0) ? t + own : t;
    int64_t srow, drow;
    int d;
    if (mode != 1) {
      const int k = find_le(P->piece_pos, P->n_pieces, i);
      const int64_t j = P->piece_src[k] + (i - P->piece_pos[k]);
      srow = (int64_t)a.src_slot[j] / a.div;
      if (mode == 3) {  // own rows: the slot's segment, after the rows of the lower-ranked sources
        const int js = P->piece_slot[k];
        d = me;
        drow = P->loff[js] + a.cj[(int64_t)js * (R + 1) + me] + (i - P->piece_pos[k]);
      } else {
        d = find_le(P->send_off, R, i);
        drow = P->dst_row0[d] + (i - P->send_off[d]);
      }
    } else {
      d = find_le(P->recv_off, R, i);
      const int64_t q2 = i - P->recv_off[d];
      const int64_t *cs = a.cs + (int64_t)d * (S + 1);
      const int j = find_le(cs, S, q2);
      srow = P->loff[j] + a.cj[(int64_t)j * (R + 1) + d] + (q2 - cs[j]);
      drow = a.ps[(int64_t)d * S + j] + (q2 - cs[j]);
    }
    copy_row(reinterpret_cast<uint4 *>(a.dst[d] + drow * a.row_bytes),
             reinterpret_cast<const uint4 *>(a.src + srow * a.row_bytes), vecs, lane);
  }
  if (mode == 3) return;  // a local copy: no flags
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < R; ++d) st_release_sys_dp(a.flag[d], a.epoch);
      *a.done = 0u;
    }
  }
}

// Local GEMM rows (slot-major, aligned segments) from the receive buffer;
// pad rows are left untouched (their GEMM outputs are never stored).
__global__ void __launch_bounds__(256) plan_regroup_kernel(const RfEpDevPlan *P, const int64_t *cs_all,
                                                           const int64_t *cj_all, const uint8_t *recv, uint8_t *xl,
                                                           int64_t row_bytes, int R, int S, int skip_me) {
  const int lane = threadIdx.x & 31;
  const int64_t vecs = row_bytes / 16;
  const int64_t n = P->overflow ? 0 : P->rows_used;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < n; r += nwarps) {
    const int j = find_le(P->loff, S, r);
    const int64_t k = r - P->loff[j];
    if (k >= P->lcount[j]) continue;
    const int64_t *cj = cj_all + (int64_t)j * (R + 1);
    const int s = find_le(cj, R, k);
    if (skip_me && s == P->me) continue;  // placed by the own-rows push
    const int64_t q = P->recv_off[s] + cs_all[(int64_t)s * (S + 1) + j] + (k - cj[s]);
    copy_row(reinterpret_cast<uint4 *>(xl + r * row_bytes), reinterpret_cast<const uint4 *>(recv + q * row_bytes),
             vecs, lane);
  }
}

}  // namespace

extern "C" size_t rf_moe_ep_devplan_workspace_size(int32_t R, int32_t E, int32_t S, int32_t n_slots) {
  if (R < 1 || E < 1 || S < 0 || n_slots < 0) return 0;
  return layout_of(R, E, S, n_slots).bytes;
}

extern "C" int rf_moe_ep_devplan_layout(int32_t R, int32_t E, int32_t S, int32_t n_slots, int64_t *out) {
  RF_CHECK_ARG(out && R >= 1 && E >= 1 && S >= 0 && n_slots >= 0, "rf_moe_ep_devplan_layout: bad arguments");
  const Layout L = layout_of(R, E, S, n_slots);
  out[0] = (int64_t)(L.plan + offsetof(RfEpDevPlan, loff32));    // int32 [S+1] GEMM segment offsets
  out[1] = (int64_t)(L.plan + offsetof(RfEpDevPlan, lcount32));  // int32 [S]   GEMM segment counts
  out[2] = (int64_t)(L.plan + offsetof(RfEpDevPlan, overflow));  // int32       overflow flag
  out[3] = (int64_t)(L.plan + offsetof(RfEpDevPlan, recv_total));
  out[4] = (int64_t)(L.plan + offsetof(RfEpDevPlan, n_send));
  out[5] = (int64_t)L.bytes;
  out[6] = (int64_t)(L.plan + offsetof(RfEpDevPlan, send_off));   // int64 [R+1]
  out[7] = (int64_t)(L.plan + offsetof(RfEpDevPlan, dst_row0));   // int64 [R]
  out[8] = (int64_t)(L.plan + offsetof(RfEpDevPlan, recv_off));   // int64 [R+1]
  out[9] = (int64_t)(L.plan + offsetof(RfEpDevPlan, back_row0));  // int64 [R]
  out[10] = (int64_t)(L.plan + offsetof(RfEpDevPlan, identity));  // int32
  out[11] = (int64_t)(L.plan + offsetof(RfEpDevPlan, rows_used)); // int64
  out[12] = (int64_t)L.cs;                                         // int64 [R][S+1] receive prefix per source
  out[13] = (int64_t)L.cj;                                         // int64 [S][R+1] receive prefix per slot
  out[14] = (int64_t)L.ps;                                         // int64 [R][S]   permuted row starts
  out[15] = (int64_t)(L.plan + offsetof(RfEpDevPlan, piece_pos));  // int64 [n_pieces+1] send pieces
  out[16] = (int64_t)(L.plan + offsetof(RfEpDevPlan, piece_src));  // int64 [n_pieces]
  out[17] = (int64_t)(L.plan + offsetof(RfEpDevPlan, n_pieces));   // int32
  out[18] = (int64_t)L.loc;  // int32 [S] offsets, [S] counts: this rank's own rows per local slot
  out[19] = (int64_t)L.rem;  // int32 [2S] offsets, [2S] counts: the other sources' rows per local slot
  out[20] = (int64_t)(L.plan + offsetof(RfEpDevPlan, piece_slot));  // int32 [n_pieces]
  return RF_OK;
}

namespace {

// Checks the sizes and lays the planner's arguments out in `workspace`.
int planner_args(PlannerArgs &a, const int32_t *counts, const int32_t *slot_experts, const int32_t *slot_offsets,
                 int32_t R, int32_t E, int32_t me, int32_t S, int32_t n_slots, int32_t align, int32_t rounds,
                 int64_t recv_capacity, int64_t back_capacity, int64_t rows_capacity, void *workspace,
                 size_t ws_bytes, const char *name) {
  const std::string nm(name);
  RF_CHECK_ARG(counts && slot_experts && slot_offsets && workspace, nm + ": null pointer");
  RF_CHECK_ARG(R >= 1 && R <= MAXR && E >= 1 && me >= 0 && me < R && S >= 0 && S <= MAXS && n_slots >= S &&
                   align >= 1 && rounds >= 0,
               nm + ": bad sizes (R <= 64, slots per rank <= 1024)");
  const Layout L = layout_of(R, E, S, n_slots);
  RF_CHECK_ARG(ws_bytes >= L.bytes && (uintptr_t)workspace % 16 == 0, nm + ": workspace too small");
  uint8_t *w = reinterpret_cast<uint8_t *>(workspace);
  a.counts = counts;
  a.slot_experts = slot_experts;
  a.slot_offsets = slot_offsets;
  a.R = R;
  a.E = E;
  a.me = me;
  a.S = S;
  a.n_slots = n_slots;
  a.align = align;
  a.rounds = rounds;
  a.recv_capacity = recv_capacity;
  a.back_capacity = back_capacity;
  a.rows_capacity = rows_capacity;
  a.plan = reinterpret_cast<RfEpDevPlan *>(w + L.plan);
  a.cs_prefix = reinterpret_cast<int64_t *>(w + L.cs);
  a.cj_prefix = reinterpret_cast<int64_t *>(w + L.cj);
  a.pstart = reinterpret_cast<int64_t *>(w + L.ps);
  a.cpre = reinterpret_cast<int64_t *>(w + L.cpre);
  a.sc.quota = reinterpret_cast<int64_t *>(w + L.quota);
  a.sc.lo = reinterpret_cast<int64_t *>(w + L.lo);
  a.sc.sbase = reinterpret_cast<int64_t *>(w + L.sbase);
  a.sc.total = reinterpret_cast<int64_t *>(w + L.total);
  a.sc.load = reinterpret_cast<int64_t *>(w + L.load);
  a.sc.repl = reinterpret_cast<int32_t *>(w + L.repl);
  a.M = reinterpret_cast<int64_t *>(w + L.M);
  a.hoff = reinterpret_cast<int32_t *>(w + L.hoff);
  a.hlist = reinterpret_cast<int32_t *>(w + L.hlist);
  a.loc = reinterpret_cast<int32_t *>(w + L.loc);
  a.rem = reinterpret_cast<int32_t *>(w + L.rem);
  a.tail = reinterpret_cast<int64_t *>(w + L.tail);
  return RF_OK;
}

}  // namespace

extern "C" int rf_moe_ep_devplan(const int32_t *counts, const int32_t *slot_experts, const int32_t *slot_offsets,
                                 int32_t R, int32_t E, int32_t me, int32_t S, int32_t n_slots, int32_t align,
                                 int32_t rounds, int64_t recv_capacity, int64_t back_capacity, int64_t rows_capacity,
                                 void *workspace, size_t ws_bytes, rf_stream_t stream) {
  PlannerArgs a;
  const int rc = planner_args(a, counts, slot_experts, slot_offsets, R, E, me, S, n_slots, align, rounds,
                              recv_capacity, back_capacity, rows_capacity, workspace, ws_bytes, "rf_moe_ep_devplan");
  if (rc != RF_OK) return rc;
  const size_t smem = smem_plan_layout(R, E, n_slots).bytes;
  if (smem <= PLAN_SMEM_MAX) {
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
      attr = cudaFuncSetAttribute(ep_planner_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)PLAN_SMEM_MAX);
    });
    if (attr != cudaSuccess) return rf::fail(RF_ERR_CUDA, std::string("rf_moe_ep_devplan: ") + cudaGetErrorString(attr));
    ep_planner_smem_kernel<<<1, 256, smem, (cudaStream_t)stream>>>(a);
  } else {
    ep_planner_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(a);
  }
  return rf::check_launch("rf_moe_ep_devplan");
}

extern "C" int rf_moe_ep_devplan_host(const int32_t *counts, const int32_t *slot_experts,
                                      const int32_t *slot_offsets, int32_t R, int32_t E, int32_t me, int32_t S,
                                      int32_t n_slots, int32_t align, int32_t rounds, int64_t recv_capacity,
                                      int64_t back_capacity, int64_t rows_capacity, void *workspace, size_t ws_bytes,
                                      int32_t *status) {
  RF_CHECK_ARG(status, "rf_moe_ep_devplan_host: null status");
  PlannerArgs a;
  const int rc = planner_args(a, counts, slot_experts, slot_offsets, R, E, me, S, n_slots, align, rounds,
                              recv_capacity, back_capacity, rows_capacity, workspace, ws_bytes,
                              "rf_moe_ep_devplan_host");
  if (rc != RF_OK) return rc;
  int bad = 0;
  PlanExec x{&bad};
  planner_body(a, x);
  *status = x.code;
  return RF_OK;
}

// dir 0: dispatch (src = token rows x, src_slot/div map send positions to them);
// dir 1: return (src = the local GEMM output rows); dir 2: dispatch to the other
// ranks only; dir 3: this rank's own dispatch rows into its slot-major GEMM rows
// dst[me] (a local copy, no flags).
extern "C" int rf_moe_ep_devplan_push(const void *workspace, int32_t R, int32_t E, int32_t S, int32_t n_slots,
                                      int32_t dir, const void *src, const int32_t *src_slot, int64_t div,
                                      int64_t row_bytes, void *const *dst, int32_t *const *flag, int32_t epoch,
                                      uint32_t *done, rf_stream_t stream) {
  RF_CHECK_ARG(workspace && dst && flag && done && dir >= 0 && dir <= 3, "rf_moe_ep_devplan_push: bad arguments");
  RF_CHECK_ARG(R >= 1 && R <= MAXR && row_bytes > 0 && row_bytes % 16 == 0 && div >= 1,
               "rf_moe_ep_devplan_push: bad sizes");
  RF_CHECK_ARG((uintptr_t)src % 16 == 0, "rf_moe_ep_devplan_push: source must be 16-byte aligned");
  const Layout L = layout_of(R, E, S, n_slots);
  const uint8_t *w = reinterpret_cast<const uint8_t *>(workspace);
  PlanPushArgs a;
  a.plan = reinterpret_cast<const RfEpDevPlan *>(w + L.plan);
  a.cs = reinterpret_cast<const int64_t *>(w + L.cs);
  a.cj = reinterpret_cast<const int64_t *>(w + L.cj);
  a.ps = reinterpret_cast<const int64_t *>(w + L.ps);
  a.src = reinterpret_cast<const uint8_t *>(src);
  a.src_slot = src_slot;
  a.div = div;
  a.row_bytes = row_bytes;
  a.R = R;
  a.S = S;
  a.ret = dir;
  a.epoch = epoch;
  a.done = done;
  for (int d = 0; d < R; ++d) {
    RF_CHECK_ARG(flag[d], "rf_moe_ep_devplan_push: missing flag");
    a.dst[d] = reinterpret_cast<uint8_t *>(dst[d]);
    a.flag[d] = flag[d];
  }
  plan_push_kernel<<<rf::num_sms() * 4, 256, 0, (cudaStream_t)stream>>>(a);
  return rf::check_launch("rf_moe_ep_devplan_push");
}

extern "C" int rf_moe_ep_devplan_regroup(const void *workspace, int32_t R, int32_t E, int32_t S, int32_t n_slots,
                                         const void *recv, void *xl, int64_t row_bytes, rf_stream_t stream) {
  RF_CHECK_ARG(workspace && recv && xl && R >= 1 && R <= MAXR && row_bytes % 16 == 0,
               "rf_moe_ep_devplan_regroup: bad arguments");
  const Layout L = layout_of(R, E, S, n_slots);
  const uint8_t *w = reinterpret_cast<const uint8_t *>(workspace);
  if (S == 0) return RF_OK;
  plan_regroup_kernel<<<rf::num_sms() * 4, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const RfEpDevPlan *>(w + L.plan), reinterpret_cast<const int64_t *>(w + L.cs),
      reinterpret_cast<const int64_t *>(w + L.cj), reinterpret_cast<const uint8_t *>(recv),
      reinterpret_cast<uint8_t *>(xl), row_bytes, R, S, 0);
  return rf::check_launch("rf_moe_ep_devplan_regroup");
}

extern "C" int rf_moe_ep_devplan_regroup_remote(const void *workspace, int32_t R, int32_t E, int32_t S,
                                                int32_t n_slots, const void *recv, void *xl, int64_t row_bytes,
                                                rf_stream_t stream) {
  RF_CHECK_ARG(workspace && recv && xl && R >= 1 && R <= MAXR && row_bytes % 16 == 0,
               "rf_moe_ep_devplan_regroup_remote: bad arguments");
  const Layout L = layout_of(R, E, S, n_slots);
  const uint8_t *w = reinterpret_cast<const uint8_t *>(workspace);
  if (S == 0) return RF_OK;
  plan_regroup_kernel<<<rf::num_sms() * 4, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const RfEpDevPlan *>(w + L.plan), reinterpret_cast<const int64_t *>(w + L.cs),
      reinterpret_cast<const int64_t *>(w + L.cj), reinterpret_cast<const uint8_t *>(recv),
      reinterpret_cast<uint8_t *>(xl), row_bytes, R, S, 1);
  return rf::check_launch("rf_moe_ep_devplan_regroup_remote");
}

// dir 1 fused into the down GEMM: y = h . w2[j]^T per local slot, each row
// stored by the GEMM epilogue into its token rank's return buffer.
extern "C" int rf_moe_ep_devplan_down_return(const void *workspace, int32_t R, int32_t E, int32_t S,
                                             int32_t n_slots, const void *h, const void *w2, int64_t rows_capacity,
                                             int64_t H, int64_t I, int32_t dtype, void *const *dst,
                                             int32_t *const *flag, int32_t epoch, uint32_t *done,
                                             rf_stream_t stream) {
  RF_CHECK_ARG(workspace && h && w2 && dst && flag && done, "rf_moe_ep_devplan_down_return: null pointer");
  RF_CHECK_ARG(R >= 1 && R <= MAXR && R <= rf::REMOTE_MAX_RANKS && S >= 1 && S <= MAXS && E >= 1 && H >= 1 &&
                   I >= 1 && rows_capacity >= 1 && rows_capacity < ((int64_t)1 << 31) && H < (1 << 30) &&
                   I < (1 << 30),
               "rf_moe_ep_devplan_down_return: bad sizes");
  RF_CHECK_ARG(rf::valid_dtype(dtype), "rf_moe_ep_devplan_down_return: unknown dtype");
  const Layout L = layout_of(R, E, S, n_slots);
  const uint8_t *w = reinterpret_cast<const uint8_t *>(workspace);
  const RfEpDevPlan *P = reinterpret_cast<const RfEpDevPlan *>(w + L.plan);
  rf::RemoteOut ro;
  ro.cj = reinterpret_cast<const int64_t *>(w + L.cj);
  ro.ps = reinterpret_cast<const int64_t *>(w + L.ps);
  ro.R = R;
  ro.S = S;
  ro.epoch = epoch;
  ro.done = done;
  for (int d = 0; d < R; ++d) {
    RF_CHECK_ARG(dst[d] && flag[d] && (uintptr_t)dst[d] % 16 == 0,
                 "rf_moe_ep_devplan_down_return: missing or unaligned peer buffer");
    ro.dst[d] = dst[d];
    ro.flag[d] = flag[d];
  }
  rf::GroupedGemmArgs g;
  g.a = h;
  g.w = w2;
  g.out = dst[0];  // rows go through ro; kept for the operand checks
  g.offsets = P->loff32;
  g.counts = P->lcount32;
  g.slot = nullptr;
  g.groups = nullptr;
  g.n_groups = S;
  g.E = S;
  g.num_slots = S;
  g.rows_capacity = rows_capacity;
  g.Kdim = (int)I;
  g.N = (int)H;
  g.dtype = dtype;
  g.act = 0;
  g.remote = &ro;
  const int rc = rf::tc_down_remote(g, (cudaStream_t)stream);
  if (rc < 0)
    return rf::fail(RF_ERR_UNSUPPORTED,
                    "rf_moe_ep_devplan_down_return: needs the tensor-core path (bf16/fp16, sizes multiple of 8)");
  return rc;
}
