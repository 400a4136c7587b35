// Host-side expert-parallel exchange planner (native; no GPU work).
//
// Given the global [R, E] routed-row counts of one step and the experts each
// rank holds (its contiguous shard of reframework/parallel/ep.py:45-55 plus
// any replica slots), computes for one rank:
//   * the per-holder row split of replicated experts (water-filling, so the
//     ranks' row counts even out; single-holder experts keep all their rows),
//   * the all-to-all split sizes,
//   * the send order (which permuted rows go to which rank, in the receiver's
//     slot order) and its inverse,
//   * the receive-side regroup: received row -> slot-major GEMM row (segments
//     aligned to `align`), and its inverse.
// The algorithm is deterministic integer arithmetic, so every rank derives the
// same split from the same counts without further communication.  It is the
// native twin of reframework_b200/parallel/{ep.py:plan_exchange,
// eplb.py:split_rows}; tests check the two agree.
#include <algorithm>
#include <cstdint>
#include <numeric>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

// Split n rows over holders whose other load is `base`, equalising final loads.
void waterfill(int64_t n, const std::vector<int64_t> &base, std::vector<int64_t> &out) {
  const int m = (int)base.size();
  std::vector<int> order(m);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return base[a] < base[b]; });
  std::vector<int64_t> loads(m);
  for (int i = 0; i < m; ++i) loads[i] = base[order[i]];
  int k = m;
  auto prefix = [&](int kk) {
    int64_t s = 0;
    for (int i = 0; i < kk; ++i) s += loads[i];
    return s;
  };
  while (k > 1 && n + prefix(k) <= loads[k - 1] * (int64_t)k) --k;
  const int64_t level = (n + prefix(k)) / k;
  std::vector<int64_t> give(m, 0);
  int64_t used = 0;
  for (int i = 0; i < k; ++i) {
    give[i] = std::max<int64_t>(0, level - loads[i]);
    used += give[i];
  }
  int64_t rem = n - used;
  for (int i = 0; rem > 0; ++i, --rem) give[i % k] += 1;
  out.assign(m, 0);
  for (int pos = 0; pos < m; ++pos) out[order[pos]] = give[pos];
}

// Holders, water-filled per-holder quotas and the row runs of one step: the
// deterministic split every rank derives from the global counts.
struct Split {
  int R = 0, E = 0;
  std::vector<int64_t> quota, lo, sbase;  // [E * R]
  const int32_t *counts = nullptr;
  // rows of source rank `src`'s pairs for expert e that holder h computes
  // (and their offset inside src's run of e)
  int64_t piece(int e, int src, int h, int64_t *offset) const {
    const int64_t qlo = lo[(int64_t)e * R + h], qhi = qlo + quota[(int64_t)e * R + h];
    const int64_t slo = sbase[(int64_t)e * R + src], shi = slo + counts[(int64_t)src * E + e];
    const int64_t a = std::max(qlo, slo), b = std::min(qhi, shi);
    if (offset) *offset = a - slo;
    return std::max<int64_t>(0, b - a);
  }
};

// Returns RF_OK or an argument error (recorded).
int build_split(const int32_t *counts, int32_t R, int32_t E, const int32_t *slot_experts,
                const int32_t *slot_offsets, int32_t rounds, Split &sp) {
  // ---- holders of every expert, in rank order
  std::vector<std::vector<int>> holders(E);
  for (int r = 0; r < R; ++r) {
    RF_CHECK_ARG(slot_offsets[r] <= slot_offsets[r + 1], "EP split: slot_offsets not ascending");
    for (int s = slot_offsets[r]; s < slot_offsets[r + 1]; ++s) {
      const int e = slot_experts[s];
      RF_CHECK_ARG(e >= 0 && e < E, "EP split: slot expert out of range");
      holders[e].push_back(r);
    }
  }
  std::vector<int64_t> total(E, 0);
  for (int r = 0; r < R; ++r)
    for (int e = 0; e < E; ++e) {
      RF_CHECK_ARG(counts[(int64_t)r * E + e] >= 0, "EP split: negative count");
      total[e] += counts[(int64_t)r * E + e];
    }
  for (int e = 0; e < E; ++e)
    RF_CHECK_ARG(!holders[e].empty() || total[e] == 0, "EP split: routed expert held by no rank");
  // ---- per-holder quota
  std::vector<int64_t> &quota = sp.quota;
  quota.assign((int64_t)E * R, 0);
  std::vector<int64_t> load(R, 0);
  std::vector<int> replicated;
  for (int e = 0; e < E; ++e) {
    const auto &hs = holders[e];
    if (hs.empty()) continue;
    if (hs.size() == 1) {
      quota[(int64_t)e * R + hs[0]] = total[e];
    } else {
      replicated.push_back(e);
      const int64_t k = (int64_t)hs.size();
      for (int64_t i = 0; i < k; ++i) quota[(int64_t)e * R + hs[i]] = total[e] / k + (i < total[e] % k ? 1 : 0);
    }
  }
  for (int e = 0; e < E; ++e)
    for (int r = 0; r < R; ++r) load[r] += quota[(int64_t)e * R + r];
  std::stable_sort(replicated.begin(), replicated.end(),
                   [&](int a, int b) { return total[a] > total[b]; });
  std::vector<int64_t> base, nq;
  for (int it = 0; it < rounds; ++it) {
    bool changed = false;
    for (int e : replicated) {
      const auto &hs = holders[e];
      base.resize(hs.size());
      for (size_t i = 0; i < hs.size(); ++i) base[i] = load[hs[i]] - quota[(int64_t)e * R + hs[i]];
      waterfill(total[e], base, nq);
      for (size_t i = 0; i < hs.size(); ++i) {
        int64_t &q = quota[(int64_t)e * R + hs[i]];
        if (q != nq[i]) {
          load[hs[i]] += nq[i] - q;
          q = nq[i];
          changed = true;
        }
      }
    }
    if (!changed) break;
  }
  // ---- runs: holder h of expert e covers global rows [lo, lo + quota) (rank order)
  std::vector<int64_t> &lo = sp.lo, &sbase = sp.sbase;
  lo.assign((int64_t)E * R, 0);
  sbase.assign((int64_t)E * R, 0);
  for (int e = 0; e < E; ++e) {
    int64_t acc = 0, src = 0;
    for (int r = 0; r < R; ++r) {
      lo[(int64_t)e * R + r] = acc;
      acc += quota[(int64_t)e * R + r];
      sbase[(int64_t)e * R + r] = src;
      src += counts[(int64_t)r * E + e];
    }
  }
  sp.R = R;
  sp.E = E;
  sp.counts = counts;
  return RF_OK;
}

}  // namespace

extern "C" int rf_moe_ep_plan(const int32_t *counts, int32_t R, int32_t E, int32_t rank,
                              const int32_t *slot_experts, const int32_t *slot_offsets, int32_t align,
                              int32_t rounds, int64_t *send_splits, int64_t *recv_splits,
                              int32_t *packed, int64_t packed_capacity, int64_t *layout) {
  RF_CHECK_ARG(counts && slot_experts && slot_offsets && send_splits && recv_splits && layout,
               "rf_moe_ep_plan: null pointer");
  RF_CHECK_ARG(R >= 1 && E >= 1 && rank >= 0 && rank < R && align >= 1 && rounds >= 0,
               "rf_moe_ep_plan: bad sizes");
  Split sp;
  {
    const int rc = build_split(counts, R, E, slot_experts, slot_offsets, rounds, sp);
    if (rc) return rc;
  }
  auto piece = [&](int e, int src, int h, int64_t *offset) -> int64_t { return sp.piece(e, src, h, offset); };
  // ---- send side
  std::vector<int64_t> seg_start(E, 0);
  for (int e = 1; e < E; ++e) seg_start[e] = seg_start[e - 1] + counts[(int64_t)rank * E + e - 1];
  std::vector<std::pair<int64_t, int64_t>> pieces;
  bool identity = true;
  int64_t pos = 0;
  for (int d = 0; d < R; ++d) {
    int64_t nd = 0;
    for (int s = slot_offsets[d]; s < slot_offsets[d + 1]; ++s) {
      int64_t off = 0;
      const int64_t ln = piece(slot_experts[s], rank, d, &off);
      if (ln > 0) {
        const int64_t start = seg_start[slot_experts[s]] + off;
        identity = identity && start == pos;
        pieces.emplace_back(start, ln);
        pos += ln;
        nd += ln;
      }
    }
    send_splits[d] = nd;
  }
  const int64_t n_send = pos;
  // ---- receive side
  const int s0 = slot_offsets[rank], S = slot_offsets[rank + 1] - s0;
  std::vector<int64_t> c((int64_t)R * S, 0), lcount(S, 0), loff(S + 1, 0);
  for (int r = 0; r < R; ++r) {
    int64_t nr = 0;
    for (int j = 0; j < S; ++j) {
      const int64_t ln = piece(slot_experts[s0 + j], r, rank, nullptr);
      c[(int64_t)r * S + j] = ln;
      lcount[j] += ln;
      nr += ln;
    }
    recv_splits[r] = nr;
  }
  for (int j = 0; j < S; ++j) loff[j + 1] = loff[j] + (lcount[j] + align - 1) / align * align;
  const int64_t rows_cap = loff[S];
  int64_t recv_total = 0;
  for (int r = 0; r < R; ++r) recv_total += recv_splits[r];
  // ---- packed output: gather | inverse | local_offsets | local_counts | send_index | pos_of_row
  const int64_t n_gather = std::max<int64_t>(rows_cap, 1);
  const int64_t n_sendix = identity ? 0 : n_send;
  const int64_t need = n_gather + recv_total + (S + 1) + S + 2 * n_sendix;
  layout[0] = 0;                              // gather_index
  layout[1] = n_gather;
  layout[2] = layout[0] + n_gather;           // inverse_index
  layout[3] = recv_total;
  layout[4] = layout[2] + recv_total;         // local_offsets
  layout[5] = S + 1;
  layout[6] = layout[4] + S + 1;              // local_counts
  layout[7] = S;
  layout[8] = layout[6] + S;                  // send_index (absent when identity)
  layout[9] = n_sendix;
  layout[10] = layout[8] + n_sendix;          // pos_of_row
  layout[11] = n_sendix;
  layout[12] = rows_cap;
  layout[13] = identity ? 1 : 0;
  layout[14] = need;
  if (!packed || packed_capacity < need)
    return rf::fail(RF_ERR_ARG, "rf_moe_ep_plan: packed buffer needs " + std::to_string(need) + " int32");
  int32_t *gather = packed + layout[0], *inverse = packed + layout[2], *lo_out = packed + layout[4];
  int32_t *lc_out = packed + layout[6], *sendix = packed + layout[8], *posrow = packed + layout[10];
  for (int64_t i = 0; i < n_gather; ++i) gather[i] = -1;
  int64_t q = 0;
  std::vector<int64_t> before(S, 0);
  for (int r = 0; r < R; ++r)
    for (int j = 0; j < S; ++j) {
      const int64_t ln = c[(int64_t)r * S + j];
      const int64_t dst0 = loff[j] + before[j];
      for (int64_t i = 0; i < ln; ++i, ++q) {
        inverse[q] = (int32_t)(dst0 + i);
        gather[dst0 + i] = (int32_t)q;
      }
      before[j] += ln;
    }
  for (int j = 0; j <= S; ++j) lo_out[j] = (int32_t)loff[j];
  for (int j = 0; j < S; ++j) lc_out[j] = (int32_t)lcount[j];
  if (!identity) {
    int64_t p = 0;
    for (const auto &pc : pieces)
      for (int64_t i = 0; i < pc.second; ++i, ++p) {
        sendix[p] = (int32_t)(pc.first + i);
        posrow[pc.first + i] = (int32_t)p;
      }
  }
  return RF_OK;
}

// M[s * R + d] = rows rank s sends to rank d this step (the all-to-all
// matrix), derived from the same split as rf_moe_ep_plan: a rank can then
// address its rows directly in a peer's receive buffer.
extern "C" int rf_moe_ep_pair_rows(const int32_t *counts, int32_t R, int32_t E, const int32_t *slot_experts,
                                   const int32_t *slot_offsets, int32_t rounds, int64_t *pair_rows) {
  RF_CHECK_ARG(counts && slot_experts && slot_offsets && pair_rows, "rf_moe_ep_pair_rows: null pointer");
  RF_CHECK_ARG(R >= 1 && E >= 1 && rounds >= 0, "rf_moe_ep_pair_rows: bad sizes");
  Split sp;
  const int rc = build_split(counts, R, E, slot_experts, slot_offsets, rounds, sp);
  if (rc) return rc;
  for (int src = 0; src < R; ++src)
    for (int d = 0; d < R; ++d) {
      int64_t n = 0;
      for (int sl = slot_offsets[d]; sl < slot_offsets[d + 1]; ++sl) n += sp.piece(slot_experts[sl], src, d, nullptr);
      pair_rows[(int64_t)src * R + d] = n;
    }
  return RF_OK;
}
