"""Residency policy of ExpertOffloadCache / Prediction — the scenarios of the
reference's tests/test_moe_prefetch.py:52-194 and
tests/test_moe_eviction_policy.py:50-186, restated against the slot-pool cache.
Runs on the CPU ("device" = host memory): only bookkeeping and copies."""

import os

import pytest
import torch

from reframework_b200 import env
from reframework_b200.moe.offload_cache import ExpertOffloadCache, Prediction

DEVICE = torch.device("cpu")


def make_cache(E, cap, H=4, I=2):
    cache = ExpertOffloadCache(device=DEVICE, lru_capacity=cap, dtype=torch.float16)
    cache.load([{"w1": torch.randn(2 * I, H, dtype=torch.float16),
                 "w2": torch.randn(H, I, dtype=torch.float16)} for _ in range(E)])
    return cache


def expert_bytes(cache):
    return cache.expert_bytes(0)


@pytest.fixture
def policy(monkeypatch):
    def _set(v):
        monkeypatch.setenv("RE_CACHE_POLICY", v)
    return _set


# ------------------------------------------------------------- Prediction
def test_predict_next_ranks_by_frequency_and_filters_resident():
    cache = make_cache(6, 6)
    cache.prefetch([0, 1])
    pred = Prediction(cache, window=16)
    pred._history.extend([frozenset({2, 4, 0}), frozenset({2, 3, 1}), frozenset({2, 3})])
    pred._age = {2: 0, 3: 1, 4: 2}
    ranked = pred.predict_next()
    assert 0 not in ranked and 1 not in ranked
    assert set(ranked) == {2, 3, 4} and ranked[0] == 2 and ranked.index(3) < ranked.index(4)


def test_predict_next_recency_tiebreak():
    cache = make_cache(4, 8)
    pred = Prediction(cache, window=16)
    pred._history.append(frozenset({0}))
    pred._history.append(frozenset({1}))
    pred._age = {0: 1, 1: 0}
    assert pred.predict_next()[0] == 1


def test_prefill_resets_history():
    cache = make_cache(4, 8)
    pred = Prediction(cache, window=16)
    pred.record_step([0], is_prefill=False, forward_ms=0.0)
    pred.record_step([1], is_prefill=False, forward_ms=0.0)
    assert pred._history
    pred.record_step([0, 1, 2, 3], is_prefill=True, forward_ms=0.0)
    assert list(pred._history) == [] and pred._age == {} and pred.predict_next() == []


# ------------------------------------------------------------- reserve
def test_reserve_bandwidth_caps_k():
    cache = make_cache(8, 16)
    b = expert_bytes(cache)
    cache._bw_headroom = 1.0
    cache._bw_gb_s = 1e9
    n = cache.reserve([0, 1, 2, 3], forward_ms=2.5 * b / 1e15, protect_current=[])
    assert n == 2
    assert set(cache._lru) == {0, 1}
    assert cache._next_reserve == frozenset({0, 1})
    assert cache.stats.predicts == 2


def test_reserve_inflight_bytes_shrink_budget():
    cache = make_cache(8, 16)
    b = expert_bytes(cache)
    cache._bw_headroom = 1.0
    cache._bw_gb_s = 1e9
    n = cache.reserve([0, 1, 2, 3], forward_ms=3.5 * b / 1e15, protect_current=[], inflight_bytes=2 * b)
    assert n == 1 and cache.stats.inflight_bytes == 2 * b


def test_reserve_lru_room_caps_k_and_evicts_stale():
    cache = make_cache(8, 4)
    cache.prefetch([0, 1, 2, 3])
    assert cache.reserve([4, 5], forward_ms=0.0, protect_current=[2, 3]) == 2
    assert set(cache._lru) == {2, 3, 4, 5}
    assert cache._next_reserve == frozenset({4, 5})


def test_reserve_stops_when_nothing_is_evictable():
    cache = make_cache(8, 2)
    cache.prefetch([0, 1])
    n = cache.reserve([2, 3, 4], forward_ms=0.0, protect_current=[0, 1])
    assert n == 1  # one load past capacity, then stop (reference behaviour)
    assert set(cache._lru) == {0, 1, 2}


def test_reserve_skips_resident_and_noop():
    cache = make_cache(4, 4)
    cache.prefetch([0])
    assert cache.reserve([0, 1, 2], forward_ms=0.0, protect_current=[0]) == 2
    assert set(cache._lru) == {0, 1, 2}
    assert cache.reserve([], forward_ms=0.0) == 0


# ------------------------------------------------------------- two-tier eviction
def test_prefetch_evicts_stale_not_soft():
    cache = make_cache(8, 4)
    cache.prefetch([0, 1, 7])
    cache._next_reserve = frozenset({0, 1})
    cache.prefetch([2, 3])
    assert set(cache._lru) == {0, 1, 2, 3}


def test_prefetch_evicts_stale_first_then_soft():
    cache = make_cache(6, 4)
    cache.prefetch([0, 1])
    cache._next_reserve = frozenset({0, 1})
    cache.prefetch([2, 3, 4])
    assert {2, 3, 4} <= set(cache._lru) and 0 not in cache._lru and 1 in cache._lru


def test_prefetch_hard_never_evicted_when_only_hard_exceeds():
    cache = make_cache(6, 2)
    cache.prefetch([0, 1, 2])
    assert set(cache._lru) == {0, 1, 2}
    assert cache.num_slots == 3  # the pool grew instead of evicting the request


def test_reset_lru_clears_reserve_and_history():
    cache = make_cache(6, 4)
    cache.attach_predictor(window=4)
    cache._predictor.record_step([0], is_prefill=False, forward_ms=0.0)
    cache.reserve([3], forward_ms=0.0, protect_current=[0])
    assert cache._next_reserve
    cache.reset_lru()
    assert len(cache._lru) == 0 and cache._next_reserve == frozenset()
    assert list(cache._predictor._history) == []
    assert sorted(cache._free) == list(range(cache.num_slots))


def test_prefetch_returns_pool_rows_holding_the_experts():
    cache = make_cache(6, 3)
    w1, w2, local = cache.prefetch([4, 1])
    assert set(local) == {1, 4}
    for e, s in local.items():
        assert torch.equal(w1[s], cache._host[e][0]) and torch.equal(w2[s], cache._host[e][1])
    cache.prefetch([0, 2, 3])  # evicts 1 and 4, reuses their slots
    w1, _, local = cache.prefetch([2])
    assert torch.equal(w1[local[2]], cache._host[2][0])
    assert cache.stats.hits == 1 and cache.stats.misses == 5 and cache.stats.evictions == 2


def test_substitution_serves_similar_resident_expert():
    cache = make_cache(4, 4)
    sim = torch.eye(4)
    sim[3, 1] = 0.9
    sim[3, 0] = 0.5
    cache.prefetch([0, 1])  # loaded before the table exists: two real fills
    cache.set_sim_table(sim)
    _, _, local = cache.prefetch([3])
    assert cache.stats.subs == 1 and local[3] == cache.slot_of(1)
    with pytest.raises(ValueError):
        cache.set_sim_table(torch.eye(3))


# ------------------------------------------------------------- RE_CACHE_POLICY
def test_lru_is_default_when_unset(monkeypatch):
    monkeypatch.delenv("RE_CACHE_POLICY", raising=False)
    cache = make_cache(6, 3)
    cache.prefetch([0, 1, 2])
    cache.prefetch([3])
    assert set(cache._lru) == {1, 2, 3}


def test_lru_invalid_value_falls_back(policy):
    policy("bogus_policy")
    cache = make_cache(6, 3)
    cache.prefetch([0, 1, 2])
    cache.prefetch([3])
    assert set(cache._lru) == {1, 2, 3}


def test_least_stale_evicts_most_stale_not_lru_oldest(policy):
    policy("least_stale")
    cache = make_cache(8, 3)
    cache.prefetch([0, 1, 2])
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 1, 1: 4, 2: 8}
    cache.prefetch([3])
    assert set(cache._lru) == {0, 1, 3}


def test_least_stale_without_predictor_degrades_to_lru(policy):
    policy("least_stale")
    cache = make_cache(6, 3)
    cache.prefetch([0, 1, 2])
    cache.prefetch([3])
    assert set(cache._lru) == {1, 2, 3}


def test_least_stale_never_seen_counts_as_maximally_stale(policy):
    policy("least_stale")
    cache = make_cache(8, 3)
    cache.prefetch([0, 1, 2])
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 1, 2: 3}
    cache.prefetch([3])
    assert set(cache._lru) == {0, 2, 3}


def test_least_stale_tie_breaks_by_lru_order(policy):
    policy("least_stale")
    cache = make_cache(8, 3)
    cache.prefetch([0, 1, 2])
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 5, 1: 5, 2: 2}
    cache.prefetch([3])
    assert set(cache._lru) == {1, 2, 3}


def test_least_stale_hard_never_evicted(policy):
    policy("least_stale")
    cache = make_cache(6, 2)
    cache.prefetch([0, 1])
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 10, 1: 10, 2: 0}
    cache.prefetch([2])
    assert 2 in cache._lru and len(cache._lru) == 2


def test_least_stale_soft_evicted_only_after_stale(policy):
    policy("least_stale")
    cache = make_cache(8, 4)
    cache.prefetch([0, 1, 7])
    cache._next_reserve = frozenset({0, 1})
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 9, 1: 9, 7: 1}
    cache.prefetch([2, 3])
    assert 7 not in cache._lru and {0, 1, 2, 3} <= set(cache._lru)


def test_least_stale_picks_stalest_soft_when_no_stale_left(policy):
    policy("least_stale")
    cache = make_cache(6, 3)
    cache.prefetch([0, 1])
    cache._next_reserve = frozenset({0, 1})
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 2, 1: 7}
    cache.prefetch([2, 3])
    assert set(cache._lru) == {0, 2, 3}


def test_lru_oldest_wins_same_scenario(policy):
    policy("lru")
    cache = make_cache(8, 3)
    cache.prefetch([0, 1, 2])
    pred = Prediction(cache, window=16)
    cache._predictor = pred
    pred._age = {0: 1, 1: 4, 2: 8}
    cache.prefetch([3])
    assert set(cache._lru) == {1, 2, 3}


def test_env_getter_normalizes(monkeypatch):
    for raw, expected in {"least_stale": "least_stale", "LEAST_STALE": "least_stale", "lru": "lru",
                          "garbage": "lru"}.items():
        monkeypatch.setenv("RE_CACHE_POLICY", raw)
        assert env.get_moe_cache_policy() == expected


def test_stats_as_dict_keys():
    cache = make_cache(4, 2)
    cache.prefetch([0, 1, 2])
    d = cache.stats.as_dict()
    assert set(d) == {"hits", "misses", "evictions", "subs", "predicts", "inflight_bytes", "transfer_mb"}
    assert "hit=" in cache.report()


# ------------------------------------------------------------- expert split
def test_split_residency_and_stats_follow_the_reference():
    """split_prefetch + reactive_load over the steps of the reference's own
    split run (golden fixture): the experts resident before every step, the
    final residency and the hit / miss / eviction / transfer counters agree."""
    from conftest import golden_config, load_golden
    from reframework_b200.workloads import generate
    rec = load_golden("int8_split_k1")
    cfg = golden_config(rec)
    d = generate(cfg)
    cache = ExpertOffloadCache(device=torch.device("cpu"), lru_capacity=4, dtype=cfg.dtype)
    cache.load([{"w1": d["w1"][e], "w2": d["w2"][e]} for e in range(cfg.experts)])
    cache.quantize_int8_host()
    assert cache.cpu_split
    for s in range(cfg.steps):
        assert sorted(cache._lru) == rec["resident_before"][s].tolist(), f"step {s}"
        (_, _, hit_slots), misses = cache.split_prefetch(rec["ids"][s].reshape(-1).tolist())
        routed = sorted(set(rec["ids"][s].reshape(-1).tolist()))
        assert sorted(hit_slots) == [e for e in routed if e in rec["resident_before"][s].tolist()]
        assert misses == [e for e in routed if e not in hit_slots]
        cache.reactive_load(misses)
    assert sorted(cache._lru) == rec["resident_after"].tolist()
    st, ref = cache.stats.as_dict(), rec["cache_stats"]
    for k in ("hits", "misses", "evictions", "subs", "transfer_mb"):
        assert st[k] == ref[k], (k, st[k], ref[k])


def test_int8_copies_match_the_reference_quantizer():
    """quantize_int8_host / cpu_banks give the codes and scales of the
    reference's symmetric per-tensor quantizer (restated in the oracle)."""
    from oracle import moe_oracle as O
    g = torch.Generator().manual_seed(3)
    cache = ExpertOffloadCache(device=torch.device("cpu"), lru_capacity=2, dtype=torch.bfloat16)
    ex = [{"w1": (torch.randn(12, 8, generator=g) * 0.02).bfloat16(), "w2": (torch.randn(8, 6, generator=g) * 0.02).bfloat16()}
          for _ in range(3)]
    ex[1]["w2"].zero_()
    cache.load(ex)
    cache.quantize_int8_host()
    w1q, w2q, s1, s2, local = cache.cpu_banks([2, 0, 1])
    assert local == {0: 0, 1: 1, 2: 2}
    for k, e in enumerate([0, 1, 2]):
        q1, r1 = O.sym_int8_quantize(ex[e]["w1"])
        q2, r2 = O.sym_int8_quantize(ex[e]["w2"])
        assert torch.equal(w1q[k], q1) and torch.equal(w2q[k], q2)
        assert float(s1[k]) == torch.tensor(r1, dtype=torch.float32).item()
        assert float(s2[k]) == torch.tensor(r2, dtype=torch.float32).item()
    assert float(s2[1]) == 1.0 and not w2q[1].any()  # an all-zero matrix: scale 1, zero codes
