"""Adapter pool + swap scheduler (ti_router_*): the policy on a NULL engine, read
back through the decision log (prefetch / evict per adapter)."""
import pytest

import ti_b200 as ti

P, E = ti.Router.PREFETCH, ti.Router.EVICT


def test_hysteresis_holds_through_flicker_and_switches_when_decisive():
    r = ti.Router(None, max_resident=4, prefetch_after=2, switch_after=3)
    assert r.observe(0, 1) == 1                 # first token: no history to hold
    assert r.actions() == []
    for c in (2, 1, 2, 1, 3, 1):                # ambiguous boundary: never two in a row
        assert r.observe(0, c) == 1
    assert r.actions() == []
    assert r.observe(0, 2) == 1
    assert r.observe(0, 2) == 1                 # led 2 tokens: prefetched ahead of the switch
    assert r.actions() == [(P, 2)]
    assert r.observe(0, 2) == 2                 # led 3 tokens: switched
    assert r.observe(0, 1) == 2                 # the new adapter is held in turn
    s = r.stats()
    assert s["switches"] == 1 and s["prefetches"] == 1 and s["observations"] == 11


def test_base_model_candidate_switches_without_prefetch():
    r = ti.Router(None, max_resident=2, prefetch_after=1, switch_after=2)
    assert r.observe(5, 0) == 0
    assert r.observe(5, -1) == 0
    assert r.observe(5, -1) == -1
    assert r.actions() == []
    with pytest.raises(ti.TiError) as ei:
        r.observe(5, -3)
    assert ei.value.status == ti.TI_ERR_INVALID


def test_lru_eviction_within_the_budget():
    r = ti.Router(None, max_resident=2, prefetch_after=1, switch_after=1)
    r.prepare([0])
    r.prepare([1, 1, -1])
    assert r.actions() == [(P, 0), (P, 1)]
    r.prepare([2])                              # 0 is least recently used
    assert r.actions() == [(E, 0), (P, 2)]
    r.prepare([1])                              # hit; 2 becomes the least recently used
    assert r.actions() == []
    r.prepare([0])
    assert r.actions() == [(E, 2), (P, 0)]
    assert r.resident() == [0, 1]
    s = r.stats()
    assert (s["prefetches"], s["evictions"], s["hits"]) == (4, 2, 1)


def test_step_adapters_are_never_evicted_and_budget_errors():
    r = ti.Router(None, max_resident=2, prefetch_after=1, switch_after=1)
    r.prepare([0, 1])
    r.actions()
    r.prepare([2, 1])                           # 1 belongs to the step: 0 goes although more recent
    assert r.actions() == [(E, 0), (P, 2)]
    with pytest.raises(ti.TiError) as ei:
        r.prepare([0, 1, 2])
    assert ei.value.status == ti.TI_ERR_OOM


def test_speculative_prefetch_spares_live_sequences():
    r = ti.Router(None, max_resident=1, prefetch_after=2, switch_after=3)
    assert r.observe(0, 0) == 0                 # sequence 0 lives on adapter 0
    r.prepare([0])
    assert r.observe(1, -1) == -1               # sequence 1 on the base model
    r.actions()
    for _ in range(2):
        assert r.observe(1, 1) == -1            # prefetch of 1 would evict 0, which is live: skipped
    assert r.actions() == []
    assert r.observe(1, 1) == 1                 # the switch is not held back by the pool
    r.prepare([1])                              # the step may evict what it does not use
    assert r.actions() == [(E, 0), (P, 1)]
    r.forget(0)
    r.forget(1)
    assert r.observe(0, 3) == 3                 # a forgotten sequence starts afresh


def test_rejects_bad_options():
    for kw in (dict(max_resident=0), dict(prefetch_after=0), dict(prefetch_after=3, switch_after=2)):
        args = dict(max_resident=2, prefetch_after=1, switch_after=2)
        args.update(kw)
        with pytest.raises(ti.TiError) as ei:
            ti.Router(None, **args)
        assert ei.value.status == ti.TI_ERR_INVALID
