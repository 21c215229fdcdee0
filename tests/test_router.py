"""Adapter pool + swap scheduler (ti_router_*): the policy on a NULL engine, read
back through the decision log (prefetch / evict per adapter)."""
import os
import subprocess
import sys

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


# ---------------------------------------------------------------- model-based
class _Policy:
    """The router's policy restated from its specification (ti_b200.h: router
    pool + scheduler), NULL-engine form: per-sequence hysteresis, LRU pool with
    a budget, step adapters never evicted, speculative prefetches sparing live
    sequences' adapters and giving up silently when nothing can go."""

    def __init__(self, max_resident, prefetch_after, switch_after):
        self.max, self.pf, self.sw = max_resident, prefetch_after, switch_after
        self.lru, self.seqs, self.in_use, self.actions = [], {}, {}, []
        self.stats = dict(observations=0, switches=0, prefetches=0, evictions=0, hits=0)

    def _evict_one(self, keep, spare_live):
        for a in reversed(self.lru):
            if a in keep or (spare_live and self.in_use.get(a, 0) > 0):
                continue
            self.lru.remove(a)
            self.actions.append((E, a))
            self.stats["evictions"] += 1
            return
        raise MemoryError

    def _ensure(self, a, keep, spare_live):
        keep = keep | {a}
        if a in self.lru:
            self.lru.remove(a)
            self.lru.insert(0, a)
            self.stats["hits"] += 1
        else:
            while len(self.lru) >= self.max:
                self._evict_one(keep, spare_live)
            self.lru.insert(0, a)
            self.actions.append((P, a))
            self.stats["prefetches"] += 1
        while len(self.lru) > self.max:
            self._evict_one(keep, spare_live)

    def _use(self, frm, to):
        if frm >= 0 and frm in self.in_use:
            self.in_use[frm] -= 1
            if self.in_use[frm] == 0:
                del self.in_use[frm]
        if to >= 0:
            self.in_use[to] = self.in_use.get(to, 0) + 1

    def observe(self, seq, c):
        self.stats["observations"] += 1
        s = self.seqs.setdefault(seq, dict(current=-2, candidate=-2, lead=0))
        if s["current"] == -2:
            s.update(current=c, candidate=c, lead=0)
            self._use(-1, c)
            return c
        if c == s["current"]:
            s.update(candidate=c, lead=0)
        else:
            if c == s["candidate"]:
                s["lead"] += 1
            else:
                s.update(candidate=c, lead=1)
            if s["lead"] == self.pf and c >= 0:
                try:
                    self._ensure(c, set(), True)
                except MemoryError:
                    pass
            if s["lead"] >= self.sw:
                self._use(s["current"], c)
                s.update(current=c, lead=0)
                self.stats["switches"] += 1
        return s["current"]

    def prepare(self, adapters):
        step = sorted({a for a in adapters if a >= 0})
        if len(step) > self.max:
            raise MemoryError
        for a in step:
            self._ensure(a, set(step), False)

    def forget(self, seq):
        s = self.seqs.pop(seq, None)
        if s is not None:
            self._use(s["current"], -1)


@pytest.mark.parametrize("seed", range(6))
def test_router_matches_its_policy_model(seed):
    import numpy as np

    rng = np.random.default_rng(seed)
    max_res = int(rng.integers(1, 5))
    pf = int(rng.integers(1, 4))
    sw = pf + int(rng.integers(0, 3))
    r = ti.Router(None, max_resident=max_res, prefetch_after=pf, switch_after=sw)
    m = _Policy(max_res, pf, sw)
    for step in range(3000):
        op = rng.random()
        if op < 0.7:
            seq, c = int(rng.integers(0, 6)), int(rng.integers(-1, 7))
            assert r.observe(seq, c) == m.observe(seq, c), step
        elif op < 0.95:
            ads = [int(a) for a in rng.integers(-1, 7, size=int(rng.integers(0, max_res + 2)))]
            try:
                m.prepare(ads)
                want = None
            except MemoryError:
                want = ti.TI_ERR_OOM
            if want is None:
                r.prepare(ads)
            else:
                with pytest.raises(ti.TiError) as ei:
                    r.prepare(ads)
                assert ei.value.status == want, step
        else:
            seq = int(rng.integers(0, 6))
            r.forget(seq)
            m.forget(seq)
        assert r.actions() == m.actions, step
        m.actions = []
        assert r.resident() == m.lru, step
        assert len(m.lru) <= max_res
    assert r.stats() == m.stats


def test_router_model_under_sanitizers(tmp_path):
    """router.cpp built with AddressSanitizer + UBSan runs the model-based test
    (iterator and container misuse, overflow abort the child)."""
    import host_sanitize

    if not host_sanitize.runtime():
        pytest.skip("gcc sanitizer runtimes not available")
    lib = str(tmp_path / "libhost_asan.so")
    ok, err = host_sanitize.build(lib)
    assert ok, err
    here = os.path.dirname(os.path.abspath(__file__))
    code = (f"import sys; sys.path[:0] = [{here!r}, {os.path.join(os.path.dirname(here), 'tensor-inference_b200')!r}]; "
            "import ti_b200 as ti, host_sanitize, test_router as T; "
            f"host_sanitize.bind(ti, {lib!r}); "
            "[T.test_router_matches_its_policy_model(s) for s in range(6)]; print('router ok')")
    r = subprocess.run([sys.executable, "-c", code], env=host_sanitize.env(), capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "router ok" in r.stdout, r.stderr[-3000:]
