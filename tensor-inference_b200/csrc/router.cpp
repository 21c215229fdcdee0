// router.cpp — adapter pool and swap scheduler over the engine's adapter slots.
//
// Spec only in the reference (README.md:170-180):
//   pool/       tracks which adapters are resident in VRAM; LRU eviction when the
//               budget is exceeded; async prefetch from RAM when a candidate is
//               identified; calls into adapter/ for the actual inject and eject
//   scheduler/  tracks semantic shift in the residual stream across tokens;
//               triggers pool/ prefetch ahead of a confirmed domain shift; a
//               hysteresis threshold prevents flicker at ambiguous boundaries;
//               holds the current adapter until the shift is decisive
// Here: the scheduler follows, per sequence, the adapter the PKM router names for
// its latest token (ti_pkm_query); a new candidate is prefetched once it has led
// for `prefetch_after` consecutive tokens and becomes the sequence's adapter after
// `switch_after`.  The pool keeps at most `max_resident` adapters in HBM, evicting
// the least recently used one that no live sequence or pending step uses, through
// ti_adapter_stage_host / ti_adapter_evict / ti_adapter_prefetch_async.  With a NULL
// engine only the decisions are recorded (ti_router_actions), to test the policy.
#include <algorithm>
#include <list>
#include <map>
#include <set>
#include <vector>

#include "internal.h"

struct ti_router {
    ti_engine* e = nullptr;
    ti_router_opts o{};
    ti_router_stats st{};
    std::list<int> lru;                              // resident adapters, most recent first
    std::map<int, std::list<int>::iterator> where;   // adapter -> its place in lru
    std::set<int> known;                             // adapters whose residency the router has learnt
    std::set<int> staged;                            // adapters with a host copy
    struct Seq {
        int current = -2;   // -2: no observation yet; -1: base model
        int candidate = -2;
        int lead = 0;
    };
    std::map<int, Seq> seqs;
    std::map<int, int> in_use;                       // adapter -> sequences using it
    std::vector<int32_t> actions;                    // (kind, adapter) pairs
};

namespace {

using ti::fail;

enum { kActPrefetch = 1, kActEvict = 2 };

void touch(ti_router* r, int a) {
    auto it = r->where.find(a);
    if (it != r->where.end()) r->lru.erase(it->second);
    r->lru.push_front(a);
    r->where[a] = r->lru.begin();
}

bool resident(const ti_router* r, int a) { return r->where.count(a) != 0; }

// learn an adapter the engine created resident (ti_adapter_create) the first time it is named
ti_status learn(ti_router* r, int a) {
    if (r->known.count(a)) return TI_OK;
    r->known.insert(a);
    if (!r->e) return TI_OK;  // policy only: adapters start evicted
    int res = 0;
    if (ti_status st = ti_adapter_is_resident(r->e, a, &res)) return st;
    if (res) touch(r, a);
    return TI_OK;
}

// evict the least recently used adapter outside `keep` (and, for a speculative
// prefetch, outside the live sequences' adapters)
ti_status evict_one(ti_router* r, const std::set<int>& keep, bool spare_live) {
    for (auto it = r->lru.rbegin(); it != r->lru.rend(); ++it) {
        const int a = *it;
        if (keep.count(a) || (spare_live && r->in_use.count(a))) continue;
        if (r->e) {
            if (!r->staged.count(a)) {
                if (ti_status st = ti_adapter_stage_host(r->e, a)) return st;
            }
            if (ti_status st = ti_adapter_evict(r->e, a)) return st;
        }
        r->staged.insert(a);
        r->where.erase(a);
        r->lru.erase(std::next(it).base());
        r->actions.push_back(kActEvict);
        r->actions.push_back(a);
        ++r->st.evictions;
        return TI_OK;
    }
    return fail(TI_ERR_OOM, "router: %d adapters resident, none evictable", (int)r->lru.size());
}

// make `a` resident (async), evicting past the budget but never an adapter in `keep`
ti_status ensure(ti_router* r, int a, const std::set<int>& keep, bool spare_live) {
    if (ti_status st = learn(r, a)) return st;
    std::set<int> keep_a = keep;
    keep_a.insert(a);
    if (resident(r, a)) {
        touch(r, a);
        ++r->st.hits;
    } else {
        while ((int)r->lru.size() >= r->o.max_resident)
            if (ti_status st = evict_one(r, keep_a, spare_live)) return st;
        if (r->e) {
            if (ti_status st = ti_adapter_prefetch_async(r->e, a)) return st;
        }
        touch(r, a);
        r->actions.push_back(kActPrefetch);
        r->actions.push_back(a);
        ++r->st.prefetches;
    }
    // adapters the engine created resident count once the router has named them
    while ((int)r->lru.size() > r->o.max_resident)
        if (ti_status st = evict_one(r, keep_a, spare_live)) return st;
    return TI_OK;
}

void use(ti_router* r, int from, int to) {
    if (from >= 0) {
        auto it = r->in_use.find(from);
        if (it != r->in_use.end() && --it->second == 0) r->in_use.erase(it);
    }
    if (to >= 0) ++r->in_use[to];
}

}  // namespace

extern "C" {

ti_status ti_router_create(ti_engine* e, const ti_router_opts* o, ti_router** out) {
    ti::clear_error();
    TI_CHECK(o && out, TI_ERR_INVALID, "ti_router_create: null argument");
    TI_CHECK(o->max_resident >= 1, TI_ERR_INVALID, "router: max_resident must be >= 1");
    TI_CHECK(o->prefetch_after >= 1 && o->switch_after >= o->prefetch_after, TI_ERR_INVALID,
             "router: need 1 <= prefetch_after <= switch_after (got %d, %d)", o->prefetch_after, o->switch_after);
    ti_router* r = new ti_router;
    r->e = e;
    r->o = *o;
    *out = r;
    return TI_OK;
}

ti_status ti_router_destroy(ti_router* r) {
    delete r;
    return TI_OK;
}

ti_status ti_router_observe(ti_router* r, int seq, int candidate, int* use_adapter) {
    ti::clear_error();
    TI_CHECK(r && use_adapter, TI_ERR_INVALID, "ti_router_observe: null argument");
    TI_CHECK(candidate >= -1, TI_ERR_INVALID, "router: candidate %d (adapter id or -1)", candidate);
    ++r->st.observations;
    ti_router::Seq& s = r->seqs[seq];
    if (s.current == -2) {  // first token of the sequence: no history to hold
        s.current = candidate;
        use(r, -1, candidate);
        s.candidate = candidate;
        s.lead = 0;
        *use_adapter = s.current;
        return TI_OK;
    }
    if (candidate == s.current) {
        s.candidate = candidate;
        s.lead = 0;
    } else {
        if (candidate == s.candidate) ++s.lead;
        else {
            s.candidate = candidate;
            s.lead = 1;
        }
        if (s.lead == r->o.prefetch_after && candidate >= 0) {
            // prefetch ahead of the switch, best effort: it evicts no adapter a live
            // sequence uses, and no room is not an error (the switch's step fetches it)
            const ti_status st = ensure(r, candidate, std::set<int>{}, true);
            if (st == TI_ERR_OOM) ti::clear_error();
            else if (st) return st;
        }
        if (s.lead >= r->o.switch_after) {
            use(r, s.current, candidate);
            s.current = candidate;
            s.lead = 0;
            ++r->st.switches;
        }
    }
    *use_adapter = s.current;
    return TI_OK;
}

ti_status ti_router_prepare(ti_router* r, const int32_t* adapters, int n) {
    ti::clear_error();
    TI_CHECK(r && (adapters || n == 0), TI_ERR_INVALID, "ti_router_prepare: null argument");
    std::set<int> step;
    for (int i = 0; i < n; ++i)
        if (adapters[i] >= 0) step.insert(adapters[i]);
    TI_CHECK((int)step.size() <= r->o.max_resident, TI_ERR_OOM,
             "router: a step uses %zu adapters, the budget is %d", step.size(), r->o.max_resident);
    for (int a : step)
        if (ti_status st = ensure(r, a, step, false)) return st;
    return TI_OK;
}

ti_status ti_router_forget(ti_router* r, int seq) {
    ti::clear_error();
    TI_CHECK(r, TI_ERR_INVALID, "ti_router_forget: null argument");
    auto it = r->seqs.find(seq);
    if (it == r->seqs.end()) return TI_OK;
    use(r, it->second.current, -1);
    r->seqs.erase(it);
    return TI_OK;
}

ti_status ti_router_stats_get(const ti_router* r, ti_router_stats* s) {
    ti::clear_error();
    TI_CHECK(r && s, TI_ERR_INVALID, "ti_router_stats_get: null argument");
    *s = r->st;
    return TI_OK;
}

ti_status ti_router_actions(ti_router* r, int32_t* out, int cap, int* n) {
    ti::clear_error();
    TI_CHECK(r && n && (out || cap == 0), TI_ERR_INVALID, "ti_router_actions: null argument");
    const int have = (int)r->actions.size() / 2;
    const int k = std::min(have, cap);
    for (int i = 0; i < 2 * k; ++i) out[i] = r->actions[i];
    r->actions.erase(r->actions.begin(), r->actions.begin() + 2 * k);
    *n = k;
    return TI_OK;
}

ti_status ti_router_resident(const ti_router* r, int32_t* out, int cap, int* n) {
    ti::clear_error();
    TI_CHECK(r && n && (out || cap == 0), TI_ERR_INVALID, "ti_router_resident: null argument");
    int k = 0;
    for (int a : r->lru) {
        if (k < cap) out[k] = a;
        ++k;
    }
    *n = k;
    return TI_OK;
}

}  // extern "C"
