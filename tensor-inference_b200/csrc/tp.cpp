// tp.cpp — tensor-parallel plumbing: the NCCL entry points (loaded at run time)
// and the shard plan of a tensor-parallel rank.
//
// NCCL is opened with dlopen rather than linked: a process that already holds
// an NCCL (PyTorch's, loaded with torch.distributed) shares that copy, and a
// single-GPU engine never needs one.
//
// Shard plan (Megatron-style, two all-reduces per layer): q/k/v are split by
// heads and gate/up by rows (column-parallel), o and down by input columns
// (row-parallel, partial sums all-reduced), the LM head by vocabulary rows
// (greedy id by an all-reduce max of packed (logit, index) keys); embeddings
// and norms are replicated.
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include "internal.h"
#include "tp.h"

namespace ti {

const NcclApi* nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's NCCL, if any
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.CommGetAsyncError =
            reinterpret_cast<decltype(api.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.AllGather &&
                 api.GetErrorString;
    });
    return api.ok ? &api : nullptr;
}

ti_status tp_plan_make(const ti_model_desc* d, int tp, int rank, ti_tp_shard* p) {
    TI_CHECK(d && p, TI_ERR_INVALID, "tp_plan: null argument");
    TI_CHECK(tp >= 1 && rank >= 0 && rank < tp, TI_ERR_INVALID, "tp_plan: rank %d of %d", rank, tp);
    TI_CHECK(d->n_heads % tp == 0 && d->n_kv_heads % tp == 0, TI_ERR_UNSUPPORTED,
             "tp_plan: %d q heads / %d kv heads do not split over %d ranks", d->n_heads, d->n_kv_heads, tp);
    TI_CHECK(d->intermediate % tp == 0 && d->vocab % tp == 0, TI_ERR_UNSUPPORTED,
             "tp_plan: intermediate %d / vocab %d do not split over %d ranks", d->intermediate, d->vocab, tp);
    const int align = d->weight_format == TI_WFMT_BF16 ? 128 : 256;  // K of the row-parallel GEMVs
    const int qw_l = d->n_heads / tp * d->head_dim, i_l = d->intermediate / tp;
    TI_CHECK(qw_l % align == 0 && i_l % align == 0, TI_ERR_UNSUPPORTED,
             "tp_plan: per-rank attention width %d / intermediate %d must be multiples of %d", qw_l, i_l, align);
    p->tp = tp;
    p->rank = rank;
    p->nq = d->n_heads / tp;
    p->nkv = d->n_kv_heads / tp;
    p->q0 = rank * p->nq;
    p->kv0 = rank * p->nkv;
    p->inter = i_l;
    p->i0 = rank * i_l;
    p->vocab = d->vocab / tp;
    p->v0 = rank * p->vocab;
    return TI_OK;
}

}  // namespace ti

using namespace ti;

extern "C" ti_status ti_nccl_unique_id(void* out) {
    clear_error();
    TI_CHECK(out, TI_ERR_INVALID, "ti_nccl_unique_id: null argument");
    const NcclApi* n = nccl_api();
    TI_CHECK(n, TI_ERR_UNSUPPORTED, "ti_nccl_unique_id: libnccl.so.2 not found");
    ncclUniqueId id;
    const ncclResult_t r = n->GetUniqueId(&id);
    TI_CHECK(r == ncclSuccess, TI_ERR_CUDA, "ncclGetUniqueId: %s", n->GetErrorString(r));
    memcpy(out, &id, sizeof id);
    return TI_OK;
}

extern "C" ti_status ti_tp_plan(const ti_model_desc* desc, int tp_size, int tp_rank, ti_tp_shard* out) {
    clear_error();
    return tp_plan_make(desc, tp_size, tp_rank, out);
}
