// Engine entry points that the host-side units call on a live engine (the GGUF
// reader loading a file into one, the router moving adapters), stubbed so that
// gguf.cpp, router.cpp and api.cpp link alone into a sanitizer build
// (tests/test_gguf_fuzz.py, tests/test_router.py).  The tests drive them with
// no engine, so the stubs never run.  Test code only.
#include "internal.h"

namespace ti {
ti_status engine_slot_info(ti_engine*, const char*, int*, size_t*, size_t*) { return TI_ERR_UNSUPPORTED; }
void rope_tables_release() {}
}  // namespace ti

extern "C" ti_status ti_engine_load_tensor(ti_engine*, const char*, int, const void*, size_t) {
    return TI_ERR_UNSUPPORTED;
}
extern "C" ti_status ti_engine_set_rope_freqs(ti_engine*, const float*, int) { return TI_ERR_UNSUPPORTED; }
extern "C" ti_status ti_adapter_stage_host(ti_engine*, int) { return TI_ERR_UNSUPPORTED; }
extern "C" ti_status ti_adapter_evict(ti_engine*, int) { return TI_ERR_UNSUPPORTED; }
extern "C" ti_status ti_adapter_prefetch_async(ti_engine*, int) { return TI_ERR_UNSUPPORTED; }
extern "C" ti_status ti_adapter_is_resident(ti_engine*, int, int*) { return TI_ERR_UNSUPPORTED; }
