// Engine entry points the GGUF reader calls when it loads a file into an
// engine, stubbed so that gguf.cpp and api.cpp link alone into a sanitizer
// build of the host-side reader (tests/test_gguf_fuzz.py).  Test code only.
#include "internal.h"

namespace ti {
ti_status engine_slot_info(ti_engine*, const char*, int*, size_t*, size_t*) { return TI_ERR_UNSUPPORTED; }
}  // namespace ti

extern "C" ti_status ti_engine_load_tensor(ti_engine*, const char*, int, const void*, size_t) {
    return TI_ERR_UNSUPPORTED;
}
extern "C" ti_status ti_engine_set_rope_freqs(ti_engine*, const float*, int) { return TI_ERR_UNSUPPORTED; }
