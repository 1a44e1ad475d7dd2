// kivi_abi.cu -- status strings, version and CUDA error bookkeeping of the C ABI.
#include "kivi_internal.h"

namespace kivi {
static thread_local int g_last_cuda_error = 0;
int record_cuda_error(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return KIVI_ERR_CUDA;
}
}  // namespace kivi

extern "C" const char* kivi_status_string(int status) {
    switch (status) {
        case KIVI_OK: return "ok";
        case KIVI_ERR_ARG: return "invalid argument (shape, null pointer or enum)";
        case KIVI_ERR_ALIGN: return "pointer or stride violates the alignment rule";
        case KIVI_ERR_UNSUPPORTED: return "unsupported configuration";
        case KIVI_ERR_CUDA: return "CUDA runtime/driver error (see kivi_last_cuda_error)";
        case KIVI_ERR_TIMEOUT: return "device-side bounded wait expired";
        case KIVI_ERR_SCRATCH: return "problem needs more scratch than the fixed no-alloc buffer (use kivi_decode with a workspace)";
        default: return "unknown status";
    }
}

extern "C" int kivi_version(void) { return 100; }
extern "C" int kivi_last_cuda_error(void) { return kivi::g_last_cuda_error; }
