// kivi_internal.h -- argument structs and host helpers shared by the .cu files.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "../../include/kivi_sm100.h"

namespace kivi {

struct StoreArgs {
    const void* k; const void* v;
    int64_t sk_h, sk_s, sk_d, sv_h, sv_s, sv_d;
    int H, S_k, S_v, D, calib_k, calib_v;
    const float* alphas; int n_alphas;
    float g_k, g_v;
    uint8_t* k_packed; void* k_scale; int kpage0, k_np_stride;
    uint8_t* v_packed; void* v_scale; int vtok0, v_s_stride;
};

struct DequantArgs {
    const uint8_t* k_packed; const void* k_scale; int k_np_stride;
    const uint8_t* v_packed; const void* v_scale; int v_s_stride;
    int H, S, D;
    float g_k, g_v;
    void* k_out; void* v_out;
    int64_t so_h, so_s, so_d;
};

struct RoundtripArgs {
    const void* x; void* y;
    int H, S, D, fmt, layout, calib;
    const float* alphas; int n_alphas;
};

// Records the CUDA error (readable through kivi_last_cuda_error) and maps it.
int record_cuda_error(cudaError_t e);

inline int check_launch() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KIVI_OK : record_cuda_error(e);
}

}  // namespace kivi
