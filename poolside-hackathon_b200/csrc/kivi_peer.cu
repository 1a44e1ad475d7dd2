// kivi_peer.cu -- cross-GPU log-sum-exp merge of sequence-parallel decode
// partials over NVLink peer memory (no collective library on the data path).
//
// Each rank owns one exchange buffer (same size on every rank), allocated
// here with cudaMalloc and mapped into the other ranks' address spaces with
// CUDA IPC handles (plain point-to-point peer mappings):
//   [0, 64)      uint32 flag[16]: flag[j] = newest epoch rank j has published
//                to this rank (written remotely by rank j, read locally)
//   [256, ...)   two slots of rows x (2 + D) fp32: m [rows], l [rows],
//                acc [rows][D]; epoch e uses slot e & 1
// A step is: kivi_peer_publish (copy this rank's partial state into slot
// e & 1 of its own buffer, then release epoch e into flag[rank] of every
// rank) and kivi_peer_merge (wait, bounded, until every flag has reached e;
// read all ranks' slots through their peer pointers; merge; bf16 out).
// Two slots make the buffer reusable without a second barrier: a rank
// publishes e + 2 into the slot of e only after its merge e + 1 saw every
// peer publish e + 1, which each peer does after finishing its merge e.
// The epoch counter lives in device memory, so the pair replays correctly
// inside a CUDA graph.  All waits are bounded and report KIVI_ERR_TIMEOUT.
#include "kivi_common.cuh"
#include "kivi_internal.h"
#include <cstring>

namespace kivi {
namespace peer {

constexpr int MAX_W = 16;
constexpr int SLOT0 = 256;            // byte offset of slot 0

__host__ __device__ inline int64_t slot_floats(int rows, int D) { return (int64_t)rows * (2 + D); }

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One CTA: advance the epoch, copy the partial state into this rank's slot,
// make it visible system-wide, then release the epoch to every rank.
__global__ void __launch_bounds__(256) publish_kernel(const float* __restrict__ m, const float* __restrict__ l,
                                                      const float* __restrict__ acc, int rows, int D,
                                                      uint8_t* my_buf, const uint64_t* __restrict__ peers, int W,
                                                      int rank, unsigned int* epoch) {
    __shared__ unsigned int e_s;
    if (threadIdx.x == 0) { e_s = *epoch + 1; *epoch = e_s; }
    __syncthreads();
    const unsigned int e = e_s;
    float* slot = reinterpret_cast<float*>(my_buf + SLOT0) + (e & 1) * slot_floats(rows, D);
    for (int i = threadIdx.x; i < rows; i += blockDim.x) { slot[i] = m[i]; slot[rows + i] = l[i]; }
    const int64_t n4 = (int64_t)rows * D / 4;
    const float4* a4 = reinterpret_cast<const float4*>(acc);
    float4* d4 = reinterpret_cast<float4*>(slot + 2 * rows);
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = a4[i];
    __syncthreads();                                   // the slot is written (CTA scope) ...
    if (threadIdx.x < W) {                             // ... and released system-wide to every rank
        __threadfence_system();
        unsigned int* flag = reinterpret_cast<unsigned int*>(peers[threadIdx.x]) + rank;
        st_release_sys(flag, e);
    }
}

// One CTA per row: wait for every rank's epoch, then merge the W states.
__global__ void __launch_bounds__(128) merge_kernel(const uint64_t* __restrict__ peers, int W, int rows, int D,
                                                    const unsigned int* epoch, const uint8_t* my_buf,
                                                    __nv_bfloat16* __restrict__ out, int* err,
                                                    long long timeout_ns) {
    __shared__ float wgt[MAX_W];
    __shared__ float lsum;
    __shared__ int ok_s;
    const int row = blockIdx.x;
    const unsigned int e = *epoch;
    if (threadIdx.x == 0) {
        const unsigned int* flags = reinterpret_cast<const unsigned int*>(my_buf);
        int ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int j = 0; j < W && ok; ++j) {
            while ((int)(ld_acquire_sys(flags + j) - e) < 0) {
                if ((long long)(globaltimer_ns() - t0) > timeout_ns) {
                    ok = 0;
                    if (err) atomicCAS(err, 0, KIVI_ERR_TIMEOUT);
                    break;
                }
            }
        }
        ok_s = ok;
    }
    __syncthreads();                                   // peers' slots acquired by thread 0
    if (!ok_s) return;
    const int64_t off = (e & 1) * slot_floats(rows, D);
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int j = 0; j < W; ++j) {
            const float* s = reinterpret_cast<const float*>(peers[j] + SLOT0) + off;
            M = fmaxf(M, s[row]);
        }
        const float Mr = (M == -INFINITY) ? 0.f : M;
        float L = 0.f;
        for (int j = 0; j < W; ++j) {
            const float* s = reinterpret_cast<const float*>(peers[j] + SLOT0) + off;
            const float w = exp2f(s[row] - Mr);
            wgt[j] = w;
            L += s[rows + row] * w;
        }
        lsum = L;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float a = 0.f;
        for (int j = 0; j < W; ++j) {
            const float* s = reinterpret_cast<const float*>(peers[j] + SLOT0) + off;
            a += s[2 * rows + (int64_t)row * D + d] * wgt[j];
        }
        out[(int64_t)row * D + d] = __float2bfloat16_rn(lsum > 0.f ? a / lsum : 0.f);
    }
}

}  // namespace peer
}  // namespace kivi

using namespace kivi;

extern "C" int64_t kivi_peer_buffer_bytes(int rows, int D, int W) {
    if (rows <= 0 || D <= 0 || D % 4 || W <= 0 || W > peer::MAX_W) return 0;
    return peer::SLOT0 + 2 * peer::slot_floats(rows, D) * (int64_t)sizeof(float);
}

extern "C" int kivi_peer_publish(const float* m, const float* l, const float* acc, int rows, int D, void* my_buf,
                                 const uint64_t* peer_bufs, int W, int rank, unsigned int* epoch,
                                 kivi_stream_t stream) {
    if (rows <= 0 || D <= 0 || D % 4 || W <= 0 || W > peer::MAX_W || rank < 0 || rank >= W) return KIVI_ERR_ARG;
    if (!m || !l || !acc || !my_buf || !peer_bufs || !epoch) return KIVI_ERR_ARG;
    if ((uintptr_t)my_buf % 16 || (uintptr_t)acc % 16) return KIVI_ERR_ALIGN;
    peer::publish_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(m, l, acc, rows, D, static_cast<uint8_t*>(my_buf),
                                                              peer_bufs, W, rank, epoch);
    return check_launch();
}

extern "C" int kivi_peer_merge(const uint64_t* peer_bufs, int W, int rows, int D, const unsigned int* epoch,
                               const void* my_buf, void* out, int* err, long long timeout_ns,
                               kivi_stream_t stream) {
    if (rows <= 0 || D <= 0 || D % 4 || W <= 0 || W > peer::MAX_W || timeout_ns <= 0) return KIVI_ERR_ARG;
    if (!peer_bufs || !epoch || !my_buf || !out) return KIVI_ERR_ARG;
    peer::merge_kernel<<<rows, 128, 0, (cudaStream_t)stream>>>(peer_bufs, W, rows, D, epoch,
                                                               static_cast<const uint8_t*>(my_buf),
                                                               reinterpret_cast<__nv_bfloat16*>(out), err,
                                                               timeout_ns);
    return check_launch();
}

// ---------------------------------------------------------------------------
// Exchange-buffer management (CUDA IPC).
// ---------------------------------------------------------------------------
extern "C" int kivi_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
    if (bytes <= 0 || !ptr || !ipc_handle) return KIVI_ERR_ARG;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e != cudaSuccess) return record_cuda_error(e);
    e = cudaMemset(p, 0, (size_t)bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) { cudaFree(p); return record_cuda_error(e); }
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return KIVI_OK;
}

extern "C" int kivi_peer_open(const void* ipc_handle, void** ptr) {
    if (!ipc_handle || !ptr) return KIVI_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? KIVI_OK : record_cuda_error(e);
}

extern "C" int kivi_peer_close(void* ptr) {
    if (!ptr) return KIVI_ERR_ARG;
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? KIVI_OK : record_cuda_error(e);
}

extern "C" int kivi_peer_free(void* ptr) {
    if (!ptr) return KIVI_ERR_ARG;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? KIVI_OK : record_cuda_error(e);
}
