// kivi_quant.cu -- quantize-and-store, dequant, roundtrip and calibrate kernels.
//
// One thread owns one 16-element quant block end to end (load, calibrate,
// quantise, pack, store).  Block geometry follows the reference
// (int4_kivi/triton_kernels.py:137-286):
//   K  'channel': block = 16 tokens of one channel (one page), threads of a
//       warp take consecutive channels, so every token row is a coalesced
//       64-byte read;
//   V  'headdim': block = 16 contiguous channels of one token (32 bytes).
// The calibration arithmetic lives in kivi_common.cuh and is bit-exact with
// kv_quant.py on CPU.
#include "kivi_common.cuh"
#include "kivi_internal.h"

namespace kivi {

template <typename T>
__device__ __forceinline__ void load_strided16(const T* __restrict__ p, int64_t stride, float x[BLK]) {
#pragma unroll
    for (int i = 0; i < BLK; ++i) x[i] = to_f32<T>(p[i * stride]);
}

template <typename T>
__device__ __forceinline__ void load_contig16(const T* __restrict__ p, int64_t stride, float x[BLK]) {
    if (stride == 1 && sizeof(T) == 2 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const uint4* p4 = reinterpret_cast<const uint4*>(p);
        uint4 a = __ldg(p4), b = __ldg(p4 + 1);
        const T* ta = reinterpret_cast<const T*>(&a);
        const T* tb = reinterpret_cast<const T*>(&b);
#pragma unroll
        for (int i = 0; i < 8; ++i) { x[i] = to_f32<T>(ta[i]); x[i + 8] = to_f32<T>(tb[i]); }
    } else {
        load_strided16<T>(p, stride, x);
    }
}

// Quantise one block into 8 packed bytes; returns the stored scale bits.
template <int FMT>
__device__ __forceinline__ void quant_pack(const float x[BLK], int calib, const float* alphas,
                                           int n_alphas, float g, uint2& packed, uint16_t& sbits) {
    uint32_t lo = 0, hi = 0;
    if (FMT == FMT_NVFP4) {
        uint8_t sc;
        float sd = nvfp4_calibrate16(x, calib, alphas, n_alphas, g, &sc);
#pragma unroll
        for (int i = 0; i < BLK; ++i) {
            uint32_t nib = 0;
            if (sd != 0.0f) {
                float y = __fdiv_rn(x[i], sd);
                nib = (uint32_t)e2m1_index(fabsf(y)) | (y < 0.0f ? 8u : 0u);
            }
            if (i < 8) lo |= nib << (4 * i); else hi |= nib << (4 * (i - 8));
        }
        sbits = sc;
    } else {
        float s = calibrate16(x, FMT, calib, alphas, n_alphas);
#pragma unroll
        for (int i = 0; i < BLK; ++i) {
            int c = (int)q_grid(__fdiv_rn(x[i], s), FMT);
            uint32_t nib = (uint32_t)c & 0xF;
            if (i < 8) lo |= nib << (4 * i); else hi |= nib << (4 * (i - 8));
        }
        sbits = __half_as_ushort(__float2half_rn(s));
    }
    packed = make_uint2(lo, hi);
}

// grid-stride over K blocks (h, p, d) then V blocks (h, t, db).
template <typename T, int FMT>
__global__ void __launch_bounds__(256) store_kernel(StoreArgs a) {
    const T* k = reinterpret_cast<const T*>(a.k);
    const T* v = reinterpret_cast<const T*>(a.v);
    const int NP = a.S_k / BLK, ND = a.D / BLK;
    const int64_t nk = (int64_t)a.H * NP * a.D;
    const int64_t nv = (int64_t)a.H * a.S_v * ND;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nk + nv;
         i += (int64_t)gridDim.x * blockDim.x) {
        float x[BLK];
        uint2 pk;
        uint16_t sb;
        if (i < nk) {
            const int d = (int)(i % a.D);
            const int64_t r = i / a.D;
            const int p = (int)(r % NP), h = (int)(r / NP);
            load_strided16<T>(k + h * a.sk_h + (int64_t)p * BLK * a.sk_s + d * a.sk_d, a.sk_s, x);
            quant_pack<FMT>(x, a.calib_k, a.alphas, a.n_alphas, a.g_k, pk, sb);
            const int64_t row = ((int64_t)h * a.D + d) * a.k_np_stride + a.kpage0 + p;
            reinterpret_cast<uint2*>(a.k_packed)[row] = pk;
            if (FMT == FMT_NVFP4) reinterpret_cast<uint8_t*>(a.k_scale)[row] = (uint8_t)sb;
            else reinterpret_cast<uint16_t*>(a.k_scale)[row] = sb;
        } else {
            const int64_t j = i - nk;
            const int db = (int)(j % ND);
            const int64_t r = j / ND;
            const int t = (int)(r % a.S_v), h = (int)(r / a.S_v);
            load_contig16<T>(v + h * a.sv_h + t * a.sv_s + (int64_t)db * BLK * a.sv_d, a.sv_d, x);
            quant_pack<FMT>(x, a.calib_v, a.alphas, a.n_alphas, a.g_v, pk, sb);
            const int64_t row = ((int64_t)h * a.v_s_stride + a.vtok0 + t) * ND + db;
            reinterpret_cast<uint2*>(a.v_packed)[row] = pk;
            if (FMT == FMT_NVFP4) reinterpret_cast<uint8_t*>(a.v_scale)[row] = (uint8_t)sb;
            else reinterpret_cast<uint16_t*>(a.v_scale)[row] = sb;
        }
    }
}

__device__ __forceinline__ float nib_value(uint32_t nib, int fmt) {
    if (fmt == FMT_NVFP4) {
        float l = e2m1_level(nib & 7);
        return (nib & 8) ? -l : l;
    }
    return (float)sx4((int)nib);
}

template <int FMT>
__device__ __forceinline__ float load_scale(const void* s, int64_t idx, float g) {
    if (FMT == FMT_NVFP4) return __fmul_rn(e4m3_to_f32(reinterpret_cast<const uint8_t*>(s)[idx]), g);
    return __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(s)[idx]));
}

template <int FMT>
__global__ void __launch_bounds__(256) dequant_kernel(DequantArgs a) {
    const int NP = a.S / BLK, ND = a.D / BLK;
    const int64_t nk = (int64_t)a.H * NP * a.D;
    const int64_t nv = (int64_t)a.H * a.S * ND;
    __nv_bfloat16* ko = reinterpret_cast<__nv_bfloat16*>(a.k_out);
    __nv_bfloat16* vo = reinterpret_cast<__nv_bfloat16*>(a.v_out);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nk + nv;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nk) {
            const int d = (int)(i % a.D);
            const int64_t r = i / a.D;
            const int p = (int)(r % NP), h = (int)(r / NP);
            const int64_t row = ((int64_t)h * a.D + d) * a.k_np_stride + p;
            const uint2 pk = reinterpret_cast<const uint2*>(a.k_packed)[row];
            const float s = load_scale<FMT>(a.k_scale, row, a.g_k);
            __nv_bfloat16* o = ko + h * a.so_h + (int64_t)p * BLK * a.so_s + d * a.so_d;
#pragma unroll
            for (int j = 0; j < BLK; ++j) {
                uint32_t nib = ((j < 8 ? pk.x : pk.y) >> (4 * (j & 7))) & 0xF;
                o[j * a.so_s] = __float2bfloat16_rn(__fmul_rn(nib_value(nib, FMT), s));
            }
        } else {
            const int64_t jj = i - nk;
            const int db = (int)(jj % ND);
            const int64_t r = jj / ND;
            const int t = (int)(r % a.S), h = (int)(r / a.S);
            const int64_t row = ((int64_t)h * a.v_s_stride + t) * ND + db;
            const uint2 pk = reinterpret_cast<const uint2*>(a.v_packed)[row];
            const float s = load_scale<FMT>(a.v_scale, row, a.g_v);
            __nv_bfloat16* o = vo + h * a.so_h + t * a.so_s + (int64_t)db * BLK * a.so_d;
#pragma unroll
            for (int c = 0; c < BLK; ++c) {
                uint32_t nib = ((c < 8 ? pk.x : pk.y) >> (4 * (c & 7))) & 0xF;
                o[c * a.so_d] = __float2bfloat16_rn(__fmul_rn(nib_value(nib, FMT), s));
            }
        }
    }
}

// kv_quant.roundtrip: one thread per block of the chosen layout.
template <typename T>
__global__ void __launch_bounds__(256) roundtrip_kernel(RoundtripArgs a) {
    const T* x = reinterpret_cast<const T*>(a.x);
    T* y = reinterpret_cast<T*>(a.y);
    const int S = a.S, D = a.D, ND = D / BLK, n_full = (S / BLK) * BLK, NP = n_full / BLK;
    const int64_t nblk = (a.layout == 0) ? (int64_t)a.H * S * ND : (int64_t)a.H * NP * D;
    const int64_t ntail = (a.layout == 1) ? (int64_t)a.H * (S - n_full) * D : 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nblk + ntail;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i >= nblk) {   // 'channel' hot tail: copied unchanged
            const int64_t j = i - nblk;
            const int d = (int)(j % D);
            const int64_t r = j / D;
            const int t = n_full + (int)(r % (S - n_full)), h = (int)(r / (S - n_full));
            const int64_t o = ((int64_t)h * S + t) * D + d;
            y[o] = x[o];
            continue;
        }
        float v[BLK];
        int64_t base, stride;
        if (a.layout == 0) {
            const int db = (int)(i % ND);
            const int64_t r = i / ND;        // h*S + t
            base = r * D + (int64_t)db * BLK;
            stride = 1;
            load_contig16<T>(x + base, 1, v);
        } else {
            const int d = (int)(i % D);
            const int64_t r = i / D;
            const int p = (int)(r % NP), h = (int)(r / NP);
            base = ((int64_t)h * S + (int64_t)p * BLK) * D + d;
            stride = D;
            load_strided16<T>(x + base, D, v);
        }
        const float s = calibrate16(v, a.fmt, a.calib, a.alphas, a.n_alphas);
#pragma unroll
        for (int j = 0; j < BLK; ++j)
            y[base + j * stride] = from_f32<T>(__fmul_rn(q_grid(__fdiv_rn(v[j], s), a.fmt), s));
    }
}

__global__ void __launch_bounds__(256) calibrate_kernel(const float* __restrict__ blocks, int64_t n,
                                                        int fmt, int calib, const float* alphas,
                                                        int n_alphas, float* scales) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float v[BLK];
        load_contig16<float>(blocks + i * BLK, 1, v);
        scales[i] = calibrate16(v, fmt, calib, alphas, n_alphas);
    }
}

static int grid_for(int64_t n) {
    int64_t g = (n + 255) / 256;
    const int64_t cap = 148LL * 16;   // grid-stride beyond 16 CTAs per SM
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace kivi

using namespace kivi;

extern "C" int kivi_store(const void* k, const void* v, int in_dtype, int64_t sk_h, int64_t sk_s,
                          int64_t sk_d, int64_t sv_h, int64_t sv_s, int64_t sv_d, int H, int S_k,
                          int S_v, int D, int fmt, int calib_k, int calib_v, const float* alphas,
                          int n_alphas, float g_k, float g_v, uint8_t* k_packed, void* k_scale,
                          int kpage0, int k_np_stride, uint8_t* v_packed, void* v_scale, int vtok0,
                          int v_s_stride, kivi_stream_t stream) {
    if (H < 0 || S_k < 0 || S_v < 0 || D <= 0 || D % BLK) return KIVI_ERR_ARG;
    if (fmt != FMT_INT4 && fmt != FMT_NVFP4) return KIVI_ERR_ARG;
    if ((unsigned)calib_k > 1 || (unsigned)calib_v > 1) return KIVI_ERR_ARG;
    if ((calib_k == CAL_MSE || calib_v == CAL_MSE) && (!alphas || n_alphas <= 0)) return KIVI_ERR_ARG;
    if (in_dtype != KIVI_DT_BF16 && in_dtype != KIVI_DT_F16) return KIVI_ERR_ARG;
    if (fmt == FMT_NVFP4 && !(g_k > 0.0f && g_v > 0.0f)) return KIVI_ERR_ARG;
    const int NP = S_k / BLK;
    if (NP > 0 && (kpage0 < 0 || k_np_stride < kpage0 + NP)) return KIVI_ERR_ARG;
    if (S_v > 0 && (vtok0 < 0 || v_s_stride < vtok0 + S_v)) return KIVI_ERR_ARG;
    if ((uintptr_t)k_packed % 8 || (uintptr_t)v_packed % 8) return KIVI_ERR_ALIGN;
    const int64_t n = (int64_t)H * NP * D + (int64_t)H * S_v * (D / BLK);
    if (n == 0) return KIVI_OK;
    if (NP > 0 && (!k || !k_packed || !k_scale)) return KIVI_ERR_ARG;
    if (S_v > 0 && (!v || !v_packed || !v_scale)) return KIVI_ERR_ARG;
    StoreArgs a{k, v, sk_h, sk_s, sk_d, sv_h, sv_s, sv_d, H, S_k, S_v, D, calib_k, calib_v, alphas,
                n_alphas, g_k, g_v, k_packed, k_scale, kpage0, k_np_stride, v_packed, v_scale,
                vtok0, v_s_stride};
    cudaStream_t st = (cudaStream_t)stream;
    const int g = grid_for(n);
    if (in_dtype == KIVI_DT_BF16) {
        if (fmt == FMT_INT4) store_kernel<__nv_bfloat16, FMT_INT4><<<g, 256, 0, st>>>(a);
        else store_kernel<__nv_bfloat16, FMT_NVFP4><<<g, 256, 0, st>>>(a);
    } else {
        if (fmt == FMT_INT4) store_kernel<__half, FMT_INT4><<<g, 256, 0, st>>>(a);
        else store_kernel<__half, FMT_NVFP4><<<g, 256, 0, st>>>(a);
    }
    return check_launch();
}

extern "C" int kivi_dequant(const uint8_t* k_packed, const void* k_scale, int k_np_stride,
                            const uint8_t* v_packed, const void* v_scale, int v_s_stride, int H,
                            int S, int D, int fmt, float g_k, float g_v, void* k_out, void* v_out,
                            int64_t so_h, int64_t so_s, int64_t so_d, kivi_stream_t stream) {
    if (H < 0 || S < 0 || D <= 0 || D % BLK) return KIVI_ERR_ARG;
    if (fmt != FMT_INT4 && fmt != FMT_NVFP4) return KIVI_ERR_ARG;
    if (k_np_stride < S / BLK || v_s_stride < S) return KIVI_ERR_ARG;
    if ((uintptr_t)k_packed % 8 || (uintptr_t)v_packed % 8) return KIVI_ERR_ALIGN;
    const int64_t n = (int64_t)H * (S / BLK) * D + (int64_t)H * S * (D / BLK);
    if (n == 0) return KIVI_OK;
    DequantArgs a{k_packed, k_scale, k_np_stride, v_packed, v_scale, v_s_stride, H, S, D,
                  g_k, g_v, k_out, v_out, so_h, so_s, so_d};
    cudaStream_t st = (cudaStream_t)stream;
    if (fmt == FMT_INT4) dequant_kernel<FMT_INT4><<<grid_for(n), 256, 0, st>>>(a);
    else dequant_kernel<FMT_NVFP4><<<grid_for(n), 256, 0, st>>>(a);
    return check_launch();
}

extern "C" int kivi_roundtrip(const void* x, void* y, int dtype, int H, int S, int D, int fmt,
                              int layout, int calib, const float* alphas, int n_alphas,
                              kivi_stream_t stream) {
    if (H < 0 || S < 0 || D <= 0 || D % BLK) return KIVI_ERR_ARG;
    if ((unsigned)fmt > 2 || (unsigned)layout > 1 || (unsigned)calib > 1) return KIVI_ERR_ARG;
    if (calib == CAL_MSE && (!alphas || n_alphas <= 0)) return KIVI_ERR_ARG;
    const int n_full = (S / BLK) * BLK;
    const int64_t n = layout == 0 ? (int64_t)H * S * (D / BLK)
                                  : (int64_t)H * (n_full / BLK) * D + (int64_t)H * (S - n_full) * D;
    if (n == 0) return KIVI_OK;
    RoundtripArgs a{x, y, H, S, D, fmt, layout, calib, alphas, n_alphas};
    cudaStream_t st = (cudaStream_t)stream;
    const int g = grid_for(n);
    switch (dtype) {
        case KIVI_DT_BF16: roundtrip_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(a); break;
        case KIVI_DT_F16: roundtrip_kernel<__half><<<g, 256, 0, st>>>(a); break;
        case KIVI_DT_F32: roundtrip_kernel<float><<<g, 256, 0, st>>>(a); break;
        default: return KIVI_ERR_ARG;
    }
    return check_launch();
}

extern "C" int kivi_calibrate(const float* blocks, int64_t n, int fmt, int calib,
                              const float* alphas, int n_alphas, float* scales,
                              kivi_stream_t stream) {
    if (n < 0 || (unsigned)fmt > 2 || (unsigned)calib > 1) return KIVI_ERR_ARG;
    if (calib == CAL_MSE && (!alphas || n_alphas <= 0)) return KIVI_ERR_ARG;
    if (n == 0) return KIVI_OK;
    calibrate_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(blocks, n, fmt, calib, alphas,
                                                                    n_alphas, scales);
    return check_launch();
}
