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

// The two 16-bit values of a 32-bit word (element 2i in the low half) as fp32.
template <typename T> __device__ __forceinline__ float lo16_f32(uint32_t w);
template <typename T> __device__ __forceinline__ float hi16_f32(uint32_t w);
template <> __device__ __forceinline__ float lo16_f32<__nv_bfloat16>(uint32_t w) { return __uint_as_float(w << 16); }
template <> __device__ __forceinline__ float hi16_f32<__nv_bfloat16>(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
template <> __device__ __forceinline__ float lo16_f32<__half>(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
template <> __device__ __forceinline__ float hi16_f32<__half>(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
template <> __device__ __forceinline__ float lo16_f32<float>(uint32_t) { return 0.f; }
template <> __device__ __forceinline__ float hi16_f32<float>(uint32_t) { return 0.f; }

// Quantise one block into 8 packed bytes; returns the stored scale bits.
template <int FMT>
__device__ __forceinline__ void quant_pack(const float x[BLK], int calib, const float* alphas,
                                           int n_alphas, float g, uint2& packed, uint16_t& sbits) {
    uint32_t lo = 0, hi = 0;
    if (FMT == FMT_NVFP4) {
        uint8_t sc;
        float sd = nvfp4_calibrate16(x, calib, alphas, n_alphas, g, &sc);
        const float r = __frcp_rn(sd);
#pragma unroll
        for (int i = 0; i < BLK; ++i) {
            uint32_t nib = 0;
            if (sd != 0.0f) {
                float y = quot_for_grid(x[i], sd, r, FMT_NVFP4);
                nib = (uint32_t)e2m1_index(fabsf(y)) | (y < 0.0f ? 8u : 0u);
            }
            if (i < 8) lo |= nib << (4 * i); else hi |= nib << (4 * (i - 8));
        }
        sbits = sc;
    } else {
        float s = calibrate16(x, FMT, calib, alphas, n_alphas);
        const float r = __frcp_rn(s);
        if (FMT == FMT_INT4 && calib == CAL_ABSMAX) {
            // s = absmax / 7, so |x / s| <= 7 (1 + 2^-23): rint never leaves
            // [-7, 7] (no clamp), and y = x * r is within 2.2e-6 of the IEEE
            // quotient, so only |frac| within 1e-5 of one half needs the
            // exact division to round like kv_quant.
            // Adding 1.5 * 2^23 rounds y to the nearest integer (ties to
            // even, like rint) and leaves it, two's complement, in the low
            // mantissa bits, so its nibble is inserted with one bit-field op.
            constexpr float MAGIC = 12582912.0f;
#pragma unroll
            for (int i = 0; i < BLK; ++i) {
                const float y = __fmul_rn(x[i], r);
                float t = __fadd_rn(y, MAGIC);
                if (fabsf(__fsub_rn(y, __fsub_rn(t, MAGIC))) > 0.5f - 1e-5f)
                    t = __fadd_rn(__fdiv_rn(x[i], s), MAGIC);
                uint32_t& w = i < 8 ? lo : hi;
                const uint32_t pos = 4 * (i & 7);
                asm("bfi.b32 %0, %1, %0, %2, 4;" : "+r"(w) : "r"(__float_as_uint(t)), "r"(pos));
            }
        } else {
#pragma unroll
            for (int i = 0; i < BLK; ++i) {
                int c = (int)q_grid_div(x[i], s, r, FMT);
                uint32_t nib = (uint32_t)c & 0xF;
                if (i < 8) lo |= nib << (4 * i); else hi |= nib << (4 * (i - 8));
            }
        }
        sbits = __half_as_ushort(__float2half_rn(s));
    }
    packed = make_uint2(lo, hi);
}

// One V block of the mixed cache: INT3 codes against the fp32 scale (scale
// stored as fp16, like every KIVI scale).
__device__ __forceinline__ void quant_v3(const float x[BLK], int calib, const float* alphas, int n_alphas,
                                         int c[BLK], uint16_t& sbits) {
    const float s = calibrate16(x, FMT_INT3, calib, alphas, n_alphas);
    const float r = __frcp_rn(s);
    if (calib == CAL_ABSMAX) {
        // s = absmax / 3: |x / s| <= 3 (1 + 2^-23), so rint stays in [-3, 3]
        // without a clamp; rounding by the 1.5 * 2^23 magic number (ties to
        // even, like rint) leaves the code two's complement in the low
        // mantissa bits (the same near-half fallback as the INT4 store)
        constexpr float MAGIC = 12582912.0f;
#pragma unroll
        for (int i = 0; i < BLK; ++i) {
            const float y = __fmul_rn(x[i], r);
            float t = __fadd_rn(y, MAGIC);
            if (fabsf(__fsub_rn(y, __fsub_rn(t, MAGIC))) > 0.5f - 1e-5f) t = __fadd_rn(__fdiv_rn(x[i], s), MAGIC);
            c[i] = (int)(__float_as_uint(t) << 29) >> 29;        // sign-extend the low 3 bits
        }
    } else {
#pragma unroll
        for (int i = 0; i < BLK; ++i) c[i] = (int)q_grid_div(x[i], s, r, FMT_INT3);
    }
    sbits = __half_as_ushort(__float2half_rn(s));
}

// K blocks (per channel, 16-token pages): a CTA owns PPC pages x D channels
// of one head.  Threads take consecutive channels, so each of a block's 16
// token loads is a contiguous row segment across the warp; the packed
// results go through shared memory and are written back grouped by channel,
// where consecutive pages are contiguous in k_packed / k_scale (a direct
// write would put neighbouring lanes k_np_stride pages apart).
// V blocks (16 channels of one token) are contiguous in the input and in the
// output, so V CTAs take one block per thread directly.
// Grid: [0, nk_ctas) K chunks (head-major), then V CTAs (grid-stride).
template <typename T, int FMT, bool ANY_MSE>
__global__ void __launch_bounds__(256) store_kernel(StoreArgs a, int ppc, int n_chunks, int nk_ctas) {
    extern __shared__ __align__(16) uint8_t st_smem[];
    constexpr int KF = FMT == FMT_MIX43 ? FMT_INT4 : FMT;    // K format
    const T* k = reinterpret_cast<const T*>(a.k);
    const T* v = reinterpret_cast<const T*>(a.v);
    const int D = a.D, ND = D / BLK, tid = threadIdx.x;
    if ((int)blockIdx.x < nk_ctas) {
        const int NP = a.S_k / BLK;
        const int h = blockIdx.x / n_chunks, p0 = (blockIdx.x % n_chunks) * ppc;
        const int np_here = min(ppc, NP - p0);
        uint2* sc = reinterpret_cast<uint2*>(st_smem);                              // [ppc][D+1]
        uint16_t* ss = reinterpret_cast<uint16_t*>(sc + (size_t)ppc * (D + 1));     // [ppc][D+2]
        const T* src = k + h * a.sk_h + (int64_t)p0 * BLK * a.sk_s;
        const int calib = ANY_MSE ? a.calib_k : (int)CAL_ABSMAX;
        if (!ANY_MSE && sizeof(T) == 2 && a.sk_d == 1 && a.sk_s % 2 == 0 &&
            (reinterpret_cast<uintptr_t>(src) & 3) == 0) {
            // absmax: a thread takes a channel pair, so each token load is one
            // 32-bit word (a 128-byte row segment across the warp) feeding two
            // blocks (the MSE search is ALU-bound and keeps one block per thread)
            const int npair = D / 2;
            for (int b = tid; b < np_here * npair; b += 256) {
                const int p = b / npair, c = 2 * (b - p * npair);
                uint32_t raw[BLK];
#pragma unroll
                for (int j = 0; j < BLK; ++j)
                    raw[j] = __ldg(reinterpret_cast<const uint32_t*>(src + ((int64_t)p * BLK + j) * a.sk_s + c));
                float x[BLK];
                uint2 pk;
                uint16_t sb;
#pragma unroll
                for (int j = 0; j < BLK; ++j) x[j] = lo16_f32<T>(raw[j]);
                quant_pack<KF>(x, calib, a.alphas, a.n_alphas, a.g_k, pk, sb);
                sc[p * (D + 1) + c] = pk;
                ss[p * (D + 2) + c] = sb;
#pragma unroll
                for (int j = 0; j < BLK; ++j) x[j] = hi16_f32<T>(raw[j]);
                quant_pack<KF>(x, calib, a.alphas, a.n_alphas, a.g_k, pk, sb);
                sc[p * (D + 1) + c + 1] = pk;
                ss[p * (D + 2) + c + 1] = sb;
            }
        } else {
            for (int b = tid; b < np_here * D; b += 256) {
                const int p = b / D, c = b - p * D;
                float x[BLK];
                load_strided16<T>(src + (int64_t)p * BLK * a.sk_s + c * a.sk_d, a.sk_s, x);
                uint2 pk;
                uint16_t sb;
                quant_pack<KF>(x, calib, a.alphas, a.n_alphas, a.g_k, pk, sb);
                sc[p * (D + 1) + c] = pk;
                ss[p * (D + 2) + c] = sb;
            }
        }
        __syncthreads();
        for (int b = tid; b < np_here * D; b += 256) {
            const int c = b / np_here, p = b - c * np_here;
            const int64_t row = ((int64_t)h * D + c) * a.k_np_stride + a.kpage0 + p0 + p;
            reinterpret_cast<uint2*>(a.k_packed)[row] = sc[p * (D + 1) + c];
            if (FMT == FMT_NVFP4) reinterpret_cast<uint8_t*>(a.k_scale)[row] = (uint8_t)ss[p * (D + 2) + c];
            else reinterpret_cast<uint16_t*>(a.k_scale)[row] = ss[p * (D + 2) + c];
        }
        return;
    }
    const int64_t nv = (int64_t)a.H * a.S_v * ND;
    const int nv_ctas = gridDim.x - nk_ctas;
    const int calib_v = ANY_MSE ? a.calib_v : (int)CAL_ABSMAX;
    if constexpr (FMT == FMT_MIX43) {
        // INT3 V: a thread takes a block pair (they share a sign word)
        for (int64_t j = (int64_t)(blockIdx.x - nk_ctas) * 256 + tid; j < nv / 2; j += (int64_t)nv_ctas * 256) {
            const int db = (int)(2 * j % ND);
            const int64_t r = 2 * j / ND;
            const int t = (int)(r % a.S_v), h = (int)(r / a.S_v);
            float x[BLK];
            int c0[BLK], c1[BLK];
            uint16_t s0, s1;
            load_contig16<T>(v + h * a.sv_h + t * a.sv_s + (int64_t)db * BLK * a.sv_d, a.sv_d, x);
            quant_v3(x, calib_v, a.alphas, a.n_alphas, c0, s0);
            load_contig16<T>(v + h * a.sv_h + t * a.sv_s + (int64_t)(db + 1) * BLK * a.sv_d, a.sv_d, x);
            quant_v3(x, calib_v, a.alphas, a.n_alphas, c1, s1);
            const int64_t row = ((int64_t)h * a.v_s_stride + a.vtok0 + t) * ND + db;
            uint32_t A0, A1, S;
            int3_pack_pair(c0, c1, A0, A1, S);
            uint32_t* o = reinterpret_cast<uint32_t*>(a.v_packed + row * PACKB3);
            o[0] = A0; o[1] = A1; o[2] = S;
            reinterpret_cast<uint16_t*>(a.v_scale)[row] = s0;
            reinterpret_cast<uint16_t*>(a.v_scale)[row + 1] = s1;
        }
        return;
    }
    if (FMT != FMT_MIX43 && !ANY_MSE && sizeof(T) == 2 && a.sv_d == 1 && ND % 2 == 0 && (a.sv_s * 2) % 16 == 0 &&
        (a.sv_h * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0) {
        // absmax: a thread takes two neighbouring blocks of one token, 64
        // contiguous bytes in four 16-byte loads all in flight before either
        // is used
        const int64_t npairs = nv / 2;
        for (int64_t q = (int64_t)(blockIdx.x - nk_ctas) * 256 + tid; q < npairs; q += (int64_t)nv_ctas * 256) {
            const int db = (int)(2 * q % ND);
            const int64_t r = 2 * q / ND;
            const int t = (int)(r % a.S_v), h = (int)(r / a.S_v);
            const uint4* src = reinterpret_cast<const uint4*>(v + h * a.sv_h + t * a.sv_s + (int64_t)db * BLK);
            const uint4 r0 = __ldg(src), r1 = __ldg(src + 1), r2 = __ldg(src + 2), r3 = __ldg(src + 3);
            const int64_t row = ((int64_t)h * a.v_s_stride + a.vtok0 + t) * ND + db;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint4 u0 = half ? r2 : r0, u1 = half ? r3 : r1;
                const uint32_t wds[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                float x[BLK];
#pragma unroll
                for (int e = 0; e < 8; ++e) { x[2 * e] = lo16_f32<T>(wds[e]); x[2 * e + 1] = hi16_f32<T>(wds[e]); }
                uint2 pk;
                uint16_t sb;
                quant_pack<FMT>(x, calib_v, a.alphas, a.n_alphas, a.g_v, pk, sb);
                reinterpret_cast<uint2*>(a.v_packed)[row + half] = pk;
                if (FMT == FMT_NVFP4) reinterpret_cast<uint8_t*>(a.v_scale)[row + half] = (uint8_t)sb;
                else reinterpret_cast<uint16_t*>(a.v_scale)[row + half] = sb;
            }
        }
        return;
    }
    for (int64_t j = (int64_t)(blockIdx.x - nk_ctas) * 256 + tid; j < nv; j += (int64_t)nv_ctas * 256) {
        const int db = (int)(j % ND);
        const int64_t r = j / ND;
        const int t = (int)(r % a.S_v), h = (int)(r / a.S_v);
        float x[BLK];
        uint2 pk;
        uint16_t sb;
        load_contig16<T>(v + h * a.sv_h + t * a.sv_s + (int64_t)db * BLK * a.sv_d, a.sv_d, x);
        const int64_t row = ((int64_t)h * a.v_s_stride + a.vtok0 + t) * ND + db;
        quant_pack<FMT>(x, calib_v, a.alphas, a.n_alphas, a.g_v, pk, sb);
        reinterpret_cast<uint2*>(a.v_packed)[row] = pk;
        if (FMT == FMT_NVFP4) reinterpret_cast<uint8_t*>(a.v_scale)[row] = (uint8_t)sb;
        else reinterpret_cast<uint16_t*>(a.v_scale)[row] = sb;
    }
}

// Small MSE stores (the per-step append): one warp per block, the clip ratios
// of the search spread over the lanes (lane a evaluates ratio a, a + 32, ...)
// and the first-index argmin found with shuffles, so a few blocks do not
// leave one thread running the whole 32-ratio search.  Same arithmetic per
// ratio as calibrate16 / nvfp4_calibrate16 and the same tie rule (the first
// ratio with the smallest error; no finite error gives scale 0).
template <typename T, int FMT>
__global__ void __launch_bounds__(256) store_warp_kernel(StoreArgs a) {
    const T* k = reinterpret_cast<const T*>(a.k);
    const T* v = reinterpret_cast<const T*>(a.v);
    const int D = a.D, ND = D / BLK, NP = a.S_k / BLK;
    const int lane = threadIdx.x & 31;
    const int64_t nk = (int64_t)a.H * NP * D, nv = (int64_t)a.H * a.S_v * ND;
    const int64_t wid = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t i = wid; i < nk + nv; i += nwarps) {
        const bool isk = i < nk;
        float x[BLK];
        int calib;
        float g;
        int64_t row;
        if (isk) {
            const int d = (int)(i % D);
            const int64_t r = i / D;
            const int p = (int)(r % NP), h = (int)(r / NP);
            load_strided16<T>(k + h * a.sk_h + (int64_t)p * BLK * a.sk_s + d * a.sk_d, a.sk_s, x);
            calib = a.calib_k; g = a.g_k;
            row = ((int64_t)h * D + d) * a.k_np_stride + a.kpage0 + p;
        } else {
            const int64_t j = i - nk;
            const int db = (int)(j % ND);
            const int64_t r = j / ND;
            const int t = (int)(r % a.S_v), h = (int)(r / a.S_v);
            load_contig16<T>(v + h * a.sv_h + t * a.sv_s + (int64_t)db * BLK * a.sv_d, a.sv_d, x);
            calib = a.calib_v; g = a.g_v;
            row = ((int64_t)h * a.v_s_stride + a.vtok0 + t) * ND + db;
        }
        const float amax = absmax16(x);
        const float qmax = FMT == FMT_NVFP4 ? 6.0f : 7.0f;
        // this lane's best ratio: (error, ratio index, scale, e4m3 byte)
        float best = __int_as_float(0x7f800000), bs = 0.0f;
        int bi = 0x7fffffff;
        uint32_t bsc = 0;
        // INT4 absmax takes amax / 7 as is; NVFP4 absmax checks its one
        // candidate's error (finite, else scale 0) with 16 lanes; MSE searches
        // the clip ratios, one per lane
        const int nA = calib == CAL_ABSMAX ? 1 : a.n_alphas;
        float xl = x[0];                                 // my element (lanes 0..15)
#pragma unroll
        for (int e = 1; e < BLK; ++e) xl = lane == e ? x[e] : xl;
        if (FMT == FMT_NVFP4 && calib == CAL_ABSMAX) {
            // one candidate: lanes 0..15 take one element's squared error each,
            // then every lane sums the 16 in kv_quant's mean order
            const uint32_t sc = f32_to_e4m3(__fdiv_rn(__fdiv_rn(amax, qmax), g));
            const float s = __fmul_rn(e4m3_to_f32((uint8_t)sc), g);
            float ei = 0.f;
            if (lane < BLK) {
                const float q = (s == 0.0f) ? 0.0f : q_grid_div(xl, s, __frcp_rn(s), FMT_NVFP4);
                const float d = __fsub_rn(xl, __fmul_rn(q, s));
                ei = __fmul_rn(d, d);
            }
            float ev[BLK];
#pragma unroll
            for (int e = 0; e < BLK; ++e) ev[e] = __shfl_sync(0xffffffffu, ei, e);
            const float err = mean16(ev);
            if (err < best) { best = err; bs = s; bi = 0; bsc = sc; }
        }
        for (int al = lane; al < nA && calib != CAL_ABSMAX; al += 32) {
            float s = calib == CAL_ABSMAX ? __fdiv_rn(amax, qmax) : __fdiv_rn(__fmul_rn(a.alphas[al], amax), qmax);
            uint32_t sc = 0;
            if (FMT == FMT_NVFP4) {
                sc = f32_to_e4m3(__fdiv_rn(s, g));
                s = __fmul_rn(e4m3_to_f32((uint8_t)sc), g);
            }
            const float err = block_err(x, s, FMT);
            if (err < best) { best = err; bs = s; bi = al; bsc = sc; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const float os = __shfl_xor_sync(0xffffffffu, bs, o);
            const uint32_t oc = __shfl_xor_sync(0xffffffffu, bsc, o);
            if (ob < best || (ob == best && oi < bi)) { best = ob; bi = oi; bs = os; bsc = oc; }
        }
        if (!(best < __int_as_float(0x7f800000))) { bs = 0.0f; bsc = 0; }   // no finite error
        if (FMT != FMT_NVFP4 && calib == CAL_ABSMAX) bs = __fdiv_rn(amax, qmax);
        // lanes 0..15 quantise one element each; the nibbles are OR-reduced
        uint32_t nib = 0;
        if (lane < BLK) {
            if (FMT == FMT_NVFP4) {
                if (bs != 0.0f) {
                    const float y = quot_for_grid(xl, bs, __frcp_rn(bs), FMT_NVFP4);
                    nib = (uint32_t)e2m1_index(fabsf(y)) | (y < 0.0f ? 8u : 0u);
                }
            } else {
                nib = (uint32_t)(int)q_grid_div(xl, bs, __frcp_rn(bs), FMT) & 0xFu;
            }
        }
        const uint32_t lo = __reduce_or_sync(0xffffffffu, lane < 8 ? nib << (4 * lane) : 0u);
        const uint32_t hi = __reduce_or_sync(0xffffffffu, (lane >= 8 && lane < BLK) ? nib << (4 * (lane - 8)) : 0u);
        if (lane == 0) {
            uint8_t* pk = isk ? a.k_packed : a.v_packed;
            void* sp = isk ? a.k_scale : a.v_scale;
            reinterpret_cast<uint2*>(pk)[row] = make_uint2(lo, hi);
            if (FMT == FMT_NVFP4) reinterpret_cast<uint8_t*>(sp)[row] = (uint8_t)bsc;
            else reinterpret_cast<uint16_t*>(sp)[row] = __half_as_ushort(__float2half_rn(bs));
        }
    }
}

// Pages per K chunk: 16 (a 32-byte run of fp16 scales per channel), fewer
// for wide heads so the staged output stays within 40 KB of shared memory
// (under the 48 KB a launch gets without opting in).
template <typename T>
static int store_ppc(int D) {
    const int p = 40960 / (D * 10 + 18);
    return p < 1 ? 1 : (p > 16 ? 16 : p);
}
template <typename T>
static size_t store_smem(int D, int ppc) {
    return (size_t)ppc * (D + 1) * 8 + (size_t)ppc * (D + 2) * 2;
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
            const float s = load_scale<FMT>(a.v_scale, row, a.g_v);
            __nv_bfloat16* o = vo + h * a.so_h + t * a.so_s + (int64_t)db * BLK * a.so_d;
            if constexpr (FMT == FMT_MIX43) {
                const uint8_t* trow = a.v_packed + ((int64_t)h * a.v_s_stride + t) * ND * PACKB3;
#pragma unroll
                for (int c = 0; c < BLK; ++c)
                    o[c * a.so_d] = __float2bfloat16_rn(__fmul_rn((float)int3_code(trow, db * BLK + c), s));
                continue;
            }
            const uint2 pk = reinterpret_cast<const uint2*>(a.v_packed)[row];
#pragma unroll
            for (int c = 0; c < BLK; ++c) {
                uint32_t nib = ((c < 8 ? pk.x : pk.y) >> (4 * (c & 7))) & 0xF;
                o[c * a.so_d] = __float2bfloat16_rn(__fmul_rn(nib_value(nib, FMT), s));
            }
        }
    }
}

// Legacy page-level dequant (kv_quant.py:70-76, QuantizedPage.dequantize):
// per-token 16-channel INT4 blocks, value = bf16(fp16(code * fp16 scale)),
// the fp16 product rounded once and then narrowed to bf16 like the
// reference's `q.to(fp16) * scale` followed by `.to(bfloat16)`.  Optionally
// also writes the unpacked int8 codes.  One thread per block.
__global__ void __launch_bounds__(256) page_dequant_kernel(const uint8_t* __restrict__ packed,
                                                           const __half* __restrict__ scale, int rows,
                                                           int tokens, int row_stride, int ND,
                                                           __nv_bfloat16* __restrict__ out,
                                                           int8_t* __restrict__ codes) {
    const int64_t n = (int64_t)rows * tokens * ND;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int db = (int)(i % ND);
        const int64_t rt = i / ND;
        const int t = (int)(rt % tokens), r = (int)(rt / tokens);
        const int64_t src = ((int64_t)r * row_stride + t) * ND + db;
        const uint2 pk = reinterpret_cast<const uint2*>(packed)[src];
        const __half s = scale[src];
        uint32_t ob[8];
        uint32_t cb[4];
#pragma unroll
        for (int j = 0; j < BLK; ++j) {
            const int c = sx4((int)(((j < 8 ? pk.x : pk.y) >> (4 * (j & 7))) & 0xF));
            const __half prod = __hmul(__int2half_rn(c), s);
            const uint32_t bits = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(prod)));
            if (j & 1) ob[j >> 1] |= bits << 16; else ob[j >> 1] = bits;
            const uint32_t cbyte = (uint32_t)(c & 0xFF) << (8 * (j & 3));
            if (j & 3) cb[j >> 2] |= cbyte; else cb[j >> 2] = cbyte;
        }
        const int64_t o = i * BLK;                     // [rows, tokens, ND, 16] == [rows, tokens, D]
        if (out) {
            uint4* o4 = reinterpret_cast<uint4*>(out + o);
            o4[0] = make_uint4(ob[0], ob[1], ob[2], ob[3]);
            o4[1] = make_uint4(ob[4], ob[5], ob[6], ob[7]);
        }
        if (codes) *reinterpret_cast<uint4*>(codes + o) = make_uint4(cb[0], cb[1], cb[2], cb[3]);
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
        const float r = __frcp_rn(s);
#pragma unroll
        for (int j = 0; j < BLK; ++j)
            y[base + j * stride] = from_f32<T>(__fmul_rn(q_grid_div(v[j], s, r, a.fmt), s));
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

namespace {
// Up to this many blocks an MSE store runs one warp per block, the 32 clip
// ratios spread over the lanes and the 16 elements quantised in parallel: one
// thread per block would keep fewer than 256 threads per SM busy, each running
// the whole search alone (the 16-token step store of 64 heads, 16384 blocks:
// NVFP4 154 -> 31 us, INT4 43 -> 16 us).  NVFP4 absmax stores too: their one
// candidate's error check (e4m3-rounded scale, non-finite error -> scale 0) is
// spread over 16 lanes.  INT4 absmax has no check and stays thread-per-block.
constexpr int64_t SMALL_STORE_BLOCKS = 148LL * 256;

template <typename T, int FMT>
int launch_store(const StoreArgs& a, cudaStream_t st) {
    const int NP = a.S_k / BLK, ND = a.D / BLK;
    // fewer pages per CTA when the K work is small, so short stores (and the
    // ALU-heavy MSE search) still fill every SM
    int ppc = store_ppc<T>(a.D);
    while (ppc > 1 && (int64_t)a.H * ((NP + ppc - 1) / ppc) < 8LL * 148) ppc >>= 1;
    const int n_chunks = (NP + ppc - 1) / ppc;
    const int64_t nk_ctas64 = (int64_t)a.H * n_chunks;
    const int64_t nv = (int64_t)a.H * a.S_v * ND;
    int64_t nv_ctas = (nv + 255) / 256;
    if (nv_ctas > 148LL * 16) nv_ctas = 148LL * 16;
    if (nk_ctas64 + nv_ctas > 0x7fffffffLL) return KIVI_ERR_UNSUPPORTED;
    const int64_t nblocks = (int64_t)a.H * NP * a.D + nv;
    if constexpr (FMT != FMT_MIX43) {        // (the mixed cache's INT3 V blocks use the thread-per-block kernel)
        if ((a.calib_k == CAL_MSE || a.calib_v == CAL_MSE || FMT == FMT_NVFP4) && nblocks <= SMALL_STORE_BLOCKS) {
            const int64_t ctas = (nblocks + 7) / 8;          // 8 warps, one block each
            store_warp_kernel<T, FMT><<<(int)ctas, 256, 0, st>>>(a);
            return check_launch();
        }
    }
    // the staged K output stays within 48 KB (store_ppc), no opt-in needed
    const size_t smem = nk_ctas64 > 0 ? store_smem<T>(a.D, ppc) : 0;
    const unsigned grid = (unsigned)(nk_ctas64 + nv_ctas);
    if (a.calib_k == CAL_MSE || a.calib_v == CAL_MSE)
        store_kernel<T, FMT, true><<<grid, 256, smem, st>>>(a, ppc, n_chunks, (int)nk_ctas64);
    else   // absmax only: the MSE search is compiled out, fewer registers, more resident threads
        store_kernel<T, FMT, false><<<grid, 256, smem, st>>>(a, ppc, n_chunks, (int)nk_ctas64);
    return check_launch();
}
}  // namespace

extern "C" int kivi_store(const void* k, const void* v, int in_dtype, int64_t sk_h, int64_t sk_s,
                          int64_t sk_d, int64_t sv_h, int64_t sv_s, int64_t sv_d, int H, int S_k,
                          int S_v, int D, int fmt, int calib_k, int calib_v, const float* alphas,
                          int n_alphas, float g_k, float g_v, uint8_t* k_packed, void* k_scale,
                          int kpage0, int k_np_stride, uint8_t* v_packed, void* v_scale, int vtok0,
                          int v_s_stride, kivi_stream_t stream) {
    if (H < 0 || S_k < 0 || S_v < 0 || D <= 0 || D % BLK) return KIVI_ERR_ARG;
    if (fmt != FMT_INT4 && fmt != FMT_NVFP4 && fmt != FMT_MIX43) return KIVI_ERR_ARG;
    if (fmt == FMT_MIX43 && D % 32) return KIVI_ERR_ARG;     // V blocks go in pairs
    if ((unsigned)calib_k > 1 || (unsigned)calib_v > 1) return KIVI_ERR_ARG;
    if ((calib_k == CAL_MSE || calib_v == CAL_MSE) && (!alphas || n_alphas <= 0)) return KIVI_ERR_ARG;
    if (in_dtype != KIVI_DT_BF16 && in_dtype != KIVI_DT_F16 && in_dtype != KIVI_DT_F32) return KIVI_ERR_ARG;
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
    switch (in_dtype) {
        case KIVI_DT_BF16: return fmt == FMT_INT4 ? launch_store<__nv_bfloat16, FMT_INT4>(a, st)
                                : fmt == FMT_NVFP4 ? launch_store<__nv_bfloat16, FMT_NVFP4>(a, st)
                                                   : launch_store<__nv_bfloat16, FMT_MIX43>(a, st);
        case KIVI_DT_F16: return fmt == FMT_INT4 ? launch_store<__half, FMT_INT4>(a, st)
                               : fmt == FMT_NVFP4 ? launch_store<__half, FMT_NVFP4>(a, st)
                                                  : launch_store<__half, FMT_MIX43>(a, st);
        default: return fmt == FMT_INT4 ? launch_store<float, FMT_INT4>(a, st)
                      : fmt == FMT_NVFP4 ? launch_store<float, FMT_NVFP4>(a, st)
                                         : launch_store<float, FMT_MIX43>(a, st);
    }
}

extern "C" int kivi_dequant(const uint8_t* k_packed, const void* k_scale, int k_np_stride,
                            const uint8_t* v_packed, const void* v_scale, int v_s_stride, int H,
                            int S, int D, int fmt, float g_k, float g_v, void* k_out, void* v_out,
                            int64_t so_h, int64_t so_s, int64_t so_d, kivi_stream_t stream) {
    if (H < 0 || S < 0 || D <= 0 || D % BLK) return KIVI_ERR_ARG;
    if (fmt != FMT_INT4 && fmt != FMT_NVFP4 && fmt != FMT_MIX43) return KIVI_ERR_ARG;
    if (fmt == FMT_MIX43 && D % 32) return KIVI_ERR_ARG;
    if (k_np_stride < S / BLK || v_s_stride < S) return KIVI_ERR_ARG;
    if ((uintptr_t)k_packed % 8 || (uintptr_t)v_packed % 8) return KIVI_ERR_ALIGN;
    const int64_t n = (int64_t)H * (S / BLK) * D + (int64_t)H * S * (D / BLK);
    if (n == 0) return KIVI_OK;
    DequantArgs a{k_packed, k_scale, k_np_stride, v_packed, v_scale, v_s_stride, H, S, D,
                  g_k, g_v, k_out, v_out, so_h, so_s, so_d};
    cudaStream_t st = (cudaStream_t)stream;
    if (fmt == FMT_INT4) dequant_kernel<FMT_INT4><<<grid_for(n), 256, 0, st>>>(a);
    else if (fmt == FMT_NVFP4) dequant_kernel<FMT_NVFP4><<<grid_for(n), 256, 0, st>>>(a);
    else dequant_kernel<FMT_MIX43><<<grid_for(n), 256, 0, st>>>(a);
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

extern "C" int kivi_page_dequant(const uint8_t* packed, const void* scale, int rows, int tokens, int row_stride,
                                 int D, void* out, int8_t* codes, kivi_stream_t stream) {
    if (rows < 0 || tokens < 0 || D <= 0 || D % BLK || row_stride < tokens) return KIVI_ERR_ARG;
    const int64_t n = (int64_t)rows * tokens * (D / BLK);
    if (n == 0) return KIVI_OK;
    if (!packed || !scale || (!out && !codes)) return KIVI_ERR_ARG;
    if ((uintptr_t)packed % 8 || (uintptr_t)scale % 2 || (uintptr_t)out % 16 || (uintptr_t)codes % 16)
        return KIVI_ERR_ALIGN;
    page_dequant_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(
        packed, reinterpret_cast<const __half*>(scale), rows, tokens, row_stride, D / BLK,
        reinterpret_cast<__nv_bfloat16*>(out), codes);
    return check_launch();
}
