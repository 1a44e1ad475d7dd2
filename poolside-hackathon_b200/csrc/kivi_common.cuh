// kivi_common.cuh -- shared device helpers for the sm_100a 4-bit KV-cache kernels.
//
// Quantiser arithmetic restates kv_quant.py:16-42, 206-266 (the reference's
// calibration) with every fp32 operation written as an explicitly rounded
// intrinsic (__fdiv_rn, __fmul_rn, __fadd_rn, __fsub_rn) so the compiler can
// neither contract nor reorder it: codes and scales are bit-identical to the
// reference on CPU.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace kivi {

constexpr int BLK = 16;   // elements per quant block; tokens per K page
constexpr int PACKB = 8;  // bytes per packed block

// FMT_MIX43: the mixed-precision cache, K INT4 (the KIVI K layout) and V INT3
// per token over 16-channel blocks (the kv_quant.py:215-217 `int3` grid,
// qmax 3), 6 bytes per block.  A code c in [-3, 3] is stored as its low two
// bits L = c & 3 and a sign bit s (c = L - 4s).  Blocks go in pairs (2k,
// 2k + 1) of 12 bytes: two 32-bit words A_{2k}, A_{2k+1} and one word S_k.
//   A_b:  L of element i < 8 at bits [4i, 4i + 2), of element 8 + i at bits
//         [4i + 2, 4i + 4);
//   S_k:  s of element i < 8 of block 2k + o at bit 4i + 2o, of element
//         8 + i at bit 4i + 1 + 2o.
// So (A & 0x33333333) and ((A >> 2) & 0x33333333) are the low two bits of
// the nibble words of elements 0..7 and 8..15, and the sign bits land on bit
// 2 of each nibble with one shift: a block becomes 3-bit nibbles c & 7 (the
// INT4 nibble layout, bit 3 clear) in a few logic operations.
enum Fmt { FMT_INT4 = 0, FMT_INT3 = 1, FMT_NVFP4 = 2, FMT_MIX43 = 3 };
constexpr int PACKB3 = 6;  // bytes per packed INT3 block (12 per block pair)
enum Calib { CAL_ABSMAX = 0, CAL_MSE = 1 };

__device__ __forceinline__ float qmax_of(int fmt) {
    return fmt == FMT_INT4 ? 7.0f : (fmt == FMT_INT3 ? 3.0f : 6.0f);
}

// kv_quant.py:220-225: bucketize(|y|, bounds, right=False) -> count of bounds
// strictly below |y|; ties resolve to the smaller magnitude.
__device__ __forceinline__ int e2m1_index(float a) {
    return (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) +
           (a > 2.5f) + (a > 3.5f) + (a > 5.0f);
}

__device__ __forceinline__ float e2m1_level(int idx) {
    // 0, .5, 1, 1.5, 2, 3, 4, 6
    return idx < 4 ? 0.5f * idx : (idx == 4 ? 2.0f : (idx == 5 ? 3.0f : (idx == 6 ? 4.0f : 6.0f)));
}

// kv_quant.py:211-225: scale-normalised value onto the format grid.
__device__ __forceinline__ float q_grid(float y, int fmt) {
    if (fmt == FMT_NVFP4) {
        float l = e2m1_level(e2m1_index(fabsf(y)));
        return y > 0.0f ? l : (y < 0.0f ? -l : 0.0f);
    }
    float r = rintf(y), qm = qmax_of(fmt);
    return r > qm ? qm : (r < -qm ? -qm : r);
}

// torch CPU order for the mean of a contiguous 16-element row:
// v[j] = e[j] + e[j+8], then ((v0+v1)+v2)+...+v7, then / 16.
__device__ __forceinline__ float mean16(const float e[BLK]) {
    float s = __fadd_rn(e[0], e[8]);
#pragma unroll
    for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __fadd_rn(e[j], e[j + 8]));
    return __fmul_rn(s, 0.0625f);      // == s / 16 exactly (a power-of-two scaling, one rounding)
}

__device__ __forceinline__ float absmax16(const float x[BLK]) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < BLK; ++i) m = fmaxf(m, fabsf(x[i]));
    return fmaxf(m, 1e-9f);   // .clamp_min(1e-9)
}

// A stand-in for the correctly rounded quotient x / s that every grid
// (rint + clamp, the e2m1 bucketing) maps to the same point, given r = 1/s
// rounded to nearest.  y = x * r is within ~2^-22 |y| of the true quotient,
// so it rounds to the same grid point as the IEEE quotient unless it lies
// that close to a rounding boundary (a half-integer, or an e2m1 bound); only
// then is the exact division done.  Valid for every x and every normal,
// nonzero s (the scales here are >= 1e-9 / 7 or e4m3 values).
__device__ __forceinline__ float quot_for_grid(float x, float s, float r, int fmt) {
    const float y = __fmul_rn(x, r);
    const float a = fabsf(y);
    const float tol = 1e-5f * fmaxf(1.0f, a);
    bool near;
    if (fmt == FMT_NVFP4) {
        const float bnd = a < 1.0f ? (a < 0.5f ? 0.25f : 0.75f)
                                   : (a < 2.125f ? (a < 1.5f ? 1.25f : 1.75f) : (a < 3.0f ? 2.5f : (a < 4.25f ? 3.5f : 5.0f)));
        near = fabsf(a - bnd) < tol;
    } else {
        near = fabsf(fabsf(y - rintf(y)) - 0.5f) < tol;
    }
    return near ? __fdiv_rn(x, s) : y;
}
__device__ __forceinline__ float q_grid_div(float x, float s, float r, int fmt) {
    return q_grid(quot_for_grid(x, s, r, fmt), fmt);
}

// Reconstruction error of one block under scale s (the kv_quant MSE term).
__device__ __forceinline__ float block_err(const float x[BLK], float s, int fmt) {
    float e[BLK];
    const float r = __frcp_rn(s);
#pragma unroll
    for (int i = 0; i < BLK; ++i) {
        float q = (s == 0.0f) ? 0.0f : q_grid_div(x[i], s, r, fmt);
        float d = __fsub_rn(x[i], __fmul_rn(q, s));
        e[i] = __fmul_rn(d, d);
    }
    return mean16(e);
}

// kv_quant.py:247-266 `_calibrate` for one block (fp32 scale).
__device__ __forceinline__ float calibrate16(const float x[BLK], int fmt, int calib,
                                             const float* __restrict__ alphas, int n_alphas) {
    const float qmax = qmax_of(fmt);
    const float amax = absmax16(x);
    if (calib == CAL_ABSMAX) return __fdiv_rn(amax, qmax);
    float best = __int_as_float(0x7f800000), bs = 0.0f;
    for (int a = 0; a < n_alphas; ++a) {
        float s = __fdiv_rn(__fmul_rn(alphas[a], amax), qmax);
        float err = block_err(x, s, fmt);
        if (err < best) { best = err; bs = s; }   // strict '<' == torch.argmin
    }
    return bs;
}

// fp32 -> e4m3 (RNE, saturating) and back; used for NVFP4 block scales.
__device__ __forceinline__ uint8_t f32_to_e4m3(float f) {
    return (uint8_t)__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
    return __half2float(__half(h));
}

// NVFP4-KIVI block: pick the e4m3 scale byte (scale rounded inside the search),
// return the dequantisable scale sd = fp32(e4m3(s/g)) * g.
__device__ __forceinline__ float nvfp4_calibrate16(const float x[BLK], int calib,
                                                   const float* __restrict__ alphas, int n_alphas,
                                                   float g, uint8_t* sc_out) {
    const float amax = absmax16(x);
    const int nA = (calib == CAL_ABSMAX) ? 1 : n_alphas;
    float best = __int_as_float(0x7f800000);
    uint8_t best_sc = 0;
    for (int a = 0; a < nA; ++a) {
        float s = (calib == CAL_ABSMAX) ? __fdiv_rn(amax, 6.0f)
                                        : __fdiv_rn(__fmul_rn(alphas[a], amax), 6.0f);
        uint8_t sc = f32_to_e4m3(__fdiv_rn(s, g));
        float sd = __fmul_rn(e4m3_to_f32(sc), g);
        float err = block_err(x, sd, FMT_NVFP4);
        if (err < best) { best = err; best_sc = sc; }
    }
    *sc_out = best_sc;
    return __fmul_rn(e4m3_to_f32(best_sc), g);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }

__device__ __forceinline__ int sx4(int n) { return n >= 8 ? n - 16 : n; }

// FMT_MIX43 V: the 8-nibble words (elements 0..7, 8..15; nibble = c & 7) of
// block 2k + o from its pair's words A (= A_{2k+o}) and S (= S_k).
__device__ __forceinline__ void int3_pair_nibbles(uint32_t A, uint32_t S, int o, uint32_t& lo, uint32_t& hi) {
    const uint32_t slo = (o ? S : S << 2) & 0x44444444u;
    const uint32_t shi = (o ? S >> 1 : S << 1) & 0x44444444u;
    lo = (A & 0x33333333u) | slo;
    hi = ((A >> 2) & 0x33333333u) | shi;
}
// Code of channel d of a token row (6 * ND bytes) of FMT_MIX43 V.
__device__ __forceinline__ int int3_code(const uint8_t* row, int d) {
    const int db = d >> 4, i = d & 15, o = db & 1;
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(row + 12 * (db >> 1));
    const uint32_t A = pw[o], S = pw[2];
    const int L = (int)(A >> (i < 8 ? 4 * i : 4 * (i - 8) + 2)) & 3;
    const int s = (int)(S >> ((i < 8 ? 4 * i : 4 * (i - 8) + 1) + 2 * o)) & 1;
    return L - 4 * s;
}
// Pack two blocks' codes (c in [-3, 3]) into the 12-byte pair.
__device__ __forceinline__ void int3_pack_pair(const int c0[16], const int c1[16], uint32_t& A0, uint32_t& A1,
                                               uint32_t& S) {
    A0 = A1 = S = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int sha = i < 8 ? 4 * i : 4 * (i - 8) + 2, shs = i < 8 ? 4 * i : 4 * (i - 8) + 1;
        A0 |= (uint32_t)(c0[i] & 3) << sha;
        A1 |= (uint32_t)(c1[i] & 3) << sha;
        S |= (uint32_t)(c0[i] < 0) << shs;
        S |= (uint32_t)(c1[i] < 0) << (shs + 2);
    }
}

// ---------------------------------------------------------------------------
// PTX wrappers: mbarrier, TMA, ldmatrix, mma.sync
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Explicit shared-window accesses by 32-bit address.  Pointers into dynamic
// shared memory that went through integer alignment arithmetic lose their
// address space; plain C++ accesses through them compile to generic loads and
// stores, which wait on the long scoreboard like global memory.
__device__ __forceinline__ uint32_t lds32s(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64s(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds8s(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts16s(uint32_t a, __half v) {
    asm volatile("st.shared.u16 [%0], %1;" :: "r"(a), "h"(__half_as_ushort(v)) : "memory");
}
__device__ __forceinline__ void sts32s(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" :: "r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void sts64s(uint32_t a, uint32_t x, uint32_t y) {
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" :: "r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ uint4 lds128s(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a)
                 : "memory");
    return v;
}
__device__ __forceinline__ void sts128s(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" :: "r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: returns false after ~timeout_ns without the phase completing.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t timeout_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
}

// TMA tiled loads into this CTA's shared memory, completion counted on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(smem_u32(dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t m, uint32_t x) {
    // (a & m) ^ x
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(m), "r"(x));
    return d;
}
__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Signed INT4 nibbles at bit offsets {0,16} (lo) or {4,20} (hi) of a word ->
// exact fp16x2 codes (fp16 magic-number method: nibble^8 placed in the
// mantissa of 1024, then the bias 1032 removed).
__device__ __forceinline__ __half2 int4_lo_to_h2(uint32_t w) {
    uint32_t v = lop3_and_xor(w, 0x000F000Fu, 0x64086408u);      // 1024 + (n ^ 8)
    return __hsub2(u32_as_h2(v), u32_as_h2(0x64086408u));         // - 1032
}
// FMT_MIX43 V nibbles hold c & 7 (bit 3 clear): (n ^ 4) = c + 4.
__device__ __forceinline__ __half2 int3n_lo_to_h2(uint32_t w) {
    uint32_t v = lop3_and_xor(w, 0x000F000Fu, 0x64046404u);      // 1024 + (n ^ 4)
    return __hsub2(u32_as_h2(v), u32_as_h2(0x64046404u));         // - 1028
}
__device__ __forceinline__ __half2 int3n_hi_to_h2(uint32_t w) {
    uint32_t v = lop3_and_xor(w, 0x00F000F0u, 0x64406440u);      // 1024 + 16 (n ^ 4)
    return __hfma2(u32_as_h2(v), u32_as_h2(0x2C002C00u), u32_as_h2(0xD440D440u));   // * 1/16 - 68
}
__device__ __forceinline__ __half2 int4_hi_to_h2(uint32_t w) {
    uint32_t v = lop3_and_xor(w, 0x00F000F0u, 0x64806480u);      // 1024 + 16 (n ^ 8)
    return __hfma2(u32_as_h2(v), u32_as_h2(0x2C002C00u), u32_as_h2(0xD480D480u));   // * 1/16 - 72
}

// Two e2m1 nibbles of one byte -> fp16x2 (exact), hardware conversion.
__device__ __forceinline__ uint32_t e2m1x2_to_h2(uint32_t byte_in_low8) {
    uint32_t d;
    asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(d) : "r"(byte_in_low8));
    return d;
}
// Four e2m1 pairs (one 32-bit word) -> four fp16x2 values, byte i -> h_i.
__device__ __forceinline__ void e2m1x8_to_h2x4(uint32_t w, uint32_t& h0, uint32_t& h1, uint32_t& h2,
                                               uint32_t& h3) {
    asm("{ .reg .b8 a, b, c, d;\n"
        "  mov.b32 {a, b, c, d}, %4;\n"
        "  cvt.rn.f16x2.e2m1x2 %0, a;\n"
        "  cvt.rn.f16x2.e2m1x2 %1, b;\n"
        "  cvt.rn.f16x2.e2m1x2 %2, c;\n"
        "  cvt.rn.f16x2.e2m1x2 %3, d; }"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3) : "r"(w));
}
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint16_t two) {
    uint32_t d;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(two));
    return d;
}

}  // namespace kivi
