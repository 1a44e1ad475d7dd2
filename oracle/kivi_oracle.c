/*
 * kivi_oracle.c -- CPU restatement of the reference's 4-bit KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against; it is never linked into, loaded by, or called from the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm use it.
 *
 * Every function names the reference code it restates (paths are relative to
 * the a1exxd0/poolside-hackathon tree).  Parity of this restatement with the
 * reference itself is pinned by tests/golden/ (fixtures produced by running the
 * reference's own kv_quant.py / scripts on CPU; see tests/golden/make_golden.py).
 *
 * Floating-point contract (compile with -O2 -ffp-contract=off, never
 * -ffast-math): every operation below is one IEEE fp32 operation in the same
 * order torch's CPU kernels perform it, so results are bit-identical.
 *   - kv_quant.py:247-266 `_calibrate`:  scale = absmax/qmax, or for 'mse'
 *     scale_a = (alpha_a*absmax)/qmax, err_a = mean((x - q(x/s)*s)**2),
 *     first argmin over a.
 *   - the 16-element `mean` is reduced by torch's CPU vector kernel as
 *     v[j] = e[j] + e[j+8] (j < 8), then ((v0+v1)+v2)+...+v7, then /16
 *     (measured against torch 2.11 CPU; pinned by the golden fixtures).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BLK 16
#define PACKB 8

enum { FMT_INT4 = 0, FMT_INT3 = 1, FMT_NVFP4 = 2 };
enum { CAL_ABSMAX = 0, CAL_MSE = 1 };
enum { LAYOUT_HEADDIM = 0, LAYOUT_CHANNEL = 1 };

/* kv_quant.py:207-208 `_E2M1_LEVELS`, `_E2M1_BOUNDS` */
static const float E2M1_LEVELS[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
static const float E2M1_BOUNDS[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};

/* kv_quant.py:228 `_FORMATS` qmax column */
static float qmax_of(int fmt) {
    return fmt == FMT_INT4 ? 7.0f : (fmt == FMT_INT3 ? 3.0f : 6.0f);
}

/* kv_quant.py:220-225 `_q_e2m1`: bucketize(|y|, bounds, right=False) gives the
 * number of bounds strictly below |y| (ties go to the lower level); result is
 * sign(y) * level.  Returns the magnitude index; *neg = (y < 0). */
static int e2m1_index(float y, int *neg) {
    float a = fabsf(y);
    int idx = 0;
    for (int i = 0; i < 7; ++i) idx += (E2M1_BOUNDS[i] < a);
    *neg = (y < 0.0f);
    return idx;
}

/* kv_quant.py:211-225: round a scale-normalised value onto the format grid. */
static float q_grid(float y, int fmt) {
    if (fmt == FMT_NVFP4) {
        int neg, idx = e2m1_index(y, &neg);
        float l = E2M1_LEVELS[idx];
        if (y > 0.0f) return l;
        if (y < 0.0f) return -l;
        return 0.0f;           /* torch.sign(+-0) * level == +0 */
    }
    float r = rintf(y), qm = qmax_of(fmt);      /* .round().clamp(-qmax, qmax) */
    if (r > qm) return qm;
    if (r < -qm) return -qm;
    return r;
}

/* torch CPU order for mean over a contiguous 16-element row (see header). */
static float mean16(const float e[BLK]) {
    float v[8];
    for (int j = 0; j < 8; ++j) v[j] = e[j] + e[j + 8];
    float s = v[0];
    for (int j = 1; j < 8; ++j) s = s + v[j];
    return s / 16.0f;
}

static float absmax16(const float x[BLK]) {
    float m = 0.0f;
    for (int i = 0; i < BLK; ++i) {
        float a = fabsf(x[i]);
        if (a > m) m = a;
    }
    return m < 1e-9f ? 1e-9f : m;   /* .clamp_min(1e-9) */
}

/* kv_quant.py:247-266 `_calibrate` for one 16-element block. */
float orc_calibrate_block(const float *x, int fmt, int calib,
                          const float *alphas, int n_alphas) {
    float qmax = qmax_of(fmt);
    float amax = absmax16(x);
    if (calib == CAL_ABSMAX) return amax / qmax;
    float best = INFINITY, bs = 0.0f;
    for (int a = 0; a < n_alphas; ++a) {
        float s = (alphas[a] * amax) / qmax;
        float e[BLK];
        for (int i = 0; i < BLK; ++i) {
            float q = q_grid(x[i] / s, fmt);
            float d = x[i] - q * s;
            e[i] = d * d;
        }
        float err = mean16(e);
        if (err < best) { best = err; bs = s; }
    }
    return bs;
}

/* Gather one block of [H, S, D] x under a layout (kv_quant.py:232-244). */
static void gather_block(const float *x, int S, int D, int layout, int h,
                         int i0, int i1, float out[BLK]) {
    /* headdim: (token i0, dblock i1); channel: (channel i0, page i1) */
    if (layout == LAYOUT_HEADDIM) {
        const float *row = x + ((size_t)h * S + i0) * D + (size_t)i1 * BLK;
        for (int c = 0; c < BLK; ++c) out[c] = row[c];
    } else {
        for (int j = 0; j < BLK; ++j)
            out[j] = x[((size_t)h * S + (size_t)i1 * BLK + j) * D + i0];
    }
}

static void scatter_block(float *y, int S, int D, int layout, int h,
                          int i0, int i1, const float v[BLK]) {
    if (layout == LAYOUT_HEADDIM) {
        float *row = y + ((size_t)h * S + i0) * D + (size_t)i1 * BLK;
        for (int c = 0; c < BLK; ++c) row[c] = v[c];
    } else {
        for (int j = 0; j < BLK; ++j)
            y[((size_t)h * S + (size_t)i1 * BLK + j) * D + i0] = v[j];
    }
}

/* kv_quant.py:299-321 `roundtrip` (fp32 result before the final dtype cast).
 * x, y: fp32 [H, S, D].  For 'channel' the trailing S % 16 tokens are copied. */
void orc_roundtrip(const float *x, float *y, int H, int S, int D, int fmt,
                   int layout, int calib, const float *alphas, int n_alphas) {
    int n_full = (S / BLK) * BLK;
    int nA = (layout == LAYOUT_HEADDIM) ? S : D;           /* i0 range */
    int nB = (layout == LAYOUT_HEADDIM) ? D / BLK : n_full / BLK;
    if (layout == LAYOUT_CHANNEL) {
        for (int h = 0; h < H; ++h)
            for (int t = n_full; t < S; ++t)
                memcpy(y + ((size_t)h * S + t) * D, x + ((size_t)h * S + t) * D,
                       sizeof(float) * D);
    }
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int a = 0; a < nA; ++a)
            for (int b = 0; b < nB; ++b) {
                float blk[BLK], out[BLK];
                gather_block(x, S, D, layout, h, a, b, blk);
                float s = orc_calibrate_block(blk, fmt, calib, alphas, n_alphas);
                for (int i = 0; i < BLK; ++i) out[i] = q_grid(blk[i] / s, fmt) * s;
                scatter_block(y, S, D, layout, h, a, b, out);
            }
}

/* kv_quant.py:247-266 over n contiguous blocks: scales[n]. */
void orc_calibrate(const float *blocks, long n, int fmt, int calib,
                   const float *alphas, int n_alphas, float *scales) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i)
        scales[i] = orc_calibrate_block(blocks + i * BLK, fmt, calib, alphas, n_alphas);
}

/* ------------------------------------------------------------------------- */
/* small-float encoders: round-to-nearest-even onto a binary format with      */
/* `mbits` mantissa bits, minimum normal exponent `emin` and bias `bias`.     */
/* ------------------------------------------------------------------------- */
static double round_fmt(double a, int mbits, int emin) {
    if (a == 0.0) return 0.0;
    int ex;
    frexp(a, &ex);                 /* a = m * 2^ex, m in [0.5, 1) */
    int E = ex - 1;
    if (E < emin) E = emin;
    double q = ldexp(1.0, E - mbits);
    return nearbyint(a / q) * q;   /* exact scaling, RNE in default mode */
}

static uint32_t encode_fmt(double r, int mbits, int emin, int bias) {
    if (r == 0.0) return 0;
    int ex;
    frexp(r, &ex);
    int E = ex - 1;
    if (E < emin) return (uint32_t)(r / ldexp(1.0, emin - mbits));   /* subnormal */
    uint32_t mant = (uint32_t)((r / ldexp(1.0, E) - 1.0) * (double)(1 << mbits));
    return ((uint32_t)(E + bias) << mbits) | mant;
}

/* fp32 -> IEEE binary16 bits, RNE, overflow to inf (torch .to(float16)). */
uint16_t orc_f32_to_f16(float f) {
    uint32_t sign = signbit(f) ? 0x8000u : 0u;
    if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
    double a = fabs((double)f);
    if (isinf(f)) return (uint16_t)(sign | 0x7c00u);
    double r = round_fmt(a, 10, -14);
    if (r > 65504.0) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | encode_fmt(r, 10, -14, 15));
}

float orc_f16_to_f32(uint16_t h) {
    int s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    double v;
    if (e == 0) v = ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexp(1.0 + m / 1024.0, e - 15);
    return (float)(s ? -v : v);
}

/* fp32 -> float8 e4m3fn bits, RNE, saturating to +-448 (cvt.rn.satfinite). */
uint8_t orc_f32_to_e4m3(float f) {
    uint32_t sign = (f < 0.0f) ? 0x80u : 0u;
    if (isnan(f)) return 0x7f;
    double a = fabs((double)f);
    double r = round_fmt(a, 3, -6);
    if (r > 448.0) r = 448.0;
    return (uint8_t)(sign | encode_fmt(r, 3, -6, 7));
}

float orc_e4m3_to_f32(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 0xf, m = b & 7;
    double v;
    if (e == 0) v = ldexp((double)m, -9);
    else if (e == 15 && m == 7) v = NAN;
    else v = ldexp(1.0 + m / 8.0, e - 7);
    return (float)(s ? -v : v);
}

/* ------------------------------------------------------------------------- */
/* INT4-KIVI store (int4_kivi/triton_kernels.py:137-178, 216-254 and          */
/* int4_kivi/cache.py:90-141): codes against the fp32 scale, scale stored     */
/* as fp16, two's-complement nibbles, element 2j -> low nibble of byte j.     */
/* ------------------------------------------------------------------------- */
static void pack16(const int c[BLK], uint8_t out[PACKB]) {
    for (int j = 0; j < PACKB; ++j)
        out[j] = (uint8_t)((c[2 * j] & 0xf) | ((c[2 * j + 1] & 0xf) << 4));
}

/* k, v: fp32 [H, S, D].  Outputs follow int4_kivi/cache.py:52-63:
 * k_packed [H, D, NP, 8], k_scale f16 [H, D, NP], v_packed [H, S, ND, 8],
 * v_scale f16 [H, S, ND].  (The bf16 hot tail is a verbatim copy.) */
void orc_store_int4(const float *k, const float *v, int H, int S, int D,
                    int calib_k, int calib_v, const float *alphas, int n_alphas,
                    uint8_t *k_packed, uint16_t *k_scale,
                    uint8_t *v_packed, uint16_t *v_scale) {
    int NP = S / BLK, ND = D / BLK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d)
            for (int p = 0; p < NP; ++p) {
                float x[BLK]; int c[BLK];
                gather_block(k, S, D, LAYOUT_CHANNEL, h, d, p, x);
                float s = orc_calibrate_block(x, FMT_INT4, calib_k, alphas, n_alphas);
                for (int j = 0; j < BLK; ++j) c[j] = (int)q_grid(x[j] / s, FMT_INT4);
                size_t r = ((size_t)h * D + d) * NP + p;
                pack16(c, k_packed + r * PACKB);
                k_scale[r] = orc_f32_to_f16(s);
            }
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int t = 0; t < S; ++t)
            for (int db = 0; db < ND; ++db) {
                float x[BLK]; int c[BLK];
                gather_block(v, S, D, LAYOUT_HEADDIM, h, t, db, x);
                float s = orc_calibrate_block(x, FMT_INT4, calib_v, alphas, n_alphas);
                for (int j = 0; j < BLK; ++j) c[j] = (int)q_grid(x[j] / s, FMT_INT4);
                size_t r = ((size_t)h * S + t) * ND + db;
                pack16(c, v_packed + r * PACKB);
                v_scale[r] = orc_f32_to_f16(s);
            }
}

static inline int sx4(int n) { return n >= 8 ? n - 16 : n; }

/* int4_kivi/triton_kernels.py:181-210,257-286: value = code * fp32(f16 scale),
 * written as fp32 (the caller rounds to bf16).  kout [H, S, D] covers the first
 * NP*16 tokens; vout [H, S, D] covers every token. */
void orc_dequant_int4(const uint8_t *k_packed, const uint16_t *k_scale,
                      const uint8_t *v_packed, const uint16_t *v_scale,
                      int H, int S, int D, float *kout, float *vout) {
    int NP = S / BLK, ND = D / BLK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d)
            for (int p = 0; p < NP; ++p) {
                size_t r = ((size_t)h * D + d) * NP + p;
                float s = orc_f16_to_f32(k_scale[r]);
                for (int j = 0; j < BLK; ++j) {
                    int b = k_packed[r * PACKB + j / 2];
                    int n = (j & 1) ? (b >> 4) : (b & 0xf);
                    kout[((size_t)h * S + p * BLK + j) * D + d] = (float)sx4(n) * s;
                }
            }
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int t = 0; t < S; ++t)
            for (int db = 0; db < ND; ++db) {
                size_t r = ((size_t)h * S + t) * ND + db;
                float s = orc_f16_to_f32(v_scale[r]);
                for (int c = 0; c < BLK; ++c) {
                    int b = v_packed[r * PACKB + c / 2];
                    int n = (c & 1) ? (b >> 4) : (b & 0xf);
                    vout[((size_t)h * S + t) * D + db * BLK + c] = (float)sx4(n) * s;
                }
            }
}

/* ------------------------------------------------------------------------- */
/* Mixed-precision cache, V half (K is orc_store_int4's K): INT3 per token    */
/* over 16-channel blocks on the kv_quant.py:215-217 `int3` grid (qmax 3,     */
/* kv_quant.py:247-266 calibration), codes against the fp32 scale, scale      */
/* stored as fp16.  The reference has no packed INT3 layout; this library's:  */
/* c in [-3, 3] kept as L = c & 3 and sign s (c = L - 4s); blocks in pairs    */
/* (2k, 2k+1) of three little-endian u32 words A_2k, A_2k+1, S_k (12 bytes):  */
/* A_b has L of element i < 8 at bit 4i, of element 8+i at bit 4i+2; S_k has  */
/* s of element i < 8 of block 2k+o at bit 4i+2o, of element 8+i at 4i+1+2o.  */
/* ------------------------------------------------------------------------- */
static void put_u32(uint8_t *p, uint32_t w) {
    for (int j = 0; j < 4; ++j) p[j] = (uint8_t)(w >> (8 * j));
}
static uint32_t get_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* v: fp32 [H, S, D] (D % 32 == 0) -> v_packed [H, S, D/32, 12], v_scale f16 [H, S, D/16]. */
void orc_store_v3(const float *v, int H, int S, int D, int calib_v, const float *alphas,
                  int n_alphas, uint8_t *v_packed, uint16_t *v_scale) {
    int ND = D / BLK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int t = 0; t < S; ++t)
            for (int pr = 0; pr < ND / 2; ++pr) {
                uint32_t A[2] = {0, 0}, Sw = 0;
                for (int o = 0; o < 2; ++o) {
                    int db = 2 * pr + o;
                    float x[BLK];
                    gather_block(v, S, D, LAYOUT_HEADDIM, h, t, db, x);
                    float s = orc_calibrate_block(x, FMT_INT3, calib_v, alphas, n_alphas);
                    for (int i = 0; i < BLK; ++i) {
                        int c = (int)q_grid(x[i] / s, FMT_INT3);
                        int sha = i < 8 ? 4 * i : 4 * (i - 8) + 2, shs = (i < 8 ? 4 * i : 4 * (i - 8) + 1) + 2 * o;
                        A[o] |= (uint32_t)(c & 3) << sha;
                        Sw |= (uint32_t)(c < 0) << shs;
                    }
                    v_scale[((size_t)h * S + t) * ND + db] = orc_f32_to_f16(s);
                }
                uint8_t *out = v_packed + (((size_t)h * S + t) * (ND / 2) + pr) * 12;
                put_u32(out, A[0]); put_u32(out + 4, A[1]); put_u32(out + 8, Sw);
            }
}

/* value = code * fp32(f16 scale), fp32; vout [H, S, D]. */
void orc_dequant_v3(const uint8_t *v_packed, const uint16_t *v_scale, int H, int S, int D, float *vout) {
    int ND = D / BLK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int t = 0; t < S; ++t)
            for (int db = 0; db < ND; ++db) {
                const uint8_t *pp = v_packed + (((size_t)h * S + t) * (ND / 2) + db / 2) * 12;
                int o = db & 1;
                uint32_t A = get_u32(pp + 4 * o), Sw = get_u32(pp + 8);
                float s = orc_f16_to_f32(v_scale[((size_t)h * S + t) * ND + db]);
                for (int i = 0; i < BLK; ++i) {
                    int sha = i < 8 ? 4 * i : 4 * (i - 8) + 2, shs = (i < 8 ? 4 * i : 4 * (i - 8) + 1) + 2 * o;
                    int c = (int)((A >> sha) & 3) - 4 * (int)((Sw >> shs) & 1);
                    vout[((size_t)h * S + t) * D + db * BLK + i] = (float)c * s;
                }
            }
}

/* ------------------------------------------------------------------------- */
/* NVFP4-KIVI store.  Reference semantics: kv_quant.py:220-229 (`nvfp4`:     */
/* e2m1 grid, qmax 6, bucketize ties toward the smaller magnitude) with the   */
/* fp8-e4m3 block scale of the paged fork (scripts/diag_kernel_perchannel.py: */
/* 30-48, WRITEUP.md:97-107: scales rounded to e4m3 inside the search).       */
/* Block scale byte sc = e4m3(s / g); the dequantisable scale is              */
/* sd = fp32(sc) * g; codes are e2m1(x / sd) (all +0 when sd == 0).  Nibble = */
/* sign << 3 | level index, i.e. the hardware e2m1 bit pattern.               */
/* ------------------------------------------------------------------------- */
static float nvfp4_block(const float x[BLK], int calib, const float *alphas,
                         int n_alphas, float g, uint8_t *sc_out, uint8_t nib[BLK]) {
    float amax = absmax16(x);
    int nA = (calib == CAL_ABSMAX) ? 1 : n_alphas;
    float best = INFINITY;
    uint8_t best_sc = 0;
    for (int a = 0; a < nA; ++a) {
        float s = (calib == CAL_ABSMAX) ? amax / 6.0f : (alphas[a] * amax) / 6.0f;
        uint8_t sc = orc_f32_to_e4m3(s / g);
        float sd = orc_e4m3_to_f32(sc) * g;
        float e[BLK];
        for (int i = 0; i < BLK; ++i) {
            float q = (sd == 0.0f) ? 0.0f : q_grid(x[i] / sd, FMT_NVFP4);
            float d = x[i] - q * sd;
            e[i] = d * d;
        }
        float err = mean16(e);
        if (err < best) { best = err; best_sc = sc; }
    }
    float sd = orc_e4m3_to_f32(best_sc) * g;
    for (int i = 0; i < BLK; ++i) {
        if (sd == 0.0f) { nib[i] = 0; continue; }
        int neg, idx = e2m1_index(x[i] / sd, &neg);
        nib[i] = (uint8_t)((neg ? 8 : 0) | idx);
    }
    *sc_out = best_sc;
    return sd;
}

/* Same tensor geometry as orc_store_int4, with 1-byte e4m3 scales. */
void orc_store_nvfp4(const float *k, const float *v, int H, int S, int D,
                     int calib_k, int calib_v, const float *alphas, int n_alphas,
                     float g_k, float g_v,
                     uint8_t *k_packed, uint8_t *k_scale,
                     uint8_t *v_packed, uint8_t *v_scale) {
    int NP = S / BLK, ND = D / BLK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d)
            for (int p = 0; p < NP; ++p) {
                float x[BLK]; uint8_t nib[BLK]; int c[BLK];
                gather_block(k, S, D, LAYOUT_CHANNEL, h, d, p, x);
                size_t r = ((size_t)h * D + d) * NP + p;
                nvfp4_block(x, calib_k, alphas, n_alphas, g_k, &k_scale[r], nib);
                for (int j = 0; j < BLK; ++j) c[j] = nib[j];
                pack16(c, k_packed + r * PACKB);
            }
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int t = 0; t < S; ++t)
            for (int db = 0; db < ND; ++db) {
                float x[BLK]; uint8_t nib[BLK]; int c[BLK];
                gather_block(v, S, D, LAYOUT_HEADDIM, h, t, db, x);
                size_t r = ((size_t)h * S + t) * ND + db;
                nvfp4_block(x, calib_v, alphas, n_alphas, g_v, &v_scale[r], nib);
                for (int j = 0; j < BLK; ++j) c[j] = nib[j];
                pack16(c, v_packed + r * PACKB);
            }
}

static inline float e2m1_val(int n) {
    float l = E2M1_LEVELS[n & 7];
    return (n & 8) ? -l : l;
}

/* value = e2m1(code) * (fp32(e4m3 scale) * g), fp32. */
void orc_dequant_nvfp4(const uint8_t *k_packed, const uint8_t *k_scale,
                       const uint8_t *v_packed, const uint8_t *v_scale,
                       int H, int S, int D, float g_k, float g_v,
                       float *kout, float *vout) {
    int NP = S / BLK, ND = D / BLK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d)
            for (int p = 0; p < NP; ++p) {
                size_t r = ((size_t)h * D + d) * NP + p;
                float s = orc_e4m3_to_f32(k_scale[r]) * g_k;
                for (int j = 0; j < BLK; ++j) {
                    int b = k_packed[r * PACKB + j / 2];
                    int n = (j & 1) ? (b >> 4) : (b & 0xf);
                    kout[((size_t)h * S + p * BLK + j) * D + d] = e2m1_val(n) * s;
                }
            }
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; ++h)
        for (int t = 0; t < S; ++t)
            for (int db = 0; db < ND; ++db) {
                size_t r = ((size_t)h * S + t) * ND + db;
                float s = orc_e4m3_to_f32(v_scale[r]) * g_v;
                for (int c = 0; c < BLK; ++c) {
                    int b = v_packed[r * PACKB + c / 2];
                    int n = (c & 1) ? (b >> 4) : (b & 0xf);
                    vout[((size_t)h * S + t) * D + db * BLK + c] = e2m1_val(n) * s;
                }
            }
}

/* ------------------------------------------------------------------------- */
/* Decode attention over dequantised K/V (scripts/validate_int4_kivi_decode.py*/
/* :73-84 `ref_decode_fp32`: GQA by repeat_interleave, softmax(q.k*sm) @ v),  */
/* evaluated in double.  k, v: fp32 [B, Hkv, S, D]; q: [B, Hq, D];            */
/* out: fp32 [B, Hq, D].  Optional per-batch lengths (NULL = all S).          */
/* ------------------------------------------------------------------------- */
void orc_decode_attention(const float *q, const float *k, const float *v,
                          const int *seq_lens, int B, int Hq, int Hkv, int S,
                          int D, float sm_scale, float *out) {
    int G = Hq / Hkv;
    #pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int hq = 0; hq < Hq; ++hq) {
            int L = seq_lens ? seq_lens[b] : S;
            int hk = hq / G;
            const float *qq = q + ((size_t)b * Hq + hq) * D;
            const float *kk = k + ((size_t)b * Hkv + hk) * (size_t)S * D;
            const float *vv = v + ((size_t)b * Hkv + hk) * (size_t)S * D;
            double *sc = (double *)malloc(sizeof(double) * (L > 0 ? L : 1));
            double m = -INFINITY;
            for (int t = 0; t < L; ++t) {
                double acc = 0.0;
                for (int d = 0; d < D; ++d) acc += (double)qq[d] * kk[(size_t)t * D + d];
                sc[t] = acc * sm_scale;
                if (sc[t] > m) m = sc[t];
            }
            double l = 0.0;
            for (int t = 0; t < L; ++t) { sc[t] = exp(sc[t] - m); l += sc[t]; }
            float *o = out + ((size_t)b * Hq + hq) * D;
            for (int d = 0; d < D; ++d) {
                double acc = 0.0;
                for (int t = 0; t < L; ++t) acc += sc[t] * vv[(size_t)t * D + d];
                o[d] = (float)(L > 0 ? acc / l : 0.0);
            }
            free(sc);
        }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count of the OpenMP loops (a launcher may have set OMP_NUM_THREADS=1). */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------- */
/* Paged cache (the vLLM-fork layout named by WRITEUP.md:82-95,117-124 and     */
/* used at scripts/validate_paged_decode.py:32-64,                             */
/* scripts/validate_store_equiv.py:34-65): kv[nb, 2, 16, H, FD] u8,            */
/* FD = D/2 + D/16, row = codes then e4m3 scale bytes; V and the K rows of a   */
/* partial block per token; K of a full block per channel, channel c's scale  */
/* at row c / (D/16), byte c % (D/16).                                         */
/* ------------------------------------------------------------------------- */
static float sum16(const float e[BLK]) {
    float v[8];
    for (int j = 0; j < 8; ++j) v[j] = e[j] + e[j + 8];
    float s = v[0];
    for (int j = 1; j < 8; ++j) s = s + v[j];
    return s;
}

/* scripts/diag_kernel_perchannel.py:30-48 `fp8` + `mse_scale`: absmax (clamp
 * 1e-9), 16-point alpha grid 0.5 + i*(0.5/15) with e4m3-rounded scales inside
 * the search, squared error summed, strict '<' from e4m3(amax/qmax).  The code
 * of a value is rint(x/s) clamped to +-7 (INT4) or the e2m1 grid (NVFP4); a
 * zero scale (e4m3 underflow) gives code 0.  Returns the e4m3 byte. */
uint8_t orc_paged_calib(const float *x, int fmt, int calib) {
    float qmax = qmax_of(fmt);
    float amax = absmax16(x);
    uint8_t best = orc_f32_to_e4m3(amax / qmax);
    if (calib == CAL_ABSMAX) return best;
    float best_err = 1e38f;
    for (int i = 0; i < 16; ++i) {
        float a = (float)(0.5 + i * (0.5 / 15.0));
        uint8_t sc = orc_f32_to_e4m3((a * amax) / qmax);
        float s = orc_e4m3_to_f32(sc);
        float e[BLK];
        for (int k = 0; k < BLK; ++k) {
            float q = (s == 0.0f) ? 0.0f : q_grid(x[k] / s, fmt);
            float d = x[k] - q * s;
            e[k] = d * d;
        }
        float err = sum16(e);
        if (err < best_err) { best_err = err; best = sc; }
    }
    return best;
}

static uint32_t paged_nibble(float x, float s, int fmt) {
    if (s == 0.0f) return 0;
    float y = x / s;
    if (fmt == FMT_NVFP4) {
        int neg, idx = e2m1_index(y, &neg);
        return (uint32_t)idx | (neg ? 8u : 0u);
    }
    return (uint32_t)(int)q_grid(y, fmt) & 0xFu;
}

static float paged_code_value(uint32_t nib, int fmt) {
    if (fmt == FMT_NVFP4) {
        float l = E2M1_LEVELS[nib & 7];
        return (nib & 8) ? -l : l;
    }
    return (float)(nib >= 8 ? (int)nib - 16 : (int)nib);
}

static uint8_t *paged_row(uint8_t *kv, int H, int D, long slot, int sel, int h) {
    long FD = D / 2 + D / 16, RB = (long)H * FD;
    return kv + ((slot / 16) * 2 + sel) * 16 * RB + (slot % 16) * RB + (long)h * FD;
}

/* Store N tokens k, v fp32 [N, H, D] at slot_mapping[N] (negative = skip).
 * A block whose last slot is written by this call, with its earlier slots at
 * the consecutive indices before it (or already in the cache), is quantised
 * per channel over its 16 tokens; rows of that block not in this call are
 * first dequantised from the cache.  Every other token's K row goes per
 * token.  Returns 0, or 1 if a slot is out of range (that token skipped). */
int orc_paged_store(const float *k, const float *v, int N, int H, int D, int fmt, int calib,
                    const int64_t *slots, uint8_t *kv, long nb) {
    int ND = D / 16, bad = 0;
    for (int i = 0; i < N; ++i) {
        long s = (long)slots[i];
        if (s < 0) continue;
        if (s >= nb * 16) { bad = 1; continue; }
        int o = (int)(s % 16), e = i + 15 - o;
        int deferred = e < N && slots[e] == s - o + 15;
        for (int h = 0; h < H; ++h)
            for (int sel = 0; sel < 2; ++sel) {
                if (sel == 0 && deferred) continue;
                const float *src = (sel ? v : k) + ((size_t)i * H + h) * D;
                uint8_t *row = paged_row(kv, H, D, s, sel, h);
                for (int db = 0; db < ND; ++db) {
                    uint8_t sc = orc_paged_calib(src + db * 16, fmt, calib);
                    float sv = orc_e4m3_to_f32(sc);
                    for (int j = 0; j < 8; ++j)
                        row[8 * db + j] = (uint8_t)(paged_nibble(src[db * 16 + 2 * j], sv, fmt) |
                                                    (paged_nibble(src[db * 16 + 2 * j + 1], sv, fmt) << 4));
                    row[D / 2 + db] = sc;
                }
            }
    }
    for (int i = 0; i < N; ++i) {
        long s = (long)slots[i];
        if (s < 0 || s >= nb * 16 || s % 16 != 15) continue;
        long s0 = s - 15;
        for (int h = 0; h < H; ++h) {
            float *x = (float *)malloc(sizeof(float) * 16 * D);   /* [token][channel] */
            for (int j = 0; j < 16; ++j) {
                int idx = i - 15 + j;
                if (idx >= 0 && slots[idx] == s0 + j) {
                    memcpy(x + (size_t)j * D, k + ((size_t)idx * H + h) * D, sizeof(float) * D);
                } else {
                    uint8_t *row = paged_row(kv, H, D, s0 + j, 0, h);
                    for (int c = 0; c < D; ++c) {
                        float sc = orc_e4m3_to_f32(row[D / 2 + c / 16]);
                        x[(size_t)j * D + c] = paged_code_value((row[c / 2] >> (4 * (c & 1))) & 0xF, fmt) * sc;
                    }
                }
            }
            for (int c = 0; c < D; ++c) {
                float col[BLK];
                for (int j = 0; j < 16; ++j) col[j] = x[(size_t)j * D + c];
                uint8_t sc = orc_paged_calib(col, fmt, calib);
                float sv = orc_e4m3_to_f32(sc);
                for (int j = 0; j < 16; ++j) {
                    uint8_t *row = paged_row(kv, H, D, s0 + j, 0, h);
                    uint32_t nib = paged_nibble(col[j], sv, fmt);
                    row[c / 2] = (uint8_t)((c & 1) ? ((row[c / 2] & 0x0F) | (nib << 4))
                                                   : ((row[c / 2] & 0xF0) | nib));
                }
                paged_row(kv, H, D, s0 + c / ND, 0, h)[D / 2 + c % ND] = sc;
            }
            free(x);
        }
    }
    return bad;
}

/* Gather-dequant to fp32 k, v [B, H, max_seq, D]; block b of a sequence of
 * length L is per channel iff (b+1)*16 <= L; tokens >= L are 0. */
void orc_paged_gather(const uint8_t *kv, long nb, const int *bt, long bt_stride, const int *seq_lens,
                      int B, int H, int D, int fmt, int max_seq, float *k_out, float *v_out) {
    int ND = D / 16;
    (void)nb;
    for (int b = 0; b < B; ++b) {
        long L = seq_lens[b] < 0 ? 0 : seq_lens[b];
        if (L > bt_stride * 16) L = bt_stride * 16;
        for (int h = 0; h < H; ++h)
            for (int t = 0; t < max_seq; ++t) {
                float *ko = k_out + (((size_t)b * H + h) * max_seq + t) * D;
                float *vo = v_out + (((size_t)b * H + h) * max_seq + t) * D;
                if (t >= L) { memset(ko, 0, sizeof(float) * D); memset(vo, 0, sizeof(float) * D); continue; }
                long pg = t / 16, phys = bt[(size_t)b * bt_stride + pg];
                int full = (pg + 1) * 16 <= L;
                const uint8_t *kr = paged_row((uint8_t *)kv, H, D, phys * 16 + t % 16, 0, h);
                const uint8_t *vr = paged_row((uint8_t *)kv, H, D, phys * 16 + t % 16, 1, h);
                for (int c = 0; c < D; ++c) {
                    float ks = orc_e4m3_to_f32(kr[D / 2 + c / 16]);
                    if (full) ks = orc_e4m3_to_f32(paged_row((uint8_t *)kv, H, D, phys * 16 + c / ND, 0, h)[D / 2 + c % ND]);
                    ko[c] = paged_code_value((kr[c / 2] >> (4 * (c & 1))) & 0xF, fmt) * ks;
                    vo[c] = paged_code_value((vr[c / 2] >> (4 * (c & 1))) & 0xF, fmt) *
                            orc_e4m3_to_f32(vr[D / 2 + c / 16]);
                }
            }
    }
}
