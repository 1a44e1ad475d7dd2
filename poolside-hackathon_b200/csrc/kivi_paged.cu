// kivi_paged.cu -- the vLLM-style paged 4-bit KV cache: store, gather-dequant
// and fused paged flash-decode.
//
// Replaces the fork kernels named by the reference (vllm/v1/attention/ops/
// triton_{int4,nvfp4}_kivi.py: int4_kivi_store, int4_kivi_gather_dequant,
// int4_kivi_paged_decode and the nvfp4_* twins; called at
// scripts/validate_paged_decode.py:59,72,91, scripts/validate_store_equiv.py:
// 50-51, scripts/validate_nvfp4_kivi.py:67-75,136-150).  The fork source is not
// part of the reference checkout; the layout below is the one its write-up
// states (WRITEUP.md:82-95,117-124) and its call sites imply.
//
// Cache: one uint8 tensor kv[num_blocks, 2, 16, H, FD], FD = D/2 + D/16;
// dim 1 selects K (0) or V (1); a row (block, kv, slot, head) holds D/2 code
// bytes (element 2j in the low nibble of byte j) then D/16 e4m3 scale bytes.
//   V, and K of a partial block: per token, scale byte j = 16 channels 16j..
//   K of a full block (16 tokens, (b+1)*16 <= seq_len): per channel over the
//     16 tokens; the 16 rows' scale bytes are read as D per-channel scales,
//     channel c at row c / (D/16), byte c % (D/16).
// INT4 codes are two's-complement in [-7, 7]; NVFP4 codes are e2m1 with the
// sign in bit 3; both scale with an e4m3 byte (value = code * fp32(scale)).
//
// Calibration (scripts/diag_kernel_perchannel.py:30-48): absmax over the 16
// values, then a 16-point clip grid alpha_i = 0.5 + i * (0.5 / 15) with the
// scale rounded to e4m3 inside the search, squared error summed over the
// block, strict '<' argmin starting from e4m3(amax / qmax).
#include "kivi_common.cuh"
#include "kivi_internal.h"
#include <algorithm>
#include <cstring>
#include <type_traits>
#include <cuda.h>

namespace kivi {
namespace paged {

constexpr int PG = 16;                 // tokens per block (page)

__host__ __device__ __forceinline__ int full_dim(int D) { return D / 2 + D / 16; }

__device__ __forceinline__ void set_err_flag(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

struct Geo {
    int H, D, FD;
    int64_t RB;    // bytes per (block, kv, slot) row: H * FD
    int64_t PGB;   // bytes per (block, kv): 16 * RB
};
__host__ __device__ __forceinline__ Geo make_geo(int H, int D) {
    Geo g;
    g.H = H; g.D = D; g.FD = full_dim(D);
    g.RB = (int64_t)H * g.FD;
    g.PGB = PG * g.RB;
    return g;
}
__device__ __forceinline__ uint8_t* row_at(uint8_t* kv, const Geo& g, int64_t slot, int sel, int h) {
    return kv + ((slot / PG) * 2 + sel) * g.PGB + (slot % PG) * g.RB + (int64_t)h * g.FD;
}
__device__ __forceinline__ const uint8_t* row_at(const uint8_t* kv, const Geo& g, int64_t slot, int sel, int h) {
    return kv + ((slot / PG) * 2 + sel) * g.PGB + (slot % PG) * g.RB + (int64_t)h * g.FD;
}

// Sum of 16 values in torch's CPU order for a contiguous row (pairs j, j+8,
// then left to right).
__device__ __forceinline__ float sum16(const float e[BLK]) {
    float s = __fadd_rn(e[0], e[8]);
#pragma unroll
    for (int j = 1; j < 8; ++j) s = __fadd_rn(s, __fadd_rn(e[j], e[j + 8]));
    return s;
}

__device__ __forceinline__ float grid_code(float y, int fmt) {
    return q_grid(y, fmt);               // INT4: rint + clamp(+-7); NVFP4: e2m1 level
}

// Squared reconstruction error of a block under the e4m3-rounded scale s.
__device__ __forceinline__ float sq_err(const float x[BLK], float s, int fmt) {
    float e[BLK];
    const float r = __frcp_rn(s);
#pragma unroll
    for (int i = 0; i < BLK; ++i) {
        const float q = (s == 0.0f) ? 0.0f : grid_code(quot_for_grid(x[i], s, r, fmt), fmt);
        const float d = __fsub_rn(x[i], __fmul_rn(q, s));
        e[i] = __fmul_rn(d, d);
    }
    return sum16(e);
}

__device__ __forceinline__ uint32_t nibble_of(float x, float s, int fmt) {
    if (s == 0.0f) return 0u;
    const float y = quot_for_grid(x, s, __frcp_rn(s), fmt);
    if (fmt == FMT_NVFP4) return (uint32_t)e2m1_index(fabsf(y)) | (y < 0.0f ? 8u : 0u);
    return (uint32_t)(int)grid_code(y, fmt) & 0xFu;
}

__device__ __forceinline__ float code_value(uint32_t nib, int fmt) {
    if (fmt == FMT_NVFP4) {
        const float l = e2m1_level(nib & 7);
        return (nib & 8) ? -l : l;
    }
    return (float)sx4((int)nib);
}

template <typename T>
__device__ __forceinline__ float ld_in(const void* p, int64_t i) {
    return to_f32<T>(reinterpret_cast<const T*>(p)[i]);
}
__device__ __forceinline__ float ld_any(const void* p, int dt, int64_t i) {
    if (dt == KIVI_DT_BF16) return ld_in<__nv_bfloat16>(p, i);
    if (dt == KIVI_DT_F16) return ld_in<__half>(p, i);
    return ld_in<float>(p, i);
}

struct StoreP {
    const void* k; const void* v; int dt;
    int64_t sk_t, sk_h, sk_d, sv_t, sv_h, sv_d;
    int N; Geo g; int fmt, calib;
    const int64_t* slots; uint8_t* kv; int64_t nb; int* err;
};

__device__ __forceinline__ bool slot_ok(const StoreP& p, int64_t s) {
    return s >= 0 && s < p.nb * PG;
}

// A token's K goes per channel when its block is completed by this call: the
// token at index i + (15 - slot % 16) exists and holds the block's last slot.
__device__ __forceinline__ bool k_deferred(const StoreP& p, int i, int64_t s) {
    const int o = (int)(s % PG);
    const int e = i + (PG - 1 - o);
    return e < p.N && p.slots[e] == s - o + (PG - 1);
}

// The 16-point clip search of one block on a half-warp: lane a (0..15)
// evaluates alpha_a; the strict-'<' first-index argmin of the sequential
// search is kept by reducing (err, index) pairs with ties to the lower index
// (NaN errors never win).  x[16] is the block, identical in every lane.
// Returns the e4m3 scale byte (same in all 16 lanes).
__device__ __forceinline__ uint8_t calib_e4m3_hw(const float x[BLK], int fmt, int calib, int a) {
    const float qmax = qmax_of(fmt);
    const float amax = absmax16(x);
    const uint8_t init = f32_to_e4m3(__fdiv_rn(amax, qmax));
    if (calib == CAL_ABSMAX) return init;
    const float al = __double2float_rn(0.5 + a * (0.5 / 15.0));
    const uint8_t sc = f32_to_e4m3(__fdiv_rn(__fmul_rn(al, amax), qmax));
    float err = sq_err(x, e4m3_to_f32(sc), fmt);
    if (!(err < 1e38f)) err = INFINITY;                 // cannot beat the initial 1e38 (or is NaN)
    int idx = a;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        const float e2 = __shfl_xor_sync(0xffffffffu, err, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (e2 < err || (e2 == err && i2 < idx)) { err = e2; idx = i2; }
    }
    const uint32_t best = __shfl_sync(0xffffffffu, (uint32_t)sc, (threadIdx.x & 16) | idx);
    return err == INFINITY ? init : (uint8_t)best;
}

// Per-token blocks: one half-warp per (token, head, 16-value block); blocks
// 0..ND-1 are V, ND..2ND-1 are K (skipped when the token's block completes in
// this call).  Lane e also quantises element e; lanes 2j, 2j+1 form byte j.
__global__ void __launch_bounds__(256) store_token_kernel(const StoreP p) {
    const int ND = p.g.D / BLK;
    const int lane = threadIdx.x & 31, a = lane & 15;
    const int64_t task = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;   // half-warp index
    const int64_t total = (int64_t)p.N * p.g.H * 2 * ND;
    const bool in = task < total;
    const int64_t tk = in ? task : total - 1;          // out-of-range half-warps shadow a valid task
    const int j = (int)(tk % (2 * ND));
    const int h = (int)((tk / (2 * ND)) % p.g.H);
    const int i = (int)(tk / (2 * ND * p.g.H));
    const int64_t s = p.slots[i];
    const bool isv = j < ND;
    const int db = isv ? j : j - ND;
    bool live = in && s >= 0;
    if (live && !slot_ok(p, s)) { if (a == 0) set_err_flag(p.err, KIVI_ERR_ARG); live = false; }
    if (live && !isv && k_deferred(p, i, s)) live = false;
    // A warp's two half-warps are neighbouring blocks of one token and head
    // (both V or both K, ND even): when neither stores anything (K that goes
    // per channel, or padding slots) the warp leaves before the search.
    if (!__any_sync(0xffffffffu, live)) return;
    // both half-warps of a warp reach the shuffles; a dead one computes on a valid block
    float x[BLK];
    const void* src = isv ? p.v : p.k;
    const int64_t st = isv ? p.sv_t : p.sk_t, sh = isv ? p.sv_h : p.sk_h, sd = isv ? p.sv_d : p.sk_d;
    const int64_t base = (int64_t)i * st + (int64_t)h * sh + (int64_t)(db * BLK) * sd;
#pragma unroll
    for (int e = 0; e < BLK; ++e) x[e] = ld_any(src, p.dt, base + e * sd);
    const uint8_t sc = calib_e4m3_hw(x, p.fmt, p.calib, a);
    const float xa = ld_any(src, p.dt, base + a * sd);   // element a (a register index would spill)
    const uint32_t nib = nibble_of(xa, e4m3_to_f32(sc), p.fmt);
    const uint32_t other = __shfl_xor_sync(0xffffffffu, nib, 1);
    if (live && s >= 0) {
        uint8_t* row = row_at(p.kv, p.g, s, isv ? 1 : 0, h);
        if ((a & 1) == 0) row[8 * db + a / 2] = (uint8_t)(nib | (other << 4));
        if (a == 0) row[p.g.D / 2 + db] = sc;
    }
}

// Per-channel K of blocks completed by this call: one 512-thread CTA per 16
// input tokens, head and group of 32 channels (blockIdx.z).  For each
// completing token the block's 16 x D values are staged in shared memory
// first (rows this call brings from the input, the others dequantised from
// their per-token form in the cache), then warps take channel pairs:
// half-warp u owns channel 2cp+u, lane a evaluates clip alpha_a, then lane e
// quantises token e.  A block whose 16 rows all come from this call's input
// is split over the channel groups (CTA z stages and quantises its 32
// channels).  A block that also needs rows from the cache is done whole by
// the z = 0 CTA: the per-token scale bytes those rows are dequantised with
// are the bytes the per-channel scales overwrite, and only one CTA can order
// its reads before those writes.
__global__ void __launch_bounds__(512) store_channel_kernel(const StoreP p) {
    extern __shared__ float xs[];                        // [16][D]
    const int h = blockIdx.y;
    const int i_lo = blockIdx.x * PG, i_hi = min(i_lo + PG, p.N);
    const int D = p.g.D, ND = D / BLK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, a = lane & 15, u = lane >> 4;
    const int nwarp = blockDim.x >> 5;
    for (int i = i_lo; i < i_hi; ++i) {
        const int64_t s = p.slots[i];                    // uniform over the CTA
        if (!slot_ok(p, s) || s % PG != PG - 1) continue;
        const int64_t s0 = s - (PG - 1);
        bool all_in = true;                              // every row of the block from this call's input
        for (int j = 0; j < PG; ++j) {
            const int idx = i - (PG - 1) + j;
            all_in = all_in && idx >= 0 && p.slots[idx] == s0 + j;
        }
        if (!all_in && blockIdx.z != 0) continue;
        const int cp_lo = all_in ? blockIdx.z * nwarp : 0;
        const int cp_hi = all_in ? min(cp_lo + nwarp, D / 2) : D / 2;   // this CTA's channel pairs
        const int c_lo = 2 * cp_lo, nc = 2 * (cp_hi - cp_lo);
        for (int e = threadIdx.x; e < PG * nc; e += blockDim.x) {
            const int j = e / nc, c = c_lo + e % nc;
            const int idx = i - (PG - 1) + j;
            float val;
            if (idx >= 0 && p.slots[idx] == s0 + j) {
                val = ld_any(p.k, p.dt, (int64_t)idx * p.sk_t + (int64_t)h * p.sk_h + (int64_t)c * p.sk_d);
            } else {
                const uint8_t* row = row_at(p.kv, p.g, s0 + j, 0, h);
                val = __fmul_rn(code_value((row[c / 2] >> (4 * (c & 1))) & 0xF, p.fmt),
                                e4m3_to_f32(row[D / 2 + c / BLK]));
            }
            xs[j * D + c] = val;
        }
        __syncthreads();                                  // all rows read before any is rewritten
        for (int cp = cp_lo + warp; cp < cp_hi; cp += nwarp) {
            const int c = 2 * cp + u;
            float x[BLK];
#pragma unroll
            for (int t = 0; t < BLK; ++t) x[t] = xs[t * D + c];
            const uint8_t sc = calib_e4m3_hw(x, p.fmt, p.calib, a);
            const uint32_t nib = nibble_of(xs[a * D + c], e4m3_to_f32(sc), p.fmt);
            const uint32_t hi = __shfl_down_sync(0xffffffffu, nib, 16);
            if (u == 0) row_at(p.kv, p.g, s0 + a, 0, h)[cp] = (uint8_t)(nib | (hi << 4));
            if (a == 0) row_at(p.kv, p.g, s0 + c / ND, 0, h)[D / 2 + c % ND] = sc;
        }
        __syncthreads();
    }
}

// Gather-dequant: bf16 k/v [B, H, max_seq, D]; tokens at or past seq_len are 0.
struct GatherP {
    const uint8_t* kv; int64_t nb; Geo g; int fmt;
    const int* bt; int64_t bt_stride; const int* seq_lens;
    int B, max_seq;
    __nv_bfloat16* k_out; __nv_bfloat16* v_out; int* err;
};
__global__ void __launch_bounds__(128) gather_kernel(const GatherP p) {
    const int D = p.g.D, ND = D / BLK, H = p.g.H;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)p.B * H * p.max_seq * ND;
    if (tid >= total) return;
    const int db = (int)(tid % ND);
    const int t = (int)((tid / ND) % p.max_seq);
    const int h = (int)((tid / ((int64_t)ND * p.max_seq)) % H);
    const int b = (int)(tid / ((int64_t)ND * p.max_seq * H));
    const int64_t cap = p.bt_stride * PG;
    const int L = (int)(p.seq_lens[b] < 0 ? 0 : (p.seq_lens[b] > cap ? cap : p.seq_lens[b]));
    const int64_t o = (((int64_t)b * H + h) * p.max_seq + t) * D + db * BLK;
    __align__(16) __nv_bfloat16 kk[BLK], vv[BLK];
    if (t >= L) {
#pragma unroll
        for (int e = 0; e < BLK; ++e) kk[e] = vv[e] = __float2bfloat16_rn(0.0f);
    } else {
        const int pg = t / PG;
        int64_t phys = p.bt[(int64_t)b * p.bt_stride + pg];
        if (phys < 0 || phys >= p.nb) { set_err_flag(p.err, KIVI_ERR_ARG); phys = 0; }
        const int64_t slot = phys * PG + t % PG;
        const bool full = (pg + 1) * PG <= L;
        const uint8_t* kr = row_at(p.kv, p.g, slot, 0, h);
        const uint8_t* vr = row_at(p.kv, p.g, slot, 1, h);
        const float vs = e4m3_to_f32(vr[D / 2 + db]);
        const float ks_tok = e4m3_to_f32(kr[D / 2 + db]);
#pragma unroll
        for (int e = 0; e < BLK; ++e) {
            const int c = db * BLK + e;
            const uint32_t kb = kr[c / 2], vb = vr[c / 2];
            float ks = ks_tok;
            if (full) {
                const uint8_t* sr = row_at(p.kv, p.g, phys * PG + c / ND, 0, h);
                ks = e4m3_to_f32(sr[D / 2 + c % ND]);
            }
            kk[e] = __float2bfloat16_rn(__fmul_rn(code_value((kb >> (4 * (c & 1))) & 0xF, p.fmt), ks));
            vv[e] = __float2bfloat16_rn(__fmul_rn(code_value((vb >> (4 * (c & 1))) & 0xF, p.fmt), vs));
        }
    }
#pragma unroll
    for (int e = 0; e < BLK; ++e) { p.k_out[o + e] = kk[e]; p.v_out[o + e] = vv[e]; }
}

// ---------------------------------------------------------------------------
// Fused paged decode.
//
// Work = flattened (sequence, TP-block tile) list split evenly over a
// persistent grid of one CTA per SM.  A CTA has one consumer warp per KV head
// plus a producer warp; the producer moves whole blocks (K and V of a block
// are one contiguous 2 * 16 * H * FD byte range) into a ring of stages guarded
// by mbarriers, one TMA tensor load per block whose box rows are wider than
// the cache row, so token rows land at a bank-spreading smem pitch and every
// byte of the cache is read once, in full rows.  Consumer warp h runs, per
// 16-token block (TP blocks of a stage interleaved):
//   QK^T  m16n8k16 with the block's 16 tokens as M, the GQA heads as N; the
//         A fragments come from 64-bit shared loads of the token rows, the
//         channel order inside each k-step is permuted to match the nibble
//         order the fp16 magic / e2m1 cvt produce (Q uses the same order);
//   PV    with channels as M and tokens as K: two token rows are interleaved
//         with a byte permute so one 32-bit word yields (token, token) pairs;
//   code * e4m3 scale is exact in fp16 (3 + 4 significant bits), so the
//   scales are applied to the A operand and every product is exact.
// Softmax is online in base 2 with lazy rescaling; per-(CTA, sequence) partial
// states are merged by paged_merge_kernel.
// ---------------------------------------------------------------------------
constexpr int DD = 128;               // head_dim of the fast path
constexpr int FDD = 72;               // row bytes per head at D = 128
constexpr int TP = 5;                 // blocks per pipeline stage
constexpr int PNST = 6;               // most pipeline stages (the launch picks what fits)
constexpr int PBP = 16 * TP + 8;     // halves per head row of the P staging buffer
constexpr int MAX_H = 16;             // KV heads (consumer warps) of the fast path

struct DecP {
    const __nv_bfloat16* q; int64_t q_sb, q_sh;
    const uint8_t* kv; int64_t nb; Geo g;
    const int* bt; int64_t bt_stride; const int* seq_lens;
    int B, Hq, G;
    float scale2;                     // sm_scale * log2(e)
    int N;                            // CTAs of the main kernel
    int nst;                          // pipeline stages of this launch (<= PNST)
    int rowp;                         // smem pitch of a token row (>= H * FD)
    int use_tma;                      // 1: blocks arrive by TMA at the padded pitch
    float* part_m; float* part_l; float* part_acc;
    int* tile_off;                    // [B + 1]
    int* err;
    __nv_bfloat16* out;               // bf16 [B, Hq, D], or null
    float* out_f32;                   // fp32 [B, Hq, D] (normalised, before the bf16 cast), or null
};

__device__ __forceinline__ int seq_len_of(const DecP& p, int b) {
    const int64_t cap = p.bt_stride * PG;
    const int L = p.seq_lens[b];
    return L < 0 ? 0 : (L > cap ? (int)cap : L);
}
__host__ __device__ __forceinline__ int64_t pslice(int64_t c, int64_t W, int N) { return c * W / N; }

// tile_off[b] = sum over earlier sequences of ceil(ceil(L / 16) / TP).
__global__ void __launch_bounds__(1024) paged_tile_offsets_kernel(const DecP p) {
    __shared__ int part[1024];
    const int t = threadIdx.x;
    const int chunk = (p.B + 1023) / 1024, a = t * chunk, e = min(a + chunk, p.B);
    auto tiles = [&](int b) { const int np = (seq_len_of(p, b) + PG - 1) / PG; return (np + TP - 1) / TP; };
    int sum = 0;
    for (int b = a; b < e; ++b) sum += tiles(b);
    part[t] = sum;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        const int v = t >= o ? part[t - o] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    int run = part[t] - sum;
    for (int b = a; b < e; ++b) { p.tile_off[b] = run; run += tiles(b); }
    if (t == 1023) p.tile_off[p.B] = part[1023];
}

struct PCursor {
    int b, t, T;
    __device__ __forceinline__ void init(const DecP& p, int64_t i) {
        int lo = 0, hi = p.B - 1;                     // last b with tile_off[b] <= i
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.tile_off[mid] <= i) lo = mid; else hi = mid - 1;
        }
        b = lo;
        while (p.tile_off[b + 1] <= i) ++b;           // skip empty sequences
        t = (int)(i - p.tile_off[b]);
        T = p.tile_off[b + 1] - p.tile_off[b];
    }
    __device__ __forceinline__ void next(const DecP& p) {
        if (++t < T) return;
        t = 0;
        ++b;
        while (b < p.B && p.tile_off[b + 1] == p.tile_off[b]) ++b;
        T = b < p.B ? p.tile_off[b + 1] - p.tile_off[b] : 1;
    }
};

struct __align__(8) PCtl {
    uint64_t full[PNST];
    uint64_t empty[PNST];
    int abort;
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t e4m3_pair(uint32_t lo_byte, uint32_t hi_byte) {
    return e4m3x2_to_h2((uint16_t)(lo_byte | (hi_byte << 8)));
}
// Eight nibbles n0..n7 of a word -> fp16x2 (n0,n4), (n1,n5), (n2,n6), (n3,n7).
template <int FMT>
__device__ __forceinline__ void nib4(uint32_t w, uint32_t (&r)[4]) {
    if (FMT == FMT_NVFP4) {
        uint32_t h0, h1, h2, h3;
        e2m1x8_to_h2x4(w, h0, h1, h2, h3);
        r[0] = __byte_perm(h0, h2, 0x5410);
        r[1] = __byte_perm(h0, h2, 0x7632);
        r[2] = __byte_perm(h1, h3, 0x5410);
        r[3] = __byte_perm(h1, h3, 0x7632);
    } else {
        const uint32_t w8 = w >> 8;
        r[0] = h2_as_u32(int4_lo_to_h2(w));
        r[1] = h2_as_u32(int4_hi_to_h2(w));
        r[2] = h2_as_u32(int4_lo_to_h2(w8));
        r[3] = h2_as_u32(int4_hi_to_h2(w8));
    }
}

// NW = warps the launch may use (KV heads + the producer warp); it sets the
// register budget.
// QK A-operand words.  INT4 needs the magic's (n, n+4) nibble pairing; the
// e2m1 cvt yields adjacent pairs (c0,c1) (c2,c3) (c4,c5) (c6,c7) directly,
// and NVFP4 keeps that order (Q and the per-channel scales follow it).
template <int FMT>
__device__ __forceinline__ void nib4_qk(uint32_t w, uint32_t (&r)[4]) {
    if (FMT == FMT_NVFP4) e2m1x8_to_h2x4(w, r[0], r[1], r[2], r[3]);
    else nib4<FMT>(w, r);
}
// NVFP4 PV words: (token A, token B) e2m1 pairs built with one shift and one
// bit-select per word: even channels 0,2,4,6 -> E[0..3], odd 1,3,5,7 -> O[0..3].
__device__ __forceinline__ void e2m1_token_pairs(uint32_t wa, uint32_t wb, uint32_t (&E)[4], uint32_t (&O)[4]) {
    const uint32_t even = (wa & 0x0F0F0F0Fu) | ((wb << 4) & 0xF0F0F0F0u);
    const uint32_t odd = ((wa >> 4) & 0x0F0F0F0Fu) | (wb & 0xF0F0F0F0u);
    e2m1x8_to_h2x4(even, E[0], E[1], E[2], E[3]);
    e2m1x8_to_h2x4(odd, O[0], O[1], O[2], O[3]);
}

// INT4 PV words with the token-pair scale folded in: each nibble pair is moved
// to bits (4, 20), the fp16 magic gives 1024 + 16 u (u = n ^ 8), and one fma
// (v * s/16 - 72 s) yields n * s exactly (n * s has <= 8 significant bits,
// s/16 and 72 s are exact in fp16).  x holds two tokens' 4-nibble halves;
// r[i] = scaled channel i of both tokens.
__device__ __forceinline__ void int4_pairs_scaled(uint32_t x, uint32_t s16, uint32_t c72, uint32_t (&r)[4]) {
    const uint32_t w[4] = {x << 4, x, x >> 4, x >> 8};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t v = lop3_and_xor(w[i], 0x00F000F0u, 0x64806480u);
        r[i] = h2_as_u32(__hfma2(u32_as_h2(v), u32_as_h2(s16), u32_as_h2(c72)));
    }
}

template <int FMT, int NW>
__global__ void __launch_bounds__(NW * 32, 1) paged_decode_kernel(const __grid_constant__ CUtensorMap tm_kv,
                                                                  const DecP p) {
    extern __shared__ __align__(128) uint8_t psm_raw[];
    uint8_t* psm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(psm_raw) + 127) & ~uintptr_t(127));
    const int H = p.g.H, G = p.G;
    const int64_t PGB = p.g.PGB, ROWP = p.rowp;
    const int64_t SB = (int64_t)TP * 32 * ROWP;                       // stage bytes
    uint8_t* stages = psm;
    __half* pbuf = reinterpret_cast<__half*>(psm + p.nst * SB);        // [H][8][PBP]
    PCtl* ctl = reinterpret_cast<PCtl*>(pbuf + H * 8 * PBP);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const int64_t Wt = p.tile_off[p.B];
    const int64_t i0 = pslice(c, Wt, p.N), i1 = pslice(c + 1, Wt, p.N);
    if (i0 >= i1) return;                                             // idle CTA

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.nst; ++s) { mbar_init(&ctl->full[s], 1); mbar_init(&ctl->empty[s], H); }
        ctl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == H) {
        // ------------------------------ producer ------------------------------
        // One TMA load per block: a (rowp/8 x 16 x 2) box of 8-byte elements
        // whose rows are wider than the cache row, so each token row lands at
        // the padded smem pitch (the extra columns are out of bounds and
        // zero-filled, not read).  Without a tensor map (odd H) the block
        // arrives by one bulk copy at the natural pitch.
        if (lane == 0) {
            if (p.use_tma) prefetch_tmap(&tm_kv);
            int it = 0;
            PCursor cu;
            cu.init(p, i0);
            for (int64_t i = i0; i < i1; ++i, ++it, cu.next(p)) {
                const int s = it % p.nst;
                if (!mbar_wait_bounded(&ctl->empty[s], ((it / p.nst) & 1) ^ 1)) {
                    set_err_flag(p.err, KIVI_ERR_TIMEOUT);
                    ctl->abort = 1;
                    break;
                }
                if (ctl->abort) break;
                const int np = (seq_len_of(p, cu.b) + PG - 1) / PG;
                const int pg0 = cu.t * TP, npg = min(TP, np - pg0);
                uint8_t* st = stages + s * SB;
                mbar_arrive_expect_tx(&ctl->full[s], (uint32_t)(npg * 32 * ROWP));
                for (int j = 0; j < npg; ++j) {
                    int64_t phys = p.bt[(int64_t)cu.b * p.bt_stride + pg0 + j];
                    if (phys < 0 || phys >= p.nb) { set_err_flag(p.err, KIVI_ERR_ARG); phys = 0; }
                    if (p.use_tma) tma_load_3d(st + j * 32 * ROWP, &tm_kv, &ctl->full[s], 0, 0, (int)(phys * 2));
                    else bulk_g2s(st + j * 32 * ROWP, p.kv + phys * 2 * PGB, (uint32_t)(2 * PGB), &ctl->full[s]);
                }
            }
            for (int j = (it > p.nst ? it - p.nst : 0); j < it; ++j)
                if (!mbar_wait_bounded(&ctl->full[j % p.nst], (j / p.nst) & 1)) set_err_flag(p.err, KIVI_ERR_TIMEOUT);
        }
        return;
    }

    // ------------------------------- consumers --------------------------------
    const int h = warp, g = lane >> 2, tq = lane & 3;
    const uint32_t rowp = (uint32_t)p.rowp;
    const uint32_t pb = smem_u32(pbuf + warp * 8 * PBP);     // P staging [8 heads][PBP] halves
    const uint32_t abort_s = smem_u32(&ctl->abort);
    uint32_t qf[2][4][2];
    float acc[8][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    int cur = -1;

    auto flush = [&](int b) {
        float L0 = l0, L1 = l1;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            L0 += __shfl_xor_sync(0xffffffffu, L0, o);
            L1 += __shfl_xor_sync(0xffffffffu, L1, o);
        }
        const int64_t rec = ((int64_t)(c + b) * H + h) * G;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int n = 2 * tq + hh;
            if (n >= G) continue;
            if (g == 0) { p.part_m[rec + n] = hh ? m1 : m0; p.part_l[rec + n] = hh ? L1 : L0; }
            float* a = p.part_acc + (rec + n) * DD + 16 * g;
            if (FMT == FMT_NVFP4) {   // m-tile e holds channel 16g + {0,2,4,6,1,3,5,7}[e] (+8 for rows g+8)
#pragma unroll
                for (int r8 = 0; r8 < 2; ++r8) {
                    const int c = 2 * r8 + hh;
                    *reinterpret_cast<float4*>(a + 8 * r8) = make_float4(acc[0][c], acc[4][c], acc[1][c], acc[5][c]);
                    *reinterpret_cast<float4*>(a + 8 * r8 + 4) = make_float4(acc[2][c], acc[6][c], acc[3][c], acc[7][c]);
                }
            } else {                  // m-tile e holds channel 16g + e (+8 for rows g+8)
                *reinterpret_cast<float4*>(a) = make_float4(acc[0][hh], acc[1][hh], acc[2][hh], acc[3][hh]);
                *reinterpret_cast<float4*>(a + 4) = make_float4(acc[4][hh], acc[5][hh], acc[6][hh], acc[7][hh]);
                *reinterpret_cast<float4*>(a + 8) = make_float4(acc[0][2 + hh], acc[1][2 + hh], acc[2][2 + hh], acc[3][2 + hh]);
                *reinterpret_cast<float4*>(a + 12) = make_float4(acc[4][2 + hh], acc[5][2 + hh], acc[6][2 + hh], acc[7][2 + hh]);
            }
        }
    };

    int it = 0;
    PCursor cu;
    cu.init(p, i0);
    int Lb = 0;
    for (int64_t i = i0; i < i1; ++i, ++it, cu.next(p)) {
        const int b = cu.b;
        if (b != cur) {
            if (cur >= 0) flush(cur);
            cur = b;
            Lb = seq_len_of(p, b);
            m0 = m1 = -INFINITY; l0 = l1 = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e][0] = acc[e][1] = acc[e][2] = acc[e][3] = 0.f;
            // B fragments of Q in the permuted channel order of the K loads
            const __nv_bfloat16* qp = p.q + (int64_t)b * p.q_sb + (int64_t)(h * G + g) * p.q_sh;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    // k-slots (2tq, 2tq+1 | 2tq+8, 2tq+9) <-> channels (ch, ch+4 | ch+1, ch+5)
                    // for INT4, (ch, ch+1 | ch+2, ch+3) for NVFP4 (nib4_qk's order)
                    constexpr bool NV = FMT == FMT_NVFP4;
                    const int ch = 64 * cc + 16 * tq + 8 * (e >> 1) + (NV ? 4 : 2) * (e & 1);
                    uint32_t b0 = 0, b1 = 0;
                    if (g < G) {
                        b0 = h2_as_u32(__floats2half2_rn(__bfloat162float(qp[ch]), __bfloat162float(qp[ch + (NV ? 1 : 4)])));
                        b1 = h2_as_u32(__floats2half2_rn(__bfloat162float(qp[ch + (NV ? 2 : 1)]),
                                                         __bfloat162float(qp[ch + (NV ? 3 : 5)])));
                    }
                    qf[cc][e][0] = b0; qf[cc][e][1] = b1;
                }
        }
        const int s = it % p.nst;
        if (!mbar_wait_bounded(&ctl->full[s], (it / p.nst) & 1)) {
            set_err_flag(p.err, KIVI_ERR_TIMEOUT);
            sts32s(abort_s, 1u);
        }
        if (lds32s(abort_s)) break;
        const uint32_t st_s = smem_u32(stages + s * SB);
        const int pg0 = cu.t * TP;
        // All TP blocks of the stage are processed together (TP independent
        // MMA chains per phase); only a stage holding a sequence's partial or
        // missing last block takes the masked body.
        auto stage_body = [&](auto masked_tag) {
            constexpr bool MASKED = decltype(masked_tag)::value;
            int lim[TP];
#pragma unroll
            for (int j = 0; j < TP; ++j) lim[j] = MASKED ? Lb - (pg0 + j) * PG : PG;
            // ------------------------------ QK^T ------------------------------
            float sc[TP][4];
#pragma unroll
            for (int j = 0; j < TP; ++j) {
                sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
                const uint32_t kpg = st_s + (uint32_t)(j * 32 * rowp + h * FDD);
                const bool full = !MASKED || lim[j] >= PG;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const uint2 ra = lds64s(kpg + g * rowp + 32 * cc + 8 * tq);
                    const uint2 rb = lds64s(kpg + (g + 8) * rowp + 32 * cc + 8 * tq);
                    uint32_t A0[4], A1[4], B0[4], B1[4];
                    nib4_qk<FMT>(ra.x, A0); nib4_qk<FMT>(ra.y, A1); nib4_qk<FMT>(rb.x, B0); nib4_qk<FMT>(rb.y, B1);
                    uint32_t S[8], T0 = 0, T1 = 0;
                    if (full) {
#pragma unroll
                        for (int sw = 0; sw < 2; ++sw) {
                            const uint2 sr = lds64s(kpg + (8 * cc + 2 * tq + sw) * rowp + DD / 2);
                            // scale pairs in the A words' channel order: (s0,s4) (s1,s5) (s2,s6)
                            // (s3,s7) for INT4, (s0,s1) (s2,s3) (s4,s5) (s6,s7) for NVFP4
                            const uint32_t x = FMT == FMT_NVFP4 ? sr.x : __byte_perm(sr.x, sr.y, 0x5140);
                            const uint32_t y = FMT == FMT_NVFP4 ? sr.y : __byte_perm(sr.x, sr.y, 0x7362);
                            S[4 * sw + 0] = e4m3x2_to_h2((uint16_t)x);
                            S[4 * sw + 1] = e4m3x2_to_h2((uint16_t)(x >> 16));
                            S[4 * sw + 2] = e4m3x2_to_h2((uint16_t)y);
                            S[4 * sw + 3] = e4m3x2_to_h2((uint16_t)(y >> 16));
                        }
                    } else {
                        const uint32_t s0 = lds8s(kpg + g * rowp + DD / 2 + 4 * cc + tq);
                        const uint32_t s1 = lds8s(kpg + (g + 8) * rowp + DD / 2 + 4 * cc + tq);
                        T0 = e4m3_pair(s0, s0);
                        T1 = e4m3_pair(s1, s1);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int sw = e >> 1, k = 2 * (e & 1);
                        uint32_t a0 = sw ? A1[k] : A0[k], a2 = sw ? A1[k + 1] : A0[k + 1];
                        uint32_t a1 = sw ? B1[k] : B0[k], a3 = sw ? B1[k + 1] : B0[k + 1];
                        if (full) {
                            const uint32_t sa = S[4 * sw + k], sb = S[4 * sw + k + 1];
                            a0 = hmul2u(a0, sa); a1 = hmul2u(a1, sa); a2 = hmul2u(a2, sb); a3 = hmul2u(a3, sb);
                        } else {
                            a0 = hmul2u(a0, T0); a2 = hmul2u(a2, T0); a1 = hmul2u(a1, T1); a3 = hmul2u(a3, T1);
                        }
                        mma_f16(sc[j], a0, a1, a2, a3, qf[cc][e][0], qf[cc][e][1]);
                    }
                }
            }
            // ----------------------------- softmax ----------------------------
            // sc[j]: (token g, head 2tq), (g, 2tq+1), (g+8, 2tq), (g+8, 2tq+1)
            float x[TP][4];
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int j = 0; j < TP; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) x[j][e] = sc[j][e] * p.scale2;
                if (MASKED) {
                    if (g >= lim[j]) x[j][0] = x[j][1] = -INFINITY;
                    if (g + 8 >= lim[j]) x[j][2] = x[j][3] = -INFINITY;
                }
                mx0 = fmaxf(mx0, fmaxf(x[j][0], x[j][2]));
                mx1 = fmaxf(mx1, fmaxf(x[j][1], x[j][3]));
            }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            // the running reference max moves only when a score exceeds it by
            // more than 2^8, so p <= 256 stays exact in fp16 staging
            const bool need = (mx0 > m0 + 8.f) || (mx1 > m1 + 8.f);
            if (__any_sync(0xffffffffu, need)) {
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float al0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - mn0);
                const float al1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - mn1);
                m0 = mn0; m1 = mn1;
                l0 *= al0; l1 *= al1;
#pragma unroll
                for (int e = 0; e < 8; ++e) { acc[e][0] *= al0; acc[e][2] *= al0; acc[e][1] *= al1; acc[e][3] *= al1; }
            }
            const float r0 = (m0 == -INFINITY) ? 0.f : m0, r1 = (m1 == -INFINITY) ? 0.f : m1;
            // PV k-slot of token t: 2 (t & 3) + ((t >> 2) & 1) + 8 (t >> 3), so the
            // four rows one PV load touches (t = tq + 4i) sit in distinct banks
            const int ks = 2 * (g & 3) + ((g >> 2) & 1);
            __syncwarp();
#pragma unroll
            for (int j = 0; j < TP; ++j) {
                const float p0 = exp2f(x[j][0] - r0), p2 = exp2f(x[j][2] - r0);
                const float p1 = exp2f(x[j][1] - r1), p3 = exp2f(x[j][3] - r1);
                l0 += p0 + p2;
                l1 += p1 + p3;
                sts16s(pb + 2 * ((2 * tq) * PBP + 16 * j + ks), __float2half_rn(p0));
                sts16s(pb + 2 * ((2 * tq + 1) * PBP + 16 * j + ks), __float2half_rn(p1));
                sts16s(pb + 2 * ((2 * tq) * PBP + 16 * j + ks + 8), __float2half_rn(p2));
                sts16s(pb + 2 * ((2 * tq + 1) * PBP + 16 * j + ks + 8), __float2half_rn(p3));
            }
            __syncwarp();
            // ------------------------------- PV -------------------------------
#pragma unroll
            for (int j = 0; j < TP; ++j) {
                const uint32_t vpg = st_s + (uint32_t)((j * 32 + 16) * rowp + h * FDD);
                const uint32_t b0 = lds32s(pb + 2 * (g * PBP + 16 * j + 2 * tq));
                const uint32_t b1 = lds32s(pb + 2 * (g * PBP + 16 * j + 2 * tq + 8));
                // k-slots (2tq, 2tq+1) = tokens (tq, tq+4); (2tq+8, 2tq+9) = (tq+8, tq+12)
                const int tA = tq, tB = tq + 4, tC = tq + 8, tD = tq + 12;
                const uint2 wa = lds64s(vpg + tA * rowp + 8 * g), wb = lds64s(vpg + tB * rowp + 8 * g);
                const uint2 wc = lds64s(vpg + tC * rowp + 8 * g), wd = lds64s(vpg + tD * rowp + 8 * g);
                uint32_t sA = lds8s(vpg + tA * rowp + DD / 2 + g), sB = lds8s(vpg + tB * rowp + DD / 2 + g);
                uint32_t sC = lds8s(vpg + tC * rowp + DD / 2 + g), sD = lds8s(vpg + tD * rowp + DD / 2 + g);
                if (MASKED) {                 // rows past the end may be unwritten (NaN scales)
                    sA = tA < lim[j] ? sA : 0u; sB = tB < lim[j] ? sB : 0u;
                    sC = tC < lim[j] ? sC : 0u; sD = tD < lim[j] ? sD : 0u;
                }
                const uint32_t sAB = e4m3_pair(sA, sB), sCD = e4m3_pair(sC, sD);
                uint32_t X0[4], Y0[4], X1[4], Y1[4], U0[4], V0[4], U1[4], V1[4];
                if (FMT == FMT_NVFP4) {       // X/U: channels 16g+{0,2,4,6}, Y/V: 16g+{1,3,5,7} (+8 in X1..V1)
                    e2m1_token_pairs(wa.x, wb.x, X0, Y0);
                    e2m1_token_pairs(wa.y, wb.y, X1, Y1);
                    e2m1_token_pairs(wc.x, wd.x, U0, V0);
                    e2m1_token_pairs(wc.y, wd.y, U1, V1);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const uint32_t a0 = hmul2u(e < 4 ? X0[e & 3] : Y0[e & 3], sAB);   // row g
                        const uint32_t a1 = hmul2u(e < 4 ? X1[e & 3] : Y1[e & 3], sAB);   // row g+8
                        const uint32_t a2 = hmul2u(e < 4 ? U0[e & 3] : V0[e & 3], sCD);
                        const uint32_t a3 = hmul2u(e < 4 ? U1[e & 3] : V1[e & 3], sCD);
                        mma_f16(acc[e], a0, a1, a2, a3, b0, b1);
                    }
                } else {                      // X/U: channels 16g+0..3, Y/V: 16g+4..7 (+8 in X1..V1), scaled
                    const uint32_t s16AB = hmul2u(sAB, 0x2C002C00u), c72AB = hmul2u(sAB, 0xD480D480u);   // s/16, -72 s
                    const uint32_t s16CD = hmul2u(sCD, 0x2C002C00u), c72CD = hmul2u(sCD, 0xD480D480u);
                    int4_pairs_scaled(__byte_perm(wa.x, wb.x, 0x5410), s16AB, c72AB, X0);   // tokens (tA, tB)
                    int4_pairs_scaled(__byte_perm(wa.x, wb.x, 0x7632), s16AB, c72AB, Y0);
                    int4_pairs_scaled(__byte_perm(wa.y, wb.y, 0x5410), s16AB, c72AB, X1);
                    int4_pairs_scaled(__byte_perm(wa.y, wb.y, 0x7632), s16AB, c72AB, Y1);
                    int4_pairs_scaled(__byte_perm(wc.x, wd.x, 0x5410), s16CD, c72CD, U0);   // tokens (tC, tD)
                    int4_pairs_scaled(__byte_perm(wc.x, wd.x, 0x7632), s16CD, c72CD, V0);
                    int4_pairs_scaled(__byte_perm(wc.y, wd.y, 0x5410), s16CD, c72CD, U1);
                    int4_pairs_scaled(__byte_perm(wc.y, wd.y, 0x7632), s16CD, c72CD, V1);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        mma_f16(acc[e], e < 4 ? X0[e & 3] : Y0[e & 3], e < 4 ? X1[e & 3] : Y1[e & 3],
                                e < 4 ? U0[e & 3] : V0[e & 3], e < 4 ? U1[e & 3] : V1[e & 3], b0, b1);
                }
            }
        };
        if ((pg0 + TP) * PG <= Lb) stage_body(std::false_type{});
        else stage_body(std::true_type{});
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->empty[s]);
    }
    if (cur >= 0 && !lds32s(abort_s)) flush(cur);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Merge of the per-(CTA, sequence) partial states of one (sequence, kv head,
// q head); one 128-thread block each.  Sequences of length 0 give zeros.
__global__ void __launch_bounds__(128) paged_merge_kernel(const DecP p) {
    extern __shared__ __align__(16) float msm[];
    const int b = blockIdx.x / p.g.H, h = blockIdx.x % p.g.H, n = blockIdx.y;
    const int G = p.G, D = DD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t Wt = p.tile_off[p.B];
    const int64_t a0 = p.tile_off[b], a1 = p.tile_off[b + 1];
    // CTA c owns tiles [floor(cW/N), floor((c+1)W/N)): the first CTA holding
    // tile a0 is the last with cW < (a0+1)N, the last holding a1-1 the last
    // with cW < a1 N
    int c_lo = 0, c_hi = -1;
    if (Wt > 0 && a1 > a0) {
        const int64_t lo = ((a0 + 1) * p.N - 1) / Wt, hi = (a1 * p.N - 1) / Wt;
        c_lo = (int)(lo < p.N - 1 ? lo : p.N - 1);
        c_hi = (int)(hi < p.N - 1 ? hi : p.N - 1);
    }
    const int ns = c_hi - c_lo + 1;
    float* w = msm;                       // [ns], padded to a multiple of 4
    float* red = msm + ((ns + 3) & ~3);   // [8]
    float* sacc = red + 8;                // [4][D], 16-byte aligned for float4
    auto rec = [&](int k) -> int64_t { return ((int64_t)(c_lo + k + b) * p.g.H + h) * G + n; };
    // CTAs with an empty slice (grids sized from bt_stride) wrote no record
    auto live = [&](int k) -> bool { return pslice(c_lo + k, Wt, p.N) < pslice(c_lo + k + 1, Wt, p.N); };
    for (int k = threadIdx.x; k < ns; k += blockDim.x) w[k] = live(k) ? p.part_m[rec(k)] : -INFINITY;
    __syncthreads();
    float M = -INFINITY;
    for (int k = threadIdx.x; k < ns; k += blockDim.x) M = fmaxf(M, w[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0) red[warp] = M;
    __syncthreads();
    M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float Mr = (M == -INFINITY) ? 0.f : M;
    __syncthreads();
    float Ls = 0.f;
    for (int k = threadIdx.x; k < ns; k += blockDim.x) {
        const float e = exp2f(w[k] - Mr);
        Ls += e != 0.f ? p.part_l[rec(k)] * e : 0.f;
        w[k] = e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
    if (lane == 0) red[4 + warp] = Ls;
    __syncthreads();
    Ls = (red[4] + red[5]) + (red[6] + red[7]);
    // four independent record loads in flight per warp iteration
    float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = warp; k0 < ns; k0 += 16) {
        float4 v4[4];
        float wk[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = k0 + 4 * u;
            wk[u] = k < ns ? w[k] : 0.f;
            v4[u] = wk[u] != 0.f ? *reinterpret_cast<const float4*>(p.part_acc + rec(k) * D + 4 * lane)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            a4.x += v4[u].x * wk[u]; a4.y += v4[u].y * wk[u]; a4.z += v4[u].z * wk[u]; a4.w += v4[u].w * wk[u];
        }
    }
    *reinterpret_cast<float4*>(sacc + warp * D + 4 * lane) = a4;
    __syncthreads();
    const int d = threadIdx.x;
    const float a = (sacc[d] + sacc[D + d]) + (sacc[2 * D + d] + sacc[3 * D + d]);
    const int64_t row = (int64_t)b * p.Hq + h * G + n;
    const float o = ns > 0 && Ls > 0.f ? a / Ls : 0.f;
    if (p.out) p.out[row * D + d] = __float2bfloat16_rn(o);
    if (p.out_f32) p.out_f32[row * D + d] = o;
}

// Any head_dim (multiple of 16, <= 256), group <= 16: one CTA per (sequence,
// kv head), four warps stride over the blocks, CUDA-core arithmetic, the four
// warp states merged in shared memory.
constexpr int GP_MAXG = 16, GP_MAXC = 8;
template <int FMT>
__global__ void __launch_bounds__(128) paged_decode_generic_kernel(const DecP p) {
    __shared__ float sm_m[4][GP_MAXG], sm_l[4][GP_MAXG];
    extern __shared__ float sm_acc[];                 // [4][G][D]
    const int b = blockIdx.x / p.g.H, h = blockIdx.x % p.g.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G, D = p.g.D, ND = D / BLK;
    const int L = seq_len_of(p, b);
    float q[GP_MAXG][GP_MAXC], acc[GP_MAXG][GP_MAXC], m[GP_MAXG], l[GP_MAXG];
    for (int n = 0; n < G; ++n) {
        m[n] = -INFINITY; l[n] = 0.f;
        const __nv_bfloat16* qp = p.q + (int64_t)b * p.q_sb + (int64_t)(h * G + n) * p.q_sh;
        for (int e = 0; e < GP_MAXC; ++e) {
            const int d = lane + 32 * e;
            q[n][e] = d < D ? __bfloat162float(qp[d]) : 0.f;
            acc[n][e] = 0.f;
        }
    }
    const float sc2 = p.scale2;
    for (int t = warp; t < L; t += 4) {
        const int pg = t / PG;
        int64_t phys = p.bt[(int64_t)b * p.bt_stride + pg];
        if (phys < 0 || phys >= p.nb) { set_err_flag(p.err, KIVI_ERR_ARG); phys = 0; }
        const bool full = (pg + 1) * PG <= L;
        const uint8_t* kr = row_at(p.kv, p.g, phys * PG + t % PG, 0, h);
        const uint8_t* vr = row_at(p.kv, p.g, phys * PG + t % PG, 1, h);
        float kv[GP_MAXC], vv[GP_MAXC];
        for (int e = 0; e < GP_MAXC; ++e) {
            const int d = lane + 32 * e;
            kv[e] = vv[e] = 0.f;
            if (d < D) {
                float ks = e4m3_to_f32(kr[D / 2 + d / BLK]);
                if (full) ks = e4m3_to_f32(row_at(p.kv, p.g, phys * PG + d / ND, 0, h)[D / 2 + d % ND]);
                kv[e] = code_value((kr[d / 2] >> (4 * (d & 1))) & 0xF, FMT) * ks;
                vv[e] = code_value((vr[d / 2] >> (4 * (d & 1))) & 0xF, FMT) * e4m3_to_f32(vr[D / 2 + d / BLK]);
            }
        }
        for (int n = 0; n < G; ++n) {
            float s = 0.f;
            for (int e = 0; e < GP_MAXC; ++e) s += q[n][e] * kv[e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            s *= sc2;
            const float mn = fmaxf(m[n], s);
            const float al = exp2f(m[n] - mn), pr = exp2f(s - mn);
            m[n] = mn;
            l[n] = l[n] * al + pr;
            for (int e = 0; e < GP_MAXC; ++e) acc[n][e] = acc[n][e] * al + pr * vv[e];
        }
    }
    for (int n = 0; n < G; ++n) {
        if (lane == 0) { sm_m[warp][n] = m[n]; sm_l[warp][n] = l[n]; }
        for (int e = 0; e < GP_MAXC; ++e) {
            const int d = lane + 32 * e;
            if (d < D) sm_acc[(warp * G + n) * D + d] = acc[n][e];
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int n = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w2 = 0; w2 < 4; ++w2) M = fmaxf(M, sm_m[w2][n]);
        const float Mr = (M == -INFINITY) ? 0.f : M;
        float Ls = 0.f, a = 0.f;
        for (int w2 = 0; w2 < 4; ++w2) {
            const float e = exp2f(sm_m[w2][n] - Mr);
            Ls += sm_l[w2][n] * e;
            a += sm_acc[(w2 * G + n) * D + d] * e;
        }
        const float o = Ls > 0.f ? a / Ls : 0.f;
        const int64_t oi = ((int64_t)b * p.Hq + h * G + n) * D + d;
        if (p.out) p.out[oi] = __float2bfloat16_rn(o);
        if (p.out_f32) p.out_f32[oi] = o;
    }
}

}  // namespace paged
}  // namespace kivi

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {
using namespace kivi;
using namespace kivi::paged;

constexpr int PAGED_MAX_OCC = 4;

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn paged_encode_fn() {
    static EncodeFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(ptr);
    }
    return fn;
}

// smem pitch of a token row: H * FD rounded up so that consecutive rows start
// 24 or 8 words apart mod 32 (rows g..g+3 then cover distinct banks).  The
// padded pitch needs the TMA path (rows of whole 16-byte multiples, even H);
// odd H keeps the natural pitch.
bool paged_tma_ok(int H) { return (H * FDD) % 16 == 0; }
int paged_rowp(int H) {
    const int rb = H * FDD;
    if (!paged_tma_ok(H)) return rb;
    for (int pad = 0; pad < 128; pad += 16) {
        const int w = ((rb + pad) / 4) % 32;
        if (w == 8 || w == 24) return rb + pad;
    }
    return rb;
}
size_t paged_stage_bytes(int H) { return (size_t)TP * 32 * paged_rowp(H); }
size_t paged_fixed_bytes(int H) { return (size_t)H * 8 * PBP * sizeof(__half) + sizeof(PCtl) + 16 + 128; }
// As many stages as fit one CTA's shared memory (227 KB on sm_100), at most PNST.
int paged_stages(int H) {
    const size_t cap = 232448, fixed = paged_fixed_bytes(H), sb = paged_stage_bytes(H);
    const int n = (int)((cap - fixed) / sb);
    return n < PNST ? n : PNST;
}
size_t paged_smem(int H) { return paged_stages(H) * paged_stage_bytes(H) + paged_fixed_bytes(H); }

int cur_device_sms(int* dev_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    static int sms[64] = {0};
    if (dev < 0 || dev >= 64) return 0;
    if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (dev_out) *dev_out = dev;
    return sms[dev];
}

template <int FMT, int NW>
int paged_occupancy(int dev, int H) {
    static int occ[64][MAX_H + 1] = {{0}};
    static bool attr[64] = {false};
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(paged_decode_kernel<FMT, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 232448) != cudaSuccess)
            return 0;
        attr[dev] = true;
    }
    if (!occ[dev][H]) {
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, paged_decode_kernel<FMT, NW>, (H + 1) * 32,
                                                          paged_smem(H)) != cudaSuccess)
            return 0;
        occ[dev][H] = o > 0 ? (o < PAGED_MAX_OCC ? o : PAGED_MAX_OCC) : 1;
    }
    return occ[dev][H];
}

struct PagedPlan { int64_t W; int N; int64_t records; int64_t off_m, off_l, off_acc, floats; };
PagedPlan paged_plan(int B, int Hkv, int G, int64_t bt_stride, int D, int sms, int occ) {
    PagedPlan pl;
    pl.W = (int64_t)B * ((bt_stride + TP - 1) / TP);
    const int64_t cap = (int64_t)sms * occ;
    pl.N = (int)(pl.W < cap ? pl.W : cap);
    if (pl.N < 1) pl.N = 1;
    pl.records = ((int64_t)pl.N + B) * Hkv * G;
    pl.off_m = ((int64_t)B + 1 + 3) / 4 * 4;           // tile table first (int32 in float slots)
    pl.off_l = pl.off_m + pl.records;
    pl.off_acc = (pl.off_l + pl.records + 3) / 4 * 4;
    pl.floats = pl.off_acc + pl.records * D;
    return pl;
}

bool dtype_ok(int dt) { return dt == KIVI_DT_BF16 || dt == KIVI_DT_F16 || dt == KIVI_DT_F32; }
bool fmt_ok(int fmt) { return fmt == FMT_INT4 || fmt == FMT_NVFP4; }
}  // namespace

extern "C" int kivi_paged_full_dim(int D) { return D > 0 && D % 16 == 0 ? full_dim(D) : 0; }

extern "C" int kivi_paged_store(const void* k, const void* v, int in_dtype, int64_t sk_t, int64_t sk_h,
                                int64_t sk_d, int64_t sv_t, int64_t sv_h, int64_t sv_d, int N, int H, int D,
                                int fmt, int calib, const int64_t* slot_mapping, uint8_t* kv_cache,
                                int64_t num_blocks, int* err, kivi_stream_t stream) {
    if (N < 0 || H <= 0 || D <= 0 || D % 16 || D > 256 || !fmt_ok(fmt) || !dtype_ok(in_dtype)) return KIVI_ERR_ARG;
    if (calib != CAL_ABSMAX && calib != CAL_MSE) return KIVI_ERR_ARG;
    if (N == 0) return KIVI_OK;
    if (!k || !v || !slot_mapping || !kv_cache || num_blocks <= 0) return KIVI_ERR_ARG;
    StoreP p{};
    p.k = k; p.v = v; p.dt = in_dtype;
    p.sk_t = sk_t; p.sk_h = sk_h; p.sk_d = sk_d; p.sv_t = sv_t; p.sv_h = sv_h; p.sv_d = sv_d;
    p.N = N; p.g = make_geo(H, D); p.fmt = fmt; p.calib = calib;
    p.slots = slot_mapping; p.kv = kv_cache; p.nb = num_blocks; p.err = err;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t halves = (int64_t)N * H * 2 * (D / BLK);          // one half-warp per block
    store_token_kernel<<<(unsigned)((halves * 16 + 255) / 256), 256, 0, st>>>(p);
    int e = check_launch();
    if (e) return e;
    store_channel_kernel<<<dim3((unsigned)((N + PG - 1) / PG), (unsigned)H, (unsigned)((D / 2 + 15) / 16)), 512,
                           (size_t)PG * D * sizeof(float), st>>>(p);
    return check_launch();
}

extern "C" int kivi_paged_gather_dequant(const uint8_t* kv_cache, int64_t num_blocks, const int* block_table,
                                         int64_t bt_stride, const int* seq_lens, int B, int H, int D, int fmt,
                                         int max_seq, void* k_out, void* v_out, int* err,
                                         kivi_stream_t stream) {
    if (B < 0 || H <= 0 || D <= 0 || D % 16 || !fmt_ok(fmt) || max_seq < 0 || bt_stride < 0) return KIVI_ERR_ARG;
    if (B == 0 || max_seq == 0) return KIVI_OK;
    if (!kv_cache || !block_table || !seq_lens || !k_out || !v_out || num_blocks <= 0) return KIVI_ERR_ARG;
    GatherP p{};
    p.kv = kv_cache; p.nb = num_blocks; p.g = make_geo(H, D); p.fmt = fmt;
    p.bt = block_table; p.bt_stride = bt_stride; p.seq_lens = seq_lens; p.B = B; p.max_seq = max_seq;
    p.k_out = reinterpret_cast<__nv_bfloat16*>(k_out); p.v_out = reinterpret_cast<__nv_bfloat16*>(v_out);
    p.err = err;
    const int64_t total = (int64_t)B * H * max_seq * (D / BLK);
    gather_kernel<<<(unsigned)((total + 127) / 128), 128, 0, (cudaStream_t)stream>>>(p);
    return check_launch();
}

extern "C" int64_t kivi_paged_decode_workspace_floats(int B, int Hq, int Hkv, int64_t bt_stride, int D) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || bt_stride < 0 || D <= 0) return 0;
    int sms = cur_device_sms(nullptr);
    if (!sms) sms = 148;
    return paged_plan(B, Hkv, Hq / Hkv, bt_stride, D, sms, PAGED_MAX_OCC).floats;
}

namespace {
int paged_decode_impl(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* kv_cache, int64_t num_blocks,
                      const int* block_table, int64_t bt_stride, const int* seq_lens, int B, int Hq, int Hkv,
                      int D, int fmt, float sm_scale, void* out, float* out_f32, float* work,
                      int64_t work_floats, int* err, kivi_stream_t stream) {
    if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || D <= 0 || D % 16 || D > 256 || !fmt_ok(fmt) || bt_stride < 0)
        return KIVI_ERR_ARG;
    if (B == 0) return KIVI_OK;
    if (!q || !kv_cache || !block_table || !seq_lens || (!out && !out_f32) || num_blocks <= 0) return KIVI_ERR_ARG;
    const int G = Hq / Hkv;
    int dev = 0;
    const int sms = cur_device_sms(&dev);
    if (!sms) return record_cuda_error(cudaGetLastError());
    DecP p{};
    p.q = reinterpret_cast<const __nv_bfloat16*>(q); p.q_sb = q_sb; p.q_sh = q_sh;
    p.kv = kv_cache; p.nb = num_blocks; p.g = make_geo(Hkv, D);
    p.bt = block_table; p.bt_stride = bt_stride; p.seq_lens = seq_lens;
    p.B = B; p.Hq = Hq; p.G = G;
    p.scale2 = sm_scale * 1.4426950408889634f;
    p.err = err; p.out = reinterpret_cast<__nv_bfloat16*>(out); p.out_f32 = out_f32;
    cudaStream_t st = (cudaStream_t)stream;
    const bool fast = D == DD && Hkv <= MAX_H && G <= 8 && (uintptr_t)kv_cache % 16 == 0 &&
                      (uintptr_t)q % 4 == 0 && q_sh % 2 == 0 && q_sb % 2 == 0;
    if (!fast) {
        if (G > GP_MAXG || D > 32 * GP_MAXC) return KIVI_ERR_UNSUPPORTED;
        const size_t smem = (size_t)4 * G * D * sizeof(float);
        if (smem > 48 * 1024) {
            cudaError_t ae = (fmt == FMT_NVFP4)
                ? cudaFuncSetAttribute(paged_decode_generic_kernel<FMT_NVFP4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                : cudaFuncSetAttribute(paged_decode_generic_kernel<FMT_INT4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (ae != cudaSuccess) return record_cuda_error(ae);
        }
        if (fmt == FMT_NVFP4) paged_decode_generic_kernel<FMT_NVFP4><<<B * Hkv, 128, smem, st>>>(p);
        else paged_decode_generic_kernel<FMT_INT4><<<B * Hkv, 128, smem, st>>>(p);
        return check_launch();
    }
    const bool wide = Hkv > 8;
    const int occ = fmt == FMT_NVFP4 ? (wide ? paged_occupancy<FMT_NVFP4, 17>(dev, Hkv) : paged_occupancy<FMT_NVFP4, 9>(dev, Hkv))
                                     : (wide ? paged_occupancy<FMT_INT4, 17>(dev, Hkv) : paged_occupancy<FMT_INT4, 9>(dev, Hkv));
    if (!occ) return record_cuda_error(cudaGetLastError());
    const PagedPlan pl = paged_plan(B, Hkv, G, bt_stride, D, sms, occ);
    if (!work || work_floats < pl.floats) return KIVI_ERR_ARG;
    p.N = pl.N;
    p.nst = paged_stages(Hkv);
    p.rowp = paged_rowp(Hkv);
    p.use_tma = paged_tma_ok(Hkv) && (uintptr_t)kv_cache % 16 == 0 && 2 * num_blocks < (1LL << 31);
    CUtensorMap tm;
    memset(&tm, 0, sizeof(tm));
    if (p.use_tma) {
        // [2 * num_blocks][16 rows][H * FD / 8] of 8-byte elements; box rows
        // are rowp / 8 elements wide (the tail past H * FD is zero fill)
        EncodeFn enc = paged_encode_fn();
        cuuint64_t dims[3] = {(cuuint64_t)(Hkv * FDD / 8), (cuuint64_t)PG, (cuuint64_t)(2 * num_blocks)};
        cuuint64_t strides[2] = {(cuuint64_t)(Hkv * FDD), (cuuint64_t)(PG * Hkv * FDD)};
        cuuint32_t box[3] = {(cuuint32_t)(p.rowp / 8), (cuuint32_t)PG, 2u};
        cuuint32_t es[3] = {1, 1, 1};
        if (!enc || enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(kv_cache), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KIVI_ERR_CUDA;
    }
    p.tile_off = reinterpret_cast<int*>(work);
    p.part_m = work + pl.off_m; p.part_l = work + pl.off_l; p.part_acc = work + pl.off_acc;
    paged_tile_offsets_kernel<<<1, 1024, 0, st>>>(p);
    int e = check_launch();
    if (e) return e;
    const size_t smem = paged_smem(Hkv);
    const dim3 blk((Hkv + 1) * 32);
    if (fmt == FMT_NVFP4 && wide) paged_decode_kernel<FMT_NVFP4, 17><<<pl.N, blk, smem, st>>>(tm, p);
    else if (fmt == FMT_NVFP4) paged_decode_kernel<FMT_NVFP4, 9><<<pl.N, blk, smem, st>>>(tm, p);
    else if (wide) paged_decode_kernel<FMT_INT4, 17><<<pl.N, blk, smem, st>>>(tm, p);
    else paged_decode_kernel<FMT_INT4, 9><<<pl.N, blk, smem, st>>>(tm, p);
    e = check_launch();
    if (e) return e;
    // a sequence's tiles touch at most N + 1 CTAs
    const size_t msm = ((size_t)pl.N + 4 + 8 + 4 * DD) * sizeof(float);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * Hkv), (unsigned)G);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = msm;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (msm > 48 * 1024) {
        cudaError_t ae = cudaFuncSetAttribute(paged_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msm);
        if (ae != cudaSuccess) return record_cuda_error(ae);
    }
    cudaError_t le = cudaLaunchKernelEx(&cfg, paged_merge_kernel, p);
    if (le != cudaSuccess) return record_cuda_error(le);
    return check_launch();
}
}  // namespace

extern "C" int kivi_paged_decode(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* kv_cache,
                                 int64_t num_blocks, const int* block_table, int64_t bt_stride,
                                 const int* seq_lens, int B, int Hq, int Hkv, int D, int fmt, float sm_scale,
                                 void* out, float* work, int64_t work_floats, int* err, kivi_stream_t stream) {
    if (!out) return KIVI_ERR_ARG;
    return paged_decode_impl(q, q_sb, q_sh, kv_cache, num_blocks, block_table, bt_stride, seq_lens, B, Hq, Hkv, D,
                             fmt, sm_scale, out, nullptr, work, work_floats, err, stream);
}

extern "C" int kivi_paged_decode_f32(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* kv_cache,
                                     int64_t num_blocks, const int* block_table, int64_t bt_stride,
                                     const int* seq_lens, int B, int Hq, int Hkv, int D, int fmt, float sm_scale,
                                     float* out, float* work, int64_t work_floats, int* err,
                                     kivi_stream_t stream) {
    if (!out) return KIVI_ERR_ARG;
    return paged_decode_impl(q, q_sb, q_sh, kv_cache, num_blocks, block_table, bt_stride, seq_lens, B, Hq, Hkv, D,
                             fmt, sm_scale, nullptr, out, work, work_floats, err, stream);
}
