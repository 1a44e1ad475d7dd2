// kivi_decode.cu -- fused split-K flash-decode over a packed INT4/NVFP4 KIVI cache.
//
// Replaces the reference's Triton decode path (int4_kivi/decode.py:53-477):
// per (sequence, kv-head) the full 16-token pages are streamed once, every
// query head of the GQA group is served from the same bytes, and a second
// launch merges the per-warp partial softmax states with log-sum-exp (the
// reference's _combine_kernel, decode.py:320-340) and adds the bf16 hot tail.
//
// Fast path (D = 128, GQA group <= 8, 16-aligned strides):
//   * work = flattened (head, 128-token tile) list split evenly over a
//     persistent grid (stream-K style), so every SM gets the same bytes;
//   * warp 4 issues TMA tile loads (K codes/scales, V codes/scales) into a
//     3-stage ring guarded by mbarriers; warps 0-3 each own 32 tokens of a
//     tile;
//   * packed nibbles go smem -> registers with ldmatrix.trans, which pairs
//     two channels (K) or two tokens (V) per 32-bit word; a LOP3 fp16 magic
//     (INT4) or the hardware e2m1 -> f16x2 cvt (NVFP4) yields exact codes,
//     which are scaled by per-page / per-token scale pairs;
//   * QK^T and PV run on mma.sync m16n8k16 (f16 in, f32 accumulate) with the
//     query heads as the N=8 side; for INT4 the fp16 scale is split into an
//     8-bit head and a 3-bit tail so every product is exact (two MMAs);
//   * online softmax in base 2 with warp-shuffle row maxima.
#include "kivi_common.cuh"
#include "kivi_internal.h"
#include <cuda.h>
#include <mutex>
#include <algorithm>
#include <type_traits>

namespace kivi {

constexpr int TILE = 128;        // tokens per pipeline stage (8 pages)
constexpr int NWARP_C = 4;       // consumer warps, 32 tokens each
constexpr int NTHREADS = (NWARP_C + 1) * 32;
constexpr int NST = 3;           // pipeline depth
constexpr int CTAS_PER_SM = 3;   // resident CTAs the register budget is sized for
constexpr int DH = 128;          // head_dim of the fast path
constexpr int PB_PITCH = 40;     // halves per head row in the P staging buffer

struct DecodeParams {
    const __nv_bfloat16* q; int64_t q_sb, q_sh;
    // multi-query decode: Tq query tokens per sequence (stride q_st), the
    // kernels' group G = Tq * Gq covers (query, head) pairs; Gq / Hq0 are the
    // real GQA group and q-head count.  Tq = 1 is the plain decode.
    int64_t q_st; int Tq, Gq, Hq0;
    int mq;                  // 1: multi-query (per-query causal limits), 0: plain decode
    int q_pos;               // multi-query: query j sits at q_pos + j and sees tokens 0 .. q_pos + j
    int nf_real;             // full-page tokens of the cache (the split kernels may see fewer)
    const uint8_t* k_packed; const void* k_scale; int k_np_stride;
    const __nv_bfloat16* k_hot; int hot_stride;
    const uint8_t* v_packed; const void* v_scale; int v_s_stride;
    int B, Hq, Hkv, G, S, D, n_full, hot;
    float scale2;        // sm_scale * log2(e) (* g_k for NVFP4)
    float g_v;
    float sm_scale, g_k;
    int T;               // tiles per head
    int64_t W;           // total tiles
    int N;               // CTAs of the main kernel
    float* part_m; float* part_l; float* part_acc;
    int* err;
    // varlen: per-sequence lengths (device, nullable) and the per-head tile
    // offsets [B*Hkv + 1] the prologue kernel derives from them
    const int* seq_lens;
    int* tile_off;
    // optional bf16 V of the tail tokens [BH, hot_stride, D] (caches that keep
    // the partial page unquantised); nullptr = the tail's V comes from v_packed
    const __nv_bfloat16* v_hot;
    // mode 2 (sequence-parallel exchange): this rank's exchange buffer, the
    // device array of all ranks' buffers, per-row epoch counters
    uint8_t* xbuf;
    const uint64_t* peers;
    int xW, xrank;                   // ranks in the exchange, this rank
    unsigned int* row_epoch;
    long long timeout_ns;
};

struct SeqPar {
    uint8_t* xbuf; const uint64_t* peers; int W, rank; unsigned int* row_epoch; long long timeout_ns;
};

// Exchange buffer of the fused sequence-parallel combine (mode 2):
//   flags uint32 [W][rows] (flag[j][row] = newest epoch rank j published for
//   the row), padded to 256 B, then two slots of fp32 m [rows], l [rows],
//   acc [rows][D]; epoch e of a row uses slot e & 1.
__host__ __device__ inline int64_t xflag_bytes(int W, int rows) { return ((int64_t)W * rows * 4 + 255) / 256 * 256; }
__host__ __device__ inline int64_t xslot_floats(int rows, int D) { return (int64_t)rows * (2 + D); }
__device__ __forceinline__ float* xslot(uint8_t* base, int W, int rows, int D, unsigned int e) {
    return reinterpret_cast<float*>(base + xflag_bytes(W, rows)) + (e & 1) * xslot_floats(rows, D);
}
__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__host__ __device__ inline int64_t tile_start(int64_t c, int64_t W, int N) { return c * W / N; }

// Per-head geometry: uniform caches use (S, n_full, hot, T); varlen caches
// read the sequence length of the head's batch entry.
__device__ __forceinline__ int head_len(const DecodeParams& p, int bh) {
    return p.seq_lens ? min(max(p.seq_lens[bh / p.Hkv], 0), p.S) : p.S;
}
// q row and output row of (sequence b, kv head kvh, column qh of the group):
// column qh is query token qh / Gq of head kvh * Gq + qh % Gq.
__device__ __forceinline__ const __nv_bfloat16* q_row(const DecodeParams& p, int b, int kvh, int qh) {
    const int j = qh / p.Gq, gh = qh - j * p.Gq;
    return p.q + b * p.q_sb + j * p.q_st + (int64_t)(kvh * p.Gq + gh) * p.q_sh;
}
__device__ __forceinline__ int64_t out_row(const DecodeParams& p, int b, int kvh, int qh) {
    const int j = qh / p.Gq, gh = qh - j * p.Gq;
    return ((int64_t)b * p.Tq + j) * p.Hq0 + kvh * p.Gq + gh;
}
__device__ __forceinline__ int64_t total_tiles(const DecodeParams& p) {
    return p.tile_off ? (int64_t)p.tile_off[p.B * p.Hkv] : p.W;
}
__device__ __forceinline__ int64_t head_tile0(const DecodeParams& p, int bh) {
    return p.tile_off ? (int64_t)p.tile_off[bh] : (int64_t)bh * p.T;
}
// Walk (head, tile) over a CTA's contiguous slice of the flattened tile list.
struct TileCursor {
    int bh, tl, T;
    __device__ __forceinline__ void init(const DecodeParams& p, int64_t i) {
        if (!p.tile_off) { bh = (int)(i / p.T); tl = (int)(i % p.T); T = p.T; return; }
        int lo = 0, hi = p.B * p.Hkv - 1;            // last head with tile_off[bh] <= i
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.tile_off[mid] <= i) lo = mid; else hi = mid - 1;
        }
        bh = lo;
        while (p.tile_off[bh + 1] <= i) ++bh;         // skip heads without tiles
        tl = (int)(i - p.tile_off[bh]);
        T = p.tile_off[bh + 1] - p.tile_off[bh];
    }
    __device__ __forceinline__ void next(const DecodeParams& p) {
        if (++tl < T) return;
        tl = 0;
        ++bh;
        if (p.tile_off) {
            const int BH = p.B * p.Hkv;
            while (bh < BH && p.tile_off[bh + 1] == p.tile_off[bh]) ++bh;
            T = bh < BH ? p.tile_off[bh + 1] - p.tile_off[bh] : 1;
        }
    }
};

// Varlen prologue: tile_off[bh] = sum of ceil(full pages / 8) over earlier heads.
__global__ void __launch_bounds__(1024) tile_offsets_kernel(const int* seq_lens, int B, int Hkv, int S,
                                                            int* tile_off) {
    __shared__ int part[1024];
    const int BH = B * Hkv, t = threadIdx.x;
    const int chunk = (BH + 1023) / 1024, a = t * chunk, e = min(a + chunk, BH);
    int sum = 0;
    for (int bh = a; bh < e; ++bh) {
        const int L = min(max(seq_lens[bh / Hkv], 0), S);
        sum += ((L / 16) * 16 + 127) / 128;
    }
    part[t] = sum;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {               // inclusive scan
        const int v = t >= o ? part[t - o] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    int run = part[t] - sum;                           // exclusive prefix of my chunk
    for (int bh = a; bh < e; ++bh) {
        tile_off[bh] = run;
        const int L = min(max(seq_lens[bh / Hkv], 0), S);
        run += ((L / 16) * 16 + 127) / 128;
    }
    if (t == 1023) tile_off[BH] = part[1023];
}

template <int FMT>
struct StageLayout {
    static constexpr int KC = 0;                        // 128 ch x 64 B, 64B-swizzled
    static constexpr int KS = 8192;                     // INT4: 128 x 16 B ; NVFP4: 128 x 16 B raw e4m3
    static constexpr int VC = 8192 + 2048;              // 128 tok x 64 B, 64B-swizzled
    static constexpr int VS = VC + 8192;                // INT4: 128 x 16 B ; NVFP4: 128 x 8 B
    static constexpr int BYTES = VS + 2048;
    // FMT_MIX43: V codes arrive as four 32-token boxes of 48-byte INT3 rows,
    // warp w's at VC + 2048 w + VC3_OFF (inside the 2 KB its nibble rows fill)
    static constexpr int VC3_OFF = 512;
    static constexpr uint32_t TX = (FMT == FMT_NVFP4) ? (8192 + 2048 + 8192 + 1024)
                                 : (FMT == FMT_MIX43) ? (8192 + 2048 + 6144 + 2048) : 20480;
};

struct __align__(8) SmemCtl {
    uint64_t full[NST];
    uint64_t empty[NST];
    int abort;
};

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Dequantise two ldmatrix words (k-halves A and B of one MMA) into the A
// fragments of tile 0 (nibble bytes 0/2) and tile 1 (bytes 1/3), unscaled.
template <int FMT>
__device__ __forceinline__ void codes4(uint32_t w, uint32_t& t0_lo, uint32_t& t0_hi,
                                       uint32_t& t1_lo, uint32_t& t1_hi) {
    if (FMT == FMT_MIX43) {
        t0_lo = h2_as_u32(int3n_lo_to_h2(w));
        t0_hi = h2_as_u32(int3n_hi_to_h2(w));
        const uint32_t w8 = w >> 8;
        t1_lo = h2_as_u32(int3n_lo_to_h2(w8));
        t1_hi = h2_as_u32(int3n_hi_to_h2(w8));
    } else if (FMT == FMT_NVFP4) {
        uint32_t h0, h1, h2, h3;
        e2m1x8_to_h2x4(w, h0, h1, h2, h3);
        t0_lo = __byte_perm(h0, h2, 0x5410);
        t0_hi = __byte_perm(h0, h2, 0x7632);
        t1_lo = __byte_perm(h1, h3, 0x5410);
        t1_hi = __byte_perm(h1, h3, 0x7632);
    } else {
        t0_lo = h2_as_u32(int4_lo_to_h2(w));
        t0_hi = h2_as_u32(int4_hi_to_h2(w));
        const uint32_t w8 = w >> 8;
        t1_lo = h2_as_u32(int4_lo_to_h2(w8));
        t1_hi = h2_as_u32(int4_hi_to_h2(w8));
    }
}

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}

// One m16n8k16 step for two M-tiles given the k-half words wA, wB and their
// scale pairs.  INT4 splits each scale into an 8-bit head and a 3-bit tail
// (two MMAs), so every code x scale product is exact in fp16; used for K,
// and for V when the GQA group is too large for the paired form.
template <int FMT, bool SPLIT>
__device__ __forceinline__ void mma_pair(float (&c0)[4], float (&c1)[4], uint32_t wA, uint32_t wB,
                                         uint32_t sA, uint32_t sB, uint32_t b0, uint32_t b1) {
    uint32_t a0l, a0h, a1l, a1h, c0l, c0h, c1l, c1h;
    codes4<FMT>(wA, a0l, a0h, a1l, a1h);     // k-half A: tile0 rows(lo,hi), tile1 rows
    codes4<FMT>(wB, c0l, c0h, c1l, c1h);     // k-half B
    if (FMT == FMT_NVFP4 || !SPLIT) {
        mma_f16(c0, hmul2u(a0l, sA), hmul2u(a0h, sA), hmul2u(c0l, sB), hmul2u(c0h, sB), b0, b1);
        mma_f16(c1, hmul2u(a1l, sA), hmul2u(a1h, sA), hmul2u(c1l, sB), hmul2u(c1h, sB), b0, b1);
    } else {
        const uint32_t sAh = sA & 0xFFF8FFF8u, sBh = sB & 0xFFF8FFF8u;
        const uint32_t sAl = h2_as_u32(__hsub2(u32_as_h2(sA), u32_as_h2(sAh)));
        const uint32_t sBl = h2_as_u32(__hsub2(u32_as_h2(sB), u32_as_h2(sBh)));
        mma_f16(c0, hmul2u(a0l, sAh), hmul2u(a0h, sAh), hmul2u(c0l, sBh), hmul2u(c0h, sBh), b0, b1);
        mma_f16(c0, hmul2u(a0l, sAl), hmul2u(a0h, sAl), hmul2u(c0l, sBl), hmul2u(c0h, sBl), b0, b1);
        mma_f16(c1, hmul2u(a1l, sAh), hmul2u(a1h, sAh), hmul2u(c1l, sBh), hmul2u(c1h, sBh), b0, b1);
        mma_f16(c1, hmul2u(a1l, sAl), hmul2u(a1h, sAl), hmul2u(c1l, sBl), hmul2u(c1h, sBl), b0, b1);
    }
}


// Paired form (INT4, GQA group <= 4): the A operand is the raw exact codes and
// the scales ride on B.  Columns n < 4 of B carry the query heads scaled for
// the first page (K) / d-block (V) of the M-tile's rows, columns n >= 4 the
// same heads scaled for the second, so one MMA serves both halves of the tile;
// each thread later keeps the half that matches its rows.
template <int FMT>
__device__ __forceinline__ void mma_raw(float (&c0)[4], float (&c1)[4], uint32_t wA, uint32_t wB,
                                        uint32_t b0, uint32_t b1) {
    uint32_t a0l, a0h, a1l, a1h, c0l, c0h, c1l, c1h;
    codes4<FMT>(wA, a0l, a0h, a1l, a1h);
    codes4<FMT>(wB, c0l, c0h, c1l, c1h);
    mma_f16(c0, a0l, a0h, c0l, c0h, b0, b1);
    mma_f16(c1, a1l, a1h, c1l, c1h, b0, b1);
}
__device__ __forceinline__ void mma_raw2(float (&c0)[4], float (&c1)[4], uint32_t wA, uint32_t wB,
                                         uint32_t b0h, uint32_t b1h, uint32_t b0l, uint32_t b1l) {
    uint32_t a0l, a0h, a1l, a1h, c0l, c0h, c1l, c1h;
    codes4<FMT_INT4>(wA, a0l, a0h, a1l, a1h);
    codes4<FMT_INT4>(wB, c0l, c0h, c1l, c1h);
    mma_f16(c0, a0l, a0h, c0l, c0h, b0h, b1h);
    mma_f16(c1, a1l, a1h, c1l, c1h, b0h, b1h);
    mma_f16(c0, a0l, a0h, c0l, c0h, b0l, b1l);
    mma_f16(c1, a1l, a1h, c1l, c1h, b0l, b1l);
}
// q (x) s as an exact hi + lo pair of fp16x2 values.
__device__ __forceinline__ void split_prod(uint32_t q, uint32_t sc, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __hmul2(u32_as_h2(q), u32_as_h2(sc));
    hi = h2_as_u32(h);
    lo = h2_as_u32(__hfma2(u32_as_h2(q), u32_as_h2(sc), __hneg2(h)));
}

__device__ __forceinline__ uint32_t swz64(uint32_t row, uint32_t chunk) {
    return row * 64u + 16u * (chunk ^ ((row >> 1) & 3u));
}

// ---------------------------------------------------------------------------
// Fast path kernel.
// ---------------------------------------------------------------------------
template <int FMT, bool PAIRED>
__global__ void __launch_bounds__(NTHREADS, CTAS_PER_SM)
decode_fast_kernel(const __grid_constant__ CUtensorMap tm_kc, const __grid_constant__ CUtensorMap tm_ks,
                   const __grid_constant__ CUtensorMap tm_vc, const __grid_constant__ CUtensorMap tm_vs,
                   const DecodeParams p) {
    using L = StageLayout<FMT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stages = smem;                                            // NST * L::BYTES
    __half* pbuf = reinterpret_cast<__half*>(stages + NST * L::BYTES); // [4][8][PB_PITCH]
    __half* scv = pbuf + NWARP_C * 8 * PB_PITCH;                       // NVFP4: [4 warps][32][8] fp16
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(scv + (FMT == FMT_NVFP4 ? NWARP_C * 32 * 8 : 0));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const int64_t Wt = total_tiles(p);
    const int64_t i0 = tile_start(c, Wt, p.N), i1 = tile_start(c + 1, Wt, p.N);
    if (i0 >= i1) return;                    // varlen grids can hold idle CTAs

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) { mbar_init(&ctl->full[s], 1); mbar_init(&ctl->empty[s], NWARP_C); }
        ctl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NWARP_C) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            prefetch_tmap(&tm_kc); prefetch_tmap(&tm_ks); prefetch_tmap(&tm_vc); prefetch_tmap(&tm_vs);
            int it = 0;
            TileCursor cu;
            cu.init(p, i0);
            for (int64_t i = i0; i < i1; ++i, ++it, cu.next(p)) {
                const int bh = cu.bh, tl = cu.tl;
                const int s = it % NST;
                if (!mbar_wait_bounded(&ctl->empty[s], ((it / NST) & 1) ^ 1)) {
                    set_err(p.err, KIVI_ERR_TIMEOUT);
                    ctl->abort = 1;
                    break;
                }
                if (ctl->abort) break;
                uint8_t* st = stages + s * L::BYTES;
                mbar_arrive_expect_tx(&ctl->full[s], L::TX);
                tma_load_2d(st + L::KC, &tm_kc, &ctl->full[s], tl * 64, bh * DH);
                if (FMT == FMT_NVFP4) tma_load_2d(st + L::KS, &tm_ks, &ctl->full[s], (tl >> 1) * 16, bh * DH);
                else tma_load_2d(st + L::KS, &tm_ks, &ctl->full[s], tl * 8, bh * DH);
                const int vrow = bh * p.v_s_stride + tl * TILE;
                if (FMT == FMT_MIX43) {
#pragma unroll
                    for (int w = 0; w < NWARP_C; ++w)
                        tma_load_2d(st + L::VC + 2048 * w + L::VC3_OFF, &tm_vc, &ctl->full[s], 0, vrow + 32 * w);
                } else {
                    tma_load_2d(st + L::VC, &tm_vc, &ctl->full[s], 0, vrow);
                }
                if (FMT == FMT_NVFP4) tma_load_2d(st + L::VS, &tm_vs, &ctl->full[s], 0, vrow >> 1);
                else tma_load_2d(st + L::VS, &tm_vs, &ctl->full[s], 0, vrow);
            }
            // Drain: every issued tile's bytes must land before the CTA retires.
            for (int j = (it > NST ? it - NST : 0); j < it; ++j)
                if (!mbar_wait_bounded(&ctl->full[j % NST], (j / NST) & 1)) set_err(p.err, KIVI_ERR_TIMEOUT);
        }
        return;
    }

    // ------------------------------- consumers --------------------------------
    constexpr int KF = FMT == FMT_MIX43 ? FMT_INT4 : FMT;   // K pages' format
    const int g = lane >> 2, tq = lane & 3;
    const int G = p.G;
    const int src_k = ((2 * warp + (g >> 2)) << 2) | tq;   // lane holding my page's K scales
    const uint32_t pb_s = smem_u32(pbuf + warp * 8 * PB_PITCH);   // P staging [8 heads][PB_PITCH] halves
    const uint32_t abort_s = smem_u32(&ctl->abort);

    uint32_t qB[8][2];
    float acc[8][4];     // [tile: 2*seg + (0:X,1:Y)][c]
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    int cur = -1;

    auto flush = [&](int bh) {
        // per-warp partial record: slot = (c + bh) * 4 + warp
        float L0 = l0, L1 = l1;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            L0 += __shfl_xor_sync(0xffffffffu, L0, o);
            L1 += __shfl_xor_sync(0xffffffffu, L1, o);
        }
        const int64_t slot = ((int64_t)(c + bh) * NWARP_C + warp) * G;
        const float gv = (FMT == FMT_NVFP4) ? p.g_v : 1.0f;
        // paired form: the acc columns of lane (g, tq) are heads 2(tq&1)(+1),
        // valid where the column half matches the rows' d-block half
        const bool acc_ok = PAIRED ? ((g < 4) == (tq < 2)) : true;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int h = (PAIRED ? 2 * (tq & 1) : 2 * tq) + hh;
            if (h < G) {
                if (g == 0 && tq < (PAIRED ? 2 : 4)) {
                    p.part_m[slot + h] = hh ? m1 : m0;
                    p.part_l[slot + h] = hh ? L1 : L0;
                }
                if (!acc_ok) continue;
                float* a = p.part_acc + (slot + h) * DH;
#pragma unroll
                for (int sg = 0; sg < 4; ++sg) {
                    float4 v = make_float4(acc[2 * sg][hh] * gv, acc[2 * sg][2 + hh] * gv,
                                           acc[2 * sg + 1][hh] * gv, acc[2 * sg + 1][2 + hh] * gv);
                    *reinterpret_cast<float4*>(a + 32 * sg + 4 * g) = v;
                }
            }
        }
    };

    int it = 0;
    TileCursor cu;
    cu.init(p, i0);
    int n_full_h = 0;
    for (int64_t i = i0; i < i1; ++i, ++it, cu.next(p)) {
        const int bh = cu.bh, tl = cu.tl;
        if (bh != cur) {
            n_full_h = (head_len(p, bh) / BLK) * BLK;
            if (cur >= 0) flush(cur);
            cur = bh;
            m0 = m1 = -INFINITY; l0 = l1 = 0.f;
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
            const int b = bh / p.Hkv, kvh = bh % p.Hkv;
            const int qh = PAIRED ? (g & 3) : g;
            const __nv_bfloat16* qp = q_row(p, b, kvh, qh < G ? qh : 0);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t v = 0;
                    if (qh < G) {
                        const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(qp + 16 * k + 8 * hf + 2 * tq);
                        v = h2_as_u32(__float22half2_rn(__bfloat1622float2(b2)));
                    }
                    qB[k][hf] = v;
                }
            }
        }
        const int s = it % NST;
        if (!mbar_wait_bounded(&ctl->full[s], (it / NST) & 1)) {
            set_err(p.err, KIVI_ERR_TIMEOUT);
            sts32s(abort_s, 1u);
        }
        if (lds32s(abort_s)) break;
        uint8_t* st = stages + s * L::BYTES;
        const uint8_t* vs_base = st + L::VS;
        if (FMT == FMT_NVFP4) {
            // my 32 tokens' e4m3 V scales -> fp16 rows [token][8] (per-warp buffer)
            __half* vw = scv + warp * 32 * 8;
            const uint2 raw = lds64s(smem_u32(st + L::VS + (32 * warp + lane) * 8));
            __syncwarp();
            sts128s(smem_u32(vw + lane * 8),
                    make_uint4(e4m3x2_to_h2((uint16_t)raw.x), e4m3x2_to_h2((uint16_t)(raw.x >> 16)),
                               e4m3x2_to_h2((uint16_t)raw.y), e4m3x2_to_h2((uint16_t)(raw.y >> 16))));
            __syncwarp();
            vs_base = reinterpret_cast<const uint8_t*>(vw) - 32 * warp * 16;
        }
        if (FMT == FMT_MIX43) {
            // my token's 48-byte INT3 row -> its 64-byte nibble row (c & 7 per
            // nibble) in the INT4 tile layout, written over my warp's 2 KB
            // (which also holds the staged INT3 rows: all lanes read first)
            const uint32_t raw = smem_u32(st + L::VC + 2048 * warp + L::VC3_OFF + 48 * lane);
            const uint4 r0 = lds128s(raw), r1 = lds128s(raw + 16), r2 = lds128s(raw + 32);
            const uint32_t wd[12] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w, r2.x, r2.y, r2.z, r2.w};
            __syncwarp();
            const uint32_t row = 32 * warp + lane, vc0 = smem_u32(st + L::VC);
#pragma unroll
            for (int k = 0; k < 4; ++k) {                 // 16-byte chunk k = blocks 2k, 2k + 1
                uint32_t l0, h0, l1, h1;
                int3_pair_nibbles(wd[3 * k], wd[3 * k + 2], 0, l0, h0);
                int3_pair_nibbles(wd[3 * k + 1], wd[3 * k + 2], 1, l1, h1);
                sts128s(vc0 + swz64(row, k), make_uint4(l0, h0, l1, h1));
            }
            __syncwarp();
        }

        const int t_span = tl * TILE + 32 * warp;      // first token of my span
        const int limit = n_full_h - t_span;           // valid tokens in my span
        // Full spans take the branch-free body; only a sequence's last tile is masked.
        auto span = [&](auto masked_tag) {
            constexpr bool MASKED = decltype(masked_tag)::value;
            // ------------------------------ QK^T ------------------------------
            float qa[2][4], qb[2][4];      // two accumulator pairs: shorter MMA chains
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) qa[j][e] = qb[j][e] = 0.f;
            const uint32_t kc_s = smem_u32(st + L::KC), ks_s = smem_u32(st + L::KS);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t row = 32 * j + lane;
                uint32_t r0, r1, r2, r3, s0, s1, s2, s3;
                ldsm_x4_t(kc_s + swz64(row, warp), r0, r1, r2, r3);
                ldsm_x4_t(ks_s + row * 16, s0, s1, s2, s3);
                if (FMT == FMT_NVFP4) {
                    // raw e4m3 rows of 16 pages: u16 column = page pair; pick my page
                    const int srcn = ((((tl & 1) * 4) + warp) << 2) | tq;
                    const uint32_t sel = (uint32_t)(g >> 2);
                    const uint32_t pm = ((2u + sel) << 4) | sel;
                    s0 = e4m3x2_to_h2((uint16_t)__byte_perm(__shfl_sync(0xffffffffu, s0, srcn), 0, pm));
                    s1 = e4m3x2_to_h2((uint16_t)__byte_perm(__shfl_sync(0xffffffffu, s1, srcn), 0, pm));
                    s2 = e4m3x2_to_h2((uint16_t)__byte_perm(__shfl_sync(0xffffffffu, s2, srcn), 0, pm));
                    s3 = e4m3x2_to_h2((uint16_t)__byte_perm(__shfl_sync(0xffffffffu, s3, srcn), 0, pm));
                } else {
                    s0 = __shfl_sync(0xffffffffu, s0, src_k);
                    s1 = __shfl_sync(0xffffffffu, s1, src_k);
                    s2 = __shfl_sync(0xffffffffu, s2, src_k);
                    s3 = __shfl_sync(0xffffffffu, s3, src_k);
                }
                if constexpr (PAIRED && KF == FMT_INT4) {
                    uint32_t h0, l0_, h1, l1_, h2, l2_, h3, l3_;
                    split_prod(qB[2 * j][0], s0, h0, l0_);
                    split_prod(qB[2 * j][1], s1, h1, l1_);
                    split_prod(qB[2 * j + 1][0], s2, h2, l2_);
                    split_prod(qB[2 * j + 1][1], s3, h3, l3_);
                    mma_raw2(qa[j & 1], qb[j & 1], r0, r1, h0, h1, l0_, l1_);
                    mma_raw2(qa[j & 1], qb[j & 1], r2, r3, h2, h3, l2_, l3_);
                } else {
                    mma_pair<KF, true>(qa[j & 1], qb[j & 1], r0, r1, s0, s1, qB[2 * j][0], qB[2 * j][1]);
                    mma_pair<KF, true>(qa[j & 1], qb[j & 1], r2, r3, s2, s3, qB[2 * j + 1][0], qB[2 * j + 1][1]);
                }
            }
            float ca[4], cb[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ca[e] = qa[0][e] + qa[1][e];
                cb[e] = qb[0][e] + qb[1][e];
            }
            if constexpr (PAIRED && KF == FMT_INT4) {
                // keep the column half that matches my rows' page; after this
                // every lane holds heads 2(tq&1), 2(tq&1)+1 of its rows
                const bool mine = (g < 4) == (tq < 2);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float oa = __shfl_xor_sync(0xffffffffu, ca[e], 2);
                    const float ob = __shfl_xor_sync(0xffffffffu, cb[e], 2);
                    ca[e] = mine ? ca[e] : oa;
                    cb[e] = mine ? cb[e] : ob;
                }
            }
            // ----------------------------- softmax ----------------------------
            // ca: tokens 4g (c0,c1), 4g+1 (c2,c3); cb: 4g+2, 4g+3; heads 2tq(+1)
            // raw scores; the softmax scale (> 0, log2 units) is applied in
            // the exp2 argument and to the running maxima
            float x[8] = {ca[0], ca[2], cb[0], cb[2], ca[1], ca[3], cb[1], cb[3]};
            if (MASKED) {
                const int tk[4] = {4 * g, 4 * g + 1, 4 * g + 2, 4 * g + 3};
#pragma unroll
                for (int e = 0; e < 8; ++e) if (tk[e & 3] >= limit) x[e] = -INFINITY;
            }
            float mx0 = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])) * p.scale2;
            float mx1 = fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7])) * p.scale2;
            // Lazy rescaling: the running reference max only moves when a new
            // score exceeds it by more than 2^8 (p stays <= 256, exact in the
            // final normalisation since l uses the same reference).  A lane's
            // own maxima decide whether any head of the warp needs it; only
            // then are the maxima reduced over the head's lanes.
            const bool need = (mx0 > m0 + 8.f) || (mx1 > m1 + 8.f);
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
                }
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float al0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - mn0);
                const float al1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - mn1);
                m0 = mn0; m1 = mn1;
                l0 *= al0; l1 *= al1;
#pragma unroll
                for (int t = 0; t < 8; ++t) { acc[t][0] *= al0; acc[t][2] *= al0; acc[t][1] *= al1; acc[t][3] *= al1; }
            }
            // m == -inf only while every token so far is masked: use 0 as reference
            const float r0 = (m0 == -INFINITY) ? 0.f : m0, r1 = (m1 == -INFINITY) ? 0.f : m1;
            float pr[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                pr[e] = exp2f(fmaf(x[e], p.scale2, -r0));
                pr[4 + e] = exp2f(fmaf(x[4 + e], p.scale2, -r1));
            }
            l0 += (pr[0] + pr[1]) + (pr[2] + pr[3]);
            l1 += (pr[4] + pr[5]) + (pr[6] + pr[7]);
            // stage P as fp16 [head][token] for the PV B-fragments
            __syncwarp();
            sts64s(pb_s + 2 * ((2 * tq) * PB_PITCH + 4 * g),
                   h2_as_u32(__floats2half2_rn(pr[0], pr[1])), h2_as_u32(__floats2half2_rn(pr[2], pr[3])));
            sts64s(pb_s + 2 * ((2 * tq + 1) * PB_PITCH + 4 * g),
                   h2_as_u32(__floats2half2_rn(pr[4], pr[5])), h2_as_u32(__floats2half2_rn(pr[6], pr[7])));
            __syncwarp();
            // ------------------------------- PV -------------------------------
            const uint32_t vc_s = smem_u32(st + L::VC), vs_s = smem_u32(vs_base);
            uint32_t vr[4];
            ldsm_x4_t(vs_s + (32 * warp + lane) * 16, vr[0], vr[1], vr[2], vr[3]);
            
#pragma unroll
            for (int lam = 0; lam < 2; ++lam) {
                const int prow = PAIRED ? (g & 3) : g;
                const uint32_t b0 = lds32s(pb_s + 2 * (prow * PB_PITCH + 16 * lam + 2 * tq));
                const uint32_t b1 = lds32s(pb_s + 2 * (prow * PB_PITCH + 16 * lam + 8 + 2 * tq));
#pragma unroll
                for (int sp = 0; sp < 2; ++sp) {          // segment pairs (2sp, 2sp+1)
                    const uint32_t trow = 32 * warp + 16 * lam + 8 * ((lane >> 3) & 1) + (lane & 7);
                    const uint32_t chunk = 2 * sp + (lane >> 4);
                    uint32_t w0, w1, w2, w3;
                    ldsm_x4_t(vc_s + swz64(trow, chunk), w0, w1, w2, w3);
#pragma unroll
                    for (int hs = 0; hs < 2; ++hs) {
                        const int sg = 2 * sp + hs;
                        const int src_v = ((2 * sg + (g >> 2)) << 2) | tq;
                        uint32_t sa = __shfl_sync(0xffffffffu, vr[2 * lam], src_v);
                        uint32_t sb = __shfl_sync(0xffffffffu, vr[2 * lam + 1], src_v);
                        if (MASKED) {
                            const int t0 = 16 * lam + 2 * tq;     // tokens of sa: t0, t0+1; sb: t0+8, t0+9
                            sa = (t0 + 1 < limit) ? sa : (t0 < limit ? (sa & 0x0000FFFFu) : 0u);
                            sb = (t0 + 9 < limit) ? sb : (t0 + 8 < limit ? (sb & 0x0000FFFFu) : 0u);
                        }
                        if constexpr (PAIRED) {
                            mma_raw<FMT>(acc[2 * sg], acc[2 * sg + 1], hs ? w2 : w0, hs ? w3 : w1,
                                    hmul2u(b0, sa), hmul2u(b1, sb));
                        } else {
                            mma_pair<FMT, true>(acc[2 * sg], acc[2 * sg + 1], hs ? w2 : w0, hs ? w3 : w1, sa, sb, b0, b1);
                        }
                    }
                }
            }
        };
        if (limit >= 32) span(std::false_type{});
        else if (limit > 0) span(std::true_type{});
        // the nibble rows written above sit where the next TMA of this stage
        // lands: order the generic-proxy writes before that async-proxy write
        if (FMT == FMT_MIX43) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->empty[s]);
    }
    if (cur >= 0 && !lds32s(abort_s)) flush(cur);
    // let the dependent merge kernel start its prologue (programmatic launch)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Generic path (any D multiple of 16 up to 256, any group <= 16, any strides):
// same work partition and partial-record format as the fast path, CUDA-core
// arithmetic, one warp streams its 32-token span of each tile token by token.
// ---------------------------------------------------------------------------
constexpr int GEN_MAXG = 16, GEN_MAXC = 8;

template <int FMT>
__device__ __forceinline__ float gen_scale(const void* s, int64_t idx, float g) {
    if (FMT == FMT_NVFP4) return e4m3_to_f32(reinterpret_cast<const uint8_t*>(s)[idx]) * g;
    return __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(s)[idx]));
}
template <int FMT>
__device__ __forceinline__ float gen_code(uint32_t nib) {
    if (FMT == FMT_NVFP4) { float l = e2m1_level(nib & 7); return (nib & 8) ? -l : l; }
    return (float)sx4((int)nib);
}
// Dequantised V at packed row vr (one token's 16-channel block), channel d.
template <int FMT>
__device__ __forceinline__ float gen_v(const DecodeParams& p, int64_t vr, int d) {
    if (FMT == FMT_MIX43)
        return (float)int3_code(p.v_packed + (vr - d / BLK) * PACKB3, d) * gen_scale<FMT>(p.v_scale, vr, p.g_v);
    const uint32_t vb = p.v_packed[vr * PACKB + (d % BLK) / 2];
    return gen_code<FMT>((vb >> (4 * (d & 1))) & 0xF) * gen_scale<FMT>(p.v_scale, vr, p.g_v);
}

template <int FMT>
__global__ void __launch_bounds__(128) decode_generic_kernel(const DecodeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x, G = p.G, D = p.D, ND = D / BLK;
    const int64_t Wt = total_tiles(p);
    const int64_t i0 = tile_start(c, Wt, p.N), i1 = tile_start(c + 1, Wt, p.N);
    const float sc2 = p.sm_scale * 1.4426950408889634f;
    float q[GEN_MAXG][GEN_MAXC], acc[GEN_MAXG][GEN_MAXC], m[GEN_MAXG], l[GEN_MAXG];
    int cur = -1;
    auto flush = [&](int bh) {
        const int64_t slot = ((int64_t)(c + bh) * NWARP_C + warp) * G;
        for (int h = 0; h < G; ++h) {
            if (lane == 0) { p.part_m[slot + h] = m[h]; p.part_l[slot + h] = l[h]; }
            for (int e = 0; e < GEN_MAXC; ++e) {
                const int d = lane + 32 * e;
                if (d < D) p.part_acc[(slot + h) * D + d] = acc[h][e];
            }
        }
    };
    TileCursor cu;
    if (i0 < i1) cu.init(p, i0);
    int n_full_h = 0;
    for (int64_t i = i0; i < i1; ++i, cu.next(p)) {
        const int bh = cu.bh, tl = cu.tl;
        if (bh != cur) {
            n_full_h = (head_len(p, bh) / BLK) * BLK;
            if (cur >= 0) flush(cur);
            cur = bh;
            const int b = bh / p.Hkv, kvh = bh % p.Hkv;
            for (int h = 0; h < G; ++h) {
                m[h] = -INFINITY; l[h] = 0.f;
                const __nv_bfloat16* qp = q_row(p, b, kvh, h);
                for (int e = 0; e < GEN_MAXC; ++e) {
                    const int d = lane + 32 * e;
                    q[h][e] = d < D ? __bfloat162float(qp[d]) : 0.f;
                    acc[h][e] = 0.f;
                }
            }
        }
        const int t_end = min(n_full_h, tl * TILE + 32 * warp + 32);
        for (int t = tl * TILE + 32 * warp; t < t_end; ++t) {
            float kv[GEN_MAXC], vv[GEN_MAXC];
            const int pg = t / BLK, j = t % BLK;
            for (int e = 0; e < GEN_MAXC; ++e) {
                const int d = lane + 32 * e;
                kv[e] = vv[e] = 0.f;
                if (d < D) {
                    const int64_t kr = ((int64_t)bh * D + d) * p.k_np_stride + pg;
                    const uint32_t kb = p.k_packed[kr * PACKB + j / 2];
                    kv[e] = gen_code<FMT>((kb >> (4 * (j & 1))) & 0xF) * gen_scale<FMT>(p.k_scale, kr, p.g_k);
                    vv[e] = gen_v<FMT>(p, ((int64_t)bh * p.v_s_stride + t) * ND + d / BLK, d);
                }
            }
            for (int h = 0; h < G; ++h) {
                float s = 0.f;
                for (int e = 0; e < GEN_MAXC; ++e) s += q[h][e] * kv[e];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                s *= sc2;
                const float mn = fmaxf(m[h], s);
                const float al = exp2f(m[h] - mn), pr = exp2f(s - mn);
                m[h] = mn;
                l[h] = l[h] * al + pr;
                for (int e = 0; e < GEN_MAXC; ++e) acc[h][e] = acc[h][e] * al + pr * vv[e];
            }
        }
    }
    if (cur >= 0) flush(cur);
}

// ---------------------------------------------------------------------------
// Combine: bf16 hot tail + LSE merge of all partial slots of one (kv-head,
// q-head) pair; one 128-thread block per pair.  The slot weights
// exp2(m_s - M) are computed once into shared memory, then every thread
// reduces its channels over the slots with coalesced loads.
// mode 0 -> normalised bf16 out; mode 1 -> merged (m, l, acc) records.
// ---------------------------------------------------------------------------
__host__ __device__ inline void head_cta_range(int64_t a0, int64_t a1, int64_t W, int N, int& c_lo, int& c_hi) {
    // CTA c owns tiles [floor(cW/N), floor((c+1)W/N)).  c_lo is the last CTA
    // whose slice starts at or before a0 (floor(cW/N) <= a0 <=> cW < (a0+1)N),
    // c_hi the last whose slice starts before a1 (cW < a1 N).
    c_lo = 0; c_hi = -1;
    if (W <= 0 || a1 <= a0) return;
    const int64_t lo = ((a0 + 1) * N - 1) / W, hi = (a1 * N - 1) / W;
    c_lo = (int)(lo < N - 1 ? lo : N - 1);
    c_hi = (int)(hi < N - 1 ? hi : N - 1);
}

// V of tail token j (absolute n_full + j) at channel d: bf16 when the caller
// keeps the partial page unquantised, else dequantised from v_packed.
template <int FMT>
__device__ __forceinline__ float tail_v(const DecodeParams& p, int bh, int n_full, int j, int d, int ND) {
    const int t = n_full + j;                           // absolute token
    // the bf16 partial page starts at the cache's last full page (plain
    // decodes: n_full itself; varlen heads each have their own n_full)
    if (p.v_hot && (!p.mq || t >= p.nf_real))
        return __bfloat162float(p.v_hot[((int64_t)bh * p.hot_stride + (p.mq ? t - p.nf_real : j)) * p.D + d]);
    return gen_v<FMT>(p, ((int64_t)bh * p.v_s_stride + t) * ND + d / BLK, d);
}

// NWC warps per row: 4, or 16 when heads spread over many CTAs (long rows of
// partial slots, e.g. batch 1), so more slot loads are in flight per row.
template <int FMT, int NWC>
__global__ void __launch_bounds__(NWC * 32, 1) combine_kernel(const DecodeParams p, int mode, __nv_bfloat16* out,
                                                              float* m_out, float* l_out, float* acc_out) {
    extern __shared__ float csm[];
    const int bh = blockIdx.x, h = blockIdx.y, b = bh / p.Hkv, kvh = bh % p.Hkv;
    const int G = p.G, D = p.D, ND = D / BLK;
    const int Lh = head_len(p, bh), n_full = (Lh / BLK) * BLK;
    // tail tokens [n_full, tail_end) merged here: the bf16 hot page; for a
    // multi-query decode also the tokens past the pages every query sees, up
    // to this query's own causal limit (a query at position S - Tq + j sees
    // tokens 0 .. S - Tq + j)
    const int hot = (p.mq ? p.q_pos + 1 + h / p.Gq : Lh) - n_full;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int c_lo = 0, c_hi = -1;
    const int64_t Wt = total_tiles(p);
    const int64_t a0 = head_tile0(p, bh), a1 = head_tile0(p, bh + 1);
    if (Wt > 0 && a1 > a0) head_cta_range(a0, a1, Wt, p.N, c_lo, c_hi);
    const int ns = (c_hi - c_lo + 1) * NWARP_C;          // partial slots of this head
    const int wcap = ns + ((16 + p.Tq - 1 + 3) & ~3);   // slots, then up to 15 + Tq - 1 tail tokens
    float* w = csm;                                      // [wcap] weights (slots, then tail tokens)
    float* red = csm + wcap;                             // [2 NWC] block reduction scratch
    const float sc2 = p.sm_scale * 1.4426950408889634f;
    const __nv_bfloat16* qp = q_row(p, b, kvh, h);
    // K of tail token n_full + j at channel d: from the packed pages when it is
    // in one (multi-query tails), else from the bf16 hot page
    auto k_tail = [&](int j, int d) -> float {
        const int t = n_full + j;
        if (p.mq && t < p.nf_real) {
            const int64_t kr = ((int64_t)bh * D + d) * p.k_np_stride + t / BLK;
            const uint32_t kb = p.k_packed[kr * PACKB + (t % BLK) / 2];
            return gen_code<FMT>((kb >> (4 * (t & 1))) & 0xF) * gen_scale<FMT>(p.k_scale, kr, p.g_k);
        }
        return __bfloat162float(p.k_hot[((int64_t)bh * p.hot_stride + (p.mq ? t - p.nf_real : j)) * D + d]);
    };
    // tail scores (log2 units), one warp per token
    for (int j = warp; j < hot; j += NWC) {
        float sdot = 0.f;
        for (int d = lane; d < D; d += 32) sdot += __bfloat162float(qp[d]) * k_tail(j, d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, o);
        if (lane == 0) w[ns + j] = sdot * sc2;
    }
    // partial slots are produced by the split kernel launched just before
    // (programmatic dependent launch): wait for its results to be visible
    asm volatile("griddepcontrol.wait;" ::: "memory");
    auto slot = [&](int i) -> int64_t {
        return ((int64_t)(c_lo + i / NWARP_C + bh) * NWARP_C + (i % NWARP_C)) * G + h;
    };
    // an idle CTA (empty slice, possible on varlen grids only: a uniform grid
    // has no more CTAs than tiles) wrote no slots
    auto live = [&](int i) -> bool {
        if (!p.tile_off) return true;
        const int64_t cc = c_lo + i / NWARP_C;
        return tile_start(cc, Wt, p.N) < tile_start(cc + 1, Wt, p.N);
    };
    // One round trip for every partial the row needs: m and l of all slots,
    // and (the long-sequence path) the first acc vectors of this warp's slots,
    // all issued before any of them is used.  Partials of another kernel are
    // read at L2.
    float* wl = w + wcap + 2 * NWC + NWC * DH;           // [ns] l of each slot
    for (int i = threadIdx.x; i < ns; i += blockDim.x) {
        const bool lv = live(i);
        w[i] = lv ? __ldcg(p.part_m + slot(i)) : -INFINITY;
        wl[i] = lv ? __ldcg(p.part_l + slot(i)) : 0.f;
    }
    constexpr int PRE = 8;                               // slots per warp loaded up front
    float4 pre[PRE];
    const bool wide = D == DH && ns >= 16;
    if (wide) {
#pragma unroll
        for (int u = 0; u < PRE; ++u) {
            const int i = warp + NWC * u;
            pre[u] = (i < ns && live(i)) ? __ldcg(reinterpret_cast<const float4*>(p.part_acc + slot(i) * DH + 4 * lane))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __syncthreads();
    // M = max over slots and hot tokens
    float M = -INFINITY;
    for (int i = threadIdx.x; i < ns + hot; i += blockDim.x) M = fmaxf(M, w[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0) red[warp] = M;
    __syncthreads();
    M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
#pragma unroll
    for (int k = 4; k < NWC; ++k) M = fmaxf(M, red[k]);
    const float Mr = (M == -INFINITY) ? 0.f : M;
    __syncthreads();
    // weights and L
    float Ls = 0.f;
    for (int i = threadIdx.x; i < ns + hot; i += blockDim.x) {
        const float e = exp2f(w[i] - Mr);
        Ls += (i < ns) ? (e != 0.f ? wl[i] * e : 0.f) : e;
        w[i] = e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
    if (lane == 0) red[NWC + warp] = Ls;
    __syncthreads();
    Ls = (red[NWC] + red[NWC + 1]) + (red[NWC + 2] + red[NWC + 3]);
#pragma unroll
    for (int k = 4; k < NWC; ++k) Ls += red[NWC + k];
    const int64_t row = out_row(p, b, kvh, h);           // == b * Hq + kvh * G + h unless multi-query
    const int rows = p.B * p.Hq;
    unsigned int e = 0;
    float* xacc = nullptr;                               // mode 2: this row's acc in my slot
    if (mode == 2) {
        e = p.row_epoch[row] + 1;
        xacc = xslot(p.xbuf, p.xW, rows, D, e) + 2 * rows + row * D;
    }
    if (wide) {
        // many slots (long sequences): warp w takes slots w, w + NWC, ...;
        // each lane owns 4 channels (float4), then a shared-memory reduction
        float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < PRE; ++u) {
            const int i = warp + NWC * u;
            const float wi = i < ns ? w[i] : 0.f;
            if (wi != 0.f) {
                a4.x += pre[u].x * wi; a4.y += pre[u].y * wi; a4.z += pre[u].z * wi; a4.w += pre[u].w * wi;
            }
        }
        for (int i0 = warp + NWC * PRE; i0 < ns; i0 += 4 * NWC) {   // four loads in flight per iteration
            float4 v4[4];
            float wi[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + NWC * u;
                wi[u] = i < ns ? w[i] : 0.f;
                v4[u] = wi[u] != 0.f ? __ldcg(reinterpret_cast<const float4*>(p.part_acc + slot(i) * DH + 4 * lane))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                a4.x += v4[u].x * wi[u]; a4.y += v4[u].y * wi[u]; a4.z += v4[u].z * wi[u]; a4.w += v4[u].w * wi[u];
            }
        }
        float* sacc = red + 2 * NWC;                     // [NWC][128]
        *reinterpret_cast<float4*>(sacc + warp * DH + 4 * lane) = a4;
        __syncthreads();
        const int d = threadIdx.x;
        if (d < DH) {
            float a = (sacc[d] + sacc[DH + d]) + (sacc[2 * DH + d] + sacc[3 * DH + d]);
#pragma unroll
            for (int k = 4; k < NWC; ++k) a += sacc[k * DH + d];
            for (int j = 0; j < hot; ++j) a += w[ns + j] * tail_v<FMT>(p, bh, n_full, j, d, ND);
            if (mode == 0) out[row * D + d] = __float2bfloat16_rn(a / Ls);
            else if (mode == 1) acc_out[row * D + d] = a;
            else xacc[d] = a;
        }
    } else {
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            float a = 0.f;
            for (int i = 0; i < ns; ++i) if (w[i] != 0.f) a += __ldcg(p.part_acc + slot(i) * D + d) * w[i];
            for (int j = 0; j < hot; ++j) a += w[ns + j] * tail_v<FMT>(p, bh, n_full, j, d, ND);
            if (mode == 0) out[row * D + d] = __float2bfloat16_rn(a / Ls);
            else if (mode == 1) acc_out[row * D + d] = a;
            else xacc[d] = a;
        }
    }
    if (mode == 1 && threadIdx.x == 0) { m_out[row] = M; l_out[row] = Ls; }
    if (mode != 2) return;
    // ---- sequence-parallel exchange: publish this row, merge every rank's ----
    float* mine = xslot(p.xbuf, p.xW, rows, D, e);
    if (threadIdx.x == 0) { mine[row] = M; mine[rows + row] = Ls; }
    __syncthreads();                                     // the row's state is written (CTA scope) ...
    if (threadIdx.x < p.xW) {                            // ... and released system-wide to every rank
        __threadfence_system();
        st_release_sys_u32(reinterpret_cast<unsigned int*>(p.peers[threadIdx.x]) + (int64_t)p.xrank * rows + row, e);
    }
    // One thread per rank (W <= 16): wait, bounded, for rank j's epoch of this
    // row (its flag sits in this rank's own buffer), then load that rank's
    // (m, l) over NVLink -- all ranks' loads in flight at once.
    __shared__ int x_ok;
    __shared__ float x_m[16], x_lr[16];
    if (threadIdx.x == 0) x_ok = 1;
    __syncthreads();
    const int W = p.xW;
    if (threadIdx.x < W) {
        const int j = threadIdx.x;
        const unsigned int* flag = reinterpret_cast<const unsigned int*>(p.xbuf) + (int64_t)j * rows + row;
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        while ((int)(ld_acquire_sys_u32(flag) - e) < 0)
            if ((long long)(globaltimer_ns() - t0) > p.timeout_ns) { ok = false; break; }
        if (ok) {
            const float* sj = xslot(reinterpret_cast<uint8_t*>(p.peers[j]), W, rows, D, e);
            x_m[j] = __ldcg(sj + row);
            x_lr[j] = __ldcg(sj + rows + row);
        } else {
            atomicAnd(&x_ok, 0);
            set_err(p.err, KIVI_ERR_TIMEOUT);
        }
    }
    __syncthreads();                                     // every rank's row acquired (or a timeout)
    if (!x_ok) return;
    float Mx = -INFINITY;
    for (int j = 0; j < W; ++j) Mx = fmaxf(Mx, x_m[j]);
    const float Mxr = (Mx == -INFINITY) ? 0.f : Mx;
    float xw[16];
    float Lx = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        xw[j] = j < W ? exp2f(x_m[j] - Mxr) : 0.f;
        if (j < W) Lx += x_lr[j] * xw[j];
    }
    if (threadIdx.x == 0) p.row_epoch[row] = e;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)                     // all ranks' loads issued before any is used
            v[j] = j < W ? __ldcg(xslot(reinterpret_cast<uint8_t*>(p.peers[j]), W, rows, D, e) + 2 * rows +
                                  row * D + d)
                         : 0.f;
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < W) a += v[j] * xw[j];
        out[row * D + d] = __float2bfloat16_rn(Lx > 0.f ? a / Lx : 0.f);
    }
}

// Merge R records [R, rows], [R, rows, D] -> bf16 [rows, D].
__global__ void __launch_bounds__(128) lse_merge_kernel(const float* m, const float* l, const float* acc,
                                                        int R, int rows, int D, __nv_bfloat16* out) {
    const int row = blockIdx.x;
    float M = -INFINITY;
    for (int r = 0; r < R; ++r) M = fmaxf(M, m[(int64_t)r * rows + row]);
    const float Mr = (M == -INFINITY) ? 0.f : M;
    float Ls = 0.f;
    for (int r = 0; r < R; ++r) Ls += l[(int64_t)r * rows + row] * exp2f(m[(int64_t)r * rows + row] - Mr);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float a = 0.f;
        for (int r = 0; r < R; ++r)
            a += acc[((int64_t)r * rows + row) * D + d] * exp2f(m[(int64_t)r * rows + row] - Mr);
        out[(int64_t)row * D + d] = __float2bfloat16_rn(a / Ls);
    }
}

}  // namespace kivi

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using namespace kivi;

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D map over [rows, cols] of `elem` bytes each, row pitch `pitch_bytes`.
bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t cols, uint64_t rows,
              uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DevInfo { int sms = 0; int occ[3] = {0, 0, 0}; };
DevInfo& dev_info(int dev) {
    static DevInfo info[64];
    return info[dev & 63];
}

template <int FMT>
size_t fast_smem_bytes() {
    return 1024 + NST * StageLayout<FMT>::BYTES + NWARP_C * 8 * PB_PITCH * 2 +
           (FMT == FMT_NVFP4 ? NWARP_C * 32 * 8 * 2 : 0) + sizeof(SmemCtl) + 16;
}

int num_sms(int* dev_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    DevInfo& di = dev_info(dev);
    if (!di.sms) cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev_out) *dev_out = dev;
    return di.sms;
}

template <int FMT>
int fast_occupancy(int dev) {
    DevInfo& di = dev_info(dev);
    const int k = (FMT == FMT_NVFP4) ? 1 : (FMT == FMT_MIX43) ? 2 : 0;
    if (!di.occ[k]) {
        const size_t smem = fast_smem_bytes<FMT>();
        if (cudaFuncSetAttribute(decode_fast_kernel<FMT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess ||
            cudaFuncSetAttribute(decode_fast_kernel<FMT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return 0;
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_fast_kernel<FMT, false>, NTHREADS, smem) !=
            cudaSuccess)
            return 0;
        di.occ[k] = occ > 0 ? occ : 1;
    }
    return di.occ[k];
}

constexpr int MAX_CTAS_PER_SM = 4;

struct Plan { int T; int64_t W; int N; int64_t slots; };

Plan make_plan(int BH, int n_full, int sms, int ctas_per_sm) {
    Plan pl;
    pl.T = (n_full + TILE - 1) / TILE;
    pl.W = (int64_t)BH * pl.T;
    int64_t cap = (int64_t)sms * (ctas_per_sm < MAX_CTAS_PER_SM ? ctas_per_sm : MAX_CTAS_PER_SM);
    pl.N = (int)(pl.W < cap ? pl.W : cap);
    pl.slots = pl.W > 0 ? (int64_t)(pl.N + BH) * NWARP_C : 0;
    return pl;
}

int decode_impl(int mode, const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                const void* k_scale, int k_np_stride, const void* k_hot, int hot_stride,
                const uint8_t* v_packed, const void* v_scale, int v_s_stride, int B, int Hq, int Hkv,
                int S, int D, int fmt, float sm_scale, float g_k, float g_v, void* out, float* m_out,
                float* l_out, float* acc_out, float* work, int64_t work_floats, int* err,
                kivi_stream_t stream, const int* seq_lens = nullptr, const void* v_hot = nullptr,
                const SeqPar* sp = nullptr, int Tq = 1, int64_t q_st = 0, int q_pos = -1) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || S < 0 || D <= 0 || D % BLK) return KIVI_ERR_ARG;
    if (fmt != FMT_INT4 && fmt != FMT_NVFP4 && fmt != FMT_MIX43) return KIVI_ERR_ARG;
    if (fmt == FMT_MIX43 && D % 32) return KIVI_ERR_ARG;
    const bool mq = q_pos >= 0;                       // multi-query decode
    if (Tq < 1 || (!mq && Tq != 1) || (mq && (mode != 0 || seq_lens || sp || q_pos + Tq > S)))
        return KIVI_ERR_ARG;
    const int Gq = Hq / Hkv, BH = B * Hkv;
    const int G = Gq * Tq;                            // columns of the group: (query, head) pairs
    const int nf_real = (S / BLK) * BLK, hot_real = S - nf_real;
    // the split kernels see the page-aligned prefix every query attends; a
    // multi-query decode's later tokens go to the merge with per-query limits
    const int S_eff = mq ? ((q_pos + 1) / BLK) * BLK : S;
    const int n_full = (S_eff / BLK) * BLK, hot = S_eff - n_full;
    const int v_tokens = v_hot ? nf_real : S;         // tokens v_packed must cover
    if (k_np_stride < nf_real / BLK || v_s_stride < v_tokens || (hot_real > 0 && hot_stride < hot_real))
        return KIVI_ERR_ARG;
    if (hot_real > 0 && v_hot && !k_hot) return KIVI_ERR_ARG;
    if (!q || (!out && mode != 1) || (mode == 1 && (!m_out || !l_out || !acc_out))) return KIVI_ERR_ARG;
    if (mode == 2 && (!sp || !sp->xbuf || !sp->peers || !sp->row_epoch || sp->W <= 0 || sp->W > 16 ||
                      sp->rank < 0 || sp->rank >= sp->W || sp->timeout_ns <= 0))
        return KIVI_ERR_ARG;
    if (nf_real > 0 && (!k_packed || !k_scale)) return KIVI_ERR_ARG;
    if (v_tokens > 0 && (!v_packed || !v_scale)) return KIVI_ERR_ARG;
    if (hot_real > 0 && !k_hot) return KIVI_ERR_ARG;
    int dev = 0;
    const int sms = num_sms(&dev);
    if (!sms) return record_cuda_error(cudaGetLastError());

    const bool fast = D == DH && G <= 8 && sm_scale > 0.0f && k_np_stride % 16 == 0 && v_s_stride % 16 == 0 &&
                      (uintptr_t)k_packed % 16 == 0 && (uintptr_t)k_scale % 16 == 0 &&
                      (uintptr_t)v_packed % 16 == 0 && (uintptr_t)v_scale % 16 == 0 &&
                      q_sh % 2 == 0 && q_st % 2 == 0 && (uintptr_t)q % 4 == 0 && n_full > 0 &&
                      (int64_t)BH * v_s_stride < (1LL << 31) && (int64_t)BH * D < (1LL << 31);
    if (!fast && (G > GEN_MAXG || D > 32 * GEN_MAXC)) return KIVI_ERR_UNSUPPORTED;
    const int occ = !fast ? 4 : fmt == FMT_NVFP4 ? fast_occupancy<FMT_NVFP4>(dev)
                             : fmt == FMT_MIX43 ? fast_occupancy<FMT_MIX43>(dev) : fast_occupancy<FMT_INT4>(dev);
    if (!occ) return record_cuda_error(cudaGetLastError());
    const Plan pl = make_plan(BH, n_full, sms, occ);   // varlen: bounds from the max length S
    const int64_t need = pl.slots * G * (2 + (int64_t)D) + (seq_lens ? BH + 2 : 0);
    if (need > 0 && (!work || work_floats < need)) return KIVI_ERR_ARG;

    DecodeParams p{};
    p.q = reinterpret_cast<const __nv_bfloat16*>(q); p.q_sb = q_sb; p.q_sh = q_sh;
    p.q_st = q_st; p.Tq = Tq; p.Gq = Gq; p.Hq0 = Hq; p.mq = mq; p.q_pos = q_pos; p.nf_real = nf_real;
    p.k_packed = k_packed; p.k_scale = k_scale; p.k_np_stride = k_np_stride;
    p.k_hot = reinterpret_cast<const __nv_bfloat16*>(k_hot); p.hot_stride = hot_stride;
    p.v_packed = v_packed; p.v_scale = v_scale; p.v_s_stride = v_s_stride;
    p.B = B; p.Hq = Hkv * G; p.Hkv = Hkv; p.G = G; p.S = S_eff; p.D = D; p.n_full = n_full; p.hot = hot;
    p.sm_scale = sm_scale; p.g_k = g_k; p.g_v = g_v;
    p.scale2 = sm_scale * 1.4426950408889634f * (fmt == FMT_NVFP4 ? g_k : 1.0f);
    p.T = pl.T; p.W = pl.W; p.N = pl.N;
    p.part_m = work; p.part_l = work + pl.slots * G; p.part_acc = work + 2 * pl.slots * G;
    p.err = err;
    p.seq_lens = seq_lens;
    p.v_hot = reinterpret_cast<const __nv_bfloat16*>(v_hot);
    if (sp) {
        p.xbuf = sp->xbuf; p.peers = sp->peers; p.xW = sp->W; p.xrank = sp->rank;
        p.row_epoch = sp->row_epoch; p.timeout_ns = sp->timeout_ns;
    }
    p.tile_off = seq_lens ? reinterpret_cast<int*>(work + pl.slots * G * (2 + (int64_t)D)) : nullptr;
    cudaStream_t st = (cudaStream_t)stream;
    if (seq_lens && pl.W > 0) {
        tile_offsets_kernel<<<1, 1024, 0, st>>>(seq_lens, B, Hkv, S, p.tile_off);
        const int e = check_launch();
        if (e) return e;
    }

    if (pl.W > 0) {
        if (fast) {
            CUtensorMap tkc, tks, tvc, tvs;
            const uint64_t rows_k = (uint64_t)BH * DH, rows_v = (uint64_t)BH * v_s_stride;
            bool ok = make_map(&tkc, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_packed, (uint64_t)k_np_stride * 8, rows_k,
                               (uint64_t)k_np_stride * 8, 64, 128, CU_TENSOR_MAP_SWIZZLE_64B) &&
                      (fmt == FMT_MIX43
                           ? make_map(&tvc, CU_TENSOR_MAP_DATA_TYPE_UINT8, v_packed, 48, rows_v, 48, 48, 32,
                                      CU_TENSOR_MAP_SWIZZLE_NONE)
                           : make_map(&tvc, CU_TENSOR_MAP_DATA_TYPE_UINT8, v_packed, 64, rows_v, 64, 64, 128,
                                      CU_TENSOR_MAP_SWIZZLE_64B));
            if (fmt == FMT_NVFP4) {
                ok = ok && make_map(&tks, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_scale, (uint64_t)k_np_stride, rows_k,
                                    (uint64_t)k_np_stride, 16, 128, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                     make_map(&tvs, CU_TENSOR_MAP_DATA_TYPE_UINT8, v_scale, 16, rows_v / 2, 16, 16, 64,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
            } else {
                ok = ok && make_map(&tks, CU_TENSOR_MAP_DATA_TYPE_UINT16, k_scale, (uint64_t)k_np_stride, rows_k,
                                    (uint64_t)k_np_stride * 2, 8, 128, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                     make_map(&tvs, CU_TENSOR_MAP_DATA_TYPE_UINT16, v_scale, 8, rows_v, 16, 8, 128,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
            }
            if (!ok) return KIVI_ERR_CUDA;
            if (fmt == FMT_MIX43 && G <= 4)
                decode_fast_kernel<FMT_MIX43, true><<<pl.N, NTHREADS, fast_smem_bytes<FMT_MIX43>(), st>>>(tkc, tks, tvc, tvs, p);
            else if (fmt == FMT_MIX43)
                decode_fast_kernel<FMT_MIX43, false><<<pl.N, NTHREADS, fast_smem_bytes<FMT_MIX43>(), st>>>(tkc, tks, tvc, tvs, p);
            else if (fmt == FMT_NVFP4 && G <= 4)
                decode_fast_kernel<FMT_NVFP4, true><<<pl.N, NTHREADS, fast_smem_bytes<FMT_NVFP4>(), st>>>(tkc, tks, tvc, tvs, p);
            else if (fmt == FMT_NVFP4)
                decode_fast_kernel<FMT_NVFP4, false><<<pl.N, NTHREADS, fast_smem_bytes<FMT_NVFP4>(), st>>>(tkc, tks, tvc, tvs, p);
            else if (G <= 4)
                decode_fast_kernel<FMT_INT4, true><<<pl.N, NTHREADS, fast_smem_bytes<FMT_INT4>(), st>>>(tkc, tks, tvc, tvs, p);
            else
                decode_fast_kernel<FMT_INT4, false><<<pl.N, NTHREADS, fast_smem_bytes<FMT_INT4>(), st>>>(tkc, tks, tvc, tvs, p);
        } else {
            if (fmt == FMT_NVFP4) decode_generic_kernel<FMT_NVFP4><<<pl.N, 128, 0, st>>>(p);
            else if (fmt == FMT_MIX43) decode_generic_kernel<FMT_MIX43><<<pl.N, 128, 0, st>>>(p);
            else decode_generic_kernel<FMT_INT4><<<pl.N, 128, 0, st>>>(p);
        }
        int e = check_launch();
        if (e) return e;
    }
    // a head of T tiles touches at most ceil(T / floor(W/N)) + 1 CTAs
    int max_ctas = 0;
    if (pl.W > 0) {
        const int64_t per = std::max<int64_t>(pl.W / pl.N, 1);
        max_ctas = seq_lens ? pl.N + 1 : (int)((pl.T + per - 1) / per) + 1;
    }
    // 16 warps per merge row when a head spans many CTAs (long slot rows)
    const int nwc = pl.N >= 16LL * BH ? 16 : 4;
    const size_t csm = ((size_t)2 * max_ctas * NWARP_C + ((16 + Tq - 1 + 3) & ~3) + 2 * nwc + nwc * DH) *
                       sizeof(float);
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
    const dim3 cgrid(BH, G);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = cgrid;
    cfg.blockDim = dim3(32 * nwc);
    cfg.dynamicSmemBytes = csm;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto launch_c = [&](auto kern) { return cudaLaunchKernelEx(&cfg, kern, p, mode, o, m_out, l_out, acc_out); };
    cudaError_t le;
    if (fmt == FMT_NVFP4) le = nwc == 16 ? launch_c(combine_kernel<FMT_NVFP4, 16>) : launch_c(combine_kernel<FMT_NVFP4, 4>);
    else if (fmt == FMT_MIX43) le = nwc == 16 ? launch_c(combine_kernel<FMT_MIX43, 16>) : launch_c(combine_kernel<FMT_MIX43, 4>);
    else le = nwc == 16 ? launch_c(combine_kernel<FMT_INT4, 16>) : launch_c(combine_kernel<FMT_INT4, 4>);
    if (le != cudaSuccess) return record_cuda_error(le);
    return check_launch();
}

}  // namespace

extern "C" int64_t kivi_decode_workspace_floats(int B, int Hq, int Hkv, int S, int D) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || S < 0 || D <= 0) return 0;
    int sms = num_sms(nullptr);
    if (!sms) sms = 148;
    const Plan pl = make_plan(B * Hkv, (S / BLK) * BLK, sms, MAX_CTAS_PER_SM);
    return pl.slots * (Hq / Hkv) * (2 + (int64_t)D) + B * Hkv + 2;   // + varlen tile table
}

extern "C" int kivi_decode_varlen(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                                  const void* k_scale, int k_np_stride, const void* k_hot, int hot_stride,
                                  const uint8_t* v_packed, const void* v_scale, int v_s_stride,
                                  const int* seq_lens, int B, int Hq, int Hkv, int S_max, int D, int fmt,
                                  float sm_scale, float g_k, float g_v, void* out, float* work,
                                  int64_t work_floats, int* err, kivi_stream_t stream) {
    if (!seq_lens) return KIVI_ERR_ARG;
    return decode_impl(0, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed, v_scale,
                       v_s_stride, B, Hq, Hkv, S_max, D, fmt, sm_scale, g_k, g_v, out, nullptr, nullptr, nullptr,
                       work, work_floats, err, stream, seq_lens);
}

extern "C" int kivi_decode(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                           const void* k_scale, int k_np_stride, const void* k_hot, int hot_stride,
                           const uint8_t* v_packed, const void* v_scale, int v_s_stride, int B, int Hq,
                           int Hkv, int S, int D, int fmt, float sm_scale, float g_k, float g_v, void* out,
                           float* work, int64_t work_floats, int* err, kivi_stream_t stream) {
    return decode_impl(0, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed, v_scale,
                       v_s_stride, B, Hq, Hkv, S, D, fmt, sm_scale, g_k, g_v, out, nullptr, nullptr, nullptr,
                       work, work_floats, err, stream);
}

extern "C" int kivi_decode_multiquery(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                                      const uint8_t* k_packed, const void* k_scale, int k_np_stride,
                                      const void* k_hot, const void* v_hot, int hot_stride,
                                      const uint8_t* v_packed, const void* v_scale, int v_s_stride, int B,
                                      int Tq, int q_pos, int Hq, int Hkv, int S, int D, int fmt, float sm_scale,
                                      float g_k, float g_v, void* out, float* work, int64_t work_floats,
                                      int* err, kivi_stream_t stream) {
    if (Tq < 1 || q_pos < 0) return KIVI_ERR_ARG;
    return decode_impl(0, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed, v_scale,
                       v_s_stride, B, Hq, Hkv, S, D, fmt, sm_scale, g_k, g_v, out, nullptr, nullptr, nullptr,
                       work, work_floats, err, stream, nullptr, v_hot, nullptr, Tq, q_st, q_pos);
}

extern "C" int kivi_decode_bf16_tail(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                                     const void* k_scale, int k_np_stride, const void* k_hot, const void* v_hot,
                                     int hot_stride, const uint8_t* v_packed, const void* v_scale,
                                     int v_s_stride, int B, int Hq, int Hkv, int S, int D, int fmt,
                                     float sm_scale, float g_k, float g_v, void* out, float* work,
                                     int64_t work_floats, int* err, kivi_stream_t stream) {
    if ((S % BLK) && !v_hot) return KIVI_ERR_ARG;
    return decode_impl(0, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed, v_scale,
                       v_s_stride, B, Hq, Hkv, S, D, fmt, sm_scale, g_k, g_v, out, nullptr, nullptr, nullptr,
                       work, work_floats, err, stream, nullptr, v_hot);
}

extern "C" int kivi_decode_partial(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                                   const void* k_scale, int k_np_stride, const void* k_hot, int hot_stride,
                                   const uint8_t* v_packed, const void* v_scale, int v_s_stride, int B,
                                   int Hq, int Hkv, int S, int D, int fmt, float sm_scale, float g_k,
                                   float g_v, float* m_out, float* l_out, float* acc_out, float* work,
                                   int64_t work_floats, int* err, kivi_stream_t stream) {
    return decode_impl(1, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed, v_scale,
                       v_s_stride, B, Hq, Hkv, S, D, fmt, sm_scale, g_k, g_v, nullptr, m_out, l_out, acc_out,
                       work, work_floats, err, stream);
}

extern "C" int64_t kivi_seqpar_buffer_bytes(int rows, int D, int W) {
    if (rows <= 0 || D <= 0 || W <= 0 || W > 16) return 0;
    return xflag_bytes(W, rows) + 2 * xslot_floats(rows, D) * (int64_t)sizeof(float);
}

extern "C" int kivi_decode_seqpar(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                                  const void* k_scale, int k_np_stride, const void* k_hot, int hot_stride,
                                  const uint8_t* v_packed, const void* v_scale, int v_s_stride, int B, int Hq,
                                  int Hkv, int S, int D, int fmt, float sm_scale, float g_k, float g_v, void* xbuf,
                                  const uint64_t* peer_bufs, int W, int rank, unsigned int* row_epoch,
                                  long long timeout_ns, void* out, float* work, int64_t work_floats, int* err,
                                  kivi_stream_t stream) {
    SeqPar sp{static_cast<uint8_t*>(xbuf), peer_bufs, W, rank, row_epoch, timeout_ns};
    return decode_impl(2, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed, v_scale,
                       v_s_stride, B, Hq, Hkv, S, D, fmt, sm_scale, g_k, g_v, out, nullptr, nullptr, nullptr,
                       work, work_floats, err, stream, nullptr, nullptr, &sp);
}

extern "C" int kivi_lse_merge(const float* m, const float* l, const float* acc, int R, int rows, int D,
                              void* out, kivi_stream_t stream) {
    if (R <= 0 || rows < 0 || D <= 0 || !m || !l || !acc || !out) return KIVI_ERR_ARG;
    if (rows == 0) return KIVI_OK;
    lse_merge_kernel<<<rows, 128, 0, (cudaStream_t)stream>>>(m, l, acc, R, rows, D,
                                                             reinterpret_cast<__nv_bfloat16*>(out));
    return check_launch();
}

// ---------------------------------------------------------------------------
// Allocation-free decode.
//
// Some callers cannot call cudaMalloc at decode time: a serving engine that
// hands out all device memory from its own pre-sized pool, or an FFI host
// (Go, Java) that owns no CUDA allocator.  For them the split-K partials live in one fixed, library-owned
// device array instead of a caller-supplied workspace.  Its size is fixed at
// KIVI_NOALLOC_SCRATCH_FLOATS fp32 values (8 MiB) and every GPU that loads the
// library keeps it until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_scratch[KIVI_NOALLOC_SCRATCH_FLOATS];

namespace {
struct NoallocSlot { float* ptr = nullptr; bool ready = false; };
std::mutex g_noalloc_mu;
NoallocSlot g_noalloc_slots[64];

// Device address of the scratch array for the current device.  In host code
// `g_noalloc_scratch` is only a host-side stand-in for the symbol, so the
// address must be looked up once per device with that device current.
int noalloc_scratch_ptr(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (dev < 0 || dev >= 64) return KIVI_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoallocSlot& s = g_noalloc_slots[dev];
    if (!s.ready) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return record_cuda_error(e);
        s.ptr = static_cast<float*>(p);
        s.ready = true;
    }
    *out = s.ptr;
    return KIVI_OK;
}
}  // namespace

extern "C" int kivi_decode_noalloc(const void* q, int64_t q_sb, int64_t q_sh, const uint8_t* k_packed,
                                   const void* k_scale, int k_np_stride, const void* k_hot, int hot_stride,
                                   const uint8_t* v_packed, const void* v_scale, int v_s_stride, int B,
                                   int Hq, int Hkv, int S, int D, int fmt, float sm_scale, float g_k,
                                   float g_v, void* out, int* err, kivi_stream_t stream) {
    const int64_t need = kivi_decode_workspace_floats(B, Hq, Hkv, S, D);
    if (need > KIVI_NOALLOC_SCRATCH_FLOATS) return KIVI_ERR_SCRATCH;
    float* scratch = nullptr;
    const int rc = noalloc_scratch_ptr(&scratch);
    if (rc != KIVI_OK) return rc;
    // Every slot the merge reads is written by the split kernel of the same
    // call, so nothing in the scratch has to start at zero.
    return decode_impl(0, q, q_sb, q_sh, k_packed, k_scale, k_np_stride, k_hot, hot_stride, v_packed,
                       v_scale, v_s_stride, B, Hq, Hkv, S, D, fmt, sm_scale, g_k, g_v, out, nullptr, nullptr,
                       nullptr, scratch, KIVI_NOALLOC_SCRATCH_FLOATS, err, stream);
}
