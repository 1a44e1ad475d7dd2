/*
 * kivi_sm100.h -- C ABI of libkivi_sm100.so, the B200 (sm_100a) 4-bit
 * KV-cache library: INT4-KIVI / NVFP4-KIVI quantize-and-store, dequant, the
 * kv_quant roundtrip primitive, and fused split-K flash-decode with an LSE
 * merge.
 *
 * Conventions
 *   - Every pointer is device memory owned by the caller; nothing here
 *     allocates, frees or synchronises.  Work is enqueued on `stream`
 *     (a cudaStream_t; NULL = legacy default stream).
 *   - Element strides are in elements of the pointed-to type.
 *   - bf16 / fp16 tensors are passed as `const void*` (raw 16-bit words).
 *   - Return value: KIVI_OK (0) or a kivi_status code; kivi_status_string()
 *     names it.  Argument errors are detected before any launch.
 *   - Device-side timeouts (a pipeline wait that never completes) do not trap:
 *     the kernel writes a nonzero code into `err` (if non-NULL) and returns.
 *
 * Reference interfaces replaced (paths inside a1exxd0/poolside-hackathon):
 * each entry point cites the Triton kernel + host wrapper it stands in for.
 */
#ifndef KIVI_SM100_H
#define KIVI_SM100_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *kivi_stream_t;   /* == cudaStream_t */

enum kivi_status {
    KIVI_OK = 0,
    KIVI_ERR_ARG = 1,          /* bad shape / null pointer / bad enum       */
    KIVI_ERR_ALIGN = 2,        /* pointer or stride violates alignment rule */
    KIVI_ERR_UNSUPPORTED = 3,  /* valid but not implemented (e.g. head_dim) */
    KIVI_ERR_CUDA = 4,         /* a CUDA runtime/driver call failed         */
    KIVI_ERR_TIMEOUT = 5,      /* device-side bounded wait expired          */
    KIVI_ERR_SCRATCH = 6       /* problem exceeds the fixed no-alloc scratch */
};

/* KIVI_FMT_INT3 is a kivi_roundtrip / kivi_calibrate grid only.  A cache of
 * KIVI_FMT_MIX43 keeps K as INT4 (the INT4 K layout) and V as INT3 on the
 * kv_quant.py:215-217 `int3` grid (qmax 3, fp16 scales), the 3-bit-V / 4-bit-K
 * cache WRITEUP.md:336-339 names (the reference ships no packed INT3 format;
 * this layout is the library's own).  V blocks go in pairs: v_packed rows are
 * [D/32][12] bytes, little-endian u32 words A_2k, A_2k+1, S_k; a code c in
 * [-3, 3] is L = c & 3 plus sign s (c = L - 4s); A_b holds L of element
 * i < 8 at bits 4i..4i+1 and of element 8+i at 4i+2..4i+3; S_k holds s of
 * element i < 8 of block 2k+o at bit 4i+2o and of element 8+i at 4i+1+2o.
 * D must be a multiple of 32.  Every store, dequant and decode entry point
 * takes it (the paged entry points do not). */
enum kivi_fmt { KIVI_FMT_INT4 = 0, KIVI_FMT_INT3 = 1, KIVI_FMT_NVFP4 = 2, KIVI_FMT_MIX43 = 3 };
enum kivi_calib { KIVI_CALIB_ABSMAX = 0, KIVI_CALIB_MSE = 1 };
enum kivi_layout { KIVI_LAYOUT_HEADDIM = 0, KIVI_LAYOUT_CHANNEL = 1 };
enum kivi_dtype { KIVI_DT_BF16 = 0, KIVI_DT_F16 = 1, KIVI_DT_F32 = 2 };

const char *kivi_status_string(int status);
int kivi_version(void);                 /* 100 * major + minor */
int kivi_last_cuda_error(void);         /* cudaError_t of the last KIVI_ERR_CUDA */

/* ------------------------------------------------------------------------ */
/* Quantize-and-store.                                                       */
/*                                                                           */
/* Replaces int4_kivi/triton_kernels.py:137-178 (k_store_kernel),            */
/* :216-254 (v_store_kernel) and their launches in int4_kivi/cache.py:90-141.*/
/*                                                                           */
/* Input K: [H, S_k, D], V: [H, S_v, D] of `in_dtype` (bf16, fp16, fp32).  */
/* (S_k and S_v differ on append: K pages vs new V tokens, one launch.)      */
/* K: the first (S_k/16)*16 tokens, per channel over 16-token pages, are     */
/*    written to k_packed[h, d, kpage0 + p, 0:8] (row stride k_np_stride     */
/*    pages) and k_scale[h, d, kpage0 + p].  Input token 0 must start a page. */
/* V: every token, per 16-channel block, to v_packed[h, vtok0 + t, db, 0:8]  */
/*    (head stride v_s_stride tokens) and v_scale[h, vtok0 + t, db].          */
/* fmt INT4: scale = fp16 (2 bytes), codes two's-complement nibbles.         */
/* fmt NVFP4: scale = e4m3 byte of (s / g), codes e2m1 nibbles (g_k, g_v).   */
/* fmt MIX43: K as INT4; V INT3, 12 bytes per block pair per token (above). */
/* alphas: device fp32 [n_alphas], the MSE clip grid linspace(0.5, 1, n).    */
/* D must be a multiple of 16.                                               */
/* ------------------------------------------------------------------------ */
int kivi_store(const void *k, const void *v, int in_dtype,
               int64_t sk_h, int64_t sk_s, int64_t sk_d,
               int64_t sv_h, int64_t sv_s, int64_t sv_d,
               int H, int S_k, int S_v, int D, int fmt, int calib_k, int calib_v,
               const float *alphas, int n_alphas, float g_k, float g_v,
               uint8_t *k_packed, void *k_scale, int kpage0, int k_np_stride,
               uint8_t *v_packed, void *v_scale, int vtok0, int v_s_stride,
               kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Dequantize to bf16 [H, S, D] (out strides in elements).                   */
/* Replaces int4_kivi/triton_kernels.py:181-210 (k_dequant_kernel),          */
/* :257-286 (v_dequant_kernel) and int4_kivi/cache.py:165-201.               */
/* K writes tokens [0, (S/16)*16) only (the bf16 hot tail is the caller's);  */
/* V writes every token.  value = code * fp32(scale) (NVFP4: * g).           */
/* ------------------------------------------------------------------------ */
int kivi_dequant(const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                 const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                 int H, int S, int D, int fmt, float g_k, float g_v,
                 void *k_out, void *v_out, int64_t so_h, int64_t so_s, int64_t so_d,
                 kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* kv_quant.roundtrip on the GPU.  Replaces kv_quant.py:299-321 (and         */
/* _calibrate/_to_blocks :232-266) for x [H, S, D] contiguous of `dtype`.    */
/* 'channel' copies the trailing S % 16 tokens unchanged.                    */
/* ------------------------------------------------------------------------ */
int kivi_roundtrip(const void *x, void *y, int dtype, int H, int S, int D,
                   int fmt, int layout, int calib, const float *alphas, int n_alphas,
                   kivi_stream_t stream);

/* kv_quant.py:247-266 `_calibrate` over n contiguous fp32 blocks [n, 16]. */
int kivi_calibrate(const float *blocks, int64_t n, int fmt, int calib,
                   const float *alphas, int n_alphas, float *scales,
                   kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Legacy page-level dequant.  Replaces kv_quant.py:70-76                    */
/* (QuantizedPage.dequantize: `q.to(fp16) * scale`, then `.to(bfloat16)`)     */
/* and the unpacked int8 codes of kv_quant.py:37-38 (quantize_block).        */
/* packed u8 [rows, row_stride, D/16, 8] and fp16 scale [rows, row_stride,   */
/* D/16] as written by kivi_store's V path (per-token 16-channel blocks).    */
/* out  : bf16 [rows, tokens, D] = bf16(fp16(code * scale)), or NULL.        */
/* codes: int8 [rows, tokens, D], or NULL.  out / codes 16-byte aligned.     */
/* ------------------------------------------------------------------------ */
int kivi_page_dequant(const uint8_t *packed, const void *scale, int rows, int tokens,
                      int row_stride, int D, void *out, int8_t *codes,
                      kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Fused split-K flash-decode over a packed cache.                           */
/*                                                                           */
/* Replaces int4_kivi/decode.py:53-219 (_kivi_decode_kernel +                */
/* kivi_decode_attention), :234-317,494-533 (split-K batched) and            */
/* :351-477 (GQA split-K) plus :320-340 (_combine_kernel).                   */
/*                                                                           */
/* q       : bf16 [B, Hq, D] (strides q_sb, q_sh; last dim contiguous)       */
/* cache   : B*Hkv stacked heads, kv-head index b*Hkv + h.                    */
/*           k_packed [BH, D, k_np_stride, 8], k_scale [BH, D, k_np_stride]  */
/*           k_hot bf16 [BH, hot_stride, D] (tokens n_full..S-1)             */
/*           v_packed [BH, v_s_stride, D/16, 8], v_scale [BH, v_s_stride, D/16]*/
/*           fmt INT4: fp16 scales; NVFP4: e4m3 scales with g_k, g_v;        */
/*           MIX43: v_packed [BH, v_s_stride, D/32, 12] (INT3 V, above).     */
/* S       : tokens attended (n_full = (S/16)*16 from pages, rest from k_hot)*/
/* out     : bf16 [B, Hq, D] contiguous.                                     */
/* work    : fp32 scratch of kivi_decode_workspace_floats(...) floats      */
/*           (any contents; calls sharing one workspace must not overlap).   */
/* err     : optional int32 device flag, set nonzero on a device timeout.    */
/* Fast path requirements: D == 128, Hq/Hkv <= 8, k_np_stride % 16 == 0,     */
/* v_s_stride % 16 == 0, 16-byte aligned pointers; otherwise a generic       */
/* CUDA-core path with identical results semantics runs.                     */
/* ------------------------------------------------------------------------ */
int64_t kivi_decode_workspace_floats(int B, int Hq, int Hkv, int S, int D);

int kivi_decode(const void *q, int64_t q_sb, int64_t q_sh,
                const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                const void *k_hot, int hot_stride,
                const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                int B, int Hq, int Hkv, int S, int D, int fmt,
                float sm_scale, float g_k, float g_v,
                void *out, float *work, int64_t work_floats, int *err,
                kivi_stream_t stream);

/* Decode over a cache that keeps its partial last page unquantised (the   */
/* HuggingFace cache layout, int4_kivi/hf_cache.py:107-190): the first      */
/* (S/16)*16 tokens from the packed pages, the last S % 16 tokens from bf16 */
/* k_hot AND v_hot (both [B*Hkv, hot_stride, D]); v_packed / v_scale cover  */
/* only the paged tokens.  Otherwise identical to kivi_decode.              */
int kivi_decode_bf16_tail(const void *q, int64_t q_sb, int64_t q_sh,
                          const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                          const void *k_hot, const void *v_hot, int hot_stride,
                          const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                          int B, int Hq, int Hkv, int S, int D, int fmt,
                          float sm_scale, float g_k, float g_v,
                          void *out, float *work, int64_t work_floats, int *err,
                          kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Variable-length batch decode.  Same as kivi_decode, but batch entry b      */
/* attends only its first seq_lens[b] tokens (device int32 [B], each in      */
/* [0, S_max]); pages, V tokens and the <16-token bf16 tail (k_hot[bh, 0:    */
/* seq_lens[b] % 16]) of every sequence live in the stacked layout sized for */
/* S_max.  Generalises the equal-length stacking of int4_kivi/decode.py:480- */
/* 491 (the reference requires one S for the whole batch); sync-free, the    */
/* per-head tile table is built on the device.                               */
/* ------------------------------------------------------------------------ */
int kivi_decode_varlen(const void *q, int64_t q_sb, int64_t q_sh,
                       const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                       const void *k_hot, int hot_stride,
                       const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                       const int *seq_lens, int B, int Hq, int Hkv, int S_max, int D, int fmt,
                       float sm_scale, float g_k, float g_v,
                       void *out, float *work, int64_t work_floats, int *err,
                       kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Partial-state variant for sequence-parallel decode across GPUs: instead   */
/* of bf16 output, writes this rank's merged (m, l, acc) per (b, q-head):     */
/* m_out/l_out fp32 [B*Hq] (m in log2 units of the scaled score), acc_out    */
/* fp32 [B*Hq, D] unnormalised.  kivi_lse_merge() combines R such records.   */
/* ------------------------------------------------------------------------ */
int kivi_decode_partial(const void *q, int64_t q_sb, int64_t q_sh,
                        const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                        const void *k_hot, int hot_stride,
                        const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                        int B, int Hq, int Hkv, int S, int D, int fmt,
                        float sm_scale, float g_k, float g_v,
                        float *m_out, float *l_out, float *acc_out,
                        float *work, int64_t work_floats, int *err,
                        kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* kivi_decode without a caller workspace: no counterpart in the reference.  */
/* For callers that cannot allocate device memory at decode time (a serving  */
/* engine that hands out all device memory from its own fixed pool, an FFI   */
/* host without a CUDA allocator).  Same arguments and result as kivi_decode,*/
/* minus `work`; the split-K partials go to a library-owned device array of  */
/* KIVI_NOALLOC_SCRATCH_FLOATS floats (8 MiB, held on every GPU that loads   */
/* the library until exit).  Problems whose kivi_decode_workspace_floats()   */
/* exceeds that return KIVI_ERR_SCRATCH before any launch.  The first call   */
/* on a device looks up the array's device address (cudaGetSymbolAddress);   */
/* make that first call before any stream capture.  All calls share the one  */
/* array: calls that overlap on the GPU (different streams, or different     */
/* host threads on the same device) race and must be serialised by the      */
/* caller.  Nothing is allocated or freed.  The looked-up address is kept    */
/* for the life of the process: after a cudaDeviceReset the library must be  */
/* reloaded before this entry point is used again on that device.           */
/* ------------------------------------------------------------------------ */
#define KIVI_NOALLOC_SCRATCH_FLOATS (1 << 21)

int kivi_decode_noalloc(const void *q, int64_t q_sb, int64_t q_sh,
                        const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                        const void *k_hot, int hot_stride,
                        const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                        int B, int Hq, int Hkv, int S, int D, int fmt,
                        float sm_scale, float g_k, float g_v,
                        void *out, int *err, kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Multi-query (speculative / chunked) decode: Tq query tokens per sequence, */
/* query j at position q_pos + j of the cache attending tokens 0..q_pos + j  */
/* (causal); q_pos + Tq <= S, so the queries' own K/V are already stored.    */
/* The reference's decode takes one query token (int4_kivi/decode.py:439-   */
/* 477 takes q [B, Hq, D]); this extends it the way a verify step of         */
/* speculative decoding needs.  q bf16 [B, Tq, Hq, D] (strides q_sb, q_st,   */
/* q_sh; last dim contiguous); out bf16 [B, Tq, Hq, D] contiguous; cache     */
/* arguments as kivi_decode; v_hot (nullable) as kivi_decode_bf16_tail: the */
/* partial page's V in bf16 [BH, hot_stride, D].  The (query, head) pairs of */
/* a kv head form the                                                        */
/* kernel's column group (Tq * Hq/Hkv <= 8 on the fast path, <= 16 on the    */
/* CUDA-core path); work: kivi_decode_workspace_floats(B, Tq * Hq, Hkv, S,   */
/* D) floats.                                                                */
/* ------------------------------------------------------------------------ */
int kivi_decode_multiquery(const void *q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                           const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                           const void *k_hot, const void *v_hot, int hot_stride,
                           const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                           int B, int Tq, int q_pos, int Hq, int Hkv, int S, int D, int fmt,
                           float sm_scale, float g_k, float g_v,
                           void *out, float *work, int64_t work_floats, int *err,
                           kivi_stream_t stream);

/* Log-sum-exp merge of R partial records laid out [R, rows] / [R, rows, D]  */
/* (int4_kivi/decode.py:320-340 semantics) -> bf16 out [rows, D].            */
int kivi_lse_merge(const float *m, const float *l, const float *acc, int R, int rows,
                   int D, void *out, kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Paged cache (vLLM block layout).                                          */
/*                                                                           */
/* Replaces the fork kernels the reference calls through                     */
/* vllm/v1/attention/ops/triton_{int4,nvfp4}_kivi.py (source not in the      */
/* reference tree; call sites scripts/validate_paged_decode.py:59,72,91,     */
/* scripts/validate_store_equiv.py:50-51, scripts/validate_nvfp4_kivi.py:    */
/* 67-75,136-150, scripts/bench_paged_decode.py:97-100): int4_kivi_store,    */
/* int4_kivi_gather_dequant, int4_kivi_paged_decode and the nvfp4_* twins.   */
/*                                                                           */
/* kv_cache: uint8 [num_blocks, 2, 16, H, FD], FD = kivi_paged_full_dim(D)   */
/*   = D/2 + D/16; dim 1 = K (0) / V (1); a row is D/2 code bytes (element   */
/*   2j in the low nibble of byte j) then D/16 e4m3 scale bytes.  V and K of */
/*   a partial block: per token (scale j covers channels 16j..16j+15).  K of */
/*   a full block ((b+1)*16 <= seq_len): per channel over its 16 tokens,     */
/*   channel c's scale at row c / (D/16), byte c % (D/16).                   */
/*   fmt INT4: codes in [-7, 7]; NVFP4: e2m1 codes (sign = bit 3).           */
/* ------------------------------------------------------------------------ */
int kivi_paged_full_dim(int D);

/* Quantise N tokens k, v [N, H, D] (dtype in_dtype, strides in elements for */
/* token, head, channel) into kv_cache at slot_mapping[N] (int64, device;    */
/* slot = block * 16 + offset; negative = padding, skipped).  A call that    */
/* writes a block's last slot quantises that block's K per channel (rows not */
/* in the call are dequantised from the cache first); other K rows go per    */
/* token.  calib: KIVI_CALIB_MSE (16-point e4m3 clip search) or ABSMAX.      */
/* Out-of-range slots set *err = KIVI_ERR_ARG and are skipped.  D <= 256.    */
int kivi_paged_store(const void *k, const void *v, int in_dtype,
                     int64_t sk_t, int64_t sk_h, int64_t sk_d,
                     int64_t sv_t, int64_t sv_h, int64_t sv_d,
                     int N, int H, int D, int fmt, int calib,
                     const int64_t *slot_mapping, uint8_t *kv_cache, int64_t num_blocks,
                     int *err, kivi_stream_t stream);

/* bf16 k_out, v_out [B, H, max_seq, D] from block_table int32 [B, bt_stride] */
/* and seq_lens int32 [B]; positions at or past seq_len are written as 0.    */
int kivi_paged_gather_dequant(const uint8_t *kv_cache, int64_t num_blocks,
                              const int *block_table, int64_t bt_stride, const int *seq_lens,
                              int B, int H, int D, int fmt, int max_seq,
                              void *k_out, void *v_out, int *err, kivi_stream_t stream);

/* Fused decode, one query token per sequence: q bf16 [B, Hq, D] (strides    */
/* q_sb, q_sh) -> out bf16 [B, Hq, D] contiguous.  Sequence b attends its    */
/* first min(seq_lens[b], 16 * bt_stride) tokens (0 gives zeros).  The grid  */
/* is sized from bt_stride, never from seq_lens, so the call never reads     */
/* device data on the host and is graph-capturable.  work: fp32 scratch of   */
/* kivi_paged_decode_workspace_floats(B, Hq, Hkv, bt_stride, D) floats.      */
/* Fast path: D == 128, Hkv <= 16, Hq/Hkv <= 8; otherwise a CUDA-core path.  */
int64_t kivi_paged_decode_workspace_floats(int B, int Hq, int Hkv, int64_t bt_stride, int D);

int kivi_paged_decode(const void *q, int64_t q_sb, int64_t q_sh,
                      const uint8_t *kv_cache, int64_t num_blocks,
                      const int *block_table, int64_t bt_stride, const int *seq_lens,
                      int B, int Hq, int Hkv, int D, int fmt, float sm_scale,
                      void *out, float *work, int64_t work_floats, int *err,
                      kivi_stream_t stream);

/* Same decode with the normalised output kept in fp32 [B, Hq, D] (the value */
/* kivi_paged_decode rounds to bf16): the fork's paged decode has no such    */
/* output; it exists for callers (and parity checks) that want the state     */
/* before the bf16 cast.                                                     */
int kivi_paged_decode_f32(const void *q, int64_t q_sb, int64_t q_sh,
                          const uint8_t *kv_cache, int64_t num_blocks,
                          const int *block_table, int64_t bt_stride, const int *seq_lens,
                          int B, int Hq, int Hkv, int D, int fmt, float sm_scale,
                          float *out, float *work, int64_t work_floats, int *err,
                          kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Sequence-parallel decode with the cross-GPU merge fused into the decode's */
/* own combine kernel (no reference counterpart; replaces decode_partial +  */
/* all-gather + merge).  Every rank calls it with its KV range of the same  */
/* B sequences; the combine CTA of each output row publishes the rank-local */
/* (m, l, acc) of that row into this rank's exchange buffer xbuf, releases  */
/* the row's epoch to every rank, waits (at most timeout_ns, else *err =    */
/* KIVI_ERR_TIMEOUT and the row is left unwritten) for every rank's state   */
/* of the row, reads them through peer_bufs[W] (all ranks' xbuf addresses, */
/* own included) and writes the merged bf16 row.  xbuf:                     */
/* kivi_seqpar_buffer_bytes(B*Hq, D, W) bytes from kivi_peer_alloc (zeroed), */
/* row_epoch: zeroed device uint32 [B*Hq] kept across calls.  Two launches  */
/* per call, graph-capturable.  Other arguments as kivi_decode.             */
/* ------------------------------------------------------------------------ */
int64_t kivi_seqpar_buffer_bytes(int rows, int D, int W);
int kivi_decode_seqpar(const void *q, int64_t q_sb, int64_t q_sh,
                       const uint8_t *k_packed, const void *k_scale, int k_np_stride,
                       const void *k_hot, int hot_stride,
                       const uint8_t *v_packed, const void *v_scale, int v_s_stride,
                       int B, int Hq, int Hkv, int S, int D, int fmt,
                       float sm_scale, float g_k, float g_v,
                       void *xbuf, const uint64_t *peer_bufs, int W, int rank,
                       unsigned int *row_epoch, long long timeout_ns,
                       void *out, float *work, int64_t work_floats, int *err,
                       kivi_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Cross-GPU merge over NVLink peer memory (sequence-parallel decode).       */
/*                                                                           */
/* No reference counterpart (the reference is single-GPU); replaces the      */
/* all-gather + kivi_lse_merge pair with direct peer reads.  Each rank       */
/* allocates kivi_peer_buffer_bytes(rows, D, W) bytes with kivi_peer_alloc   */
/* (zeroed; returns a 64-byte CUDA IPC handle), exchanges the handles over   */
/* the host, maps the others with kivi_peer_open, and passes the device     */
/* array of all W ranks' buffer addresses (peer_bufs[W], own one included)  */
/* and a zeroed device uint32 epoch counter.  Per decode step:              */
/*   kivi_peer_publish: copy this rank's (m [rows] in log2 units, l [rows],  */
/*     acc [rows, D]) into its buffer and release the next epoch to every    */
/*     rank's flag for this rank;                                            */
/*   kivi_peer_merge: wait until every rank published that epoch (at most    */
/*     timeout_ns, else *err = KIVI_ERR_TIMEOUT and the rows are left        */
/*     unwritten), read all W states through the peer pointers and write     */
/*     bf16 out [rows, D].                                                   */
/* Both are stream-ordered and graph-capturable; W <= 16, D % 4 == 0.        */
/* ------------------------------------------------------------------------ */
int64_t kivi_peer_buffer_bytes(int rows, int D, int W);
int kivi_peer_alloc(int64_t bytes, void **ptr, void *ipc_handle);   /* handle: 64 bytes out */
int kivi_peer_open(const void *ipc_handle, void **ptr);
int kivi_peer_close(void *ptr);                                      /* unmap a peer buffer  */
int kivi_peer_free(void *ptr);                                       /* free own buffer      */
int kivi_peer_publish(const float *m, const float *l, const float *acc, int rows, int D,
                      void *my_buf, const uint64_t *peer_bufs, int W, int rank,
                      unsigned int *epoch, kivi_stream_t stream);
int kivi_peer_merge(const uint64_t *peer_bufs, int W, int rows, int D, const unsigned int *epoch,
                    const void *my_buf, void *out, int *err, long long timeout_ns,
                    kivi_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KIVI_SM100_H */
