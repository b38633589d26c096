/* bw_attn.h -- C ABI of the B200 (sm_100a) GQA / MHA attention forward.
 *
 * Drop-in boundary for the attention path of the reference workbench
 * (sanjaykrishnablubridge-bit/Blackwell).  Each entry point names the reference
 * launcher it replaces.  Conventions, shared by every call:
 *
 *  - Tensors are caller-owned DEVICE buffers on the current CUDA device.  The
 *    library allocates nothing; the decode path takes a caller workspace.
 *  - Q, K, V, O are bf16 (raw 16-bit storage, `const void*`).  LSE is fp32,
 *    natural log, [B, Hq, Sq] contiguous (may be NULL: not written).
 *  - Default layout is the reference's BHSD, contiguous: [B, H, S, D].  Any other
 *    layout whose head dimension is contiguous (e.g. BSHD) is passed with
 *    `bw_strides` (element strides of the b, h, s axes).  Strides must be
 *    multiples of 8 elements (16 bytes); base pointers 16-byte aligned.
 *  - GQA routing: query head hq reads KV head hq / G, G = Hq / Hkv.
 *  - D (head dimension) is 64 or 128.  The reference fixes it as a template
 *    parameter (`template<int Br,int Bc,int D>`); here it is a runtime argument.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *    asynchronous; they are reentrant and may be made from several host threads.
 *  - Return codes (never exit()): BW_OK, or an error below.  Argument errors are
 *    detected before any launch.  Device-side failures (a bounded wait that
 *    timed out, a workspace that was too small for the actual lengths) are
 *    recorded in the error word of the call's stream, which bw_stream_status()
 *    reads and clears.
 */
#ifndef BW_ATTN_H_
#define BW_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BW_API __attribute__((visibility("default")))
#else
#define BW_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BW_OK = 0,
  BW_ERR_SHAPE = 1,     /* unsupported or inconsistent sizes */
  BW_ERR_ALIGN = 2,     /* pointer or stride not 16-byte aligned */
  BW_ERR_CUDA = 3,      /* a CUDA runtime / driver call failed */
  BW_ERR_TIMEOUT = 4,   /* a device-side wait exceeded its bound */
  BW_ERR_NCCL = 5,      /* collective failure (multi-GPU helpers) */
  BW_ERR_NULL = 6,      /* required pointer is NULL */
  BW_ERR_WORKSPACE = 7  /* workspace too small */
};

/* Element strides of the batch, head and sequence axes (head-dim stride is 1). */
typedef struct bw_strides {
  int64_t q[3];
  int64_t k[3];
  int64_t v[3];
  int64_t o[3];
} bw_strides;

/* Non-causal GQA forward, Sq = Skv = S.
 * Replaces launch_gqa_v0..v23<Br,Bc,D>(Q,K,V,O,LSE,B,Hq,Hkv,S,G,scale)
 * (src/SM103/attention/GQA_sm103.cu:5733-6516; the sm_120 twins in
 * src/SM120/attention/GQA_sm120.cu:353-380). */
BW_API int bw_gqa_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv, int S,
               int G, int D, float scale, const bw_strides* strides, void* stream);

/* Causal GQA forward (key j visible to query i iff j <= i).
 * Replaces launch_gqa_vN_causal<Br,Bc,D>(Q,K,V,O,LSE,B,Hq,Hkv,S,G,scale)
 * (src/SM103/attention/GQA_sm103_causal.cu:4155-7760,
 *  src/SM103/attention/GQA_sm103_causal_v3.cu:2156-2180). */
BW_API int bw_gqa_causal_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv,
                      int S, int G, int D, float scale, const bw_strides* strides, void* stream);

/* Split-length GQA forward, Sq != Skv (cross-attention / KV-cache prefill).
 * Replaces launch_gqa_v1<Br,Bc,D>(Q,K,V,O,LSE,B,Hq,Hkv,Sq,Skv,G,scale)
 * (src/SM120/attention/adhitya_GQA.cu:199-213).  `causal` = 0 matches the
 * reference; 1 applies the top-left mask j <= i. */
BW_API int bw_gqa_split_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv,
                     int Sq, int Skv, int G, int D, float scale, int causal, const bw_strides* strides,
                     void* stream);

/* Causal attention of a chunk of queries against a longer key prefix
 * (chunked prefill / prefix caching): query row i is sequence position
 * q_offset + i and sees keys j <= q_offset + i; with Skv = q_offset + Sq this
 * is the bottom-right-aligned causal mask.  q_offset = 0 is bw_gqa_split_fwd
 * with causal = 1.  Extends the reference's split-length launcher
 * (adhitya_GQA.cu:199-213), which has no offset. */
BW_API int bw_gqa_causal_offset_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B,
                                    int Hq, int Hkv, int Sq, int Skv, int G, int D, float scale, int q_offset,
                                    const bw_strides* strides, void* stream);

/* MHA forward (G = 1), bf16 in/out, optional LSE.
 * Replaces mha_v3_tc<Br,Bc,D><<<(S/Br,B*H),32,smem>>>(Q,K,V,O,scale,S)
 * (src/SM120/attention/MHA_sm120.cu:64-71, launch :333-345), which is fp32
 * in/out without LSE. */
BW_API int bw_mha_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int H, int S, int D,
               float scale, const bw_strides* strides, void* stream);

/* MHA forward with fp32 inputs and output at fp32 accuracy: the data types and
 * the 3xTF32 split of the reference's mha_v3_tc
 * (src/SM120/attention/MHA_sm120.cu:64-71; split_tf32 :39-62 applied to Q, K
 * and V :119-138).  Each operand is split into TF32 hi / lo parts (written to
 * `workspace`, bw_mha_f32_workspace_size bytes, 256-byte aligned) and
 * Q K^T and P V each run as three kind::tf32 tensor-core products
 * (hi*hi + hi*lo + lo*hi); softmax, sums and O / l in fp32.  D = 64; LSE
 * optional.  Strides are fp32 element strides (multiples of 4). */
BW_API size_t bw_mha_f32_workspace_size(int B, int H, int S, int D);
BW_API int bw_mha_fwd_f32(const float* Q, const float* K, const float* V, float* O, float* LSE, int B, int H, int S,
                          int D, float scale, const bw_strides* strides, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Split-KV single-token decode.  No counterpart kernel exists in the reference;
 * the semantics are its split-length GQA (adhitya_GQA.cu:63-188) with Sq = 1
 * and Skv = kv_lens[b] per sequence.
 *   Q:  bf16 [B, Hq, D] contiguous
 *   K, V: bf16 [total_tokens, Hkv, D] contiguous; sequence b owns tokens
 *         [kv_offsets[b], kv_offsets[b] + kv_lens[b])   (device int64 / int32)
 *   O:  bf16 [B, Hq, D];  LSE: fp32 [B, Hq] or NULL
 * `chunk` = tokens per split (multiple of 64; 0 = default 1024).  The KV of one
 * sequence is split into ceil(L_b / chunk) pieces whose partials are merged by
 * the LSE-combine kernel on the same stream.  `workspace` must hold
 * bw_gqa_decode_workspace_size(B, Hq, Hkv, D, total_tokens, chunk) bytes. */
BW_API size_t bw_gqa_decode_workspace_size(int B, int Hq, int Hkv, int D, int64_t total_tokens, int chunk);
BW_API int bw_gqa_decode(const void* Q, const void* K, const void* V, const int* kv_lens, const int64_t* kv_offsets,
                  void* O, float* LSE, int B, int Hq, int Hkv, int D, int64_t total_tokens, float scale, int chunk,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Split-KV decode over a paged KV cache (new; no reference counterpart -- the
 * closest relative is the reference's split-length launcher, adhitya_GQA.cu:50-55).
 *   K_cache, V_cache: bf16 [num_pages, page_size, Hkv, D] contiguous
 *   block_table: int32 [B, max_pages_per_seq]; token i of sequence b is slot
 *                i % page_size of page block_table[b][i / page_size]
 *   kv_lens: int32 [B];  Q, O, LSE as in bw_gqa_decode.
 * page_size: 8, 16, 32, 64 or any multiple of 64.  Workspace:
 * bw_gqa_decode_workspace_size(B, Hq, Hkv, D, min(num_pages * page_size,
 * B * max_pages_per_seq * page_size), chunk) bytes. */
BW_API int bw_gqa_decode_paged(const void* Q, const void* K_cache, const void* V_cache, const int* block_table,
                               const int* kv_lens, void* O, float* LSE, int B, int Hq, int Hkv, int D, int page_size,
                               int num_pages, int max_pages_per_seq, float scale, int chunk, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Split-KV decode that leaves fp32 partial results for a cross-GPU merge (new;
 * no reference counterpart).  Same arguments as bw_gqa_decode, but O is fp32
 * [B, Hq, D] normalised by this call's own softmax sum and LSE (required) is
 * the natural-log sum over this call's keys (-inf for an empty sequence).  When
 * each GPU holds a slice of every sequence's KV, every GPU runs this on its
 * slice, the partials are all-gathered into [world, B, Hq, D] / [world, B, Hq]
 * and bw_lse_combine merges them. */
BW_API int bw_gqa_decode_partial(const void* Q, const void* K, const void* V, const int* kv_lens,
                                 const int64_t* kv_offsets, float* O, float* LSE, int B, int Hq, int Hkv, int D,
                                 int64_t total_tokens, float scale, int chunk, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* The same decode for callers that cannot allocate device memory (no
 * counterpart in the reference: it is an addition of this library).  Callers
 * such as allocator hooks, memory-pool callbacks or host runtimes that own no
 * allocator cannot supply bw_gqa_decode's workspace; this variant takes none
 * and allocates nothing.  Its scratch is a fixed array of
 * bw_gqa_decode_static_scratch_bytes() (32 MiB) in the library's device data,
 * held on every GPU that loads the library until exit; calls needing more
 * (bw_gqa_decode_workspace_size with the same arguments) fail with
 * BW_ERR_WORKSPACE.  All calls on a device share the array, so calls that
 * overlap on the GPU race.  The first call on a device does a one-time set-up
 * (symbol-address lookup); make it before any stream capture. */
BW_API size_t bw_gqa_decode_static_scratch_bytes(void);
BW_API int bw_gqa_decode_static(const void* Q, const void* K, const void* V, const int* kv_lens,
                                const int64_t* kv_offsets, void* O, float* LSE, int B, int Hq, int Hkv, int D,
                                int64_t total_tokens, float scale, int chunk, void* stream);

/* Merge `splits` partial attention results (new; no reference counterpart).
 *   O_part fp32 [splits, B, Hq, D], each normalised by its own softmax sum;
 *   LSE_part fp32 [splits, B, Hq] (natural log; -inf = empty split).
 * Writes O bf16 [B, Hq, D] and LSE fp32 [B, Hq] (may be NULL). */
BW_API int bw_lse_combine(const float* O_part, const float* LSE_part, int splits, int B, int Hq, int D, void* O,
                   float* LSE, void* stream);

/* Packed partials for a cross-GPU merge in ONE collective (new; no reference
 * counterpart).  A packed split is fp32 [bw_decode_packed_split_floats(B, Hq, D)]:
 * O [B, Hq, D] (as bw_gqa_decode_partial writes it), then LSE [B, Hq], then
 * padding to a multiple of 4 floats, so that each rank's O and LSE travel in a
 * single all-gather.  bw_lse_combine_packed merges `splits` such buffers laid
 * end to end (the all-gather's output, 16-byte aligned) into O bf16 [B, Hq, D]
 * and LSE fp32 [B, Hq] (may be NULL), like bw_lse_combine. */
BW_API size_t bw_decode_packed_split_floats(int B, int Hq, int D);
BW_API int bw_lse_combine_packed(const float* parts, int splits, int B, int Hq, int D, void* O, float* LSE,
                                 void* stream);

/* QK-norm + RoPE prologue of the reference's fused op
 * (src/SM103/attention/GQA_fused_sm103.cu:59-104; its ground truth :328-420),
 * on a [B, H, S, D] bf16 tensor X -> Y (Y may equal X).  Per row:
 *   rstd = 1/sqrt(mean(x^2) + eps); x = bf16(x * rstd * gamma)  (gamma NULL: skipped)
 *   RoPE at p = s + pos_offset when 0 <= p < cache_seq_len, with the fp32
 *   cos|sin cache [cache_seq_len, D]; interleaved = 0: NeoX pairs (i, i+D/2),
 *   1: GPT-J pairs (2i, 2i+1).  rstd (fp32 [B, H, S]) may be NULL.
 * x_strides / y_strides: element strides of (b, h, s), NULL = contiguous.
 * X, Y and the cache must be 16-byte aligned (BW_ERR_ALIGN otherwise). */
BW_API int bw_qk_norm_rope(const void* X, void* Y, int B, int H, int S, int D, const int64_t* x_strides,
                           const int64_t* y_strides, const float* cos_sin_cache, int cache_seq_len, int pos_offset,
                           const float* gamma, float eps, int interleaved, float* rstd, void* stream);

/* QK-norm + RoPE + GQA attention: replaces launch_gqa_fused_v0<Br,Bc,D>(Q,K,V,O,LSE,
 * cache, q_gamma, k_gamma, q_rstd, k_rstd, B,Hq,Hkv,G,S, cache_seq_len,
 * pos_offset, eps, interleaved, scale, is_causal) (GQA_fused_sm103.cu:284-313),
 * BHSD contiguous.  The normalised Q and K go to a caller workspace of
 * bw_gqa_fused_workspace_size(B, Hq, Hkv, S, D) bytes; Q, K are not modified. */
BW_API size_t bw_gqa_fused_workspace_size(int B, int Hq, int Hkv, int S, int D);
BW_API int bw_gqa_fused_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE,
                            const float* cos_sin_cache, const float* q_gamma, const float* k_gamma, float* q_rstd,
                            float* k_rstd, int B, int Hq, int Hkv, int S, int G, int D, int cache_seq_len,
                            int pos_offset, float eps, int interleaved, float scale, int causal, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Host tensor layouts for bw_attn_fwd_host. */
enum { BW_LAYOUT_BHSD = 0, BW_LAYOUT_BSHD = 1 };

/* Attention forward on HOST buffers: the reference harness's copy-in /
 * launch / copy-out sequence (kernelBench.cuh:34-98 around launch_gqa_vN,
 * GQA_sm103_causal_v3.cu:2156-2180) as one call, with the PCIe copies
 * pipelined against the kernels in `chunks` pieces (<= 32; 0 = 4): causal
 * calls are cut along the sequence (query rows [s0, s1) need keys [0, s1)
 * only), non-causal calls along the batch.  Q, K, V, O are contiguous host
 * tensors in `layout` (BHSD or BSHD), LSE host [B, Hq, S] fp32 or NULL.
 * `workspace` (device, 256-byte aligned, bw_attn_fwd_host_workspace_size
 * bytes) holds the device copies.  Asynchronous: O and LSE are complete when
 * `stream` reaches this point (synchronise it before reading them).  The
 * copies overlap only if the host buffers are page-locked.  Calls on one
 * device are serialised inside the library while they enqueue. */
BW_API size_t bw_attn_fwd_host_workspace_size(int B, int Hq, int Hkv, int S, int D);
BW_API int bw_attn_fwd_host(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv,
                            int S, int D, float scale, int causal, int layout, int chunks, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Synchronise `stream`, then read and clear the error word of `stream` on the
 * current device.  Every stream has its own word (the first 1023 distinct
 * streams of a device; later ones share one), so a call on one stream neither
 * sees nor clears the errors of calls on another.
 * Returns BW_OK, BW_ERR_TIMEOUT, BW_ERR_WORKSPACE or BW_ERR_CUDA. */
BW_API int bw_stream_status(void* stream);

/* Library options (process-wide).  Keys:
 *   BW_OPT_TIMEOUT_NS      bound on every device-side wait (default 2e9)
 *   BW_OPT_DEBUG_FLAGS     test hook; bit 0 makes the prefill producer withhold
 *                          its first K tile so that the consumers' bounded waits
 *                          expire and the call reports BW_ERR_TIMEOUT
 *   BW_OPT_MAX_CTAS        cap on the persistent prefill grid (0 = SM count)
 *   BW_OPT_EXP_POLY        of every 8 pairs of softmax exponentials, how many
 *                          are computed by an FMA-pipe polynomial instead of
 *                          MUFU ex2: 0, 2, 3 or 4; -1 (default) picks the
 *                          measured best per head dimension
 *   BW_OPT_PREFILL_KERNEL  0 (default): kernel 5 at D = 64, kernel 4 at
 *                          D = 128 (the fastest at every measured shape on
 *                          B200);
 *                          4: one query tile per CTA, three score buffers and
 *                          one O accumulator (four threads per row share the
 *                          running max), separate QK^T and PV issuing threads
 *                          and an epilogue warpgroup, so QK^T never waits for
 *                          the PV of the previous tile;
 *                          5 (D = 64; at D = 128 it selects 4): three score
 *                          buffers and two O accumulators, the two softmax
 *                          warpgroups taking alternate key tiles (one row per
 *                          thread), merged by the epilogue warps.
 *                          Other values return BW_ERR_SHAPE (kernels 1-3 were
 *                          removed as slower at every measured shape).
 *   BW_OPT_P_IN_TMEM       retired with kernel 1; setting it returns
 *                          BW_ERR_SHAPE. */
enum {
  BW_OPT_TIMEOUT_NS = 1,
  BW_OPT_P_IN_TMEM = 2,
  BW_OPT_DEBUG_FLAGS = 3,
  BW_OPT_MAX_CTAS = 4,
  BW_OPT_EXP_POLY = 5,
  BW_OPT_PREFILL_KERNEL = 6
};
BW_API int bw_set_option(int key, int64_t value);
BW_API int64_t bw_get_option(int key);

/* Contiguous share [*begin, *end) of `units` work units for `rank` of `world`
 * (multi-GPU sharding by (batch x KV-head group); no collective). */
BW_API int bw_shard_plan(int64_t units, int world, int rank, int64_t* begin, int64_t* end);

BW_API const char* bw_strerror(int code);
BW_API const char* bw_version(void);

#ifdef __cplusplus
}
#endif
#endif /* BW_ATTN_H_ */
