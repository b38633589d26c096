// Internal launch interface between the C-ABI layer (api.cu) and the kernels.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/bw_attn.h"

namespace bw {

// Prefill / full-sequence attention forward (GQA, MHA = GQA with G = 1).
struct FmhaParams {
  void* O;                       // bf16, element strides below (d stride 1)
  int64_t o_sb, o_sh, o_ss;
  float* LSE;                    // fp32 [B, Hq, Sq] contiguous, may be null
  int B, Hq, Hkv, G, Sq, Skv, D;
  int causal;                    // 1: key j visible to query i iff j <= i
  float scale_log2;              // softmax scale * log2(e)
  int n_qtiles, n_kvtiles;       // ceil(Sq / 128), ceil(Skv / 128)
  int num_items;                 // work items (one query tile, or a causal pair of them)
  int* err;                      // device error word
  uint64_t timeout_ns;           // bound for every device-side wait
  int debug_flags;               // bit 0: producer withholds its first K load (timeout test)
  int q_offset;                  // causal: query row i is sequence row q_offset + i (key j visible
                                 // iff j <= q_offset + i); 0 = top-left alignment
  int lse_sh;                    // LSE element stride between heads (>= Sq); LSE[b][h][i] at
                                 // (b * Hq + h) * lse_sh + i
};

struct FmhaMaps {
  CUtensorMap q, k, v;           // 4-D (D, S, H, B) bf16, box (64, rows, 1, 1), SWIZZLE_128B;
                                 // rows = 128
  CUtensorMap o;                 // 4-D (D, Sq, Hq, B) bf16 output, box (64, 32, 1, 1), SWIZZLE_128B
};

// fp32 MHA at fp32 accuracy (3xTF32 split, D = 64): split passes and the
// attention kernel (fmha_f32x3.cu).  The split arrays: Q and K hi / lo as
// contiguous [B, H, S, 64] fp32, V hi / lo transposed [B, H, 64, S32] fp32
// (S32 = S rounded up to 32, zero columns past S).
struct F32x3Params {
  float* O;                      // fp32, element strides below (d stride 1)
  int64_t o_sb, o_sh, o_ss;
  float* LSE;                    // fp32 [B, H, S] or null
  int B, H, S;
  int n_qtiles, n_kvtiles;       // ceil(S / 128), ceil(S / 32)
  float scale_log2;
  int* err;
  uint64_t timeout_ns;
};
struct F32x3Maps {
  // fp32, SWIZZLE_128B, 32-element (128-byte) inner box: Q (64, S, H, B) box
  // (32, 128); K (64, S, H, B) box (32, 32); VT (S32, 64, H, B) box (32, 64)
  CUtensorMap q_hi, q_lo, k_hi, k_lo, vt_hi, vt_lo;
};
cudaError_t launch_f32x3_split(const float* x, int64_t sb, int64_t sh, int64_t ss, float* hi, float* lo, int B,
                               int H, int S, int num_sms, cudaStream_t stream);
cudaError_t launch_f32x3_split_vt(const float* x, int64_t sb, int64_t sh, int64_t ss, float* hi, float* lo, int B,
                                  int H, int S, int S32, cudaStream_t stream);
cudaError_t launch_fmha_f32x3(const F32x3Params& p, const F32x3Maps& maps, cudaStream_t stream);

// Prefill kernels (fmha_fwd3.cu), one query tile per work item.  exp_poly: of
// every 8 pairs of exponentials, how many run as the FMA-pipe polynomial
// instead of MUFU ex2 (0, 2, 3 or 4).
// Kernel 4: three score buffers and one O accumulator (rows read through the
// 16-lane TMEM shapes, four threads per row sharing the running max).
cudaError_t launch_fmha_fwd4(const FmhaParams& p, const FmhaMaps& maps, int exp_poly, int num_sms,
                             cudaStream_t stream);
// Kernel 5 (D = 64): three score buffers, two O accumulators; the two softmax
// warpgroups own alternate key tiles, one row per thread.
cudaError_t launch_fmha_fwd5(const FmhaParams& p, const FmhaMaps& maps, int exp_poly, int num_sms,
                             cudaStream_t stream);

// Split-KV single-token decode over ragged, contiguous per-sequence KV.
struct DecodeParams {
  const void* Q;                 // bf16 [B, Hq, D], strides q_sb, q_sh
  int64_t q_sb, q_sh;
  const int* kv_lens;            // [B]
  const int64_t* kv_offsets;     // [B] first token of sequence b
  int B, Hq, Hkv, G, D;
  int chunk;                     // tokens per split (multiple of 64)
  float scale_log2;
  float* o_part;                 // [parts, G, D] fp32, normalised by its own sum
  float* lse_part;               // [parts, G]   natural-log LSE of the split
  int* chunk_prefix;             // [B + 1] written by the decode kernel
  int max_parts;                 // capacity of o_part / lse_part (bounds check)
  int* err;
  uint64_t timeout_ns;
  // Paged KV cache (block_table != null): K/V rows are page * page_size + slot,
  // token i of sequence b lives in page block_table[b * max_pages + i / page_size].
  const int* block_table;
  int page_size, max_pages;
};

struct DecodeMaps {
  // 3-D (64, rows, Hkv * D / 64) bf16 over a [rows, Hkv, D] K or V array: dim 1
  // steps rows (stride Hkv * D * 2 bytes), dim 2 steps 64-element panels
  // (stride 128 bytes); box (64, min(64, page_size), D / 64), SWIZZLE_128B.
  // One load brings both panels of a piece of up to 64 rows of one KV head.
  CUtensorMap k, v;
};

cudaError_t launch_decode(const DecodeParams& p, const DecodeMaps& maps, int num_sms, cudaStream_t stream);

// Merge of split partials.
struct CombineParams {
  const float* o_part;           // ragged: [parts, G, D] via chunk_prefix; uniform: [splits, B, Hq, D]
  const float* lse_part;         // ragged: [parts, G];                     uniform: [splits, B, Hq]
  const int* chunk_prefix;       // null => uniform `splits`
  int splits;
  int64_t o_split_stride;        // uniform: elements between splits of o_part (B * Hq * D when contiguous)
  int64_t lse_split_stride;      // uniform: elements between splits of lse_part (B * Hq when contiguous)
  int B, Hq, Hkv, G, D;
  void* O;                       // bf16 [B, Hq, D] (strides o_sb, o_sh)
  int64_t o_sb, o_sh;
  float* LSE;                    // fp32 [B, Hq], may be null
  int o_fp32;                    // 1: O is fp32 (strides in fp32 elements) instead of bf16
};

cudaError_t launch_lse_combine(const CombineParams& p, cudaStream_t stream);

// QK-norm + RoPE prologue over a [B, H, S, D] bf16 tensor (in place allowed).
struct NormRopeParams {
  const void* in;
  void* out;
  int64_t in_sb, in_sh, in_ss, out_sb, out_sh, out_ss;   // element strides
  int B, H, S, D;
  const float* cache;        // fp32 [cache_seq_len, D]: cos | sin
  int cache_seq_len, pos_offset;
  const float* gamma;        // fp32 [D] or null (no norm)
  float eps;
  float* rstd;               // fp32 [B, H, S] or null
  int neox;                  // 1: pairs (i, i + D/2); 0: pairs (2i, 2i + 1)
};

cudaError_t launch_norm_rope(const NormRopeParams& p, int num_sms, cudaStream_t stream);

// The attention forward of the C ABI with the internal extras: causal query
// offset (multiple of 128) and LSE head stride (0 = Sq).  Returns a status code.
int attn_forward(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv, int Sq,
                 int Skv, int G, int D, float scale, int causal, const bw_strides* strides, void* stream,
                 int q_offset, int lse_sh);

// The split-KV decode + combine of bw_gqa_decode / bw_gqa_decode_partial on a
// given scratch buffer (`workspace`, `workspace_bytes`): argument checks, tensor
// maps, scratch layout and both launches.  o_fp32 = 1 writes fp32 O (partial
// results).  Returns a status code.
int decode_run(const void* Q, const void* K, const void* V, const int* kv_lens, const int64_t* kv_offsets, void* O,
               int o_fp32, float* LSE, int B, int Hq, int Hkv, int D, int64_t total_tokens, float scale, int chunk,
               void* workspace, size_t workspace_bytes, void* stream);

}  // namespace bw
