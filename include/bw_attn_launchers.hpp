// bw_attn_launchers.hpp -- C++ templates with the reference's launcher shapes,
// forwarding to the C ABI in bw_attn.h so the reference's harness code
// (`launch_gqa_vN<Br,Bc,D>(d_Q, d_K, d_V, d_O, d_LSE, B, Hq, Hkv, S, G, scale)`)
// compiles against this library unchanged apart from the include.
//
// Br and Bc are accepted for signature compatibility and ignored: the sm_100a
// kernel always uses 128-row query blocks and 128-row K/V tiles.  The calls run
// on the legacy default stream like the reference's launchers; they return the
// bw_attn status code (the reference returns void, so existing call sites that
// ignore the result still compile).
#pragma once
#include <cstddef>
#include <cstdio>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "bw_attn.h"

namespace bw_compat {

// src/SM103/attention/GQA_sm103.cu:5733-6516 (launch_gqa_v0 .. v23)
template <int Br, int Bc, int D>
inline int launch_gqa(__nv_bfloat16* Q, __nv_bfloat16* K, __nv_bfloat16* V, __nv_bfloat16* O, float* LSE, int B,
                      int Hq, int Hkv, int S, int G, float scale) {
  return bw_gqa_fwd(Q, K, V, O, LSE, B, Hq, Hkv, S, G, D, scale, nullptr, nullptr);
}

// src/SM103/attention/GQA_sm103_causal_v3.cu:2156-2180 (launch_gqa_vN_causal)
template <int Br, int Bc, int D>
inline int launch_gqa_causal(__nv_bfloat16* Q, __nv_bfloat16* K, __nv_bfloat16* V, __nv_bfloat16* O, float* LSE,
                             int B, int Hq, int Hkv, int S, int G, float scale) {
  return bw_gqa_causal_fwd(Q, K, V, O, LSE, B, Hq, Hkv, S, G, D, scale, nullptr, nullptr);
}

// src/SM120/attention/adhitya_GQA.cu:199-213 (launch_gqa_v1 with Sq, Skv)
template <int Br, int Bc, int D>
inline int launch_gqa_split(__nv_bfloat16* Q, __nv_bfloat16* K, __nv_bfloat16* V, __nv_bfloat16* O, float* LSE,
                            int B, int Hq, int Hkv, int Sq, int Skv, int G, float scale) {
  return bw_gqa_split_fwd(Q, K, V, O, LSE, B, Hq, Hkv, Sq, Skv, G, D, scale, 0, nullptr, nullptr);
}

// src/SM120/attention/MHA_sm120.cu:64-71 (mha_v3_tc: Q, K, V, O, scale, S), bf16
// storage; B and H are explicit because the reference derives them from its grid.
template <int Br, int Bc, int D>
inline int launch_mha(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V, __nv_bfloat16* O,
                      float scale, int S, int B, int H) {
  return bw_mha_fwd(Q, K, V, O, nullptr, B, H, S, D, scale, nullptr, nullptr);
}

// src/SM120/attention/MHA_sm120.cu:64-71 (mha_v3_tc: fp32 Q, K, V, O, scale, S),
// launch :333-345.  The reference's call has no workspace slot, so this
// launcher keeps one (for the 3xTF32 hi / lo split) in a cudaMalloc'd buffer it
// grows on demand and reuses; it is not thread-safe and is released at process
// exit.  B and H are explicit because the reference derives them from its grid.
template <int Br, int Bc, int D>
inline int launch_mha_f32(const float* Q, const float* K, const float* V, float* O, float scale, int S, int B,
                          int H) {
  struct Workspace {
    void* ptr = nullptr;
    size_t bytes = 0;
    ~Workspace() {
      if (ptr) cudaFree(ptr);
    }
  };
  static Workspace ws;
  const size_t need = bw_mha_f32_workspace_size(B, H, S, D);
  if (need == 0) return BW_ERR_SHAPE;
  if (need > ws.bytes) {
    if (ws.ptr) cudaFree(ws.ptr);
    ws.ptr = nullptr;
    ws.bytes = 0;
    if (cudaMalloc(&ws.ptr, need) != cudaSuccess) return BW_ERR_CUDA;
    ws.bytes = need;
  }
  return bw_mha_fwd_f32(Q, K, V, O, nullptr, B, H, S, D, scale, nullptr, ws.ptr, ws.bytes, nullptr);
}

// Reads `n` float32 values from a headerless file written by the reference's
// Python generators (base/baseline_gqa.py:165-170); the reference's own loadBin
// (include/utils/kernelUtils.cuh:191-199) exits on error, this returns false.
inline bool loadBin(const char* path, float* buf, size_t n) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return false;
  const size_t got = std::fread(buf, sizeof(float), n, f);
  std::fclose(f);
  return got == n;
}

// Writes `n` float32 values in the same headerless format.
inline bool saveBin(const char* path, const float* buf, size_t n) {
  FILE* f = std::fopen(path, "wb");
  if (!f) return false;
  const size_t put = std::fwrite(buf, sizeof(float), n, f);
  return std::fclose(f) == 0 && put == n;
}

}  // namespace bw_compat
