// C-ABI entry points (include/bw_attn.h): argument validation, TMA tensor-map
// encoding, per-device state, and dispatch to the kernels.
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include <cudaTypedefs.h>

#include "../../include/bw_attn.h"
#include "kernels.h"

namespace {

// Device error words: 0, or 0x100|site for a timed-out wait, 0x200 for a
// decode workspace overflow, 0x400 for a shared-memory window the prefill
// kernel could not align.  One word per stream (slot), so that calls on
// different streams neither see nor clear each other's errors; module
// globals are per context, so every device has its own array.  Slot 0 is
// shared by the streams beyond the first kErrSlots - 1 distinct ones.
constexpr int kErrSlots = 1024;
__device__ int g_bw_err[kErrSlots];

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool init = false;
  int num_sms = 0;
  int* err_base = nullptr;
  std::unordered_map<cudaStream_t, int> slot_of;
  int next_slot = 1;
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

std::atomic<int64_t> g_timeout_ns{2000000000LL};
std::atomic<int64_t> g_debug_flags{0};
std::atomic<int64_t> g_max_ctas{0};
std::atomic<int64_t> g_exp_poly{-1};        // -1: per head dimension (kExpPolyD64 / kExpPolyD128)
std::atomic<int64_t> g_prefill_kernel{0};   // 0: default (kernel 5 at D = 64, else 4)

// Measured defaults of the exponential split (of every 8 pairs, how many run as
// the FMA-pipe polynomial) per head dimension.
constexpr int kExpPolyD128 = 2;
constexpr int kExpPolyD64 = 2;

int exp_poly_for(int D) {
  const int64_t v = g_exp_poly.load();
  if (v >= 0) return (int)v;
  return D == 64 ? kExpPolyD64 : kExpPolyD128;
}

int get_device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BW_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    if (cudaDeviceGetAttribute(&st.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return BW_ERR_CUDA;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bw_err) != cudaSuccess) return BW_ERR_CUDA;
    st.err_base = static_cast<int*>(p);
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn)
        return BW_ERR_CUDA;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    st.init = true;
  }
  *out = &st;
  return BW_OK;
}

// The error word of `stream` on this device (assigned on first use).
int* err_slot(DeviceState* dev, void* stream) {
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = dev->slot_of.find(s);
  int slot = 0;
  if (it != dev->slot_of.end()) {
    slot = it->second;
  } else if (dev->next_slot < kErrSlots) {
    slot = dev->next_slot++;
    dev->slot_of.emplace(s, slot);
  }
  return dev->err_base + slot;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 4-D map over a [B, H, S, D] bf16 tensor with element strides (sb, sh, ss, 1):
// dims (D, S, H, B), box (64, 128, 1, 1), 128-byte swizzle, zero fill out of bounds.
int make_map_bhsd(CUtensorMap* m, const void* base, int B, int H, int S, int D, const int64_t st[3],
                  uint32_t box_rows = 128, bool fp32 = false) {
  const uint32_t eb = fp32 ? 4 : 2;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * eb, (cuuint64_t)st[1] * eb, (cuuint64_t)st[0] * eb};
  cuuint32_t box[4] = {128 / eb, box_rows, 1, 1};   // 128-byte rows (the swizzle span)
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                        const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BW_OK : BW_ERR_CUDA;
}

// 4-D store map over the [B, Hq, Sq, D] bf16 output with element strides
// st (sb, sh, ss, 1): box (64, 32, 1, 1), one 128-byte-swizzled panel of the
// 32 rows an epilogue warp of the prefill kernel writes (D / 64 stores).
int make_map_out(CUtensorMap* m, void* base, int B, int H, int S, int D, const int64_t st[3]) {
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * 2, (cuuint64_t)st[1] * 2, (cuuint64_t)st[0] * 2};
  cuuint32_t box[4] = {64, 32, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BW_OK : BW_ERR_CUDA;
}

// 3-D map over a [rows, Hkv, D] bf16 K or V array for the decode kernels:
// dims (64, rows, Hkv * D / 64), strides (Hkv * D * 2, 128) bytes, box
// (64, box_rows, D / 64): one load = both 64-column panels of box_rows rows of
// one KV head, written panel after panel.
int make_map_kv3d(CUtensorMap* m, const void* base, int64_t rows, int Hkv, int D, uint32_t box_rows) {
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)Hkv * D / 64};
  cuuint64_t strides[2] = {(cuuint64_t)Hkv * D * 2, 128};
  cuuint32_t box[3] = {64, box_rows, (cuuint32_t)(D / 64)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BW_OK : BW_ERR_CUDA;
}

bool strides_ok(const int64_t s[3]) {
  for (int i = 0; i < 3; ++i)
    if (s[i] <= 0 || (s[i] % 8) != 0 || s[i] * 2 >= (int64_t(1) << 40)) return false;
  return true;
}

void contiguous(int H, int S, int D, int64_t out[3]) {
  out[2] = D;
  out[1] = (int64_t)S * D;
  out[0] = (int64_t)H * S * D;
}

// q_offset: causal query row i is sequence row q_offset + i;
// lse_sh: LSE stride between heads (0 = Sq).
int attn_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv, int Sq,
             int Skv, int G, int D, float scale, int causal, const bw_strides* strides, void* stream,
             int q_offset = 0, int lse_sh = 0) {
  if (!Q || !K || !V || !O) return BW_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0 || G <= 0) return BW_ERR_SHAPE;
  if (Hq % Hkv != 0 || Hq / Hkv != G) return BW_ERR_SHAPE;
  if (D != 64 && D != 128) return BW_ERR_SHAPE;
  if (!(scale > 0.f) || !std::isfinite(scale)) return BW_ERR_SHAPE;
  if ((int64_t)B * Hq * ((Sq + 255) / 256) >= (int64_t(1) << 30)) return BW_ERR_SHAPE;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return BW_ERR_ALIGN;
  bw_strides st;
  if (strides) {
    st = *strides;
  } else {
    contiguous(Hq, Sq, D, st.q);
    contiguous(Hkv, Skv, D, st.k);
    contiguous(Hkv, Skv, D, st.v);
    contiguous(Hq, Sq, D, st.o);
  }
  if (!strides_ok(st.q) || !strides_ok(st.k) || !strides_ok(st.v) || !strides_ok(st.o)) return BW_ERR_ALIGN;

  DeviceState* dev = nullptr;
  int rc = get_device_state(&dev);
  if (rc != BW_OK) return rc;

  if (q_offset < 0 || (lse_sh != 0 && lse_sh < Sq)) return BW_ERR_SHAPE;
  int kern = (int)g_prefill_kernel.load();
  if (kern == 0) kern = D == 64 ? 5 : 4;
  if (kern == 5 && D != 64) kern = 4;   // kernel 5 exists for D = 64 only
  const uint32_t kv_rows = 128u;
  bw::FmhaMaps maps;
  if (make_map_bhsd(&maps.q, Q, B, Hq, Sq, D, st.q) != BW_OK) return BW_ERR_CUDA;
  if (make_map_bhsd(&maps.k, K, B, Hkv, Skv, D, st.k, kv_rows) != BW_OK) return BW_ERR_CUDA;
  if (make_map_bhsd(&maps.v, V, B, Hkv, Skv, D, st.v, kv_rows) != BW_OK) return BW_ERR_CUDA;
  if (make_map_out(&maps.o, O, B, Hq, Sq, D, st.o) != BW_OK) return BW_ERR_CUDA;

  bw::FmhaParams p{};
  p.O = O;
  p.o_sb = st.o[0];
  p.o_sh = st.o[1];
  p.o_ss = st.o[2];
  p.LSE = LSE;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = G;
  p.Sq = Sq;
  p.Skv = Skv;
  p.D = D;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.n_qtiles = (Sq + 127) / 128;
  p.n_kvtiles = (Skv + 127) / 128;
  p.num_items = B * Hq * (causal ? (p.n_qtiles + 1) / 2 : p.n_qtiles);
  p.err = err_slot(dev, stream);
  p.timeout_ns = (uint64_t)g_timeout_ns.load();
  p.debug_flags = (int)g_debug_flags.load();
  p.q_offset = q_offset;
  p.lse_sh = lse_sh > 0 ? lse_sh : Sq;
  int ctas = dev->num_sms;
  const int64_t cap = g_max_ctas.load();
  if (cap > 0 && cap < ctas) ctas = (int)cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int poly = exp_poly_for(D);
  cudaError_t e = kern == 5 ? bw::launch_fmha_fwd5(p, maps, poly, ctas, s) : bw::launch_fmha_fwd4(p, maps, poly, ctas, s);
  return e == cudaSuccess ? BW_OK : BW_ERR_CUDA;
}

constexpr int kDefaultChunk = 1024;

int64_t decode_max_parts(int B, int Hkv, int64_t total_tokens, int chunk) {
  return (int64_t)Hkv * ((total_tokens + chunk - 1) / chunk + B);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

namespace bw {

int attn_forward(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv, int Sq,
                 int Skv, int G, int D, float scale, int causal, const bw_strides* strides, void* stream,
                 int q_offset, int lse_sh) {
  return attn_fwd(Q, K, V, O, LSE, B, Hq, Hkv, Sq, Skv, G, D, scale, causal, strides, stream, q_offset, lse_sh);
}
}  // namespace bw

extern "C" {

int bw_gqa_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv, int S,
               int G, int D, float scale, const bw_strides* strides, void* stream) {
  return attn_fwd(Q, K, V, O, LSE, B, Hq, Hkv, S, S, G, D, scale, 0, strides, stream);
}

int bw_gqa_causal_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv,
                      int S, int G, int D, float scale, const bw_strides* strides, void* stream) {
  return attn_fwd(Q, K, V, O, LSE, B, Hq, Hkv, S, S, G, D, scale, 1, strides, stream);
}

int bw_gqa_split_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv,
                     int Sq, int Skv, int G, int D, float scale, int causal, const bw_strides* strides,
                     void* stream) {
  return attn_fwd(Q, K, V, O, LSE, B, Hq, Hkv, Sq, Skv, G, D, scale, causal, strides, stream);
}

int bw_gqa_causal_offset_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq,
                             int Hkv, int Sq, int Skv, int G, int D, float scale, int q_offset,
                             const bw_strides* strides, void* stream) {
  if (q_offset < 0 || (int64_t)q_offset + Sq > (int64_t(1) << 30)) return BW_ERR_SHAPE;
  return attn_fwd(Q, K, V, O, LSE, B, Hq, Hkv, Sq, Skv, G, D, scale, 1, strides, stream, q_offset, 0);
}

int bw_mha_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int H, int S, int D,
               float scale, const bw_strides* strides, void* stream) {
  return attn_fwd(Q, K, V, O, LSE, B, H, H, S, S, 1, D, scale, 0, strides, stream);
}

size_t bw_mha_f32_workspace_size(int B, int H, int S, int D) {
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return 0;
  const size_t rows = align256((size_t)B * H * S * D * 4);
  const size_t vt = align256((size_t)B * H * D * (((size_t)S + 31) & ~size_t(31)) * 4);
  return 4 * rows + 2 * vt;
}

int bw_mha_fwd_f32(const float* Q, const float* K, const float* V, float* O, float* LSE, int B, int H, int S, int D,
                   float scale, const bw_strides* strides, void* workspace, size_t workspace_bytes, void* stream) {
  if (!Q || !K || !V || !O || !workspace) return BW_ERR_NULL;
  if (B <= 0 || H <= 0 || S <= 0 || D != 64) return BW_ERR_SHAPE;
  if (workspace_bytes < bw_mha_f32_workspace_size(B, H, S, D)) return BW_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return BW_ERR_ALIGN;
  if (!(scale > 0.f) || !std::isfinite(scale)) return BW_ERR_SHAPE;
  if ((int64_t)B * H * ((S + 127) / 128) >= (int64_t(1) << 31) || (int64_t)B * H > 65535) return BW_ERR_SHAPE;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return BW_ERR_ALIGN;
  bw_strides st;
  if (strides) {
    st = *strides;
  } else {
    contiguous(H, S, D, st.q);
    contiguous(H, S, D, st.k);
    contiguous(H, S, D, st.v);
    contiguous(H, S, D, st.o);
  }
  for (const int64_t* a : {st.q, st.k, st.v, st.o})
    for (int i = 0; i < 3; ++i)
      if (a[i] <= 0 || (a[i] % 4) != 0) return BW_ERR_ALIGN;
  DeviceState* dev = nullptr;
  int rc = get_device_state(&dev);
  if (rc != BW_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 3xTF32 split: Q, K hi / lo row-major, V hi / lo transposed, in the workspace
  const int S32 = (S + 31) & ~31;
  const size_t rows = align256((size_t)B * H * S * D * 4);
  const size_t vtb = align256((size_t)B * H * D * S32 * 4);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* qh = reinterpret_cast<float*>(ws);
  float* ql = reinterpret_cast<float*>(ws + rows);
  float* kh = reinterpret_cast<float*>(ws + 2 * rows);
  float* kl = reinterpret_cast<float*>(ws + 3 * rows);
  float* vth = reinterpret_cast<float*>(ws + 4 * rows);
  float* vtl = reinterpret_cast<float*>(ws + 4 * rows + vtb);
  if (bw::launch_f32x3_split(Q, st.q[0], st.q[1], st.q[2], qh, ql, B, H, S, dev->num_sms, s) != cudaSuccess ||
      bw::launch_f32x3_split(K, st.k[0], st.k[1], st.k[2], kh, kl, B, H, S, dev->num_sms, s) != cudaSuccess ||
      bw::launch_f32x3_split_vt(V, st.v[0], st.v[1], st.v[2], vth, vtl, B, H, S, S32, s) != cudaSuccess)
    return BW_ERR_CUDA;
  bw::F32x3Maps maps;
  auto map = [&](CUtensorMap* m, const float* base, uint64_t d0, uint64_t d1, uint32_t b1) {
    cuuint64_t dims[4] = {d0, d1, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t str[3] = {d0 * 4, d0 * d1 * 4, d0 * d1 * H * 4};
    cuuint32_t box[4] = {32, b1, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, str, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  if (!map(&maps.q_hi, qh, D, S, 128) || !map(&maps.q_lo, ql, D, S, 128) || !map(&maps.k_hi, kh, D, S, 32) ||
      !map(&maps.k_lo, kl, D, S, 32) || !map(&maps.vt_hi, vth, S32, D, 64) || !map(&maps.vt_lo, vtl, S32, D, 64))
    return BW_ERR_CUDA;
  bw::F32x3Params p{};
  p.O = O;
  p.o_sb = st.o[0];
  p.o_sh = st.o[1];
  p.o_ss = st.o[2];
  p.LSE = LSE;
  p.B = B;
  p.H = H;
  p.S = S;
  p.n_qtiles = (S + 127) / 128;
  p.n_kvtiles = (S + 31) / 32;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err_slot(dev, stream);
  p.timeout_ns = (uint64_t)g_timeout_ns.load();
  return bw::launch_fmha_f32x3(p, maps, s) == cudaSuccess ? BW_OK : BW_ERR_CUDA;
}

size_t bw_gqa_decode_workspace_size(int B, int Hq, int Hkv, int D, int64_t total_tokens, int chunk) {
  if (B <= 0 || Hkv <= 0 || Hq % Hkv != 0 || total_tokens < 0) return 0;
  if (chunk <= 0) chunk = kDefaultChunk;
  const int G = Hq / Hkv;
  const int64_t parts = decode_max_parts(B, Hkv, total_tokens, chunk);
  return align256((size_t)(B + 1) * 4) + align256((size_t)parts * G * 4) + (size_t)parts * G * D * 4;
}

}  // extern "C"

namespace bw {

int decode_run(const void* Q, const void* K, const void* V, const int* kv_lens, const int64_t* kv_offsets, void* O,
               int o_fp32, float* LSE, int B, int Hq, int Hkv, int D, int64_t total_tokens, float scale, int chunk,
               void* workspace, size_t workspace_bytes, void* stream) {
  if (!Q || !K || !V || !kv_lens || !kv_offsets || !O || !workspace) return BW_ERR_NULL;
  if (B <= 0 || B > 4096 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0) return BW_ERR_SHAPE;
  const int G = Hq / Hkv;
  if (G > 16 || (D != 64 && D != 128) || total_tokens <= 0 || total_tokens >= (int64_t(1) << 31))
    return BW_ERR_SHAPE;
  if (!(scale > 0.f) || !std::isfinite(scale)) return BW_ERR_SHAPE;
  if (chunk <= 0) chunk = kDefaultChunk;
  if (chunk % 64 != 0) return BW_ERR_SHAPE;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(workspace))
    return BW_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(kv_offsets) & 7u) || (reinterpret_cast<uintptr_t>(kv_lens) & 3u))
    return BW_ERR_ALIGN;
  if (workspace_bytes < bw_gqa_decode_workspace_size(B, Hq, Hkv, D, total_tokens, chunk)) return BW_ERR_WORKSPACE;

  DeviceState* dev = nullptr;
  int rc = get_device_state(&dev);
  if (rc != BW_OK) return rc;

  bw::DecodeMaps maps;
  if (make_map_kv3d(&maps.k, K, total_tokens, Hkv, D, 64) != BW_OK) return BW_ERR_CUDA;
  if (make_map_kv3d(&maps.v, V, total_tokens, Hkv, D, 64) != BW_OK) return BW_ERR_CUDA;

  const int64_t parts = decode_max_parts(B, Hkv, total_tokens, chunk);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* prefix = reinterpret_cast<int*>(ws);
  float* lse_part = reinterpret_cast<float*>(ws + align256((size_t)(B + 1) * 4));
  float* o_part = reinterpret_cast<float*>(ws + align256((size_t)(B + 1) * 4) + align256((size_t)parts * G * 4));

  bw::DecodeParams p{};
  p.Q = Q;
  p.q_sb = (int64_t)Hq * D;
  p.q_sh = D;
  p.kv_lens = kv_lens;
  p.kv_offsets = kv_offsets;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = G;
  p.D = D;
  p.chunk = chunk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.chunk_prefix = prefix;
  p.max_parts = (int)parts;
  p.err = err_slot(dev, stream);
  p.timeout_ns = (uint64_t)g_timeout_ns.load();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = bw::launch_decode(p, maps, dev->num_sms, s);
  if (e != cudaSuccess) return BW_ERR_CUDA;

  bw::CombineParams c{};
  c.o_part = o_part;
  c.lse_part = lse_part;
  c.chunk_prefix = prefix;
  c.splits = 0;
  c.B = B;
  c.Hq = Hq;
  c.Hkv = Hkv;
  c.G = G;
  c.D = D;
  c.O = O;
  c.o_sb = (int64_t)Hq * D;
  c.o_sh = D;
  c.LSE = LSE;
  c.o_fp32 = o_fp32;
  e = bw::launch_lse_combine(c, s);
  return e == cudaSuccess ? BW_OK : BW_ERR_CUDA;
}

}  // namespace bw

extern "C" {

int bw_gqa_decode(const void* Q, const void* K, const void* V, const int* kv_lens, const int64_t* kv_offsets,
                  void* O, float* LSE, int B, int Hq, int Hkv, int D, int64_t total_tokens, float scale, int chunk,
                  void* workspace, size_t workspace_bytes, void* stream) {
  return bw::decode_run(Q, K, V, kv_lens, kv_offsets, O, 0, LSE, B, Hq, Hkv, D, total_tokens, scale, chunk, workspace,
                     workspace_bytes, stream);
}

int bw_gqa_decode_partial(const void* Q, const void* K, const void* V, const int* kv_lens,
                          const int64_t* kv_offsets, float* O, float* LSE, int B, int Hq, int Hkv, int D,
                          int64_t total_tokens, float scale, int chunk, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (!LSE) return BW_ERR_NULL;
  return bw::decode_run(Q, K, V, kv_lens, kv_offsets, O, 1, LSE, B, Hq, Hkv, D, total_tokens, scale, chunk, workspace,
                     workspace_bytes, stream);
}

int bw_gqa_decode_paged(const void* Q, const void* K_cache, const void* V_cache, const int* block_table,
                        const int* kv_lens, void* O, float* LSE, int B, int Hq, int Hkv, int D, int page_size,
                        int num_pages, int max_pages_per_seq, float scale, int chunk, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!Q || !K_cache || !V_cache || !block_table || !kv_lens || !O || !workspace) return BW_ERR_NULL;
  if (B <= 0 || B > 4096 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0) return BW_ERR_SHAPE;
  const int G = Hq / Hkv;
  if (G > 16 || (D != 64 && D != 128) || num_pages <= 0 || max_pages_per_seq <= 0) return BW_ERR_SHAPE;
  // page pieces must start on 1024-byte (8-row) boundaries of the swizzled stage
  const bool ps_ok = page_size >= 8 && ((page_size <= 64 && 64 % page_size == 0) || page_size % 64 == 0);
  if (!ps_ok) return BW_ERR_SHAPE;
  const int64_t rows = (int64_t)num_pages * page_size;
  if (rows >= (int64_t(1) << 31)) return BW_ERR_SHAPE;
  if (!(scale > 0.f) || !std::isfinite(scale)) return BW_ERR_SHAPE;
  if (chunk <= 0) chunk = kDefaultChunk;
  if (chunk % 64 != 0) return BW_ERR_SHAPE;
  if (!aligned16(Q) || !aligned16(K_cache) || !aligned16(V_cache) || !aligned16(O) || !aligned16(workspace))
    return BW_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(block_table) & 3u) || (reinterpret_cast<uintptr_t>(kv_lens) & 3u))
    return BW_ERR_ALIGN;
  const int64_t max_tokens = (int64_t)B * max_pages_per_seq * page_size;
  const int64_t bound = max_tokens < rows ? max_tokens : rows;
  if (workspace_bytes < bw_gqa_decode_workspace_size(B, Hq, Hkv, D, bound, chunk)) return BW_ERR_WORKSPACE;

  DeviceState* dev = nullptr;
  int rc = get_device_state(&dev);
  if (rc != BW_OK) return rc;
  const uint32_t box_rows = page_size < 64 ? (uint32_t)page_size : 64u;
  bw::DecodeMaps maps;
  if (make_map_kv3d(&maps.k, K_cache, rows, Hkv, D, box_rows) != BW_OK) return BW_ERR_CUDA;
  if (make_map_kv3d(&maps.v, V_cache, rows, Hkv, D, box_rows) != BW_OK) return BW_ERR_CUDA;

  const int64_t parts = decode_max_parts(B, Hkv, bound, chunk);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* prefix = reinterpret_cast<int*>(ws);
  float* lse_part = reinterpret_cast<float*>(ws + align256((size_t)(B + 1) * 4));
  float* o_part = reinterpret_cast<float*>(ws + align256((size_t)(B + 1) * 4) + align256((size_t)parts * G * 4));

  bw::DecodeParams p{};
  p.Q = Q;
  p.q_sb = (int64_t)Hq * D;
  p.q_sh = D;
  p.kv_lens = kv_lens;
  p.kv_offsets = nullptr;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = G;
  p.D = D;
  p.chunk = chunk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.chunk_prefix = prefix;
  p.max_parts = (int)parts;
  p.err = err_slot(dev, stream);
  p.timeout_ns = (uint64_t)g_timeout_ns.load();
  p.block_table = block_table;
  p.page_size = page_size;
  p.max_pages = max_pages_per_seq;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bw::launch_decode(p, maps, dev->num_sms, s) != cudaSuccess) return BW_ERR_CUDA;

  bw::CombineParams c{};
  c.o_part = o_part;
  c.lse_part = lse_part;
  c.chunk_prefix = prefix;
  c.B = B;
  c.Hq = Hq;
  c.Hkv = Hkv;
  c.G = G;
  c.D = D;
  c.O = O;
  c.o_sb = (int64_t)Hq * D;
  c.o_sh = D;
  c.LSE = LSE;
  c.o_fp32 = 0;
  return bw::launch_lse_combine(c, s) == cudaSuccess ? BW_OK : BW_ERR_CUDA;
}

int bw_qk_norm_rope(const void* X, void* Y, int B, int H, int S, int D, const int64_t* x_strides,
                    const int64_t* y_strides, const float* cos_sin_cache, int cache_seq_len, int pos_offset,
                    const float* gamma, float eps, int interleaved, float* rstd, void* stream) {
  if (!X || !Y || !cos_sin_cache) return BW_ERR_NULL;
  if (B <= 0 || H <= 0 || S <= 0 || (D != 64 && D != 128) || cache_seq_len < 0 || !(eps >= 0.f))
    return BW_ERR_SHAPE;
  if ((int64_t)B * H * S >= (int64_t(1) << 31)) return BW_ERR_SHAPE;
  int64_t xs[3], ys[3];
  if (x_strides) { for (int i = 0; i < 3; ++i) xs[i] = x_strides[i]; } else { contiguous(H, S, D, xs); }
  if (y_strides) { for (int i = 0; i < 3; ++i) ys[i] = y_strides[i]; } else { contiguous(H, S, D, ys); }
  for (int i = 0; i < 3; ++i)
    if (xs[i] <= 0 || ys[i] <= 0 || (xs[i] % 8) || (ys[i] % 8)) return BW_ERR_ALIGN;
  if (!aligned16(X) || !aligned16(Y) || !aligned16(cos_sin_cache)) return BW_ERR_ALIGN;
  DeviceState* dev = nullptr;
  int rc = get_device_state(&dev);
  if (rc != BW_OK) return rc;
  bw::NormRopeParams p{};
  p.in = X;
  p.out = Y;
  p.in_sb = xs[0]; p.in_sh = xs[1]; p.in_ss = xs[2];
  p.out_sb = ys[0]; p.out_sh = ys[1]; p.out_ss = ys[2];
  p.B = B; p.H = H; p.S = S; p.D = D;
  p.cache = cos_sin_cache;
  p.cache_seq_len = cache_seq_len;
  p.pos_offset = pos_offset;
  p.gamma = gamma;
  p.eps = eps;
  p.rstd = rstd;
  p.neox = interleaved ? 0 : 1;
  return bw::launch_norm_rope(p, dev->num_sms, static_cast<cudaStream_t>(stream)) == cudaSuccess ? BW_OK
                                                                                                 : BW_ERR_CUDA;
}

size_t bw_gqa_fused_workspace_size(int B, int Hq, int Hkv, int S, int D) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return 0;
  return align256((size_t)B * Hq * S * D * 2) + align256((size_t)B * Hkv * S * D * 2);
}

int bw_gqa_fused_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, const float* cos_sin_cache,
                     const float* q_gamma, const float* k_gamma, float* q_rstd, float* k_rstd, int B, int Hq,
                     int Hkv, int S, int G, int D, int cache_seq_len, int pos_offset, float eps, int interleaved,
                     float scale, int causal, void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace) return BW_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0) return BW_ERR_SHAPE;
  if (workspace_bytes < bw_gqa_fused_workspace_size(B, Hq, Hkv, S, D)) return BW_ERR_WORKSPACE;
  if (!aligned16(workspace)) return BW_ERR_ALIGN;
  if (!cos_sin_cache) return BW_ERR_NULL;
  if (cache_seq_len < 0 || !(eps >= 0.f)) return BW_ERR_SHAPE;
  // Q and K are normalised and rotated into the workspace by the HBM-bound
  // prologue kernel (one pass each), then read by the attention kernel.
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* q2 = ws;
  void* k2 = ws + align256((size_t)B * Hq * S * D * 2);
  int rc = bw_qk_norm_rope(Q, q2, B, Hq, S, D, nullptr, nullptr, cos_sin_cache, cache_seq_len, pos_offset, q_gamma,
                           eps, interleaved, q_rstd, stream);
  if (rc != BW_OK) return rc;
  rc = bw_qk_norm_rope(K, k2, B, Hkv, S, D, nullptr, nullptr, cos_sin_cache, cache_seq_len, pos_offset, k_gamma,
                       eps, interleaved, k_rstd, stream);
  if (rc != BW_OK) return rc;
  return attn_fwd(q2, k2, V, O, LSE, B, Hq, Hkv, S, S, G, D, scale, causal, nullptr, stream);
}

}  // extern "C"

namespace {

int combine_uniform(const float* O_part, const float* LSE_part, int64_t o_ss, int64_t l_ss, int splits, int B, int Hq,
                    int D, void* O, float* LSE, void* stream) {
  if (!O_part || !LSE_part || !O) return BW_ERR_NULL;
  if (splits <= 0 || B <= 0 || Hq <= 0 || D <= 0 || D % 4 != 0 || D > 128) return BW_ERR_SHAPE;
  if (!aligned16(O_part) || (reinterpret_cast<uintptr_t>(O) & 7u) || (o_ss % 4) != 0) return BW_ERR_ALIGN;
  bw::CombineParams c{};
  c.o_part = O_part;
  c.lse_part = LSE_part;
  c.chunk_prefix = nullptr;
  c.splits = splits;
  c.o_split_stride = o_ss;
  c.lse_split_stride = l_ss;
  c.B = B;
  c.Hq = Hq;
  c.Hkv = Hq;
  c.G = 1;
  c.D = D;
  c.O = O;
  c.o_sb = (int64_t)Hq * D;
  c.o_sh = D;
  c.LSE = LSE;
  c.o_fp32 = 0;
  cudaError_t e = bw::launch_lse_combine(c, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BW_OK : BW_ERR_CUDA;
}

}  // namespace

extern "C" {

int bw_lse_combine(const float* O_part, const float* LSE_part, int splits, int B, int Hq, int D, void* O,
                   float* LSE, void* stream) {
  return combine_uniform(O_part, LSE_part, (int64_t)B * Hq * D, (int64_t)B * Hq, splits, B, Hq, D, O, LSE, stream);
}

size_t bw_decode_packed_split_floats(int B, int Hq, int D) {
  if (B <= 0 || Hq <= 0 || D <= 0) return 0;
  return (size_t)B * Hq * D + (((size_t)B * Hq + 3) & ~size_t(3));
}

int bw_lse_combine_packed(const float* parts, int splits, int B, int Hq, int D, void* O, float* LSE, void* stream) {
  if (!parts) return BW_ERR_NULL;
  const int64_t ss = (int64_t)bw_decode_packed_split_floats(B, Hq, D);
  if (ss == 0) return BW_ERR_SHAPE;
  return combine_uniform(parts, parts + (int64_t)B * Hq * D, ss, ss, splits, B, Hq, D, O, LSE, stream);
}

int bw_stream_status(void* stream) {
  DeviceState* dev = nullptr;
  int rc = get_device_state(&dev);
  if (rc != BW_OK) return rc;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return BW_ERR_CUDA;
  int* slot = err_slot(dev, stream);
  int v = 0;
  if (cudaMemcpy(&v, slot, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return BW_ERR_CUDA;
  if (v != 0) {
    const int zero = 0;
    if (cudaMemcpy(slot, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return BW_ERR_CUDA;
  }
  if (v == 0) return BW_OK;
  if (v & 0x400) return BW_ERR_CUDA;
  if (v & 0x200) return BW_ERR_WORKSPACE;
  return BW_ERR_TIMEOUT;
}

int bw_set_option(int key, int64_t value) {
  switch (key) {
    case BW_OPT_TIMEOUT_NS:
      if (value <= 0) return BW_ERR_SHAPE;
      g_timeout_ns = value;
      return BW_OK;
    case BW_OPT_DEBUG_FLAGS: g_debug_flags = value; return BW_OK;
    case BW_OPT_MAX_CTAS:
      if (value < 0) return BW_ERR_SHAPE;
      g_max_ctas = value;
      return BW_OK;
    case BW_OPT_PREFILL_KERNEL:
      if (value != 0 && value != 4 && value != 5) return BW_ERR_SHAPE;
      g_prefill_kernel = value;
      return BW_OK;
    case BW_OPT_EXP_POLY:
      if (value != -1 && value != 0 && value != 2 && value != 3 && value != 4) return BW_ERR_SHAPE;
      g_exp_poly = value;
      return BW_OK;
    default: return BW_ERR_SHAPE;
  }
}

int64_t bw_get_option(int key) {
  switch (key) {
    case BW_OPT_TIMEOUT_NS: return g_timeout_ns.load();
    case BW_OPT_DEBUG_FLAGS: return g_debug_flags.load();
    case BW_OPT_MAX_CTAS: return g_max_ctas.load();
    case BW_OPT_EXP_POLY: return g_exp_poly.load();
    case BW_OPT_PREFILL_KERNEL: return g_prefill_kernel.load();
    default: return -1;
  }
}

int bw_shard_plan(int64_t units, int world, int rank, int64_t* begin, int64_t* end) {
  if (!begin || !end) return BW_ERR_NULL;
  if (units < 0 || world <= 0 || rank < 0 || rank >= world) return BW_ERR_SHAPE;
  const int64_t base = units / world, rem = units % world;
  *begin = rank * base + (rank < rem ? rank : rem);
  *end = *begin + base + (rank < rem ? 1 : 0);
  return BW_OK;
}

const char* bw_strerror(int code) {
  switch (code) {
    case BW_OK: return "ok";
    case BW_ERR_SHAPE: return "unsupported or inconsistent shape";
    case BW_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case BW_ERR_CUDA: return "CUDA call failed";
    case BW_ERR_TIMEOUT: return "device-side wait timed out";
    case BW_ERR_NCCL: return "collective failed";
    case BW_ERR_NULL: return "required pointer is NULL";
    case BW_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown error";
  }
}

const char* bw_version(void) { return "bw_attn 0.1.0 (sm_100a)"; }

}  // extern "C"
