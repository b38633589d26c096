// bw_gqa_decode_static: the split-KV decode for callers that cannot allocate
// device memory.
//
// bw_gqa_decode needs a caller-provided workspace for its per-split partials.
// Some callers have no way to provide one: code that runs inside an allocator
// hook or a memory-pool callback (where calling cudaMalloc would re-enter the
// allocator), a C host runtime that was handed fixed device buffers and owns no
// allocator, or a process whose device memory is fully reserved up front.  This
// entry point serves them: its scratch lives in a fixed-size array in the
// library's own device data (`g_decode_scratch` below), so the call allocates
// nothing and takes no workspace.  The caller still passes the inputs and
// outputs.
//
// Limits and sharing rules:
//  * The scratch is kStaticScratchBytes (32 MiB) per device.  It is part of the
//    library's module image: every GPU on which the library is loaded holds it
//    until the process exits.  Calls whose partials would not fit (see
//    bw_gqa_decode_workspace_size with the same arguments) are rejected with
//    BW_ERR_WORKSPACE before anything is launched.
//  * Every call on a device uses the same array and it keeps the previous
//    call's contents.  Nothing in it needs to start at zero: each call writes
//    its chunk table and every partial it later reads.  Two calls whose kernels
//    overlap on the GPU (different streams, no ordering between them) race on
//    the array and give wrong results; order such calls on one stream or with
//    events.
//  * The first call on each device performs a one-time set-up with that device
//    current (it looks up the array's device address with
//    cudaGetSymbolAddress).  Make that first call before any stream capture.
#include <mutex>

#include <cudaTypedefs.h>

#include "../../include/bw_attn.h"
#include "kernels.h"

constexpr size_t kStaticScratchBytes = size_t(32) << 20;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol, not a device address: a kernel must be given the address returned by
// cudaGetSymbolAddress for the current device.
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

namespace {
constexpr int kDefaultChunk = 1024;
constexpr int kMaxDevices = 64;


std::mutex g_static_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Set-up, once per device, with that device current.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BW_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || ptr == nullptr) return BW_ERR_CUDA;
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return BW_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

extern "C" {

size_t bw_gqa_decode_static_scratch_bytes(void) { return kStaticScratchBytes; }

int bw_gqa_decode_static(const void* Q, const void* K, const void* V, const int* kv_lens, const int64_t* kv_offsets,
                         void* O, float* LSE, int B, int Hq, int Hkv, int D, int64_t total_tokens, float scale,
                         int chunk, void* stream) {
  if (!Q || !K || !V || !kv_lens || !kv_offsets || !O) return BW_ERR_NULL;
  if (B <= 0 || B > 4096 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0) return BW_ERR_SHAPE;
  const int G = Hq / Hkv;
  if (G > 16 || (D != 64 && D != 128) || total_tokens <= 0 || total_tokens >= (int64_t(1) << 31))
    return BW_ERR_SHAPE;
  if (!(scale > 0.f) || !(scale < 3.4e38f)) return BW_ERR_SHAPE;
  if (chunk <= 0) chunk = kDefaultChunk;
  if (chunk % 64 != 0) return BW_ERR_SHAPE;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(Q) || !a16(K) || !a16(V) || !a16(O)) return BW_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(kv_offsets) & 7u) || (reinterpret_cast<uintptr_t>(kv_lens) & 3u))
    return BW_ERR_ALIGN;
  // Same scratch layout and size rule as the workspace of bw_gqa_decode.
  if (bw_gqa_decode_workspace_size(B, Hq, Hkv, D, total_tokens, chunk) > kStaticScratchBytes)
    return BW_ERR_WORKSPACE;

  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != BW_OK) return rc;
  int* err = nullptr;
  int num_sms = 0;
  void* enc = nullptr;
  rc = bw::device_context(&err, &num_sms, &enc);
  if (rc != BW_OK) return rc;
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(enc);

  bw::DecodeMaps maps;   // the 3-D layout launch_decode expects (kernels.h)
  for (int i = 0; i < 2; ++i) {
    cuuint64_t dims[3] = {64, (cuuint64_t)total_tokens, (cuuint64_t)Hkv * D / 64};
    cuuint64_t strides[2] = {(cuuint64_t)Hkv * D * 2, 128};
    cuuint32_t box[3] = {64, 64, (cuuint32_t)(D / 64)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = encode(i == 0 ? &maps.k : &maps.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                        const_cast<void*>(i == 0 ? K : V), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return BW_ERR_CUDA;
  }

  const int64_t parts = (int64_t)Hkv * ((total_tokens + chunk - 1) / chunk + B);
  uint8_t* ws = static_cast<uint8_t*>(scratch);
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
  p.err = err;
  p.timeout_ns = (uint64_t)bw_get_option(BW_OPT_TIMEOUT_NS);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bw::launch_decode(p, maps, num_sms, s) != cudaSuccess) return BW_ERR_CUDA;

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

}  // extern "C"
