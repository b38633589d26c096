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

#include "../../include/bw_attn.h"
#include "kernels.h"

constexpr size_t kStaticScratchBytes = size_t(32) << 20;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol, not a device address: a kernel must be given the address returned by
// cudaGetSymbolAddress for the current device.
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

namespace {
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

}  // namespace

extern "C" {

size_t bw_gqa_decode_static_scratch_bytes(void) { return kStaticScratchBytes; }

int bw_gqa_decode_static(const void* Q, const void* K, const void* V, const int* kv_lens, const int64_t* kv_offsets,
                         void* O, float* LSE, int B, int Hq, int Hkv, int D, int64_t total_tokens, float scale,
                         int chunk, void* stream) {
  // Argument checks first, so that a bad call reports its own error before the
  // set-up touches the device.  The size rule is bw_gqa_decode's workspace rule.
  if (!Q || !K || !V || !kv_lens || !kv_offsets || !O) return BW_ERR_NULL;
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0 || total_tokens <= 0) return BW_ERR_SHAPE;
  if (bw_gqa_decode_workspace_size(B, Hq, Hkv, D, total_tokens, chunk) > kStaticScratchBytes)
    return BW_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != BW_OK) return rc;
  // The shared decode path (validation, tensor maps, scratch layout, launches)
  // on the static array instead of a caller workspace.
  return bw::decode_run(Q, K, V, kv_lens, kv_offsets, O, 0, LSE, B, Hq, Hkv, D, total_tokens, scale, chunk, scratch,
                        kStaticScratchBytes, stream);
}

}  // extern "C"
