// bw_attn_fwd_host: attention forward on HOST buffers, with the PCIe copies
// pipelined against the kernels.
//
// The reference's harnesses copy their inputs to the device, launch, and copy
// the outputs back in series (kernelBench.cuh and the main() of every
// launcher file).  Here the work is cut into chunks and three queues overlap:
//   copy-in stream   H2D of chunk c + 1
//   caller's stream  the attention kernel on chunk c
//   copy-out stream  D2H of chunk c - 1
// Causal calls are cut along the sequence: query rows [s0, s1) need keys
// [0, s1) only, all of which have arrived with chunks 0 .. c, so chunk c runs
// as a split-length call with a query offset of s0 (rows in multiples of 128).
// Non-causal calls are cut along the batch.  Chunks shrink from first to last
// (weights nc .. 1), so that little work remains once the last copy-in lands.  The copies are strided 2-D
// copies (one per tensor and chunk), so both host layouts work without a
// staging copy.  Overlap needs page-locked host memory.
#include <mutex>

#include "../../include/bw_attn.h"
#include "kernels.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxChunks = 32;

struct PipeState {
  bool init = false;
  cudaStream_t s_in = nullptr, s_out = nullptr;
  cudaEvent_t ev_start = nullptr, ev_done = nullptr;
  cudaEvent_t ev_in[kMaxChunks] = {}, ev_cmp[kMaxChunks] = {};
};

std::mutex g_pipe_mu;   // held for the whole enqueue: the events are reused call to call
PipeState g_pipe[kMaxDevices];

int pipe_state(PipeState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BW_ERR_CUDA;
  PipeState& st = g_pipe[dev];
  if (!st.init) {
    const unsigned f = cudaEventDisableTiming;
    if (cudaStreamCreateWithFlags(&st.s_in, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&st.s_out, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&st.ev_start, f) != cudaSuccess ||
        cudaEventCreateWithFlags(&st.ev_done, f) != cudaSuccess)
      return BW_ERR_CUDA;
    for (int i = 0; i < kMaxChunks; ++i)
      if (cudaEventCreateWithFlags(&st.ev_in[i], f) != cudaSuccess ||
          cudaEventCreateWithFlags(&st.ev_cmp[i], f) != cudaSuccess)
        return BW_ERR_CUDA;
    st.init = true;
  }
  *out = &st;
  return BW_OK;
}

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

// Element strides (b, h, s) of a [B, H, S, D] tensor in the given layout.
void layout_strides(int layout, int H, int S, int D, int64_t st[3]) {
  if (layout == BW_LAYOUT_BSHD) {
    st[0] = (int64_t)S * H * D;
    st[1] = D;
    st[2] = (int64_t)H * D;
  } else {
    st[0] = (int64_t)H * S * D;
    st[1] = (int64_t)S * D;
    st[2] = D;
  }
}

// Copies rows [s0, s1) of every (b, h) of a [B, H, S, D] tensor (element size
// es, D elements per row) between host and device buffers of the same layout.
cudaError_t copy_rows(void* dst, const void* src, int layout, int B, int H, int S, int D, int es, int s0, int s1,
                      cudaMemcpyKind kind, cudaStream_t s) {
  const size_t row = (size_t)D * es;
  if (layout == BW_LAYOUT_BSHD) {
    // per b: rows s0 .. s1 of all heads are one contiguous run
    const size_t pitch = (size_t)S * H * row, off = (size_t)s0 * H * row;
    return cudaMemcpy2DAsync(static_cast<char*>(dst) + off, pitch, static_cast<const char*>(src) + off, pitch,
                             (size_t)(s1 - s0) * H * row, B, kind, s);
  }
  // BHSD: per (b, h) one run
  const size_t pitch = (size_t)S * row, off = (size_t)s0 * row;
  return cudaMemcpy2DAsync(static_cast<char*>(dst) + off, pitch, static_cast<const char*>(src) + off, pitch,
                           (size_t)(s1 - s0) * row, (size_t)B * H, kind, s);
}

}  // namespace

extern "C" {

size_t bw_attn_fwd_host_workspace_size(int B, int Hq, int Hkv, int S, int D) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return 0;
  const size_t q = (size_t)B * Hq * S * D * 2, kv = (size_t)B * Hkv * S * D * 2;
  return 2 * a256(q) + 2 * a256(kv) + a256((size_t)B * Hq * S * 4);
}

int bw_attn_fwd_host(const void* Q, const void* K, const void* V, void* O, float* LSE, int B, int Hq, int Hkv, int S,
                     int D, float scale, int causal, int layout, int chunks, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (!Q || !K || !V || !O || !workspace) return BW_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || Hq % Hkv != 0 || (D != 64 && D != 128)) return BW_ERR_SHAPE;
  if (layout != BW_LAYOUT_BHSD && layout != BW_LAYOUT_BSHD) return BW_ERR_SHAPE;
  if (workspace_bytes < bw_attn_fwd_host_workspace_size(B, Hq, Hkv, S, D)) return BW_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return BW_ERR_ALIGN;
  const int G = Hq / Hkv;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t qb = a256((size_t)B * Hq * S * D * 2), kvb = a256((size_t)B * Hkv * S * D * 2);
  void* dq = ws;
  void* dk = ws + qb;
  void* dv = ws + qb + kvb;
  void* dout = ws + qb + 2 * kvb;
  float* dl = reinterpret_cast<float*>(ws + 2 * qb + 2 * kvb);

  bw_strides st;
  layout_strides(layout, Hq, S, D, st.q);
  layout_strides(layout, Hkv, S, D, st.k);
  layout_strides(layout, Hkv, S, D, st.v);
  layout_strides(layout, Hq, S, D, st.o);

  // chunk plan: sequence rows (causal, multiples of 128) or batch entries
  const int ntiles = (S + 127) / 128;
  const bool by_rows = causal != 0;
  int nc = chunks <= 0 ? 4 : chunks;
  nc = nc > kMaxChunks ? kMaxChunks : nc;
  nc = nc > (by_rows ? ntiles : B) ? (by_rows ? ntiles : B) : nc;
  // Chunk sizes fall linearly (weights nc, nc - 1, .., 1): what is left after
  // the last copy-in (the last chunk's kernel and copy-out) is small, while the
  // copy-in stream, the bound, runs without gaps from the first chunk on.
  const int units = by_rows ? ntiles : B;
  const int64_t wsum = (int64_t)nc * (nc + 1) / 2;
  auto bound = [&](int c) -> int {
    const int64_t w = (int64_t)c * nc - (int64_t)c * (c - 1) / 2;   // weights of chunks 0 .. c - 1
    const int u = (int)((w * units + wsum / 2) / wsum);
    if (by_rows) return c == nc ? S : (u * 128 > S ? S : u * 128);
    return u;
  };

  cudaStream_t s_cmp = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  PipeState* ps = nullptr;
  int rc = pipe_state(&ps);
  if (rc != BW_OK) return rc;
  // the copy-in must not overwrite the device buffers before the caller's
  // earlier work on its stream is done
  if (cudaEventRecord(ps->ev_start, s_cmp) != cudaSuccess) return BW_ERR_CUDA;
  if (cudaStreamWaitEvent(ps->s_in, ps->ev_start, 0) != cudaSuccess) return BW_ERR_CUDA;
  if (cudaStreamWaitEvent(ps->s_out, ps->ev_start, 0) != cudaSuccess) return BW_ERR_CUDA;

  // An error after the first enqueue still orders the caller's stream after
  // every copy already queued on the copy-in and copy-out streams, so that a
  // caller who frees the buffers after the error (having synchronised its
  // stream) cannot race them.
  auto fail = [&](int code) -> int {
    if (cudaEventRecord(ps->ev_start, ps->s_in) == cudaSuccess) cudaStreamWaitEvent(s_cmp, ps->ev_start, 0);
    if (cudaEventRecord(ps->ev_done, ps->s_out) == cudaSuccess) cudaStreamWaitEvent(s_cmp, ps->ev_done, 0);
    return code;
  };
  for (int c = 0; c < nc; ++c) {
    const int lo = bound(c), hi = bound(c + 1);
    if (hi <= lo) continue;
    // ---- copy in
    cudaError_t e = cudaSuccess;
    if (by_rows) {
      e = copy_rows(dq, Q, layout, B, Hq, S, D, 2, lo, hi, cudaMemcpyHostToDevice, ps->s_in);
      if (e == cudaSuccess) e = copy_rows(dk, K, layout, B, Hkv, S, D, 2, lo, hi, cudaMemcpyHostToDevice, ps->s_in);
      if (e == cudaSuccess) e = copy_rows(dv, V, layout, B, Hkv, S, D, 2, lo, hi, cudaMemcpyHostToDevice, ps->s_in);
    } else {
      const size_t qs = (size_t)Hq * S * D * 2, ks = (size_t)Hkv * S * D * 2;
      e = cudaMemcpyAsync(static_cast<char*>(dq) + lo * qs, static_cast<const char*>(Q) + lo * qs, (hi - lo) * qs,
                          cudaMemcpyHostToDevice, ps->s_in);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(static_cast<char*>(dk) + lo * ks, static_cast<const char*>(K) + lo * ks, (hi - lo) * ks,
                            cudaMemcpyHostToDevice, ps->s_in);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(static_cast<char*>(dv) + lo * ks, static_cast<const char*>(V) + lo * ks, (hi - lo) * ks,
                            cudaMemcpyHostToDevice, ps->s_in);
    }
    if (e != cudaSuccess || cudaEventRecord(ps->ev_in[c], ps->s_in) != cudaSuccess) return fail(BW_ERR_CUDA);
    // ---- compute on the caller's stream
    if (cudaStreamWaitEvent(s_cmp, ps->ev_in[c], 0) != cudaSuccess) return fail(BW_ERR_CUDA);
    if (by_rows) {
      const size_t qoff = (size_t)lo * st.q[2], ooff = (size_t)lo * st.o[2];
      rc = bw::attn_forward(static_cast<const uint16_t*>(dq) + qoff, dk, dv, static_cast<uint16_t*>(dout) + ooff,
                            LSE ? dl + lo : nullptr, B, Hq, Hkv, hi - lo, hi, G, D, scale, 1, &st, stream, lo, S);
    } else {
      rc = bw::attn_forward(static_cast<const uint16_t*>(dq) + (size_t)lo * st.q[0],
                            static_cast<const uint16_t*>(dk) + (size_t)lo * st.k[0],
                            static_cast<const uint16_t*>(dv) + (size_t)lo * st.v[0],
                            static_cast<uint16_t*>(dout) + (size_t)lo * st.o[0],
                            LSE ? dl + (size_t)lo * Hq * S : nullptr, hi - lo, Hq, Hkv, S, S, G, D, scale, causal, &st,
                            stream, 0, S);
    }
    if (rc != BW_OK) return fail(rc);
    if (cudaEventRecord(ps->ev_cmp[c], s_cmp) != cudaSuccess) return fail(BW_ERR_CUDA);
    // ---- copy out
    if (cudaStreamWaitEvent(ps->s_out, ps->ev_cmp[c], 0) != cudaSuccess) return fail(BW_ERR_CUDA);
    if (by_rows) {
      e = copy_rows(O, dout, layout, B, Hq, S, D, 2, lo, hi, cudaMemcpyDeviceToHost, ps->s_out);
      if (e == cudaSuccess && LSE)
        e = cudaMemcpy2DAsync(LSE + lo, (size_t)S * 4, dl + lo, (size_t)S * 4, (size_t)(hi - lo) * 4,
                              (size_t)B * Hq, cudaMemcpyDeviceToHost, ps->s_out);
    } else {
      const size_t os = (size_t)Hq * S * D * 2;
      e = cudaMemcpyAsync(static_cast<char*>(O) + lo * os, static_cast<const char*>(dout) + lo * os, (hi - lo) * os,
                          cudaMemcpyDeviceToHost, ps->s_out);
      if (e == cudaSuccess && LSE)
        e = cudaMemcpyAsync(LSE + (size_t)lo * Hq * S, dl + (size_t)lo * Hq * S, (size_t)(hi - lo) * Hq * S * 4,
                            cudaMemcpyDeviceToHost, ps->s_out);
    }
    if (e != cudaSuccess) return fail(BW_ERR_CUDA);
  }
  // the caller's stream is ordered after the last copy-out (and the copy-in
  // stream is drained by it too, since every compute waited on a copy-in)
  if (cudaEventRecord(ps->ev_done, ps->s_out) != cudaSuccess) return BW_ERR_CUDA;
  if (cudaStreamWaitEvent(s_cmp, ps->ev_done, 0) != cudaSuccess) return BW_ERR_CUDA;
  return BW_OK;
}

}  // extern "C"
