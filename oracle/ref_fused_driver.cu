// Driver for the reference's own ground truth of the fused QK-norm + RoPE +
// attention op (TEST INFRASTRUCTURE ONLY).
//
// The reference computes its fused-op ground truth on the GPU with two naive
// kernels, ref_norm_rope<D> and ref_attention<D>
// (src/SM103/attention/GQA_fused_sm103.cu:328-420), driven by its own main()
// (:424-525) at one fixed configuration.  This translation unit includes that
// reference source file unmodified from the reference tree (its main() is
// renamed by the define around the #include below; build recipe:
// oracle/build_ref.py) and
// runs the same two kernels, with the same launch shape as the reference's
// main() (256 threads, one thread per row), on inputs given in files:
//
//   ref_fused <dir> B Hq Hkv S D neox causal use_norm pos_offset cache_len eps
//
// reads   <dir>/q.bin k.bin v.bin     bf16 [B,H,S,D] raw (BHSD, contiguous)
//         <dir>/cache.bin             fp32 [cache_len, D] (cos | sin)
//         <dir>/qg.bin kg.bin         fp32 [D]          (when use_norm)
// writes  <dir>/qn.bin kn.bin o.bin   bf16 raw
//         <dir>/lse.bin               fp32 [B,Hq,S]
//         <dir>/qrstd.bin krstd.bin   fp32              (when use_norm)
// Exit code 0 on success.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

// The reference file's own main() becomes reference_fused_main (never called).
#define main reference_fused_main
#include "GQA_fused_sm103.cu"
#undef main

namespace {

template <typename T>
bool read_file(const std::string& path, std::vector<T>& v) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  const size_t n = std::fread(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
  return n == v.size();
}

template <typename T>
bool write_file(const std::string& path, const std::vector<T>& v) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return false;
  const size_t n = std::fwrite(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
  return n == v.size();
}

template <typename T>
T* to_device(const std::vector<T>& h) {
  T* d = nullptr;
  if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
  cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
  return d;
}

template <typename T>
std::vector<T> from_device(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
  return h;
}

template <int D>
int run(const std::string& dir, int B, int Hq, int Hkv, int S, bool neox, bool causal, bool use_norm, int pos_offset,
        int cache_len, float eps) {
  const int G = Hq / Hkv;
  const size_t nq = (size_t)B * Hq * S * D, nkv = (size_t)B * Hkv * S * D;
  const size_t nlse = (size_t)B * Hq * S, nkr = (size_t)B * Hkv * S;
  std::vector<__nv_bfloat16> q(nq), k(nkv), v(nkv);
  std::vector<float> cache((size_t)cache_len * D), qg(D), kg(D);
  if (!read_file(dir + "/q.bin", q) || !read_file(dir + "/k.bin", k) || !read_file(dir + "/v.bin", v) ||
      !read_file(dir + "/cache.bin", cache))
    return 2;
  if (use_norm && (!read_file(dir + "/qg.bin", qg) || !read_file(dir + "/kg.bin", kg))) return 2;
  __nv_bfloat16 *dq = to_device(q), *dk = to_device(k), *dv = to_device(v);
  float *dcache = to_device(cache), *dqg = to_device(qg), *dkg = to_device(kg);
  __nv_bfloat16 *dqn, *dkn, *dout;
  float *dlse, *dqr, *dkr;
  cudaMalloc(&dqn, nq * 2);
  cudaMalloc(&dkn, nkv * 2);
  cudaMalloc(&dout, nq * 2);
  cudaMalloc(&dlse, nlse * 4);
  cudaMalloc(&dqr, nlse * 4);
  cudaMalloc(&dkr, nkr * 4);
  const float scale = 1.0f / std::sqrt((float)D);
  const int T = 256;
  const long q_rows = (long)B * Hq * S, k_rows = (long)B * Hkv * S;
  ref_norm_rope<D><<<(unsigned)((q_rows + T - 1) / T), T>>>(dq, dqn, use_norm ? dqr : nullptr, dcache,
                                                          use_norm ? dqg : nullptr, q_rows, S, cache_len,
                                                          pos_offset, eps, neox);
  ref_norm_rope<D><<<(unsigned)((k_rows + T - 1) / T), T>>>(dk, dkn, use_norm ? dkr : nullptr, dcache,
                                                          use_norm ? dkg : nullptr, k_rows, S, cache_len,
                                                          pos_offset, eps, neox);
  ref_attention<D><<<(unsigned)((q_rows + T - 1) / T), T>>>(dqn, dkn, dv, dout, dlse, B, Hq, Hkv, G, S, scale,
                                                          causal);
  if (cudaDeviceSynchronize() != cudaSuccess || cudaGetLastError() != cudaSuccess) return 3;
  bool ok = write_file(dir + "/qn.bin", from_device(dqn, nq)) && write_file(dir + "/kn.bin", from_device(dkn, nkv)) &&
            write_file(dir + "/o.bin", from_device(dout, nq)) && write_file(dir + "/lse.bin", from_device(dlse, nlse));
  if (use_norm)
    ok = ok && write_file(dir + "/qrstd.bin", from_device(dqr, nlse)) &&
         write_file(dir + "/krstd.bin", from_device(dkr, nkr));
  for (void* p : {(void*)dq, (void*)dk, (void*)dv, (void*)dcache, (void*)dqg, (void*)dkg, (void*)dqn, (void*)dkn,
                  (void*)dout, (void*)dlse, (void*)dqr, (void*)dkr})
    cudaFree(p);
  return ok ? 0 : 4;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 13) {
    std::fprintf(stderr, "usage: %s dir B Hq Hkv S D neox causal use_norm pos_offset cache_len eps\n", argv[0]);
    return 1;
  }
  const std::string dir = argv[1];
  const int B = std::atoi(argv[2]), Hq = std::atoi(argv[3]), Hkv = std::atoi(argv[4]), S = std::atoi(argv[5]);
  const int D = std::atoi(argv[6]);
  const bool neox = std::atoi(argv[7]) != 0, causal = std::atoi(argv[8]) != 0, use_norm = std::atoi(argv[9]) != 0;
  const int pos_offset = std::atoi(argv[10]), cache_len = std::atoi(argv[11]);
  const float eps = (float)std::atof(argv[12]);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || S <= 0) return 1;
  if (D == 64) return run<64>(dir, B, Hq, Hkv, S, neox, causal, use_norm, pos_offset, cache_len, eps);
  if (D == 128) return run<128>(dir, B, Hq, Hkv, S, neox, causal, use_norm, pos_offset, cache_len, eps);
  return 1;
}
