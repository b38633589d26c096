// bw_harness: the reference's per-launcher main() programs (load the
// data/*.bin files written by base/baseline_*.py, run the launcher, check O and
// LSE, benchmark) as one C++ program over this library's C ABI.
//
//   bw_harness <mode> [--B n] [--Hq n] [--Hkv n] [--S n] [--Sq n] [--Skv n] [--D n]
//              [--data DIR] [--iters n] [--warmup n] [--tol x]
//   mode: gqa | gqa_causal | gqa_split | mha | mha_f32
//
// Files (headerless float32, the reference's format; base/baseline_gqa.py:165-170):
//   gqa:        DIR/gqa_{q,k,v,o,lse}.bin           (src/SM120/attention/GQA_sm120.cu:427-433)
//   gqa_causal: DIR/gqa_causal_{q,k,v,o,lse}.bin
//   gqa_split:  DIR/gqa_split_{q,k,v,o,lse}.bin     (adhitya_GQA.cu:243-255)
//   mha:        DIR/mha_{q,k,v,out}.bin             (MHA_sm120.cu:314-318; bf16 compute here)
//   mha_f32:    the same files, fp32 in / out through launch_mha_f32 (the
//               reference's mha_v3_tc call shape; 3xTF32, D = 64)
// Inputs are narrowed to bf16 as the reference's loaders do.  Without the
// files the inputs are N(0,1) from a fixed seed and only the benchmark runs.
//
// Check: |ref - got| <= tol + tol |ref| on every element (the reference's
// checkResult with atol = rtol = 2e-2, include/utils/kernelUtils.cuh:91-110).
// Benchmark: warm-ups, then timed launches each preceded by a 256 MiB memset
// that evicts L2, CUDA events around the launch alone, average / median / min
// / max (include/utils/kernelBench.cuh:34-98).  Exit status 0 = all checks
// passed (or nothing to check), 1 = mismatch, 2 = usage or CUDA error.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "bw_attn_launchers.hpp"

namespace {

struct Args {
  std::string mode;
  int B = 4, Hq = 32, Hkv = 8, S = 4096, Sq = 0, Skv = 0, D = 128;
  std::string data = "data";
  int iters = 100, warmup = 25;
  float tol = 2e-2f;
};

int usage() {
  std::fprintf(stderr,
               "usage: bw_harness gqa|gqa_causal|gqa_split|mha|mha_f32 [--B n] [--Hq n] [--Hkv n] [--S n] [--Sq n] "
               "[--Skv n] [--D 64|128] [--data DIR] [--iters n] [--warmup n] [--tol x]\n");
  return 2;
}

#define CK(x)                                                                              \
  do {                                                                                     \
    cudaError_t e_ = (x);                                                                  \
    if (e_ != cudaSuccess) {                                                               \
      std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
      std::exit(2);                                                                        \
    }                                                                                      \
  } while (0)

bool file_has(const std::string& p, size_t n) {
  FILE* f = std::fopen(p.c_str(), "rb");
  if (!f) return false;
  std::fseek(f, 0, SEEK_END);
  const long bytes = std::ftell(f);
  std::fclose(f);
  return bytes == (long)(n * sizeof(float));
}

void to_bf16(const std::vector<float>& a, std::vector<__nv_bfloat16>& b) {
  b.resize(a.size());
  for (size_t i = 0; i < a.size(); ++i) b[i] = __float2bfloat16(a[i]);
}

void randn(std::vector<float>& a, unsigned seed) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> nd(0.f, 1.f);
  for (auto& x : a) x = nd(gen);
}

// The reference's reportPrecision / checkResult, on host float arrays.
bool check(const char* label, const std::vector<float>& ref, const std::vector<float>& got, float tol) {
  double max_abs = 0, sum_abs = 0;
  size_t bad = ref.size();
  for (size_t i = 0; i < ref.size(); ++i) {
    const double d = std::fabs((double)ref[i] - got[i]);
    max_abs = std::max(max_abs, d);
    sum_abs += d;
    if (bad == ref.size() && d > tol + tol * std::fabs(ref[i])) bad = i;
  }
  std::printf("  %-4s max_abs=%.3e  mean_abs=%.3e  ", label, max_abs, sum_abs / std::max<size_t>(1, ref.size()));
  if (bad == ref.size()) {
    std::printf("Values match!\n");
    return true;
  }
  std::printf("Values don't match at index %zu! Ref: %.8f, GPU: %.8f\n", bad, ref[bad], got[bad]);
  return false;
}

template <typename F>
void bench(const char* name, F launch, int iters, int warmup, double flops) {
  void* flush = nullptr;
  const size_t kFlush = size_t(256) << 20;
  CK(cudaMalloc(&flush, kFlush));
  for (int i = 0; i < warmup; ++i) launch();
  CK(cudaDeviceSynchronize());
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  std::vector<float> t;
  for (int i = 0; i < iters; ++i) {
    CK(cudaMemset(flush, 0, kFlush));
    CK(cudaEventRecord(a));
    launch();
    CK(cudaEventRecord(b));
    CK(cudaEventSynchronize(b));
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, a, b));
    t.push_back(ms);
  }
  std::sort(t.begin(), t.end());
  const double avg = std::accumulate(t.begin(), t.end(), 0.0) / t.size();
  const double med = t.size() % 2 ? t[t.size() / 2] : 0.5 * (t[t.size() / 2 - 1] + t[t.size() / 2]);
  std::printf("\n----------------------------------------------------------\n");
  std::printf("Benchmark: %s\n", name);
  std::printf("----------------------------------------------------------\n");
  std::printf("Average Time:  %10.4f ms\nMedian Time:   %10.4f ms\nMin Time:      %10.4f ms\nMax Time:      %10.4f ms\n",
              avg, med, t.front(), t.back());
  std::printf("Performance:   %10.4f TFLOPS\n", flops / (avg * 1e9));
  std::printf("----------------------------------------------------------\n");
  CK(cudaEventDestroy(a));
  CK(cudaEventDestroy(b));
  CK(cudaFree(flush));
}

template <int D>
int run(const Args& a) {
  const bool split = a.mode == "gqa_split", mha = a.mode == "mha";
  const bool causal = a.mode == "gqa_causal";
  const int Hkv = mha ? a.Hq : a.Hkv;
  const int Sq = split ? (a.Sq ? a.Sq : a.S) : a.S, Skv = split ? (a.Skv ? a.Skv : a.S) : a.S;
  if (a.Hq % Hkv != 0) return usage();
  const int G = a.Hq / Hkv;
  const size_t nq = (size_t)a.B * a.Hq * Sq * D, nkv = (size_t)a.B * Hkv * Skv * D, nl = (size_t)a.B * a.Hq * Sq;
  const std::string pre = a.data + "/" + (mha ? std::string("mha") : a.mode) + "_";
  const std::string o_name = mha ? "out" : "o";
  const bool has_ref = file_has(pre + "q.bin", nq) && file_has(pre + "k.bin", nkv) && file_has(pre + "v.bin", nkv) &&
                       file_has(pre + o_name + ".bin", nq);
  const bool has_lse = !mha && file_has(pre + "lse.bin", nl);
  std::vector<float> q(nq), k(nkv), v(nkv), o_ref, lse_ref;
  if (has_ref) {
    bw_compat::loadBin((pre + "q.bin").c_str(), q.data(), nq);
    bw_compat::loadBin((pre + "k.bin").c_str(), k.data(), nkv);
    bw_compat::loadBin((pre + "v.bin").c_str(), v.data(), nkv);
    o_ref.resize(nq);
    bw_compat::loadBin((pre + o_name + ".bin").c_str(), o_ref.data(), nq);
    if (has_lse) {
      lse_ref.resize(nl);
      bw_compat::loadBin((pre + "lse.bin").c_str(), lse_ref.data(), nl);
    }
    std::printf("Loaded reference data from %s*.bin\n", pre.c_str());
  } else {
    randn(q, 1);
    randn(k, 2);
    randn(v, 3);
    std::printf("No matching reference files under %s -- random inputs, benchmark only\n", a.data.c_str());
  }
  std::vector<__nv_bfloat16> hq, hk, hv;
  to_bf16(q, hq);
  to_bf16(k, hk);
  to_bf16(v, hv);
  __nv_bfloat16 *dq, *dk, *dv, *dout;
  float* dl;
  CK(cudaMalloc(&dq, nq * 2));
  CK(cudaMalloc(&dk, nkv * 2));
  CK(cudaMalloc(&dv, nkv * 2));
  CK(cudaMalloc(&dout, nq * 2));
  CK(cudaMalloc(&dl, nl * 4));
  CK(cudaMemcpy(dq, hq.data(), nq * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dk, hk.data(), nkv * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dv, hv.data(), nkv * 2, cudaMemcpyHostToDevice));
  const float scale = 1.f / std::sqrt((float)D);
  auto launch = [&]() -> int {
    if (mha) return bw_compat::launch_mha<128, 128, D>(dq, dk, dv, dout, scale, a.S, a.B, a.Hq);
    if (split) return bw_compat::launch_gqa_split<128, 128, D>(dq, dk, dv, dout, dl, a.B, a.Hq, Hkv, Sq, Skv, G, scale);
    if (causal) return bw_compat::launch_gqa_causal<128, 128, D>(dq, dk, dv, dout, dl, a.B, a.Hq, Hkv, a.S, G, scale);
    return bw_compat::launch_gqa<128, 128, D>(dq, dk, dv, dout, dl, a.B, a.Hq, Hkv, a.S, G, scale);
  };
  std::printf("%s: B=%d Hq=%d Hkv=%d Sq=%d Skv=%d D=%d (%s)\n", a.mode.c_str(), a.B, a.Hq, Hkv, Sq, Skv, D,
              bw_version());
  const int rc = launch();
  if (rc != BW_OK) {
    std::fprintf(stderr, "launch failed: %s\n", bw_strerror(rc));
    return 2;
  }
  CK(cudaDeviceSynchronize());
  if (bw_stream_status(nullptr) != BW_OK) {
    std::fprintf(stderr, "device-side error reported by bw_stream_status\n");
    return 2;
  }
  bool ok = true;
  if (has_ref) {
    std::vector<__nv_bfloat16> ho(nq);
    std::vector<float> o(nq), l(nl);
    CK(cudaMemcpy(ho.data(), dout, nq * 2, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < nq; ++i) o[i] = __bfloat162float(ho[i]);
    std::printf("\nCorrectness (tolerance atol = rtol = %.0e):\n", a.tol);
    ok = check("O", o_ref, o, a.tol) && ok;
    if (has_lse) {
      CK(cudaMemcpy(l.data(), dl, nl * 4, cudaMemcpyDeviceToHost));
      ok = check("LSE", lse_ref, l, a.tol) && ok;
    }
  }
  double flops = 4.0 * a.B * a.Hq * (double)Sq * Skv * D;
  if (causal) flops /= 2;
  bench(("bw_attn " + a.mode).c_str(), [&]() { launch(); }, a.iters, a.warmup, flops);
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dout);
  cudaFree(dl);
  return ok ? 0 : 1;
}

// fp32 MHA through the reference's mha_v3_tc call shape (launch_mha_f32).
int run_mha_f32(const Args& a) {
  constexpr int D = 64;
  const size_t n = (size_t)a.B * a.Hq * a.S * D;
  const std::string pre = a.data + "/mha_";
  const bool has_ref = file_has(pre + "q.bin", n) && file_has(pre + "k.bin", n) && file_has(pre + "v.bin", n) &&
                       file_has(pre + "out.bin", n);
  std::vector<float> q(n), k(n), v(n), o_ref, o(n);
  if (has_ref) {
    bw_compat::loadBin((pre + "q.bin").c_str(), q.data(), n);
    bw_compat::loadBin((pre + "k.bin").c_str(), k.data(), n);
    bw_compat::loadBin((pre + "v.bin").c_str(), v.data(), n);
    o_ref.resize(n);
    bw_compat::loadBin((pre + "out.bin").c_str(), o_ref.data(), n);
    std::printf("Loaded reference data from %s*.bin\n", pre.c_str());
  } else {
    randn(q, 1);
    randn(k, 2);
    randn(v, 3);
    std::printf("No matching reference files under %s -- random inputs, benchmark only\n", a.data.c_str());
  }
  float *dq, *dk, *dv, *dout;
  CK(cudaMalloc(&dq, n * 4));
  CK(cudaMalloc(&dk, n * 4));
  CK(cudaMalloc(&dv, n * 4));
  CK(cudaMalloc(&dout, n * 4));
  CK(cudaMemcpy(dq, q.data(), n * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dk, k.data(), n * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dv, v.data(), n * 4, cudaMemcpyHostToDevice));
  const float scale = 1.f / std::sqrt((float)D);
  auto launch = [&]() { return bw_compat::launch_mha_f32<16, 32, D>(dq, dk, dv, dout, scale, a.S, a.B, a.Hq); };
  std::printf("mha_f32: B=%d H=%d S=%d D=%d (%s)\n", a.B, a.Hq, a.S, D, bw_version());
  const int rc = launch();
  if (rc != BW_OK) {
    std::fprintf(stderr, "launch failed: %s\n", bw_strerror(rc));
    return 2;
  }
  CK(cudaDeviceSynchronize());
  if (bw_stream_status(nullptr) != BW_OK) {
    std::fprintf(stderr, "device-side error reported by bw_stream_status\n");
    return 2;
  }
  bool ok = true;
  if (has_ref) {
    CK(cudaMemcpy(o.data(), dout, n * 4, cudaMemcpyDeviceToHost));
    std::printf("\nCorrectness (tolerance atol = rtol = %.0e):\n", a.tol);
    ok = check("O", o_ref, o, a.tol);
  }
  bench("bw_attn mha_f32", [&]() { launch(); }, a.iters, a.warmup, 4.0 * a.B * a.Hq * (double)a.S * a.S * D);
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dout);
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) return usage();
  Args a;
  a.mode = argv[1];
  if (a.mode != "gqa" && a.mode != "gqa_causal" && a.mode != "gqa_split" && a.mode != "mha" && a.mode != "mha_f32")
    return usage();
  for (int i = 2; i < argc; ++i) {
    const std::string k = argv[i];
    if (i + 1 >= argc) return usage();
    const char* v = argv[++i];
    if (k == "--B") a.B = std::atoi(v);
    else if (k == "--Hq") a.Hq = std::atoi(v);
    else if (k == "--Hkv") a.Hkv = std::atoi(v);
    else if (k == "--S") a.S = std::atoi(v);
    else if (k == "--Sq") a.Sq = std::atoi(v);
    else if (k == "--Skv") a.Skv = std::atoi(v);
    else if (k == "--D") a.D = std::atoi(v);
    else if (k == "--data") a.data = v;
    else if (k == "--iters") a.iters = std::atoi(v);
    else if (k == "--warmup") a.warmup = std::atoi(v);
    else if (k == "--tol") a.tol = (float)std::atof(v);
    else return usage();
  }
  if (a.B <= 0 || a.Hq <= 0 || a.Hkv <= 0 || a.S <= 0 || a.iters <= 0 || a.warmup < 0) return usage();
  if (a.mode == "mha_f32") return run_mha_f32(a);   // D = 64, the reference's instantiation
  if (a.D == 64) return run<64>(a);
  if (a.D == 128) return run<128>(a);
  return usage();
}
