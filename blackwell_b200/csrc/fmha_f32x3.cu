// fp32 MHA forward at fp32 accuracy on the TF32 tensor cores: the 3xTF32 split.
//
// The reference's fp32 MHA kernel (mha_v3_tc, src/SM120/attention/MHA_sm120.cu:
// split_tf32 :39-62, used on Q, K and V at :119-138) keeps fp32 accuracy on
// TF32 MMAs by splitting each operand x into a TF32 "big" part and the TF32
// rounding of the remainder, x = hi + lo, and summing three products:
//     a b ~ a_hi b_hi + a_hi b_lo + a_lo b_hi     (the lo * lo term is ~2^-22 a b).
// Here the same split drives tcgen05 kind::tf32 MMAs:
//   split pass      fp32 Q, K -> hi / lo arrays (row-major, [B, H, S, 64]) and
//                   V -> hi / lo TRANSPOSED ([B, H, 64, S32], S32 = S rounded
//                   up to 32), so that every MMA operand is K-major (the form
//                   the QK^T path of the tensor cores is known to take for
//                   TF32 operands);
//   attention       S = Qhi Khi^T + Qhi Klo^T + Qlo Khi^T    (24 MMAs per tile)
//                   O += Phi Vhi + Phi Vlo + Plo Vhi         (12 MMAs per tile)
//                   with P = 2^(s - m) split the same way by the softmax
//                   threads and staged in shared memory (SS form: both
//                   operands in shared memory).
// Everything else is fp32: the online softmax in the log2 domain (exact running
// max, ex2.approx: relative error ~2^-22), the row sums, O / l and
// LSE = ln 2 (m + log2 l).  The result sits ~1e-6 from the fp64 ground truth,
// the order of the reference kernel's own error.
//
// Kernel layout (one CTA per (b, h, 128-row query tile), 192 threads):
//   warps 0-3  softmax: thread t owns query row t (TMEM lane t)
//   warp 4     TMA producer: Qhi, Qlo once, then a 3-stage ring of 32-key
//              stages (Khi, Klo, VThi, VTlo: 4 x 8 KB)
//   warp 5     MMA issuer (one thread) and TMEM owner
// TMEM (128 columns): S_0 | S_1 (32 fp32 columns each, double-buffered so that
// QK^T of tile j + 1 runs during the softmax of tile j) | O (64 columns).
// Head dimension 64 (the reference's mha_v3_tc is instantiated at D = 64).
#include "kernels.h"
#include "ptx.cuh"
#include "softmax_math.cuh"
#include "tmem_io.cuh"

namespace bw {
namespace {

constexpr int kD = 64;
constexpr int kRows = 128;      // query rows per CTA
constexpr int kKeys = 32;       // keys per stage
constexpr int kNS = 3;          // ring stages
constexpr int kThreads = 192;

// Shared memory (offsets from a 1024-aligned base).  Tiles are 128-byte
// swizzled, K-major: 128 B = 32 fp32 of the reduction dimension per row.
constexpr int kQTile = kRows * kD * 4;            // 32 KB: 2 panels of 128 rows x 128 B
constexpr int kQPanel = kRows * 128;
constexpr int kKTile = kKeys * kD * 4;            // 8 KB: 2 panels of 32 rows x 128 B
constexpr int kKPanel = kKeys * 128;
constexpr int kVTile = kD * kKeys * 4;            // 8 KB: 64 rows (d) x 128 B (32 keys)
constexpr int kStage = 2 * kKTile + 2 * kVTile;   // Khi, Klo, VThi, VTlo
constexpr int kPTile = kRows * kKeys * 4;         // 16 KB: 128 rows x 128 B
constexpr int kOffQ = 0;                          // Qhi, Qlo
constexpr int kOffKV = 2 * kQTile;
constexpr int kOffP = kOffKV + kNS * kStage;      // Phi, Plo
constexpr int kOffBar = kOffP + 2 * kPTile;
constexpr int kBytes = kOffBar + 256;
constexpr int kSmemAlloc = kBytes + 1024;
static_assert(kSmemAlloc <= 232448, "shared memory");

struct BarsX3 {
  uint64_t q_full, s_full[2], p_full, pv_done, mma_done;
  uint64_t kv_full[kNS], kv_empty[kNS];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(BarsX3) <= 256, "barrier block");

__device__ __forceinline__ float round_tf32(float x) {
  // round to nearest on the 13 mantissa bits a TF32 operand drops
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// ------------------------------------------------------------- split pass
// Row-major hi / lo of one [B, H, S, 64] fp32 tensor (element strides sb, sh,
// ss; d contiguous) into contiguous arrays.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int64_t sb, int64_t sh,
                                                         int64_t ss, float* __restrict__ hi, float* __restrict__ lo,
                                                         int B, int H, int S) {
  const int64_t n4 = (int64_t)B * H * S * (kD / 4);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (kD / 4);
    const int c = (int)(i - row * (kD / 4));
    const int s = (int)(row % S);
    const int64_t bh = row / S;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const float4 v = *reinterpret_cast<const float4*>(x + b * sb + h * sh + s * ss + 4 * c);
    float4 a, r;
    a.x = round_tf32(v.x); r.x = round_tf32(v.x - a.x);
    a.y = round_tf32(v.y); r.y = round_tf32(v.y - a.y);
    a.z = round_tf32(v.z); r.z = round_tf32(v.z - a.z);
    a.w = round_tf32(v.w); r.w = round_tf32(v.w - a.w);
    reinterpret_cast<float4*>(hi)[i] = a;
    reinterpret_cast<float4*>(lo)[i] = r;
  }
}

// Transposed hi / lo of V: [B, H, S, 64] -> [B, H, 64, S32] through a 32 x 32
// shared-memory tile per block (coalesced reads and writes); columns s >= S
// are written as zero.
__global__ void __launch_bounds__(256) split_vt_kernel(const float* __restrict__ x, int64_t sb, int64_t sh,
                                                       int64_t ss, float* __restrict__ hi, float* __restrict__ lo,
                                                       int B, int H, int S, int S32) {
  __shared__ float th[32][33], tl[32][33];
  const int tiles_s = S32 / 32;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  for (int tile = blockIdx.x; tile < tiles_s * (kD / 32); tile += gridDim.x) {
    const int s0 = (tile / (kD / 32)) * 32, d0 = (tile % (kD / 32)) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
    for (int r = ty; r < 32; r += 8) {
      const int s = s0 + r;
      float v = s < S ? x[b * sb + h * sh + (int64_t)s * ss + d0 + tx] : 0.f;
      const float a = round_tf32(v);
      th[r][tx] = a;
      tl[r][tx] = round_tf32(v - a);
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
      const int64_t o = ((int64_t)bh * kD + d0 + r) * S32 + s0 + tx;
      hi[o] = th[tx][r];
      lo[o] = tl[tx][r];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------- attention
struct F32x3Item {
  int b, h, qt;
};
__device__ __forceinline__ F32x3Item x3_item(const F32x3Params& p) {
  F32x3Item it;
  const int per = p.n_qtiles;
  const int r = blockIdx.x / per;
  it.qt = blockIdx.x - r * per;
  it.b = r / p.H;
  it.h = r - it.b * p.H;
  return it;
}

__device__ void x3_producer(const F32x3Params& p, const F32x3Maps& maps, uint8_t* smem, BarsX3& bars,
                            const WaitCtl& wc) {
  const F32x3Item it = x3_item(p);
  const int n = p.n_kvtiles;
  mbar_arrive_expect_tx(&bars.q_full, 2 * kQTile);
  for (int part = 0; part < 2; ++part)
    for (int c = 0; c < 2; ++c)
      tma_load_4d(smem + kOffQ + part * kQTile + c * kQPanel, part ? &maps.q_lo : &maps.q_hi, &bars.q_full, c * 32,
                  it.qt * kRows, it.h, it.b);
  int j = 0;
  bool ok = true;
  for (; j < n; ++j) {
    const int st = j % kNS;
    if (!wc.wait(&bars.kv_empty[st], ((j / kNS) & 1) ^ 1)) { ok = false; break; }
    mbar_arrive_expect_tx(&bars.kv_full[st], kStage);
    uint8_t* dst = smem + kOffKV + st * kStage;
    for (int part = 0; part < 2; ++part) {
      for (int c = 0; c < 2; ++c)
        tma_load_4d(dst + part * kKTile + c * kKPanel, part ? &maps.k_lo : &maps.k_hi, &bars.kv_full[st], c * 32,
                    j * kKeys, it.h, it.b);
      tma_load_4d(dst + 2 * kKTile + part * kVTile, part ? &maps.vt_lo : &maps.vt_hi, &bars.kv_full[st], j * kKeys,
                  0, it.h, it.b);
    }
  }
  if (!ok) {
    // unwinding: wait for the loads already issued before the CTA exits
    for (int i = j > kNS ? j - kNS : 0; i < j; ++i) drain_wait(&bars.kv_full[i % kNS], (i / kNS) & 1, wc.timeout_ns);
    drain_wait(&bars.q_full, 0, wc.timeout_ns);
  }
}

__device__ void x3_mma(const F32x3Params& p, uint8_t* smem, BarsX3& bars, const WaitCtl& wc, uint32_t tmem) {
  constexpr uint32_t IDESC_QK = idesc_tf32_f32(kRows, kKeys, false);
  constexpr uint32_t IDESC_PV = idesc_tf32_f32(kRows, kD, false);
  constexpr uint32_t HI = sdesc_hi_sbo1024();
  const uint32_t base = smem_u32(smem);
  const uint32_t q_hi = sdesc_lo(base + kOffQ, 16), q_lo = sdesc_lo(base + kOffQ + kQTile, 16);
  const uint32_t p_hi = sdesc_lo(base + kOffP, 16), p_lo = sdesc_lo(base + kOffP + kPTile, 16);
  const int n = p.n_kvtiles;
  const uint32_t o_tm = tmem + 64;
  auto kv = [&](int j, int off) { return sdesc_lo(base + kOffKV + (j % kNS) * kStage + off, 16); };
  // S(j) = Qhi Khi^T + Qhi Klo^T + Qlo Khi^T into buffer j % 2; a k-step is 8
  // fp32 (32 bytes) of the head dimension: panel ks / 4, offset (ks % 4) * 32.
  auto issue_qk = [&](int j) {
    const uint32_t k_hi = kv(j, 0), k_lo = kv(j, kKTile);
    const uint32_t d = tmem + (j & 1) * 32;
#pragma unroll
    for (int ks = 0; ks < kD / 8; ++ks) {
      const uint32_t qo = ((ks >> 2) * kQPanel + (ks & 3) * 32) / 16;
      const uint32_t ko = ((ks >> 2) * kKPanel + (ks & 3) * 32) / 16;
      mma_ss_lh_tf32(d, q_hi + qo, HI, k_hi + ko, HI, IDESC_QK, ks > 0);
      mma_ss_lh_tf32(d, q_hi + qo, HI, k_lo + ko, HI, IDESC_QK, 1);
      mma_ss_lh_tf32(d, q_lo + qo, HI, k_hi + ko, HI, IDESC_QK, 1);
    }
  };
  bool ok = wc.wait(&bars.q_full, 0);
  if (ok) ok = wc.wait(&bars.kv_full[0], 0);
  if (ok) {
    tc_fence_after();
    issue_qk(0);
    tc_commit(&bars.s_full[0]);
  }
  for (int j = 0; ok && j < n; ++j) {
    if (j + 1 < n) {
      if (!wc.wait(&bars.kv_full[(j + 1) % kNS], ((j + 1) / kNS) & 1)) { ok = false; break; }
      tc_fence_after();
      issue_qk(j + 1);   // its buffer held S(j - 1), consumed before P(j - 1) was published
      tc_commit(&bars.s_full[(j + 1) & 1]);
    }
    if (!spin_wait(wc, &bars.p_full, j & 1)) { ok = false; break; }
    tc_fence_after();
    // O += Phi VThi + Phi VTlo + Plo VThi; a k-step is 8 keys (32 bytes)
    const uint32_t v_hi = kv(j, 2 * kKTile), v_lo = kv(j, 2 * kKTile + kVTile);
#pragma unroll
    for (int ks = 0; ks < kKeys / 8; ++ks) {
      const uint32_t o = (ks * 32) / 16;
      mma_ss_lh_tf32(o_tm, p_hi + o, HI, v_hi + o, HI, IDESC_PV, (j > 0 || ks > 0) ? 1u : 0u);
      mma_ss_lh_tf32(o_tm, p_hi + o, HI, v_lo + o, HI, IDESC_PV, 1);
      mma_ss_lh_tf32(o_tm, p_lo + o, HI, v_hi + o, HI, IDESC_PV, 1);
    }
    tc_commit(&bars.pv_done);
    tc_commit(&bars.kv_empty[j % kNS]);
  }
  tc_commit(&bars.mma_done);
  drain_wait(&bars.mma_done, 0, wc.timeout_ns);
}

__device__ void x3_softmax(const F32x3Params& p, uint8_t* smem, BarsX3& bars, const WaitCtl& wc, uint32_t tmem,
                           int t) {
  const F32x3Item it = x3_item(p);
  const int n = p.n_kvtiles;
  const int row = it.qt * kRows + t;
  const uint32_t lane_off = (uint32_t)((t >> 5) * 32) << 16;
  const uint32_t o_tm = tmem + lane_off + 64;
  const float c = p.scale_log2;
  float m_run = -INFINITY, l_run = 0.f;
  uint8_t* p_hi = smem + kOffP + t * 128;
  uint8_t* p_lo = p_hi + kPTile;
  for (int j = 0; j < n; ++j) {
    if (!wc.wait(&bars.s_full[j & 1], (j >> 1) & 1)) return;
    tc_fence_after();
    uint32_t r[32];
    tmem_ld32(tmem + lane_off + (j & 1) * 32, r);
    float* s = reinterpret_cast<float*>(r);
    const int lim = p.S - j * kKeys;   // keys past the end of the sequence are masked
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kKeys; ++i) {
      if (i >= lim) s[i] = -INFINITY;
      mx = fmaxf(mx, s[i]);
    }
    const float m_new = fmaxf(m_run, mx * c);   // finite: every tile has a key
    const float corr = m_run == -INFINITY ? 0.f : ex2_mufu(m_run - m_new);
    m_run = m_new;
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kKeys; ++i) {
      s[i] = ex2_mufu(fmaf(s[i], c, -m_new));
      sum += s[i];
    }
    l_run = l_run * corr + sum;
    // PV(j - 1) has read P(j - 1) and finished with O: P(j) may be written and O rescaled
    if (j > 0) {
      if (!wc.wait(&bars.pv_done, (j - 1) & 1)) return;
      tc_fence_after();
      if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
        for (int c0 = 0; c0 < kD; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_tm + c0, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st32(o_tm + c0, o);
        }
        tmem_wait_st();
      }
    }
    // P hi / lo, K-major 128-byte-swizzled rows: chunk q (keys 4q .. 4q + 3) at q ^ (t % 8)
#pragma unroll
    for (int q = 0; q < kKeys / 4; ++q) {
      float4 a, b;
      a.x = round_tf32(s[4 * q]);     b.x = round_tf32(s[4 * q] - a.x);
      a.y = round_tf32(s[4 * q + 1]); b.y = round_tf32(s[4 * q + 1] - a.y);
      a.z = round_tf32(s[4 * q + 2]); b.z = round_tf32(s[4 * q + 2] - a.z);
      a.w = round_tf32(s[4 * q + 3]); b.w = round_tf32(s[4 * q + 3] - a.w);
      const int off = (q ^ (t & 7)) * 16;
      *reinterpret_cast<float4*>(p_hi + off) = a;
      *reinterpret_cast<float4*>(p_lo + off) = b;
    }
    fence_proxy_async_smem();   // the tensor core reads P through the async proxy
    tc_fence_before();
    __syncwarp();
    if ((t & 31) == 0) mbar_arrive(&bars.p_full);
  }
  if (!wc.wait(&bars.pv_done, (n - 1) & 1)) return;
  tc_fence_after();
  const float inv_l = 1.f / l_run;
  float* O = p.O + (int64_t)it.b * p.o_sb + (int64_t)it.h * p.o_sh + (int64_t)row * p.o_ss;
#pragma unroll
  for (int c0 = 0; c0 < kD; c0 += 32) {
    uint32_t o[32];
    tmem_ld32(o_tm + c0, o);
    if (row < p.S) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(O + c0 + i) =
            make_float4(__uint_as_float(o[i]) * inv_l, __uint_as_float(o[i + 1]) * inv_l,
                        __uint_as_float(o[i + 2]) * inv_l, __uint_as_float(o[i + 3]) * inv_l);
    }
  }
  if (p.LSE != nullptr && row < p.S)
    p.LSE[((int64_t)it.b * p.H + it.h) * p.S + row] = (m_run + __log2f(l_run)) * 0.69314718055994531f;
}

__global__ void __launch_bounds__(kThreads, 1) fmha_f32x3_kernel(const F32x3Params p,
                                                                 const __grid_constant__ F32x3Maps maps) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BarsX3& bars = *reinterpret_cast<BarsX3*>(smem + kOffBar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(&bars.q_full, 1);
    mbar_init(&bars.s_full[0], 1);
    mbar_init(&bars.s_full[1], 1);
    mbar_init(&bars.p_full, 4);
    mbar_init(&bars.pv_done, 1);
    mbar_init(&bars.mma_done, 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    bars.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&maps.q_hi);
    prefetch_tmap(&maps.k_hi);
    prefetch_tmap(&maps.vt_hi);
  }
  if (warp == 5) tmem_alloc(&bars.tmem_base, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  WaitCtl wc{&bars.abort_flag, p.err, p.timeout_ns, 40 + warp};
  if (warp < 4) {
    x3_softmax(p, smem, bars, wc, tmem, tid);
  } else if (lane == 0) {
    if (warp == 4) x3_producer(p, maps, smem, bars, wc);
    else x3_mma(p, smem, bars, wc, tmem);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace

cudaError_t launch_f32x3_split(const float* x, int64_t sb, int64_t sh, int64_t ss, float* hi, float* lo, int B,
                               int H, int S, int num_sms, cudaStream_t stream) {
  const int64_t n4 = (int64_t)B * H * S * (kD / 4);
  int64_t blocks = (n4 + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  split_rows_kernel<<<(int)blocks, 256, 0, stream>>>(x, sb, sh, ss, hi, lo, B, H, S);
  return cudaGetLastError();
}

cudaError_t launch_f32x3_split_vt(const float* x, int64_t sb, int64_t sh, int64_t ss, float* hi, float* lo, int B,
                                  int H, int S, int S32, cudaStream_t stream) {
  if (B * H > 65535) return cudaErrorInvalidValue;
  const int tiles = (S32 / 32) * (kD / 32);
  dim3 grid(tiles < 64 ? tiles : 64, B * H);
  split_vt_kernel<<<grid, 256, 0, stream>>>(x, sb, sh, ss, hi, lo, B, H, S, S32);
  return cudaGetLastError();
}

cudaError_t launch_fmha_f32x3(const F32x3Params& p, const F32x3Maps& maps, cudaStream_t stream) {
  auto kern = fmha_f32x3_kernel;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
  if (e != cudaSuccess) return e;
  const int64_t grid = (int64_t)p.B * p.H * p.n_qtiles;
  if (grid <= 0 || grid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  kern<<<(unsigned)grid, kThreads, kSmemAlloc, stream>>>(p, maps);
  return cudaGetLastError();
}

}  // namespace bw
