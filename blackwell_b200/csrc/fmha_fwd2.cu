// GQA / MHA flash-attention forward for sm_100a, double-buffered-S variant.
//
// Same contract as fmha_fwd.cu (reference launchers launch_gqa_vN /
// gqa_causal / gqa_split, GQA_sm103.cu:5733-6516, GQA_sm103_causal_v3.cu:2156-2180,
// adhitya_GQA.cu:199-213) and the same CTA work items (two 128-row query blocks
// sharing one K/V stream), but K/V are streamed in 64-row tiles so that each
// softmax warpgroup owns TWO score buffers in tensor memory:
//
//   TMEM columns of warpgroup w (256 each):  S[0] (64) | S[1] (64) | O (D <= 128)
//
// With two S buffers the MMA thread computes S(j+1) = Q K(j+1)^T while the
// softmax works on S(j); P(j) (bf16, 32 columns) overwrites the first half of
// S(j)'s buffer and feeds the PV MMA from TMEM.  Per warpgroup the MMA order is
//   QK(0), QK(1), then for each tile j:  PV(j) [after P(j)], QK(j+2) [into
//   S(j)'s buffer, behind PV(j) in the in-order tcgen05 pipe]
// so the softmax of tile j+1 no longer waits for PV(j) + QK(j+1): the tensor
// core and the two warpgroups' exp work overlap.  A softmax that must rescale O
// (rare: only when its running max rises by more than 8 in log2 units) first
// waits for PV(j-1) through the pv_done barrier.
//
// Barriers with two phases in flight get one barrier per S buffer (s_full,
// p_full), so no waiter ever falls two phases behind a barrier.
#include "kernels.h"
#include "ptx.cuh"
#include "softmax_math.cuh"
#include "tmem_io.cuh"

namespace bw {
namespace {

constexpr int kQRows = 128;           // query rows per block
constexpr int kKRows = 64;            // keys per K/V tile
constexpr int kThreads2 = 320;        // 2 softmax warpgroups + producer warp + MMA warp
constexpr int kSmemBudget2 = 232448 - 2048;

template <int D>
struct Cfg2 {
  static constexpr int kQBytes = kQRows * D * 2;       // one Q block
  static constexpr int kQPanel = kQRows * 128;         // 64-column panel of a Q block
  static constexpr int kKVBytes = kKRows * D * 2;      // one K or V tile
  static constexpr int kKVPanel = kKRows * 128;        // 64-column panel of a K/V tile
  static constexpr int kKV = 2 * kQBytes;              // ring start
  static constexpr int kNSraw = (kSmemBudget2 - kKV) / kKVBytes;
  static constexpr int NS = kNSraw > 16 ? 16 : kNSraw;
  static constexpr int kBar = kKV + NS * kKVBytes;
  static constexpr int kBytes = kBar + 1024;
  static_assert(NS >= 6, "K/V ring needs at least 6 slots");
};

struct Bars2 {
  uint64_t q_full[2], q_empty[2], o_full[2], pv_done[2], mma_done;
  uint64_t s_full[2][2], p_full[2][2];   // [warpgroup][S buffer]
  uint64_t kv_full[16], kv_empty[16];
  uint32_t tmem_base;
  int abort_flag;
};

struct Item2 {
  int b, kvh;
  int head[2], qt[2], nkv[2];   // nkv: 64-row K/V tiles visited by each block
  int nmax;
};

__device__ __forceinline__ Item2 decode_item2(const FmhaParams& p, int idx) {
  Item2 it;
  int t0, t1;
  if (p.pair_heads) {
    const int hp = p.Hq >> 1;
    const int per_t = p.B * hp;
    int t = idx / per_t;
    const int r = idx - t * per_t;
    if (p.causal) t = p.n_qtiles - 1 - t;
    it.b = r / hp;
    const int h0 = 2 * (r - it.b * hp);
    it.head[0] = h0;
    it.head[1] = h0 + 1;
    t0 = t1 = t;
  } else {
    const int ntp = (p.n_qtiles + 1) >> 1;
    const int per_t = p.B * p.Hq;
    int tp = idx / per_t;
    const int r = idx - tp * per_t;
    if (p.causal) tp = ntp - 1 - tp;
    it.b = r / p.Hq;
    it.head[0] = it.head[1] = r - it.b * p.Hq;
    t0 = 2 * tp;
    t1 = 2 * tp + 1;
  }
  it.kvh = it.head[0] / p.G;
  it.qt[0] = t0;
  it.qt[1] = t1;
  const int n64 = (p.Skv + kKRows - 1) / kKRows;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const int t = it.qt[w];
    int n = 0;
    if (t < p.n_qtiles) n = p.causal ? min(2 * t + 2, n64) : n64;
    it.nkv[w] = n;
  }
  it.nmax = max(it.nkv[0], it.nkv[1]);
  return it;
}

__device__ __forceinline__ uint32_t pack_bf16_2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------------ producer warp
template <int D>
__device__ void producer2(const FmhaParams& p, const FmhaMaps& maps, uint8_t* smem, Bars2& bars, const WaitCtl& wc) {
  using C = Cfg2<D>;
  constexpr int NS = C::NS;
  constexpr int NPANEL = D / 64;
  uint32_t ld = 0;
  uint32_t qc[2] = {0, 0};
  bool ok = true;
  bool first_k = true;
  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item2 it = decode_item2(p, idx);
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      if (!ok || it.nkv[w] == 0) continue;
      if (!wc.wait(&bars.q_empty[w], (qc[w] & 1) ^ 1)) { ok = false; break; }
      mbar_arrive_expect_tx(&bars.q_full[w], C::kQBytes);
      uint8_t* dst = smem + w * C::kQBytes;
#pragma unroll
      for (int c = 0; c < NPANEL; ++c)
        tma_load_4d(dst + c * C::kQPanel, &maps.q, &bars.q_full[w], c * 64, it.qt[w] * kQRows, it.head[w], it.b);
      ++qc[w];
    }
    for (int j = 0; ok && j < it.nmax; ++j) {
#pragma unroll
      for (int kind = 0; kind < 2; ++kind) {
        const uint32_t slot = ld % NS;
        if (!wc.wait(&bars.kv_empty[slot], ((ld / NS) & 1) ^ 1)) { ok = false; break; }
        const bool withhold = kind == 0 && first_k && (p.debug_flags & 1);
        if (kind == 0) first_k = false;
        if (!withhold) {
          mbar_arrive_expect_tx(&bars.kv_full[slot], C::kKVBytes);
          uint8_t* dst = smem + C::kKV + slot * C::kKVBytes;
          const CUtensorMap* m = kind == 0 ? &maps.k : &maps.v;
#pragma unroll
          for (int c = 0; c < NPANEL; ++c)
            tma_load_4d(dst + c * C::kKVPanel, m, &bars.kv_full[slot], c * 64, j * kKRows, it.kvh, it.b);
        }
        ++ld;
      }
    }
  }
  if (!ok) {
    for (uint32_t i = (ld > NS ? ld - NS : 0); i < ld; ++i)
      drain_wait(&bars.kv_full[i % NS], (i / NS) & 1, wc.timeout_ns);
    for (int w = 0; w < 2; ++w)
      if (qc[w]) drain_wait(&bars.q_full[w], (qc[w] - 1) & 1, wc.timeout_ns);
  }
}

// ---------------------------------------------------------------- MMA warp
template <int D>
__device__ void mma2(const FmhaParams& p, uint8_t* smem, Bars2& bars, const WaitCtl& wc, uint32_t tmem) {
  using C = Cfg2<D>;
  constexpr int NS = C::NS;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, kKRows, false);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, D, true);
  constexpr uint32_t HI = sdesc_hi_sbo1024();
  const uint32_t smem_base = smem_u32(smem);
  const uint32_t q_lo0 = sdesc_lo(smem_base, 16);
  const uint32_t k_lo0 = sdesc_lo(smem_base + C::kKV, 16);
  const uint32_t v_lo0 = sdesc_lo(smem_base + C::kKV, C::kKVPanel);
  uint32_t ld = 0;
  uint32_t qc[2] = {0, 0};
  uint32_t pc[2][2] = {{0, 0}, {0, 0}};
  uint32_t mt[2] = {0, 0};   // tiles per warpgroup (trace index)
  bool ok = true;

  auto kv_wait = [&](uint32_t i) -> bool { return wc.wait(&bars.kv_full[i % NS], (i / NS) & 1); };
  auto issue_qk = [&](int w, uint32_t kslot, int buf) {
    const uint32_t qa = q_lo0 + (uint32_t)(w * C::kQBytes) / 16;
    const uint32_t ka = k_lo0 + kslot * (uint32_t)(C::kKVBytes / 16);
    const uint32_t d_tmem = tmem + w * 256 + buf * 64;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const uint32_t a_off = ((ks >> 2) * C::kQPanel + (ks & 3) * 32) / 16;
      const uint32_t b_off = ((ks >> 2) * C::kKVPanel + (ks & 3) * 32) / 16;
      mma_ss_lh(d_tmem, qa + a_off, HI, ka + b_off, HI, IDESC_QK, ks > 0);
    }
  };
  auto issue_pv = [&](int w, uint32_t vslot, int buf, bool acc) {
    const uint32_t va = v_lo0 + vslot * (uint32_t)(C::kKVBytes / 16);
    const uint32_t o_tmem = tmem + w * 256 + 128;
    const uint32_t p_tmem = tmem + w * 256 + buf * 64;
#pragma unroll
    for (int ks = 0; ks < kKRows / 16; ++ks)
      mma_ts_lh(o_tmem, p_tmem + ks * 8, va + (ks * 16 * 128) / 16, HI, IDESC_PV, (acc || ks > 0) ? 1u : 0u);
  };

  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item2 it = decode_item2(p, idx);
    for (int w = 0; w < 2 && ok; ++w) {
      if (it.nkv[w] == 0) continue;
      ok = wc.wait(&bars.q_full[w], qc[w] & 1);
      ++qc[w];
    }
    if (!ok) break;
    // prologue: S for tiles 0 and 1 into buffers 0 and 1
    for (int jj = 0; jj < 2 && jj < it.nmax; ++jj) {
      if (!kv_wait(ld + 2 * jj)) { ok = false; break; }
      tc_fence_after();
      for (int w = 0; w < 2; ++w) {
        if (jj >= it.nkv[w]) continue;
        issue_qk(w, (ld + 2 * jj) % NS, jj);
        tc_commit(&bars.s_full[w][jj]);
        if (jj == it.nkv[w] - 1) tc_commit(&bars.q_empty[w]);
      }
      tc_commit(&bars.kv_empty[(ld + 2 * jj) % NS]);
    }
    if (!ok) break;
    for (int j = 0; j < it.nmax; ++j) {
      const int b = j & 1;
      const uint32_t iv = ld + 2 * j + 1;
      const uint32_t ik = ld + 2 * (j + 2);
      const bool more = j + 2 < it.nmax;
      BW_TRACE_AT(true, 20, mt[0]);
      if (!kv_wait(iv)) { ok = false; break; }
      BW_TRACE_AT(true, 21, mt[0]);
      if (more && !kv_wait(ik)) { ok = false; break; }
      BW_TRACE_AT(true, 22, mt[0]);
      for (int w = 0; w < 2; ++w) {
        if (j < it.nkv[w]) {
          if (!wc.wait(&bars.p_full[w][b], pc[w][b] & 1)) { ok = false; break; }
          ++pc[w][b];
          tc_fence_after();
          BW_TRACE_AT(true, 50 + w, mt[w]);
          issue_pv(w, iv % NS, b, j > 0);
          BW_TRACE_AT(true, 55 + w, mt[w]);
          ++mt[w];
          tc_commit(&bars.pv_done[w]);
          if (j == it.nkv[w] - 1) tc_commit(&bars.o_full[w]);
        }
        if (j + 2 < it.nkv[w]) {
          issue_qk(w, ik % NS, b);
          tc_commit(&bars.s_full[w][b]);
          BW_TRACE_AT(true, 60 + w, mt[w] - 1);
          if (j + 3 == it.nkv[w]) tc_commit(&bars.q_empty[w]);
        }
      }
      if (!ok) break;
      tc_commit(&bars.kv_empty[iv % NS]);
      if (more) tc_commit(&bars.kv_empty[ik % NS]);
    }
    ld += 2 * it.nmax;
  }
  tc_commit(&bars.mma_done);
  drain_wait(&bars.mma_done, 0, wc.timeout_ns);
}

// ------------------------------------------------------ softmax warpgroups
template <int D, int POLY>
__device__ void softmax2(const FmhaParams& p, Bars2& bars, const WaitCtl& wc, uint32_t tmem, int w, int t) {
  const int wq = t >> 5;
  const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
  const uint32_t s_base = tmem + lane_off + w * 256;
  const uint32_t o_tmem = s_base + 128;
  const float c = p.scale_log2;
  uint32_t sc[2] = {0, 0}, oc = 0, gt = 0;

  for (int idx = blockIdx.x; idx < p.num_items; idx += gridDim.x) {
    const Item2 it = decode_item2(p, idx);
    const int n = it.nkv[w];
    if (n == 0) continue;
    const int row = it.qt[w] * kQRows + t;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < n; ++j, ++gt) {
      const int b = j & 1;
      if (!wc.wait(&bars.s_full[w][b], sc[b] & 1)) return;
      ++sc[b];
      tc_fence_after();
      BW_TRACE_AT(t == 0, 10 + w, gt);
      uint32_t r[64];
      tmem_ld64(s_base + b * 64, r);
      float* s = reinterpret_cast<float*>(r);
      const int kv0 = j * kKRows;
      const bool diag = p.causal && (kv0 + kKRows - 1 > it.qt[w] * kQRows);
      if (diag || kv0 + kKRows > p.Skv) {
        int lim = p.Skv - kv0;
        if (p.causal) lim = min(lim, row + 1 - kv0);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= lim) s[i] = -INFINITY;
      }
      float mx;
      {
        float a[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = fmaxf(s[u], s[8 + u]);
#pragma unroll
        for (int i = 16; i < 64; i += 16)
#pragma unroll
          for (int u = 0; u < 8; ++u) a[u] = fmax3(a[u], s[i + u], s[i + 8 + u]);
        mx = fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
      }
      const float m_cand = mx * c;
      float corr = 1.f;
      const bool upd = m_cand > m_run + 8.f;
      if (upd) {
        corr = ex2_mufu(m_run - m_cand);
        m_run = m_cand;
      }
      const float msub = (m_run == -INFINITY) ? 0.f : m_run;
      const f2 cc2{c, c}, nm2{-msub, -msub};
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const f2 x = ffma2(f2{s[2 * k], s[2 * k + 1]}, cc2, nm2);
        s[2 * k] = x.x;
        s[2 * k + 1] = x.y;
      }
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        if ((k & 7) < POLY) {
          const f2 e = ex2_poly2(f2{s[2 * k], s[2 * k + 1]});
          s[2 * k] = e.x;
          s[2 * k + 1] = e.y;
        } else {
          s[2 * k] = ex2_mufu(s[2 * k]);
          s[2 * k + 1] = ex2_mufu(s[2 * k + 1]);
        }
      }
      f2 acc0{0.f, 0.f}, acc1{0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        acc0 = fadd2(acc0, f2{s[2 * k], s[2 * k + 1]});
        acc1 = fadd2(acc1, f2{s[2 * k + 2], s[2 * k + 3]});
      }
      uint32_t pk[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) pk[k] = pack_bf16_2(s[2 * k], s[2 * k + 1]);
      acc0 = fadd2(acc0, acc1);
      l_run = l_run * corr + (acc0.x + acc0.y);
      BW_TRACE_AT(t == 0, 30 + w, gt);
      tmem_st32(s_base + b * 64, pk);   // P(j) over the first 32 columns of its S buffer
      if (j > 0 && __any_sync(0xffffffffu, upd)) {
        // O must hold PV(j-1) before it is rescaled
        if (!wc.wait(&bars.pv_done[w], (gt - 1) & 1)) return;
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_tmem + c0, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st32(o_tmem + c0, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars.p_full[w][b]);
      BW_TRACE_AT(t == 0, 40 + w, gt);
    }
    if (!wc.wait(&bars.o_full[w], oc & 1)) return;
    ++oc;
    tc_fence_after();
    const float inv_l = 1.f / l_run;
    const int h = it.head[w];
    __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.O) + it.b * p.o_sb + h * p.o_sh + (int64_t)row * p.o_ss;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t o[32];
      tmem_ld32(o_tmem + c0, o);
      uint32_t q[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        q[i] = pack_bf16_2(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
      if (row < p.Sq) {
        uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(q[4 * i], q[4 * i + 1], q[4 * i + 2], q[4 * i + 3]);
      }
    }
    if (p.LSE != nullptr && row < p.Sq)
      p.LSE[((int64_t)it.b * p.Hq + h) * p.lse_sh + row] = (m_run + __log2f(l_run)) * 0.69314718055994531f;
    tc_fence_before();
  }
}

template <int D, int POLY>
__global__ void __launch_bounds__(kThreads2, 1)
    fmha_fwd2_kernel(const FmhaParams p, const __grid_constant__ FmhaMaps maps) {
  using C = Cfg2<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars2& bars = *reinterpret_cast<Bars2*>(smem + C::kBar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bars.q_full[w], 1);
      mbar_init(&bars.q_empty[w], 1);
      mbar_init(&bars.o_full[w], 1);
      mbar_init(&bars.pv_done[w], 1);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&bars.s_full[w][b], 1);
        mbar_init(&bars.p_full[w][b], 128);
      }
    }
    mbar_init(&bars.mma_done, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    bars.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    prefetch_tmap(&maps.q);
    prefetch_tmap(&maps.k);
    prefetch_tmap(&maps.v);
  }
  if (warp == 9) tmem_alloc(&bars.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  WaitCtl wc{&bars.abort_flag, p.err, p.timeout_ns, warp};
  if (warp < 8) {
    softmax2<D, POLY>(p, bars, wc, tmem, warp >> 2, tid & 127);
  } else if (warp == 8) {
    if (lane == 0) producer2<D>(p, maps, smem, bars, wc);
  } else {
    if (lane == 0) mma2<D>(p, smem, bars, wc, tmem);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, int POLY>
cudaError_t launch2_impl(const FmhaParams& p, const FmhaMaps& maps, int num_sms, cudaStream_t stream) {
  constexpr int bytes = Cfg2<D>::kBytes + 1024;
  auto kern = fmha_fwd2_kernel<D, POLY>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  const int grid = p.num_items < num_sms ? p.num_items : num_sms;
  kern<<<grid, kThreads2, bytes, stream>>>(p, maps);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch2_poly(const FmhaParams& p, const FmhaMaps& maps, int poly, int num_sms, cudaStream_t stream) {
  switch (poly) {
    case 0: return launch2_impl<D, 0>(p, maps, num_sms, stream);
    case 2: return launch2_impl<D, 2>(p, maps, num_sms, stream);
    case 3: return launch2_impl<D, 3>(p, maps, num_sms, stream);
    case 4: return launch2_impl<D, 4>(p, maps, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_fmha_fwd2(const FmhaParams& p, const FmhaMaps& maps, int exp_poly, int num_sms,
                             cudaStream_t stream) {
  if (p.D == 128) return launch2_poly<128>(p, maps, exp_poly, num_sms, stream);
  if (p.D == 64) return launch2_poly<64>(p, maps, exp_poly, num_sms, stream);
  return cudaErrorInvalidValue;
}

}  // namespace bw

#ifdef BW_TRACE
extern "C" __attribute__((visibility("default"))) int bw_trace2_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, g_bw_trace, sizeof(g_bw_trace));
  return 64 * 512;
}
#endif
