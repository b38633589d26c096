// GQA / MHA flash-attention forward for sm_100a.
//
// Computes, per query row i of head hq (KV head hkv = hq / G):
//     O[i]   = softmax(scale * Q[i] K^T) V          (bf16 out, fp32 math)
//     LSE[i] = ln sum_j exp(scale * Q[i].K[j])       (fp32, natural log)
// with an optional causal mask (key j visible iff j <= i).  This is the
// behaviour of the reference's launch_gqa_vN / gqa_causal launchers
// (src/SM103/attention/GQA_sm103.cu:5733-6516, GQA_sm103_causal_v3.cu:2156-2180)
// and the split-length launcher (src/SM120/attention/adhitya_GQA.cu:199-213).
//
// Design (one persistent CTA per SM, 10 warps):
//   warps 0-3  softmax warpgroup 0 -> query block 0 (128 rows, one row per thread)
//   warps 4-7  softmax warpgroup 1 -> query block 1
//   warp  8    TMA producer: Q blocks, then a K/V ring of NS 128-row tiles
//   warp  9    tcgen05 MMA issuer (one thread) and TMEM owner
// The two query blocks of a work item share one K/V stream: either two query
// heads of the same KV group at the same rows (GQA, G even) or two adjacent
// 128-row tiles of one head.  Tensor memory (512 columns) holds
//   S0 | S1 (128 fp32 columns each) | O0 | O1 (D columns each);
// the softmax writes P as packed bf16 over the first 64 columns of its S block and
// the P*V MMA reads A straight from TMEM (or, in the P-in-shared-memory variant,
// from a 128B-swizzled shared tile).  The two warpgroups ping-pong: while one
// runs exp2 the tensor core works on the other's QK^T / PV.
//
// Online softmax works in the log2 domain: s' = s * scale * log2(e) folded into
// one FFMA, p = 2^(s' - m).  The running max m is only raised when the new tile
// max exceeds it by more than 8 (a factor 256), as in FlashAttention-4; the O
// rescale in TMEM is skipped otherwise.  Values of p stay <= 256, well within
// bf16/fp32 range, and the final O / l and LSE = ln2 * (m + log2 l) are exact
// for whichever m was used.
#include "kernels.h"
#include "ptx.cuh"
#include "softmax_math.cuh"
#include "tmem_io.cuh"

namespace bw {
namespace {

constexpr int kRows = 128;          // query rows per block == KV rows per tile
constexpr int kSmemBudget = 232448 - 2048;

template <int D>
struct Cfg {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileBytes = kRows * kRowBytes;      // one 128-row tile
  static constexpr int kSub = kRows * 128;                  // one 128-byte swizzle panel
  static constexpr int kPanels = kRowBytes / 128;
  static constexpr int kPanelElems = 64;                    // elements per panel row
  static constexpr int kPBytes = kRows * kRows * 2;         // P tile (smem variant)
  static constexpr int kKStep = 16;                         // MMA K per instruction (32 bytes)
};

template <int D, bool PT>
struct Layout {
  static constexpr int kQ = 0;
  static constexpr int kP = 2 * Cfg<D>::kTileBytes;
  static constexpr int kKV = kP + (PT ? 0 : 2 * Cfg<D>::kPBytes);
  static constexpr int kNSraw = (kSmemBudget - kKV) / Cfg<D>::kTileBytes;
  static constexpr int NS = kNSraw > 8 ? 8 : kNSraw;
  static constexpr int kBar = kKV + NS * Cfg<D>::kTileBytes;
  static constexpr int kBytes = kBar + 512;
  static_assert(NS >= 3, "K/V ring needs at least 3 slots");
};

struct Bars {
  uint64_t q_full[2], q_empty[2], s_full[2], p_full[2], o_full[2], mma_done;
  uint64_t kv_full[8], kv_empty[8];
  uint32_t tmem_base;
  int abort_flag;
};

struct Item {
  int b, kvh;
  int head[2], qt[2], nkv[2];
  int nmax;
};

__device__ __forceinline__ Item decode_item(const FmhaParams& p, int idx) {
  Item it;
  int t0, t1;
  if (p.pair_heads) {
    const int hp = p.Hq >> 1;
    const int per_t = p.B * hp;
    int t = idx / per_t;
    const int r = idx - t * per_t;
    if (p.causal) t = p.n_qtiles - 1 - t;  // heaviest query tiles first
    it.b = r / hp;
    const int h0 = 2 * (r - it.b * hp);
    it.head[0] = h0;
    it.head[1] = h0 + 1;
    t0 = t1 = t;
  } else {
    const int ntp = (p.n_qtiles + 1) >> 1;
    const int per_t = p.B * p.Hq;
    int tp, r;
    if (p.causal) {
      tp = idx / per_t;
      r = idx - tp * per_t;
      tp = ntp - 1 - tp;  // heaviest query tiles first
    } else {
      // head-major: the CTAs running at once share a few heads' K / V in L2
      r = idx / ntp;
      tp = idx - r * ntp;
    }
    it.b = r / p.Hq;
    it.head[0] = it.head[1] = r - it.b * p.Hq;
    t0 = 2 * tp;
    t1 = 2 * tp + 1;
  }
  it.kvh = it.head[0] / p.G;
  it.qt[0] = t0;
  it.qt[1] = t1;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const int t = it.qt[w];
    int n = 0;
    if (t < p.n_qtiles) n = p.causal ? min((p.q_offset + t * kRows + kRows - 1) / kRows + 1, p.n_kvtiles) : p.n_kvtiles;
    it.nkv[w] = n;
  }
  it.nmax = max(it.nkv[0], it.nkv[1]);
  return it;
}

// ------------------------------------------------------------ producer warp
template <int D, bool PT>
__device__ void producer_role(const FmhaParams& p, const FmhaMaps& maps, uint8_t* smem, Bars& bars,
                              const WaitCtl& wc) {
  using L = Layout<D, PT>;
  constexpr int NS = L::NS;
  constexpr int TB = Cfg<D>::kTileBytes;
  constexpr int NPANEL = Cfg<D>::kPanels;
  constexpr int PE = Cfg<D>::kPanelElems;
  uint32_t ld = 0;                 // K/V loads issued (ring position)
  uint32_t qc[2] = {0, 0};
  uint32_t armed = 0;              // bit s: slot s has a load whose completion is pending/known
  bool ok = true;
  bool first_k = true;
  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item it = decode_item(p, idx);
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      if (!ok || it.nkv[w] == 0) continue;
      if (!wc.wait(&bars.q_empty[w], (qc[w] & 1) ^ 1)) { ok = false; break; }
      mbar_arrive_expect_tx(&bars.q_full[w], TB);
      uint8_t* dst = smem + L::kQ + w * TB;
#pragma unroll
      for (int c = 0; c < NPANEL; ++c)
        tma_load_4d(dst + c * Cfg<D>::kSub, &maps.q, &bars.q_full[w], c * PE, it.qt[w] * kRows, it.head[w], it.b);
      ++qc[w];
    }
    for (int j = 0; ok && j < it.nmax; ++j) {
#pragma unroll
      for (int kind = 0; kind < 2; ++kind) {
        const uint32_t slot = ld % NS;
        const uint32_t ph = (ld / NS) & 1;
        BW_TRACE_AT(true, 23, ld);
        if (!wc.wait(&bars.kv_empty[slot], ph ^ 1)) { ok = false; break; }
        BW_TRACE_AT(true, 24, ld);
        const bool withhold = kind == 0 && first_k && (p.debug_flags & 1);
        if (kind == 0) first_k = false;
        if (!withhold) {
          const int np = NPANEL;
          const int pe = PE;
          mbar_arrive_expect_tx(&bars.kv_full[slot], TB);
          uint8_t* dst = smem + L::kKV + slot * TB;
          const CUtensorMap* m = kind == 0 ? &maps.k : &maps.v;
          for (int c = 0; c < np; ++c)
            tma_load_4d(dst + c * Cfg<D>::kSub, m, &bars.kv_full[slot], c * pe, j * kRows, it.kvh, it.b);
          armed |= 1u << slot;
        } else {
          armed &= ~(1u << slot);
        }
        ++ld;
      }
    }
  }
  if (!ok) {
    // Wait for every load this warp issued before the CTA releases its memory.
    for (uint32_t i = (ld > NS ? ld - NS : 0); i < ld; ++i) {
      const uint32_t slot = i % NS;
      if (armed & (1u << slot)) drain_wait(&bars.kv_full[slot], (i / NS) & 1, wc.timeout_ns);
    }
    for (int w = 0; w < 2; ++w)
      if (qc[w]) drain_wait(&bars.q_full[w], (qc[w] - 1) & 1, wc.timeout_ns);
  }
}

// ---------------------------------------------------------------- MMA warp
// One thread issues every tcgen05.mma.  Order per work item (w = 0, 1):
//   QK_w(0) ... then for each KV tile j:  PV_w(j), QK_w(j+1)
// tcgen05 operations from one thread execute in issue order, so the commit that
// signals S_w(j+1) ready also guarantees PV_w(j) has finished reading P_w(j)
// (which shares S_w's columns) and that O_w is stable for the softmax's rescale.
template <int D, bool PT>
__device__ void mma_role(const FmhaParams& p, uint8_t* smem, Bars& bars, const WaitCtl& wc, uint32_t tmem) {
  using L = Layout<D, PT>;
  constexpr int NS = L::NS;
  constexpr int TB = Cfg<D>::kTileBytes;
  constexpr int SUB = Cfg<D>::kSub;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 128, false);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, D, true);
  constexpr int KS = Cfg<D>::kKStep;
  const uint32_t smem_base = smem_u32(smem);
  uint32_t ld = 0;
  uint32_t qc[2] = {0, 0}, pc[2] = {0, 0};
  bool ok = true;

  auto kv_wait = [&](uint32_t i) -> bool { return wc.wait(&bars.kv_full[i % NS], (i / NS) & 1); };
  // Descriptor low halves of the tile bases, computed once; each K-step adds
  // its byte offset / 16.
  constexpr uint32_t HI = sdesc_hi_sbo1024();
  const uint32_t q_lo0 = sdesc_lo(smem_base + L::kQ, 16);
  const uint32_t kv_lo_k0 = sdesc_lo(smem_base + L::kKV, 16);       // K operand (K-major)
  const uint32_t kv_lo_v0 = sdesc_lo(smem_base + L::kKV, SUB);      // V operand (MN-major)
  const uint32_t p_lo0 = sdesc_lo(smem_base + L::kP, 16);
  auto issue_qk = [&](int w, uint32_t kslot) {
    const uint32_t qa = q_lo0 + (uint32_t)(w * TB) / 16;
    const uint32_t ka = kv_lo_k0 + kslot * (uint32_t)(TB / 16);
    const uint32_t d_tmem = tmem + w * 128;
#pragma unroll
    for (int ks = 0; ks < D / KS; ++ks) {
      const uint32_t off = ((ks >> 2) * SUB + (ks & 3) * 32) / 16;
      mma_ss_lh(d_tmem, qa + off, HI, ka + off, HI, IDESC_QK, ks > 0);
    }
  };
  auto issue_pv = [&](int w, uint32_t vslot, bool acc) {
    const uint32_t va = kv_lo_v0 + vslot * (uint32_t)(TB / 16);
    const uint32_t o_tmem = tmem + 256 + w * D;
    const uint32_t acc0 = acc ? 1u : 0u;
#pragma unroll
    for (int ks = 0; ks < kRows / 16; ++ks) {
      const uint32_t b_lo = va + (ks * 16 * 128) / 16;
      if constexpr (PT) {
        mma_ts_lh(o_tmem, tmem + w * 128 + ks * 8, b_lo, HI, IDESC_PV, ks > 0 ? 1u : acc0);
      } else {
        const uint32_t pa = p_lo0 + (uint32_t)(w * Cfg<D>::kPBytes) / 16 + ((ks >> 2) * SUB + (ks & 3) * 32) / 16;
        mma_ss_lh(o_tmem, pa, HI, b_lo, HI, IDESC_PV, ks > 0 ? 1u : acc0);
      }
    }
  };

  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item it = decode_item(p, idx);
    for (int w = 0; w < 2 && ok; ++w) {
      if (it.nkv[w] == 0) continue;
      ok = wc.wait(&bars.q_full[w], qc[w] & 1);
      ++qc[w];
    }
    if (!ok) break;
    if (!kv_wait(ld)) { ok = false; break; }
    tc_fence_after();
    for (int w = 0; w < 2; ++w) {
      if (it.nkv[w] == 0) continue;
      issue_qk(w, ld % NS);
      tc_commit(&bars.s_full[w]);
      if (it.nkv[w] == 1) tc_commit(&bars.q_empty[w]);
    }
    tc_commit(&bars.kv_empty[ld % NS]);
    for (int j = 0; j < it.nmax; ++j) {
      const uint32_t iv = ld + 2 * j + 1;
      const uint32_t ik = ld + 2 * j + 2;
      const bool next = j + 1 < it.nmax;
      BW_TRACE_AT(true, 20, pc[0]);
      if (!kv_wait(iv)) { ok = false; break; }
      BW_TRACE_AT(true, 21, pc[0]);
      if (next && !kv_wait(ik)) { ok = false; break; }
      BW_TRACE_AT(true, 22, pc[0]);
      for (int w = 0; w < 2; ++w) {
        if (j < it.nkv[w]) {
          if (!wc.wait(&bars.p_full[w], pc[w] & 1)) { ok = false; break; }
          ++pc[w];
          tc_fence_after();
          BW_TRACE_AT(true, 50 + w, pc[w] - 1);
          issue_pv(w, iv % NS, j > 0);
          BW_TRACE_AT(true, 55 + w, pc[w] - 1);
          if (j == it.nkv[w] - 1) tc_commit(&bars.o_full[w]);
        }
        if (j + 1 < it.nkv[w]) {
          issue_qk(w, ik % NS);
          tc_commit(&bars.s_full[w]);
          BW_TRACE_AT(true, 60 + w, pc[w] - 1);
          if (j + 2 == it.nkv[w]) tc_commit(&bars.q_empty[w]);
        }
      }
      if (!ok) break;
      tc_commit(&bars.kv_empty[iv % NS]);
      if (next) tc_commit(&bars.kv_empty[ik % NS]);
    }
    ld += 2 * it.nmax;
  }
  // Whether finished or unwinding: wait until every MMA issued here is complete
  // before TMEM can be released.
  tc_commit(&bars.mma_done);
  drain_wait(&bars.mma_done, 0, wc.timeout_ns);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ----------------------------------------------------------- softmax warpgroups
// Thread t of warpgroup w owns query row t of block w (TMEM lane t).
template <int D, bool PT, int POLY>
__device__ void softmax_role(const FmhaParams& p, uint8_t* smem, Bars& bars, const WaitCtl& wc, uint32_t tmem,
                             int w, int t) {
  using L = Layout<D, PT>;
  const int wq = t >> 5;                                 // warp within warpgroup -> lane quarter
  const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
  const uint32_t s_tmem = tmem + lane_off + w * 128;
  const uint32_t o_tmem = tmem + lane_off + 256 + w * D;
  const float c = p.scale_log2;
  uint32_t sc = 0, oc = 0;
  uint8_t* p_smem = smem + L::kP + w * Cfg<D>::kPBytes;

  for (int idx = blockIdx.x; idx < p.num_items; idx += gridDim.x) {
    const Item it = decode_item(p, idx);
    const int n = it.nkv[w];
    if (n == 0) continue;
    const int row = it.qt[w] * kRows + t;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < n; ++j) {
      if (!wc.wait(&bars.s_full[w], sc & 1)) return;
      ++sc;
      tc_fence_after();
      BW_TRACE_AT(t == 0, 10 + w, sc - 1);
      uint32_t r[128];
      tmem_ld128(s_tmem, r);
      float* s = reinterpret_cast<float*>(r);
      const int kv0 = j * kRows;
      const bool diag = p.causal && (kv0 + kRows - 1 > p.q_offset + it.qt[w] * kRows);
      if (diag || kv0 + kRows > p.Skv) {
        int lim = p.Skv - kv0;
        if (p.causal) lim = min(lim, p.q_offset + row + 1 - kv0);
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= lim) s[i] = -INFINITY;
      }
      // Row max: eight independent three-input max chains.
      float mx;
      {
        float a[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = fmaxf(s[u], s[8 + u]);
#pragma unroll
        for (int i = 16; i < 128; i += 16)
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
      // Argument, exponential (POLY of every 8 pairs on the FMA pipe, the rest on
      // MUFU) and row sum per pair in one pass, so the scheduler can overlap the
      // FMA/ALU work with the MUFU stream.
      f2 acc0{0.f, 0.f}, acc1{0.f, 0.f}, acc2{0.f, 0.f}, acc3{0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        const f2 x = ffma2(f2{s[2 * k], s[2 * k + 1]}, cc2, nm2);
        f2 e;
        if ((k & 7) < POLY) {
          e = ex2_poly2(x);
        } else {
          e.x = ex2_mufu(x.x);
          e.y = ex2_mufu(x.y);
        }
        s[2 * k] = e.x;
        s[2 * k + 1] = e.y;
        if constexpr (PT) {
          // first half of P (key columns 0..63 -> TMEM columns 0..31) goes out
          // while the second half is still being exponentiated
          if (k == 31) {
            uint32_t pk0[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) pk0[i] = pack_bf16(s[2 * i], s[2 * i + 1]);
            tmem_st32(s_tmem, pk0);
          }
        }
        if ((k & 3) == 0) acc0 = fadd2(acc0, e);
        else if ((k & 3) == 1) acc1 = fadd2(acc1, e);
        else if ((k & 3) == 2) acc2 = fadd2(acc2, e);
        else acc3 = fadd2(acc3, e);
      }
      acc0 = fadd2(fadd2(acc0, acc1), fadd2(acc2, acc3));
      l_run = l_run * corr + (acc0.x + acc0.y);
      BW_TRACE_AT(t == 0, 30 + w, sc - 1);
      if constexpr (PT) {
        uint32_t pk[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) pk[k] = pack_bf16(s[64 + 2 * k], s[64 + 2 * k + 1]);
        tmem_st32(s_tmem + 32, pk);
      } else {
        uint32_t pk[64];
#pragma unroll
        for (int k = 0; k < 64; ++k) pk[k] = pack_bf16(s[2 * k], s[2 * k + 1]);
        // 128B-swizzled K-major tile: panel k/64, row t, 16B chunk (k%64)/8 ^ (t%8)
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const int panel = ch >> 3, cc = ch & 7;
          uint4 v = make_uint4(pk[ch * 4], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
          *reinterpret_cast<uint4*>(p_smem + panel * Cfg<D>::kSub + t * 128 + ((cc ^ (t & 7)) << 4)) = v;
        }
      }
      if (j > 0 && __any_sync(0xffffffffu, upd)) {
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
      if constexpr (!PT) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&bars.p_full[w]);
      BW_TRACE_AT(t == 0, 40 + w, sc - 1);
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
        q[i] = pack_bf16(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
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

struct Roles {
  static constexpr int kSoftThreads = 128;   // per warpgroup
  static constexpr int kProducerWarp = 2 * kSoftThreads / 32;
  static constexpr int kMmaWarp = kProducerWarp + 1;
  static constexpr int kThreads = 32 * (kMmaWarp + 1);
};

template <int D, bool PT, int POLY>
__global__ void __launch_bounds__(Roles::kThreads, 1)
    fmha_fwd_kernel(const FmhaParams p, const __grid_constant__ FmhaMaps maps) {
  using L = Layout<D, PT>;
  using R = Roles;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBar);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bars.q_full[w], 1);
      mbar_init(&bars.q_empty[w], 1);
      mbar_init(&bars.s_full[w], 1);
      mbar_init(&bars.p_full[w], R::kSoftThreads);
      mbar_init(&bars.o_full[w], 1);
    }
    mbar_init(&bars.mma_done, 1);
    for (int s = 0; s < L::NS; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    bars.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == R::kProducerWarp && lane == 0) {
    prefetch_tmap(&maps.q);
    prefetch_tmap(&maps.k);
    prefetch_tmap(&maps.v);
  }
  if (warp == R::kMmaWarp) tmem_alloc(&bars.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  WaitCtl wc{&bars.abort_flag, p.err, p.timeout_ns, warp};

  if (warp < R::kProducerWarp) {
    const int w = tid / R::kSoftThreads;
    softmax_role<D, PT, POLY>(p, smem, bars, wc, tmem, w, tid % R::kSoftThreads);
  } else if (warp == R::kProducerWarp) {
    if (lane == 0) producer_role<D, PT>(p, maps, smem, bars, wc);
  } else {
    if (lane == 0) mma_role<D, PT>(p, smem, bars, wc, tmem);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == R::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool PT, int POLY>
cudaError_t launch_impl(const FmhaParams& p, const FmhaMaps& maps, int num_sms, cudaStream_t stream) {
  constexpr int bytes = Layout<D, PT>::kBytes + 1024;
  constexpr int kThreads = Roles::kThreads;
  auto kern = fmha_fwd_kernel<D, PT, POLY>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  const int grid = p.num_items < num_sms ? p.num_items : num_sms;
  kern<<<grid, kThreads, bytes, stream>>>(p, maps);
  return cudaGetLastError();
}

template <int D, bool PT>
cudaError_t launch_poly(const FmhaParams& p, const FmhaMaps& maps, int poly, int num_sms, cudaStream_t stream) {
  switch (poly) {
    case 0: return launch_impl<D, PT, 0>(p, maps, num_sms, stream);
    case 2: return launch_impl<D, PT, 2>(p, maps, num_sms, stream);
    case 3: return launch_impl<D, PT, 3>(p, maps, num_sms, stream);
    case 4: return launch_impl<D, PT, 4>(p, maps, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_fmha_fwd(const FmhaParams& p, const FmhaMaps& maps, bool p_in_tmem, int exp_poly, int num_sms,
                            cudaStream_t stream) {
  if (p.D == 128) return p_in_tmem ? launch_poly<128, true>(p, maps, exp_poly, num_sms, stream)
                                   : launch_poly<128, false>(p, maps, exp_poly, num_sms, stream);
  if (p.D == 64) return p_in_tmem ? launch_poly<64, true>(p, maps, exp_poly, num_sms, stream)
                                  : launch_poly<64, false>(p, maps, exp_poly, num_sms, stream);
  return cudaErrorInvalidValue;
}

}  // namespace bw

#ifdef BW_TRACE
extern "C" __attribute__((visibility("default"))) int bw_trace_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, g_bw_trace, sizeof(g_bw_trace));
  return 64 * 512;
}
#endif
