// GQA / MHA flash-attention forward for sm_100a, one query tile per work item:
// kernel 4 (three score buffers, one O accumulator; the default at D = 128) and
// kernel 5 (D = 64: three score buffers, two O accumulators owned by the two
// softmax warpgroups in turn), the same roles and pipeline otherwise.
//
// Operator (per query row i of head hq, KV head hq / G):
//   O[i] = softmax(scale * Q[i] K^T) V,  LSE[i] = ln sum_j exp(scale * Q[i].K[j]),
// optional causal mask j <= q_offset + i; the behaviour of the reference's
// launch_gqa_vN / gqa_causal launchers (src/SM103/attention/GQA_sm103.cu:5733-6516,
// GQA_sm103_causal_v3.cu:2156-2180) and the split-length launcher
// (src/SM120/attention/adhitya_GQA.cu:199-213).
//
// Design (one persistent CTA per SM, four warpgroups):
//   warps 0 .. 7     softmax: one 128-row query tile (two warpgroups)
//   warps 8 .. 11    epilogue: row r of each finished tile (O / L, LSE; kernel
//                    5 first merges its two accumulators)
//   warp 12          TMA producer: the Q tile, then K and V tiles in MMA order
//   warp 13          PV MMA issuer (one thread) and TMEM owner
//   warp 14          QK^T MMA issuer (one thread); warp 15 idle
// Tensor memory: S_0 | S_1 | S_2 (128 fp32 columns each) | O (D columns;
// kernel 5: O_0 | O_1).  Global key tile g (counted over all items of the
// CTA) uses score buffer g % 3; the softmax writes its P (bf16) over the first
// 64 columns of that buffer, and the PV MMA reads it from there (TS form).
// MMA order per item of n key tiles:
//   QK(0), QK(1), then for each j: PV(j), QK(j + 2)   (two issuing threads)
// so while the softmax works on tile j the tensor core runs PV(j - 1) and
// QK(j + 1) is already waiting in another buffer: the softmax of one tile
// overlaps the MMAs of its neighbours instead of waiting for them.  The
// epilogue warpgroup takes the end of a tile (O read, division, store) off the
// softmax warps, which go from a tile's last key tile straight to the next
// tile's first.
//
// Online softmax in the log2 domain with the FlashAttention-4 lazy rescale
// (running max raised only when a tile's max exceeds it by more than 8).
#include "kernels.h"
#include "ptx.cuh"
#include "softmax_math.cuh"
#include "tmem_io.cuh"

namespace bw {
namespace {

constexpr int kRows = 128;
// The dynamic shared memory window is requested 512 bytes larger than the
// layout, for the round-up of its base to 1024 bytes (the kernel checks it).
constexpr int kAlignSlack = 512;
constexpr int kSmemBudget = 232448 - kAlignSlack;
constexpr int kMaxSlots = 12;

// Kernel 4 (V = 4): one accumulator O and three score buffers (TMEM S_0 | S_1
// | S_2 | O, 3 x 128 + D <= 512 columns), so that QK(g + 1) never waits for
// PV(g - 1): each softmax warp covers 16 rows of its TMEM lane quadrant
// through the 16-lane access shapes, four threads per row and two rows per
// thread, and the four threads of a row share one running max (two shuffles
// per row and tile), so all keys of a row accumulate into the same O.
// Kernel 5 (V = 5, D = 64): the same three buffers and two accumulators
// O_0 | O_1 (3 x 128 + 2 x 64 = 512 columns); see softmax5.
template <int D, int V>
struct Split {
  static_assert(V == 4 || (V == 5 && D == 64), "kernel 4 (D = 64, 128) or kernel 5 (D = 64)");
  static constexpr int N = 2;                      // softmax warpgroups
  static constexpr int NACC = V == 5 ? 2 : 1;      // O accumulators
  static constexpr int NB = 3;                     // score buffers
  static constexpr int kOCol = NB * 128;           // first TMEM column of O_0
  // softmax (4 N warps), output epilogue (4 warps), producer / PV issuer /
  // QK issuer (+ one idle warp): four warpgroups for the register split
  static constexpr int kThreads = 512;
  static_assert(N == 2, "warpgroup roles assume two softmax warpgroups");
  static_assert(kOCol + NACC * D <= 512, "TMEM: score buffers and accumulators");
};

template <int D>
struct L3 {
  static constexpr int kTile = kRows * D * 2;   // one 128-row bf16 tile
  static constexpr int kSub = kRows * 128;      // one 128-byte swizzle panel
  static constexpr int kPanels = D / 64;
  static constexpr int kQ = 0;                  // two Q slots: the next segment's tile loads during this one
  static constexpr int kKV = 2 * kTile;
  static constexpr int kXBytes = 2 * kRows * 8;   // (m, l) per row and accumulator: [2][128] float2
  // output staging: each epilogue warp's 32 rows x D columns as D / 64
  // panels of 32 x 128 bytes in the 128-byte-swizzled layout of the O tensor
  // map (one TMA store per panel)
  static constexpr int kStgWarp = 32 * D * 2;
  static constexpr int kNSraw = (kSmemBudget - kKV - kTile - 512 - kXBytes) / kTile;
  static constexpr int NS = kNSraw > kMaxSlots ? kMaxSlots : kNSraw;
  static constexpr int kStg = kKV + NS * kTile;
  static constexpr int kBar = kStg + kTile;
  static constexpr int kX = kBar + 512;
  static constexpr int kBytes = kX + kXBytes;
  static_assert(NS >= 4, "K/V ring needs at least 4 slots");
  static_assert(kBytes + kAlignSlack <= 232448, "shared memory");
  static_assert(kStgWarp * 4 == kTile, "staging = one tile");
};

struct Bars3 {
  uint64_t q_full[2], q_empty[2], s_full[3], p_full[3], pv_done[3], o_full, o_empty, mma_done, qk_done;
  uint64_t xch_full, xch_empty;
  uint64_t kv_full[kMaxSlots], kv_empty[kMaxSlots];
  uint32_t tmem_base;
  int abort_flag;
};

// A work item is one (b, hq) head and one query tile (non-causal) or the
// pair of query tiles (nqt - 1 - p, p) (causal: nqt + 1 key tiles in total
// whatever p, so items weigh the same).  Items are numbered head-major, so the
// CTAs running at any moment work on a few neighbouring heads and the K / V
// tiles they share stay in L2 (query-tile-major order made 148 concurrent CTAs
// stream 148 different heads and re-read K / V from DRAM about six times).
struct Item3 {
  int b, h, kvh, nseg;
  int qt[2], n[2];
};

__device__ __forceinline__ Item3 decode_item3(const FmhaParams& p, int idx) {
  Item3 it;
  const int per_head = p.causal ? (p.n_qtiles + 1) >> 1 : p.n_qtiles;
  const int r = idx / per_head;
  const int u = idx - r * per_head;
  it.b = r / p.Hq;
  it.h = r - it.b * p.Hq;
  it.kvh = it.h / p.G;
  if (p.causal) {
    it.qt[0] = p.n_qtiles - 1 - u;
    it.qt[1] = u;
    it.nseg = it.qt[1] == it.qt[0] ? 1 : 2;
    it.n[0] = min((p.q_offset + it.qt[0] * kRows + kRows - 1) / kRows + 1, p.n_kvtiles);
    it.n[1] = min((p.q_offset + it.qt[1] * kRows + kRows - 1) / kRows + 1, p.n_kvtiles);
  } else {
    it.qt[0] = it.qt[1] = u;
    it.nseg = 1;
    it.n[0] = it.n[1] = p.n_kvtiles;
  }
  return it;
}

// ------------------------------------------------------------ producer warp
// Loads, per item, the Q tile and then the K / V tiles in the order the MMA
// thread consumes them: K0, K1, then V(j), K(j + 2) for j = 0 .. n - 1.
template <int D, int V>
__device__ void producer3(const FmhaParams& p, const FmhaMaps& maps, uint8_t* smem, Bars3& bars, const WaitCtl& wc) {
  using L = L3<D>;
  constexpr int NS = L::NS;
  uint32_t ld = 0, qn = 0;
  uint32_t armed = 0;
  bool ok = true;
  bool first_k = true;
  auto load_kv = [&](bool is_k, int tile, const Item3& it) -> bool {
    const uint32_t slot = ld % NS;
    if (!wc.wait(&bars.kv_empty[slot], ((ld / NS) & 1) ^ 1)) return false;
    const bool withhold = is_k && first_k && (p.debug_flags & 1);
    if (is_k) first_k = false;
    if (!withhold) {
      mbar_arrive_expect_tx(&bars.kv_full[slot], L::kTile);
      uint8_t* dst = smem + L::kKV + slot * L::kTile;
      const CUtensorMap* m = is_k ? &maps.k : &maps.v;
      for (int c = 0; c < L::kPanels; ++c)
        tma_load_4d(dst + c * L::kSub, m, &bars.kv_full[slot], c * 64, tile * kRows, it.kvh, it.b);
      armed |= 1u << slot;
    } else {
      armed &= ~(1u << slot);
    }
    ++ld;
    return true;
  };
  // Q tiles run one segment ahead: the next segment's Q load is issued right
  // after the current segment's first K tiles, into the other Q slot (freed
  // by the previous segment's last QK^T), so it has a whole segment to land.
  auto load_q = [&](const Item3& it, int sg) -> bool {
    const uint32_t qs = qn & 1;
    if (!wc.wait(&bars.q_empty[qs], ((qn >> 1) & 1) ^ 1)) return false;
    mbar_arrive_expect_tx(&bars.q_full[qs], L::kTile);
    const int qt = sg == 0 ? it.qt[0] : it.qt[1];
    for (int c = 0; c < L::kPanels; ++c)
      tma_load_4d(smem + L::kQ + qs * L::kTile + c * L::kSub, &maps.q, &bars.q_full[qs], c * 64, qt * kRows, it.h,
                  it.b);
    ++qn;
    return true;
  };
  if (blockIdx.x < p.num_items) ok = load_q(decode_item3(p, blockIdx.x), 0);
  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item3 it = decode_item3(p, idx);
    for (int sg = 0; ok && sg < it.nseg; ++sg) {
      const int n = sg == 0 ? it.n[0] : it.n[1];
      ok = load_kv(true, 0, it);
      if (ok && n > 1) ok = load_kv(true, 1, it);
      if (ok) {   // the next segment's Q
        if (sg + 1 < it.nseg) ok = load_q(it, sg + 1);
        else if (idx + (int)gridDim.x < p.num_items) ok = load_q(decode_item3(p, idx + gridDim.x), 0);
      }
      for (int j = 0; ok && j < n; ++j) {
        ok = load_kv(false, j, it);
        if (ok && j + 2 < n) ok = load_kv(true, j + 2, it);
      }
    }
  }
  if (!ok) {
    for (uint32_t i = (ld > NS ? ld - NS : 0); i < ld; ++i) {
      const uint32_t slot = i % NS;
      if (armed & (1u << slot)) drain_wait(&bars.kv_full[slot], (i / NS) & 1, wc.timeout_ns);
    }
    for (uint32_t i = qn > 2 ? qn - 2 : 0; i < qn; ++i) drain_wait(&bars.q_full[i & 1], (i >> 1) & 1, wc.timeout_ns);
  }
}

// ---------------------------------------------------------------- MMA warps
// Two issuing threads, one per MMA kind, so that one thread's barrier waits
// overlap the other's issue (an issuing thread blocks while the tensor pipe
// drains its queue, ~70 cycles per 128x128x16 MMA; a single issuer waiting for
// P, K and V in series left the pipe idle for about a third of every tile).
//   QK issuer: QK(g) into score buffer g % 3 for the global tile index g, once
//              PV(g - 3) (which reads P(g - 3) from that buffer) has completed.
//   PV issuer: PV(g) once the softmax has written P(g).
// Ring positions of an item's K / V tiles (the producer's order): K0 at 0,
// K1 at 1, then V(j) and K(j + 2) alternate; with e0 the item's first position
// and n >= 2: K(j) at e0 + (j < 2 ? j : 2j - 1); V(j) at e0 + 2 + 2j for
// j <= n - 2 and e0 + 2n - 1 for j = n - 1; with n = 1: K0 at e0, V0 at e0 + 1.
// The issuers poll without suspending (a suspended thread wakes a few hundred
// cycles after the phase completes); measured equal to suspending waits, which
// would matter only if the polling took issue slots from the softmax warps.
__device__ __forceinline__ bool issuer_wait(const WaitCtl& wc, uint64_t* bar, uint32_t parity) {
  return spin_wait(wc, bar, parity);
}
__device__ __forceinline__ uint32_t pos_k(int j) { return j < 2 ? (uint32_t)j : (uint32_t)(2 * j - 1); }
__device__ __forceinline__ uint32_t pos_v(int j, int n) {
  if (n == 1) return 1;
  return j <= n - 2 ? (uint32_t)(2 + 2 * j) : (uint32_t)(2 * n - 1);
}

template <int D, int V>
__device__ void qk_issuer3(const FmhaParams& p, uint8_t* smem, Bars3& bars, const WaitCtl& wc, uint32_t tmem) {
  using L = L3<D>;
  constexpr int NS = L::NS;
  constexpr int SUB = L::kSub;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 128, false);
  constexpr uint32_t HI = sdesc_hi_sbo1024();
  const uint32_t smem_base = smem_u32(smem);
  const uint32_t q_lo = sdesc_lo(smem_base + L::kQ, 16);
  const uint32_t k_lo0 = sdesc_lo(smem_base + L::kKV, 16);
  uint32_t e0 = 0, qn = 0, tc = 0;
  bool ok = true;
  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item3 it = decode_item3(p, idx);
    for (int sg = 0; ok && sg < it.nseg; ++sg) {
      const int n = sg == 0 ? it.n[0] : it.n[1];
      const uint32_t qs = qn & 1;
      if (!wc.wait(&bars.q_full[qs], (qn >> 1) & 1)) { ok = false; break; }
      ++qn;
      const uint32_t qa = q_lo + qs * (uint32_t)(L::kTile / 16);
      for (int j = 0; j < n; ++j) {
        constexpr uint32_t NB = Split<D, V>::NB;
        const uint32_t g = tc + j, buf = g % NB;
        const uint32_t e = e0 + pos_k(j);
        if (!wc.wait(&bars.kv_full[e % NS], (e / NS) & 1)) { ok = false; break; }
        BW_TRACE_AT(true, 22, g);
        if (g >= NB && !issuer_wait(wc, &bars.pv_done[buf], ((g - NB) / NB) & 1)) { ok = false; break; }
        BW_TRACE_AT(true, 23, g);
        tc_fence_after();
        const uint32_t ka = k_lo0 + (e % NS) * (uint32_t)(L::kTile / 16);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = ((ks >> 2) * SUB + (ks & 3) * 32) / 16;
          mma_ss_lh(tmem + buf * 128, qa + off, HI, ka + off, HI, IDESC_QK, ks > 0);
        }
        BW_TRACE_AT(true, 24, g);
        tc_commit(&bars.s_full[buf]);
        tc_commit(&bars.kv_empty[e % NS]);
        if (j == n - 1) tc_commit(&bars.q_empty[qs]);
      }
      if (!ok) break;
      tc += n;
      e0 += 2 * n;
    }
  }
  tc_commit(&bars.qk_done);
  drain_wait(&bars.qk_done, 0, wc.timeout_ns);
}

template <int D, int V>
__device__ void pv_issuer3(const FmhaParams& p, uint8_t* smem, Bars3& bars, const WaitCtl& wc, uint32_t tmem) {
  using L = L3<D>;
  constexpr int NS = L::NS;
  constexpr int SUB = L::kSub;
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, D, true);
  constexpr uint32_t HI = sdesc_hi_sbo1024();
  const uint32_t v_lo0 = sdesc_lo(smem_u32(smem) + L::kKV, SUB);   // V operand (MN-major)
  uint32_t e0 = 0, tc = 0, itn = 0;
  bool ok = true;
  for (int idx = blockIdx.x; ok && idx < p.num_items; idx += gridDim.x) {
    const Item3 it = decode_item3(p, idx);
    for (int sg = 0; ok && sg < it.nseg; ++sg) {
      const int n = sg == 0 ? it.n[0] : it.n[1];
      for (int j = 0; j < n; ++j) {
        constexpr uint32_t NB = Split<D, V>::NB;
        const uint32_t g = tc + j, buf = g % NB;
        const uint32_t e = e0 + pos_v(j, n);
        if (!wc.wait(&bars.kv_full[e % NS], (e / NS) & 1)) { ok = false; break; }
        // the previous tile's epilogue must have read O before PV(0) overwrites it
        if (j == 0 && itn > 0 && !wc.wait(&bars.o_empty, (itn - 1) & 1)) { ok = false; break; }
        if (!issuer_wait(wc, &bars.p_full[buf], (g / NB) & 1)) { ok = false; break; }
        BW_TRACE_AT(true, 6, g);
        tc_fence_after();
        const uint32_t va = v_lo0 + (e % NS) * (uint32_t)(L::kTile / 16);
        if constexpr (V == 5) {
          // key tile j accumulates into O_{j % 2} (the part that owns it)
          const uint32_t o_col = Split<D, V>::kOCol + (uint32_t)(j & 1) * D;
#pragma unroll
          for (int ks = 0; ks < kRows / 16; ++ks)
            mma_ts_lh(tmem + o_col, tmem + buf * 128 + ks * 8, va + (ks * 16 * 128) / 16, HI, IDESC_PV,
                      (ks > 0 || j >= 2) ? 1u : 0u);
        } else {
          // O += P (bf16, key k at column k / 2 of the buffer) * V; k-step ks: keys 16 ks ..
#pragma unroll
          for (int ks = 0; ks < kRows / 16; ++ks)
            mma_ts_lh(tmem + Split<D, V>::kOCol, tmem + buf * 128 + ks * 8, va + (ks * 16 * 128) / 16, HI, IDESC_PV,
                      (ks > 0 || j > 0) ? 1u : 0u);
        }
        BW_TRACE_AT(true, 8, g);
        tc_commit(&bars.pv_done[buf]);
        tc_commit(&bars.kv_empty[e % NS]);
      }
      if (!ok) break;
      tc_commit(&bars.o_full);
      tc += n;
      e0 += 2 * n;
      ++itn;
    }
  }
  tc_commit(&bars.mma_done);
  drain_wait(&bars.mma_done, 0, wc.timeout_ns);
}

__device__ __forceinline__ uint32_t pack_bf16_3(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------- softmax warps, kernel 4
// Warp w (0 .. 7) covers TMEM lanes 32 (w % 4) + 16 (w / 4) .. + 15 with the
// 16-lane shapes: thread i holds rows r0 = that base + i / 4 and r1 = r0 + 8,
// keys 8 c + 2 (i % 4) and + 1 of chunk c = 0 .. 15 of every key tile (64
// scores, 32 per row).  The four threads of a row (lanes 4k .. 4k + 3) reduce
// the tile max with two shuffles and so keep the same running max; each keeps
// its own partial row sum, reduced at the end of the query tile.  P (bf16)
// goes back over the first 64 columns of the score buffer in the order the PV
// MMA reads it (key k at column k / 2).
template <int D, int POLY>
__device__ void softmax4(const FmhaParams& p, uint8_t* smem, Bars3& bars, const WaitCtl& wc, uint32_t tmem, int t) {
  using L = L3<D>;
  using Split = bw::Split<D, 4>;
  constexpr uint32_t NB = Split::NB;
  const int w = t >> 5, ln = t & 31;
  const int rb = 32 * (w & 3) + 16 * (w >> 2);           // first TMEM lane of the warp
  const int r0 = rb + (ln >> 2), kq = 2 * (ln & 3);      // rows r0, r0 + 8; key offset in a chunk
  const uint32_t lane_off = (uint32_t)rb << 16;
  const uint32_t o_tm = tmem + lane_off + Split::kOCol;
  const float c = p.scale_log2;
  float2* xch = reinterpret_cast<float2*>(smem + L::kX);
  uint32_t tc = 0, itn = 0;

  for (int idx = blockIdx.x; idx < p.num_items; idx += gridDim.x) {
    const Item3 it = decode_item3(p, idx);
    for (int sg = 0; sg < it.nseg; ++sg) {
    const int n = sg == 0 ? it.n[0] : it.n[1];
    const int qt = sg == 0 ? it.qt[0] : it.qt[1];
    const int row0 = qt * kRows + r0;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    for (int j = 0; j < n; ++j) {
      const uint32_t g = tc + j, buf = g % NB;
      const uint32_t s_tmem = tmem + lane_off + buf * 128;
      if (!wc.wait(&bars.s_full[buf], (g / NB) & 1)) return;
      BW_TRACE_AT(t == 0, 0, g);
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_16x256b_x16(s_tmem, r);
      BW_TRACE_AT(t == 0, 1, g);
      float* s = reinterpret_cast<float*>(r);
      const int kv0 = j * kRows;
      if ((p.causal && kv0 + kRows - 1 > p.q_offset + qt * kRows) || kv0 + kRows > p.Skv) {
        int lim0 = p.Skv - kv0, lim1 = lim0;
        if (p.causal) {
          lim0 = min(lim0, p.q_offset + row0 + 1 - kv0);
          lim1 = min(lim1, p.q_offset + row0 + 9 - kv0);
        }
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const int k = 8 * ch + kq;
          if (k >= lim0) s[4 * ch] = -INFINITY;
          if (k + 1 >= lim0) s[4 * ch + 1] = -INFINITY;
          if (k >= lim1) s[4 * ch + 2] = -INFINITY;
          if (k + 1 >= lim1) s[4 * ch + 3] = -INFINITY;
        }
      }
      float mx0, mx1;
      {
        float a0 = fmaxf(s[0], s[1]), b0 = fmaxf(s[4], s[5]), a1 = fmaxf(s[2], s[3]), b1 = fmaxf(s[6], s[7]);
#pragma unroll
        for (int ch = 2; ch < 16; ch += 2) {
          a0 = fmax3(a0, s[4 * ch], s[4 * ch + 1]);
          b0 = fmax3(b0, s[4 * ch + 4], s[4 * ch + 5]);
          a1 = fmax3(a1, s[4 * ch + 2], s[4 * ch + 3]);
          b1 = fmax3(b1, s[4 * ch + 6], s[4 * ch + 7]);
        }
        mx0 = fmaxf(a0, b0);
        mx1 = fmaxf(a1, b1);
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      }
      // lazy rescale per row (the same decision in the row's four threads)
      const float mc0 = mx0 * c, mc1 = mx1 * c;
      float corr0 = 1.f, corr1 = 1.f;
      const bool up0 = mc0 > m0 + 8.f, up1 = mc1 > m1 + 8.f;
      if (up0) {
        corr0 = ex2_mufu(m0 - mc0);
        m0 = mc0;
      }
      if (up1) {
        corr1 = ex2_mufu(m1 - mc1);
        m1 = mc1;
      }
      const float ms0 = (m0 == -INFINITY) ? 0.f : m0, ms1 = (m1 == -INFINITY) ? 0.f : m1;
      const f2 cc2{c, c}, nm0{-ms0, -ms0}, nm1{-ms1, -ms1};
      f2 sa0{0.f, 0.f}, sb0{0.f, 0.f}, sa1{0.f, 0.f}, sb1{0.f, 0.f};
      // pair k: chunk k / 2, row k & 1 (registers 4 (k / 2) + 2 (k & 1) and + 1)
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int i = 4 * (k >> 1) + 2 * (k & 1);
        const f2 x = ffma2(f2{s[i], s[i + 1]}, cc2, (k & 1) ? nm1 : nm0);
        f2 e;
        if ((k & 7) < POLY) {
          e = ex2_poly2(x);
        } else {
          e.x = ex2_mufu(x.x);
          e.y = ex2_mufu(x.y);
        }
        s[i] = e.x;
        s[i + 1] = e.y;
        if ((k & 1) == 0) {
          if ((k & 2) == 0) sa0 = fadd2(sa0, e);
          else sb0 = fadd2(sb0, e);
        } else {
          if ((k & 2) == 0) sa1 = fadd2(sa1, e);
          else sb1 = fadd2(sb1, e);
        }
      }
      sa0 = fadd2(sa0, sb0);
      sa1 = fadd2(sa1, sb1);
      l0 = l0 * corr0 + (sa0.x + sa0.y);
      l1 = l1 * corr1 + (sa1.x + sa1.y);
      BW_TRACE_AT(t == 0, 2, g);
      {
        // 16x128b repetition ch: column 4 ch + i % 4 (keys 8 ch + 2 (i % 4), + 1) of rows r0, r0 + 8
        uint32_t pk[32];
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          pk[2 * ch] = pack_bf16_3(s[4 * ch], s[4 * ch + 1]);
          pk[2 * ch + 1] = pack_bf16_3(s[4 * ch + 2], s[4 * ch + 3]);
        }
        tmem_st_16x128b_x16(s_tmem, pk);
      }
      if (j > 0 && __any_sync(0xffffffffu, up0 || up1)) {
        // O must hold PV(j - 1) before it is rescaled
        if (!wc.wait(&bars.pv_done[(g - 1) % NB], ((g - 1) / NB) & 1)) return;
        tc_fence_after();
        if constexpr (D == 128) {
          uint32_t o[64];
          tmem_ld_16x256b_x16(o_tm, o);
#pragma unroll
          for (int i = 0; i < 64; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * ((i & 2) ? corr1 : corr0));
          tmem_st_16x256b_x16(o_tm, o);
        } else {
          uint32_t o[32];
          tmem_ld_16x256b_x8(o_tm, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * ((i & 2) ? corr1 : corr0));
          tmem_st_16x256b_x8(o_tm, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (ln == 0) mbar_arrive(&bars.p_full[buf]);
      BW_TRACE_AT(t == 0, 3, g);
      BW_TRACE_AT(ln == 0 && t < 256, 10 + w, g);
    }
    // the row sums of the four threads, then (m, l) per row for the epilogue
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (itn > 0 && !wc.wait(&bars.xch_empty, (itn - 1) & 1)) return;
    if ((ln & 3) == 0) {
      xch[r0] = make_float2(m0, l0);
      xch[r0 + 8] = make_float2(m1, l1);
    }
    __syncwarp();
    if (ln == 0) mbar_arrive(&bars.xch_full);
    tc += n;
    ++itn;
    }
  }
}

// ------------------------------------------------- softmax warps, kernel 5
// D = 64 only.  The two softmax warpgroups own alternate key tiles of a query
// tile: part q = t / 128 takes key tiles j = q, q + 2, .. and accumulates them
// into its own O_q; thread t holds row t % 128 and all 128 scores of its tile
// (32x32b shape).  The two warps of one SM sub-partition therefore work on
// neighbouring key tiles, not on the same one, so one warp's barrier waits and
// TMEM round trips overlap the other's exponentials.  Each part keeps its own
// running max and sum; the epilogue merges the two accumulators.  TMEM:
// S_0 | S_1 | S_2 | O_0 | O_1 (3 x 128 + 2 x 64 columns); P(g) goes
// over the first 64 columns of its score buffer.  A rescale of O_q at tile j
// waits for PV(j - 2), the part's previous tile.
template <int D, int POLY>
__device__ void softmax5(const FmhaParams& p, uint8_t* smem, Bars3& bars, const WaitCtl& wc, uint32_t tmem, int t) {
  using L = L3<D>;
  using Split = bw::Split<D, 5>;
  constexpr uint32_t NB = Split::NB;
  const int rl = t & 127, part = t >> 7;
  const uint32_t lane_off = (uint32_t)((rl >> 5) * 32) << 16;
  const uint32_t o_own = tmem + lane_off + Split::kOCol + part * D;
  const float c = p.scale_log2;
  float2* xch = reinterpret_cast<float2*>(smem + L::kX);
  uint32_t tc = 0, itn = 0;
  // Score buffer g % 3 is reused by tile g + 3, and a parity wait for S(g) is
  // only exact once S(g - 3) is known complete.  A part skips the other part's
  // tiles (up to three in a row across segment boundaries), so it first waits,
  // in order, for every score tile before its own: those complete in order
  // before S(g) anyway, so this adds no latency.
  uint32_t s_next = 0;

  for (int idx = blockIdx.x; idx < p.num_items; idx += gridDim.x) {
    const Item3 it = decode_item3(p, idx);
    for (int sg = 0; sg < it.nseg; ++sg) {
    const int n = sg == 0 ? it.n[0] : it.n[1];
    const int qt = sg == 0 ? it.qt[0] : it.qt[1];
    const int row = qt * kRows + rl;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = part; j < n; j += 2) {
      const uint32_t g = tc + j, buf = g % NB;
      const uint32_t s_tmem = tmem + lane_off + buf * 128;
      for (; s_next <= g; ++s_next)
        if (!wc.wait(&bars.s_full[s_next % NB], (s_next / NB) & 1)) return;
      BW_TRACE_AT(t == 0, 0, g);
      BW_TRACE_AT(t == 128, 4, g);
      tc_fence_after();
      uint32_t r[128];
      tmem_ld128(s_tmem, r);
      BW_TRACE_AT(t == 0, 1, g);
      BW_TRACE_AT(t == 128, 18, g);
      float* s = reinterpret_cast<float*>(r);
      const int kv0 = j * kRows;
      if ((p.causal && kv0 + kRows - 1 > p.q_offset + qt * kRows) || kv0 + kRows > p.Skv) {
        int lim = p.Skv - kv0;
        if (p.causal) lim = min(lim, p.q_offset + row + 1 - kv0);
#pragma unroll
        for (int i = 0; i < kRows; ++i)
          if (i >= lim) s[i] = -INFINITY;
      }
      float mx;
      {
        float a[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = fmaxf(s[u], s[8 + u]);
#pragma unroll
        for (int i = 16; i < kRows; i += 16)
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
      f2 acc0{0.f, 0.f}, acc1{0.f, 0.f}, acc2{0.f, 0.f}, acc3{0.f, 0.f};
      uint32_t pk[kRows / 2];
#pragma unroll
      for (int k = 0; k < kRows / 2; ++k) {
        const f2 x = ffma2(f2{s[2 * k], s[2 * k + 1]}, cc2, nm2);
        f2 e;
        if ((k & 7) < POLY) {
          e = ex2_poly2(x);
        } else {
          e.x = ex2_mufu(x.x);
          e.y = ex2_mufu(x.y);
        }
        pk[k] = pack_bf16_3(e.x, e.y);
        if ((k & 3) == 0) acc0 = fadd2(acc0, e);
        else if ((k & 3) == 1) acc1 = fadd2(acc1, e);
        else if ((k & 3) == 2) acc2 = fadd2(acc2, e);
        else acc3 = fadd2(acc3, e);
      }
      acc0 = fadd2(fadd2(acc0, acc1), fadd2(acc2, acc3));
      l_run = l_run * corr + (acc0.x + acc0.y);
      BW_TRACE_AT(t == 0, 2, g);
      BW_TRACE_AT(t == 128, 19, g);
      // P (bf16, key k at column k / 2) over the first 64 columns of the buffer
      tmem_st32(s_tmem, pk);
      tmem_st32(s_tmem + 32, pk + 32);
      if (j >= 2 && __any_sync(0xffffffffu, upd)) {
        // O_part must hold PV(j - 2) before it is rescaled (exact parity: QK(g)
        // waited for PV(g - 3), so PV(g - 5) is complete)
        if (!wc.wait(&bars.pv_done[(g - 2) % NB], ((g - 2) / NB) & 1)) return;
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_own + c0, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st32(o_own + c0, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if ((t & 31) == 0) mbar_arrive(&bars.p_full[buf]);
      BW_TRACE_AT(t == 0, 3, g);
      BW_TRACE_AT(t == 128, 5, g);
      BW_TRACE_AT((t & 31) == 0 && t < 256, 10 + (t >> 5), g);
    }
    // (m, l) of the row's part for the epilogue (a part with no key tile in
    // this segment hands over m = -inf, l = 0)
    if (itn > 0 && !wc.wait(&bars.xch_empty, (itn - 1) & 1)) return;
    xch[part * kRows + rl] = make_float2(m_run, l_run);
    __syncwarp();
    if ((t & 31) == 0) mbar_arrive(&bars.xch_full);
    tc += n;
    ++itn;
    }
  }
}

// 16 or 32 consecutive TMEM columns of this thread's lane (32x32b shape).
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld32(taddr, r); }

// ---------------------------------------------------------- epilogue warps
// Thread t (0 .. 127): row t of every segment's query tile (TMEM lane t).  Per
// segment: merge the parts of the row (kernel 5) from their (m, l) (m = max_q m_q,
// w_q = 2^(m_q - m) / L, L = sum_q l_q 2^(m_q - m)), read O_0 .. O_{N-1} once
// PV of the segment's last tile is done, free O for the next segment's first
// PV, and write O = sum_q w_q O_q through the warp's staging area with TMA
// stores (rows past Sq are clipped by the map) and LSE = ln 2 (m + log2 L).
// The softmax warps never wait for any of this unless they finish a whole
// segment before the previous one's (m, l) has been read.
// (Kernel 4: one accumulator, N = 1 below: O / L.)
template <int D, int V>
__device__ void epilogue3(const FmhaParams& p, const FmhaMaps& maps, uint8_t* smem, Bars3& bars, const WaitCtl& wc,
                          uint32_t tmem, int t) {
  using L = L3<D>;
  constexpr int N = Split<D, V>::NACC;
  const int ln = t & 31, wq = t >> 5;
  const uint32_t o0 = tmem + ((uint32_t)(wq * 32) << 16) + Split<D, V>::kOCol;
  const float2* xch = reinterpret_cast<const float2*>(smem + L::kX);
  uint8_t* stg = smem + L::kStg + wq * L::kStgWarp;
  uint32_t itn = 0;
  for (int idx = blockIdx.x; idx < p.num_items; idx += gridDim.x) {
    const Item3 it = decode_item3(p, idx);
    for (int sg = 0; sg < it.nseg; ++sg) {
      const int qt = sg == 0 ? it.qt[0] : it.qt[1];
      const int row = qt * kRows + t;
      if (!wc.wait(&bars.xch_full, itn & 1)) return;
      float mp[N], lp[N];
#pragma unroll
      for (int q = 0; q < N; ++q) {
        const float2 v = xch[q * kRows + t];
        mp[q] = v.x;
        lp[q] = v.y;
      }
      __syncwarp();
      if (ln == 0) mbar_arrive(&bars.xch_empty);
      float m = mp[0];
#pragma unroll
      for (int q = 1; q < N; ++q) m = fmaxf(m, mp[q]);
      float w[N], lsum = 0.f;
#pragma unroll
      for (int q = 0; q < N; ++q) {
        w[q] = mp[q] == -INFINITY ? 0.f : ex2_mufu(mp[q] - m);
        lsum = fmaf(lp[q], w[q], lsum);
      }
      const float inv_l = 1.f / lsum;
#pragma unroll
      for (int q = 0; q < N; ++q) w[q] *= inv_l;
      if (ln == 0) bulk_wait_read0();   // the warp's previous stores have read the staging area
      __syncwarp();
      if (!wc.wait(&bars.o_full, itn & 1)) return;
      tc_fence_after();
      // columns per TMEM load: 16 for kernel 5, whose epilogue runs in 64 registers
      constexpr int CW = V == 5 ? 16 : 32;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += CW) {
        float acc[CW];
        uint32_t x[CW];
        tmem_ld_cols(o0 + c0, x);
#pragma unroll
        for (int i = 0; i < CW; ++i) acc[i] = __uint_as_float(x[i]) * w[0];
#pragma unroll
        for (int q = 1; q < N; ++q) {
          tmem_ld_cols(o0 + q * D + c0, x);
          // kernel 5: a part that owned no key tile of the segment (n = 1) never
          // wrote its accumulator, whose stale contents must not reach O
          if (V == 5 && w[q] == 0.f) continue;
#pragma unroll
          for (int i = 0; i < CW; ++i) acc[i] = fmaf(__uint_as_float(x[i]), w[q], acc[i]);
        }
        // columns c0 .. c0 + CW - 1: panel c0 / 64, 16-byte chunks (c0 % 64) / 8 + i
#pragma unroll
        for (int i = 0; i < CW / 8; ++i) {
          const int ch = (c0 & 63) / 8 + i;
          *reinterpret_cast<uint4*>(stg + (c0 / 64) * (32 * 128) + ln * 128 + ((ch ^ (ln & 7)) << 4)) =
              make_uint4(pack_bf16_3(acc[8 * i], acc[8 * i + 1]), pack_bf16_3(acc[8 * i + 2], acc[8 * i + 3]),
                         pack_bf16_3(acc[8 * i + 4], acc[8 * i + 5]), pack_bf16_3(acc[8 * i + 6], acc[8 * i + 7]));
        }
      }
      // O has been read: the next segment's first PV may overwrite it
      tc_fence_before();
      __syncwarp();
      if (ln == 0) mbar_arrive(&bars.o_empty);
      fence_proxy_async_smem();
      __syncwarp();
      if (ln == 0) {
#pragma unroll
        for (int c = 0; c < D / 64; ++c) tma_store_4d(&maps.o, stg + c * (32 * 128), c * 64, row - ln, it.h, it.b);
        bulk_commit();
      }
      if (p.LSE != nullptr && row < p.Sq)
        p.LSE[((int64_t)it.b * p.Hq + it.h) * p.lse_sh + row] = (m + __log2f(lsum)) * 0.69314718055994531f;
      ++itn;
    }
  }
}

template <int D, int POLY, int V>
__global__ void __launch_bounds__(512, 1) fmha_fwd3_kernel(const FmhaParams p, const __grid_constant__ FmhaMaps maps) {
  using Split = bw::Split<D, V>;
  static_assert(Split::kThreads == 512, "launch bounds");
  using L = L3<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad > (uint32_t)kAlignSlack) {
    // the window cannot hold the 1024-aligned layout: report, do nothing
    if (threadIdx.x == 0) atomicCAS(p.err, 0, 0x400);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  Bars3& bars = *reinterpret_cast<Bars3*>(smem + L::kBar);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  constexpr int kSoftWarps = 4 * Split::N;
  constexpr int kEpilogue = kSoftWarps;                     // warpgroup 2
  constexpr int kProducer = kSoftWarps + 4, kPvIssuer = kSoftWarps + 5, kQkIssuer = kSoftWarps + 6;

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars.q_full[b], 1);
      mbar_init(&bars.q_empty[b], 1);
    }
    for (int b = 0; b < Split::NB; ++b) {
      mbar_init(&bars.s_full[b], 1);
      mbar_init(&bars.p_full[b], V == 5 ? 4 : 4 * Split::N);   // one arrival per softmax warp of the tile
    }
    for (int b = 0; b < Split::NB; ++b) mbar_init(&bars.pv_done[b], 1);
    mbar_init(&bars.qk_done, 1);
    mbar_init(&bars.o_full, 1);
    mbar_init(&bars.o_empty, 4);                     // one arrival per epilogue warp
    mbar_init(&bars.xch_full, 4 * Split::N);         // one per softmax warp
    mbar_init(&bars.xch_empty, 4);
    mbar_init(&bars.mma_done, 1);
    for (int s = 0; s < L::NS; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    bars.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducer && lane == 0) {
    prefetch_tmap(&maps.q);
    prefetch_tmap(&maps.k);
    prefetch_tmap(&maps.v);
    prefetch_tmap(&maps.o);
  }
  if (warp == kPvIssuer) tmem_alloc(&bars.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  WaitCtl wc{&bars.abort_flag, p.err, p.timeout_ns, warp};

  // Register split (the block is launched with 128 per thread, 65536 in all):
  // softmax 2 x 128 x 168 + epilogue 128 x 128 + producer / issuers 128 x 40
  // = 64512; kernel 5 (a whole 128-score row per thread): softmax 2 x 128 x
  // 200 + epilogue 128 x 64 + producer / issuers 128 x 48 = 65536 (no spills;
  // issuers at 32 spilled, run once per key tile).
  constexpr int kSoftRegs = V == 5 ? 200 : 168, kEpiRegs = V == 5 ? 64 : 128, kAuxRegs = V == 5 ? 48 : 40;
  static_assert(2 * 128 * kSoftRegs + 128 * kEpiRegs + 128 * kAuxRegs <= 65536, "register split");
  if (warp < kSoftWarps) {
    reg_alloc<kSoftRegs>();
    if constexpr (V == 5) softmax5<D, POLY>(p, smem, bars, wc, tmem, tid);
    else softmax4<D, POLY>(p, smem, bars, wc, tmem, tid);
  } else if (warp < kEpilogue + 4) {
    reg_dealloc<kEpiRegs>();   // 128 keeps the launch count; states this role's bound to the register allocator
    epilogue3<D, V>(p, maps, smem, bars, wc, tmem, tid - 32 * kEpilogue);
    // the warp's output stores read shared memory until they complete
    if (lane == 0) bulk_wait0();
  } else {
    reg_dealloc<kAuxRegs>();
    if (lane == 0) {
      if (warp == kProducer) producer3<D, V>(p, maps, smem, bars, wc);
      else if (warp == kPvIssuer) pv_issuer3<D, V>(p, smem, bars, wc, tmem);
      else if (warp == kQkIssuer) qk_issuer3<D, V>(p, smem, bars, wc, tmem);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPvIssuer) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, int POLY, int V>
cudaError_t launch3(const FmhaParams& p, const FmhaMaps& maps, int num_sms, cudaStream_t stream) {
  constexpr int bytes = L3<D>::kBytes + kAlignSlack;
  auto kern = fmha_fwd3_kernel<D, POLY, V>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  const int grid = p.num_items < num_sms ? p.num_items : num_sms;
  kern<<<grid, Split<D, V>::kThreads, bytes, stream>>>(p, maps);
  return cudaGetLastError();
}

template <int D, int V>
cudaError_t launch3_poly(const FmhaParams& p, const FmhaMaps& maps, int poly, int num_sms, cudaStream_t stream) {
  switch (poly) {
    case 0: return launch3<D, 0, V>(p, maps, num_sms, stream);
    case 2: return launch3<D, 2, V>(p, maps, num_sms, stream);
    case 3: return launch3<D, 3, V>(p, maps, num_sms, stream);
    case 4: return launch3<D, 4, V>(p, maps, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_fmha_fwd5(const FmhaParams& p, const FmhaMaps& maps, int exp_poly, int num_sms,
                             cudaStream_t stream) {
  if (p.D == 64) return launch3_poly<64, 5>(p, maps, exp_poly, num_sms, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_fmha_fwd4(const FmhaParams& p, const FmhaMaps& maps, int exp_poly, int num_sms,
                             cudaStream_t stream) {
  if (p.D == 128) return launch3_poly<128, 4>(p, maps, exp_poly, num_sms, stream);
  if (p.D == 64) return launch3_poly<64, 4>(p, maps, exp_poly, num_sms, stream);
  return cudaErrorInvalidValue;
}

}  // namespace bw

#ifdef BW_TRACE
extern "C" __attribute__((visibility("default"))) int bw_trace_read3(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, g_bw_trace, sizeof(g_bw_trace));
  return 64 * 512;
}
#endif
