// Split-KV single-token GQA decode and the LSE-combine of split partials.
//
// The reference has no decode kernel; the behaviour restated here is its
// split-length GQA (src/SM120/attention/adhitya_GQA.cu:63-188,
// base/baseline_gqa_split.py:33-48) with Sq = 1 and one Skv = L_b per sequence.
//
// Decode is HBM-bound (about 8 FLOP per byte of K/V), so the kernel is built
// around streaming: a persistent grid; per CTA one TMA producer thread feeding a
// 3-stage ring of 64-token K and V tiles (128B-swizzled, one 2-D tensor map over
// [total_tokens, Hkv * D]); four consumer warps each taking 16 tokens of a stage.
// The G query heads of one KV head form the M dimension of mma.sync m16n8k16
// (M = 16 >= G, rows >= G are zero); a tcgen05 MMA needs M >= 64 and would only
// add padding, and the tensor pipe is far from the bound here.
//
// Work item = (sequence b, chunk c of `chunk` tokens, KV head).  Each item writes
// a partial (O normalised by its own sum, natural-log LSE) for its G heads; the
// combine kernel merges the chunks of a sequence.  An item reads chunk*4*D bytes
// of K/V and writes G*D*4 bytes of partial, so partial traffic is G/chunk of the
// K/V bytes (1/128 at G = 8, chunk = 1024).
#include "kernels.h"
#include "ptx.cuh"

namespace bw {
namespace {

constexpr int kTok = 64;          // tokens per stage
constexpr int kStages = 3;
constexpr int kConsumers = 4;     // warps
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kMaxB = 4096;
constexpr int kBtCacheEntries = 160;   // page indices cached per work item (chunk / page_size + 1)

template <int D>
struct DecCfg {
  static constexpr int kHalf = kTok * D * 2;               // K (or V) part of a stage
  static constexpr int kStage = 2 * kHalf;
  static constexpr int kAcc = kStages * kStage;            // fp32 [16][D] accumulator
  static constexpr int kRed = kAcc + 16 * D * 4;           // m, l [4][16] each
  static constexpr int kBar = kRed + 2 * kConsumers * 16 * 4;
  static constexpr int kBtCache = kBar + 128;                // paged: page indices of one item
  static constexpr int kPrefix = kBtCache + kBtCacheEntries * 4;
};

struct DecBars {
  uint64_t full[kStages], empty[kStages];
  int abort_flag;
  int total_parts;
  long long warp_sum[kThreads / 32];
};
static_assert(sizeof(DecBars) <= 128, "DecBars must fit the 128 bytes reserved at kBar");

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
}

struct DecItem {
  int b, c, kvh, part;
  int64_t t0, t1;
};

__device__ __forceinline__ DecItem dec_item(const DecodeParams& p, const int* prefix, int idx) {
  DecItem it;
  const int pc = idx / p.Hkv;
  it.kvh = idx - pc * p.Hkv;
  int lo = 0, hi = p.B - 1;               // last b with prefix[b] <= pc
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= pc) lo = mid; else hi = mid - 1;
  }
  it.b = lo;
  it.c = pc - prefix[lo];
  it.part = idx;
  const int64_t base = p.block_table ? 0 : p.kv_offsets[it.b];   // paged: sequence-relative tokens
  const int len = p.kv_lens[it.b];
  it.t0 = base + (int64_t)it.c * p.chunk;
  const int64_t end = base + len;
  it.t1 = min(it.t0 + p.chunk, end);
  return it;
}

template <int D>
__global__ void __launch_bounds__(kThreads)
    decode_kernel(const DecodeParams p, const __grid_constant__ DecodeMaps maps) {
  using C = DecCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DecBars& bars = *reinterpret_cast<DecBars*>(smem + C::kBar);
  float* acc = reinterpret_cast<float*>(smem + C::kAcc);
  float* red_m = reinterpret_cast<float*>(smem + C::kRed);
  float* red_l = red_m + kConsumers * 16;
  int* prefix = reinterpret_cast<int*>(smem + C::kPrefix);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], kConsumers);
    }
    bars.abort_flag = 0;
    fence_mbar_init();
  }
  // Chunk prefix over the B sequences: a block-wide exclusive scan (each thread
  // sums a contiguous run of sequences, a warp scan plus the warp totals give
  // its offset), O(B / threads) per thread.  The counts are summed in 64 bits;
  // when the parts exceed the workspace capacity the prefix is all zeros (no
  // items, the combine writes empty rows) and block 0 flags BW_ERR_WORKSPACE,
  // so no kernel reads or writes past the workspace.
  {
    const int per = (p.B + kThreads - 1) / kThreads;
    const int b0 = min(tid * per, p.B), b1 = min(b0 + per, p.B);
    long long mine = 0;
    for (int b = b0; b < b1; ++b) {
      const int len = p.kv_lens[b];
      mine += len > 0 ? (len + p.chunk - 1) / p.chunk : 0;
    }
    long long x = mine;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) bars.warp_sum[warp] = x;
    __syncthreads();
    long long before = x - mine, total_c = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      if (w < warp) before += bars.warp_sum[w];
      total_c += bars.warp_sum[w];
    }
    const bool over = total_c * p.Hkv > (long long)p.max_parts;
    for (int b = b0; b < b1; ++b) {
      prefix[b] = over ? 0 : (int)before;
      const int len = p.kv_lens[b];
      before += len > 0 ? (len + p.chunk - 1) / p.chunk : 0;
    }
    if (tid == 0) {
      prefix[p.B] = over ? 0 : (int)total_c;
      bars.total_parts = over ? 0 : (int)(total_c * p.Hkv);
      if (over && blockIdx.x == 0) atomicCAS(p.err, 0, 0x200);
    }
  }
  for (int i = tid; i < 16 * D; i += kThreads) acc[i] = 0.f;
  __syncthreads();
  if (blockIdx.x == 0)
    for (int b = tid; b <= p.B; b += kThreads) p.chunk_prefix[b] = prefix[b];
  const int total = bars.total_parts;
  WaitCtl wc{&bars.abort_flag, p.err, p.timeout_ns, 16 + warp};
  const uint32_t sbase = smem_u32(smem);

  if (warp == kConsumers) {
    // ------------------------------------------------------------ producer
    // For a paged cache the whole warp first copies the item's page indices
    // into shared memory (one coalesced load), so no load waits on the block
    // table; each lane then issues the loads of one page piece of a stage.
    int* bt_cache = reinterpret_cast<int*>(smem + C::kBtCache);
    if (lane == 0) {
      prefetch_tmap(&maps.k);
      prefetch_tmap(&maps.v);
    }
    uint32_t n = 0;
    bool ok = true;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      const DecItem it = dec_item(p, prefix, idx);
      const int len_b = p.kv_lens[it.b];
      const int* bt_b = p.block_table ? p.block_table + (int64_t)it.b * p.max_pages : nullptr;
      int pg0 = 0;
      bool cached = false;
      if (bt_b != nullptr) {
        pg0 = (int)(it.t0 / p.page_size);
        const int pg1 = (int)((it.t1 - 1) / p.page_size);
        cached = pg1 - pg0 + 1 <= kBtCacheEntries;
        if (cached)
          for (int i = pg0 + lane; i <= pg1; i += 32) bt_cache[i - pg0] = bt_b[i];
        __syncwarp();
      }
      // Lane 0 waits for the slot and posts the byte count; then the loads are
      // issued, for a paged cache one page piece per lane.
      for (int64_t t = it.t0; t < it.t1; t += kTok, ++n) {
        const uint32_t s = n % kStages;
        bool got = true;
        if (lane == 0) {
          got = wc.wait(&bars.empty[s], ((n / kStages) & 1) ^ 1);
          if (got) mbar_arrive_expect_tx(&bars.full[s], C::kStage);
        }
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          break;
        }
        uint8_t* dst = smem + s * C::kStage;
        if (bt_b == nullptr) {
          if (lane == 0) {
            tma_load_3d(dst, &maps.k, &bars.full[s], 0, (int)t, it.kvh * (D / 64));
            tma_load_3d(dst + C::kHalf, &maps.v, &bars.full[s], 0, (int)t, it.kvh * (D / 64));
          }
        } else {
          // Paged: the 64-token stage is gathered page piece by page piece
          // (bh = min(64, page_size) rows per box, both panels per load).
          // Pieces past the end of the sequence re-read its last piece (in
          // range; masked by the consumers).
          const int bh = p.page_size < kTok ? p.page_size : kTok;
          const int sub = lane;
          if (sub < kTok / bh) {
            const int last = ((len_b - 1) / bh) * bh;
            int tok = (int)t + sub * bh;
            if (tok > last) tok = last;
            const int pi = tok / p.page_size;
            const int page = cached ? bt_cache[pi - pg0] : bt_b[pi];
            const int row = page * p.page_size + tok % p.page_size;
            const int off = sub * (D / 64) * bh * 128;
            tma_load_3d(dst + off, &maps.k, &bars.full[s], 0, row, it.kvh * (D / 64));
            tma_load_3d(dst + C::kHalf + off, &maps.v, &bars.full[s], 0, row, it.kvh * (D / 64));
          }
        }
      }
      __syncwarp();
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
    }
    if (!ok && lane == 0) {
      // unwinding: wait for the loads already in flight before exiting
      for (uint32_t i = n > kStages ? n - kStages : 0; i < n; ++i)
        drain_wait(&bars.full[i % kStages], (i / kStages) & 1, p.timeout_ns);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2, q4 = lane & 3;
  const float cl2 = p.scale_log2;
  uint32_t n = 0;
  // Shared-memory layout of a K (or V) stage: pieces of bh rows (bh = 64, or
  // the page size below 64), each piece holding its D / 64 panels one after
  // the other (bh x 128 bytes, 128-byte swizzled): token tl, 16-byte chunk c
  // sits at piece(tl) + (c / 8) * bh * 128 + (tl % bh) * 128 + ((c % 8) ^ (tl % 8)) * 16.
  const int bh = (p.block_table != nullptr && p.page_size < kTok) ? p.page_size : kTok;
  const uint32_t panel_b = (uint32_t)bh * 128;
  auto tok_off = [&](int tl) -> uint32_t {
    return (uint32_t)(tl / bh) * (D / 64) * panel_b + (uint32_t)(tl % bh) * 128;
  };
  uint32_t k_off[2], v_off;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) k_off[nt] = tok_off(warp * 16 + nt * 8 + (lane & 7));
  v_off = tok_off(warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7));
  bool ok = true;
  for (int idx = blockIdx.x; ok && idx < total; idx += gridDim.x) {
    const DecItem it = dec_item(p, prefix, idx);
    // Q fragments: A[16 x 16] per k-step, rows >= G are zero.
    uint32_t qa[D / 16][4];
    {
      const __nv_bfloat16* Q = reinterpret_cast<const __nv_bfloat16*>(p.Q) + it.b * p.q_sb;
      const int h0 = it.kvh * p.G;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int k0 = ks * 16 + q4 * 2;
        qa[ks][0] = g < p.G ? *reinterpret_cast<const uint32_t*>(Q + (h0 + g) * p.q_sh + k0) : 0u;
        qa[ks][1] = g + 8 < p.G ? *reinterpret_cast<const uint32_t*>(Q + (h0 + g + 8) * p.q_sh + k0) : 0u;
        qa[ks][2] = g < p.G ? *reinterpret_cast<const uint32_t*>(Q + (h0 + g) * p.q_sh + k0 + 8) : 0u;
        qa[ks][3] = g + 8 < p.G ? *reinterpret_cast<const uint32_t*>(Q + (h0 + g + 8) * p.q_sh + k0 + 8) : 0u;
      }
    }
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

    for (int64_t t = it.t0; t < it.t1; t += kTok, ++n) {
      const uint32_t s = n % kStages;
      // On a timeout the warp still runs this item's merge below, so that the
      // named barriers stay matched across the consumer warps, then stops.
      if (!wc.wait(&bars.full[s], (n / kStages) & 1)) { ok = false; break; }
      const int64_t tw = t + warp * 16;         // first token of this warp's slice
      if (tw < it.t1) {
        const uint32_t kb = sbase + s * C::kStage;
        const uint32_t vb = kb + C::kHalf;
        // S = Q K^T for 16 tokens (two n8 tiles)
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int tl = warp * 16 + nt * 8 + (lane & 7);
#pragma unroll
          for (int qq = 0; qq < D / 32; ++qq) {
            const int chunk = qq * 4 + (lane >> 3);
            const uint32_t addr = kb + k_off[nt] + (chunk >> 3) * panel_b + (((chunk & 7) ^ (tl & 7)) << 4);
            uint32_t r[4];
            ldsm_x4(addr, r);
            mma_bf16_16816(sacc[nt], qa[2 * qq], r[0], r[1]);
            mma_bf16_16816(sacc[nt], qa[2 * qq + 1], r[2], r[3]);
          }
        }
        // mask tokens past the end of the chunk
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t tok = tw + nt * 8 + q4 * 2 + (e & 1);
            if (tok >= it.t1) sacc[nt][e] = -INFINITY;
          }
        // online softmax for rows g (e = 0,1) and g + 8 (e = 2,3)
        float pr[2][4];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          float mx = fmaxf(fmaxf(sacc[0][2 * rr], sacc[0][2 * rr + 1]), fmaxf(sacc[1][2 * rr], sacc[1][2 * rr + 1]));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float mc = mx * cl2;
          if (mc > m_run[rr] + 8.f) {
            const float corr = ex2f(m_run[rr] - mc);
            m_run[rr] = mc;
            l_run[rr] *= corr;
#pragma unroll
            for (int i = 0; i < D / 8; ++i) {
              o[i][2 * rr] *= corr;
              o[i][2 * rr + 1] *= corr;
            }
          }
          const float msub = m_run[rr] == -INFINITY ? 0.f : m_run[rr];
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            pr[nt][2 * rr] = ex2f(fmaf(sacc[nt][2 * rr], cl2, -msub));
            pr[nt][2 * rr + 1] = ex2f(fmaf(sacc[nt][2 * rr + 1], cl2, -msub));
            l_run[rr] += pr[nt][2 * rr] + pr[nt][2 * rr + 1];
          }
        }
        uint32_t pa[4];
        pa[0] = pack2(pr[0][0], pr[0][1]);
        pa[1] = pack2(pr[0][2], pr[0][3]);
        pa[2] = pack2(pr[1][0], pr[1][1]);
        pa[3] = pack2(pr[1][2], pr[1][3]);
        // O += P V  (V via transposed ldmatrix)
#pragma unroll
        for (int e = 0; e < D / 16; ++e) {
          const int mi = lane >> 3;
          const int tl = warp * 16 + (mi & 1) * 8 + (lane & 7);
          const int chunk = 2 * e + (mi >> 1);
          const uint32_t addr = vb + v_off + (chunk >> 3) * panel_b + (((chunk & 7) ^ (tl & 7)) << 4);
          uint32_t r[4];
          ldsm_x4_t(addr, r);
          mma_bf16_16816(o[2 * e], pa, r[0], r[1]);
          mma_bf16_16816(o[2 * e + 1], pa, r[2], r[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.empty[s]);
    }

    // ---- merge the four warps' partial softmax states for this item
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 1);
      l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 2);
    }
    if (q4 == 0) {
      red_m[warp * 16 + g] = m_run[0];
      red_m[warp * 16 + g + 8] = m_run[1];
      red_l[warp * 16 + g] = l_run[0];
      red_l[warp * 16 + g + 8] = l_run[1];
    }
    consumer_sync();
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = g + 8 * rr;
      if (row >= p.G) continue;
      float M = -INFINITY;
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, red_m[w * 16 + row]);
      const float f = m_run[rr] == -INFINITY ? 0.f : ex2f(m_run[rr] - M);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        atomicAdd(&acc[row * D + i * 8 + q4 * 2], o[i][2 * rr] * f);
        atomicAdd(&acc[row * D + i * 8 + q4 * 2 + 1], o[i][2 * rr + 1] * f);
      }
    }
    consumer_sync();
    for (int i = tid; i < p.G * D; i += kConsumers * 32) {
      const int row = i / D;
      float M = -INFINITY;
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, red_m[w * 16 + row]);
      float Ls = 0.f;
      for (int w = 0; w < kConsumers; ++w) {
        const float mw = red_m[w * 16 + row];
        if (mw != -INFINITY) Ls += red_l[w * 16 + row] * ex2f(mw - M);
      }
      p.o_part[(int64_t)it.part * p.G * D + i] = acc[i] / Ls;
      acc[i] = 0.f;
      if ((i % D) == 0) p.lse_part[(int64_t)it.part * p.G + row] = (M + __log2f(Ls)) * 0.69314718055994531f;
    }
    consumer_sync();
    if (*wc.abort_flag) ok = false;
  }
}

// One warp per (b, hq).  Two passes over the splits: the max LSE, then the
// weighted sum with weights e^{LSE_i - LSE*}.
__global__ void __launch_bounds__(128) lse_combine_kernel(const CombineParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.B * p.Hq) return;
  const int b = warp / p.Hq, hq = warp - b * p.Hq;
  const int kvh = hq / p.G, gi = hq - kvh * p.G;
  int nsp;
  int64_t base_part = 0;
  if (p.chunk_prefix) {
    base_part = p.chunk_prefix[b];
    nsp = p.chunk_prefix[b + 1] - p.chunk_prefix[b];
  } else {
    nsp = p.splits;
  }
  auto lse_at = [&](int i) -> float {
    if (p.chunk_prefix) return p.lse_part[((base_part + i) * p.Hkv + kvh) * p.G + gi];
    return p.lse_part[(int64_t)i * p.lse_split_stride + (int64_t)b * p.Hq + hq];
  };
  auto o_at = [&](int i) -> const float* {
    if (p.chunk_prefix) return p.o_part + (((base_part + i) * p.Hkv + kvh) * p.G + gi) * p.D;
    return p.o_part + (int64_t)i * p.o_split_stride + ((int64_t)b * p.Hq + hq) * p.D;
  };
  float mx = -INFINITY;
  for (int i = lane; i < nsp; i += 32) mx = fmaxf(mx, lse_at(i));
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float msafe = mx == -INFINITY ? 0.f : mx;
  float accv[4] = {0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  const int d0 = lane * 4;
  for (int i = 0; i < nsp; ++i) {
    const float l = lse_at(i);
    const float w = l == -INFINITY ? 0.f : __expf(l - msafe);
    wsum += w;
    if (d0 < p.D) {
      const float4 v = *reinterpret_cast<const float4*>(o_at(i) + d0);
      accv[0] += w * v.x; accv[1] += w * v.y; accv[2] += w * v.z; accv[3] += w * v.w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  if (d0 < p.D) {
    if (p.o_fp32) {
      float* O = reinterpret_cast<float*>(p.O) + b * p.o_sb + hq * p.o_sh + d0;
      *reinterpret_cast<float4*>(O) = make_float4(accv[0] * inv, accv[1] * inv, accv[2] * inv, accv[3] * inv);
    } else {
      __nv_bfloat16* O = reinterpret_cast<__nv_bfloat16*>(p.O) + b * p.o_sb + hq * p.o_sh + d0;
      uint2 u = make_uint2(pack2(accv[0] * inv, accv[1] * inv), pack2(accv[2] * inv, accv[3] * inv));
      *reinterpret_cast<uint2*>(O) = u;
    }
  }
  if (p.LSE && lane == 0) p.LSE[(int64_t)b * p.Hq + hq] = wsum > 0.f ? msafe + __logf(wsum) : -INFINITY;
}

template <int D>
cudaError_t launch_decode_impl(const DecodeParams& p, const DecodeMaps& maps, int num_sms, cudaStream_t stream) {
  using C = DecCfg<D>;
  const int bytes = C::kPrefix + (p.B + 1) * 4 + 1024;
  auto kern = decode_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, bytes);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  kern<<<num_sms * per_sm, kThreads, bytes, stream>>>(p, maps);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode(const DecodeParams& p, const DecodeMaps& maps, int num_sms, cudaStream_t stream) {
  if (p.B > kMaxB || p.G > 16) return cudaErrorInvalidValue;
  if (p.D == 128) return launch_decode_impl<128>(p, maps, num_sms, stream);
  if (p.D == 64) return launch_decode_impl<64>(p, maps, num_sms, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_lse_combine(const CombineParams& p, cudaStream_t stream) {
  if (p.D % 4 != 0 || p.D > 128) return cudaErrorInvalidValue;
  const int warps = p.B * p.Hq;
  const int blocks = (warps + 3) / 4;
  if (blocks == 0) return cudaSuccess;
  lse_combine_kernel<<<blocks, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace bw
