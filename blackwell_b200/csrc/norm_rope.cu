// QK-norm (RMSNorm over the head dimension) + rotary position embedding, the
// prologue of the reference's fused attention op
// (src/SM103/attention/GQA_fused_sm103.cu:59-104, ground truth :328-420):
//   rstd  = 1 / sqrt(mean(x^2) + eps)
//   x_hat = bf16(x * rstd * gamma[d])            (skipped when gamma == null)
//   RoPE at position p = token + pos_offset, if 0 <= p < cache_seq_len:
//     pairs (i, i + D/2) (NeoX) or (2i, 2i + 1) (GPT-J interleaved), i < D/2,
//     c = cache[p][i], s = cache[p][D/2 + i]  (fp32 cos | sin cache [len, D])
//     a' = bf16(a c - b s),  b' = bf16(a s + b c)
// fp32 math, bf16 storage, a bf16 rounding between norm and RoPE as in the
// reference.  Optional per-row rstd output (fp32, [B, H, S]).
//
// HBM-bound streaming kernel.  Each lane holds 8 consecutive elements of a row
// (one 16-byte load and store), so a row spans LPR = D/8 lanes and one warp
// instruction covers 32/LPR rows (512 bytes); a warp keeps kGroups such
// instructions in flight before any arithmetic.  The NeoX partner of a lane's
// elements sits D/2 elements away, in lane l ^ (LPR/2) (one shuffle); GPT-J
// pairs are inside a lane.  The row's norm is a shuffle reduction over its LPR
// lanes.  cos/sin are read with 16-byte loads (the cache is 16-byte aligned and
// a row is D*4 bytes).  Grid-stride over row groups, grid sized to the SM count.
#include <cuda_bf16.h>

#include "kernels.h"

namespace bw {
namespace {

constexpr int kGroups = 4;       // row groups (warp-wide 512-byte loads) in flight per warp
constexpr int kMinBlocks = 4;    // 256-thread blocks per SM (64 registers per thread)

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int D, bool NEOX>
__global__ void __launch_bounds__(256, kMinBlocks) norm_rope_kernel(const NormRopeParams p) {
  constexpr int LPR = D / 8;           // lanes per row
  constexpr int RPI = 32 / LPR;        // rows per warp instruction
  constexpr int RPW = RPI * kGroups;   // rows per warp iteration
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;          // lane within its row
  const int e0 = sub * 8;              // first element held
  const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);
  const uint32_t rows = (uint32_t)p.B * p.H * p.S;   // < 2^31, checked by the caller

  for (uint32_t base = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW; base < rows;
       base += warps_total * RPW) {
    uint4 raw[kGroups];
    int64_t out_off[kGroups];
    int pos[kGroups];
    uint32_t rs_idx[kGroups];  // [B, H, S] index of the row (rstd output)
    // Rows are enumerated (b, s, h) with h fastest, so the rows in flight share
    // few positions and their cos/sin reads hit L1.  (b, s, h) of this lane's
    // first row by division, the later ones by stepping h forward RPI at a time.
    uint32_t r = base + lane / LPR;
    if (r >= rows) r = rows - 1;
    uint32_t bs = r / (uint32_t)p.H;
    int h = (int)(r - bs * (uint32_t)p.H);
    int b = (int)(bs / (uint32_t)p.S);
    int s = (int)(bs - (uint32_t)b * p.S);
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      if (u > 0 && base + u * RPI + lane / LPR < rows) {
        h += RPI;
        while (h >= p.H) {
          h -= p.H;
          if (++s == p.S) { s = 0; ++b; }
        }
      }
      raw[u] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.in) + b * p.in_sb +
                                               h * p.in_sh + (int64_t)s * p.in_ss + e0);
      out_off[u] = b * p.out_sb + h * p.out_sh + (int64_t)s * p.out_ss + e0;
      pos[u] = s + p.pos_offset;
      rs_idx[u] = ((uint32_t)b * p.H + h) * (uint32_t)p.S + s;
    }
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      const uint32_t r = base + u * RPI + lane / LPR;
      float x[8];
      {
        const uint32_t w4[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[2 * i] = __uint_as_float(w4[i] << 16);
          x[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
        }
      }
      if (p.gamma != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
        for (int off = LPR / 2; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float rstd = rsqrtf(ss * (1.f / (float)D) + p.eps);   // D is a power of two: exact
        if (p.rstd != nullptr && sub == 0 && r < rows) p.rstd[rs_idx[u]] = rstd;
        const float4 g0 = ldg4(p.gamma + e0), g1 = ldg4(p.gamma + e0 + 4);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const uint32_t v = pack2(x[i] * rstd * g[i], x[i + 1] * rstd * g[i + 1]);   // bf16 rounding
          x[i] = __uint_as_float(v << 16);
          x[i + 1] = __uint_as_float(v & 0xffff0000u);
        }
      }
      const bool rot = pos[u] >= 0 && pos[u] < p.cache_seq_len;
      const float* cs = p.cache + (int64_t)(rot ? pos[u] : 0) * D;
      if constexpr (NEOX) {
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = __shfl_xor_sync(0xffffffffu, x[i], LPR / 2);
        if (rot) {
          // lanes with d < D/2 hold a (x' = a c - b s), the others b (x' = a s + b c):
          // both are x' = x c + y s' with s' = -s in the first half, y the partner
          const bool first = sub < LPR / 2;
          const int i0 = first ? e0 : e0 - D / 2;
          const float4 c0 = ldg4(cs + i0), c1 = ldg4(cs + i0 + 4);
          const float4 s0 = ldg4(cs + D / 2 + i0), s1 = ldg4(cs + D / 2 + i0 + 4);
          const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          const float sg = first ? -1.f : 1.f;
          const float sn[8] = {s0.x * sg, s0.y * sg, s0.z * sg, s0.w * sg, s1.x * sg, s1.y * sg, s1.z * sg, s1.w * sg};
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = x[i] * c[i] + y[i] * sn[i];
        }
      } else {
        if (rot) {
          const float4 c = ldg4(cs + e0 / 2), sn = ldg4(cs + D / 2 + e0 / 2);
          const float cc[4] = {c.x, c.y, c.z, c.w}, ss4[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a = x[2 * i], bb = x[2 * i + 1];
            x[2 * i] = a * cc[i] - bb * ss4[i];
            x[2 * i + 1] = a * ss4[i] + bb * cc[i];
          }
        }
      }
      if (r < rows)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + out_off[u]) =
            make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
    }
  }
}

// fp32 -> bf16 (round to nearest even), 4 elements per thread, grid-stride.
__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* src, int64_t sb, int64_t sh, int64_t ss,
                                                          __nv_bfloat16* dst, int B, int H, int S, int D) {
  const int64_t quads = (int64_t)B * H * S * D / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 4;
    const int d = (int)(e % D);
    const int64_t r = e / D;
    const int s = (int)(r % S);
    const int64_t bh = r / S;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const float4 v = *reinterpret_cast<const float4*>(src + b * sb + h * sh + (int64_t)s * ss + d);
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst + e) = u;
  }
}

}  // namespace

cudaError_t launch_f32_to_bf16(const float* src, int64_t sb, int64_t sh, int64_t ss, void* dst, int B, int H, int S,
                               int D, int num_sms, cudaStream_t stream) {
  const int64_t quads = (int64_t)B * H * S * D / 4;
  if (quads == 0) return cudaSuccess;
  int64_t blocks = (quads + 255) / 256;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  f32_to_bf16_kernel<<<(int)blocks, 256, 0, stream>>>(src, sb, sh, ss, static_cast<__nv_bfloat16*>(dst), B, H, S, D);
  return cudaGetLastError();
}

cudaError_t launch_norm_rope(const NormRopeParams& p, int num_sms, cudaStream_t stream) {
  const int64_t rows = (int64_t)p.B * p.H * p.S;
  if (rows == 0) return cudaSuccess;
  const int64_t rows_per_block = 8 * (32 / (p.D / 8)) * kGroups;
  int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)num_sms * kMinBlocks;
  if (blocks > cap) blocks = cap;
  if (p.D == 128) {
    if (p.neox) norm_rope_kernel<128, true><<<(int)blocks, 256, 0, stream>>>(p);
    else norm_rope_kernel<128, false><<<(int)blocks, 256, 0, stream>>>(p);
  } else if (p.D == 64) {
    if (p.neox) norm_rope_kernel<64, true><<<(int)blocks, 256, 0, stream>>>(p);
    else norm_rope_kernel<64, false><<<(int)blocks, 256, 0, stream>>>(p);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace bw
