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
// HBM-bound streaming kernel.  Each lane holds two 16-byte chunks (16
// elements) of a row, so a row spans LPR = D/16 lanes and one warp covers RPI =
// 32/LPR rows.  A warp task is RPI consecutive positions of one sequence over
// all H heads: each lane's position is fixed for the task, so its 8 cos and 8
// sin values are read once per task (not once per row), and the kGroups heads
// in flight are RPI neighbouring rows each (contiguous in BHSD, adjacent runs
// in BSHD).  The NeoX partner of a lane's elements is in the same lane (its
// two chunks are D/2 elements apart); GPT-J pairs are inside a chunk.  The
// row's norm is a shuffle reduction over its LPR lanes.  Grid-stride over
// tasks, grid sized to the SM count.
#include <cuda_bf16.h>

#include "kernels.h"

namespace bw {
namespace {

constexpr int kGroups = 2;       // heads (two 16-byte loads per lane each) in flight per warp
constexpr int kMinBlocks = 4;    // 256-thread blocks per SM (64 registers per thread)

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int D, bool NEOX>
__global__ void __launch_bounds__(256, kMinBlocks) norm_rope_kernel(const NormRopeParams p) {
  constexpr int NCH = D / 8;           // 16-byte chunks per row
  constexpr int LPR = NCH / 2;         // lanes per row: two chunks per lane
  constexpr int RPI = 32 / LPR;        // rows (positions) per warp instruction
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;          // lane within its row
  // NeoX: chunks sub and sub + NCH/2 (each element's rotation partner is in the
  // same lane); interleaved: chunks 2 sub, 2 sub + 1 (pairs inside a chunk).
  const int c0 = NEOX ? sub : 2 * sub, c1 = NEOX ? sub + NCH / 2 : 2 * sub + 1;
  const int ci = 8 * sub;              // first cos / sin index this lane uses (8 of them)
  const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);
  const int nsb = (p.S + RPI - 1) / RPI;                 // position blocks per sequence
  const uint32_t tasks = (uint32_t)p.B * nsb;
  // A warp task is RPI consecutive positions of one sequence, all H heads: the
  // lane's position, and so its cos / sin, is fixed for the whole task (read
  // once), and the kGroups heads in flight are RPI contiguous rows each.
  for (uint32_t task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks; task += warps_total) {
    const int b = (int)(task / (uint32_t)nsb);
    const int s = (int)(task - (uint32_t)b * nsb) * RPI + lane / LPR;
    const bool valid = s < p.S;
    const int pos = s + p.pos_offset;
    const bool rope = valid && pos >= 0 && pos < p.cache_seq_len;
    float c[8], sn[8];
    if (rope) {
      const float* cs = p.cache + (int64_t)pos * D;
      const float4 ca = ldg4(cs + ci), cb = ldg4(cs + ci + 4);
      const float4 sa = ldg4(cs + D / 2 + ci), sb = ldg4(cs + D / 2 + ci + 4);
      c[0] = ca.x; c[1] = ca.y; c[2] = ca.z; c[3] = ca.w; c[4] = cb.x; c[5] = cb.y; c[6] = cb.z; c[7] = cb.w;
      sn[0] = sa.x; sn[1] = sa.y; sn[2] = sa.z; sn[3] = sa.w; sn[4] = sb.x; sn[5] = sb.y; sn[6] = sb.z; sn[7] = sb.w;
    }
    for (int h0 = 0; h0 < p.H; h0 += kGroups) {
      uint4 raw[kGroups][2];
#pragma unroll
      for (int u = 0; u < kGroups; ++u) {
        const int h = h0 + u;
        if (valid && h < p.H) {
          const __nv_bfloat16* src =
              reinterpret_cast<const __nv_bfloat16*>(p.in) + b * p.in_sb + h * p.in_sh + (int64_t)s * p.in_ss;
          raw[u][0] = *reinterpret_cast<const uint4*>(src + 8 * c0);
          raw[u][1] = *reinterpret_cast<const uint4*>(src + 8 * c1);
        } else {
          raw[u][0] = raw[u][1] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < kGroups; ++u) {
        const int h = h0 + u;
        float x[16];
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          const uint32_t w4[4] = {raw[u][hc].x, raw[u][hc].y, raw[u][hc].z, raw[u][hc].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            x[8 * hc + 2 * i] = __uint_as_float(w4[i] << 16);
            x[8 * hc + 2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
          }
        }
        if (p.gamma != nullptr) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
          for (int off = LPR / 2; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
          const float rstd = rsqrtf(ss * (1.f / (float)D) + p.eps);   // D is a power of two: exact
          if (p.rstd != nullptr && sub == 0 && valid && h < p.H)
            p.rstd[((int64_t)b * p.H + h) * p.S + s] = rstd;
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {
            const int e = 8 * (hc ? c1 : c0);
            const float4 g0 = ldg4(p.gamma + e), g1 = ldg4(p.gamma + e + 4);
            const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              const uint32_t v = pack2(x[8 * hc + i] * rstd * g[i], x[8 * hc + i + 1] * rstd * g[i + 1]);   // bf16
              x[8 * hc + i] = __uint_as_float(v << 16);
              x[8 * hc + i + 1] = __uint_as_float(v & 0xffff0000u);
            }
          }
        }
        if (rope) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            // NeoX: element i of chunk c0 pairs with element i of chunk c1;
            // interleaved: elements 2i and 2i + 1 of the lane's 16
            const int ia = NEOX ? i : 2 * i, ib = NEOX ? 8 + i : 2 * i + 1;
            const float av = x[ia], bv = x[ib];
            x[ia] = av * c[i] - bv * sn[i];
            x[ib] = av * sn[i] + bv * c[i];
          }
        }
        if (valid && h < p.H) {
          __nv_bfloat16* dst =
              reinterpret_cast<__nv_bfloat16*>(p.out) + b * p.out_sb + h * p.out_sh + (int64_t)s * p.out_ss;
          *reinterpret_cast<uint4*>(dst + 8 * c0) =
              make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
          *reinterpret_cast<uint4*>(dst + 8 * c1) =
              make_uint4(pack2(x[8], x[9]), pack2(x[10], x[11]), pack2(x[12], x[13]), pack2(x[14], x[15]));
        }
      }
    }
  }
}

}  // namespace


cudaError_t launch_norm_rope(const NormRopeParams& p, int num_sms, cudaStream_t stream) {
  const int64_t rows = (int64_t)p.B * p.H * p.S;
  if (rows == 0) return cudaSuccess;
  const int64_t rpi = 32 / (p.D / 16);                       // positions per warp task
  const int64_t tasks = (int64_t)p.B * ((p.S + rpi - 1) / rpi);
  int64_t blocks = (tasks + 7) / 8;                          // 8 warps per block
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
