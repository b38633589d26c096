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
// Memory-bound: one warp per (b, h, token) row, each lane holding D/32
// consecutive elements (8 bytes at D = 128); the NeoX partner of a lane's
// elements sits D/2 elements away, i.e. in lane l ^ 16, fetched with one
// shuffle.  Grid-stride over rows, grid sized to the SM count.
#include <cuda_bf16.h>

#include "kernels.h"

namespace bw {
namespace {

template <int D, bool NEOX>
__global__ void __launch_bounds__(256) norm_rope_kernel(const NormRopeParams p) {
  constexpr int PER = D / 32;  // elements per lane: 2 (D=64) or 4 (D=128)
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t rows = (int64_t)p.B * p.H * p.S;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps_total) {
    const int s = (int)(r % p.S);
    const int64_t bh = r / p.S;
    const int h = (int)(bh % p.H);
    const int b = (int)(bh / p.H);
    const __nv_bfloat16* in = reinterpret_cast<const __nv_bfloat16*>(p.in) + b * p.in_sb + h * p.in_sh +
                              (int64_t)s * p.in_ss + lane * PER;
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out) + b * p.out_sb + h * p.out_sh +
                         (int64_t)s * p.out_ss + lane * PER;
    float x[PER];
    if constexpr (PER == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(in);
      const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
      const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
      x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(c); x[3] = __high2float(c);
    } else {
      const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(in);
      x[0] = __low2float(a); x[1] = __high2float(a);
    }
    if (p.gamma != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
      for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float rstd = rsqrtf(ss / (float)D + p.eps);
      if (p.rstd != nullptr && lane == 0) p.rstd[r] = rstd;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        x[i] = __bfloat162float(__float2bfloat16(x[i] * rstd * p.gamma[lane * PER + i]));
    }
    const int pos = s + p.pos_offset;
    if (pos >= 0 && pos < p.cache_seq_len) {
      const float* cs = p.cache + (int64_t)pos * D;
      if constexpr (NEOX) {
        // element d = lane*PER + i pairs with d +- D/2, held by lane +- 16
        float y[PER];
#pragma unroll
        for (int i = 0; i < PER; ++i) y[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
        const bool first = lane < 16;  // holds the "a" element of the pair
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int pi = (lane & 15) * PER + i;  // pair index in [0, D/2)
          const float c = cs[pi], sn = cs[D / 2 + pi];
          const float a = first ? x[i] : y[i];
          const float bb = first ? y[i] : x[i];
          x[i] = first ? (a * c - bb * sn) : (a * sn + bb * c);
        }
      } else {
#pragma unroll
        for (int i = 0; i < PER; i += 2) {
          const int pi = (lane * PER + i) >> 1;
          const float c = cs[pi], sn = cs[D / 2 + pi];
          const float a = x[i], bb = x[i + 1];
          x[i] = a * c - bb * sn;
          x[i + 1] = a * sn + bb * c;
        }
      }
    }
    if constexpr (PER == 4) {
      __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
      __nv_bfloat162 c = __floats2bfloat162_rn(x[2], x[3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&a);
      u.y = *reinterpret_cast<uint32_t*>(&c);
      *reinterpret_cast<uint2*>(out) = u;
    } else {
      *reinterpret_cast<__nv_bfloat162*>(out) = __floats2bfloat162_rn(x[0], x[1]);
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
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)num_sms * 8;
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
