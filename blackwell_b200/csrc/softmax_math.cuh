// Arithmetic helpers for the online softmax: paired fp32 (f32x2) FMA/ADD,
// three-input max, and a software exp2 that runs on the FMA pipe so that part of
// the exponentials bypass the MUFU unit.
//
// Software exp2 (Cody-Waite style range reduction + polynomial, the split used
// by FlashAttention-4 to balance MUFU and FMA throughput):
//   x  = max(x, -126)                      (keeps the exponent add in range)
//   t  = x + 1.5*2^23                      (round-to-nearest integer n in the low mantissa bits)
//   f  = x - (t - 1.5*2^23)   in [-0.5, 0.5]
//   p  = 1 + f*(a1 + f*(a2 + f*a3))       ~ 2^f
//   2^x = bits(p) + (bits(t) << 23)       (adds n to p's exponent field)
// a1..a3 were fitted for this library by iteratively re-weighted least squares
// on the relative error of 2^f over [-0.5, 0.5] with p(0) = 1 fixed; max
// relative error 1.02e-4 (checked in fp32, tests/test_exp2_poly.py), below the
// 3.9e-3 step of the bf16 P that consumes it.
#pragma once
#include <cstdint>

namespace bw {

struct f2 {
  float x, y;
};

#ifdef BW_SCALAR_F2
__device__ __forceinline__ f2 ffma2(f2 a, f2 b, f2 c) { return f2{fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y)}; }
__device__ __forceinline__ f2 fadd2(f2 a, f2 b) { return f2{a.x + b.x, a.y + b.y}; }
__device__ __forceinline__ f2 fsub2(f2 a, f2 b) { return f2{a.x - b.x, a.y - b.y}; }
#else
__device__ __forceinline__ f2 ffma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ f2 fadd2(f2 a, f2 b) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ f2 fsub2(f2 a, f2 b) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
#endif
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kExpA1 = 0.6932830810546875f;
constexpr float kExpA2 = 0.24220921099185944f;
constexpr float kExpA3 = 0.05500814691185951f;
constexpr float kRound = 12582912.0f;  // 1.5 * 2^23

// 2^x for a pair of values on the FMA/ALU pipes.
__device__ __forceinline__ f2 ex2_poly2(f2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const f2 t = fadd2(x, f2{kRound, kRound});
  const f2 j = fsub2(t, f2{kRound, kRound});
  const f2 f = fsub2(x, j);
  f2 p = ffma2(f, f2{kExpA3, kExpA3}, f2{kExpA2, kExpA2});
  p = ffma2(p, f, f2{kExpA1, kExpA1});
  p = ffma2(p, f, f2{1.f, 1.f});
  f2 r;
  r.x = __uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23));
  r.y = __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23));
  return r;
}

}  // namespace bw
