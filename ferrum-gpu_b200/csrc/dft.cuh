// Register-resident forward DFT building blocks (radix 2, 4, 8, 16, 32) on
// interleaved complex64 values held as float2.
//
// Every dft<R>(u) takes u[0..R) in natural order and leaves X[0..R) in natural
// order, X[k] = sum_n u[n] * exp(-2*pi*i*n*k/R) — the forward sign convention
// of the reference (crates/ferrum-gpu-fft/src/plan.rs:7-13). Radix 8 is a
// radix-2 split over two radix-4 DFTs; radix 16 is the 4 x 4 split
//   X[k1 + 4 k2] = sum_n2 W4^(n2 k2) W16^(n2 k1) sum_n1 u[4 n1 + n2] W4^(n1 k1);
// radix 32 is a radix-2 split over two radix-16 DFTs. The constants are cos
// and sin of pi/4, pi/8, pi/16 and 3 pi/16.
#pragma once

#include <cuda_runtime.h>
#include <math.h>

#include "plan.h"

namespace ferrum {

FERRUM_HD __forceinline__ float2 c_add(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
FERRUM_HD __forceinline__ float2 c_sub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
// a * w (complex)
FERRUM_HD __forceinline__ float2 c_mul(float2 a, float2 w) {
  return make_float2(fmaf(a.x, w.x, -a.y * w.y), fmaf(a.x, w.y, a.y * w.x));
}
// a * (-i)
FERRUM_HD __forceinline__ float2 c_mul_neg_i(float2 a) { return make_float2(a.y, -a.x); }

constexpr float kCos4 = 0.70710678118654752440f;   // cos(pi/4)
constexpr float kCos8 = 0.92387953251128675613f;   // cos(pi/8)
constexpr float kSin8 = 0.38268343236508977173f;   // sin(pi/8)

// a * exp(-i*pi/4) = c * ((x + y) + i (y - x))
FERRUM_HD __forceinline__ float2 c_mul_w8_1(float2 a) {
  return make_float2(kCos4 * (a.x + a.y), kCos4 * (a.y - a.x));
}
// a * exp(-3i*pi/4) = c * ((y - x) - i (x + y))
FERRUM_HD __forceinline__ float2 c_mul_w8_3(float2 a) {
  return make_float2(kCos4 * (a.y - a.x), -kCos4 * (a.x + a.y));
}

FERRUM_HD __forceinline__ void dft2(float2 (&u)[2]) {
  float2 a = u[0], b = u[1];
  u[0] = c_add(a, b);
  u[1] = c_sub(a, b);
}

FERRUM_HD __forceinline__ void dft4_vals(float2& a, float2& b, float2& c, float2& d) {
  float2 t0 = c_add(a, c), t1 = c_sub(a, c);
  float2 t2 = c_add(b, d), t3 = c_mul_neg_i(c_sub(b, d));
  a = c_add(t0, t2);
  c = c_sub(t0, t2);
  b = c_add(t1, t3);
  d = c_sub(t1, t3);
}

FERRUM_HD __forceinline__ void dft4(float2 (&u)[4]) { dft4_vals(u[0], u[1], u[2], u[3]); }

FERRUM_HD __forceinline__ void dft8(float2 (&u)[8]) {
  float2 e0 = u[0], e1 = u[2], e2 = u[4], e3 = u[6];
  float2 o0 = u[1], o1 = u[3], o2 = u[5], o3 = u[7];
  dft4_vals(e0, e1, e2, e3);
  dft4_vals(o0, o1, o2, o3);
  o1 = c_mul_w8_1(o1);
  o2 = c_mul_neg_i(o2);
  o3 = c_mul_w8_3(o3);
  u[0] = c_add(e0, o0); u[4] = c_sub(e0, o0);
  u[1] = c_add(e1, o1); u[5] = c_sub(e1, o1);
  u[2] = c_add(e2, o2); u[6] = c_sub(e2, o2);
  u[3] = c_add(e3, o3); u[7] = c_sub(e3, o3);
}

FERRUM_HD __forceinline__ void dft16(float2 (&u)[16]) {
  // Column DFT-4s over n1 for each n2; result Y[n2][k1] in slot n2 + 4*k1.
  dft4_vals(u[0], u[4], u[8], u[12]);
  dft4_vals(u[1], u[5], u[9], u[13]);
  dft4_vals(u[2], u[6], u[10], u[14]);
  dft4_vals(u[3], u[7], u[11], u[15]);
  // Twiddles W16^(n2*k1).
  const float2 w1 = make_float2(kCos8, -kSin8);   // W16^1
  const float2 w3 = make_float2(kSin8, -kCos8);   // W16^3
  const float2 w9 = make_float2(-kCos8, kSin8);   // W16^9
  u[5] = c_mul(u[5], w1);          // n2=1,k1=1
  u[9] = c_mul_w8_1(u[9]);         // n2=1,k1=2: W16^2
  u[13] = c_mul(u[13], w3);        // n2=1,k1=3
  u[6] = c_mul_w8_1(u[6]);         // n2=2,k1=1: W16^2
  u[10] = c_mul_neg_i(u[10]);      // n2=2,k1=2: W16^4
  u[14] = c_mul_w8_3(u[14]);       // n2=2,k1=3: W16^6
  u[7] = c_mul(u[7], w3);          // n2=3,k1=1
  u[11] = c_mul_w8_3(u[11]);       // n2=3,k1=2: W16^6
  u[15] = c_mul(u[15], w9);        // n2=3,k1=3
  // Row DFT-4s over n2 for each k1; output k2 lands in slot 4*k1 + k2.
  dft4_vals(u[0], u[1], u[2], u[3]);
  dft4_vals(u[4], u[5], u[6], u[7]);
  dft4_vals(u[8], u[9], u[10], u[11]);
  dft4_vals(u[12], u[13], u[14], u[15]);
  // X[k1 + 4 k2] = slot[4 k1 + k2]: a 4 x 4 transpose of the slots.
  float2 t;
  t = u[1]; u[1] = u[4]; u[4] = t;
  t = u[2]; u[2] = u[8]; u[8] = t;
  t = u[3]; u[3] = u[12]; u[12] = t;
  t = u[6]; u[6] = u[9]; u[9] = t;
  t = u[7]; u[7] = u[13]; u[13] = t;
  t = u[11]; u[11] = u[14]; u[14] = t;
}

// cos / sin of pi/16 and 3*pi/16.
constexpr float kCos16 = 0.98078528040323044913f;
constexpr float kSin16 = 0.19509032201612826785f;
constexpr float kCos3_16 = 0.83146961230254523708f;
constexpr float kSin3_16 = 0.55557023301960222474f;

// a * W32^j (W32 = exp(-2 pi i / 32)). Meant for exponents that are
// compile-time constants after unrolling: quarter turns are swaps and sign
// changes, other angles multiply by constants of the first octant moved by
// symmetry (cos / sin of 2 pi r / 32 for r <= 4 are 1, kCos16, kCos8,
// kCos3_16, kCos4 and 0, kSin16, kSin8, kSin3_16, kCos4).
FERRUM_HD __forceinline__ float2 c_mul_w32(float2 a, int j) {
  j &= 31;
  if (j == 0) return a;
  if (j == 8) return make_float2(a.y, -a.x);
  if (j == 16) return make_float2(-a.x, -a.y);
  if (j == 24) return make_float2(-a.y, a.x);
  const int q = j >> 3, r = j & 7;
  const float c0[5] = {1.0f, kCos16, kCos8, kCos3_16, kCos4};
  const float s0[5] = {0.0f, kSin16, kSin8, kSin3_16, kCos4};
  // (c, s) = (cos, sin) of 2 pi r / 32, r in 1..7
  const float c = r <= 4 ? c0[r] : s0[8 - r];
  const float sn = r <= 4 ? s0[r] : c0[8 - r];
  // exp(-i 2 pi j / 32) = (-i)^q (c - i s)
  float2 w;
  if (q == 0)
    w = make_float2(c, -sn);
  else if (q == 1)
    w = make_float2(-sn, -c);
  else if (q == 2)
    w = make_float2(-c, sn);
  else
    w = make_float2(sn, c);
  return c_mul(a, w);
}

// Radix 32 = radix-2 split over two radix-16 DFTs:
// X[k] = E[k] + W32^k O[k], X[k+16] = E[k] - W32^k O[k].
FERRUM_HD __forceinline__ void dft32(float2 (&u)[32]) {
  float2 e[16], o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    e[i] = u[2 * i];
    o[i] = u[2 * i + 1];
  }
  dft16(e);
  dft16(o);
  o[1] = c_mul(o[1], make_float2(kCos16, -kSin16));
  o[2] = c_mul(o[2], make_float2(kCos8, -kSin8));
  o[3] = c_mul(o[3], make_float2(kCos3_16, -kSin3_16));
  o[4] = c_mul_w8_1(o[4]);
  o[5] = c_mul(o[5], make_float2(kSin3_16, -kCos3_16));
  o[6] = c_mul(o[6], make_float2(kSin8, -kCos8));
  o[7] = c_mul(o[7], make_float2(kSin16, -kCos16));
  o[8] = c_mul_neg_i(o[8]);
  o[9] = c_mul(o[9], make_float2(-kSin16, -kCos16));
  o[10] = c_mul(o[10], make_float2(-kSin8, -kCos8));
  o[11] = c_mul(o[11], make_float2(-kSin3_16, -kCos3_16));
  o[12] = c_mul_w8_3(o[12]);
  o[13] = c_mul(o[13], make_float2(-kCos3_16, -kSin3_16));
  o[14] = c_mul(o[14], make_float2(-kCos8, -kSin8));
  o[15] = c_mul(o[15], make_float2(-kCos16, -kSin16));
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    u[k] = c_add(e[k], o[k]);
    u[k + 16] = c_sub(e[k], o[k]);
  }
}

template <int R>
FERRUM_HD __forceinline__ void dft(float2 (&u)[R]);
template <> FERRUM_HD __forceinline__ void dft<1>(float2 (&)[1]) {}
template <> FERRUM_HD __forceinline__ void dft<2>(float2 (&u)[2]) { dft2(u); }
template <> FERRUM_HD __forceinline__ void dft<4>(float2 (&u)[4]) { dft4(u); }
template <> FERRUM_HD __forceinline__ void dft<8>(float2 (&u)[8]) { dft8(u); }
template <> FERRUM_HD __forceinline__ void dft<16>(float2 (&u)[16]) { dft16(u); }
template <> FERRUM_HD __forceinline__ void dft<32>(float2 (&u)[32]) { dft32(u); }

}  // namespace ferrum
