// Portable arithmetic on the device: the functions of the reference's scalar contract
// (crates/yskn-ref/src/portable_math.rs) for the layer kernels, so that their results
// equal yskn-ref's bit for bit instead of depending on CUDA's math library.
//
// Every binary32/binary64 step is one explicit round-to-nearest operation (__fadd_rn,
// __fmul_rn, __fdiv_rn, __dadd_rn, ...), in the order of the Rust source; the square
// root is IEEE's correctly rounded __fsqrt_rn, which equals the reference's integer
// bisection (portable_math.rs:59-104) for every input. Float-to-integer conversions
// truncate toward zero, as Rust's `as` does.
#pragma once
#include <stdint.h>

namespace yskn {

__device__ __forceinline__ float pm_f(uint32_t b) { return __uint_as_float(b); }

// portable_math.rs:106-109: the rounded square root, then a rounded division.
__device__ __forceinline__ float pm_rsqrt(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

// portable_math.rs:111-156.
__device__ __forceinline__ float pm_exp(float x) {
  const uint32_t bits = __float_as_uint(x), ab = bits & 0x7fffffffu;
  const bool neg = (bits >> 31) != 0;
  if (ab > 0x7f800000u) return __fadd_rn(x, x);
  if (!neg && ab >= 0x42b17218u) return pm_f(0x7f800000u);
  if (bits > 0xc2cff1b5u) return 0.0f;
  const float ln2_hi = pm_f(0x3f317200u), ln2_lo = pm_f(0x35bfbe8eu);
  float hi = 0.0f, lo = 0.0f, r = x;
  int k = 0;
  if (ab > 0x3eb17218u) {
    if (ab < 0x3f851592u) {
      hi = __fsub_rn(x, neg ? -ln2_hi : ln2_hi);
      lo = neg ? -ln2_lo : ln2_lo;
      k = neg ? -1 : 1;
    } else {
      k = __float2int_rz(__fadd_rn(__fmul_rn(pm_f(0x3fb8aa3bu), x), neg ? -0.5f : 0.5f));
      const float kf = (float)k;  // exact: |k| <= 150
      hi = __fsub_rn(x, __fmul_rn(kf, ln2_hi));
      lo = __fmul_rn(kf, ln2_lo);
    }
    r = __fsub_rn(hi, lo);
  } else if (ab < 0x39000000u) {
    return __fadd_rn(1.0f, x);
  }
  const float sq = __fmul_rn(r, r);
  const float c = __fsub_rn(r, __fmul_rn(sq, __fadd_rn(pm_f(0x3e2aaa8fu), __fmul_rn(sq, pm_f(0xbb355215u)))));
  if (k == 0) return __fsub_rn(1.0f, __fsub_rn(__fdiv_rn(__fmul_rn(r, c), __fsub_rn(c, 2.0f)), r));
  const float y = __fsub_rn(1.0f, __fsub_rn(__fsub_rn(lo, __fdiv_rn(__fmul_rn(r, c), __fsub_rn(2.0f, c))), hi));
  if (k >= -125) {
    if (k == 128) return __fmul_rn(__fmul_rn(y, 2.0f), pm_f(0x7f000000u));
    return __fmul_rn(y, pm_f((uint32_t)(127 + k) << 23));
  }
  return __fmul_rn(__fmul_rn(y, pm_f((uint32_t)(127 + k + 100) << 23)), pm_f(0x0d800000u));
}

// portable_math.rs:158-183 (positive finite argument).
__device__ __forceinline__ float pm_log(float x) {
  uint32_t bits = __float_as_uint(x);
  int e = 0;
  if (bits < 0x00800000u) {
    x = __fmul_rn(x, 33554432.0f);
    e = -25;
    bits = __float_as_uint(x);
  }
  e += (int)(bits >> 23) - 127;
  bits &= 0x007fffffu;
  const uint32_t adj = (bits + 0x004afb20u) & 0x00800000u;
  const float mant = pm_f(bits | (adj ^ 0x3f800000u));
  e += (int)(adj >> 23);
  const float f = __fsub_rn(mant, 1.0f);
  const float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  const float z = __fmul_rn(s, s), w = __fmul_rn(z, z);
  const float even = __fmul_rn(w, __fadd_rn(pm_f(0x3eccce13u), __fmul_rn(w, pm_f(0x3e789e26u))));
  const float odd = __fmul_rn(z, __fadd_rn(pm_f(0x3f2aaaaau), __fmul_rn(w, pm_f(0x3e91e9eeu))));
  const float rem = __fadd_rn(odd, even);
  const float hfsq = __fmul_rn(__fmul_rn(0.5f, f), f);
  const float ef = (float)e;
  return __fsub_rn(__fmul_rn(ef, pm_f(0x3f317180u)),
                   __fsub_rn(__fsub_rn(hfsq, __fadd_rn(__fmul_rn(s, __fadd_rn(hfsq, rem)), __fmul_rn(ef, pm_f(0x3717f7d1u)))),
                             f));
}

// portable_math.rs:185-194 (nonnegative argument).
__device__ __forceinline__ float pm_log1p(float x) {
  const float u = __fadd_rn(1.0f, x);
  const float c = x <= 1.0f ? __fsub_rn(x, __fsub_rn(u, 1.0f)) : __fsub_rn(1.0f, __fsub_rn(u, x));
  return __fadd_rn(pm_log(u), __fdiv_rn(c, u));
}

// portable_math.rs:196-216.
__device__ __forceinline__ float pm_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, pm_exp(-x))); }
__device__ __forceinline__ float pm_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, pm_exp(-x))); }
__device__ __forceinline__ float pm_softplus(float x) { return x > 20.0f ? x : pm_log1p(pm_exp(x)); }
__device__ __forceinline__ float pm_exp2(float x) { return pm_exp(__fmul_rn(x, pm_f(0x3f317218u))); }

__device__ __forceinline__ double pm_d(uint32_t hi, uint32_t lo) {
  return __hiloint2double((int)hi, (int)lo);
}

// portable_math.rs:364-378 (binary64; Horner from the innermost coefficient out).
__device__ __forceinline__ double pm_kernel_sin(double r) {
  const double z = __dmul_rn(r, r), v = __dmul_rn(z, r);
  double p = pm_d(0x3de5d93au, 0x5acfd57cu);
  p = __dadd_rn(pm_d(0xbe5ae5e6u, 0x8a2b9cebu), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0x3ec71de3u, 0x57b1fe7du), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0xbf2a01a0u, 0x19c161d5u), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0x3f811111u, 0x1110f8a6u), __dmul_rn(z, p));
  return __dadd_rn(r, __dmul_rn(v, __dadd_rn(pm_d(0xbfc55555u, 0x55555549u), __dmul_rn(z, p))));
}

// portable_math.rs:380-404 (binary64).
__device__ __forceinline__ double pm_kernel_cos(double r) {
  const double z = __dmul_rn(r, r);
  double p = pm_d(0xbda8fae9u, 0xbe8838d4u);
  p = __dadd_rn(pm_d(0x3e21ee9eu, 0xbdb4b1c4u), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0xbe927e4fu, 0x809c52adu), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0x3efa01a0u, 0x19cb1590u), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0xbf56c16cu, 0x16c15177u), __dmul_rn(z, p));
  p = __dadd_rn(pm_d(0x3fa55555u, 0x5555554cu), __dmul_rn(z, p));
  p = __dmul_rn(z, p);
  const uint32_t ahi = (uint32_t)__double2hiint(r) & 0x7fffffffu;
  const double corr = __dmul_rn(z, p);
  if (ahi < 0x3fd33333u) return __dsub_rn(1.0, __dsub_rn(__dmul_rn(0.5, z), corr));
  const double qx = ahi > 0x3fe90000u ? 0.28125 : pm_d(ahi - 0x00200000u, 0u);
  return __dsub_rn(__dsub_rn(1.0, qx), __dsub_rn(__dsub_rn(__dmul_rn(0.5, z), qx), corr));
}

// portable_math.rs:406-434: cosine and sine of a binary32 angle after binary64
// reduction. Returns false for a non-finite angle or one outside the reduction's
// 32-bit quadrant range (the reference returns an error there); *c and *s are then 0.
__device__ __forceinline__ bool pm_sincos(float angle, float* c, float* s) {
  *c = 0.0f;
  *s = 0.0f;
  if (!isfinite(angle)) return false;
  const double v = (double)angle;
  const double qf = __dadd_rn(__dmul_rn(v, pm_d(0x3fe45f30u, 0x6dc9c883u)), 0.5);
  if (!(qf >= -2147483648.0 && qf < 2147483648.0)) return false;
  const int q = __double2int_rz(qf);
  const double qd = (double)q;
  const double r = __dsub_rn(__dsub_rn(__dsub_rn(v, __dmul_rn(qd, pm_d(0x3ff921fbu, 0x54400000u))),
                                       __dmul_rn(qd, pm_d(0x3dd0b461u, 0x1a600000u))),
                             __dmul_rn(qd, pm_d(0x3ba3198au, 0x2e037073u)));
  const double sn = pm_kernel_sin(r), cs = pm_kernel_cos(r);
  double cc, ss;
  switch (q & 3) {
    case 0: cc = cs; ss = sn; break;
    case 1: cc = -sn; ss = cs; break;
    case 2: cc = -cs; ss = -sn; break;
    default: cc = sn; ss = -cs; break;
  }
  *c = __double2float_rn(cc);
  *s = __double2float_rn(ss);
  return true;
}

}  // namespace yskn
