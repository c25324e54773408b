/*
 * portable_math.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's portable arithmetic
 * (crates/yskn-ref/src/portable_math.rs), the functions the scalar reference calls
 * wherever the model needs a square root, exponential, logarithm or rotary sine and
 * cosine. Each function follows the Rust source statement by statement: every
 * binary32/binary64 operation is one round-to-nearest operation (this file is built
 * with -ffp-contract=off, on x86-64 SSE arithmetic), integer conversions truncate
 * toward zero like Rust's `as`. The layer oracles (oracle.py) and the attention
 * oracle (kv_oracle.c) call these so that they reproduce yskn-ref bit for bit; the
 * tests pin them to the reference's own known answers (portable_math.rs:440-588).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float f_bits(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static uint32_t bits_f(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}
static double d_bits(uint32_t high, uint32_t low) {
  const uint64_t b = ((uint64_t)high << 32) | low;
  double d;
  memcpy(&d, &b, 8);
  return d;
}
static uint64_t bits_d(double d) {
  uint64_t b;
  memcpy(&b, &d, 8);
  return b;
}

/* portable_math.rs:59-104: correctly rounded binary32 square root by integer bisection
 * of the normalised radicand (no platform square root involved). */
float orc_pm_sqrt_rn(float value) {
  const uint32_t bits = bits_f(value);
  if ((bits & 0x7fffffffu) == 0 || bits == 0x7f800000u) return value;
  if ((bits & 0x80000000u) || (bits & 0x7f800000u) == 0x7f800000u) return NAN;
  const int exponent_bits = (int)((bits >> 23) & 255u);
  uint64_t significand;
  int exponent;
  if (exponent_bits == 0) {
    significand = bits & 0x007fffffu;
    exponent = -149;
  } else {
    significand = (bits & 0x007fffffu) | 0x00800000u;
    exponent = exponent_bits - 150;
  }
  const int leading_exponent = 63 - __builtin_clzll(significand) + exponent;
  /* Rust's div_euclid(2): floor division for a positive divisor. */
  int result_exponent = leading_exponent >= 0 ? leading_exponent / 2 : -((-leading_exponent + 1) / 2);
  const int shift = exponent - 2 * result_exponent + 46;
  const uint64_t radicand = significand << shift;
  uint64_t lower = 1ull << 23, upper = 1ull << 24;
  while (upper - lower > 1) {
    const uint64_t middle = lower + (upper - lower) / 2;
    if (middle * middle <= radicand)
      lower = middle;
    else
      upper = middle;
  }
  if (radicand - lower * lower > lower) lower += 1;
  if (lower == 1ull << 24) {
    lower >>= 1;
    result_exponent += 1;
  }
  return f_bits(((uint32_t)(result_exponent + 127) << 23) | ((uint32_t)lower & 0x007fffffu));
}

/* portable_math.rs:106-109: the rounded square root, then a separately rounded division. */
float orc_pm_rsqrt(float value) { return 1.0f / orc_pm_sqrt_rn(value); }

/* portable_math.rs:111-156. */
float orc_pm_exp(float value) {
  const uint32_t bits = bits_f(value);
  const uint32_t absolute_bits = bits & 0x7fffffffu;
  const int negative = (bits >> 31) != 0;
  if (absolute_bits > 0x7f800000u) return value + value;
  if (!negative && absolute_bits >= 0x42b17218u) return INFINITY;
  if (bits > 0xc2cff1b5u) return 0.0f;
  const float ln2_high = f_bits(0x3f317200u), ln2_low = f_bits(0x35bfbe8eu);
  float high = 0.0f, low = 0.0f, reduced = value;
  int exponent = 0;
  if (absolute_bits > 0x3eb17218u) {
    if (absolute_bits < 0x3f851592u) {
      high = value - (negative ? -ln2_high : ln2_high);
      low = negative ? -ln2_low : ln2_low;
      exponent = negative ? -1 : 1;
    } else {
      exponent = (int)(f_bits(0x3fb8aa3bu) * value + (negative ? -0.5f : 0.5f));
      const float exponent_float = (float)exponent;
      high = value - exponent_float * ln2_high;
      low = exponent_float * ln2_low;
    }
    reduced = high - low;
  } else if (absolute_bits < 0x39000000u) {
    return 1.0f + value;
  }
  const float square = reduced * reduced;
  const float correction = reduced - square * (f_bits(0x3e2aaa8fu) + square * f_bits(0xbb355215u));
  if (exponent == 0) return 1.0f - ((reduced * correction) / (correction - 2.0f) - reduced);
  const float result = 1.0f - ((low - (reduced * correction) / (2.0f - correction)) - high);
  if (exponent >= -125) {
    if (exponent == 128) return (result * 2.0f) * f_bits(0x7f000000u);
    return result * f_bits((uint32_t)(127 + exponent) << 23);
  }
  return (result * f_bits((uint32_t)(127 + exponent + 100) << 23)) * f_bits(0x0d800000u);
}

/* portable_math.rs:158-183 (the caller supplies a positive finite value). */
float orc_pm_log(float value) {
  uint32_t bits = bits_f(value);
  int exponent = 0;
  if (bits < 0x00800000u) {
    value *= 33554432.0f;
    exponent = -25;
    bits = bits_f(value);
  }
  exponent += (int)(bits >> 23) - 127;
  bits &= 0x007fffffu;
  const uint32_t adjustment = (bits + 0x004afb20u) & 0x00800000u;
  const float mantissa = f_bits(bits | (adjustment ^ 0x3f800000u));
  exponent += (int)(adjustment >> 23);
  const float fraction = mantissa - 1.0f;
  const float ratio = fraction / (2.0f + fraction);
  const float square = ratio * ratio;
  const float fourth = square * square;
  const float even = fourth * (f_bits(0x3eccce13u) + fourth * f_bits(0x3e789e26u));
  const float odd = square * (f_bits(0x3f2aaaaau) + fourth * f_bits(0x3e91e9eeu));
  const float remainder = odd + even;
  const float half_square = (0.5f * fraction) * fraction;
  const float exponent_float = (float)exponent;
  return exponent_float * f_bits(0x3f317180u) -
         ((half_square - (ratio * (half_square + remainder) + exponent_float * f_bits(0x3717f7d1u))) - fraction);
}

/* portable_math.rs:185-194 (nonnegative domain). */
float orc_pm_log1p(float value) {
  const float shifted = 1.0f + value;
  const float correction = value <= 1.0f ? value - (shifted - 1.0f) : 1.0f - (shifted - value);
  return orc_pm_log(shifted) + correction / shifted;
}

/* portable_math.rs:196-210. */
float orc_pm_sigmoid(float value) { return 1.0f / (1.0f + orc_pm_exp(-value)); }
float orc_pm_silu(float value) { return value / (1.0f + orc_pm_exp(-value)); }
float orc_pm_softplus(float value) { return value > 20.0f ? value : orc_pm_log1p(orc_pm_exp(value)); }

/* portable_math.rs:212-216: the product with binary32 ln(2), then the portable exp. */
float orc_pm_exp2(float value) { return orc_pm_exp(value * f_bits(0x3f317218u)); }

/* portable_math.rs:274-281: the high-word exponent adjustment. */
static double scale_double_exponent(double value, int adjustment) {
  const uint64_t bits = bits_d(value);
  const uint32_t high = (uint32_t)(bits >> 32);
  const uint32_t adjusted_high = high + (uint32_t)adjustment * 1048576u;
  return d_bits(adjusted_high, (uint32_t)bits);
}

/* portable_math.rs:218-272. */
double orc_pm_exp_d(double value) {
  const uint64_t bits = bits_d(value);
  const uint32_t high_bits = (uint32_t)(bits >> 32), low_bits = (uint32_t)bits;
  const int negative = (high_bits >> 31) != 0;
  const uint32_t absolute_high = high_bits & 0x7fffffffu;
  if (absolute_high >= 0x40862e42u) {
    if (absolute_high >= 0x7ff00000u) {
      if (((absolute_high & 0x000fffffu) | low_bits) != 0) return value + value;
      return negative ? 0.0 : value;
    }
    if (value > d_bits(0x40862e42u, 0xfefa39efu)) return INFINITY;
    if (value < d_bits(0xc0874910u, 0xd52d3051u)) return 0.0;
  }
  const double ln2_high = d_bits(0x3fe62e42u, 0xfee00000u), ln2_low = d_bits(0x3dea39efu, 0x35793c76u);
  double high = 0.0, low = 0.0, reduced = value;
  int exponent = 0;
  if (absolute_high > 0x3fd62e42u) {
    if (absolute_high < 0x3ff0a2b2u) {
      high = value - (negative ? -ln2_high : ln2_high);
      low = negative ? -ln2_low : ln2_low;
      exponent = negative ? -1 : 1;
    } else {
      exponent = (int)(d_bits(0x3ff71547u, 0x652b82feu) * value + (negative ? -0.5 : 0.5));
      const double exponent_float = (double)exponent;
      high = value - exponent_float * ln2_high;
      low = exponent_float * ln2_low;
    }
    reduced = high - low;
  } else if (absolute_high < 0x3e300000u) {
    return 1.0 + value;
  }
  const double square = reduced * reduced;
  const double polynomial =
      d_bits(0x3fc55555u, 0x5555553eu) +
      square * (d_bits(0xbf66c16cu, 0x16bebd93u) +
                square * (d_bits(0x3f11566au, 0xaf25de2cu) +
                          square * (d_bits(0xbebbbd41u, 0xc5d26bf1u) + square * d_bits(0x3e663769u, 0x72bea4d0u))));
  const double correction = reduced - square * polynomial;
  if (exponent == 0) return 1.0 - ((reduced * correction) / (correction - 2.0) - reduced);
  const double result = 1.0 - ((low - (reduced * correction) / (2.0 - correction)) - high);
  if (exponent >= -1021) return scale_double_exponent(result, exponent);
  return scale_double_exponent(result, exponent + 1000) * d_bits(0x01700000u, 0);
}

/* portable_math.rs:283-362, including its finite results at +0 and -0. */
double orc_pm_log_d(double value) {
  int32_t high = (int32_t)(bits_d(value) >> 32);
  int exponent = 0;
  if (high < 0x00100000) {
    value *= d_bits(0x43500000u, 0);
    exponent = -54;
    high = (int32_t)(bits_d(value) >> 32);
  }
  exponent += (high >> 20) - 1023;
  high &= 0x000fffff;
  const int32_t adjustment = (high + 0x00095f64) & 0x00100000;
  value = d_bits((uint32_t)(high | (adjustment ^ 0x3ff00000)), (uint32_t)bits_d(value));
  exponent += adjustment >> 20;
  const double ln2_high = d_bits(0x3fe62e42u, 0xfee00000u), ln2_low = d_bits(0x3dea39efu, 0x35793c76u);
  const double fraction = value - 1.0;
  if ((0x000fffff & (2 + high)) < 3) {
    if (fraction == 0.0) {
      if (exponent == 0) return 0.0;
      const double exponent_float = (double)exponent;
      return exponent_float * ln2_high + exponent_float * ln2_low;
    }
    const double remainder = (fraction * fraction) * (0.5 - d_bits(0x3fd55555u, 0x55555555u) * fraction);
    if (exponent == 0) return fraction - remainder;
    const double exponent_float = (double)exponent;
    return exponent_float * ln2_high - ((remainder - exponent_float * ln2_low) - fraction);
  }
  const double ratio = fraction / (2.0 + fraction);
  const double exponent_float = (double)exponent;
  const double square = ratio * ratio;
  const double fourth = square * square;
  const int32_t interval = (high - 0x0006147a) | (0x0006b851 - high);
  const double even =
      fourth * (d_bits(0x3fd99999u, 0x9997fa04u) +
                fourth * (d_bits(0x3fcc71c5u, 0x1d8e78afu) + fourth * d_bits(0x3fc39a09u, 0xd078c69fu)));
  const double odd =
      square * (d_bits(0x3fe55555u, 0x55555593u) +
                fourth * (d_bits(0x3fd24924u, 0x94229359u) +
                          fourth * (d_bits(0x3fc74664u, 0x96cb03deu) + fourth * d_bits(0x3fc2f112u, 0xdf3e5244u))));
  const double remainder = odd + even;
  if (interval > 0) {
    const double half_square = (0.5 * fraction) * fraction;
    if (exponent == 0) return fraction - (half_square - ratio * (half_square + remainder));
    return exponent_float * ln2_high -
           ((half_square - (ratio * (half_square + remainder) + exponent_float * ln2_low)) - fraction);
  }
  if (exponent == 0) return fraction - ratio * (fraction - remainder);
  return exponent_float * ln2_high - ((ratio * (fraction - remainder) - exponent_float * ln2_low) - fraction);
}

/* portable_math.rs:364-378. */
static double kernel_sin(double reduced) {
  const double square = reduced * reduced;
  const double cube = square * reduced;
  const double remainder =
      d_bits(0x3f811111u, 0x1110f8a6u) +
      square * (d_bits(0xbf2a01a0u, 0x19c161d5u) +
                square * (d_bits(0x3ec71de3u, 0x57b1fe7du) +
                          square * (d_bits(0xbe5ae5e6u, 0x8a2b9cebu) + square * d_bits(0x3de5d93au, 0x5acfd57cu))));
  return reduced + cube * (d_bits(0xbfc55555u, 0x55555549u) + square * remainder);
}

/* portable_math.rs:380-404. */
static double kernel_cos(double reduced) {
  const double square = reduced * reduced;
  const double remainder =
      square *
      (d_bits(0x3fa55555u, 0x5555554cu) +
       square * (d_bits(0xbf56c16cu, 0x16c15177u) +
                 square * (d_bits(0x3efa01a0u, 0x19cb1590u) +
                           square * (d_bits(0xbe927e4fu, 0x809c52adu) +
                                     square * (d_bits(0x3e21ee9eu, 0xbdb4b1c4u) +
                                               square * d_bits(0xbda8fae9u, 0xbe8838d4u))))));
  const uint32_t absolute_high = (uint32_t)(bits_d(reduced) >> 32) & 0x7fffffffu;
  const double correction = square * remainder;
  if (absolute_high < 0x3fd33333u) return 1.0 - (0.5 * square - correction);
  const double quarter = absolute_high > 0x3fe90000u ? 0.28125 : d_bits(absolute_high - 0x00200000u, 0);
  return (1.0 - quarter) - ((0.5 * square - quarter) - correction);
}

/* portable_math.rs:406-434: (cosine, sine) after binary64 reduction and polynomials.
 * Returns 0, or -1 for a non-finite angle or one beyond the reduction's i32 domain
 * (the reference returns an error there). */
int orc_pm_sincos(float angle, float* cosine_out, float* sine_out) {
  if (!isfinite(angle)) return -1;
  const double value = (double)angle;
  double quadrant_float = value * d_bits(0x3fe45f30u, 0x6dc9c883u) + 0.5;
  if (!(quadrant_float >= -2147483648.0 && quadrant_float < 2147483648.0)) return -1;
  const int32_t quadrant = (int32_t)quadrant_float;
  quadrant_float = (double)quadrant;
  const double reduced = ((value - quadrant_float * d_bits(0x3ff921fbu, 0x54400000u)) -
                          quadrant_float * d_bits(0x3dd0b461u, 0x1a600000u)) -
                         quadrant_float * d_bits(0x3ba3198au, 0x2e037073u);
  const double sine = kernel_sin(reduced), cosine = kernel_cos(reduced);
  double c, s;
  switch (quadrant & 3) {
    case 0: c = cosine; s = sine; break;
    case 1: c = -sine; s = cosine; break;
    case 2: c = -cosine; s = -sine; break;
    default: c = sine; s = -cosine; break;
  }
  *cosine_out = (float)c;
  *sine_out = (float)s;
  return 0;
}

/* Elementwise maps over arrays for the numpy oracles: fn 0 exp, 1 exp2, 2 log, 3 log1p,
 * 4 sigmoid, 5 silu, 6 softplus, 7 rsqrt, 8 sqrt_rn. Returns -1 for an unknown fn. */
int orc_pm_map(int fn, const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    switch (fn) {
      case 0: y[i] = orc_pm_exp(v); break;
      case 1: y[i] = orc_pm_exp2(v); break;
      case 2: y[i] = orc_pm_log(v); break;
      case 3: y[i] = orc_pm_log1p(v); break;
      case 4: y[i] = orc_pm_sigmoid(v); break;
      case 5: y[i] = orc_pm_silu(v); break;
      case 6: y[i] = orc_pm_softplus(v); break;
      case 7: y[i] = orc_pm_rsqrt(v); break;
      case 8: y[i] = orc_pm_sqrt_rn(v); break;
      default: return -1;
    }
  }
  return 0;
}

/* sincos over an array; returns -1 at the first angle the reduction rejects. */
int orc_pm_sincos_map(const float* angle, float* cosine, float* sine, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    if (orc_pm_sincos(angle[i], cosine + i, sine + i)) return -1;
  return 0;
}
