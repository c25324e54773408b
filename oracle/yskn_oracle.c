/*
 * yskn_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU algorithm for the compressed
 * integer linear path (YASAKANI `.yskn` weights). It is the parity checker for
 * the CUDA library under yasakani-for-mac_b200/ and the timed CPU baseline in
 * bench.py. Nothing in the product links, loads or calls this file.
 *
 * Every function cites the reference file:line it restates (paths are relative
 * to the reference project root). Floating point: binary32 only, compiled with
 * -ffp-contract=off and without -ffast-math, so every mul/add/div rounds once to
 * nearest-even, as crates/yskn-ref does in Rust.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_EINVAL -1
#define ORC_EOVERFLOW -2

/* ------------------------------------------------------------------ signs --
 * crates/yskn-format/src/signs.rs:12-38 and docs/FORMAT.md:159-180.
 * rule 0 = splitmix64, rule 1 = mulberry32_7919_13. */
int orc_signs(int rule, uint64_t seed, uint64_t offset, int64_t count, int8_t* out) {
  if (count < 0 || (rule != 0 && rule != 1)) return ORC_EINVAL;
  for (int64_t i = 0; i < count; ++i) {
    uint64_t position = offset + (uint64_t)i + 1u;
    int positive;
    if (rule == 0) {
      uint64_t v = seed + position * 0x9e3779b97f4a7c15ull;
      v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
      v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
      v ^= v >> 31;
      positive = (v >> 63) != 0;
    } else {
      uint32_t initial = (uint32_t)seed * 7919u + 13u;
      if (initial == 0) initial = 0x9e3779b9u;
      uint32_t v = initial + (uint32_t)position * 0x6d2b79f5u;
      v = (v ^ (v >> 15)) * (v | 1u);
      v ^= v + (v ^ (v >> 7)) * (v | 61u);
      v ^= v >> 14;
      positive = v >= 0x80000000u;
    }
    out[i] = positive ? 1 : -1;
  }
  return ORC_OK;
}

/* ----------------------------------------------------------------- floats --
 * crates/yskn-format/src/floats.rs:4-67 (exact widening, RNE narrowing). */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_f16_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exponent = (bits >> 10) & 0x1fu;
  uint32_t fraction = bits & 0x03ffu;
  uint32_t widened;
  if (exponent == 0 && fraction == 0) {
    widened = sign;
  } else if (exponent == 0) {
    uint32_t shift = (uint32_t)__builtin_clz(fraction) - 21u;
    uint32_t normalized = fraction << shift;
    widened = sign | ((113u - shift) << 23) | ((normalized & 0x03ffu) << 13);
  } else if (exponent == 31) {
    widened = sign | 0x7f800000u | (fraction << 13);
  } else {
    widened = sign | ((exponent + 112u) << 23) | (fraction << 13);
  }
  return u2f(widened);
}

static uint32_t round_shift_even(uint32_t value, uint32_t shift) {
  uint32_t retained = value >> shift;
  uint32_t discarded = value & ((1u << shift) - 1u);
  uint32_t midpoint = 1u << (shift - 1u);
  return retained + (uint32_t)(discarded > midpoint || (discarded == midpoint && (retained & 1u)));
}

uint16_t orc_f32_to_f16(float value) {
  uint32_t bits = f2u(value);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  int32_t exponent = (int32_t)((bits >> 23) & 0xffu);
  uint32_t fraction = bits & 0x007fffffu;
  if (exponent == 255) return (uint16_t)(sign | 0x7c00u | (fraction == 0 ? 0u : 0x0200u));
  int32_t half_exponent = exponent - 127 + 15;
  if (half_exponent >= 31) return (uint16_t)(sign | 0x7c00u);
  if (half_exponent < -10) return sign;
  if (half_exponent <= 0) {
    uint32_t significand = fraction | 0x00800000u;
    uint32_t shift = (uint32_t)(14 - half_exponent);
    return (uint16_t)(sign | round_shift_even(significand, shift));
  }
  uint32_t magnitude = ((uint32_t)half_exponent << 10) + round_shift_even(fraction, 13);
  return (uint16_t)(sign | magnitude);
}

uint16_t orc_f32_to_bf16(float value) {
  uint32_t bits = f2u(value);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
  return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

/* crates/yskn-ref/src/portable_math.rs:12-14 */
float orc_half(float value) { return orc_f16_to_f32(orc_f32_to_f16(value)); }

/* ----------------------------------------------------- trellis addressing --
 * crates/yskn-format/src/tensor.rs:403-418 and docs/FORMAT.md:139-151.
 * layout 0 = row, layout 1 = warp. */
static inline int64_t word_index(int layout, int64_t phys_rows, int64_t cols, int64_t bits,
                                 int64_t row, int64_t seq, int64_t word) {
  if (layout == 0) return (row * (cols / 256) + seq) * (4 * bits) + word;
  int64_t q = seq * phys_rows + row;
  int64_t group = q / 32, lane = q % 32;
  return ((group * bits + word / 4) * 32 + lane) * 4 + word % 4;
}

int64_t orc_word_index(int layout, int64_t phys_rows, int64_t cols, int bits, int64_t row,
                       int64_t seq, int64_t word) {
  return word_index(layout, phys_rows, cols, bits, row, seq, word);
}

/* crates/yskn-format/src/tensor.rs:385-401 (bit-by-bit, zero before the start). */
uint16_t orc_state(const uint32_t* words, int layout, int64_t phys_rows, int64_t cols, int bits,
                   int64_t row, int64_t seq, int step) {
  int end = bits * (step + 1);
  uint16_t state = 0;
  for (int state_bit = 0; state_bit < 12; ++state_bit) {
    int position = end - 12 + state_bit;
    if (position >= 0) {
      uint32_t word = words[word_index(layout, phys_rows, cols, bits, row, seq, position / 32)];
      state |= (uint16_t)(((word >> (position % 32)) & 1u) << state_bit);
    }
  }
  return state;
}

/* All states, ordered [physical_rows][sequences][128] as docs/FORMAT.md:257-262
 * and tools/yskn_decode.py hash them. */
int orc_states_all(const uint32_t* words, int layout, int64_t phys_rows, int64_t cols, int bits,
                   uint16_t* out) {
  if (bits < 4 || bits > 8 || cols <= 0 || cols % 512 != 0 || phys_rows <= 0) return ORC_EINVAL;
  const int64_t seqs = cols / 256;
  for (int64_t r = 0; r < phys_rows; ++r)
    for (int64_t s = 0; s < seqs; ++s)
      for (int j = 0; j < 128; ++j)
        out[(r * seqs + s) * 128 + j] = orc_state(words, layout, phys_rows, cols, bits, r, s, j);
  return ORC_OK;
}

/* -------------------------------------------------------- weight table -----
 * crates/yskn-ref/src/compressed_linear.rs:138-158; docs/spec/02_COMPRESSED_LINEAR.md:39-70;
 * the reference loader src/loader.cpp:19-25. */
int orc_quantize_weight_table(const uint16_t* table16, const uint16_t* scale16, int64_t n,
                              int8_t* lut8, float* tau) {
  float table_maximum = 0.0f;
  for (int i = 0; i < 8192; ++i) {
    float v = orc_f16_to_f32(table16[i]);
    if (!isfinite(v)) return ORC_EINVAL;
    float a = fabsf(v);
    table_maximum = table_maximum > a ? table_maximum : a;
  }
  if (table_maximum == 0.0f) return ORC_EINVAL;
  const float table_scale = table_maximum / 127.0f;
  for (int i = 0; i < 8192; ++i) {
    float r = nearbyintf(orc_f16_to_f32(table16[i]) / table_scale);
    r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
    lut8[i] = (int8_t)r;
  }
  for (int64_t r = 0; r < n; ++r) {
    float s = orc_f16_to_f32(scale16[r]);
    if (!isfinite(s)) return ORC_EINVAL;
    tau[r] = s * table_scale;
    if (!isfinite(tau[r])) return ORC_EINVAL;
  }
  return ORC_OK;
}

/* ---------------------------------------------------------------- H512 -----
 * crates/yskn-ref/src/compressed_linear.rs:14-29: ascending strides, each
 * sum/difference rounded separately. */
void orc_hadamard512(float* v) {
  for (int stride = 1; stride < 512; stride *= 2)
    for (int base = 0; base < 512; base += 2 * stride)
      for (int o = 0; o < stride; ++o) {
        float lower = v[base + o], upper = v[base + o + stride];
        v[base + o] = lower + upper;
        v[base + o + stride] = lower - upper;
      }
}

static const uint32_t HADAMARD_NORMALIZATION_BITS = 0x3d3504f3u; /* compressed_linear.rs:9 */
static const uint32_t INTEGER_SCALE_QUANTUM_BITS = 0x33800000u;  /* 2^-24, compressed_linear.rs:11 */

/* ------------------------------------------------- activation quantiser ----
 * crates/yskn-ref/src/compressed_linear.rs:57-135; spec 02_COMPRESSED_LINEAR.md:129-196.
 * One call quantises M rows of Kc columns. Returns ORC_EINVAL for non-finite
 * values (before or after the FP16 rounding) and for bad signs. */
int orc_quantize_activation(const float* x, const int8_t* signs, int64_t M, int64_t Kc,
                            int8_t* act8, float* alpha, int32_t* A, float* row_quantum) {
  if (M <= 0 || Kc <= 0 || Kc % 512 != 0) return ORC_EINVAL;
  for (int64_t i = 0; i < Kc; ++i)
    if (signs[i] != 1 && signs[i] != -1) return ORC_EINVAL;
  const float K512 = u2f(HADAMARD_NORMALIZATION_BITS);
  const int64_t G = Kc / 512;
  float rotated[512];
  for (int64_t m = 0; m < M; ++m) {
    const float* xr = x + m * Kc;
    for (int64_t i = 0; i < Kc; ++i)
      if (!isfinite(xr[i])) return ORC_EINVAL;
    for (int64_t g = 0; g < G; ++g) {
      for (int j = 0; j < 512; ++j) rotated[j] = xr[g * 512 + j] * (float)signs[g * 512 + j];
      orc_hadamard512(rotated);
      for (int j = 0; j < 512; ++j) rotated[j] = orc_half(rotated[j] * K512);
      float maximum = 0.0f;
      for (int j = 0; j < 512; ++j) {
        if (!isfinite(rotated[j])) return ORC_EINVAL;
        float a = fabsf(rotated[j]);
        maximum = maximum > a ? maximum : a;
      }
      const float scale = maximum / 127.0f;
      alpha[m * G + g] = scale;
      for (int j = 0; j < 512; ++j) {
        float ratio = scale > 0.0f ? rotated[j] / scale : 0.0f;
        float r = nearbyintf(ratio);
        r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
        act8[m * Kc + g * 512 + j] = (int8_t)r;
      }
    }
    float maximum_scale = 0.0f;
    for (int64_t g = 0; g < G; ++g)
      maximum_scale = maximum_scale > alpha[m * G + g] ? maximum_scale : alpha[m * G + g];
    const float multiplier = maximum_scale > 0.0f ? 16777216.0f / maximum_scale : 0.0f;
    row_quantum[m] = maximum_scale * u2f(INTEGER_SCALE_QUANTUM_BITS);
    for (int64_t g = 0; g < G; ++g) A[m * G + g] = (int32_t)nearbyintf(alpha[m * G + g] * multiplier);
  }
  return ORC_OK;
}

/* ------------------------------------------------------- weighted sums -----
 * crates/yskn-ref/src/compressed_linear.rs:205-252 (scalar; checked i64 add).
 * out is [M][rows] row-major; rows <= phys_rows. */
int orc_weighted_sums(const uint32_t* words, int layout, int64_t phys_rows, int64_t cols, int bits,
                      const int8_t* lut8, const int8_t* act8, const int32_t* A, int64_t M,
                      int64_t rows, int64_t* out) {
  if (bits < 4 || bits > 8 || cols <= 0 || cols % 512 != 0 || rows < 0 || rows > phys_rows || M <= 0)
    return ORC_EINVAL;
  const int64_t G = cols / 512;
  uint16_t st[256];
  int rc = ORC_OK;
  for (int64_t row = 0; row < rows; ++row) {
    for (int64_t m = 0; m < M; ++m) out[m * rows + row] = 0;
    for (int64_t g = 0; g < G; ++g) {
      /* Two adjacent 256-weight sequences form one 512-term dot (compressed_linear.rs:230-243). */
      for (int si = 0; si < 2; ++si)
        for (int step = 0; step < 128; ++step)
          st[si * 128 + step] = orc_state(words, layout, phys_rows, cols, bits, row, g * 2 + si, step);
      for (int64_t m = 0; m < M; ++m) {
        int32_t dot = 0;
        for (int k = 0; k < 256; ++k) {
          const int state = st[k];
          const int64_t column = g * 512 + k * 2;
          dot += (int32_t)lut8[state * 2] * (int32_t)act8[m * cols + column];
          dot += (int32_t)lut8[state * 2 + 1] * (int32_t)act8[m * cols + column + 1];
        }
        const int64_t weighted = (int64_t)A[m * G + g] * (int64_t)dot;
        int64_t* sum = &out[m * rows + row];
        if (__builtin_add_overflow(*sum, weighted, sum)) rc = ORC_EOVERFLOW;
      }
    }
  }
  return rc;
}

/* ------------------------------------------------------------- restore -----
 * crates/yskn-ref/src/compressed_linear.rs:288-370; spec 02_COMPRESSED_LINEAR.md:198-241.
 * ws is [M][phys_rows]; out is [M][rows]. inv_rms (per activation row) and
 * signs_out may be NULL. */
int orc_restore(const int64_t* ws, int64_t M, int64_t phys_rows, const float* row_quantum,
                const float* inv_rms, const float* tau, const int8_t* signs_out, int64_t rows,
                float* out) {
  if (M <= 0 || rows < 0 || rows > phys_rows) return ORC_EINVAL;
  if (signs_out) {
    if (phys_rows % 512 != 0) return ORC_EINVAL;
    for (int64_t i = 0; i < phys_rows; ++i)
      if (signs_out[i] != 1 && signs_out[i] != -1) return ORC_EINVAL;
  }
  const float K512 = u2f(HADAMARD_NORMALIZATION_BITS);
  float* lin = (float*)malloc(sizeof(float) * (size_t)phys_rows);
  if (!lin) return ORC_EINVAL;
  for (int64_t m = 0; m < M; ++m) {
    if (inv_rms && !isfinite(inv_rms[m])) { free(lin); return ORC_EINVAL; }
    for (int64_t r = 0; r < phys_rows; ++r) {
      float v = (float)ws[m * phys_rows + r] * row_quantum[m];
      if (inv_rms) v = v * inv_rms[m];
      v = v * tau[r];
      if (!isfinite(v)) { free(lin); return ORC_EINVAL; }
      lin[r] = v;
    }
    if (signs_out) {
      for (int64_t b = 0; b < phys_rows / 512; ++b) {
        float blk[512];
        memcpy(blk, lin + b * 512, sizeof blk);
        orc_hadamard512(blk);
        for (int j = 0; j < 512; ++j) {
          float v = (blk[j] * K512) * (float)signs_out[b * 512 + j];
          if (!isfinite(v)) { free(lin); return ORC_EINVAL; }
          lin[b * 512 + j] = v;
        }
      }
    }
    memcpy(out + m * rows, lin, sizeof(float) * (size_t)rows);
  }
  free(lin);
  return ORC_OK;
}

/* -------------------------------------------------------------- repack -----
 * src/repack.cu:10-18: warp-layout words -> the reference's "frag" order. */
int orc_repack_warp_to_frag(const uint32_t* w, uint32_t* f, int rows, int seqs, int wps) {
  if (rows <= 0 || seqs <= 0 || wps <= 0 || rows % 64 || wps % 4) return ORC_EINVAL;
  const int64_t total = (int64_t)rows * seqs * wps;
  for (int64_t i = 0; i < total; ++i) {
    const int word = (int)(i % wps);
    const int64_t t2 = i / wps;
    const int seq = (int)(t2 % seqs), row = (int)(t2 / seqs);
    const int64_t q = (int64_t)seq * rows + row, tile = q / 32, lane = q % 32;
    const int64_t src = ((tile * (wps / 4) + word / 4) * 32 + lane) * 4 + (word % 4);
    const int64_t wt = row / 64, j = (row % 64) / 8, r = row % 8, c = word / 4;
    const int64_t dst = ((((wt * seqs + seq) * 8 + j) * (wps / 4) + c) * 8 + r) * 4 + (word % 4);
    f[dst] = w[src];
  }
  return ORC_OK;
}

/* --------------------------------------------------- threaded CPU kernel ---
 * Restatement of the Mac port's CPU engine: crates/yskn-engine/src/kernel.rs:92-233
 * (constant-shift decode for bits 6 and 8, generic window otherwise; one 512-weight
 * decode per (row, group) reused for up to 16 input rows; portable i32 dot) on a
 * pool of worker threads taking 32- or 256-row tasks (crates/yskn-engine/src/pool.rs:284-288).
 * This is the CPU baseline that bench.py times. */
typedef struct {
  const uint32_t* words; int layout; int64_t phys_rows, cols; int bits;
  const int8_t* lut8; const int8_t* act8; const int32_t* A; int64_t M, rows;
  int64_t* out; int64_t task_rows, n_tasks; atomic_long next; atomic_int failed;
} fast_job;

static void decode_seq(const fast_job* J, int64_t row, int64_t seq, int8_t* w) {
  const int B = J->bits;
  uint32_t words[33];
  for (int k = 0; k < 4 * B; ++k)
    words[k] = J->words[word_index(J->layout, J->phys_rows, J->cols, B, row, seq, k)];
  words[4 * B] = 0;
  const int8_t* T = J->lut8;
  uint64_t carry = 0;
  if (B == 6) {
    for (int chunk = 0; chunk < 8; ++chunk) {
      uint64_t a = (uint64_t)words[chunk * 3] | ((uint64_t)words[chunk * 3 + 1] << 32);
      uint64_t c = words[chunk * 3 + 2];
      uint64_t s[16] = {(a << 6) | carry, a, a >> 6, a >> 12, a >> 18, a >> 24, a >> 30, a >> 36,
                        a >> 42, a >> 48, (a >> 54) | (c << 10), (a >> 60) | (c << 4), c >> 2,
                        c >> 8, c >> 14, c >> 20};
      for (int j = 0; j < 16; ++j) {
        int idx = (int)(s[j] & 4095) * 2;
        w[chunk * 32 + 2 * j] = T[idx];
        w[chunk * 32 + 2 * j + 1] = T[idx + 1];
      }
      carry = c >> 26;
    }
    return;
  }
  if (B == 8) {
    for (int chunk = 0; chunk < 16; ++chunk) {
      uint64_t a = (uint64_t)words[chunk * 2] | ((uint64_t)words[chunk * 2 + 1] << 32);
      uint64_t s[8] = {(a << 4) | carry, a >> 4, a >> 12, a >> 20, a >> 28, a >> 36, a >> 44, a >> 52};
      for (int j = 0; j < 8; ++j) {
        int idx = (int)(s[j] & 4095) * 2;
        w[chunk * 16 + 2 * j] = T[idx];
        w[chunk * 16 + 2 * j + 1] = T[idx + 1];
      }
      carry = a >> 60;
    }
    return;
  }
  for (int step = 0; step < 128; ++step) {
    int end = B * (step + 1);
    uint32_t state;
    if (end < 12) {
      state = (words[0] << (12 - end)) & 4095u;
    } else {
      int start = end - 12;
      uint64_t window = (uint64_t)words[start / 32] | ((uint64_t)words[start / 32 + 1] << 32);
      state = (uint32_t)((window >> (start % 32)) & 4095u);
    }
    w[step * 2] = T[state * 2];
    w[step * 2 + 1] = T[state * 2 + 1];
  }
}

static void* fast_worker(void* arg) {
  fast_job* J = (fast_job*)arg;
  const int64_t G = J->cols / 512;
  int8_t weights[512];
  for (;;) {
    const long t = atomic_fetch_add(&J->next, 1);
    if (t >= J->n_tasks || atomic_load(&J->failed)) break;
    const int64_t r0 = t * J->task_rows;
    const int64_t r1 = r0 + J->task_rows < J->rows ? r0 + J->task_rows : J->rows;
    for (int64_t batch = 0; batch < J->M; batch += 16) {
      const int64_t bend = batch + 16 < J->M ? batch + 16 : J->M;
      for (int64_t tile = r0; tile < r1; tile += 32) {
        for (int64_t g = 0; g < G; ++g) {
          const int64_t tend = tile + 32 < r1 ? tile + 32 : r1;
          for (int64_t row = tile; row < tend; ++row) {
            decode_seq(J, row, g * 2, weights);
            decode_seq(J, row, g * 2 + 1, weights + 256);
            for (int64_t in = batch; in < bend; ++in) {
              const int8_t* a = J->act8 + in * J->cols + g * 512;
              int32_t dot = 0;
              for (int k = 0; k < 512; ++k) dot += (int32_t)weights[k] * (int32_t)a[k];
              int64_t* sum = &J->out[in * J->rows + row];
              if (__builtin_add_overflow(*sum, (int64_t)dot * (int64_t)J->A[in * G + g], sum))
                atomic_store(&J->failed, 1);
            }
          }
        }
      }
    }
  }
  return NULL;
}

int orc_fast_weighted_sums(const uint32_t* words, int layout, int64_t phys_rows, int64_t cols, int bits,
                           const int8_t* lut8, const int8_t* act8, const int32_t* A, int64_t M,
                           int64_t rows, int64_t* out, int threads) {
  if (bits < 4 || bits > 8 || cols <= 0 || cols % 512 != 0 || rows < 0 || rows > phys_rows || M <= 0 ||
      threads <= 0)
    return ORC_EINVAL;
  memset(out, 0, sizeof(int64_t) * (size_t)(M * rows));
  fast_job J;
  J.words = words; J.layout = layout; J.phys_rows = phys_rows; J.cols = cols; J.bits = bits;
  J.lut8 = lut8; J.act8 = act8; J.A = A; J.M = M; J.rows = rows; J.out = out;
  J.task_rows = (rows / threads < 256) ? 32 : 256;
  J.n_tasks = (rows + J.task_rows - 1) / J.task_rows;
  atomic_init(&J.next, 0);
  atomic_init(&J.failed, 0);
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  if (!tid) return ORC_EINVAL;
  int started = 0;
  for (int i = 0; i < threads; ++i)
    if (pthread_create(&tid[i], NULL, fast_worker, &J) == 0) ++started;
  if (started == 0) fast_worker(&J);
  for (int i = 0; i < started; ++i) pthread_join(tid[i], NULL);
  free(tid);
  return atomic_load(&J.failed) ? ORC_EOVERFLOW : ORC_OK;
}
