/*
 * kv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's quantised-KV row codec and decode
 * attention (crates/yskn-ref/src/kv_codec.rs, kv_profile.rs, attention.rs) used as
 * the checker of the CUDA KV kernels. The codec is pinned by the reference's frozen
 * SHA-256 (crates/yskn-ref/src/kv_codec_tests.rs:427-470). Binary32 operations are
 * separate round-to-nearest operations (-ffp-contract=off), as in the Rust source.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

float orc_f16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float value);
uint16_t orc_f32_to_bf16(float value);

#define KV_OK 0
#define KV_EINVAL -1

float orc_pm_exp(float value);
float orc_pm_exp2(float value);

static float half_r(float x) { return orc_f16_to_f32(orc_f32_to_f16(x)); }
static float bfloat_r(float x) {
  uint32_t u = (uint32_t)orc_f32_to_bf16(x) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static int finite32(float x) { return isfinite(x); }

/* kv_profile.rs:12-14 */
static float reconstruction(const int16_t* codes, float gain, int state) {
  return ((float)codes[state] * 0.00390625f) * gain;
}

/* kv_codec.rs:228-245: warp XOR butterflies 16,8,4,2,1; eight warp sums fold from +0. */
static float warp_sum(const float* v32) {
  float v[32], old[32];
  memcpy(v, v32, sizeof v);
  for (int offset = 16; offset > 0; offset >>= 1) {
    memcpy(old, v, sizeof v);
    for (int i = 0; i < 32; ++i) v[i] = old[i] + old[i ^ offset];
  }
  return v[0];
}
static float sum256(const float* v) {
  float total = 0.0f;
  for (int c = 0; c < 8; ++c) total += warp_sum(v + 32 * c);
  return total;
}

/* kv_codec.rs:112-115: checked i32 arithmetic. */
static int add_c(int32_t a, int32_t b, int32_t* r) { return __builtin_add_overflow(a, b, r); }
static int sub_c(int32_t a, int32_t b, int32_t* r) { return __builtin_sub_overflow(a, b, r); }
static int mul_c(int32_t a, int32_t b, int32_t* r) { return __builtin_mul_overflow(a, b, r); }

/* kv_codec.rs:117-146 (src/kvq_fast.cuh:108-135): lowest predecessor j, then lowest final state. */
static int general_chain(const int32_t* target, const int16_t* codes, int bits, uint8_t* path) {
  const int fields = 1 << bits, stride = 256 >> bits;
  int32_t cost[256], next[256];
  static uint8_t bp[64][32];
  for (int s = 0; s < 256; ++s) cost[s] = 0x40000000;
  cost[0] = 0;
  for (int t = 0; t < 64; ++t) {
    const int32_t x = target[t];
    for (int u = 0; u < stride; ++u) {
      int32_t best = cost[u];
      int choice = 0;
      for (int j = 1; j < fields; ++j)
        if (cost[j * stride + u] < best) {
          best = cost[j * stride + u];
          choice = j;
        }
      bp[t][u] = (uint8_t)choice;
      for (int j = 0; j < fields; ++j) {
        const int state = (u << bits) | j;
        int32_t dx, sq, r;
        if (sub_c(x, codes[state], &dx) || mul_c(dx, dx, &sq) || add_c(sq, best, &r)) return KV_EINVAL;
        next[state] = r;
      }
    }
    memcpy(cost, next, sizeof cost);
  }
  int state = 0;
  for (int s = 1; s < 256; ++s)
    if ((uint32_t)cost[s] < (uint32_t)cost[state]) state = s;
  for (int t = 63; t >= 0; --t) {
    path[t] = (uint8_t)state;
    state = ((int)bp[t][state >> bits] << (8 - bits)) | (state >> bits);
  }
  return KV_OK;
}

/* kv_codec.rs:148-211 (src/kvq_vit2.cuh:64-88,143-192): compressed cost recurrence. */
static int vit2_chain(const int32_t* target, const int16_t* codes, int bits, uint8_t* path) {
  const int fields = 1 << bits, stride = 256 >> bits;
  const int32_t f = fields;
  int32_t ac[256], bc[256], cost[64], next[64];
  static uint8_t bp[64][16];
  for (int d = 0; d < 256; ++d) {
    const int32_t c = codes[d];
    int32_t t1, t2, r;
    if (mul_c(f, c, &t1) || mul_c(t1, c, &t2) || add_c(t2, d / stride, &r)) return KV_EINVAL;
    ac[d] = r;
    if (mul_c(-2, f, &t1) || mul_c(t1, c, &r)) return KV_EINVAL;
    bc[d] = r;
  }
  for (int g = 0; g < stride; ++g) cost[g] = f << 24;
  cost[0] = 0;
  int64_t final_k = INT32_MAX;
  int final_state = -1;
  int have_final = 0;
  for (int t = 0; t < 64; ++t) {
    const int32_t x = target[t];
    int32_t sq0, square;
    if (mul_c(x, x, &sq0) || mul_c(sq0, f, &square)) return KV_EINVAL;
    for (int g = 0; g < stride; ++g) {
      int32_t best = INT32_MAX;
      const int step = bits == 5 ? 2 : 1;
      for (int j = 0; j < fields; j += step) {
        const int d = stride * j + g;
        int32_t m, emission, r;
        if (mul_c(bc[d], x, &m) || add_c(ac[d], m, &emission)) return KV_EINVAL;
        if (bits == 5) {
          const int other = d + stride;
          int32_t m2, e2;
          if (mul_c(bc[other], x, &m2) || add_c(ac[other], m2, &e2)) return KV_EINVAL;
          if (e2 < emission) emission = e2;
        }
        if (add_c(emission, cost[d >> bits], &r)) return KV_EINVAL;
        if (r < best) best = r;
      }
      int32_t k;
      if (add_c(best, square, &k)) return KV_EINVAL;
      if (t == 63) {
        const int state = stride * (k & (fields - 1)) + g;
        const int32_t key = k >> bits;
        if (!have_final || key < final_k || (key == final_k && state < final_state)) {
          final_k = key;
          final_state = state;
          have_final = 1;
        }
      } else {
        int32_t k2;
        if (sub_c(k, cost[0], &k2)) return KV_EINVAL;
        next[g] = k2 & ~(f - 1);
        bp[t + 1][g] = (uint8_t)(k2 & (f - 1));
      }
    }
    if (t < 63) memcpy(cost, next, sizeof(int32_t) * stride);
  }
  int state = final_state;
  for (int t = 63; t >= 1; --t) {
    path[t] = (uint8_t)state;
    state = ((int)bp[t][state >> bits] << (8 - bits)) | (state >> bits);
  }
  path[0] = (uint8_t)state;
  return KV_OK;
}

/* kv_codec.rs:247-264 (src/kvx_codec.cuh:50-69) */
static int initial_int8(const float* row, int8_t* q, float* scale_out) {
  float maximum = 0.0f;
  for (int i = 0; i < 256; ++i) {
    if (!finite32(row[i])) return KV_EINVAL;
    const float a = fabsf(row[i]);
    maximum = maximum > a ? maximum : a;
  }
  const float scale = maximum / 127.0f;
  for (int i = 0; i < 256; ++i) {
    if (scale > 0.0f) {
      float r = nearbyintf(row[i] / scale);
      r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
      q[i] = (int8_t)r;
    } else {
      q[i] = 0;
    }
  }
  *scale_out = scale;
  return KV_OK;
}

typedef struct {
  int mode, bits, guard, n_basis, has_mean, vit2;
  const int16_t* codes;
  float gain;
  const float* mean;   /* 256 or NULL */
  const float* basis;  /* n_basis x 256 */
  const float* mults;
  int n_mult;
} kv_group;

/* kv_codec.rs:272-396: select(). */
static int kv_select(const kv_group* g, int position, const float* row, float* rec, uint8_t* states, float* sel_scale) {
  int8_t q[256];
  float s0;
  if (initial_int8(row, q, &s0)) return KV_EINVAL;
  float y[256];
  for (int i = 0; i < 256; ++i) y[i] = (float)q[i] * s0;
  memset(states, 0, 256);
  if (position < g->guard) {
    memcpy(rec, y, sizeof y);
    *sel_scale = 1.0f;
    return KV_OK;
  }
  float residual[256], tmp[256];
  memcpy(residual, y, sizeof y);
  if (g->has_mean)
    for (int i = 0; i < 256; ++i) residual[i] -= g->mean[i];
  float coef[2] = {0.0f, 0.0f};
  const int nb = g->n_basis < 2 ? g->n_basis : 2;
  for (int j = 0; j < nb; ++j) {
    for (int i = 0; i < 256; ++i) tmp[i] = residual[i] * g->basis[j * 256 + i];
    coef[j] = half_r(sum256(tmp));
    for (int i = 0; i < 256; ++i) residual[i] -= coef[j] * g->basis[j * 256 + i];
  }
  for (int i = 0; i < 256; ++i)
    if (!finite32(residual[i])) return KV_EINVAL;
  for (int i = 0; i < 256; ++i) tmp[i] = residual[i] * residual[i];
  float rms = sqrtf(sum256(tmp) / 256.0f);
  if (rms == 0.0f) rms = 1.0f;
  if (!finite32(rms)) return KV_EINVAL;
  memcpy(rec, residual, sizeof residual);
  *sel_scale = 1.0f;
  if (g->mode == 0) {
    int have = 0;
    float best_error = 0.0f;
    for (int mi = 0; mi < g->n_mult; ++mi) {
      float scale = half_r(rms * g->mults[mi]);
      if (scale == 0.0f) scale = 1.0f;
      if (!finite32(scale)) return KV_EINVAL;
      int32_t targets[256];
      for (int i = 0; i < 256; ++i) {
        float r = nearbyintf((residual[i] / scale) * 256.0f);
        r = r < -2048.0f ? -2048.0f : (r > 2048.0f ? 2048.0f : r);
        targets[i] = (int32_t)r;
      }
      uint8_t st[256];
      for (int c = 0; c < 4; ++c) {
        int rc = g->vit2 ? vit2_chain(targets + 64 * c, g->codes, g->bits, st + 64 * c)
                         : general_chain(targets + 64 * c, g->codes, g->bits, st + 64 * c);
        if (rc) return rc;
      }
      float r2[256];
      for (int i = 0; i < 256; ++i) r2[i] = reconstruction(g->codes, g->gain, st[i]) * scale;
      for (int i = 0; i < 256; ++i) {
        const float d = residual[i] - r2[i];
        tmp[i] = d * d;
      }
      const float error = sum256(tmp);
      if (!finite32(error)) return KV_EINVAL;
      if (!have || error < best_error) {
        have = 1;
        best_error = error;
        memcpy(rec, r2, sizeof r2);
        memcpy(states, st, 256);
        *sel_scale = scale;
      }
    }
  } else if (g->mode == 1) {
    float m = 0.0f;
    for (int i = 0; i < 256; ++i) {
      const float a = fabsf(residual[i]);
      m = m > a ? m : a;
    }
    float scale = m / 7.0f;
    if (scale == 0.0f) scale = 1.0f;
    for (int i = 0; i < 256; ++i) {
      float r = nearbyintf(residual[i] / scale);
      r = r < -7.0f ? -7.0f : (r > 7.0f ? 7.0f : r);
      rec[i] = r * scale;
    }
    *sel_scale = scale;
  }
  for (int j = 0; j < nb; ++j)
    for (int i = 0; i < 256; ++i) rec[i] += coef[j] * g->basis[j * 256 + i];
  if (g->has_mean)
    for (int i = 0; i < 256; ++i) rec[i] += g->mean[i];
  for (int i = 0; i < 256; ++i)
    if (!finite32(rec[i])) return KV_EINVAL;
  return KV_OK;
}

/* kv_codec.rs:447-458: MSB-first fields in little-endian u32 words. */
static void pack_fields(const uint8_t* fields, int bits, uint32_t* words) {
  memset(words, 0, sizeof(uint32_t) * 8 * bits);
  for (int e = 0; e < 256; ++e)
    for (int j = 0; j < bits; ++j) {
      const int bit = e * bits + j;
      words[bit / 32] |= (uint32_t)((fields[e] >> (bits - 1 - j)) & 1) << (31 - bit % 32);
    }
}
static int field_of(const uint32_t* words, int bits, int channel) {
  int r = 0;
  for (int j = 0; j < bits; ++j) {
    const int bit = channel * bits + j;
    r = (r << 1) | (int)((words[bit / 32] >> (31 - bit % 32)) & 1);
  }
  return r;
}
/* kv_codec.rs:467-475 (src/q35_atxpk.cu:69-74): the last eight stream bits, reset each chain. */
int orc_kv_packed_state(const uint32_t* words, int bits, int channel) {
  int first = channel - 7 / bits;
  if (first < channel / 64 * 64) first = channel / 64 * 64;
  int state = 0;
  for (int i = first; i <= channel; ++i) state = ((state << bits) | field_of(words, bits, i)) & 0xff;
  return state;
}

/* encode_packed (kv_codec.rs:408-441) and requantize_int8 (:398-406) for one row.
 * Outputs: *kind = bits (packed) or 8 (int8); words (8*bits), ints (256), bases (256 bf16),
 * *scale; *req_scale + req_ints = requantize_int8 of the same row. */
int orc_kv_encode(const float* row, int position, int mode, int bits, const int16_t* codes, float gain, int guard,
                  int n_basis, const float* basis, const float* mean, const float* mults, int n_mult, int vit2,
                  int packable, int* kind, float* scale, uint32_t* words, int8_t* ints, uint16_t* bases,
                  float* req_scale, int8_t* req_ints) {
  kv_group g = {mode, bits, guard, n_basis, mean != 0, vit2, codes, gain, mean, basis, mults, n_mult};
  float rec[256], sel_scale;
  uint8_t states[256];
  int rc = kv_select(&g, position, row, rec, states, &sel_scale);
  if (rc) return rc;
  if (initial_int8(rec, req_ints, req_scale)) return KV_EINVAL;
  if (!packable) {
    *kind = 8;
    memcpy(ints, req_ints, 256);
    *scale = *req_scale;
    return KV_OK;
  }
  uint8_t fields[256];
  const int mask = (1 << bits) - 1;
  for (int i = 0; i < 256; ++i) fields[i] = states[i] & mask;
  pack_fields(fields, bits, words);
  *kind = bits;
  *scale = sel_scale;
  for (int i = 0; i < 256; ++i)
    bases[i] = orc_f32_to_bf16(reconstruction(codes, gain, orc_kv_packed_state(words, bits, i)));
  return KV_OK;
}

/* ------------------------------------------------------------ attention --
 * One query head, decode (one row), following crates/yskn-ref/src/attention.rs:
 * prefix_schedule splits, per-row 32-slot tiles (D9), online softmax with exp2,
 * BF16 prefix value weights, separate FP32 self term, packed value mean, split
 * combination with exp, division. Output: the rotated head (before the inverse
 * cache rotation). exp2 and exp are the reference's portable functions
 * (portable_math.rs:111-156,212-216, restated in portable_math.c), so this
 * reproduces attend_head bit for bit (pinned by attention.rs:1244-1306); the GPU
 * kernel sums in its own order and is checked within a tolerance.
 *   kb/vb: [length][256] bases as floats (bf16 values or int8 integers); ks/vs: scales. */
static const float LOG2E = 1.4426950408889634f;
int orc_kv_attend_head(const float* q, const float* kb, const float* ks, const float* vb, const float* vs,
                       const float* vmean /*256 or NULL*/, int length, int n_splits, float* out) {
  const int per_split = (length + n_splits - 1) / n_splits;
  int padded = 1;
  while (padded < n_splits) padded <<= 1;
  static float smax[64], sden[64], snum[64][256];
  for (int s = 0; s < padded; ++s) {
    smax[s] = -1e30f;
    sden[s] = 0.0f;
    memset(snum[s], 0, sizeof snum[s]);
  }
  for (int s = 0; s < n_splits; ++s) {
    const int first = s * per_split;
    const int last = first + per_split < length ? first + per_split : length;
    int prefix_end = last < length - 1 ? last : length - 1;
    if (prefix_end < first) prefix_end = first;
    const int include_self = first <= length - 1 && length - 1 < first + per_split;
    float mx = -1e30f, den = 0.0f, *num = snum[s];
    for (int t0 = first / 32 * 32; t0 < prefix_end; t0 += 32) {
      float sc[32], pr[32];
      int vis[32];
      float nm = mx;
      for (int k = 0; k < 32; ++k) {
        const int pos = t0 + k;
        vis[k] = pos >= first && pos < prefix_end;
        sc[k] = -INFINITY;
        if (vis[k]) {
          float acc = 0.0f;
          for (int c = 0; c < 256; ++c) acc += q[c] * kb[(size_t)pos * 256 + c];
          sc[k] = acc * (ks[pos] * 0.0625f);
        }
        if (sc[k] > nm) nm = sc[k];
      }
      const float rescale = orc_pm_exp2((mx - nm) * LOG2E);
      const float smx = nm * LOG2E;
      mx = nm;
      for (int k = 0; k < 32; ++k) pr[k] = vis[k] ? orc_pm_exp2(sc[k] * LOG2E - smx) : 0.0f;
      float part[4] = {0, 0, 0, 0};
      for (int lane = 0; lane < 4; ++lane)
        for (int grp = 0; grp < 4; ++grp) part[lane] += pr[8 * grp + 2 * lane] + pr[8 * grp + 2 * lane + 1];
      for (int d = 1; d <= 2; d <<= 1) {
        float old[4];
        memcpy(old, part, sizeof old);
        for (int lane = 0; lane < 4; ++lane) part[lane] = old[lane] + old[lane ^ d];
      }
      den = den * rescale + part[0];
      for (int c = 0; c < 256; ++c) num[c] *= rescale;
      for (int k = 0; k < 32; ++k) {
        if (!vis[k]) continue;
        const float w = bfloat_r(pr[k] * vs[t0 + k]);
        for (int c = 0; c < 256; ++c) num[c] += w * vb[(size_t)(t0 + k) * 256 + c];
      }
    }
    if (include_self) {
      const int self = length - 1;
      float part[4] = {0, 0, 0, 0};
      for (int lane = 0; lane < 4; ++lane)
        for (int ch = 0; ch < 16; ++ch) {
          const int offs[4] = {2 * lane, 2 * lane + 1, 8 + 2 * lane, 9 + 2 * lane};
          for (int o = 0; o < 4; ++o) {
            const int c = 16 * ch + offs[o];
            part[lane] += q[c] * kb[(size_t)self * 256 + c];
          }
        }
      for (int d = 1; d <= 2; d <<= 1) {
        float old[4];
        memcpy(old, part, sizeof old);
        for (int lane = 0; lane < 4; ++lane) part[lane] = old[lane] + old[lane ^ d];
      }
      const float score = part[0] * (ks[self] * 0.0625f);
      const float nm = mx > score ? mx : score;
      const float rescale = orc_pm_exp2((mx - nm) * LOG2E);
      const float p = orc_pm_exp2((score - nm) * LOG2E);
      mx = nm;
      den = den * rescale + p;
      const float w = p * vs[self];
      for (int c = 0; c < 256; ++c) num[c] = num[c] * rescale + w * vb[(size_t)self * 256 + c];
    }
    if (vmean)
      for (int c = 0; c < 256; ++c) num[c] += den * vmean[c];
    smax[s] = mx;
    sden[s] = den;
  }
  float largest = -1e30f;
  for (int s = 0; s < padded; ++s) largest = smax[s] > largest ? smax[s] : largest;
  float scl[64];
  for (int s = 0; s < padded; ++s) scl[s] = smax[s] > -1e29f ? orc_pm_exp(smax[s] - largest) : 0.0f;
  float total = 0.0f;
  for (int s = 0; s < padded; ++s) total += scl[s] * sden[s];
  if (!(total > 0.0f)) return KV_EINVAL;
  for (int c = 0; c < 256; ++c) {
    float n = 0.0f;
    for (int s = 0; s < padded; ++s) n += scl[s] * snum[s][c];
    out[c] = n / total;
  }
  return KV_OK;
}

/* attention.rs:997-1044: hash signs and the inverse cache rotation (H256, x1/16, signs). */
float orc_kv_cache_sign(int channel) {
  uint32_t v = (uint32_t)channel + 1u;
  v ^= v >> 16;
  v *= 0x7feb352du;
  v ^= v >> 15;
  v *= 0x846ca68bu;
  v ^= v >> 16;
  return (v & 1u) == 0 ? 1.0f : -1.0f;
}
void orc_kv_inverse_rotate(float* v) {
  for (int d = 1; d < 256; d *= 2)
    for (int b = 0; b < 256; b += 2 * d)
      for (int o = 0; o < d; ++o) {
        const float a = v[b + o], c = v[b + o + d];
        v[b + o] = a + c;
        v[b + o + d] = a - c;
      }
  for (int c = 0; c < 256; ++c) v[c] = (v[c] * 0.0625f) * orc_kv_cache_sign(c);
}

/* decode_packed (kv_codec.rs:485-495) for n_rows rows as floats: book[packed_state]. The
 * running fold (acc << bits | field) & 0xff, reset at each 64-channel chain, keeps exactly
 * the last eight stream bits, which is packed_state's window (kv_codec.rs:467-475). */
void orc_kv_decode_rows(const uint32_t* words, int64_t n_rows, int bits, const uint16_t* book_bf16, float* out) {
  const int W = 8 * bits;
  for (int64_t r = 0; r < n_rows; ++r) {
    const uint32_t* w = words + r * W;
    int acc = 0;
    for (int c = 0; c < 256; ++c) {
      if (c % 64 == 0) acc = 0;
      acc = ((acc << bits) | field_of(w, bits, c)) & 0xff;
      const uint32_t u = (uint32_t)book_bf16[acc] << 16;
      memcpy(out + r * 256 + c, &u, 4);
    }
  }
}
