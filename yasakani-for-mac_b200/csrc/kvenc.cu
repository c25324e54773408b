// Quantised-KV row encoder for packed rows (trellis, kb = 4 or 5 bits per channel).
//
// Reference: launch_tb_fast -> tbf_vit_kernel / tbf2_vit_kernel + tbf_sel_kernel
// (src/kvq_fast.cuh:150-249, src/kvq_vit2.cuh:217); scalar spec encode_packed and
// select (crates/yskn-ref/src/kv_codec.rs:117-264,272-396,408-458); the profile
// predicates of kv_profile.rs:251-286 decide which rows are packed and whether the
// compressed (vit2) recurrence is used.
//
// A packed row's group has mode 0, no guard and no basis (the packable condition),
// so select() reduces to: initial int8 row (max/127, rne, clamp), y = q * s0,
// residual = y - mean, rms = sqrt(sum256(residual^2) / 256) (1 if zero), then per
// profile multiplier: scale = half(rms * mult) (1 if zero), targets = clamp(rne(
// residual / scale * 256), +-2048), a 64-step Viterbi on each of the four 64-channel
// chains, and error = sum256((residual - reconstruction(state) * scale)^2); the
// lowest error wins, the first multiplier on ties.
//
// kv_encode_kernel: one CTA of 16 warps per row. The float steps run one thread per
// channel, single-rounded binary32 operations in the scalar order (sum256: XOR
// butterflies 16..1 in each warp, the eight warp sums folded from +0). The chains
// of up to 4 multipliers run at once, each chain in one warp: each lane evaluates 8
// candidate transitions per step and costs are double-buffered in shared memory, so
// a step needs one __syncwarp. Integer arithmetic is i32 like the reference; where a
// bound does not already rule overflow out (|target| <= 2048, |code| <= 32768; vit2
// requires |code| <= 1100 and the kernel checks it), the add is checked, and an
// overflow or a non-finite value fails the row (nothing is written for it). The CTA
// then keeps the lowest-error candidate and packs its fields MSB-first into 8*kb
// words at the row's destination, with its scale.
#include <cuda_fp16.h>

#include "common.cuh"

namespace yskn {

struct KvEncParams {
  const float* rows;          // [n_rows][256]
  const int32_t* row_group;   // [n_rows]
  const int16_t* tables;      // [n_groups][256]
  const float* gains;         // [n_groups]
  const float* means;         // [n_groups][256] or nullptr
  const uint8_t* has_mean;    // [n_groups] or nullptr (all groups have a mean if means != nullptr)
  const float* mults;         // [n_mult]
  const int64_t* dest;        // [n_rows] destination row index, or nullptr (row i)
  uint32_t* words;            // [*][8*kb]
  float* scales;              // [*]
  int n_rows, n_mult, kb, vit2;
  unsigned* err;
};

__device__ __forceinline__ bool kv_finite(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

// kv_codec.rs:228-245: XOR butterflies 16, 8, 4, 2, 1 in each warp, then the eight
// warp sums folded from +0 in order. Every thread gets the total. red: 8 floats.
__device__ __forceinline__ float kv_sum256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) total = __fadd_rn(total, red[w]);
  __syncthreads();
  return total;
}

__device__ __forceinline__ bool add_ovf(int32_t a, int32_t b, int32_t& r) {
  r = (int32_t)((uint32_t)a + (uint32_t)b);
  return ((a ^ r) & (b ^ r)) < 0;
}
__device__ __forceinline__ bool sub_ovf(int32_t a, int32_t b, int32_t& r) {
  r = (int32_t)((uint32_t)a - (uint32_t)b);
  return ((a ^ b) & (a ^ r)) < 0;
}

// general_chain (kv_codec.rs:117-146), one warp: predecessor group u = lane / PER
// (PER = 32 / stride lanes per group) takes its lowest cost over j, lowest j on
// ties; lane q = lane % PER owns j = q*8 .. q*8+7 and the 8 states (u << KB) | j.
// (x - code)^2 <= 34816^2 fits in i32; only the add of the best cost is checked.
template <int KB>
__device__ void general_chain_warp(const int32_t* target, const int16_t* codes, int lane, int32_t* cbuf /*[2][256]*/,
                                   uint8_t* bp /*[64][16]*/, uint8_t* path, bool& bad) {
  constexpr int STRIDE = 256 >> KB, PER = 32 / STRIDE;
  const int u = lane / PER, q = lane % PER;
  int32_t code[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) code[k] = codes[(u << KB) | (q * 8 + k)];
  for (int s = lane; s < 256; s += 32) cbuf[s] = s == 0 ? 0 : 0x40000000;
  __syncwarp();
  int cur = 0;
  for (int step = 0; step < 64; ++step) {
    const int32_t* cost = cbuf + cur * 256;
    int32_t* next = cbuf + (cur ^ 1) * 256;
    const int32_t x = target[step];
    int32_t best = cost[(q * 8) * STRIDE + u];
    int choice = q * 8;
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      const int32_t c = cost[(q * 8 + k) * STRIDE + u];
      if (c < best) {
        best = c;
        choice = q * 8 + k;
      }
    }
#pragma unroll
    for (int o = 1; o < PER; o <<= 1) {
      const int32_t ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oc = __shfl_xor_sync(0xffffffffu, choice, o);
      if (ob < best || (ob == best && oc < choice)) {
        best = ob;
        choice = oc;
      }
    }
    if (q == 0) bp[step * 16 + u] = (uint8_t)choice;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int32_t dx = x - code[k];
      int32_t r;
      bad |= add_ovf(dx * dx, best, r);
      next[(u << KB) | (q * 8 + k)] = r;
    }
    __syncwarp();
    cur ^= 1;
  }
  // Lowest final cost as u32, lowest state on ties.
  const int32_t* cost = cbuf + cur * 256;
  uint32_t bv = (uint32_t)cost[lane * 8];
  int bs = lane * 8;
#pragma unroll
  for (int k = 1; k < 8; ++k)
    if ((uint32_t)cost[lane * 8 + k] < bv) {
      bv = (uint32_t)cost[lane * 8 + k];
      bs = lane * 8 + k;
    }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int os = __shfl_xor_sync(0xffffffffu, bs, o);
    if (ov < bv || (ov == bv && os < bs)) {
      bv = ov;
      bs = os;
    }
  }
  if (lane == 0) {
    int state = bs;
    for (int step = 63; step >= 0; --step) {
      path[step] = (uint8_t)state;
      state = ((int)bp[step * 16 + (state >> KB)] << (8 - KB)) | (state >> KB);
    }
  }
  __syncwarp();
}

// vit2_chain (kv_codec.rs:148-211), one warp: the compressed recurrence whose costs
// carry the backpointer in their low KB bits. Group g = lane / PER (stride groups);
// lane q = lane % PER evaluates NS = 8 / (KB - 3) transitions j (kb 5: j even, each
// with the odd partner d + stride folded in by min). With |code| <= 1100 every term
// fits in i32 (|bc * x| <= 2*32*1100*2048); the cost adds are checked.
template <int KB>
__device__ void vit2_chain_warp(const int32_t* target, const int16_t* codes, int lane, int32_t* cbuf /*[2][16]*/,
                                uint8_t* bp /*[64][16]*/, uint8_t* path, bool& bad) {
  constexpr int FIELDS = 1 << KB, STRIDE = 256 >> KB, PER = 32 / STRIDE, NS = KB == 5 ? 4 : 8;
  constexpr int32_t F = FIELDS;
  const int g = lane / PER, q = lane % PER;
  int32_t ac[NS], bc[NS], ac2[NS], bc2[NS];
  int ci[NS];
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    const int j = KB == 5 ? (q * NS + k) * 2 : q * NS + k;
    const int d = STRIDE * j + g;
    const int32_t c = codes[d];
    ac[k] = F * c * c + d / STRIDE;
    bc[k] = -2 * F * c;
    ci[k] = d >> KB;
    if (KB == 5) {
      const int32_t c2 = codes[d + STRIDE];
      ac2[k] = F * c2 * c2 + (d + STRIDE) / STRIDE;
      bc2[k] = -2 * F * c2;
    } else {
      ac2[k] = 0;
      bc2[k] = 0;
    }
  }
  if (lane < STRIDE) cbuf[lane] = lane == 0 ? 0 : (F << 24);
  __syncwarp();
  int cur = 0;
  int32_t final_k = 0x7fffffff, final_state = 0x7fffffff;
  for (int step = 0; step < 64; ++step) {
    const int32_t* cost = cbuf + cur * 16;
    const int32_t x = target[step];
    const int32_t square = x * x * F;
    int32_t best = 0x7fffffff;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      int32_t e = ac[k] + bc[k] * x;
      if (KB == 5) e = min(e, ac2[k] + bc2[k] * x);
      int32_t r;
      bad |= add_ovf(e, cost[ci[k]], r);
      best = min(best, r);
    }
#pragma unroll
    for (int o = 1; o < PER; o <<= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
    int32_t k;
    bad |= add_ovf(best, square, k);
    if (step == 63) {
      if (q == 0) {
        final_k = k >> KB;
        final_state = STRIDE * (k & (FIELDS - 1)) + g;
      }
    } else if (q == 0) {
      int32_t k2;
      bad |= sub_ovf(k, cost[0], k2);
      cbuf[(cur ^ 1) * 16 + g] = k2 & ~(F - 1);
      bp[(step + 1) * 16 + g] = (uint8_t)(k2 & (F - 1));
    }
    __syncwarp();
    cur ^= 1;
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {  // lowest key, then lowest state
    const int32_t ok = __shfl_xor_sync(0xffffffffu, final_k, o);
    const int32_t os = __shfl_xor_sync(0xffffffffu, final_state, o);
    if (ok < final_k || (ok == final_k && os < final_state)) {
      final_k = ok;
      final_state = os;
    }
  }
  if (lane == 0) {
    int state = final_state;
    for (int step = 63; step >= 1; --step) {
      path[step] = (uint8_t)state;
      state = ((int)bp[step * 16 + (state >> KB)] << (8 - KB)) | (state >> KB);
    }
    path[0] = (uint8_t)state;
  }
  __syncwarp();
}

constexpr int ENC_THREADS = 512;  // 16 warps: 4 multipliers x 4 chains at a time
constexpr int ENC_BATCH = 4;      // multipliers per pass

struct EncSmem {
  int32_t cost[ENC_BATCH * 4][2 * 256];  // per (multiplier of the pass, chain), double-buffered
  uint8_t bp[ENC_BATCH * 4][64 * 16];
  int32_t target[ENC_BATCH][256];
  uint8_t states[ENC_BATCH][256];
  uint8_t best_states[256];
  int16_t codes[256];
  float red[16];
  float s_max[16];
  float scale[ENC_BATCH];
  float best_scale;
  int bad;
};

// One CTA (512 threads) per row: the float steps with thread = channel (warps
// 0..7), the chains of up to 4 multipliers at once (warp w: multiplier w / 4 of the
// pass, chain w % 4), the candidate errors, the choice and the packed fields.
__global__ void __launch_bounds__(ENC_THREADS) kv_encode_kernel(const __grid_constant__ KvEncParams p) {
  extern __shared__ __align__(16) uint8_t enc_raw[];
  EncSmem& S = *reinterpret_cast<EncSmem*>(enc_raw);
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool chan = tid < 256;
  const int c = tid & 255;
  pdl_begin();  // the rows may be the previous kernel's output; the attention may start its set-up
  const int grp = p.row_group[row];
  const float x = chan ? p.rows[(size_t)row * 256 + c] : 0.0f;
  bool bad = false;
  if (chan) {
    const int16_t code = p.tables[(size_t)grp * 256 + c];
    S.codes[c] = code;
    bad = !kv_finite(x) || (p.vit2 && (code > 1100 || code < -1100));
  }
  if (tid == 0) {
    S.bad = 0;
    S.best_scale = 0.0f;
  }
  // initial_int8 (kv_codec.rs:247-264)
  float a = fabsf(x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if (lane == 0) S.s_max[warp] = a;
  __syncthreads();
  float maximum = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) maximum = fmaxf(maximum, S.s_max[w]);
  const float s0 = __fdiv_rn(maximum, 127.0f);
  float q = 0.0f;
  if (s0 > 0.0f) q = fminf(127.0f, fmaxf(-127.0f, rintf(__fdiv_rn(x, s0))));
  const float y = __fmul_rn(q, s0);
  const bool has_mean = p.means && (!p.has_mean || p.has_mean[grp]);
  const float res = (has_mean && chan) ? __fsub_rn(y, p.means[(size_t)grp * 256 + c]) : y;
  bad |= !kv_finite(res);
  float rms = __fsqrt_rn(__fdiv_rn(kv_sum256(chan ? __fmul_rn(res, res) : 0.0f, S.red), 256.0f));
  if (rms == 0.0f) rms = 1.0f;
  bad |= !kv_finite(rms);
  float best_error = 0.0f;
  for (int m0 = 0; m0 < p.n_mult; m0 += ENC_BATCH) {
    const int nb = min(ENC_BATCH, p.n_mult - m0);
    if (tid < nb) {
      float scale = __half2float(__float2half_rn(__fmul_rn(rms, p.mults[m0 + tid])));
      if (scale == 0.0f) scale = 1.0f;
      bad |= !kv_finite(scale);
      S.scale[tid] = scale;
    }
    __syncthreads();
    if (chan) {  // targets of the pass's multipliers
      for (int b = 0; b < nb; ++b) {
        const float tr = fminf(2048.0f, fmaxf(-2048.0f, rintf(__fmul_rn(__fdiv_rn(res, S.scale[b]), 256.0f))));
        S.target[b][c] = (int32_t)tr;
      }
    }
    __syncthreads();
    {
      const int b = warp >> 2, chain = warp & 3;
      if (b < nb) {
        const int32_t* tg = S.target[b] + 64 * chain;
        uint8_t* path = S.states[b] + 64 * chain;
        int32_t* cb = S.cost[warp];
        uint8_t* bpp = S.bp[warp];
        if (p.vit2) {
          if (p.kb == 4) vit2_chain_warp<4>(tg, S.codes, lane, cb, bpp, path, bad);
          else vit2_chain_warp<5>(tg, S.codes, lane, cb, bpp, path, bad);
        } else {
          if (p.kb == 4) general_chain_warp<4>(tg, S.codes, lane, cb, bpp, path, bad);
          else general_chain_warp<5>(tg, S.codes, lane, cb, bpp, path, bad);
        }
      }
    }
    __syncthreads();
    const float gain = p.gains[grp];
    for (int b = 0; b < nb; ++b) {
      float d2 = 0.0f;
      if (chan) {
        const float r2 =
            __fmul_rn(__fmul_rn(__fmul_rn((float)S.codes[S.states[b][c]], 0.00390625f), gain), S.scale[b]);
        const float d = __fsub_rn(res, r2);
        d2 = __fmul_rn(d, d);
      }
      const float error = kv_sum256(d2, S.red);
      bad |= !kv_finite(error);
      if (m0 + b == 0 || error < best_error) {  // first multiplier wins ties
        best_error = error;
        if (chan) S.best_states[c] = S.states[b][c];
        if (tid == 0) S.best_scale = S.scale[b];
      }
    }
    __syncthreads();
  }
  if (bad) S.bad = 1;
  __syncthreads();
  if (S.bad) {
    if (tid == 0) raise_device_error(p.err, DERR_NONFINITE);
    return;
  }
  // Pack the chosen fields MSB-first (kv_codec.rs:447-458).
  const int kb = p.kb, W = 8 * kb, mask = (1 << kb) - 1;
  const int64_t dst = p.dest ? p.dest[row] : row;
  if (tid < W) {
    uint32_t w = 0;
    for (int bb = 0; bb < 32; ++bb) {
      const int bit = 32 * tid + bb, e = bit / kb, j = bit - e * kb;
      w |= (uint32_t)(((S.best_states[e] & mask) >> (kb - 1 - j)) & 1) << (31 - bb);
    }
    p.words[dst * W + tid] = w;
  }
  if (tid == 0) p.scales[dst] = S.best_scale;
}

int launch_kv_encode(const KvEncArgs& a, cudaStream_t st) {
  KvEncParams p{};
  p.rows = a.rows;
  p.row_group = a.row_group;
  p.tables = a.tables;
  p.gains = a.gains;
  p.means = a.means;
  p.has_mean = a.has_mean;
  p.mults = a.mults;
  p.dest = a.dest;
  p.words = a.words;
  p.scales = a.scales;
  p.n_rows = a.n_rows;
  p.n_mult = a.n_mult;
  p.kb = a.kb;
  p.vit2 = a.vit2;
  p.err = device_error_word();
  static bool attr[64] = {};
  int dev = 0;
  if (int rc = cuda_fail(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(YSKN_EINVAL, "device ordinal out of range");
  if (!attr[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kv_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(EncSmem));
    if (e != cudaSuccess) return cuda_fail(e, "kv encode attributes");
    attr[dev] = true;
  }
  return cuda_fail(launch_pdl(kv_encode_kernel, a.n_rows, ENC_THREADS, sizeof(EncSmem), st, p), "kv_encode_kernel");
}

}  // namespace yskn
