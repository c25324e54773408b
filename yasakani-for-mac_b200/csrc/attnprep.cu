// Attention inputs from the q/k/v projections: per-head RMS norm, RoPE and the 256-element
// cache rotation (the step between the q/k/v operator and the KV encoder / attention).
//
// Reference: the head preparation of q35 attention (src/q35_kernels.cu:1013-1059, RoPE table
// :1091-1104), the cache rotation (src/kvx_codec.cuh:11-48); scalar spec docs/spec/
// 04_ATTENTION.md:15-106 with the helpers of 03_GATED_DELTANET.md:5-32. Per row and head:
//   y = bf16(projection); the query heads' gate halves are saved as bf16;
//   queries and keys: normalised by the head's RMS (8 groups of 32, xor_sum32, rsqrt) times
//   (1 + weight), bf16; RoPE on channels i, i+32 (i < 32) with bf16(cos/sin(p * freq[i]));
//   every query, key and value: x * cache_sign -> H256 (distances 1..128) -> * 1/16;
//   queries rounded to bf16, keys and values left in f32 (the encoder's input).
// rsqrt and sincos are the scalar contract's portable functions (attention.rs:732-775,
// portable_math.rs:106-109,406-434; pmath.cuh), so every output equals yskn-ref's bits.
//
// B200 design: one warp per (row, head); lane l holds channels l + 32g (g = 0..7), so a
// group of 32 channels is one value per lane (xor_sum32 is a shuffle butterfly), RoPE's
// pairs (l, l+32) are in the lane, and the cache rotation's distances 1..16 are lane
// shuffles and 32..128 are in the lane, in the spec's ascending order.
#include <cuda_bf16.h>

#include "common.cuh"
#include "pmath.cuh"

namespace yskn {

// Binary32 bit patterns of the 32 RoPE frequencies (docs/spec/04_ATTENTION.md:42-52).
__constant__ uint32_t c_rope_freq[32] = {
    0x3f800000u, 0x3f1ab32bu, 0x3ebaf81bu, 0x3e61f835u, 0x3e088d77u, 0x3da50956u, 0x3d47763fu, 0x3cf11177u,
    0x3c91ad39u, 0x3c301052u, 0x3bd4ca15u, 0x3b80967du, 0x3b1b690du, 0x3abbd3edu, 0x3a6301e2u, 0x3a092e02u,
    0x39a5cb60u, 0x394860c1u, 0x38f22ce2u, 0x3892587eu, 0x3830df52u, 0x37d5c441u, 0x37812dabu, 0x371c1fc4u,
    0x36bcb0c1u, 0x36640cc6u, 0x3609cf4au, 0x35a68e4cu, 0x35494c57u, 0x34f3499du, 0x3493048eu, 0x3431af44u};

__device__ __forceinline__ float bf(float x) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x)) << 16);
}

// src/kvx_codec.cuh:28-36: the fixed sign of cache channel c (unsigned 32-bit hash).
__device__ __forceinline__ float cache_sign(int c) {
  uint32_t x = (uint32_t)(c + 1);
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return (x & 1u) ? -1.0f : 1.0f;
}

struct PrepParams {
  const float* q;  // [M][n_qh][512]: 256 query channels, then 256 gate channels per head
  const float* k;  // [M][n_kvh][256]
  const float* v;  // [M][n_kvh][256]
  const uint16_t* q_norm;  // bf16 [256]
  const uint16_t* k_norm;  // bf16 [256]
  const int32_t* positions;  // [M]
  float eps;
  int M, n_qh, n_kvh;
  uint16_t* query;  // bf16 [M][n_qh][256]
  uint16_t* gate;   // bf16 [M][n_qh][256]
  float* k_rot;     // [M][n_kvh][256]
  float* v_rot;     // [M][n_kvh][256]
  unsigned* err;    // device error word
};

constexpr int PREP_WARPS = 8;

__global__ void __launch_bounds__(PREP_WARPS * 32) attention_prep_kernel(const __grid_constant__ PrepParams p) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int heads = p.n_qh + 2 * p.n_kvh;  // query heads, then key heads, then value heads
  const int item = blockIdx.x * PREP_WARPS + (threadIdx.x >> 5);
  if (item >= p.M * heads) return;
  const int m = item / heads, h = item - m * heads;
  const int kind = h < p.n_qh ? 0 : (h < p.n_qh + p.n_kvh ? 1 : 2);  // query, key, value
  const int hh = kind == 0 ? h : (kind == 1 ? h - p.n_qh : h - p.n_qh - p.n_kvh);
  const float* src = kind == 0 ? p.q + ((size_t)m * p.n_qh + hh) * 512
                               : (kind == 1 ? p.k : p.v) + ((size_t)m * p.n_kvh + hh) * 256;
  float x[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) x[g] = bf(src[32 * g + lane]);
  if (kind == 0) {  // the raw projected gate, bf16
    uint16_t* gd = p.gate + ((size_t)m * p.n_qh + hh) * 256;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      gd[32 * g + lane] = __bfloat16_as_ushort(__float2bfloat16_rn(src[256 + 32 * g + lane]));
  }
  if (kind != 2) {
    // normalize_head (04_ATTENTION.md:27-37): xor_sum32 of each group's squares, the
    // groups added from 0, rsqrtf(total / 256 + eps), bf16(y * inv * (1 + w)).
    float total = 0.0f;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      float s = __fmul_rn(x[g], x[g]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
      total = __fadd_rn(total, s);
    }
    const float inv = pm_rsqrt(__fadd_rn(__fdiv_rn(total, 256.0f), p.eps));
    const uint16_t* w = kind == 0 ? p.q_norm : p.k_norm;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      x[g] = bf(__fmul_rn(__fmul_rn(x[g], inv), __fadd_rn(1.0f, __uint_as_float((uint32_t)w[32 * g + lane] << 16))));
    // RoPE on channels (lane, lane + 32) = slots 0 and 1.
    const float arg = __fmul_rn((float)p.positions[m], __uint_as_float(c_rope_freq[lane]));
    float cs, sn;
    if (!pm_sincos(arg, &cs, &sn)) raise_device_error(p.err, DERR_RANGE);  // a position beyond the reduction's range
    const float c = bf(cs), s = bf(sn);
    const float n0 = x[0], n1 = x[1];
    x[0] = bf(__fadd_rn(bf(__fmul_rn(n0, c)), bf(__fmul_rn(-n1, s))));
    x[1] = bf(__fadd_rn(bf(__fmul_rn(n1, c)), bf(__fmul_rn(n0, s))));
  }
  // rotate_cache: signs, H256 with distances 1..128 ascending, * 1/16.
#pragma unroll
  for (int g = 0; g < 8; ++g) x[g] = __fmul_rn(x[g], cache_sign(32 * g + lane));
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const bool upper = (lane & d) != 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const float o = __shfl_xor_sync(0xffffffffu, x[g], d);
      x[g] = upper ? __fsub_rn(o, x[g]) : __fadd_rn(x[g], o);
    }
  }
#pragma unroll
  for (int b = 1; b < 8; b <<= 1) {  // distances 32, 64, 128: slot bits
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g & b) continue;
      const float lo = x[g], hi = x[g | b];
      x[g] = __fadd_rn(lo, hi);
      x[g | b] = __fsub_rn(lo, hi);
    }
  }
  if (kind == 0) {
    uint16_t* qd = p.query + ((size_t)m * p.n_qh + hh) * 256;
#pragma unroll
    for (int g = 0; g < 8; ++g) qd[32 * g + lane] = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(x[g], 0.0625f)));
  } else {
    float* od = (kind == 1 ? p.k_rot : p.v_rot) + ((size_t)m * p.n_kvh + hh) * 256;
#pragma unroll
    for (int g = 0; g < 8; ++g) od[32 * g + lane] = __fmul_rn(x[g], 0.0625f);
  }
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_attention_prep(const float* d_q, const float* d_k, const float* d_v,
                                                     const uint16_t* d_q_norm, const uint16_t* d_k_norm,
                                                     const int32_t* d_positions, float eps, int M, int n_qh,
                                                     int n_kvh, uint16_t* d_query, uint16_t* d_gate, float* d_k_rot,
                                                     float* d_v_rot, void* stream) {
  if (!d_q || !d_k || !d_v || !d_q_norm || !d_k_norm || !d_positions || !d_query || !d_gate || !d_k_rot || !d_v_rot ||
      M < 1 || n_qh < 1 || n_kvh < 1)
    return fail(YSKN_EINVAL, "attention_prep: null argument or empty shape");
  PrepParams p{d_q, d_k, d_v, d_q_norm, d_k_norm, d_positions, eps, M, n_qh, n_kvh, d_query, d_gate, d_k_rot, d_v_rot,
               device_error_word()};
  const int64_t items = (int64_t)M * (n_qh + 2 * n_kvh);
  if (items > (int64_t)INT32_MAX) return fail(YSKN_EINVAL, "attention_prep: too many rows");
  return cuda_fail(launch_pdl(attention_prep_kernel, (unsigned)((items + PREP_WARPS - 1) / PREP_WARPS),
                              PREP_WARPS * 32, 0, reinterpret_cast<cudaStream_t>(stream), p),
                   "attention_prep_kernel");
}
