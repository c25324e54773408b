// Device functions of the operator prologue (activation quantiser) and epilogue
// (restore + output rotation), shared by the standalone kernels (quant.cu) and the
// fused decode operator (gemv.cu), so both produce the same bits.
//
// Bit-exact restatements of the reference's scalar order (docs/spec/
// 02_COMPRESSED_LINEAR.md:84-101,129-241; crates/yskn-ref/src/compressed_linear.rs:
// 14-29,57-135,288-370). Every binary32 operation is an explicit round-to-nearest
// intrinsic, so no multiply-add contraction can occur (the reference build relies on
// --fmad=false, CMakeLists.txt:47-51).
//
// One warp transforms one 512-element block: lane l holds elements 16l..16l+15. The
// Hadamard butterflies run in ascending stride order as the spec requires: strides
// 1..8 inside a lane, 16..256 across lanes (shfl_xor with lane bit stride/16). Each
// element's value after every stage is the same binary32 value the scalar loop
// produces, so the parallel transform is bit-identical.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "pmath.cuh"

namespace yskn {

// One butterfly across lanes: the lower lane keeps v + other, the upper lane other - v.
// Both are fma(v, s, other) with s = +1 or -1: v * s is exact, so the single rounding
// of the fma gives exactly fadd_rn(v, other) or fsub_rn(other, v) (signed zeros, infinities
// and NaN included), in one instruction instead of an add, a subtract and a select.
__device__ __forceinline__ float cross_butterfly(float v, float other, float s) { return __fmaf_rn(v, s, other); }

__device__ __forceinline__ void hadamard512_warp(float (&v)[16], int lane) {
#pragma unroll
  for (int stride = 1; stride < 16; stride <<= 1) {
#pragma unroll
    for (int base = 0; base < 16; base += 2 * stride) {
#pragma unroll
      for (int o = 0; o < stride; ++o) {
        const float lower = v[base + o], upper = v[base + o + stride];
        v[base + o] = __fadd_rn(lower, upper);
        v[base + o + stride] = __fsub_rn(lower, upper);
      }
    }
  }
#pragma unroll
  for (int mask = 1; mask < 32; mask <<= 1) {
    const float s = (lane & mask) ? -1.0f : 1.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = cross_butterfly(v[e], __shfl_xor_sync(0xffffffffu, v[e], mask), s);
  }
}

__device__ __forceinline__ bool finite32(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

// The lane's share of one 512-column group: inputs 16*lane .. 16*lane+15 and their signs.
struct Group512In {
  float4 x[4];
  int4 s;
};
__device__ __forceinline__ void load_group512(const float* __restrict__ xg, const int8_t* __restrict__ sg, int lane,
                                              Group512In& in) {
  const float4* xp = reinterpret_cast<const float4*>(xg + lane * 16);
  in.s = __ldg(reinterpret_cast<const int4*>(sg + lane * 16));
#pragma unroll
  for (int q = 0; q < 4; ++q) in.x[q] = __ldg(xp + q);
}

// rne(fl(v / scale)) as an int, where scale > 0 and |v / scale| <= 128: the quotient
// is estimated as y = v * rcp (rcp = 1/scale correctly rounded), within 1.5 * 2^-23
// relative of the correctly rounded quotient, i.e. within 2.3e-5 of it. Unless y lies
// within 2^-14 of a half-integer, both round to the same integer, read off
// y + 1.5 * 2^23 (exact round-to-nearest-even into the low mantissa bits). Otherwise,
// and for non-finite values, the exact division decides.
__device__ __forceinline__ int quotient_rne(float v, float scale, float rcp) {
  const float y = __fmul_rn(v, rcp);
  const float t = __fadd_rn(y, 12582912.0f);                 // 1.5 * 2^23
  const float d = __fsub_rn(y, __fsub_rn(t, 12582912.0f));  // y - rne(y), exact
  if (fabsf(d) < 0.49993896484375f) return (int)(__float_as_uint(t) - 0x4B400000u);  // 0.5 - 2^-14
  return __float2int_rn(__fdiv_rn(v, scale));
}

// One 512-column group of one activation row (compressed_linear.rs:57-112): x*s_in,
// H512, half(v * 1/sqrt(512)), alpha = max|v|/127, q = clamp(rne(v/alpha), +-127).
// in: the lane's inputs and signs (load_group512); the lane's 16 int8 go to dst
// (16-byte aligned). Returns alpha on every lane; `bad` collects non-finite values.
__device__ __forceinline__ float quantize_loaded512(const Group512In& in, int8_t* dst, int lane, bool& bad) {
  float v[16];
  const uint32_t* sw = reinterpret_cast<const uint32_t*>(&in.s);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = in.x[q];
    v[4 * q + 0] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
  }
  // x * s for s = +1/-1 is x with its sign bit flipped when s < 0 (bit 7 of the sign
  // byte). For a NaN x the product would be the canonical NaN instead, but every value
  // then passes through an add of the first butterfly, which makes any NaN canonical.
  // Inputs are not checked for finiteness here: every output of the transform is a
  // signed sum of all 512 inputs, so a NaN or infinite input leaves every output NaN or
  // infinite, and the check after the transform reports it.
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const uint32_t flip = (sw[e >> 2] << (24 - 8 * (e & 3))) & 0x80000000u;
    v[e] = __uint_as_float(__float_as_uint(v[e]) ^ flip);
  }
  hadamard512_warp(v, lane);
  float mx = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    v[e] = __half2float(__float2half_rn(__fmul_rn(v[e], kHadamardNorm)));
    bad |= !finite32(v[e]);
    mx = fmaxf(mx, fabsf(v[e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float scale = __fdiv_rn(mx, 127.0f);
  const float rcp = __frcp_rn(scale);
  uint32_t packed[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      int r = scale > 0.0f ? quotient_rne(v[4 * q + b], scale, rcp) : 0;
      r = max(-127, min(127, r));
      w |= (uint32_t)(r & 0xff) << (8 * b);
    }
    packed[q] = w;
  }
  *reinterpret_cast<uint4*>(dst + lane * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  return scale;
}
// xg, sg: the group's 512 inputs and input signs.
__device__ __forceinline__ float quantize_group512(const float* __restrict__ xg, const int8_t* __restrict__ sg,
                                                   int8_t* dst, int lane, bool& bad) {
  Group512In in;
  load_group512(xg, sg, lane, in);
  return quantize_loaded512(in, dst, lane, bad);
}

// The row's common 2^24 integer grid (compressed_linear.rs:113-128) from its group
// scales: multiplier 2^24 / max alpha, and row_quantum = max alpha * 2^-24.
__device__ __forceinline__ float row_grid_multiplier(float max_alpha) {
  return max_alpha > 0.0f ? __fdiv_rn(16777216.0f, max_alpha) : 0.0f;
}
__device__ __forceinline__ int32_t integer_group_scale(float alpha, float mult) {
  return __float2int_rn(__fmul_rn(alpha, mult));
}
__device__ __forceinline__ float row_quantum_of(float max_alpha) {
  return __fmul_rn(max_alpha, 5.9604644775390625e-08f /* 2^-24 */);
}

// f32(ws) * row_quantum (* inv_rms) * tau (compressed_linear.rs:288-312).
__device__ __forceinline__ float restore_value(long long ws, float rq, const float* inv_rms_m, float tau) {
  float t = __fmul_rn(__ll2float_rn(ws), rq);
  if (inv_rms_m) t = __fmul_rn(t, *inv_rms_m);
  return __fmul_rn(t, tau);
}

// One 512-row block of one token (compressed_linear.rs:313-348): restore, H512,
// * 1/sqrt(512), * s_out; rows >= n_rows are not stored. Lane l holds rows
// 64k + 2l + b (k = 0..7, b = 0..1), so each of the warp's loads and stores is one
// contiguous access (512 B of int64, 256 B of f32), and the butterflies still run in
// ascending stride order: stride 1 in the lane (b), 2..32 across lanes (lane bits),
// 64..256 in the lane (k). ws is read through L2 (other SMs may have written it in
// the same launch).
// The same in separate load and transform steps, for a caller restoring several tokens
// of a block: it requests the next token's sums before transforming this token's.
struct Rows512 {  // the block's row scales and output signs, the same for every token
  float2 tau[8];
  char2 sg[8];
};
__device__ __forceinline__ void load_rows512(const float* __restrict__ tau, const int8_t* __restrict__ s_out, int r0,
                                             int lane, Rows512& rr) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + 64 * k + 2 * lane;
    rr.tau[k] = __ldg(reinterpret_cast<const float2*>(tau + r));
    rr.sg[k] = __ldg(reinterpret_cast<const char2*>(s_out + r));
  }
}
__device__ __forceinline__ void load_sums512(const int64_t* wsr, int r0, int lane, longlong2 (&w)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) w[k] = __ldcg(reinterpret_cast<const longlong2*>(wsr + r0 + 64 * k + 2 * lane));
}
// The block's outputs y (restored, H512, / sqrt(512), output signs) in v[2k + b] for rows
// r0 + 64k + 2l + b, from sums already loaded.
__device__ __forceinline__ void restore_values512(const longlong2 (&w)[8], const Rows512& rr, float rq,
                                                  const float* inv_rms_m, int lane, bool& bad, float (&v)[16]) {
  if (inv_rms_m) bad |= !finite32(*inv_rms_m);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[2 * k] = restore_value(w[k].x, rq, inv_rms_m, rr.tau[k].x);
    v[2 * k + 1] = restore_value(w[k].y, rq, inv_rms_m, rr.tau[k].y);
    bad |= !finite32(v[2 * k]) | !finite32(v[2 * k + 1]);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // stride 1
    const float lower = v[2 * k], upper = v[2 * k + 1];
    v[2 * k] = __fadd_rn(lower, upper);
    v[2 * k + 1] = __fsub_rn(lower, upper);
  }
#pragma unroll
  for (int mask = 1; mask < 32; mask <<= 1) {  // strides 2..32
    const float s = (lane & mask) ? -1.0f : 1.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = cross_butterfly(v[e], __shfl_xor_sync(0xffffffffu, v[e], mask), s);
  }
#pragma unroll
  for (int kb = 1; kb < 8; kb <<= 1) {  // strides 64, 128, 256
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k & kb) continue;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const float lower = v[2 * k + b], upper = v[2 * (k + kb) + b];
        v[2 * k + b] = __fadd_rn(lower, upper);
        v[2 * (k + kb) + b] = __fsub_rn(lower, upper);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[2 * k] = __fmul_rn(__fmul_rn(v[2 * k], kHadamardNorm), (float)rr.sg[k].x);
    v[2 * k + 1] = __fmul_rn(__fmul_rn(v[2 * k + 1], kHadamardNorm), (float)rr.sg[k].y);
    bad |= !finite32(v[2 * k]) | !finite32(v[2 * k + 1]);
  }
}
// Rows r0 + 64k + 2l + b of y (rows >= n_rows not stored).
__device__ __forceinline__ void store_rows512(const float (&v)[16], int r0, int n_rows, float* __restrict__ yr,
                                              int lane) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + 64 * k + 2 * lane;
    float* dst = yr + r;
    if (r + 1 < n_rows && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
      *reinterpret_cast<float2*>(dst) = make_float2(v[2 * k], v[2 * k + 1]);
    } else {
      if (r < n_rows) dst[0] = v[2 * k];
      if (r + 1 < n_rows) dst[1] = v[2 * k + 1];
    }
  }
}
__device__ __forceinline__ void restore_loaded512(const longlong2 (&w)[8], const Rows512& rr, float rq,
                                                  const float* inv_rms_m, int r0, int n_rows, float* __restrict__ yr,
                                                  int lane, bool& bad) {
  float v[16];
  restore_values512(w, rr, rq, inv_rms_m, lane, bad, v);
  store_rows512(v, r0, n_rows, yr, lane);
}

// ---------------------------------------------------------------------------------------
// Residual epilogue (the f1 chain): a restored and rotated 512-row block of a projection
// whose output is added to the residual stream, the block's part of the next RMS
// normalisation and the next operator's quantised input, in the restore's lane mapping
// (lane l holds rows 64k + 2l + b). Every step keeps the scalar order of the reference
// (residual_norm_mlp.rs:14-61,120-135; compressed_linear.rs:57-112):
//   h = bf16(h + bf16(y));  x = h * (1 + w);  gate copy bf16(x);
//   block sum of squares of h: partial t = sum_{j<4} h[t + 128 j]^2 from +0, an XOR butterfly
//   (offsets 16..1) over each group of 32 partials, the four group sums added in order;
//   quantiser: x * s_next -> H512 (strides 1..256 ascending) -> half(v / sqrt(512)) ->
//   alpha = max |v| / 127 -> q = clamp(rne(v / alpha), +-127).
struct ResidualOut {
  uint16_t* hidden;        // bf16 [rows] of this token (in and out)
  const uint16_t* norm_w;  // bf16 [rows]
  const int8_t* s_next;    // the next operator's input signs [rows]
  int8_t* act;             // int8 [rows] of this token
  float* alpha;            // [rows / 512] of this token
  float* bss;              // [rows / 512] of this token
  uint16_t* gate;          // bf16 [rows] of this token, or nullptr
};

// The residual prologue's inputs (see GemvParams::rin).
struct ResidualIn {
  const float* y;           // f32 [M][cols]: the previous projection's restored rows
  const uint16_t* h_in;     // bf16 [M][cols]: the residual stream before it
  uint16_t* h_out;          // bf16 [M][cols]: after it (CTA 0)
  const uint16_t* norm_w;   // bf16 [cols]
  uint16_t* gate_out;       // bf16 [M][cols] copy of h * (1 + w), or nullptr (CTA 0)
  float* inv_out;           // f32 [M] 1/rms, or nullptr (CTA 0)
  float eps;
};

__device__ __forceinline__ float bf16_round(float x) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x)) << 16);
}

// The MLP's gated product of one element in the scalar order of the reference
// (residual_norm_mlp.rs; docs/spec/05_RESIDUAL_NORM_MLP.md): bf16(bf16(silu(bf16(g))) * bf16(u)).
__device__ __forceinline__ float gated_product_value(float g, float u) {
  return bf16_round(__fmul_rn(bf16_round(pm_silu(bf16_round(g))), bf16_round(u)));
}

// The residual epilogue of one token's 512-row block from its projection values v (the
// restore's lane mapping) and the block's residual-stream, norm-weight and next-sign words
// (hws, wws, sws: rows r + 2l, r + 2l + 1 at k = 0..7, r = 64k), in the scalar order above.
// Writes the updated residual words to hidden_out and the gate copy to gate_out (each if
// non-null; rows 64k + 2l + b from each pointer), the block's int8 input to act (same
// rows), and lane 0 writes the block's group scale to *alpha and its sum of squares to *bss.
__device__ __forceinline__ void residual_block512(float (&v)[16], const uint32_t (&hws)[8], const uint32_t (&wws)[8],
                                                  const uint32_t (&sws)[8], uint16_t* hidden_out, uint16_t* gate_out,
                                                  int8_t* act, float* alpha, float* bss, int lane, bool& bad) {
  float x[16];  // the next operator's unnormalised input h * (1 + w)
  // residual and the next normalisation's input
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = 64 * k + 2 * lane;
    const uint32_t hw = hws[k], ww = wws[k];
    uint32_t hn = 0, gw = 0;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const float h = __uint_as_float((b ? hw & 0xffff0000u : hw << 16));
      const float w = __uint_as_float((b ? ww & 0xffff0000u : ww << 16));
      const float nh = bf16_round(__fadd_rn(h, bf16_round(v[2 * k + b])));
      const float xv = __fmul_rn(nh, __fadd_rn(1.0f, w));
      x[2 * k + b] = xv;
      v[2 * k + b] = nh;
      hn |= (__float_as_uint(nh) >> 16) << (16 * b);
      gw |= (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(xv)) << (16 * b);
      bad |= !finite32(nh) | !finite32(xv);
    }
    if (hidden_out) *reinterpret_cast<uint32_t*>(hidden_out + r) = hn;
    if (gate_out) *reinterpret_cast<uint32_t*>(gate_out + r) = gw;
  }
  // block sum of squares of h: lane l holds partials 2l + b (k even) and 64 + 2l + b (k odd)
  float pt[2][2];
#pragma unroll
  for (int hi = 0; hi < 2; ++hi)
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) s = __fadd_rn(s, __fmul_rn(v[2 * (2 * j + hi) + b], v[2 * (2 * j + hi) + b]));
      pt[hi][b] = s;
    }
  // XOR offsets 16, 8, 4, 2 on the partial index are lane offsets 8, 4, 2, 1; offset 1 is b.
#pragma unroll
  for (int lm = 8; lm > 0; lm >>= 1)
#pragma unroll
    for (int hi = 0; hi < 2; ++hi)
#pragma unroll
      for (int b = 0; b < 2; ++b) pt[hi][b] = __fadd_rn(pt[hi][b], __shfl_xor_sync(0xffffffffu, pt[hi][b], lm));
  const float g_lo = __fadd_rn(pt[0][0], pt[0][1]), g_hi = __fadd_rn(pt[1][0], pt[1][1]);
  // groups 0, 1, 2, 3: (lanes 0..15, k even), (lanes 16..31, k even), (0..15, k odd), (16..31, k odd)
  const float G0 = __shfl_sync(0xffffffffu, g_lo, 0), G1 = __shfl_sync(0xffffffffu, g_lo, 16);
  const float G2 = __shfl_sync(0xffffffffu, g_hi, 0), G3 = __shfl_sync(0xffffffffu, g_hi, 16);
  const float block = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, G0), G1), G2), G3);
  // the next operator's quantiser on x * s_next
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t sw = sws[k];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const uint32_t flip = (sw << (24 - 8 * b)) & 0x80000000u;  // sign bit of byte b
      x[2 * k + b] = __uint_as_float(__float_as_uint(x[2 * k + b]) ^ flip);
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // stride 1
    const float lower = x[2 * k], upper = x[2 * k + 1];
    x[2 * k] = __fadd_rn(lower, upper);
    x[2 * k + 1] = __fsub_rn(lower, upper);
  }
#pragma unroll
  for (int mask = 1; mask < 32; mask <<= 1) {  // strides 2..32
    const float s = (lane & mask) ? -1.0f : 1.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) x[e] = cross_butterfly(x[e], __shfl_xor_sync(0xffffffffu, x[e], mask), s);
  }
#pragma unroll
  for (int kb = 1; kb < 8; kb <<= 1) {  // strides 64, 128, 256
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k & kb) continue;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const float lower = x[2 * k + b], upper = x[2 * (k + kb) + b];
        x[2 * k + b] = __fadd_rn(lower, upper);
        x[2 * (k + kb) + b] = __fsub_rn(lower, upper);
      }
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    x[e] = __half2float(__float2half_rn(__fmul_rn(x[e], kHadamardNorm)));
    bad |= !finite32(x[e]);
    mx = fmaxf(mx, fabsf(x[e]));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float scale = __fdiv_rn(mx, 127.0f);
  const float rcp = __frcp_rn(scale);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t w2 = 0;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      int q = scale > 0.0f ? quotient_rne(x[2 * k + b], scale, rcp) : 0;
      q = max(-127, min(127, q));
      w2 |= (uint32_t)(q & 0xff) << (8 * b);
    }
    *reinterpret_cast<uint16_t*>(act + 64 * k + 2 * lane) = (uint16_t)w2;
  }
  if (lane == 0) {
    *alpha = scale;
    *bss = block;
  }
}

// The block's residual-stream, norm-weight and next-sign words (residual_block512's
// inputs) for rows r0 + 64k + 2l + b.
__device__ __forceinline__ void load_residual_words512(const uint16_t* hidden, const uint16_t* __restrict__ norm_w,
                                                       const int8_t* __restrict__ s_next, int r0, int lane,
                                                       uint32_t (&hws)[8], uint32_t (&wws)[8], uint32_t (&sws)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + 64 * k + 2 * lane;
    hws[k] = __ldcg(reinterpret_cast<const unsigned int*>(hidden + r));
    wws[k] = __ldg(reinterpret_cast<const unsigned int*>(norm_w + r));
    sws[k] = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(s_next + r));
  }
}

// Restores token block r0 of the int64 sums wsr (restore_values512) and applies the
// residual epilogue to it. Every load the block needs is issued first, together: the sums,
// the row scales and output signs, and the residual-stream, norm-weight and next-sign words
// (the stores below go through some of the same pointers, so the compiler could not move
// the later loads ahead of them). The caller clears the sums afterwards.
__device__ __forceinline__ void residual_restore512(const int64_t* wsr, const float* __restrict__ tau,
                                                        const int8_t* __restrict__ s_out, float rq,
                                                        const float* inv_rms_m, const ResidualOut o, int r0, int lane,
                                                        bool& bad) {
  longlong2 ws[8];
  Rows512 rr;
  load_sums512(wsr, r0, lane, ws);
  load_rows512(tau, s_out, r0, lane, rr);
  uint32_t hws[8], wws[8], sws[8];
  load_residual_words512(o.hidden, o.norm_w, o.s_next, r0, lane, hws, wws, sws);
  float v[16];  // the block's outputs y; then the updated residual stream h
  restore_values512(ws, rr, rq, inv_rms_m, lane, bad, v);
  residual_block512(v, hws, wws, sws, o.hidden + r0, o.gate ? o.gate + r0 : nullptr, o.act + r0, o.alpha + r0 / 512,
                    o.bss + r0 / 512, lane, bad);
}

__device__ __forceinline__ void restore_block512(const int64_t* wsr, float rq, const float* inv_rms_m,
                                                 const float* __restrict__ tau, const int8_t* __restrict__ s_out,
                                                 int r0, int n_rows, float* __restrict__ yr, int lane, bool& bad) {
  float v[16];
  char2 sg[8];  // output signs, requested with the sums so their latency overlaps
  if (inv_rms_m) bad |= !finite32(*inv_rms_m);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + 64 * k + 2 * lane;
    const longlong2 w = __ldcg(reinterpret_cast<const longlong2*>(wsr + r));
    const float2 t = __ldg(reinterpret_cast<const float2*>(tau + r));
    sg[k] = __ldg(reinterpret_cast<const char2*>(s_out + r));
    v[2 * k] = restore_value(w.x, rq, inv_rms_m, t.x);
    v[2 * k + 1] = restore_value(w.y, rq, inv_rms_m, t.y);
    bad |= !finite32(v[2 * k]) | !finite32(v[2 * k + 1]);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // stride 1
    const float lower = v[2 * k], upper = v[2 * k + 1];
    v[2 * k] = __fadd_rn(lower, upper);
    v[2 * k + 1] = __fsub_rn(lower, upper);
  }
#pragma unroll
  for (int mask = 1; mask < 32; mask <<= 1) {  // strides 2..32
    const float s = (lane & mask) ? -1.0f : 1.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = cross_butterfly(v[e], __shfl_xor_sync(0xffffffffu, v[e], mask), s);
  }
#pragma unroll
  for (int kb = 1; kb < 8; kb <<= 1) {  // strides 64, 128, 256
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k & kb) continue;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const float lower = v[2 * k + b], upper = v[2 * (k + kb) + b];
        v[2 * k + b] = __fadd_rn(lower, upper);
        v[2 * (k + kb) + b] = __fsub_rn(lower, upper);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = r0 + 64 * k + 2 * lane;
    const float t0 = __fmul_rn(__fmul_rn(v[2 * k], kHadamardNorm), (float)sg[k].x);
    const float t1 = __fmul_rn(__fmul_rn(v[2 * k + 1], kHadamardNorm), (float)sg[k].y);
    bad |= !finite32(t0) | !finite32(t1);
    float* dst = yr + r;
    if (r + 1 < n_rows && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
      *reinterpret_cast<float2*>(dst) = make_float2(t0, t1);
    } else {
      if (r < n_rows) dst[0] = t0;
      if (r + 1 < n_rows) dst[1] = t1;
    }
  }
}

}  // namespace yskn
