// Operator prologue and epilogue: the activation quantiser and the restore.
//
// Both are bit-exact restatements of the reference's scalar order
// (docs/spec/02_COMPRESSED_LINEAR.md:84-101,129-241; crates/yskn-ref/src/
// compressed_linear.rs:14-29,57-135,288-370). Every binary32 operation is an
// explicit round-to-nearest intrinsic, so no multiply-add contraction can occur
// (the reference build relies on --fmad=false, CMakeLists.txt:47-51).
//
// One warp transforms one 512-element block: lane l holds elements 16l..16l+15.
// The Hadamard butterflies run in ascending stride order as the spec requires:
// strides 1..8 inside a lane, 16..256 across lanes (shfl_xor with lane bit
// stride/16). Each element's value after every stage is the same binary32 value
// the scalar loop produces, so the parallel transform is bit-identical.
#include <cuda_fp16.h>

#include "common.cuh"

namespace yskn {

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
    const bool upper_half = (lane & mask) != 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, v[e], mask);
      v[e] = upper_half ? __fsub_rn(other, v[e]) : __fadd_rn(v[e], other);
    }
  }
}

__device__ __forceinline__ bool finite32(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

// grid: M blocks; block: nw warps; dynamic smem: G floats.
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ x, const int8_t* __restrict__ signs,
                                                       int Kc, int8_t* __restrict__ act, float* __restrict__ alpha,
                                                       int32_t* __restrict__ scales, float* __restrict__ row_quantum,
                                                       unsigned* __restrict__ err) {
  extern __shared__ float s_alpha[];
  const int m = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int G = Kc / 512;
  const float* xr = x + (int64_t)m * Kc;
  bool bad = false;
  for (int g = warp; g < G; g += nw) {
    const int base = g * 512 + lane * 16;
    float v[16];
    const float4* xp = reinterpret_cast<const float4*>(xr + base);
    const int4 sp = *reinterpret_cast<const int4*>(signs + base);
    const int8_t* sb = reinterpret_cast<const int8_t*>(&sp);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 f = __ldg(xp + q);
      v[4 * q + 0] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      bad |= !finite32(v[e]);
      v[e] = __fmul_rn(v[e], (float)sb[e]);
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
    uint32_t packed[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        int r = scale > 0.0f ? __float2int_rn(__fdiv_rn(v[4 * q + b], scale)) : 0;
        r = max(-127, min(127, r));
        w |= (uint32_t)(r & 0xff) << (8 * b);
      }
      packed[q] = w;
    }
    *reinterpret_cast<uint4*>(act + (int64_t)m * Kc + base) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    if (lane == 0) {
      s_alpha[g] = scale;
      alpha[(int64_t)m * G + g] = scale;
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(err, DERR_NONFINITE);
  __syncthreads();
  // Common 2^24 integer grid for the row (compressed_linear.rs:113-128).
  float mxs = 0.0f;
  for (int g = 0; g < G; ++g) mxs = fmaxf(mxs, s_alpha[g]);
  const float mult = mxs > 0.0f ? __fdiv_rn(16777216.0f, mxs) : 0.0f;
  for (int g = threadIdx.x; g < G; g += blockDim.x)
    scales[(int64_t)m * G + g] = __float2int_rn(__fmul_rn(s_alpha[g], mult));
  if (threadIdx.x == 0) row_quantum[m] = __fmul_rn(mxs, 5.9604644775390625e-08f /* 2^-24 */);
}

int launch_quantize(const float* x, const int8_t* signs, int M, int Kc, int8_t* act, float* alpha, int32_t* scales,
                    float* row_quantum, cudaStream_t st) {
  const int G = Kc / 512;
  const int nw = G < 8 ? G : 8;
  quantize_kernel<<<M, nw * 32, G * sizeof(float), st>>>(x, signs, Kc, act, alpha, scales, row_quantum,
                                                                device_error_word());
  return cuda_fail(cudaGetLastError(), "quantize_kernel");
}

// Restore with output rotation: one warp per (row m, 512-row block).
__global__ void __launch_bounds__(256) restore_rot_kernel(int64_t* __restrict__ ws, int ws_ld,
                                                          const float* __restrict__ row_quantum,
                                                          const float* __restrict__ inv_rms,
                                                          const float* __restrict__ tau,
                                                          const int8_t* __restrict__ s_out, int M, int blocks,
                                                          int n_rows, int clear_ws, float* __restrict__ y,
                                                          unsigned* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= (int64_t)M * blocks) return;
  const int m = (int)(item / blocks), b = (int)(item % blocks);
  const int r0 = b * 512 + lane * 16;
  const float rq = row_quantum[m];
  const float ir = inv_rms ? inv_rms[m] : 1.0f;
  bool bad = inv_rms ? !finite32(ir) : false;
  int64_t* wsr = ws + (int64_t)m * ws_ld + r0;
  float v[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    float t = __fmul_rn(__ll2float_rn(wsr[e]), rq);
    if (inv_rms) t = __fmul_rn(t, ir);
    t = __fmul_rn(t, __ldg(tau + r0 + e));
    bad |= !finite32(t);
    v[e] = t;
  }
  if (clear_ws) {
#pragma unroll
    for (int e = 0; e < 16; e += 2) *reinterpret_cast<longlong2*>(wsr + e) = make_longlong2(0, 0);
  }
  hadamard512_warp(v, lane);
  const int4 sp = *reinterpret_cast<const int4*>(s_out + r0);
  const int8_t* sb = reinterpret_cast<const int8_t*>(&sp);
  float* yr = y + (int64_t)m * n_rows;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float t = __fmul_rn(__fmul_rn(v[e], kHadamardNorm), (float)sb[e]);
    bad |= !finite32(t);
    if (r0 + e < n_rows) yr[r0 + e] = t;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(err, DERR_NONFINITE);
}

// Restore without output rotation (vocabulary head, draft): elementwise.
__global__ void __launch_bounds__(256) restore_plain_kernel(int64_t* __restrict__ ws, int ws_ld,
                                                            const float* __restrict__ row_quantum,
                                                            const float* __restrict__ inv_rms,
                                                            const float* __restrict__ tau, int M, int phys,
                                                            int n_rows, int clear_ws, float* __restrict__ y,
                                                            unsigned* __restrict__ err) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * phys) return;
  const int m = (int)(i / phys), r = (int)(i % phys);
  int64_t* p = ws + (int64_t)m * ws_ld + r;
  float t = __fmul_rn(__ll2float_rn(*p), row_quantum[m]);
  bool bad = false;
  if (inv_rms) {
    bad |= !finite32(inv_rms[m]);
    t = __fmul_rn(t, inv_rms[m]);
  }
  t = __fmul_rn(t, __ldg(tau + r));
  bad |= !finite32(t);
  if (clear_ws) *p = 0;
  if (r < n_rows) y[(int64_t)m * n_rows + r] = t;
  if (bad) raise_device_error(err, DERR_NONFINITE);
}

int launch_restore(int64_t* ws, int ws_ld, const float* row_quantum, const float* inv_rms, const float* tau,
                   const int8_t* s_out, int M, int phys, int n_rows, int clear_ws, float* y, cudaStream_t st) {
  if (s_out) {
    const int blocks = phys / 512;
    const int64_t items = (int64_t)M * blocks;
    restore_rot_kernel<<<(unsigned)ceil_div(items, 8), 256, 0, st>>>(ws, ws_ld, row_quantum, inv_rms, tau, s_out, M,
                                                                     blocks, n_rows, clear_ws, y, device_error_word());
    return cuda_fail(cudaGetLastError(), "restore_rot_kernel");
  }
  const int64_t total = (int64_t)M * phys;
  restore_plain_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(ws, ws_ld, row_quantum, inv_rms, tau, M, phys,
                                                                       n_rows, clear_ws, y, device_error_word());
  return cuda_fail(cudaGetLastError(), "restore_plain_kernel");
}

}  // namespace yskn
