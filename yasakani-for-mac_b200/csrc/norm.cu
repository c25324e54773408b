// The steps between two projections: residual addition with deferred RMS
// normalisation (what turns one projection's restored output into the next projection's
// input), and the MLP's gated product (gate and up into down's input).
//
// Reference: the residual + normalisation part of q35_res_norm_xsm_kernel
// (src/q35_kernels.cu:1437-1463) and q35_xsm_r (src/q35_kernels.cu:81-85); scalar spec
// docs/spec/05_RESIDUAL_NORM_MLP.md:53-141. Per token row (cols a multiple of 512):
//   hidden[i] = bf16(hidden[i] + bf16(projection[i]))         (skipped without a projection)
//   sum of squares of hidden, in the spec's reduction shape, per 512 columns, blocks in order
//   inverse_rms = rsqrt(total / cols + eps)                  (the portable rsqrt: rounded sqrt, rounded division)
//   input[i] = hidden[i] * (1 + norm_weight[i])               (binary32, the next operator's x)
//   gate[i] = bf16(input[i])                                   (optional copy)
// The next compressed operator quantises `input` and applies inverse_rms in its restore
// (yskn_b200_linear's inv_rms), so the normalised vector is never formed, as in the
// reference.
//
// B200 design: one 1024-thread CTA per row, eight 128-thread groups; group s takes the
// 512-column blocks s, s+8, ... and its thread t owns partial sum t of each (elements t,
// t+128, t+256, t+384), so the spec's reduction — four products added from +0, an XOR
// butterfly over each group of 32 partials — is a per-thread loop and one warp shuffle
// butterfly, all blocks of a row at once (a decode row is latency-bound); the group sums
// wait in shared memory and one thread adds them in the spec's order (four per block from
// +0, blocks in order). Every element is read and written once.
#include <cuda_bf16.h>

#include "common.cuh"
#include "pmath.cuh"
#include "quant.cuh"

namespace yskn {

constexpr int NORM_THREADS = 128;
constexpr int NORM_GROUPS = 8;  // 128-thread groups per CTA

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(NORM_THREADS * NORM_GROUPS) residual_prepare_kernel(
    uint16_t* hidden, const float* projection, const uint16_t* norm_weight, int cols, float eps, float* input,
    float* inv_rms, uint16_t* gate) {
  extern __shared__ float s_group[];  // [cols / 512][4] group sums
  pdl_begin();
  const int t = threadIdx.x & (NORM_THREADS - 1), lane = t & 31, warp = t >> 5, s = threadIdx.x / NORM_THREADS;
  const size_t row = blockIdx.x;
  uint16_t* h = hidden + row * cols;
  const float* pr = projection ? projection + row * cols : nullptr;
  for (int b = 512 * s; b < cols; b += 512 * NORM_GROUPS) {
    // Every load of the block first (the stores below may alias them as far as the
    // compiler knows, which would otherwise serialise one memory round trip per element).
    uint16_t hv[4], wv[4];
    float pv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = b + t + 128 * j;
      hv[j] = h[i];
      wv[j] = norm_weight[i];
      pv[j] = pr ? pr[i] : 0.0f;
    }
    float partial = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = b + t + 128 * j;
      float x = bf16_to_f32(hv[j]);
      if (pr) {
        x = bf16_to_f32(f32_to_bf16(__fadd_rn(x, bf16_to_f32(f32_to_bf16(pv[j])))));
        h[i] = f32_to_bf16(x);  // exact: x already has bf16 precision
      }
      partial = __fadd_rn(partial, __fmul_rn(x, x));
      const float in = __fmul_rn(x, __fadd_rn(1.0f, bf16_to_f32(wv[j])));
      input[row * cols + i] = in;
      if (gate) gate[row * cols + i] = f32_to_bf16(in);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) partial = __fadd_rn(partial, __shfl_xor_sync(0xffffffffu, partial, off));
    if (lane == 0) s_group[(b / 512) * 4 + warp] = partial;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int b = 0; b < cols / 512; ++b) {
      float block = 0.0f;
#pragma unroll
      for (int g = 0; g < NORM_THREADS / 32; ++g) block = __fadd_rn(block, s_group[4 * b + g]);
      total = __fadd_rn(total, block);
    }
    inv_rms[row] = pm_rsqrt(__fadd_rn(__fdiv_rn(total, (float)cols), eps));
  }
}

// MLP nonlinear step (src/q35_kernels.cu:1402-1421, 113-116; docs/spec/
// 05_RESIDUAL_NORM_MLP.md:156-176): with g = bf16(gate), u = bf16(up),
// out = bf16(bf16(silu(g)) * u), written as f32 so it is the down projection's x directly;
// silu(g) = g / (1 + exp(-g)) with the portable exp of the scalar contract
// (residual_norm_mlp.rs:137-156, portable_math.rs:201-203). Four elements per thread.
__global__ void __launch_bounds__(256) gated_product_kernel(const float* gate, const float* up, int64_t n, float* out) {
  pdl_begin();
  const int64_t i0 = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i0 >= n) return;
  const int k_end = n - i0 < 4 ? (int)(n - i0) : 4;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (k >= k_end) break;
    out[i0 + k] = gated_product_value(gate[i0 + k], up[i0 + k]);
  }
}

// The gated product of one 512-element group, quantised at once for the down projection
// (the f1 chain): the same values as gated_product_kernel, then the operator's quantiser
// (quantize_loaded512: signs, H512, half, alpha, int8) on them, so the down operator starts
// from int8 rows instead of quantising the f32 product in every CTA. One 128-thread CTA
// per (group, row): every thread forms four products (the SiLU is the costly part), then
// warp 0 quantises the group from shared memory (lane l: elements 16l..16l+15).
__global__ void __launch_bounds__(128) gated_product_q8_kernel(const float* gate, const float* up, int n,
                                                               const int8_t* signs, int8_t* act, float* alpha,
                                                               unsigned* err) {
  __shared__ __align__(16) float s_prod[512];
  pdl_begin();
  const int g = blockIdx.x, m = blockIdx.y;
  const size_t base = (size_t)m * n + (size_t)g * 512;
  {
    const float4 gv = *reinterpret_cast<const float4*>(gate + base + 4 * threadIdx.x);
    const float4 uv = *reinterpret_cast<const float4*>(up + base + 4 * threadIdx.x);
    const float gs[4] = {gv.x, gv.y, gv.z, gv.w}, us[4] = {uv.x, uv.y, uv.z, uv.w};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = gated_product_value(gs[e], us[e]);
    reinterpret_cast<float4*>(s_prod)[threadIdx.x] = make_float4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  Group512In in;
  in.s = __ldg(reinterpret_cast<const int4*>(signs + (size_t)g * 512 + 16 * lane));
#pragma unroll
  for (int q = 0; q < 4; ++q) in.x[q] = reinterpret_cast<const float4*>(s_prod)[4 * lane + q];
  bool bad = false;
  const float a = quantize_loaded512(in, act + base, lane, bad);
  if (lane == 0) alpha[(size_t)m * (n / 512) + g] = a;
  if (__any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(err, DERR_NONFINITE);
}

int launch_gated_product_q8(const float* gate, const float* up, int M, int n, const int8_t* signs, int8_t* act,
                            float* alpha, cudaStream_t st) {
  return cuda_fail(launch_pdl(gated_product_q8_kernel, dim3((unsigned)(n / 512), (unsigned)M), 128, 0, st, gate, up,
                              n, signs, act, alpha, device_error_word()),
                   "gated_product_q8_kernel");
}

// bf16 -> f32, exact (an operator's input from a bf16 producer such as the attention).
__global__ void __launch_bounds__(256) widen_bf16_kernel(const uint16_t* in, int64_t n, float* out) {
  pdl_begin();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = bf16_to_f32(in[i]);
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_widen_bf16(const uint16_t* d_in, int64_t n, float* d_out, void* stream) {
  if (!d_in || !d_out || n < 1 || n > (int64_t)INT32_MAX * 256) return fail(YSKN_EINVAL, "widen_bf16: bad argument");
  return cuda_fail(launch_pdl(widen_bf16_kernel, (unsigned)((n + 255) / 256), 256, 0,
                              reinterpret_cast<cudaStream_t>(stream), d_in, n, d_out),
                   "widen_bf16_kernel");
}

extern "C" YSKN_B200_API int yskn_b200_gated_product(const float* d_gate, const float* d_up, int M, int n,
                                                    float* d_out, void* stream) {
  if (!d_gate || !d_up || !d_out || M < 1 || n < 1) return fail(YSKN_EINVAL, "gated_product: bad argument");
  const int64_t total = (int64_t)M * n;
  const int64_t threads = (total + 3) / 4;
  return cuda_fail(launch_pdl(gated_product_kernel, (unsigned)((threads + 255) / 256), 256, 0,
                              reinterpret_cast<cudaStream_t>(stream), d_gate, d_up, total, d_out),
                   "gated_product_kernel");
}

extern "C" YSKN_B200_API int yskn_b200_gated_product_q8(const float* d_gate, const float* d_up, int M, int n,
                                                       const int8_t* d_signs, int8_t* d_act, float* d_alpha,
                                                       void* stream) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!d_gate || !d_up || !d_signs || !d_act || !d_alpha || M < 1 || M > 65535 || n < 512 || n % 512 ||
      !a16(d_gate) || !a16(d_up) || !a16(d_signs) || !a16(d_act))
    return fail(YSKN_EINVAL, "gated_product_q8: null or unaligned argument, M outside 1..65535, or n not a multiple of 512");
  return launch_gated_product_q8(d_gate, d_up, M, n, d_signs, d_act, d_alpha, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" YSKN_B200_API int yskn_b200_residual_prepare(uint16_t* d_hidden, const float* d_projection,
                                                       const uint16_t* d_norm_weight, int M, int cols, float eps,
                                                       float* d_input, float* d_inv_rms, uint16_t* d_gate,
                                                       void* stream) {
  if (!d_hidden || !d_norm_weight || !d_input || !d_inv_rms || M < 1 || cols <= 0 || cols % 512)
    return fail(YSKN_EINVAL, "residual_prepare: null argument, M < 1, or cols not a multiple of 512");
  if (cols > 512 * 3072) return fail(YSKN_EINVAL, "residual_prepare: cols above 1572864");
  const size_t smem = (size_t)(cols / 512) * 4 * sizeof(float);  // at most 48 KB
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < M; m0 += 65535) {
    const int n = M - m0 < 65535 ? M - m0 : 65535;
    const size_t off = (size_t)m0 * cols;
    if (cudaError_t e = launch_pdl(residual_prepare_kernel, n, NORM_THREADS * NORM_GROUPS, smem, st, d_hidden + off,
                                   d_projection ? d_projection + off : nullptr, d_norm_weight, cols, eps,
                                   d_input + off, d_inv_rms + m0, d_gate ? d_gate + off : nullptr))
      return cuda_fail(e, "residual_prepare_kernel");
  }
  return YSKN_OK;
}
