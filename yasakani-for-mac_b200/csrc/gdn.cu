// Gated DeltaNet decode step: the dense gates, the four-tap convolution, the q/k
// normalisation and gates, the recurrent state update and the gated output norm — the
// layer between in_proj_qkv/in_proj_z and out_proj of a linear-attention layer.
//
// Reference: src/q35_kernels.cu:746-820 (dense gates), :864-980 (convolution, gates,
// recurrence, output); scalar spec docs/spec/03_GATED_DELTANET.md:33-160 (helpers :5-32).
// Ordinary causal rows (depth = row); the verification-row table is not covered. A call
// commits after n_commit rows (:160-186): the state is saved when row + 1 == n_commit and
// the history takes the newest committed rows; n_commit = 0 is the provisional
// verification pass that changes neither. The
// transcendental helpers are CUDA's expf, rsqrtf and log1pf, as in the reference
// (GDN-01 of the spec: their bits are not portable).
//
// B200 design:
//  * gates: one 128-thread CTA per (row, output); thread p forms partial p (40 products in
//    the spec's order), each warp is one xor_sum32 group (a shuffle butterfly: every lane
//    ends with the same bits), the four groups combine in sum4 order.
//  * step: one 128-thread CTA per value head, its 128x128 f32 state in shared memory for
//    all rows (the recurrence is sequential over rows); thread j owns state column j, so
//    the spec's 32-term sequential groups are per-thread loops and the column is read and
//    written once per launch (saved when the committed row is reached). q/k of the head's key head are recomputed by its three value
//    heads (128 channels each, cheap).
//  * history: the three newest projected rows are written after the step, in place (another
//    launch, since three CTAs read each key head's history).
#include <cuda_bf16.h>

#include "common.cuh"

namespace yskn {

constexpr int GDN_DK = 128;   // channels per head
constexpr int GDN_QK_HEADS = 16;
constexpr int GDN_V_HEADS = 48;
constexpr int GDN_QKV = 2 * GDN_QK_HEADS * GDN_DK + GDN_V_HEADS * GDN_DK;  // 10240

__device__ __forceinline__ float bf(float x) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x)) << 16);
}
__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float xor_sum32(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float sum4(const float* v) { return __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), v[2]), v[3]); }

// squares128 (03_GATED_DELTANET.md:24-27) of the value each of the 128 threads holds.
__device__ __forceinline__ float squares128(float x, float* s4) {
  const float g = xor_sum32(__fmul_rn(x, x));
  __syncthreads();  // s4 is free
  if ((threadIdx.x & 31) == 0) s4[threadIdx.x >> 5] = g;
  __syncthreads();
  return sum4(s4);
}

// 03_GATED_DELTANET.md:57-76: the 96 dense gates of each row (b, then a).
__global__ void __launch_bounds__(128) gdn_gates_kernel(const uint16_t* x, const float* inv_rms, const uint16_t* wb,
                                                        const uint16_t* wa, int hidden, float* gates) {
  __shared__ float s4[4];
  const int o = blockIdx.x, row = blockIdx.y, p = threadIdx.x;
  const uint16_t* w = o < GDN_V_HEADS ? wb + (size_t)o * hidden : wa + (size_t)(o - GDN_V_HEADS) * hidden;
  const uint16_t* xr = x + (size_t)row * hidden;
  float partial = 0.0f;
  for (int chunk = 0; chunk < hidden / 1024; ++chunk)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = 8 * p + 1024 * chunk + e;
      partial = __fadd_rn(partial, __fmul_rn(bf16f(w[i]), bf16f(xr[i])));
    }
  const float g = xor_sum32(partial);
  if ((p & 31) == 0) s4[p >> 5] = g;
  __syncthreads();
  if (p == 0) gates[(size_t)row * 2 * GDN_V_HEADS + o] = bf(__fmul_rn(sum4(s4), inv_rms[row]));
}

struct GdnParams {
  const float* qkv;       // [M][10240] restored in_proj_qkv
  const float* z;         // [M][6144] restored in_proj_z
  const float* gates;     // [M][96]
  const uint16_t* conv_w; // bf16 [10240][4], oldest coefficient first
  const uint16_t* a_log;  // bf16 [48]
  const uint16_t* dt_bias;
  const uint16_t* norm_w; // bf16 [128]
  float eps;
  int M, n_commit;
  float* state;              // [48][128][128]
  const uint16_t* history;   // bf16 [3][10240], oldest first
  float* out;                // [M][6144]: the gated output (bf16 values), out_proj's x
};

// The convolved (bf16(silu(bf16(conv))) channel c of row `row` (03_GATED_DELTANET.md:86-100).
__device__ __forceinline__ float gdn_conv(const GdnParams& p, int row, int c) {
  auto past = [&](int r) { return r < 0 ? bf16f(p.history[(size_t)(3 + r) * GDN_QKV + c]) : bf(p.qkv[(size_t)r * GDN_QKV + c]); };
  const uint16_t* w = p.conv_w + (size_t)c * 4;
  float a = __fmul_rn(bf16f(w[0]), past(row - 3));
  a = __fadd_rn(a, __fmul_rn(bf16f(w[1]), past(row - 2)));
  a = __fadd_rn(a, __fmul_rn(bf16f(w[2]), past(row - 1)));
  a = __fadd_rn(a, __fmul_rn(bf16f(w[3]), past(row)));
  return bf(silu(bf(a)));
}

__global__ void __launch_bounds__(128) gdn_step_kernel(const __grid_constant__ GdnParams p) {
  extern __shared__ __align__(16) float R[];  // [128][128] this head's state
  __shared__ float s_q[GDN_DK], s_k[GDN_DK], s4[4];
  const int vh = blockIdx.x, kh = vh / 3, j = threadIdx.x;
  float* state = p.state + (size_t)vh * GDN_DK * GDN_DK;
  for (int i = 0; i < GDN_DK; ++i) R[i * GDN_DK + j] = state[i * GDN_DK + j];
  const float a_log = bf16f(p.a_log[vh]), dt_bias = bf16f(p.dt_bias[vh]);
  for (int row = 0; row < p.M; ++row) {
    // 03_GATED_DELTANET.md:102-116: q/k of the key head, the value, beta and the decay.
    const float q = gdn_conv(p, row, GDN_DK * kh + j);
    const float k = gdn_conv(p, row, GDN_QK_HEADS * GDN_DK + GDN_DK * kh + j);
    const float v = gdn_conv(p, row, 2 * GDN_QK_HEADS * GDN_DK + GDN_DK * vh + j);
    const float rq = rsqrtf(__fadd_rn(squares128(q, s4), 1e-6f));
    const float rk = rsqrtf(__fadd_rn(squares128(k, s4), 1e-6f));
    __syncthreads();  // the previous row's readers of s_q / s_k are done
    s_q[j] = __fmul_rn(__fmul_rn(q, rq), 0.08838834764831845f);
    s_k[j] = __fmul_rn(k, rk);
    __syncthreads();
    const float* g = p.gates + (size_t)row * 2 * GDN_V_HEADS;
    const float beta = bf(sigmoid(g[vh]));
    const float log_decay = __fmul_rn(-expf(a_log), softplus(__fadd_rn(g[GDN_V_HEADS + vh], dt_bias)));
    const float decay = expf(log_decay);
    // 03_GATED_DELTANET.md:123-143: column j of the state.
    float part[4];
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      float acc = 0.0f;
      for (int r = 0; r < 32; ++r) {
        const int i = 32 * grp + r;
        const float x = __fmul_rn(R[i * GDN_DK + j], decay);
        R[i * GDN_DK + j] = x;
        acc = __fadd_rn(acc, __fmul_rn(x, s_k[i]));
      }
      part[grp] = acc;
    }
    const float correction = __fmul_rn(__fsub_rn(v, sum4(part)), beta);
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      float acc = 0.0f;
      for (int r = 0; r < 32; ++r) {
        const int i = 32 * grp + r;
        const float x = __fadd_rn(R[i * GDN_DK + j], __fmul_rn(s_k[i], correction));
        R[i * GDN_DK + j] = x;
        acc = __fadd_rn(acc, __fmul_rn(x, s_q[i]));
      }
      part[grp] = acc;
    }
    const float core = bf(sum4(part));
    // 03_GATED_DELTANET.md:145-155: the output norm (weight used directly) and the z gate.
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(squares128(core, s4), 128.0f), p.eps));
    const float normalized = bf(__fmul_rn(bf16f(p.norm_w[j]), bf(__fmul_rn(core, inv))));
    const float zz = p.z[(size_t)row * GDN_V_HEADS * GDN_DK + GDN_DK * vh + j];
    p.out[(size_t)row * GDN_V_HEADS * GDN_DK + GDN_DK * vh + j] = bf(__fmul_rn(normalized, silu(zz)));
    if (row + 1 == p.n_commit)
      for (int i = 0; i < GDN_DK; ++i) state[i * GDN_DK + j] = R[i * GDN_DK + j];
  }
}

// The three newest committed rows (bf16, M = n_commit here) become the history, in place
// after the step: row a takes old row M + a when fewer than 3 - a new rows exist, a later
// row than a, so
// each thread (one channel) reads every old value before it writes over it.
__global__ void gdn_history_kernel(const float* qkv, int M, uint16_t* history) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= GDN_QKV) return;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const int r = M - 3 + a;
    history[(size_t)a * GDN_QKV + c] = r < 0 ? history[(size_t)(3 + r) * GDN_QKV + c]
                                             : __bfloat16_as_ushort(__float2bfloat16_rn(qkv[(size_t)r * GDN_QKV + c]));
  }
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_gdn_gates(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb,
                                                const uint16_t* d_wa, int M, int hidden, float* d_gates, void* stream) {
  if (!d_hidden || !d_inv_rms || !d_wb || !d_wa || !d_gates || M < 1 || hidden <= 0 || hidden % 1024)
    return fail(YSKN_EINVAL, "gdn_gates: null argument, M < 1 or hidden not a multiple of 1024");
  if (M > 65535) return fail(YSKN_EINVAL, "gdn_gates: at most 65535 rows per call");
  gdn_gates_kernel<<<dim3(2 * GDN_V_HEADS, M), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      d_hidden, d_inv_rms, d_wb, d_wa, hidden, d_gates);
  return cuda_fail(cudaGetLastError(), "gdn_gates_kernel");
}

extern "C" YSKN_B200_API int yskn_b200_gdn_step(const float* d_qkv, const float* d_z, const float* d_gates,
                                               const uint16_t* d_conv_w, const uint16_t* d_a_log,
                                               const uint16_t* d_dt_bias, const uint16_t* d_norm_w, float eps, int M,
                                               int n_commit, float* d_state, uint16_t* d_history, float* d_out, void* stream) {
  if (!d_qkv || !d_z || !d_gates || !d_conv_w || !d_a_log || !d_dt_bias || !d_norm_w || !d_state || !d_history ||
      !d_out || M < 1 || n_commit < 0 || n_commit > M)
    return fail(YSKN_EINVAL, "gdn_step: null argument, M < 1 or n_commit outside 0..M");
  static bool attr_set[64] = {};
  constexpr int smem = GDN_DK * GDN_DK * sizeof(float);
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return cuda_fail(e, "gdn_step: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(YSKN_EINVAL, "gdn_step: device index out of range");
  if (!attr_set[dev]) {
    if (cudaError_t e = cudaFuncSetAttribute(gdn_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))
      return cuda_fail(e, "gdn_step_kernel attributes");
    attr_set[dev] = true;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  GdnParams p{d_qkv, d_z, d_gates, d_conv_w, d_a_log, d_dt_bias, d_norm_w, eps, M, n_commit, d_state, d_history, d_out};
  gdn_step_kernel<<<GDN_V_HEADS, 128, smem, st>>>(p);
  if (cudaError_t e = cudaGetLastError()) return cuda_fail(e, "gdn_step_kernel");
  if (n_commit == 0) return YSKN_OK;
  // After the step (the same stream): every head has read the old history.
  gdn_history_kernel<<<(GDN_QKV + 255) / 256, 256, 0, st>>>(d_qkv, n_commit, d_history);
  return cuda_fail(cudaGetLastError(), "gdn_history_kernel");
}
