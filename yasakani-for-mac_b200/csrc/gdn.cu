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
// transcendental helpers are the scalar contract's portable exp, rsqrt, sigmoid, softplus
// and silu (gated_deltanet.rs:332-577, portable_math.rs; pmath.cuh), so the outputs and
// the state equal yskn-ref's bits.
//
// B200 design:
//  * gates: one 128-thread CTA per (output, 8 rows); thread p forms partial p (40 products in
//    the spec's order, eight bf16 pairs per 16-byte load of weights and input), each warp is
//    one xor_sum32 group (a shuffle butterfly: every lane ends with the same bits), the four
//    groups combine in sum4 order.
//  * step: one 512-thread CTA per value head, its 128x128 f32 state in registers for all
//    rows (the recurrence is sequential over rows); thread (g, j) holds rows 32g..32g+31 of
//    state column j, so each of the spec's 32-term sequential groups is one thread's loop
//    over its registers and the four group sums meet in shared memory for sum4. The state
//    is read once per launch (32 coalesced loads per thread, in flight while the first
//    row's convolution and gates are formed) and written once (when the committed row is
//    reached); each row's raw inputs are loaded during the previous row's recurrence. Thread groups 0, 1 and 2 convolve the query, key and value channel j
//    (q/k of the key head are recomputed by its three value heads: 128 channels each).
//  * history: the three newest projected rows are written after the step, in place (another
//    launch, since three CTAs read each key head's history).
//  * the whole mixer in one launch (yskn_b200_gdn_mixer[_heads]): the step CTA of value head h
//    also forms its two dense gates (thread groups 0 and 1 in the gates kernel's order, every
//    row's before the first) and, once every row is done, writes its value channels' history;
//    the query/key history of a key head is written by the last of the key head's value-head
//    CTAs to finish (an arrival counter per key head), after every reader has used its taps;
//    CTA 0 writes that of the run's key heads that none of its value heads reads.
//  * tensor parallelism: a rank runs a run of value heads with the key heads they read
//    (the *_heads entry points); every head's arithmetic is the whole layer's, so the runs
//    of all ranks together give the whole layer's bits.
#include <cuda_bf16.h>

#include "common.cuh"
#include "pmath.cuh"

namespace yskn {

constexpr int GDN_DK = 128;   // channels per head
constexpr int GDN_QK_HEADS = 16;
constexpr int GDN_V_HEADS = 48;
constexpr int GDN_GATE_ROWS = 8;  // rows per gates CTA
constexpr int GDN_MIXER_MAX_M = 64;  // rows per call of the one-launch mixer (gates in shared memory)

// Arrivals of the one-launch mixer's value-head CTAs per key head (zero between launches;
// the last arriver resets its counter): one such launch in flight per device.
__device__ unsigned g_gdn_arrivals[GDN_QK_HEADS];

__device__ __forceinline__ float bf(float x) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x)) << 16);
}
__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ float xor_sum32(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float sum4(const float* v) { return __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), v[2]), v[3]); }

__device__ __forceinline__ float sum4(float a, float b, float c, float d) {
  return __fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d);
}

// Adds the eight products of a 16-byte group of bf16 weights and inputs to `acc`, element 0
// (the low half of the first word) first.
__device__ __forceinline__ float dot8(float acc, uint4 w, uint4 x) {
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w}, xx[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(ww[k] << 16), __uint_as_float(xx[k] << 16)));
    acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(ww[k] & 0xffff0000u), __uint_as_float(xx[k] & 0xffff0000u)));
  }
  return acc;
}

// 03_GATED_DELTANET.md:57-76: the 96 dense gates of each row (b, then a).
__global__ void __launch_bounds__(128) gdn_gates_kernel(const uint16_t* x, const float* inv_rms, const uint16_t* wb,
                                                        const uint16_t* wa, int n_heads, int hidden, int M,
                                                        float* gates) {
  __shared__ float s4[2][4];
  pdl_begin();
  const int o = blockIdx.x, p = threadIdx.x;
  const uint16_t* w = o < n_heads ? wb + (size_t)o * hidden : wa + (size_t)(o - n_heads) * hidden;
  const int row0 = blockIdx.y * GDN_GATE_ROWS;
  const int rows = M - row0 < GDN_GATE_ROWS ? M - row0 : GDN_GATE_ROWS;
  const int chunks = hidden / 1024;
  for (int rr = 0; rr < rows; ++rr) {
    const int row = row0 + rr;
    const uint16_t* xr = x + (size_t)row * hidden;
    float partial = 0.0f;
#pragma unroll 5
    for (int chunk = 0; chunk < chunks; ++chunk) {
      const int i = 1024 * chunk + 8 * p;
      partial = dot8(partial, __ldg(reinterpret_cast<const uint4*>(w + i)), __ldg(reinterpret_cast<const uint4*>(xr + i)));
    }
    const float g = xor_sum32(partial);
    if ((p & 31) == 0) s4[rr & 1][p >> 5] = g;
    __syncthreads();  // (the other buffer is written only after every thread passed the next barrier)
    if (p == 0) gates[(size_t)row * 2 * n_heads + o] = bf(__fmul_rn(sum4(s4[rr & 1]), inv_rms[row]));
  }
}

// A run of value heads: n_v heads from global head v0, with the query and key channels of
// global key heads qk0 .. qk0 + qk_ch / 128 - 1 (value head h reads key head h / 3). A
// row of the projected input is [query channels | key channels | value channels], W wide
// (the whole layer: v0 = qk0 = 0, n_v = 48, qk_ch = 2048, W = 10240).
struct GdnParams {
  const float* qkv;       // [M][W] restored in_proj_qkv rows of the run
  const float* z;         // [M][128 n_v] restored in_proj_z rows of the run
  const float* gates;     // [M][2 n_v]: b, then a
  const uint16_t* conv_w; // bf16 [W][4], oldest coefficient first
  const uint16_t* a_log;  // bf16 [n_v]
  const uint16_t* dt_bias;
  const uint16_t* norm_w; // bf16 [128]
  float eps;
  int M, n_commit;
  float* state;              // [n_v][128][128]
  uint16_t* history;         // bf16 [3][W], oldest first (written by the one-launch mixer)
  float* out;                // [M][128 n_v]: the gated output (bf16 values), out_proj's x
  int n_v, v0, qk0, qk_ch, W;
  // One-launch mixer only: the dense gates' input rows and weights (rows of the run's heads).
  const uint16_t* x;         // bf16 [M][hidden]
  const float* inv_rms;      // [M]
  const uint16_t* wb;        // bf16 [n_v][hidden]
  const uint16_t* wa;
  int hidden;
};

constexpr int GDN_STEP_THREADS = 4 * GDN_DK;  // four threads per state column, one per 32-row group

// One row's raw inputs of one thread, loaded a row ahead of their use: the four
// convolution taps (oldest first) of channel c (none when c < 0), z of column j (group 0)
// and the head's two gates.
struct GdnRowIn {
  float x[4];
  float z, gb, ga;
};

// The gates come from gsrc: [row][gstride], b at gb_off and a at gb_off + ga_step.
__device__ __forceinline__ void gdn_load_row(const GdnParams& p, int row, int c, int vh, int j, const float* gsrc,
                                             int gstride, int gb_off, int ga_step, GdnRowIn& in) {
  if (c >= 0) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = row - 3 + t;  // 03_GATED_DELTANET.md:86-100, depth = row
      in.x[t] = r < 0 ? bf16f(p.history[(size_t)(3 + r) * p.W + c]) : bf(p.qkv[(size_t)r * p.W + c]);
    }
  }
  if (c >= 0 && c < p.qk_ch) in.z = p.z[(size_t)row * p.n_v * GDN_DK + GDN_DK * vh + j];
  in.gb = gsrc[(size_t)row * gstride + gb_off];
  in.ga = gsrc[(size_t)row * gstride + gb_off + ga_step];
}

// The history of channel c after a call that commits n_commit rows: row a takes the newest
// committed row n_commit - 3 + a, or old row n_commit + a when fewer than 3 - a new rows
// exist (a later row than a, read before anything overwrites it).
__device__ __forceinline__ void gdn_history_channel(const float* qkv, int n_commit, int W, int c, uint16_t* history) {
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const int r = n_commit - 3 + a;
    history[(size_t)a * W + c] = r < 0 ? history[(size_t)(3 + r) * W + c]
                                       : __bfloat16_as_ushort(__float2bfloat16_rn(qkv[(size_t)r * W + c]));
  }
}

// bf(silu(bf(conv))) of one channel from its taps and weights.
__device__ __forceinline__ float gdn_conv(const float (&x)[4], const float (&w)[4]) {
  float a = __fmul_rn(w[0], x[0]);
  a = __fadd_rn(a, __fmul_rn(w[1], x[1]));
  a = __fadd_rn(a, __fmul_rn(w[2], x[2]));
  a = __fadd_rn(a, __fmul_rn(w[3], x[3]));
  return bf(pm_silu(bf(a)));
}

template <bool MIXER>
__global__ void __launch_bounds__(GDN_STEP_THREADS) gdn_step_kernel(const __grid_constant__ GdnParams p) {
  __shared__ float s_gate[MIXER ? GDN_MIXER_MAX_M : 1][2];  // mixer: every row's b, a
  __shared__ float s_g4[2][4];
  __shared__ bool s_last;
  __shared__ __align__(16) float s_q[GDN_DK];
  __shared__ __align__(16) float s_k[GDN_DK];
  __shared__ float s_v[GDN_DK];
  __shared__ float s_part[2][4][GDN_DK];  // the four group sums of the two inner products
  __shared__ float s_sq[2][4], s_so[4];   // per-warp squares: query, key; core
  pdl_begin();
  const int t = threadIdx.x, j = t & (GDN_DK - 1), grp = t >> 7, warp = t >> 5, lane = t & 31;
  const int vh = blockIdx.x, kh = (p.v0 + vh) / 3 - p.qk0, i0 = 32 * grp;  // local value and key head
  float* state = p.state + (size_t)vh * GDN_DK * GDN_DK + (size_t)i0 * GDN_DK + j;  // element (i0, j)
  float R[32];  // state rows i0..i0+31 of column j
#pragma unroll
  for (int r = 0; r < 32; ++r) R[r] = state[r * GDN_DK];
  // group 0: query channel j of the key head; 1: key channel; 2: value channel; 3: none
  const int c = grp == 0   ? GDN_DK * kh + j
                : grp == 1 ? p.qk_ch + GDN_DK * kh + j
                : grp == 2 ? 2 * p.qk_ch + GDN_DK * vh + j
                           : -1;
  float cw[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (c >= 0) {
    const uint2 w4 = __ldg(reinterpret_cast<const uint2*>(p.conv_w + (size_t)c * 4));
    cw[0] = __uint_as_float(w4.x << 16), cw[1] = __uint_as_float(w4.x & 0xffff0000u);
    cw[2] = __uint_as_float(w4.y << 16), cw[3] = __uint_as_float(w4.y & 0xffff0000u);
  }
  const float a_log = bf16f(p.a_log[vh]), dt_bias = bf16f(p.dt_bias[vh]);
  if constexpr (MIXER) {
    // 03_GATED_DELTANET.md:57-76: this head's dense gates of every row, in gdn_gates_kernel's
    // order: group 0 forms b, group 1 a; thread j adds its 40 products (5120 columns), each
    // warp is one xor_sum32 group, the four groups meet in sum4 order.
    const uint16_t* w = (grp == 0 ? p.wb : p.wa) + (size_t)vh * p.hidden;
    const int chunks = p.hidden / 1024;
    for (int row = 0; row < p.M; ++row) {
      if (grp < 2) {
        const uint16_t* xr = p.x + (size_t)row * p.hidden;
        float partial = 0.0f;
#pragma unroll 5
        for (int chunk = 0; chunk < chunks; ++chunk) {
          const int i = 1024 * chunk + 8 * j;
          partial =
              dot8(partial, __ldg(reinterpret_cast<const uint4*>(w + i)), __ldg(reinterpret_cast<const uint4*>(xr + i)));
        }
        const float g = xor_sum32(partial);
        if (lane == 0) s_g4[grp][warp & 3] = g;
      }
      __syncthreads();
      if (j == 0 && grp < 2) s_gate[row][grp] = bf(__fmul_rn(sum4(s_g4[grp]), p.inv_rms[row]));
      __syncthreads();
    }
  }
  const float* gsrc = MIXER ? &s_gate[0][0] : p.gates;
  const int gstride = MIXER ? 2 : 2 * p.n_v, gb_off = MIXER ? 0 : vh, ga_step = MIXER ? 1 : p.n_v;
  GdnRowIn cur;
  gdn_load_row(p, 0, c, vh, j, gsrc, gstride, gb_off, ga_step, cur);
  for (int row = 0; row < p.M; ++row) {
    GdnRowIn nxt;
    if (row + 1 < p.M) gdn_load_row(p, row + 1, c, vh, j, gsrc, gstride, gb_off, ga_step, nxt);
    // 03_GATED_DELTANET.md:102-116: the convolved channel; squares of query and key per warp.
    const float y = c >= 0 ? gdn_conv(cur.x, cw) : 0.0f;
    if (grp < 2) {
      const float g = xor_sum32(__fmul_rn(y, y));
      if (lane == 0) s_sq[grp][warp & 3] = g;
    } else if (grp == 2) {
      s_v[j] = y;
    }
    __syncthreads();
    if (grp == 0)
      s_q[j] = __fmul_rn(__fmul_rn(y, pm_rsqrt(__fadd_rn(sum4(s_sq[0]), 1e-6f))), 0.08838834764831845f);
    else if (grp == 1)
      s_k[j] = __fmul_rn(y, pm_rsqrt(__fadd_rn(sum4(s_sq[1]), 1e-6f)));
    const float beta = bf(pm_sigmoid(cur.gb));
    const float log_decay = __fmul_rn(-pm_exp(a_log), pm_softplus(__fadd_rn(cur.ga, dt_bias)));
    const float decay = pm_exp(log_decay);
    __syncthreads();
    // 03_GATED_DELTANET.md:123-143: rows i0..i0+31 of column j.
    const float4* k4 = reinterpret_cast<const float4*>(s_k + i0);
    const float4* q4 = reinterpret_cast<const float4*>(s_q + i0);
    float acc = 0.0f;
#pragma unroll
    for (int r4 = 0; r4 < 8; ++r4) {
      const float4 kk = k4[r4];
      const float kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        R[4 * r4 + e] = __fmul_rn(R[4 * r4 + e], decay);
        acc = __fadd_rn(acc, __fmul_rn(R[4 * r4 + e], kv[e]));
      }
    }
    s_part[0][grp][j] = acc;
    __syncthreads();
    const float correction =
        __fmul_rn(__fsub_rn(s_v[j], sum4(s_part[0][0][j], s_part[0][1][j], s_part[0][2][j], s_part[0][3][j])), beta);
    acc = 0.0f;
#pragma unroll
    for (int r4 = 0; r4 < 8; ++r4) {
      const float4 kk = k4[r4], qq = q4[r4];
      const float kv[4] = {kk.x, kk.y, kk.z, kk.w}, qv[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        R[4 * r4 + e] = __fadd_rn(R[4 * r4 + e], __fmul_rn(kv[e], correction));
        acc = __fadd_rn(acc, __fmul_rn(R[4 * r4 + e], qv[e]));
      }
    }
    s_part[1][grp][j] = acc;
    __syncthreads();
    // 03_GATED_DELTANET.md:145-155: the output norm (weight used directly) and the z gate.
    float core = 0.0f;
    if (grp == 0) {
      core = bf(sum4(s_part[1][0][j], s_part[1][1][j], s_part[1][2][j], s_part[1][3][j]));
      const float g = xor_sum32(__fmul_rn(core, core));
      if (lane == 0) s_so[warp] = g;
    }
    __syncthreads();
    if (grp == 0) {
      const float inv = pm_rsqrt(__fadd_rn(__fdiv_rn(sum4(s_so), 128.0f), p.eps));
      const float normalized = bf(__fmul_rn(bf16f(p.norm_w[j]), bf(__fmul_rn(core, inv))));
      p.out[(size_t)row * p.n_v * GDN_DK + GDN_DK * vh + j] = bf(__fmul_rn(normalized, pm_silu(cur.z)));
    }
    if (row + 1 == p.n_commit)
#pragma unroll
      for (int r = 0; r < 32; ++r) state[r * GDN_DK] = R[r];
    cur = nxt;
  }
  if constexpr (MIXER) {
    if (p.n_commit > 0) {
      // Every tap of every row has been used. This head alone reads its value channels;
      // the query/key channels of its key head are read by up to three heads, so the last
      // of them to get here writes those.
      if (grp == 2) gdn_history_channel(p.qkv, p.n_commit, p.W, c, p.history);
      __syncthreads();
      const int kg = p.v0 + vh;  // global value head; its key head kg / 3
      if (t == 0) {
        const int k3 = kg / 3 * 3;
        const unsigned readers = (unsigned)(min(p.v0 + p.n_v, k3 + 3) - max(p.v0, k3));
        __threadfence();
        s_last = atomicAdd(&g_gdn_arrivals[kg / 3], 1u) == readers - 1u;
      }
      __syncthreads();
      if (s_last) {
        if (grp < 2) gdn_history_channel(p.qkv, p.n_commit, p.W, c, p.history);
        if (t == 0) g_gdn_arrivals[kg / 3] = 0u;
      }
      // Key heads of the run that no value head of the run reads (a run's query/key
      // channels come in whole 512-column blocks): nobody reads them here, CTA 0 writes them.
      if (vh == 0 && grp < 2)
        for (int kl = 0; kl < p.qk_ch / GDN_DK; ++kl) {
          const int k3 = 3 * (p.qk0 + kl);
          if (k3 + 2 < p.v0 || k3 >= p.v0 + p.n_v)
            gdn_history_channel(p.qkv, p.n_commit, p.W, grp * p.qk_ch + GDN_DK * kl + j, p.history);
        }
    }
  }
}

// The three newest committed rows (bf16, M = n_commit here) become the history, in place
// after the step; each thread (one channel) reads every old value before it writes over it.
__global__ void gdn_history_kernel(const float* qkv, int M, int W, uint16_t* history) {
  pdl_begin();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= W) return;
  gdn_history_channel(qkv, M, W, c, history);
}

}  // namespace yskn

using namespace yskn;

static int gdn_gates(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb, const uint16_t* d_wa,
                     int n_heads, int M, int hidden, float* d_gates, void* stream) {
  if (!d_hidden || !d_inv_rms || !d_wb || !d_wa || !d_gates || M < 1 || hidden <= 0 || hidden % 1024 || n_heads < 1 ||
      n_heads > GDN_V_HEADS)
    return fail(YSKN_EINVAL, "gdn_gates: null argument, M < 1, hidden not a multiple of 1024 or heads outside 1..48");
  if (((uintptr_t)d_hidden | (uintptr_t)d_wb | (uintptr_t)d_wa) & 15)
    return fail(YSKN_EINVAL, "gdn_gates: hidden rows and weights must be 16-byte aligned");
  const int groups = (M + GDN_GATE_ROWS - 1) / GDN_GATE_ROWS;
  if (groups > 65535) return fail(YSKN_EINVAL, "gdn_gates: too many rows per call");
  return cuda_fail(launch_pdl(gdn_gates_kernel, dim3(2 * n_heads, groups), 128, 0, reinterpret_cast<cudaStream_t>(stream),
                              d_hidden, d_inv_rms, d_wb, d_wa, n_heads, hidden, M, d_gates),
                   "gdn_gates_kernel");
}

// The one-launch mixer's dense-gate inputs (gdn_step with them: gates and history in the launch).
struct MixerIn {
  const uint16_t* x;
  const float* inv_rms;
  const uint16_t* wb;
  const uint16_t* wa;
  int hidden;
};

static int gdn_step(const float* d_qkv, const float* d_z, const float* d_gates, const uint16_t* d_conv_w,
                    const uint16_t* d_a_log, const uint16_t* d_dt_bias, const uint16_t* d_norm_w, float eps, int M,
                    int n_commit, int n_v, int v0, int qk0, int qk_ch, float* d_state, uint16_t* d_history,
                    float* d_out, void* stream, const MixerIn* mixer = nullptr) {
  if (!d_qkv || !d_z || !(d_gates || mixer) || !d_conv_w || !d_a_log || !d_dt_bias || !d_norm_w || !d_state ||
      !d_history || !d_out || M < 1 || n_commit < 0 || n_commit > M)
    return fail(YSKN_EINVAL, "gdn_step: null argument, M < 1 or n_commit outside 0..M");
  if (mixer && (!mixer->x || !mixer->inv_rms || !mixer->wb || !mixer->wa || mixer->hidden <= 0 ||
                mixer->hidden % 1024 || M > GDN_MIXER_MAX_M ||
                (((uintptr_t)mixer->x | (uintptr_t)mixer->wb | (uintptr_t)mixer->wa) & 15)))
    return fail(YSKN_EINVAL, "gdn_mixer: null or unaligned gate input, hidden not a multiple of 1024, or M above 64");
  if (n_v < 1 || v0 < 0 || v0 + n_v > GDN_V_HEADS || qk0 < 0 || qk_ch < GDN_DK || qk_ch % GDN_DK ||
      qk0 * GDN_DK + qk_ch > GDN_QK_HEADS * GDN_DK || v0 / 3 < qk0 || (v0 + n_v - 1) / 3 >= qk0 + qk_ch / GDN_DK)
    return fail(YSKN_EINVAL, "gdn_step: the value heads need their key heads among the given query/key channels");
  if ((uintptr_t)d_conv_w & 7) return fail(YSKN_EINVAL, "gdn_step: convolution weights must be 8-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int W = 2 * qk_ch + GDN_DK * n_v;
  GdnParams p{d_qkv, d_z, d_gates, d_conv_w, d_a_log, d_dt_bias, d_norm_w, eps, M, n_commit, d_state, d_history,
              d_out, n_v, v0, qk0, qk_ch, W};
  if (mixer) {  // the gates and the history in the step's launch
    p.gates = nullptr;
    p.x = mixer->x;
    p.inv_rms = mixer->inv_rms;
    p.wb = mixer->wb;
    p.wa = mixer->wa;
    p.hidden = mixer->hidden;
    return cuda_fail(launch_pdl(gdn_step_kernel<true>, n_v, GDN_STEP_THREADS, 0, st, p), "gdn_step_kernel");
  }
  if (cudaError_t e = launch_pdl(gdn_step_kernel<false>, n_v, GDN_STEP_THREADS, 0, st, p))
    return cuda_fail(e, "gdn_step_kernel");
  if (n_commit == 0) return YSKN_OK;
  // After the step (the same stream): every head has read the old history.
  return cuda_fail(launch_pdl(gdn_history_kernel, (W + 255) / 256, 256, 0, st, d_qkv, n_commit, W, d_history),
                   "gdn_history_kernel");
}


extern "C" YSKN_B200_API int yskn_b200_gdn_gates(const uint16_t* d_hidden, const float* d_inv_rms, const uint16_t* d_wb,
                                                const uint16_t* d_wa, int M, int hidden, float* d_gates, void* stream) {
  return gdn_gates(d_hidden, d_inv_rms, d_wb, d_wa, GDN_V_HEADS, M, hidden, d_gates, stream);
}

extern "C" YSKN_B200_API int yskn_b200_gdn_gates_heads(const uint16_t* d_hidden, const float* d_inv_rms,
                                                      const uint16_t* d_wb, const uint16_t* d_wa, int n_heads, int M,
                                                      int hidden, float* d_gates, void* stream) {
  return gdn_gates(d_hidden, d_inv_rms, d_wb, d_wa, n_heads, M, hidden, d_gates, stream);
}

extern "C" YSKN_B200_API int yskn_b200_gdn_step(const float* d_qkv, const float* d_z, const float* d_gates,
                                               const uint16_t* d_conv_w, const uint16_t* d_a_log,
                                               const uint16_t* d_dt_bias, const uint16_t* d_norm_w, float eps, int M,
                                               int n_commit, float* d_state, uint16_t* d_history, float* d_out, void* stream) {
  return gdn_step(d_qkv, d_z, d_gates, d_conv_w, d_a_log, d_dt_bias, d_norm_w, eps, M, n_commit, GDN_V_HEADS, 0, 0,
                  GDN_QK_HEADS * GDN_DK, d_state, d_history, d_out, stream);
}

extern "C" YSKN_B200_API int yskn_b200_gdn_mixer_heads(const uint16_t* d_hidden, const float* d_inv_rms,
                                                      const uint16_t* d_wb, const uint16_t* d_wa, int hidden,
                                                      const float* d_qkv, const float* d_z, const uint16_t* d_conv_w,
                                                      const uint16_t* d_a_log, const uint16_t* d_dt_bias,
                                                      const uint16_t* d_norm_w, float eps, int M, int n_commit,
                                                      int n_v_heads, int v_head0, int qk_head0, int qk_channels,
                                                      float* d_state, uint16_t* d_history, float* d_out,
                                                      void* stream) {
  const MixerIn in{d_hidden, d_inv_rms, d_wb, d_wa, hidden};
  return gdn_step(d_qkv, d_z, nullptr, d_conv_w, d_a_log, d_dt_bias, d_norm_w, eps, M, n_commit, n_v_heads, v_head0,
                  qk_head0, qk_channels, d_state, d_history, d_out, stream, &in);
}

extern "C" YSKN_B200_API int yskn_b200_gdn_mixer(const uint16_t* d_hidden, const float* d_inv_rms,
                                                const uint16_t* d_wb, const uint16_t* d_wa, int hidden,
                                                const float* d_qkv, const float* d_z, const uint16_t* d_conv_w,
                                                const uint16_t* d_a_log, const uint16_t* d_dt_bias,
                                                const uint16_t* d_norm_w, float eps, int M, int n_commit,
                                                float* d_state, uint16_t* d_history, float* d_out, void* stream) {
  return yskn_b200_gdn_mixer_heads(d_hidden, d_inv_rms, d_wb, d_wa, hidden, d_qkv, d_z, d_conv_w, d_a_log, d_dt_bias,
                                   d_norm_w, eps, M, n_commit, GDN_V_HEADS, 0, 0, GDN_QK_HEADS * GDN_DK, d_state,
                                   d_history, d_out, stream);
}

extern "C" YSKN_B200_API int yskn_b200_gdn_step_heads(const float* d_qkv, const float* d_z, const float* d_gates,
                                                     const uint16_t* d_conv_w, const uint16_t* d_a_log,
                                                     const uint16_t* d_dt_bias, const uint16_t* d_norm_w, float eps,
                                                     int M, int n_commit, int n_v_heads, int v_head0, int qk_head0,
                                                     int qk_channels, float* d_state, uint16_t* d_history,
                                                     float* d_out, void* stream) {
  return gdn_step(d_qkv, d_z, d_gates, d_conv_w, d_a_log, d_dt_bias, d_norm_w, eps, M, n_commit, n_v_heads, v_head0,
                  qk_head0, qk_channels, d_state, d_history, d_out, stream);
}
