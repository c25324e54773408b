// Quantised-KV (packed 4-bit trellis rows) decode attention and split combination.
//
// Reference: launch_q35_atx_pk / q35_atxpk3 (src/q35_atxpk.cu:702-741,
// src/q35_atxpk3.cuh), combine q35_combine_kernel (src/q35_kernels.cu:1279-1399);
// scalar spec docs/spec/04_ATTENTION.md:310-453, crates/yskn-ref/src/attention.rs:
// 740-1075, row decode crates/yskn-ref/src/kv_codec.rs:467-495.
//
// Cache layout (per KV head h, per side): rows [length][8*kb words] of MSB-first
// kb-bit fields (kv_codec.rs:447-458), f32 row scales [length], the side's 256-entry
// BF16 codebook (bfloat(reconstruction(state))) and, for values, an optional mean.
// Channel c's 8-bit state is the last eight stream bits ending at its field, reset
// at every 64-channel chain: for kb = 4, (field[c-1] << 4 | field[c]) & 0xff.
//
// kv4_split_kernel: one CTA per (split, KV head), serving the G query heads of the
// KV head so each cache row is read once. Per 32-key tile: the packed K and V rows
// are staged in shared memory; warp w scores keys 4w..4w+3, 8 lanes per key over 32
// channels each, against the G queries; warp 0 updates the online softmax (exp2,
// LOG2E products as the spec orders them) and writes BF16-rounded value weights;
// thread t then accumulates value channel t for all G heads. Codebook lookups go to
// 32 bank-private copies (copy l in bank l), so a warp's 32 lookups are one
// shared-memory wavefront. The self row is handled separately with an FP32 weight,
// then den*mean is added. Sums are FP32 in this kernel's own order: parity with the
// scalar spec is within a tolerance (the reference's own kernels use an unspecified
// mma order, ATT-01).
//
// kv4_combine_kernel: one CTA per query head: combine the splits (padded to a
// power of two, native expf), divide, inverse H256 cache rotation with hash signs,
// BF16, times BF16 sigmoid(gate) when a gate is given.
#include <cuda_bf16.h>

#include "common.cuh"

namespace yskn {

constexpr int KV_THREADS = 256;
constexpr int KV_MAXG = KV_MAX_GROUP;
constexpr float KV_LOG2E = 1.4426950408889634f;

struct KvParams {
  const uint16_t* q;  // [n_qh][256] bf16
  const uint32_t* kw;
  const float* ks;
  const uint32_t* vw;
  const float* vs;
  const uint16_t* kbase;  // [n_kvh][256] bf16
  const uint16_t* vbase;
  const float* vmean;  // [n_kvh][256] or nullptr
  float* partials;     // [M][n_qh][max_splits][2 + 256]
  int M, n_qh, n_kvh, G, length, capacity, n_splits, max_splits, words;  // words per row = 8*kb
};

// Splits of query row m (reference schedule unless fixed by the caller).
__host__ __device__ __forceinline__ int kv_row_length(int length, int M, int m) { return length - M + 1 + m; }
__host__ __device__ __forceinline__ int kv_row_splits(int fixed, int len) { return fixed ? fixed : (len < 4096 ? 31 : 42); }

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// State of channel c of a packed row (kb = 4) from its 32 words in shared memory.
__device__ __forceinline__ uint32_t kv_state4(const uint32_t* row, int c) {
  const uint32_t w = row[c >> 3];
  const int i = c & 7;
  if (i != 0) return (w >> (28 - 4 * i)) & 0xffu;
  const uint32_t f = w >> 28;
  if ((c & 63) == 0) return f;
  return ((row[(c >> 3) - 1] & 0xfu) << 4) | f;
}

// Bank-private codebook: copy l of entry s at byte ((s >> 1) * 32 + l) * 4 + (s & 1) * 2.
__device__ __forceinline__ float lut_get(const uint8_t* lut, uint32_t s, int lane) {
  return bf16_to_f32(*reinterpret_cast<const uint16_t*>(lut + ((((s >> 1) << 5) + lane) << 2) + ((s & 1u) << 1)));
}

__global__ void __launch_bounds__(KV_THREADS) kv4_split_kernel(const __grid_constant__ KvParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t* lutK = sm;                                                    // 16 KiB
  uint8_t* lutV = sm + 16384;                                            // 16 KiB
  float* q_s = reinterpret_cast<float*>(sm + 32768);                     // [G][256]
  uint32_t* kt = reinterpret_cast<uint32_t*>(q_s + KV_MAXG * 256);       // [33][32] (row 32: self)
  uint32_t* vt = kt + 33 * 32;                                           // [33][32]
  float* ksc = reinterpret_cast<float*>(vt + 33 * 32);                   // [33]
  float* vsc = ksc + 33;                                                 // [33]
  float* sc_s = vsc + 33;                                                // [G][32] scores
  float* w_s = sc_s + KV_MAXG * 32;                                      // [G][32] value weights
  float* st_s = w_s + KV_MAXG * 32;                                      // [G][4]: max, den, rescale, self w

  const int h = blockIdx.y, s = blockIdx.x, m = blockIdx.z, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.G, W = p.words;
  const int length = kv_row_length(p.length, p.M, m);
  const int n_splits = kv_row_splits(p.n_splits, length);
  if (s >= n_splits) return;
  for (int i = tid; i < 256 * 32; i += KV_THREADS) {  // 32 copies of each 256-entry table
    const int e = i >> 5, l = i & 31;
    reinterpret_cast<uint16_t*>(lutK)[(((e >> 1) << 5) + l) * 2 + (e & 1)] = p.kbase[h * 256 + e];
    reinterpret_cast<uint16_t*>(lutV)[(((e >> 1) << 5) + l) * 2 + (e & 1)] = p.vbase[h * 256 + e];
  }
  for (int i = tid; i < G * 256; i += KV_THREADS) q_s[i] = bf16_to_f32(p.q[((size_t)m * p.n_qh + h * G) * 256 + i]);
  if (tid < G) {
    st_s[tid * 4 + 0] = -1e30f;
    st_s[tid * 4 + 1] = 0.0f;
  }
  const int per_split = (length + n_splits - 1) / n_splits;
  const int first = s * per_split;
  const int last = min(length, first + per_split);
  const int prefix_end = max(first, min(last, length - 1));
  const bool include_self = first <= length - 1 && length - 1 < first + per_split;
  float num[KV_MAXG];
#pragma unroll
  for (int g = 0; g < KV_MAXG; ++g) num[g] = 0.0f;
  const uint32_t* Kh = p.kw + (size_t)h * p.capacity * W;
  const uint32_t* Vh = p.vw + (size_t)h * p.capacity * W;
  const float* Ks = p.ks + (size_t)h * p.capacity;
  const float* Vs = p.vs + (size_t)h * p.capacity;
  __syncthreads();

  const int kk = warp * 4 + (lane >> 3), chunk = lane & 7;  // scoring role: key of the tile, 32-channel chunk
  for (int t0 = first / 32 * 32; t0 < prefix_end; t0 += 32) {
    for (int i = tid; i < 32 * 32; i += KV_THREADS) {  // stage 32 rows of K and V (kb = 4: 32 words each)
      const int r = i >> 5, wd = i & 31, pos = t0 + r;
      const bool in = pos < length;
      kt[r * 32 + wd] = in ? __ldg(Kh + (size_t)pos * W + wd) : 0u;
      vt[r * 32 + wd] = in ? __ldg(Vh + (size_t)pos * W + wd) : 0u;
    }
    if (tid < 32) {
      const int pos = t0 + tid;
      ksc[tid] = pos < length ? __ldg(Ks + pos) : 0.0f;
      vsc[tid] = pos < length ? __ldg(Vs + pos) : 0.0f;
    }
    __syncthreads();
    {
      const int pos = t0 + kk;
      const bool vis = pos >= first && pos < prefix_end;
      float acc[KV_MAXG];
#pragma unroll
      for (int g = 0; g < KV_MAXG; ++g) acc[g] = 0.0f;
      const uint32_t* row = kt + kk * 32;
#pragma unroll 8
      for (int c = 0; c < 32; ++c) {
        const int ch = chunk * 32 + c;
        const float kv = lut_get(lutK, kv_state4(row, ch), lane);
#pragma unroll
        for (int g = 0; g < KV_MAXG; ++g)
          if (g < G) acc[g] = __fmaf_rn(q_s[g * 256 + ch], kv, acc[g]);
      }
#pragma unroll
      for (int g = 0; g < KV_MAXG; ++g) {
        float a = acc[g];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        a += __shfl_xor_sync(0xffffffffu, a, 4);
        if (chunk == 0 && g < G) sc_s[g * 32 + kk] = vis ? a * (ksc[kk] * 0.0625f) : -INFINITY;
      }
    }
    __syncthreads();
    if (warp == 0) {  // online softmax update, lane = key of the tile
      for (int g = 0; g < G; ++g) {
        const float sc = sc_s[g * 32 + lane];
        float m = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float old = st_s[g * 4 + 0];
        const float nm = fmaxf(old, m);
        const float rescale = exp2f((old - nm) * KV_LOG2E);
        const float pr = sc == -INFINITY ? 0.0f : exp2f(sc * KV_LOG2E - nm * KV_LOG2E);
        float sum = pr;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        w_s[g * 32 + lane] = __bfloat162float(__float2bfloat16_rn(pr * vsc[lane]));
        __syncwarp();
        if (lane == 0) {
          st_s[g * 4 + 0] = nm;
          st_s[g * 4 + 1] = st_s[g * 4 + 1] * rescale + sum;
          st_s[g * 4 + 2] = rescale;
        }
        __syncwarp();
      }
    }
    __syncthreads();
    {  // values: thread = channel
      const int ch = tid;
#pragma unroll
      for (int g = 0; g < KV_MAXG; ++g)
        if (g < G) num[g] *= st_s[g * 4 + 2];
      for (int k = 0; k < 32; ++k) {
        const float vv = lut_get(lutV, kv_state4(vt + k * 32, ch), lane);
#pragma unroll
        for (int g = 0; g < KV_MAXG; ++g)
          if (g < G) num[g] = __fmaf_rn(w_s[g * 32 + k], vv, num[g]);
      }
    }
    __syncthreads();
  }

  if (include_self) {
    const int self = length - 1;
    for (int i = tid; i < 32; i += KV_THREADS) {
      kt[32 * 32 + i] = __ldg(Kh + (size_t)self * W + i);
      vt[32 * 32 + i] = __ldg(Vh + (size_t)self * W + i);
    }
    if (tid == 0) {
      ksc[32] = __ldg(Ks + self);
      vsc[32] = __ldg(Vs + self);
    }
    __syncthreads();
    if (warp == 0) {  // lane covers channels lane*8 .. lane*8+7
      for (int g = 0; g < G; ++g) {
        float a = 0.0f;
        for (int c = lane * 8; c < lane * 8 + 8; ++c)
          a = __fmaf_rn(q_s[g * 256 + c], lut_get(lutK, kv_state4(kt + 32 * 32, c), lane), a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) {
          const float score = a * (ksc[32] * 0.0625f);
          const float old = st_s[g * 4 + 0];
          const float nm = fmaxf(old, score);
          const float rescale = exp2f((old - nm) * KV_LOG2E);
          const float pr = exp2f((score - nm) * KV_LOG2E);
          st_s[g * 4 + 0] = nm;
          st_s[g * 4 + 1] = st_s[g * 4 + 1] * rescale + pr;
          st_s[g * 4 + 2] = rescale;
          st_s[g * 4 + 3] = pr * vsc[32];
        }
        __syncwarp();
      }
    }
    __syncthreads();
    const float vv = lut_get(lutV, kv_state4(vt + 32 * 32, tid), lane);
#pragma unroll
    for (int g = 0; g < KV_MAXG; ++g)
      if (g < G) num[g] = num[g] * st_s[g * 4 + 2] + st_s[g * 4 + 3] * vv;
  }
  if (p.vmean) {
    const float m = p.vmean[h * 256 + tid];
#pragma unroll
    for (int g = 0; g < KV_MAXG; ++g)
      if (g < G) num[g] += st_s[g * 4 + 1] * m;
  }
  for (int g = 0; g < G; ++g) {
    float* out = p.partials + (((size_t)m * p.n_qh + h * G + g) * p.max_splits + s) * 258;
    if (tid == 0) {
      out[0] = st_s[g * 4 + 0];
      out[1] = st_s[g * 4 + 1];
    }
    out[2 + tid] = num[g];
  }
}

__device__ __forceinline__ float kv_cache_sign(int channel) {  // attention.rs:997-1005
  unsigned v = (unsigned)channel + 1u;
  v ^= v >> 16;
  v *= 0x7feb352du;
  v ^= v >> 15;
  v *= 0x846ca68bu;
  v ^= v >> 16;
  return (v & 1u) ? -1.0f : 1.0f;
}

__global__ void __launch_bounds__(256) kv4_combine_kernel(const __grid_constant__ KvParams p,
                                                          const uint16_t* __restrict__ gate, float* __restrict__ attended,
                                                          uint16_t* __restrict__ out) {
  __shared__ float sc[KV_MAX_SPLITS];
  __shared__ float buf[256];
  __shared__ float tot;
  const int qh = blockIdx.x, m = blockIdx.y, t = threadIdx.x;
  const int n_splits = kv_row_splits(p.n_splits, kv_row_length(p.length, p.M, m));
  const size_t row = (size_t)m * p.n_qh + qh;
  const float* P = p.partials + row * p.max_splits * 258;
  int padded = 1;
  while (padded < n_splits) padded <<= 1;
  if (t < 32) {
    float mx = -1e30f;
    for (int s = t; s < padded; s += 32) mx = fmaxf(mx, s < n_splits ? P[(size_t)s * 258] : -1e30f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int s = t; s < padded; s += 32) {
      const float ms = s < n_splits ? P[(size_t)s * 258] : -1e30f;
      sc[s] = ms > -1e29f ? expf(ms - mx) : 0.0f;
    }
    __syncwarp();
    if (t == 0) {
      float d = 0.0f;
      for (int s = 0; s < n_splits; ++s) d += sc[s] * P[(size_t)s * 258 + 1];
      tot = d;
    }
  }
  __syncthreads();
  float n = 0.0f;
  for (int s = 0; s < n_splits; ++s) n += sc[s] * P[(size_t)s * 258 + 2 + t];
  const float a = n / tot;
  if (attended) attended[row * 256 + t] = a;
  buf[t] = a;
  __syncthreads();
  for (int d = 1; d < 256; d <<= 1) {  // inverse cache rotation: ascending H256 strides
    const float x = buf[t], y = buf[t ^ d];
    __syncthreads();
    buf[t] = (t & d) ? y - x : x + y;
    __syncthreads();
  }
  const float r = __bfloat162float(__float2bfloat16_rn((buf[t] * 0.0625f) * kv_cache_sign(t)));
  float o = r;
  if (gate) {
    const float gv = __uint_as_float((uint32_t)gate[row * 256 + t] << 16);
    const float sg = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-gv))));
    o = r * sg;
  }
  out[row * 256 + t] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
}

static size_t kv4_smem_bytes() {
  return 32768 + (KV_MAXG * 256) * 4 + 2 * 33 * 32 * 4 + 2 * 33 * 4 + 2 * KV_MAXG * 32 * 4 + KV_MAXG * 4 * 4;
}

int kv_max_splits(const KvArgs& a) {
  return a.n_splits ? a.n_splits : (kv_row_length(a.length, a.M, a.M - 1) < 4096 ? 31 : 42);
}

int64_t kv_partials_floats(int M, int n_qh, int max_splits) { return (int64_t)M * n_qh * max_splits * 258; }

int launch_kv4_attention(const KvArgs& a, cudaStream_t st) {
  KvParams p{};
  p.q = a.q;
  p.kw = a.kw;
  p.ks = a.ks;
  p.vw = a.vw;
  p.vs = a.vs;
  p.kbase = a.kbase;
  p.vbase = a.vbase;
  p.vmean = a.vmean;
  p.partials = a.partials;
  p.M = a.M;
  p.n_qh = a.n_qh;
  p.n_kvh = a.n_kvh;
  p.G = a.n_qh / a.n_kvh;
  p.length = a.length;
  p.capacity = a.capacity;
  p.n_splits = a.n_splits;
  p.max_splits = kv_max_splits(a);
  p.words = 8 * a.kb;
  static bool attr[64] = {};
  int dev = 0;
  if (int rc = cuda_fail(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(YSKN_EINVAL, "device ordinal out of range");
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kv4_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kv4_smem_bytes());
    if (e != cudaSuccess) return cuda_fail(e, "kv4 attributes");
    attr[dev] = true;
  }
  kv4_split_kernel<<<dim3(p.max_splits, a.n_kvh, a.M), KV_THREADS, kv4_smem_bytes(), st>>>(p);
  if (int rc = cuda_fail(cudaGetLastError(), "kv4_split_kernel")) return rc;
  kv4_combine_kernel<<<dim3(a.n_qh, a.M), 256, 0, st>>>(p, a.gate, a.attended, a.out);
  return cuda_fail(cudaGetLastError(), "kv4_combine_kernel");
}

}  // namespace yskn
