// Quantised-KV (packed 4-bit trellis rows) decode attention with the split
// combination, inverse cache rotation and output gate, in one launch.
//
// Reference: launch_q35_atx_pk / q35_atxpk3 (src/q35_atxpk.cu:702-741,
// src/q35_atxpk3.cuh), combine q35_combine_kernel (src/q35_kernels.cu:1279-1399);
// scalar spec docs/spec/04_ATTENTION.md:310-453, crates/yskn-ref/src/attention.rs:
// 207-232,740-1075, row decode crates/yskn-ref/src/kv_codec.rs:467-495.
//
// Cache layout (per KV head h, per side): rows [capacity][32 words] of MSB-first
// 4-bit fields (kv_codec.rs:447-458), f32 row scales [capacity], the side's
// 256-entry BF16 codebook (bfloat(reconstruction(state))) and, for values, an
// optional mean. Channel c's 8-bit state is (field[c-1] << 4 | field[c]) & 0xff,
// with field[-1] = 0 at every 64-channel chain start.
//
// kv4_attention_kernel: one CTA (8 warps) per (split, KV head, query row); the CTA
// serves the G <= 8 query heads of the KV head, so each cache row is read once per
// query row. Warps take the split's 32-key tiles round-robin (two 16-key blocks
// each). Rows and row scales arrive by cp.async into per-warp two-stage rings, K and
// V separately (16-byte chunks XOR-swizzled by row, so the fragment reads below are
// conflict-free); the first blocks' K, V and scales and the self row are requested
// before the codebooks are built, so their DRAM latency overlaps the set-up.
// Per chunk of up to 64 tiles:
//   (A) S^T = K Q^T with mma.sync m16n8k16 bf16 (A = 16 keys x 16 channels, B = Q^T
//       with the heads as the 8 columns). Lane (g, t) supplies keys g, g+8 and owns
//       channels 64t..64t+63 (words 8t..8t+7 of each row): exactly one 64-channel
//       chain, so every state is built from the lane's own words. MMA i takes
//       channels 64t+4i..+3. Scores (C layout: keys g, g+8 x heads 2t, 2t+1) go to
//       shared memory with the tile maxima.
//   (B) the split's running maximum at each tile: a prefix max over the tiles, the
//       value the scalar schedule holds when it reaches that tile.
//   (C) p = exp2(score * LOG2E - max * LOG2E) against that running max and BF16
//       value weights p * Vscale (the spec's BF16 boundary, so the rounded weights are
//       the scalar schedule's), then O^T += V^T P^T with mma.sync (A = 16 channels x
//       16 keys, B = P^T through a 256-byte shared transpose). Lane (g, t) decodes keys
//       2t, 2t+1, 2t+8, 2t+9 over words 4g..4g+3 (channels 32g..32g+31: nibble n ->
//       MMA tile n/2, row g or g+8); the first state of an odd g takes one nibble from
//       lane g-1 (one shuffle).
// Codebook lookups go to 32 bank-private copies (entry s, copy l at word 32s + l),
// so a warp's 32 lookups are one shared-memory wavefront; the address is one shift
// (a funnel shift for a word's first state) and one LOP3.
// Then the warps' (max, den, O) are merged, the self row added (FP32 weight, as the
// spec keeps it separate) and den * mean; the CTA writes its split partial. The splits
// of a (query row, KV head) are combined (padded to a power of two, the portable exp),
// divided, inverse-rotated (H256 with the hash signs), rounded to BF16 and multiplied by
// the BF16 sigmoid of the gate: when the grid is one wave of CTAs, by the last G CTAs to
// arrive (an arrival counter in a static device array), one query head each with the
// whole CTA, the earlier ones waiting (bounded) for the last arrival; otherwise by the
// last CTA, one warp per head. The combiners count themselves in after the arrivals and
// the last of them resets the counter.
// Sums are FP32 in this kernel's own order: parity with the scalar spec is within a
// tolerance (the reference's own kernels also use an unspecified MMA order, ATT-01).
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "pmath.cuh"

namespace yskn {

constexpr int KV_WARPS = 8;
constexpr int KV_THREADS = KV_WARPS * 32;
constexpr float KV_LOG2E = 1.4426950408889634f;
constexpr int KV_CHUNK_TILES = 64;  // 32-key tiles per chunk (2048 keys)
// A split partial: max, den, two pad floats, num[256]; 260 floats keep every record and
// its numerator 16-byte aligned for the combine's vector loads.
constexpr int KV_PART = 260;
constexpr int KV_NUM = 4;

// Arrival counters of the (query row, KV head) pairs of a launch: zero when the module
// loads, and reset by the last CTA of each pair, so they are zero between launches.
__device__ unsigned g_kv_arrivals[KV_MAX_ARRIVALS];

struct KvParams {
  const uint16_t* q;  // [M][n_qh][256] bf16
  const uint32_t* kw;
  const float* ks;
  const uint32_t* vw;
  const float* vs;
  const uint16_t* kbase;  // [n_kvh][256] bf16
  const uint16_t* vbase;
  const float* vmean;     // [n_kvh][256] or nullptr
  const uint16_t* gate;   // [M][n_qh][256] bf16 or nullptr
  float* partials;        // [M][n_qh][max_splits][KV_PART]: max, den, 2 pad, num[256]
  float* attended;        // [M][n_qh][256] or nullptr
  uint16_t* out;          // [M][n_qh][256] bf16
  int M, n_qh, n_kvh, G, length, capacity, n_splits, max_splits;
  int one_wave;  // every CTA of the grid fits on the SMs at once
  unsigned* err;
};
constexpr long long KV_WAIT_LIMIT = 2000000000ll;  // clock cycles (~1 s) before a combiner's wait gives up

// Splits of query row m (reference schedule unless fixed by the caller).
__host__ __device__ __forceinline__ int kv_row_length(int length, int M, int m) { return length - M + 1 + m; }
__host__ __device__ __forceinline__ int kv_row_splits(int fixed, int len) { return fixed ? fixed : (len < 4096 ? 31 : 42); }

struct KvSmem {
  uint32_t lut[2][256 * 32];          // K, V codebooks: 32 bank-private copies, BF16 bits in the low half
  uint4 stage[2][KV_WARPS][2][128];   // K|V, warp, stage: 16 rows x 8 swizzled 16-byte chunks
  float sscale[2][KV_WARPS][2][16];   // K|V row scales of the staged blocks
  union {
    float score[KV_CHUNK_TILES * 32][8];  // the chunk's scores [key][head]
    float merge[KV_WARPS][8][256];        // after the chunks: each warp's O per head
  } u;
  float tmax[KV_CHUNK_TILES][8];  // per tile max, then the running (prefix) max
  float run[8];                   // running max after the previous chunks
  uint16_t pt[KV_WARPS][8 * 16];  // per warp: P^T transpose, [head][key] bf16
  float wmax[KV_WARPS][8], wden[KV_WARPS][8];
  float self_score[8];
  uint4 selfrow[2][8];   // the self row's K and V words
  float selfscale[4];    // its K and V scales
  float comb[KV_WARPS][KV_MAX_SPLITS];  // per combining warp: the splits' weights
  float vmean[256];                      // the value mean (zeros without one), staged at set-up
  uint16_t qrow[KV_MAX_GROUP][256];      // the G query rows (bf16), staged at set-up for the self score
  int last;
};

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of the codebook entry of nibble n's state in this lane's copy: the
// state's 8 bits land in address bits 7..14 (entry * 128) with one shift, the copy
// (lane * 4) is OR-ed in. prev: the word before w in the chain (0 at a chain start).
__device__ __forceinline__ uint32_t lut_off(uint32_t w, uint32_t prev, int n, uint32_t lane4) {
  uint32_t x;
  if (n == 0) x = __funnelshift_r(w, prev, 21);
  else if (n <= 5) x = w >> (21 - 4 * n);
  else x = w << (4 * n - 21);
  return (x & 0x7f80u) | lane4;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t pack2(uint32_t lo, uint32_t hi) {  // lo | hi << 16 on the FMA pipe
  uint32_t r;
  asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(r) : "r"(hi), "r"(lo));
  return r;
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait(bool keep_one) {
  if (keep_one) asm volatile("cp.async.wait_group 1;" ::: "memory");
  else asm volatile("cp.async.wait_group 0;" ::: "memory");
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

// The split combination of one query head's partials (q35_combine_kernel; spec
// 04_ATTENTION.md:428-453: pad to a power of two, the portable exp, divide), the inverse
// cache rotation, BF16 and the gate, by one warp: lane l owns channels 8l..8l+7, so
// the H256 strides 1..4 stay in the lane and 8..128 are lane shuffles (ascending).
// One warp: the splits' weights comb[s] = exp(max_s - max) (zero for the padding) and
// the total den, lane-parallel over s = lane + 32 i, then a butterfly sum.
__device__ __forceinline__ float kv_split_weights(const float* P, int n_splits, float* comb, int lane) {
  float ms[2], ds[2];  // split s = lane + 32 i (at most 64 splits): its max and den, loaded once
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int s = lane + 32 * i;
    const float2 md = s < n_splits ? __ldcg(reinterpret_cast<const float2*>(P + (size_t)s * KV_PART))
                                   : make_float2(-1e30f, 0.0f);
    ms[i] = md.x;
    ds[i] = md.y;
  }
  int padded = 1;
  while (padded < n_splits) padded <<= 1;
  float mx = fmaxf(ms[0], ms[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int s = lane + 32 * i;
    if (s >= padded) break;
    const float f = ms[i] > -1e29f ? pm_exp(ms[i] - mx) : 0.0f;
    comb[s] = f;
    if (s < n_splits) tot += f * ds[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  __syncwarp();
  return tot;
}

__device__ void finish_head(const KvParams& p, float (&v)[8], uint4 gate8, size_t row, int lane);

// comb: this warp's 64 floats of scratch. The gate and the first KV_COMB_BATCH splits'
// numerators are requested before the split weights are formed, and the splits are
// then taken in batches of that many with all their loads in flight (the sums still
// run over the splits in ascending order).
constexpr int KV_COMB_BATCH = 20;
__device__ void combine_head_warp(const KvParams& p, float* comb, size_t row, int n_splits, int lane) {
  const float* P = p.partials + row * p.max_splits * KV_PART;
  uint4 gate8 = make_uint4(0, 0, 0, 0);
  if (p.gate) gate8 = __ldg(reinterpret_cast<const uint4*>(p.gate + row * 256 + 8 * lane));
  float4 nb[KV_COMB_BATCH][2];
  auto load_batch = [&](int s0) {
#pragma unroll
    for (int j = 0; j < KV_COMB_BATCH; ++j)
      if (s0 + j < n_splits) {
        const float4* src = reinterpret_cast<const float4*>(P + (size_t)(s0 + j) * KV_PART + KV_NUM + 8 * lane);
        nb[j][0] = __ldcg(src);
        nb[j][1] = __ldcg(src + 1);
      }
  };
  load_batch(0);
  const float tot = kv_split_weights(P, n_splits, comb, lane);
  float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  for (int s0 = 0; s0 < n_splits; s0 += KV_COMB_BATCH) {
#pragma unroll
    for (int j = 0; j < KV_COMB_BATCH; ++j)
      if (s0 + j < n_splits) {
        const float f = comb[s0 + j];
        const float4 a = nb[j][0], b = nb[j][1];
        v[0] += f * a.x; v[1] += f * a.y; v[2] += f * a.z; v[3] += f * a.w;
        v[4] += f * b.x; v[5] += f * b.y; v[6] += f * b.z; v[7] += f * b.w;
      }
    load_batch(s0 + KV_COMB_BATCH);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = v[e] / tot;
  finish_head(p, v, gate8, row, lane);
}

// The same combination of one query head by a whole CTA: thread t owns channel t and
// has all the splits' numerators of its channel in flight at once, warp 0 forms the
// weights meanwhile; the per-channel sums run over the splits in the same ascending
// order as above (same bits). Then warp 0 finishes the head from shared memory.
// stage: 256 floats of shared scratch; comb: 64; tot_s: 1.
__device__ void combine_head_cta(const KvParams& p, float* comb, float* stage, float* tot_s, size_t row,
                                 int n_splits) {
  const int tid = threadIdx.x, lane = tid & 31;
  const float* P = p.partials + row * p.max_splits * KV_PART;
  constexpr int CH = 32;  // splits in flight per thread
  float val[CH];
  auto load = [&](int s0) {
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (s0 + j < n_splits) val[j] = __ldcg(P + (size_t)(s0 + j) * KV_PART + KV_NUM + tid);
  };
  load(0);
  uint4 gate8 = make_uint4(0, 0, 0, 0);
  if (tid < 32 && p.gate) gate8 = __ldg(reinterpret_cast<const uint4*>(p.gate + row * 256 + 8 * lane));
  if (tid < 32) {
    const float tot = kv_split_weights(P, n_splits, comb, lane);
    if (lane == 0) *tot_s = tot;
  }
  __syncthreads();
  float v = 0.0f;
  for (int s0 = 0; s0 < n_splits; s0 += CH) {
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (s0 + j < n_splits) v += comb[s0 + j] * val[j];
    if (s0 + CH < n_splits) load(s0 + CH);
  }
  stage[tid] = v / *tot_s;
  __syncthreads();
  if (tid < 32) {
    float w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = stage[8 * lane + e];
    finish_head(p, w, gate8, row, lane);
  }
}

// The divided head (lane l: channels 8l..8l+7): the attended values, the inverse H256
// cache rotation with the hash signs, BF16, times the BF16 sigmoid of the gate.
__device__ void finish_head(const KvParams& p, float (&v)[8], uint4 gate8, size_t row, int lane) {
  if (p.attended) {
    float4* dst = reinterpret_cast<float4*>(p.attended + row * 256 + 8 * lane);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
#pragma unroll
  for (int d = 1; d < 8; d <<= 1) {  // strides 1, 2, 4 inside the lane
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (!(e & d)) {
        const float x = v[e], y = v[e | d];
        v[e] = x + y;
        v[e | d] = x - y;
      }
  }
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {  // strides 8..128: lane bit d
    const bool upper = (lane & d) != 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, v[e], d);
      v[e] = upper ? other - v[e] : v[e] + other;
    }
  }
  uint32_t packed[4];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int ch = 8 * lane + e;
    const float r = __bfloat162float(__float2bfloat16_rn((v[e] * 0.0625f) * kv_cache_sign(ch)));
    float o = r;
    if (p.gate) {
      const uint32_t gw = (&gate8.x)[e >> 1];
      const float gv = __uint_as_float((e & 1) ? (gw & 0xffff0000u) : (gw << 16));
      const float sg = __bfloat162float(__float2bfloat16_rn(pm_sigmoid(gv)));
      o = r * sg;
    }
    const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(o));
    packed[e >> 1] = (e & 1) ? (packed[e >> 1] | (b << 16)) : b;
  }
  *reinterpret_cast<uint4*>(p.out + row * 256 + 8 * lane) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

__global__ void __launch_bounds__(KV_THREADS, 1) kv4_attention_kernel(const __grid_constant__ KvParams p) {
  extern __shared__ __align__(128) uint8_t kv_raw[];
  KvSmem& S = *reinterpret_cast<KvSmem*>(kv_raw);
  const int s = blockIdx.x, h = blockIdx.y, m = blockIdx.z, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.G;
  const int length = kv_row_length(p.length, p.M, m);
  const int n_splits = kv_row_splits(p.n_splits, length);
  if (s >= n_splits) return;
  const int per_split = (length + n_splits - 1) / n_splits;
  const int first = s * per_split;
  const int last = min(length, first + per_split);
  const int prefix_end = max(first, min(last, length - 1));
  const bool include_self = first <= length - 1 && length - 1 < first + per_split;
  const int self = length - 1;
  const uint32_t* Kh = p.kw + (size_t)h * p.capacity * 32;
  const uint32_t* Vh = p.vw + (size_t)h * p.capacity * 32;
  const float* Ks = p.ks + (size_t)h * p.capacity;
  const float* Vs = p.vs + (size_t)h * p.capacity;

  // The split's 32-key tiles (absolute alignment, attention.rs:207-232) overlapping
  // [first, prefix_end), in chunks of up to 64 tiles; warp w takes tiles w, w+8, ...
  const int tile0 = first >> 5;
  const int n_tiles = prefix_end > first ? ((prefix_end - 1) >> 5) - tile0 + 1 : 0;
  auto blocks_of = [&](int c0) {  // this warp's 16-key blocks in the chunk starting at tile c0
    const int nt = min(KV_CHUNK_TILES, n_tiles - c0);
    return nt > warp ? 2 * ((nt - warp + KV_WARPS - 1) / KV_WARPS) : 0;
  };
  auto block_pos = [&](int c0, int j) { return (tile0 + c0 + warp + KV_WARPS * (j >> 1)) * 32 + (j & 1) * 16; };
  // Rows [pos0, pos0 + 16) of one side into stage st (rows past the cache end: zeros).
  auto copy_rows = [&](int side, int pos0, int st) {
    const uint32_t* base = side ? Vh : Kh;
    const float* sc = side ? Vs : Ks;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int q = lane + 32 * k, r = q >> 3, c = q & 7;
      const int pos = pos0 + r;
      const bool ok = pos < length;
      cp_async16(&S.stage[side][warp][st][r * 8 + (c ^ (r & 7))], base + (size_t)(ok ? pos : 0) * 32 + c * 4,
                 ok ? 16 : 0);
    }
    if (lane < 16) {
      const bool ok = pos0 + lane < length;
      cp_async4(&S.sscale[side][warp][st][lane], sc + (ok ? pos0 + lane : 0), ok ? 4 : 0);
    }
  };

  // Programmatic dependent launch: the next kernel on the stream may be scheduled as SMs
  // free up (it waits before it reads anything this grid writes).
  asm volatile("griddepcontrol.launch_dependents;");
  // 32 copies of each codebook: one coalesced load of the 256 entries (staged in the
  // transpose buffers), then consecutive-word stores read back as broadcasts. The
  // codebooks and the value mean belong to the model, so they are fetched and expanded
  // before this grid waits for the previous kernel on the stream.
  uint16_t* raw_k = &S.pt[0][0];
  uint16_t* raw_v = &S.pt[2][0];
  raw_k[tid] = p.kbase[h * 256 + tid];
  raw_v[tid] = p.vbase[h * 256 + tid];
  S.vmean[tid] = p.vmean ? __ldg(p.vmean + h * 256 + tid) : 0.0f;  // for the end of the kernel
  __syncthreads();
#pragma unroll 8
  for (int i = tid; i < 256 * 32; i += KV_THREADS) {
    S.lut[0][i] = raw_k[i >> 5];
    S.lut[1][i] = raw_v[i >> 5];
  }
  if (tid < 8) S.run[tid] = -1e30f;
  // First requests: the chunk's first two blocks of this warp (K, V, scales) and the self row.
  // Blocks wholly before the call's M new rows hold earlier steps' rows, which no kernel
  // just before this one writes: they are requested before the wait.
  int nb = n_tiles > 0 ? blocks_of(0) : 0;
  int j0 = 0;
  for (; j0 < min(nb, 2) && block_pos(0, j0) + 16 <= p.length - p.M; ++j0) {
    copy_rows(0, block_pos(0, j0), j0);
    copy_rows(1, block_pos(0, j0), j0);
    cp_commit();
  }
  // The new rows (from the encoder just before), the queries and the gate may be the
  // previous kernel's output: wait for it (a no-op without a programmatic launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int j = j0; j < min(nb, 2); ++j) {
    copy_rows(0, block_pos(0, j), j);
    copy_rows(1, block_pos(0, j), j);
    cp_commit();
  }
  if (include_self && warp == KV_WARPS - 1) {
    if (lane < 16) cp_async16(&S.selfrow[lane >> 3][lane & 7], (lane < 8 ? Kh : Vh) + (size_t)self * 32 + (lane & 7) * 4, 16);
    else if (lane < 18) cp_async4(&S.selfscale[lane - 16], (lane == 16 ? Ks : Vs) + self, 4);
    cp_commit();
  }
  // The query rows, staged for the self score at the end of the kernel.
  for (int hh = 0; hh < G; ++hh) S.qrow[hh][tid] = __ldg(p.q + ((size_t)m * p.n_qh + h * G + hh) * 256 + tid);
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  // B fragments of Q^T: head g (zero beyond G), channels 64t + 4i + {0,1} and {2,3}.
  uint32_t qb[16][2];
  {
    const uint16_t* qr = p.q + ((size_t)m * p.n_qh + h * G + min(g, G - 1)) * 256 + 64 * t;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(qr + 4 * i));
      qb[i][0] = g < G ? v.x : 0u;
      qb[i][1] = g < G ? v.y : 0u;
    }
  }
  __syncthreads();
  const uint32_t lutK = (uint32_t)__cvta_generic_to_shared(S.lut[0]);
  const uint32_t lutV = (uint32_t)__cvta_generic_to_shared(S.lut[1]);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  // Heads 2t, 2t+1: the running max of this warp's latest tile, and den over this lane's keys.
  float mx0 = -1e30f, mx1 = -1e30f, den0 = 0.0f, den1 = 0.0f;

  for (int c0 = 0; c0 < n_tiles; c0 += KV_CHUNK_TILES) {
    const int nt = min(KV_CHUNK_TILES, n_tiles - c0);
    nb = blocks_of(c0);
    const int chunk_pos = (tile0 + c0) * 32;
    if (c0 > 0) {
      for (int j = 0; j < min(nb, 2); ++j) {
        copy_rows(0, block_pos(c0, j), j);
        copy_rows(1, block_pos(c0, j), j);
        cp_commit();
      }
    }

    // ---- (A) scores S^T = K Q^T and tile maxima
    float tm0 = -INFINITY, tm1 = -INFINITY;
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      cp_wait(j + 1 < nb);
      __syncwarp();
      const int pos0 = block_pos(c0, j);
      const int kg = pos0 + g, kg8 = kg + 8;
      const bool vis0 = kg >= first && kg < prefix_end, vis1 = kg8 >= first && kg8 < prefix_end;
      const float ksc0 = S.sscale[0][warp][st][g] * 0.0625f, ksc1 = S.sscale[0][warp][st][g + 8] * 0.0625f;
      const uint4* Kt = S.stage[0][warp][st];
      float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      float cc[3][4] = {};  // four independent accumulation chains (i % 4), added at the end
      {
        uint32_t wa[8], wb[8];
        const uint4 a0 = Kt[g * 8 + ((2 * t) ^ g)], a1 = Kt[g * 8 + ((2 * t + 1) ^ g)];
        const uint4 b0 = Kt[(g + 8) * 8 + ((2 * t) ^ g)], b1 = Kt[(g + 8) * 8 + ((2 * t + 1) ^ g)];
        wa[0] = a0.x; wa[1] = a0.y; wa[2] = a0.z; wa[3] = a0.w; wa[4] = a1.x; wa[5] = a1.y; wa[6] = a1.z; wa[7] = a1.w;
        wb[0] = b0.x; wb[1] = b0.y; wb[2] = b0.z; wb[3] = b0.w; wb[4] = b1.x; wb[5] = b1.y; wb[6] = b1.z; wb[7] = b1.w;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k = i >> 1, n0 = (i & 1) * 4;
          const uint32_t pa = k ? wa[k - 1] : 0u, pb = k ? wb[k - 1] : 0u;
          const uint32_t x0 = pack2(lds32(lutK + lut_off(wa[k], pa, n0, lane4)),
                                    lds32(lutK + lut_off(wa[k], pa, n0 + 1, lane4)));
          const uint32_t x2 = pack2(lds32(lutK + lut_off(wa[k], pa, n0 + 2, lane4)),
                                    lds32(lutK + lut_off(wa[k], pa, n0 + 3, lane4)));
          const uint32_t x1 = pack2(lds32(lutK + lut_off(wb[k], pb, n0, lane4)),
                                    lds32(lutK + lut_off(wb[k], pb, n0 + 1, lane4)));
          const uint32_t x3 = pack2(lds32(lutK + lut_off(wb[k], pb, n0 + 2, lane4)),
                                    lds32(lutK + lut_off(wb[k], pb, n0 + 3, lane4)));
          if ((i & 3) == 0) mma_bf16(c, x0, x1, x2, x3, qb[i][0], qb[i][1]);
          else mma_bf16(cc[(i & 3) - 1], x0, x1, x2, x3, qb[i][0], qb[i][1]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) c[e] = (c[e] + cc[0][e]) + (cc[1][e] + cc[2][e]);
      }
      const float s00 = vis0 ? c[0] * ksc0 : -INFINITY, s01 = vis0 ? c[1] * ksc0 : -INFINITY;
      const float s10 = vis1 ? c[2] * ksc1 : -INFINITY, s11 = vis1 ? c[3] * ksc1 : -INFINITY;
      const int kc = pos0 - chunk_pos + g;
      S.u.score[kc][2 * t] = s00;
      S.u.score[kc][2 * t + 1] = s01;
      S.u.score[kc + 8][2 * t] = s10;
      S.u.score[kc + 8][2 * t + 1] = s11;
      tm0 = fmaxf(tm0, fmaxf(s00, s10));
      tm1 = fmaxf(tm1, fmaxf(s01, s11));
      if (j & 1) {  // the tile's two blocks are done
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
          tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
        }
        if (g == 0) {
          const int tt = warp + KV_WARPS * (j >> 1);
          S.tmax[tt][2 * t] = tm0;
          S.tmax[tt][2 * t + 1] = tm1;
        }
        tm0 = tm1 = -INFINITY;
      }
      __syncwarp();
      if (j + 2 < nb) {
        copy_rows(0, block_pos(c0, j + 2), st);
        cp_commit();
      }
    }
    cp_wait(false);
    __syncthreads();

    // ---- (B) the split's running max at each tile of the chunk
    if (tid < 8) {
      float r = S.run[tid];
      for (int tt = 0; tt < nt; ++tt) {
        r = fmaxf(r, S.tmax[tt][tid]);
        S.tmax[tt][tid] = r;
      }
      S.run[tid] = r;
    }
    __syncthreads();

    // ---- (C) BF16 value weights against the running max; O^T += V^T P^T
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      cp_wait(j + 1 < nb);
      __syncwarp();
      const int pos0 = block_pos(c0, j);
      if ((j & 1) == 0) {  // a new tile: move to the split's running max there
        const int tt = warp + KV_WARPS * (j >> 1);
        const float nm0 = S.tmax[tt][2 * t], nm1 = S.tmax[tt][2 * t + 1];
        const float r0 = exp2f((mx0 - nm0) * KV_LOG2E), r1 = exp2f((mx1 - nm1) * KV_LOG2E);
        den0 *= r0;
        den1 *= r1;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[i][0] *= r0;
          o[i][1] *= r1;
          o[i][2] *= r0;
          o[i][3] *= r1;
        }
        mx0 = nm0;
        mx1 = nm1;
      }
      const int kg = pos0 + g, kg8 = kg + 8;
      const bool vis0 = kg >= first && kg < prefix_end, vis1 = kg8 >= first && kg8 < prefix_end;
      const float vsc0 = S.sscale[1][warp][st][g], vsc1 = S.sscale[1][warp][st][g + 8];
      const int kc = pos0 - chunk_pos + g;
      const float l0 = mx0 * KV_LOG2E, l1 = mx1 * KV_LOG2E;
      const float p00 = vis0 ? exp2f(S.u.score[kc][2 * t] * KV_LOG2E - l0) : 0.0f;
      const float p01 = vis0 ? exp2f(S.u.score[kc][2 * t + 1] * KV_LOG2E - l1) : 0.0f;
      const float p10 = vis1 ? exp2f(S.u.score[kc + 8][2 * t] * KV_LOG2E - l0) : 0.0f;
      const float p11 = vis1 ? exp2f(S.u.score[kc + 8][2 * t + 1] * KV_LOG2E - l1) : 0.0f;
      den0 += p00 + p10;
      den1 += p01 + p11;
      uint16_t* pt = S.pt[warp];
      pt[(2 * t) * 16 + g] = __bfloat16_as_ushort(__float2bfloat16_rn(p00 * vsc0));
      pt[(2 * t + 1) * 16 + g] = __bfloat16_as_ushort(__float2bfloat16_rn(p01 * vsc0));
      pt[(2 * t) * 16 + g + 8] = __bfloat16_as_ushort(__float2bfloat16_rn(p10 * vsc1));
      pt[(2 * t + 1) * 16 + g + 8] = __bfloat16_as_ushort(__float2bfloat16_rn(p11 * vsc1));
      __syncwarp();
      const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(pt + g * 16 + 2 * t);
      const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(pt + g * 16 + 2 * t + 8);
      const uint4* Vt = S.stage[1][warp][st];
      uint32_t v[4][4], pv[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // keys 2t, 2t+1, 2t+8, 2t+9; words 4g..4g+3
        const int key = 2 * t + (kk & 1) + (kk >> 1) * 8;
        const uint4 x = Vt[key * 8 + (g ^ (key & 7))];
        v[kk][0] = x.x; v[kk][1] = x.y; v[kk][2] = x.z; v[kk][3] = x.w;
        const uint32_t up = __shfl_up_sync(0xffffffffu, x.w, 4);  // lane g-1's last word of the same key
        pv[kk] = (g & 1) ? up : 0u;                               // even g starts a 64-channel chain
      }
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        const int wd = mt >> 2, n0 = (2 * mt) & 7;  // nibbles 2mt (row g) and 2mt+1 (row g+8)
        uint32_t e[4][2];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t prev = wd ? v[kk][wd - 1] : pv[kk];
          e[kk][0] = lds32(lutV + lut_off(v[kk][wd], prev, n0, lane4));
          e[kk][1] = lds32(lutV + lut_off(v[kk][wd], prev, n0 + 1, lane4));
        }
        mma_bf16(o[mt], pack2(e[0][0], e[1][0]), pack2(e[0][1], e[1][1]), pack2(e[2][0], e[3][0]),
                 pack2(e[2][1], e[3][1]), pb0, pb1);
      }
      __syncwarp();
      if (j + 2 < nb) {
        copy_rows(1, block_pos(c0, j + 2), st);
        cp_commit();
      }
    }
    cp_wait(false);
    __syncthreads();  // the next chunk reuses the scores and maxima
  }

  // ---- merge the warps' sub-splits
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    den0 += __shfl_xor_sync(0xffffffffu, den0, off);
    den1 += __shfl_xor_sync(0xffffffffu, den1, off);
  }
  cp_wait(false);   // the self row (warp 7's request)
  __syncthreads();  // every warp is done with the scores and its stages
  if (g == 0) {
    S.wmax[warp][2 * t] = mx0;
    S.wmax[warp][2 * t + 1] = mx1;
    S.wden[warp][2 * t] = den0;
    S.wden[warp][2 * t + 1] = den1;
  }
#pragma unroll
  for (int mt = 0; mt < 16; ++mt) {
    const int ch = 32 * g + 2 * mt;
    S.u.merge[warp][2 * t][ch] = o[mt][0];
    S.u.merge[warp][2 * t + 1][ch] = o[mt][1];
    S.u.merge[warp][2 * t][ch + 1] = o[mt][2];
    S.u.merge[warp][2 * t + 1][ch + 1] = o[mt][3];
  }
  const uint32_t* selfk = reinterpret_cast<const uint32_t*>(S.selfrow[0]);
  const uint32_t* selfv = reinterpret_cast<const uint32_t*>(S.selfrow[1]);
  // Self score of head `warp` in FP32 (the spec's separate self term).
  if (include_self && warp < G) {
    const uint32_t w = selfk[lane], pw = (lane & 7) ? selfk[lane - 1] : 0u;
    const uint16_t* qr = &S.qrow[warp][8 * lane];
    float a = 0.0f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const uint32_t e = lds32(lutK + lut_off(w, pw, n, lane4));
      a = fmaf(__uint_as_float((uint32_t)qr[n] << 16), __uint_as_float(e << 16), a);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    if (lane == 0) S.self_score[warp] = a * (S.selfscale[0] * 0.0625f);
  }
  __syncthreads();
  const int ch = tid;  // one thread per output channel
  float vself = 0.0f, vs_self = 0.0f;
  if (include_self) {
    const int wi = ch >> 3, n = ch & 7;
    const uint32_t w = selfv[wi], pw = (wi & 7) ? selfv[wi - 1] : 0u;
    vself = __uint_as_float(lds32(lutV + lut_off(w, pw, n, lane4)) << 16);
    vs_self = S.selfscale[1];
  }
  const float mean = S.vmean[ch];
  for (int hh = 0; hh < G; ++hh) {
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < KV_WARPS; ++w) M = fmaxf(M, S.wmax[w][hh]);
    float num = 0.0f, den = 0.0f;
#pragma unroll
    for (int w = 0; w < KV_WARPS; ++w) {
      const float f = exp2f((S.wmax[w][hh] - M) * KV_LOG2E);
      num += f * S.u.merge[w][hh][ch];
      den += f * S.wden[w][hh];
    }
    if (include_self) {
      const float score = S.self_score[hh];
      const float nm = fmaxf(M, score);
      const float r = exp2f((M - nm) * KV_LOG2E);
      const float ps = exp2f((score - nm) * KV_LOG2E);
      num = num * r + (ps * vs_self) * vself;
      den = den * r + ps;
      M = nm;
    }
    num += den * mean;
    float* out = p.partials + (((size_t)m * p.n_qh + h * G + hh) * p.max_splits + s) * KV_PART;
    if (ch == 0) {
      out[0] = M;
      out[1] = den;
    }
    out[KV_NUM + ch] = num;
  }

  // ---- the last CTA of this (query row, KV head) combines the splits. Release: every
  // thread's partial stores, then the CTA barrier, then one arrival; the last arriver
  // acquires before it reads the other splits' partials (acq_rel fences, lighter than
  // the sequentially consistent __threadfence).
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  __syncthreads();
  unsigned* arrivals = g_kv_arrivals + (size_t)m * p.n_kvh + h;
  if (tid == 0) S.last = (int)atomicAdd(arrivals, 1u);
  __syncthreads();
  // The last G CTAs to arrive combine one query head each (k = 0: the last one), when
  // the whole grid is one wave of CTAs (they all run at once, so the others' waits for
  // the final arrival end); otherwise the last CTA combines all G heads.
  const int ncomb = p.one_wave ? min(G, n_splits) : 1;  // combiner k takes heads k, k + ncomb, ...
  const int k = n_splits - 1 - S.last;
  if (k >= ncomb) return;
  if (k > 0 && tid == 0) {  // wait (bounded) until every split's partial is in
    const long long t0 = clock64();
    unsigned v;
    do {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(arrivals) : "memory");
      if (clock64() - t0 > KV_WAIT_LIMIT) {
        raise_device_error(p.err, DERR_TIMEOUT);
        break;
      }
    } while (v < (unsigned)n_splits);
  }
  __syncthreads();
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  if (ncomb == 1) {
    if (warp < G) combine_head_warp(p, S.comb[warp], (size_t)m * p.n_qh + h * G + warp, n_splits, lane);
  } else {
    for (int hh = k; hh < G; hh += ncomb) {
      combine_head_cta(p, S.comb[0], &S.u.merge[0][0][0], &S.wden[0][0], (size_t)m * p.n_qh + h * G + hh, n_splits);
      __syncthreads();  // the shared scratch is reused by the next head
    }
  }
  // The combiners count themselves in after the arrivals; the last of them resets the
  // counter for the next launch.
  __syncthreads();
  if (tid == 0 && atomicAdd(arrivals, 1u) == (unsigned)(n_splits + ncomb - 1)) *arrivals = 0u;
}

static int sm_count_kv() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// n_splits < 0: as many splits per (KV head, row) as fill one wave of CTAs.
static int kv_resolved_splits(const KvArgs& a) {
  if (a.n_splits >= 0) return a.n_splits;
  return std::max(1, std::min(KV_MAX_SPLITS, sm_count_kv() / std::max(1, a.n_kvh * a.M)));
}

int kv_max_splits(const KvArgs& a) {
  const int fixed = kv_resolved_splits(a);
  return fixed ? fixed : (kv_row_length(a.length, a.M, a.M - 1) < 4096 ? 31 : 42);
}

int64_t kv_partials_floats(int M, int n_qh, int max_splits) { return (int64_t)M * n_qh * max_splits * KV_PART; }

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
  p.gate = a.gate;
  p.partials = a.partials;
  p.attended = a.attended;
  p.out = a.out;
  p.M = a.M;
  p.n_qh = a.n_qh;
  p.n_kvh = a.n_kvh;
  p.G = a.n_qh / a.n_kvh;
  p.length = a.length;
  p.capacity = a.capacity;
  p.n_splits = kv_resolved_splits(a);
  p.max_splits = kv_max_splits(a);
  p.err = device_error_word();
  p.one_wave = (int64_t)p.max_splits * a.n_kvh * a.M <= sm_count_kv() ? 1 : 0;
  if ((int64_t)a.M * a.n_kvh > KV_MAX_ARRIVALS) return fail(YSKN_EINVAL, "kv4 attention: M * n_kv_heads > 4096");
  static bool attr[64] = {};
  int dev = 0;
  if (int rc = cuda_fail(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(YSKN_EINVAL, "device ordinal out of range");
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kv4_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(KvSmem));
    if (e != cudaSuccess) return cuda_fail(e, "kv4 attributes");
    attr[dev] = true;
  }
  // A programmatic dependent of the previous kernel on the stream: the CTAs may start
  // on SMs that kernel has left and build their codebooks while it finishes.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, a.n_kvh, a.M);
  cfg.blockDim = dim3(KV_THREADS);
  cfg.dynamicSmemBytes = sizeof(KvSmem);
  cfg.stream = st;
  cudaLaunchAttribute attr_pdl[1];
  attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr_pdl;
  cfg.numAttrs = 1;
  return cuda_fail(cudaLaunchKernelEx(&cfg, kv4_attention_kernel, p), "kv4_attention_kernel");
}

}  // namespace yskn
