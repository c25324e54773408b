// Greedy token selection and the top-8 raw logits of each row of head logits.
//
// Reference: the greedy and top-k kernels after the head (src/misc_kernels.cu:59-88,
// 100-140; src/q35_sample.cu:131-178); docs/spec/06_OUTPUT_HEAD_SAMPLER.md:31-64,232-250.
// The logits are the head operator's restored outputs (yskn_b200_linear on the head
// matrix with the row's inverse RMS: f32(sum) * row quantum * inverse RMS * tau, no
// rotation). Candidates compare by (larger logit, smaller token id), starting from
// (-FLT_MAX, INT_MAX) as the reference does, so a NaN or -inf logit is never chosen;
// the top 8 are the first eight of that order, unfilled places (fewer than eight
// eligible logits) keep (-FLT_MAX, INT_MAX).
//
// B200 design: the candidates are totally ordered, so the first eight of a row are the
// first eight of the union of any partition's first eights. Rows up to HEAD_SPLIT_ROWS per
// call run in two levels inside one launch: HEAD_CHUNKS CTAs per row each take a
// contiguous chunk of the row and write its first eight to scratch; the last CTA of the
// row to arrive (a counter per row, reset by that CTA) merges the chunks' candidates.
// Both levels use the same block selection: every thread keeps the best eight of a
// strided share in registers (an insertion into a sorted list), then eight rounds of a
// block-wide maximum over the threads' current heads pick the order, the winner of each
// round stepping to its next entry. Larger calls take one CTA per row. The row is read
// once either way. The scratch and the counters are static device arrays: calls on one
// device that overlap on the GPU (different streams at the same time) race on them.
#include <cfloat>
#include <climits>

#include "common.cuh"

namespace yskn {

constexpr int HEAD_THREADS = 512;
constexpr int HEAD_K = 8;
constexpr int HEAD_CHUNKS = 148;     // CTAs per row in the two-level selection
constexpr int HEAD_SPLIT_ROWS = 64;  // rows per call handled in two levels
constexpr int HEAD_SPLIT_THREADS = 256;

struct Cand {
  float v;
  int id;
};

// a comes first in the row's order.
__device__ __forceinline__ bool before(float av, int ai, float bv, int bi) { return av > bv || (av == bv && ai < bi); }

__device__ __forceinline__ Cand shfl_cand(Cand c, int lane_mask) {
  return {__shfl_xor_sync(0xffffffffu, c.v, lane_mask), __shfl_xor_sync(0xffffffffu, c.id, lane_mask)};
}

template <int THREADS>
__device__ Cand block_best(Cand c, Cand* s_warp) {
  for (int off = 16; off > 0; off >>= 1) {
    const Cand o = shfl_cand(c, off);
    if (before(o.v, o.id, c.v, c.id)) c = o;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // s_warp is free (previous round read it)
  if (lane == 0) s_warp[warp] = c;
  __syncthreads();
  c = lane < THREADS / 32 ? s_warp[lane] : Cand{-FLT_MAX, INT_MAX};
  for (int off = 16; off > 0; off >>= 1) {
    const Cand o = shfl_cand(c, off);
    if (before(o.v, o.id, c.v, c.id)) c = o;
  }
  return c;  // every lane of every warp holds the block's best
}

// One candidate into a thread's sorted list of eight (the list keeps the first eight seen
// of the order; NaN and -inf never enter).
__device__ __forceinline__ void insert8(float (&v)[HEAD_K], int (&id)[HEAD_K], float cv, int ci) {
  if (!before(cv, ci, v[HEAD_K - 1], id[HEAD_K - 1])) return;
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) {
    if (before(cv, ci, v[k], id[k])) {
      const float tv = v[k];
      const int ti = id[k];
      v[k] = cv, id[k] = ci;
      cv = tv, ci = ti;
    }
  }
}

// The block's first eight from every thread's list, in order: out(r, best) for r = 0..7.
template <int THREADS, typename Out>
__device__ __forceinline__ void block_first8(const float (&v)[HEAD_K], const int (&id)[HEAD_K], Cand* s_warp, Out out) {
  int head = 0;  // the next entry of this thread's list
  for (int r = 0; r < HEAD_K; ++r) {
    Cand mine{-FLT_MAX, INT_MAX};
#pragma unroll
    for (int k = 0; k < HEAD_K; ++k)
      if (k == head) mine = {v[k], id[k]};
    const Cand best = block_best<THREADS>(mine, s_warp);
    if (head < HEAD_K && mine.id == best.id && mine.v == best.v && best.id != INT_MAX) ++head;
    if (threadIdx.x == 0) out(r, best);
  }
}

// Strided share [lo, hi) of a row of logits into a thread's list (8 loads in flight).
template <int THREADS>
__device__ __forceinline__ void scan_share(const float* row, int lo, int hi, float (&v)[HEAD_K], int (&id)[HEAD_K]) {
  constexpr int BATCH = 8;
  for (int i0 = lo + threadIdx.x; i0 < hi; i0 += BATCH * THREADS) {
    float xs[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int i = i0 + u * THREADS;
      xs[u] = i < hi ? __ldg(row + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {  // in increasing index order, as one element at a time
      const int i = i0 + u * THREADS;
      if (i < hi) insert8(v, id, xs[u], i);
    }
  }
}

__global__ void __launch_bounds__(HEAD_THREADS) head_select_kernel(const float* logits, int n, int32_t* token,
                                                                   float* top_v, int32_t* top_id) {
  __shared__ Cand s_warp[HEAD_THREADS / 32];
  pdl_begin();
  float v[HEAD_K];
  int id[HEAD_K];
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) v[k] = -FLT_MAX, id[k] = INT_MAX;
  scan_share<HEAD_THREADS>(logits + (size_t)blockIdx.x * n, 0, n, v, id);
  const size_t r0 = blockIdx.x;
  block_first8<HEAD_THREADS>(v, id, s_warp, [&](int r, Cand best) {
    if (r == 0 && token) token[r0] = best.id;
    if (top_v) top_v[r0 * HEAD_K + r] = best.v;
    if (top_id) top_id[r0 * HEAD_K + r] = best.id;
  });
}

// Two-level scratch: the first eight of every chunk of every row, and one arrival counter
// per row (zero between launches: the merging CTA resets it).
__device__ Cand g_head_part[HEAD_SPLIT_ROWS][HEAD_CHUNKS][HEAD_K];
__device__ unsigned g_head_arrivals[HEAD_SPLIT_ROWS];

// grid (HEAD_CHUNKS, rows): CTA (c, m) selects within chunk c of row m; the row's last
// arriving CTA merges the HEAD_CHUNKS x 8 candidates into the row's first eight.
__global__ void __launch_bounds__(HEAD_SPLIT_THREADS) head_select_split_kernel(const float* logits, int n,
                                                                               int32_t* token, float* top_v,
                                                                               int32_t* top_id) {
  __shared__ Cand s_warp[HEAD_SPLIT_THREADS / 32];
  __shared__ bool s_last;
  pdl_begin();
  const int c = blockIdx.x, m = blockIdx.y;
  const int chunk = (n + HEAD_CHUNKS - 1) / HEAD_CHUNKS;
  const int lo = min(n, c * chunk), hi = min(n, lo + chunk);
  float v[HEAD_K];
  int id[HEAD_K];
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) v[k] = -FLT_MAX, id[k] = INT_MAX;
  scan_share<HEAD_SPLIT_THREADS>(logits + (size_t)m * n, lo, hi, v, id);
  block_first8<HEAD_SPLIT_THREADS>(v, id, s_warp, [&](int r, Cand best) { g_head_part[m][c][r] = best; });
  if (threadIdx.x == 0) {
    __threadfence();  // this chunk's eight before the arrival
    s_last = atomicAdd(&g_head_arrivals[m], 1u) == HEAD_CHUNKS - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // the other chunks' eights after seeing the final count
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) v[k] = -FLT_MAX, id[k] = INT_MAX;
  for (int i = threadIdx.x; i < HEAD_CHUNKS * HEAD_K; i += HEAD_SPLIT_THREADS) {
    const Cand* p = &g_head_part[m][i / HEAD_K][i % HEAD_K];
    insert8(v, id, __ldcg(&p->v), __ldcg(&p->id));  // through L2: other SMs wrote them in this launch
  }
  block_first8<HEAD_SPLIT_THREADS>(v, id, s_warp, [&](int r, Cand best) {
    if (r == 0 && token) token[m] = best.id;
    if (top_v) top_v[(size_t)m * HEAD_K + r] = best.v;
    if (top_id) top_id[(size_t)m * HEAD_K + r] = best.id;
  });
  if (threadIdx.x == 0) g_head_arrivals[m] = 0u;
}

// The first eight of each row from several parts' first eights (the parts partition the
// row's ids; part q's ids are local, its first id is offset q): one thread per row inserts
// every part's candidates. The order is total on the eligible candidates, so the result is
// the first eight of the whole row, as head_select over the whole row gives.
struct MergeOffsets {
  int off[TP_MAX_WORLD];
};

__global__ void head_merge_kernel(const float* part_v, const int32_t* part_id, int64_t part_stride,
                                  const MergeOffsets offs, int n_parts, int M, int32_t* token, float* top_v,
                                  int32_t* top_id) {
  pdl_begin();
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float v[HEAD_K];
  int id[HEAD_K];
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) v[k] = -FLT_MAX, id[k] = INT_MAX;
  for (int q = 0; q < n_parts; ++q)
    for (int k = 0; k < HEAD_K; ++k) {
      const size_t i = (size_t)q * part_stride + (size_t)m * HEAD_K + k;
      const int li = part_id[i];
      if (li == INT_MAX) continue;  // an unfilled place of that part
      insert8(v, id, part_v[i], li + offs.off[q]);
    }
  if (token) token[m] = id[0];
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) {
    if (top_v) top_v[(size_t)m * HEAD_K + k] = v[k];
    if (top_id) top_id[(size_t)m * HEAD_K + k] = id[k];
  }
}

// Greedy token only (no top-8 requested): the same two levels with one candidate per
// thread and one block-wide round per level instead of eight. The first of the order is
// the best of the first candidates of any partition, so the token is the same.
__device__ Cand g_head_best[HEAD_SPLIT_ROWS][HEAD_CHUNKS];
__device__ unsigned g_head_best_arrivals[HEAD_SPLIT_ROWS];

__global__ void __launch_bounds__(HEAD_SPLIT_THREADS) head_greedy_split_kernel(const float* logits, int n,
                                                                                int32_t* token) {
  __shared__ Cand s_warp[HEAD_SPLIT_THREADS / 32];
  __shared__ bool s_last;
  pdl_begin();
  const int c = blockIdx.x, m = blockIdx.y;
  const int chunk = (n + HEAD_CHUNKS - 1) / HEAD_CHUNKS;
  const int lo = min(n, c * chunk), hi = min(n, lo + chunk);
  const float* row = logits + (size_t)m * n;
  Cand mine{-FLT_MAX, INT_MAX};
  constexpr int BATCH = 8;
  for (int i0 = lo + threadIdx.x; i0 < hi; i0 += BATCH * HEAD_SPLIT_THREADS) {
    float xs[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int i = i0 + u * HEAD_SPLIT_THREADS;
      xs[u] = i < hi ? __ldg(row + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {  // in increasing index order, as one element at a time
      const int i = i0 + u * HEAD_SPLIT_THREADS;
      if (i < hi && before(xs[u], i, mine.v, mine.id)) mine = {xs[u], i};
    }
  }
  const Cand best = block_best<HEAD_SPLIT_THREADS>(mine, s_warp);
  if (threadIdx.x == 0) {
    g_head_best[m][c] = best;
    __threadfence();  // this chunk's best before the arrival
    s_last = atomicAdd(&g_head_best_arrivals[m], 1u) == HEAD_CHUNKS - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // the other chunks' bests after seeing the final count
  Cand cand{-FLT_MAX, INT_MAX};
  for (int i = threadIdx.x; i < HEAD_CHUNKS; i += HEAD_SPLIT_THREADS) {
    const Cand* q = &g_head_best[m][i];
    const Cand o{__ldcg(&q->v), __ldcg(&q->id)};  // through L2: other SMs wrote them in this launch
    if (before(o.v, o.id, cand.v, cand.id)) cand = o;
  }
  const Cand total = block_best<HEAD_SPLIT_THREADS>(cand, s_warp);
  if (threadIdx.x == 0) {
    token[m] = total.id;
    g_head_best_arrivals[m] = 0u;
  }
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_head_merge(const float* d_part_logits, const int32_t* d_part_ids,
                                                 int64_t part_stride, const int32_t* h_id_offsets, int n_parts, int M,
                                                 int32_t* d_token, float* d_top8_logits, int32_t* d_top8_ids,
                                                 void* stream) {
  if (!d_part_logits || !d_part_ids || !h_id_offsets || n_parts < 1 || n_parts > TP_MAX_WORLD || M < 1 ||
      part_stride < (int64_t)M * HEAD_K || (!d_token && !d_top8_logits && !d_top8_ids))
    return fail(YSKN_EINVAL, "head_merge: null argument, parts outside 1..8, M < 1, stride below 8 M or no output");
  MergeOffsets offs{};
  for (int q = 0; q < n_parts; ++q) {
    if (h_id_offsets[q] < 0) return fail(YSKN_EINVAL, "head_merge: negative id offset");
    offs.off[q] = h_id_offsets[q];
  }
  return cuda_fail(launch_pdl(head_merge_kernel, (M + 31) / 32, 32, 0, reinterpret_cast<cudaStream_t>(stream),
                              d_part_logits, d_part_ids, part_stride, offs, n_parts, M, d_token, d_top8_logits,
                              d_top8_ids),
                   "head_merge_kernel");
}

extern "C" YSKN_B200_API int yskn_b200_head_select(const float* d_logits, int M, int n, int32_t* d_token,
                                                  float* d_top8_logits, int32_t* d_top8_ids, void* stream) {
  if (!d_logits || M < 1 || n < 1 || (!d_token && !d_top8_logits && !d_top8_ids))
    return fail(YSKN_EINVAL, "head_select: null logits, M < 1, n < 1 or no output");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (M <= HEAD_SPLIT_ROWS && n >= 4 * HEAD_CHUNKS && !d_top8_logits && !d_top8_ids)
    return cuda_fail(launch_pdl(head_greedy_split_kernel, dim3(HEAD_CHUNKS, M), HEAD_SPLIT_THREADS, 0, st, d_logits,
                                n, d_token),
                     "head_greedy_split_kernel");
  if (M <= HEAD_SPLIT_ROWS && n >= 4 * HEAD_CHUNKS)
    return cuda_fail(launch_pdl(head_select_split_kernel, dim3(HEAD_CHUNKS, M), HEAD_SPLIT_THREADS, 0, st, d_logits, n,
                                d_token, d_top8_logits, d_top8_ids),
                     "head_select_split_kernel");
  for (int m0 = 0; m0 < M; m0 += 65535) {
    const int rows = M - m0 < 65535 ? M - m0 : 65535;
    if (cudaError_t e = launch_pdl(head_select_kernel, rows, HEAD_THREADS, 0, st, d_logits + (size_t)m0 * n, n,
                                   d_token ? d_token + m0 : nullptr,
                                   d_top8_logits ? d_top8_logits + (size_t)m0 * HEAD_K : nullptr,
                                   d_top8_ids ? d_top8_ids + (size_t)m0 * HEAD_K : nullptr))
      return cuda_fail(e, "head_select_kernel");
  }
  return YSKN_OK;
}
