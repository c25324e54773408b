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
// B200 design: one CTA per row; every thread keeps the best eight of a strided share of
// the row in registers (an insertion into a sorted list), then eight rounds of a
// block-wide maximum over the threads' current heads pick the row's order, the winner
// of each round stepping to its next entry. The row is read once.
#include <cfloat>
#include <climits>

#include "common.cuh"

namespace yskn {

constexpr int HEAD_THREADS = 512;
constexpr int HEAD_K = 8;

struct Cand {
  float v;
  int id;
};

// a comes first in the row's order.
__device__ __forceinline__ bool before(float av, int ai, float bv, int bi) { return av > bv || (av == bv && ai < bi); }

__device__ __forceinline__ Cand shfl_cand(Cand c, int lane_mask) {
  return {__shfl_xor_sync(0xffffffffu, c.v, lane_mask), __shfl_xor_sync(0xffffffffu, c.id, lane_mask)};
}

__device__ Cand block_best(Cand c, Cand* s_warp) {
  for (int off = 16; off > 0; off >>= 1) {
    const Cand o = shfl_cand(c, off);
    if (before(o.v, o.id, c.v, c.id)) c = o;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // s_warp is free (previous round read it)
  if (lane == 0) s_warp[warp] = c;
  __syncthreads();
  c = lane < HEAD_THREADS / 32 ? s_warp[lane] : Cand{-FLT_MAX, INT_MAX};
  for (int off = 16; off > 0; off >>= 1) {
    const Cand o = shfl_cand(c, off);
    if (before(o.v, o.id, c.v, c.id)) c = o;
  }
  return c;  // every lane of every warp holds the block's best
}

__global__ void __launch_bounds__(HEAD_THREADS) head_select_kernel(const float* logits, int n, int32_t* token,
                                                                   float* top_v, int32_t* top_id) {
  __shared__ Cand s_warp[HEAD_THREADS / 32];
  pdl_begin();
  const float* row = logits + (size_t)blockIdx.x * n;
  float v[HEAD_K];
  int id[HEAD_K];
#pragma unroll
  for (int k = 0; k < HEAD_K; ++k) v[k] = -FLT_MAX, id[k] = INT_MAX;
  constexpr int BATCH = 8;  // loads in flight per thread
  for (int i0 = threadIdx.x; i0 < n; i0 += BATCH * HEAD_THREADS) {
    float xs[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int i = i0 + u * HEAD_THREADS;
      xs[u] = i < n ? __ldg(row + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {  // in increasing index order, as one element at a time
      const int i = i0 + u * HEAD_THREADS;
      if (i >= n || !before(xs[u], i, v[HEAD_K - 1], id[HEAD_K - 1])) continue;  // NaN and -inf stop here
      float cv = xs[u];
      int ci = i;
#pragma unroll
      for (int k = 0; k < HEAD_K; ++k) {  // insert, keeping the list in order
        if (before(cv, ci, v[k], id[k])) {
          const float tv = v[k];
          const int ti = id[k];
          v[k] = cv, id[k] = ci;
          cv = tv, ci = ti;
        }
      }
    }
  }
  int head = 0;  // the next entry of this thread's list
  for (int r = 0; r < HEAD_K; ++r) {
    Cand mine{-FLT_MAX, INT_MAX};
#pragma unroll
    for (int k = 0; k < HEAD_K; ++k)
      if (k == head) mine = {v[k], id[k]};
    const Cand best = block_best(mine, s_warp);
    if (head < HEAD_K && mine.id == best.id && mine.v == best.v && best.id != INT_MAX) ++head;
    if (threadIdx.x == 0) {
      if (r == 0 && token) token[blockIdx.x] = best.id;
      if (top_v) top_v[(size_t)blockIdx.x * HEAD_K + r] = best.v;
      if (top_id) top_id[(size_t)blockIdx.x * HEAD_K + r] = best.id;
    }
  }
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_head_select(const float* d_logits, int M, int n, int32_t* d_token,
                                                  float* d_top8_logits, int32_t* d_top8_ids, void* stream) {
  if (!d_logits || M < 1 || n < 1 || (!d_token && !d_top8_logits && !d_top8_ids))
    return fail(YSKN_EINVAL, "head_select: null logits, M < 1, n < 1 or no output");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
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
