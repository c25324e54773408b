// Load-time layout transforms of the code stream.
//
//  * pack: the file's row or warp layout (docs/FORMAT.md:139-151) -> the B200
//    streaming layout. The streaming layout IS the format's warp layout, taken
//    with the physical row count rounded up to a multiple of 32 (padding rows are
//    zero codes whose sums are never written out). Every 16-byte chunk of 32
//    sequences is one fully coalesced 512-byte segment, and the two sequences of a
//    512-column group for one 32-row group are two contiguous bits*512-byte runs,
//    which is exactly what the GEMV streams with 16-byte loads (gemv.cu). So the
//    warp-layout files of the released models need no reorder beyond a copy.
//  * repack_frag: the reference's own load-time permutation into its mma.sync
//    "frag" order (src/repack.cu:10-18), kept bit-identical for the C ABI, written
//    with 16-byte moves (one thread per chunk of 4 words) instead of one per word.
#include "common.cuh"

namespace yskn {

__global__ void __launch_bounds__(256) pack_kernel(const uint4* __restrict__ src, int layout, int phys, int phys_pad,
                                                   int seqs, int bits, uint4* __restrict__ dst, int64_t total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31);
  const int64_t t = i >> 5;
  const int c = (int)(t % bits);
  const int64_t rest = t / bits;
  const int groups = phys_pad >> 5;
  const int rg = (int)(rest % groups);
  const int64_t seq = rest / groups;
  const int row = rg * 32 + lane;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (row < phys) {
    int64_t s;
    if (layout == YSKN_LAYOUT_WARP) {
      const int64_t q = seq * phys + row;
      s = ((q >> 5) * bits + c) * 32 + (q & 31);
    } else {
      s = ((int64_t)row * seqs + seq) * bits + c;
    }
    v = __ldg(src + s);
  }
  dst[i] = v;
}

int launch_pack(const uint32_t* words, int layout, int phys, int cols, int bits, uint4* out, cudaStream_t st) {
  const int phys_pad = (int)ceil_div(phys, 32) * 32;
  const int seqs = cols / 256;
  const int64_t total = (int64_t)seqs * (phys_pad / 32) * bits * 32;
  if (total == 0) return YSKN_OK;
  pack_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(words), layout, phys,
                                                              phys_pad, seqs, bits, out, total);
  return cuda_fail(cudaGetLastError(), "pack_kernel");
}

// One thread per 16-byte chunk of the warp-layout source: chunk k belongs to
// sequence-group tile = k / (32*wps/4), chunk c, lane; destination order as
// src/repack.cu:15-16 defines it.
__global__ void __launch_bounds__(256) repack_frag_kernel(const uint4* __restrict__ w, uint4* __restrict__ f, int rows,
                                                          int seqs, int wps, int64_t total) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= total) return;
  const int cpw = wps >> 2;
  const int lane = (int)(k & 31);
  const int64_t t = k >> 5;
  const int c = (int)(t % cpw);
  const int64_t tile = t / cpw;
  const int64_t q = tile * 32 + lane;
  const int64_t seq = q / rows;
  const int row = (int)(q % rows);
  const int64_t wt = row >> 6, j = (row & 63) >> 3, r = row & 7;
  const int64_t d = (((wt * seqs + seq) * 8 + j) * cpw + c) * 8 + r;
  f[d] = __ldg(w + k);
}

int launch_repack_frag(const uint32_t* w, uint32_t* f, int rows, int seqs, int wps, cudaStream_t st) {
  const int64_t total = (int64_t)rows * seqs * (wps / 4);
  if (total == 0) return YSKN_OK;
  repack_frag_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(w),
                                                                     reinterpret_cast<uint4*>(f), rows, seqs, wps,
                                                                     total);
  return cuda_fail(cudaGetLastError(), "repack_frag_kernel");
}

}  // namespace yskn
