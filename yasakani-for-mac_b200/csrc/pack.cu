// Load-time layout transforms of the code stream.
//
//  * pack: the file's row or warp layout (docs/FORMAT.md:139-151) -> the B200
//    streaming layout the decode GEMV reads (gemv.cu). Physical rows are padded
//    to a multiple of 8 with zero codes (their sums are never written). Tiles of
//    8 rows x one 256-column sequence are stored row-block-major, sequence-minor,
//    so the two tiles of a 512-column group are adjacent. Inside a tile, lane
//    (n = row%8, q = quarter) owns words q*bits .. q*bits+bits-1 of row n's
//    sequence (its 32 trellis steps), stored in chunks of U words
//    (U = 4 for bits 4/8, 2 for bits 6, 1 otherwise) interleaved across the 32
//    lanes: chunk j of lane l at tile + (j*32 + l)*U. A warp's load of one chunk
//    is one contiguous 128*U-byte segment. At bits = 8 each byte is stored with its
//    bits moved (stream8_store, common.cuh) for the GEMV's table addressing.
//  * repack_frag: the reference's own load-time permutation into its mma.sync
//    "frag" order (src/repack.cu:10-18), kept bit-identical for the C ABI, written
//    with 16-byte moves (one thread per chunk of 4 words) instead of one per word.
#include "common.cuh"

namespace yskn {

// The packed matrix may be a shard of the source tensor: physical rows
// [row0, row0 + phys) and sequences [seq0, seq0 + seqs) of a source with src_phys
// rows and src_seqs sequences (the addressing of docs/FORMAT.md:139-151 uses the
// source's geometry).
__global__ void __launch_bounds__(256) pack_kernel(const uint32_t* __restrict__ src, int layout, int src_phys,
                                                   int src_seqs, int row0, int seq0, int phys, int seqs, int bits,
                                                   int U, uint32_t* __restrict__ dst, int64_t total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (row block, sequence, lane)
  if (i >= total) return;
  const int lane = (int)(i & 31);
  const int64_t tile = i >> 5;
  const int64_t seq = tile % seqs, rb = tile / seqs;
  const int n = lane >> 2, q = lane & 3;
  const int64_t row = rb * 8 + n;
  uint32_t* t = dst + tile * (int64_t)bits * 32;
  for (int j = 0; j < bits; ++j) {
    uint32_t v = 0;
    if (row < phys) {
      const int64_t w = (int64_t)q * bits + j;  // word of the sequence
      const int64_t sr = row0 + row, ss = seq0 + seq;
      int64_t s;
      if (layout == YSKN_LAYOUT_WARP) {
        const int64_t qq = ss * src_phys + sr;
        s = (((qq >> 5) * bits + (w >> 2)) * 32 + (qq & 31)) * 4 + (w & 3);
      } else {
        s = (sr * src_seqs + ss) * (4 * (int64_t)bits) + w;
      }
      v = __ldg(src + s);
      if (bits == 8) v = stream8_store(v);  // bit order inside each byte (common.cuh)
    }
    t[((j / U) * 32 + lane) * U + (j % U)] = v;
  }
}

int launch_pack_range(const uint32_t* words, int layout, int src_phys, int src_cols, int row0, int col0, int phys,
                      int cols, int bits, uint32_t* out, cudaStream_t st) {
  const int64_t pad8 = ceil_div(phys, 8) * 8;
  const int seqs = cols / 256;
  const int U = bits % 4 == 0 ? 4 : (bits % 2 == 0 ? 2 : 1);
  const int64_t total = pad8 / 8 * seqs * 32;
  if (total == 0) return YSKN_OK;
  pack_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(words, layout, src_phys, src_cols / 256, row0,
                                                              col0 / 256, phys, seqs, bits, U, out, total);
  return cuda_fail(cudaGetLastError(), "pack_kernel");
}

int launch_pack(const uint32_t* words, int layout, int phys, int cols, int bits, uint32_t* out, cudaStream_t st) {
  return launch_pack_range(words, layout, phys, cols, 0, 0, phys, cols, bits, out, st);
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
