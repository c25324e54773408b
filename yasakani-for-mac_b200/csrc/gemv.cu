// Weighted integer sums for skinny inputs (M <= 16 per pass): the decode GEMV.
//
// Contract (crates/yskn-ref/src/compressed_linear.rs:205-252; docs/spec/
// 02_COMPRESSED_LINEAR.md:160-196):
//   ws[m][n] = sum_g A[m][g] * sum_{j<512} lut8[state(n, 512g+j)] * act[m][512g+j]
// with an i32 dot per 512-column group and i64 across groups. Integer adds are
// associative, so any split of the groups across warps gives identical bits.
//
// B200 design. The hot loop is an HBM stream of the code words. The streaming
// layout (pack.cu) puts the 32 rows of a row group side by side in 16-byte
// chunks, so lane l of a warp owns row 32*rg + l: it loads its sequence's
// 4*bits words with bits 16-byte loads (each warp-wide load is one contiguous
// 512-byte segment), rebuilds its 128 trellis states with constant shifts,
// looks the int8 pairs up in a shared-memory copy of the table and feeds dp4a.
// No lane ever needs another lane's data: there are no shuffles and no partial
// sums to reduce inside a warp. The work unit is (row group, 512-column group);
// each warp takes a contiguous run of units in row-group-major order, keeps i64
// sums in registers while the row group stays the same, and adds them to the
// output with one 64-bit atomic per row when it leaves the row group (the output
// is zeroed first). The grid is sized to the SM count times the resident blocks.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace yskn {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_MAX_SEG = 3;

struct GemvSeg {
  const uint4* codes;
  const uint16_t* lut;
  int64_t* out;
  int64_t unit_begin;  // first unit of this segment
  int rowgroups;       // phys_pad / 32
  int out_rows;        // rows written (<= phys)
  int out_ld;          // leading dimension of out (elements per activation row)
};

struct GemvParams {
  GemvSeg seg[GEMV_MAX_SEG];
  int n_seg;
  int G;  // 512-column groups per row (cols / 512)
  int Kc;
  const int8_t* act;
  const int32_t* scales;
  int mv;  // valid activation rows in this pass (<= MT)
  int64_t total_units;
  int checked;  // 1: one warp owns whole rows and checks every i64 add (cols >= 262144)
  unsigned* err;
};

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// State of step j (docs/FORMAT.md:121-128): the 12 code bits ending at bits*(j+1),
// zeros before the start of the sequence. j is a compile-time constant after unrolling.
template <int BITS>
__device__ __forceinline__ uint32_t state_at(const uint32_t (&w)[4 * BITS], int j) {
  const int end = BITS * (j + 1);
  if (end < 12) return (w[0] << (12 - end)) & 0xfffu;
  const int start = end - 12, wi = start >> 5, sh = start & 31;
  if (sh + 12 <= 32) return (w[wi] >> sh) & 0xfffu;
  return __funnelshift_r(w[wi], w[wi + 1], sh) & 0xfffu;
}

template <int BITS, int MT>
__device__ __forceinline__ void sequence_dot(const uint32_t (&w)[4 * BITS], const uint16_t* __restrict__ lut,
                                             const int8_t* __restrict__ act, int Kc, int mv, int (&dot)[MT]) {
#pragma unroll
  for (int qb = 0; qb < 16; ++qb) {
    uint32_t wq[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int j0 = qb * 8 + 2 * t;
      const uint32_t lo = lut[state_at<BITS>(w, j0)];
      const uint32_t hi = lut[state_at<BITS>(w, j0 + 1)];
      wq[t] = __byte_perm(lo, hi, 0x5410);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const int mm = m < mv ? m : mv - 1;
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(act + (int64_t)mm * Kc) + qb);
      dot[m] = __dp4a((int)wq[0], (int)a.x, dot[m]);
      dot[m] = __dp4a((int)wq[1], (int)a.y, dot[m]);
      dot[m] = __dp4a((int)wq[2], (int)a.z, dot[m]);
      dot[m] = __dp4a((int)wq[3], (int)a.w, dot[m]);
    }
  }
}

template <int BITS, int MT>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_kernel(const __grid_constant__ GemvParams p) {
  __shared__ uint16_t s_lut[GEMV_MAX_SEG][4096];
  for (int s = 0; s < p.n_seg; ++s)
    for (int i = threadIdx.x; i < 2048; i += blockDim.x)
      reinterpret_cast<uint32_t*>(s_lut[s])[i] = __ldg(reinterpret_cast<const uint32_t*>(p.seg[s].lut) + i);
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * GEMV_WARPS;
  (void)nw;
  int64_t u, u_end;
  if (p.checked) {
    // One warp per row group, groups in ascending order: every i64 add is
    // checked in the reference's order (compressed_linear.rs:229-248).
    u = gw * p.G;
    u_end = std::min<int64_t>(u + p.G, p.total_units);
  } else {
    u = gw * p.total_units / nw;
    u_end = (gw + 1) * p.total_units / nw;
  }
  if (u >= u_end) return;

  int seg = 0;
  while (seg + 1 < p.n_seg && u >= p.seg[seg + 1].unit_begin) ++seg;
  int64_t local = u - p.seg[seg].unit_begin;
  int rg = (int)(local / p.G), g = (int)(local % p.G);
  long long acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0;
  bool overflow = false;

  for (;;) {
    const GemvSeg& S = p.seg[seg];
    int dot[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) dot[m] = 0;
    uint32_t w0[4 * BITS], w1[4 * BITS];
    const uint4* c0 = S.codes + ((int64_t)(2 * g) * S.rowgroups + rg) * (BITS * 32) + lane;
    const uint4* c1 = S.codes + ((int64_t)(2 * g + 1) * S.rowgroups + rg) * (BITS * 32) + lane;
#pragma unroll
    for (int c = 0; c < BITS; ++c) {
      const uint4 v = ld_stream(c0 + c * 32);
      w0[4 * c] = v.x; w0[4 * c + 1] = v.y; w0[4 * c + 2] = v.z; w0[4 * c + 3] = v.w;
    }
#pragma unroll
    for (int c = 0; c < BITS; ++c) {
      const uint4 v = ld_stream(c1 + c * 32);
      w1[4 * c] = v.x; w1[4 * c + 1] = v.y; w1[4 * c + 2] = v.z; w1[4 * c + 3] = v.w;
    }
    const int8_t* a0 = p.act + (int64_t)g * 512;
    sequence_dot<BITS, MT>(w0, s_lut[seg], a0, p.Kc, p.mv, dot);
    sequence_dot<BITS, MT>(w1, s_lut[seg], a0 + 256, p.Kc, p.mv, dot);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const int mm = m < p.mv ? m : p.mv - 1;
      const long long t = (long long)__ldg(p.scales + (int64_t)mm * p.G + g) * (long long)dot[m];
      const long long r = (long long)((unsigned long long)acc[m] + (unsigned long long)t);
      overflow |= ((acc[m] ^ r) & (t ^ r)) < 0;
      acc[m] = r;
    }

    ++u;
    const bool done = u >= u_end;
    int nseg = seg, nrg = rg, ng = g + 1;
    if (ng == p.G) {
      ng = 0;
      ++nrg;
      if (nrg == S.rowgroups) {
        nrg = 0;
        ++nseg;
      }
    }
    if (done || nrg != rg || nseg != seg) {
      const int row = rg * 32 + lane;
      if (row < S.out_rows) {
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (m < p.mv)
            atomicAdd(reinterpret_cast<unsigned long long*>(S.out + (int64_t)m * S.out_ld + row),
                      (unsigned long long)acc[m]);
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] = 0;
    }
    if (done) break;
    seg = nseg;
    rg = nrg;
    g = ng;
  }
  if (p.checked && __any_sync(0xffffffffu, overflow) && lane == 0) raise_device_error(p.err, DERR_OVERFLOW);
}

template <int BITS, int MT>
static int launch_one(const GemvParams& p, cudaStream_t st) {
  static int grid_per_sm = 0;
  static int sm_count = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&grid_per_sm, gemv_kernel<BITS, MT>, GEMV_WARPS * 32, 0);
    if (grid_per_sm < 1) grid_per_sm = 1;
  });
  int64_t grid;
  if (p.checked) {
    // One warp per whole row group: ranges are multiples of G units.
    grid = ceil_div(p.total_units / p.G, GEMV_WARPS);
  } else {
    grid = std::min<int64_t>((int64_t)sm_count * grid_per_sm, ceil_div(p.total_units, GEMV_WARPS));
  }
  if (grid < 1) grid = 1;
  gemv_kernel<BITS, MT><<<(unsigned)grid, GEMV_WARPS * 32, 0, st>>>(p);
  return cuda_fail(cudaGetLastError(), "gemv_kernel");
}

template <int BITS>
static int launch_bits(const GemvParams& p, int mt, cudaStream_t st) {
  switch (mt) {
    case 1: return launch_one<BITS, 1>(p, st);
    case 2: return launch_one<BITS, 2>(p, st);
    case 4: return launch_one<BITS, 4>(p, st);
    case 8: return launch_one<BITS, 8>(p, st);
    default: return launch_one<BITS, 16>(p, st);
  }
}

int launch_gemv(const MatrixDev* mats, int n_mats, const int8_t* act, const int32_t* scales, int M, int64_t* const* out,
                const int* out_rows, cudaStream_t st) {
  const int Kc = mats[0].cols, G = Kc / 512, bits = mats[0].bits;
  GemvParams p{};
  p.n_seg = n_mats;
  p.G = G;
  p.Kc = Kc;
  p.checked = G >= 512 ? 1 : 0;
  p.err = device_error_word();
  int64_t units = 0;
  for (int i = 0; i < n_mats; ++i) {
    p.seg[i].codes = mats[i].codes;
    p.seg[i].lut = mats[i].lut8;
    p.seg[i].unit_begin = units;
    p.seg[i].rowgroups = mats[i].phys_pad / 32;
    p.seg[i].out_rows = out_rows[i];
    p.seg[i].out_ld = out_rows[i];
    units += (int64_t)p.seg[i].rowgroups * G;
  }
  p.total_units = units;
  for (int i = 0; i < n_mats; ++i) {
    cudaError_t e = cudaMemsetAsync(out[i], 0, sizeof(int64_t) * (size_t)M * out_rows[i], st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  }
  for (int m0 = 0; m0 < M; m0 += 16) {
    const int mv = std::min(16, M - m0);
    const int mt = mv == 1 ? 1 : mv == 2 ? 2 : mv <= 4 ? 4 : mv <= 8 ? 8 : 16;
    p.act = act + (int64_t)m0 * Kc;
    p.scales = scales + (int64_t)m0 * G;
    p.mv = mv;
    for (int i = 0; i < n_mats; ++i) p.seg[i].out = out[i] + (int64_t)m0 * out_rows[i];
    int rc;
    switch (bits) {
      case 4: rc = launch_bits<4>(p, mt, st); break;
      case 5: rc = launch_bits<5>(p, mt, st); break;
      case 6: rc = launch_bits<6>(p, mt, st); break;
      case 7: rc = launch_bits<7>(p, mt, st); break;
      default: rc = launch_bits<8>(p, mt, st); break;
    }
    if (rc) return rc;
  }
  return YSKN_OK;
}

}  // namespace yskn
