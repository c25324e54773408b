// Weighted integer sums for many activation rows (prefill / long verify): the
// tcgen05 GEMM.
//
// Same contract as gemv.cu (crates/yskn-ref/src/compressed_linear.rs:205-252):
//   ws[m][n] = sum_g A[m][g] * sum_{k in group g} W[n][k] * act[m][k]
// computed exactly: int8 x int8 -> int32 per 512-column group on the tensor
// cores, i64 across groups.
//
// B200 design (replaces the reference's mt_predecode2_kernel + mt_gemm6_kernel,
// src/q35_g6.cu:35-277, and pfa_kernel, src/pfa.cu:85-321):
//  1. trellis_predecode_kernel: the codes of the matrix -> dense int8 W [N][Kc] (K-major)
//     in a workspace, once per call (decoding inside the MMA loop would cost
//     shared-memory bandwidth the tensor cores need; this is the reference's own
//     choice for >= 256 rows, q35_g6.cu:35-69).
//  2. trellis_mma_kernel: persistent, one CTA per SM looping over 128 x 128 output tiles
//     (128 activation rows x 128 weight rows) in a grouped raster. Warp 0 streams
//     128-byte K chunks of both operands with TMA (128B swizzle, 5-stage mbarrier
//     ring, counted across tiles); one thread of warp 1 issues
//     tcgen05.mma.cta_group::1.kind::i8 (M=128, N=128, K=32) into TMEM; warps
//     2..9 drain each 512-column group's int32 tile with tcgen05.ld, multiply it
//     by the activation row's integer group scale and accumulate i64 in registers,
//     then write the tile through a shared staging buffer. TMEM holds four group
//     accumulators (all 512 columns), so the MMAs run up to four groups ahead of
//     the drain, also across a tile's output write. Activation rows are the MMA's M
//     dimension, so each epilogue thread owns one activation row and one scale per
//     group.
//  Every mbarrier wait is bounded: on timeout the CTA raises YSKN_ETIMEDOUT in
//  the device error word, stops issuing work, waits (bounded) for its own copies
//  and frees its TMEM before returning.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "async.cuh"
#include "common.cuh"

namespace yskn {

constexpr int GM_BM = 128;    // activation rows per tile (MMA M)
constexpr int GM_BN = 128;    // weight rows per tile (MMA N)
constexpr int GM_BK = 128;    // bytes of K per stage (one 128-byte swizzle row)
constexpr int GM_STAGES = 5;
constexpr int GM_THREADS = 320;  // 10 warps
constexpr int GM_STAGE_BYTES = (GM_BM + GM_BN) * GM_BK;
constexpr int GM_TMEM_BUFS = 4;  // group accumulators of 128 columns: the whole TMEM
constexpr int GM_OUT_LD = 32 + 2;  // int64 per staged output row (16 bytes of padding)
constexpr int GM_OUT_BYTES = GM_BM * GM_OUT_LD * 8;
constexpr int GM_SMEM = GM_STAGES * GM_STAGE_BYTES + GM_OUT_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr long long GM_WAIT_LIMIT = 4000000000ll;  // clock cycles (~2 s) before a wait gives up

// ------------------------------------------------------------------ PTX helpers
// (mbarrier basics in async.cuh)
// Bounded wait; false if this CTA aborted (timeout here or elsewhere in the CTA).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > GM_WAIT_LIMIT) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in 128-byte-swizzled rows: 8-row atoms of 1024 bytes (SBO), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3fff) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::i8: D s32, A s8, B s8, both K-major, N = 128, M = 128.
constexpr uint32_t GM_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(GM_BN >> 3) << 17) |
                              ((uint32_t)(GM_BM >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(GM_IDESC), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// -------------------------------------------------------------- predecode
// Codes (streaming layout, pack.cu) -> dense int8 W [phys_pad8][Kc]. One warp per
// tile (8 rows x 256 columns); lane (n, q) decodes its 32 steps into 64 bytes of
// row n. The table is read straight from L1 (4096 x 2 bytes).
template <int BITS>
__global__ void __launch_bounds__(256) trellis_predecode_kernel(const uint32_t* __restrict__ codes,
                                                        const uint16_t* __restrict__ lut, int row_blocks, int S,
                                                        int Kc, int8_t* __restrict__ W) {
  __shared__ uint16_t s_lut[4096];
  for (int i = threadIdx.x; i < 2048; i += blockDim.x)
    reinterpret_cast<uint32_t*>(s_lut)[i] = __ldg(reinterpret_cast<const uint32_t*>(lut) + i);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t tiles = (int64_t)row_blocks * S;
  constexpr int U = (BITS % 4 == 0) ? 4 : (BITS % 2 == 0 ? 2 : 1);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < tiles;
       t += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int rb = (int)(t / S), s = (int)(t % S);
    const uint32_t* tile = codes + t * (BITS * 32);
    uint32_t w[BITS];
#pragma unroll
    for (int j = 0; j < BITS; ++j) {
      w[j] = __ldg(tile + ((j / U) * 32 + lane) * U + (j % U));
      if constexpr (BITS == 8) w[j] = stream8_load(w[j]);  // the file's bit order (common.cuh)
    }
    uint32_t carry = __shfl_up_sync(0xffffffffu, w[BITS - 1], 1);
    if ((lane & 3) == 0) carry = 0u;
    uint32_t out[16];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      // 12-bit state ending at bit BITS*(i+1) of the quarter; V = [carry | w].
      const int P = 32 + BITS * (i + 1) - 12;
      const int wi = P >> 5, sh = P & 31;
      const uint32_t lo = wi == 0 ? carry : w[wi - 1];
      const uint32_t hi = wi >= BITS ? 0u : w[wi];
      const uint32_t x = sh == 0 ? lo : (sh + 12 <= 32 ? lo >> sh : __funnelshift_r(lo, hi, sh));
      const uint32_t e = s_lut[x & 0xfffu];
      if (i & 1) out[i >> 1] |= e << 16;
      else out[i >> 1] = e;
    }
    int8_t* dst = W + (int64_t)(rb * 8 + (lane >> 2)) * Kc + s * 256 + (lane & 3) * 64;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      reinterpret_cast<uint4*>(dst)[k] = make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
  }
}

// ------------------------------------------------------------------- GEMM
struct GemmParams {
  const int32_t* scales;  // [M][G]
  int64_t* out;           // [M][out_ld] int64
  int M, G, out_rows, out_ld;
  int m_tiles, n_tiles;
  unsigned* err;
};

constexpr int GM_GROUP = 16;  // activation tiles per raster group

__global__ void __launch_bounds__(GM_THREADS, 1)
    trellis_mma_kernel(const __grid_constant__ CUtensorMap map_act, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                 // [stage][128 rows][128 B]
  uint8_t* sB = smem + GM_STAGES * GM_BM * GM_BK;     // [stage][128 rows][128 B]
  long long* stage_out = reinterpret_cast<long long*>(smem + GM_STAGES * GM_STAGE_BYTES);  // [128][GM_OUT_LD]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GM_STAGES * GM_STAGE_BYTES + GM_OUT_BYTES);
  uint64_t* full = bars;                           // [GM_STAGES] TMA landed
  uint64_t* empty = bars + GM_STAGES;              // [GM_STAGES] MMAs done reading
  uint64_t* tmem_full = bars + 2 * GM_STAGES;      // [GM_TMEM_BUFS] group accumulator ready
  uint64_t* tmem_empty = tmem_full + GM_TMEM_BUFS; // [GM_TMEM_BUFS] group accumulator drained
  uint64_t* drained = tmem_empty + GM_TMEM_BUFS;   // all MMAs of this CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_total = p.m_tiles * p.n_tiles;
  // Grouped tile order: consecutive tiles sweep GM_GROUP activation tiles for each
  // weight tile, so the tiles in flight across the SMs (~16 MB of operands) stay in
  // the 126 MB L2 and each weight tile is read from HBM about once per GM_GROUP
  // activation tiles. CTA c takes tiles c, c + grid, c + 2*grid, ...
  auto coords = [&](int t, int& m0, int& n0) {
    const int per_group = GM_GROUP * p.n_tiles;
    const int first_m = (t / per_group) * GM_GROUP;
    const int gsize = min(p.m_tiles - first_m, GM_GROUP);
    m0 = (first_m + (t % per_group) % gsize) * GM_BM;
    n0 = ((t % per_group) / gsize) * GM_BN;
  };
  const int G = p.G, KB = G * 4;  // 128-byte chunks per tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < GM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < GM_TMEM_BUFS; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);
    }
    mbar_init(drained, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(GM_TMEM_BUFS * GM_BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer: K chunks of every tile of this CTA through the stage ring
    if (lane == 0) {
      int c = 0;  // chunks issued by this CTA
      for (int t = blockIdx.x; t < n_total && !*abort_flag; t += gridDim.x) {
        int m0, n0;
        coords(t, m0, n0);
        for (int kb = 0; kb < KB; ++kb, ++c) {
          const int s = c % GM_STAGES, u = c / GM_STAGES;
          if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1, abort_flag)) break;
          mbar_expect_tx(&full[s], GM_STAGE_BYTES);
          tma_load_2d(sA + s * GM_BM * GM_BK, &map_act, &full[s], kb * GM_BK, m0);
          tma_load_2d(sB + s * GM_BN * GM_BK, &map_w, &full[s], kb * GM_BK, n0);
        }
      }
      if (*abort_flag) {
        // Let the copies this thread started land before the CTA leaves.
        for (int k = std::max(0, c - GM_STAGES); k < c; ++k) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[k % GM_STAGES], (k / GM_STAGES) & 1) && clock64() - t0 < GM_WAIT_LIMIT) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (one thread): groups of every tile into the TMEM ring
    if (lane == 0) {
      int c = 0, q = 0;  // chunks consumed, groups issued
      bool ok = true;
      for (int t = blockIdx.x; t < n_total && ok; t += gridDim.x) {
        for (int g = 0; g < G && ok; ++g, ++q) {
          const int b = q % GM_TMEM_BUFS, v = q / GM_TMEM_BUFS;
          if (v > 0 && !mbar_wait(&tmem_empty[b], (v - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + b * GM_BN;
          for (int cc = 0; cc < 4; ++cc, ++c) {
            const int s = c % GM_STAGES;
            if (!mbar_wait(&full[s], (c / GM_STAGES) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + s * GM_BM * GM_BK), b0 = smem_u32(sB + s * GM_BN * GM_BK);
#pragma unroll
            for (int k = 0; k < GM_BK / 32; ++k)
              umma_i8(d, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), (cc > 0 || k > 0) ? 1u : 0u);
            umma_commit(&empty[s]);  // frees the stage when these MMAs have read it
          }
          if (ok) umma_commit(&tmem_full[b]);
        }
      }
      // Every MMA this thread issued has completed before TMEM can be freed.
      umma_commit(drained);
      const long long t0 = clock64();
      while (!mbar_try_wait(drained, 0) && clock64() - t0 < GM_WAIT_LIMIT) {
      }
    }
  } else {
    // ---- Epilogue: warps 2..9. TMEM lanes 32*(warp%4).. ; column half (warp-2)/4.
    // Every epilogue warp runs the same tiles and the same named barriers whether or
    // not the CTA aborted (then it skips the waits and the stores).
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    int q = 0;  // groups drained
    for (int t = blockIdx.x; t < n_total; t += gridDim.x) {
      int m0, n0;
      coords(t, m0, n0);
      const int row = m0 + quarter * 32 + lane;  // activation row of this thread
      const int32_t* sc = p.scales + (size_t)min(row, p.M - 1) * G;
      long long acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0;
      int s_next = __ldg(sc);  // the row's scale of the next group, loaded one group ahead
      for (int g = 0; g < G; ++g, ++q) {
        const int b = q % GM_TMEM_BUFS, v = q / GM_TMEM_BUFS;
        const long long s = s_next;
        if (g + 1 < G) s_next = __ldg(sc + g + 1);
        if (!mbar_wait(&tmem_full[b], v & 1, abort_flag)) continue;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + b * GM_BN + half * 64;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t r[32];
          tmem_ld32(taddr + h * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[h * 32 + j] += s * (long long)(int)r[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[b]);
      }
      // Output tile through the staging buffer: one 32-column quarter at a time (a small
      // buffer leaves shared memory to the operand ring), rows padded by 16 bytes; then
      // the warps write whole 256-byte row segments (direct per-row stores from
      // registers measured 24 % slower). The MMA issuer meanwhile runs the next tile's
      // groups into the other TMEM buffers.
      const bool live = !*abort_flag;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        if (half == (h >> 1)) {
#pragma unroll
          for (int j = 0; j < 32; j += 2)
            *reinterpret_cast<longlong2*>(stage_out + (quarter * 32 + lane) * GM_OUT_LD + j) =
                make_longlong2(acc[(h & 1) * 32 + j], acc[(h & 1) * 32 + j + 1]);
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (live) {
          const int et = threadIdx.x - 64;  // 0..255
          const int c0 = n0 + h * 32;
          for (int idx = et; idx < GM_BM * 16; idx += 256) {
            const int r = idx >> 4, ch = idx & 15;
            const int orow = m0 + r, col = c0 + 2 * ch;
            if (orow >= p.M) continue;
            const longlong2 val = *reinterpret_cast<const longlong2*>(stage_out + r * GM_OUT_LD + 2 * ch);
            int64_t* dst = p.out + (size_t)orow * p.out_ld + col;
            if (col + 1 < p.out_rows && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
              *reinterpret_cast<longlong2*>(dst) = val;
            } else {
              if (col < p.out_rows) dst[0] = val.x;
              if (col + 1 < p.out_rows) dst[1] = val.y;
            }
          }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) raise_device_error(p.err, DERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GM_TMEM_BUFS * GM_BN));
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// 2-D int8 matrix [rows][cols] (row stride = cols bytes), box 128 x 128, 128B swizzle.
static int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols) {
  EncodeTiled fn = encode_fn();
  if (!fn) return fail(YSKN_ECUDA, "cuTensorMapEncodeTiled is not available");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols % 16)) return fail(YSKN_EINVAL, "gemm: operand not 16-byte aligned");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols};
  const cuuint32_t box[2] = {GM_BK, 128};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(YSKN_ECUDA, "cuTensorMapEncodeTiled failed");
  return YSKN_OK;
}

int64_t gemm_workspace_bytes(const MatrixDev& m) { return (int64_t)m.phys_pad8 * m.cols; }

int launch_predecode(const MatrixDev& m, int8_t* W, cudaStream_t st) {
  const int S = m.cols / 256, rb = m.phys_pad8 / 8;
  const int64_t tiles = (int64_t)rb * S;
  const int blocks = (int)std::min<int64_t>(ceil_div(tiles, 8), 148 * 16);
  switch (m.bits) {
    case 4: trellis_predecode_kernel<4><<<blocks, 256, 0, st>>>(m.codes, m.lut8, rb, S, m.cols, W); break;
    case 5: trellis_predecode_kernel<5><<<blocks, 256, 0, st>>>(m.codes, m.lut8, rb, S, m.cols, W); break;
    case 6: trellis_predecode_kernel<6><<<blocks, 256, 0, st>>>(m.codes, m.lut8, rb, S, m.cols, W); break;
    case 7: trellis_predecode_kernel<7><<<blocks, 256, 0, st>>>(m.codes, m.lut8, rb, S, m.cols, W); break;
    default: trellis_predecode_kernel<8><<<blocks, 256, 0, st>>>(m.codes, m.lut8, rb, S, m.cols, W); break;
  }
  return cuda_fail(cudaGetLastError(), "trellis_predecode_kernel");
}

int launch_gemm(const MatrixDev& m, const int8_t* act, const int32_t* scales, int M, int64_t* out, int out_rows,
                int8_t* W, cudaStream_t st) {
  if (int rc = launch_predecode(m, W, st)) return rc;
  CUtensorMap map_act, map_w;
  if (int rc = make_map(&map_act, act, M, m.cols)) return rc;
  if (int rc = make_map(&map_w, W, m.phys_pad8, m.cols)) return rc;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] { attr = cudaFuncSetAttribute(trellis_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GM_SMEM); });
  if (attr != cudaSuccess) return cuda_fail(attr, "trellis_mma_kernel attributes");
  GemmParams p{};
  p.scales = scales;
  p.out = out;
  p.M = M;
  p.G = m.cols / 512;
  p.out_rows = out_rows;
  p.out_ld = out_rows;
  p.err = device_error_word();
  p.n_tiles = (int)ceil_div(out_rows, GM_BN);
  p.m_tiles = (int)ceil_div(M, GM_BM);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>((int64_t)p.n_tiles * p.m_tiles, sms);  // persistent: one CTA per SM
  trellis_mma_kernel<<<grid, GM_THREADS, GM_SMEM, st>>>(map_act, map_w, p);
  return cuda_fail(cudaGetLastError(), "trellis_mma_kernel");
}

}  // namespace yskn
