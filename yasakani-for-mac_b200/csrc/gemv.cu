// Weighted integer sums for skinny inputs (M <= 16 per pass): the decode GEMV.
//
// Contract (crates/yskn-ref/src/compressed_linear.rs:205-252; docs/spec/
// 02_COMPRESSED_LINEAR.md:160-196):
//   ws[m][n] = sum_g A[m][g] * sum_{j<512} lut8[state(n, 512g+j)] * act[m][512g+j]
// with an i32 dot per 512-column group and i64 across groups. Integer adds are
// associative, so any split of the groups across warps gives identical bits.
//
// B200 design
// -----------
// * Streaming layout (pack.cu): tiles of 8 rows x one 256-column sequence. Lane
//   (n = lane/4, q = lane%4) of a warp owns the q-th quarter (32 trellis steps,
//   `bits` words) of row n's sequence; the two tiles of a 512-column group are
//   adjacent, and a warp's run of units is one contiguous byte range of HBM.
// * Decode: each lane rebuilds its 32 states with constant shifts (the
//   12-bit window of its first step reaches into the previous quarter: one
//   shfl_up of the neighbour's last word), and looks the int8 pairs up in
//   shared memory. The table is stored 16 times (two lanes per copy); the
//   address is one shift (a funnel shift only where the 12-bit window straddles
//   two words) plus one LOP3, because B200's integer pipe (16 lanes/clk per SM
//   sub-partition) is as scarce as shared-memory bandwidth here. At bits = 8 the
//   stored bit order lets each copy own two banks (~2 wavefronts per warp-wide
//   lookup); at other bits four lanes share four banks (~3 wavefronts).
// * Math: the 8 decoded weights of a lane per 32-column chunk are exactly its
//   B fragment of mma.sync.m16n8k32.s8 (n = row, k = 8 consecutive columns of its
//   quarter); the activations (A, 16 token rows) are loaded in the same column
//   permutation, so one MMA replaces 4*M dp4a and M = 1..16 cost the same.
//   The i32 accumulator is scaled by the token's integer group scale into i64
//   after each 512-column group.
// * Work: one persistent CTA per SM; CTAs are split between the (up to 3)
//   matrices of a call in proportion to their work; each warp streams a
//   contiguous run of (8-row block, group) units, prefetching the next unit's
//   codes while it computes the current one. A row block whose groups are split
//   between warps is reduced without atomics on the output: every contributor
//   writes its i64 partial to scratch, and the last one to arrive (a counter per
//   row block) adds the partials and stores the result, then resets the counter.
//   The output is written exactly once, so it needs no zeroing.
// * Fused operator, rows with an output rotation: contributors add their partials
//   into int64 sums kept zero in library scratch (64-bit integer reductions, exact
//   in any order) and count the groups they added per 512-row block; the warp that
//   completes a block restores and rotates it, then clears the sums and the count.
//   One arrival per warp and block replaces the per-row-block hand-over.
// * Prologue: the first unit's codes and the 128 KiB table image (one bulk
//   asynchronous copy) are requested before the kernel waits for its predecessor on
//   the stream (programmatic dependent launch), then the input groups: the code
//   fetch and the table copy overlap the previous kernel's tail and the quantiser.
#include <algorithm>
#include <mutex>

#include "async.cuh"
#include "pmath.cuh"
#include "quant.cuh"

namespace yskn {

constexpr int GEMV_MAX_SEG = 3;
constexpr int LUT_COPY_BYTES = 128 * 1024;  // 16 copies x 4096 entries x 2 bytes
constexpr int LUT_BAR_BYTES = 16;           // the table copy's mbarrier, after the table
constexpr long long TABLE_WAIT_LIMIT = 2000000000ll;  // clock cycles (~1 s) before the table wait gives up

struct GemvSeg {
  const uint32_t* codes;
  const uint8_t* lutx;  // shared-memory image of the table (MatrixDev::lutx)
  int64_t* out;
  unsigned* counters;  // one per row block, zero between launches
  int64_t tiles;       // row blocks * 2G
  int row_blocks;
  int out_rows;        // rows written (<= physical rows)
  int out_ld;
  int cta_begin;       // first CTA of this segment
  int n_ctas;
  int base, rem;       // balanced tile ranges of the segment's warps
  // Fused operator only: restore into y instead of returning int64 sums.
  const float* tau;
  const int8_t* s_out;     // output rotation signs (sums go to `out` first), or nullptr
  float* y;                // f32 [mv][y_rows]
  int y_rows;
  unsigned* blk_counters;  // one per 512-row block (rotated restore), zero between launches
};

struct GemvParams {
  GemvSeg seg[GEMV_MAX_SEG];
  int n_seg;
  int G;
  int Kc;
  const int8_t* act;
  const int32_t* scales;
  int mv;  // valid activation rows (1..16)
  int checked;
  long long* partials;  // [2 * warps][32 lanes][4] i64
  unsigned* err;
  // Fused operator only: f32 input rows, input signs, optional 1/rms per row.
  const float* x;
  const int8_t* s_in;
  const float* inv_rms;
  // Fused operator with a quantised input (q_act != nullptr): the int8 rows [mv][Kc] and
  // group scales [mv][G] from the producing kernel, replacing the in-kernel quantiser; with
  // q_bss the rows' 1/rms is formed here from their per-512-block sums of squares
  // (rsqrt(sum / Kc + q_eps), blocks added in order from +0) and, if inv_out, stored.
  const int8_t* q_act;
  const float* q_alpha;
  const float* q_bss;
  float q_eps;
  float* inv_out;
  // Residual epilogue (res.hidden != nullptr; one matrix with an output rotation): the
  // restored rows go into the residual stream and become the next operator's quantised
  // input (residual_block512), token m's arrays at m * rows (alpha, bss at m * rows / 512).
  ResidualOut res;
  // Residual prologue (rin.y != nullptr): the input is formed in every CTA from the previous
  // projection's restored rows (residual_block512 per 512-group: the residual stream plus y,
  // times 1 + norm weight, quantised with the matrix's input signs); each row's 1/rms from
  // its block sums of squares. CTA 0 stores the updated stream to h_out (a buffer other than
  // h_in, which every CTA reads), the gate copy and 1/rms.
  ResidualIn rin;
  // Row-parallel tensor-parallel operator (tp.world > 1): exchange areas of all ranks.
  TpView tp;
};

template <int BITS>
struct Unit {
  static constexpr int U = (BITS % 4 == 0) ? 4 : (BITS % 2 == 0 ? 2 : 1);
  uint32_t w[2][BITS];
};

template <int BITS>
__device__ __forceinline__ void load_unit(Unit<BITS>& u, const uint32_t* tile0, int lane) {
  constexpr int U = Unit<BITS>::U;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const uint32_t* t = tile0 + s * (BITS * 32);
#pragma unroll
    for (int j = 0; j < BITS / U; ++j) {
      const uint32_t* p = t + (j * 32 + lane) * U;
      if constexpr (U == 4) {
        uint4 v;
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
        u.w[s][4 * j] = v.x; u.w[s][4 * j + 1] = v.y; u.w[s][4 * j + 2] = v.z; u.w[s][4 * j + 3] = v.w;
      } else if constexpr (U == 2) {
        uint2 v;
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
        u.w[s][2 * j] = v.x; u.w[s][2 * j + 1] = v.y;
      } else {
        uint32_t v;
        asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
        u.w[s][j] = v;
      }
    }
  }
}

// One unit's codes (2 tiles, 256 * BITS bytes) requested into L2, a 128-byte line per lane.
template <int BITS>
__device__ __forceinline__ void l2_prefetch_unit(const uint32_t* unit, int lane) {
  constexpr int LINES = 2 * BITS * 32 * 4 / 128;
  if (lane < LINES) asm volatile("prefetch.global.L2 [%0];" ::"l"(unit + lane * 32));
}

template <int BITS>
__device__ __forceinline__ uint32_t lut_copy_off(int lane) {
  return (uint32_t)(lane >> 1) << 3;
}

// hi32(a * b) + c and lo32(a * b) + c in one instruction each: with b a power of two they
// are a right or left shift and an add.
__device__ __forceinline__ uint32_t mad_hi(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("mad.hi.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t mad_lo(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
// One table entry at a shared-memory address (zero-extended).
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// Shared-memory address of state(step i) in this lane's table copy. V = [carry | w0 ..
// w_{BITS-1} | 0] is the lane's code words with the previous lane's last word in front;
// the state's 12 bits end at bit 32 + BITS(i+1) of V, and the 17-bit window that
// starts 5 bits below that end's state start holds them. Masked, they give the address
// bits of the table image:
// * bits = 8: the stored bytes carry the state's bits at 0,1 and 6..15 of bytes
//   (i-1, i) (stream8_store, common.cuh); shifted left by one and masked, they fill
//   address bits 1,2 and 7..16 around the copy (lane/2) in bits 3..6, so copy c sits
//   in banks 2c and 2c+1 and only the two lanes of a copy can conflict: ~2 shared-
//   memory wavefronts per 32 random lookups.
// * other bits: the same image layout (copy c in banks 2c, 2c+1; state bits 0,1 at
//   address bits 1,2 and bits 2..11 at 7..16, lutx_split_state in common.cuh), so the
//   same ~2 wavefronts per lookup; the stored stream has no spare bits between the two
//   parts of a state, so the address takes the state's window shifted to bit 1, two
//   masks and a multiply-add.
// base is the image's shared address plus the lane's copy offset (the masked state
// bits never overlap the copy field, so adding the copy equals or-ing it). Where the
// state's bits come from one word, the mask and one multiply-add form the address
// (hi32(x * 2^(32-sh)) + base is (x >> sh) + base, lo32(x * 2^k) + base is (x << k) +
// base); where they straddle two words, a funnel shift, the mask and an add. All shift
// amounts are compile-time constants after unrolling.
template <int BITS>
__device__ __forceinline__ uint32_t lut_abs(uint32_t carry, const uint32_t (&w)[BITS], int i, uint32_t base) {
  if constexpr (BITS != 8) {
    const int p = 32 + BITS * (i + 1) - 12 - 1;  // the bit of V below the state's first
    const int wi = p >> 5, sh = p & 31;
    const uint32_t lo = wi == 0 ? carry : w[wi - 1];
    const uint32_t hi = wi >= BITS ? 0u : w[wi];
    const uint32_t x = sh == 0 ? lo : sh + 13 <= 32 ? lo >> sh : __funnelshift_r(lo, hi, sh);  // state at 1..12
    return mad_lo(x & 0x1ff8u, 16u, (x & 6u) | base);
  }
  constexpr uint32_t MASK = 0x1ff86u;
  constexpr int LO = 1, HI = 17;
  const int p = 32 + BITS * (i + 1) - 12 - 5;
  const int wi = p >> 5, sh = p & 31;
  const uint32_t lo = wi == 0 ? carry : w[wi - 1];
  const uint32_t hi = wi >= BITS ? 0u : w[wi];
  if (sh == 0) return (lo & MASK) + base;
  if (sh + HI <= 32) return mad_hi(lo & (MASK << sh), 1u << (32 - sh), base);
  if (sh + LO >= 32) return mad_lo(hi & (MASK >> (32 - sh)), 1u << (32 - sh), base);
  return (__funnelshift_r(lo, hi, sh) & MASK) + base;
}

// lo | hi << 16 on the FMA pipe (lo, hi are zero-extended 16-bit entries).
__device__ __forceinline__ uint32_t pack_pair(uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(r) : "r"(hi), "r"(lo));
  return r;
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One sequence of one tile: 8 MMAs (k = 32 each) over this lane's quarter.
// a0p / a1p: the 64 activation bytes of quarter q for tokens n and n + 8 (shared
// memory or global, same column permutation as the B fragments).
template <int BITS, bool M1>
__device__ __forceinline__ void sequence_mma(const uint32_t (&w)[BITS], int lane, uint32_t lut_base, const uint4* a0p,
                                             const uint4* a1p, bool row0, bool row1, int (&c)[4]) {
  uint32_t carry = __shfl_up_sync(0xffffffffu, w[BITS - 1], 1);
  if ((lane & 3) == 0) carry = 0u;  // zeros before the start of the sequence (docs/FORMAT.md:121-128)
#pragma unroll
  for (int tp = 0; tp < 4; ++tp) {
    // Activations of two 32-column chunks, loaded before the 16 lookups that hide their latency.
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
    if (row0) x0 = a0p[tp];
    if (!M1 && row1) x1 = a1p[tp];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int t = 2 * tp + half;
      uint32_t b[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i0 = 4 * t + 2 * h;
        b[h] = pack_pair(lds_u16(lut_abs<BITS>(carry, w, i0, lut_base)), lds_u16(lut_abs<BITS>(carry, w, i0 + 1, lut_base)));
      }
      const uint32_t a0 = half ? x0.z : x0.x, a2 = half ? x0.w : x0.y;
      const uint32_t a1 = half ? x1.z : x1.x, a3 = half ? x1.w : x1.y;
      mma_s8(c, a0, a1, a2, a3, b[0], b[1]);
    }
  }
}

// Arrival of a warp on a GPU-scope counter: the fence (acq_rel, lighter than the
// sequentially consistent __threadfence) releases every lane's earlier writes, then one
// lane adds n. Returns the counter's previous value on every lane. The warp that sees
// the final count runs gpu_acquire() before it reads what the others wrote.
__device__ __forceinline__ unsigned warp_arrive(unsigned* counter, unsigned n, int lane) {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  __syncwarp();
  unsigned prev = 0;
  if (lane == 0) prev = atomicAdd(counter, n);
  return __shfl_sync(0xffffffffu, prev, 0);
}
__device__ __forceinline__ void gpu_acquire() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Cross-GPU exchange of the row-parallel operator. Each 32-bit datum goes to a peer's
// area as one 64-bit word (datum | epoch << 32) with a plain (volatile) store over
// NVLink; an aligned 64-bit access is single-copy atomic, so a receiver that reads a
// word carrying its epoch has the datum too, without fences. Every wait of a CTA on its
// peers runs against deadlines of TpView::wait_cycles clock cycles taken once per wait
// phase (not per word), and a CTA-wide abort flag ends every later wait at once: a
// peer that never arrives costs a launch at most two limits, after which the device
// error word holds DERR_TIMEOUT and the call's output is not valid.
__device__ __forceinline__ uint64_t ll_word(uint32_t datum, uint32_t epoch) {
  return (uint64_t)datum | ((uint64_t)epoch << 32);
}
__device__ __forceinline__ void st_ll(uint64_t* p, uint64_t w) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_ll2(uint64_t* p, uint64_t w0, uint64_t w1) {  // two words, each atomic
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_ll2(const uint64_t* p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The int64 sum of two epoch-tagged words (low half first), polling until both carry
// `epoch` or the clock passes `deadline`. Once `ok` is false (this lane timed out
// before, or the CTA's abort flag is up) it returns 0 without polling.
__device__ __forceinline__ long long recv_sum(const uint64_t* p, uint32_t epoch, long long deadline,
                                              const volatile int* abort_flag, bool& ok) {
  if (!ok) return 0;
  ulonglong2 v = ld_ll2(p);
  while ((uint32_t)(v.x >> 32) != epoch || (uint32_t)(v.y >> 32) != epoch) {
    if (clock64() > deadline || *abort_flag) {
      ok = false;
      return 0;
    }
    v = ld_ll2(p);
  }
  return (long long)(((uint64_t)(uint32_t)v.y << 32) | (uint32_t)v.x);
}
template <typename T>
__device__ __forceinline__ T* tp_at(const TpView& tp, int q, size_t off) {
  return reinterpret_cast<T*>(tp.base[q] + off);
}

// Balanced contiguous ranges: warp w of a segment owns tiles
// [w*base + min(w, rem), (w+1)*base + min(w+1, rem)), base = tiles / warps.
struct Ranges {
  int base, rem;
  __device__ __forceinline__ int begin(int w) const { return w * base + min(w, rem); }
  __device__ __forceinline__ int owner(int t) const {
    const int cut = rem * (base + 1);
    return t < cut ? t / (base + 1) : rem + (t - cut) / base;
  }
};

// Residual prologue of the fused operator (GemvParams::rin): warp w forms input groups
// w, w + 16, ... from the previous projection's rows (every load of a group issued before
// its arithmetic) into the CTA's int8 rows, group scales and block sums. Kept out of line:
// its registers stay out of the streaming loop's allocation.
__device__ __noinline__ void residual_prologue(const ResidualIn rin, const int8_t* s_in, int Kc, int items,
                                               int8_t* s_act, int act_ld, float* s_alpha, float* s_bss,
                                               unsigned* err, int warp, int lane) {
  const int G = Kc / 512;
  bool bad = false;
  const bool writer = blockIdx.x == 0;
  for (int k = warp; k < items; k += GEMV_WARPS) {
    const int m = k / G, r0 = (k - m * G) * 512;
    float v[16];
    uint32_t hws[8], wws[8], sws[8];
    const float* yr = rin.y + (size_t)m * Kc + r0;
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) {
      const float2 t = __ldcg(reinterpret_cast<const float2*>(yr + 64 * k2 + 2 * lane));
      v[2 * k2] = t.x;
      v[2 * k2 + 1] = t.y;
    }
    load_residual_words512(rin.h_in + (size_t)m * Kc, rin.norm_w, s_in, r0, lane, hws, wws, sws);
    residual_block512(v, hws, wws, sws, writer ? rin.h_out + (size_t)m * Kc + r0 : nullptr,
                      writer && rin.gate_out ? rin.gate_out + (size_t)m * Kc + r0 : nullptr,
                      s_act + (size_t)m * act_ld + r0, s_alpha + k, s_bss + k, lane, bad);
  }
  if (writer && __any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(err, DERR_NONFINITE);
}

// ACT_SMEM: activations and scales staged once per CTA in shared memory after
// the table (rows padded by 16 bytes so the 8 token rows fall in different banks).
// FUSED (implies ACT_SMEM): the whole operator. Every CTA quantises the f32 input
// rows itself while it builds the table (the same device functions as the
// standalone quantiser, so the same bits), and results leave as restored f32:
// rows without an output rotation are restored where they are stored; with a
// rotation the int64 sums go to `out` and the warp that completes the last 8-row
// block of a 512-row block (a counter per 512-row block) restores and rotates it.
template <int BITS, bool M1, bool ACT_SMEM, bool FUSED>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 1) trellis_sums_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) uint8_t s_lut[];
  // Which matrix this CTA serves.
  int si = 0;
  while (si + 1 < p.n_seg && (int)blockIdx.x >= p.seg[si + 1].cta_begin) ++si;
  const GemvSeg& S = p.seg[si];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, Kc = p.Kc, act_ld = Kc + 16;
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(s_lut + LUT_COPY_BYTES);
  int8_t* s_act = reinterpret_cast<int8_t*>(s_lut + LUT_COPY_BYTES + LUT_BAR_BYTES);
  int32_t* s_scale = reinterpret_cast<int32_t*>(s_lut + LUT_COPY_BYTES + LUT_BAR_BYTES + (size_t)p.mv * act_ld);
  float* s_alpha = reinterpret_cast<float*>(s_scale + p.mv * G);  // FUSED: group scales
  float* s_rq = s_alpha + p.mv * G;                                // FUSED: row quanta
  float* s_bss = s_rq + TP_MAX_M;                                  // FUSED, residual prologue: block sums

  // Programmatic dependent launch: the next kernel on the stream may be scheduled as
  // SMs free up; it waits (griddepcontrol.wait) before it reads anything this grid writes.
  asm volatile("griddepcontrol.launch_dependents;");
  const int items = FUSED ? p.mv * G : 0;
  Group512In nxt;

  // This warp's tiles [t_begin, t_end) (tile t = sequence t % 2G of row block t / 2G),
  // walked as units u = (row block, group) = tiles 2u, 2u+1; only the first and the
  // last unit can be half units. Its first unit's codes are requested before the table
  // is built, so their HBM latency overlaps the table copy (and, fused, the quantiser).
  const int w_id = (blockIdx.x - S.cta_begin) * GEMV_WARPS + warp;
  const Ranges R{S.base, S.rem};
  const int T2 = 2 * G;  // tiles per row block
  int t_begin, t_end;
  if (p.checked) {
    // One warp per whole row block, groups in ascending order: every i64 add is
    // checked in the reference's order (compressed_linear.rs:229-248).
    t_begin = w_id < S.row_blocks ? w_id * T2 : 0;
    t_end = w_id < S.row_blocks ? t_begin + T2 : 0;
  } else {
    t_begin = R.begin(w_id);
    t_end = R.begin(w_id + 1);
  }
  int u = t_begin >> 1;
  const int u_end = (t_end + 1) >> 1;
  constexpr int TILE_WORDS = BITS * 32;
  // The tiles of a row block are consecutive in memory, so units are a stride of two
  // tiles apart and the walk needs no division.
  const uint32_t* ptr = S.codes + (size_t)u * 2 * TILE_WORDS;
  Unit<BITS> ua, ub;
  if (u < u_end) load_unit<BITS>(ua, ptr, lane);
  if (u + 1 < u_end) l2_prefetch_unit<BITS>(ptr + 2 * TILE_WORDS, lane);

  // 16 copies of the int8-pair table, copy c in banks 2c, 2c+1 (lut_abs). The
  // matrix keeps this image prebuilt (MatrixDev::lutx); one thread starts bulk
  // asynchronous copies of it at once, and they land while the warps quantise the
  // input (fused) or stage the activations. (Expanding the stored 8 KiB table in
  // shared memory instead costs every SM about 0.5 us more, measured.)
  if (threadIdx.x == 0) {
    mbar_init(s_bar, 1);
    mbar_init_fence();
    mbar_expect_tx(s_bar, LUT_COPY_BYTES);
    // Every CTA of the segment copies the same image: each starts at another quarter, so
    // the CTAs' first requests spread over the L2 slices instead of queueing on the same lines.
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = (k + blockIdx.x) & 3;
      bulk_copy_g2s(s_lut + c * (LUT_COPY_BYTES / 4), S.lutx + c * (LUT_COPY_BYTES / 4), LUT_COPY_BYTES / 4, s_bar);
    }
  }
  if (FUSED && S.s_out) {
    // The restores at the end of the launch read the row scales and output signs of
    // whole 512-row blocks; the segment's CTAs bring both into L2 now, a share each.
    const size_t t_lines = ((size_t)S.y_rows * 4 + 127) / 128, s_lines = ((size_t)S.y_rows + 127) / 128;
    for (size_t l = (size_t)(blockIdx.x - S.cta_begin) * blockDim.x + threadIdx.x; l < t_lines + s_lines;
         l += (size_t)S.n_ctas * blockDim.x) {
      const char* a = l < t_lines ? reinterpret_cast<const char*>(S.tau) + 128 * l
                                  : reinterpret_cast<const char*>(S.s_out) + 128 * (l - t_lines);
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
    }
    if (p.res.hidden) {
      // Likewise the residual epilogue's rows: the residual stream (each token), the norm
      // weights and the next operator's input signs. L2 is the point of coherence, so the
      // stream's lines may be brought in before the previous kernel has finished.
      const size_t h_lines = ((size_t)p.mv * S.y_rows * 2 + 127) / 128, w_lines = ((size_t)S.y_rows * 2 + 127) / 128;
      const size_t n_lines = h_lines + w_lines + s_lines;
      for (size_t l = (size_t)(blockIdx.x - S.cta_begin) * blockDim.x + threadIdx.x; l < n_lines;
           l += (size_t)S.n_ctas * blockDim.x) {
        const char* a = l < h_lines ? reinterpret_cast<const char*>(p.res.hidden) + 128 * l
                        : l < h_lines + w_lines
                            ? reinterpret_cast<const char*>(p.res.norm_w) + 128 * (l - h_lines)
                            : reinterpret_cast<const char*>(p.res.s_next) + 128 * (l - h_lines - w_lines);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
      }
    }
  }
  // Everything above reads only the matrix (codes, table), which no kernel writes. The
  // inputs, the scales and every scratch word may belong to the previous kernel on the
  // stream until it completes: wait for it here (a no-op without a programmatic launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Fused: each warp's first input group is requested first, ahead of the staging below.
  // Warp w quantises items w, w + 16, ... counted from a CTA-dependent start, so the CTAs
  // do not all read the same input lines at the same moment.
  const int item_rot = FUSED ? (int)(blockIdx.x % (unsigned)items) : 0;
  auto item_of = [&](int k) { return k + item_rot < items ? k + item_rot : k + item_rot - items; };
  if (FUSED && !p.q_act && !p.rin.y && warp < items) {
    const int it = item_of(warp);
    load_group512(p.x + (size_t)(it / G) * Kc + (it % G) * 512, p.s_in + (it % G) * 512, lane, nxt);
  }
  __shared__ float s_inv[TP_MAX_M];  // quantised input with block sums of squares: the rows' 1/rms
  {
    if (FUSED && p.q_act) {
      // Quantised input: stage the int8 rows and the group scales (8 independent 16-byte
      // loads per thread before their stores); each row's 1/rms from its block sums. The
      // first two scales (and block sums) of each thread are requested before the rows, so
      // all of the staging is one round of loads.
      const int n_sc = p.mv * G;
      const int i0 = threadIdx.x, i1 = threadIdx.x + GEMV_WARPS * 32;
      float al0 = 0.0f, al1 = 0.0f, bs0 = 0.0f, bs1 = 0.0f;
      if (i0 < n_sc) {
        al0 = __ldcg(p.q_alpha + i0);
        if (p.q_bss) bs0 = __ldcg(p.q_bss + i0);
      }
      if (i1 < n_sc) {
        al1 = __ldcg(p.q_alpha + i1);
        if (p.q_bss) bs1 = __ldcg(p.q_bss + i1);
      }
      const int vec = Kc / 16, total = p.mv * vec;
      for (int base = 0; base < total; base += 8 * GEMV_WARPS * 32) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int idx = base + threadIdx.x + k * GEMV_WARPS * 32;
          if (idx < total) v[k] = __ldcg(reinterpret_cast<const uint4*>(p.q_act + (size_t)(idx / vec) * Kc) + idx % vec);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int idx = base + threadIdx.x + k * GEMV_WARPS * 32;
          if (idx < total) reinterpret_cast<uint4*>(s_act + (idx / vec) * act_ld)[idx % vec] = v[k];
        }
      }
      if (i0 < n_sc) {
        s_alpha[i0] = al0;
        s_bss[i0] = bs0;  // summed per row after the barrier
      }
      if (i1 < n_sc) {
        s_alpha[i1] = al1;
        s_bss[i1] = bs1;
      }
      for (int idx = threadIdx.x + 2 * GEMV_WARPS * 32; idx < n_sc; idx += blockDim.x) {
        s_alpha[idx] = __ldcg(p.q_alpha + idx);
        if (p.q_bss) s_bss[idx] = __ldcg(p.q_bss + idx);
      }
    } else if (FUSED && p.rin.y) {
      residual_prologue(p.rin, p.s_in, Kc, items, s_act, act_ld, s_alpha, s_bss, p.err, warp, lane);
    } else if (FUSED) {
      // A warp's groups in turn, each one's inputs requested before the previous is quantised.
      bool bad = false;
      for (int k = warp; k < items; k += GEMV_WARPS) {
        const int item = item_of(k);
        const int m = item / G, g = item - m * G;
        const Group512In cur = nxt;
        if (k + GEMV_WARPS < items) {
          const int after = item_of(k + GEMV_WARPS);
          load_group512(p.x + (size_t)(after / G) * Kc + (after % G) * 512, p.s_in + (after % G) * 512, lane, nxt);
        }
        const float a = quantize_loaded512(cur, s_act + (size_t)m * act_ld + g * 512, lane, bad);
        if (lane == 0) s_alpha[item] = a;
      }
      if (blockIdx.x == 0 && __any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(p.err, DERR_NONFINITE);
    } else if (ACT_SMEM) {
      // Batches of 8 independent 16-byte loads per thread before their stores.
      const int vec = Kc / 16, total = p.mv * vec;
      for (int base = 0; base < total; base += 8 * GEMV_WARPS * 32) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int idx = base + threadIdx.x + k * GEMV_WARPS * 32;
          if (idx < total) v[k] = __ldg(reinterpret_cast<const uint4*>(p.act + (size_t)(idx / vec) * Kc) + idx % vec);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int idx = base + threadIdx.x + k * GEMV_WARPS * 32;
          if (idx < total) reinterpret_cast<uint4*>(s_act + (idx / vec) * act_ld)[idx % vec] = v[k];
        }
      }
      for (int idx = threadIdx.x; idx < p.mv * G; idx += blockDim.x) s_scale[idx] = __ldg(p.scales + idx);
    }
  }
  __syncthreads();  // the barrier is initialised; fused: the group scales are in place
  // Every thread waits (bounded) for the table. A timeout is reported and the CTA still
  // runs its units, so the arrival counters and the zero-kept sums stay consistent.
  if (!mbar_wait_bounded(s_bar, 0, TABLE_WAIT_LIMIT) && lane == 0) raise_device_error(p.err, DERR_TIMEOUT);
  // Row-parallel tensor parallelism: this launch's epoch (every CTA of every launch on
  // this rank adds one to the rank's counter, and every such launch has one CTA per SM)
  // and the slot parity that double-buffers the exchange.
  __shared__ unsigned s_epoch;
  __shared__ float s_rowmax[TP_MAX_M];
  __shared__ int s_abort;  // row-parallel: a wait on a peer gave up; later waits return at once
  const bool tp = FUSED && p.tp.world > 1;
  if (tp && threadIdx.x == 0) {
    const unsigned long long prev = atomicAdd(tp_at<unsigned long long>(p.tp, p.tp.rank, p.tp.off_counter), 1ull);
    s_epoch = (unsigned)(prev / gridDim.x) + 1u;
    s_abort = 0;
  }
  if (FUSED) {  // the rows' common integer grids (compressed_linear.rs:113-128)
    if (threadIdx.x < p.mv) {
      float mx = 0.0f;
      for (int g = 0; g < G; ++g) mx = fmaxf(mx, s_alpha[threadIdx.x * G + g]);
      s_rowmax[threadIdx.x] = mx;
      if (p.rin.y || (p.q_act && p.q_bss)) {  // the row's 1/rms from its block sums, added in order from +0
        float total_sq = 0.0f;
        for (int g = 0; g < G; ++g) total_sq = __fadd_rn(total_sq, s_bss[threadIdx.x * G + g]);
        const float inv = pm_rsqrt(__fadd_rn(__fdiv_rn(total_sq, (float)Kc), p.rin.y ? p.rin.eps : p.q_eps));
        s_inv[threadIdx.x] = inv;
        float* inv_out = p.rin.y ? p.rin.inv_out : p.inv_out;
        if (inv_out && blockIdx.x == 0) inv_out[threadIdx.x] = inv;
      }
    }
    if (tp) {
      // The grid of a row is set by its largest group scale over all ranks' groups:
      // CTA 0 of every rank sends its row maxima to every rank (epoch-tagged words),
      // every CTA polls them in its own area and takes the max.
      __syncthreads();
      const unsigned epoch = s_epoch, par = epoch & 1u;
      const int W = p.tp.world, me = p.tp.rank;
      if (blockIdx.x == 0 && threadIdx.x < p.mv)
        for (int q = 0; q < W; ++q)
          st_ll(tp_at<uint64_t>(p.tp, q, p.tp.off_maxbox) + (par * W + me) * TP_MAX_M + threadIdx.x,
                ll_word(__float_as_uint(s_rowmax[threadIdx.x]), epoch));
      if (threadIdx.x < 32 && lane < p.mv) {
        const uint64_t* box = tp_at<uint64_t>(p.tp, me, p.tp.off_maxbox) + (size_t)par * W * TP_MAX_M;
        bool ok = true;
        float mx = 0.0f;
        const long long deadline = clock64() + p.tp.wait_cycles;  // one limit for all sources
        for (int src = 0; src < W && ok; ++src) {
          const uint64_t* w = box + src * TP_MAX_M + lane;
          uint64_t v = ld_ll(w);
          while ((uint32_t)(v >> 32) != epoch) {
            if (clock64() > deadline) {
              ok = false;
              break;
            }
            v = ld_ll(w);
          }
          mx = fmaxf(mx, __uint_as_float((uint32_t)v));
        }
        if (!ok) {
          s_abort = 1;
          raise_device_error(p.err, DERR_TIMEOUT);
        }
        s_rowmax[lane] = mx;
      }
    }
    __syncthreads();
    for (int item = threadIdx.x; item < p.mv * G; item += blockDim.x) {
      const int m = item / G;
      const float mx = s_rowmax[m];
      s_scale[item] = integer_group_scale(s_alpha[item], row_grid_multiplier(mx));
      if (item == m * G) s_rq[m] = row_quantum_of(mx);
    }
  }
  __syncthreads();

  if (t_begin >= t_end) return;

  const uint32_t copy_off = lut_copy_off<BITS>(lane);
  // The lane's table copy as a shared-memory address. Passed through a volatile move
  // after the barriers above, so no lookup that depends on it can be scheduled earlier.
  uint32_t lut_base;
  asm volatile("mov.u32 %0, %1;" : "=r"(lut_base) : "r"(smem_u32(s_lut) + copy_off));
  const int q = lane & 3, n = lane >> 2;
  const int tok0 = n < p.mv ? n : p.mv - 1;
  const int tok1 = n + 8 < p.mv ? n + 8 : p.mv - 1;
  const bool row0 = n < p.mv, row1 = n + 8 < p.mv;
  const int8_t* act0 = ACT_SMEM ? s_act + tok0 * act_ld : p.act + (size_t)tok0 * Kc;
  const int8_t* act1 = ACT_SMEM ? s_act + tok1 * act_ld : p.act + (size_t)tok1 * Kc;
  const int32_t* sc0 = ACT_SMEM ? s_scale + tok0 * G : p.scales + (size_t)tok0 * G;
  const int32_t* sc1 = ACT_SMEM ? s_scale + tok1 * G : p.scales + (size_t)tok1 * G;

  int rb = u / G, g = u % G;
  long long acc[4] = {0, 0, 0, 0};
  bool overflow = false;
  bool bad = false;       // FUSED: non-finite restored values
  unsigned pend = 0;      // FUSED, rotated rows: tiles added to the current 512-row block, not yet counted
  // 512-row blocks this warp completed (bit i: block blk_lo + i) and restores after its
  // last unit: row-parallel, the blocks whose sums it sent to the peers; several tokens,
  // every block it completed (one token: restored at once, inside the loop).
  const int blk_lo = (t_begin / T2) >> 6;
  unsigned done_mask = 0;

  // The rows' 1/rms for the restore: formed here from a quantised input's block sums, or given.
  const float* inv_base = (FUSED && ((p.q_act && p.q_bss) || p.rin.y)) ? s_inv : p.inv_rms;
  // Final sums of rows row0, row0 + 1 for tokens n, n + 8 (the C fragment): stored
  // as int64, or (fused operator, rows without an output rotation) restored to f32.
  auto emit = [&](const long long (&v)[4], int row0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = n + (i >> 1) * 8, row = row0 + (i & 1);
      if constexpr (FUSED) {
        if (tok < p.mv && row < S.y_rows) {
          const float t = restore_value(v[i], s_rq[tok], inv_base ? inv_base + tok : nullptr, __ldg(S.tau + row));
          bad |= !finite32(t) || (inv_base && !finite32(inv_base[tok]));
          S.y[(size_t)tok * S.y_rows + row] = t;
        }
      } else {
        if (tok < p.mv && row < S.out_rows) S.out[(size_t)tok * S.out_ld + row] = v[i];
      }
    }
  };
  // Rotated rows (fused): restore + H512 of a complete 512-row block of sums, then clear
  // the sums and the block's counter for the next launch.
  // Several tokens: restored after the streaming loop (see done_mask), tokens in turn,
  // each token's sums requested before the previous token is transformed.
  // Residual epilogue: token tok's block, restored, into the residual stream and the next
  // operator's quantised input.
  auto residual = [&](const int64_t* wsr, int tok, int blk) {
    const int rows = S.y_rows;
    ResidualOut o = p.res;
    o.hidden += (size_t)tok * rows;
    o.act += (size_t)tok * rows;
    o.alpha += (size_t)tok * (rows / 512);
    o.bss += (size_t)tok * (rows / 512);
    if (o.gate) o.gate += (size_t)tok * rows;
    residual_restore512(wsr, S.tau, S.s_out, s_rq[tok], inv_base ? inv_base + tok : nullptr, o, blk * 512, lane, bad);
  };
  auto clear_sums = [&](int64_t* wsr, int blk) {  // the rows this lane read (the restore's lane mapping)
#pragma unroll
    for (int k = 0; k < 8; ++k)
      __stcg(reinterpret_cast<longlong2*>(wsr + blk * 512 + 64 * k + 2 * lane), make_longlong2(0, 0));
  };
  // One token, no residual output: the block restored inside the streaming loop by the
  // warp that completed it (kept free of the residual code, which would raise the loop's
  // register pressure; the residual epilogue runs after the loop).
  auto restore_plain = [&](int blk) {
    restore_block512(S.out, s_rq[0], inv_base, S.tau, S.s_out, blk * 512, S.y_rows, S.y, lane, bad);
    clear_sums(S.out, blk);
    if (lane == 0) S.blk_counters[blk] = 0u;
  };
  auto restore_block = [&](int blk) {
    if (FUSED && p.res.hidden) {
      for (int tok = 0; tok < p.mv; ++tok) {
        int64_t* wsr = S.out + (size_t)tok * S.out_ld;
        residual(wsr, tok, blk);
        clear_sums(wsr, blk);
      }
    } else if constexpr (M1) {
      for (int tok = 0; tok < p.mv; ++tok) {
        int64_t* wsr = S.out + (size_t)tok * S.out_ld;
        restore_block512(wsr, s_rq[tok], inv_base ? inv_base + tok : nullptr, S.tau, S.s_out, blk * 512, S.y_rows,
                         S.y + (size_t)tok * S.y_rows, lane, bad);
        clear_sums(wsr, blk);
      }
    } else {
      Rows512 rr;
      longlong2 w[8], wn[8];
      load_sums512(S.out, blk * 512, lane, w);
      load_rows512(S.tau, S.s_out, blk * 512, lane, rr);
      for (int tok = 0; tok < p.mv; ++tok) {
        int64_t* wsr = S.out + (size_t)tok * S.out_ld;
        if (tok + 1 < p.mv) load_sums512(wsr + S.out_ld, blk * 512, lane, wn);
        clear_sums(wsr, blk);  // after their reads
        restore_loaded512(w, rr, s_rq[tok], inv_base ? inv_base + tok : nullptr, blk * 512, S.y_rows,
                          S.y + (size_t)tok * S.y_rows, lane, bad);
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = wn[k];
      }
    }
    if (lane == 0) S.blk_counters[blk] = 0u;
  };
  // Row-parallel: this rank's int64 sums of block blk into the receive slot of every
  // peer, each sum as two epoch-tagged words (plain stores over NVLink, no fence).
  // Slot word (2 per sum) of row r, token tok, source src: recv + ((par*W + src)*16 + tok) * 2*rows + 2r.
  auto send_block = [&](int blk) {
    const unsigned epoch = s_epoch, par = epoch & 1u;
    const int W = p.tp.world, me = p.tp.rank;
    const size_t slot = (size_t)p.tp.max_blocks * 512 * 2;
    for (int tok = 0; tok < p.mv; ++tok) {
      const int64_t* src = S.out + (size_t)tok * S.out_ld + blk * 512;
      longlong2 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __ldcg(reinterpret_cast<const longlong2*>(src + 64 * k + 2 * lane));
      for (int qd = 0; qd < W; ++qd) {
        if (qd == me) continue;
        uint64_t* dst = tp_at<uint64_t>(p.tp, qd, p.tp.off_recv) + (((size_t)par * W + me) * TP_MAX_M + tok) * slot +
                        (size_t)blk * 1024;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = 64 * k + 2 * lane;  // rows r, r + 1 of the block (restore_block512's lane mapping)
          st_ll2(dst + 2 * r, ll_word((uint32_t)v[k].x, epoch), ll_word((uint32_t)((uint64_t)v[k].x >> 32), epoch));
          st_ll2(dst + 2 * r + 2, ll_word((uint32_t)v[k].y, epoch), ll_word((uint32_t)((uint64_t)v[k].y >> 32), epoch));
        }
      }
    }
  };
  // One unit: prefetch the next one into `nxt`, compute `cur`; true when done.
  // The loop below alternates the two buffers, so no registers are copied.
  auto step = [&](Unit<BITS>& cur, Unit<BITS>& nxt) -> bool {
    const bool has_next = u + 1 < u_end;
    int rbn = rb, gn = g + 1;
    if (gn == G) {
      gn = 0;
      ++rbn;
    }
    ptr += 2 * TILE_WORDS;
    if (has_next) load_unit<BITS>(nxt, ptr, lane);
    // The unit after the next one into L2 now, so its load next step waits on L2, not HBM
    // (one unit in registers per warp is too few bytes in flight to cover HBM latency).
    if (u + 2 < u_end) l2_prefetch_unit<BITS>(ptr + 2 * TILE_WORDS, lane);
    int c[4] = {0, 0, 0, 0};
    const int col = g * 512 + q * 64;
    const uint4* a0p = reinterpret_cast<const uint4*>(act0 + col);
    const uint4* a1p = reinterpret_cast<const uint4*>(act1 + col);
    // A half unit at either end of the range holds one tile (the integer dot of a half
    // group, scaled by the group's scale, adds up exactly with the other half's).
    if (2 * u >= t_begin) sequence_mma<BITS, M1>(cur.w[0], lane, lut_base, a0p, a1p, row0, row1, c);
    if (2 * u + 1 < t_end) sequence_mma<BITS, M1>(cur.w[1], lane, lut_base, a0p + 16, a1p + 16, row0, row1, c);
    const long long s0 = sc0[g], s1 = sc1[g];
    const long long t[4] = {s0 * c[0], s0 * c[1], s1 * c[2], s1 * c[3]};
    if (p.checked) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const long long r = (long long)((unsigned long long)acc[i] + (unsigned long long)t[i]);
        overflow |= ((acc[i] ^ r) & (t[i] ^ r)) < 0;
        acc[i] = r;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += t[i];  // cannot overflow below 512 groups
    }

    ++u;
    if (!has_next || rbn != rb) {
      // Rows 2q, 2q+1 of the block for tokens n and n+8 (the C fragment).
      const int row0 = rb * 8 + 2 * q;
      const int first = rb * T2, last = first + T2 - 1;  // the row block's tiles
      const bool sole = p.checked || (t_begin <= first && t_end > last);
      if (FUSED && S.s_out) {
        // Rotated rows: every contributor adds its partial into the zeroed sums (integer
        // adds commute, so any order gives the same bits) and counts the tiles it added
        // per 512-row block; the warp that brings a block to 64 x 2G tiles restores it,
        // then clears the sums and the counter for the next launch.
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tok = n + (i >> 1) * 8;
          if (tok < p.mv)
            atomicAdd(reinterpret_cast<unsigned long long*>(S.out + (size_t)tok * S.out_ld + row0 + (i & 1)),
                      (unsigned long long)acc[i]);
        }
        pend += (unsigned)(min(2 * u, t_end) - max(t_begin, first));
        if (!has_next || (rbn >> 6) != (rb >> 6)) {
          const int blk = rb >> 6;
          const unsigned prev = warp_arrive(S.blk_counters + blk, pend, lane);
          if (prev + pend == 64u * (unsigned)T2) {
            gpu_acquire();
            if (tp) {
              // This rank's sums of the block go to every peer; the block is restored
              // (with theirs added) after this warp's last unit, so no warp ever waits
              // for a peer while it still holds work that a peer may wait for.
              send_block(blk);
              done_mask |= 1u << (blk - blk_lo);
            } else {
              if (M1 && !p.res.hidden)
                restore_plain(blk);
              else
                done_mask |= 1u << (blk - blk_lo);
            }
          }
          pend = 0;
        }
      } else if (sole) {
        emit(acc, row0);
      } else {
        // Split row block: publish this warp's partial; the last of the
        // contributing warps (consecutive, all non-empty) adds them up.
        const int gw = blockIdx.x * GEMV_WARPS + warp;  // global warp id: scratch slot owner
        const int slot_kind = t_begin >= first ? 0 : 1;
        long long* mine = p.partials + ((size_t)(gw * 2 + slot_kind) * 32 + lane) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) __stcg(mine + i, acc[i]);
        const int wf = R.owner(first), wl = R.owner(last);
        const unsigned prev = warp_arrive(S.counters + rb, 1u, lane);
        if (prev == (unsigned)(wl - wf)) {
          gpu_acquire();
          long long sum[4] = {0, 0, 0, 0};
          for (int cw = wf; cw <= wl; ++cw) {
            const int kind = R.begin(cw) >= first ? 0 : 1;
            const int cgw = S.cta_begin * GEMV_WARPS + cw;
            const long long* src = p.partials + ((size_t)(cgw * 2 + kind) * 32 + lane) * 4;
#pragma unroll
            for (int i = 0; i < 4; ++i) sum[i] += __ldcg(src + i);
          }
          if (lane == 0) S.counters[rb] = 0u;
          emit(sum, row0);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = 0;
    }
    rb = rbn;
    g = gn;
    return !has_next;
  };
  // Row-parallel: the peers' sums of block blk added to this rank's, then the restore.
  auto recv_restore = [&](int blk, long long deadline, bool& ok) {
    const unsigned epoch = s_epoch, par = epoch & 1u;
    const int W = p.tp.world, me = p.tp.rank;
    const size_t slot = (size_t)p.tp.max_blocks * 512 * 2;
    const uint64_t* recv = tp_at<uint64_t>(p.tp, me, p.tp.off_recv);
    for (int tok = 0; tok < p.mv; ++tok) {
      int64_t* mine = S.out + (size_t)tok * S.out_ld + blk * 512;
      longlong2 s[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] = __ldcg(reinterpret_cast<const longlong2*>(mine + 64 * k + 2 * lane));
      for (int src = 0; src < W; ++src) {
        if (src == me) continue;
        // All 16 tagged word pairs of this lane requested at once (one round trip when the
        // peer's block has arrived, instead of one per pair); a pair whose tag is not yet
        // this epoch's is polled on its own, against the same deadline.
        const uint64_t* w = recv + (((size_t)par * W + src) * TP_MAX_M + tok) * slot + (size_t)blk * 1024 + 4 * lane;
        ulonglong2 v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = ld_ll2(w + 128 * (j >> 1) + 2 * (j & 1));
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          long long add;
          if ((uint32_t)(v[j].x >> 32) == epoch && (uint32_t)(v[j].y >> 32) == epoch)
            add = (long long)(((uint64_t)(uint32_t)v[j].y << 32) | (uint32_t)v[j].x);
          else
            add = recv_sum(w + 128 * (j >> 1) + 2 * (j & 1), epoch, deadline, &s_abort, ok);
          if (j & 1)
            s[j >> 1].y += add;
          else
            s[j >> 1].x += add;
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) __stcg(reinterpret_cast<longlong2*>(mine + 64 * k + 2 * lane), s[k]);
    }
    if (__any_sync(0xffffffffu, !ok)) {
      ok = false;
      if (lane == 0) {
        s_abort = 1;
        raise_device_error(p.err, DERR_TIMEOUT);
      }
    }
    restore_block(blk);
  };
  for (;;) {
    if (step(ua, ub)) break;
    if (step(ub, ua)) break;
  }
  if (tp) {
    // Every peer's sums of the blocks this warp completed: wait for them (their warps
    // send as soon as each block completes there, without waiting on anything), add
    // them to this rank's, restore the whole block. One deadline for all of this warp's
    // blocks; after a timeout (here or in another warp of the CTA) the remaining words
    // are not polled.
    const long long deadline = clock64() + p.tp.wait_cycles;
    bool ok = true;
    while (done_mask) {
      const int blk = blk_lo + __ffs(done_mask) - 1;
      done_mask &= done_mask - 1;
      recv_restore(blk, deadline, ok);
    }
  }
  if constexpr (FUSED) {
    if (!tp && (!M1 || p.res.hidden)) {  // several tokens, or the residual epilogue
      while (done_mask) {
        const int blk = blk_lo + __ffs(done_mask) - 1;
        done_mask &= done_mask - 1;
        restore_block(blk);
      }
    }
  }
  if (p.checked && __any_sync(0xffffffffu, overflow) && lane == 0) raise_device_error(p.err, DERR_OVERFLOW);
  if (FUSED && __any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(p.err, DERR_NONFINITE);
}

static int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  });
  return n;
}

int gemv_max_warps() { return (sm_count() + 8) * GEMV_WARPS; }

// Dynamic shared memory per CTA: B200's opt-in 232448 bytes less room for the kernel's
// few static shared words (launch epoch, row maxima).
constexpr int SMEM_LIMIT = 232448 - 1024;

static size_t act_smem_bytes(int mv, int Kc, bool fused) {
  const size_t G = Kc / 512;
  // int8 rows | integer scales | fused: group scales, row quanta (TP_MAX_M), block sums
  return (size_t)mv * (Kc + 16) + 4 * (size_t)mv * G + (fused ? 8 * (size_t)mv * G + 4 * TP_MAX_M : 0);
}
static size_t table_smem_bytes() { return LUT_COPY_BYTES + LUT_BAR_BYTES; }

template <int BITS, bool M1, bool ACT_SMEM, bool FUSED>
static int launch_one(const GemvParams& p, int grid, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(trellis_sums_kernel<BITS, M1, ACT_SMEM, FUSED>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "trellis_sums_kernel attributes");
  const size_t smem = table_smem_bytes() + (ACT_SMEM ? act_smem_bytes(p.mv, p.Kc, FUSED) : 0);
  // Launched as a programmatic dependent of the previous kernel on the stream: the CTAs
  // may start on SMs that kernel has left and fetch their table and first codes while it
  // finishes (the kernel waits for it before touching its inputs or the scratch).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMV_WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_fail(cudaLaunchKernelEx(&cfg, trellis_sums_kernel<BITS, M1, ACT_SMEM, FUSED>, p), "trellis_sums_kernel");
}

template <int BITS>
static int launch_bits(const GemvParams& p, int grid, bool fused, cudaStream_t st) {
  if (fused)
    return p.mv == 1 ? launch_one<BITS, true, true, true>(p, grid, st) : launch_one<BITS, false, true, true>(p, grid, st);
  const bool fits = table_smem_bytes() + act_smem_bytes(p.mv, p.Kc, false) <= (size_t)SMEM_LIMIT;
  if (p.mv == 1)
    return fits ? launch_one<BITS, true, true, false>(p, grid, st) : launch_one<BITS, true, false, false>(p, grid, st);
  return fits ? launch_one<BITS, false, true, false>(p, grid, st) : launch_one<BITS, false, false, false>(p, grid, st);
}

static int launch_bits_any(int bits, const GemvParams& p, int grid, bool fused, cudaStream_t st) {
  switch (bits) {
    case 4: return launch_bits<4>(p, grid, fused, st);
    case 5: return launch_bits<5>(p, grid, fused, st);
    case 6: return launch_bits<6>(p, grid, fused, st);
    case 7: return launch_bits<7>(p, grid, fused, st);
    default: return launch_bits<8>(p, grid, fused, st);
  }
}

// Segments, CTA split and scratch for one call. The CTAs (one per SM) are split
// between the matrices in proportion to their units by largest remainders, so the
// grid never exceeds the SM count (a CTA beyond it would run as a second wave).
// full_grid (one matrix): exactly one CTA per SM, whatever the work (the row-parallel
// operator's launch epoch counts CTAs).
static int build_params(const MatrixDev* mats, int n_mats, const int* out_rows, const GemvScratch& scratch,
                        bool fused, GemvParams& p, int& grid, bool full_grid = false) {
  const int Kc = mats[0].cols, G = Kc / 512;
  const int sms = sm_count();
  p = GemvParams{};
  p.n_seg = n_mats;
  p.G = G;
  p.Kc = Kc;
  p.checked = G >= 512 ? 1 : 0;
  p.partials = scratch.partials;
  p.err = device_error_word();
  int64_t total = 0;  // tiles of the call
  for (int i = 0; i < n_mats; ++i) total += (int64_t)(mats[i].phys_pad8 / 8) * 2 * G;
  if (total >= (int64_t)1 << 31) return fail(YSKN_EINVAL, "gemv: matrix too large for one call");
  int64_t want[GEMV_MAX_SEG];
  if (p.checked) {
    for (int i = 0; i < n_mats; ++i) want[i] = ceil_div(mats[i].phys_pad8 / 8, GEMV_WARPS);  // a warp per row block
  } else {
    const int budget = std::max(sms, n_mats);
    double frac[GEMV_MAX_SEG];
    int64_t used = 0;
    for (int i = 0; i < n_mats; ++i) {
      const int64_t tiles = (int64_t)(mats[i].phys_pad8 / 8) * 2 * G;
      const double exact = (double)budget * tiles / total;
      want[i] = std::max<int64_t>(1, (int64_t)exact);
      frac[i] = exact - (double)(int64_t)exact;
      used += want[i];
    }
    while (used < budget) {  // hand the remaining CTAs to the largest remainders
      int best = 0;
      for (int i = 1; i < n_mats; ++i)
        if (frac[i] > frac[best]) best = i;
      ++want[best];
      frac[best] = -1.0;
      ++used;
    }
    while (used > budget) {  // only when a tiny segment was lifted to one CTA
      int big = 0;
      for (int i = 1; i < n_mats; ++i)
        if (want[i] > want[big]) big = i;
      --want[big];
      --used;
    }
    for (int i = 0; i < n_mats; ++i)  // no more CTAs than tile runs of 16 warps
      want[i] = std::max<int64_t>(1, std::min<int64_t>(want[i], ceil_div((int64_t)(mats[i].phys_pad8 / 8) * 2 * G,
                                                                          GEMV_WARPS)));
    if (full_grid && n_mats == 1) want[0] = sms;
  }
  grid = 0;
  unsigned* cnt = scratch.counters;
  for (int i = 0; i < n_mats; ++i) {
    GemvSeg& s = p.seg[i];
    s.codes = mats[i].codes;
    s.lutx = mats[i].lutx;
    s.row_blocks = mats[i].phys_pad8 / 8;
    s.tiles = (int64_t)s.row_blocks * 2 * G;
    s.out_rows = out_rows[i];
    s.out_ld = out_rows[i];
    s.counters = cnt;
    cnt += s.row_blocks;
    if (fused && mats[i].s_out) {
      s.blk_counters = cnt;
      cnt += s.row_blocks / 64;
    }
    s.cta_begin = grid;
    s.n_ctas = (int)want[i];
    const int64_t nw = want[i] * GEMV_WARPS;
    s.base = (int)(s.tiles / nw);
    s.rem = (int)(s.tiles % nw);
    grid += (int)want[i];
  }
  if ((int64_t)(cnt - scratch.counters) > scratch.n_counters ||
      (!p.checked && (int64_t)grid * GEMV_WARPS > scratch.max_warps))
    return fail(YSKN_EINVAL, "gemv: scratch too small for this call");
  return YSKN_OK;
}

int launch_gemv(const MatrixDev* mats, int n_mats, const int8_t* act, const int32_t* scales, int M, int64_t* const* out,
                const int* out_rows, const GemvScratch& scratch, cudaStream_t st) {
  const int Kc = mats[0].cols, G = Kc / 512;
  GemvParams p;
  int grid = 0;
  if (int rc = build_params(mats, n_mats, out_rows, scratch, false, p, grid)) return rc;
  for (int m0 = 0; m0 < M; m0 += 16) {
    const int mv = std::min(16, M - m0);
    p.act = act + (int64_t)m0 * Kc;
    p.scales = scales + (int64_t)m0 * G;
    p.mv = mv;
    for (int i = 0; i < n_mats; ++i) p.seg[i].out = out[i] + (int64_t)m0 * out_rows[i];
    if (int rc = launch_bits_any(mats[0].bits, p, grid, false, st)) return rc;
  }
  return YSKN_OK;
}

bool fused_linear_fits(int M, int Kc) {
  return M >= 1 && M <= 16 && Kc / 512 < 512 &&
         table_smem_bytes() + act_smem_bytes(M, Kc, true) <= (size_t)SMEM_LIMIT;
}

int launch_linear_fused(const MatrixDev* mats, int n_mats, const float* x, int M, const float* inv_rms,
                        float* const* y, const GemvScratch& scratch, cudaStream_t st, const FusedIO& io) {
  if (!fused_linear_fits(M, mats[0].cols)) return fail(YSKN_EINVAL, "fused linear: shape out of range");
  if (io.res_hidden && (n_mats != 1 || !mats[0].s_out || mats[0].rows != mats[0].phys || mats[0].rows % 512))
    return fail(YSKN_EINVAL, "fused linear: the residual output needs one rotated matrix of whole 512-row blocks");
  int out_rows[GEMV_MAX_SEG];
  for (int i = 0; i < n_mats; ++i) out_rows[i] = mats[i].phys;
  GemvParams p;
  int grid = 0;
  if (int rc = build_params(mats, n_mats, out_rows, scratch, true, p, grid)) return rc;
  p.x = x;
  p.s_in = mats[0].s_in;
  p.inv_rms = inv_rms;
  p.mv = M;
  p.q_act = io.q_act;
  p.q_alpha = io.q_alpha;
  p.q_bss = io.q_bss;
  p.q_eps = io.q_eps;
  p.inv_out = io.inv_out;
  p.res = ResidualOut{io.res_hidden, io.res_norm_w, io.res_next_signs, io.res_act, io.res_alpha, io.res_bss,
                      io.res_gate};
  p.rin = ResidualIn{io.rin_y, io.rin_h_in, io.rin_h_out, io.rin_norm_w, io.rin_gate_out, io.rin_inv_out, io.rin_eps};
  int64_t sums_used = 0;  // rotated rows add into the zero-kept scratch sums
  for (int i = 0; i < n_mats; ++i) {
    GemvSeg& s = p.seg[i];
    s.out = nullptr;
    if (mats[i].s_out) {
      s.out = reinterpret_cast<int64_t*>(scratch.fused_sums) + sums_used;
      sums_used += (int64_t)M * mats[i].phys;
      if (sums_used > scratch.fused_sums_len) return fail(YSKN_EINVAL, "fused linear: sums scratch too small");
    }
    s.tau = mats[i].tau;
    s.s_out = mats[i].s_out;
    s.y = y[i];
    s.y_rows = mats[i].rows;
    // With several tokens a warp restores the rotated blocks it completed after its last
    // unit (a 32-bit mask of them).
    if ((M > 1 || io.res_hidden) && mats[i].s_out && (s.base + 1) / (64 * 2 * (int64_t)p.G) + 2 > 32)
      return fail(YSKN_EINVAL, "fused linear: too many rows per warp");
  }

  return launch_bits_any(mats[0].bits, p, grid, true, st);
}

int launch_linear_rowpar(const MatrixDev& mat, const TpView& tp, const float* x_local, int M, const float* inv_rms,
                         float* y, const GemvScratch& scratch, cudaStream_t st, const FusedIO& io) {
  if (!fused_linear_fits(M, mat.cols) || M > TP_MAX_M)
    return fail(YSKN_EINVAL, "row-parallel linear: M must be 1..16 with the input in shared memory");
  if (!mat.s_out) return fail(YSKN_EINVAL, "row-parallel linear: the matrix needs an output rotation");
  if (io.q_bss) return fail(YSKN_EINVAL, "row-parallel linear: no input normalisation from block sums");
  if (io.res_hidden && (mat.rows != mat.phys || mat.rows % 512))
    return fail(YSKN_EINVAL, "row-parallel linear: the residual output needs whole 512-row blocks");
  if (mat.phys / 512 > tp.max_blocks) return fail(YSKN_EINVAL, "row-parallel linear: matrix taller than the exchange");
  const int out_rows = mat.phys;
  GemvParams p;
  int grid = 0;
  if (int rc = build_params(&mat, 1, &out_rows, scratch, true, p, grid, true)) return rc;
  if (grid != sm_count()) return fail(YSKN_EINVAL, "row-parallel linear: needs one CTA per SM");
  // A warp restores the blocks it completed after its last unit (a 32-bit mask of them).
  const int64_t span = p.seg[0].base + 1, per_blk = 64 * 2 * (int64_t)p.G;
  if (span / per_blk + 2 > 32) return fail(YSKN_EINVAL, "row-parallel linear: too many rows per warp");
  p.x = x_local;
  p.s_in = mat.s_in;
  p.inv_rms = inv_rms;
  p.mv = M;
  p.tp = tp;
  p.q_act = io.q_act;
  p.q_alpha = io.q_alpha;
  p.res = ResidualOut{io.res_hidden, io.res_norm_w, io.res_next_signs, io.res_act, io.res_alpha, io.res_bss,
                      io.res_gate};
  GemvSeg& s = p.seg[0];
  s.out = reinterpret_cast<int64_t*>(scratch.fused_sums);
  if ((int64_t)M * mat.phys > scratch.fused_sums_len) return fail(YSKN_EINVAL, "row-parallel linear: sums scratch");
  s.tau = mat.tau;
  s.s_out = mat.s_out;
  s.y = y;
  s.y_rows = mat.rows;
  return launch_bits_any(mat.bits, p, grid, true, st);
}

}  // namespace yskn
