// The C ABI (include/yskn_b200.h): matrix handles, argument checks, dispatch.
//
// Host-side arithmetic here (the int8 table and the effective row scales) follows
// crates/yskn-ref/src/compressed_linear.rs:138-158 and the reference loader
// src/loader.cpp:19-25; it is compiled with -ffp-contract=off so each binary32
// operation rounds once, as the Rust reference does.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace yskn {

__device__ unsigned g_device_error = 0;

unsigned* device_error_word() {
  static unsigned* words[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!words[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) words[dev] = reinterpret_cast<unsigned*>(p);
  }
  return words[dev];
}

static thread_local std::string t_last_error;

// Per-device scratch of the GEMV reduction, sized at matrix-creation time so the
// hot calls never allocate. Grows (synchronously) when a larger matrix is loaded.
struct DeviceScratch {
  GemvScratch s{};
  void* block = nullptr;
};
static DeviceScratch g_scratch[64];
static std::mutex g_scratch_mutex;

// rot_rows: physical rows of a matrix with an output rotation (0 without), whose
// fused decode operator adds its int64 sums into scratch.fused_sums.
static int ensure_scratch(int row_blocks, int64_t gemm_bytes, int64_t rot_rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(YSKN_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  DeviceScratch& d = g_scratch[dev];
  const int64_t want_sums = 3 * 16 * rot_rows;
  if (want_sums > d.s.fused_sums_len) {
    void* s = nullptr;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMalloc(&s, (size_t)want_sums * sizeof(long long));
    if (e == cudaSuccess) e = cudaMemset(s, 0, (size_t)want_sums * sizeof(long long));
    if (e != cudaSuccess) {
      if (s) cudaFree(s);
      return cuda_fail(e, "fused sums scratch");
    }
    if (d.s.fused_sums) cudaFree(d.s.fused_sums);
    d.s.fused_sums = reinterpret_cast<long long*>(s);
    d.s.fused_sums_len = want_sums;
  }
  if (gemm_bytes > d.s.gemm_w_bytes) {
    void* w = nullptr;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMalloc(&w, (size_t)gemm_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "gemm workspace");
    if (d.s.gemm_w) cudaFree(d.s.gemm_w);
    d.s.gemm_w = reinterpret_cast<int8_t*>(w);
    d.s.gemm_w_bytes = gemm_bytes;
  }
  // Row-block counters of up to 3 matrices per call, plus one per 512-row block for the fused restore.
  const int64_t want_counters = std::max<int64_t>(4 * (int64_t)row_blocks, 4096);
  const int64_t want_warps = gemv_max_warps();
  if (d.block && d.s.n_counters >= want_counters && d.s.max_warps >= want_warps) return YSKN_OK;
  const int64_t n_counters = std::max(want_counters, d.s.n_counters);
  const size_t part_bytes = (size_t)want_warps * 2 * 32 * 4 * sizeof(long long);
  const size_t bytes = part_bytes + (size_t)n_counters * sizeof(unsigned);
  void* block = nullptr;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMalloc(&block, bytes);
  if (e == cudaSuccess) e = cudaMemset(reinterpret_cast<char*>(block) + part_bytes, 0, bytes - part_bytes);
  if (e != cudaSuccess) {
    if (block) cudaFree(block);
    return cuda_fail(e, "gemv scratch");
  }
  if (d.block) cudaFree(d.block);
  d.block = block;
  d.s.partials = reinterpret_cast<long long*>(block);
  d.s.counters = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(block) + part_bytes);
  d.s.n_counters = n_counters;
  d.s.max_warps = want_warps;
  return YSKN_OK;
}

static const GemvScratch* current_scratch() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !g_scratch[dev].block) return nullptr;
  return &g_scratch[dev].s;
}

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return YSKN_OK;
  t_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return YSKN_ECUDA;
}

static float f16_to_f32(uint16_t bits) {  // crates/yskn-format/src/floats.rs:4-19
  const uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  const uint32_t exponent = (bits >> 10) & 0x1fu, fraction = bits & 0x3ffu;
  uint32_t out;
  if (exponent == 0 && fraction == 0) {
    out = sign;
  } else if (exponent == 0) {
    const uint32_t shift = (uint32_t)__builtin_clz(fraction) - 21u;
    out = sign | ((113u - shift) << 23) | (((fraction << shift) & 0x3ffu) << 13);
  } else if (exponent == 31) {
    out = sign | 0x7f800000u | (fraction << 13);
  } else {
    out = sign | ((exponent + 112u) << 23) | (fraction << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

float half_bits_to_float(uint16_t bits) { return f16_to_f32(bits); }

static void sign_stream(int rule, uint64_t seed, uint64_t offset, int64_t n, int8_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t position = offset + (uint64_t)i + 1u;
    bool positive;
    if (rule == YSKN_SIGNS_SPLITMIX64) {
      uint64_t v = seed + position * 0x9e3779b97f4a7c15ull;
      v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
      v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
      v ^= v >> 31;
      positive = (v >> 63) != 0;
    } else {
      uint32_t s0 = (uint32_t)seed * 7919u + 13u;
      if (s0 == 0) s0 = 0x9e3779b9u;
      uint32_t v = s0 + (uint32_t)position * 0x6d2b79f5u;
      v = (v ^ (v >> 15)) * (v | 1u);
      v ^= v + (v ^ (v >> 7)) * (v | 61u);
      v ^= v >> 14;
      positive = v >= 0x80000000u;
    }
    out[i] = positive ? 1 : -1;
  }
}

}  // namespace yskn

using namespace yskn;

struct yskn_b200_matrix {
  MatrixDev dev{};
  void* codes = nullptr;
  void* small = nullptr;  // lut8 | tau | s_in | s_out | lutx in one allocation
  int64_t packed_bytes = 0;
  bool has_rot = false;
};

namespace yskn {
const MatrixDev* matrix_dev(const yskn_b200_matrix* m) { return m ? &m->dev : nullptr; }
}  // namespace yskn

// One rank's side of the row-parallel exchange: its own area (cudaMalloc, shared by
// CUDA IPC) and the peers' areas mapped into this process.
struct yskn_b200_tp {
  TpView view{};
  void* local = nullptr;
  bool mapped[TP_MAX_WORLD] = {};
  bool connected = false;
};

static cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" {

YSKN_B200_API const char* yskn_b200_last_error(void) { return t_last_error.c_str(); }

YSKN_B200_API int yskn_b200_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "yskn_b200_status");
  unsigned bits = 0;
  const unsigned zero = 0;
  e = cudaMemcpyFromSymbol(&bits, g_device_error, sizeof bits);
  if (e == cudaSuccess && bits) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero);
  if (e != cudaSuccess) return cuda_fail(e, "yskn_b200_status");
  if (bits & DERR_TIMEOUT) return fail(YSKN_ETIMEDOUT, "a bounded device wait timed out");
  if (bits & DERR_OVERFLOW) return fail(YSKN_EOVERFLOW, "compressed integer accumulation exceeds i64");
  if (bits & DERR_NONFINITE) return fail(YSKN_ENONFINITE, "non-finite activation or restored value");
  if (bits & DERR_RANGE) return fail(YSKN_EINVAL, "a token id lies outside the embedding's rows");
  return YSKN_OK;
}

YSKN_B200_API int yskn_repack_warp_to_frag(const uint32_t* d_words, uint32_t* d_frag, int rows, int seqs, int wps,
                                           void* cuda_stream) {
  if (rows % 64 || wps % 4) return -1;  // src/repack.cu:22
  if (rows <= 0 || seqs <= 0 || wps <= 0 || !d_words || !d_frag) return fail(YSKN_EINVAL, "repack: bad arguments");
  return launch_repack_frag(d_words, d_frag, rows, seqs, wps, as_stream(cuda_stream));
}

YSKN_B200_API int yskn_repack_warp_to_frag_host(const uint32_t* h_words, uint32_t* h_frag, int rows, int seqs,
                                                int wps) {
  if (rows % 64 || wps % 4) return -1;
  if (rows <= 0 || seqs <= 0 || wps <= 0 || !h_words || !h_frag) return fail(YSKN_EINVAL, "repack: bad arguments");
  const size_t bytes = (size_t)rows * seqs * wps * 4;
  uint32_t *dw = nullptr, *df = nullptr;
  cudaError_t e = cudaMalloc(&dw, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&df, bytes);
  if (e == cudaSuccess) e = cudaMemcpy(dw, h_words, bytes, cudaMemcpyHostToDevice);
  int rc = e == cudaSuccess ? launch_repack_frag(dw, df, rows, seqs, wps, nullptr) : cuda_fail(e, "repack_host");
  if (rc == YSKN_OK) {
    e = cudaMemcpy(h_frag, df, bytes, cudaMemcpyDeviceToHost);
    rc = cuda_fail(e, "repack_host");
  }
  cudaFree(dw);
  cudaFree(df);
  return rc;
}

YSKN_B200_API int yskn_b200_signs(int rule, uint64_t seed, uint64_t offset, int64_t n, int8_t* h_out) {
  if ((rule != YSKN_SIGNS_SPLITMIX64 && rule != YSKN_SIGNS_MULBERRY32) || n < 0 || (n && !h_out))
    return fail(YSKN_EINVAL, "signs: bad arguments");
  sign_stream(rule, seed, offset, n, h_out);
  return YSKN_OK;
}

YSKN_B200_API int64_t yskn_b200_pack_bytes(int physical_rows, int cols, int bits) {
  if (physical_rows <= 0 || cols <= 0 || cols % 512 || bits < 4 || bits > 8) return -1;
  return ceil_div(physical_rows, 8) * 8 * (int64_t)(cols / 256) * bits * 16;
}

static int check_shape(int layout, int phys, int cols, int bits) {
  if (cols <= 0 || cols % 512 || phys <= 0 || bits < 4 || bits > 8 ||
      (layout != YSKN_LAYOUT_ROW && layout != YSKN_LAYOUT_WARP))
    return fail(YSKN_EINVAL, "invalid matrix dimensions, bits or layout");
  if (layout == YSKN_LAYOUT_WARP && ((int64_t)phys * (cols / 256)) % 32)
    return fail(YSKN_EINVAL, "warp layout requires a multiple of 32 sequences");
  return YSKN_OK;
}

YSKN_B200_API int yskn_b200_pack(const uint32_t* d_words, int layout, int physical_rows, int cols, int bits,
                                 void* d_out, void* stream) {
  if (int rc = check_shape(layout, physical_rows, cols, bits)) return rc;
  if (!d_words || !d_out || !aligned16(d_words) || !aligned16(d_out))
    return fail(YSKN_EINVAL, "pack: pointers must be non-null and 16-byte aligned");
  return launch_pack(d_words, layout, physical_rows, cols, bits, reinterpret_cast<uint32_t*>(d_out),
                     as_stream(stream));
}

// A matrix handle for physical rows [row0, row1) and columns [col0, col1) of a source
// tensor of src_rows x src_phys x src_cols (the whole tensor, or one tensor-parallel
// shard). The lookup table is per tensor, so every shard quantises it identically.
// A matrix handle for the physical rows of n_ranges ranges [row0, row1) (stored in
// that order: the handle's rows are the ranges' rows one after another) and columns
// [col0, col1) of a source tensor of src_rows x src_phys x src_cols (the whole tensor,
// one tensor-parallel shard, or the row blocks one rank needs of several parts of it).
static yskn_b200_matrix* create_matrix(const uint32_t* d_codes, int layout, int src_rows, int src_phys, int src_cols,
                                       int bits, const uint16_t* lut16_host, const uint16_t* scale16_src,
                                       const int8_t* signs_in_src, const int8_t* signs_out_src, int n_ranges,
                                       const int* ranges, int col0, int col1) {
  if (check_shape(layout, src_phys, src_cols, bits)) return nullptr;
  if (src_rows <= 0 || src_rows > src_phys) return fail(YSKN_EINVAL, "rows must be in 1..physical_rows"), nullptr;
  if (!d_codes || !aligned16(d_codes) || !lut16_host || !scale16_src || !signs_in_src)
    return fail(YSKN_EINVAL, "matrix_create: missing or misaligned input"), nullptr;
  if (n_ranges < 1 || n_ranges > 16 || !ranges)
    return fail(YSKN_EINVAL, "shard: 1 to 16 row ranges"), nullptr;
  if (col0 < 0 || col1 > src_cols || col0 >= col1 || col0 % 512 || col1 % 512)
    return fail(YSKN_EINVAL, "shard: columns must be whole 512-groups of the tensor"), nullptr;
  int physical_rows = 0, rows = 0;
  for (int k = 0; k < n_ranges; ++k) {
    const int r0 = ranges[2 * k], r1 = ranges[2 * k + 1];
    // Every range but the last holds real rows only, a whole number of 8-row blocks.
    if (r0 < 0 || r1 > src_phys || r0 >= r1 || r0 % 8 || r0 >= src_rows ||
        (k + 1 < n_ranges && (r1 > src_rows || (r1 - r0) % 8)))
      return fail(YSKN_EINVAL, "shard: rows [row0, row1) need row0 % 8 == 0 and real rows; every range but the last "
                               "whole 8-row blocks of real rows"),
             nullptr;
    if (signs_out_src && ((r1 - r0) % 512 || r0 % 512))
      return fail(YSKN_EINVAL, "an output rotation needs whole 512-row blocks"), nullptr;
    physical_rows += r1 - r0;
    rows += std::min(src_rows, r1) - r0;
  }
  const int cols = col1 - col0;
  std::vector<uint16_t> scale16_rows(physical_rows);
  std::vector<int8_t> signs_out_rows(signs_out_src ? physical_rows : 0);
  for (int k = 0, o = 0; k < n_ranges; ++k)
    for (int r = ranges[2 * k]; r < ranges[2 * k + 1]; ++r, ++o) {
      scale16_rows[o] = scale16_src[r];
      if (signs_out_src) signs_out_rows[o] = signs_out_src[r];
    }
  const uint16_t* scale16_host = scale16_rows.data();
  const int8_t* signs_in_host = signs_in_src + col0;
  const int8_t* signs_out_host = signs_out_src ? signs_out_rows.data() : nullptr;
  for (int i = 0; i < cols; ++i)
    if (signs_in_host[i] != 1 && signs_in_host[i] != -1) return fail(YSKN_EINVAL, "signs must be -1 or +1"), nullptr;
  if (signs_out_host)
    for (int i = 0; i < physical_rows; ++i)
      if (signs_out_host[i] != 1 && signs_out_host[i] != -1)
        return fail(YSKN_EINVAL, "signs must be -1 or +1"), nullptr;

  // compressed_linear.rs:138-158: one table maximum over all 8192 values.
  float table_maximum = 0.0f;
  for (int i = 0; i < 8192; ++i) {
    const float v = f16_to_f32(lut16_host[i]);
    if (!std::isfinite(v)) return fail(YSKN_EINVAL, "non-finite weight lookup table"), nullptr;
    table_maximum = std::fmax(table_maximum, std::fabs(v));
  }
  if (table_maximum == 0.0f)
    return fail(YSKN_EINVAL, "a compressed projection cannot use an all-zero lookup table (LIN-01)"), nullptr;
  const float table_scale = table_maximum / 127.0f;
  std::vector<int8_t> lut8(8192);
  for (int i = 0; i < 8192; ++i) {
    float r = std::nearbyint(f16_to_f32(lut16_host[i]) / table_scale);
    r = std::fmin(127.0f, std::fmax(-127.0f, r));
    lut8[i] = (int8_t)r;
  }
  std::vector<float> tau(physical_rows);
  for (int r = 0; r < physical_rows; ++r) {
    const float s = f16_to_f32(scale16_host[r]);
    tau[r] = s * table_scale;
    if (!std::isfinite(s) || !std::isfinite(tau[r]))
      return fail(YSKN_EINVAL, "non-finite weight row scales"), nullptr;
  }

  if (ensure_scratch((int)ceil_div(physical_rows, 8), ceil_div(physical_rows, 8) * 8 * (int64_t)cols,
                     signs_out_host ? physical_rows : 0))
    return nullptr;
  std::unique_ptr<yskn_b200_matrix> m(new yskn_b200_matrix);
  const int64_t packed = yskn_b200_pack_bytes(physical_rows, cols, bits);
  const size_t off_tau = 8192, off_sin = off_tau + ceil_div(4 * (int64_t)physical_rows, 256) * 256;
  const size_t off_sout = off_sin + ceil_div(cols, 256) * 256;
  const size_t off_lutx = off_sout + ceil_div(physical_rows, 256) * 256;
  const size_t small_bytes = off_lutx + 4096 * 32;
  // The GEMV's shared-memory image of the table (MatrixDev::lutx).
  std::vector<uint16_t> lutx(4096 * 16);
  auto pair = [&](uint32_t s) { return (uint16_t)((uint8_t)lut8[2 * s] | ((uint8_t)lut8[2 * s + 1] << 8)); };
  for (uint32_t e = 0; e < 4096 * 16; ++e) lutx[e] = pair(bits == 8 ? lutx8_state(2 * e) : lutx_split_state(2 * e));
  cudaError_t e = cudaMalloc(&m->codes, (size_t)packed);
  if (e == cudaSuccess) e = cudaMalloc(&m->small, small_bytes);
  if (e != cudaSuccess) {
    cudaFree(m->codes);
    cuda_fail(e, "matrix_create: cudaMalloc");
    return nullptr;
  }
  char* small = reinterpret_cast<char*>(m->small);
  e = cudaMemcpy(small, lut8.data(), 8192, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(small + off_lutx, lutx.data(), 4096 * 32, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(small + off_tau, tau.data(), 4 * (size_t)physical_rows, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(small + off_sin, signs_in_host, cols, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && signs_out_host)
    e = cudaMemcpy(small + off_sout, signs_out_host, physical_rows, cudaMemcpyHostToDevice);
  int rc = e == cudaSuccess ? YSKN_OK : cuda_fail(e, "matrix_create: copy");
  for (int k = 0, done = 0; k < n_ranges && rc == YSKN_OK; ++k) {  // each range's 8-row blocks after the previous
    const int r0 = ranges[2 * k], n = ranges[2 * k + 1] - r0;
    char* dst = reinterpret_cast<char*>(m->codes) + (int64_t)done * (cols / 256) * bits * 16;
    rc = launch_pack_range(d_codes, layout, src_phys, src_cols, r0, col0, n, cols, bits, reinterpret_cast<uint32_t*>(dst),
                           nullptr);
    done += n;
  }
  if (rc == YSKN_OK) rc = cuda_fail(cudaDeviceSynchronize(), "matrix_create: pack");
  if (rc != YSKN_OK) {
    cudaFree(m->codes);
    cudaFree(m->small);
    return nullptr;
  }
  m->packed_bytes = packed;
  m->has_rot = signs_out_host != nullptr;
  MatrixDev& d = m->dev;
  d.codes = reinterpret_cast<const uint32_t*>(m->codes);
  d.lut8 = reinterpret_cast<const uint16_t*>(small);
  d.lutx = reinterpret_cast<const uint8_t*>(small + off_lutx);
  d.tau = reinterpret_cast<const float*>(small + off_tau);
  d.s_in = reinterpret_cast<const int8_t*>(small + off_sin);
  d.s_out = m->has_rot ? reinterpret_cast<const int8_t*>(small + off_sout) : nullptr;
  d.rows = rows;
  d.phys = physical_rows;
  d.phys_pad8 = (int)ceil_div(physical_rows, 8) * 8;
  d.cols = cols;
  d.bits = bits;
  return m.release();
}

YSKN_B200_API yskn_b200_matrix* yskn_b200_matrix_create(const uint32_t* d_codes, int layout, int rows,
                                                        int physical_rows, int cols, int bits,
                                                        const uint16_t* lut16_host, const uint16_t* scale16_host,
                                                        const int8_t* signs_in_host, const int8_t* signs_out_host) {
  const int all[2] = {0, physical_rows};
  return create_matrix(d_codes, layout, rows, physical_rows, cols, bits, lut16_host, scale16_host, signs_in_host,
                       signs_out_host, 1, all, 0, cols);
}

YSKN_B200_API yskn_b200_matrix* yskn_b200_matrix_create_shard(const uint32_t* d_codes, int layout, int rows,
                                                              int physical_rows, int cols, int bits,
                                                              const uint16_t* lut16_host,
                                                              const uint16_t* scale16_host,
                                                              const int8_t* signs_in_host,
                                                              const int8_t* signs_out_host, int row_begin, int row_end,
                                                              int col_begin, int col_end) {
  const int range[2] = {row_begin, row_end};
  return create_matrix(d_codes, layout, rows, physical_rows, cols, bits, lut16_host, scale16_host, signs_in_host,
                       signs_out_host, 1, range, col_begin, col_end);
}

YSKN_B200_API yskn_b200_matrix* yskn_b200_matrix_create_rows(const uint32_t* d_codes, int layout, int rows,
                                                             int physical_rows, int cols, int bits,
                                                             const uint16_t* lut16_host,
                                                             const uint16_t* scale16_host,
                                                             const int8_t* signs_in_host,
                                                             const int8_t* signs_out_host, int n_ranges,
                                                             const int* row_ranges, int col_begin, int col_end) {
  return create_matrix(d_codes, layout, rows, physical_rows, cols, bits, lut16_host, scale16_host, signs_in_host,
                       signs_out_host, n_ranges, row_ranges, col_begin, col_end);
}

YSKN_B200_API int yskn_b200_rescale(const float* d_alpha, const float* d_row_max, int M, int groups,
                                    int32_t* d_scales, float* d_row_quantum, void* stream) {
  if (M < 1 || groups < 1 || !d_alpha || !d_row_max || !d_scales || !d_row_quantum)
    return fail(YSKN_EINVAL, "rescale: bad arguments");
  return launch_rescale(d_alpha, d_row_max, M, groups, d_scales, d_row_quantum, as_stream(stream));
}

YSKN_B200_API yskn_b200_tp* yskn_b200_tp_create(int world, int rank, int max_physical_rows, void* ipc_handle_out) {
  if (world < 2 || world > TP_MAX_WORLD || rank < 0 || rank >= world || max_physical_rows < 512 ||
      max_physical_rows % 512 || !ipc_handle_out)
    return fail(YSKN_EINVAL, "tp_create: need 2 <= world <= 8, 0 <= rank < world, rows a multiple of 512"), nullptr;
  std::unique_ptr<yskn_b200_tp> t(new yskn_b200_tp);
  t->view = tp_layout(world, rank, max_physical_rows / 512);
  cudaError_t e = cudaMalloc(&t->local, t->view.bytes);
  if (e == cudaSuccess) e = cudaMemset(t->local, 0, t->view.bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, t->local);
  if (e != cudaSuccess) {
    if (t->local) cudaFree(t->local);
    return cuda_fail(e, "tp_create"), nullptr;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == YSKN_B200_TP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle_out, &h, sizeof h);
  t->view.base[rank] = reinterpret_cast<char*>(t->local);
  return t.release();
}

YSKN_B200_API int yskn_b200_tp_connect(yskn_b200_tp* t, const void* handles) {
  if (!t || !handles || t->connected) return fail(YSKN_EINVAL, "tp_connect: bad arguments");
  const auto* h = reinterpret_cast<const unsigned char*>(handles);
  for (int q = 0; q < t->view.world; ++q) {
    if (q == t->view.rank) continue;
    cudaIpcMemHandle_t hq;
    std::memcpy(&hq, h + (size_t)q * YSKN_B200_TP_HANDLE_BYTES, sizeof hq);
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, hq, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "tp_connect: mapping a peer's exchange area");
    t->view.base[q] = reinterpret_cast<char*>(ptr);
    t->mapped[q] = true;
  }
  t->connected = true;
  return YSKN_OK;
}

YSKN_B200_API void* yskn_b200_tp_area(yskn_b200_tp* t) {
  if (!t) return fail(YSKN_EINVAL, "tp_area: null exchange"), nullptr;
  return t->local;
}

YSKN_B200_API int yskn_b200_tp_connect_peers(yskn_b200_tp* t, void* const* peer_areas) {
  if (!t || !peer_areas || t->connected) return fail(YSKN_EINVAL, "tp_connect_peers: bad arguments");
  for (int q = 0; q < t->view.world; ++q) {
    if (q == t->view.rank) continue;
    if (!peer_areas[q] || (reinterpret_cast<uintptr_t>(peer_areas[q]) & 255u))
      return fail(YSKN_EINVAL, "tp_connect_peers: a peer area is null or not 256-byte aligned");
  }
  for (int q = 0; q < t->view.world; ++q)
    if (q != t->view.rank) t->view.base[q] = reinterpret_cast<char*>(peer_areas[q]);
  t->connected = true;
  return YSKN_OK;
}

YSKN_B200_API int yskn_b200_tp_set_wait(yskn_b200_tp* t, double seconds) {
  if (!t || !(seconds >= 1e-6 && seconds <= 60.0)) return fail(YSKN_EINVAL, "tp_set_wait: need 1e-6 <= seconds <= 60");
  int dev = 0, khz = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
  if (e != cudaSuccess) return cuda_fail(e, "tp_set_wait");
  t->view.wait_cycles = std::max(1ll, (long long)(seconds * 1e3 * (double)khz));
  return YSKN_OK;
}

YSKN_B200_API void yskn_b200_tp_destroy(yskn_b200_tp* t) {
  if (!t) return;
  cudaDeviceSynchronize();
  for (int q = 0; q < t->view.world; ++q)
    if (t->mapped[q]) cudaIpcCloseMemHandle(t->view.base[q]);
  if (t->local) cudaFree(t->local);
  delete t;
}

YSKN_B200_API int yskn_b200_linear_rowpar(yskn_b200_tp* t, const yskn_b200_matrix* mat, const float* d_x_local, int M,
                                          const float* d_inv_rms, float* d_y, void* stream) {
  if (!t || !t->connected || !mat || !d_x_local || !d_y || !aligned16(d_x_local))
    return fail(YSKN_EINVAL, "linear_rowpar: bad arguments (connected exchange, matrix, aligned input, output)");
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear_rowpar: no matrix was created on this device");
  return launch_linear_rowpar(mat->dev, t->view, d_x_local, M, d_inv_rms, d_y, *sc, as_stream(stream));
}

YSKN_B200_API int yskn_b200_linear_rowpar_q8(yskn_b200_tp* t, const yskn_b200_matrix* mat, const int8_t* d_act_local,
                                             const float* d_alpha_local, int M, float* d_y, void* stream) {
  if (!t || !t->connected || !mat || !d_act_local || !d_alpha_local || !d_y || !aligned16(d_act_local))
    return fail(YSKN_EINVAL, "linear_rowpar_q8: bad arguments (connected exchange, matrix, aligned input, output)");
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear_rowpar_q8: no matrix was created on this device");
  FusedIO io;
  io.q_act = d_act_local;
  io.q_alpha = d_alpha_local;
  return launch_linear_rowpar(mat->dev, t->view, nullptr, M, nullptr, d_y, *sc, as_stream(stream), io);
}

YSKN_B200_API int yskn_b200_linear_rowpar_residual(yskn_b200_tp* t, const yskn_b200_matrix* mat,
                                                   const float* d_x_local, const int8_t* d_act_local,
                                                   const float* d_alpha_local, int M, uint16_t* d_hidden,
                                                   const uint16_t* d_norm_weight, const int8_t* d_next_signs,
                                                   int8_t* d_act_out, float* d_alpha_out, float* d_bss_out,
                                                   uint16_t* d_gate_out, void* stream) {
  if (!t || !t->connected || !mat || M < 1 || (!d_x_local == !d_act_local) || (d_act_local && !d_alpha_local) ||
      !d_hidden || !d_norm_weight || !d_next_signs || !d_act_out || !d_alpha_out || !d_bss_out ||
      (d_x_local && !aligned16(d_x_local)) || (d_act_local && !aligned16(d_act_local)) || !aligned16(d_act_out) ||
      (reinterpret_cast<uintptr_t>(d_hidden) & 3) || (d_gate_out && (reinterpret_cast<uintptr_t>(d_gate_out) & 3)))
    return fail(YSKN_EINVAL, "linear_rowpar_residual: bad arguments (connected exchange, exactly one of f32 or int8 "
                             "input, aligned buffers)");
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear_rowpar_residual: no matrix was created on this device");
  FusedIO io;
  io.q_act = d_act_local;
  io.q_alpha = d_alpha_local;
  io.res_hidden = d_hidden;
  io.res_norm_w = d_norm_weight;
  io.res_next_signs = d_next_signs;
  io.res_act = d_act_out;
  io.res_alpha = d_alpha_out;
  io.res_bss = d_bss_out;
  io.res_gate = d_gate_out;
  return launch_linear_rowpar(mat->dev, t->view, d_x_local, M, nullptr, nullptr, *sc, as_stream(stream), io);
}

YSKN_B200_API void yskn_b200_matrix_destroy(yskn_b200_matrix* m) {
  if (!m) return;
  cudaFree(m->codes);
  cudaFree(m->small);
  delete m;
}

YSKN_B200_API int yskn_b200_matrix_info(const yskn_b200_matrix* m, int64_t* out6) {
  if (!m || !out6) return fail(YSKN_EINVAL, "matrix_info: null argument");
  out6[0] = m->dev.rows;
  out6[1] = m->dev.phys;
  out6[2] = m->dev.cols;
  out6[3] = m->dev.bits;
  out6[4] = m->has_rot ? 1 : 0;
  out6[5] = m->packed_bytes;
  return YSKN_OK;
}

YSKN_B200_API const int8_t* yskn_b200_matrix_lut8(const yskn_b200_matrix* m) {
  return m ? reinterpret_cast<const int8_t*>(m->dev.lut8) : nullptr;
}
YSKN_B200_API const float* yskn_b200_matrix_tau(const yskn_b200_matrix* m) { return m ? m->dev.tau : nullptr; }
YSKN_B200_API const int8_t* yskn_b200_matrix_signs_in(const yskn_b200_matrix* m) { return m ? m->dev.s_in : nullptr; }
YSKN_B200_API const int8_t* yskn_b200_matrix_signs_out(const yskn_b200_matrix* m) {
  return m ? m->dev.s_out : nullptr;
}

static int check_group(const yskn_b200_matrix* const* mats, int n_mats) {
  if (!mats || n_mats < 1 || n_mats > 3) return fail(YSKN_EINVAL, "1 to 3 matrices per call");
  for (int i = 0; i < n_mats; ++i) {
    if (!mats[i]) return fail(YSKN_EINVAL, "null matrix");
    if (mats[i]->dev.cols != mats[0]->dev.cols || mats[i]->dev.bits != mats[0]->dev.bits)
      return fail(YSKN_EINVAL, "grouped matrices must share cols and bits");
  }
  return YSKN_OK;
}

// Skinny inputs stream the codes through the decode GEMV; from GEMM_MIN_M rows
// the weights are expanded once and multiplied on the tensor cores. Inputs of
// >= 512 groups stay on the GEMV, whose ordered variant checks every i64 add.
static int run_sums(const MatrixDev* devs, int n_mats, const int8_t* act, const int32_t* scales, int M,
                    int64_t* const* out, const int* rows, const GemvScratch& sc, cudaStream_t st) {
  if (M >= GEMM_MIN_M && devs[0].cols / 512 < 512) {
    for (int i = 0; i < n_mats; ++i) {
      if (gemm_workspace_bytes(devs[i]) > sc.gemm_w_bytes) return fail(YSKN_EINVAL, "gemm workspace too small");
      if (int rc = launch_gemm(devs[i], act, scales, M, out[i], rows[i], sc.gemm_w, st)) return rc;
    }
    return YSKN_OK;
  }
  return launch_gemv(devs, n_mats, act, scales, M, out, rows, sc, st);
}

static int finish_checked(int cols, void* stream) {
  // Overflow is only possible with at least 512 groups: |dot| < 2^23, |A| <= 2^31.
  if (cols / 512 < 512) return YSKN_OK;
  return yskn_b200_status(stream);
}

YSKN_B200_API int yskn_b200_weighted_sums(const yskn_b200_matrix* const* mats, int n_mats, const int8_t* d_act,
                                          const int32_t* d_scales, int M, int64_t* const* d_out, void* stream) {
  if (int rc = check_group(mats, n_mats)) return rc;
  if (M < 1 || !d_act || !d_scales || !d_out || !aligned16(d_act) || !aligned16(d_scales))
    return fail(YSKN_EINVAL, "weighted_sums: bad activation arguments");
  MatrixDev devs[3];
  int rows[3];
  for (int i = 0; i < n_mats; ++i) {
    if (!d_out[i]) return fail(YSKN_EINVAL, "weighted_sums: null output");
    devs[i] = mats[i]->dev;
    rows[i] = mats[i]->dev.phys;
  }
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "weighted_sums: no matrix was created on this device");
  if (int rc = run_sums(devs, n_mats, d_act, d_scales, M, d_out, rows, *sc, as_stream(stream))) return rc;
  return finish_checked(mats[0]->dev.cols, stream);
}

YSKN_B200_API int yskn_b200_weighted_sums_prefix(const yskn_b200_matrix* mat, const int8_t* d_act,
                                                 const int32_t* d_scales, int M, int n_rows, int64_t* d_out,
                                                 void* stream) {
  if (!mat) return fail(YSKN_EINVAL, "null matrix");
  if (M < 1 || !d_act || !d_scales || !d_out || !aligned16(d_act) || !aligned16(d_scales))
    return fail(YSKN_EINVAL, "weighted_sums_prefix: bad activation arguments");
  if (n_rows < 1 || n_rows > mat->dev.phys)
    return fail(YSKN_EINVAL, "requested projection rows exceed the physical row count");
  int rows = n_rows;
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "weighted_sums: no matrix was created on this device");
  if (int rc = run_sums(&mat->dev, 1, d_act, d_scales, M, &d_out, &rows, *sc, as_stream(stream))) return rc;
  return finish_checked(mat->dev.cols, stream);
}

YSKN_B200_API int yskn_b200_quantize(const float* d_x, const int8_t* d_signs, int M, int Kc, int8_t* d_act,
                                     float* d_alpha, int32_t* d_scales, float* d_row_quantum, void* stream) {
  if (M < 1 || Kc <= 0 || Kc % 512)
    return fail(YSKN_EINVAL, "activation and input signs must have matching, nonzero multiples of 512 elements");
  if (!d_x || !d_signs || !d_act || !d_alpha || !d_scales || !d_row_quantum || !aligned16(d_x) ||
      !aligned16(d_signs) || !aligned16(d_act))
    return fail(YSKN_EINVAL, "quantize: null or misaligned pointer");
  return launch_quantize(d_x, d_signs, M, Kc, d_act, d_alpha, d_scales, d_row_quantum, as_stream(stream));
}

YSKN_B200_API int yskn_b200_restore(int64_t* d_ws, const float* d_row_quantum, const float* d_inv_rms,
                                    const yskn_b200_matrix* mat, int M, int rotate_out, int n_rows, int clear_ws,
                                    float* d_y, void* stream) {
  if (!mat || M < 1 || !d_ws || !d_row_quantum || !d_y || !aligned16(d_ws))
    return fail(YSKN_EINVAL, "restore: bad arguments");
  if (n_rows < 1 || n_rows > mat->dev.phys) return fail(YSKN_EINVAL, "restore: row count out of range");
  if (rotate_out && !mat->dev.s_out)
    return fail(YSKN_EINVAL, "a body projection requires complete 512-row output rotations");
  return launch_restore(d_ws, mat->dev.phys, d_row_quantum, d_inv_rms, mat->dev.tau, rotate_out ? mat->dev.s_out : nullptr,
                        M, mat->dev.phys, n_rows, clear_ws, d_y, as_stream(stream));
}

// Work area of yskn_b200_linear: act8 | alpha | scales | row_quantum | ws[i].
struct LinearWork {
  size_t act, alpha, scales, rq, ws[3], total;
};

static LinearWork linear_work(const yskn_b200_matrix* const* mats, int n_mats, int M) {
  LinearWork w{};
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const int Kc = mats[0]->dev.cols, G = Kc / 512;
  size_t o = 0;
  w.act = o; o += up((size_t)M * Kc);
  w.alpha = o; o += up(4 * (size_t)M * G);
  w.scales = o; o += up(4 * (size_t)M * G);
  w.rq = o; o += up(4 * (size_t)M);
  for (int i = 0; i < n_mats; ++i) {
    w.ws[i] = o;
    o += up(8 * (size_t)M * mats[i]->dev.phys);
  }
  w.total = o;
  return w;
}

YSKN_B200_API int64_t yskn_b200_linear_work_bytes(const yskn_b200_matrix* const* mats, int n_mats, int M) {
  if (check_group(mats, n_mats) || M < 1) return -1;
  return (int64_t)linear_work(mats, n_mats, M).total;
}

YSKN_B200_API int yskn_b200_linear(const yskn_b200_matrix* const* mats, int n_mats, const float* d_x, int M,
                                   const float* d_inv_rms, void* d_work, float* const* d_y, void* stream) {
  if (int rc = check_group(mats, n_mats)) return rc;
  if (M < 1 || !d_x || !d_work || !d_y || !aligned16(d_x) || !aligned16(d_work))
    return fail(YSKN_EINVAL, "linear: bad arguments");
  const LinearWork w = linear_work(mats, n_mats, M);
  char* base = reinterpret_cast<char*>(d_work);
  int8_t* act = reinterpret_cast<int8_t*>(base + w.act);
  float* alpha = reinterpret_cast<float*>(base + w.alpha);
  int32_t* scales = reinterpret_cast<int32_t*>(base + w.scales);
  float* rq = reinterpret_cast<float*>(base + w.rq);
  const int Kc = mats[0]->dev.cols;
  cudaStream_t st = as_stream(stream);
  MatrixDev devs[3];
  int rows[3];
  int64_t* ws[3];
  for (int i = 0; i < n_mats; ++i) {
    if (!d_y[i]) return fail(YSKN_EINVAL, "linear: null output");
    devs[i] = mats[i]->dev;
    rows[i] = mats[i]->dev.phys;
    ws[i] = reinterpret_cast<int64_t*>(base + w.ws[i]);
  }
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear: no matrix was created on this device");
  if (fused_linear_fits(M, Kc)) {  // decode: one launch for the whole operator
    if (int rc = launch_linear_fused(devs, n_mats, d_x, M, d_inv_rms, d_y, *sc, st)) return rc;
    return finish_checked(Kc, stream);
  }
  if (int rc = launch_quantize(d_x, mats[0]->dev.s_in, M, Kc, act, alpha, scales, rq, st)) return rc;
  if (int rc = run_sums(devs, n_mats, act, scales, M, ws, rows, *sc, st)) return rc;
  for (int i = 0; i < n_mats; ++i) {
    const MatrixDev& d = mats[i]->dev;
    if (int rc = launch_restore(ws[i], d.phys, rq, d_inv_rms, d.tau, d.s_out, M, d.phys, d.rows, 0, d_y[i], st))
      return rc;
  }
  return finish_checked(Kc, stream);
}

YSKN_B200_API int yskn_b200_linear_q8(const yskn_b200_matrix* const* mats, int n_mats, const int8_t* d_act,
                                      const float* d_alpha, const float* d_bss, float eps, int M, float* d_inv_rms_out,
                                      float* const* d_y, void* stream) {
  if (int rc = check_group(mats, n_mats)) return rc;
  const int Kc = mats[0]->dev.cols;
  if (M < 1 || !d_act || !d_alpha || !d_y || !aligned16(d_act) || (d_bss && !(eps > 0.0f)))
    return fail(YSKN_EINVAL, "linear_q8: bad arguments (aligned int8 input, group scales, outputs, eps > 0 with bss)");
  if (!fused_linear_fits(M, Kc)) return fail(YSKN_EINVAL, "linear_q8: M must be 1..16 with the input in shared memory");
  MatrixDev devs[3];
  for (int i = 0; i < n_mats; ++i) {
    if (!d_y[i]) return fail(YSKN_EINVAL, "linear_q8: null output");
    devs[i] = mats[i]->dev;
  }
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear_q8: no matrix was created on this device");
  FusedIO io;
  io.q_act = d_act;
  io.q_alpha = d_alpha;
  io.q_bss = d_bss;
  io.q_eps = eps;
  io.inv_out = d_bss ? d_inv_rms_out : nullptr;
  if (int rc = launch_linear_fused(devs, n_mats, nullptr, M, nullptr, d_y, *sc, as_stream(stream), io)) return rc;
  return finish_checked(Kc, stream);
}

YSKN_B200_API int yskn_b200_linear_residual(const yskn_b200_matrix* mat, const float* d_x, const int8_t* d_act,
                                            const float* d_alpha, int M, uint16_t* d_hidden,
                                            const uint16_t* d_norm_weight, const int8_t* d_next_signs,
                                            int8_t* d_act_out, float* d_alpha_out, float* d_bss_out,
                                            uint16_t* d_gate_out, void* stream) {
  if (!mat || M < 1 || (!d_x == !d_act) || (d_act && !d_alpha) || !d_hidden || !d_norm_weight || !d_next_signs ||
      !d_act_out || !d_alpha_out || !d_bss_out || (d_x && !aligned16(d_x)) || (d_act && !aligned16(d_act)) ||
      !aligned16(d_act_out) || (reinterpret_cast<uintptr_t>(d_hidden) & 3) ||
      (d_gate_out && (reinterpret_cast<uintptr_t>(d_gate_out) & 3)))
    return fail(YSKN_EINVAL, "linear_residual: bad arguments (exactly one of f32 or int8 input, aligned buffers)");
  const MatrixDev& d = mat->dev;
  if (!fused_linear_fits(M, d.cols))
    return fail(YSKN_EINVAL, "linear_residual: M must be 1..16 with the input in shared memory");
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear_residual: no matrix was created on this device");
  FusedIO io;
  io.q_act = d_act;
  io.q_alpha = d_alpha;
  io.res_hidden = d_hidden;
  io.res_norm_w = d_norm_weight;
  io.res_next_signs = d_next_signs;
  io.res_act = d_act_out;
  io.res_alpha = d_alpha_out;
  io.res_bss = d_bss_out;
  io.res_gate = d_gate_out;
  float* no_y[1] = {nullptr};
  if (int rc = launch_linear_fused(&d, 1, d_x, M, nullptr, no_y, *sc, as_stream(stream), io)) return rc;
  return finish_checked(d.cols, stream);
}

YSKN_B200_API int yskn_b200_linear_from_residual(const yskn_b200_matrix* const* mats, int n_mats, const float* d_y_prev,
                                                 const uint16_t* d_hidden_in, uint16_t* d_hidden_out,
                                                 const uint16_t* d_norm_weight, float eps, int M, uint16_t* d_gate_out,
                                                 float* d_inv_rms_out, float* const* d_y, void* stream) {
  if (int rc = check_group(mats, n_mats)) return rc;
  const int Kc = mats[0]->dev.cols;
  if (M < 1 || !d_y_prev || !d_hidden_in || !d_hidden_out || !d_norm_weight || !d_y || !(eps > 0.0f) ||
      d_hidden_in == d_hidden_out || !aligned16(d_y_prev) || (reinterpret_cast<uintptr_t>(d_hidden_in) & 3) ||
      (reinterpret_cast<uintptr_t>(d_hidden_out) & 3) || (reinterpret_cast<uintptr_t>(d_norm_weight) & 3) ||
      (d_gate_out && (reinterpret_cast<uintptr_t>(d_gate_out) & 3)))
    return fail(YSKN_EINVAL, "linear_from_residual: bad arguments (aligned buffers, two residual buffers, eps > 0)");
  if (!fused_linear_fits(M, Kc))
    return fail(YSKN_EINVAL, "linear_from_residual: M must be 1..16 with the input in shared memory");
  MatrixDev devs[3];
  for (int i = 0; i < n_mats; ++i) {
    if (!d_y[i]) return fail(YSKN_EINVAL, "linear_from_residual: null output");
    devs[i] = mats[i]->dev;
  }
  const GemvScratch* sc = current_scratch();
  if (!sc) return fail(YSKN_EINVAL, "linear_from_residual: no matrix was created on this device");
  FusedIO io;
  io.rin_y = d_y_prev;
  io.rin_h_in = d_hidden_in;
  io.rin_h_out = d_hidden_out;
  io.rin_norm_w = d_norm_weight;
  io.rin_gate_out = d_gate_out;
  io.rin_inv_out = d_inv_rms_out;
  io.rin_eps = eps;
  if (int rc = launch_linear_fused(devs, n_mats, nullptr, M, nullptr, d_y, *sc, as_stream(stream), io)) return rc;
  return finish_checked(Kc, stream);
}

static int kv_check(int M, int n_qh, int n_kvh, int length, int capacity, int kb, int n_splits) {
  if (M < 1 || n_qh < 1 || n_kvh < 1 || n_qh % n_kvh != 0 || n_qh / n_kvh > KV_MAX_GROUP)
    return fail(YSKN_EINVAL, "kv4 attention: query heads must be a multiple (at most 8x) of the KV heads");
  if (length < M || capacity < length) return fail(YSKN_EINVAL, "kv4 attention: need M <= length <= capacity");
  if (kb != 4) return fail(YSKN_EINVAL, "kv4 attention: only kb = 4 packed rows are supported");
  if (n_splits < -1 || n_splits > KV_MAX_SPLITS) return fail(YSKN_EINVAL, "kv4 attention: n_splits outside [-1, 64]");
  return YSKN_OK;
}

YSKN_B200_API int64_t yskn_b200_kv4_attention_work_bytes(int M, int n_query_heads, int length, int n_splits) {
  if (M < 1 || n_query_heads < 1 || length < M || n_splits < -1 || n_splits > KV_MAX_SPLITS) return -1;
  if (n_splits < 0) return 4 * kv_partials_floats(M, n_query_heads, KV_MAX_SPLITS);  // depends on the device
  KvArgs a{};
  a.M = M;
  a.length = length;
  a.n_splits = n_splits;
  return 4 * kv_partials_floats(M, n_query_heads, kv_max_splits(a));
}

YSKN_B200_API int yskn_b200_kv4_attention(const uint16_t* d_q, const uint16_t* d_gate, const uint32_t* d_k_rows,
                                          const float* d_k_scales, const uint32_t* d_v_rows, const float* d_v_scales,
                                          const uint16_t* d_k_codebook, const uint16_t* d_v_codebook,
                                          const float* d_v_mean, int M, int n_query_heads, int n_kv_heads, int length,
                                          int capacity, int kb, int n_splits, void* d_work, float* d_attended,
                                          uint16_t* d_out, void* stream) {
  if (int rc = kv_check(M, n_query_heads, n_kv_heads, length, capacity, kb, n_splits)) return rc;
  if (!d_q || !d_k_rows || !d_k_scales || !d_v_rows || !d_v_scales || !d_k_codebook || !d_v_codebook || !d_work ||
      !d_out)
    return fail(YSKN_EINVAL, "kv4 attention: null argument");
  if (!aligned16(d_k_rows) || !aligned16(d_v_rows) || !aligned16(d_work) || !aligned16(d_q) || !aligned16(d_out) ||
      (d_attended && !aligned16(d_attended)) || (d_gate && !aligned16(d_gate)))
    return fail(YSKN_EINVAL, "kv4 attention: queries, gate, rows, outputs and work area must be 16-byte aligned");
  KvArgs a{};
  a.q = d_q;
  a.gate = d_gate;
  a.kw = d_k_rows;
  a.ks = d_k_scales;
  a.vw = d_v_rows;
  a.vs = d_v_scales;
  a.kbase = d_k_codebook;
  a.vbase = d_v_codebook;
  a.vmean = d_v_mean;
  a.partials = reinterpret_cast<float*>(d_work);
  a.attended = d_attended;
  a.out = d_out;
  a.M = M;
  a.n_qh = n_query_heads;
  a.n_kvh = n_kv_heads;
  a.length = length;
  a.capacity = capacity;
  a.kb = kb;
  a.n_splits = n_splits;
  return launch_kv4_attention(a, as_stream(stream));
}

YSKN_B200_API int yskn_b200_kv_encode(const float* d_rows, const int32_t* d_row_group, int n_rows,
                                      const int16_t* d_tables, const float* d_gains, const float* d_means,
                                      const uint8_t* d_has_mean, const float* d_mults, int n_mult, int kb, int vit2,
                                      const int64_t* d_dest, uint32_t* d_words, float* d_scales, void* stream) {
  if (n_rows < 1 || n_rows > 65535) return fail(YSKN_EINVAL, "kv encode: n_rows outside [1, 65535]");
  if (n_mult < 1 || n_mult > 16) return fail(YSKN_EINVAL, "kv encode: 1 to 16 scale multipliers");
  if (kb != 4 && kb != 5) return fail(YSKN_EINVAL, "kv encode: packed rows have 4 or 5 bits per channel");
  if (!d_rows || !d_row_group || !d_tables || !d_gains || !d_mults || !d_words || !d_scales)
    return fail(YSKN_EINVAL, "kv encode: null argument");
  KvEncArgs a{};
  a.rows = d_rows;
  a.row_group = d_row_group;
  a.tables = d_tables;
  a.gains = d_gains;
  a.means = d_means;
  a.has_mean = d_has_mean;
  a.mults = d_mults;
  a.dest = d_dest;
  a.words = d_words;
  a.scales = d_scales;
  a.n_rows = n_rows;
  a.n_mult = n_mult;
  a.kb = kb;
  a.vit2 = vit2 ? 1 : 0;
  return launch_kv_encode(a, as_stream(stream));
}

}  // extern "C"
