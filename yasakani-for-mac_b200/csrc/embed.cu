// Coded embedding rows: the bf16 input vectors of tokens, decoded from a compressed
// `embed_tokens` tensor and up to two residual tables.
//
// Reference: Engine35's embedding set-up and launch (src/engine35.cpp:272-299), the
// block kernel q35_embed (src/q35_kernels.cu:1501-1522, 1527-1554, 1571-1574); scalar
// spec docs/spec/02_COMPRESSED_LINEAR.md:271-303. Per token and column i:
//   value[i] = f16 table[state(i)][i mod 2] * f16 row scale[token]    (binary32, one rounding)
//            (+ the same for each residual table, added in order)
// then per 512 columns H512 (ascending strides), * 1/sqrt(512), * the main table's
// input sign, rounded once to bf16. The tables keep their 16-bit values (no int8 table:
// an embedding is not a linear operator here).
//
// B200 design: one warp per (token, 512-column block); lane l holds columns 16l..16l+15
// of the block, which are steps 8(l%16)..+7 of sequence 2*block + l/16, so the states
// come from the codes as stored (row layout: each row's sequences are contiguous) with
// at most two word reads per state, the sums are exact per-element products, and the
// transform is the activation quantiser's warp H512 (same op order). A token outside the
// table raises DERR_RANGE (yskn_b200_status reports YSKN_EINVAL) and its row is zeros.
#include <cuda_bf16.h>

#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "quant.cuh"

namespace yskn {

constexpr int EMB_MAX_PARTS = 3;
constexpr int EMB_WARPS = 4;

struct EmbPart {
  const uint32_t* codes;  // row layout, rows * (cols / 256) * 4 * bits words
  const float* table;     // 8192 binary32 (exact copies of the binary16 table)
  const float* scale;     // rows binary32
  int bits;
};

struct EmbParams {
  EmbPart part[EMB_MAX_PARTS];
  int n_parts, rows, cols;
  const int8_t* signs;  // the main table's input signs, cols
  const int32_t* tokens;
  uint16_t* out;  // bf16 [M][cols]
  unsigned* err;
};

// The 12-bit state of step j of a sequence whose words start at w (docs/FORMAT.md:116-125):
// the 12 bits that end just after the step's own, zeros before the sequence start.
__device__ __forceinline__ uint32_t sequence_state(const uint32_t* w, int bits, int j) {
  const int e = bits * (j + 1);
  if (e < 12) return (__ldg(w) & ((1u << e) - 1u)) << (12 - e);
  const int p = e - 12, wi = p >> 5, sh = p & 31;
  uint32_t x = __ldg(w + wi) >> sh;
  if (sh > 20) x |= __ldg(w + wi + 1) << (32 - sh);  // the window reaches into the next word
  return x & 0xfffu;
}

__global__ void __launch_bounds__(EMB_WARPS * 32) embed_kernel(const __grid_constant__ EmbParams p, int m0) {
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x * EMB_WARPS + (threadIdx.x >> 5);
  if (blk >= p.cols / 512) return;
  const int m = m0 + blockIdx.y;
  const int token = __ldg(p.tokens + m);
  uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)m * p.cols + blk * 512 + 16 * lane);
  if (token < 0 || token >= p.rows) {
    if (lane == 0) raise_device_error(p.err, DERR_RANGE);
    dst[0] = make_uint4(0, 0, 0, 0);
    dst[1] = make_uint4(0, 0, 0, 0);
    return;
  }
  const int seqs = p.cols / 256, s = 2 * blk + (lane >> 4), j0 = 8 * (lane & 15);
  float v[16];
#pragma unroll
  for (int q = 0; q < EMB_MAX_PARTS; ++q) {
    if (q >= p.n_parts) break;
    const EmbPart& P = p.part[q];
    const uint32_t* w = P.codes + ((size_t)token * seqs + s) * (4 * P.bits);
    const float sc = __ldg(P.scale + token);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 t = __ldg(reinterpret_cast<const float2*>(P.table) + sequence_state(w, P.bits, j0 + k));
      const float a = __fmul_rn(t.x, sc), b = __fmul_rn(t.y, sc);
      v[2 * k] = q == 0 ? a : __fadd_rn(v[2 * k], a);
      v[2 * k + 1] = q == 0 ? b : __fadd_rn(v[2 * k + 1], b);
    }
  }
  hadamard512_warp(v, lane);
  const int8_t* sg = p.signs + blk * 512 + 16 * lane;
  uint32_t packed[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float a = __fmul_rn(__fmul_rn(v[2 * k], kHadamardNorm), (float)__ldg(sg + 2 * k));
    const float b = __fmul_rn(__fmul_rn(v[2 * k + 1], kHadamardNorm), (float)__ldg(sg + 2 * k + 1));
    packed[k] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
                ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
  }
  dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
}

}  // namespace yskn

using namespace yskn;

struct yskn_b200_embedding {
  EmbParams p{};
  void* mem = nullptr;  // every device copy in one allocation
};

extern "C" YSKN_B200_API yskn_b200_embedding* yskn_b200_embedding_create(int n_parts, const uint32_t* const* d_codes,
                                                                      const int* bits, int rows, int cols,
                                                                      const uint16_t* const* lut16_host,
                                                                      const uint16_t* const* scale16_host,
                                                                      const int8_t* signs_in_host) {
  if (n_parts < 1 || n_parts > EMB_MAX_PARTS || !d_codes || !bits || !lut16_host || !scale16_host || !signs_in_host ||
      rows <= 0 || cols <= 0 || cols % 512) {
    fail(YSKN_EINVAL, "embedding_create: 1..3 tables, rows > 0, cols a multiple of 512, non-null arguments");
    return nullptr;
  }
  for (int q = 0; q < n_parts; ++q)
    if (!d_codes[q] || !lut16_host[q] || !scale16_host[q] || bits[q] < 4 || bits[q] > 8) {
      fail(YSKN_EINVAL, "embedding_create: table " + std::to_string(q) + ": null pointer or bits outside 4..8");
      return nullptr;
    }
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  size_t code_bytes[EMB_MAX_PARTS], off_code[EMB_MAX_PARTS], off_table[EMB_MAX_PARTS], off_scale[EMB_MAX_PARTS];
  size_t total = 0;
  for (int q = 0; q < n_parts; ++q) {
    code_bytes[q] = (size_t)rows * (cols / 256) * 4 * bits[q] * 4;
    off_code[q] = total;
    total += up(code_bytes[q]);
    off_table[q] = total;
    total += up(8192 * sizeof(float));
    off_scale[q] = total;
    total += up((size_t)rows * sizeof(float));
  }
  const size_t off_signs = total;
  total += up((size_t)cols);
  std::unique_ptr<yskn_b200_embedding> e(new yskn_b200_embedding);
  cudaError_t err = cudaMalloc(&e->mem, total);
  if (err != cudaSuccess) {
    cuda_fail(err, "embedding_create: cudaMalloc");
    return nullptr;
  }
  char* base = static_cast<char*>(e->mem);
  std::vector<float> table(8192), scale((size_t)rows);
  for (int q = 0; q < n_parts && err == cudaSuccess; ++q) {
    for (int i = 0; i < 8192; ++i) table[i] = half_bits_to_float(lut16_host[q][i]);
    for (int r = 0; r < rows; ++r) scale[r] = half_bits_to_float(scale16_host[q][r]);
    err = cudaMemcpy(base + off_code[q], d_codes[q], code_bytes[q], cudaMemcpyDeviceToDevice);
    if (err == cudaSuccess) err = cudaMemcpy(base + off_table[q], table.data(), 8192 * sizeof(float), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
      err = cudaMemcpy(base + off_scale[q], scale.data(), (size_t)rows * sizeof(float), cudaMemcpyHostToDevice);
    e->p.part[q] = {reinterpret_cast<const uint32_t*>(base + off_code[q]),
                    reinterpret_cast<const float*>(base + off_table[q]),
                    reinterpret_cast<const float*>(base + off_scale[q]), bits[q]};
  }
  if (err == cudaSuccess) err = cudaMemcpy(base + off_signs, signs_in_host, (size_t)cols, cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    cudaFree(e->mem);
    cuda_fail(err, "embedding_create: copies");
    return nullptr;
  }
  e->p.n_parts = n_parts;
  e->p.rows = rows;
  e->p.cols = cols;
  e->p.signs = reinterpret_cast<const int8_t*>(base + off_signs);
  return e.release();
}

extern "C" YSKN_B200_API void yskn_b200_embedding_destroy(yskn_b200_embedding* e) {
  if (!e) return;
  cudaFree(e->mem);
  delete e;
}

extern "C" YSKN_B200_API int yskn_b200_embedding_lookup(const yskn_b200_embedding* e, const int32_t* d_tokens, int M,
                                                       uint16_t* d_out, void* stream) {
  if (!e || !d_tokens || !d_out || M < 1 || (reinterpret_cast<uintptr_t>(d_out) & 15) ||
      (reinterpret_cast<uintptr_t>(d_tokens) & 3))
    return fail(YSKN_EINVAL, "embedding_lookup: null handle, M < 1, or misaligned tokens/output (4 / 16 bytes)");
  EmbParams p = e->p;
  p.tokens = d_tokens;
  p.out = d_out;
  p.err = device_error_word();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned gx = (unsigned)((p.cols / 512 + EMB_WARPS - 1) / EMB_WARPS);
  for (int m0 = 0; m0 < M; m0 += 65535) {  // grid.y holds at most 65535 tokens per launch
    const unsigned gy = (unsigned)std::min(M - m0, 65535);
    embed_kernel<<<dim3(gx, gy), EMB_WARPS * 32, 0, st>>>(p, m0);
    if (cudaError_t err = cudaGetLastError()) return cuda_fail(err, "embed_kernel");
  }
  return YSKN_OK;
}
