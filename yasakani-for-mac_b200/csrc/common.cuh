// Shared declarations of the B200 compressed-linear library (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "yskn_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library is written for sm_100a (B200) only"
#endif

namespace yskn {

// Device-side error word: kernels OR in one of these bits; yskn_b200_status()
// reads and clears it. Never a trap, never a fault.
enum : unsigned {
  DERR_NONFINITE = 1u,
  DERR_OVERFLOW = 2u,
  DERR_TIMEOUT = 4u,
  DERR_RANGE = 8u,  // an index read on the device (a token id) lies outside its table
};
// Address of this device's error word (a __device__ variable in api.cu).
unsigned* device_error_word();

__device__ __forceinline__ void raise_device_error(unsigned* word, unsigned bits) { atomicOr(word, bits); }

// Programmatic dependent launch for the small kernels between operators: launched with
// launch_pdl, a kernel may be scheduled while the previous kernel of the stream drains; its
// first statement, pdl_begin(), waits for that kernel's completion and memory (before any
// access to memory) and then lets the next kernel of the stream be scheduled early, so a
// following operator loads its tables while this kernel runs. Both are no-ops in a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Thread-local error message (src/c_api.cpp:11-14 keeps one per thread as well).
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* where);
// IEEE binary16 bits -> binary32, exact (crates/yskn-format/src/floats.rs:4-19).
float half_bits_to_float(uint16_t bits);

// 1/sqrt(512) as the binary32 literal 0.044194173824159216f (bits 0x3d3504f3).
constexpr float kHadamardNorm = 0.044194173824159216f;

// bits = 8: the streaming layout stores every byte c of the code stream with its bits
// moved, b = file byte: c[0,1] = b[4,5], c[2..5] = b[0..3], c[6,7] = b[6,7]. A 12-bit
// state is the high nibble of byte i-1 and all of byte i, so in the 16 stored bits of
// bytes i-1, i the state's bits sit at 0,1 and 6..15 and bits 2..5 (the low nibble of
// byte i-1) are not part of it. Shifted left by one, those four bits land on the
// table image's copy field (address bits 3..6): the GEMV forms a lookup address with
// one shift and one LOP3 while each table copy spans two banks (gemv.cu).
__host__ __device__ inline uint32_t stream8_store(uint32_t b) {
  return ((b >> 4) & 0x03030303u) | ((b & 0x0f0f0f0fu) << 2) | (b & 0xc0c0c0c0u);
}
__host__ __device__ inline uint32_t stream8_load(uint32_t c) {
  return ((c & 0x03030303u) << 4) | ((c >> 2) & 0x0f0f0f0fu) | (c & 0xc0c0c0c0u);
}
// The state whose entry the bits = 8 table image holds at byte address a (even,
// < 128 KiB): address bit j is stored bit j-1 of bytes (i-1, i); bits 3..6 pick the copy.
__host__ __device__ inline uint32_t lutx8_state(uint32_t a) {
  const uint32_t c_prev = ((a >> 1) & 3u) | (((a >> 7) & 3u) << 6);  // stored byte i-1, bits 2..5 unused
  const uint32_t c_cur = (a >> 9) & 0xffu;                           // stored byte i
  const uint32_t b_prev = stream8_load(c_prev), b_cur = stream8_load(c_cur);
  return (b_prev >> 4) | (b_cur << 4);
}

// The state whose entry the table image of the other widths holds at byte address a
// (even, < 128 KiB): address bits 1, 2 are state bits 0, 1, bits 7..16 state bits 2..11;
// bits 3..6 pick the copy.
__host__ __device__ inline uint32_t lutx_split_state(uint32_t a) {
  return ((a >> 1) & 3u) | (((a >> 7) & 0x3ffu) << 2);
}

struct MatrixDev {
  const uint32_t* codes;  // B200 streaming layout (see pack.cu)
  const uint16_t* lut8;   // 4096 entries: int8 pair (component 0 low byte, component 1 high byte)
  // The GEMV's shared-memory image of lut8 (128 KiB, 16 copies). bits = 8: the entry of
  // lutx8_state(a) at every even byte address a, copy (a >> 3) & 15 in banks 2c, 2c+1;
  // other bits: the same with lutx_split_state(a).
  const uint8_t* lutx;
  const float* tau;       // effective row scale, f32[physical_rows]
  const int8_t* s_in;     // i8[cols]
  const int8_t* s_out;    // i8[physical_rows] or nullptr
  int rows, phys, phys_pad8, cols, bits;
};

// Scratch of the decode GEMV's split-row-block reduction (gemv.cu): per-warp i64
// partials and one arrival counter per 8-row block (zero between launches); for the
// fused operator's rotated rows, int64 sums that every contributing warp adds into
// (zero between launches: the warp that restores a 512-row block clears it).
struct GemvScratch {
  long long* partials;  // [2 * max_warps][32][4]
  unsigned* counters;   // [n_counters], zeroed at allocation, reset by the kernel
  int64_t n_counters;
  int64_t max_warps;
  long long* fused_sums;   // [fused_sums_len], zeroed at allocation, cleared by the kernel
  int64_t fused_sums_len;  // >= 16 tokens x the physical rows of any 3 rotated matrices
  int8_t* gemm_w;        // dense int8 weights of one matrix for the GEMM path
  int64_t gemm_w_bytes;
};

constexpr int GEMV_WARPS = 16;  // warps per persistent GEMV CTA (one CTA per SM)
int gemv_max_warps();

// Exchange areas of the tensor-parallel row-parallel operator (gemv.cu). Every rank
// allocates one area with this layout (zeroed); base[q] is rank q's area as mapped in
// this process (peer memory through CUDA IPC over NVLink; base[rank] is local).
// Every exchanged 32-bit datum travels as one 64-bit word (datum | launch epoch << 32),
// a single-copy-atomic access: the receiver polls the words themselves until they
// carry its epoch, so no fences are needed. Double-buffered by launch parity.
constexpr int TP_MAX_WORLD = 8;
constexpr int TP_MAX_M = 16;
struct TpView {
  char* base[TP_MAX_WORLD];
  int world, rank;
  int max_blocks;                   // 512-row blocks of the largest matrix
  size_t off_counter;               // u64: launches x CTAs on this rank (the epoch source)
  size_t off_maxbox;                // u64 [2][world][TP_MAX_M]: row maxima (f32 bits) by source rank
  size_t off_recv;                  // u64 x2 [2][world][TP_MAX_M][max_blocks * 512]: int64 block sums by source
  size_t bytes;
  long long wait_cycles;            // limit of each wait phase on the peers, in SM clock cycles
};
constexpr long long TP_DEFAULT_WAIT_CYCLES = 2000000000ll;  // ~1 s at B200 clocks
inline TpView tp_layout(int world, int rank, int max_blocks) {
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  TpView v{};
  v.world = world;
  v.rank = rank;
  v.max_blocks = max_blocks;
  v.off_counter = 0;
  v.off_maxbox = 256;
  v.off_recv = v.off_maxbox + up(2 * (size_t)world * TP_MAX_M * 8);
  v.bytes = v.off_recv + up(2 * (size_t)world * TP_MAX_M * max_blocks * 512 * 16);
  v.wait_cycles = TP_DEFAULT_WAIT_CYCLES;
  return v;
}

// Activation rows from which the tcgen05 GEMM (gemm.cu) replaces the GEMV.
constexpr int GEMM_MIN_M = 64;
int64_t gemm_workspace_bytes(const MatrixDev& m);  // dense int8 copy of the weights
int launch_gemm(const MatrixDev& m, const int8_t* act, const int32_t* scales, int M, int64_t* out, int out_rows,
                int8_t* W, cudaStream_t st);

// The device view of a matrix handle (nullptr for a null handle).
const MatrixDev* matrix_dev(const yskn_b200_matrix* m);

// Launchers (one per .cu file).
int launch_gemv(const MatrixDev* mats, int n_mats, const int8_t* act, const int32_t* scales, int M, int64_t* const* out,
                const int* out_rows, const GemvScratch& scratch, cudaStream_t st);
// The whole decode operator in one launch (quantise, sums, restore): M <= 16 rows
// whose activations fit in shared memory next to the table, fewer than 512 groups.
bool fused_linear_fits(int M, int Kc);
// The f1 chain's options of the fused operator (all null: plain f32 input, f32 output).
// Quantised input: q_act [M][Kc] int8 and q_alpha [M][Kc/512] group scales from the
// producing kernel (the in-kernel quantiser is skipped); with q_bss [M][Kc/512] block sums
// of squares the rows' 1/rms is formed in the kernel (and stored to inv_out if given).
// Residual output (res_hidden set; one matrix with an output rotation, rows a multiple of
// 512): the restored rows are added to the bf16 residual stream, which is normalised with
// res_norm_w and quantised with the next operator's input signs res_next_signs into
// res_act / res_alpha, its block sums of squares into res_bss, and (if res_gate) a bf16
// copy of the unnormalised input; y is not written.
struct FusedIO {
  const int8_t* q_act = nullptr;
  const float* q_alpha = nullptr;
  const float* q_bss = nullptr;
  float q_eps = 0.0f;
  float* inv_out = nullptr;
  uint16_t* res_hidden = nullptr;
  const uint16_t* res_norm_w = nullptr;
  const int8_t* res_next_signs = nullptr;
  int8_t* res_act = nullptr;
  float* res_alpha = nullptr;
  float* res_bss = nullptr;
  uint16_t* res_gate = nullptr;
  const float* rin_y = nullptr;  // residual prologue (GemvParams::rin)
  const uint16_t* rin_h_in = nullptr;
  uint16_t* rin_h_out = nullptr;
  const uint16_t* rin_norm_w = nullptr;
  uint16_t* rin_gate_out = nullptr;
  float* rin_inv_out = nullptr;
  float rin_eps = 0.0f;
};
int launch_linear_fused(const MatrixDev* mats, int n_mats, const float* x, int M, const float* inv_rms,
                        float* const* y, const GemvScratch& scratch, cudaStream_t st, const FusedIO& io = FusedIO());
// Gated product followed by the down projection's quantiser (per 512-element group):
// act [M][n] int8 and alpha [M][n/512] (n a multiple of 512).
int launch_gated_product_q8(const float* gate, const float* up, int M, int n, const int8_t* signs, int8_t* act,
                            float* alpha, cudaStream_t st);
// The row-parallel operator of one rank in one launch: this rank's 512-column groups
// of a matrix with an output rotation, the row maxima and the int64 block sums
// exchanged with the peers through `tp`, the whole output restored on every rank.
// With io: an int8 input (q_act, q_alpha) instead of x_local, and the residual epilogue
// (res_*) instead of y, as in launch_linear_fused.
int launch_linear_rowpar(const MatrixDev& mat, const TpView& tp, const float* x_local, int M, const float* inv_rms,
                         float* y, const GemvScratch& scratch, cudaStream_t st, const FusedIO& io = FusedIO());
int launch_quantize(const float* x, const int8_t* signs, int M, int Kc, int8_t* act, float* alpha, int32_t* scales,
                    float* row_quantum, cudaStream_t st);
int launch_restore(int64_t* ws, int ws_ld, const float* row_quantum, const float* inv_rms, const float* tau,
                   const int8_t* s_out, int M, int phys, int n_rows, int clear_ws, float* y, cudaStream_t st);
int launch_pack(const uint32_t* words, int layout, int phys, int cols, int bits, uint32_t* out, cudaStream_t st);
int launch_pack_range(const uint32_t* words, int layout, int src_phys, int src_cols, int row0, int col0, int phys,
                      int cols, int bits, uint32_t* out, cudaStream_t st);
// Integer grid of each activation row from a given row maximum of the group scales
// (tensor parallelism: the maximum over all ranks' groups).
int launch_rescale(const float* alpha, const float* row_max, int M, int G, int32_t* scales, float* row_quantum,
                   cudaStream_t st);
int launch_repack_frag(const uint32_t* w, uint32_t* f, int rows, int seqs, int wps, cudaStream_t st);

// Quantised-KV decode attention (kvattn.cu). Query row m of M sees cache rows
// [0, length - M + m], the last of which is its own (the self term).
struct KvArgs {
  const uint16_t* q;      // bf16 [M][n_qh][256], cache-rotated
  const uint32_t* kw;     // [n_kvh][capacity][8*kb] packed key rows
  const float* ks;        // [n_kvh][capacity]
  const uint32_t* vw;     // [n_kvh][capacity][8*kb] packed value rows
  const float* vs;        // [n_kvh][capacity]
  const uint16_t* kbase;  // bf16 [n_kvh][256] codebooks
  const uint16_t* vbase;
  const float* vmean;     // [n_kvh][256] or nullptr
  const uint16_t* gate;   // bf16 [M][n_qh][256] or nullptr
  float* partials;        // kv_partials_floats(...) floats
  float* attended;        // f32 [M][n_qh][256] before the inverse rotation, or nullptr
  uint16_t* out;          // bf16 [M][n_qh][256]
  int M, n_qh, n_kvh, length, capacity, kb, n_splits;  // n_splits 0: 31 below 4096 rows, else 42
};
constexpr int KV_MAX_SPLITS = 64;
constexpr int KV_MAX_GROUP = 8;        // query heads per KV head
constexpr int KV_MAX_ARRIVALS = 4096;  // (query row, KV head) pairs per launch
int kv_max_splits(const KvArgs& a);
int64_t kv_partials_floats(int M, int n_qh, int max_splits);
int launch_kv4_attention(const KvArgs& a, cudaStream_t st);

// Quantised-KV row encoder for packed rows (kvenc.cu).
struct KvEncArgs {
  const float* rows;         // f32 [n_rows][256] (cache-rotated)
  const int32_t* row_group;  // [n_rows] profile group of each row
  const int16_t* tables;     // [n_groups][256] trellis table codes
  const float* gains;        // [n_groups]
  const float* means;        // [n_groups][256] or nullptr
  const uint8_t* has_mean;   // [n_groups] or nullptr
  const float* mults;        // [n_mult] profile scale multipliers
  const int64_t* dest;       // [n_rows] destination row, or nullptr (row i)
  uint32_t* words;           // [*][8*kb]
  float* scales;             // [*]
  int n_rows, n_mult, kb, vit2;
};
int launch_kv_encode(const KvEncArgs& a, cudaStream_t st);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace yskn
