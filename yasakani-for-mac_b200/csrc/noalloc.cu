// yskn_b200_weighted_sums_noalloc: the decode GEMV with its scratch in a static
// device array, for callers that must not have the library allocate device memory.
//
// Who needs it: a serving process that handed almost all of HBM to its own pool
// at start-up, or a latency-critical decode loop in which a cudaMalloc/cudaFree
// could synchronise the device. yskn_b200_weighted_sums allocates nothing per
// call either, but its reduction scratch is allocated (and grown) per device by
// yskn_b200_matrix_create; this variant needs no library allocation at all.
//
// The scratch (per-warp i64 partials and one arrival counter per 8-row block of
// gemv.cu's split-row-block reduction) lives in g_noalloc_scratch below,
// 5,373,952 bytes, which every GPU that loads the library holds until exit.
// Limits (a call beyond them returns YSKN_EINVAL with a message): at most 64
// activation rows, at most 32768 blocks of 8 physical rows over the call's
// matrices (262,144 rows), cols below 262,144, and a GEMV grid of at most 2560
// warps (160 CTAs: every B200 configuration).
//
// Every call on a device shares the one array and it keeps the last call's
// contents; the counters that must start at zero are cleared (cudaMemsetAsync,
// which allocates nothing) on the caller's stream before each launch. Calls that
// overlap on the GPU (other streams at the same time) race on the array: issue
// them in order on one stream. The first call on each device looks up the
// array's device address (cudaGetSymbolAddress, with that device current); make
// that first call before any stream capture.
#include <mutex>

#include "common.cuh"

namespace yskn {

constexpr int NOALLOC_MAX_M = 64;
constexpr int64_t NOALLOC_MAX_ROW_BLOCKS = 32768;
constexpr int64_t NOALLOC_MAX_WARPS = 2560;
constexpr size_t NOALLOC_PARTIAL_BYTES = (size_t)NOALLOC_MAX_WARPS * 2 * 32 * 4 * sizeof(long long);
constexpr size_t NOALLOC_BYTES = NOALLOC_PARTIAL_BYTES + (size_t)NOALLOC_MAX_ROW_BLOCKS * sizeof(unsigned);

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

// Device address of g_noalloc_scratch per device (host code must not use the
// symbol itself as a pointer: on the host it names a stand-in, not device memory).
static unsigned char* g_noalloc_addr[64];
static std::mutex g_noalloc_mutex;

static int noalloc_scratch(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "weighted_sums_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(YSKN_EINVAL, "weighted_sums_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "weighted_sums_noalloc: cudaGetSymbolAddress");
    g_noalloc_addr[dev] = reinterpret_cast<unsigned char*>(p);
  }
  *out = g_noalloc_addr[dev];
  return YSKN_OK;
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_weighted_sums_noalloc(const yskn_b200_matrix* const* mats, int n_mats,
                                                              const int8_t* d_act, const int32_t* d_scales, int M,
                                                              int64_t* const* d_out, void* stream) {
  if (!mats || n_mats < 1 || n_mats > 3) return fail(YSKN_EINVAL, "weighted_sums_noalloc: 1 to 3 matrices per call");
  if (M < 1 || M > NOALLOC_MAX_M)
    return fail(YSKN_EINVAL, "weighted_sums_noalloc: M must be 1..64 (the static scratch holds one GEMV grid)");
  if (!d_act || !d_scales || !d_out || (reinterpret_cast<uintptr_t>(d_act) & 15) ||
      (reinterpret_cast<uintptr_t>(d_scales) & 15))
    return fail(YSKN_EINVAL, "weighted_sums_noalloc: null or misaligned activation arguments");
  MatrixDev devs[3];
  int rows[3];
  int64_t row_blocks = 0;
  for (int i = 0; i < n_mats; ++i) {
    const MatrixDev* d = matrix_dev(mats[i]);
    if (!d || !d_out[i]) return fail(YSKN_EINVAL, "weighted_sums_noalloc: null matrix or output");
    if (d->cols != matrix_dev(mats[0])->cols || d->bits != matrix_dev(mats[0])->bits)
      return fail(YSKN_EINVAL, "weighted_sums_noalloc: grouped matrices must share cols and bits");
    devs[i] = *d;
    rows[i] = d->phys;
    row_blocks += d->phys_pad8 / 8;
  }
  if (devs[0].cols / 512 >= 512)
    return fail(YSKN_EINVAL, "weighted_sums_noalloc: cols must be below 262144 (no overflow-checked variant)");
  if (row_blocks > NOALLOC_MAX_ROW_BLOCKS)
    return fail(YSKN_EINVAL, "weighted_sums_noalloc: more than 262144 physical rows in one call");
  unsigned char* base = nullptr;
  if (int rc = noalloc_scratch(&base)) return rc;
  GemvScratch sc{};
  sc.partials = reinterpret_cast<long long*>(base);
  sc.counters = reinterpret_cast<unsigned*>(base + NOALLOC_PARTIAL_BYTES);
  sc.n_counters = NOALLOC_MAX_ROW_BLOCKS;
  sc.max_warps = NOALLOC_MAX_WARPS;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(sc.counters, 0, (size_t)row_blocks * sizeof(unsigned), st);
  if (e != cudaSuccess) return cuda_fail(e, "weighted_sums_noalloc: clearing the counters");
  return launch_gemv(devs, n_mats, d_act, d_scales, M, d_out, rows, sc, st);
}
