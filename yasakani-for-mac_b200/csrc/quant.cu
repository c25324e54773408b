// Operator prologue and epilogue as standalone kernels: the activation quantiser
// and the restore (+ output rotation). The arithmetic lives in quant.cuh, shared
// with the fused decode operator in gemv.cu.
#include "quant.cuh"

namespace yskn {

// grid: M blocks; block: nw warps; dynamic smem: G floats.
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ x, const int8_t* __restrict__ signs,
                                                       int Kc, int8_t* __restrict__ act, float* __restrict__ alpha,
                                                       int32_t* __restrict__ scales, float* __restrict__ row_quantum,
                                                       unsigned* __restrict__ err) {
  extern __shared__ float s_alpha[];
  const int m = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int G = Kc / 512;
  const float* xr = x + (int64_t)m * Kc;
  bool bad = false;
  for (int g = warp; g < G; g += nw) {
    const float scale = quantize_group512(xr + g * 512, signs + g * 512, act + (int64_t)m * Kc + g * 512, lane, bad);
    if (lane == 0) {
      s_alpha[g] = scale;
      alpha[(int64_t)m * G + g] = scale;
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(err, DERR_NONFINITE);
  __syncthreads();
  float mxs = 0.0f;
  for (int g = 0; g < G; ++g) mxs = fmaxf(mxs, s_alpha[g]);
  const float mult = row_grid_multiplier(mxs);
  for (int g = threadIdx.x; g < G; g += blockDim.x) scales[(int64_t)m * G + g] = integer_group_scale(s_alpha[g], mult);
  if (threadIdx.x == 0) row_quantum[m] = row_quantum_of(mxs);
}

int launch_quantize(const float* x, const int8_t* signs, int M, int Kc, int8_t* act, float* alpha, int32_t* scales,
                    float* row_quantum, cudaStream_t st) {
  const int G = Kc / 512;
  const int nw = G < 8 ? G : 8;
  quantize_kernel<<<M, nw * 32, G * sizeof(float), st>>>(x, signs, Kc, act, alpha, scales, row_quantum,
                                                         device_error_word());
  return cuda_fail(cudaGetLastError(), "quantize_kernel");
}

// The integer grid from a given row maximum (compressed_linear.rs:113-128): under
// tensor parallelism the maximum over every rank's groups, so all ranks form the
// integers of the whole row.
__global__ void __launch_bounds__(256) rescale_kernel(const float* __restrict__ alpha,
                                                      const float* __restrict__ row_max, int M, int G,
                                                      int32_t* __restrict__ scales, float* __restrict__ row_quantum) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * G) return;
  const int m = (int)(i / G);
  const float mx = row_max[m];
  scales[i] = integer_group_scale(alpha[i], row_grid_multiplier(mx));
  if (i == (int64_t)m * G) row_quantum[m] = row_quantum_of(mx);
}

int launch_rescale(const float* alpha, const float* row_max, int M, int G, int32_t* scales, float* row_quantum,
                   cudaStream_t st) {
  const int64_t n = (int64_t)M * G;
  rescale_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(alpha, row_max, M, G, scales, row_quantum);
  return cuda_fail(cudaGetLastError(), "rescale_kernel");
}

// Restore with output rotation: one warp per (row m, 512-row block).
__global__ void __launch_bounds__(256) restore_rot_kernel(int64_t* __restrict__ ws, int ws_ld,
                                                          const float* __restrict__ row_quantum,
                                                          const float* __restrict__ inv_rms,
                                                          const float* __restrict__ tau,
                                                          const int8_t* __restrict__ s_out, int M, int blocks,
                                                          int n_rows, int clear_ws, float* __restrict__ y,
                                                          unsigned* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= (int64_t)M * blocks) return;
  const int m = (int)(item / blocks), b = (int)(item % blocks);
  bool bad = false;
  int64_t* wsr = ws + (int64_t)m * ws_ld;
  restore_block512(wsr, row_quantum[m], inv_rms ? inv_rms + m : nullptr, tau, s_out, b * 512, n_rows,
                   y + (int64_t)m * n_rows, lane, bad);
  if (clear_ws) {  // the rows this lane read (restore_block512's lane mapping)
#pragma unroll
    for (int k = 0; k < 8; ++k)
      *reinterpret_cast<longlong2*>(wsr + b * 512 + 64 * k + 2 * lane) = make_longlong2(0, 0);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) raise_device_error(err, DERR_NONFINITE);
}

// Restore without output rotation (vocabulary head, draft): elementwise.
__global__ void __launch_bounds__(256) restore_plain_kernel(int64_t* __restrict__ ws, int ws_ld,
                                                            const float* __restrict__ row_quantum,
                                                            const float* __restrict__ inv_rms,
                                                            const float* __restrict__ tau, int M, int phys,
                                                            int n_rows, int clear_ws, float* __restrict__ y,
                                                            unsigned* __restrict__ err) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * phys) return;
  const int m = (int)(i / phys), r = (int)(i % phys);
  int64_t* p = ws + (int64_t)m * ws_ld + r;
  bool bad = inv_rms ? !finite32(inv_rms[m]) : false;
  const float t = restore_value(*p, row_quantum[m], inv_rms ? inv_rms + m : nullptr, __ldg(tau + r));
  bad |= !finite32(t);
  if (clear_ws) *p = 0;
  if (r < n_rows) y[(int64_t)m * n_rows + r] = t;
  if (bad) raise_device_error(err, DERR_NONFINITE);
}

int launch_restore(int64_t* ws, int ws_ld, const float* row_quantum, const float* inv_rms, const float* tau,
                   const int8_t* s_out, int M, int phys, int n_rows, int clear_ws, float* y, cudaStream_t st) {
  if (s_out) {
    const int blocks = phys / 512;
    const int64_t items = (int64_t)M * blocks;
    restore_rot_kernel<<<(unsigned)ceil_div(items, 8), 256, 0, st>>>(ws, ws_ld, row_quantum, inv_rms, tau, s_out, M,
                                                                     blocks, n_rows, clear_ws, y, device_error_word());
    return cuda_fail(cudaGetLastError(), "restore_rot_kernel");
  }
  const int64_t total = (int64_t)M * phys;
  restore_plain_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(ws, ws_ld, row_quantum, inv_rms, tau, M, phys,
                                                                       n_rows, clear_ws, y, device_error_word());
  return cuda_fail(cudaGetLastError(), "restore_plain_kernel");
}

}  // namespace yskn
