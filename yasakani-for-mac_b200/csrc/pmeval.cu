// yskn_b200_portable_math: the library's device portable functions (pmath.cuh) over an
// array, so callers (and the tests) can compare them with the scalar contract directly.
#include <algorithm>

#include "common.cuh"
#include "pmath.cuh"

namespace yskn {

__global__ void portable_math_kernel(int fn, const float* x, float* y, float* y2, int64_t n) {
  pdl_begin();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    float r = 0.0f;
    switch (fn) {
      case YSKN_PM_EXP: r = pm_exp(v); break;
      case YSKN_PM_EXP2: r = pm_exp2(v); break;
      case YSKN_PM_LOG: r = pm_log(v); break;
      case YSKN_PM_LOG1P: r = pm_log1p(v); break;
      case YSKN_PM_SIGMOID: r = pm_sigmoid(v); break;
      case YSKN_PM_SILU: r = pm_silu(v); break;
      case YSKN_PM_SOFTPLUS: r = pm_softplus(v); break;
      case YSKN_PM_RSQRT: r = pm_rsqrt(v); break;
      default: {  // YSKN_PM_SINCOS: cosine to y, sine to y2 (0 and 0 where the reduction refuses)
        float c, s;
        pm_sincos(v, &c, &s);
        r = c;
        y2[i] = s;
      }
    }
    y[i] = r;
  }
}

}  // namespace yskn

using namespace yskn;

extern "C" YSKN_B200_API int yskn_b200_portable_math(int fn, const float* d_x, int64_t n, float* d_y, float* d_y2,
                                                     void* stream) {
  if (fn < YSKN_PM_EXP || fn > YSKN_PM_SINCOS || !d_x || !d_y || n < 1 || (fn == YSKN_PM_SINCOS && !d_y2))
    return fail(YSKN_EINVAL, "portable_math: bad argument");
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
  return cuda_fail(launch_pdl(portable_math_kernel, blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream), fn, d_x,
                              d_y, d_y2, n),
                   "portable_math_kernel");
}
