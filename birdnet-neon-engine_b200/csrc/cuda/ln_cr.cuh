// The natural logarithm of the dB-image front end, rounded once: CUDA's double-precision log of the float argument,
// rounded to nearest float. Used by k_dbimg_frames and exported for tests through bnn_cuda_fn (function 9).
#pragma once
#include <math.h>

namespace bnn {
__device__ __forceinline__ float ln_cr(float x) { return __double2float_rn(log((double)x)); }
}  // namespace bnn
