// Instantiates the compile-time-K separable kernels for float storage (see sep_fast_launch.cuh).
#include "sep_fast_launch.cuh"

namespace serron {
template int sep_fast_fwd_t<float>(int, int, bool, bool, const void*, void*, void*, uint32_t*, long long, int, int,
                                   int, cudaStream_t);
}  // namespace serron
