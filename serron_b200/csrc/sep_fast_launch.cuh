// Host launchers of the compile-time-K separable kernels (sep_fast.cuh), instantiated once per storage
// type in sep_fast_<type>.cu so the type variants compile in parallel.
#pragma once

#include "sep_fast.cuh"

namespace serron {

// Window lengths with a compiled fast path; other flat windows take the generic kernels.
#define SERRON_SEP_FAST_KS(X) X(3) X(5) X(7) X(9) X(11) X(13) X(15) X(17) X(21) X(25) X(31)

template <int K>
using FastIndex = typename std::conditional<(K <= 15), uint8_t, uint16_t>::type;

template <typename K_>
inline cudaError_t set_smem_attr(K_ kernel, size_t bytes) {
    if (bytes > 48 * 1024) return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    return cudaSuccess;
}

template <typename T, int OP, int K, bool V, bool X>
int sep_fast_fwd_launch(const void* x, void* y, void* win, long long planes, int H, int W, int border,
                        cudaStream_t stream) {
    using G = FastGeom<K>;
    using I = FastIndex<K>;
    const int tx = (W + kFastTW - 1) / kFastTW, ty = (H + G::TH - 1) / G::TH;
    const size_t smem = G::smem_bytes();
    auto kernel = sep_fast_fwd_kernel<T, OP, I, V, X, K>;
    cudaError_t err = set_smem_attr(kernel, smem);
    if (err != cudaSuccess) return static_cast<int>(err);
    const long long blocks = static_cast<long long>(tx) * ty * planes;
    kernel<<<static_cast<unsigned>(blocks), kFastThreads, smem, stream>>>(
        static_cast<const T*>(x), static_cast<T*>(y), static_cast<I*>(win), H, W, border, tx, ty);
    return static_cast<int>(cudaGetLastError());
}

template <typename T, int OP, int K>
int sep_fast_fwd_k(bool with_value, bool with_index, const void* x, void* y, void* win, long long planes, int H,
                   int W, int border, cudaStream_t stream) {
    if (with_value && with_index) return sep_fast_fwd_launch<T, OP, K, true, true>(x, y, win, planes, H, W, border, stream);
    if (with_index) return sep_fast_fwd_launch<T, OP, K, false, true>(x, y, win, planes, H, W, border, stream);
    return sep_fast_fwd_launch<T, OP, K, true, false>(x, y, win, planes, H, W, border, stream);
}

// Returns 0 on success, a cudaError_t code on a launch failure, or -1 when K has no fast path.
template <typename T>
int sep_fast_fwd_t(int op, int K, bool with_value, bool with_index, const void* x, void* y, void* win,
                   long long planes, int H, int W, int border, cudaStream_t stream) {
#define SERRON_SEP_FAST_FWD_CASE(k)                                                                       \
    case k:                                                                                               \
        return op == kErode ? sep_fast_fwd_k<T, kErode, k>(with_value, with_index, x, y, win, planes, H, W, \
                                                           border, stream)                                \
                            : sep_fast_fwd_k<T, kDilate, k>(with_value, with_index, x, y, win, planes, H, W, \
                                                            border, stream);
    switch (K) {
        SERRON_SEP_FAST_KS(SERRON_SEP_FAST_FWD_CASE)
    default:
        return -1;
    }
#undef SERRON_SEP_FAST_FWD_CASE
}

template <typename T, int K>
int sep_fast_gather_launch(const void* go, const void* win, void* gi, long long planes, int H, int W, int border,
                           cudaStream_t stream) {
    using G = FastGeom<K>;
    using I = FastIndex<K>;
    const int tx = (W + kFastTW - 1) / kFastTW, ty = (H + G::GTH - 1) / G::GTH;
    const size_t smem = G::gather_smem_bytes(sizeof(I));
    auto kernel = sep_fast_gather_kernel<T, I, K>;
    cudaError_t err = set_smem_attr(kernel, smem);
    if (err != cudaSuccess) return static_cast<int>(err);
    const long long blocks = static_cast<long long>(tx) * ty * planes;
    kernel<<<static_cast<unsigned>(blocks), kFastThreads, smem, stream>>>(
        static_cast<const T*>(go), static_cast<const I*>(win), static_cast<T*>(gi), H, W, border, tx, ty);
    return static_cast<int>(cudaGetLastError());
}

template <typename T>
int sep_fast_gather_t(int K, const void* go, const void* win, void* gi, long long planes, int H, int W, int border,
                      cudaStream_t stream) {
#define SERRON_SEP_FAST_GATHER_CASE(k) \
    case k:                            \
        return sep_fast_gather_launch<T, k>(go, win, gi, planes, H, W, border, stream);
    switch (K) {
        SERRON_SEP_FAST_KS(SERRON_SEP_FAST_GATHER_CASE)
    default:
        return -1;
    }
#undef SERRON_SEP_FAST_GATHER_CASE
}

}  // namespace serron
