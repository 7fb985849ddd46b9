// Launcher of the autocast forward (tiled_autocast.cuh), in a translation unit of its own so its
// window sizes compile in parallel with the rest of the library.
#include "tiled_autocast.cuh"

namespace serron {

namespace {

template <typename TI, int OP, int K>
cudaError_t launch(const void* x, const float* w, __half* y, uint8_t* win, uint32_t* map, long long planes, int C,
                   int H, int W, int kcs, int border, int bulk, int out_vec, cudaStream_t stream) {
    using G = AcGeom<K, sizeof(TI)>;
    auto kernel = tiled_autocast_fwd_kernel<TI, OP, K>;
    const size_t smem = G::smem();
    if (smem > 48 * 1024) {
        const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     static_cast<int>(smem));
        if (err != cudaSuccess) return err;
    }
    const int tx = (W + kAcCols - 1) / kAcCols, ty = (H + kAcRows - 1) / kAcRows;
    const long long blocks = planes * tx * ty;
    if (blocks >= (1ll << 31)) return cudaErrorInvalidConfiguration;
    kernel<<<static_cast<unsigned>(blocks), kAcThreads, smem, stream>>>(static_cast<const TI*>(x), w, y, win, map, C,
                                                                         H, W, kcs, border, tx, ty, bulk, out_vec);
    return cudaGetLastError();
}

template <typename TI, int OP>
cudaError_t launch_k(int K, const void* x, const float* w, __half* y, uint8_t* win, uint32_t* map, long long planes,
                     int C, int H, int W, int kcs, int border, int bulk, int out_vec, cudaStream_t stream) {
    switch (K) {
#define SERRON_AC_CASE(k) \
    case k: return launch<TI, OP, k>(x, w, y, win, map, planes, C, H, W, kcs, border, bulk, out_vec, stream);
        SERRON_AC_CASE(3) SERRON_AC_CASE(5) SERRON_AC_CASE(7) SERRON_AC_CASE(9) SERRON_AC_CASE(11)
        SERRON_AC_CASE(13) SERRON_AC_CASE(15)
#undef SERRON_AC_CASE
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

// Windows the autocast forward compiles for: odd and square, 3 to 15.
bool autocast_fwd_supported_k(int kH, int kW) { return kH == kW && (kH & 1) && kH >= 3 && kH <= 15; }

// input_dtype: kF32, kF16 or kBF16; weights float32; output float16; one-byte direct records with the
// target map (zeroed by the caller).
cudaError_t autocast_fwd_launch(int op, int input_dtype, int K, const void* x, const float* w, __half* y,
                                uint8_t* win, uint32_t* map, long long planes, int C, int H, int W, int kcs,
                                int border, int bulk, int out_vec, cudaStream_t stream) {
    auto go = [&](auto t) {
        using TI = decltype(t);
        return op == kErode
                   ? launch_k<TI, kErode>(K, x, w, y, win, map, planes, C, H, W, kcs, border, bulk, out_vec, stream)
                   : launch_k<TI, kDilate>(K, x, w, y, win, map, planes, C, H, W, kcs, border, bulk, out_vec, stream);
    };
    switch (input_dtype) {
    case kF32: return go(float{});
    case kF16: return go(__half{});
    case kBF16: return go(__nv_bfloat16{});
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace serron
