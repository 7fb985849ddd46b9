// Launcher of the one-launch derived operations (derived.cuh), in a translation unit of its own so its
// instantiations compile in parallel with the rest of the library.
#include "derived.cuh"

namespace serron {

namespace {

template <typename T, int MODE>
cudaError_t launch(const void* x, const void* w, void* y, uint8_t* win_a, uint8_t* win_b, uint32_t* map_a,
                   uint32_t* map_b, long long planes, int C, int H, int W, int kH, int kW, int kcs, int border,
                   cudaStream_t stream) {
    using A = typename Storage<T>::acc;
    auto kernel = derived_fwd_kernel<T, uint8_t, MODE>;
    const DerivedGeom geo(kH, kW, derived_two_stage(MODE));
    const size_t smem = geo.bytes(kH, kW, sizeof(A));
    if (smem > 48 * 1024) {
        const cudaError_t err =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err != cudaSuccess) return err;
    }
    const int tx = (W + kTile - 1) / kTile, ty = (H + kTile - 1) / kTile;
    const long long blocks = planes * tx * ty;
    if (blocks >= (1ll << 31)) return cudaErrorInvalidConfiguration;
    kernel<<<static_cast<unsigned>(blocks), dim3(kTile, kTileThreadsY), smem, stream>>>(
        static_cast<const T*>(x), static_cast<const T*>(w), static_cast<T*>(y), win_a, win_b, map_a, map_b, C, H, W,
        kH, kW, kcs, border, tx, ty);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_mode(int mode, const void* x, const void* w, void* y, uint8_t* win_a, uint8_t* win_b,
                        uint32_t* map_a, uint32_t* map_b, long long planes, int C, int H, int W, int kH, int kW,
                        int kcs, int border, cudaStream_t stream) {
    switch (mode) {
#define SERRON_DERIVED_CASE(m) \
    case m: return launch<T, m>(x, w, y, win_a, win_b, map_a, map_b, planes, C, H, W, kH, kW, kcs, border, stream);
        SERRON_DERIVED_CASE(kDerivedGradient) SERRON_DERIVED_CASE(kDerivedOpening) SERRON_DERIVED_CASE(kDerivedClosing)
        SERRON_DERIVED_CASE(kDerivedTopHat) SERRON_DERIVED_CASE(kDerivedBlackHat)
#undef SERRON_DERIVED_CASE
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

// Windows and images the one-launch derived operations take: both window sides at most kDerivedMaxK (the
// two-stage ones also need an image at least as large as the window, so a folded position of the
// intermediate lies in the CTA's grown tile), and a one-byte record.
bool derived_supported(int mode, long long H, long long W, long long kH, long long kW) {
    if (mode < kDerivedGradient || mode > kDerivedBlackHat) return false;
    if (kH < 1 || kW < 1 || kH > kDerivedMaxK || kW > kDerivedMaxK || kH * kW > 255) return false;
    return !derived_two_stage(mode) || (H >= kH && W >= kW);
}

// dtype: kF32, kF64, kF16 or kBF16 (input, kernel and output); one-byte direct records with their target
// maps (zeroed by the caller): a = dilation / first stage, b = erosion / second stage.
cudaError_t derived_fwd_launch(int mode, int dtype, const void* x, const void* w, void* y, uint8_t* win_a,
                               uint8_t* win_b, uint32_t* map_a, uint32_t* map_b, long long planes, int C, int H, int W,
                               int kH, int kW, int kcs, int border, cudaStream_t stream) {
    switch (dtype) {
    case kF32:
        return launch_mode<float>(mode, x, w, y, win_a, win_b, map_a, map_b, planes, C, H, W, kH, kW, kcs, border, stream);
    case kF64:
        return launch_mode<double>(mode, x, w, y, win_a, win_b, map_a, map_b, planes, C, H, W, kH, kW, kcs, border,
                                   stream);
    case kF16:
        return launch_mode<__half>(mode, x, w, y, win_a, win_b, map_a, map_b, planes, C, H, W, kH, kW, kcs, border,
                                   stream);
    case kBF16:
        return launch_mode<__nv_bfloat16>(mode, x, w, y, win_a, win_b, map_a, map_b, planes, C, H, W, kH, kW, kcs,
                                          border, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace serron
