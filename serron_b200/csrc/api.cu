// C ABI of the sm_100a morphology library: validation, algorithm resolution, buffer sizing and kernel
// launches.  Declarations and the contract of every entry point: include/serron_b200.h.
//
// Host-side behaviour follows the reference's CUDA operators (vhrabar/serron 0.6.0, packages/serron/):
// validation and messages csrc/gpu/morphology/operators.cpp:153-190 and backward.cpp:154-194,
// algorithm resolution csrc/gpu/morphology/algorithm.h:103-137, thresholds
// csrc/gpu/morphology/thresholds.h:46-71 with the SERRON_SEPARABLE_MIN_K override of
// csrc/gpu/morphology/separable.h:104-116, flatness read-back separable.h:150-169.
#include "serron_b200.h"

#include "common.cuh"
#include "direct.cuh"
#include "recon.cuh"
#include "recon_persist.cuh"
#include "derived.cuh"
#include "recon_scan.cuh"
#include "segrad.cuh"
#include "separable.cuh"
#include "gather_pull.cuh"
#include "gather_stream.cuh"

namespace serron {
// compile-time-K separable kernels, instantiated per storage type in sep_fast_<type>.cu; they return
// 0, a cudaError_t code, or -1 when the window length has no fast path; with `map` they also set the
// winners in the gather's target map
template <typename T>
int sep_fast_fwd_t(int op, int K, bool with_value, bool with_index, const void* x, void* y, void* win, uint32_t* map,
                   long long planes, int H, int W, int border, cudaStream_t stream);
// the one-launch derived operations (derived.cu)
bool derived_supported(int mode, long long H, long long W, long long kH, long long kW);
cudaError_t derived_fwd_launch(int mode, int dtype, const void* x, const void* w, void* y, uint8_t* win_a,
                               uint8_t* win_b, uint32_t* map_a, uint32_t* map_b, long long planes, int C, int H, int W,
                               int kH, int kW, int kcs, int border, cudaStream_t stream);
// the autocast forward (tiled_autocast.cu): float16 values and float32 winners in one pass
bool autocast_fwd_supported_k(int kH, int kW);
cudaError_t autocast_fwd_launch(int op, int input_dtype, int K, const void* x, const float* w, __half* y,
                                uint8_t* win, uint32_t* map, long long planes, int C, int H, int W, int kcs,
                                int border, int bulk, int out_vec, cudaStream_t stream);
}  // namespace serron

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace serron {
namespace {

thread_local std::string g_last_error;

struct Failure {
    int code;
    std::string message;
};

template <typename... Args>
std::string concat(const Args&... args) {
    std::ostringstream oss;
    ((oss << args), ...);
    return oss.str();
}

#define SB_CHECK(cond, ...)                                                  \
    do {                                                                     \
        if (!(cond)) throw Failure{SERRON_ERR_INVALID, concat(__VA_ARGS__)}; \
    } while (0)

#define SB_CUDA(expr)                                                                                         \
    do {                                                                                                      \
        const cudaError_t err_ = (expr);                                                                      \
        if (err_ != cudaSuccess)                                                                              \
            throw Failure{SERRON_ERR_CUDA, concat("serron: CUDA error ", cudaGetErrorName(err_), ": ",      \
                                                  cudaGetErrorString(err_), " (", #expr, ")")};              \
    } while (0)

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return SERRON_OK;
    } catch (const Failure& e) {
        g_last_error = e.message;
        return e.code;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return SERRON_ERR_INVALID;
    }
}

// Makes `device` current for the scope of a call and restores the previous device.
struct DeviceScope {
    int previous = -1;
    explicit DeviceScope(int device) {
        if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
        cudaGetLastError();
        if (previous != device) SB_CUDA(cudaSetDevice(device));
    }
    ~DeviceScope() {
        int now = -1;
        if (previous >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous) cudaSetDevice(previous);
    }
};

size_t elem_size(int dtype) { return dtype == kF64 ? 8 : dtype == kF32 ? 4 : 2; }
size_t acc_size(int dtype) { return dtype == kF64 ? 8 : 4; }

struct DeviceInfo {
    size_t smem_optin = 0;
    int sm_count = 0;
};
DeviceInfo device_info(int device) {
    static std::mutex mutex;
    static std::map<int, DeviceInfo> cache;
    const std::scoped_lock lock(mutex);
    auto it = cache.find(device);
    if (it != cache.end()) return it->second;
    DeviceInfo info;
    int v = 0;
    SB_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    info.smem_optin = static_cast<size_t>(v);
    SB_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device));
    info.sm_count = v;
    cache[device] = info;
    return info;
}

// ------------------------------------------------------------------------------------------------
// geometry and validation
// ------------------------------------------------------------------------------------------------
struct Geometry {
    int64_t N = 0, C = 0, H = 0, W = 0;
    int64_t kH = 0, kW = 0, kcs = 0;
    int64_t numel() const { return N * C * H * W; }
    int64_t kernel_numel() const { return kcs ? C * kcs : kH * kW; }
};

Geometry parse_geometry(const char* name, const int64_t* in_sizes, int64_t in_dim, const int64_t* k_sizes,
                        int64_t k_dim) {
    SB_CHECK(in_dim == 4, name, ": input must be 4-D (N, C, H, W), got ", in_dim, "-D");
    SB_CHECK(k_dim == 2 || k_dim == 3, name, ": kernel must be 2-D (kH, kW) or 3-D (C, kH, kW), got ", k_dim, "-D");
    SB_CHECK(in_sizes != nullptr && k_sizes != nullptr, name, ": sizes must not be null");
    Geometry g;
    g.N = in_sizes[0];
    g.C = in_sizes[1];
    g.H = in_sizes[2];
    g.W = in_sizes[3];
    SB_CHECK(g.N >= 0 && g.C >= 0 && g.H >= 0 && g.W >= 0, name, ": input sizes must be non-negative");
    if (k_dim == 3) {
        SB_CHECK(k_sizes[0] == g.C, name, ": kernel channel dim (", k_sizes[0], ") must match input channels (", g.C,
                 ")");
        g.kH = k_sizes[1];
        g.kW = k_sizes[2];
        g.kcs = g.kH * g.kW;
    } else {
        g.kH = k_sizes[0];
        g.kW = k_sizes[1];
        g.kcs = 0;
    }
    SB_CHECK(g.kH > 0 && g.kW > 0, name, ": kernel spatial dims must be positive");
    SB_CHECK(g.H < (int64_t(1) << 30) && g.W < (int64_t(1) << 30) && g.kH < (int64_t(1) << 20) &&
                 g.kW < (int64_t(1) << 20) && g.C < (int64_t(1) << 31),
             name, ": extents beyond the supported range (H, W < 2^30, kH, kW < 2^20)");
    return g;
}

void check_common(const char* name, int32_t dtype, int64_t border) {
    SB_CHECK(dtype >= kF32 && dtype <= kBF16, name, ": unsupported dtype code ", dtype);
    SB_CHECK(border >= kReflect && border <= kConstant, name, ": invalid border mode ", border);
}

int parse_algo(const char* name, int64_t algo) {
    SB_CHECK(algo >= 0 && algo <= 3, name, ": invalid algo ", algo);
    return static_cast<int>(algo);
}

// Flatness of the SE, read back from the device when the caller does not know it (a synchronising
// copy on `stream`, as the reference does).
bool resolve_flat(int32_t flat, const void* kernel, int64_t numel, int32_t dtype, cudaStream_t stream) {
    if (flat >= 0) return flat != 0;
    if (numel == 0) return true;
    std::vector<unsigned char> host(static_cast<size_t>(numel) * elem_size(dtype));
    SB_CUDA(cudaMemcpyAsync(host.data(), kernel, host.size(), cudaMemcpyDeviceToHost, stream));
    SB_CUDA(cudaStreamSynchronize(stream));
    for (int64_t i = 0; i < numel; ++i) {
        float v = 0.0f;
        switch (dtype) {
        case kF32: std::memcpy(&v, host.data() + 4 * i, 4); break;
        case kF64: {
            double d;
            std::memcpy(&d, host.data() + 8 * i, 8);
            if (d != 0.0) return false;
            continue;
        }
        default: {
            uint16_t h;
            std::memcpy(&h, host.data() + 2 * i, 2);
            // zero in both half and bfloat16: only +0 and -0
            if ((h & 0x7fffu) != 0) return false;
            continue;
        }
        }
        if (v != 0.0f) return false;
    }
    return true;
}

// ------------------------------------------------------------------------------------------------
// thresholds (csrc/gpu/morphology/thresholds.h:46-71)
// ------------------------------------------------------------------------------------------------
// The reference ships 11 (csrc/gpu/morphology/thresholds.h:16).  Measured on a B200 with x (4,64,512,512) and
// square(K) SEs, K = 3..15, float32 / float16 / bfloat16, forward and backward: the separable sweep was the
// faster algorithm at every K from 3 on (K = 3, float32: forward 0.21 vs 0.49 ms, backward 0.49 vs 1.12 ms
// for the tiled kernel), so every flat rectangle of at least three taps along a side takes it.
constexpr int64_t kDefaultSeparableMinK = 3;

int64_t separable_min_k_override() {
    static const int64_t value = [] {
        if (const char* env = std::getenv("SERRON_SEPARABLE_MIN_K")) {
            char* end = nullptr;
            const long parsed = std::strtol(env, &end, 10);
            if (end != env && *end == '\0' && parsed > 0) return static_cast<int64_t>(parsed);
        }
        return static_cast<int64_t>(0);
    }();
    return value;
}

struct ThresholdTable {
    std::mutex mutex;
    std::map<std::tuple<int, int, bool>, int64_t> values;
};
ThresholdTable& thresholds() {
    static ThresholdTable table;
    return table;
}

int64_t separable_min_k(int device, int dtype, bool backward) {
    if (const int64_t forced = separable_min_k_override(); forced > 0) return forced;
    auto& t = thresholds();
    const std::scoped_lock lock(t.mutex);
    const auto it = t.values.find({device, dtype, backward});
    return it == t.values.end() ? kDefaultSeparableMinK : it->second;
}

// ------------------------------------------------------------------------------------------------
// algorithm feasibility and resolution (csrc/gpu/morphology/algorithm.h:59-137)
// ------------------------------------------------------------------------------------------------
enum Algo : int { kAuto = 0, kElement = 1, kTiled = 2, kSeparable = 3 };

int direct_format(int64_t kH, int64_t kW) {
    const int64_t taps = kH * kW;
    return taps <= 255 ? SERRON_WINNERS_DIRECT_U8 : taps <= 65535 ? SERRON_WINNERS_DIRECT_U16 : SERRON_WINNERS_DIRECT_U32;
}
int separable_format(int64_t kH, int64_t kW) {
    if (kH <= 15 && kW <= 16) return SERRON_WINNERS_SEPARABLE_U8;
    if (kH <= 255 && kW <= 256) return SERRON_WINNERS_SEPARABLE_U16;
    return SERRON_WINNERS_SEPARABLE_U32;
}
int base_format(int fmt) { return fmt & ~SERRON_WINNERS_MAP; }
bool format_has_map(int fmt) { return (fmt & SERRON_WINNERS_MAP) != 0; }
int format_bytes(int fmt) {
    switch (base_format(fmt)) {
    case SERRON_WINNERS_DIRECT_U8:
    case SERRON_WINNERS_SEPARABLE_U8: return 1;
    case SERRON_WINNERS_DIRECT_U16:
    case SERRON_WINNERS_SEPARABLE_U16: return 2;
    case SERRON_WINNERS_DIRECT_U32:
    case SERRON_WINNERS_SEPARABLE_U32: return 4;
    default: return 0;
    }
}
bool format_is_separable(int fmt) { return base_format(fmt) >= SERRON_WINNERS_SEPARABLE_U8; }

// the tile with its halo and weights, then the target-map bitmap of the halo
size_t tiled_smem_bytes(int64_t kH, int64_t kW, int dtype) {
    const int h = static_cast<int>(kH), w = static_cast<int>(kW);
    return (tiled_smem(h, w, acc_size(dtype)) + 15) / 16 * 16 + mark_bytes(kTile, kTile, h, w);
}
size_t wide_smem_bytes(int kH, int kW, size_t acc) {
    return (wide_smem(kH, kW, acc) + 15) / 16 * 16 + mark_bytes(kWideRows, kWideCols, kH, kW);
}
size_t sep_smem_bytes(int64_t kH, int64_t kW, int dtype) {
    return dtype == kF64 ? SepSmem<double>::bytes(static_cast<int>(kH), static_cast<int>(kW))
                         : SepSmem<float>::bytes(static_cast<int>(kH), static_cast<int>(kW));
}

struct Problem {
    int64_t kH, kW;
    bool flat;
    int dtype;
    size_t budget;
    int64_t min_k;
};

bool tiled_feasible(const Problem& p) { return tiled_smem_bytes(p.kH, p.kW, p.dtype) <= p.budget; }
bool separable_feasible(const Problem& p) {
    return p.flat && p.kW <= 256 && p.kH <= 65534 && p.kH + kSepTH < 65536 && p.kW + kSepTW < 65536 &&
           sep_smem_bytes(p.kH, p.kW, p.dtype) <= p.budget;
}
int heuristic(const Problem& p) {
    if (std::max(p.kH, p.kW) >= p.min_k && separable_feasible(p)) return kSeparable;
    return tiled_feasible(p) ? kTiled : kElement;
}
int resolve_algorithm(int requested, const Problem& p, const char* name) {
    switch (requested) {
    case kAuto: return heuristic(p);
    case kElement: return kElement;
    case kTiled:
        SB_CHECK(tiled_feasible(p), name, ": algo 'tiled' needs ", tiled_smem_bytes(p.kH, p.kW, p.dtype),
                 " bytes of shared memory for a ", p.kH, "x", p.kW, " window, over the ", p.budget, " available");
        return kTiled;
    default:
        SB_CHECK(p.flat, name, ": algo 'separable' needs a flat structuring element");
        SB_CHECK(separable_feasible(p), name, ": algo 'separable' does not fit in shared memory for a ", p.kH, "x",
                 p.kW, " window");
        return kSeparable;
    }
}
// every forward algorithm writes direct taps, with the gather's target map where the gather can use one;
// the packed separable formats are accepted as input only
int winners_format_for(int /*algo*/, int64_t kH, int64_t kW) {
    const int fmt = direct_format(kH, kW);
    return pull_taps_fit(kH, kW, format_bytes(fmt)) ? fmt | SERRON_WINNERS_MAP : fmt;
}

// ------------------------------------------------------------------------------------------------
// type dispatch
// ------------------------------------------------------------------------------------------------
template <typename F>
void dispatch_dtype(int dtype, F&& f) {
    switch (dtype) {
    case kF32: f(float{}); break;
    case kF64: f(double{}); break;
    case kF16: f(__half{}); break;
    default: f(__nv_bfloat16{}); break;
    }
}
template <typename F>
void dispatch_op(int op, F&& f) {
    if (op == kErode)
        f(std::integral_constant<int, kErode>{});
    else
        f(std::integral_constant<int, kDilate>{});
}
template <typename F>
void dispatch_index(int fmt, F&& f) {
    switch (format_bytes(fmt)) {
    case 1: f(uint8_t{}); break;
    case 2: f(uint16_t{}); break;
    default: f(uint32_t{}); break;
    }
}

constexpr size_t kSmemOptin = 227 * 1024;  // sm_100 shared memory per CTA with the opt-in

template <typename K>
void set_smem(K kernel, size_t bytes) {
    if (bytes > 48 * 1024) SB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
}

unsigned int grid_1d(long long blocks) {
    SB_CHECK(blocks < (1ll << 31), "serron: problem too large for one launch");
    return static_cast<unsigned int>(blocks);
}

// ------------------------------------------------------------------------------------------------
// launches
// ------------------------------------------------------------------------------------------------
// Returns true when the launch also filled `map` (the separable sweep, for its window lengths, and the
// tiled kernels do).
template <typename T, int OP, typename I, bool V, bool X>
bool launch_forward_t(int algo, const Geometry& g, const void* x, const void* w, void* y, void* win, uint32_t* map,
                      int border, cudaStream_t stream) {
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W), C = static_cast<int>(g.C);
    const int kH = static_cast<int>(g.kH), kW = static_cast<int>(g.kW), kcs = static_cast<int>(g.kcs);
    const T* xp = static_cast<const T*>(x);
    const T* wp = static_cast<const T*>(w);
    T* yp = static_cast<T*>(y);
    I* ip = static_cast<I*>(win);
    if (algo == kElement) {
        const long long total = g.numel();
        element_fwd_kernel<T, OP, I, V, X><<<grid_1d((total + 255) / 256), 256, 0, stream>>>(
            xp, wp, yp, ip, total, C, H, W, kH, kW, kcs, border);
    } else if (algo == kTiled) {
        const size_t acc = sizeof(typename Storage<T>::acc);
        // eight outputs per thread pay off from 9 columns, and from 5 for 16-bit storage (whose taps
        // need no float-tie tracking, which costs the wide kernel registers)
        const bool wide = kW >= kWideQ + 1 || (kW >= 5 && sizeof(T) == 2);
        // both kernels fill the target map themselves, for less than a mark launch costs (config 3's
        // step: 15.47 ms against 15.99 ms with the launch)
        uint32_t* marks = X ? map : nullptr;
        if (wide && wide_smem_bytes(kH, kW, acc) <= kSmemOptin) {
            const int tx = ceil_div(W, kWideCols), ty = ceil_div(H, kWideRows);
            const size_t smem = wide_smem_bytes(kH, kW, acc);
            auto kernel = wide_fwd_kernel<T, OP, I, V, X>;
            set_smem(kernel, smem);
            kernel<<<grid_1d(static_cast<long long>(tx) * ty * g.N * g.C), 256, smem, stream>>>(
                xp, wp, yp, ip, C, H, W, kH, kW, kcs, border, tx, ty, marks);
        } else {
            const int tx = ceil_div(W, kTile), ty = ceil_div(H, kTile);
            const size_t smem = tiled_smem_bytes(kH, kW, std::is_same<T, double>::value ? kF64 : kF32);
            auto kernel = tiled_fwd_kernel<T, OP, I, V, X>;
            set_smem(kernel, smem);
            kernel<<<grid_1d(static_cast<long long>(tx) * ty * g.N * g.C), dim3(kTile, kTileThreadsY), smem, stream>>>(
                xp, wp, yp, ip, C, H, W, kH, kW, kcs, border, tx, ty, marks);
        }
        SB_CUDA(cudaGetLastError());
        return marks != nullptr;
    } else {
        if constexpr (!std::is_same<T, double>::value) {
            // the sweep indexes a plane in 32 bits, including the masked rows a segment's last step runs
            // past the image (fewer than 64)
            if (kH == kW && g.N * g.C < (1ll << 31) / 4096 && (g.H + 64) * (g.W + 64) < (1ll << 31)) {
                const int rc = sep_fast_fwd_t<T>(OP, kH, V, X, x, y, win, X ? map : nullptr, g.N * g.C, H, W, border,
                                                 stream);
                if (rc > 0) SB_CUDA(static_cast<cudaError_t>(rc));
                if (rc == 0) return X && map != nullptr;
            }
        }
        const int tx = ceil_div(W, kSepTW), ty = ceil_div(H, kSepTH);
        const size_t smem = SepSmem<typename Storage<T>::acc>::bytes(kH, kW);
        auto kernel = sep_fwd_kernel<T, OP, I, V, X>;
        set_smem(kernel, smem);
        kernel<<<grid_1d(static_cast<long long>(tx) * ty * g.N * g.C), kSepThreads, smem, stream>>>(
            xp, yp, ip, H, W, kH, kW, border, tx, ty);
    }
    SB_CUDA(cudaGetLastError());
    return false;
}

int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }
int64_t map_workspace(const Geometry& g) { return align256(pull_map_words(g.N * g.C, g.H, g.W) * 4); }
// a record buffer with the map flag: the records, then the map from the next 256-byte boundary
int64_t records_bytes(const Geometry& g, int fmt) { return align256(g.numel() * format_bytes(fmt)); }
int64_t winners_buffer_bytes(const Geometry& g, int fmt) {
    return format_has_map(fmt) ? records_bytes(g, fmt) + map_workspace(g) : g.numel() * format_bytes(fmt);
}

// The mark-and-pull gather applies: candidates within one border fold, box taps that fit the record,
// and both of its kernels within the shared-memory budget and the grid limits.
bool pull_applicable(const Geometry& g, int border, size_t elem, int idx, size_t budget) {
    const int64_t H = g.H, W = g.W, kH = g.kH, kW = g.kW;
    const bool single_fold =
        border != kReflect || (kH / 2 <= H - 1 && kH - 1 - kH / 2 <= H - 1 && kW / 2 <= W - 1 && kW - 1 - kW / 2 <= W - 1);
    if (!single_fold || !pull_taps_fit(kH, kW, idx)) return false;
    const PullGeom mg(static_cast<int>(kH), static_cast<int>(kW), idx);
    const SumGeom sg(static_cast<int>(kH), static_cast<int>(kW), static_cast<int>(elem), idx);
    const long long strips = (W + kPullTQ - 1) / kPullTQ, bands = (H + kSumTP - 1) / kSumTP;
    return mg.smem() <= budget && sg.smem() <= budget && g.N * g.C * strips < (1ll << 31) / 64 &&
           g.N * g.C * strips * bands < (1ll << 31);
}

// The gather's target map from direct records (every word of it is written).
template <typename I>
void launch_pull_mark_t(const Geometry& g, const void* win, uint32_t* map, int border, cudaStream_t stream) {
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W);
    const int kH = static_cast<int>(g.kH), kW = static_cast<int>(g.kW);
    const PullGeom geo(kH, kW, sizeof(I));
    const int strips = ceil_div(W, kPullTQ);
    const long long ctas = g.N * g.C * strips;
    // enough CTAs for several waves; each segment re-reads 2aH rows, so keep them >= 4 bands
    const long long want = std::clamp<long long>((2400 + ctas - 1) / ctas, 1, std::max(1, H / (4 * kPullTB)));
    const int seg_h = static_cast<int>((H + want - 1) / want);
    const int segs = ceil_div(H, seg_h);
    const int rec_vec = (reinterpret_cast<uintptr_t>(win) & 15) == 0 && (W * sizeof(I)) % 16 == 0;
    auto mark = pull_mark_kernel<I>;
    set_smem(mark, geo.smem());
    mark<<<grid_1d(ctas * segs), kPullThreads, geo.smem(), stream>>>(static_cast<const I*>(win), map, H, W, kH, kW,
                                                                      border, strips, segs, seg_h, rec_vec);
    SB_CUDA(cudaGetLastError());
}

// Forward; with a record buffer of a map format, the target map too (set by the separable sweep as it
// writes the records, or built from the records afterwards).
void launch_forward(int op, int dtype, int algo, const Geometry& g, const void* x, const void* w, void* y, void* win,
                    int fmt, int border, size_t budget, cudaStream_t stream) {
    dispatch_dtype(dtype, [&](auto t) {
        using T = decltype(t);
        dispatch_op(op, [&](auto o) {
            constexpr int OP = decltype(o)::value;
            if (win == nullptr) {
                launch_forward_t<T, OP, uint8_t, true, false>(algo, g, x, w, y, nullptr, nullptr, border, stream);
                return;
            }
            uint32_t* map = nullptr;
            if (format_has_map(fmt)) {
                map = reinterpret_cast<uint32_t*>(static_cast<char*>(win) + records_bytes(g, fmt));
                SB_CUDA(cudaMemsetAsync(map, 0, pull_map_words(g.N * g.C, g.H, g.W) * 4, stream));
            }
            dispatch_index(fmt, [&](auto i) {
                using I = decltype(i);
                const bool filled = y != nullptr
                                        ? launch_forward_t<T, OP, I, true, true>(algo, g, x, w, y, win, map, border, stream)
                                        : launch_forward_t<T, OP, I, false, true>(algo, g, x, w, nullptr, win, map,
                                                                                  border, stream);
                if (map && !filled && pull_applicable(g, border, sizeof(T), sizeof(I), budget))
                    launch_pull_mark_t<I>(g, win, map, border, stream);
            });
        });
    });
}

// backward workspace layout: [winner records][target map][segrad partials][segrad global bins], each
// 256-byte aligned; the records only when the backward computes them (the map then follows them, as in a
// record buffer of a map format), the map only when the records come without one, the segrad parts
// only for grad_kernel
struct SegradPlan {
    int chunks = 0;
    int threads = 0;
    bool global_bins = false;
    long long per_chunk = 0;
    int64_t partial_bytes = 0;
    int64_t bins_bytes = 0;
};
SegradPlan segrad_plan(const Geometry& g) {
    SegradPlan p;
    const int64_t bins = g.kH * g.kW;
    const int64_t per_channel = g.N * g.H * g.W;
    p.threads = bins <= 96 ? 128 : 32;
    p.global_bins = bins > 768;
    // about 32 chunks per SM over all channels, enough threads in flight to hide the loads, with the
    // partials held to 4 MiB; per-thread bins in global memory keep the old 4 chunks per SM
    const int64_t total_chunks = p.global_bins ? 592 : std::min<int64_t>(4736, (int64_t(4) << 20) / (bins * 8));
    const int64_t max_chunks = std::max<int64_t>(1, total_chunks / std::max<int64_t>(g.C, 1));
    p.chunks = static_cast<int>(std::clamp<int64_t>((per_channel + 16383) / 16384, 1, max_chunks));
    p.per_chunk = (per_channel + p.chunks - 1) / p.chunks;
    p.per_chunk = (p.per_chunk + 15) / 16 * 16;  // whole 16-output groups for the vector path
    p.partial_bytes = g.C * p.chunks * bins * 8;
    p.bins_bytes = p.global_bins ? g.C * p.chunks * int64_t(p.threads) * bins * 8 : 0;
    return p;
}
// The SE-gradient kernel's 16-output vector path: direct records, whole 16-output groups per plane,
// 16-byte aligned go and records.
int segrad_vec_ok(const Geometry& g, const void* go, const void* win, bool sep) {
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return !sep && (g.H * g.W) % 16 == 0 && aligned(go) && aligned(win) ? 1 : 0;
}
int64_t segrad_workspace(const Geometry& g, bool need_kg) {
    if (!need_kg) return 0;
    const SegradPlan p = segrad_plan(g);
    return align256(p.partial_bytes) + align256(p.bins_bytes);
}
int64_t backward_workspace(const Geometry& g, bool need_kg, int fmt, bool with_winners) {
    int64_t bytes = 0;
    if (!with_winners) bytes += records_bytes(g, fmt);
    if (!with_winners || !format_has_map(fmt)) bytes += map_workspace(g);
    return bytes + segrad_workspace(g, need_kg);
}

template <typename T, typename I, bool SEP>
void launch_gather_t(const Geometry& g, const void* go, const void* win, void* gi, uint32_t* map, bool map_ready,
                     int border, size_t budget, cudaStream_t stream) {
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W);
    const int kH = static_cast<int>(g.kH), kW = static_cast<int>(g.kW);
    const int dtype = std::is_same<T, double>::value ? kF64 : kF32;
    const int fmt_bytes = sizeof(I);
    const int tw = SEP ? kGTW : kTile, th = SEP ? kGTH : kTile;
    const int tx = ceil_div(W, tw), ty = ceil_div(H, th);
    size_t smem = static_cast<size_t>((tw + 2 * (kW / 2)) * (th + 2 * (kH / 2))) * (acc_size(dtype) + fmt_bytes) + 16;
    const long long blocks = static_cast<long long>(tx) * ty * g.N * g.C;
    // a halo too large for shared memory walks the candidates in global memory instead
    const int force_global = smem > budget ? 1 : 0;
    if (force_global) smem = 0;
    {
        // mark-and-pull and raster-order stream gathers: every candidate must lie within a single border fold
        const bool single_fold = border != kReflect || (kH / 2 <= H - 1 && kH - 1 - kH / 2 <= H - 1 &&
                                                        kW / 2 <= W - 1 && kW - 1 - kW / 2 <= W - 1);
        if (!SEP && map != nullptr && pull_applicable(g, border, sizeof(T), sizeof(I), budget)) {
            if (!map_ready) launch_pull_mark_t<I>(g, win, map, border, stream);
            const SumGeom sgeo(kH, kW, sizeof(T), sizeof(I));
            const int tiles_x = ceil_div(W, kPullTQ), tiles_y = ceil_div(H, kSumTP);
            auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
            const int go_vec = aligned(go) && (W * sizeof(T)) % 16 == 0;
            const int rec_vec = aligned(win) && (W * sizeof(I)) % 16 == 0;
            const int out_vec = aligned(gi) && (W * sizeof(T)) % 16 == 0;
            // rows of both staged arrays start on 16-byte boundaries: one bulk copy per row
            const int bulk = go_vec && rec_vec;
            auto run = [&](auto sum) {
                set_smem(sum, sgeo.smem());
                SB_CUDA(cudaFuncSetAttribute(sum, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
                sum<<<grid_1d(g.N * g.C * tiles_x * tiles_y), kSumThreads, sgeo.smem(), stream>>>(
                    static_cast<const T*>(go), static_cast<const I*>(win), map, static_cast<T*>(gi), H, W, kH, kW,
                    border, tiles_x, tiles_y, go_vec, rec_vec, out_vec, bulk);
            };
            // odd square windows up to 15 x 15 with one-byte records: the unrolled box of that size
            const int box = (sizeof(I) == 1 && kH == kW && (kW & 1) && kW >= 3 && kW <= 15) ? kW : 0;
            if constexpr (sizeof(I) == 1) {
                switch (box) {
                case 3: run(pull_sum_kernel<T, I, 3>); break;
                case 5: run(pull_sum_kernel<T, I, 5>); break;
                case 7: run(pull_sum_kernel<T, I, 7>); break;
                case 9: run(pull_sum_kernel<T, I, 9>); break;
                case 11: run(pull_sum_kernel<T, I, 11>); break;
                case 13: run(pull_sum_kernel<T, I, 13>); break;
                case 15: run(pull_sum_kernel<T, I, 15>); break;
                default: run(pull_sum_kernel<T, I, 0>); break;
                }
            } else {
                run(pull_sum_kernel<T, I, 0>);
            }
            SB_CUDA(cudaGetLastError());
            return;
        }
        const StreamGeom geo(kH, kW, sizeof(I));
        const size_t stream_smem = geo.smem(sizeof(typename GradAcc<T>::type), sizeof(I));
        if (single_fold && stream_smem <= budget && g.N * g.C < (1ll << 31) / 64) {
            const int strips = ceil_div(W, kStreamTW);
            const long long ctas = g.N * g.C * strips;
            // enough single-warp CTAs to fill the machine several times over; each segment re-walks
            // 2aH halo rows, so segments stay at least 64 rows tall
            const long long want = std::clamp<long long>((9472 + ctas - 1) / ctas, 1, std::max(1, H / 64));
            const int seg_h = static_cast<int>((H + want - 1) / want);
            const int segs = ceil_div(H, seg_h);
            auto kernel = stream_gather_kernel<T, I, SEP>;
            set_smem(kernel, stream_smem);
            kernel<<<grid_1d(ctas * segs), 32, stream_smem, stream>>>(
                static_cast<const T*>(go), static_cast<const I*>(win), static_cast<T*>(gi), H, W, kH, kW, border,
                strips, segs, seg_h);
            SB_CUDA(cudaGetLastError());
            return;
        }
    }
    if (SEP) {
        auto kernel = sep_gather_kernel<T, I>;
        set_smem(kernel, smem);
        kernel<<<grid_1d(blocks), dim3(kGTW, 8), smem, stream>>>(static_cast<const T*>(go), static_cast<const I*>(win),
                                                               static_cast<T*>(gi), H, W, kH, kW, border, tx, ty,
                                                               force_global);
    } else {
        auto kernel = direct_gather_kernel<T, I>;
        set_smem(kernel, smem);
        kernel<<<grid_1d(blocks), dim3(kTile, kTileThreadsY), smem, stream>>>(
            static_cast<const T*>(go), static_cast<const I*>(win), static_cast<T*>(gi), static_cast<int>(g.C), H, W,
            kH, kW, border, tx, ty, force_global);
    }
    SB_CUDA(cudaGetLastError());
}

template <typename T, typename I, bool SEP>
void launch_segrad_t(int op, const Geometry& g, const void* go, const void* win, void* gk, void* ws, int border,
                     cudaStream_t stream) {
    const SegradPlan p = segrad_plan(g);
    const int bins = static_cast<int>(g.kH * g.kW);
    double* partial = static_cast<double*>(ws);
    double* gbins = p.global_bins ? reinterpret_cast<double*>(static_cast<char*>(ws) + align256(p.partial_bytes)) : nullptr;
    const size_t smem = p.global_bins ? 0 : static_cast<size_t>(p.threads) * bins * 8;
    auto kernel = segrad_partial_kernel<T, I, SEP>;
    set_smem(kernel, smem);
    const int vec = segrad_vec_ok(g, go, win, SEP);
    kernel<<<dim3(p.chunks, static_cast<unsigned>(g.C)), p.threads, smem, stream>>>(
        static_cast<const T*>(go), static_cast<const I*>(win), partial, gbins, static_cast<int>(g.N),
        static_cast<int>(g.C), static_cast<int>(g.H), static_cast<int>(g.W), static_cast<int>(g.kH),
        static_cast<int>(g.kW), border, p.per_chunk, vec);
    SB_CUDA(cudaGetLastError());
    const int out_cells = static_cast<int>(g.kcs ? g.C * bins : bins);
    const double sign = op == kErode ? -1.0 : 1.0;
    segrad_final_kernel<T><<<out_cells, kSegradFinalThreads, 0, stream>>>(partial, static_cast<T*>(gk),
                                                                          static_cast<int>(g.C), p.chunks, bins,
                                                                          g.kcs ? 0 : 1, sign);
    SB_CUDA(cudaGetLastError());
}

// The pull gather and the structuring-element gradient with float arithmetic, grad_output read as TG and
// grad_input written as TO (one-byte or two-byte direct records with their target map).
template <typename TG, typename TO, typename I>
void launch_backward_widened_t(int op, const Geometry& g, const void* go, const void* win, void* gi, void* gk,
                               bool need_kg, const uint32_t* map, void* ws, int border, cudaStream_t stream) {
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W);
    const int kH = static_cast<int>(g.kH), kW = static_cast<int>(g.kW);
    const SumGeom sgeo(kH, kW, sizeof(TG), sizeof(I));
    const int tiles_x = ceil_div(W, kPullTQ), tiles_y = ceil_div(H, kSumTP);
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const int go_vec = aligned(go) && (W * sizeof(TG)) % 16 == 0;
    const int rec_vec = aligned(win) && (W * sizeof(I)) % 16 == 0;
    const int out_vec = aligned(gi) && (W * sizeof(TO)) % 16 == 0;
    const int bulk = go_vec && rec_vec;
    auto run = [&](auto sum) {
        set_smem(sum, sgeo.smem());
        SB_CUDA(cudaFuncSetAttribute(sum, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        sum<<<grid_1d(g.N * g.C * tiles_x * tiles_y), kSumThreads, sgeo.smem(), stream>>>(
            static_cast<const TG*>(go), static_cast<const I*>(win), map, static_cast<TO*>(gi), H, W, kH, kW, border,
            tiles_x, tiles_y, go_vec, rec_vec, out_vec, bulk);
    };
    const int box = (sizeof(I) == 1 && kH == kW && (kW & 1) && kW >= 3 && kW <= 15) ? kW : 0;
    if constexpr (sizeof(I) == 1) {
        switch (box) {
        case 3: run(pull_sum_kernel<float, I, 3, TG, TO>); break;
        case 5: run(pull_sum_kernel<float, I, 5, TG, TO>); break;
        case 7: run(pull_sum_kernel<float, I, 7, TG, TO>); break;
        case 9: run(pull_sum_kernel<float, I, 9, TG, TO>); break;
        case 11: run(pull_sum_kernel<float, I, 11, TG, TO>); break;
        case 13: run(pull_sum_kernel<float, I, 13, TG, TO>); break;
        case 15: run(pull_sum_kernel<float, I, 15, TG, TO>); break;
        default: run(pull_sum_kernel<float, I, 0, TG, TO>); break;
        }
    } else {
        run(pull_sum_kernel<float, I, 0, TG, TO>);
    }
    SB_CUDA(cudaGetLastError());
    if (!need_kg) {
        SB_CUDA(cudaMemsetAsync(gk, 0, g.kernel_numel() * sizeof(float), stream));
        return;
    }
    const SegradPlan p = segrad_plan(g);
    const int bins = static_cast<int>(g.kH * g.kW);
    double* partial = static_cast<double*>(ws);
    double* gbins = p.global_bins ? reinterpret_cast<double*>(static_cast<char*>(ws) + align256(p.partial_bytes)) : nullptr;
    const size_t smem = p.global_bins ? 0 : static_cast<size_t>(p.threads) * bins * 8;
    auto kernel = segrad_partial_kernel<TG, I, false>;
    set_smem(kernel, smem);
    kernel<<<dim3(p.chunks, static_cast<unsigned>(g.C)), p.threads, smem, stream>>>(
        static_cast<const TG*>(go), static_cast<const I*>(win), partial, gbins, static_cast<int>(g.N),
        static_cast<int>(g.C), H, W, kH, kW, border, p.per_chunk, segrad_vec_ok(g, go, win, false));
    SB_CUDA(cudaGetLastError());
    const int out_cells = static_cast<int>(g.kcs ? g.C * bins : bins);
    segrad_final_kernel<float><<<out_cells, kSegradFinalThreads, 0, stream>>>(
        partial, static_cast<float*>(gk), static_cast<int>(g.C), p.chunks, bins, g.kcs ? 0 : 1,
        op == kErode ? -1.0 : 1.0);
    SB_CUDA(cudaGetLastError());
}

// `map`: the target map (ready: filled from these records), `ws`: the segrad workspace.
void launch_backward_from_winners(int op, int dtype, const Geometry& g, const void* go, const void* win, int fmt,
                                  void* gi, void* gk, bool need_kg, uint32_t* map, bool map_ready, void* ws,
                                  int border, size_t budget, cudaStream_t stream) {
    const bool sep = format_is_separable(fmt);
    dispatch_dtype(dtype, [&](auto t) {
        using T = decltype(t);
        dispatch_index(fmt, [&](auto i) {
            using I = decltype(i);
            if (sep)
                launch_gather_t<T, I, true>(g, go, win, gi, map, map_ready, border, budget, stream);
            else
                launch_gather_t<T, I, false>(g, go, win, gi, map, map_ready, border, budget, stream);
            if (need_kg) {
                if (sep)
                    launch_segrad_t<T, I, true>(op, g, go, win, gk, ws, border, stream);
                else
                    launch_segrad_t<T, I, false>(op, g, go, win, gk, ws, border, stream);
            }
        });
    });
    if (!need_kg) SB_CUDA(cudaMemsetAsync(gk, 0, g.kernel_numel() * elem_size(dtype), stream));
}

const char* op_name(int op) { return op == kErode ? "serron::erode" : "serron::dilate"; }
const char* bwd_name(int op) { return op == kErode ? "serron::erode_backward" : "serron::dilate_backward"; }

int forward_impl(int op, const void* input, const int64_t* in_sizes, int64_t in_dim, const void* kernel,
                 const int64_t* k_sizes, int64_t k_dim, int32_t dtype, int64_t border, int32_t flat, int64_t algo,
                 void* output, void* winners, int32_t winners_format, int32_t device, void* stream_) {
    return guarded([&] {
        const char* name = op_name(op);
        SB_CHECK(op == kErode || op == kDilate, "serron: invalid op ", op);
        const Geometry g = parse_geometry(name, in_sizes, in_dim, k_sizes, k_dim);
        check_common(name, dtype, border);
        const int requested = parse_algo(name, algo);
        if (g.numel() == 0) return;
        SB_CHECK(input && kernel && (output || winners), name, ": null tensor pointer");
        DeviceScope scope(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_);
        const DeviceInfo info = device_info(device);
        // a forced tiled or element-wise launch never reads the flatness
        const bool needs_flat = requested == kAuto || requested == kSeparable;
        const bool is_flat = needs_flat && resolve_flat(flat, kernel, g.kernel_numel(), dtype, stream);
        const Problem p{g.kH, g.kW, is_flat, dtype, info.smem_optin, separable_min_k(device, dtype, false)};
        const int resolved = resolve_algorithm(requested, p, name);
        if (winners) {
            // the plan's format, or the same records without the map
            const int want = winners_format_for(resolved, g.kH, g.kW);
            SB_CHECK(winners_format == want || winners_format == base_format(want), name, ": winner format ",
                     winners_format, " does not match the resolved algorithm (expected ", want, ")");
        }
        launch_forward(op, dtype, resolved, g, input, kernel, output, winners, winners_format, static_cast<int>(border),
                       info.smem_optin, stream);
    });
}

int backward_impl(int op, const void* grad_output, const int64_t* go_sizes, int64_t go_dim, const void* input,
                  const int64_t* in_sizes, int64_t in_dim, const void* kernel, const int64_t* k_sizes, int64_t k_dim,
                  int32_t dtype, int64_t border, int32_t flat, int32_t need_kg, int64_t algo, void* grad_input,
                  void* grad_kernel, void* workspace, int64_t workspace_bytes, int32_t device, void* stream_) {
    return guarded([&] {
        const char* name = bwd_name(op);
        const Geometry g = parse_geometry(name, in_sizes, in_dim, k_sizes, k_dim);
        SB_CHECK(go_dim == 4, name, ": grad_output must be 4-D (N, C, H, W), got ", go_dim, "-D");
        check_common(name, dtype, border);
        const int requested = parse_algo(name, algo);
        SB_CHECK(go_sizes[0] == g.N && go_sizes[1] == g.C && go_sizes[2] == g.H && go_sizes[3] == g.W, name,
                 ": grad_output shape must match input");
        DeviceScope scope(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_);
        if (g.numel() == 0) {
            if (g.kernel_numel() > 0) SB_CUDA(cudaMemsetAsync(grad_kernel, 0, g.kernel_numel() * elem_size(dtype), stream));
            return;
        }
        SB_CHECK(grad_output && input && kernel && grad_input && grad_kernel, name, ": null tensor pointer");
        const DeviceInfo info = device_info(device);
        const bool needs_flat = requested == kAuto || requested == kSeparable;
        const bool is_flat = needs_flat && resolve_flat(flat, kernel, g.kernel_numel(), dtype, stream);
        const Problem p{g.kH, g.kW, is_flat, dtype, info.smem_optin, separable_min_k(device, dtype, true)};
        const int resolved = resolve_algorithm(requested, p, name);
        const int fmt = winners_format_for(resolved, g.kH, g.kW);
        const int64_t need = backward_workspace(g, need_kg != 0, fmt, false);
        if (workspace_bytes < need)
            throw Failure{SERRON_ERR_WORKSPACE, concat(name, ": workspace of ", workspace_bytes, " bytes, ", need, " needed")};
        char* ws = static_cast<char*>(workspace);
        void* win = ws;
        uint32_t* map = reinterpret_cast<uint32_t*>(ws + records_bytes(g, fmt));
        launch_forward(op, dtype, resolved, g, input, kernel, nullptr, win, fmt, static_cast<int>(border),
                       info.smem_optin, stream);
        launch_backward_from_winners(op, dtype, g, grad_output, win, fmt, grad_input, grad_kernel, need_kg != 0, map,
                                     format_has_map(fmt), ws + records_bytes(g, fmt) + map_workspace(g),
                                     static_cast<int>(border), info.smem_optin, stream);
    });
}

// ------------------------------------------------------------------------------------------------
// reconstruction
// ------------------------------------------------------------------------------------------------
// Wall-clock budget of each wait of the persistent worklist (a CTA waiting for a tile to be queued):
// two seconds, or SERRON_RECON_WAIT_NS.  A healthy wait lasts at most a few tile runs per CTA of the
// grid; one that runs out ends the call with SERRON_ERR_TIMEOUT instead of holding the GPU.
unsigned long long recon_wait_budget_ns() {
    if (const char* env = std::getenv("SERRON_RECON_WAIT_NS")) {
        char* end = nullptr;
        const unsigned long long v = std::strtoull(env, &end, 10);
        if (end != env && *end == '\0' && v > 0) return v;
    }
    return 2000000000ull;
}

// seed_top / seed_bottom < 0: a full reconstruction.  Otherwise the marker (clipped by the mask) is already
// at the fixed point except near the image's top and bottom edges: only the tiles within seed_top rows of
// the top and seed_bottom rows of the bottom start queued, and the worklist carries any change from there.
int reconstruct_impl(int32_t dilate, const void* marker, const void* mask, const int64_t* sizes, int64_t dim,
                     const void* kernel, const int64_t* k_sizes, int64_t k_dim, int32_t dtype, int64_t border,
                     int64_t max_iter, int64_t check_every, void* output, void* workspace, int64_t workspace_bytes,
                     int32_t device, void* stream_, int64_t* steps, int64_t seed_top = -1, int64_t seed_bottom = -1) {
    return guarded([&] {
        const char* name = dilate ? "serron.reconstruction_by_dilation" : "serron.reconstruction_by_erosion";
        const Geometry g = parse_geometry(name, sizes, dim, k_sizes, k_dim);
        check_common(name, dtype, border);
        SB_CHECK(check_every >= 1, name, ": check_every must be >= 1, got ", check_every);
        const bool seeded = seed_top >= 0 || seed_bottom >= 0;
        SB_CHECK(!seeded || max_iter <= 0, name, ": an edge-seeded reconstruction runs to the fixed point (max_iter <= 0)");
        const int64_t total = g.numel();
        const int64_t need = serron_reconstruct_workspace_bytes(sizes, dim, dtype, max_iter);
        if (workspace_bytes < need)
            throw Failure{SERRON_ERR_WORKSPACE, concat(name, ": workspace of ", workspace_bytes, " bytes, ", need, " needed")};
        if (steps) *steps = 0;
        if (total == 0) return;
        DeviceScope scope(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_);
        int* flags = static_cast<int*>(workspace);
        void* tmp = static_cast<char*>(workspace) + 256;
        const int H = static_cast<int>(g.H), W = static_cast<int>(g.W), C = static_cast<int>(g.C);
        const int kH = static_cast<int>(g.kH), kW = static_cast<int>(g.kW), kcs = static_cast<int>(g.kcs);
        const int op = dilate ? kDilate : kErode;
        int host_flags[3] = {0, 0, 0};
        int64_t taken = 0;
        bool converged = false;
        dispatch_dtype(dtype, [&](auto t) {
            using T = decltype(t);
            dispatch_op(op, [&](auto o) {
                constexpr int OP = decltype(o)::value;
                SB_CUDA(cudaMemsetAsync(flags, 0, 3 * sizeof(int), stream));
                recon_init_kernel<T, OP><<<grid_1d((total + 255) / 256), 256, 0, stream>>>(
                    static_cast<const T*>(marker), static_cast<const T*>(mask), static_cast<T*>(output), total, flags);
                SB_CUDA(cudaGetLastError());
                if (max_iter <= 0 && kcs == 0) {
                    recon_se_class_kernel<T, OP><<<1, 32, 0, stream>>>(static_cast<const T*>(kernel), kH, kW, flags + 2);
                    SB_CUDA(cudaGetLastError());
                }
                SB_CUDA(cudaMemcpyAsync(host_flags, flags, 3 * sizeof(int), cudaMemcpyDeviceToHost, stream));
                SB_CUDA(cudaStreamSynchronize(stream));
                const bool has_nan = host_flags[1] != 0;
                if (max_iter <= 0) {
                    // a NaN never compares equal, so the reference's loop would never end
                    if (has_nan)
                        throw Failure{SERRON_ERR_NOT_CONVERGED,
                                      concat(name, ": no fixed point after None iterations; raise max_iter, or pass "
                                                   "finite inputs (a NaN never compares equal, so the convergence test "
                                                   "can never fire)")};
                    const int tx = ceil_div(W, kRecTile), ty = ceil_div(H, kRecTile);
                    const size_t smem = (static_cast<size_t>(kRecTile + kW - 1) * (kRecTile + kH - 1) +
                                         kRecTile * kRecTile + static_cast<size_t>(kH) * kW) *
                                        sizeof(typename Storage<T>::acc);
                    const long long blocks = static_cast<long long>(tx) * ty * g.N * g.C;
                    // a flat SE with an anchor and a direct neighbour: first rounds of row and column scans,
                    // which carry fronts across the image; when only the scans' taps exist and a round
                    // changes nothing, that is the fixed point
                    const int cls = host_flags[2];
                    const int lines = cls & (kScanLeft | kScanRight | kScanUp | kScanDown);
                    bool complete = false;  // the scans cover every tap of the full step
                    const int diags = cls & kScanDiag;
                    if ((cls & kScanFlat) && (lines || diags)) {
                        using A = typename Storage<T>::acc;
                        const size_t row_smem = 2 * static_cast<size_t>(kScanChunk) * sizeof(A);
                        auto rows_fn = recon_rows_kernel<T, OP>;
                        set_smem(rows_fn, row_smem);
                        const int strips = ceil_div(W, kScanCols);
                        const long long rows = g.N * g.C * g.H, strip_blocks = g.N * g.C * strips;
                        // under REFLECT a one-sided line tap at the image edge reads the pixel on its other
                        // side, which only the opposite scan covers
                        const bool lop = ((cls & kScanLeft) != 0) != ((cls & kScanRight) != 0);
                        const bool vop = ((cls & kScanUp) != 0) != ((cls & kScanDown) != 0);
                        // a folded diagonal tap lands on another tap of the 3x3 neighbourhood, which only
                        // the full square is sure to hold
                        const bool square = lines == (kScanLeft | kScanRight | kScanUp | kScanDown) && diags == kScanDiag;
                        complete = !(cls & kScanOther) &&
                                   (diags ? border == kConstant || square : !(border == kReflect && (lop || vop)));
                        // the shared-memory scan tiles alone do best when they cover the SE (measured on the
                        // 8192^2 blob mask: 176 ms with no global round, 208 ms with 8); the full-step tiles
                        // need the global rounds to carry the fronts
                        // (an edge-seeded call starts near its fixed point: no global rounds)
                        const int rounds = complete || seeded ? 0 : kScanRounds;
                        for (int round = 0; round < (lines ? rounds : 0); ++round) {
                            SB_CUDA(cudaMemsetAsync(flags, 0, sizeof(int), stream));
                            if (lines & (kScanLeft | kScanRight))
                                rows_fn<<<grid_1d(rows), kScanThreads, row_smem, stream>>>(
                                    static_cast<T*>(output), static_cast<const T*>(mask), W, cls, flags);
                            if (lines & (kScanUp | kScanDown))
                                recon_cols_kernel<T, OP><<<grid_1d(strip_blocks), kScanThreads, 0, stream>>>(
                                    static_cast<T*>(output), static_cast<const T*>(mask), H, W, strips, cls, flags);
                            SB_CUDA(cudaGetLastError());
                            ++taken;
                            SB_CUDA(cudaMemcpyAsync(host_flags, flags, sizeof(int), cudaMemcpyDeviceToHost, stream));
                            SB_CUDA(cudaStreamSynchronize(stream));
                            if (host_flags[0] == 0) {
                                converged = complete;
                                break;
                            }
                        }
                    }
                    // then tile relaxation to the fixed point in one persistent launch: a device worklist of
                    // tiles whose halo moved, solved by scans in shared memory when the scans cover the SE,
                    // else by the full step; the fixed point is reached when no tile is queued or running
                    if (!converged) {
                        ReconQueue q;
                        q.counters = reinterpret_cast<unsigned int*>(flags + 16);
                        q.state = static_cast<int*>(tmp);
                        q.cells = reinterpret_cast<unsigned long long*>(static_cast<char*>(tmp) + align256(4 * blocks));
                        q.cap = static_cast<unsigned int>(recon_queue_cap(blocks));
                        SB_CHECK(blocks < (1ll << 30), name, ": too many tiles for one call");
                        // tile rows [0, row0_end) and [row1_begin, ty) start queued: all of them, or those near the
                        // seeded edges
                        int row0_end = ty, row1_begin = ty;
                        if (seeded) {
                            const int st = static_cast<int>(std::min<int64_t>(std::max<int64_t>(seed_top, 0), H));
                            const int sb = static_cast<int>(std::min<int64_t>(std::max<int64_t>(seed_bottom, 0), H));
                            row0_end = std::min(ty, ceil_div(st, kRecTile));
                            // the tile row holding row H - sb (a last tile row can be short)
                            row1_begin = sb > 0 ? std::max(row0_end, (H - sb) / kRecTile) : ty;
                        }
                        recon_queue_init_kernel<<<grid_1d((q.cap + 255) / 256), 256, 0, stream>>>(
                            q, static_cast<int>(g.N * g.C), tx, ty, row0_end, row1_begin);
                        SB_CUDA(cudaGetLastError());
                        const unsigned long long budget = recon_wait_budget_ns();
                        const int sms = device_info(device).sm_count;
                        int per_sm = 0;
                        if (complete) {
                            using A = typename Storage<T>::acc;
                            const size_t scan_smem = scan_tile_smem<A>();
                            auto kfn = recon_persist_scan_kernel<T, OP>;
                            // six tiles per SM: registers capped by the launch bounds, shared memory by the carveout
                            set_smem(kfn, scan_smem);
                            SB_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
                            SB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kScanTileThreads, scan_smem));
                            const long long grid = std::min<long long>(blocks, std::min<long long>(kReconMaxGrid, std::max(1, per_sm) * sms));
                            kfn<<<static_cast<unsigned>(grid), kScanTileThreads, scan_smem, stream>>>(
                                static_cast<T*>(output), static_cast<const T*>(mask), H, W, tx, ty, cls, 4 * kRecTile, q,
                                budget);
                        } else {
                            auto kfn = recon_persist_full_kernel<T, OP>;
                            set_smem(kfn, smem);
                            SB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kRecThreads, smem));
                            const long long grid = std::min<long long>(blocks, std::min<long long>(kReconMaxGrid, std::max(1, per_sm) * sms));
                            // a halo within the eight neighbours, or (a window wider than a tile, or folded across an
                            // image narrower than itself) the whole plane
                            const int reach = (kH < kRecTile && kW < kRecTile && H > kH && W > kW) ? 1 : std::max(tx, ty);
                            kfn<<<static_cast<unsigned>(grid), kRecThreads, smem, stream>>>(
                                static_cast<T*>(output), static_cast<const T*>(mask), static_cast<const T*>(kernel), C, H,
                                W, kH, kW, kcs, static_cast<int>(border), tx, ty, 4 * kRecTile, reach, q, budget);
                        }
                        SB_CUDA(cudaGetLastError());
                        unsigned int counters[5] = {0, 0, 0, 0, 0};
                        SB_CUDA(cudaMemcpyAsync(counters, q.counters, sizeof(counters), cudaMemcpyDeviceToHost, stream));
                        SB_CUDA(cudaStreamSynchronize(stream));
                        if (counters[3] != 0u)
                            throw Failure{SERRON_ERR_TIMEOUT,
                                          concat(name, ": a wait of the device worklist ran out after ", budget,
                                                 " ns (status ", counters[3], "); the result is incomplete")};
                        SB_CHECK(counters[2] == 0u, name, ": the device worklist ended with ", counters[2],
                                 " tiles outstanding");
                        taken += counters[4];
                        converged = true;
                    }
                } else {
                    // the reference's Jacobi schedule: check every `check_every` steps, stop at max_iter
                    T* cur = static_cast<T*>(output);
                    T* nxt = static_cast<T*>(tmp);
                    for (int64_t it = 1; it <= max_iter; ++it) {
                        recon_step_kernel<T, OP><<<grid_1d((total + 255) / 256), 256, 0, stream>>>(
                            cur, nxt, static_cast<const T*>(mask), static_cast<const T*>(kernel), total, C, H, W, kH,
                            kW, kcs, static_cast<int>(border), flags);
                        SB_CUDA(cudaGetLastError());
                        std::swap(cur, nxt);
                        taken = it;
                        if (it % check_every == 0) {
                            SB_CUDA(cudaMemcpyAsync(host_flags, flags, sizeof(int), cudaMemcpyDeviceToHost, stream));
                            SB_CUDA(cudaStreamSynchronize(stream));
                            if (host_flags[0] == 0 && !has_nan) {
                                converged = true;
                                break;
                            }
                            SB_CUDA(cudaMemsetAsync(flags, 0, sizeof(int), stream));
                        }
                    }
                    if (!converged) {
                        SB_CUDA(cudaMemcpyAsync(host_flags, flags, sizeof(int), cudaMemcpyDeviceToHost, stream));
                        SB_CUDA(cudaStreamSynchronize(stream));
                        converged = host_flags[0] == 0 && !has_nan;
                    }
                    if (cur != static_cast<T*>(output))
                        SB_CUDA(cudaMemcpyAsync(output, cur, total * sizeof(T), cudaMemcpyDeviceToDevice, stream));
                    if (!converged)
                        throw Failure{SERRON_ERR_NOT_CONVERGED,
                                      concat(name, ": no fixed point after ", max_iter,
                                             " iterations; raise max_iter, or pass finite inputs (a NaN never "
                                             "compares equal, so the convergence test can never fire)")};
                }
            });
        });
        if (steps) *steps = taken;
        (void)converged;
    });
}

}  // namespace

// Lets the library's other translation units report a failure through serron_last_error.
void set_last_error(const std::string& message) { g_last_error = message; }

}  // namespace serron

using namespace serron;

extern "C" {

const char* serron_last_error(void) { return g_last_error.c_str(); }

int32_t serron_abi_version(void) { return 1; }

int serron_erode(const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                 const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                 int64_t algo, void* output, int32_t device, void* stream) {
    return forward_impl(kErode, input, input_sizes, input_dim, kernel, kernel_sizes, kernel_dim, dtype, border, flat,
                        algo, output, nullptr, 0, device, stream);
}

int serron_dilate(const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                  const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                  int64_t algo, void* output, int32_t device, void* stream) {
    return forward_impl(kDilate, input, input_sizes, input_dim, kernel, kernel_sizes, kernel_dim, dtype, border, flat,
                        algo, output, nullptr, 0, device, stream);
}

int serron_forward(int32_t op, const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                   const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                   int64_t algo, void* output, void* winners, int32_t winners_format, int32_t device, void* stream) {
    return forward_impl(op, input, input_sizes, input_dim, kernel, kernel_sizes, kernel_dim, dtype, border, flat, algo,
                        output, winners, winners_format, device, stream);
}

int serron_forward_autocast(int32_t op, const void* input, const int64_t* input_sizes, int64_t input_dim,
                            int32_t input_dtype, const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim,
                            int32_t kernel_dtype, int64_t border, void* output, void* winners, int32_t winners_format,
                            int32_t device, void* stream) {
    return guarded([&] {
        SB_CHECK(op == kErode || op == kDilate, "serron: invalid op ", op);
        const char* name = op_name(op);
        const Geometry g = parse_geometry(name, input_sizes, input_dim, kernel_sizes, kernel_dim);
        check_common(name, input_dtype, border);
        SB_CHECK(input_dtype == kF32 || input_dtype == kF16 || input_dtype == kBF16, name,
                 ": the autocast forward takes a float32, float16 or bfloat16 input");
        SB_CHECK(kernel_dtype == kF32, name, ": the autocast forward needs a float32 structuring element");
        SB_CHECK(autocast_fwd_supported_k(static_cast<int>(g.kH), static_cast<int>(g.kW)), name,
                 ": the autocast forward needs an odd square window of 3 to 15, got ", g.kH, "x", g.kW);
        const int fmt = winners_format_for(kTiled, g.kH, g.kW);
        SB_CHECK(winners_format == fmt, name, ": winner format ", winners_format, " (", fmt, " expected)");
        DeviceScope scope(device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (g.numel() == 0) return;
        SB_CHECK(input && kernel && output && winners, name, ": null tensor pointer");
        uint32_t* map = reinterpret_cast<uint32_t*>(static_cast<char*>(winners) + records_bytes(g, fmt));
        SB_CUDA(cudaMemsetAsync(map, 0, pull_map_words(g.N * g.C, g.H, g.W) * 4, s));
        auto aligned = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; };
        const int bulk = aligned(input, 16) && (g.W * static_cast<int64_t>(elem_size(input_dtype))) % 16 == 0;
        const int out_vec = aligned(output, 16) && aligned(winners, 8) && g.W % 8 == 0;
        SB_CUDA(autocast_fwd_launch(op, input_dtype, static_cast<int>(g.kH), input, static_cast<const float*>(kernel),
                                    static_cast<__half*>(output), static_cast<uint8_t*>(winners), map, g.N * g.C,
                                    static_cast<int>(g.C), static_cast<int>(g.H), static_cast<int>(g.W),
                                    static_cast<int>(g.kcs), static_cast<int>(border), bulk, out_vec, s));
    });
}

int serron_derived_supported(int32_t mode, const int64_t* input_sizes, int64_t input_dim, const int64_t* kernel_sizes,
                             int64_t kernel_dim) {
    if (input_dim != 4 || input_sizes == nullptr || kernel_sizes == nullptr || (kernel_dim != 2 && kernel_dim != 3))
        return 0;
    return derived_supported(mode, input_sizes[2], input_sizes[3], kernel_sizes[kernel_dim - 2],
                             kernel_sizes[kernel_dim - 1])
               ? 1
               : 0;
}

int serron_derived_forward(int32_t mode, const void* input, const int64_t* input_sizes, int64_t input_dim,
                           const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype,
                           int64_t border, void* output, void* winners_a, void* winners_b, int32_t winners_format,
                           int32_t device, void* stream) {
    return guarded([&] {
        static const char* const names[] = {"serron.gradient", "serron.opening", "serron.closing", "serron.top_hat",
                                            "serron.black_hat"};
        SB_CHECK(mode >= 0 && mode <= 4, "serron: invalid derived operation ", mode);
        const char* name = names[mode];
        const Geometry g = parse_geometry(name, input_sizes, input_dim, kernel_sizes, kernel_dim);
        check_common(name, dtype, border);
        SB_CHECK(derived_supported(mode, g.H, g.W, g.kH, g.kW), name, ": no one-launch form for a ", g.kH, "x", g.kW,
                 " window on a ", g.H, "x", g.W, " image (windows up to ", kDerivedMaxK, " a side)");
        const int fmt = SERRON_WINNERS_DIRECT_U8 | SERRON_WINNERS_MAP;
        SB_CHECK(winners_format == fmt, name, ": winner format ", winners_format, " (", fmt, " expected)");
        DeviceScope scope(device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (g.numel() == 0) return;
        SB_CHECK(input && kernel && output && winners_a && winners_b, name, ": null tensor pointer");
        const int64_t map_bytes = pull_map_words(g.N * g.C, g.H, g.W) * 4;
        uint32_t* map_a = reinterpret_cast<uint32_t*>(static_cast<char*>(winners_a) + records_bytes(g, fmt));
        uint32_t* map_b = reinterpret_cast<uint32_t*>(static_cast<char*>(winners_b) + records_bytes(g, fmt));
        SB_CUDA(cudaMemsetAsync(map_a, 0, map_bytes, s));
        SB_CUDA(cudaMemsetAsync(map_b, 0, map_bytes, s));
        SB_CUDA(derived_fwd_launch(mode, dtype, input, kernel, output, static_cast<uint8_t*>(winners_a),
                                   static_cast<uint8_t*>(winners_b), map_a, map_b, g.N * g.C, static_cast<int>(g.C),
                                   static_cast<int>(g.H), static_cast<int>(g.W), static_cast<int>(g.kH),
                                   static_cast<int>(g.kW), static_cast<int>(g.kcs), static_cast<int>(border), s));
    });
}

int64_t serron_winners_bytes(const int64_t* sizes, int64_t dim, int32_t winners_format) {
    int64_t out = -1;
    const int rc = guarded([&] {
        const char* name = "serron::winners_bytes";
        SB_CHECK(dim == 4 && sizes != nullptr, name, ": input must be 4-D (N, C, H, W), got ", dim, "-D");
        const int base = base_format(winners_format);
        SB_CHECK(base >= SERRON_WINNERS_DIRECT_U8 && base <= SERRON_WINNERS_SEPARABLE_U32 &&
                     (winners_format & ~(SERRON_WINNERS_MAP | 0xf)) == 0 &&
                     !(format_has_map(winners_format) && format_is_separable(winners_format)),
                 name, ": invalid winner format ", winners_format);
        Geometry g;
        g.N = sizes[0];
        g.C = sizes[1];
        g.H = sizes[2];
        g.W = sizes[3];
        SB_CHECK(g.N >= 0 && g.C >= 0 && g.H >= 0 && g.W >= 0, name, ": input sizes must be non-negative");
        out = winners_buffer_bytes(g, winners_format);
    });
    return rc == SERRON_OK ? out : -1;
}

int serron_plan(const int64_t* input_sizes, int64_t input_dim, const void* kernel, const int64_t* kernel_sizes,
                int64_t kernel_dim, int32_t dtype, int32_t flat, int64_t algo, int32_t backward, int32_t device,
                void* stream, serron_plan_t* plan) {
    return guarded([&] {
        const char* name = backward ? "serron::plan(backward)" : "serron::plan";
        const Geometry g = parse_geometry(name, input_sizes, input_dim, kernel_sizes, kernel_dim);
        check_common(name, dtype, 0);
        const int requested = parse_algo(name, algo);
        SB_CHECK(plan != nullptr, name, ": plan must not be null");
        DeviceScope scope(device);
        const DeviceInfo info = device_info(device);
        const bool needs_flat = requested == kAuto || requested == kSeparable;
        const bool is_flat = needs_flat && resolve_flat(flat, kernel, g.kernel_numel(), dtype,
                                                        static_cast<cudaStream_t>(stream));
        const Problem p{g.kH, g.kW, is_flat, dtype, info.smem_optin, separable_min_k(device, dtype, backward != 0)};
        const int resolved = resolve_algorithm(requested, p, name);
        plan->algo = resolved;
        plan->winners_format = winners_format_for(resolved, g.kH, g.kW);
        plan->winners_bytes = format_bytes(plan->winners_format);
        plan->reserved = 0;
        plan->workspace_bytes = backward_workspace(g, true, plan->winners_format, false);
    });
}

int serron_erode_backward(const void* grad_output, const int64_t* grad_output_sizes, int64_t grad_output_dim,
                          const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                          const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                          int32_t need_kernel_grad, int64_t algo, void* grad_input, void* grad_kernel, void* workspace,
                          int64_t workspace_bytes, int32_t device, void* stream) {
    return backward_impl(kErode, grad_output, grad_output_sizes, grad_output_dim, input, input_sizes, input_dim, kernel,
                         kernel_sizes, kernel_dim, dtype, border, flat, need_kernel_grad, algo, grad_input,
                         grad_kernel, workspace, workspace_bytes, device, stream);
}

int serron_dilate_backward(const void* grad_output, const int64_t* grad_output_sizes, int64_t grad_output_dim,
                           const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                           const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border,
                           int32_t flat, int32_t need_kernel_grad, int64_t algo, void* grad_input, void* grad_kernel,
                           void* workspace, int64_t workspace_bytes, int32_t device, void* stream) {
    return backward_impl(kDilate, grad_output, grad_output_sizes, grad_output_dim, input, input_sizes, input_dim,
                         kernel, kernel_sizes, kernel_dim, dtype, border, flat, need_kernel_grad, algo, grad_input,
                         grad_kernel, workspace, workspace_bytes, device, stream);
}

int serron_backward_from_winners(int32_t op, const void* grad_output, const int64_t* sizes, int64_t dim,
                                 const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border,
                                 int32_t need_kernel_grad, const void* winners, int32_t winners_format,
                                 void* grad_input, void* grad_kernel, void* workspace, int64_t workspace_bytes,
                                 int32_t device, void* stream) {
    return guarded([&] {
        const char* name = bwd_name(op);
        SB_CHECK(op == kErode || op == kDilate, "serron: invalid op ", op);
        const Geometry g = parse_geometry(name, sizes, dim, kernel_sizes, kernel_dim);
        check_common(name, dtype, border);
        const int base = base_format(winners_format);
        SB_CHECK(base >= SERRON_WINNERS_DIRECT_U8 && base <= SERRON_WINNERS_SEPARABLE_U32 &&
                     (winners_format & ~(SERRON_WINNERS_MAP | 0xf)) == 0 &&
                     !(format_has_map(winners_format) && format_is_separable(winners_format)),
                 name, ": invalid winner format ", winners_format);
        const int want = format_is_separable(base) ? separable_format(g.kH, g.kW) : direct_format(g.kH, g.kW);
        SB_CHECK(base == want, name, ": winner format ", winners_format, " does not fit a ", g.kH, "x", g.kW,
                 " window");
        DeviceScope scope(device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (g.numel() == 0) {
            if (g.kernel_numel() > 0) SB_CUDA(cudaMemsetAsync(grad_kernel, 0, g.kernel_numel() * elem_size(dtype), s));
            return;
        }
        const int64_t need = backward_workspace(g, need_kernel_grad != 0, winners_format, true);
        if (workspace_bytes < need)
            throw Failure{SERRON_ERR_WORKSPACE, concat(name, ": workspace of ", workspace_bytes, " bytes, ", need, " needed")};
        SB_CHECK(grad_output && winners && grad_input && grad_kernel, name, ": null tensor pointer");
        const DeviceInfo info = device_info(device);
        const bool has_map = format_has_map(winners_format);
        char* ws = static_cast<char*>(workspace);
        uint32_t* map = has_map ? reinterpret_cast<uint32_t*>(static_cast<char*>(const_cast<void*>(winners)) +
                                                              records_bytes(g, winners_format))
                                : reinterpret_cast<uint32_t*>(ws);
        launch_backward_from_winners(op, dtype, g, grad_output, winners, winners_format, grad_input, grad_kernel,
                                     need_kernel_grad != 0, map, has_map, has_map ? ws : ws + map_workspace(g),
                                     static_cast<int>(border), info.smem_optin, s);
    });
}

int serron_backward_from_winners_widened(int32_t op, const void* grad_output, int32_t grad_output_dtype,
                                         const int64_t* sizes, int64_t dim, const int64_t* kernel_sizes,
                                         int64_t kernel_dim, int64_t border, int32_t need_kernel_grad,
                                         const void* winners, int32_t winners_format, void* grad_input,
                                         int32_t grad_input_dtype, void* grad_kernel, void* workspace,
                                         int64_t workspace_bytes, int32_t device, void* stream) {
    return guarded([&] {
        const char* name = bwd_name(op);
        SB_CHECK(op == kErode || op == kDilate, "serron: invalid op ", op);
        const Geometry g = parse_geometry(name, sizes, dim, kernel_sizes, kernel_dim);
        check_common(name, kF32, border);
        auto half_or_float = [](int32_t d) { return d == kF32 || d == kF16 || d == kBF16; };
        SB_CHECK(half_or_float(grad_output_dtype) && half_or_float(grad_input_dtype), name,
                 ": the widened backward reads and writes float32, float16 or bfloat16");
        const int base = base_format(winners_format);
        SB_CHECK((base == SERRON_WINNERS_DIRECT_U8 || base == SERRON_WINNERS_DIRECT_U16) &&
                     format_has_map(winners_format) && (winners_format & ~(SERRON_WINNERS_MAP | 0xf)) == 0 &&
                     base == direct_format(g.kH, g.kW),
                 name, ": the widened backward needs direct one- or two-byte records with their target map, got format ",
                 winners_format);
        DeviceScope scope(device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (g.numel() == 0) {
            if (g.kernel_numel() > 0) SB_CUDA(cudaMemsetAsync(grad_kernel, 0, g.kernel_numel() * sizeof(float), s));
            return;
        }
        const int64_t need = backward_workspace(g, need_kernel_grad != 0, winners_format, true);
        if (workspace_bytes < need)
            throw Failure{SERRON_ERR_WORKSPACE, concat(name, ": workspace of ", workspace_bytes, " bytes, ", need, " needed")};
        SB_CHECK(grad_output && winners && grad_input && grad_kernel, name, ": null tensor pointer");
        const DeviceInfo info = device_info(device);
        SB_CHECK(pull_applicable(g, static_cast<int>(border), elem_size(grad_output_dtype), format_bytes(winners_format),
                                 info.smem_optin),
                 name, ": the widened backward does not fit this window and image");
        const uint32_t* map = reinterpret_cast<const uint32_t*>(static_cast<const char*>(winners) +
                                                                records_bytes(g, winners_format));
        auto with_index = [&](auto tg, auto to) {
            using TG = decltype(tg);
            using TO = decltype(to);
            if (base == SERRON_WINNERS_DIRECT_U8)
                launch_backward_widened_t<TG, TO, uint8_t>(op, g, grad_output, winners, grad_input, grad_kernel,
                                                           need_kernel_grad != 0, map, workspace, static_cast<int>(border), s);
            else
                launch_backward_widened_t<TG, TO, uint16_t>(op, g, grad_output, winners, grad_input, grad_kernel,
                                                            need_kernel_grad != 0, map, workspace, static_cast<int>(border), s);
        };
        auto with_out = [&](auto tg) {
            switch (grad_input_dtype) {
            case kF32: with_index(tg, float{}); break;
            case kF16: with_index(tg, __half{}); break;
            default: with_index(tg, __nv_bfloat16{}); break;
            }
        };
        switch (grad_output_dtype) {
        case kF32: with_out(float{}); break;
        case kF16: with_out(__half{}); break;
        default: with_out(__nv_bfloat16{}); break;
        }
    });
}

int64_t serron_backward_workspace_bytes(const int64_t* sizes, int64_t dim, const int64_t* kernel_sizes,
                                        int64_t kernel_dim, int32_t need_kernel_grad, int32_t winners_format,
                                        int32_t with_winners) {
    int64_t out = -1;
    const int rc = guarded([&] {
        const Geometry g = parse_geometry("serron::backward_workspace_bytes", sizes, dim, kernel_sizes, kernel_dim);
        out = backward_workspace(g, need_kernel_grad != 0, winners_format, with_winners != 0);
    });
    return rc == SERRON_OK ? out : -1;
}

int64_t serron_feasible_algos(const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int32_t flat,
                              int32_t backward, int32_t device) {
    int64_t mask = -1;
    const int rc = guarded([&] {
        const char* name = "serron::feasible_algos";
        SB_CHECK(kernel_dim == 2 || kernel_dim == 3, name, ": kernel must be 2-D (kH, kW) or 3-D (C, kH, kW), got ",
                 kernel_dim, "-D");
        const int64_t kH = kernel_sizes[kernel_dim - 2], kW = kernel_sizes[kernel_dim - 1];
        SB_CHECK(kH > 0 && kW > 0, name, ": kernel spatial dims must be positive");
        check_common(name, dtype, 0);
        DeviceScope scope(device);
        const Problem p{kH, kW, flat > 0, dtype, device_info(device).smem_optin,
                        separable_min_k(device, dtype, backward != 0)};
        mask = (int64_t(1) << kElement) | (tiled_feasible(p) ? (int64_t(1) << kTiled) : 0) |
               (separable_feasible(p) ? (int64_t(1) << kSeparable) : 0);
    });
    return rc == SERRON_OK ? mask : -1;
}

int64_t serron_heuristic_algo(const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int32_t flat,
                              int32_t backward, int32_t device) {
    int64_t algo = -1;
    const int rc = guarded([&] {
        const char* name = "serron::heuristic_algo";
        SB_CHECK(kernel_dim == 2 || kernel_dim == 3, name, ": kernel must be 2-D (kH, kW) or 3-D (C, kH, kW), got ",
                 kernel_dim, "-D");
        const int64_t kH = kernel_sizes[kernel_dim - 2], kW = kernel_sizes[kernel_dim - 1];
        SB_CHECK(kH > 0 && kW > 0, name, ": kernel spatial dims must be positive");
        check_common(name, dtype, 0);
        DeviceScope scope(device);
        const Problem p{kH, kW, flat > 0, dtype, device_info(device).smem_optin,
                        separable_min_k(device, dtype, backward != 0)};
        algo = heuristic(p);
    });
    return rc == SERRON_OK ? algo : -1;
}

int64_t serron_set_separable_min_k(int32_t device, int32_t dtype, int32_t backward, int64_t min_k) {
    auto& t = thresholds();
    {
        const std::scoped_lock lock(t.mutex);
        const std::tuple<int, int, bool> key{device, dtype, backward != 0};
        if (min_k > 0)
            t.values[key] = min_k;
        else
            t.values.erase(key);
    }
    return separable_min_k(device, dtype, backward != 0);
}

int64_t serron_get_separable_min_k(int32_t device, int32_t dtype, int32_t backward) {
    return separable_min_k(device, dtype, backward != 0);
}

int serron_reconstruct(int32_t dilate, const void* marker, const void* mask, const int64_t* sizes, int64_t dim,
                       const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype,
                       int64_t border, int64_t max_iter, int64_t check_every, void* output, void* workspace,
                       int64_t workspace_bytes, int32_t device, void* stream, int64_t* steps) {
    return reconstruct_impl(dilate, marker, mask, sizes, dim, kernel, kernel_sizes, kernel_dim, dtype, border, max_iter,
                            check_every, output, workspace, workspace_bytes, device, stream, steps);
}

int serron_reconstruct_from_edges(int32_t dilate, const void* marker, const void* mask, const int64_t* sizes,
                                  int64_t dim, const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim,
                                  int32_t dtype, int64_t border, int64_t seed_top, int64_t seed_bottom, void* output,
                                  void* workspace, int64_t workspace_bytes, int32_t device, void* stream,
                                  int64_t* steps) {
    if (seed_top < 0 || seed_bottom < 0) {
        g_last_error = "serron.reconstruction: seed_top and seed_bottom must be >= 0";
        return SERRON_ERR_INVALID;
    }
    return reconstruct_impl(dilate, marker, mask, sizes, dim, kernel, kernel_sizes, kernel_dim, dtype, border, 0, 1,
                            output, workspace, workspace_bytes, device, stream, steps, seed_top, seed_bottom);
}

int64_t serron_reconstruct_workspace_bytes(const int64_t* sizes, int64_t dim, int32_t dtype, int64_t max_iter) {
    if (dim != 4 || sizes == nullptr || dtype < kF32 || dtype > kBF16) return -1;
    const int64_t total = sizes[0] * sizes[1] * sizes[2] * sizes[3];
    // the Jacobi schedule's second buffer, or the device worklist: a state word per tile and the ring
    const int64_t tiles = sizes[0] * sizes[1] * ((sizes[2] + kRecTile - 1) / kRecTile) * ((sizes[3] + kRecTile - 1) / kRecTile);
    return 256 + (max_iter > 0 ? align256(total * static_cast<int64_t>(elem_size(dtype)))
                               : align256(4 * tiles) + align256(8 * recon_queue_cap(tiles)));
}

}  // extern "C"
