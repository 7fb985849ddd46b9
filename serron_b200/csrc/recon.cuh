// Geodesic reconstruction.
//
// Reference: torch-ext/serron/functional.py:144-202 iterates y <- clip(step(y), mask) (step = dilate
// and clip = minimum for reconstruction by dilation; erode / maximum for the dual) with a Jacobi
// schedule until a check every `check_every` steps sees no change.
//
// The step map is monotone and the iteration starts below its least fixed point (the anchor tap is
// >= 0), so every schedule that keeps applying the step to some pixels until none changes reaches the
// same fixed point.  `full_tile_solve` exploits that: a CTA loads a tile plus halo, iterates it in
// shared memory until the tile is stable, writes it back and asks for its neighbours to run again if
// anything changed (recon_persist.cuh runs that worklist in one launch).  One tile run advances a front
// across a whole tile instead of one pixel.  `recon_step_kernel` is the plain Jacobi step, used when the caller
// bounds the iteration count (max_iter), whose outcome depends on the reference's exact schedule.
#pragma once

#include "common.cuh"

#include <type_traits>

namespace serron {

constexpr int kRecTile = 64;     // recon tile: 64 x 64 pixels, 256 threads, 16 pixels per thread
constexpr int kRecThreads = 256;

// A load that bypasses L1 (ld.global.cg): pixels another CTA may have written during this launch.
template <typename T>
__device__ __forceinline__ T load_cg(const T* p) {
    if constexpr (std::is_same<T, __half>::value) {
        return __ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(p)));
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        return __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(p)));
    } else {
        return __ldcg(p);
    }
}

template <int OP>
struct Clip;  // the clip against the mask that follows a step
template <>
struct Clip<kDilate> {  // reconstruction by dilation: torch.minimum (NaN propagates)
    template <typename A>
    static __device__ __forceinline__ A apply(A v, A m) { return (v != v) ? v : (m != m) ? m : (m < v ? m : v); }
};
template <>
struct Clip<kErode> {  // reconstruction by erosion: torch.maximum
    template <typename A>
    static __device__ __forceinline__ A apply(A v, A m) { return (v != v) ? v : (m != m) ? m : (m > v ? m : v); }
};

// one step for pixel (h, w): op over the window (samples from `sample(dr, dc, s)`), rounded to the
// storage type, then clipped
template <typename T, int OP, typename Sample, typename Weight>
__device__ __forceinline__ typename Storage<T>::acc recon_update(const Sample& sample, const Weight& weight, int kH,
                                                                 int kW, typename Storage<T>::acc m) {
    using A = typename Storage<T>::acc;
    A best = Op<OP>::template neutral<A>();
    for (int di = 0; di < kH; ++di)
        for (int dj = 0; dj < kW; ++dj) {
            A s;
            if (!sample(di, dj, s)) continue;
            const A v = Op<OP>::tap(s, weight(di, dj));
            if (Op<OP>::better(v, best)) best = v;
        }
    best = Storage<T>::load(Storage<T>::store(best));
    return Clip<OP>::apply(best, m);
}

// y <- clip(marker, mask), and a NaN probe (flags[1] |= 1 when any NaN is present)
template <typename T, int OP>
__global__ void recon_init_kernel(const T* __restrict__ marker, const T* __restrict__ mask, T* __restrict__ y,
                                  long long total, int* __restrict__ flags) {
    using A = typename Storage<T>::acc;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const A a = Storage<T>::load(marker[i]), m = Storage<T>::load(mask[i]);
    if (a != a || m != m) atomicOr(flags + 1, 1);
    y[i] = Storage<T>::store(Clip<OP>::apply(a, m));
}

// Full-step tile: solves tile b (tiles numbered plane by plane, row-major within a plane) in shared
// memory with the step itself, writes it back if it changed, and returns the neighbours to run again
// as bits 3 * (dy + 1) + (dx + 1): all eight when anything changed, bit 4 (this tile) when its inner
// iterations ran out.  y is read through L2 (the persistent driver runs a tile on whichever CTA pops
// it).
template <typename T, int OP>
__device__ __forceinline__ unsigned full_tile_solve(long long b, T* __restrict__ y, const T* __restrict__ mask,
                                                    const T* __restrict__ w, int C, int H, int W, int kH, int kW,
                                                    int kcs, int border, int tiles_x, int tiles_y, int max_inner,
                                                    unsigned char* smem_raw) {
    using A = typename Storage<T>::acc;
    const int aH = kH / 2, aW = kW / 2;
    const int sw = kRecTile + kW - 1, sh = kRecTile + kH - 1;
    A* ys = reinterpret_cast<A*>(smem_raw);       // [sh][sw] current values with halo
    A* ms = ys + sw * sh;                          // [TILE][TILE] mask
    A* ws = ms + kRecTile * kRecTile;              // [kH*kW]

    const int tx = static_cast<int>(b % tiles_x), ty = static_cast<int>((b / tiles_x) % tiles_y);
    const long long plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    const int c = static_cast<int>(plane % C);
    const int h0 = ty * kRecTile, w0 = tx * kRecTile;
    T* yp = y + plane * H * W;
    const T* mp = mask + plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int tid = threadIdx.x;
    const A neutral = Op<OP>::template neutral<A>();

    for (int i = tid; i < kH * kW; i += kRecThreads) ws[i] = Storage<T>::load(wc[i]);
    for (int i = tid; i < sw * sh; i += kRecThreads) {
        const int r = i / sw, q = i - r * sw;
        int gr = h0 - aH + r, gq = w0 - aW + q;
        A v = neutral;
        if (resolve(gr, H, border) && resolve(gq, W, border))
            v = Storage<T>::load(load_cg(yp + static_cast<long long>(gr) * W + gq));
        ys[i] = v;
    }
    for (int i = tid; i < kRecTile * kRecTile; i += kRecThreads) {
        const int r = i / kRecTile, q = i - r * kRecTile;
        const int gr = h0 + r, gq = w0 + q;
        ms[i] = (gr < H && gq < W) ? Storage<T>::load(mp[static_cast<long long>(gr) * W + gq]) : neutral;
    }
    __syncthreads();

    // Border-resolved halo cells that alias a pixel of this tile (REFLECT/REPLICATE at the image edge)
    // must follow that pixel; the sample function reads through the resolved coordinate when the
    // aliased pixel lies inside the tile.
    auto sample_at = [&](int lr, int lq, int di, int dj, A& s) {
        int gr = h0 + lr + di - aH, gq = w0 + lq + dj - aW;
        if (!resolve(gr, H, border) || !resolve(gq, W, border)) return false;
        const int sr = gr - h0 + aH, sq = gq - w0 + aW;
        if (sr < 0 || sr >= sh || sq < 0 || sq >= sw) {
            // a window folded from beyond the staged halo (REFLECT on an image narrower than the
            // window): read the current global value; a stale value only delays convergence
            s = Storage<T>::load(load_cg(yp + static_cast<long long>(gr) * W + gq));
            return true;
        }
        s = ys[sr * sw + sq];
        return true;
    };
    auto weight = [&](int di, int dj) { return ws[di * kW + dj]; };

    bool any_change = false, settled = false;
    for (int it = 0; it < max_inner; ++it) {
        bool changed = false;
        for (int i = tid; i < kRecTile * kRecTile; i += kRecThreads) {
            const int lr = i / kRecTile, lq = i - lr * kRecTile;
            if (h0 + lr >= H || w0 + lq >= W) continue;
            auto sample = [&](int di, int dj, A& s) { return sample_at(lr, lq, di, dj, s); };
            const int si = (lr + aH) * sw + lq + aW;
            const A old = ys[si];
            const A v = recon_update<T, OP>(sample, weight, kH, kW, ms[i]);
            if (!(v == old) && !(v != v && old != old)) {
                ys[si] = v;
                changed = true;
            }
        }
        changed = __syncthreads_or(changed);
        if (!changed) {
            settled = true;
            break;
        }
        any_change = true;
    }
    if (!any_change) return 0u;
    for (int i = tid; i < kRecTile * kRecTile; i += kRecThreads) {
        const int lr = i / kRecTile, lq = i - lr * kRecTile;
        const int gr = h0 + lr, gq = w0 + lq;
        if (gr < H && gq < W) yp[static_cast<long long>(gr) * W + gq] = Storage<T>::store(ys[(lr + aH) * sw + lq + aW]);
    }
    // the eight neighbours, and the tile itself when its inner iterations ran out before it settled
    return 0x1efu | (settled ? 0u : 0x10u);
}

// One Jacobi step y_out = clip(op(y_in), mask); changed[0] |= any pixel differs from y_in.
template <typename T, int OP>
__global__ void __launch_bounds__(256) recon_step_kernel(const T* __restrict__ yin, T* __restrict__ yout,
                                                         const T* __restrict__ mask, const T* __restrict__ w,
                                                         long long total, int C, int H, int W, int kH, int kW,
                                                         int kcs, int border, int* __restrict__ changed) {
    using A = typename Storage<T>::acc;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int ow = static_cast<int>(idx % W), oh = static_cast<int>((idx / W) % H);
    const long long plane = idx / (static_cast<long long>(W) * H);
    const int c = static_cast<int>(plane % C);
    const T* xp = yin + plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int aH = kH / 2, aW = kW / 2;
    auto sample = [&](int di, int dj, A& s) {
        int r = oh + di - aH, q = ow + dj - aW;
        if (!resolve(r, H, border) || !resolve(q, W, border)) return false;
        s = Storage<T>::load(xp[static_cast<long long>(r) * W + q]);
        return true;
    };
    auto weight = [&](int di, int dj) { return Storage<T>::load(wc[di * kW + dj]); };
    const A v = recon_update<T, OP>(sample, weight, kH, kW, Storage<T>::load(mask[idx]));
    const A old = Storage<T>::load(yin[idx]);
    yout[idx] = Storage<T>::store(v);
    if (!(v == old)) atomicOr(changed, 1);
}

}  // namespace serron
