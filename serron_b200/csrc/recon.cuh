// Geodesic reconstruction.
//
// Reference: torch-ext/serron/functional.py:144-202 iterates y <- clip(step(y), mask) (step = dilate
// and clip = minimum for reconstruction by dilation; erode / maximum for the dual) with a Jacobi
// schedule until a check every `check_every` steps sees no change.
//
// The step map is monotone and the iteration starts below its least fixed point (the anchor tap is
// >= 0), so every schedule that keeps applying the step to some pixels until none changes reaches the
// same fixed point.  `recon_tile_kernel` exploits that: each CTA loads a tile plus halo, iterates it in
// shared memory until the tile is stable, writes it back and raises a device flag if anything
// changed; the host relaunches until a launch changes nothing.  One launch advances a front across a
// whole tile instead of one pixel.  `recon_step_kernel` is the plain Jacobi step, used when the caller
// bounds the iteration count (max_iter), whose outcome depends on the reference's exact schedule.
#pragma once

#include "common.cuh"

namespace serron {

constexpr int kRecTile = 64;     // recon tile: 64 x 64 pixels, 256 threads, 16 pixels per thread
constexpr int kRecThreads = 256;

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

// With `dirty_in`, a launch runs only the tiles flagged in it, and a tile that changed flags its eight
// neighbours (and itself, if its inner iterations ran out) in `dirty_out`.  Two arrays, swapped and
// cleared by the host between launches: a tile that read a neighbour's halo while the neighbour was
// still changing it is flagged for the next launch, which sees the neighbour's final writes.
// flags[0] is raised whenever a flag is set; the host stops when a launch sets none.  Without
// `dirty_in` every tile runs and flags[0] says whether anything changed.
template <typename T, int OP>
__global__ void __launch_bounds__(kRecThreads) recon_tile_kernel(T* __restrict__ y, const T* __restrict__ mask,
                                                                 const T* __restrict__ w, int C, int H, int W, int kH,
                                                                 int kW, int kcs, int border, int tiles_x,
                                                                 int tiles_y, int max_inner, int* __restrict__ flags,
                                                                 const uint8_t* __restrict__ dirty_in,
                                                                 uint8_t* __restrict__ dirty_out) {
    using A = typename Storage<T>::acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int aH = kH / 2, aW = kW / 2;
    const int sw = kRecTile + kW - 1, sh = kRecTile + kH - 1;
    A* ys = reinterpret_cast<A*>(smem_raw);       // [sh][sw] current values with halo
    A* ms = ys + sw * sh;                          // [TILE][TILE] mask
    A* ws = ms + kRecTile * kRecTile;              // [kH*kW]

    const long long b = blockIdx.x;
    const int tx = static_cast<int>(b % tiles_x), ty = static_cast<int>((b / tiles_x) % tiles_y);
    const long long plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    const int c = static_cast<int>(plane % C);
    const int h0 = ty * kRecTile, w0 = tx * kRecTile;
    T* yp = y + plane * H * W;
    const T* mp = mask + plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int tid = threadIdx.x;
    const A neutral = Op<OP>::template neutral<A>();

    if (dirty_in && !dirty_in[b]) return;  // one byte, read alike by every thread
    for (int i = tid; i < kH * kW; i += kRecThreads) ws[i] = Storage<T>::load(wc[i]);
    for (int i = tid; i < sw * sh; i += kRecThreads) {
        const int r = i / sw, q = i - r * sw;
        int gr = h0 - aH + r, gq = w0 - aW + q;
        A v = neutral;
        if (resolve(gr, H, border) && resolve(gq, W, border)) v = Storage<T>::load(yp[static_cast<long long>(gr) * W + gq]);
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
            s = Storage<T>::load(yp[static_cast<long long>(gr) * W + gq]);
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
    if (any_change) {
        for (int i = tid; i < kRecTile * kRecTile; i += kRecThreads) {
            const int lr = i / kRecTile, lq = i - lr * kRecTile;
            const int gr = h0 + lr, gq = w0 + lq;
            if (gr < H && gq < W) yp[static_cast<long long>(gr) * W + gq] = Storage<T>::store(ys[(lr + aH) * sw + lq + aW]);
        }
        if (dirty_in) {
            // the neighbours, and the tile itself when its inner iterations ran out before it settled
            if (tid < 9 && (tid != 4 || !settled)) {
                const int nx = tx + tid % 3 - 1, ny = ty + tid / 3 - 1;
                if (nx >= 0 && nx < tiles_x && ny >= 0 && ny < tiles_y)
                    dirty_out[plane * tiles_x * tiles_y + static_cast<long long>(ny) * tiles_x + nx] = 1;
            }
        }
        if (tid == 0) atomicOr(flags, 1);
    }
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
