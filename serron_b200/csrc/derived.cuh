// Derived operations in one launch: the morphological gradient from one staged tile, and opening,
// closing, top-hat and black-hat with the intermediate image kept in shared memory.
//
// The reference composes them from primitive calls (packages/serron/torch-ext/serron/functional.py:40-92):
//   gradient  = dilation(x) - erosion(x)        top_hat   = x - opening(x)
//   opening   = dilation(erosion(x))            black_hat = closing(x) - x
//   closing   = erosion(dilation(x))
// each primitive writing a tensor of the storage type, each subtraction done in that type.  A CTA here
// owns a 32x32 output tile:
//   gradient  stages x with the window's halo once and finds, per output, both the dilation and the
//             erosion winner over the same samples; y = T(D) - T(E).
//   two-stage stages x with twice the halo, computes the first operation on the tile grown by one halo
//             (the intermediate z, rounded to the storage type like the reference's intermediate tensor),
//             gives z's positions outside the image the border's treatment (REPLICATE / REFLECT: the z of
//             the folded pixel, which lies in the grown tile because the image is at least as large as
//             the window), then the second operation on the tile; top_hat and black_hat subtract in the
//             epilogue.
// A CONSTANT pad (of x, or of z) is staged as a NaN: no compare with it is true, so it never wins, exactly
// as the reference's neutral padding never does, for either operation of the gradient.
// Winners: the first strict improvement in (di, dj) order, float ties settled in double for inexact float
// weights, as the primitive kernels do.  Both stages write direct records (the first stage only for the
// intermediate pixels the tile owns) and set their gather target maps, so the backward is two gathers.
#pragma once

#include "direct.cuh"

namespace serron {

constexpr int kDerivedGradient = 0, kDerivedOpening = 1, kDerivedClosing = 2, kDerivedTopHat = 3,
              kDerivedBlackHat = 4;
constexpr int kDerivedMaxK = 7;  // the grown tile's extra work stays below (1 + 6/32)^2 = 1.41x

__host__ __device__ constexpr bool derived_two_stage(int mode) { return mode != kDerivedGradient; }
// the first stage's operation: erosion for opening and top-hat, dilation for closing and black-hat
__host__ __device__ constexpr int derived_first_op(int mode) {
    return (mode == kDerivedOpening || mode == kDerivedTopHat) ? kErode : kDilate;
}

// Shared-memory layout (in elements of the arithmetic type A, then ints and mark words):
//   xs  staged x: rows TO + s * (kH - 1), pitch px (s = 2 for two stages, 1 for the gradient)
//   zs  intermediate (two stages): rows TO + kH - 1, pitch pz
//   ws  weights [kH * kW], span [kH][2]
// Pitches are odd and leave three columns past the last quad's samples.
struct DerivedGeom {
    int sx, px, rz, cz, pz;
    size_t xs_elems, zs_elems;
    __host__ __device__ DerivedGeom(int kH, int kW, bool two) {
        const int s = two ? 2 : 1;
        sx = kTile + s * (kH - 1);
        rz = kTile + kH - 1;
        cz = kTile + kW - 1;
        // stage one computes quads over cz columns (the last quad may pass cz by up to 3)
        const int first_cols = two ? (cz + 3) / 4 * 4 : kTile;
        px = (first_cols + kW - 1 + 3) | 1;
        pz = (kTile + kW - 1 + 3) | 1;
        xs_elems = static_cast<size_t>(sx) * px;
        zs_elems = two ? static_cast<size_t>(rz + 1) * pz : 0;
    }
    __host__ __device__ size_t marks_offset(int kH, int kW, size_t acc) const {
        const size_t core = (xs_elems + zs_elems + static_cast<size_t>(kH) * kW) * acc + static_cast<size_t>(kH) * 2 * 4;
        return (core + 15) / 16 * 16;
    }
    __host__ __device__ size_t bytes(int kH, int kW, size_t acc) const {
        return marks_offset(kH, kW, acc) + 2 * mark_bytes(kTile, kTile, kH, kW);
    }
};

// Best value and winning tap of four adjacent outputs of op OP: output k reads rows lr .. lr + kH - 1 and
// columns q0 + k .. q0 + k + kW - 1 of `src` (pitch sp); a float tie with the running best is settled in
// double over the same samples when the weights are not exact.
template <typename T, int OP>
__device__ __forceinline__ void derived_quad(const typename Storage<T>::acc* src, int sp,
                                             const typename Storage<T>::acc* ws, const int* span, int kH, int kW,
                                             int lr, int q0, bool exact, typename Storage<T>::acc (&best)[kTileQuad],
                                             int (&tap)[kTileQuad]) {
    using A = typename Storage<T>::acc;
    const A neutral = Op<OP>::template neutral<A>();
    bool tie[kTileQuad];
#pragma unroll
    for (int k = 0; k < kTileQuad; ++k) {
        best[k] = neutral;
        tap[k] = -1;
        tie[k] = false;
    }
    for (int di = 0; di < kH; ++di) {
        const int lo = span[2 * di], hi = span[2 * di + 1];
        if (hi < lo) continue;
        const A* row = src + (lr + di) * sp + q0 + lo;
        const A* wrow = ws + di * kW;
        A s0 = row[0], s1 = row[1], s2 = row[2];
        for (int dj = lo; dj <= hi; ++dj) {
            const A s3 = row[dj - lo + 3];
            const A wv = wrow[dj];
            const A v[kTileQuad] = {Op<OP>::tap(s0, wv), Op<OP>::tap(s1, wv), Op<OP>::tap(s2, wv), Op<OP>::tap(s3, wv)};
#pragma unroll
            for (int k = 0; k < kTileQuad; ++k) {
                if (!exact) tie[k] |= v[k] == best[k];
                if (Op<OP>::better(v[k], best[k])) {
                    best[k] = v[k];
                    tap[k] = di * kW + dj;
                }
            }
            s0 = s1;
            s1 = s2;
            s2 = s3;
        }
    }
#pragma unroll
    for (int k = 0; k < kTileQuad; ++k) {
        if (!exact && tie[k] && best[k] != neutral) {
            auto sample = [&](int di, int dj, A& s_) {
                s_ = src[(lr + di) * sp + q0 + k + dj];
                return true;
            };
            auto weight = [&](int di, int dj) { return ws[di * kW + dj]; };
            A b_;
            window_winner<T, OP, true>(sample, weight, kH, kW, b_, tap[k]);
        }
    }
}

template <typename T, typename I, int MODE>
__global__ void __launch_bounds__(256) derived_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          T* __restrict__ y, I* __restrict__ win_a,
                                                          I* __restrict__ win_b, uint32_t* __restrict__ map_a,
                                                          uint32_t* __restrict__ map_b, int C, int H, int W, int kH,
                                                          int kW, int kcs, int border, int tiles_x, int tiles_y) {
    using A = typename Storage<T>::acc;
    constexpr bool TWO = derived_two_stage(MODE);
    // gradient: a = dilation, b = erosion; two stages: a = the first operation, b = the second
    constexpr int OPA = TWO ? derived_first_op(MODE) : kDilate;
    constexpr int OPB = OPA == kErode ? kDilate : kErode;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const DerivedGeom geo(kH, kW, TWO);
    A* const xs = reinterpret_cast<A*>(smem_raw);
    A* const zs = xs + geo.xs_elems;
    A* const ws = zs + geo.zs_elems;
    int* const span = reinterpret_cast<int*>(ws + kH * kW);
    __shared__ int exact_flag;

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int c = static_cast<int>(tc.plane % C);
    const int oh0 = tc.ty * kTile, ow0 = tc.tx * kTile;
    const int aH = kH / 2, aW = kW / 2;
    const T* xp = x + tc.plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int tid = threadIdx.y * kTile + threadIdx.x;
    const A pad = __int_as_float(0x7fffffff);  // never wins
    const A never = -std::numeric_limits<A>::infinity();
    const long long pbase = tc.plane * H * W;
    const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;

    uint32_t* const mbits = reinterpret_cast<uint32_t*>(smem_raw + geo.marks_offset(kH, kW, sizeof(A)));
    const int mrows = kTile + kH - 1, mwords = mark_words(kTile, kW);
    const TileMarks marks_a{mbits, oh0 - aH, floor_div32(ow0 - aW), mrows, mwords};
    const TileMarks marks_b{mbits + mrows * mwords, oh0 - aH, floor_div32(ow0 - aW), mrows, mwords};
    marks_a.clear(tid, 256);
    marks_b.clear(tid, 256);
    if (tid == 0) exact_flag = 1;
    __syncthreads();
    for (int i = tid; i < kH * kW; i += 256) {
        const A v = Storage<T>::load(wc[i]);
        ws[i] = v;
        if (NeedsExactCheck<T>::value && !weight_is_exact(static_cast<float>(v))) exact_flag = 0;
    }
    // x from (oh0 - s * aH, ow0 - s * aW), border resolved (CONSTANT pads as NaN)
    const int xr0 = oh0 - (TWO ? 2 : 1) * aH, xc0 = ow0 - (TWO ? 2 : 1) * aW;
    for (int i = tid; i < geo.sx * geo.px; i += 256) {
        const int r = i / geo.px, q = i - r * geo.px;
        int gr = xr0 + r, gq = xc0 + q;
        A v = pad;
        if (resolve(gr, H, border) && resolve(gq, W, border)) v = Storage<T>::load(xp[static_cast<long long>(gr) * W + gq]);
        xs[i] = v;
    }
    for (int di = tid; di < kH; di += 256) {
        int lo = kW, hi = -1;
        for (int dj = 0; dj < kW; ++dj)
            if (!(ws[di * kW + dj] == never)) {
                lo = min(lo, dj);
                hi = dj;
            }
        span[2 * di] = lo;
        span[2 * di + 1] = hi;
    }
    __syncthreads();
    const bool exact = !NeedsExactCheck<T>::value || exact_flag;
    auto round_t = [](A v) { return Storage<T>::load(Storage<T>::store(v)); };

    if constexpr (!TWO) {
        // the gradient: both operations over the same samples, four adjacent outputs per thread
        const int lr = tid >> 3, q0 = (tid & 7) * kTileQuad;
        const int oh = oh0 + lr;
        if (oh < H && ow0 + q0 < W) {
            A bd[kTileQuad], be[kTileQuad];
            int td[kTileQuad], te[kTileQuad];
            derived_quad<T, kDilate>(xs, geo.px, ws, span, kH, kW, lr, q0, exact, bd, td);
            derived_quad<T, kErode>(xs, geo.px, ws, span, kH, kW, lr, q0, exact, be, te);
            int last_a = -1, last_b = -1;
#pragma unroll
            for (int k = 0; k < kTileQuad; ++k) {
                const int ow = ow0 + q0 + k;
                if (ow >= W) break;
                const long long o = pbase + static_cast<long long>(oh) * W + ow;
                y[o] = Storage<T>::store(round_t(bd[k]) - round_t(be[k]));
                win_a[o] = encode_direct<I>(td[k]);
                win_b[o] = encode_direct<I>(te[k]);
                if (td[k] >= 0) marks_a.mark(map_a, tc.plane, H, W, kW, kw_magic, aH, aW, border, oh, ow, td[k], last_a);
                if (te[k] >= 0) marks_b.mark(map_b, tc.plane, H, W, kW, kw_magic, aH, aW, border, oh, ow, te[k], last_b);
            }
        }
    } else {
        // stage one: z over the tile grown by the halo, rows [oh0 - aH, oh0 - aH + rz), columns [ow0 - aW, ...)
        const int nq = (geo.cz + kTileQuad - 1) / kTileQuad;
        for (int qi = tid; qi < geo.rz * nq; qi += 256) {
            const int lr = qi / nq, q0 = (qi - lr * nq) * kTileQuad;
            const int zr = oh0 - aH + lr;
            if (zr < 0 || zr >= H) continue;
            A bz[kTileQuad];
            int tz[kTileQuad];
            derived_quad<T, OPA>(xs, geo.px, ws, span, kH, kW, lr, q0, exact, bz, tz);
            int last = -1;
#pragma unroll
            for (int k = 0; k < kTileQuad; ++k) {
                const int q = q0 + k, zc = ow0 - aW + q;
                if (q >= geo.cz || zc < 0 || zc >= W) continue;
                zs[lr * geo.pz + q] = round_t(bz[k]);
                // the intermediate pixels this tile owns carry the first stage's records
                if (lr >= aH && lr < aH + kTile && q >= aW && q < aW + kTile) {
                    win_a[pbase + static_cast<long long>(zr) * W + zc] = encode_direct<I>(tz[k]);
                    if (tz[k] >= 0) marks_a.mark(map_a, tc.plane, H, W, kW, kw_magic, aH, aW, border, zr, zc, tz[k], last);
                }
            }
        }
        __syncthreads();
        // z's positions outside the image: CONSTANT pads, or the z of the folded pixel (when it lies in the
        // grown tile; others are read by no output inside the image)
        for (int i = tid; i < geo.rz * geo.cz; i += 256) {
            const int r = i / geo.cz, q = i - r * geo.cz;
            int zr = oh0 - aH + r, zc = ow0 - aW + q;
            if (zr >= 0 && zr < H && zc >= 0 && zc < W) continue;
            A v = pad;
            if (resolve(zr, H, border) && resolve(zc, W, border)) {
                const int fr = zr - (oh0 - aH), fq = zc - (ow0 - aW);
                const bool inside = fr >= 0 && fr < geo.rz && fq >= 0 && fq < geo.cz &&
                                    !(fr == r && fq == q);
                if (inside) v = zs[fr * geo.pz + fq];
            }
            zs[r * geo.pz + q] = v;
        }
        __syncthreads();
        // stage two over z: the tile's outputs, with the top-hat / black-hat epilogue
        const int lr = tid >> 3, q0 = (tid & 7) * kTileQuad;
        const int oh = oh0 + lr;
        if (oh < H && ow0 + q0 < W) {
            A bo[kTileQuad];
            int to[kTileQuad];
            derived_quad<T, OPB>(zs, geo.pz, ws, span, kH, kW, lr, q0, exact, bo, to);
            int last = -1;
#pragma unroll
            for (int k = 0; k < kTileQuad; ++k) {
                const int ow = ow0 + q0 + k;
                if (ow >= W) break;
                const long long o = pbase + static_cast<long long>(oh) * W + ow;
                const A v = round_t(bo[k]);
                const A xv = xs[(lr + 2 * aH) * geo.px + q0 + k + 2 * aW];  // x at the output (inside the image)
                A out = v;
                if (MODE == kDerivedTopHat) out = xv - v;
                if (MODE == kDerivedBlackHat) out = v - xv;
                y[o] = Storage<T>::store(out);
                win_b[o] = encode_direct<I>(to[k]);
                if (to[k] >= 0) marks_b.mark(map_b, tc.plane, H, W, kW, kw_magic, aH, aW, border, oh, ow, to[k], last);
            }
        }
    }
    __syncthreads();
    marks_a.flush(map_a, tc.plane, H, W, tid, 256);
    marks_b.flush(map_b, tc.plane, H, W, tid, 256);
}

}  // namespace serron
