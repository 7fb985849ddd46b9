// Direct (2-D window) kernels: element-wise and shared-memory tiled forward, optionally recording
// the winning tap, and the atomic-free gather that forms grad_input.
//
// Reference behaviour followed: forward csrc/gpu/morphology/forward_kernels.cu:43-178 and
// csrc/cpu/morphology/operators.cpp:38-80; winner selection csrc/cpu/morphology/backward.cpp:46-99;
// grad_input accumulation order and precision csrc/cpu/morphology/backward.cpp:250-263 (serial
// scatter in output raster order, in the storage type's arithmetic).  The gather visits, for each
// input pixel, the outputs that can select it in ascending raster order, so every sum is formed in
// exactly the order and precision the reference CPU forms it, with no atomics.
#pragma once

#include <limits>

#include "common.cuh"

namespace serron {

constexpr int kTile = 32;        // tiled forward / gather: 32x32 outputs (pixels) per CTA
constexpr int kTileThreadsY = 8; // 32 x 8 threads, 4 rows per thread
constexpr int kRowsPerThread = kTile / kTileThreadsY;

// Decodes a 1-D grid index into (plane, tile row, tile column).
struct TileCoord {
    long long plane;
    int ty, tx;
};
__device__ __forceinline__ TileCoord tile_coord(int tiles_x, int tiles_y) {
    const long long b = blockIdx.x;
    TileCoord t;
    t.tx = static_cast<int>(b % tiles_x);
    t.ty = static_cast<int>((b / tiles_x) % tiles_y);
    t.plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    return t;
}

// ------------------------------------------------------------------------------------------------
// winner search over one window
//
// `sample(di, dj, v)` stores the (border-resolved) sample and returns false when the tap lies outside
// a CONSTANT border.  Returns the extreme value and the first strictly-improving tap, or tap = -1.
// ------------------------------------------------------------------------------------------------
template <typename T, int OP, bool EXACT, typename Sample, typename Weight>
__device__ __forceinline__ void window_winner(const Sample& sample, const Weight& weight, int kH, int kW,
                                              typename Storage<T>::acc& best_out, int& tap_out) {
    using A = typename Storage<T>::acc;
    const A neutral = Op<OP>::template neutral<A>();
    A best = neutral;
    int tap = -1;
    bool tie = false;
    for (int di = 0; di < kH; ++di) {
        for (int dj = 0; dj < kW; ++dj) {
            A s;
            if (!sample(di, dj, s)) continue;  // CONSTANT outside: neutral, never wins
            const A v = Op<OP>::tap(s, weight(di, dj));
            if (EXACT) tie |= (v == best);
            if (Op<OP>::better(v, best)) {
                best = v;
                tap = di * kW + dj;
            }
        }
    }
    if (EXACT && tie && best != neutral) {
        // a float tie with the running best: settle it the way the reference CPU does, in double
        double bd = Op<OP>::template neutral<double>();
        tap = -1;
        for (int di = 0; di < kH; ++di) {
            for (int dj = 0; dj < kW; ++dj) {
                A s;
                if (!sample(di, dj, s)) continue;
                const double v = Op<OP>::tap(static_cast<double>(s), static_cast<double>(weight(di, dj)));
                if (Op<OP>::better(v, bd)) {
                    bd = v;
                    tap = di * kW + dj;
                }
            }
        }
    }
    best_out = best;
    tap_out = tap;
}

template <typename I>
__device__ __forceinline__ I encode_direct(int tap) {
    return tap < 0 ? static_cast<I>(IndexTraits<I>::none) : static_cast<I>(tap);
}

// ------------------------------------------------------------------------------------------------
// element-wise forward (algo = element): one thread per output, samples read from global memory
// ------------------------------------------------------------------------------------------------
template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX>
__global__ void __launch_bounds__(256) element_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          T* __restrict__ y, I* __restrict__ win, long long total,
                                                          int C, int H, int W, int kH, int kW, int kcs,
                                                          int border) {
    using A = typename Storage<T>::acc;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int ow = static_cast<int>(idx % W);
    const int oh = static_cast<int>((idx / W) % H);
    const long long plane = idx / (static_cast<long long>(W) * H);
    const int c = static_cast<int>(plane % C);
    const T* xp = x + plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int aH = kH / 2, aW = kW / 2;
    auto sample = [&](int di, int dj, A& s) {
        int r = oh + di - aH, q = ow + dj - aW;
        if (!resolve(r, H, border) || !resolve(q, W, border)) return false;
        s = Storage<T>::load(xp[static_cast<long long>(r) * W + q]);
        return true;
    };
    auto weight = [&](int di, int dj) { return Storage<T>::load(wc[di * kW + dj]); };
    A best;
    int tap;
    // float inputs always track ties here; a tied window is settled in double, which is exact for any
    // weights (for 0/inf weights the redo merely repeats the float answer)
    window_winner<T, OP, NeedsExactCheck<T>::value>(sample, weight, kH, kW, best, tap);
    if (WITH_VALUE) y[idx] = Storage<T>::store(best);
    if (WITH_INDEX) win[idx] = encode_direct<I>(tap);
}

// ------------------------------------------------------------------------------------------------
// tiled forward (algo = tiled): a 32x32 output tile, its halo staged once in shared memory with the
// border resolved at staging (CONSTANT cells hold the neutral element, which never wins).
//
// A thread computes four adjacent outputs of one row: for each SE row it walks the columns with a
// sliding window of four samples in registers, so one shared-memory load and one (broadcast) weight
// load serve four taps.  An SE row is walked only over its span of finite weights: a -inf weight never
// wins (x + -inf for dilation, x - -inf for erosion), which skips most of a mask SE's corners.
// ------------------------------------------------------------------------------------------------
// Target-map marking inside a tiled forward (`map` non-null, with records): the winners of a tile's
// outputs lie in its halo, so a CTA sets them in a shared bitmap of the halo's rows, in whole target-map
// words, and ORs the non-zero words into the map at the end (a winner folded from beyond the halo goes
// straight to the map).
__host__ __device__ inline int mark_words(int tile_cols, int kW) { return (tile_cols + kW - 2) / 32 + 2; }
__host__ __device__ inline size_t mark_bytes(int tile_rows, int tile_cols, int kH, int kW) {
    return static_cast<size_t>(tile_rows + kH - 1) * mark_words(tile_cols, kW) * sizeof(uint32_t);
}
__device__ __forceinline__ int floor_div32(int v) { return v >= 0 ? v / 32 : -((31 - v) / 32); }

struct TileMarks {
    uint32_t* bits;
    int rbase, wbase, rows, words;
    __device__ void clear(int tid, int nthr) const {
        for (int i = tid; i < rows * words; i += nthr) bits[i] = 0u;
    }
    // winner of output (oh, ow) through direct tap t (>= 0); `last` holds the previous output's winner
    // (plane-relative pixel, -1 for none), and an output with the same winner sets nothing
    __device__ void mark(uint32_t* map, long long plane, int H, int W, int kW, uint32_t kw_magic, int aH, int aW,
                         int border, int oh, int ow, int t, int& last) const {
        const uint32_t ut = static_cast<uint32_t>(t);
        const int di = kW == 1 ? t
                               : static_cast<int>(ut <= 0xffffu ? __umulhi(ut, kw_magic) : ut / static_cast<uint32_t>(kW));
        int x = oh + di - aH, y = ow + (t - di * kW) - aW;
        if (!resolve(x, H, border) || !resolve(y, W, border)) return;
        const int key = x * W + y;  // < H * W < 2^31
        if (key == last) return;
        last = key;
        const int ri = x - rbase, wi = (y >> 5) - wbase;
        if (ri >= 0 && ri < rows && wi >= 0 && wi < words)
            atomicOr(&bits[ri * words + wi], 1u << (y & 31));
        else
            atomicOr(&map[(plane * H + x) * ((W + 31) / 32) + (y >> 5)], 1u << (y & 31));
    }
    __device__ void flush(uint32_t* map, long long plane, int H, int W, int tid, int nthr) const {
        const int WW = (W + 31) / 32;
        for (int i = tid; i < rows * words; i += nthr) {
            const uint32_t v = bits[i];
            if (v) {
                const int ri = i / words;
                atomicOr(&map[(plane * H + rbase + ri) * WW + wbase + (i - ri * words)], v);
            }
        }
    }
};

constexpr int kTileQuad = 4;  // adjacent outputs per thread

// staged row pitch: odd, so that the 4 rows x 8 column groups of a warp hit distinct banks
__host__ __device__ inline int tiled_pitch(int kW) { return (kTile + kW - 1) | 1; }
__host__ __device__ inline size_t tiled_smem(int kH, int kW, size_t acc) {
    return (static_cast<size_t>(kTile + kH - 1) * tiled_pitch(kW) + static_cast<size_t>(kH) * kW) * acc +
           static_cast<size_t>(kH) * 2 * sizeof(int);
}

template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX>
__global__ void __launch_bounds__(256) tiled_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                        T* __restrict__ y, I* __restrict__ win, int C, int H, int W,
                                                        int kH, int kW, int kcs, int border, int tiles_x,
                                                        int tiles_y, uint32_t* __restrict__ map) {
    using A = typename Storage<T>::acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int sw = tiled_pitch(kW), sh = kTile + kH - 1;
    A* xs = reinterpret_cast<A*>(smem_raw);
    A* ws = xs + sw * sh;
    int* span = reinterpret_cast<int*>(ws + kH * kW);  // [kH][2]: first and last finite column of an SE row
    __shared__ int exact_flag;

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int c = static_cast<int>(tc.plane % C);
    const int oh0 = tc.ty * kTile, ow0 = tc.tx * kTile;
    const int aH = kH / 2, aW = kW / 2;
    const T* xp = x + tc.plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int tid = threadIdx.y * kTile + threadIdx.x;
    const A neutral = Op<OP>::template neutral<A>();
    const A never = -std::numeric_limits<A>::infinity();  // a weight that never wins

    const TileMarks marks{reinterpret_cast<uint32_t*>(smem_raw + (tiled_smem(kH, kW, sizeof(A)) + 15) / 16 * 16),
                          oh0 - aH, floor_div32(ow0 - aW), kTile + kH - 1, mark_words(kTile, kW)};
    if (map) marks.clear(tid, 256);
    if (tid == 0) exact_flag = 1;
    __syncthreads();
    for (int i = tid; i < kH * kW; i += 256) {
        const A v = Storage<T>::load(wc[i]);
        ws[i] = v;
        if (NeedsExactCheck<T>::value && !weight_is_exact(static_cast<float>(v))) exact_flag = 0;
    }
    const int cw = kTile + kW - 1;  // staged columns (the pitch may add one)
    for (int i = tid; i < sh * cw; i += 256) {
        const int r = i / cw, q = i - r * cw;
        int gr = oh0 - aH + r, gq = ow0 - aW + q;
        A v = neutral;
        if (resolve(gr, H, border) && resolve(gq, W, border)) v = Storage<T>::load(xp[static_cast<long long>(gr) * W + gq]);
        xs[r * sw + q] = v;
    }
    __syncthreads();
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

    const int lr = tid >> 3, q0 = (tid & 7) * kTileQuad;  // output row, first of four columns
    const int oh = oh0 + lr;
    const bool active = !(oh >= H || ow0 + q0 >= W);
    if (active) {
        const bool exact = !NeedsExactCheck<T>::value || exact_flag;
        A best[kTileQuad];
        int tap[kTileQuad];
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
            const A* row = xs + (lr + di) * sw + q0 + lo;
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
        int last_winner = -1;  // marking: the previous output's winner pixel
        const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;
#pragma unroll
        for (int k = 0; k < kTileQuad; ++k) {
            const int ow = ow0 + q0 + k;
            if (ow >= W) break;
            if (!exact && tie[k] && best[k] != neutral) {
                // a float tie with the running best: settle it the way the reference CPU does, in double
                auto sample = [&](int di, int dj, A& s_) {
                    s_ = xs[(lr + di) * sw + q0 + k + dj];
                    return true;
                };
                auto weight = [&](int di, int dj) { return ws[di * kW + dj]; };
                A b_;
                window_winner<T, OP, true>(sample, weight, kH, kW, b_, tap[k]);
            }
            const long long o = tc.plane * H * W + static_cast<long long>(oh) * W + ow;
            if (WITH_VALUE) y[o] = Storage<T>::store(best[k]);
            if (WITH_INDEX) win[o] = encode_direct<I>(tap[k]);
            if (WITH_INDEX && map && tap[k] >= 0)
                marks.mark(map, tc.plane, H, W, kW, kw_magic, aH, aW, border, oh, ow, tap[k], last_winner);
        }
    }
    if (map) {
        __syncthreads();
        marks.flush(map, tc.plane, H, W, tid, 256);
    }
}

// ------------------------------------------------------------------------------------------------
// wide tiled forward (algo = tiled, windows 9 or more columns wide, 5 or more for 16-bit storage):
// a 32x64 output tile, eight
// adjacent outputs per thread.  An SE row whose span holds one weight of zero (every row of a flat
// disk, diamond or square) needs no per-tap weight: the eight windows over that row share the core
// [c0 + lo + 7, c0 + hi], so the thread takes the core's first extremum once, suffix extrema of the
// seven columns left of it and prefix extrema of the seven right of it, and combines three
// candidates per output in column order (ties keep the leftmost): span + 27 compare-selects for
// eight outputs instead of 8 x span.  Other rows are walked like tiled_fwd_kernel, eight samples in
// registers.  NaN samples are staged as the neutral element (neither wins).
// ------------------------------------------------------------------------------------------------
constexpr int kWideRows = 32, kWideCols = 64, kWideQ = 8;

__host__ __device__ inline int wide_pitch(int kW) { return (kWideCols + kW - 1) | 1; }
__host__ __device__ inline size_t wide_smem(int kH, int kW, size_t acc) {
    return (static_cast<size_t>(kWideRows + kH - 1) * wide_pitch(kW) + static_cast<size_t>(kH) * kW) * acc +
           static_cast<size_t>(kH) * 3 * sizeof(int);
}

// Keyed samples (16-bit storage, every non-empty SE row one run of one zero weight).  A staged sample
// becomes a 32-bit key that orders like the candidates of the first-extremum rule: the value's 16 bits in
// an order where better is smaller (-0 taken as +0, so the two compare equal as they do as floats), then
// the staged row and column.  For any one output the staged row and column grow with the SE row and
// column of the tap, so among equal values the first tap in raster order has the smallest key, and the
// window's winner is the unsigned minimum of its keys.  The lowest bit keeps a -0's sign for the output,
// below the position, where it never decides.  Neutral and NaN samples (never winners) are all ones, the
// minimum's starting value; no other key has all of its low 16 bits set.
//   bits 31..16 ordered value, 15..9 staged row (< 128), 8..2 staged column (< 128), 0 negative zero
constexpr uint32_t kKeyNone = 0xffffffffu;
constexpr int kKeyMaxRows = 128, kKeyMaxCols = 128;

template <typename T>
struct Bits16;
template <>
struct Bits16<__half> {
    static constexpr uint32_t inf = 0x7c00u;
    static __device__ __forceinline__ uint32_t of(__half v) { return __half_as_ushort(v); }
    static __device__ __forceinline__ float value(uint32_t b) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
    }
};
template <>
struct Bits16<__nv_bfloat16> {
    static constexpr uint32_t inf = 0x7f80u;
    static __device__ __forceinline__ uint32_t of(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
    static __device__ __forceinline__ float value(uint32_t b) {
        return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(b)));
    }
};

// b: a sample's 16-bit pattern at staged row r, column q
template <typename T, int OP>
__device__ __forceinline__ uint32_t sample_key(uint32_t b, int r, int q) {
    constexpr uint32_t inf = Bits16<T>::inf, neutral = OP == kErode ? inf : (inf | 0x8000u);
    if ((b & 0x7fffu) > inf || b == neutral) return kKeyNone;
    const uint32_t negzero = b == 0x8000u ? 1u : 0u;
    if (negzero) b = 0u;
    uint32_t ord = (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);  // ascending with the value
    if (OP == kDilate) ord = ~ord & 0xffffu;                         // better = larger: descending
    return (ord << 16) | (static_cast<uint32_t>(r) << 9) | (static_cast<uint32_t>(q) << 2) | negzero;
}
// the 16-bit pattern of the sample a key holds
template <int OP>
__device__ __forceinline__ uint32_t key_bits16(uint32_t key) {
    if (key & 1u) return 0x8000u;
    uint32_t ord = key >> 16;
    if (OP == kDilate) ord = ~ord & 0xffffu;
    return (ord & 0x8000u) ? (ord & 0x7fffu) : (~ord & 0xffffu);
}
template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX>
__global__ void __launch_bounds__(256) wide_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                       T* __restrict__ y, I* __restrict__ win, int C, int H, int W,
                                                       int kH, int kW, int kcs, int border, int tiles_x,
                                                       int tiles_y, uint32_t* __restrict__ map) {
    using A = typename Storage<T>::acc;
    constexpr int Q = kWideQ;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int sw = wide_pitch(kW), sh = kWideRows + kH - 1;
    A* xs = reinterpret_cast<A*>(smem_raw);
    A* ws = xs + sw * sh;
    int* info = reinterpret_cast<int*>(ws + kH * kW);  // [kH][3]: first and last finite column, one weight
    __shared__ int exact_flag;

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int c = static_cast<int>(tc.plane % C);
    const int oh0 = tc.ty * kWideRows, ow0 = tc.tx * kWideCols;
    const int aH = kH / 2, aW = kW / 2;
    const T* xp = x + tc.plane * H * W;
    const T* wc = w + static_cast<long long>(c) * kcs;
    const int tid = threadIdx.x;
    const A neutral = Op<OP>::template neutral<A>();
    const A never = -std::numeric_limits<A>::infinity();

    const TileMarks marks{reinterpret_cast<uint32_t*>(smem_raw + (wide_smem(kH, kW, sizeof(A)) + 15) / 16 * 16),
                          oh0 - aH, floor_div32(ow0 - aW), kWideRows + kH - 1, mark_words(kWideCols, kW)};
    if (map) marks.clear(tid, 256);
    if (tid == 0) exact_flag = 1;
    __syncthreads();
    for (int i = tid; i < kH * kW; i += 256) {
        const A v = Storage<T>::load(wc[i]);
        ws[i] = v;
        if (NeedsExactCheck<T>::value && !weight_is_exact(static_cast<float>(v))) exact_flag = 0;
    }
    const int cw = kWideCols + kW - 1;
    __syncthreads();
    for (int di = tid; di < kH; di += 256) {
        int lo = kW, hi = -1;
        for (int dj = 0; dj < kW; ++dj)
            if (!(ws[di * kW + dj] == never)) {
                lo = min(lo, dj);
                hi = dj;
            }
        // one weight over the whole span, of value zero (bit-identical, so the row's taps add the same)
        bool one = hi >= lo && ws[di * kW + lo] == A(0);
        for (int dj = lo; one && dj <= hi; ++dj)
            one = ws[di * kW + dj] == A(0) && signbit(ws[di * kW + dj]) == signbit(ws[di * kW + lo]);
        info[3 * di] = lo;
        info[3 * di + 1] = hi;
        info[3 * di + 2] = one ? 1 : 0;
    }
    bool keyed = false;
    if constexpr (sizeof(T) == 2) {
        bool rows_ok = true;
        for (int di = tid; di < kH; di += 256)  // rows this thread classified above
            rows_ok &= info[3 * di + 1] < info[3 * di] || info[3 * di + 2] != 0;
        keyed = __syncthreads_and(rows_ok && sh <= kKeyMaxRows && cw <= kKeyMaxCols);
    } else {
        __syncthreads();
    }
    if (keyed) {
        if constexpr (sizeof(T) == 2) {
            uint32_t* ks = reinterpret_cast<uint32_t*>(xs);
            for (int i = tid; i < sh * cw; i += 256) {
                const int r = i / cw, q = i - r * cw;
                int gr = oh0 - aH + r, gq = ow0 - aW + q;
                uint32_t key = kKeyNone;
                if (resolve(gr, H, border) && resolve(gq, W, border))
                    key = sample_key<T, OP>(Bits16<T>::of(xp[static_cast<long long>(gr) * W + gq]), r, q);
                ks[r * sw + q] = key;
            }
        }
    } else {
        for (int i = tid; i < sh * cw; i += 256) {
            const int r = i / cw, q = i - r * cw;
            int gr = oh0 - aH + r, gq = ow0 - aW + q;
            A v = neutral;
            if (resolve(gr, H, border) && resolve(gq, W, border))
                v = Storage<T>::load(xp[static_cast<long long>(gr) * W + gq]);
            xs[r * sw + q] = v != v ? neutral : v;
        }
    }
    __syncthreads();

    // output row and first of eight columns: a warp takes 8 rows x 4 column groups, so with the odd pitch
    // its 32 loads of a sample position hit 32 distinct banks
    const int lane = tid & 31, wq = tid >> 5;
    const int lr = 8 * (wq & 3) + (lane & 7), c0 = (4 * (wq >> 2) + (lane >> 3)) * Q;
    const int oh = oh0 + lr;
    const bool active = !(oh >= H || ow0 + c0 >= W);
    if (keyed) {
        const uint32_t* ks = reinterpret_cast<const uint32_t*>(xs);
        if (active) {
            uint32_t best[Q];
#pragma unroll
            for (int k = 0; k < Q; ++k) best[k] = kKeyNone;
            for (int di = 0; di < kH; ++di) {
                const int lo = info[3 * di], hi = info[3 * di + 1];
                if (hi < lo) continue;
                const uint32_t* row = ks + (lr + di) * sw + c0;  // output k's window starts at row[k]
                if (hi - lo + 1 >= Q) {
                    // output k: suffix row[lo + k .. lo + Q - 2], core row[lo + Q - 1 .. hi], prefix
                    // row[hi + 1 .. hi + k]
                    uint32_t sk[Q - 1];
                    sk[Q - 2] = row[lo + Q - 2];
#pragma unroll
                    for (int k = Q - 3; k >= 0; --k) sk[k] = min(row[lo + k], sk[k + 1]);
                    uint32_t ck = row[lo + Q - 1];
                    int j = lo + Q;
                    for (; j < hi; j += 2) ck = __vimin3_u32(ck, row[j], row[j + 1]);
                    if (j == hi) ck = min(ck, row[j]);
                    best[0] = __vimin3_u32(best[0], sk[0], ck);
#pragma unroll
                    for (int k = 1; k < Q; ++k) {
                        ck = min(ck, row[hi + k]);  // the core and the prefix of output k
                        best[k] = k < Q - 1 ? __vimin3_u32(best[k], sk[k], ck) : min(best[k], ck);
                    }
                } else {
                    uint32_t s8[Q];
#pragma unroll
                    for (int k = 0; k < Q - 1; ++k) s8[k] = row[lo + k];
                    for (int dj = lo; dj <= hi; ++dj) {
                        s8[Q - 1] = row[dj + Q - 1];
#pragma unroll
                        for (int k = 0; k < Q; ++k) best[k] = min(best[k], s8[k]);
#pragma unroll
                        for (int k = 0; k < Q - 1; ++k) s8[k] = s8[k + 1];
                    }
                }
            }
            int last_winner = -1;
            const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;
#pragma unroll
            for (int k = 0; k < Q; ++k) {
                const int ow = ow0 + c0 + k;
                if (ow >= W) break;
                A val = neutral;
                int t = -1;
                if (best[k] != kKeyNone) {
                    const int di = static_cast<int>((best[k] >> 9) & 127u) - lr;
                    const int dj = static_cast<int>((best[k] >> 2) & 127u) - (c0 + k);
                    t = di * kW + dj;
                    if constexpr (sizeof(T) == 2)
                        val = Op<OP>::tap(Bits16<T>::value(key_bits16<OP>(best[k])), ws[di * kW + info[3 * di]]);
                }
                const long long o = tc.plane * H * W + static_cast<long long>(oh) * W + ow;
                if (WITH_VALUE) y[o] = Storage<T>::store(val);
                if (WITH_INDEX) win[o] = encode_direct<I>(t);
                if (WITH_INDEX && map && t >= 0)
                    marks.mark(map, tc.plane, H, W, kW, kw_magic, aH, aW, border, oh, ow, t, last_winner);
            }
        }
        if (map) {
            __syncthreads();
            marks.flush(map, tc.plane, H, W, tid, 256);
        }
        return;
    }
    if (active) {
        const bool exact = !NeedsExactCheck<T>::value || exact_flag;
        A best[Q];
        int tap[Q];
        bool tie[Q];
#pragma unroll
        for (int k = 0; k < Q; ++k) {
            best[k] = neutral;
            tap[k] = -1;
            tie[k] = false;
        }
        for (int di = 0; di < kH; ++di) {
            const int lo = info[3 * di], hi = info[3 * di + 1];
            if (hi < lo) continue;
            const A* row = xs + (lr + di) * sw + c0;  // output k's window starts at row[k]
            const A* wrow = ws + di * kW;
            if (info[3 * di + 2] && hi - lo + 1 >= Q) {
                // suffix extrema of row[lo .. lo + Q - 2] (ties: the left one)
                A sv[Q - 1];
                int sc[Q - 1];
                sv[Q - 2] = row[lo + Q - 2];
                sc[Q - 2] = lo + Q - 2;
#pragma unroll
                for (int k = Q - 3; k >= 0; --k) {
                    const A v = row[lo + k];
                    const bool take = !Op<OP>::better(sv[k + 1], v);
                    sv[k] = take ? v : sv[k + 1];
                    sc[k] = take ? lo + k : sc[k + 1];
                }
                // core row[lo + Q - 1 .. hi], first extremum
                A cv = row[lo + Q - 1];
                int cc = lo + Q - 1;
                for (int j = lo + Q; j <= hi; ++j) {
                    const A v = row[j];
                    if (Op<OP>::better(v, cv)) {
                        cv = v;
                        cc = j;
                    }
                }
                const A wz = wrow[lo];
                A pv = neutral;
                int pc = 0;
#pragma unroll
                for (int k = 0; k < Q; ++k) {
                    // window of output k: row[lo + k .. lo + Q - 2], the core, row[hi + 1 .. hi + k]
                    A rv = cv;
                    int rc = cc;
                    if (k < Q - 1 && !Op<OP>::better(cv, sv[k])) {
                        rv = sv[k];
                        rc = sc[k];
                    }
                    if (k > 0) {
                        const A v = row[hi + k];
                        if (k == 1 || Op<OP>::better(v, pv)) {
                            pv = v;
                            pc = hi + k;
                        }
                        if (Op<OP>::better(pv, rv)) {
                            rv = pv;
                            rc = pc;
                        }
                    }
                    const A t = Op<OP>::tap(rv, wz);
                    if (!exact) tie[k] |= t == best[k];
                    if (Op<OP>::better(t, best[k])) {
                        best[k] = t;
                        tap[k] = di * kW + rc - k;
                    }
                }
            } else {
                A s[Q];
#pragma unroll
                for (int k = 0; k < Q - 1; ++k) s[k] = row[lo + k];
                for (int dj = lo; dj <= hi; ++dj) {
                    s[Q - 1] = row[dj + Q - 1];
                    const A wv = wrow[dj];
#pragma unroll
                    for (int k = 0; k < Q; ++k) {
                        const A v = Op<OP>::tap(s[k], wv);
                        if (!exact) tie[k] |= v == best[k];
                        if (Op<OP>::better(v, best[k])) {
                            best[k] = v;
                            tap[k] = di * kW + dj;
                        }
                    }
#pragma unroll
                    for (int k = 0; k < Q - 1; ++k) s[k] = s[k + 1];
                }
            }
        }
        int last_winner = -1;  // marking: the previous output's winner pixel
        const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;
#pragma unroll
        for (int k = 0; k < Q; ++k) {
            const int ow = ow0 + c0 + k;
            if (ow >= W) break;
            if (!exact && tie[k] && best[k] != neutral) {
                // a float tie with the running best: settle it the way the reference CPU does, in double
                auto sample = [&](int di, int dj, A& s_) {
                    s_ = xs[(lr + di) * sw + c0 + k + dj];
                    return true;
                };
                auto weight = [&](int di, int dj) { return ws[di * kW + dj]; };
                A b_;
                window_winner<T, OP, true>(sample, weight, kH, kW, b_, tap[k]);
            }
            const long long o = tc.plane * H * W + static_cast<long long>(oh) * W + ow;
            if (WITH_VALUE) y[o] = Storage<T>::store(best[k]);
            if (WITH_INDEX) win[o] = encode_direct<I>(tap[k]);
            if (WITH_INDEX && map && tap[k] >= 0)
                marks.mark(map, tc.plane, H, W, kW, kw_magic, aH, aW, border, oh, ow, tap[k], last_winner);
        }
    }
    if (map) {
        __syncthreads();
        marks.flush(map, tc.plane, H, W, tid, 256);
    }
}

// ------------------------------------------------------------------------------------------------
// grad_input gather for direct winners
//
// Each CTA owns a 32x32 tile of input pixels and stages the winners and grad_output of every output
// that can reach the tile.  A pixel walks its candidate outputs in ascending raster order and adds
// grad_output wherever the output's winner resolves to it.
// ------------------------------------------------------------------------------------------------
template <typename T, typename I>
__global__ void __launch_bounds__(256) direct_gather_kernel(const T* __restrict__ go, const I* __restrict__ win,
                                                            T* __restrict__ gi, int C, int H, int W, int kH, int kW,
                                                            int border, int tiles_x, int tiles_y, int force_global) {
    using G = typename GradAcc<T>::type;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int aH = kH / 2, aW = kW / 2;
    // halo of aH rows / aW columns on every side: it holds every candidate output, including the one an
    // even window reaches through a REFLECT fold beyond its plain window (see candidate_range)
    const int rh0 = -aH, rw0 = -aW;
    const int sw = kTile + 2 * aW, sh = kTile + 2 * aH;
    const int offh = 2 * aH - (kH - 1), offw = 2 * aW - (kW - 1);  // 1 for an even window, else 0
    G* gs = reinterpret_cast<G*>(smem_raw);
    I* is = reinterpret_cast<I*>(gs + sw * sh);

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int ph0 = tc.ty * kTile, pw0 = tc.tx * kTile;
    const long long base = tc.plane * H * W;
    const int tid = threadIdx.y * kTile + threadIdx.x;
    const bool full_h = border == kReflect && (aH > H - 1 || kH - 1 - aH > H - 1);
    const bool full_w = border == kReflect && (aW > W - 1 || kW - 1 - aW > W - 1);

    if (force_global || full_h || full_w) {
        // windows wider than the image under REFLECT (any output may fold back onto any pixel), or a
        // halo too large for shared memory: walk the candidates in global memory
        for (int i = 0; i < kRowsPerThread; ++i) {
            const int ph = ph0 + threadIdx.y * kRowsPerThread + i, pw = pw0 + threadIdx.x;
            if (ph >= H || pw >= W) continue;
            int lh, hh, lw, hw;
            candidate_range(ph, H, kH, aH, border, lh, hh);
            candidate_range(pw, W, kW, aW, border, lw, hw);
            G acc = G(0);
            for (int oh = lh; oh <= hh; ++oh)
                for (int ow = lw; ow <= hw; ++ow) {
                    const long long o = base + static_cast<long long>(oh) * W + ow;
                    const uint32_t t = win[o];
                    if (t == IndexTraits<I>::none) continue;
                    int r = oh + static_cast<int>(t / kW) - aH, q = ow + static_cast<int>(t % kW) - aW;
                    if (resolve(r, H, border) && resolve(q, W, border) && r == ph && q == pw)
                        acc = GradAcc<T>::add(acc, static_cast<G>(Storage<T>::load(go[o])));
                }
            gi[base + static_cast<long long>(ph) * W + pw] = Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
        }
        return;
    }

    for (int i = tid; i < sw * sh; i += 256) {
        const int r = i / sw, q = i - r * sw;
        const int oh = ph0 + rh0 + r, ow = pw0 + rw0 + q;
        I t = static_cast<I>(IndexTraits<I>::none);
        G g = G(0);
        if (oh >= 0 && oh < H && ow >= 0 && ow < W) {
            const long long o = base + static_cast<long long>(oh) * W + ow;
            t = win[o];
            g = static_cast<G>(Storage<T>::load(go[o]));
        }
        is[i] = t;
        gs[i] = g;
    }
    __syncthreads();

    const bool deep = ph0 >= kH - 1 && ph0 + kTile - 1 <= H - kH && pw0 >= kW - 1 && pw0 + kTile - 1 <= W - kW;
    for (int i = 0; i < kRowsPerThread; ++i) {
        const int lr = threadIdx.y * kRowsPerThread + i;
        const int ph = ph0 + lr, pw = pw0 + threadIdx.x;
        if (ph >= H || pw >= W) continue;
        G acc = G(0);
        if (deep) {
            // no border mapping anywhere in reach: output (ph - aH' + a, ...) selects the pixel only
            // through the tap that points straight at it
            for (int a = 0; a < kH; ++a) {        // output row = ph - (kH - 1 - aH) + a, ascending
                const int di = kH - 1 - a;          // tap row pointing from that output to ph
                const int srow = (lr + a + offh) * sw + threadIdx.x + offw;
                for (int b = 0; b < kW; ++b) {
                    const uint32_t want = static_cast<uint32_t>(di * kW + (kW - 1 - b));
                    if (static_cast<uint32_t>(is[srow + b]) == want) acc = GradAcc<T>::add(acc, gs[srow + b]);
                }
            }
        } else {
            int lh, hh, lw, hw;
            candidate_range(ph, H, kH, aH, border, lh, hh);
            candidate_range(pw, W, kW, aW, border, lw, hw);
            for (int oh = lh; oh <= hh; ++oh) {
                const int srow = (oh - ph0 - rh0) * sw - pw0 - rw0;
                for (int ow = lw; ow <= hw; ++ow) {
                    const uint32_t t = is[srow + ow];
                    if (t == IndexTraits<I>::none) continue;
                    int r = oh + static_cast<int>(t / kW) - aH, q = ow + static_cast<int>(t % kW) - aW;
                    if (resolve(r, H, border) && resolve(q, W, border) && r == ph && q == pw)
                        acc = GradAcc<T>::add(acc, gs[srow + ow]);
                }
            }
        }
        gi[base + static_cast<long long>(ph) * W + pw] = Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
    }
}

}  // namespace serron
