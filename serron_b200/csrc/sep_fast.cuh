// Separable flat-square path with the window length K known at compile time: the hot kernels of the
// flat structuring-element workloads.  Same results as the generic kernels in separable.cuh (winners,
// records and gradients are bit-identical); only the schedule differs.
//
// Forward: a CTA stages a (TH+K-1) x (TW+K-1) halo tile once, then
//   row pass     one thread per (row, K-chunk): the K+K-1 samples of its windows in registers, a
//                suffix arg-scan over the chunk and a prefix arg-scan over the next chunk combined per
//                output (van Herk / Gil-Werman: about three compare-selects per output, any K);
//   column pass  the same over the row results, one thread per (column, K-chunk of output rows).
// TH is a multiple of K, so every column chunk is full.
//
// Gather (grad_input): output o selects pixel p iff its column winner resolves to row ph (bit in
// Rmask[o's row][ph - oh + a]) and the row winner of row ph at o's column resolves to pw (bit in
// Smask[p]).  Both masks are built once per tile with shared-memory ORs; a pixel with an empty
// Smask gets zero at once, the others walk their 2a+1 candidate rows, AND the two masks and add
// grad_output over the set bits in ascending column order: the reference's raster order.
#pragma once

#include "common.cuh"
#include "direct.cuh"

namespace serron {

constexpr int kFastTW = 64;        // output (pixel) columns per tile
constexpr int kFastThreads = 256;

template <int K>
struct FastGeom {
    static constexpr int a = K / 2;
    static constexpr int TH = K * ((32 + K - 1) / K);  // output rows per forward tile: a multiple of K
    static constexpr int R = TH + K - 1;                // staged rows
    static constexpr int Cc = kFastTW + K - 1;          // staged columns
    static constexpr int XS = Cc | 1;                   // odd row pitch: conflict-free column-wise reads
    static constexpr int RS = kFastTW + 1;              // row-result pitch
    static constexpr int NCR = (kFastTW + K - 1) / K;   // row-pass chunks per row
    static constexpr int NCC = TH / K;                  // column-pass chunks per column
    static size_t smem_bytes() { return (size_t(R) * XS + size_t(R) * RS) * 4 + size_t(R) * RS; }
    // gather
    static constexpr int GTH = 32;                       // pixel rows per gather tile
    static constexpr int GH = GTH + 2 * a;               // halo rows
    static constexpr int GW = kFastTW + 2 * a;           // halo columns
    static constexpr int NW = (GW + 31) / 32 + 1;        // mask words per halo row (+1 for funnel reads)
    static size_t gather_smem_bytes(int idx_bytes) {
        return size_t(GH) * GW * 4 + size_t(GTH) * kFastTW * 4 + size_t(GH) * (2 * a + 1) * NW * 4 +
               ((size_t(GH) * GW * idx_bytes + 15) / 16) * 16;
    }
};

// One run of K windows [m, m+K-1], m = 0..K-1, over samples v[0..2K-2]: value and first-extremum
// offset (window-relative) of each, by a suffix arg-scan over v[0..K-1] and a prefix arg-scan over
// v[K..2K-2].  Ties keep the lower offset.
template <int K, int OP, bool IDX, typename Emit>
__device__ __forceinline__ void van_herk_run(const float (&v)[2 * K - 1], Emit emit) {
    float sv[K];
    int si[K];
    sv[K - 1] = v[K - 1];
    si[K - 1] = K - 1;
#pragma unroll
    for (int m = K - 2; m >= 0; --m) {
        // the lower position m is kept unless the suffix beyond it is strictly better
        const bool take = Op<OP>::better(sv[m + 1], v[m]);
        sv[m] = take ? sv[m + 1] : v[m];
        si[m] = IDX ? (take ? si[m + 1] : m) : 0;
    }
    emit(0, sv[0], si[0]);
    float pv = 0.0f;
    int pi = 0;
#pragma unroll
    for (int m = 1; m < K; ++m) {
        const float x = v[K + m - 1];
        if (m == 1) {
            pv = x;
            pi = K;
        } else {
            const bool take = Op<OP>::better(x, pv);
            pv = take ? x : pv;
            if (IDX) pi = take ? K + m - 1 : pi;
        }
        const bool take = Op<OP>::better(pv, sv[m]);
        emit(m, take ? pv : sv[m], take ? pi - m : si[m] - m);
    }
}

template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX, int K>
__global__ void __launch_bounds__(kFastThreads) sep_fast_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                                    I* __restrict__ win, int H, int W, int border,
                                                                    int tiles_x, int tiles_y) {
    using G = FastGeom<K>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);                  // [R][XS] staged samples
    float* rv = xs + G::R * G::XS;                                    // [R][RS] row results
    uint8_t* rdj = reinterpret_cast<uint8_t*>(rv + G::R * G::RS);    // [R][RS] row winner offsets

    const long long b = blockIdx.x;
    const int tx = static_cast<int>(b % tiles_x), ty = static_cast<int>((b / tiles_x) % tiles_y);
    const long long plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    const int oh0 = ty * G::TH, ow0 = tx * kFastTW;
    const T* xp = x + plane * H * W;
    const int tid = threadIdx.x;
    const float neutral = Op<OP>::template neutral<float>();

    // ---- stage: border resolved here, NaN staged as the neutral element (it never wins) ----
    const bool interior = oh0 - G::a >= 0 && oh0 + G::R - G::a <= H && ow0 - G::a >= 0 && ow0 + G::Cc - G::a <= W;
    for (int i = tid; i < G::R * G::Cc; i += kFastThreads) {
        const int r = i / G::Cc, q = i - r * G::Cc;
        int gr = oh0 - G::a + r, gq = ow0 - G::a + q;
        float v = neutral;
        if (interior || (resolve(gr, H, border) && resolve(gq, W, border))) {
            v = Storage<T>::load(xp[static_cast<long long>(gr) * W + gq]);
            if (v != v) v = neutral;
        }
        xs[r * G::XS + q] = v;
    }
    __syncthreads();

    // ---- row pass ----
    for (int task = tid; task < G::NCR * G::R; task += kFastThreads) {
        const int c = task / G::R, r = task - c * G::R;
        const int base = c * K;
        float v[2 * K - 1];
#pragma unroll
        for (int m = 0; m < 2 * K - 1; ++m) v[m] = (base + m < G::Cc) ? xs[r * G::XS + base + m] : neutral;
        van_herk_run<K, OP, true>(v, [&](int m, float val, int off) {
            const int j = base + m;
            if (j < kFastTW) {
                rv[r * G::RS + j] = val;
                rdj[r * G::RS + j] = static_cast<uint8_t>(off);
            }
        });
    }
    __syncthreads();

    // ---- column pass ----
    for (int task = tid; task < G::NCC * kFastTW; task += kFastThreads) {
        const int c = task / kFastTW, j = task - c * kFastTW;
        const int base = c * K;
        const int ow = ow0 + j;
        float v[2 * K - 1];
#pragma unroll
        for (int m = 0; m < 2 * K - 1; ++m) v[m] = rv[(base + m) * G::RS + j];
        van_herk_run<K, OP, WITH_INDEX>(v, [&](int m, float val, int off) {
            const int i = base + m;
            const int oh = oh0 + i;
            if (oh < H && ow < W) {
                const long long o = plane * H * W + static_cast<long long>(oh) * W + ow;
                if (WITH_VALUE) y[o] = Storage<T>::store(val);
                if (WITH_INDEX) {
                    const uint32_t hi = val == neutral ? sep_none_hi<I>() : static_cast<uint32_t>(off);
                    const uint32_t lo = rdj[(i + G::a) * G::RS + j];
                    win[o] = static_cast<I>((hi << IndexTraits<I>::half_bits) | lo);
                }
            }
        });
    }
}

template <typename T, typename I, int K>
__global__ void __launch_bounds__(kFastThreads) sep_fast_gather_kernel(const T* __restrict__ go,
                                                                       const I* __restrict__ win, T* __restrict__ gi,
                                                                       int H, int W, int border, int tiles_x,
                                                                       int tiles_y) {
    using G = FastGeom<K>;
    using A = typename GradAcc<T>::type;
    constexpr int a = G::a, GH = G::GH, GW = G::GW, NW = G::NW, TH = G::GTH, TW = kFastTW;
    constexpr uint32_t win_mask = (2 * a + 1) >= 32 ? 0xffffffffu : ((1u << (2 * a + 1)) - 1u);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* gs = reinterpret_cast<float*>(smem_raw);                       // [GH][GW] grad_output
    uint32_t* smask = reinterpret_cast<uint32_t*>(gs + GH * GW);          // [TH][TW]
    uint32_t* rmask = smask + TH * TW;                                    // [GH][2a+1][NW]
    I* ws = reinterpret_cast<I*>(rmask + GH * (2 * a + 1) * NW);          // [GH][GW] winner records

    const long long b = blockIdx.x;
    const int tx = static_cast<int>(b % tiles_x), ty = static_cast<int>((b / tiles_x) % tiles_y);
    const long long plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    const int ph0 = ty * TH, pw0 = tx * TW;
    const long long base = plane * H * W;
    const int tid = threadIdx.x;
    const uint32_t none_hi = sep_none_hi<I>();

    for (int i = tid; i < TH * TW; i += kFastThreads) smask[i] = 0u;
    for (int i = tid; i < GH * (2 * a + 1) * NW; i += kFastThreads) rmask[i] = 0u;
    for (int i = tid; i < GH * GW; i += kFastThreads) {
        const int r = i / GW, q = i - r * GW;
        const int oh = ph0 - a + r, ow = pw0 - a + q;
        I t = static_cast<I>(none_hi << IndexTraits<I>::half_bits);
        float g = 0.0f;
        if (oh >= 0 && oh < H && ow >= 0 && ow < W) {
            const long long o = base + static_cast<long long>(oh) * W + ow;
            t = win[o];
            g = Storage<T>::load(go[o]);
        }
        ws[i] = t;
        gs[i] = g;
    }
    __syncthreads();

    // Smask: row ph of the tile, every halo column ow -> the column its row winner resolves to
    for (int i = tid; i < TH * GW; i += kFastThreads) {
        const int rl = i / GW, ql = i - rl * GW;
        const int ph = ph0 + rl, ow = pw0 - a + ql;
        if (ph >= H || ow < 0 || ow >= W) continue;
        int c = ow + static_cast<int>(sep_lo<I>(ws[(rl + a) * GW + ql])) - a;
        if (!resolve(c, W, border)) continue;
        const int cl = c - pw0, bit = ow - (c - a);
        if (cl < 0 || cl >= TW || bit < 0 || bit > 2 * a) continue;
        atomicOr(&smask[rl * TW + cl], 1u << bit);
    }
    // Rmask: every halo output -> the row its column winner resolves to, if that row is in the tile
    for (int i = tid; i < GH * GW; i += kFastThreads) {
        const uint32_t h = sep_hi<I>(ws[i]);
        if (h == none_hi) continue;
        const int r0 = i / GW, q = i - r0 * GW;
        const int oh = ph0 - a + r0;
        int r = oh + static_cast<int>(h) - a;
        if (!resolve(r, H, border)) continue;
        const int rl = r - ph0;
        if (rl < 0 || rl >= TH) continue;
        const int d = r - oh + a;  // in [0, 2a] for single folds
        if (d < 0 || d > 2 * a) continue;
        atomicOr(&rmask[(r0 * (2 * a + 1) + d) * NW + (q >> 5)], 1u << (q & 31));
    }
    __syncthreads();

    for (int i = tid; i < TH * TW; i += kFastThreads) {
        const int rl = i / TW, pl = i - rl * TW;
        const int ph = ph0 + rl, pw = pw0 + pl;
        if (ph >= H || pw >= W) continue;
        const uint32_t s = smask[i];
        A acc = A(0);
        if (s) {
            const int lo_row = max(ph - a, 0), hi_row = min(ph + a, H - 1);
            for (int oh = lo_row; oh <= hi_row; ++oh) {
                const int r0 = oh - ph0 + a;
                const int d = ph - oh + a;
                const uint32_t* words = rmask + (r0 * (2 * a + 1) + d) * NW + (pl >> 5);
                uint32_t m = __funnelshift_r(words[0], words[1], pl & 31) & win_mask & s;
                while (m) {
                    const int bit = __ffs(m) - 1;
                    m &= m - 1;
                    acc = GradAcc<T>::add(acc, gs[r0 * GW + pl + bit]);
                }
            }
        }
        gi[base + static_cast<long long>(ph) * W + pw] = Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
    }
}

}  // namespace serron
