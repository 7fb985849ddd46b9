// Flat-rectangle separable path (van Herk / Gil-Werman), forward and grad_input gather.
//
// Reference behaviour followed: csrc/gpu/morphology/forward_kernels.cu:201-269 and
// csrc/cpu/morphology/operators.cpp:101-168 (row pass, then column pass, each a chunked
// prefix/suffix scan combined once per output); winners csrc/cpu/morphology/backward.cpp:116-236
// (arg-scans keep the lower offset unless the higher one is strictly better, so a row keeps its
// first extremum and the column keeps the first row).
//
// B200 layout: one CTA owns a TH x TW output tile and runs both passes out of shared memory, so the
// row result never goes to HBM.  With a winner buffer the tile also writes the direct tap
// di * kW + dj of every output's winner (di from the column pass, dj from the winning row's row pass).
#pragma once

#include "common.cuh"
#include "direct.cuh"

namespace serron {

constexpr int kSepTW = 64;   // output columns per tile
constexpr int kSepTH = 32;   // output rows per tile
constexpr int kSepThreads = 256;

template <typename A>
struct SepSmem {
    // bytes of shared memory the fused forward needs for window (kH, kW)
    static size_t bytes(int kH, int kW) {
        const size_t R = kSepTH + kH - 1, Cc = kSepTW + kW - 1;
        const size_t xs = R * Cc * sizeof(A);
        const size_t col_suffix = static_cast<size_t>(kSepTH) * kSepTW * (sizeof(A) + 2);
        const size_t a = xs > col_suffix ? xs : col_suffix;          // staged samples, later column suffix
        const size_t b = R * kSepTW * (sizeof(A) + 2);               // row suffix (value, position)
        const size_t c = R * kSepTW * (sizeof(A) + 1);               // row result (value, dj)
        return ((a + 15) / 16 + (b + 15) / 16 + (c + 15) / 16) * 16;
    }
};

template <typename A, int OP>
__device__ __forceinline__ void arg_combine(A& lo_v, int& lo_i, A hi_v, int hi_i) {
    if (Op<OP>::better(hi_v, lo_v)) {
        lo_v = hi_v;
        lo_i = hi_i;
    }
}

template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX>
__global__ void __launch_bounds__(kSepThreads) sep_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                              I* __restrict__ win, int H, int W, int kH, int kW,
                                                              int border, int tiles_x, int tiles_y) {
    using A = typename Storage<T>::acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int R = kSepTH + kH - 1, Cc = kSepTW + kW - 1;
    const int aH = kH / 2, aW = kW / 2;
    const size_t xs_bytes = static_cast<size_t>(R) * Cc * sizeof(A);
    const size_t cs_bytes = static_cast<size_t>(kSepTH) * kSepTW * (sizeof(A) + 2);
    const size_t a_bytes = ((xs_bytes > cs_bytes ? xs_bytes : cs_bytes) + 15) / 16 * 16;
    const size_t b_bytes = (static_cast<size_t>(R) * kSepTW * (sizeof(A) + 2) + 15) / 16 * 16;
    A* xs = reinterpret_cast<A*>(smem_raw);                                  // [R][Cc]
    A* cs_val = reinterpret_cast<A*>(smem_raw);                              // [TH][TW] (after row pass)
    uint16_t* cs_pos = reinterpret_cast<uint16_t*>(cs_val + kSepTH * kSepTW);
    A* rs_val = reinterpret_cast<A*>(smem_raw + a_bytes);                    // [R][TW]
    uint16_t* rs_pos = reinterpret_cast<uint16_t*>(rs_val + R * kSepTW);
    A* rv = reinterpret_cast<A*>(smem_raw + a_bytes + b_bytes);              // [R][TW]
    uint8_t* rdj = reinterpret_cast<uint8_t*>(rv + R * kSepTW);              // kW <= 256 (checked on host)

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int oh0 = tc.ty * kSepTH, ow0 = tc.tx * kSepTW;
    const T* xp = x + tc.plane * H * W;
    const int tid = threadIdx.x;
    const A neutral = Op<OP>::template neutral<A>();

    // stage the halo tile; border resolved here, NaN staged as the neutral element (it never wins)
    for (int i = tid; i < R * Cc; i += kSepThreads) {
        const int r = i / Cc, q = i - r * Cc;
        int gr = oh0 - aH + r, gq = ow0 - aW + q;
        A v = neutral;
        if (resolve(gr, H, border) && resolve(gq, W, border)) {
            v = Storage<T>::load(xp[static_cast<long long>(gr) * W + gq]);
            if (v != v) v = neutral;
        }
        xs[i] = v;
    }
    __syncthreads();

    // ---- row pass: suffix scans of each kW-chunk, stored for window starts j < TW ----
    const int nch_r = (Cc + kW - 1) / kW;
    for (int task = tid; task < R * nch_r; task += kSepThreads) {
        const int r = task / nch_r, c = task - r * nch_r;
        const int start = c * kW;
        if (start >= kSepTW) continue;
        const int end = min(start + kW, Cc) - 1;
        A sv = xs[r * Cc + end];
        int si = end;
        if (end < kSepTW) {
            rs_val[r * kSepTW + end] = sv;
            rs_pos[r * kSepTW + end] = static_cast<uint16_t>(si);
        }
        for (int p = end - 1; p >= start; --p) {
            // the lower position is the "lo" candidate: it wins ties
            A v = xs[r * Cc + p];
            int vi = p;
            arg_combine<A, OP>(v, vi, sv, si);
            sv = v;
            si = vi;
            if (p < kSepTW) {
                rs_val[r * kSepTW + p] = sv;
                rs_pos[r * kSepTW + p] = static_cast<uint16_t>(si);
            }
        }
    }
    __syncthreads();
    // ---- row pass: prefix of the next chunk, combined with the suffix ----
    for (int task = tid; task < R * nch_r; task += kSepThreads) {
        const int r = task / nch_r, c = task - r * nch_r;
        const int start = c * kW;
        if (start >= kSepTW) continue;
        A pv = A(0);
        int pi = 0;
        for (int m = 0; m < kW; ++m) {
            const int j = start + m;
            if (j >= kSepTW) break;
            A bv = rs_val[r * kSepTW + j];
            int bi = rs_pos[r * kSepTW + j];
            if (m > 0) {
                const int p = start + kW + m - 1;  // < Cc because j < TW
                const A v = xs[r * Cc + p];
                if (m == 1) {
                    pv = v;
                    pi = p;
                } else {
                    arg_combine<A, OP>(pv, pi, v, p);
                }
                arg_combine<A, OP>(bv, bi, pv, pi);
            }
            rv[r * kSepTW + j] = bv;
            rdj[r * kSepTW + j] = static_cast<uint8_t>(bi - j);
        }
    }
    __syncthreads();

    // ---- column pass over the row results: suffix scans of each kH-chunk of rows ----
    const int nch_c = (R + kH - 1) / kH;
    for (int task = tid; task < nch_c * kSepTW; task += kSepThreads) {
        const int c = task / kSepTW, j = task - c * kSepTW;
        const int start = c * kH;
        if (start >= kSepTH) continue;
        const int end = min(start + kH, R) - 1;
        A sv = rv[end * kSepTW + j];
        int si = end;
        if (end < kSepTH) {
            cs_val[end * kSepTW + j] = sv;
            cs_pos[end * kSepTW + j] = static_cast<uint16_t>(si);
        }
        for (int p = end - 1; p >= start; --p) {
            A v = rv[p * kSepTW + j];
            int vi = p;
            arg_combine<A, OP>(v, vi, sv, si);
            sv = v;
            si = vi;
            if (p < kSepTH) {
                cs_val[p * kSepTW + j] = sv;
                cs_pos[p * kSepTW + j] = static_cast<uint16_t>(si);
            }
        }
    }
    __syncthreads();
    for (int task = tid; task < nch_c * kSepTW; task += kSepThreads) {
        const int c = task / kSepTW, j = task - c * kSepTW;
        const int start = c * kH;
        if (start >= kSepTH) continue;
        const int ow = ow0 + j;
        A pv = A(0);
        int pi = 0;
        for (int m = 0; m < kH; ++m) {
            const int i = start + m;
            if (i >= kSepTH) break;
            A bv = cs_val[i * kSepTW + j];
            int bi = cs_pos[i * kSepTW + j];
            if (m > 0) {
                const int p = start + kH + m - 1;  // < R because i < TH
                const A v = rv[p * kSepTW + j];
                if (m == 1) {
                    pv = v;
                    pi = p;
                } else {
                    arg_combine<A, OP>(pv, pi, v, p);
                }
                arg_combine<A, OP>(bv, bi, pv, pi);
            }
            const int oh = oh0 + i;
            if (oh < H && ow < W) {
                const long long o = tc.plane * H * W + static_cast<long long>(oh) * W + ow;
                if (WITH_VALUE) y[o] = Storage<T>::store(bv);
                if (WITH_INDEX) {
                    // direct tap of the winner: row bi of the row results, column from its row pass
                    const uint32_t t = bv == neutral ? IndexTraits<I>::none
                                                     : static_cast<uint32_t>(bi - i) * static_cast<uint32_t>(kW) +
                                                           rdj[bi * kSepTW + j];
                    win[o] = static_cast<I>(t);
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// grad_input gather for separable winners
//
// Output o = (oh, ow) selects pixel p = (ph, pw) iff its column winner resolves to row ph and the row
// winner of row ph at column ow resolves to column pw.  The second condition does not depend on oh,
// so each pixel first collects the columns ow that pass it (a bit mask), then walks the candidate
// rows in ascending order and, within a row, the passing columns in ascending order: the reference's
// raster order.
// ------------------------------------------------------------------------------------------------
constexpr int kGTW = 32, kGTH = 32;  // pixel tile of the separable gather (256 threads, 4 rows each)

template <typename T, typename I>
__global__ void __launch_bounds__(256) sep_gather_kernel(const T* __restrict__ go, const I* __restrict__ win,
                                                         T* __restrict__ gi, int H, int W, int kH, int kW,
                                                         int border, int tiles_x, int tiles_y, int force_global) {
    using G = typename GradAcc<T>::type;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int aH = kH / 2, aW = kW / 2;
    const int rh0 = -aH, rw0 = -aW;  // symmetric halo: see direct_gather_kernel
    const int sw = kGTW + 2 * aW, sh = kGTH + 2 * aH;
    G* gs = reinterpret_cast<G*>(smem_raw);
    I* is = reinterpret_cast<I*>(gs + sw * sh);

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int ph0 = tc.ty * kGTH, pw0 = tc.tx * kGTW;
    const long long base = tc.plane * H * W;
    const int tid = threadIdx.y * kGTW + threadIdx.x;
    const uint32_t none_hi = sep_none_hi<I>();
    const bool full_h = border == kReflect && (aH > H - 1 || kH - 1 - aH > H - 1);
    const bool full_w = border == kReflect && (aW > W - 1 || kW - 1 - aW > W - 1);

    if (force_global || full_h || full_w) {
        for (int i = 0; i < kGTH / 8; ++i) {
            const int ph = ph0 + threadIdx.y * (kGTH / 8) + i, pw = pw0 + threadIdx.x;
            if (ph >= H || pw >= W) continue;
            int lh, hh, lw, hw;
            candidate_range(ph, H, kH, aH, border, lh, hh);
            candidate_range(pw, W, kW, aW, border, lw, hw);
            G acc = G(0);
            for (int oh = lh; oh <= hh; ++oh)
                for (int ow = lw; ow <= hw; ++ow) {
                    const long long o = base + static_cast<long long>(oh) * W + ow;
                    const uint32_t h = sep_hi<I>(win[o]);
                    if (h == none_hi) continue;
                    int r = oh + static_cast<int>(h) - aH;
                    if (!resolve(r, H, border) || r != ph) continue;
                    int q = ow + static_cast<int>(sep_lo<I>(win[base + static_cast<long long>(ph) * W + ow])) - aW;
                    if (resolve(q, W, border) && q == pw)
                        acc = GradAcc<T>::add(acc, static_cast<G>(Storage<T>::load(go[o])));
                }
            gi[base + static_cast<long long>(ph) * W + pw] =
                Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
        }
        return;
    }

    for (int i = tid; i < sw * sh; i += 256) {
        const int r = i / sw, q = i - r * sw;
        const int oh = ph0 + rh0 + r, ow = pw0 + rw0 + q;
        I t = static_cast<I>(none_hi << IndexTraits<I>::half_bits);
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

    for (int i = 0; i < kGTH / 8; ++i) {
        const int lr = threadIdx.y * (kGTH / 8) + i;
        const int ph = ph0 + lr, pw = pw0 + threadIdx.x;
        if (ph >= H || pw >= W) continue;
        int lh, hh, lw, hw;
        candidate_range(ph, H, kH, aH, border, lh, hh);
        candidate_range(pw, W, kW, aW, border, lw, hw);
        // the pixel's own row in shared memory (row ph sits at halo row ph - ph0 - rh0)
        const int prow = (lr - rh0) * sw - pw0 - rw0;
        G acc = G(0);
        if (kW <= 64) {
            uint64_t mask = 0;
            for (int ow = lw; ow <= hw; ++ow) {
                int q = ow + static_cast<int>(sep_lo<I>(is[prow + ow])) - aW;
                if (resolve(q, W, border) && q == pw) mask |= uint64_t(1) << (ow - lw);
            }
            if (mask) {
                for (int oh = lh; oh <= hh; ++oh) {
                    const int srow = (oh - ph0 - rh0) * sw - pw0 - rw0 + lw;
                    uint64_t m = mask;
                    while (m) {
                        const int b = __ffsll(static_cast<long long>(m)) - 1;
                        m &= m - 1;
                        const uint32_t h = sep_hi<I>(is[srow + b]);
                        if (h == none_hi) continue;
                        int r = oh + static_cast<int>(h) - aH;
                        if (resolve(r, H, border) && r == ph) acc = GradAcc<T>::add(acc, gs[srow + b]);
                    }
                }
            }
        } else {
            for (int oh = lh; oh <= hh; ++oh) {
                const int srow = (oh - ph0 - rh0) * sw - pw0 - rw0;
                for (int ow = lw; ow <= hw; ++ow) {
                    const uint32_t h = sep_hi<I>(is[srow + ow]);
                    if (h == none_hi) continue;
                    int r = oh + static_cast<int>(h) - aH;
                    if (!resolve(r, H, border) || r != ph) continue;
                    int q = ow + static_cast<int>(sep_lo<I>(is[prow + ow])) - aW;
                    if (resolve(q, W, border) && q == pw) acc = GradAcc<T>::add(acc, gs[srow + ow]);
                }
            }
        }
        gi[base + static_cast<long long>(ph) * W + pw] = Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
    }
}

}  // namespace serron
