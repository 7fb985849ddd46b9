// grad_input by pulling, strip by strip: the atomic-free gather for direct winner records.
//
// The reference forms grad_input[p] by adding grad_output of every output whose winner is p, in
// output raster order, in the storage type's arithmetic (csrc/cpu/morphology/backward.cpp:250-263).
// Only a few pixels are winners (about 1.5 % for a flat 15x15 window on noise), each of many outputs.
//
// A CTA owns a strip of kPullTQ pixel columns of one plane and a segment of its rows, and walks the
// segment in bands of kPullTB pixel rows.  For the strip it keeps, in shared-memory rings indexed by
// image row, grad_output and the winner records of the outputs that can select its pixels (the strip
// widened by aW columns each side):
//   1. the rows a band needs are staged with cp.async one band ahead, so loads overlap the work;
//   2. each staged output decodes its record into the pixel it selects (borders folded) and marks that
//      pixel when it lies in the strip; its record becomes the box tap of that pixel relative to the
//      output, (dr + aH) * S + (dc + aW) with S = 2aW + 1, which is the record itself for an odd window
//      inside the image;
//   3. the marked pixels of the band, the only ones with a non-zero gradient, are listed;
//   4. one thread per listed pixel walks the (2aH+1) x (2aW+1) box of outputs around it in raster
//      order and adds grad_output of each output whose tap points at it (four one-byte taps per
//      compare): the reference's sequence of additions for that pixel, with no atomics and no
//      ordering between threads;
//   5. the band is written out, zeros where nothing was marked.
// Every candidate must lie within a single border fold; the host sends windows wider than the image
// under REFLECT elsewhere.
#pragma once

#include "common.cuh"

namespace serron {

constexpr int kPullTQ = 64;       // pixel columns per strip
constexpr int kPullTB = 32;       // pixel rows per band
constexpr int kPullThreads = 256;

__device__ __forceinline__ void pg_cp_async16(void* smem_dst, const void* gmem_src) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void pg_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void pg_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Position of unresolved coordinate c on an axis of `size` pixels, for a candidate within one fold;
// false when it falls on a CONSTANT pad.
__device__ __forceinline__ bool fold1(int& c, int size, int border) {
    if (c >= 0 && c < size) return true;
    if (border == kConstant) return false;
    if (border == kReplicate || size == 1) {
        c = c < 0 ? 0 : size - 1;
        return true;
    }
    c = c < 0 ? -c : 2 * (size - 1) - c;
    return true;
}

// Shared-memory layout.  A staged row covers image columns from a 16-byte boundary: tap column lw
// (image column c0 - aW + lw) is element lw + goff of a grad_output row and lw + roff of a record row.
struct PullGeom {
    int aH, aW, S, hq, rr, mr, gv, goff, gq, rv, roff, rq;
    size_t go_b, rec_b, mark_b, list_b, res_b;
    __host__ __device__ static size_t up16(size_t v) { return (v + 15) / 16 * 16; }
    __host__ __device__ PullGeom(int kH, int kW, int elem, int idx)
        : aH(kH / 2), aW(kW / 2), S(2 * (kW / 2) + 1), hq(kPullTQ + 2 * (kW / 2)) {
        rr = 2 * kPullTB + 2 * aH;  // record / grad_output ring: the band's box rows and the next band
        mr = kPullTB + 2 * aH;      // mark ring: pixel rows a band's outputs can select
        gv = 16 / elem;
        goff = (gv - aW % gv) % gv;
        gq = (goff + hq + gv - 1) / gv * gv;
        rv = 16 / idx;
        roff = (rv - aW % rv) % rv;
        rq = (roff + hq + 7 + rv - 1) / rv * rv;  // + 7: the word-wise box reads run up to 6 bytes past a row
        go_b = up16(size_t(rr) * gq * elem);
        rec_b = up16(size_t(rr) * rq * idx);
        mark_b = size_t(mr) * kPullTQ;
        list_b = size_t(kPullTB) * kPullTQ * 2;
        res_b = size_t(kPullTB) * kPullTQ * elem;
    }
    __host__ __device__ size_t smem() const { return go_b + rec_b + mark_b + list_b + res_b + 16; }
    // the box taps of a (kH, kW) window fit in a record of `idx` bytes next to the all-ones "none"
    __host__ __device__ static bool taps_fit(int kH, int kW, int idx) {
        const long long box = static_cast<long long>(2 * (kH / 2) + 1) * (2 * (kW / 2) + 1);
        return idx >= 4 ? box < 0xffffffffll : box < (1ll << (8 * idx)) - 1;
    }
};

// Exact zero-byte mask of v: bit 8k+7 set where byte k of v is zero.
__device__ __forceinline__ uint32_t pg_zero_bytes(uint32_t v) {
    return ~(((v & 0x7f7f7f7fu) + 0x7f7f7f7fu) | v) & 0x80808080u;
}

// Sum for one pixel over a KB x KB box of one-byte taps (KB = 2a + 1 known at compile time).  The box
// is unrolled: the taps of a row are matched four at a time against constants, and every matching
// grad_output load is issued before the row's additions, which then run back to back in order.
//   tw       record ring as 32-bit words (rqw words per slot); slot0 ring slot of box row 0;
//   pc0      byte offset in a record row of box column 0;
//   gp       grad_output ring at box column 0 of slot 0 (gq elements per slot);
//   rows_ok  bit r: box row r lies in the image;  keep[g]: 0x80 in byte k where box column 4g+k does.
template <int KB, typename T>
__device__ __forceinline__ typename GradAcc<T>::type pull_box_fixed(const uint32_t* tw, const T* gp, int slot0,
                                                                    int RR, int rqw, int gq, int pc0,
                                                                    uint32_t rows_ok,
                                                                    const uint32_t (&keep)[(KB + 3) / 4]) {
    using G = typename GradAcc<T>::type;
    constexpr int NG = (KB + 3) / 4;
    const int sh = (pc0 & 3) * 8;
    const int w0 = pc0 >> 2;
    G acc = G(0);
    int slot = slot0;
#pragma unroll
    for (int r = 0; r < KB; ++r) {
        if (rows_ok & (1u << r)) {
            const uint32_t* row = tw + slot * rqw + w0;
            const T* grow = gp + slot * gq;
            uint32_t wd[NG + 1];
#pragma unroll
            for (int i = 0; i <= NG; ++i) wd[i] = row[i];
            uint32_t m[NG];
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                // box column j = 4g + k of row r is selected by the tap (KB - 1 - r) * KB + (KB - 1) - j;
                // bytes past the box may borrow, and are dropped by keep
                const uint32_t pat =
                    static_cast<uint32_t>((KB - 1 - r) * KB + (KB - 1) - 4 * g) * 0x01010101u - 0x03020100u;
                m[g] = pg_zero_bytes(__funnelshift_r(wd[g], wd[g + 1], sh) ^ pat) & keep[g];
            }
            G v[KB];
#pragma unroll
            for (int j = 0; j < KB; ++j)
                v[j] = (m[j >> 2] >> (8 * (j & 3) + 7)) & 1u ? static_cast<G>(Storage<T>::load(grow[j])) : G(0);
#pragma unroll
            for (int j = 0; j < KB; ++j)
                if ((m[j >> 2] >> (8 * (j & 3) + 7)) & 1u) acc = GradAcc<T>::add(acc, v[j]);
        }
        if (++slot == RR) slot = 0;
    }
    return acc;
}

template <int KB, typename T>
__device__ __forceinline__ typename GradAcc<T>::type pull_box_fixed_at(const uint8_t* tapS, const T* goS, int slot0,
                                                                       int RR, int rq, int gq, int roff, int goff,
                                                                       int pc, int x, int y, int H, int W) {
    constexpr int a = KB / 2, NG = (KB + 3) / 4;
    const int rlo = max(0, a - x), rhi = min(KB - 1, H - 1 - x + a);
    const uint32_t rows_ok = (rhi < rlo) ? 0u : ((2u << rhi) - 1u) & ~((1u << rlo) - 1u);
    const int jlo = max(0, a - y), jhi = min(KB - 1, W - 1 - y + a);
    uint32_t keep[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        uint32_t k = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = 4 * g + e;
            if (j < KB && j >= jlo && j <= jhi) k |= 0x80u << (8 * e);
        }
        keep[g] = k;
    }
    return pull_box_fixed<KB, T>(reinterpret_cast<const uint32_t*>(tapS), goS + goff + pc, slot0, RR, rq / 4, gq,
                                 roff + pc, rows_ok, keep);
}

template <typename T, typename I>
__global__ void __launch_bounds__(kPullThreads, 4) pull_gather_kernel(const T* __restrict__ go,
                                                                   const I* __restrict__ win, T* __restrict__ gi,
                                                                   int H, int W, int kH, int kW, int border,
                                                                   int strips, int segs, int seg_h, int go_vec,
                                                                   int rec_vec, int out_vec) {
    using G = typename GradAcc<T>::type;
    constexpr int TQ = kPullTQ, TB = kPullTB, NT = kPullThreads;
    constexpr uint32_t kNone = IndexTraits<I>::none;
    const PullGeom geo(kH, kW, sizeof(T), sizeof(I));
    const int aH = geo.aH, aW = geo.aW, S = geo.S, hq = geo.hq, RR = geo.rr, MR = geo.mr;
    const int gv = geo.gv, goff = geo.goff, gq = geo.gq, rv = geo.rv, roff = geo.roff, rq = geo.rq;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* goS = reinterpret_cast<T*>(smem_raw);                                             // [RR][gq]
    I* tapS = reinterpret_cast<I*>(smem_raw + geo.go_b);                                 // [RR][rq]
    uint8_t* markS = smem_raw + geo.go_b + geo.rec_b;                                    // [MR][TQ]
    uint16_t* listS = reinterpret_cast<uint16_t*>(markS + geo.mark_b);                   // [TB * TQ]
    T* resS = reinterpret_cast<T*>(smem_raw + geo.go_b + geo.rec_b + geo.mark_b + geo.list_b);  // [TB][TQ]
    int* countS = reinterpret_cast<int*>(smem_raw + geo.go_b + geo.rec_b + geo.mark_b + geo.list_b + geo.res_b);

    const long long b = blockIdx.x;
    const int strip = static_cast<int>(b % strips);
    const int seg = static_cast<int>((b / strips) % segs);
    const long long plane = b / (static_cast<long long>(strips) * segs);
    const int c0 = strip * TQ;
    const int ph0 = seg * seg_h, ph1 = min(H, ph0 + seg_h);
    const T* gop = go + plane * H * W;
    const I* wp = win + plane * H * W;
    T* gip = gi + plane * H * W;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hbase = ph0 - aH;  // ring slot of output row h: (h - hbase) mod RR
    const int hend = min(H, ph1 + aH);

    // stage output rows [lo, hi) into their ring slots (warp per row)
    // stage output rows [lo, hi) into their ring slots; the (row, 16-byte chunk) copies are spread over
    // all threads, grad_output first, then records
    const int nchg = gq / gv, nchr = rq / rv;
    const uint32_t nchg_magic = static_cast<uint32_t>(((1ull << 32) + nchg - 1) / nchg);  // i < 2^16: exact
    const uint32_t nchr_magic = static_cast<uint32_t>(((1ull << 32) + nchr - 1) / nchr);
    auto stage = [&](int lo, int hi) {
        lo = max(lo, 0);
        const int n = hi - lo;  // <= RR rows
        if (n > 0) {
            const int slot_lo = (lo - hbase) % RR;
            for (int i = tid; i < n * nchg; i += NT) {
                const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), nchg_magic));
                const int k = i - r * nchg;
                int slot = slot_lo + r;
                if (slot >= RR) slot -= RR;
                const int col = c0 - aW - goff + k * gv;
                T* dst = goS + slot * gq + k * gv;
                const T* src = gop + static_cast<long long>(lo + r) * W + col;
                if (go_vec && col >= 0 && col + gv <= W) {
                    pg_cp_async16(dst, src);
                } else {
                    for (int e = 0; e < gv; ++e) dst[e] = (col + e >= 0 && col + e < W) ? src[e] : Storage<T>::store(0.0f);
                }
            }
            for (int i = tid; i < n * nchr; i += NT) {
                const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), nchr_magic));
                const int k = i - r * nchr;
                int slot = slot_lo + r;
                if (slot >= RR) slot -= RR;
                const int col = c0 - aW - roff + k * rv;
                I* dst = tapS + slot * rq + k * rv;
                const I* src = wp + static_cast<long long>(lo + r) * W + col;
                if (rec_vec && col >= 0 && col + rv <= W) {
                    pg_cp_async16(dst, src);
                } else {
                    for (int e = 0; e < rv; ++e) dst[e] = (col + e >= 0 && col + e < W) ? src[e] : static_cast<I>(kNone);
                }
            }
        }
        pg_commit();
    };

    for (int i = tid; i < MR * TQ / 4; i += NT) reinterpret_cast<uint32_t*>(markS)[i] = 0u;
    for (int i = tid; i < int(geo.res_b / 16); i += NT) reinterpret_cast<uint4*>(resS)[i] = make_uint4(0, 0, 0, 0);
    // the first band needs output rows up to ph0 + TB + aH
    stage(hbase, min(hend, ph0 + TB + aH));

    const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;
    const bool odd_w = (kW & 1) != 0;
    // odd square windows up to 15 x 15 with one-byte records take the unrolled box sum
    const bool box_fixed = sizeof(I) == 1 && kH == kW && odd_w && kW >= 3 && kW <= 15;
    int decoded = max(hbase, 0);  // output rows below this are decoded
    int mbase = 0;                // mark-ring slot of pixel row R

    for (int R = ph0; R < ph1; R += TB) {
        const int nb = min(TB, ph1 - R);
        const int need = min(hend, R + TB + aH);  // output rows the band's boxes reach
        pg_wait_all();
        __syncthreads();
        // prefetch the next band's new rows into slots no box of this band uses
        if (R + TB < ph1) stage(need, min(hend, R + 2 * TB + aH));

        // 2. decode output rows [decoded, need): tap of the selected pixel, mark it when in the strip.
        //    A mark lands in pixel rows [xlo, xhi) (the segment, and the rows the mark ring holds) and
        //    columns [c0, c0 + ylen).
        {
            const int xlo = max(ph0, R), xhi = min(ph1, R + MR);
            const int ylen = min(TQ, W - c0);
            auto decode = [&](I& rec, int h, int w) {
                const uint32_t t = rec;
                if (t == kNone) return;
                const uint32_t di = sizeof(I) <= 2 ? (kW > 1 ? __umulhi(t, kw_magic) : t) : t / static_cast<uint32_t>(kW);
                const int dj = static_cast<int>(t - di * static_cast<uint32_t>(kW));
                int x = h + static_cast<int>(di) - aH, y = w + dj - aW;
                if (static_cast<unsigned>(x) >= static_cast<unsigned>(H) ||
                    static_cast<unsigned>(y) >= static_cast<unsigned>(W)) {
                    if (!fold1(x, H, border) || !fold1(y, W, border)) {  // a CONSTANT pad never wins
                        rec = static_cast<I>(kNone);
                        return;
                    }
                    rec = static_cast<I>((x - h + aH) * S + (y - w + aW));
                } else if (!odd_w) {
                    rec = static_cast<I>((x - h + aH) * S + (y - w + aW));
                }
                if (static_cast<unsigned>(x - xlo) < static_cast<unsigned>(xhi - xlo) &&
                    static_cast<unsigned>(y - c0) < static_cast<unsigned>(ylen)) {
                    int ms = mbase + (x - R);
                    if (ms >= MR) ms -= MR;
                    markS[ms * TQ + (y - c0)] = 1;
                }
            };
            // every target of rows [decoded, need) in this strip lies inside the image: no folding, and the
            // record of an odd window is its own tap
            const bool fast = odd_w && decoded - aH >= 0 && need - 1 + aH <= H - 1 && c0 - 2 * aW >= 0 &&
                              c0 + TQ + 2 * aW <= W;
            if (sizeof(I) == 1 && fast) {
                // (row, word) items over all threads: four records per word, staged columns
                // [4 * wfirst, 4 * (wfirst + nwords)) hold tap columns [0, hq) and a few real neighbours,
                // whose targets fall outside the strip.  A "none" record decodes to some pixel that no
                // tap selects: marking it costs a sum of zero terms, so it is not filtered.
                const int wfirst = roff >> 2, nwords = ((roff + hq - 1) >> 2) - wfirst + 1;
                const uint32_t nw_magic = static_cast<uint32_t>(((1ull << 32) + nwords - 1) / nwords);
                const int nrows = need - decoded;
                const int slot_d = (decoded - hbase) % RR;
                const int rqw = rq / 4;
                const uint32_t* tw = reinterpret_cast<const uint32_t*>(tapS);
                const int mrow0 = mbase - R;  // mark-ring row of pixel row x: x + mrow0, less MR past the end
                for (int i = tid; i < nrows * nwords; i += NT) {
                    const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), nw_magic));
                    const int q = i - r * nwords;
                    int slot = slot_d + r;
                    if (slot >= RR) slot -= RR;
                    const uint32_t word = tw[slot * rqw + wfirst + q];
                    const int xb = decoded + r - aH;                       // target row = xb + di
                    const int yb = 4 * (wfirst + q) - roff - 2 * aW;        // target column - c0 = yb + e + dj
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t t = (word >> (8 * e)) & 0xffu;
                        const uint32_t di = kW > 1 ? __umulhi(t, kw_magic) : t;
                        const int x = xb + static_cast<int>(di);
                        const int yc = yb + e + static_cast<int>(t - di * static_cast<uint32_t>(kW));
                        if (static_cast<unsigned>(yc) < static_cast<unsigned>(ylen) &&
                            static_cast<unsigned>(x - xlo) < static_cast<unsigned>(xhi - xlo)) {
                            int ms = x + mrow0;
                            if (ms >= MR) ms -= MR;
                            markS[ms * TQ + yc] = 1;
                        }
                    }
                }
            } else if constexpr (sizeof(I) == 1) {
                // four records per word; tap columns [0, hq) are bytes [roff, roff + hq) of a row
                const int wfirst = roff >> 2, nwords = ((roff + hq - 1) >> 2) - wfirst + 1;
                for (int h = decoded + warp; h < need; h += NT / 32) {
                    const int slot = (h - hbase) % RR;
                    uint32_t* trow = reinterpret_cast<uint32_t*>(tapS + slot * rq);
                    for (int q = lane; q < nwords; q += 32) {
                        const int wi = wfirst + q;
                        uint32_t word = trow[wi];
                        if (word == 0xffffffffu) continue;
                        uint8_t* bytes = reinterpret_cast<uint8_t*>(&word);
                        const uint32_t before = word;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int lw = wi * 4 + e - roff;
                            const int w = c0 - aW + lw;
                            if (static_cast<unsigned>(lw) < static_cast<unsigned>(hq) &&
                                static_cast<unsigned>(w) < static_cast<unsigned>(W))
                                decode(*reinterpret_cast<I*>(bytes + e), h, w);
                        }
                        if (word != before) trow[wi] = word;
                    }
                }
            } else {
                for (int h = decoded + warp; h < need; h += NT / 32) {
                    const int slot = (h - hbase) % RR;
                    I* trow = tapS + slot * rq + roff;
                    for (int lw = lane; lw < hq; lw += 32) {
                        const int w = c0 - aW + lw;
                        if (static_cast<unsigned>(w) < static_cast<unsigned>(W)) decode(trow[lw], h, w);
                    }
                }
            }
        }
        decoded = need;
        if (tid == 0) *countS = 0;
        __syncthreads();

        // 3. list the band's marked pixels and clear their marks
        for (int base = 0; base < TB * TQ / 4; base += NT) {
            const int i = base + tid;  // word i: band row i / (TQ / 4), pixels 4 * (i % (TQ / 4)) + 0..3
            uint32_t m = 0;
            if (i < nb * (TQ / 4)) {
                const int r = i / (TQ / 4);
                int ms = mbase + r;
                if (ms >= MR) ms -= MR;
                uint32_t* wptr = reinterpret_cast<uint32_t*>(markS + ms * TQ) + (i - r * (TQ / 4));
                const uint32_t v = *wptr;
                if (v) {
                    *wptr = 0u;
                    m = ~pg_zero_bytes(v) & 0x80808080u;
                }
            }
            const int cnt = __popc(m);
            int incl = cnt;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, incl, d);
                if (lane >= d) incl += o;
            }
            int wbase = 0;
            if (lane == 31 && incl) wbase = atomicAdd(countS, incl);
            wbase = __shfl_sync(0xffffffffu, wbase, 31);
            int pos = wbase + incl - cnt;
            while (m) {
                const int k = (__ffs(m) - 8) >> 3;
                m &= m - 1;
                listS[pos++] = static_cast<uint16_t>(4 * i + k);
            }
        }
        __syncthreads();

        // 4. one thread per marked pixel: the outputs of its box in raster order
        const int n = *countS;
        for (int k = tid; k < n; k += NT) {
            const int p = listS[k];
            const int pr = p / TQ, pc = p - pr * TQ;
            const int x = R + pr, y = c0 + pc;
            const int hlo = max(0, x - aH), hhi = min(H - 1, x + aH);
            const int jlo = max(0, aW - y), jhi = min(2 * aW, W - 1 - y + aW);  // box columns in the image
            G acc = G(0);
            if constexpr (sizeof(I) == 1) {
                if (box_fixed) {
                    const int slot0 = (x - aH - hbase) % RR;  // x - aH - hbase = x - ph0 >= 0
                    const uint8_t* t8 = reinterpret_cast<const uint8_t*>(tapS);
                    switch (kW) {
#define SERRON_PULL_FIXED(KB)                                                                                \
    case KB: acc = pull_box_fixed_at<KB, T>(t8, goS, slot0, RR, rq, gq, roff, goff, pc, x, y, H, W); break;
                        SERRON_PULL_FIXED(3) SERRON_PULL_FIXED(5) SERRON_PULL_FIXED(7) SERRON_PULL_FIXED(9)
                        SERRON_PULL_FIXED(11) SERRON_PULL_FIXED(13) SERRON_PULL_FIXED(15)
#undef SERRON_PULL_FIXED
                    default: break;
                    }
                    resS[p] = Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
                    continue;
                }
            }
            int slot = (hlo - hbase) % RR;
            for (int h = hlo; h <= hhi; ++h) {
                const I* trow = tapS + slot * rq + roff + pc;  // box column j at trow[j]
                const T* grow = goS + slot * gq + goff + pc;
                const int e0 = (x - h + aH) * S + 2 * aW;      // tap expected at box column 0
                if constexpr (sizeof(I) == 1) {
                    const uint32_t* wrow = reinterpret_cast<const uint32_t*>(tapS + slot * rq);
                    const int byte0 = roff + pc;
                    const int sh = (byte0 & 3) * 8;
                    const uint32_t* wq = wrow + (byte0 >> 2);
                    uint32_t lo_w = wq[0];
                    for (int j0 = 0; j0 <= jhi; j0 += 4) {
                        const uint32_t hi_w = wq[(j0 >> 2) + 1];
                        const uint32_t g = __funnelshift_r(lo_w, hi_w, sh);
                        lo_w = hi_w;
                        // bytes j0 .. j0+3 expected e0 - j0 - k (borrows only reach bytes past the box)
                        const uint32_t pat = static_cast<uint32_t>(e0 - j0) * 0x01010101u - 0x03020100u;
                        uint32_t m = pg_zero_bytes(g ^ pat);
                        // keep box columns jlo .. jhi
                        const int a0 = jlo - j0, a1 = jhi - j0;
                        const uint32_t keep_lo = a0 <= 0 ? 0xffffffffu : (a0 >= 4 ? 0u : 0xffffffffu << (8 * a0));
                        const uint32_t keep_hi = a1 >= 3 ? 0xffffffffu : (a1 < 0 ? 0u : 0xffffffffu >> (8 * (3 - a1)));
                        m &= keep_lo & keep_hi;
                        while (m) {
                            const int kk = (__ffs(m) - 8) >> 3;
                            m &= m - 1;
                            acc = GradAcc<T>::add(acc, static_cast<G>(Storage<T>::load(grow[j0 + kk])));
                        }
                    }
                } else {
                    for (int j = jlo; j <= jhi; ++j)
                        if (static_cast<int>(trow[j]) == e0 - j)
                            acc = GradAcc<T>::add(acc, static_cast<G>(Storage<T>::load(grow[j])));
                }
                if (++slot == RR) slot = 0;
            }
            resS[p] = Storage<T>::store(static_cast<typename Storage<T>::acc>(acc));
        }
        __syncthreads();

        // 5. write the band and clear the result tile
        {
            const int ov = 16 / int(sizeof(T));
            for (int i = tid; i < nb * (TQ / ov); i += NT) {
                const int pr = i / (TQ / ov), pc = (i - pr * (TQ / ov)) * ov;
                const int c = c0 + pc;
                uint4* src = reinterpret_cast<uint4*>(resS) + i;
                if (c < W) {
                    T* dst = gip + static_cast<long long>(R + pr) * W + c;
                    if (out_vec && c + ov <= W) {
                        *reinterpret_cast<uint4*>(dst) = *src;
                    } else {
                        for (int e = 0; e < ov && c + e < W; ++e) dst[e] = resS[pr * TQ + pc + e];
                    }
                }
                *src = make_uint4(0, 0, 0, 0);
            }
        }
        mbase += TB;
        if (mbase >= MR) mbase -= MR;
    }
    pg_wait_all();
}

}  // namespace serron
