// grad_input by marking and pulling: the atomic-free gather for direct winner records.
//
// The reference forms grad_input[p] by adding grad_output of every output whose winner is p, in
// output raster order, in the storage type's arithmetic (csrc/cpu/morphology/backward.cpp:250-263).
// Only a few pixels are winners (about 1.5 % for a flat 15x15 window on noise), each of many outputs,
// so the work splits in two launches:
//
//   pull_mark_kernel  finds the winners.  A CTA owns a strip of kPullTQ pixel columns of one plane and
//                     a segment of its rows, and streams the records of the outputs that can select
//                     them (the strip widened by aW columns) through a shared-memory ring, one band of
//                     kPullTB rows ahead with cp.async.  Every record is decoded into the pixel it
//                     selects (borders folded) and that pixel is marked.  Each finished band leaves
//                     as one bit per pixel in the target map.  (The separable sweep forward sets the
//                     map itself while it writes the records; then this launch is skipped.)
//   pull_sum_kernel   computes grad_input.  A CTA owns a kSumTP x kPullTQ tile, writes it as zeros
//                     (16-byte stores), reads its map words (done when they are empty), stages
//                     grad_output and the records of the tile grown by the box halo in shared memory
//                     with cp.async, lists the set
//                     bits, and one thread per winner p walks the (2aH+1) x (2aW+1) box of outputs around
//                     p in raster order, adding grad_output of each output that selects p: exactly the
//                     reference's sequence of additions for p, with no atomics and no ordering between
//                     threads.  Inside the image an odd window's record IS the box tap of its winner,
//                     (dr + aH) * kW + (dc + aW), so for boxes up to 15 x 15 the test runs on four
//                     one-byte records at a time against constants, with the box unrolled.  Each
//                     winner's sum is stored over the zeros.
//
// Every candidate must lie within a single border fold; the host sends windows wider than the image
// under REFLECT elsewhere.
#pragma once

#include "bulk_copy.cuh"
#include "common.cuh"

namespace serron {

constexpr int kPullTQ = 64;       // pixel columns per strip (two target-map words)
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

// Pixel selected by the direct record t of output (h, w); false for "none" and for a CONSTANT pad.
__device__ __forceinline__ bool pg_target(uint32_t t, uint32_t none, int h, int w, int H, int W, int kW, int aH,
                                          int aW, int border, uint32_t kw_magic, int& x, int& y) {
    if (t == none) return false;
    const uint32_t di = t <= 0xffffu ? (kW > 1 ? __umulhi(t, kw_magic) : t) : t / static_cast<uint32_t>(kW);
    x = h + static_cast<int>(di) - aH;
    y = w + static_cast<int>(t - di * static_cast<uint32_t>(kW)) - aW;
    return fold1(x, H, border) && fold1(y, W, border);
}

// Shared-memory layout of the mark kernel: a record row covers image columns from a 16-byte
// boundary, tap column lw (image column c0 - aW + lw) at element lw + roff.
struct PullGeom {
    int aH, aW, hq, rr, mr, rv, roff, rq;
    size_t rec_b, mark_b;
    __host__ __device__ PullGeom(int kH, int kW, int idx) : aH(kH / 2), aW(kW / 2), hq(kPullTQ + 2 * (kW / 2)) {
        rr = 2 * kPullTB + 2 * aH;  // record ring: the band's rows and the next band's
        mr = kPullTB + 2 * aH;      // mark ring: pixel rows a band's outputs can select
        rv = 16 / idx;
        roff = (rv - aW % rv) % rv;
        rq = (roff + hq + 3 + rv - 1) / rv * rv;
        rec_b = (size_t(rr) * rq * idx + 15) / 16 * 16;
        mark_b = size_t(mr) * kPullTQ;
    }
    __host__ __device__ size_t smem() const { return rec_b + mark_b; }
};

// Words of the target map of `planes` images of H x W: one bit per pixel, rows of ceil(W / 32) words.
__host__ __device__ inline long long pull_map_words(long long planes, long long H, long long W) {
    return planes * H * ((W + 31) / 32);
}

template <typename I>
__global__ void __launch_bounds__(kPullThreads, 4) pull_mark_kernel(const I* __restrict__ win, uint32_t* __restrict__ map,
                                                                    int H, int W, int kH, int kW, int border,
                                                                    int strips, int segs, int seg_h, int rec_vec) {
    constexpr int TQ = kPullTQ, TB = kPullTB, NT = kPullThreads;
    constexpr uint32_t kNone = IndexTraits<I>::none;
    const PullGeom geo(kH, kW, sizeof(I));
    const int aH = geo.aH, aW = geo.aW, hq = geo.hq, RR = geo.rr, MR = geo.mr;
    const int rv = geo.rv, roff = geo.roff, rq = geo.rq;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    I* recS = reinterpret_cast<I*>(smem_raw);  // [RR][rq]
    uint8_t* markS = smem_raw + geo.rec_b;     // [MR][TQ]

    const long long b = blockIdx.x;
    const int strip = static_cast<int>(b % strips);
    const int seg = static_cast<int>((b / strips) % segs);
    const long long plane = b / (static_cast<long long>(strips) * segs);
    const int c0 = strip * TQ;
    const int ph0 = seg * seg_h, ph1 = min(H, ph0 + seg_h);
    const I* wp = win + plane * H * W;
    const int WW = (W + 31) / 32;
    uint32_t* mapp = map + plane * H * WW;
    const int tid = threadIdx.x;
    const int hbase = ph0 - aH;  // ring slot of output row h: (h - hbase) mod RR
    const int hend = min(H, ph1 + aH);

    // stage output rows [lo, hi) into their ring slots, (row, 16-byte chunk) copies over all threads
    const int nch = rq / rv;
    const uint32_t nch_magic = static_cast<uint32_t>(((1ull << 32) + nch - 1) / nch);  // i < 2^16: exact
    auto stage = [&](int lo, int hi) {
        lo = max(lo, 0);
        const int n = hi - lo;  // <= RR rows
        if (n > 0) {
            const int slot_lo = (lo - hbase) % RR;
            for (int i = tid; i < n * nch; i += NT) {
                const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), nch_magic));
                const int k = i - r * nch;
                int slot = slot_lo + r;
                if (slot >= RR) slot -= RR;
                const int col = c0 - aW - roff + k * rv;
                I* dst = recS + slot * rq + k * rv;
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
    stage(hbase, min(hend, ph0 + TB + aH));  // the first band's rows

    const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;
    int decoded = max(hbase, 0);  // output rows below this are decoded
    int mbase = 0;                // mark-ring row of pixel row R

    for (int R = ph0; R < ph1; R += TB) {
        const int nb = min(TB, ph1 - R);
        const int need = min(hend, R + TB + aH);  // every output that can select a pixel of the band
        pg_wait_all();
        __syncthreads();
        if (R + TB < ph1) stage(need, min(hend, R + 2 * TB + aH));  // slots no row of this band uses

        // decode output rows [decoded, need); marks land in pixel rows [xlo, xhi) (the segment, and the
        // rows the mark ring holds) and strip columns [0, ylen)
        {
            const int xlo = max(ph0, R), xhi = min(ph1, R + MR);
            const int ylen = min(TQ, W - c0);
            const int mrow0 = mbase - R;  // mark-ring row of pixel row x: x + mrow0, less MR past the end
            auto mark = [&](int x, int yc) {
                if (static_cast<unsigned>(yc) < static_cast<unsigned>(ylen) &&
                    static_cast<unsigned>(x - xlo) < static_cast<unsigned>(xhi - xlo)) {
                    int ms = x + mrow0;
                    if (ms >= MR) ms -= MR;
                    markS[ms * TQ + yc] = 1;
                }
            };
            const int nrows = need - decoded;
            const int slot_d = (decoded - hbase) % RR;
            if constexpr (sizeof(I) == 1) {
                // (row, word) items, four records per word.  The words span tap columns [0, hq) and a few
                // real neighbours, whose targets (folded or not) fall outside the strip; staged columns
                // outside the image hold "none".  Only outputs near the image edge take the fold branch.
                const int wfirst = roff >> 2, nwords = ((roff + hq - 1) >> 2) - wfirst + 1;
                const uint32_t nw_magic = static_cast<uint32_t>(((1ull << 32) + nwords - 1) / nwords);
                const uint32_t* tw = reinterpret_cast<const uint32_t*>(recS);
                const int rqw = rq / 4;
                for (int i = tid; i < nrows * nwords; i += NT) {
                    const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), nw_magic));
                    const int q = i - r * nwords;
                    int slot = slot_d + r;
                    if (slot >= RR) slot -= RR;
                    const uint32_t word = tw[slot * rqw + wfirst + q];
                    const int h = decoded + r;
                    const int wb = c0 - aW + 4 * (wfirst + q) - roff;  // image column of byte 0
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t t = (word >> (8 * e)) & 0xffu;
                        if (t == 0xffu) continue;
                        const uint32_t di = kW > 1 ? __umulhi(t, kw_magic) : t;
                        int x = h + static_cast<int>(di) - aH;
                        int y = wb + e + static_cast<int>(t - di * static_cast<uint32_t>(kW)) - aW;
                        if (static_cast<unsigned>(x) >= static_cast<unsigned>(H) ||
                            static_cast<unsigned>(y) >= static_cast<unsigned>(W)) {
                            if (!fold1(x, H, border) || !fold1(y, W, border)) continue;  // CONSTANT pad
                        }
                        mark(x, y - c0);
                    }
                }
            } else {
                const uint32_t hq_magic = static_cast<uint32_t>(((1ull << 32) + hq - 1) / hq);
                for (int i = tid; i < nrows * hq; i += NT) {
                    const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), hq_magic));
                    const int lw = i - r * hq;
                    int slot = slot_d + r;
                    if (slot >= RR) slot -= RR;
                    const int h = decoded + r, w = c0 - aW + lw;
                    int x, y;
                    if (static_cast<unsigned>(w) < static_cast<unsigned>(W) &&
                        pg_target(recS[slot * rq + roff + lw], kNone, h, w, H, W, kW, aH, aW, border, kw_magic, x, y))
                        mark(x, y - c0);
                }
            }
        }
        decoded = need;
        __syncthreads();

        // the band leaves as target-map words (a thread packs the 32 mark bytes of a word, each 0 or 1)
        for (int i = tid; i < nb * (TQ / 32); i += NT) {
            const int r = i / (TQ / 32), k = i - r * (TQ / 32);
            int ms = mbase + r;
            if (ms >= MR) ms -= MR;
            uint4* mrow = reinterpret_cast<uint4*>(markS + ms * TQ + 32 * k);
            const uint4 lo4 = mrow[0], hi4 = mrow[1];
            mrow[0] = mrow[1] = make_uint4(0, 0, 0, 0);
            const uint32_t q[8] = {lo4.x, lo4.y, lo4.z, lo4.w, hi4.x, hi4.y, hi4.z, hi4.w};
            uint32_t bits = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) bits |= ((q[e] | (q[e] >> 7) | (q[e] >> 14) | (q[e] >> 21)) & 0xfu) << (4 * e);
            if (c0 / 32 + k < WW) mapp[static_cast<long long>(R + r) * WW + c0 / 32 + k] = bits;
        }
        mbase += TB;
        if (mbase >= MR) mbase -= MR;
    }
    pg_wait_all();
}

// Exact zero-byte mask of v: bit 8k+7 set where byte k of v is zero.
__device__ __forceinline__ uint32_t pg_zero_bytes(uint32_t v) {
    return ~(((v & 0x7f7f7f7fu) + 0x7f7f7f7fu) | v) & 0x80808080u;
}

constexpr int kSumTP = 32;        // pixel rows per sum tile (kPullTQ columns)
constexpr int kSumThreads = 128;

// Shared-memory layout of the sum kernel: the tile's outputs and their box halo, rows
// [r0 - aH, r0 + kSumTP + aH); a staged row starts on a 16-byte boundary of the image row, so box
// column lw (image column c0 - aW + lw) is element lw + goff of a grad_output row, lw + roff of a record
// row, with a few bytes of slack behind the record row for word-wise reads.
struct SumGeom {
    int aH, aW, hr, hq, gv, goff, gq, rv, roff, rq;
    size_t go_b, rec_b, list_b;
    __host__ __device__ SumGeom(int kH, int kW, int elem, int idx)
        : aH(kH / 2), aW(kW / 2), hr(kSumTP + 2 * (kH / 2)), hq(kPullTQ + 2 * (kW / 2)) {
        gv = 16 / elem;
        goff = (gv - aW % gv) % gv;
        gq = (goff + hq + gv - 1) / gv * gv;
        rv = 16 / idx;
        roff = (rv - aW % rv) % rv;
        rq = (roff + hq + 7 + rv - 1) / rv * rv;  // + 7: the word reads of a box row run 6 bytes past it
        go_b = (size_t(hr) * gq * elem + 15) / 16 * 16;
        rec_b = (size_t(hr) * rq * idx + 15) / 16 * 16;
        list_b = size_t(kSumTP) * kPullTQ * 2;

    }
    __host__ __device__ size_t smem() const { return go_b + rec_b + list_b + 16; }
};

// Sum for one pixel over its KB x KB box (KB = 2a + 1) of one-byte box taps staged in shared memory.
// Box rows run in a loop unrolled three times (the fully unrolled box overflowed the instruction cache;
// three rows let the next rows' loads issue early: -2 % on the 15 x 15 gather, five rows +4 %); within a
// row the taps are matched four at a time against constants, and the matching grad_output loads are
// issued before the row's additions, which then run back to back in order.
//   rec      tap row of box row 0 at box column 0 (a byte address; rows rq bytes apart, rq % 4 == 0)
//   gp       grad_output of box row 0 at box column 0 (rows gq elements apart)
//   rows_ok  bit r: box row r lies in the image;  keep[g]: 0x80 in byte k where box column 4g+k does
template <int KB, typename T, typename TG>
__device__ __forceinline__ typename GradAcc<T>::type pull_box_fixed(const uint8_t* rec, int rq, const TG* gp, int gq,
                                                                    uint32_t rows_ok,
                                                                    const uint32_t (&keep)[(KB + 3) / 4]) {
    using G = typename GradAcc<T>::type;
    constexpr int NG = (KB + 3) / 4;
    G acc = G(0);
    const uintptr_t addr = reinterpret_cast<uintptr_t>(rec);
    const uint32_t* row = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
    const int sh = static_cast<int>(addr & 3) * 8;  // the same in every row: rows are a multiple of 4 bytes apart
    const int rqw = rq >> 2;
    // box column j = 4g + k of row r selects the pixel with tap (KB - 1 - r) * KB + (KB - 1) - j: byte k of
    // group g of row r is matched against pat - (4g * 0x01010101), pat dropping by KB in every byte per row
    // (bytes past the box may borrow, and are dropped by keep)
    uint32_t pat = static_cast<uint32_t>((KB - 1) * KB + (KB - 1)) * 0x01010101u - 0x03020100u;
#pragma unroll 3
    for (int r = 0; r < KB; ++r, row += rqw, gp += gq, pat -= static_cast<uint32_t>(KB) * 0x01010101u) {
        if (!(rows_ok & (1u << r))) continue;
        uint32_t wd[NG + 1];
#pragma unroll
        for (int i = 0; i <= NG; ++i) wd[i] = row[i];
        uint32_t m[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g)
            m[g] = pg_zero_bytes(__funnelshift_r(wd[g], wd[g + 1], sh) ^ (pat - static_cast<uint32_t>(4 * g) * 0x01010101u)) &
                   keep[g];
        G v[KB];
#pragma unroll
        for (int j = 0; j < KB; ++j)
            v[j] = (m[j >> 2] >> (8 * (j & 3) + 7)) & 1u ? static_cast<G>(Storage<TG>::load(gp[j])) : G(0);
#pragma unroll
        for (int j = 0; j < KB; ++j)
            if ((m[j >> 2] >> (8 * (j & 3) + 7)) & 1u) acc = GradAcc<T>::add(acc, v[j]);
    }
    return acc;
}

template <int KB, typename T, typename TG>
__device__ __forceinline__ typename GradAcc<T>::type pull_box_fixed_clip(const uint8_t* rec, int rq, const TG* gp,
                                                                         int gq, int x, int y, int H, int W) {
    constexpr int a = KB / 2, NG = (KB + 3) / 4;
    const int rlo = max(0, a - x), rhi = min(KB - 1, H - 1 - x + a);
    const uint32_t rows_ok = ((2u << rhi) - 1u) & ~((1u << rlo) - 1u);
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
    return pull_box_fixed<KB, T, TG>(rec, rq, gp, gq, rows_ok, keep);
}

// KB > 0: the box of a KB x KB window with one-byte records, unrolled (one kernel per size keeps each
// one's code small); KB == 0: any window, walked generically.  With `bulk`, grad_output and the records
// of each staged row arrive by one bulk copy each (rows 16-byte aligned: the host checks pointers and W).
// T is the arithmetic (the sums run as the reference adds in T); grad_output is read as TG and grad_input
// written as TO, by default T: with TG = float16 / bfloat16 and T = float, grad_output is widened on load
// (exactly) and each sum rounded to TO once at its store, which equals casting grad_output to float,
// gathering in float and casting the result.
// Registers capped for nine CTAs per SM, as many as the 15 x 15 float32 tile's shared memory allows (the
// headline gather: 1.86 ms per launch against 1.89 at eight).
template <typename T, typename I, int KB, typename TG = T, typename TO = T>
__global__ void __launch_bounds__(kSumThreads, 9) pull_sum_kernel(const TG* __restrict__ go, const I* __restrict__ win,
                                                               const uint32_t* __restrict__ map,
                                                               TO* __restrict__ gi, int H, int W, int kH, int kW,
                                                               int border, int tiles_x, int tiles_y, int go_vec,
                                                               int rec_vec, int out_vec, int bulk) {
    static_assert(KB == 0 || sizeof(I) == 1, "the unrolled box reads one-byte records");
    using G = typename GradAcc<T>::type;
    constexpr int TP = kSumTP, TQ = kPullTQ, NT = kSumThreads, NWORDS = TP * TQ / 32;
    constexpr uint32_t kNone = IndexTraits<I>::none;
    const SumGeom geo(kH, kW, sizeof(TG), sizeof(I));
    const int aH = geo.aH, aW = geo.aW, hq = geo.hq, gv = geo.gv, goff = geo.goff, gq = geo.gq;
    const int rv = geo.rv, roff = geo.roff, rq = geo.rq;
    const int S = 2 * aW + 1;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TG* goS = reinterpret_cast<TG*>(smem_raw);                                        // [hr][gq]
    I* recS = reinterpret_cast<I*>(smem_raw + geo.go_b);                              // [hr][rq]
    uint16_t* listS = reinterpret_cast<uint16_t*>(smem_raw + geo.go_b + geo.rec_b);   // [TP * TQ]
    int* countS = reinterpret_cast<int*>(smem_raw + geo.go_b + geo.rec_b + geo.list_b);

    const long long b = blockIdx.x;
    const int tx = static_cast<int>(b % tiles_x);
    const int ty = static_cast<int>((b / tiles_x) % tiles_y);
    const long long plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    const int r0 = ty * TP, c0 = tx * TQ;
    const int tid = threadIdx.x, lane = tid & 31;
    const int WW = (W + 31) / 32;

    // the tile's target-map words: band row tid / 2, word tid % 2 (NWORDS == 64)
    uint32_t bits = 0;
    int wrow = 0, wcol = 0;
    if (tid < NWORDS) {
        wrow = r0 + tid / (TQ / 32);
        wcol = c0 / 32 + tid % (TQ / 32);
        if (wrow < H && wcol < WW) bits = map[(plane * H + wrow) * WW + wcol];
    }
    // the tile is zeroed first, in 16-byte stores; the winners' sums are stored over the zeros after the
    // barriers below (ordered within the CTA)
    TO* gip = gi + plane * H * W;
    {
        constexpr int OV = 16 / int(sizeof(TO));
        for (int i = tid; i < TP * TQ / OV; i += NT) {
            const int pr = i / (TQ / OV), pc = (i - pr * (TQ / OV)) * OV;
            const int r = r0 + pr, c = c0 + pc;
            if (r >= H || c >= W) continue;
            TO* dst = gip + static_cast<long long>(r) * W + c;
            if (out_vec && c + OV <= W) {
                *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
            } else {
                for (int e = 0; e < OV && c + e < W; ++e) dst[e] = Storage<TO>::store(0.0f);
            }
        }
    }
    if (!__syncthreads_or(bits != 0u)) return;  // no winner in the tile

    // stage grad_output and records of output rows [r0 - aH, r0 + TP + aH) inside the image
    const TG* gop = go + plane * H * W;
    const I* wp = win + plane * H * W;
    const int lo = max(0, r0 - aH), hi = min(H, r0 + TP + aH);
    __shared__ __align__(8) uint64_t bar;
    if (bulk) {
        // one bulk copy per row and array of the part inside the image; the columns outside it are filled
        const int gcol0 = c0 - aW - goff, rcol0 = c0 - aW - roff;  // 16-byte aligned in the image row
        const int gc_lo = max(gcol0, 0), gc_hi = min(gcol0 + gq, W);
        const int rc_lo = max(rcol0, 0), rc_hi = min(rcol0 + rq, W);
        const unsigned gbytes = static_cast<unsigned>(gc_hi - gc_lo) * sizeof(TG);
        const unsigned rbytes = static_cast<unsigned>(rc_hi - rc_lo) * sizeof(I);
        if (tid == 0) {
            mbar_init(&bar, 1);
            mbar_arrive_expect_tx(&bar, (gbytes + rbytes) * static_cast<unsigned>(hi - lo));
        }
        __syncthreads();
        for (int i = tid; i < 2 * (hi - lo); i += NT) {
            const int h = lo + (i >> 1), sr = h - (r0 - aH);
            if (i & 1)
                bulk_load(recS + sr * rq + (rc_lo - rcol0), wp + static_cast<long long>(h) * W + rc_lo, rbytes, &bar);
            else
                bulk_load(goS + sr * gq + (gc_lo - gcol0), gop + static_cast<long long>(h) * W + gc_lo, gbytes, &bar);
        }
        if (gc_lo > gcol0 || gc_hi < gcol0 + gq || rc_lo > rcol0 || rc_hi < rcol0 + rq) {
            const int gpad = gq - (gc_hi - gc_lo), rpad = rq - (rc_hi - rc_lo);
            for (int i = tid; i < (hi - lo) * gpad; i += NT) {
                const int sr = lo + i / gpad - (r0 - aH), q = i % gpad;
                const int col = q < gc_lo - gcol0 ? q : gc_hi - gcol0 + (q - (gc_lo - gcol0));
                goS[sr * gq + col] = Storage<TG>::store(0.0f);
            }
            for (int i = tid; i < (hi - lo) * rpad; i += NT) {
                const int sr = lo + i / rpad - (r0 - aH), q = i % rpad;
                const int col = q < rc_lo - rcol0 ? q : rc_hi - rcol0 + (q - (rc_lo - rcol0));
                recS[sr * rq + col] = static_cast<I>(kNone);
            }
        }
    } else {
        const int nchg = gq / gv, nchr = rq / rv;
        const uint32_t mg = static_cast<uint32_t>(((1ull << 32) + nchg - 1) / nchg);  // i < 2^16: exact
        const uint32_t mr = static_cast<uint32_t>(((1ull << 32) + nchr - 1) / nchr);
        for (int i = tid; i < (hi - lo) * nchg; i += NT) {
            const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), mg)), k = i - r * nchg;
            const int h = lo + r, col = c0 - aW - goff + k * gv;
            TG* dst = goS + (h - (r0 - aH)) * gq + k * gv;
            const TG* src = gop + static_cast<long long>(h) * W + col;
            if (go_vec && col >= 0 && col + gv <= W) {
                pg_cp_async16(dst, src);
            } else {
                for (int e = 0; e < gv; ++e) dst[e] = (col + e >= 0 && col + e < W) ? src[e] : Storage<TG>::store(0.0f);
            }
        }
        for (int i = tid; i < (hi - lo) * nchr; i += NT) {
            const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), mr)), k = i - r * nchr;
            const int h = lo + r, col = c0 - aW - roff + k * rv;
            I* dst = recS + (h - (r0 - aH)) * rq + k * rv;
            const I* src = wp + static_cast<long long>(h) * W + col;
            if (rec_vec && col >= 0 && col + rv <= W) {
                pg_cp_async16(dst, src);
            } else {
                for (int e = 0; e < rv; ++e) dst[e] = (col + e >= 0 && col + e < W) ? src[e] : static_cast<I>(kNone);
            }
        }
        pg_commit();
    }

    // list the tile's winners as (row - r0) * TQ + (column - c0)
    if (tid == 0) *countS = 0;
    __syncthreads();
    if (tid < NWORDS) {  // the first two warps
        const int cnt = __popc(bits);
        int incl = cnt;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += o;
        }
        int base = 0;
        if (lane == 31) base = atomicAdd(countS, incl);
        base = __shfl_sync(0xffffffffu, base, 31);
        int pos = base + incl - cnt;
        const int pbase = (wrow - r0) * TQ + (wcol * 32 - c0);
        for (uint32_t m = bits; m; m &= m - 1) listS[pos++] = static_cast<uint16_t>(pbase + __ffs(m) - 1);
    }
    if (bulk) {
        // a byte count that never arrives ends the wait: the tile is poisoned (NaN) instead of hanging
        if (!__syncthreads_and(mbar_wait(&bar, 0))) {
            for (int i = tid; i < TP * TQ; i += NT) {
                const int r = r0 + i / TQ, c = c0 + i % TQ;
                if (r < H && c < W) gip[static_cast<long long>(r) * W + c] = Storage<TO>::store(__int_as_float(0x7fffffff));
            }
            return;
        }
    } else {
        pg_wait_all();
        __syncthreads();
    }

    // records become box taps: (dr + aH) * S + (dc + aW) of the pixel each output selects.  An odd window's
    // record already is one unless a border folds its target, which only happens near the image edge.
    const bool folds = r0 - 2 * aH < 0 || r0 + TP + 2 * aH > H || c0 - 2 * aW < 0 || c0 + TQ + 2 * aW > W;
    if (folds || !(kW & 1)) {
        const uint32_t kw_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;
        auto convert = [&](int h, int lw) {
            const int w = c0 - aW + lw;
            if (static_cast<unsigned>(w) >= static_cast<unsigned>(W)) return;
            I& rec = recS[(h - (r0 - aH)) * rq + roff + lw];
            int x, y;
            if (!pg_target(rec, kNone, h, w, H, W, kW, aH, aW, border, kw_magic, x, y))
                rec = static_cast<I>(kNone);
            else
                rec = static_cast<I>((x - h + aH) * S + (y - w + aW));
        };
        if (!(kW & 1)) {
            const uint32_t mq = static_cast<uint32_t>(((1ull << 32) + hq - 1) / hq);
            for (int i = tid; i < (hi - lo) * hq; i += NT) {
                const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), mq));
                convert(lo + r, i - r * hq);
            }
        } else {
            // an odd window inside the image selects a pixel inside it, and its record already is its box
            // tap: only the outputs within the window's half-width of an image edge are converted.  Rows
            // [lo, e0) and [e1, hi) in full; the other rows' first and last columns.
            const int e0 = min(hi, max(lo, aH)), e1 = max(e0, min(hi, H - aH));
            const int edge_rows = (e0 - lo) + (hi - e1);
            const int lw_l1 = max(0, min(hq, 2 * aW - c0));        // columns w < aW: lw < 2aW - c0
            const int lw_r0 = max(lw_l1, min(hq, W - c0));         // columns w >= W - aW: lw >= W - c0
            const int side = lw_l1 + (hq - lw_r0);
            for (int i = tid; i < edge_rows * hq; i += NT) {
                const int r = i / hq, lw = i - r * hq;
                convert(r < e0 - lo ? lo + r : e1 + r - (e0 - lo), lw);
            }
            if (side > 0)
                for (int i = tid; i < (e1 - e0) * side; i += NT) {
                    const int r = i / side, k = i - r * side;
                    convert(e0 + r, k < lw_l1 ? k : lw_r0 + (k - lw_l1));
                }
        }
        __syncthreads();
    }

    // one thread per winner: the outputs of its box, in raster order
    const int n = *countS;
    for (int k = tid; k < n; k += NT) {
        const int p = listS[k];
        const int pr = p / TQ, pc = p - pr * TQ;  // box rows pr .. pr + 2aH, columns pc .. pc + 2aW (staged)
        const int x = r0 + pr, y = c0 + pc;
        G acc = G(0);
        if constexpr (KB > 0) {
            const uint8_t* rec = reinterpret_cast<const uint8_t*>(recS) + pr * rq + roff + pc;
            const TG* gp = goS + pr * gq + goff + pc;
            acc = pull_box_fixed_clip<KB, T, TG>(rec, rq, gp, gq, x, y, H, W);
        } else {
            for (int h = max(0, x - aH); h <= min(H - 1, x + aH); ++h) {
                const int lh = h - (r0 - aH);
                const int jlo = max(0, aW - y), jhi = min(2 * aW, W - 1 - y + aW);
                const I* trow = recS + lh * rq + roff + pc;  // box column j at trow[j]
                const TG* grow = goS + lh * gq + goff + pc;
                const int e0 = (x - h + aH) * S + 2 * aW;     // tap selecting (x, y) from box column 0
                for (int j = jlo; j <= jhi; ++j)
                    if (static_cast<int>(trow[j]) == e0 - j)
                        acc = GradAcc<T>::add(acc, static_cast<G>(Storage<TG>::load(grow[j])));
            }
        }
        gip[static_cast<long long>(x) * W + y] = Storage<TO>::store(static_cast<typename Storage<TO>::acc>(acc));
    }
}

// The box taps of a (kH, kW) window, and the "none" record, fit in a record of `idx` bytes.
inline bool pull_taps_fit(long long kH, long long kW, int idx) {
    const long long box = (2 * (kH / 2) + 1) * (2 * (kW / 2) + 1);
    return idx >= 4 ? box < 0xffffffffll : box < (1ll << (8 * idx)) - 1;
}

}  // namespace serron
