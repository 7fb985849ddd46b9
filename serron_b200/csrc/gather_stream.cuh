// grad_input by a raster-order stream: the atomic-free gather for any winner encoding.
//
// The reference forms grad_input[p] by adding grad_output of every output whose winner is p, in
// output raster order, in the storage type's arithmetic (csrc/cpu/morphology/backward.cpp:250-263).
// This kernel reproduces exactly that order with each output visited once:
//
// * one warp (one CTA) owns a strip of kStreamTW pixel columns of one plane and a segment of its rows,
//   and walks the output rows that can reach them (aH above to aH below the segment) top to bottom;
// * an output row is taken 32 columns at a time in ascending order; each lane decodes its output's
//   winner into a target pixel; lanes aiming at the same pixel form a group (warp match) whose lowest
//   lane adds the group's grad_output values to the pixel's accumulator in lane (= column) order;
// * accumulators live in a ring of 2aH+1 pixel rows: once output row oh is done, pixel row oh - aH can
//   receive nothing more (its outputs lie within aH rows), so it is written out and its slot reused;
// * output rows are prefetched kStreamPF rows ahead with cp.async (records and grad_output).
//
// Candidates are assumed to lie within a single border fold (aH / aW of the pixel); the host routes
// windows wider than the image under REFLECT to the generic kernels.
#pragma once

#include "common.cuh"

namespace serron {

constexpr int kStreamTW = 64;     // pixel columns per strip
constexpr int kStreamPF = 6;      // output rows prefetched ahead of the one being processed

__device__ __forceinline__ void sg_cp_async4(void* smem_dst, const void* gmem_src) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void sg_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void sg_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

struct StreamGeom {
    int aH, aW, gw, rrows, arows, gwb;
    __host__ __device__ StreamGeom(int kH, int kW, int idx_bytes)
        : aH(kH / 2), aW(kW / 2), gw(kStreamTW + 2 * (kW / 2)), rrows(2 * (kH / 2) + 1 + kStreamPF + 1),
          arows(2 * (kH / 2) + 1), gwb(0) {
        // record rows: a word-aligned superset of the halo columns (see record_offset)
        const int per_word = 4 / idx_bytes;
        gwb = ((gw + 3 + per_word - 1) / per_word) * per_word;
    }
    // byte size of each shared-memory region
    __host__ __device__ size_t go_bytes(size_t acc) const { return ((size_t(rrows) * gw * acc + 15) / 16) * 16; }
    __host__ __device__ size_t rec_bytes(size_t idx) const { return ((size_t(rrows) * gwb * idx + 15) / 16) * 16; }
    __host__ __device__ size_t acc_bytes(size_t acc) const { return size_t(arows) * kStreamTW * acc; }
    __host__ __device__ size_t smem(size_t acc, size_t idx) const {
        return go_bytes(acc) + rec_bytes(idx) + acc_bytes(acc);
    }
};

template <typename T, typename I, bool SEP>
__global__ void __launch_bounds__(32) stream_gather_kernel(const T* __restrict__ go, const I* __restrict__ win,
                                                           T* __restrict__ gi, int H, int W, int kH, int kW,
                                                           int border, int strips, int segs, int seg_h) {
    using G = typename GradAcc<T>::type;
    constexpr int PER_WORD = 4 / int(sizeof(I));
    const StreamGeom geo(kH, kW, sizeof(I));
    const int aH = geo.aH, aW = geo.aW, GW = geo.gw, RR = geo.rrows, AR = geo.arows, GWB = geo.gwb;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    G* gs = reinterpret_cast<G*>(smem_raw);                                                      // [RR][GW]
    I* rs = reinterpret_cast<I*>(smem_raw + geo.go_bytes(sizeof(G)));                            // [RR][GWB]
    G* acc = reinterpret_cast<G*>(smem_raw + geo.go_bytes(sizeof(G)) + geo.rec_bytes(sizeof(I))); // [AR][TW]

    const long long b = blockIdx.x;
    const int strip = static_cast<int>(b % strips);
    const int seg = static_cast<int>((b / strips) % segs);
    const long long plane = b / (static_cast<long long>(strips) * segs);
    const int pw0 = strip * kStreamTW;
    const int ph_begin = seg * seg_h, ph_end = min(H, ph_begin + seg_h);
    const T* gop = go + plane * H * W;
    const I* wp = win + plane * H * W;
    T* gip = gi + plane * H * W;
    const int lane = threadIdx.x;
    const I none_rec = SEP ? static_cast<I>(sep_none_hi<I>() << IndexTraits<I>::half_bits)
                           : static_cast<I>(IndexTraits<I>::none);
    // record row layout: element e holds image column rc0 + e, rc0 word-aligned so whole 4-byte words
    // can be copied; halo column q (image column pw0 - aW + q) sits at element roff + q
    const int rc0 = ((pw0 - aW) >= 0 ? (pw0 - aW) / PER_WORD : -((-(pw0 - aW) + PER_WORD - 1) / PER_WORD)) * PER_WORD;
    const int roff = (pw0 - aW) - rc0;
    const bool words_ok = (static_cast<long long>(W) * sizeof(I)) % 4 == 0;

    const int oh_first = ph_begin - aH, oh_last = ph_end - 1 + aH;  // output rows walked
    // ring slots advance with the row; wrap by a compare, never by a division
    auto wrap = [](int s, int n) { return s < 0 ? s + n : (s >= n ? s - n : s); };
    // stage output row oh into ring slot `slot` (rows outside the image: no winner, zero)
    auto stage = [&](int oh, int slot) {
        G* gdst = gs + slot * GW;
        I* rdst = rs + slot * GWB;
        const bool row_ok = oh >= 0 && oh < H;
        for (int q = lane; q < GW; q += 32) {
            const int ow = pw0 - aW + q;
            if (row_ok && ow >= 0 && ow < W) {
                const T* src = gop + static_cast<long long>(oh) * W + ow;
                if constexpr (sizeof(T) == 4)
                    sg_cp_async4(gdst + q, src);
                else
                    gdst[q] = static_cast<G>(Storage<T>::load(*src));
            } else {
                gdst[q] = G(0);
            }
        }
        for (int wd = lane; wd < GWB / PER_WORD; wd += 32) {
            const int c = rc0 + wd * PER_WORD;
            I* dst = rdst + wd * PER_WORD;
            if (row_ok && words_ok && c >= 0 && c + PER_WORD <= W) {
                sg_cp_async4(dst, wp + static_cast<long long>(oh) * W + c);
            } else {
#pragma unroll
                for (int e = 0; e < PER_WORD; ++e)
                    dst[e] = (row_ok && c + e >= 0 && c + e < W) ? wp[static_cast<long long>(oh) * W + c + e] : none_rec;
            }
        }
    };

    for (int i = lane; i < AR * kStreamTW; i += 32) acc[i] = G(0);
    // prologue: rows needed before the first one is processed (records reach aH rows below)
    int staged = oh_first - 1;  // last staged row
    const int ahead = aH + kStreamPF;  // < RR
    int slot = ((oh_first % RR) + RR) % RR;   // ring slot of row oh
    int aslot = ((oh_first % AR) + AR) % AR;  // accumulator slot of pixel row oh
    for (int r = oh_first; r <= min(oh_last, oh_first + ahead); ++r) {
        stage(r, wrap(slot + (r - oh_first), RR));
        sg_commit();
        staged = r;
    }
    // exact division of a record (< 2^16) by kW: multiply-high by ceil(2^32 / kW)
    const uint32_t div_magic = kW > 1 ? static_cast<uint32_t>(((1ull << 32) + kW - 1) / kW) : 0u;

    for (int oh = oh_first; oh <= oh_last; ++oh) {
        // keep the ring filled `ahead` rows past oh; rows up to oh + aH must have landed
        if (staged < oh_last && staged < oh + ahead) {
            ++staged;
            stage(staged, wrap(slot + (staged - oh), RR));
        }
        sg_commit();
        sg_wait<kStreamPF>();
        __syncwarp();

        const G* grow = gs + slot * GW;
        const I* rrow = rs + slot * GWB + roff;
        for (int q0 = 0; q0 < GW; q0 += 32) {
            const int q = q0 + lane;
            int key = -1;
            if (q < GW) {
                const uint32_t v = rrow[q];
                const int ow = pw0 - aW + q;
                int r = -1, c = -1;
                if (SEP) {
                    const uint32_t hi = sep_hi<I>(v);
                    if (hi != sep_none_hi<I>()) {
                        r = oh + static_cast<int>(hi) - aH;
                        if (resolve(r, H, border) && r >= ph_begin && r < ph_end) {
                            const int rslot = wrap(slot + (r - oh), RR);  // |r - oh| <= aH
                            c = ow + static_cast<int>(sep_lo<I>(rs[rslot * GWB + roff + q])) - aW;
                            if (!resolve(c, W, border)) r = -1;
                        } else {
                            r = -1;
                        }
                    }
                } else if (v != IndexTraits<I>::none) {
                    const uint32_t di = sizeof(I) <= 2 ? (kW > 1 ? __umulhi(v, div_magic) : v)
                                                       : v / static_cast<uint32_t>(kW);
                    r = oh + static_cast<int>(di) - aH;
                    c = ow + static_cast<int>(v - di * static_cast<uint32_t>(kW)) - aW;
                    if (!resolve(r, H, border) || !resolve(c, W, border) || r < ph_begin || r >= ph_end) r = -1;
                }
                if (r >= 0 && c >= pw0 && c < pw0 + kStreamTW) key = wrap(aslot + (r - oh), AR) * kStreamTW + (c - pw0);
            }
            const unsigned group = __match_any_sync(0xffffffffu, key);
            if (key >= 0 && lane == __ffs(group) - 1) {
                G a = acc[key];
                unsigned m = group;
                while (m) {
                    const int l = __ffs(m) - 1;
                    m &= m - 1;
                    a = GradAcc<T>::add(a, grow[q0 + l]);
                }
                acc[key] = a;
            }
            __syncwarp();
        }
        // pixel row oh - aH is complete: write it and free its slot
        const int done = oh - aH;
        if (done >= ph_begin && done < ph_end) {
            G* arow = acc + wrap(aslot - aH, AR) * kStreamTW;
            for (int c = lane; c < kStreamTW; c += 32) {
                if (pw0 + c < W)
                    gip[static_cast<long long>(done) * W + pw0 + c] =
                        Storage<T>::store(static_cast<typename Storage<T>::acc>(arow[c]));
                arow[c] = G(0);
            }
        }
        __syncwarp();
        slot = wrap(slot + 1, RR);
        aslot = wrap(aslot + 1, AR);
    }
    sg_wait<0>();
}

}  // namespace serron
