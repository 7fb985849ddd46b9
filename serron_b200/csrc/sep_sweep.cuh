// Separable flat-square forward with the window length K known at compile time: the forward kernel
// of the flat structuring-element workloads.  Results are bit-identical to separable.cuh.
//
// The kernel sweeps: a CTA owns a 64-column strip of one plane (or a row segment of it) and walks it
// downwards in steps of TH output rows (a multiple of K), carrying the last K-1 row results from one
// step to the next, so every image row is staged and row-scanned once; the rows of the next step are
// prefetched with cp.async while the current step computes.
//   row pass     one thread per (row, K-chunk): 2K-1 samples in registers, a suffix arg-scan over the
//                chunk, a prefix arg-scan over the next chunk, one compare-select per output to combine
//                (van Herk / Gil-Werman: three compare-selects per output, any K);
//   column pass  the same over the row results.
// With a winner buffer every output gets the direct tap di * K + dj of its winner (di from the column
// pass, dj from the row pass of the winning row), the record the direct kernels write.
// Compare-selects keep the first extremum (the reference's tie rule).  A NaN sample never wins: a sample
// is taken only when it compares at least as good (suffix scan, towards lower offsets) or strictly better
// (prefix scan) than the running best, which starts at the neutral element, and a compare with a NaN is
// false.  Three CTAs per SM (80 registers: no spills).
#pragma once

#include "common.cuh"

#include <type_traits>

namespace serron {

constexpr int kSweepTW = 64;      // strip width (output / pixel columns)
constexpr int kSweepThreads = 256;

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all_but_one() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

constexpr int kSweepMarkPitch = 128;  // mark bytes per buffer row: image columns [ow0 - 32, ow0 + 96)

template <int K, int ELEM>
struct SweepGeom {
    static constexpr int a = K / 2;
    static constexpr int TH = K * ((32 + K - 1) / K);   // output rows per forward step
    static constexpr int Cc = kSweepTW + K - 1;          // staged input columns
    static constexpr int NCR = (kSweepTW + K - 1) / K;   // row-pass chunks per row
    // pitches padded so every row-pass chunk reads and writes whole chunks without bounds checks;
    // odd so that threads on consecutive rows hit distinct banks
    static constexpr int XS = (NCR * K + K - 1) | 1;     // staged-sample pitch (columns >= Cc: neutral)
    static constexpr int RS = (NCR * K) | 1;             // row-result pitch
    static constexpr int RR = TH + K - 1;                // row-result rows: K-1 carried + TH new
    static constexpr int NCC = TH / K;                   // column-pass chunks per column
    static constexpr size_t XS_BYTES = ((size_t(TH) * XS * ELEM + 15) / 16) * 16;
    static constexpr size_t RD_END = ((2 * XS_BYTES + size_t(RR) * RS * 4 + size_t(RR) * RS) + 15) / 16 * 16;
    // winner marks of one step, a byte per pixel of the buffer rows; they live in the step's staging
    // buffer, dead once its row pass is done, where they fit
    static constexpr size_t MARK_BYTES = size_t(RR) * kSweepMarkPitch;
    static constexpr bool MARK_IN_STAGE = XS_BYTES >= MARK_BYTES;
    static constexpr int MARK_ROWS_IN_STAGE = int((MARK_BYTES + size_t(XS) * ELEM - 1) / (size_t(XS) * ELEM));
    static constexpr size_t fwd_smem() { return RD_END + (MARK_IN_STAGE ? 0 : MARK_BYTES); }
};

// One run of K windows [m, m+K-1], m = 0..K-1, over samples v[0..2K-2]: value and first-extremum
// offset (window-relative) of each.  Ties keep the lower offset; a window of NaNs only yields the neutral
// element (its offset is then meaningless: such outputs get the "none" record).
template <int K, int OP, bool IDX, typename Emit>
__device__ __forceinline__ void sweep_run(const float (&v)[2 * K - 1], Emit emit) {
    const float neutral = Op<OP>::template neutral<float>();
    float sv[K];
    int si[K];
    float cv = neutral;
    int ci = K - 1;
#pragma unroll
    for (int m = K - 1; m >= 0; --m) {
        const bool take = Op<OP>::better_eq(v[m], cv);
        cv = take ? v[m] : cv;
        if (IDX) ci = take ? m : ci;
        sv[m] = cv;
        si[m] = ci;
    }
    emit(0, sv[0], si[0]);
    float pv = neutral;
    int pi = K;
#pragma unroll
    for (int m = 1; m < K; ++m) {
        const float xv = v[K + m - 1];
        const bool tk = Op<OP>::better(xv, pv);
        pv = tk ? xv : pv;
        if (IDX) pi = tk ? K + m - 1 : pi;
        const bool take = Op<OP>::better(pv, sv[m]);
        emit(m, take ? pv : sv[m], (take ? pi : si[m]) - m);
    }
}

// 32 mark bytes (each 0 or 1) as the bits of one word, byte i -> bit i.
__device__ __forceinline__ uint32_t pack_marks(uint4 lo, uint4 hi) {
    const uint32_t q[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint32_t bits = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) bits |= ((q[e] | (q[e] >> 7) | (q[e] >> 14) | (q[e] >> 21)) & 0xfu) << (4 * e);
    return bits;
}

// With `map` (records only), every winner is also set in the target map of the gather (one bit per
// pixel, rows of ceil(W / 32) words, zero on entry).  The column pass marks the winning pixel of each
// output with a byte in a step-local window of the buffer rows (image columns [ow0 - 32, ow0 + 96));
// after the pass, each 32-byte run of marks leaves as one word ORed into the map (words across the image
// edge bit by bit, through the border's folding).
template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX, int K>
__global__ void __launch_bounds__(kSweepThreads, (K <= 15 ? 3 : 1)) sep_sweep_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                                      I* __restrict__ win, uint32_t* __restrict__ map,
                                                                      int H, int W, int border, int strips, int segs,
                                                                      int seg_h) {
    static_assert(K <= 255, "dj is a byte");
    using G = SweepGeom<K, sizeof(T)>;
    constexpr int a = G::a, TH = G::TH, Cc = G::Cc, XS = G::XS, RS = G::RS, NCR = G::NCR, NCC = G::NCC;
    constexpr int RR = G::RR, MP = kSweepMarkPitch;
    constexpr bool ASYNC = sizeof(T) == 4;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* const xsb0 = reinterpret_cast<T*>(smem_raw);
    T* const xsb1 = reinterpret_cast<T*>(smem_raw + G::XS_BYTES);
    float* rv = reinterpret_cast<float*>(smem_raw + 2 * G::XS_BYTES);   // [RR][RS]
    uint8_t* rdj = reinterpret_cast<uint8_t*>(rv + RR * RS);             // [RR][RS]

    const long long b = blockIdx.x;
    const int strip = static_cast<int>(b % strips);
    const int seg = static_cast<int>((b / strips) % segs);
    const long long plane = b / (static_cast<long long>(strips) * segs);
    const int ow0 = strip * kSweepTW;
    const int oh_begin = seg * seg_h, oh_end = min(H, oh_begin + seg_h);
    const T* xp = x + plane * H * W;
    const int tid = threadIdx.x;
    const float neutral = Op<OP>::template neutral<float>();
    const T neutral_t = Storage<T>::store(neutral);
    const bool cols_inside = ow0 - a >= 0 && ow0 - a + Cc <= W;

    const int warp = tid >> 5, lane = tid & 31;
    const bool marking = WITH_INDEX && map != nullptr;
    const int WW = (W + 31) / 32;

    // rows [r0, r0 + nrows) of the image (unresolved) -> buffer rows [0, nrows); one warp per row
    auto stage = [&](T* buf, int r0, int nrows) {
        for (int r = warp; r < nrows; r += kSweepThreads / 32) {
            int gr = r0 + r;
            T* dst = buf + r * XS;
            if (!resolve(gr, H, border)) {  // a CONSTANT row outside the image: all neutral
#pragma unroll
                for (int q0 = 0; q0 < Cc; q0 += 32)
                    if (q0 + lane < Cc) dst[q0 + lane] = neutral_t;
                continue;
            }
            const T* row = xp + static_cast<long long>(gr) * W;
            if (cols_inside) {
                const T* src = row + (ow0 - a);
#pragma unroll
                for (int q0 = 0; q0 < Cc; q0 += 32) {
                    const int q = q0 + lane;
                    if (q < Cc) {
                        if constexpr (ASYNC)
                            cp_async4(dst + q, src + q);
                        else
                            dst[q] = src[q];
                    }
                }
            } else {
#pragma unroll
                for (int q0 = 0; q0 < Cc; q0 += 32) {
                    const int q = q0 + lane;
                    if (q >= Cc) continue;
                    int gq = ow0 - a + q;
                    if (resolve(gq, W, border)) {
                        if constexpr (ASYNC)
                            cp_async4(dst + q, row + gq);
                        else
                            dst[q] = row[gq];
                    } else {
                        dst[q] = neutral_t;
                    }
                }
            }
        }
    };
    // row pass over buffer rows [0, NR) -> row results rows [dst0, dst0 + NR); every chunk is whole (the
    // padding columns hold the neutral element), so no bounds checks
    auto row_pass = [&](const T* buf, int dst0, auto nr) {
        constexpr int NR = decltype(nr)::value;
#pragma unroll 1
        for (int task = tid; task < NCR * NR; task += kSweepThreads) {
            const int c = task / NR, r = task - c * NR;
            const T* src = buf + r * XS + c * K;
            float v[2 * K - 1];
#pragma unroll
            for (int m = 0; m < 2 * K - 1; ++m) v[m] = Storage<T>::load(src[m]);
            float* rvr = rv + (dst0 + r) * RS + c * K;
            uint8_t* rdr = rdj + (dst0 + r) * RS + c * K;
            sweep_run<K, OP, true>(v, [&](int m, float val, int off) {
                rvr[m] = val;
                rdr[m] = static_cast<uint8_t>(off);
            });
        }
    };

    // the padding columns of both staging buffers are never staged: neutral once (and again after a step
    // whose marks lived in the buffer)
    for (int i = tid; i < 2 * TH * (XS - Cc); i += kSweepThreads) {
        const int r = i / (XS - Cc), q = Cc + i % (XS - Cc);
        (r < TH ? xsb0 : xsb1)[(r % TH) * XS + q] = neutral_t;
    }

    // prologue: the K-1 rows above the first output row's window end
    stage(xsb0, oh_begin - a, K - 1);
    if constexpr (ASYNC) cp_async_commit();
    stage(xsb1, oh_begin - a + K - 1, TH);  // the first step's new rows
    if constexpr (ASYNC) {
        cp_async_commit();
        cp_async_wait_all_but_one();
    }
    __syncthreads();
    row_pass(xsb0, 0, std::integral_constant<int, K - 1>{});

    int step = 0;
    for (int s0 = oh_begin; s0 < oh_end; s0 += TH, ++step) {
        T* cur = (step & 1) ? xsb0 : xsb1;
        T* nxt = (step & 1) ? xsb1 : xsb0;
        // (the next step's rows go to nxt, and cur is restaged only two steps on, after barriers)
        uint8_t* const marks =
            G::MARK_IN_STAGE ? reinterpret_cast<uint8_t*>(cur) : smem_raw + G::RD_END;  // [RR][MP]
        __syncthreads();  // nxt is no longer read
        if constexpr (ASYNC) {
            if (s0 + TH < oh_end) stage(nxt, s0 + TH - a + K - 1, TH);
            cp_async_commit();
            cp_async_wait_all_but_one();
        } else if (step > 0) {
            stage(cur, s0 - a + K - 1, TH);
        }
        __syncthreads();
        row_pass(cur, K - 1, std::integral_constant<int, TH>{});
        __syncthreads();
        if (marking) {  // cur is dead: its bytes become this step's marks
            for (int i = tid; i < int(G::MARK_BYTES / 16); i += kSweepThreads)
                reinterpret_cast<uint4*>(marks)[i] = make_uint4(0, 0, 0, 0);
            __syncthreads();
        }

        // column pass: output row s0 + i uses row results [i, i + K - 1]
        const int rows_left = oh_end - s0;  // >= TH except in a segment's last step
#pragma unroll 1
        for (int task = tid; task < NCC * kSweepTW; task += kSweepThreads) {
            const int c = task / kSweepTW, j = task - c * kSweepTW;
            const int base = c * K;
            const int ow = ow0 + j;
            const bool col_ok = ow < W;
            float v[2 * K - 1];
#pragma unroll
            for (int m = 0; m < 2 * K - 1; ++m) v[m] = rv[(base + m) * RS + j];
            // offsets within the plane fit in 32 bits, rows up to TH past the image included
            // ((H + 64) * (W + 64) < 2^31 is checked on the host)
            const int o0 = (s0 + base) * W + ow;
            T* yp = y + plane * H * W;
            I* wp = win + plane * H * W;
            const uint8_t* dj_col = rdj + base * RS + j;
            uint8_t* mark_col = marks + base * MP + (32 - a) + j;
            sweep_run<K, OP, WITH_INDEX>(v, [&](int m, float val, int off) {
                const bool out_ok = col_ok && base + m < rows_left;
                const int o = o0 + m * W;
                if (WITH_VALUE && out_ok) yp[o] = Storage<T>::store(val);
                if (WITH_INDEX && out_ok) {
                    // winning row base + m + off, and the column its own row pass chose
                    const uint32_t djb = dj_col[(m + off) * RS];
                    const bool none = val == neutral;
                    wp[o] = static_cast<I>(none ? IndexTraits<I>::none : static_cast<uint32_t>(off * K) + djb);
                    if (marking && !none) mark_col[(m + off) * MP + djb] = 1;
                }
            });
        }
        __syncthreads();
        if (marking) {
            // the marks of buffer rows (image rows s0 - a + i) leave as map words; words and rows inside
            // the image whole, the others bit by bit through the border's folding.  Rows a later step
            // marks again (the carried ones) are ORed again then.
            const long long map_plane = plane * H;
#pragma unroll 1
            for (int t = tid; t < RR * (MP / 32); t += kSweepThreads) {
                const int i = t / (MP / 32), k = t - i * (MP / 32);
                const uint4* src = reinterpret_cast<const uint4*>(marks + i * MP + 32 * k);
                const uint32_t bits = pack_marks(src[0], src[1]);
                if (bits == 0u) continue;
                const int gr = s0 - a + i, gc0 = ow0 - 32 + 32 * k;
                if (gr >= 0 && gr < H && gc0 >= 0 && gc0 + 32 <= W) {
                    atomicOr(&map[(map_plane + gr) * WW + (gc0 >> 5)], bits);
                } else {
                    for (uint32_t m = bits; m; m &= m - 1) {
                        int r = gr, cc = gc0 + __ffs(m) - 1;
                        if (resolve(r, H, border) && resolve(cc, W, border))
                            atomicOr(&map[(map_plane + r) * WW + (cc >> 5)], 1u << (cc & 31));
                    }
                }
            }
            // the marks overwrote cur's padding columns: neutral again before its next row pass (once
            // every mark is read)
            if constexpr (G::MARK_IN_STAGE) {
                __syncthreads();
                for (int i = tid; i < G::MARK_ROWS_IN_STAGE * (XS - Cc); i += kSweepThreads)
                    cur[(i / (XS - Cc)) * XS + Cc + i % (XS - Cc)] = neutral_t;
            }
        }
        // carry the last K-1 row results to the top
        for (int i = tid; i < (K - 1) * RS; i += kSweepThreads) {
            rv[i] = rv[TH * RS + i];
            rdj[i] = rdj[TH * RS + i];
        }
    }
    if constexpr (ASYNC) cp_async_wait_all();
}

}  // namespace serron
