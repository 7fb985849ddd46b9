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
#pragma once

#include "common.cuh"

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
    static constexpr int QCAP = 32 * K;  // winner-cell queue of a warp: one task's pushes at most
    static constexpr size_t QUEUE_BYTES = size_t(kSweepThreads / 32) * QCAP * 2;
    // the queues live in the step's staging buffer, dead once its row pass is done, where they fit
    static constexpr bool QUEUE_IN_STAGE = XS_BYTES >= QUEUE_BYTES;
    static constexpr size_t fwd_smem() { return RD_END + (QUEUE_IN_STAGE ? 0 : QUEUE_BYTES); }
};

// One run of K windows [m, m+K-1], m = 0..K-1, over samples v[0..2K-2]: value and first-extremum
// offset (window-relative) of each.  Ties keep the lower offset.
template <int K, int OP, bool IDX, typename Emit>
__device__ __forceinline__ void sweep_run(const float (&v)[2 * K - 1], Emit emit) {
    float sv[K];
    int si[K];
    sv[K - 1] = v[K - 1];
    si[K - 1] = K - 1;
#pragma unroll
    for (int m = K - 2; m >= 0; --m) {
        const bool take = Op<OP>::better(sv[m + 1], v[m]);
        sv[m] = take ? sv[m + 1] : v[m];
        si[m] = IDX ? (take ? si[m + 1] : m) : 0;
    }
    emit(0, sv[0], si[0]);
    float pv = 0.0f;
    int pi = 0;
#pragma unroll
    for (int m = 1; m < K; ++m) {
        const float xv = v[K + m - 1];
        if (m == 1) {
            pv = xv;
            pi = K;
        } else {
            const bool take = Op<OP>::better(xv, pv);
            pv = take ? xv : pv;
            pi = IDX ? (take ? K + m - 1 : pi) : 0;
        }
        const bool take = Op<OP>::better(pv, sv[m]);
        emit(m, take ? pv : sv[m], take ? pi - m : si[m] - m);
    }
}

template <typename T>
__device__ __forceinline__ float load_clean(T v, float neutral) {
    const float f = Storage<T>::load(v);
    return f != f ? neutral : f;  // NaN never wins: staged as the neutral element
}

// With `map` (records only), every winner is also set in the target map of the gather (one bit per
// pixel, rows of ceil(W / 32) words, zero on entry).  In the column pass a lane whose winning row
// result differs from the one of the output above pushes it to its warp's queue (ballot + popc: only
// the few changes take a slot); the warp then decodes its queue densely into winner pixels and ORs
// each into the map, skipping one equal to its queue neighbour's.
template <typename T, int OP, typename I, bool WITH_VALUE, bool WITH_INDEX, int K>
__global__ void __launch_bounds__(kSweepThreads, (K <= 15 ? 4 : 1)) sep_sweep_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                                      I* __restrict__ win, uint32_t* __restrict__ map,
                                                                      int H, int W, int border, int strips, int segs,
                                                                      int seg_h) {
    static_assert(K <= 255, "dj is a byte");
    using G = SweepGeom<K, sizeof(T)>;
    constexpr int a = G::a, TH = G::TH, Cc = G::Cc, XS = G::XS, RS = G::RS;
    constexpr bool ASYNC = sizeof(T) == 4;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* const xsb0 = reinterpret_cast<T*>(smem_raw);
    T* const xsb1 = reinterpret_cast<T*>(smem_raw + G::XS_BYTES);
    float* rv = reinterpret_cast<float*>(smem_raw + 2 * G::XS_BYTES);   // [RR][RS]
    uint8_t* rdj = reinterpret_cast<uint8_t*>(rv + G::RR * RS);         // [RR][RS]
    uint16_t* const queue_own = reinterpret_cast<uint16_t*>(smem_raw + G::RD_END) + (threadIdx.x >> 5) * G::QCAP;

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
                for (int q = lane; q < Cc; q += 32) dst[q] = neutral_t;
                continue;
            }
            const T* row = xp + static_cast<long long>(gr) * W;
            if (cols_inside) {
                const T* src = row + (ow0 - a);
                for (int q = lane; q < Cc; q += 32) {
                    if constexpr (ASYNC)
                        cp_async4(dst + q, src + q);
                    else
                        dst[q] = src[q];
                }
            } else {
                for (int q = lane; q < Cc; q += 32) {
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
    // row pass over buffer rows [0, nrows) -> row results rows [dst0, dst0 + nrows); every chunk is
    // whole (the padding columns hold the neutral element), so no bounds checks
    auto row_pass = [&](const T* buf, int nrows, int dst0) {
        for (int task = tid; task < G::NCR * nrows; task += kSweepThreads) {
            const int c = task / nrows, r = task - c * nrows;
            const T* src = buf + r * XS + c * K;
            float v[2 * K - 1];
#pragma unroll
            for (int m = 0; m < 2 * K - 1; ++m) v[m] = load_clean(src[m], neutral);
            float* rvr = rv + (dst0 + r) * RS + c * K;
            uint8_t* rdr = rdj + (dst0 + r) * RS + c * K;
            sweep_run<K, OP, true>(v, [&](int m, float val, int off) {
                rvr[m] = val;
                rdr[m] = static_cast<uint8_t>(off);
            });
        }
    };

    // the padding columns of both staging buffers are never staged: neutral once (and again after a step
    // whose winner queues lived in the buffer)
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
    row_pass(xsb0, K - 1, 0);

    int step = 0;
    for (int s0 = oh_begin; s0 < oh_end; s0 += TH, ++step) {
        T* cur = (step & 1) ? xsb0 : xsb1;
        T* nxt = (step & 1) ? xsb1 : xsb0;
        // (the next step's rows go to nxt, and cur is restaged only two steps on, after barriers)
        uint16_t* const queue =
            G::QUEUE_IN_STAGE ? reinterpret_cast<uint16_t*>(cur) + (threadIdx.x >> 5) * G::QCAP : queue_own;
        __syncthreads();  // nxt is no longer read
        if constexpr (ASYNC) {
            if (s0 + TH < oh_end) stage(nxt, s0 + TH - a + K - 1, TH);
            cp_async_commit();
            cp_async_wait_all_but_one();
        } else if (step > 0) {
            stage(cur, s0 - a + K - 1, TH);
        }
        __syncthreads();
        row_pass(cur, TH, K - 1);
        __syncthreads();

        // column pass: output row s0 + i uses row results [i, i + K - 1]
        const int rows_left = oh_end - s0;  // >= TH except in a segment's last step
        // (the task count is a multiple of 32, so every warp runs whole: lanes past the image edge stay in
        // the loop with nothing to write, and the winner de-duplication below can shuffle across the warp)
        for (int task = tid; task < G::NCC * kSweepTW; task += kSweepThreads) {
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
            int qn = 0, prev = -1;  // queue length (warp-uniform), this lane's last pushed row result
            sweep_run<K, OP, WITH_INDEX>(v, [&](int m, float val, int off) {
                const bool out_ok = col_ok && base + m < rows_left;
                const int o = o0 + m * W;
                if (WITH_VALUE && out_ok) yp[o] = Storage<T>::store(val);
                if (WITH_INDEX && out_ok) {
                    // winning row base + m + off, and the column its own row pass chose
                    const uint32_t djb = dj_col[(m + off) * RS];
                    wp[o] = static_cast<I>(val == neutral ? IndexTraits<I>::none : static_cast<uint32_t>(off * K) + djb);
                }
                if (marking) {
                    const int cell = out_ok && val != neutral ? base + m + off : -1;
                    const bool push = cell >= 0 && cell != prev;
                    prev = cell;
                    const unsigned bal = __ballot_sync(0xffffffffu, push);
                    if (push) queue[qn + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(cell * kSweepTW + j);
                    qn += __popc(bal);
                }
            });
            if (marking) {
                // the queued row results' winners (row s0 - a + i, column ow0 + j - a + dj, border folded)
                __syncwarp();
                for (int q0 = 0; q0 < qn; q0 += 32) {
                    int key = -1, wx = 0, wy = 0;
                    if (q0 + lane < qn) {
                        const int e = queue[q0 + lane];
                        const int i = e / kSweepTW, jj = e - i * kSweepTW;
                        wx = s0 - a + i;
                        wy = ow0 + jj - a + static_cast<int>(rdj[i * RS + jj]);
                        if ((static_cast<unsigned>(wx) < static_cast<unsigned>(H) || resolve(wx, H, border)) &&
                            (static_cast<unsigned>(wy) < static_cast<unsigned>(W) || resolve(wy, W, border)))
                            key = wx * W + wy;  // < H * W < 2^31
                    }
                    const int left = __shfl_up_sync(0xffffffffu, key, 1);
                    if (key >= 0 && (lane == 0 || left != key))
                        atomicOr(&map[(plane * H + wx) * WW + (wy >> 5)], 1u << (wy & 31));
                }
                __syncwarp();  // the queue is refilled by the warp's next task
            }
        }
        __syncthreads();
        // the queues overwrote cur: its padding columns back to neutral before its next row pass
        if (G::QUEUE_IN_STAGE && marking)
            for (int i = tid; i < TH * (XS - Cc); i += kSweepThreads)
                cur[(i / (XS - Cc)) * XS + Cc + i % (XS - Cc)] = neutral_t;
        // carry the last K-1 row results to the top
        for (int i = tid; i < (K - 1) * RS; i += kSweepThreads) {
            rv[i] = rv[TH * RS + i];
            rdj[i] = rdj[TH * RS + i];
        }
    }
    if constexpr (ASYNC) cp_async_wait_all();
}

}  // namespace serron
