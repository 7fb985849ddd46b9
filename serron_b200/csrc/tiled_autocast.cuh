// Forward under CUDA autocast with the backward's winners in the same pass.
//
// Under torch.autocast("cuda") the reference casts serron::erode/dilate's arguments to float16
// (packages/serron/torch-ext/serron/_cmake_ops.py:175-189), so the forward value is the op on the
// float16 casts, while the backward works on the tensors the autograd function saved, promoted to their
// common dtype (float32 for a bfloat16 or float16 input and a float32 layer weight; autograd.py:37-76)
// and finds that dtype's winners again.  This kernel produces both at once for a compile-time odd
// K x K window: the float16 value of every output and the direct record (tap di * K + dj) of its
// float32 winner, with the gather's target map, so the backward only gathers.
//
//   value    min (max) over taps of h(x) - h(w) (h(x) + h(w)) in half2 arithmetic, two adjacent outputs
//            per instruction (__hsub2/__hmin2 or __hadd2/__hmax2).  The reference computes each tap in
//            float and rounds the extremum to half once; rounding is monotone and a float difference of
//            two halves rounds to half exactly as the half difference does (24 >= 2 * 11 + 2 bits), so the
//            results agree bit for bit.  NaN taps never win (the half2 min/max returns the other value);
//            the neutral element stays when nothing else is there.
//   winner   the first strict improvement in (di, dj) order of float(x) -/+ w in float32; a thread notes
//            whether any tap of its outputs compared equal to a running best, and then settles its
//            outputs' windows in double, as the reference CPU compares (exact weights need neither).
//
// A CTA computes a 32 x 64 output tile, eight adjacent outputs per thread (lane = tile row, warp = group
// of eight columns).  The tile's input rows (plus the window's halo) arrive by one bulk copy each (the
// part inside the image, 16-byte aligned), then one pass converts them into a float32 image and a
// float16 image in shared memory with the border applied (REPLICATE / REFLECT read the folded pixel,
// CONSTANT the neutral element).  Row pitches are 4 (mod 8) words with an odd multiple of 4 (mod 32), so
// the 16-byte loads of eight lanes on eight consecutive rows hit distinct banks.
#pragma once

#include "bulk_copy.cuh"
#include "direct.cuh"

namespace serron {

constexpr int kAcRows = 32, kAcCols = 64, kAcQ = 8, kAcThreads = 256;

// Smallest pitch (in 32-bit words) >= need whose residue mod 32 is an odd multiple of 4.
__host__ __device__ constexpr int ac_pitch_words(int need) {
    int p = need;
    while (!((p % 32) % 4 == 0 && ((p % 32) / 4) % 2 == 1)) ++p;
    return p;
}

template <int K, int TI_BYTES>
struct AcGeom {
    static constexpr int a = K / 2;
    static constexpr int SR = kAcRows + K - 1;                     // staged rows
    static constexpr int SC = kAcCols + K - 1;                     // staged columns
    static constexpr int NX = kAcQ + K - 1;                        // samples a thread reads per row
    static constexpr int NX4 = (NX + 3) / 4 * 4;                   // ... in whole 16-byte loads (floats)
    static constexpr int NH8 = (NX + 7) / 8 * 8;                   // ... (halves)
    static constexpr int XP = ac_pitch_words(kAcCols - kAcQ + NX4);  // float32 image pitch (floats)
    static constexpr int HP = 2 * ac_pitch_words((kAcCols - kAcQ + NH8) / 2);  // float16 image pitch (halves)
    // landing rows: image columns [gcA, gcA + LP), gcA = ow0 - a - SH aligned to 16 bytes
    static constexpr int AL = 16 / TI_BYTES;
    static constexpr int SH = (AL - a % AL) % AL;
    static constexpr int LP = (SH + SC + AL - 1) / AL * AL;
    static constexpr size_t X_BYTES = size_t(SR) * XP * 4;
    static constexpr size_t H_BYTES = size_t(SR) * HP * 2;
    static constexpr size_t L_BYTES = (size_t(SR) * LP * TI_BYTES + 15) / 16 * 16;
    static constexpr size_t W_BYTES = (size_t(K) * K * 8 + 15) / 16 * 16;
    static constexpr size_t MARK_OFF = X_BYTES + H_BYTES + L_BYTES + W_BYTES;
    static size_t smem() { return MARK_OFF + mark_bytes(kAcRows, kAcCols, K, K); }
};

template <typename TI>
__device__ __forceinline__ float ac_load(TI v) {
    return Storage<TI>::load(v);
}

template <int OP>
__device__ __forceinline__ __half2 ac_tap2(__half2 s, __half2 w) {
    return OP == kErode ? __hsub2(s, w) : __hadd2(s, w);
}
template <int OP>
__device__ __forceinline__ __half2 ac_best2(__half2 a, __half2 b) {
    return OP == kErode ? __hmin2(a, b) : __hmax2(a, b);
}

// TI: input storage (float, __half, __nv_bfloat16); weights are float32, per channel (kcs = K * K) or
// shared (kcs = 0).  `bulk`: rows of x start on 16-byte boundaries (pointer and W checked by the host).
template <typename TI, int OP, int K>
__global__ void __launch_bounds__(kAcThreads, 3) tiled_autocast_fwd_kernel(
    const TI* __restrict__ x, const float* __restrict__ w, __half* __restrict__ y, uint8_t* __restrict__ win,
    uint32_t* __restrict__ map, int C, int H, int W, int kcs, int border, int tiles_x, int tiles_y, int bulk,
    int out_vec) {
    static_assert(K % 2 == 1 && K * K <= 255, "odd window, one-byte taps");
    using G = AcGeom<K, sizeof(TI)>;
    constexpr int a = G::a, SR = G::SR, SC = G::SC, XP = G::XP, HP = G::HP, LP = G::LP, NX = G::NX;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);                                   // [SR][XP]
    __half* hs = reinterpret_cast<__half*>(smem_raw + G::X_BYTES);                    // [SR][HP]
    TI* land = reinterpret_cast<TI*>(smem_raw + G::X_BYTES + G::H_BYTES);             // [SR][LP]
    float* w32 = reinterpret_cast<float*>(smem_raw + G::X_BYTES + G::H_BYTES + G::L_BYTES);  // [K*K]
    __half2* w16 = reinterpret_cast<__half2*>(w32 + K * K);                           // [K*K]
    __shared__ __align__(8) uint64_t bar;
    __shared__ int exact_flag;

    const TileCoord tc = tile_coord(tiles_x, tiles_y);
    const int c = static_cast<int>(tc.plane % C);
    const int oh0 = tc.ty * kAcRows, ow0 = tc.tx * kAcCols;
    const TI* xp = x + tc.plane * H * W;
    const float* wc = w + static_cast<long long>(c) * kcs;
    const int tid = threadIdx.x;
    const float neutral = Op<OP>::template neutral<float>();
    const int r_lo = max(0, oh0 - a), r_hi = min(H, oh0 - a + SR);  // landed image rows
    const int gcA = ow0 - a - G::SH;
    const int c_lo = max(0, gcA), c_hi = min(W, gcA + LP);          // landed image columns

    const TileMarks marks{reinterpret_cast<uint32_t*>(smem_raw + G::MARK_OFF), oh0 - a, floor_div32(ow0 - a),
                          kAcRows + K - 1, mark_words(kAcCols, K)};
    if (map) marks.clear(tid, kAcThreads);
    if (tid == 0) exact_flag = 1;
    if (bulk && tid == 0) {
        mbar_init(&bar, 1);
        mbar_arrive_expect_tx(&bar, static_cast<unsigned>((r_hi - r_lo) * (c_hi - c_lo) * sizeof(TI)));
    }
    __syncthreads();
    if (bulk) {
        for (int r = r_lo + tid; r < r_hi; r += kAcThreads)
            bulk_load(land + (r - (oh0 - a)) * LP + (c_lo - gcA), xp + static_cast<long long>(r) * W + c_lo,
                      static_cast<unsigned>((c_hi - c_lo) * sizeof(TI)), &bar);
    } else {
        for (int i = tid; i < (r_hi - r_lo) * (c_hi - c_lo); i += kAcThreads) {
            const int r = r_lo + i / (c_hi - c_lo), q = c_lo + i % (c_hi - c_lo);
            land[(r - (oh0 - a)) * LP + (q - gcA)] = xp[static_cast<long long>(r) * W + q];
        }
    }
    for (int i = tid; i < K * K; i += kAcThreads) {
        const float v = wc[i];
        w32[i] = v;
        w16[i] = __half2half2(__float2half_rn(v));
        if (!weight_is_exact(v)) exact_flag = 0;
    }
    if (bulk) {
        // a byte count that never arrives ends the wait: the tile's values are poisoned (NaN)
        if (!__syncthreads_and(mbar_wait(&bar, 0))) {
            for (int i = tid; i < kAcRows * kAcCols; i += kAcThreads) {
                const int oh = oh0 + i / kAcCols, ow = ow0 + i % kAcCols;
                if (oh < H && ow < W) y[tc.plane * H * W + static_cast<long long>(oh) * W + ow] = __float2half_rn(__int_as_float(0x7fffffff));
            }
            return;
        }
    } else {
        __syncthreads();
    }
    // the float32 and float16 images of the staged window, border applied
    for (int i = tid; i < SR * SC; i += kAcThreads) {
        const int r = i / SC, q = i - r * SC;
        int gr = oh0 - a + r, gq = ow0 - a + q;
        float v = neutral;
        if (resolve(gr, H, border) && resolve(gq, W, border)) {
            if (gr >= r_lo && gr < r_hi && gq >= c_lo && gq < c_hi)
                v = ac_load(land[(gr - (oh0 - a)) * LP + (gq - gcA)]);
            else  // folded from beyond the landed rows or columns (an image narrower than the window)
                v = ac_load(xp[static_cast<long long>(gr) * W + gq]);
        }
        xs[r * XP + q] = v;
        hs[r * HP + q] = __float2half_rn(v);
    }
    __syncthreads();

    const int lr = tid & 31, q0 = (tid >> 5) * kAcQ;  // output row and first of eight columns
    const int oh = oh0 + lr;
    const bool exact = exact_flag != 0;
    __half2 acc[kAcQ / 2];
    float best[kAcQ];
    int tap[kAcQ];
    bool tie = false;  // some tap of some output compared equal to that output's running best
    {
        const __half hn = __float2half_rn(neutral);
#pragma unroll
        for (int p = 0; p < kAcQ / 2; ++p) acc[p] = __halves2half2(hn, hn);
#pragma unroll
        for (int k = 0; k < kAcQ; ++k) {
            best[k] = neutral;
            tap[k] = -1;
        }
    }
#pragma unroll 1
    for (int di = 0; di < K; ++di) {
        // this row's samples: float32 x[q0 .. q0 + NX), float16 pairs at even and odd offsets
        float s[G::NX4];
        const float4* xr = reinterpret_cast<const float4*>(xs + (lr + di) * XP + q0);
#pragma unroll
        for (int v4 = 0; v4 < G::NX4 / 4; ++v4) {
            const float4 t = xr[v4];
            s[4 * v4] = t.x;
            s[4 * v4 + 1] = t.y;
            s[4 * v4 + 2] = t.z;
            s[4 * v4 + 3] = t.w;
        }
        uint32_t he[G::NH8 / 2];  // he[i] = (h[2i], h[2i + 1])
        const uint4* hr = reinterpret_cast<const uint4*>(hs + (lr + di) * HP + q0);
#pragma unroll
        for (int v4 = 0; v4 < G::NH8 / 8; ++v4) {
            const uint4 t = hr[v4];
            he[4 * v4] = t.x;
            he[4 * v4 + 1] = t.y;
            he[4 * v4 + 2] = t.z;
            he[4 * v4 + 3] = t.w;
        }
#pragma unroll
        for (int dj = 0; dj < K; ++dj) {
            const int t_idx = di * K + dj;
            const float wv = w32[t_idx];
            const __half2 wh = w16[t_idx];
#pragma unroll
            for (int p = 0; p < kAcQ / 2; ++p) {
                // samples of outputs 2p and 2p + 1 at this tap: h[2p + dj], h[2p + dj + 1]
                const int e = 2 * p + dj;
                const uint32_t pair = (e & 1) ? __byte_perm(he[e >> 1], he[(e >> 1) + 1], 0x5432) : he[e >> 1];
                __half2 sp;
                memcpy(&sp, &pair, 4);
                acc[p] = ac_best2<OP>(acc[p], ac_tap2<OP>(sp, wh));
            }
#pragma unroll
            for (int k = 0; k < kAcQ; ++k) {
                const float v = Op<OP>::tap(s[k + dj], wv);
                if (!exact) tie |= v == best[k];
                if (Op<OP>::better(v, best[k])) {
                    best[k] = v;
                    tap[k] = t_idx;
                }
            }
        }
    }
    static_assert(NX <= G::NX4 && NX <= G::NH8, "samples per row");

    const bool active = oh < H && ow0 + q0 < W;
    if (active) {
        int last_winner = -1;
        const uint32_t kw_magic = static_cast<uint32_t>(((1ull << 32) + K - 1) / K);
        __half vals[kAcQ];
        uint8_t recs[kAcQ];
#pragma unroll
        for (int k = 0; k < kAcQ; ++k) {
            vals[k] = (k & 1) ? __high2half(acc[k >> 1]) : __low2half(acc[k >> 1]);
            if (tie && best[k] != neutral) {
                // a float tie with a running best in this thread: settle its outputs the way the reference
                // CPU does, in double (rare: it takes two taps whose float32 results coincide)
                auto sample = [&](int di_, int dj_, float& s_) {
                    s_ = xs[(lr + di_) * XP + q0 + k + dj_];
                    return true;
                };
                auto weight = [&](int di_, int dj_) { return w32[di_ * K + dj_]; };
                float b_;
                window_winner<float, OP, true>(sample, weight, K, K, b_, tap[k]);
            }
            recs[k] = encode_direct<uint8_t>(tap[k]);
        }
        const long long o = tc.plane * H * W + static_cast<long long>(oh) * W + ow0 + q0;
        if (out_vec && ow0 + q0 + kAcQ <= W) {
            uint4 vv;
            memcpy(&vv, vals, 16);
            *reinterpret_cast<uint4*>(y + o) = vv;
            uint2 rr;
            memcpy(&rr, recs, 8);
            *reinterpret_cast<uint2*>(win + o) = rr;
        } else {
#pragma unroll
            for (int k = 0; k < kAcQ; ++k)
                if (ow0 + q0 + k < W) {
                    y[o + k] = vals[k];
                    win[o + k] = recs[k];
                }
        }
        if (map) {
#pragma unroll
            for (int k = 0; k < kAcQ; ++k)
                if (tap[k] >= 0 && ow0 + q0 + k < W)
                    marks.mark(map, tc.plane, H, W, K, kw_magic, a, a, border, oh, ow0 + q0 + k, tap[k], last_winner);
        }
    }
    if (map) {
        __syncthreads();
        marks.flush(map, tc.plane, H, W, tid, kAcThreads);
    }
}

}  // namespace serron
