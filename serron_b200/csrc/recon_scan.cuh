// Geodesic reconstruction by directional scans, for flat structuring elements.
//
// The reference (torch-ext/serron/functional.py:144-202) iterates y <- clip(step(y), mask) until
// nothing changes.  Any schedule that keeps raising pixels to a value the full step could give them
// reaches the same fixed point (recon.cuh states why), so these kernels raise whole rows and columns
// at once.  For a flat element whose anchor row holds the left neighbour tap, the left-to-right
// update of one row,
//     y[c] <- C(m[c], B(y[c], y[c - 1]))        B = max, C = min for reconstruction by dilation,
// is a composition of clamps f_c(x) = C(m[c], B(a[c], x)), and clamps compose into clamps using
// selections only: g(f(x)) = C(g(fq), B(g(fp), x)) for f = (fp, fq), f(x) = C(fq, B(fp, x)).  So a
// row scan is a parallel prefix over (p, q) pairs whose result is the sequential scan's, value for
// value.  `recon_rows_kernel` runs left-to-right then right-to-left over each row, one CTA per row;
// `recon_cols_kernel` runs top-to-bottom then bottom-to-top over 32-column strips, each warp holding
// one run of rows.  A round of both carries a front across the image along any path that turns a
// few times, where the tile relaxation moves it one tile per launch.  The host runs a few such rounds
// ahead of recon_tile_kernel (SEs with taps the scans do not cover), which also confirms the fixed
// point; SEs the scans cover go straight to the worklist of recon_tile_scan_kernel below.
//
// Border taps are skipped by the scans (a partial update is still a valid one); where that leaves a
// tap of the full step uncovered (REFLECT with a one-sided line tap, whose edge sample lies on the
// other side) a round without change is not taken as the fixed point.  Inputs hold no NaN: the host
// routes NaN inputs elsewhere before any scan runs.
#pragma once

#include "recon.cuh"

namespace serron {

constexpr int kScanThreads = 1024;
constexpr int kScanPer = 8;                          // elements per thread in a row chunk
constexpr int kScanChunk = kScanThreads * kScanPer;  // row chunk held in shared memory
constexpr int kScanCols = 32;                        // columns per CTA of the column scan
constexpr int kScanRounds = 8;                       // global scan rounds before full-step tile relaxation

// SE classes found on the device (bits of flags[2])
constexpr int kScanFlat = 1;     // every present tap has weight 0 and the anchor is present
constexpr int kScanLeft = 2;     // tap sampling (row, column - 1)
constexpr int kScanRight = 4;    // (row, column + 1)
constexpr int kScanUp = 8;       // (row - 1, column)
constexpr int kScanDown = 16;    // (row + 1, column)
constexpr int kScanOther = 32;   // a present tap outside the 3x3 neighbourhood
constexpr int kScanUL = 64;      // (row - 1, column - 1)
constexpr int kScanUR = 128;     // (row - 1, column + 1)
constexpr int kScanDL = 256;     // (row + 1, column - 1)
constexpr int kScanDR = 512;     // (row + 1, column + 1)
constexpr int kScanDiag = kScanUL | kScanUR | kScanDL | kScanDR;

// one step of the reconstruction as a clamp: f(x) = C(q, B(p, x))
template <int OP>
struct ReconClamp {
    template <typename A>
    static __device__ __forceinline__ A B(A a, A x) { return Op<OP>::better(x, a) ? x : a; }
    template <typename A>
    static __device__ __forceinline__ A C(A m, A v) { return Clip<OP>::apply(v, m); }
    template <typename A>
    static __device__ __forceinline__ A apply(A p, A q, A x) { return C(q, B(p, x)); }
    // (p, q) <- g o f with f = (p, q) applied first
    template <typename A>
    static __device__ __forceinline__ void then(A& p, A& q, A gp, A gq) {
        p = apply(gp, gq, p);
        q = apply(gp, gq, q);
    }
};

template <typename T, int OP>
__global__ void recon_se_class_kernel(const T* __restrict__ w, int kH, int kW, int* __restrict__ out) {
    using A = typename Storage<T>::acc;
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int aH = kH / 2, aW = kW / 2;
    const A never = Op<kDilate>::template neutral<A>();  // a weight of -inf never wins
    bool flat = true, anchor = false;
    int cls = 0;
    for (int di = 0; di < kH; ++di)
        for (int dj = 0; dj < kW; ++dj) {
            const A v = Storage<T>::load(w[di * kW + dj]);
            if (v == never) continue;
            if (!(v == A(0))) flat = false;
            const int dr = di - aH, dc = dj - aW;
            if (dr == 0 && dc == 0) anchor = true;
            else if (dr == 0 && dc == -1) cls |= kScanLeft;
            else if (dr == 0 && dc == 1) cls |= kScanRight;
            else if (dr == -1 && dc == 0) cls |= kScanUp;
            else if (dr == 1 && dc == 0) cls |= kScanDown;
            else if (dr == -1 && dc == -1) cls |= kScanUL;
            else if (dr == -1 && dc == 1) cls |= kScanUR;
            else if (dr == 1 && dc == -1) cls |= kScanDL;
            else if (dr == 1 && dc == 1) cls |= kScanDR;
            else cls |= kScanOther;
        }
    if (flat && anchor) cls |= kScanFlat;
    *out = cls;
}

// Block-wide exclusive prefix of the clamps (p, q) of all threads, in thread order, applied to `x`.
template <int OP, typename A>
__device__ __forceinline__ A scan_prefix_apply(A p, A q, A x, A* sp, A* sq) {
    using R = ReconClamp<OP>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // inclusive warp scan
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const A pp = __shfl_up_sync(0xffffffffu, p, off), pq = __shfl_up_sync(0xffffffffu, q, off);
        if (lane >= off) {
            // earlier lanes first: (p, q) <- (p, q) o (pp, pq)
            A np = pp, nq = pq;
            R::then(np, nq, p, q);
            p = np;
            q = nq;
        }
    }
    if (lane == 31) {
        sp[warp] = p;
        sq[warp] = q;
    }
    __syncthreads();
    if (warp == 0) {
        A wp = sp[lane], wq = sq[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const A pp = __shfl_up_sync(0xffffffffu, wp, off), pq = __shfl_up_sync(0xffffffffu, wq, off);
            if (lane >= off) {
                A np = pp, nq = pq;
                R::then(np, nq, wp, wq);
                wp = np;
                wq = nq;
            }
        }
        sp[32 + lane] = wp;  // inclusive prefix over warps
        sq[32 + lane] = wq;
    }
    __syncthreads();
    // exclusive: the warps before this one, then the lanes before this one
    if (warp > 0) x = R::apply(sp[32 + warp - 1], sq[32 + warp - 1], x);
    const A lp = __shfl_up_sync(0xffffffffu, p, 1), lq = __shfl_up_sync(0xffffffffu, q, 1);
    if (lane > 0) x = R::apply(lp, lq, x);
    return x;
}

// One CTA per image row: left-to-right (when the SE has the left tap), then right-to-left (right tap),
// in chunks of kScanChunk columns staged in shared memory.
template <typename T, int OP>
__global__ void __launch_bounds__(kScanThreads) recon_rows_kernel(T* __restrict__ y, const T* __restrict__ mask,
                                                                  int W, int cls, int* __restrict__ flags) {
    using A = typename Storage<T>::acc;
    using R = ReconClamp<OP>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    A* ys = reinterpret_cast<A*>(smem_raw);  // [kScanChunk], thread t's elements at t * kScanPer + k
    A* ms = ys + kScanChunk;
    __shared__ A sp[64], sq[64];
    __shared__ A carry_s;
    const long long row = blockIdx.x;
    T* yr = y + row * W;
    const T* mr = mask + row * W;
    const int tid = threadIdx.x;
    const A idp = Op<OP>::template neutral<A>();                                   // B's neutral
    const A idq = Op<OP == kDilate ? kErode : kDilate>::template neutral<A>();     // C's neutral
    const int chunks = (W + kScanChunk - 1) / kScanChunk;
    bool changed = false;
    for (int dir = 0; dir < 2; ++dir) {
        if (!(cls & (dir == 0 ? kScanLeft : kScanRight))) continue;
        A carry = idp;
        for (int ci = 0; ci < chunks; ++ci) {
            const int c0 = (dir == 0 ? ci : chunks - 1 - ci) * kScanChunk;
            const int n = min(kScanChunk, W - c0);
            const bool fresh = chunks > 1 || dir == 0 || !(cls & kScanLeft);
            if (fresh) {
                __syncthreads();
                for (int i = tid; i < n; i += kScanThreads) {
                    ys[i] = Storage<T>::load(yr[c0 + i]);
                    ms[i] = Storage<T>::load(mr[c0 + i]);
                }
            }
            __syncthreads();
            // logical position l = tid * kScanPer + k runs along the scan direction
            A p = idp, q = idq;
#pragma unroll
            for (int k = 0; k < kScanPer; ++k) {
                const int l = tid * kScanPer + k;
                if (l < n) {
                    const int i = dir == 0 ? l : n - 1 - l;
                    const A a = ys[i], m = ms[i];
                    R::then(p, q, R::C(m, a), m);
                }
            }
            A x = scan_prefix_apply<OP>(p, q, carry, sp, sq);
#pragma unroll
            for (int k = 0; k < kScanPer; ++k) {
                const int l = tid * kScanPer + k;
                if (l < n) {
                    const int i = dir == 0 ? l : n - 1 - l;
                    const A a = ys[i];
                    const A v = R::apply(a, ms[i], x);
                    if (!(v == a)) {
                        changed = true;
                        ys[i] = v;
                    }
                    x = v;
                    if (l == n - 1) carry_s = v;
                }
            }
            __syncthreads();
            carry = carry_s;
            const bool last = chunks > 1 || dir == 1 || !(cls & kScanRight);
            if (last)
                for (int i = tid; i < n; i += kScanThreads) yr[c0 + i] = Storage<T>::store(ys[i]);
        }
    }
    if (__syncthreads_or(changed) && tid == 0) atomicOr(flags, 1);
}

// One CTA per 32-column strip of a plane; warp s holds rows [s * L, (s + 1) * L), lane j column j of
// the strip.  Top-to-bottom (up tap), then bottom-to-top (down tap).  Each direction composes every
// warp's run, scans the 32 runs of a column in order, and applies.  The top-to-bottom apply also
// composes the bottom-to-top runs from the values it writes.
template <typename T, int OP>
__global__ void __launch_bounds__(kScanThreads) recon_cols_kernel(T* __restrict__ y, const T* __restrict__ mask,
                                                                  int H, int W, int strips, int cls,
                                                                  int* __restrict__ flags) {
    using A = typename Storage<T>::acc;
    using R = ReconClamp<OP>;
    __shared__ A sp[32][kScanCols + 1], sq[32][kScanCols + 1];
    const long long plane = blockIdx.x / strips;
    const int strip = static_cast<int>(blockIdx.x % strips);
    const int j = threadIdx.x & 31, s = threadIdx.x >> 5;
    const int col = strip * kScanCols + j;
    const bool ok = col < W;
    const int L = (H + 31) / 32;
    const int r0 = min(H, s * L), r1 = min(H, r0 + L);
    T* yc = y + plane * H * W + col;
    const T* mc = mask + plane * H * W + col;
    const A idp = Op<OP>::template neutral<A>();
    const A idq = Op<OP == kDilate ? kErode : kDilate>::template neutral<A>();
    const bool down = cls & kScanUp, up = cls & kScanDown;
    bool changed = false;

    // exclusive prefix over the runs of this lane's column, in run order `order` (0: top first)
    auto run_scan = [&](int order) {
        __syncthreads();
        if (s == 0) {
            A p = idp, q = idq;
            for (int t = 0; t < 32; ++t) {
                const int r = order == 0 ? t : 31 - t;
                const A fp = sp[r][j], fq = sq[r][j];
                sp[r][j] = p;
                sq[r][j] = q;
                R::then(p, q, fp, fq);
            }
        }
        __syncthreads();
    };

    if (down) {
        A p = idp, q = idq;
        if (ok)
            for (int r = r0; r < r1; ++r) {
                const A m = Storage<T>::load(mc[static_cast<long long>(r) * W]);
                R::then(p, q, R::C(m, Storage<T>::load(yc[static_cast<long long>(r) * W])), m);
            }
        sp[s][j] = p;
        sq[s][j] = q;
        run_scan(0);
        A x = R::apply(sp[s][j], sq[s][j], idp);
        A bp = idp, bq = idq;  // bottom-to-top composition of this run, from the new values
        if (ok)
            for (int r = r0; r < r1; ++r) {
                const long long o = static_cast<long long>(r) * W;
                const A a = Storage<T>::load(yc[o]), m = Storage<T>::load(mc[o]);
                const A v = R::apply(a, m, x);
                if (!(v == a)) {
                    changed = true;
                    yc[o] = Storage<T>::store(v);
                }
                x = v;
                if (up) {
                    // prepend: the run's lower rows act first
                    A np = R::C(m, v), nq = m;
                    R::then(np, nq, bp, bq);
                    bp = np;
                    bq = nq;
                }
            }
        __syncthreads();
        sp[s][j] = bp;
        sq[s][j] = bq;
    } else if (up) {
        A p = idp, q = idq;
        if (ok)
            for (int r = r1 - 1; r >= r0; --r) {
                const A m = Storage<T>::load(mc[static_cast<long long>(r) * W]);
                R::then(p, q, R::C(m, Storage<T>::load(yc[static_cast<long long>(r) * W])), m);
            }
        sp[s][j] = p;
        sq[s][j] = q;
    }
    if (up) {
        run_scan(1);
        A x = R::apply(sp[s][j], sq[s][j], idp);
        if (ok)
            for (int r = r1 - 1; r >= r0; --r) {
                const long long o = static_cast<long long>(r) * W;
                const A a = Storage<T>::load(yc[o]), m = Storage<T>::load(mc[o]);
                const A v = R::apply(a, m, x);
                if (!(v == a)) {
                    changed = true;
                    yc[o] = Storage<T>::store(v);
                }
                x = v;
            }
    }
    if (__syncthreads_or(changed) && threadIdx.x == 0) atomicOr(flags, 1);
}

// Worklist tile for flat SEs within the 3x3 neighbourhood (anchor plus any of the eight neighbours):
// a 64x64 tile with a one-pixel halo in shared memory, solved by repeated row and column scans (the
// four line taps) and an in-place pass of the diagonal taps, until none changes anything.  Four threads share a row (or a column), 16 pixels each: each
// composes its run's clamps, the four runs are scanned with shuffles, then applied.  Halo cells outside
// the image hold the neutral element (a border tap is left to the opposite scan, which reads the same
// pixel).  A tile that changed a pixel on an edge asks for the neighbour across that edge to run again
// (recon_persist.cuh runs the worklist).
constexpr int kScanTile = 64;
constexpr int kScanTileThreads = 256;                           // four threads per line
constexpr int kLineLanes = kScanTileThreads / kScanTile, kLineRun = kScanTile / kLineLanes;
template <typename A>
constexpr size_t scan_tile_smem() { return static_cast<size_t>((kScanTile + 2) + kScanTile) * (kScanTile + 3) * sizeof(A); }

// Solves tile b (tiles numbered plane by plane, row-major within a plane) in shared memory, writes it
// back if it changed, and returns the neighbours to run again as bits 3 * (dy + 1) + (dx + 1) (bit 4:
// this tile, when its inner iterations ran out).  y is read through L2: the persistent driver runs a
// tile on whichever CTA pops it.
template <typename T, int OP>
__device__ __forceinline__ unsigned scan_tile_solve(long long b, T* __restrict__ y, const T* __restrict__ mask, int H,
                                                    int W, int tiles_x, int tiles_y, int cls, int max_inner,
                                                    unsigned char* smem_raw) {
    using A = typename Storage<T>::acc;
    using R = ReconClamp<OP>;
    constexpr int TS = kScanTile, P = TS + 3;  // pitch: odd
    A* ys = reinterpret_cast<A*>(smem_raw);  // [TS + 2][P], pixel (r, c) of the tile at (r + 1, c + 1)
    A* ms = ys + (TS + 2) * P;                // [TS][P]
    const int tx = static_cast<int>(b % tiles_x), ty = static_cast<int>((b / tiles_x) % tiles_y);
    const long long plane = b / (static_cast<long long>(tiles_x) * tiles_y);
    const int h0 = ty * TS, w0 = tx * TS;
    T* yp = y + plane * H * W;
    const T* mp = mask + plane * H * W;
    const int tid = threadIdx.x;
    const A idp = Op<OP>::template neutral<A>();
    const A idq = Op<OP == kDilate ? kErode : kDilate>::template neutral<A>();

    const int th = min(TS, H - h0), tw = min(TS, W - w0);
    for (int i = tid; i < (TS + 2) * (TS + 2); i += kScanTileThreads) {
        const int r = i / (TS + 2), q = i - r * (TS + 2);
        const int gr = h0 + r - 1, gq = w0 + q - 1;
        A v = idp;
        if (gr >= 0 && gr < H && gq >= 0 && gq < W && r <= th + 1 && q <= tw + 1)
            v = Storage<T>::load(load_cg(yp + static_cast<long long>(gr) * W + gq));
        ys[r * P + q] = v;
    }
    for (int i = tid; i < TS * TS; i += kScanTileThreads) {
        const int r = i / TS, q = i - r * TS;
        ms[r * P + q] = (r < th && q < tw) ? Storage<T>::load(mp[static_cast<long long>(h0 + r) * W + w0 + q]) : idq;
    }
    __syncthreads();

    // one line of n <= 64 cells, four runs of 16; `at(k)` is the k-th cell along the scan direction
    // (a pointer into ys), `mk(k)` its mask, `x0` the cell before the first (halo)
    const int line = tid / kLineLanes, g = tid % kLineLanes;
    // returns 1 when the first cell changed, 2 when the last did, 4 when any did; `moved_at(k)` hears
    // of every cell that changed
    auto sweep = [&](auto at, auto mk, int n, A x0, auto moved_at) {
        __syncwarp();  // the line's cells written by the other lanes in the previous sweep
        const int k0 = g * kLineRun, k1 = min(n, k0 + kLineRun);
        A p = idp, q = idq;
        for (int k = k0; k < k1; ++k) R::then(p, q, R::C(mk(k), *at(k)), mk(k));
#pragma unroll
        for (int off = 1; off < kLineLanes; off <<= 1) {
            const A pp = __shfl_up_sync(0xffffffffu, p, off, kLineLanes);
            const A pq = __shfl_up_sync(0xffffffffu, q, off, kLineLanes);
            if (g >= off) {
                A np = pp, nq = pq;
                R::then(np, nq, p, q);
                p = np;
                q = nq;
            }
        }
        const A lp = __shfl_up_sync(0xffffffffu, p, 1, kLineLanes), lq = __shfl_up_sync(0xffffffffu, q, 1, kLineLanes);
        A x = g > 0 ? R::apply(lp, lq, x0) : x0;
        int moved = 0;
        for (int k = k0; k < k1; ++k) {
            A* c = at(k);
            const A v = R::apply(*c, mk(k), x);
            if (!(v == *c)) {
                *c = v;
                moved |= 4 | (k == 0 ? 1 : 0) | (k == n - 1 ? 2 : 0);
                moved_at(k);
            }
            x = v;
        }
        return moved;
    };

    // lines to sweep: a row is swept again only after a column sweep moved one of its pixels, and a
    // column only after a row sweep did (a line whose pixels did not move is still at its own fixed
    // point, its halo ends being fixed during the launch)
    __shared__ unsigned row_dirty[2], col_dirty[2];
    if (tid < 2) {
        row_dirty[tid] = ~0u;
        col_dirty[tid] = ~0u;
    }
    __syncthreads();
    bool any = false, settled = false;
    int edges = 0;  // bit 0: top row changed, 1: bottom, 2: left column, 3: right
    auto mark = [](unsigned* set, int i) { atomicOr(&set[i >> 5], 1u << (i & 31)); };
    for (int it = 0; it < max_inner; ++it) {
        int moved = 0;
        const bool rows_go = (row_dirty[line >> 5] >> (line & 31)) & 1u;
        __syncthreads();
        if (tid < 2) row_dirty[tid] = 0;
        const bool row_ok = line < th && rows_go;
        const int row_edges = (line == 0 ? 1 : 0) | (line == th - 1 ? 2 : 0);
        const int col_edges = (line == 0 ? 4 : 0) | (line == tw - 1 ? 8 : 0);
        // corner bits (read by diagonal neighbours): 16 top-left, 32 top-right, 64 bottom-left, 128 bottom-right
        const int left_c = (line == 0 ? 16 : 0) | (line == th - 1 ? 64 : 0);   // row `line`, column 0
        const int right_c = (line == 0 ? 32 : 0) | (line == th - 1 ? 128 : 0); // row `line`, last column
        const int top_c = (line == 0 ? 16 : 0) | (line == tw - 1 ? 32 : 0);    // column `line`, row 0
        const int bot_c = (line == 0 ? 64 : 0) | (line == tw - 1 ? 128 : 0);   // column `line`, last row
        if (cls & kScanLeft) {
            const int m = sweep([&](int k) { return &ys[(line + 1) * P + k + 1]; },
                                [&](int k) { return ms[line * P + k]; }, row_ok ? tw : 0,
                                row_ok ? ys[(line + 1) * P] : idp, [&](int k) { mark(col_dirty, k); });
            if (m) edges |= row_edges | (m & 1 ? 4 | left_c : 0) | (m & 2 ? 8 | right_c : 0);
            moved |= m;
        }
        if (cls & kScanRight) {
            const int m = sweep([&](int k) { return &ys[(line + 1) * P + tw - k]; },
                                [&](int k) { return ms[line * P + tw - 1 - k]; }, row_ok ? tw : 0,
                                row_ok ? ys[(line + 1) * P + tw + 1] : idp, [&](int k) { mark(col_dirty, tw - 1 - k); });
            if (m) edges |= row_edges | (m & 1 ? 8 | right_c : 0) | (m & 2 ? 4 | left_c : 0);
            moved |= m;
        }
        __syncthreads();
        const bool cols_go = (col_dirty[line >> 5] >> (line & 31)) & 1u;
        __syncthreads();
        if (tid < 2) col_dirty[tid] = 0;
        const bool col_ok = line < tw && cols_go;
        if (cls & kScanUp) {
            const int m = sweep([&](int k) { return &ys[(k + 1) * P + line + 1]; },
                                [&](int k) { return ms[k * P + line]; }, col_ok ? th : 0, col_ok ? ys[line + 1] : idp,
                                [&](int k) { mark(row_dirty, k); });
            if (m) edges |= col_edges | (m & 1 ? 1 | top_c : 0) | (m & 2 ? 2 | bot_c : 0);
            moved |= m;
        }
        if (cls & kScanDown) {
            const int m = sweep([&](int k) { return &ys[(th - k) * P + line + 1]; },
                                [&](int k) { return ms[(th - 1 - k) * P + line]; }, col_ok ? th : 0,
                                col_ok ? ys[(th + 1) * P + line + 1] : idp, [&](int k) { mark(row_dirty, th - 1 - k); });
            if (m) edges |= col_edges | (m & 1 ? 2 | bot_c : 0) | (m & 2 ? 1 | top_c : 0);
            moved |= m;
        }
        if (cls & kScanDiag) {
            // the diagonal taps, in place (a neighbour read before or after its own update is a value the
            // step could give: either way the update is a valid one)
            __syncthreads();
            for (int i = tid; i < th * tw; i += kScanTileThreads) {
                const int r = i / tw, c = i - r * tw;
                A* cell = &ys[(r + 1) * P + c + 1];
                A x = idp;
                if (cls & kScanUL) x = R::B(x, cell[-P - 1]);
                if (cls & kScanUR) x = R::B(x, cell[-P + 1]);
                if (cls & kScanDL) x = R::B(x, cell[P - 1]);
                if (cls & kScanDR) x = R::B(x, cell[P + 1]);
                const A a0 = *cell;
                const A v = R::apply(a0, ms[r * P + c], x);
                if (!(v == a0)) {
                    *cell = v;
                    mark(row_dirty, r);
                    mark(col_dirty, c);
                    moved |= 4;
                    edges |= (r == 0 ? 1 : 0) | (r == th - 1 ? 2 : 0) | (c == 0 ? 4 : 0) | (c == tw - 1 ? 8 : 0);
                    edges |= (r == 0 && c == 0 ? 16 : 0) | (r == 0 && c == tw - 1 ? 32 : 0) |
                             (r == th - 1 && c == 0 ? 64 : 0) | (r == th - 1 && c == tw - 1 ? 128 : 0);
                }
            }
        }
        if (!__syncthreads_or(moved)) {
            settled = true;
            break;
        }
        any = true;
    }
    if (!any) return 0u;
    for (int i = tid; i < th * tw; i += kScanTileThreads) {
        const int r = i / tw, q = i - r * tw;
        yp[static_cast<long long>(h0 + r) * W + w0 + q] = Storage<T>::store(ys[(r + 1) * P + q + 1]);
    }
    // the neighbours across the edges (and, with diagonal taps, corners) that moved, and the tile itself
    // if it did not settle
    __shared__ int edge_s;
    if (tid == 0) edge_s = 0;
    __syncthreads();
    if (edges) atomicOr(&edge_s, edges);
    __syncthreads();
    const int e = edge_s;
    unsigned bits = (e & 1 ? 1u << 1 : 0u) | (e & 2 ? 1u << 7 : 0u) | (e & 4 ? 1u << 3 : 0u) | (e & 8 ? 1u << 5 : 0u) |
                    (settled ? 0u : 1u << 4);
    if (cls & kScanDiag)
        bits |= (e & 16 ? 1u << 0 : 0u) | (e & 32 ? 1u << 2 : 0u) | (e & 64 ? 1u << 6 : 0u) | (e & 128 ? 1u << 8 : 0u);
    return bits;
}

}  // namespace serron
