// Reconstruction to the fixed point in one persistent launch.
//
// The worklist of 64x64 tiles lives on the device.  A grid of co-resident CTAs pops tiles, solves each
// in shared memory (recon_scan.cuh's scan tiles, or recon.cuh's full-step tiles) and, when the tile's
// values changed where a neighbour reads them, asks for that neighbour to run again.  The call is
// done when no tile is queued or running: that is the device-side convergence test, and the host
// reads it once, after the launch.
//
// Per tile, a state word keeps the worklist exact without ever solving one tile on two CTAs at once:
//   IDLE -> QUEUED        a neighbour's request; the tile is pushed (pending + 1)
//   QUEUED -> RUNNING     a CTA pops it
//   RUNNING -> RUNNING|1  a request while it runs: it will run again
//   RUNNING -> IDLE       it finished, nothing asked for it meanwhile (pending - 1)
//   RUNNING|1 -> QUEUED   it finished and is pushed again (its inner iterations ran out, or a neighbour
//                         changed its halo while it ran)
// A tile therefore sits in the queue at most once, a run always starts after the last change of its
// halo that it must see (the neighbour writes, fences, then requests), and `pending` counts tiles
// queued or running; it reaches zero only at the fixed point, because a tile's requests for its
// neighbours are made before its own state is released.
//
// The queue is a ring of 64-bit cells tagged with their slot number, so a consumer that took slot s
// (head) waits for exactly the item a producer put in slot s (tail).  Every wait is bounded by a
// budget of wall-clock nanoseconds (%globaltimer): a wait that runs out records kReconTimedOut in the
// status word and the CTA returns; every other wait sees that status and returns too.  y is read
// through L2 (ld.global.cg), since a tile's pixels are written by whichever CTA ran it last.
#pragma once

#include "recon.cuh"
#include "recon_scan.cuh"

namespace serron {

constexpr int kTileIdle = 0, kTileQueued = 1, kTileRunning = 2;
constexpr int kReconTimedOut = 1;

// Device-side worklist state (workspace memory; set up by recon_queue_init_kernel).
struct ReconQueue {
    unsigned long long* cells;  // [cap]: (slot + 1) << 32 | tile
    int* state;                 // [tiles]
    unsigned int* counters;     // head, tail, pending, status, tile runs
    unsigned int cap;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned int ld_volatile(const unsigned int* p) {
    return *reinterpret_cast<const volatile unsigned int*>(p);
}

__device__ __forceinline__ void rq_push(const ReconQueue& q, int tile) {
    const unsigned int slot = atomicAdd(&q.counters[1], 1u);
    const unsigned long long cell = (static_cast<unsigned long long>(slot + 1u) << 32) | static_cast<unsigned int>(tile);
    atomicExch(&q.cells[slot % q.cap], cell);
}

// A neighbour's request that `tile` runs (again); made after the requester's writes were fenced.
__device__ __forceinline__ void rq_request(const ReconQueue& q, int tile) {
    const int old = atomicOr(&q.state[tile], 1);
    if (old == kTileIdle) {
        atomicAdd(&q.counters[2], 1u);
        rq_push(q, tile);
    }
}

// The end of a run: queued again when asked for (`again`, or a request meanwhile), else idle.
__device__ __forceinline__ void rq_finish(const ReconQueue& q, int tile, bool again) {
    if (again) atomicOr(&q.state[tile], 1);
    const int old = atomicCAS(&q.state[tile], kTileRunning, kTileIdle);
    if (old == kTileRunning) {
        __threadfence();
        atomicSub(&q.counters[2], 1u);
    } else {  // RUNNING | 1: pending stays, the tile goes back in the queue
        atomicExch(&q.state[tile], kTileQueued);
        rq_push(q, tile);
    }
}

// Next tile for this CTA (one thread), -1 when the fixed point is reached, -2 on a timeout or after
// another CTA's.
__device__ __forceinline__ int rq_pop(const ReconQueue& q, unsigned long long budget_ns) {
    if (ld_volatile(&q.counters[3]) != 0u) return -2;
    if (ld_volatile(&q.counters[2]) == 0u) return -1;
    const unsigned int slot = atomicAdd(&q.counters[0], 1u);
    const unsigned long long want = static_cast<unsigned long long>(slot + 1u);
    const unsigned long long t0 = global_ns();
    unsigned int backoff = 32;
    for (;;) {
        const unsigned long long cell = atomicAdd(&q.cells[slot % q.cap], 0ull);
        if ((cell >> 32) == want) {
            const int tile = static_cast<int>(cell & 0xffffffffull);
            atomicExch(&q.state[tile], kTileRunning);
            __threadfence();
            return tile;
        }
        if (ld_volatile(&q.counters[2]) == 0u) return -1;  // nothing queued or running: nothing will come
        if (ld_volatile(&q.counters[3]) != 0u) return -2;
        if (global_ns() - t0 > budget_ns) {
            atomicOr(&q.counters[3], static_cast<unsigned int>(kReconTimedOut));
            return -2;
        }
        __nanosleep(backoff);
        if (backoff < 1024) backoff *= 2;
    }
}

// The tiles of tile rows [0, row0_end) and [row1_begin, tiles_y) of every plane queued once, in order
// (all of them when row0_end == tiles_y), the others idle; the rest of the ring cleared (a cell left
// by an earlier call must not match a slot of this one).  The tail and pending counters start at the
// number queued.
__global__ void recon_queue_init_kernel(ReconQueue q, int planes, int tiles_x, int tiles_y, int row0_end,
                                        int row1_begin) {
    const unsigned int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int per_plane = tiles_x * tiles_y;
    const int tiles = planes * per_plane;
    const int seeded_rows = row0_end + (tiles_y - row1_begin);
    const int per_plane_seeded = seeded_rows * tiles_x;
    const unsigned int queued = static_cast<unsigned int>(planes * per_plane_seeded);
    if (i < static_cast<unsigned int>(tiles)) {
        const int ty = static_cast<int>(i % per_plane) / tiles_x;
        q.state[i] = (ty < row0_end || ty >= row1_begin) ? kTileQueued : kTileIdle;
    }
    if (i < q.cap) {
        unsigned long long cell = 0ull;
        if (i < queued) {
            const int p = static_cast<int>(i) / per_plane_seeded, rem = static_cast<int>(i) - p * per_plane_seeded;
            const int sr = rem / tiles_x, tx = rem - sr * tiles_x;
            const int ty = sr < row0_end ? sr : row1_begin + (sr - row0_end);
            cell = (static_cast<unsigned long long>(i + 1) << 32) | static_cast<unsigned int>(p * per_plane + ty * tiles_x + tx);
        }
        q.cells[i] = cell;
    }
    if (i == 0) {
        q.counters[0] = 0u;
        q.counters[1] = queued;
        q.counters[2] = queued;
        q.counters[3] = 0u;
        q.counters[4] = 0u;
    }
}

// The persistent driver: `solve(tile)` runs one tile and returns the neighbours to request as bits
// 3 * (dy + 1) + (dx + 1) (bit 4: the tile itself).  With `reach` > 1 (a window wider than a tile, or
// folded across an image narrower than the window) a change asks for every tile within `reach` tiles.
// Runs counts the tile runs in counters[4].
template <typename Solve>
__device__ __forceinline__ void recon_persist_loop(const ReconQueue& q, int tiles_x, int tiles_y, int reach,
                                                   unsigned long long budget_ns, Solve solve) {
    __shared__ int s_tile;
    __shared__ unsigned int s_bits;
    const int tid = threadIdx.x;
    const int per_plane = tiles_x * tiles_y;
    for (;;) {
        if (tid == 0) s_tile = rq_pop(q, budget_ns);
        __syncthreads();
        const int t = s_tile;
        if (t < 0) return;
        const unsigned int bits = solve(t);
        __threadfence();  // this thread's writes of the tile, before any neighbour hears of them
        if (tid == 0) s_bits = 0u;
        __syncthreads();
        if (bits) atomicOr(&s_bits, bits);
        __syncthreads();
        const unsigned int nb = s_bits;
        const int plane = t / per_plane, r = t - plane * per_plane;
        const int ty = r / tiles_x, tx = r - ty * tiles_x;
        if (reach <= 1) {
            if (tid < 9 && tid != 4 && ((nb >> tid) & 1u)) {
                const int nx = tx + tid % 3 - 1, ny = ty + tid / 3 - 1;
                if (nx >= 0 && nx < tiles_x && ny >= 0 && ny < tiles_y) rq_request(q, plane * per_plane + ny * tiles_x + nx);
            }
        } else if (nb & ~0x10u) {
            const int x0 = max(0, tx - reach), x1 = min(tiles_x - 1, tx + reach);
            const int y0 = max(0, ty - reach), y1 = min(tiles_y - 1, ty + reach);
            const int bw = x1 - x0 + 1, n = bw * (y1 - y0 + 1);
            for (int i = tid; i < n; i += blockDim.x) {
                const int nx = x0 + i % bw, ny = y0 + i / bw;
                if (nx != tx || ny != ty) rq_request(q, plane * per_plane + ny * tiles_x + nx);
            }
        }
        __threadfence();  // the requests (and their pending counts) before this tile's state is released
        __syncthreads();
        if (tid == 0) {
            rq_finish(q, t, (nb >> 4) & 1u);
            atomicAdd(&q.counters[4], 1u);
        }
        __syncthreads();  // s_tile and s_bits are reused
    }
}

// Flat structuring elements within the 3x3 neighbourhood: scan tiles (six CTAs per SM).
template <typename T, int OP>
__global__ void __launch_bounds__(kScanTileThreads, 6) recon_persist_scan_kernel(
    T* __restrict__ y, const T* __restrict__ mask, int H, int W, int tiles_x, int tiles_y, int cls, int max_inner,
    ReconQueue q, unsigned long long budget_ns) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    recon_persist_loop(q, tiles_x, tiles_y, 1, budget_ns, [&](int t) {
        return scan_tile_solve<T, OP>(t, y, mask, H, W, tiles_x, tiles_y, cls, max_inner, smem_raw);
    });
}

// Any other structuring element: full-step tiles.
template <typename T, int OP>
__global__ void __launch_bounds__(kRecThreads) recon_persist_full_kernel(
    T* __restrict__ y, const T* __restrict__ mask, const T* __restrict__ w, int C, int H, int W, int kH, int kW,
    int kcs, int border, int tiles_x, int tiles_y, int max_inner, int reach, ReconQueue q,
    unsigned long long budget_ns) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    recon_persist_loop(q, tiles_x, tiles_y, reach, budget_ns, [&](int t) {
        return full_tile_solve<T, OP>(t, y, mask, w, C, H, W, kH, kW, kcs, border, tiles_x, tiles_y, max_inner,
                                      smem_raw);
    });
}

// Ring cells for `tiles` tiles: every tile can be queued once, and consumers (at most the grid, capped
// at kReconMaxGrid CTAs) may take slots ahead of the producers; four times both keeps a slot's cell
// from being reused while its consumer still waits on it.
constexpr int kReconMaxGrid = 4096;
inline long long recon_queue_cap(long long tiles) { return 4 * tiles + 4ll * kReconMaxGrid + 64; }

}  // namespace serron
