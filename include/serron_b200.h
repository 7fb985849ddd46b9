/*
 * serron_b200 -- C ABI of the B200 (sm_100a) grayscale-morphology library.
 *
 * Every entry point takes plain device pointers and sizes; nothing here uses torch or any other
 * framework type.  The operator entry points mirror the reference's torch operator schemas
 * (vhrabar/serron 0.6.0, packages/serron/csrc/bindings.cpp:8-19) one for one: same argument meaning,
 * same validation and the same error messages, with the tensor arguments spelled out as
 * (pointer, sizes, number of dims) and the outputs passed in by the caller.
 *
 * Conventions
 *   - Images are contiguous (N, C, H, W); a structuring element (SE) is contiguous (kH, kW), shared by
 *     all channels, or (C, kH, kW).  All tensors of one call share `dtype`.
 *   - `device` is the CUDA device owning the pointers; the call makes it current for its duration, so
 *     any host thread may call, including one that never touched CUDA.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Work is enqueued on it and the
 *     call returns without synchronising, except where a function says otherwise.
 *   - Every function returns SERRON_OK (0) on success.  On failure it returns a non-zero status and
 *     serron_last_error() holds the message for the calling thread, worded as the reference's
 *     SERRON_CHECK messages (packages/serron/csrc/compat/check.h:26-31), e.g.
 *     "serron::erode: input must be 4-D (N, C, H, W), got 2-D".
 *   - `flat` is 1 / 0 when the caller knows whether every SE entry is zero, or -1 to let the library
 *     read the SE back (a device-to-host copy that synchronises `stream`), like the reference's
 *     `bool? flat=None`.
 *   - `algo`: 0 auto, 1 element, 2 tiled, 3 separable (packages/serron/csrc/morph_algorithm.h:16-21).
 *   - `border`: 0 reflect, 1 replicate, 2 constant (packages/serron/torch-ext/serron/enums.py:34-38).
 *     CONSTANT pads with the neutral element (+inf for erode, -inf for dilate).
 */
#ifndef SERRON_B200_H
#define SERRON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SERRON_API __attribute__((visibility("default")))
#else
#define SERRON_API
#endif

/* status codes */
#define SERRON_OK 0
#define SERRON_ERR_INVALID 1       /* bad argument; message in serron_last_error() */
#define SERRON_ERR_CUDA 2          /* a CUDA runtime call failed */
#define SERRON_ERR_NOT_CONVERGED 3 /* reconstruction: max_iter ran out */
#define SERRON_ERR_WORKSPACE 4     /* workspace too small */
#define SERRON_ERR_TIMEOUT 5       /* reconstruction: a bounded wait of the device worklist ran out */

/* dtype codes */
#define SERRON_F32 0
#define SERRON_F64 1
#define SERRON_F16 2
#define SERRON_BF16 3

/* operations */
#define SERRON_ERODE 0
#define SERRON_DILATE 1

/* winner-record formats (one record per output).  serron_forward writes the direct formats for every
 * algorithm: t = di * kW + dj of the winning SE cell, all ones when the window has no winner.  The
 * separable formats (hi = di, lo = dj of the output's own row) are accepted by
 * serron_backward_from_winners. */
#define SERRON_WINNERS_NONE 0
#define SERRON_WINNERS_DIRECT_U8 1
#define SERRON_WINNERS_DIRECT_U16 2
#define SERRON_WINNERS_DIRECT_U32 3
#define SERRON_WINNERS_SEPARABLE_U8 4
#define SERRON_WINNERS_SEPARABLE_U16 5
#define SERRON_WINNERS_SEPARABLE_U32 6
/* Flag on a direct format: the record buffer also carries the gather's target map (one bit per pixel
 * that wins some window; rows of ceil(W/32) 32-bit words, planes one after the other), starting at the
 * first 256-byte boundary after the records.  serron_forward fills it; serron_backward_from_winners
 * then skips finding the winners again.  Size of such a buffer: serron_winners_bytes. */
#define SERRON_WINNERS_MAP 0x10

/* How the library will run one call. */
typedef struct serron_plan_t {
    int32_t algo;                /* resolved algorithm: 1 element, 2 tiled, 3 separable */
    int32_t winners_format;      /* SERRON_WINNERS_* of the records serron_forward writes (with the map flag
                                    where the gather can use a target map) */
    int32_t winners_bytes;       /* bytes per output of that record (1, 2 or 4) */
    int32_t reserved;
    int64_t workspace_bytes;     /* backward: device workspace needed when no winner records are given */
} serron_plan_t;

/* Message of the last failed call on this thread ("" when none). */
SERRON_API const char* serron_last_error(void);

/* ABI version of this header (incremented on incompatible changes). */
SERRON_API int32_t serron_abi_version(void);

/* ---------------------------------------------------------------------------------------------
 * Forward.  Replaces serron::erode / serron::dilate
 *   "erode(Tensor input, Tensor kernel, int border, bool? flat=None, int algo=0) -> Tensor"
 *   (packages/serron/csrc/bindings.cpp:8-9; CUDA impl packages/serron/csrc/gpu/morphology/operators.cpp:153-256).
 * `output` has the shape and dtype of `input`.
 * --------------------------------------------------------------------------------------------- */
SERRON_API int serron_erode(const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                            const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border,
                            int32_t flat, int64_t algo, void* output, int32_t device, void* stream);
SERRON_API int serron_dilate(const void* input, const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                             const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int64_t border,
                             int32_t flat, int64_t algo, void* output, int32_t device, void* stream);

/* Resolves algorithm, winner-record format and backward workspace for a call (host only, no GPU
 * work; with flat == -1 it reads the SE back).  `backward` selects the backward pass's threshold.
 * Has no single reference counterpart: it folds together the reference's resolve_algorithm
 * (packages/serron/csrc/gpu/morphology/algorithm.h:119-137) and its buffer sizing. */
SERRON_API int serron_plan(const int64_t* input_sizes, int64_t input_dim, const void* kernel,
                           const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int32_t flat, int64_t algo,
                           int32_t backward, int32_t device, void* stream, serron_plan_t* plan);

/* Forward of `op` that also writes, per output, the record of its winning tap in the format of
 * serron_plan(backward=0) (`winners` may be NULL to skip it; `output` may be NULL to write only the
 * records).  Feeding the records to serron_backward skips the winner search of the backward pass.
 * The reference has no counterpart; it recomputes winners in its backward
 * (packages/serron/csrc/gpu/morphology/backward_kernels.cu:41-101). */
SERRON_API int serron_forward(int32_t op, const void* input, const int64_t* input_sizes, int64_t input_dim,
                              const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype,
                              int64_t border, int32_t flat, int64_t algo, void* output, void* winners,
                              int32_t winners_format, int32_t device, void* stream);
/* The forward under CUDA autocast, with the backward's winners.  Replaces, for the calls it takes, the
 * reference's autocast path: serron::erode/dilate on float16 casts of their arguments
 * (packages/serron/torch-ext/serron/_cmake_ops.py:175-189) followed, in the backward, by a winner search
 * on the saved tensors promoted to float32 (packages/serron/torch-ext/serron/autograd.py:37-76).
 * `output` (float16, the shape of `input`) gets the op on the float16 casts of `input` (float32, float16
 * or bfloat16, `input_dtype`) and `kernel` (float32); `winners` (serron_winners_bytes of `winners_format`,
 * which must be the one serron_plan gives for the tiled algorithm: one-byte direct taps with the target
 * map) gets the float32 winners, so serron_backward_from_winners can follow with a float32 grad_output.
 * Windows: odd and square, 3 to 15.  The reference has no counterpart. */
SERRON_API int serron_forward_autocast(int32_t op, const void* input, const int64_t* input_sizes, int64_t input_dim,
                                       int32_t input_dtype, const void* kernel, const int64_t* kernel_sizes,
                                       int64_t kernel_dim, int32_t kernel_dtype, int64_t border, void* output,
                                       void* winners, int32_t winners_format, int32_t device, void* stream);

/* Bytes of a record buffer of `winners_format` for an input of `sizes` (4-D): one record per output,
 * plus the target map when the format carries SERRON_WINNERS_MAP; -1 for bad arguments.  No
 * reference counterpart (the reference keeps no winner records). */
SERRON_API int64_t serron_winners_bytes(const int64_t* sizes, int64_t dim, int32_t winners_format);

/* ---------------------------------------------------------------------------------------------
 * Backward.  Replaces serron::erode_backward / serron::dilate_backward
 *   "erode_backward(Tensor grad_output, Tensor input, Tensor kernel, int border, bool? flat=None,
 *    bool need_kernel_grad=True, int algo=0) -> (Tensor, Tensor)"
 *   (packages/serron/csrc/bindings.cpp:10-13; CUDA impl packages/serron/csrc/gpu/morphology/backward.cpp:154-262).
 * grad_input has the input's shape, grad_kernel the kernel's; both are fully written (grad_kernel is
 * zero when need_kernel_grad == 0).  grad_input is bit-identical to the reference CPU backward
 * (serial raster-order accumulation in the storage type's arithmetic) and computed without atomics;
 * grad_kernel is a deterministic reduction.  `workspace` must hold serron_plan(...).workspace_bytes.
 * --------------------------------------------------------------------------------------------- */
SERRON_API int serron_erode_backward(const void* grad_output, const int64_t* grad_output_sizes, int64_t grad_output_dim,
                                     const void* input, const int64_t* input_sizes, int64_t input_dim,
                                     const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim,
                                     int32_t dtype, int64_t border, int32_t flat, int32_t need_kernel_grad,
                                     int64_t algo, void* grad_input, void* grad_kernel, void* workspace,
                                     int64_t workspace_bytes, int32_t device, void* stream);
SERRON_API int serron_dilate_backward(const void* grad_output, const int64_t* grad_output_sizes,
                                      int64_t grad_output_dim, const void* input, const int64_t* input_sizes,
                                      int64_t input_dim, const void* kernel, const int64_t* kernel_sizes,
                                      int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                                      int32_t need_kernel_grad, int64_t algo, void* grad_input, void* grad_kernel,
                                      void* workspace, int64_t workspace_bytes, int32_t device, void* stream);

/* Backward from winner records written by serron_forward (format `winners_format`); `input` is only
 * used for validation and may be NULL.  Workspace: serron_backward_workspace_bytes(...). */
SERRON_API int serron_backward_from_winners(int32_t op, const void* grad_output, const int64_t* sizes, int64_t dim,
                                            const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype,
                                            int64_t border, int32_t need_kernel_grad, const void* winners,
                                            int32_t winners_format, void* grad_input, void* grad_kernel,
                                            void* workspace, int64_t workspace_bytes, int32_t device, void* stream);
SERRON_API int64_t serron_backward_workspace_bytes(const int64_t* sizes, int64_t dim, const int64_t* kernel_sizes,
                                                   int64_t kernel_dim, int32_t need_kernel_grad,
                                                   int32_t winners_format, int32_t with_winners);
/* serron_backward_from_winners in float32 arithmetic with grad_output read as `grad_output_dtype` and
 * grad_input written as `grad_input_dtype` (each float32, float16 or bfloat16; grad_kernel float32):
 * the same results as widening grad_output to float32, running serron_backward_from_winners with
 * dtype float32 and rounding grad_input to its dtype (to nearest even), without those two copies.  It
 * serves the backward that follows serron_forward_autocast, where the reference's autograd casts the
 * float16 grad_output up to the promoted float32 and the float32 grad_input down to the input's dtype
 * (packages/serron/torch-ext/serron/autograd.py:37-76).  Direct one- or two-byte records with their
 * target map only.  Workspace: serron_backward_workspace_bytes(..., with_winners = 1). */
SERRON_API int serron_backward_from_winners_widened(int32_t op, const void* grad_output, int32_t grad_output_dtype,
                                                    const int64_t* sizes, int64_t dim, const int64_t* kernel_sizes,
                                                    int64_t kernel_dim, int64_t border, int32_t need_kernel_grad,
                                                    const void* winners, int32_t winners_format, void* grad_input,
                                                    int32_t grad_input_dtype, void* grad_kernel, void* workspace,
                                                    int64_t workspace_bytes, int32_t device, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Derived operations in one launch.  Replace, for the calls they take, the reference's compositions
 * (packages/serron/torch-ext/serron/functional.py:40-92): mode 0 gradient = dilation(x) - erosion(x),
 * 1 opening = dilation(erosion(x)), 2 closing = erosion(dilation(x)), 3 top_hat = x - opening(x),
 * 4 black_hat = closing(x) - x, each bit-identical to the composition (the intermediate image rounded to
 * `dtype` as the reference's intermediate tensor is, the subtraction in `dtype`).  The gradient finds
 * both extremes over one staged tile; the others keep the intermediate in shared memory.  `winners_a` and
 * `winners_b` (serron_winners_bytes of SERRON_WINNERS_DIRECT_U8 | SERRON_WINNERS_MAP each) get the direct
 * records and target maps of the two operations (gradient: a = dilation, b = erosion, both over x;
 * otherwise a = the first operation over x, b = the second over the intermediate), for
 * serron_backward_from_winners.  serron_derived_supported says whether a call is taken: both window
 * sides at most 7 and, for modes 1-4, an image at least as large as the window.  No reference
 * counterpart.
 * --------------------------------------------------------------------------------------------- */
SERRON_API int serron_derived_supported(int32_t mode, const int64_t* input_sizes, int64_t input_dim,
                                        const int64_t* kernel_sizes, int64_t kernel_dim);
SERRON_API int serron_derived_forward(int32_t mode, const void* input, const int64_t* input_sizes, int64_t input_dim,
                                      const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim,
                                      int32_t dtype, int64_t border, void* output, void* winners_a, void* winners_b,
                                      int32_t winners_format, int32_t device, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Algorithm selection.  Replace serron::feasible_algos / heuristic_algo / set_separable_min_k /
 * get_separable_min_k (packages/serron/csrc/bindings.cpp:16-19, gpu/morphology/dispatch_info.cpp:54-81).
 * Return values are as the reference's (bit mask, algorithm code, threshold) or -1 on error.
 * --------------------------------------------------------------------------------------------- */
SERRON_API int64_t serron_feasible_algos(const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int32_t flat,
                                         int32_t backward, int32_t device);
SERRON_API int64_t serron_heuristic_algo(const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype, int32_t flat,
                                         int32_t backward, int32_t device);
SERRON_API int64_t serron_set_separable_min_k(int32_t device, int32_t dtype, int32_t backward, int64_t min_k);
SERRON_API int64_t serron_get_separable_min_k(int32_t device, int32_t dtype, int32_t backward);

/* ---------------------------------------------------------------------------------------------
 * Geodesic reconstruction.  Replaces the Python loop of serron.functional._reconstruct
 * (packages/serron/torch-ext/serron/functional.py:144-202): out = the fixed point of
 * clip(step(y), mask) from y = clip(marker, mask), step = dilate/clip = min when dilate != 0, else
 * erode/max.  With max_iter <= 0 the fixed point is found by tile-local relaxation in one persistent
 * launch over a device worklist of the 64x64 tiles whose halo moved (scan tiles for flat SEs within the
 * 3x3 neighbourhood, after a few global row and column scan rounds for other flat SEs); the device
 * decides convergence (no tile queued or running) and the host reads it once.  Every wait of that
 * worklist is bounded (SERRON_RECON_WAIT_NS, default 2 s); one that runs out returns
 * SERRON_ERR_TIMEOUT.  With max_iter > 0 the reference's Jacobi schedule and check_every test are
 * reproduced, so the call fails exactly when the reference would.  Synchronous.  *steps receives the
 * scan rounds plus tile runs, or the Jacobi steps, taken.  Workspace:
 * serron_reconstruct_workspace_bytes (256 bytes of flags and counters, then for max_iter <= 0 a state
 * word per tile and the worklist ring, for max_iter > 0 a second image).
 * --------------------------------------------------------------------------------------------- */
SERRON_API int serron_reconstruct(int32_t dilate, const void* marker, const void* mask, const int64_t* sizes,
                                  int64_t dim, const void* kernel, const int64_t* kernel_sizes, int64_t kernel_dim,
                                  int32_t dtype, int64_t border, int64_t max_iter, int64_t check_every, void* output,
                                  void* workspace, int64_t workspace_bytes, int32_t device, void* stream,
                                  int64_t* steps);
SERRON_API int64_t serron_reconstruct_workspace_bytes(const int64_t* sizes, int64_t dim, int32_t dtype,
                                                      int64_t max_iter);
/* Continues a reconstruction whose marker (clipped by the mask) is already at the fixed point except
 * near the top and bottom edges of each plane: the device worklist starts with only the tiles within
 * `seed_top` rows of the top and `seed_bottom` rows of the bottom (both >= 0), and any change spreads
 * from there, to the same fixed point serron_reconstruct reaches.  The halo exchange of a reconstruction
 * sharded along H calls this after its first round, when only rows next to the received halos can move.
 * Arguments and workspace as serron_reconstruct with max_iter = 0.  No reference counterpart (the
 * reference is single-process). */
SERRON_API int serron_reconstruct_from_edges(int32_t dilate, const void* marker, const void* mask,
                                             const int64_t* sizes, int64_t dim, const void* kernel,
                                             const int64_t* kernel_sizes, int64_t kernel_dim, int32_t dtype,
                                             int64_t border, int64_t seed_top, int64_t seed_bottom, void* output,
                                             void* workspace, int64_t workspace_bytes, int32_t device, void* stream,
                                             int64_t* steps);

/* ---------------------------------------------------------------------------------------------
 * Backward without any allocation.  No counterpart in the reference (its backward allocates its own
 * temporaries through torch); this is an addition for callers that cannot allocate device memory: a
 * host binding this ABI that owns only its input and output buffers, or one that must not call
 * cudaMalloc / cudaFree between launches (they synchronise the device and can fail under a fixed
 * memory budget).
 *
 * Same arguments and results as serron_erode_backward / serron_dilate_backward (`op` selects which),
 * with the workspace taken from a fixed array of SERRON_STATIC_SCRATCH_BYTES per device that the
 * library reserves when it loads on that device.  A call needing more is rejected with
 * SERRON_ERR_WORKSPACE before anything is enqueued.  Every call looks the array's address up with
 * the device current (so a device reset between calls is harmless); the first call on a device may
 * load the library's module there: make it before any stream capture.  All calls on a device
 * share the array, so calls that can overlap on the GPU (two streams, two host threads) race: order
 * them on one stream or with events.  Nothing in the array needs clearing between calls.
 * --------------------------------------------------------------------------------------------- */
#define SERRON_STATIC_SCRATCH_BYTES (32ll << 20)
SERRON_API int serron_backward_static_scratch(int32_t op, const void* grad_output, const int64_t* grad_output_sizes,
                                              int64_t grad_output_dim, const void* input, const int64_t* input_sizes,
                                              int64_t input_dim, const void* kernel, const int64_t* kernel_sizes,
                                              int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                                              int32_t need_kernel_grad, int64_t algo, void* grad_input,
                                              void* grad_kernel, int32_t device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SERRON_B200_H */
