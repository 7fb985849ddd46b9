/*
 * ORACLE -- test infrastructure only; see morph_oracle.h.
 *
 * A restatement in C of the reference's CPU algorithm.  Each routine names the
 * reference lines it follows (paths relative to packages/serron/).  The
 * reference computes in acc_type<scalar_t, false> (csrc/compat/acc_type.h:23-53):
 * double for float and double, float for half and bfloat16.  Here the inputs are
 * widened once to that type, the algorithm runs on the widened copy, and the
 * results are rounded back to the storage type exactly where the reference
 * rounds.
 */
#include "morph_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* storage conversions                                                        */
/* ------------------------------------------------------------------------- */

static inline uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static inline float u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t oracle_f32_to_f16(float f) {
    const uint32_t u = f2u(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t absu = u & 0x7fffffffu;
    if (absu > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((absu >> 13) & 0x3ffu)); /* NaN */
    if (absu >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf (>= 65520) */
    const int32_t exp = (int32_t)(absu >> 23) - 127;
    if (exp >= -14) {
        /* normal half: 10 mantissa bits, round the dropped 13 to nearest even */
        uint32_t mant = absu & 0x7fffffu;
        uint32_t h = ((uint32_t)(exp + 15) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u; /* carry into exponent is correct */
        return (uint16_t)(sign | h);
    }
    if (exp < -25) return (uint16_t)sign; /* below half of the smallest subnormal */
    /* subnormal half: value = m * 2^-24 with m = round(abs * 2^24) */
    const uint32_t mant = (absu & 0x7fffffu) | 0x800000u; /* 24-bit significand, value mant*2^(exp-23) */
    const int shift = -exp - 1;                             /* mant * 2^(exp-23) / 2^-24 = mant >> (-1-exp) */
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t mant = h & 0x3ffu;
    if (exp == 0) {
        const float v = (float)mant * 0x1p-24f;
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (mant << 13));
    return u2f(sign | ((exp + 112u) << 23) | (mant << 13));
}

/* ------------------------------------------------------------------------- */
/* borders: csrc/cpu/utils/boundaries.h:26-51                                 */
/* ------------------------------------------------------------------------- */

static inline int resolve_coord(int64_t* coord, int64_t size, int border) {
    int64_t c = *coord;
    if (c >= 0 && c < size) return 1;
    switch (border) {
    case OR_REPLICATE:
        *coord = c < 0 ? 0 : size - 1;
        return 1;
    case OR_REFLECT: {
        if (size == 1) {
            *coord = 0;
            return 1;
        }
        const int64_t period = 2 * size - 2;
        int64_t m = c % period;
        if (m < 0) m += period;
        *coord = m < size ? m : period - m;
        return 1;
    }
    default:
        return 0;
    }
}

/* ------------------------------------------------------------------------- */
/* widening / narrowing                                                       */
/* ------------------------------------------------------------------------- */

static void widen_d(int dtype, const void* src, double* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = dtype == OR_F32 ? (double)((const float*)src)[i] : ((const double*)src)[i];
}
static void widen_f(int dtype, const void* src, float* dst, int64_t n) {
    const uint16_t* s = (const uint16_t*)src;
    for (int64_t i = 0; i < n; ++i) dst[i] = dtype == OR_F16 ? oracle_f16_to_f32(s[i]) : oracle_bf16_to_f32(s[i]);
}
static void narrow_d(int dtype, const double* src, void* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        if (dtype == OR_F32)
            ((float*)dst)[i] = (float)src[i];
        else
            ((double*)dst)[i] = src[i];
    }
}
static void narrow_f(int dtype, const float* src, void* dst, int64_t n) {
    uint16_t* d = (uint16_t*)dst;
    for (int64_t i = 0; i < n; ++i) d[i] = dtype == OR_F16 ? oracle_f32_to_f16(src[i]) : oracle_f32_to_bf16(src[i]);
}

/* ------------------------------------------------------------------------- */
/* the algorithm, once per accumulate type                                    */
/* ------------------------------------------------------------------------- */

/* op policy: csrc/cpu/morphology/ops_policy.h:11-49 */
#define NEUTRAL(ACC, op) ((op) == OR_ERODE ? (ACC)INFINITY : -(ACC)INFINITY)
#define TAP(op, s, w) ((op) == OR_ERODE ? (s) - (w) : (s) + (w))
#define REDUCE(op, acc, val) ((op) == OR_ERODE ? ((val) < (acc) ? (val) : (acc)) : ((val) > (acc) ? (val) : (acc)))

#define DEFINE_ALGO(ACC, SFX)                                                                                          \
    /* direct 2-D window: csrc/cpu/morphology/operators.cpp:38-80 */                                                 \
    static void fwd_direct_##SFX(int op, const ACC* x, const ACC* w, ACC* y, int64_t N, int64_t C, int64_t H,      \
                                 int64_t W, int64_t kH, int64_t kW, int64_t kcs, int border) {                     \
        const int64_t ah = kH / 2, aw = kW / 2, total = N * C * H * W;                                            \
        const ACC neutral = NEUTRAL(ACC, op);                                                                      \
        _Pragma("omp parallel for schedule(static)") for (int64_t idx = 0; idx < total; ++idx) {                   \
            const int64_t w_ = idx % W, h = (idx / W) % H, c = (idx / (W * H)) % C, n = idx / (W * H * C);        \
            const ACC* xin = x + (n * C + c) * H * W;                                                              \
            const ACC* kc = w + c * kcs;                                                                           \
            ACC acc = neutral;                                                                                     \
            for (int64_t di = 0; di < kH; ++di) {                                                                  \
                int64_t ih = h + di - ah;                                                                          \
                const int ihv = resolve_coord(&ih, H, border);                                                     \
                for (int64_t dj = 0; dj < kW; ++dj) {                                                              \
                    ACC val = neutral;                                                                             \
                    if (ihv) {                                                                                     \
                        int64_t iw = w_ + dj - aw;                                                                 \
                        if (resolve_coord(&iw, W, border)) val = TAP(op, xin[ih * W + iw], kc[di * kW + dj]);      \
                    }                                                                                              \
                    acc = REDUCE(op, acc, val);                                                                    \
                }                                                                                                  \
            }                                                                                                      \
            y[idx] = acc;                                                                                          \
        }                                                                                                          \
    }                                                                                                              \
                                                                                                                   \
    /* one separable line pass: csrc/cpu/morphology/operators.cpp:101-148.  The reference rounds the row      */  \
    /* result to the storage type between passes; a flat SE only copies samples, so that rounding is exact. */  \
    static void line_pass_##SFX(int op, const ACC* in, ACC* out, int64_t N, int64_t C, int64_t H, int64_t W,     \
                                int64_t k, int border, int col) {                                                  \
        const int64_t line_len = col ? H : W, lines = col ? W : H, stride = col ? W : 1;                          \
        const int64_t anchor = k / 2, span = line_len + k - 1, padded = (span + k - 1) / k * k;                   \
        const ACC neutral = NEUTRAL(ACC, op);                                                                      \
        _Pragma("omp parallel") {                                                                                  \
            ACC* samples = (ACC*)malloc(sizeof(ACC) * (size_t)padded);                                             \
            ACC* prefix = (ACC*)malloc(sizeof(ACC) * (size_t)padded);                                              \
            ACC* suffix = (ACC*)malloc(sizeof(ACC) * (size_t)padded);                                              \
            for (int64_t t = 0; t < padded; ++t) samples[t] = neutral;                                             \
            _Pragma("omp for schedule(static)") for (int64_t idx = 0; idx < N * C * lines; ++idx) {                \
                const int64_t line = idx % lines, nc = idx / lines;                                                \
                const ACC* inc = in + nc * H * W;                                                                  \
                ACC* outc = out + nc * H * W;                                                                      \
                const int64_t off = col ? line : line * W;                                                         \
                for (int64_t t = 0; t < span; ++t) {                                                               \
                    int64_t pos = t - anchor;                                                                      \
                    samples[t] = resolve_coord(&pos, line_len, border) ? inc[off + pos * stride] : neutral;        \
                }                                                                                                  \
                for (int64_t t = 0; t < padded; ++t)                                                               \
                    prefix[t] = (t % k == 0) ? samples[t] : REDUCE(op, prefix[t - 1], samples[t]);                 \
                for (int64_t t = padded - 1; t >= 0; --t)                                                          \
                    suffix[t] = (t % k == k - 1) ? samples[t] : REDUCE(op, suffix[t + 1], samples[t]);             \
                for (int64_t o = 0; o < line_len; ++o) outc[off + o * stride] = REDUCE(op, suffix[o], prefix[o + k - 1]); \
            }                                                                                                      \
            free(samples);                                                                                         \
            free(prefix);                                                                                          \
            free(suffix);                                                                                          \
        }                                                                                                          \
    }                                                                                                              \
                                                                                                                   \
    /* winners, direct: csrc/cpu/morphology/backward.cpp:46-99 (strict improvement = first extremum) */         \
    static void winners_direct_##SFX(int op, const ACC* x, const ACC* w, int64_t* best_in, int64_t* best_k,      \
                                     int64_t N, int64_t C, int64_t H, int64_t W, int64_t kH, int64_t kW,          \
                                     int64_t kcs, int border) {                                                    \
        const int64_t ah = kH / 2, aw = kW / 2, total = N * C * H * W;                                            \
        const ACC neutral = NEUTRAL(ACC, op);                                                                      \
        _Pragma("omp parallel for schedule(static)") for (int64_t idx = 0; idx < total; ++idx) {                   \
            const int64_t w_ = idx % W, h = (idx / W) % H, c = (idx / (W * H)) % C, n = idx / (W * H * C);        \
            const ACC* xin = x + (n * C + c) * H * W;                                                              \
            const ACC* kc = w + c * kcs;                                                                           \
            ACC best = neutral;                                                                                    \
            int64_t bk = -1, bi = -1;                                                                              \
            for (int64_t di = 0; di < kH; ++di) {                                                                  \
                int64_t ih = h + di - ah;                                                                          \
                const int ihv = resolve_coord(&ih, H, border);                                                     \
                for (int64_t dj = 0; dj < kW; ++dj) {                                                              \
                    ACC val = neutral;                                                                             \
                    int64_t off = -1;                                                                              \
                    if (ihv) {                                                                                     \
                        int64_t iw = w_ + dj - aw;                                                                 \
                        if (resolve_coord(&iw, W, border)) {                                                       \
                            off = ih * W + iw;                                                                     \
                            val = TAP(op, xin[off], kc[di * kW + dj]);                                             \
                        }                                                                                          \
                    }                                                                                              \
                    const ACC merged = REDUCE(op, best, val);                                                      \
                    if (merged != best) {                                                                          \
                        best = merged;                                                                             \
                        bk = di * kW + dj;                                                                         \
                        bi = off;                                                                                  \
                    }                                                                                              \
                }                                                                                                  \
            }                                                                                                      \
            best_in[idx] = bi < 0 ? -1 : (n * C + c) * H * W + bi;                                                 \
            best_k[idx] = bk < 0 ? -1 : c * kcs + bk;                                                              \
        }                                                                                                          \
    }                                                                                                              \
                                                                                                                   \
    /* separable argreduce: csrc/cpu/morphology/backward.cpp:116-236 */                                             \
    typedef struct {                                                                                               \
        ACC val;                                                                                                   \
        int64_t idx;                                                                                               \
    } argtap_##SFX;                                                                                                \
    static inline argtap_##SFX arg_combine_##SFX(int op, argtap_##SFX lo, argtap_##SFX hi) {                      \
        return REDUCE(op, lo.val, hi.val) != lo.val ? hi : lo;                                                     \
    }                                                                                                              \
    /* mode 0: row pass over the image; mode 1: column pass over the row results */                               \
    static void argreduce_##SFX(int op, const ACC* rows_in, ACC* row_val, int32_t* row_dj, int64_t* best_in,     \
                                int64_t* best_k, int64_t N, int64_t C, int64_t H, int64_t W, int64_t kH, int64_t kW, \
                                int64_t kcs, int border, int mode) {                                               \
        const int64_t k = mode ? kH : kW, line_len = mode ? H : W, lines = mode ? N * C * W : N * C * H;           \
        const int64_t anchor = k / 2, span = line_len + k - 1, padded = (span + k - 1) / k * k;                   \
        const ACC neutral = NEUTRAL(ACC, op);                                                                      \
        _Pragma("omp parallel") {                                                                                  \
            argtap_##SFX* s = (argtap_##SFX*)malloc(sizeof(argtap_##SFX) * (size_t)padded);                        \
            argtap_##SFX* pre = (argtap_##SFX*)malloc(sizeof(argtap_##SFX) * (size_t)padded);                     \
            argtap_##SFX* suf = (argtap_##SFX*)malloc(sizeof(argtap_##SFX) * (size_t)padded);                      \
            _Pragma("omp for schedule(static)") for (int64_t line = 0; line < lines; ++line) {                     \
                for (int64_t t = 0; t < padded; ++t) {                                                             \
                    int64_t pos = t - anchor;                                                                      \
                    const int inside = t < span && resolve_coord(&pos, line_len, border);                          \
                    ACC v = neutral;                                                                               \
                    if (inside) {                                                                                  \
                        if (mode == 0)                                                                             \
                            v = rows_in[line * W + pos];                                                           \
                        else                                                                                       \
                            v = row_val[(line / W) * H * W + pos * W + line % W];                                  \
                    }                                                                                              \
                    s[t].val = v;                                                                                  \
                    s[t].idx = t;                                                                                  \
                }                                                                                                  \
                for (int64_t t = 0; t < padded; ++t) pre[t] = (t % k == 0) ? s[t] : arg_combine_##SFX(op, pre[t - 1], s[t]); \
                for (int64_t t = padded - 1; t >= 0; --t)                                                          \
                    suf[t] = (t % k == k - 1) ? s[t] : arg_combine_##SFX(op, s[t], suf[t + 1]);                    \
                for (int64_t o = 0; o < line_len; ++o) {                                                           \
                    const argtap_##SFX tap = arg_combine_##SFX(op, suf[o], pre[o + k - 1]);                        \
                    const int64_t d = tap.idx - o;                                                                 \
                    if (mode == 0) {                                                                               \
                        row_val[line * W + o] = tap.val;                                                           \
                        row_dj[line * W + o] = (int32_t)d;                                                         \
                    } else {                                                                                       \
                        const int64_t nc = line / W, w_ = line % W, c = nc % C;                                    \
                        int64_t ih = o + d - kH / 2;                                                               \
                        const int okh = resolve_coord(&ih, H, border);                                             \
                        const int64_t idx = nc * H * W + o * W + w_;                                               \
                        if (!okh) {                                                                                \
                            best_in[idx] = -1;                                                                     \
                            best_k[idx] = -1;                                                                      \
                            continue;                                                                              \
                        }                                                                                          \
                        const int32_t dj = row_dj[nc * H * W + ih * W + w_];                                       \
                        int64_t iw = w_ + dj - kW / 2;                                                             \
                        if (!resolve_coord(&iw, W, border)) {                                                      \
                            best_in[idx] = -1;                                                                     \
                            best_k[idx] = -1;                                                                      \
                            continue;                                                                              \
                        }                                                                                          \
                        best_in[idx] = nc * H * W + ih * W + iw;                                                   \
                        best_k[idx] = c * kcs + d * kW + dj;                                                       \
                    }                                                                                              \
                }                                                                                                  \
            }                                                                                                      \
            free(s);                                                                                               \
            free(pre);                                                                                             \
            free(suf);                                                                                             \
        }                                                                                                          \
    }

DEFINE_ALGO(double, d)
DEFINE_ALGO(float, f)

/* ------------------------------------------------------------------------- */
/* entry points                                                               */
/* ------------------------------------------------------------------------- */

static int is_wide(int dtype) { return dtype == OR_F32 || dtype == OR_F64; }

static int check_args(int op, int dtype, int border) {
    if (op != OR_ERODE && op != OR_DILATE) return 1;
    if (dtype < OR_F32 || dtype > OR_BF16) return 2;
    if (border < OR_REFLECT || border > OR_CONSTANT) return 3;
    return 0;
}

int oracle_forward(int op, int dtype, const void* x, const void* w, void* y, int64_t N, int64_t C, int64_t H,
                   int64_t W, int64_t kH, int64_t kW, int64_t kcs, int border, int separable) {
    int rc = check_args(op, dtype, border);
    if (rc) return rc;
    const int64_t total = N * C * H * W, nk = kcs ? C * kcs : kH * kW;
    if (total == 0) return 0;
    if (is_wide(dtype)) {
        double* xa = malloc(sizeof(double) * (size_t)total);
        double* wa = malloc(sizeof(double) * (size_t)nk);
        double* ya = malloc(sizeof(double) * (size_t)total);
        widen_d(dtype, x, xa, total);
        widen_d(dtype, w, wa, nk);
        if (separable) {
            double* tmp = malloc(sizeof(double) * (size_t)total);
            line_pass_d(op, xa, tmp, N, C, H, W, kW, border, 0);
            /* the reference's row scratch is scalar_t: round it (exact for a flat SE) */
            if (dtype == OR_F32)
                for (int64_t i = 0; i < total; ++i) tmp[i] = (double)(float)tmp[i];
            line_pass_d(op, tmp, ya, N, C, H, W, kH, border, 1);
            free(tmp);
        } else {
            fwd_direct_d(op, xa, wa, ya, N, C, H, W, kH, kW, kcs, border);
        }
        narrow_d(dtype, ya, y, total);
        free(xa);
        free(wa);
        free(ya);
    } else {
        float* xa = malloc(sizeof(float) * (size_t)total);
        float* wa = malloc(sizeof(float) * (size_t)nk);
        float* ya = malloc(sizeof(float) * (size_t)total);
        widen_f(dtype, x, xa, total);
        widen_f(dtype, w, wa, nk);
        if (separable) {
            float* tmp = malloc(sizeof(float) * (size_t)total);
            line_pass_f(op, xa, tmp, N, C, H, W, kW, border, 0);
            uint16_t* r = malloc(sizeof(uint16_t) * (size_t)total);
            narrow_f(dtype, tmp, r, total);
            widen_f(dtype, r, tmp, total);
            free(r);
            line_pass_f(op, tmp, ya, N, C, H, W, kH, border, 1);
            free(tmp);
        } else {
            fwd_direct_f(op, xa, wa, ya, N, C, H, W, kH, kW, kcs, border);
        }
        narrow_f(dtype, ya, y, total);
        free(xa);
        free(wa);
        free(ya);
    }
    return 0;
}

int oracle_winners(int op, int dtype, const void* x, const void* w, int64_t* best_in, int64_t* best_k, int64_t N,
                   int64_t C, int64_t H, int64_t W, int64_t kH, int64_t kW, int64_t kcs, int border, int separable) {
    int rc = check_args(op, dtype, border);
    if (rc) return rc;
    const int64_t total = N * C * H * W, nk = kcs ? C * kcs : kH * kW;
    if (total == 0) return 0;
    if (is_wide(dtype)) {
        double* xa = malloc(sizeof(double) * (size_t)total);
        double* wa = malloc(sizeof(double) * (size_t)nk);
        widen_d(dtype, x, xa, total);
        widen_d(dtype, w, wa, nk);
        if (separable) {
            double* rv = malloc(sizeof(double) * (size_t)total);
            int32_t* rd = malloc(sizeof(int32_t) * (size_t)total);
            argreduce_d(op, xa, rv, rd, best_in, best_k, N, C, H, W, kH, kW, kcs, border, 0);
            if (dtype == OR_F32)
                for (int64_t i = 0; i < total; ++i) rv[i] = (double)(float)rv[i];
            argreduce_d(op, xa, rv, rd, best_in, best_k, N, C, H, W, kH, kW, kcs, border, 1);
            free(rv);
            free(rd);
        } else {
            winners_direct_d(op, xa, wa, best_in, best_k, N, C, H, W, kH, kW, kcs, border);
        }
        free(xa);
        free(wa);
    } else {
        float* xa = malloc(sizeof(float) * (size_t)total);
        float* wa = malloc(sizeof(float) * (size_t)nk);
        widen_f(dtype, x, xa, total);
        widen_f(dtype, w, wa, nk);
        if (separable) {
            float* rv = malloc(sizeof(float) * (size_t)total);
            int32_t* rd = malloc(sizeof(int32_t) * (size_t)total);
            argreduce_f(op, xa, rv, rd, best_in, best_k, N, C, H, W, kH, kW, kcs, border, 0);
            argreduce_f(op, xa, rv, rd, best_in, best_k, N, C, H, W, kH, kW, kcs, border, 1);
            free(rv);
            free(rd);
        } else {
            winners_direct_f(op, xa, wa, best_in, best_k, N, C, H, W, kH, kW, kcs, border);
        }
        free(xa);
        free(wa);
    }
    return 0;
}

/* serial scatter in the storage type's arithmetic: csrc/cpu/morphology/backward.cpp:250-263 */
int oracle_backward(int op, int dtype, const void* go, const void* x, const void* w, void* gi, void* gk, int64_t N,
                    int64_t C, int64_t H, int64_t W, int64_t kH, int64_t kW, int64_t kcs, int border, int separable,
                    int need_kernel_grad) {
    int rc = check_args(op, dtype, border);
    if (rc) return rc;
    const int64_t total = N * C * H * W, nk = kcs ? C * kcs : kH * kW;
    const size_t esz = dtype == OR_F64 ? 8 : dtype == OR_F32 ? 4 : 2;
    memset(gi, 0, esz * (size_t)total);
    memset(gk, 0, esz * (size_t)nk);
    if (total == 0) return 0;
    int64_t* bi = malloc(sizeof(int64_t) * (size_t)total);
    int64_t* bk = malloc(sizeof(int64_t) * (size_t)total);
    rc = oracle_winners(op, dtype, x, w, bi, bk, N, C, H, W, kH, kW, kcs, border, separable);
    if (rc) {
        free(bi);
        free(bk);
        return rc;
    }
    for (int64_t idx = 0; idx < total; ++idx) {
        if (bi[idx] < 0) continue;
        switch (dtype) {
        case OR_F32: {
            const float g = ((const float*)go)[idx];
            float* gif = (float*)gi;
            gif[bi[idx]] = gif[bi[idx]] + g;
            if (need_kernel_grad) {
                float* gkf = (float*)gk;
                gkf[bk[idx]] = gkf[bk[idx]] + (float)((op == OR_ERODE ? -1.0 : 1.0) * (double)g);
            }
            break;
        }
        case OR_F64: {
            const double g = ((const double*)go)[idx];
            double* gid = (double*)gi;
            gid[bi[idx]] = gid[bi[idx]] + g;
            if (need_kernel_grad) {
                double* gkd = (double*)gk;
                gkd[bk[idx]] = gkd[bk[idx]] + (op == OR_ERODE ? -1.0 : 1.0) * g;
            }
            break;
        }
        default: {
            float (*load)(uint16_t) = dtype == OR_F16 ? oracle_f16_to_f32 : oracle_bf16_to_f32;
            uint16_t (*store)(float) = dtype == OR_F16 ? oracle_f32_to_f16 : oracle_f32_to_bf16;
            const float g = load(((const uint16_t*)go)[idx]);
            uint16_t* gih = (uint16_t*)gi;
            gih[bi[idx]] = store(load(gih[bi[idx]]) + g);
            if (need_kernel_grad) {
                uint16_t* gkh = (uint16_t*)gk;
                const float sg = load(store((op == OR_ERODE ? -1.0f : 1.0f) * g));
                gkh[bk[idx]] = store(load(gkh[bk[idx]]) + sg);
            }
            break;
        }
        }
    }
    free(bi);
    free(bk);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* reconstruction: torch-ext/serron/functional.py:144-202                      */
/* ------------------------------------------------------------------------- */

/* torch.minimum / torch.maximum propagate NaN */
#define CLIP(dil, a, b)                                                                                                \
    (((a) != (a)) ? (a) : ((b) != (b)) ? (b) : (dil) ? ((b) < (a) ? (b) : (a)) : ((b) > (a) ? (b) : (a)))

int64_t oracle_reconstruct(int dilate, int dtype, const void* marker, const void* mask, const void* w, void* out,
                           int64_t N, int64_t C, int64_t H, int64_t W, int64_t kH, int64_t kW, int64_t kcs,
                           int border, int flat, int64_t max_iter, int64_t check_every) {
    if (check_args(0, dtype, border) || check_every < 1) return -2;
    const int64_t total = N * C * H * W, nk = kcs ? C * kcs : kH * kW;
    const int op = dilate ? OR_DILATE : OR_ERODE;
    const int sep = flat && (kH > 1 || kW > 1);
    int64_t result = -1;
    if (is_wide(dtype)) {
        double *cur = malloc(8 * (size_t)total), *nxt = malloc(8 * (size_t)total), *snap = malloc(8 * (size_t)total),
               *mk = malloc(8 * (size_t)total), *wa = malloc(8 * (size_t)nk), *tmp = malloc(8 * (size_t)total);
        widen_d(dtype, marker, cur, total);
        widen_d(dtype, mask, mk, total);
        widen_d(dtype, w, wa, nk);
        for (int64_t i = 0; i < total; ++i) cur[i] = CLIP(dilate, cur[i], mk[i]);
        memcpy(snap, cur, 8 * (size_t)total);
        int64_t it = 0;
        for (;;) {
            if (max_iter > 0 && it >= max_iter) break;
            if (sep) {
                line_pass_d(op, cur, tmp, N, C, H, W, kW, border, 0);
                line_pass_d(op, tmp, nxt, N, C, H, W, kH, border, 1);
            } else {
                fwd_direct_d(op, cur, wa, nxt, N, C, H, W, kH, kW, kcs, border);
            }
            /* the step's output is rounded to the storage type before the clip */
            for (int64_t i = 0; i < total; ++i) {
                double v = dtype == OR_F32 ? (double)(float)nxt[i] : nxt[i];
                cur[i] = CLIP(dilate, v, mk[i]);
            }
            ++it;
            if (it % check_every == 0) {
                int same = 1;
                for (int64_t i = 0; i < total && same; ++i) same = cur[i] == snap[i];
                if (same) {
                    result = it;
                    break;
                }
                memcpy(snap, cur, 8 * (size_t)total);
            }
        }
        if (result < 0) {
            int same = 1;
            for (int64_t i = 0; i < total && same; ++i) same = cur[i] == snap[i];
            if (same) result = it;
        }
        narrow_d(dtype, cur, out, total);
        free(cur);
        free(nxt);
        free(snap);
        free(mk);
        free(wa);
        free(tmp);
    } else {
        float *cur = malloc(4 * (size_t)total), *nxt = malloc(4 * (size_t)total), *snap = malloc(4 * (size_t)total),
              *mk = malloc(4 * (size_t)total), *wa = malloc(4 * (size_t)nk), *tmp = malloc(4 * (size_t)total);
        uint16_t* r = malloc(2 * (size_t)total);
        widen_f(dtype, marker, cur, total);
        widen_f(dtype, mask, mk, total);
        widen_f(dtype, w, wa, nk);
        for (int64_t i = 0; i < total; ++i) cur[i] = CLIP(dilate, cur[i], mk[i]);
        memcpy(snap, cur, 4 * (size_t)total);
        int64_t it = 0;
        for (;;) {
            if (max_iter > 0 && it >= max_iter) break;
            if (sep) {
                line_pass_f(op, cur, tmp, N, C, H, W, kW, border, 0);
                line_pass_f(op, tmp, nxt, N, C, H, W, kH, border, 1);
            } else {
                fwd_direct_f(op, cur, wa, nxt, N, C, H, W, kH, kW, kcs, border);
            }
            narrow_f(dtype, nxt, r, total);
            widen_f(dtype, r, nxt, total);
            for (int64_t i = 0; i < total; ++i) cur[i] = CLIP(dilate, nxt[i], mk[i]);
            ++it;
            if (it % check_every == 0) {
                int same = 1;
                for (int64_t i = 0; i < total && same; ++i) same = cur[i] == snap[i];
                if (same) {
                    result = it;
                    break;
                }
                memcpy(snap, cur, 4 * (size_t)total);
            }
        }
        if (result < 0) {
            int same = 1;
            for (int64_t i = 0; i < total && same; ++i) same = cur[i] == snap[i];
            if (same) result = it;
        }
        narrow_f(dtype, cur, out, total);
        free(cur);
        free(nxt);
        free(snap);
        free(mk);
        free(wa);
        free(tmp);
        free(r);
    }
    return result;
}

/* ------------------------------------------------------------------------- */
/* reconstruction to the fixed point by flooding (exact, any schedule)        */
/* ------------------------------------------------------------------------- */

/* The reference iterates y <- clip(op(y), mask) from clip(marker, mask) until
 * nothing changes (torch-ext/serron/functional.py:144-202).  For a structuring
 * element whose finite taps all weigh zero and include the anchor, under the
 * CONSTANT border (out-of-image taps are neutral), a step only moves values
 * along the taps' edges, so the fixed point is unique: for dilation, y(p) is the
 * largest over paths q -> ... -> p (each node reading the previous through a
 * tap) of min(y0(q), mask of every later node).  That is a widest-path problem,
 * solved here by a max-heap flood in O(n log n) instead of thousands of full
 * steps; erosion is the same on negated values.  Only min/max and copies are
 * involved, so the result is bit-identical to the reference's loop.
 * Returns 0, or -2 for arguments outside that class (another border, a
 * non-zero finite weight, a missing anchor tap, NaN). */

typedef struct {
    double key;
    uint32_t idx;
} flood_item;

static void flood_push(flood_item** heap, int64_t* n, int64_t* cap, double key, uint32_t idx) {
    if (*n == *cap) {
        *cap = *cap ? 2 * *cap : 1024;
        *heap = realloc(*heap, (size_t)*cap * sizeof(flood_item));
    }
    flood_item* h = *heap;
    int64_t i = (*n)++;
    while (i > 0) {
        const int64_t parent = (i - 1) / 2;
        if (h[parent].key >= key) break;
        h[i] = h[parent];
        i = parent;
    }
    h[i].key = key;
    h[i].idx = idx;
}

static flood_item flood_pop(flood_item* h, int64_t* n) {
    const flood_item top = h[0];
    const flood_item last = h[--(*n)];
    int64_t i = 0;
    for (;;) {
        int64_t c = 2 * i + 1;
        if (c >= *n) break;
        if (c + 1 < *n && h[c + 1].key > h[c].key) ++c;
        if (h[c].key <= last.key) break;
        h[i] = h[c];
        i = c;
    }
    if (*n > 0) h[i] = last;
    return top;
}

int oracle_reconstruct_flood(int dilate, int dtype, const void* marker, const void* mask, const void* w, void* out,
                             int64_t N, int64_t C, int64_t H, int64_t W, int64_t kH, int64_t kW, int64_t kcs,
                             int border) {
    if (check_args(0, dtype, border) || border != OR_CONSTANT) return -2;
    const int64_t total = N * C * H * W, nk = kcs ? C * kcs : kH * kW, plane = H * W;
    if (plane >= ((int64_t)1 << 32)) return -2;
    const int64_t aH = kH / 2, aW = kW / 2;
    double* wk = malloc(8 * (size_t)(nk > 0 ? nk : 1));
    double* mk = malloc(8 * (size_t)(total > 0 ? total : 1));
    double* y = malloc(8 * (size_t)(total > 0 ? total : 1));
    float* tmpf = malloc(4 * (size_t)((total > nk ? total : nk) > 0 ? (total > nk ? total : nk) : 1));
    int rc = 0;
    /* widen to double (exact for every storage type) */
    if (is_wide(dtype)) {
        widen_d(dtype, w, wk, nk);
        widen_d(dtype, mask, mk, total);
        widen_d(dtype, marker, y, total);
    } else {
        widen_f(dtype, w, tmpf, nk);
        for (int64_t i = 0; i < nk; ++i) wk[i] = tmpf[i];
        widen_f(dtype, mask, tmpf, total);
        for (int64_t i = 0; i < total; ++i) mk[i] = tmpf[i];
        widen_f(dtype, marker, tmpf, total);
        for (int64_t i = 0; i < total; ++i) y[i] = tmpf[i];
    }
    for (int64_t i = 0; i < nk; ++i)
        if (!(wk[i] == 0.0 || (isinf(wk[i]) && wk[i] < 0))) rc = -2;
    for (int64_t c = 0; c < (kcs ? C : 1) && !rc; ++c)
        if (wk[c * kH * kW + aH * kW + aW] != 0.0) rc = -2;
    for (int64_t i = 0; i < total && !rc; ++i)
        if (isnan(mk[i]) || isnan(y[i])) rc = -2;
    if (!rc) {
        const double s = dilate ? 1.0 : -1.0; /* erosion: the same flood on negated values */
        for (int64_t i = 0; i < total; ++i) {
            mk[i] *= s;
            y[i] *= s;
            if (mk[i] < y[i]) y[i] = mk[i];
        }
        /* tap offsets of each plane's SE: u = v + (di - aH, dj - aW) is read by v */
        int64_t* tdi = malloc(8 * (size_t)(kH * kW));
        int64_t* tdj = malloc(8 * (size_t)(kH * kW));
        flood_item* heap = NULL;
        int64_t cap = 0;
        for (int64_t pl = 0; pl < N * C; ++pl) {
            const double* wp = wk + (kcs ? (pl % C) * kcs : 0);
            int64_t nt = 0;
            for (int64_t di = 0; di < kH; ++di)
                for (int64_t dj = 0; dj < kW; ++dj)
                    if (wp[di * kW + dj] == 0.0 && !(di == aH && dj == aW)) {
                        tdi[nt] = di - aH;
                        tdj[nt] = dj - aW;
                        ++nt;
                    }
            double* yp = y + pl * plane;
            const double* mp = mk + pl * plane;
            int64_t n = 0;
            /* every pixel that can raise a reader starts in the heap */
            for (int64_t v = 0; v < plane; ++v) {
                const int64_t vy = v / W, vx = v % W;
                int raises = 0;
                for (int64_t t = 0; t < nt && !raises; ++t) {
                    const int64_t ry = vy - tdi[t], rx = vx - tdj[t];
                    if (ry < 0 || ry >= H || rx < 0 || rx >= W) continue;
                    const int64_t r = ry * W + rx;
                    const double cand = yp[v] < mp[r] ? yp[v] : mp[r];
                    raises = cand > yp[r];
                }
                if (raises) flood_push(&heap, &n, &cap, yp[v], (uint32_t)v);
            }
            while (n > 0) {
                const flood_item it = flood_pop(heap, &n);
                if (it.key != yp[it.idx]) continue; /* superseded by a later raise */
                const int64_t uy = it.idx / W, ux = it.idx % W;
                for (int64_t t = 0; t < nt; ++t) {
                    /* the reader r of u through tap t: r + (di, dj) = u */
                    const int64_t ry = uy - tdi[t], rx = ux - tdj[t];
                    if (ry < 0 || ry >= H || rx < 0 || rx >= W) continue;
                    const int64_t r = ry * W + rx;
                    const double cand = it.key < mp[r] ? it.key : mp[r];
                    if (cand > yp[r]) {
                        yp[r] = cand;
                        flood_push(&heap, &n, &cap, cand, (uint32_t)r);
                    }
                }
            }
        }
        free(heap);
        free(tdi);
        free(tdj);
        for (int64_t i = 0; i < total; ++i) y[i] *= s;
        if (is_wide(dtype)) {
            narrow_d(dtype, y, out, total);
        } else {
            for (int64_t i = 0; i < total; ++i) tmpf[i] = (float)y[i];
            narrow_f(dtype, tmpf, out, total);
        }
    }
    free(wk);
    free(mk);
    free(y);
    free(tmpf);
    return rc;
}
