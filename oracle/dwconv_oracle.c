/*
 * dwconv_oracle.c -- CPU restatement of the reference's depthwise path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (depthwise_conv_b200/)
 * links or calls this file; only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg use it, as the checker.
 *
 * What it restates (file:line in luckychen/depthwise_conv):
 *   - the convolution every reference kernel computes: NHWC fp16 input,
 *     [K][K][C] fp16 weights, stride 1, pad K/2, output(b,h,w,c) =
 *     sum_{ki,kj} x(b, h+ki-pad, w+kj-pad, c) * w(ki,kj,c) over in-image taps
 *     (convmixer/kernels/depthwise_integration.cu:71-101,
 *      replknet/kernels/depthWise_ch_128_k_31_t_56_half_forward.cu:688-741);
 *     the reference validates its kernels against exactly this sum computed
 *     by F.conv2d(groups=C) in fp32 (benchmark_sensitivity.py:254-259,
 *     benchmark_triton.py:141-144); here it is accumulated in double;
 *   - the fused epilogue y = act(conv + bias) * scale + shift, act = ReLU or
 *     exact-erf GELU (benchmark_cudnn_fused_e2e.py:65-74 with the BN fold of
 *     :125-131; nn.GELU() default at convmixer/convmixer.py:91), plus the
 *     residual add of convmixer/convmixer.py:58-59;
 *   - the reference kernels' own arithmetic, fp16 accumulation in row-major
 *     tap order with one rounding per fused multiply-add (__hfma / __hfma2 at
 *     depthwise_integration.cu:88-99, depthWise_ch_128_k_31_t_56_half_forward.cu:694,
 *     depthWise_ch_512_k_27_t_14_half_forward.cu:380), used only to report
 *     how far the reference kernels themselves sit from the exact result.
 *
 * binary16 conversions are written from the IEEE 754 definition (no
 * dependency on a compiler's half type).
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

enum { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2 };

/* ---- a minimal parallel-for over [0, n) with dynamic chunks ---------------- */
typedef void (*range_fn)(int64_t lo, int64_t hi, void* ctx);
typedef struct {
    int64_t n, chunk;
    int64_t next;
    pthread_mutex_t mu;
    range_fn fn;
    void* ctx;
} pool_job;

static void* pool_worker(void* arg) {
    pool_job* job = (pool_job*)arg;
    for (;;) {
        pthread_mutex_lock(&job->mu);
        const int64_t lo = job->next;
        job->next += job->chunk;
        pthread_mutex_unlock(&job->mu);
        if (lo >= job->n) break;
        const int64_t hi = lo + job->chunk < job->n ? lo + job->chunk : job->n;
        job->fn(lo, hi, job->ctx);
    }
    return NULL;
}

static void parallel_for(int64_t n, int64_t chunk, int nthreads, range_fn fn, void* ctx) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pool_job job = {n, chunk < 1 ? 1 : chunk, 0, PTHREAD_MUTEX_INITIALIZER, fn, ctx};
    pthread_t tids[256];
    int started = 0;
    for (int i = 1; i < nthreads; ++i)
        if (pthread_create(&tids[started], NULL, pool_worker, &job) == 0) ++started;
    pool_worker(&job);
    for (int i = 0; i < started; ++i) pthread_join(tids[i], NULL);
}

ORACLE_API double oracle_half_to_double(uint16_t h) {
    const int sign = (h >> 15) & 1;
    const int exp = (h >> 10) & 0x1f;
    const int mant = h & 0x3ff;
    double v;
    if (exp == 0) {
        v = ldexp((double)mant, -24); /* subnormal: mant * 2^-24 */
    } else if (exp == 31) {
        v = mant ? NAN : INFINITY;
    } else {
        v = ldexp(1.0 + mant / 1024.0, exp - 15);
    }
    return sign ? -v : v;
}

/* Decoded value of every binary16 bit pattern (filled once). */
static double g_h2d[65536];
static pthread_once_t g_h2d_once = PTHREAD_ONCE_INIT;
static void fill_h2d(void) {
    for (uint32_t i = 0; i < 65536u; ++i) g_h2d[i] = oracle_half_to_double((uint16_t)i);
}
#define H2D(h) (g_h2d[(h)])

/* Round a double to the nearest binary16 value, ties to even. */
ORACLE_API uint16_t oracle_double_to_half(double v) {
    uint16_t sign = 0;
    if (isnan(v)) return 0x7e00;
    if (signbit(v)) {
        sign = 0x8000;
        v = -v;
    }
    if (v >= 65520.0) return sign | 0x7c00; /* rounds to infinity */
    if (v < ldexp(1.0, -14)) {
        /* subnormal range: units of 2^-24 */
        double q = nearbyint(ldexp(v, 24));
        return sign | (uint16_t)q; /* q == 1024 encodes the smallest normal */
    }
    int e;
    double m = frexp(v, &e); /* v = m * 2^e, m in [0.5, 1) */
    m *= 2.0;
    e -= 1; /* v = m * 2^e, m in [1, 2) */
    double q = nearbyint((m - 1.0) * 1024.0);
    if (q >= 1024.0) {
        q = 0.0;
        e += 1;
    }
    if (e > 15) return sign | 0x7c00;
    return sign | (uint16_t)((e + 15) << 10) | (uint16_t)q;
}

static double apply_epilogue(double acc, int64_t c, const uint16_t* bias, const uint16_t* scale,
                             const uint16_t* shift, int act) {
    double v = acc;
    if (bias) v += H2D(bias[c]);
    if (act == ACT_RELU) {
        v = v > 0.0 ? v : 0.0;
    } else if (act == ACT_GELU) {
        v = 0.5 * v * (1.0 + erf(v / sqrt(2.0)));
    }
    if (scale) v *= H2D(scale[c]);
    if (shift) v += H2D(shift[c]);
    return v;
}

/* One output pixel (all C channels) in double precision. */
static void pixel_forward(const uint16_t* x, const uint16_t* w, const uint16_t* bias, const uint16_t* scale,
                          const uint16_t* shift, const uint16_t* residual, int64_t H, int64_t W, int64_t C, int K,
                          int act, int64_t b, int64_t h, int64_t wc, double* acc, float* y32, uint16_t* y16) {
    const int pad = K / 2;
    for (int64_t c = 0; c < C; ++c) acc[c] = 0.0;
    for (int ki = 0; ki < K; ++ki) {
        const int64_t hi = h + ki - pad;
        if (hi < 0 || hi >= H) continue;
        for (int kj = 0; kj < K; ++kj) {
            const int64_t wi = wc + kj - pad;
            if (wi < 0 || wi >= W) continue;
            const uint16_t* xp = x + ((b * H + hi) * W + wi) * C;
            const uint16_t* wp = w + ((int64_t)ki * K + kj) * C;
            for (int64_t c = 0; c < C; ++c) acc[c] += H2D(xp[c]) * H2D(wp[c]);
        }
    }
    const int64_t off = ((b * H + h) * W + wc) * C;
    for (int64_t c = 0; c < C; ++c) {
        double v = apply_epilogue(acc[c], c, bias, scale, shift, act);
        if (residual) v += H2D(residual[off + c]);
        if (y32) y32[off + c] = (float)v;
        if (y16) y16[off + c] = oracle_double_to_half(v);
    }
}

/*
 * Full forward.  Any of bias/scale/shift/residual/y32/y16 may be NULL.
 * Scratch: one double per channel per thread, on the stack for C <= 4096.
 */
typedef struct {
    const uint16_t *x, *w, *bias, *scale, *shift, *residual;
    int64_t B, H, W, C;
    int K, act;
    float* y32;
    uint16_t* y16;
    const int64_t* pix;
} fwd_ctx;

static void forward_rows(int64_t lo, int64_t hi, void* vctx) {
    const fwd_ctx* q = (const fwd_ctx*)vctx;
    double acc[4096];
    for (int64_t r = lo; r < hi; ++r) {
        const int64_t b = r / q->H, h = r % q->H;
        for (int64_t wc = 0; wc < q->W; ++wc)
            pixel_forward(q->x, q->w, q->bias, q->scale, q->shift, q->residual, q->H, q->W, q->C, q->K, q->act, b, h,
                          wc, acc, q->y32, q->y16);
    }
}

ORACLE_API int oracle_dw_forward(const uint16_t* x, const uint16_t* w, const uint16_t* bias, const uint16_t* scale,
                                 const uint16_t* shift, const uint16_t* residual, int64_t B, int64_t H, int64_t W,
                                 int64_t C, int K, int act, float* y32, uint16_t* y16, int nthreads) {
    pthread_once(&g_h2d_once, fill_h2d);
    if (C > 4096 || K < 1 || (K % 2) == 0) return 1;
    fwd_ctx q = {x, w, bias, scale, shift, residual, B, H, W, C, K, act, y32, y16, NULL};
    parallel_for(B * H, 1, nthreads, forward_rows, &q);
    return 0;
}

/*
 * Forward at a list of output pixels only (linear index (b*H + h)*W + w).
 * out32 / out16 are [npix][C] (packed, in list order).
 */
static void forward_pixels(int64_t lo, int64_t hi, void* vctx) {
    const fwd_ctx* q = (const fwd_ctx*)vctx;
    const uint16_t *x = q->x, *w = q->w, *bias = q->bias, *scale = q->scale, *shift = q->shift,
                   *residual = q->residual;
    const int64_t H = q->H, W = q->W, C = q->C;
    const int K = q->K, act = q->act, pad = q->K / 2;
    const int64_t* pix = q->pix;
    float* out32 = q->y32;
    uint16_t* out16 = q->y16;
    double acc[4096];
    for (int64_t i = lo; i < hi; ++i) {
        const int64_t p = pix[i];
        const int64_t b = p / (H * W), h = (p / W) % H, wc = p % W;
        for (int64_t c = 0; c < C; ++c) acc[c] = 0.0;
        for (int ki = 0; ki < K; ++ki) {
            const int64_t hi = h + ki - pad;
            if (hi < 0 || hi >= H) continue;
            for (int kj = 0; kj < K; ++kj) {
                const int64_t wi = wc + kj - pad;
                if (wi < 0 || wi >= W) continue;
                const uint16_t* xp = x + ((b * H + hi) * W + wi) * C;
                const uint16_t* wp = w + ((int64_t)ki * K + kj) * C;
                for (int64_t c = 0; c < C; ++c) acc[c] += H2D(xp[c]) * H2D(wp[c]);
            }
        }
        const int64_t off = ((b * H + h) * W + wc) * C;
        for (int64_t c = 0; c < C; ++c) {
            double v = apply_epilogue(acc[c], c, bias, scale, shift, act);
            if (residual) v += H2D(residual[off + c]);
            if (out32) out32[i * C + c] = (float)v;
            if (out16) out16[i * C + c] = oracle_double_to_half(v);
        }
    }
}

ORACLE_API int oracle_dw_forward_pixels(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                                        const uint16_t* scale, const uint16_t* shift, const uint16_t* residual,
                                        int64_t B, int64_t H, int64_t W, int64_t C, int K, int act,
                                        const int64_t* pix, int64_t npix, float* out32, uint16_t* out16,
                                        int nthreads) {
    pthread_once(&g_h2d_once, fill_h2d);
    if (C > 4096 || K < 1 || (K % 2) == 0) return 1;
    fwd_ctx q = {x, w, bias, scale, shift, residual, B, H, W, C, K, act, out32, out16, pix};
    parallel_for(npix, 4, nthreads, forward_pixels, &q);
    return 0;
}

/*
 * The reference kernels' arithmetic: fp16 accumulator, taps in row-major
 * (ki, kj) order, each a fused multiply-add rounded once to binary16, then
 * (replknet path) an fp16 bias add (__hadd, depthwise_replknet_nhwc_integration.cu:26).
 */
static void f16acc_rows(int64_t lo, int64_t hi_row, void* vctx) {
    const fwd_ctx* q = (const fwd_ctx*)vctx;
    const uint16_t *x = q->x, *w = q->w, *bias = q->bias;
    const int64_t H = q->H, W = q->W, C = q->C;
    const int K = q->K, pad = q->K / 2;
    uint16_t* y16 = q->y16;
    for (int64_t r = lo; r < hi_row; ++r) {
        const int64_t b = r / H, h = r % H;
        for (int64_t wc = 0; wc < W; ++wc) {
            for (int64_t c = 0; c < C; ++c) {
                uint16_t acc = 0;
                for (int ki = 0; ki < K; ++ki) {
                    const int64_t hi = h + ki - pad;
                    if (hi < 0 || hi >= H) continue;
                    for (int kj = 0; kj < K; ++kj) {
                        const int64_t wi = wc + kj - pad;
                        if (wi < 0 || wi >= W) continue;
                        /* binary16 * binary16 is exact in double, as is adding a binary16 */
                        const double prod = H2D(x[((b * H + hi) * W + wi) * C + c]) *
                                            H2D(w[((int64_t)ki * K + kj) * C + c]);
                        acc = oracle_double_to_half(prod + H2D(acc));
                    }
                }
                if (bias) acc = oracle_double_to_half(H2D(acc) + H2D(bias[c]));
                y16[((b * H + h) * W + wc) * C + c] = acc;
            }
        }
    }
}

ORACLE_API int oracle_dw_forward_f16acc(const uint16_t* x, const uint16_t* w, const uint16_t* bias, int64_t B,
                                        int64_t H, int64_t W, int64_t C, int K, uint16_t* y16, int nthreads) {
    pthread_once(&g_h2d_once, fill_h2d);
    if (K < 1 || (K % 2) == 0) return 1;
    fwd_ctx q = {x, w, bias, NULL, NULL, NULL, B, H, W, C, K, 0, NULL, y16, NULL};
    parallel_for(B * H, 1, nthreads, f16acc_rows, &q);
    return 0;
}

/*
 * Per-channel sum of the convolution over all output pixels of image b,
 * computed in O(H*W*C + K*K*C) from 2-D prefix sums of the input:
 *   sum_{h,w} y(b,h,w,c) = sum_{ki,kj} w(ki,kj,c) * S_c(rows(ki), cols(kj))
 * where S_c is the sum of x over the input rectangle tap (ki,kj) touches.
 * A size-independent property for full-size parity checks.
 */
ORACLE_API int oracle_dw_channel_sums(const uint16_t* x, const uint16_t* w, int64_t B, int64_t H, int64_t W,
                                      int64_t C, int K, double* sums /* [B][C] */, double* scratch
                                      /* (H+1)*(W+1)*C doubles */) {
    pthread_once(&g_h2d_once, fill_h2d);
    const int pad = K / 2;
    const int64_t W1 = W + 1;
    for (int64_t b = 0; b < B; ++b) {
        memset(scratch, 0, sizeof(double) * (size_t)((H + 1) * W1 * C));
        for (int64_t h = 0; h < H; ++h)
            for (int64_t wc = 0; wc < W; ++wc) {
                const uint16_t* xp = x + ((b * H + h) * W + wc) * C;
                double* o = scratch + ((h + 1) * W1 + (wc + 1)) * C;
                const double* up = scratch + (h * W1 + (wc + 1)) * C;
                const double* left = scratch + ((h + 1) * W1 + wc) * C;
                const double* diag = scratch + (h * W1 + wc) * C;
                for (int64_t c = 0; c < C; ++c) o[c] = H2D(xp[c]) + up[c] + left[c] - diag[c];
            }
        for (int64_t c = 0; c < C; ++c) sums[b * C + c] = 0.0;
        for (int ki = 0; ki < K; ++ki) {
            /* output rows h in [0,H) read input rows h+ki-pad clipped to [0,H) */
            const int64_t r0 = ki - pad < 0 ? 0 : ki - pad;
            const int64_t r1 = (H + ki - pad) > H ? H : (H + ki - pad);
            if (r1 <= r0) continue;
            for (int kj = 0; kj < K; ++kj) {
                const int64_t c0 = kj - pad < 0 ? 0 : kj - pad;
                const int64_t c1 = (W + kj - pad) > W ? W : (W + kj - pad);
                if (c1 <= c0) continue;
                const uint16_t* wp = w + ((int64_t)ki * K + kj) * C;
                for (int64_t c = 0; c < C; ++c) {
                    const double s = scratch[(r1 * W1 + c1) * C + c] - scratch[(r0 * W1 + c1) * C + c] -
                                     scratch[(r1 * W1 + c0) * C + c] + scratch[(r0 * W1 + c0) * C + c];
                    sums[b * C + c] += H2D(wp[c]) * s;
                }
            }
        }
    }
    return 0;
}
