/*
 * dwconv_b200.h -- C ABI of the B200 (sm_100a) depthwise-convolution engine.
 *
 * Scope: the FP16 NHWC forward depthwise convolution, stride 1, "same"
 * padding (pad = K/2 on every side), odd kernel sizes 1..31, with an optional
 * fused epilogue  y = act(conv(x) + bias) * scale + shift (+ residual).
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are DEVICE pointers to IEEE binary16 data.
 *   - x, y, residual: NHWC, i.e. the physical layout of a channels_last
 *     [B, C, H, W] tensor; element (b, h, w, c) at ((b*H + h)*W + w)*C + c.
 *   - w: [K][K][C] contiguous (tap-major, channel innermost), the layout the
 *     reference's torch ops take (convmixer/kernels/depthwise_torch_ops.py:202-205,
 *     replknet/kernels/depthwise_replknet_nhwc_ops.py:113).
 *   - bias, scale, shift: [C] or NULL (NULL means 0 / 1 / 0 respectively).
 *   - stream: a cudaStream_t passed as void*; NULL is the legacy default
 *     stream.  Every launch goes on this stream only, and no entry point
 *     synchronises, allocates device memory or calls back into the host, so
 *     all of them can be captured into CUDA graphs.
 *   - Return value: a dwb_status code.  Errors are reported, never exit().
 *   - Requirements: C % 8 == 0 (16-byte channel rows for TMA), x / w / y
 *     16-byte aligned, 1 <= K <= 31 and K odd, B,H,W >= 1 (B == 0 is a no-op).
 *
 * The engine allocates nothing: the caller owns every buffer.
 */
#ifndef DWCONV_B200_H
#define DWCONV_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DWB_ABI_VERSION 6

#if defined(__GNUC__)
#define DWB_API __attribute__((visibility("default")))
#else
#define DWB_API
#endif

typedef enum dwb_status {
    DWB_OK = 0,
    DWB_ERR_NULL_POINTER = 1,   /* a required pointer is NULL                    */
    DWB_ERR_BAD_SHAPE = 2,      /* shape outside the supported range / mismatch  */
    DWB_ERR_BAD_ALIGN = 3,      /* pointer not 16-byte aligned                   */
    DWB_ERR_UNSUPPORTED = 4,    /* valid request this build has no kernel for    */
    DWB_ERR_CUDA = 5,           /* a CUDA runtime / driver call failed           */
    DWB_ERR_NO_DEVICE = 6,      /* no usable sm_100 device                       */
    DWB_ERR_DEVICE_TIMEOUT = 7, /* a kernel's bounded wait expired (device flag) */
    DWB_ERR_BAD_ARG = 8         /* an enum / flag argument is out of range       */
} dwb_status;

typedef enum dwb_act {
    DWB_ACT_NONE = 0,
    DWB_ACT_RELU = 1,
    DWB_ACT_GELU = 2            /* exact erf GELU, as nn.GELU() default          */
} dwb_act;

typedef enum dwb_accum {
    DWB_ACCUM_F32 = 0,          /* every tap accumulated in fp32 (FFMA2)          */
    DWB_ACCUM_MIXED = 1         /* fp16x2 HFMA2 chains of <= 24 taps, added into
                                   fp32 accumulators (rel-L2 ~6e-4 vs exact)      */
} dwb_accum;

/* Accumulation used by the entry points that take no `accum` argument. */
#define DWB_ACCUM_DEFAULT DWB_ACCUM_MIXED

/* Problem description used by the planner. */
typedef struct dwb_problem {
    int64_t batch, height, width, channels;
    int32_t kernel_size;
    int32_t accum;              /* dwb_accum */
} dwb_problem;

/* Launch plan chosen by the planner (all fields are outputs). */
typedef struct dwb_plan {
    int32_t kernel_size;
    int32_t cols_per_thread;    /* R: output columns a thread owns              */
    int32_t rows_per_thread;    /* M: output rows a thread owns                 */
    int32_t channel_block;      /* CB: channels per CTA (2 per lane)            */
    int32_t tile_h, tile_w;     /* output tile per CTA                          */
    int32_t tile_w_in;          /* input columns staged per row (tile_w + K-1)  */
    int32_t ring_rows;          /* stage ring slots (one input row + one weight
                                   row each); at least tile_h                   */
    int32_t ring_wrows;         /* unused, 0                                    */
    int32_t consumer_warps;
    int32_t threads;
    int32_t smem_bytes;
    int32_t ctas_per_sm;
    int64_t grid;               /* CTAs launched (persistent: <= tiles)         */
    int64_t tiles;              /* work units the CTAs walk in strides: output
                                   tiles, or (band mode) bands                  */
    int32_t accum;              /* dwb_accum actually used                      */
    int32_t regs_estimate;      /* registers/thread assumed by the planner      */
    double model_cost;          /* planner's modelled time (arbitrary units)     */
    int32_t row_splits;         /* S: warps sharing one output slot, each taking
                                   every S-th kernel row; their fp32 partial sums
                                   are added in shared memory (0 or 1 = none)    */
    int32_t load_schedule;      /* 0: input columns read next to their FMAs;
                                   1: the row segment read into registers first
                                   (mixed accumulation only)                     */
    int32_t band_tiles;         /* 0: every tile stages its own tile_h + K - 1
                                   input rows and K weight rows.  n > 0 (band
                                   mode, mixed accumulation, K <= 17): a CTA
                                   walks bands of n row tiles of one column
                                   strip, staging each input row once per band
                                   and the K x K weights once; ring_rows must be
                                   at least tile_h + K - 1                      */
} dwb_plan;

/* ---- library information ------------------------------------------------ */

DWB_API int dwb_abi_version(void);
DWB_API const char* dwb_status_string(int status);

/* Plan a problem without touching the GPU (pure host arithmetic).
 * sm_count / smem_optin_bytes describe the target (148 / 232448 on B200);
 * pass 0 for both to use the B200 defaults. */
DWB_API int dwb_plan_query(const dwb_problem* problem, int sm_count, int smem_optin_bytes,
                   dwb_plan* plan_out);

/* The plan the launcher uses for a problem on the current device: the tuned
 * table entry measured fastest on B200 for the same H, W, C, K and
 * accumulation (nearest batch), else the cost model with this device's
 * register counts.  Needs a device. */
DWB_API int dwb_plan_select(const dwb_problem* problem, dwb_plan* plan_out);

/* Every feasible plan for a problem (host arithmetic only), in the planner's
 * enumeration order, for autotuning.  Writes at most `capacity` plans and
 * the total number of feasible plans to *count_out. */
DWB_API int dwb_plan_candidates(const dwb_problem* problem, int sm_count, int smem_optin_bytes,
                                dwb_plan* plans_out, int capacity, int* count_out);

/* Text of the last CUDA runtime/driver failure seen by the calling thread
 * (behind a DWB_ERR_CUDA status), or "" if none. */
DWB_API const char* dwb_last_error(void);

/* ---- generic entry points ------------------------------------------------ */

/* y = conv(x, w): the plain depthwise convolution (no bias), DWB_ACCUM_DEFAULT. */
DWB_API int dwb_conv2d_nhwc_fwd(const void* x, const void* w, void* y,
                        int64_t B, int64_t H, int64_t W, int64_t C, int K,
                        void* stream);

/* y = act(conv(x, w) + bias) * scale + shift (+ residual), in one kernel.
 * Any of bias / scale / shift / residual may be NULL.  accum: dwb_accum. */
DWB_API int dwb_conv2d_nhwc_fused_fwd(const void* x, const void* w, const void* bias,
                              const void* scale, const void* shift,
                              const void* residual, void* y,
                              int64_t B, int64_t H, int64_t W, int64_t C, int K,
                              int act, int accum, void* stream);

/* As dwb_conv2d_nhwc_fused_fwd, with a caller-chosen plan instead of the
 * planner's (for autotuning).  The plan's cols_per_thread, rows_per_thread,
 * tile_h, tile_w, ring_rows, ring_wrows and accum are used; every derived
 * field is recomputed, and an inconsistent plan returns DWB_ERR_BAD_ARG. */
DWB_API int dwb_conv2d_nhwc_fwd_planned(const void* x, const void* w, const void* bias,
                                        const void* scale, const void* shift,
                                        const void* residual, void* y,
                                        int64_t B, int64_t H, int64_t W, int64_t C, int K,
                                        int act, const dwb_plan* plan, void* stream);

/* y = act(x + bias) * scale + shift over `pixels` NHWC pixels of C channels
 * (x, y fp16, 16-byte aligned, C % 8 == 0; bias/scale/shift [C] or NULL).
 * The elementwise tail of a ConvMixer pointwise block (1x1 conv -> bias ->
 * act -> BatchNorm, convmixer/convmixer.py:116-118) in one pass; x == y is
 * allowed.  No counterpart kernel in the reference (PyTorch ops there). */
DWB_API int dwb_bias_act_affine_nhwc(const void* x, const void* bias, const void* scale,
                                     const void* shift, void* y, int64_t pixels, int64_t C,
                                     int act, void* stream);

/* y = act(x * w^T + bias) * scale + shift: a whole ConvMixer pointwise block
 * (1x1 conv -> bias -> act -> BatchNorm, convmixer/convmixer.py:116-118), or a
 * patch stem given its patch matrix, as one tensor-core kernel (tcgen05 MMAs
 * into tensor memory, the epilogue applied on the way out; no intermediate in
 * HBM).  x: [pixels][C_in] fp16 row-major (NHWC activations), w: [C_out][C_in]
 * fp16 row-major (the 1x1 weight as PyTorch stores it), y: [pixels][C_out]
 * fp16; bias/scale/shift: [C_out] fp16 or NULL.  C_in, C_out multiples of 8,
 * x / w / y 16-byte aligned, y must not overlap x or w.  fp32 accumulation.
 * tile_n: output channels per CTA tile (64, 96, 128 or 256), 0 = chosen by
 * the launcher.  In the reference these are PyTorch's conv2d (cuDNN), bias,
 * GELU and BatchNorm kernels; there is no reference entry point to replace. */
DWB_API int dwb_pointwise_conv_nhwc(const void* x, const void* w, const void* bias,
                                    const void* scale, const void* shift, void* y,
                                    int64_t pixels, int64_t C_in, int64_t C_out, int act,
                                    int tile_n, void* stream);

/* ---- reference-facing entry points --------------------------------------
 * One per launcher of luckychen/depthwise_conv on this path, with the same
 * argument meaning.  Where the reference loops over the batch in Python
 * (depthwise_torch_ops.py:113,122,131) the batch B is passed here instead and
 * all images run in one launch.  A shape that does not match the launcher's
 * fixed (H, W, C, K) returns DWB_ERR_BAD_SHAPE where the reference prints and
 * calls exit(1). */

/* replaces depthwise_forward_32_768_7, convmixer/kernels/depthwise_integration.cu:114-133 */
DWB_API int dwb_depthwise_forward_32_768_7(const void* input, const void* weight, void* output,
                                   int tensorHeight, int tensorWidth, int Ch,
                                   int windowSize, int B, void* stream);

/* replaces depthwise_forward_32_1536_9, convmixer/kernels/depthwise_integration.cu:398-421 */
DWB_API int dwb_depthwise_forward_32_1536_9(const void* input, const void* weight, void* output,
                                    int tensorHeight, int tensorWidth, int Ch,
                                    int windowSize, int B, int batchStride,
                                    void* stream);

/* replaces depthwise_forward_32_1536_9_v2, convmixer/kernels/depthwise_integration.cu:707-730 */
DWB_API int dwb_depthwise_forward_32_1536_9_v2(const void* input, const void* weight, void* output,
                                       int tensorHeight, int tensorWidth, int Ch,
                                       int windowSize, int B, int batchStride,
                                       void* stream);

/* replaces depthwise_forward_16_1536_9, convmixer/kernels/depthwise_integration.cu:984-1003 */
DWB_API int dwb_depthwise_forward_16_1536_9(const void* input, const void* weight, void* output,
                                    int tensorHeight, int tensorWidth, int Ch,
                                    int windowSize, int B, void* stream);

/* replaces depthwise_forward_32_1536_13, convmixer/kernels/depthwise_integration.cu:1013-1030
 * (a stub that exits in the reference; implemented here) */
DWB_API int dwb_depthwise_forward_32_1536_13(const void* input, const void* weight, void* output,
                                     int tensorHeight, int tensorWidth, int Ch,
                                     int windowSize, int B, void* stream);

/* replaces depthwise_31x31_128_nhwc, replknet/kernels/depthwise_replknet_nhwc_integration.cu:60-98
 * bias may be NULL (the reference's empty-tensor case, :73); the bias add is
 * fused instead of the reference's separate bias_add_nhwc_kernel (:23-28). */
DWB_API int dwb_depthwise_31x31_128_nhwc(const void* input, const void* weight, const void* bias,
                                 void* output, int B, int C, int H, int W, void* stream);

/* replaces depthwise_29x29_256_nhwc, replknet/kernels/depthwise_replknet_nhwc_integration.cu:103-141 */
DWB_API int dwb_depthwise_29x29_256_nhwc(const void* input, const void* weight, const void* bias,
                                 void* output, int B, int C, int H, int W, void* stream);

/* replaces depthwise_27x27_512_nhwc, replknet/kernels/depthwise_replknet_nhwc_integration.cu:146-184 */
DWB_API int dwb_depthwise_27x27_512_nhwc(const void* input, const void* weight, const void* bias,
                                 void* output, int B, int C, int H, int W, void* stream);

/* ---- gradients ---------------------------------------------------------------
 * No counterpart in the reference, whose ops are inference-only
 * (convmixer/kernels/depthwise_torch_ops.py:157-159).  Same layouts as the
 * forward: x, dy, dx NHWC fp16; w [K][K][C] fp16. */

/* w_rot180[kh][kw][c] = w[K-1-kh][K-1-kw][c] (C % 8 == 0, 16-byte aligned). */
DWB_API int dwb_weight_rot180(const void* w, void* w_rot180, int64_t C, int K, void* stream);

/* Input gradient: dx = depthwise conv of dy with w_rot180 (from dwb_weight_rot180);
 * the forward kernel and plan, mixed accumulation. */
DWB_API int dwb_conv2d_nhwc_bwd_data(const void* dy, const void* w_rot180, void* dx, int64_t B, int64_t H,
                                     int64_t W, int64_t C, int K, void* stream);

/* Weight gradient, accumulated in fp32: dw[kh][kw][c] += sum over b, h, w of
 * dy[b][h][w][c] * x[b][h+kh-K/2][w+kw-K/2][c].  dw is [K][K][C] fp32 (8-byte
 * aligned); zero it first for a plain gradient.  The summation order (atomic
 * adds of per-warp partial sums) is not fixed, so results may differ in the
 * last bits between calls. */
DWB_API int dwb_conv2d_nhwc_bwd_weight(const void* x, const void* dy, float* dw, int64_t B, int64_t H, int64_t W,
                                       int64_t C, int K, void* stream);

/* The weight gradient with a fixed summation order (the same bits on every
 * run, as torch.use_deterministic_algorithms asks): every CTA warp writes its
 * partial sums to its own slice of `workspace` (fp32, 16-byte aligned, at
 * least the size dwb_conv2d_nhwc_bwd_weight_workspace reports for the
 * problem on the current device) instead of adding them into dw atomically,
 * and a second kernel adds the slices into dw in slice order.  dw: [K][K][C]
 * fp32, 16-byte aligned, accumulated into as by dwb_conv2d_nhwc_bwd_weight. */
DWB_API int dwb_conv2d_nhwc_bwd_weight_workspace(int64_t B, int64_t H, int64_t W, int64_t C, int K,
                                                 int64_t* bytes);
DWB_API int dwb_conv2d_nhwc_bwd_weight_det(const void* x, const void* dy, float* dw, void* workspace,
                                           int64_t workspace_bytes, int64_t B, int64_t H, int64_t W,
                                           int64_t C, int K, void* stream);

/* Input gradient that allocates nothing (no counterpart in the reference): the
 * same result as dwb_weight_rot180 + dwb_conv2d_nhwc_bwd_data, for callers
 * that cannot allocate device memory where they need it (a serving loop with
 * memory fixed after warm-up, a framework that owns every allocation).  Takes
 * the unrotated w; the rotated taps go to a 4 MiB buffer built into the
 * library (every GPU that loads the library holds it until exit), so K*K*C
 * must be at most 2097152 (DWB_ERR_BAD_SHAPE and a dwb_last_error message
 * otherwise).  The first call on a device looks up the buffer's address
 * (cudaGetSymbolAddress): make that first call before any stream capture
 * (a lookup that fails is not remembered; the next call tries again).
 * All calls share the buffer: calls on one device whose work overlaps on the
 * GPU race on it. */
DWB_API int dwb_conv2d_nhwc_bwd_data_noalloc(const void* dy, const void* w, void* dx, int64_t B, int64_t H,
                                             int64_t W, int64_t C, int K, void* stream);

/* ---- diagnostics ----------------------------------------------------------- */

/* Read (and optionally clear) the device-side error word of the current
 * device: 0 = no error, otherwise a code set by a kernel whose bounded
 * mbarrier wait expired.  Synchronises the given stream first. */
DWB_API int dwb_device_error(int* code_out, int clear, void* stream);

/* Self-test of the failure path: launch a one-warp kernel whose bounded
 * mbarrier wait can never complete, with a limit of limit_cycles clock
 * cycles (1 .. 2e9).  The wait expires, the kernel records code 5 in the
 * device error word (read it with dwb_device_error) and returns; the context
 * stays usable.  No counterpart in the reference, whose kernels have no
 * waits. */
DWB_API int dwb_selftest_bounded_wait(int64_t limit_cycles, void* stream);

/* Measure the CUDA-core FMA rate of the current device with a short
 * microbenchmark (fp16x2 HFMA2 and fp32x2 FFMA2), in TFLOP/s. */
DWB_API int dwb_probe_fma_peak(double* hfma2_tflops, double* ffma2_tflops, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DWCONV_B200_H */
