// dw_capi.cu -- the C ABI of the engine (include/dwconv_b200.h): argument
// validation, planning, TMA descriptor encoding and kernel launch.
//
// Nothing here allocates device memory, synchronises (except the explicit
// diagnostics call) or launches on any stream but the caller's.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/dwconv_b200.h"
#include "dw_backward.h"
#include "dw_kernel.cuh"
#include "dw_launch.h"
#include "dw_planner.h"
#include "dw_pointwise_gemm.h"

namespace dwb {

// ---- variant registry --------------------------------------------------------
#define DWB_DECLARE_TABLE(K)             \
  extern const KernelEntry kTableK##K[]; \
  extern const int kCountK##K;
DWB_DECLARE_TABLE(1)
DWB_DECLARE_TABLE(3)
DWB_DECLARE_TABLE(5)
DWB_DECLARE_TABLE(7)
DWB_DECLARE_TABLE(9)
DWB_DECLARE_TABLE(11)
DWB_DECLARE_TABLE(13)
DWB_DECLARE_TABLE(15)
DWB_DECLARE_TABLE(17)
DWB_DECLARE_TABLE(19)
DWB_DECLARE_TABLE(21)
DWB_DECLARE_TABLE(23)
DWB_DECLARE_TABLE(25)
DWB_DECLARE_TABLE(27)
DWB_DECLARE_TABLE(29)
DWB_DECLARE_TABLE(31)

int kernels_for_k(int K, const KernelEntry** out) {
  switch (K) {
#define DWB_CASE(KK)       \
  case KK:                 \
    *out = kTableK##KK;    \
    return kCountK##KK;
    DWB_CASE(1) DWB_CASE(3) DWB_CASE(5) DWB_CASE(7) DWB_CASE(9) DWB_CASE(11) DWB_CASE(13) DWB_CASE(15)
    DWB_CASE(17) DWB_CASE(19) DWB_CASE(21) DWB_CASE(23) DWB_CASE(25) DWB_CASE(27) DWB_CASE(29) DWB_CASE(31)
#undef DWB_CASE
    default:
      *out = nullptr;
      return 0;
  }
}

static const KernelEntry* find_variant(int K, int R, int M, int acc, int pre) {
  const KernelEntry* tab = nullptr;
  const int n = kernels_for_k(K, &tab);
  for (int i = 0; i < n; ++i)
    if (tab[i].r == R && tab[i].m == M && tab[i].acc == acc && tab[i].pre == pre) return &tab[i];
  return nullptr;
}

// Self-test of the bounded-wait path: one thread waits on an mbarrier that
// nothing ever arrives at.  The wait gives up after `limit` cycles, records
// code 5 in the device error word and the kernel returns normally, so the
// context stays usable -- the same path a kernel takes when its data never
// arrives.
__global__ void bounded_wait_selftest(int* err, long long limit) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    (void)mbar_wait_bounded(&bar, 0u, err, 5, limit);
  }
}

// ---- per-device state -----------------------------------------------------------
// The device error word: written by kernels whose bounded waits expire.
static __device__ int g_device_error;

constexpr int kMaxDevices = 64;
constexpr int kMaxVariants = 2 * 16 * kNumVariantR * 8;  // (tile, band) x K values x R x M x accum x load schedule

struct VariantState {
  int regs = -1;         // -1 unknown, 0 unavailable
  bool smem_set = false;
  int smem_max = 0;
  int occ_threads = 0, occ_smem = -1, occ_ctas = 0;  // last occupancy query
};

// B, H, W, C, K, accum, residual is the input (a ConvMixer block)
using PlanKey = std::tuple<long long, long long, long long, long long, int, int, int>;

struct DeviceState {
  std::once_flag once;
  int status = DWB_ERR_NO_DEVICE;
  HwInfo hw;
  int* err_word = nullptr;
  std::mutex mu;
  VariantState variants[kMaxVariants];
  std::mutex plan_mu;
  std::map<PlanKey, dwb_plan> plans;  // planner results, computed once per problem
};

// Last CUDA failure of this thread, for dwb_last_error().
static thread_local char g_last_error[256] = "";

static int cuda_fail(const char* what, cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
  return DWB_ERR_CUDA;
}

static int driver_fail(const char* what, int code) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: CUresult %d", what, code);
  return DWB_ERR_CUDA;
}

static DeviceState g_devices[kMaxDevices];

static int variant_slot(int K, int R, int M, int acc, int pre, bool band = false) {
  int ri = 0;
  for (; ri < kNumVariantR - 1; ++ri)
    if (kVariantR[ri] == R) break;
  const int mi = (M == 2) ? 0 : 1;
  return (((band ? 16 : 0) + K / 2) * kNumVariantR + ri) * 8 + mi * 4 + acc * 2 + (pre ? 1 : 0);
}

static void init_device(int dev, DeviceState* st) {
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) {
    st->status = cuda_fail("cudaDeviceGetAttribute", e);
    return;
  }
  if (major != 10) {  // the library is built for sm_100a only
    st->status = DWB_ERR_NO_DEVICE;
    return;
  }
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  st->hw.sm_count = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  st->hw.smem_optin = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  st->hw.smem_per_sm = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrReservedSharedMemoryPerBlock, dev);
  st->hw.smem_reserved = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
  st->hw.regs_per_sm = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
  st->hw.max_threads_sm = v;
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_device_error);
  if (e != cudaSuccess) {
    st->status = cuda_fail("cudaGetSymbolAddress(g_device_error)", e);
    return;
  }
  st->err_word = static_cast<int*>(p);
  st->status = DWB_OK;
}

static int get_device_state(DeviceState** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DWB_ERR_NO_DEVICE;
  DeviceState* st = &g_devices[dev];
  std::call_once(st->once, init_device, dev, st);
  *out = st;
  return st->status;
}

static int regs_of_variant(int K, int R, int M, int acc, int pre, void* ctx) {
  DeviceState* st = static_cast<DeviceState*>(ctx);
  const KernelEntry* e = find_variant(K, R, M, acc, pre);
  if (!e) return 0;
  VariantState& vs = st->variants[variant_slot(K, R, M, acc, pre)];
  std::lock_guard<std::mutex> lk(st->mu);
  if (vs.regs < 0) {
    cudaFuncAttributes fa;
    vs.regs = (cudaFuncGetAttributes(&fa, e->fn) == cudaSuccess) ? fa.numRegs : 0;
  }
  return vs.regs;
}

static int ensure_smem_attr(DeviceState* st, const KernelEntry* e, bool band, int smem) {
  VariantState& vs = st->variants[variant_slot(e->k, e->r, e->m, e->acc, e->pre, band)];
  std::lock_guard<std::mutex> lk(st->mu);
  if (vs.smem_max >= smem) return DWB_OK;
  const cudaError_t ce =
      cudaFuncSetAttribute(band ? e->band : e->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (ce != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(MaxDynamicSharedMemorySize)", ce);
  vs.smem_max = smem;
  return DWB_OK;
}

// ---- TMA descriptors ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// x: NHWC fp16 viewed as (C, W, H, B); box = 64 channels x tile_w_in columns x 1 row.
static int encode_x_map(CUtensorMap* m, const void* x, long long B, long long H, long long W, long long C,
                        int tile_w_in) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return driver_fail("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", -1);
  const cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)(C * 2), (cuuint64_t)(W * C * 2), (cuuint64_t)(H * W * C * 2)};
  const cuuint32_t box[4] = {(cuuint32_t)kChannelsPerCta, (cuuint32_t)tile_w_in, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DWB_OK : driver_fail("cuTensorMapEncodeTiled(x)", static_cast<int>(r));
}

// w: [K][K][C] fp16 viewed as (C, K, K); box = 64 channels x K taps x `rows` kernel rows
// (1: one weight row per stage; K: all of a channel block's taps at once, band mode).
static int encode_w_map(CUtensorMap* m, const void* w, long long C, int K, int rows = 1) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return driver_fail("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", -1);
  const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)K, (cuuint64_t)K};
  const cuuint64_t strides[2] = {(cuuint64_t)(C * 2), (cuuint64_t)(K * C * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)kChannelsPerCta, (cuuint32_t)K, (cuuint32_t)rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DWB_OK : driver_fail("cuTensorMapEncodeTiled(w)", static_cast<int>(r));
}

static inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Argument checks shared by every entry point (no CUDA calls).  An empty
// batch is accepted before the pointer checks: an empty tensor may report a
// null data pointer.
static int validate_args(const void* x, const void* w, const void* bias, const void* scale, const void* shift,
                         const void* residual, const void* y, long long B, long long H, long long W, long long C,
                         int K, int act, int accum) {
  if (act < DWB_ACT_NONE || act > DWB_ACT_GELU) return DWB_ERR_BAD_ARG;
  if (accum != DWB_ACCUM_F32 && accum != DWB_ACCUM_MIXED) return DWB_ERR_BAD_ARG;
  if (B < 0 || H < 1 || W < 1 || C < 1 || K < 1 || K > 31 || (K % 2) == 0 || (C % 8) != 0) return DWB_ERR_BAD_SHAPE;
  if (B == 0) return DWB_OK;
  if (!x || !w || !y) return DWB_ERR_NULL_POINTER;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16)) return DWB_ERR_BAD_ALIGN;
  if ((bias && !aligned(bias, 4)) || (scale && !aligned(scale, 4)) || (shift && !aligned(shift, 4)) ||
      (residual && !aligned(residual, 4)))
    return DWB_ERR_BAD_ALIGN;
  return DWB_OK;
}

static dwb_problem make_problem(long long B, long long H, long long W, long long C, int K, int accum) {
  dwb_problem pr;
  pr.batch = B;
  pr.height = H;
  pr.width = W;
  pr.channels = C;
  pr.kernel_size = K;
  pr.accum = accum;
  return pr;
}

// Launch one plan (already checked against the problem).
static int launch_plan(DeviceState* st, const dwb_plan& plan, const void* x, const void* w, const void* bias,
                       const void* scale, const void* shift, const void* residual, void* y, long long B, long long H,
                       long long W, long long C, int K, int act, void* stream) {
  const KernelEntry* e = find_variant(K, plan.cols_per_thread, plan.rows_per_thread, plan.accum, plan.load_schedule);
  if (!e) return DWB_ERR_UNSUPPORTED;
  const bool band = plan.band_tiles > 0;
  if (band && !e->band) return DWB_ERR_UNSUPPORTED;
  const void* fn = band ? e->band : e->fn;
  int rc = ensure_smem_attr(st, e, band, plan.smem_bytes);
  if (rc != DWB_OK) return rc;

  CUtensorMap tmx, tmw;
  rc = encode_x_map(&tmx, x, B, H, W, C, plan.tile_w_in);
  if (rc != DWB_OK) return rc;
  rc = encode_w_map(&tmw, w, C, K, band ? K : 1);
  if (rc != DWB_OK) return rc;

  DwParams p;
  p.y = static_cast<__half*>(y);
  p.bias = static_cast<const __half*>(bias);
  p.scale = static_cast<const __half*>(scale);
  p.shift = static_cast<const __half*>(shift);
  p.residual = static_cast<const __half*>(residual);
  p.B = static_cast<int>(B);
  p.H = static_cast<int>(H);
  p.W = static_cast<int>(W);
  p.C = static_cast<int>(C);
  p.tile_h = plan.tile_h;
  p.tile_w = plan.tile_w;
  p.tile_w_in = plan.tile_w_in;
  p.tiles_h = static_cast<int>((H + plan.tile_h - 1) / plan.tile_h);
  p.tiles_w = static_cast<int>((W + plan.tile_w - 1) / plan.tile_w);
  p.cblocks = static_cast<int>((C + kChannelsPerCta - 1) / kChannelsPerCta);
  if (plan.tiles > 0x7fffffffLL) return DWB_ERR_BAD_SHAPE;
  p.num_tiles = static_cast<uint32_t>(plan.tiles);
  p.ncg = plan.tile_w / plan.cols_per_thread;
  p.nsplit = plan.row_splits > 1 ? plan.row_splits : 1;
  p.slots = p.ncg * (plan.tile_h / plan.rows_per_thread);
  p.consumer_warps = plan.consumer_warps;
  if (p.consumer_warps != p.nsplit * p.slots) return DWB_ERR_BAD_ARG;
  p.stages = plan.ring_rows;
  p.act = act;
  p.ring_off = kBarrierBytes;
  // a stage holds one staged input row (band mode) or an input row and a weight row
  p.stage_bytes = static_cast<uint32_t>(plan.tile_w_in + (band ? 0 : K)) * kPixelBytes;
  long long red_off = 0, wbuf_off = 0;
  const long long smem_need =
      band ? band_smem_bytes(K, plan.tile_w_in, plan.ring_rows, p.nsplit, p.slots, plan.rows_per_thread,
                             plan.cols_per_thread, &red_off, &wbuf_off)
           : plan_smem_bytes(K, plan.tile_w_in, plan.ring_rows, p.nsplit, p.slots, plan.rows_per_thread,
                             plan.cols_per_thread, &red_off);
  if (smem_need > plan.smem_bytes) return DWB_ERR_BAD_ARG;
  p.red_off = static_cast<uint32_t>(red_off);
  p.wbuf_off = static_cast<uint32_t>(wbuf_off);
  p.band_tiles = band ? plan.band_tiles : 0;
  p.bands_h = band ? static_cast<int>((p.tiles_h + plan.band_tiles - 1) / plan.band_tiles) : 0;
  p.num_bands = band ? static_cast<uint32_t>(plan.tiles) : 0u;
  p.err = st->err_word;
  p.res_in_ring = 0;  // set below, once the grid is known

  // grid < 0: persistent, as many CTAs as fit on the device at once (measured
  // by the occupancy calculator for this variant); otherwise the plan's CTA
  // count (one tile per CTA when it equals the tile count).
  long long grid = plan.grid;
  {
    VariantState& vs = st->variants[variant_slot(e->k, e->r, e->m, e->acc, e->pre, band)];
    std::lock_guard<std::mutex> lk(st->mu);
    if (vs.occ_threads != plan.threads || vs.occ_smem != plan.smem_bytes) {
      int occ = 0;
      const cudaError_t oe =
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, plan.threads, static_cast<size_t>(plan.smem_bytes));
      if (oe != cudaSuccess) return cuda_fail("cudaOccupancyMaxActiveBlocksPerMultiprocessor", oe);
      vs.occ_threads = plan.threads;
      vs.occ_smem = plan.smem_bytes;
      vs.occ_ctas = occ;
    }
    if (vs.occ_ctas < 1) return DWB_ERR_UNSUPPORTED;
    const long long fit = static_cast<long long>(vs.occ_ctas) * st->hw.sm_count;
    if (grid < 0) grid = fit;
    if (grid <= 0 || grid > plan.tiles) grid = plan.tiles;
  }

  // A ConvMixer block's residual is the convolution's own input: when every CTA runs exactly one
  // tile and the ring holds all of that tile's input rows (nothing is ever refilled), the epilogue
  // reads it from shared memory.
  p.res_in_ring = (!band && residual != nullptr && residual == x && grid == plan.tiles &&
                   plan.ring_rows >= plan.tile_h + K - 1) ? 1 : 0;
  void* args[3] = {&tmx, &tmw, &p};
  const cudaError_t ce = launch_kernel(fn, dim3(static_cast<unsigned>(grid)), dim3(plan.threads), args,
                                       static_cast<size_t>(plan.smem_bytes), static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) {
    (void)cudaGetLastError();
    return cuda_fail(band ? "cudaLaunchKernelExC(dw_band_kernel)" : "cudaLaunchKernelExC(dw_stream_kernel)", ce);
  }
  return DWB_OK;
}

// Plans measured fastest on B200 (depthwise_conv_b200/tune.py).  A problem
// with the same H, W, C, K and accumulation takes the entry with the nearest
// batch (the tile shape does not depend on the batch); the plan is checked
// against this device before use.
struct TunedPlan {
  long long B, H, W, C;
  int K, accum, R, M, tile_h, tile_w, ring_rows, ring_wrows, grid;
  int splits;  // row split (0 or 1 = none)
  int pre;     // load schedule
  int band;    // band mode: row tiles per band (0 = tile mode)
};
static const TunedPlan kTunedPlans[] = {
#include "dw_tuned_plans.inc"
};
// Plans measured fastest for a ConvMixer block (residual = the convolution's input, which the
// epilogue can read from the stage ring when each CTA keeps its tile whole); a launch whose
// residual is its input looks here first.  The zero row only keeps the array non-empty.
static const TunedPlan kTunedResPlans[] = {
#include "dw_tuned_plans_res.inc"
    {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0}};

static bool tuned_plan(DeviceState* st, const dwb_problem& pr, dwb_plan* out, bool res_input = false) {
  const TunedPlan* best = nullptr;
  long long best_d = 0;
  const TunedPlan* tables[2] = {kTunedPlans, kTunedResPlans};
  const size_t sizes[2] = {sizeof(kTunedPlans) / sizeof(TunedPlan), sizeof(kTunedResPlans) / sizeof(TunedPlan)};
  for (int ti = res_input ? 1 : 0; ti >= 0 && !best; --ti)
  for (size_t i = 0; i < sizes[ti]; ++i) {
    const TunedPlan& t = tables[ti][i];
    if (t.B == 0 || t.H != pr.height || t.W != pr.width || t.C != pr.channels || t.K != pr.kernel_size ||
        t.accum != pr.accum)
      continue;
    const long long d = t.B > pr.batch ? t.B - pr.batch : pr.batch - t.B;
    if (!best || d < best_d) {
      best = &t;
      best_d = d;
    }
  }
  if (!best) return false;
  dwb_plan p;
  std::memset(&p, 0, sizeof(p));
  p.kernel_size = best->K;
  p.accum = best->accum;
  p.cols_per_thread = best->R;
  p.rows_per_thread = best->M;
  p.tile_h = best->tile_h;
  p.tile_w = best->tile_w;
  p.ring_rows = best->ring_rows;
  p.ring_wrows = best->ring_wrows;
  p.grid = best->grid;
  p.row_splits = best->splits;
  p.load_schedule = best->pre;
  p.band_tiles = best->band;
  const int regs = regs_of_variant(p.kernel_size, p.cols_per_thread, p.rows_per_thread, p.accum, p.load_schedule, st);
  if (regs <= 0 || check_plan(pr, st->hw, regs, &p) != DWB_OK) return false;
  p.ctas_per_sm = 0;  // not modelled for tuned plans
  *out = p;
  return true;
}

// The plan for a problem on this device (tuned table, else the planner's
// cost model), computed once.
static int cached_plan(DeviceState* st, const dwb_problem& pr, dwb_plan* out, bool res_input = false) {
  const PlanKey key{pr.batch, pr.height, pr.width, pr.channels, pr.kernel_size, pr.accum, res_input ? 1 : 0};
  {
    std::lock_guard<std::mutex> lk(st->plan_mu);
    auto it = st->plans.find(key);
    if (it != st->plans.end()) {
      *out = it->second;
      return DWB_OK;
    }
  }
  if (!tuned_plan(st, pr, out, res_input)) {
    const int rc = plan_problem(pr, st->hw, regs_of_variant, st, out);
    if (rc != DWB_OK) return rc;
    out->grid = -1;  // persistent
  }
  std::lock_guard<std::mutex> lk(st->plan_mu);
  if (st->plans.size() > 4096) st->plans.clear();  // bound the cache
  st->plans[key] = *out;
  return DWB_OK;
}

// The single planner-driven launch path behind every entry point.
static int launch_forward(const void* x, const void* w, const void* bias, const void* scale, const void* shift,
                          const void* residual, void* y, long long B, long long H, long long W, long long C, int K,
                          int act, int accum, void* stream) {
  int rc = validate_args(x, w, bias, scale, shift, residual, y, B, H, W, C, K, act, accum);
  if (rc != DWB_OK || B == 0) return rc;
  DeviceState* st = nullptr;
  rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  dwb_plan plan;
  rc = cached_plan(st, make_problem(B, H, W, C, K, accum), &plan, residual != nullptr && residual == x);
  if (rc != DWB_OK) return rc;
  return launch_plan(st, plan, x, w, bias, scale, shift, residual, y, B, H, W, C, K, act, stream);
}

// Shared by the fixed-shape reference launchers.
static int fixed_shape(int H, int W, int C, int K, int eH, int eW, int eC, int eK) {
  return (H == eH && W == eW && C == eC && K == eK) ? DWB_OK : DWB_ERR_BAD_SHAPE;
}

}  // namespace dwb

using namespace dwb;

extern "C" {

int dwb_abi_version(void) { return DWB_ABI_VERSION; }

const char* dwb_status_string(int status) {
  switch (status) {
    case DWB_OK: return "ok";
    case DWB_ERR_NULL_POINTER: return "a required pointer is NULL";
    case DWB_ERR_BAD_SHAPE: return "shape outside the supported range or not the launcher's fixed shape";
    case DWB_ERR_BAD_ALIGN: return "pointer not aligned (x, w, y need 16 bytes; bias/scale/shift/residual 4 bytes)";
    case DWB_ERR_UNSUPPORTED: return "no compiled kernel variant fits this problem";
    case DWB_ERR_CUDA: return "a CUDA runtime or driver call failed";
    case DWB_ERR_NO_DEVICE: return "no usable sm_100 device is current";
    case DWB_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired (device error word set)";
    case DWB_ERR_BAD_ARG: return "an enum or flag argument is out of range";
    default: return "unknown status";
  }
}

int dwb_plan_query(const dwb_problem* problem, int sm_count, int smem_optin_bytes, dwb_plan* plan_out) {
  if (!problem || !plan_out) return DWB_ERR_NULL_POINTER;
  HwInfo hw;
  if (sm_count > 0) hw.sm_count = sm_count;
  if (smem_optin_bytes > 0) hw.smem_optin = smem_optin_bytes;
  return plan_problem(*problem, hw, nullptr, nullptr, plan_out);
}

namespace {
struct CandSink {
  dwb_plan* out;
  int cap;
  int n;
};
void collect(const dwb_plan& p, void* vctx) {
  CandSink* c = static_cast<CandSink*>(vctx);
  if (c->n < c->cap) c->out[c->n] = p;
  ++c->n;
}
}  // namespace

int dwb_plan_candidates(const dwb_problem* problem, int sm_count, int smem_optin_bytes, dwb_plan* plans_out,
                        int capacity, int* count_out) {
  if (!problem || !count_out || (capacity > 0 && !plans_out)) return DWB_ERR_NULL_POINTER;
  HwInfo hw;
  if (sm_count > 0) hw.sm_count = sm_count;
  if (smem_optin_bytes > 0) hw.smem_optin = smem_optin_bytes;
  CandSink c{plans_out, capacity, 0};
  const int rc = enumerate_plans(*problem, hw, nullptr, nullptr, collect, &c);
  *count_out = c.n;
  return rc;
}

const char* dwb_last_error(void) { return g_last_error; }

int dwb_plan_select(const dwb_problem* problem, dwb_plan* plan_out) {
  if (!problem || !plan_out) return DWB_ERR_NULL_POINTER;
  int rc = validate_problem(*problem);
  if (rc != DWB_OK) return rc;
  DeviceState* st = nullptr;
  rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  return cached_plan(st, *problem, plan_out);
}

int dwb_conv2d_nhwc_fwd_planned(const void* x, const void* w, const void* bias, const void* scale, const void* shift,
                                const void* residual, void* y, int64_t B, int64_t H, int64_t W, int64_t C, int K,
                                int act, const dwb_plan* plan, void* stream) {
  if (!plan) return DWB_ERR_NULL_POINTER;
  int rc = validate_args(x, w, bias, scale, shift, residual, y, B, H, W, C, K, act, plan->accum);
  if (rc != DWB_OK || B == 0) return rc;
  DeviceState* st = nullptr;
  rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  dwb_plan p = *plan;
  const int regs = regs_of_variant(K, p.cols_per_thread, p.rows_per_thread, p.accum, p.load_schedule, st);
  if (regs <= 0) return DWB_ERR_UNSUPPORTED;
  rc = check_plan(make_problem(B, H, W, C, K, p.accum), st->hw, regs, &p);
  if (rc != DWB_OK) return rc;
  return launch_plan(st, p, x, w, bias, scale, shift, residual, y, B, H, W, C, K, act, stream);
}

int dwb_conv2d_nhwc_fwd(const void* x, const void* w, void* y, int64_t B, int64_t H, int64_t W, int64_t C, int K,
                        void* stream) {
  return launch_forward(x, w, nullptr, nullptr, nullptr, nullptr, y, B, H, W, C, K, DWB_ACT_NONE, DWB_ACCUM_DEFAULT,
                        stream);
}

int dwb_conv2d_nhwc_bwd_data(const void* dy, const void* w_rot180, void* dx, int64_t B, int64_t H, int64_t W,
                             int64_t C, int K, void* stream) {
  // "same" padding with an odd K: the adjoint of the convolution is the convolution with the taps
  // rotated by 180 degrees, so the forward kernel computes the input gradient.
  return launch_forward(dy, w_rot180, nullptr, nullptr, nullptr, nullptr, dx, B, H, W, C, K, DWB_ACT_NONE,
                        DWB_ACCUM_DEFAULT, stream);
}

// Grid of the weight-gradient kernel: CTA = (64 channels, kernel row, column tile, chunk of rows);
// up to 4 consumer warps of 16 columns; chunks sized for ~4 CTAs per SM.
struct WgradGeometry {
  int ncw, tile_w;
  long long col_tiles, cblocks, chunks, rows_per_chunk;
};
static int wgrad_geometry(long long B, long long H, long long W, long long C, int K, int sm_count, WgradGeometry* g) {
  if (B < 0 || H < 1 || W < 1 || C < 8 || (C % 8) != 0 || K < 1 || K > 31 || (K % 2) == 0) return DWB_ERR_BAD_SHAPE;
  if (H > (1 << 30) || W > (1 << 30) || C > (1 << 30) || B > (1 << 30)) return DWB_ERR_BAD_SHAPE;
  g->ncw = static_cast<int>(std::min<long long>(4, (W + kWgradColumnsPerWarp - 1) / kWgradColumnsPerWarp));
  g->tile_w = g->ncw * kWgradColumnsPerWarp;
  g->col_tiles = (W + g->tile_w - 1) / g->tile_w;
  g->cblocks = (C + kChannelsPerCta - 1) / kChannelsPerCta;
  const long long rows = std::max<long long>(1, B * H);
  const long long base = g->cblocks * K * g->col_tiles;
  long long chunks = (4LL * sm_count + base - 1) / base;
  chunks = std::max<long long>(1, std::min(chunks, rows));
  g->rows_per_chunk = (rows + chunks - 1) / chunks;
  g->chunks = (rows + g->rows_per_chunk - 1) / g->rows_per_chunk;
  if (g->cblocks > 0x7fffffffLL || g->col_tiles * g->chunks > 65535) return DWB_ERR_BAD_SHAPE;
  return DWB_OK;
}

// The deterministic mode's workspace: one fp32 [K][K][C] slice per (row chunk, column tile, warp).
static long long wgrad_workspace_bytes(const WgradGeometry& g, long long C, int K) {
  return g.col_tiles * g.chunks * g.ncw * static_cast<long long>(K) * K * C * 4;
}

static int launch_wgrad(const void* x, const void* dy, float* dw, void* workspace, long long workspace_bytes,
                        long long B, long long H, long long W, long long C, int K, void* stream) {
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  WgradGeometry g;
  rc = wgrad_geometry(B, H, W, C, K, st->hw.sm_count, &g);
  if (rc != DWB_OK || B == 0) return rc;
  const void* fn = wgrad_kernel_for(K);
  if (!fn) return DWB_ERR_UNSUPPORTED;
  if (workspace && workspace_bytes < wgrad_workspace_bytes(g, C, K)) return DWB_ERR_BAD_ARG;

  WgradParams p;
  p.dw = dw;
  p.B = static_cast<int>(B);
  p.H = static_cast<int>(H);
  p.W = static_cast<int>(W);
  p.C = static_cast<int>(C);
  p.tile_w = g.tile_w;
  p.col_tiles = static_cast<int>(g.col_tiles);
  p.rows_per_chunk = g.rows_per_chunk;
  p.consumer_warps = g.ncw;
  p.stages = 4;
  p.ring_off = kBarrierBytes;
  p.stage_bytes = static_cast<uint32_t>(2 * g.tile_w + K - 1) * kPixelBytes;
  p.partial = static_cast<float*>(workspace);
  p.err = st->err_word;
  const int smem = static_cast<int>(p.ring_off + p.stages * p.stage_bytes);
  {
    static int smem_set[kMaxDevices][32];  // largest dynamic smem allowed so far, per device and K
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(st->mu);
    if (smem_set[dev][K] < smem) {
      const cudaError_t ce = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (ce != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(dw_wgrad_kernel)", ce);
      smem_set[dev][K] = smem;
    }
  }
  CUtensorMap tmx, tmdy;
  rc = encode_x_map(&tmx, x, B, H, W, C, g.tile_w + K - 1);
  if (rc != DWB_OK) return rc;
  rc = encode_x_map(&tmdy, dy, B, H, W, C, g.tile_w);
  if (rc != DWB_OK) return rc;
  void* args[3] = {&tmx, &tmdy, &p};
  cudaError_t ce = launch_kernel(fn, dim3(static_cast<unsigned>(g.cblocks), K, static_cast<unsigned>(g.col_tiles * g.chunks)),
                                 dim3(32 * (g.ncw + 1)), args, static_cast<size_t>(smem), static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) {
    (void)cudaGetLastError();
    return cuda_fail("cudaLaunchKernelExC(dw_wgrad_kernel)", ce);
  }
  if (workspace) {  // the slices, summed in a fixed order
    const float4* part = static_cast<const float4*>(workspace);
    float4* out = reinterpret_cast<float4*>(dw);
    long long n4 = static_cast<long long>(K) * K * C / 4;
    int slices = static_cast<int>(g.col_tiles * g.chunks * g.ncw);
    const long long want = (n4 + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(std::min<long long>(want, 8LL * st->hw.sm_count));
    void* rargs[4] = {&part, &out, &n4, &slices};
    ce = launch_kernel(wgrad_reduce_kernel_fn(), dim3(blocks), dim3(256), rargs, 0, static_cast<cudaStream_t>(stream));
    if (ce != cudaSuccess) {
      (void)cudaGetLastError();
      return cuda_fail("cudaLaunchKernelExC(wgrad_reduce_kernel)", ce);
    }
  }
  return DWB_OK;
}

int dwb_conv2d_nhwc_bwd_weight(const void* x, const void* dy, float* dw, int64_t B, int64_t H, int64_t W,
                               int64_t C, int K, void* stream) {
  if (B < 0 || H < 1 || W < 1 || C < 8 || (C % 8) != 0 || K < 1 || K > 31 || (K % 2) == 0)
    return DWB_ERR_BAD_SHAPE;
  if (B == 0) return DWB_OK;
  if (!x || !dy || !dw) return DWB_ERR_NULL_POINTER;
  if (!aligned(x, 16) || !aligned(dy, 16) || !aligned(dw, 8)) return DWB_ERR_BAD_ALIGN;
  return launch_wgrad(x, dy, dw, nullptr, 0, B, H, W, C, K, stream);
}

int dwb_conv2d_nhwc_bwd_weight_workspace(int64_t B, int64_t H, int64_t W, int64_t C, int K, int64_t* bytes) {
  if (!bytes) return DWB_ERR_NULL_POINTER;
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  WgradGeometry g;
  rc = wgrad_geometry(B, H, W, C, K, st->hw.sm_count, &g);
  if (rc != DWB_OK) return rc;
  *bytes = B == 0 ? 0 : wgrad_workspace_bytes(g, C, K);
  return DWB_OK;
}

int dwb_conv2d_nhwc_bwd_weight_det(const void* x, const void* dy, float* dw, void* workspace, int64_t workspace_bytes,
                                   int64_t B, int64_t H, int64_t W, int64_t C, int K, void* stream) {
  if (B < 0 || H < 1 || W < 1 || C < 8 || (C % 8) != 0 || K < 1 || K > 31 || (K % 2) == 0)
    return DWB_ERR_BAD_SHAPE;
  if (B == 0) return DWB_OK;
  if (!x || !dy || !dw || !workspace) return DWB_ERR_NULL_POINTER;
  if (!aligned(x, 16) || !aligned(dy, 16) || !aligned(dw, 16) || !aligned(workspace, 16)) return DWB_ERR_BAD_ALIGN;
  return launch_wgrad(x, dy, dw, workspace, workspace_bytes, B, H, W, C, K, stream);
}

// ---- pointwise block: the fused 1x1-convolution GEMM -------------------------------------
// [rows][cols] fp16 row-major matrix as a 2-D TMA tensor; box = kPwTileK columns (128 bytes) x
// box_rows rows with the 128-byte swizzle the MMA's shared-memory descriptors describe.
static int encode_matrix_map(CUtensorMap* m, const void* base, long long rows, long long cols, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return driver_fail("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", -1);
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kPwTileK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DWB_OK : driver_fail("cuTensorMapEncodeTiled(matrix)", static_cast<int>(r));
}

static bool pw_tile_n_compiled(int bn) {
  for (int v : kPwTileNs)
    if (v == bn) return true;
  return false;
}

// Output channels per tile for an M x N product on `sms` SMs (one CTA per SM): the fewest
// waves of tiles, each costing its BN columns of MMAs plus a fixed ~32-column-equivalent of
// fill and epilogue latency.
static int pw_choose_tile_n(long long M, long long N, int sms) {
  int best = kPwTileNs[0];
  double best_cost = 0.0;
  for (int bn : kPwTileNs) {
    const long long tiles = ((M + kPwTileM - 1) / kPwTileM) * ((N + bn - 1) / bn);
    const long long waves = (tiles + sms - 1) / sms;
    const double cost = static_cast<double>(waves) * (bn + 32.0);
    if (best_cost == 0.0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

int dwb_pointwise_conv_nhwc(const void* x, const void* w, const void* bias, const void* scale, const void* shift,
                            void* y, int64_t pixels, int64_t C_in, int64_t C_out, int act, int tile_n,
                            void* stream) {
  if (act < DWB_ACT_NONE || act > DWB_ACT_GELU) return DWB_ERR_BAD_ARG;
  if (tile_n != 0 && !pw_tile_n_compiled(tile_n)) return DWB_ERR_BAD_ARG;
  if (pixels < 0 || C_in < 8 || (C_in % 8) != 0 || C_out < 8 || (C_out % 8) != 0) return DWB_ERR_BAD_SHAPE;
  if (pixels > 0x7fffff00LL || C_in > (1LL << 24) || C_out > 65535LL * kPwTileNs[0]) return DWB_ERR_BAD_SHAPE;
  if (pixels == 0) return DWB_OK;
  if (!x || !w || !y) return DWB_ERR_NULL_POINTER;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16) || (bias && !aligned(bias, 2)) ||
      (scale && !aligned(scale, 2)) || (shift && !aligned(shift, 2)))
    return DWB_ERR_BAD_ALIGN;
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  const int bn = tile_n ? tile_n : pw_choose_tile_n(pixels, C_out, st->hw.sm_count);
  if ((C_out + bn - 1) / bn > 65535) return DWB_ERR_BAD_SHAPE;
  const void* fn = pw_gemm_kernel_for(bn, act);
  if (!fn) return DWB_ERR_UNSUPPORTED;

  PwGemmParams p;
  p.bias = static_cast<const __half*>(bias);
  p.scale = static_cast<const __half*>(scale);
  p.shift = static_cast<const __half*>(shift);
  p.y = static_cast<__half*>(y);
  p.M = static_cast<int>(pixels);
  p.N = static_cast<int>(C_out);
  p.K = static_cast<int>(C_in);
  p.num_kb = static_cast<int>((C_in + kPwTileK - 1) / kPwTileK);
  int stages = std::min(kPwMaxStages, std::max(2, p.num_kb));
  while (stages > 2 && pw_smem_bytes(bn, stages) > st->hw.smem_optin) --stages;
  if (pw_smem_bytes(bn, stages) > st->hw.smem_optin) return DWB_ERR_UNSUPPORTED;
  p.stages = stages;
  p.err = st->err_word;
  const int smem = pw_smem_bytes(bn, stages);
  {
    static int smem_set[kMaxDevices][4][3];  // largest dynamic smem allowed so far: device, tile_n, act
    int dev = 0, bi = 0;
    cudaGetDevice(&dev);
    while (kPwTileNs[bi] != bn) ++bi;
    std::lock_guard<std::mutex> lk(st->mu);
    if (smem_set[dev][bi][act] < smem) {
      const cudaError_t ce = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (ce != cudaSuccess) return cuda_fail("cudaFuncSetAttribute(pw_gemm_kernel)", ce);
      smem_set[dev][bi][act] = smem;
    }
  }
  CUtensorMap tmx, tmw;
  rc = encode_matrix_map(&tmx, x, pixels, C_in, kPwTileM);
  if (rc != DWB_OK) return rc;
  rc = encode_matrix_map(&tmw, w, C_out, C_in, bn);
  if (rc != DWB_OK) return rc;
  void* args[3] = {&tmx, &tmw, &p};
  const dim3 grid(static_cast<unsigned>((pixels + kPwTileM - 1) / kPwTileM), static_cast<unsigned>((C_out + bn - 1) / bn));
  const cudaError_t ce = launch_kernel(fn, grid, dim3(kPwThreads), args, static_cast<size_t>(smem),
                                       static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) {
    (void)cudaGetLastError();
    return cuda_fail("cudaLaunchKernelExC(pw_gemm_kernel)", ce);
  }
  return DWB_OK;
}

int dwb_conv2d_nhwc_fused_fwd(const void* x, const void* w, const void* bias, const void* scale, const void* shift,
                              const void* residual, void* y, int64_t B, int64_t H, int64_t W, int64_t C, int K,
                              int act, int accum, void* stream) {
  return launch_forward(x, w, bias, scale, shift, residual, y, B, H, W, C, K, act, accum, stream);
}

int dwb_depthwise_forward_32_768_7(const void* input, const void* weight, void* output, int tensorHeight,
                                   int tensorWidth, int Ch, int windowSize, int B, void* stream) {
  int rc = fixed_shape(tensorHeight, tensorWidth, Ch, windowSize, 32, 32, 768, 7);
  if (rc != DWB_OK) return rc;
  return launch_forward(input, weight, nullptr, nullptr, nullptr, nullptr, output, B, 32, 32, 768, 7, DWB_ACT_NONE,
                        DWB_ACCUM_DEFAULT, stream);
}

static int forward_32_1536_9(const void* input, const void* weight, void* output, int tensorHeight, int tensorWidth,
                             int Ch, int windowSize, int B, int batchStride, void* stream) {
  int rc = fixed_shape(tensorHeight, tensorWidth, Ch, windowSize, 32, 32, 1536, 9);
  if (rc != DWB_OK) return rc;
  if (batchStride != 32 * 32 * 1536) return DWB_ERR_BAD_SHAPE;  // images are packed NHWC
  return launch_forward(input, weight, nullptr, nullptr, nullptr, nullptr, output, B, 32, 32, 1536, 9, DWB_ACT_NONE,
                        DWB_ACCUM_DEFAULT, stream);
}

int dwb_depthwise_forward_32_1536_9(const void* input, const void* weight, void* output, int tensorHeight,
                                    int tensorWidth, int Ch, int windowSize, int B, int batchStride, void* stream) {
  return forward_32_1536_9(input, weight, output, tensorHeight, tensorWidth, Ch, windowSize, B, batchStride, stream);
}

int dwb_depthwise_forward_32_1536_9_v2(const void* input, const void* weight, void* output, int tensorHeight,
                                       int tensorWidth, int Ch, int windowSize, int B, int batchStride,
                                       void* stream) {
  return forward_32_1536_9(input, weight, output, tensorHeight, tensorWidth, Ch, windowSize, B, batchStride, stream);
}

int dwb_depthwise_forward_16_1536_9(const void* input, const void* weight, void* output, int tensorHeight,
                                    int tensorWidth, int Ch, int windowSize, int B, void* stream) {
  int rc = fixed_shape(tensorHeight, tensorWidth, Ch, windowSize, 16, 16, 1536, 9);
  if (rc != DWB_OK) return rc;
  return launch_forward(input, weight, nullptr, nullptr, nullptr, nullptr, output, B, 16, 16, 1536, 9, DWB_ACT_NONE,
                        DWB_ACCUM_DEFAULT, stream);
}

int dwb_depthwise_forward_32_1536_13(const void* input, const void* weight, void* output, int tensorHeight,
                                     int tensorWidth, int Ch, int windowSize, int B, void* stream) {
  int rc = fixed_shape(tensorHeight, tensorWidth, Ch, windowSize, 32, 32, 1536, 13);
  if (rc != DWB_OK) return rc;
  return launch_forward(input, weight, nullptr, nullptr, nullptr, nullptr, output, B, 32, 32, 1536, 13,
                        DWB_ACT_NONE, DWB_ACCUM_DEFAULT, stream);
}

static int replknet_forward(const void* input, const void* weight, const void* bias, void* output, int B, int C,
                            int H, int W, int eC, int eHW, int eK, void* stream) {
  if (C != eC || H != eHW || W != eHW) return DWB_ERR_BAD_SHAPE;
  return launch_forward(input, weight, bias, nullptr, nullptr, nullptr, output, B, H, W, C, eK, DWB_ACT_NONE,
                        DWB_ACCUM_DEFAULT, stream);
}

int dwb_depthwise_31x31_128_nhwc(const void* input, const void* weight, const void* bias, void* output, int B, int C,
                                 int H, int W, void* stream) {
  return replknet_forward(input, weight, bias, output, B, C, H, W, 128, 56, 31, stream);
}

int dwb_depthwise_29x29_256_nhwc(const void* input, const void* weight, const void* bias, void* output, int B, int C,
                                 int H, int W, void* stream) {
  return replknet_forward(input, weight, bias, output, B, C, H, W, 256, 28, 29, stream);
}

int dwb_depthwise_27x27_512_nhwc(const void* input, const void* weight, const void* bias, void* output, int B, int C,
                                 int H, int W, void* stream) {
  return replknet_forward(input, weight, bias, output, B, C, H, W, 512, 14, 27, stream);
}

int dwb_selftest_bounded_wait(int64_t limit_cycles, void* stream) {
  if (limit_cycles < 1 || limit_cycles > kWaitLimitCycles) return DWB_ERR_BAD_ARG;
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  bounded_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(st->err_word, limit_cycles);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DWB_OK : cuda_fail("launch(bounded_wait_selftest)", e);
}

int dwb_device_error(int* code_out, int clear, void* stream) {
  if (!code_out) return DWB_ERR_NULL_POINTER;
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != DWB_OK) return rc;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("cudaStreamSynchronize", e);
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_fail("cudaMemcpyFromSymbol(g_device_error)", e);
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail("cudaMemcpyToSymbol(g_device_error)", e);
  }
  *code_out = v;
  return DWB_OK;
}

// ---- input gradient without any allocation ------------------------------------
// Some callers cannot allocate device memory at the point where they need the
// input gradient: code that must not call cudaMalloc there (a serving or
// training loop whose memory is fixed after warm-up, a host framework that
// owns every device allocation and exposes no allocator to its plugins).
// dwb_conv2d_nhwc_bwd_data
// needs a buffer for the rotated taps that its caller allocates; this variant
// keeps them in a buffer compiled into the library instead, so it takes the
// unrotated weights and allocates nothing.
//
// The buffer is a file-scope device array: every GPU that loads the library
// reserves kNoAllocMaxTaps halves (4 MiB) for it until the process exits.  In
// host code its name is only a stand-in for the device symbol, so its device
// address is looked up once per device (cudaGetSymbolAddress, the device
// current) on the first call of this entry point on that device.  All calls
// share the one buffer: each call overwrites the K*K*C entries it uses before
// reading them (nothing needs to start at zero), and calls on one device whose
// work overlaps on the GPU (for example on two streams) race on it: order them.
// Only a successful lookup is remembered: a lookup that failed (for example one
// attempted during a stream capture) is tried again by the next call.
constexpr long long kNoAllocMaxTaps = 1LL << 21;  // K*K*C fp16 taps
static __device__ __align__(256) __half g_noalloc_rot_taps[kNoAllocMaxTaps];
static std::mutex g_noalloc_mu[kMaxDevices];
static void* g_noalloc_taps[kMaxDevices];

// Device address of the built-in buffer on device `dev` (current), looked up once.
static int noalloc_taps(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu[dev]);
  if (!g_noalloc_taps[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_rot_taps);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return cuda_fail("cudaGetSymbolAddress(g_noalloc_rot_taps)", e);
    }
    g_noalloc_taps[dev] = p;
  }
  *out = g_noalloc_taps[dev];
  return DWB_OK;
}

int dwb_conv2d_nhwc_bwd_data_noalloc(const void* dy, const void* w, void* dx, int64_t B, int64_t H, int64_t W,
                                     int64_t C, int K, void* stream) {
  int rc = validate_args(dy, w, nullptr, nullptr, nullptr, nullptr, dx, B, H, W, C, K, DWB_ACT_NONE,
                         DWB_ACCUM_DEFAULT);
  if (rc != DWB_OK) return rc;
  if (static_cast<long long>(K) * K * C > kNoAllocMaxTaps) {
    std::snprintf(g_last_error, sizeof(g_last_error),
                  "dwb_conv2d_nhwc_bwd_data_noalloc: K*K*C = %lld taps exceeds the built-in buffer of %lld",
                  static_cast<long long>(K) * K * C, kNoAllocMaxTaps);
    return DWB_ERR_BAD_SHAPE;
  }
  if (B == 0) return DWB_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DWB_ERR_NO_DEVICE;
  void* taps = nullptr;
  rc = noalloc_taps(dev, &taps);
  if (rc != DWB_OK) return rc;
  rc = dwb_weight_rot180(w, taps, C, K, stream);
  if (rc != DWB_OK) return rc;
  return launch_forward(dy, taps, nullptr, nullptr, nullptr, nullptr, dx, B, H, W, C, K, DWB_ACT_NONE,
                        DWB_ACCUM_DEFAULT, stream);
}

}  // extern "C"
