// dw_backward.cu -- gradients of the depthwise convolution (NHWC fp16, "same"
// padding, stride 1, odd K).
//
//   input gradient  dx = conv(dy, w rotated by 180 degrees): the forward
//                   kernel on dy with the rotated taps (dwb_weight_rot180 +
//                   dwb_conv2d_nhwc_bwd_data in dw_capi.cu);
//   weight gradient dw[kh][kw][c] = sum over b, h, w of
//                   dy[b][h][w][c] * x[b][h + kh - K/2][w + kw - K/2][c]
//                   (this file).
//
// Weight gradient decomposition: one CTA per (64-channel block, kernel row
// kh, column tile, chunk of output rows).  A producer warp streams, for every
// output row h of the chunk whose input row ih = h + kh - K/2 lies in the
// image, one stage holding the dy row segment (tile_w columns) and the x row
// segment it meets (tile_w + K - 1 columns, zero outside the image from the
// TMA fill) through a ring of shared-memory stages with full/empty mbarriers
// (bounded waits), like the forward kernel.  Each consumer warp owns R = 16
// columns of the tile (lane = channel pair): per stage it converts its R dy
// values and R + K - 1 x values to fp32 and adds the R x K products into K
// packed fp32 accumulators, one per kw.  At the end it adds them into dw with
// fp32 atomics, so the result needs no buffer beyond dw itself (the caller
// zeroes dw, or passes a sum to add to).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/dwconv_b200.h"
#include "dw_backward.h"
#include "dw_device.cuh"
#include "dw_launch.h"

namespace dwb {

constexpr int kWgradR = 16;  // output columns per consumer warp

template <int K>
__global__ void __launch_bounds__(160, 1) dw_wgrad_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                          const __grid_constant__ CUtensorMap tm_dy,
                                                          const WgradParams p) {
  constexpr int PAD = K / 2;
  constexpr int R = kWgradR;
  constexpr int NJ = R + K - 1;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int NS = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NS;
  unsigned char* ring = smem + p.ring_off;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t dy_bytes = static_cast<uint32_t>(p.tile_w) * 128u;
  const uint32_t x_bytes = static_cast<uint32_t>(p.tile_w + K - 1) * 128u;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_dy);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], p.consumer_warps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // x and dy may come from the previous kernel
  griddep_launch_dependents();

  const int c0 = blockIdx.x * 64;
  const int kh = blockIdx.y;
  const int ct = static_cast<int>(blockIdx.z % static_cast<unsigned>(p.col_tiles));
  const long long chunk = blockIdx.z / static_cast<unsigned>(p.col_tiles);
  const int w0 = ct * p.tile_w;
  const long long rows = static_cast<long long>(p.B) * p.H;
  const long long r0 = chunk * p.rows_per_chunk;
  const long long r1 = r0 + p.rows_per_chunk < rows ? r0 + p.rows_per_chunk : rows;

  if (warp == p.consumer_warps) {
    // ---- producer: one stage per output row with an in-image input row ----
    if (lane == 0) {
      RingPos fr;
      long long fills = 0;
      for (long long r = r0; r < r1; ++r) {
        const int b = static_cast<int>(r / p.H);
        const int h = static_cast<int>(r - static_cast<long long>(b) * p.H);
        const int ih = h + kh - PAD;
        if (ih < 0 || ih >= p.H) continue;
        if (fills >= NS && !mbar_wait_bounded<true>(&empty[fr.slot], fr.phase ^ 1u, p.err, 3)) break;
        unsigned char* dst = ring + fr.slot * p.stage_bytes;
        mbar_arrive_expect_tx(&full[fr.slot], dy_bytes + x_bytes);
        tma_load_4d(dst, &tm_dy, &full[fr.slot], c0, w0, h, b);
        tma_load_4d(dst + dy_bytes, &tm_x, &full[fr.slot], c0, w0 - PAD, ih, b);
        fr.next(NS);
        ++fills;
      }
    }
    return;
  }

  // ---- consumers: R columns each, K accumulators per channel pair ----
  const int col0 = warp * R;
  f32x2 acc[K];
#pragma unroll
  for (int k = 0; k < K; ++k) acc[k] = f32x2_zero();
  RingPos ws;
  bool ok = true;
  for (long long r = r0; r < r1 && ok; ++r) {
    const int b = static_cast<int>(r / p.H);
    const int h = static_cast<int>(r - static_cast<long long>(b) * p.H);
    const int ih = h + kh - PAD;
    if (ih < 0 || ih >= p.H) continue;  // the producer skipped it too
    ok = mbar_wait_bounded(&full[ws.slot], ws.phase, p.err, 2);
    if (!ok) break;
    const unsigned char* st = ring + ws.slot * p.stage_bytes;
    const __half2* dyr = reinterpret_cast<const __half2*>(st) + col0 * 32 + lane;
    const __half2* xr = reinterpret_cast<const __half2*>(st + dy_bytes) + col0 * 32 + lane;
    f32x2 dv[R];
#pragma unroll
    for (int i = 0; i < R; ++i) dv[i] = h2_to_f32x2(dyr[i * 32]);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const f32x2 xv = h2_to_f32x2(xr[j * 32]);
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int kw = j - i;
        if (kw >= 0 && kw < K) ffma2(acc[kw], dv[i], xv);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[ws.slot]);
    ws.next(NS);
  }
  const int c = c0 + 2 * lane;
  if (!ok || c >= p.C) return;
  if (p.partial) {  // deterministic: this warp's own slice, summed in order by wgrad_reduce_kernel
    const long long slice = static_cast<long long>(blockIdx.z) * p.consumer_warps + warp;
    float* out = p.partial + (slice * K + kh) * K * p.C + c;
#pragma unroll
    for (int kw = 0; kw < K; ++kw)
      *reinterpret_cast<float2*>(out + static_cast<long long>(kw) * p.C) = bits_f2(acc[kw]);
    return;
  }
  float* out = p.dw + static_cast<long long>(kh) * K * p.C + c;
#pragma unroll
  for (int kw = 0; kw < K; ++kw) {
    const float2 v = bits_f2(acc[kw]);
    atomicAdd(out + static_cast<long long>(kw) * p.C, v.x);
    atomicAdd(out + static_cast<long long>(kw) * p.C + 1, v.y);
  }
}

__global__ void __launch_bounds__(256) wgrad_reduce_kernel(const float4* __restrict__ partial, float4* __restrict__ dw,
                                                           long long n4, int slices) {
  griddep_wait();  // the partial sums come from the previous kernel
  griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 a = dw[i];
    for (int s = 0; s < slices; ++s) {  // fixed order: the same bits on every run
      const float4 v = partial[static_cast<long long>(s) * n4 + i];
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    dw[i] = a;
  }
}

const void* wgrad_reduce_kernel_fn() { return reinterpret_cast<const void*>(&wgrad_reduce_kernel); }

// w_rot[kh][kw][c] = w[K-1-kh][K-1-kw][c], 8 channels (16 bytes) per thread.
__global__ void weight_rot180_kernel(const uint4* __restrict__ w, uint4* __restrict__ wr, int K, int C8) {
  griddep_wait();
  griddep_launch_dependents();
  const int n = K * K * C8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int c8 = i % C8;
    const int tap = i / C8;  // kh * K + kw
    wr[i] = w[(K * K - 1 - tap) * C8 + c8];
  }
}

template <int K>
const void* wgrad_fn() {
  return reinterpret_cast<const void*>(&dw_wgrad_kernel<K>);
}

const void* wgrad_kernel_for(int K) {
  switch (K) {
#define DWB_WG(KK) \
  case KK:         \
    return wgrad_fn<KK>();
    DWB_WG(1) DWB_WG(3) DWB_WG(5) DWB_WG(7) DWB_WG(9) DWB_WG(11) DWB_WG(13) DWB_WG(15)
    DWB_WG(17) DWB_WG(19) DWB_WG(21) DWB_WG(23) DWB_WG(25) DWB_WG(27) DWB_WG(29) DWB_WG(31)
#undef DWB_WG
    default:
      return nullptr;
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace dwb

extern "C" int dwb_weight_rot180(const void* w, void* w_rot180, int64_t C, int K, void* stream) {
  using namespace dwb;
  if (C < 8 || (C % 8) != 0 || C > (1 << 24) || K < 1 || K > 31 || (K % 2) == 0) return DWB_ERR_BAD_SHAPE;
  if (!w || !w_rot180) return DWB_ERR_NULL_POINTER;
  if (!aligned16(w) || !aligned16(w_rot180)) return DWB_ERR_BAD_ALIGN;
  int C8 = static_cast<int>(C / 8), Ki = K;
  const int n = K * K * C8;
  const uint4* wp = static_cast<const uint4*>(w);
  uint4* wr = static_cast<uint4*>(w_rot180);
  void* args[4] = {&wp, &wr, &Ki, &C8};
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
  const cudaError_t e = launch_kernel(reinterpret_cast<const void*>(&weight_rot180_kernel), dim3(blocks), dim3(256),
                                      args, 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return DWB_ERR_CUDA;
  }
  return DWB_OK;
}
