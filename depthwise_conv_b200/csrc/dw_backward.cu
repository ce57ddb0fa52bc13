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
// Weight gradient decomposition: a warp owns one kernel row kh (for K > 13
// half of its taps), 64 channels (lane = channel pair) and a chunk of output
// rows (b, h).  For each output row it slides along the row in blocks of R
// columns: R dy values and the R + KW - 1 x values they meet are read
// (coalesced 128-byte rows per warp, converted to fp32), and the R x KW
// products go into KW packed fp32 accumulators, one per tap.  At the end the
// warp adds its KW x 64 partial sums into dw with fp32 atomics, so the result
// needs no buffer beyond dw itself
// (the caller zeroes dw, or passes a sum to add to).  Chunks are sized so the
// grid holds at least ~16 warps per SM.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/dwconv_b200.h"
#include "dw_device.cuh"
#include "dw_launch.h"

namespace dwb {

constexpr int kWgradR = 16;      // output columns per register block
constexpr int kWgradWarps = 4;   // warps (chunks) per CTA

// KW taps of the kernel row per warp (kw0 = blockIdx.y % nkw * KW): large K
// splits the row over warps, which halves each warp's accumulators and x reads
// and lets more warps share an SM.
template <int K>
constexpr int wgrad_kw() {
  return K <= 13 ? K : (K + 1) / 2;
}

template <int K>
__global__ void __launch_bounds__(kWgradWarps * 32, 4) dw_wgrad_kernel(const __half2* __restrict__ x,
                                                                    const __half2* __restrict__ dy,
                                                                    float* __restrict__ dw, int B, int H, int W,
                                                                    int C, long long rows_per_chunk,
                                                                    long long nchunks) {
  griddep_launch_dependents();
  griddep_wait();  // x and dy may come from the previous kernel
  constexpr int PAD = K / 2;
  constexpr int R = kWgradR;
  constexpr int KW = wgrad_kw<K>();
  constexpr int NKW = (K + KW - 1) / KW;
  constexpr int NJ = R + KW - 1;
  const int lane = threadIdx.x & 31;
  const long long chunk = static_cast<long long>(blockIdx.z) * kWgradWarps + (threadIdx.x >> 5);
  const int kh = blockIdx.y / NKW;
  const int kw0 = (blockIdx.y - kh * NKW) * KW;
  const int c = blockIdx.x * 64 + 2 * lane;  // this lane's channel pair
  if (chunk >= nchunks || c >= C) return;
  const int C2 = C / 2;  // half2 per pixel
  const long long rows = static_cast<long long>(B) * H;
  const long long r0 = chunk * rows_per_chunk;
  const long long r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;

  f32x2 acc[KW];
#pragma unroll
  for (int k = 0; k < KW; ++k) acc[k] = f32x2_zero();

  for (long long r = r0; r < r1; ++r) {
    const int b = static_cast<int>(r / H);
    const int h = static_cast<int>(r - static_cast<long long>(b) * H);
    const int ih = h + kh - PAD;
    if (ih < 0 || ih >= H) continue;  // warp-uniform
    const __half2* dyrow = dy + (static_cast<long long>(b) * H + h) * W * C2 + c / 2;
    const __half2* xrow = x + (static_cast<long long>(b) * H + ih) * W * C2 + c / 2;
    for (int w0 = 0; w0 < W; w0 += R) {
      f32x2 dv[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int w = w0 + i;
        dv[i] = w < W ? h2_to_f32x2(dyrow[static_cast<long long>(w) * C2]) : f32x2_zero();
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int iw = w0 + kw0 + j - PAD;
        const f32x2 xv = (iw >= 0 && iw < W) ? h2_to_f32x2(xrow[static_cast<long long>(iw) * C2]) : f32x2_zero();
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const int k = j - i;
          if (k >= 0 && k < KW) ffma2(acc[k], dv[i], xv);
        }
      }
    }
  }
  float* out = dw + static_cast<long long>(kh) * K * C + c;
#pragma unroll
  for (int k = 0; k < KW; ++k) {
    if (kw0 + k >= K) break;  // the last warp of an odd row has one tap fewer
    const float2 v = bits_f2(acc[k]);
    atomicAdd(out + static_cast<long long>(kw0 + k) * C, v.x);
    atomicAdd(out + static_cast<long long>(kw0 + k) * C + 1, v.y);
  }
}

// w_rot[kh][kw][c] = w[K-1-kh][K-1-kw][c], 8 channels (16 bytes) per thread.
__global__ void weight_rot180_kernel(const uint4* __restrict__ w, uint4* __restrict__ wr, int K, int C8) {
  griddep_launch_dependents();
  griddep_wait();
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

// Warps per kernel row (the kw split of wgrad_kw) for a runtime K.
static int wgrad_nkw(int K) {
  const int kw = K <= 13 ? K : (K + 1) / 2;
  return (K + kw - 1) / kw;
}

static const void* wgrad_for(int K) {
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

extern "C" int dwb_conv2d_nhwc_bwd_weight(const void* x, const void* dy, float* dw, int64_t B, int64_t H, int64_t W,
                                          int64_t C, int K, void* stream) {
  using namespace dwb;
  if (B < 0 || H < 1 || W < 1 || C < 8 || (C % 8) != 0 || K < 1 || K > 31 || (K % 2) == 0)
    return DWB_ERR_BAD_SHAPE;
  if (H > (1 << 30) || W > (1 << 30) || C > (1 << 30) || B > (1 << 30)) return DWB_ERR_BAD_SHAPE;
  if (B == 0) return DWB_OK;
  if (!x || !dy || !dw) return DWB_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(dy) || (reinterpret_cast<uintptr_t>(dw) & 7u) != 0) return DWB_ERR_BAD_ALIGN;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return DWB_ERR_NO_DEVICE;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long rows = B * H;
  const long long cblocks = (C + 63) / 64;
  // at least ~16 warps per SM over (channel block, kernel row, chunk)
  const long long rowsets = cblocks * K * wgrad_nkw(K);  // (channel block, kernel row, kw part)
  const long long want = (16LL * sms + rowsets - 1) / rowsets;
  const long long nchunks = want < rows ? (want > 0 ? want : 1) : rows;
  const long long rows_per_chunk = (rows + nchunks - 1) / nchunks;
  const long long nchunks_used = (rows + rows_per_chunk - 1) / rows_per_chunk;
  const long long zblocks = (nchunks_used + kWgradWarps - 1) / kWgradWarps;
  if (cblocks > 0x7fffffffLL || zblocks > 65535) return DWB_ERR_BAD_SHAPE;
  const __half2* xp = static_cast<const __half2*>(x);
  const __half2* dyp = static_cast<const __half2*>(dy);
  int Bi = static_cast<int>(B), Hi = static_cast<int>(H), Wi = static_cast<int>(W), Ci = static_cast<int>(C);
  long long rpc = rows_per_chunk, nch = nchunks_used;
  void* args[9] = {&xp, &dyp, &dw, &Bi, &Hi, &Wi, &Ci, &rpc, &nch};
  const cudaError_t e = launch_kernel(wgrad_for(K),
                                      dim3(static_cast<unsigned>(cblocks), K * wgrad_nkw(K), static_cast<unsigned>(zblocks)),
                                      dim3(kWgradWarps * 32), args, 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return DWB_ERR_CUDA;
  }
  return DWB_OK;
}

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
