// dw_pointwise.cu -- the elementwise epilogue of a ConvMixer pointwise block:
//   y = act(x + bias) * scale + shift      (per channel; x, y NHWC fp16)
// i.e. the bias, activation and inference BatchNorm that follow a 1x1
// convolution (convmixer/convmixer.py:116-118), as one HBM pass instead of
// PyTorch's separate bias-add, GELU and BatchNorm kernels.  The arithmetic is
// the fused depthwise kernel's epilogue (dw_device.cuh); memory traffic is
// 16-byte vectors, grid-stride over 8-channel groups (the parameter vectors
// read 16 bytes at a time too where they are 16-byte aligned).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/dwconv_b200.h"
#include "dw_device.cuh"
#include "dw_launch.h"

namespace dwb {

// Per-channel parameter pairs i = 0..3 of the 8 channels starting at c: one
// 16-byte load when the vectors are 16-byte aligned (VP), else 4-byte loads.
template <bool VP>
__device__ __forceinline__ void load_param8(const __half* __restrict__ p, int c, __half2 (&out)[4]) {
  if constexpr (VP) {
    const uint4 u = *reinterpret_cast<const uint4*>(p + c);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = h[i];
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = *reinterpret_cast<const __half2*>(p + c + 2 * i);
  }
}

template <int ACT, bool VP>
__global__ void __launch_bounds__(256) bias_act_affine_kernel(const uint4* __restrict__ x, const __half* __restrict__ bias,
                                                              const __half* __restrict__ scale,
                                                              const __half* __restrict__ shift, uint4* __restrict__ y,
                                                              long long groups, int cgroups) {
  griddep_wait();  // x may be the previous kernel's output (programmatic dependent launch)
  griddep_launch_dependents();
  const int stride = static_cast<int>(gridDim.x * blockDim.x);  // the launcher keeps the grid below 2^31 threads
  const int g0 = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  // channel group of the current vector, advanced by stride mod cgroups per
  // iteration, so the loop has no (64-bit) division
  int cg = g0 % cgroups;
  const int cstep = stride % cgroups;
  for (long long g = g0; g < groups; g += stride) {
    const int c = cg * 8;  // first of this vector's 8 channels
    cg += cstep;
    if (cg >= cgroups) cg -= cgroups;
    uint4 vec = x[g];
    __half2 b2[4], s2[4], t2[4];
    if (bias) load_param8<VP>(bias, c, b2);
    if (scale) load_param8<VP>(scale, c, s2);
    if (shift) load_param8<VP>(shift, c, t2);
    __half2* h = reinterpret_cast<__half2*>(&vec);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f32x2 v = h2_to_f32x2(h[i]);
      if (bias) fadd2(v, h2_to_f32x2(b2[i]));
      if (ACT == kActGelu) {
        v = gelu_erf2(v);
      } else if (ACT == kActRelu) {
        const float2 f = bits_f2(v);
        v = f2_bits(make_float2(fmaxf(f.x, 0.0f), fmaxf(f.y, 0.0f)));
      }
      const f32x2 sc = scale ? h2_to_f32x2(s2[i]) : splat2(1.0f);
      const f32x2 sh = shift ? h2_to_f32x2(t2[i]) : splat2(0.0f);
      const float2 o = bits_f2(fma2(v, sc, sh));
      h[i] = __floats2half2_rn(o.x, o.y);
    }
    y[g] = vec;
  }
}

template <int ACT>
const void* bias_act_affine_fn(bool vp) {
  return vp ? reinterpret_cast<const void*>(&bias_act_affine_kernel<ACT, true>)
            : reinterpret_cast<const void*>(&bias_act_affine_kernel<ACT, false>);
}

}  // namespace dwb

extern "C" int dwb_bias_act_affine_nhwc(const void* x, const void* bias, const void* scale, const void* shift, void* y,
                                         int64_t pixels, int64_t C, int act, void* stream) {
  using namespace dwb;
  if (act < DWB_ACT_NONE || act > DWB_ACT_GELU) return DWB_ERR_BAD_ARG;
  if (pixels < 0 || C < 8 || (C % 8) != 0) return DWB_ERR_BAD_SHAPE;
  if (pixels == 0) return DWB_OK;
  if (!x || !y) return DWB_ERR_NULL_POINTER;
  auto al = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; };
  if (!al(x, 16) || !al(y, 16) || (bias && !al(bias, 4)) || (scale && !al(scale, 4)) || (shift && !al(shift, 4)))
    return DWB_ERR_BAD_ALIGN;
  const long long groups = pixels * (C / 8);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (groups + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(want < sms * 8LL ? want : sms * 8LL);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* yv = static_cast<uint4*>(y);
  const __half *b = static_cast<const __half*>(bias), *sc = static_cast<const __half*>(scale),
               *sh = static_cast<const __half*>(shift);
  int cg = static_cast<int>(C / 8);
  long long ng = groups;
  void* args[7] = {&xv, &b, &sc, &sh, &yv, &ng, &cg};
  const bool vp = (!bias || al(bias, 16)) && (!scale || al(scale, 16)) && (!shift || al(shift, 16));
  const void* fn = act == DWB_ACT_GELU   ? bias_act_affine_fn<kActGelu>(vp)
                   : act == DWB_ACT_RELU ? bias_act_affine_fn<kActRelu>(vp)
                                         : bias_act_affine_fn<kActNone>(vp);
  if (launch_kernel(fn, dim3(blocks), dim3(256), args, 0, s) != cudaSuccess) {
    (void)cudaGetLastError();
    return DWB_ERR_CUDA;
  }
  return DWB_OK;
}
