// dw_pointwise.cu -- the elementwise epilogue of a ConvMixer pointwise block:
//   y = act(x + bias) * scale + shift      (per channel; x, y NHWC fp16)
// i.e. the bias, activation and inference BatchNorm that follow a 1x1
// convolution (convmixer/convmixer.py:116-118), as one HBM pass instead of
// PyTorch's separate bias-add, GELU and BatchNorm kernels.  The arithmetic is
// the fused depthwise kernel's epilogue (dw_device.cuh); memory traffic is
// 16-byte vectors, grid-stride over 8-channel groups.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/dwconv_b200.h"
#include "dw_device.cuh"
#include "dw_launch.h"

namespace dwb {

template <int ACT>
__global__ void __launch_bounds__(256) bias_act_affine_kernel(const uint4* __restrict__ x, const __half* __restrict__ bias,
                                                              const __half* __restrict__ scale,
                                                              const __half* __restrict__ shift, uint4* __restrict__ y,
                                                              long long groups, int cgroups) {
  griddep_launch_dependents();
  griddep_wait();  // x may be the previous kernel's output (programmatic dependent launch)
  for (long long g = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(g % cgroups) * 8;  // first of this vector's 8 channels
    uint4 v = x[g];
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ci = c + 2 * i;
      f32x2 v = h2_to_f32x2(h[i]);
      if (bias) fadd2(v, h2_to_f32x2(*reinterpret_cast<const __half2*>(bias + ci)));
      if (ACT == kActGelu) {
        v = gelu_erf2(v);
      } else if (ACT == kActRelu) {
        const float2 f = bits_f2(v);
        v = f2_bits(make_float2(fmaxf(f.x, 0.0f), fmaxf(f.y, 0.0f)));
      }
      const f32x2 s = scale ? h2_to_f32x2(*reinterpret_cast<const __half2*>(scale + ci)) : splat2(1.0f);
      const f32x2 t = shift ? h2_to_f32x2(*reinterpret_cast<const __half2*>(shift + ci)) : splat2(0.0f);
      const float2 o = bits_f2(fma2(v, s, t));
      h[i] = __floats2half2_rn(o.x, o.y);
    }
    y[g] = v;
  }
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
  const void* fn = act == DWB_ACT_GELU   ? reinterpret_cast<const void*>(&bias_act_affine_kernel<kActGelu>)
                   : act == DWB_ACT_RELU ? reinterpret_cast<const void*>(&bias_act_affine_kernel<kActRelu>)
                                         : reinterpret_cast<const void*>(&bias_act_affine_kernel<kActNone>);
  if (launch_kernel(fn, dim3(blocks), dim3(256), args, 0, s) != cudaSuccess) {
    (void)cudaGetLastError();
    return DWB_ERR_CUDA;
  }
  return DWB_OK;
}
