// ref_shim.cu -- extern "C" entry points over the reference's own RepLKNet
// depthwise kernels (TEST INFRASTRUCTURE ONLY).
//
// Built by oracle/build_ref.py together with the reference's unmodified
// sources replknet/kernels/depthWise_ch_{128_k_31_t_56,256_k_29_t_28,
// 512_k_27_t_14}_half_forward.cu into oracle/_ref/libref_replknet.so.  The
// kernels are the ones the reference's torch ops launch
// (replknet/kernels/depthwise_replknet_nhwc_integration.cu:86-90,129-133,
// 172-176); their C interfaces (depthWise128_56_k31.hpp:33, depthWise256_28_k29.hpp:13,
// depthWise512_14_k27.hpp:28) launch one image on the default stream.  The
// tests use them to pin the oracle's emulation of the reference arithmetic
// and to time the reference kernels rebuilt for sm_100a.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "depthWise128_56_k31.hpp"
#include "depthWise256_28_k29.hpp"
#include "depthWise512_14_k27.hpp"

#define REF_API extern "C" __attribute__((visibility("default")))

static int last_status() { return static_cast<int>(cudaGetLastError()); }

// One 56x56x128 image, k31 (colmerge 8x12), output without bias.
REF_API int ref_dw_k31_c128_h56(const void* in, const void* w, void* out) {
  depthWise_forward_ch_128_kernel_31_tensor_56_fp16_colmerge_8x12_C_interface(
      static_cast<half*>(const_cast<void*>(in)), static_cast<const half*>(w), static_cast<half*>(out), 56, 56, 128,
      31);
  return last_status();
}

// One 28x28x256 image, k29 (colmerge 8x12).
REF_API int ref_dw_k29_c256_h28(const void* in, const void* w, void* out) {
  depthWise_forward_ch_256_kernel_29_tensor_28_fp16_colmerge_8x12_C_interface(
      static_cast<half*>(const_cast<void*>(in)), static_cast<const half*>(w), static_cast<half*>(out), 28, 28, 256,
      29);
  return last_status();
}

// One 14x14x512 image, k27 (allshared branch-free half2).
REF_API int ref_dw_k27_c512_h14(const void* in, const void* w, void* out) {
  depthWise_forward_ch_512_kernel_27_tensor_14_fp16_allshared_branchfree_h2_cb32_C_interface(
      static_cast<half*>(const_cast<void*>(in)), static_cast<const half*>(w), static_cast<half*>(out), 14, 14, 512,
      27);
  return last_status();
}
