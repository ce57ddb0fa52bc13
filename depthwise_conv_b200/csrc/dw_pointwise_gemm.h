// dw_pointwise_gemm.h -- the pointwise (1x1 convolution) block's fused GEMM:
// parameters, tile geometry and kernel registry, shared by
// dw_pointwise_gemm.cu (kernels) and dw_capi.cu (launcher).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace dwb {

// One CTA computes a kPwTileM x BN tile of y = act(x * w^T + bias) * scale + shift
// over K blocks of kPwTileK input channels.
constexpr int kPwTileM = 128;
constexpr int kPwTileK = 64;                      // 128 bytes of fp16: one swizzle row
constexpr int kPwThreads = 192;                   // warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer
constexpr int kPwMaxStages = 8;
constexpr int kPwTileNs[] = {64, 96, 128, 256};   // compiled BN values

struct PwGemmParams {
  const __half* bias;   // [N] or null
  const __half* scale;  // [N] or null
  const __half* shift;  // [N] or null
  __half* y;            // [M][N] row-major (NHWC pixels x output channels)
  int M, N, K;          // pixels, output channels, input channels
  int num_kb;           // ceil(K / kPwTileK)
  int stages;           // operand ring depth
  int* err;             // device error word
};

constexpr int pw_stage_bytes(int bn) { return (kPwTileM + bn) * kPwTileK * 2; }
// Dynamic shared memory of a launch: 1024 bytes of alignment slack, the
// operand ring, 2 * stages + 1 mbarriers, the TMEM address slot and the
// staged per-channel parameters (3 x BN floats).
constexpr int pw_smem_bytes(int bn, int stages) {
  return 1024 + stages * pw_stage_bytes(bn) + (2 * stages + 1) * 8 + 16 + 3 * bn * 4;
}

// pw_gemm_kernel<BN, ACT> (nullptr when BN is not compiled).
const void* pw_gemm_kernel_for(int bn, int act);

}  // namespace dwb
