// dw_backward.h -- the weight-gradient kernel's parameters and registry,
// shared by dw_backward.cu (kernels) and dw_capi.cu (launcher).
#pragma once

#include <stdint.h>

namespace dwb {

struct WgradParams {
  float* dw;                  // [K][K][C] fp32, accumulated into
  int B, H, W, C;
  int tile_w;                 // columns per CTA (consumer_warps * 16)
  int col_tiles;              // column tiles across W
  long long rows_per_chunk;   // output rows (b, h) per CTA
  int consumer_warps;
  int stages;                 // ring depth
  uint32_t ring_off;          // byte offset of stage 0 in dynamic smem
  uint32_t stage_bytes;       // (2 tile_w + K - 1) * 128
  float* partial;             // deterministic mode: [gridDim.z * consumer_warps][K][K][C] partial sums,
                              // one slice per (row chunk, column tile, warp); nullptr: atomics into dw
  int* err;                   // device error word
};

constexpr int kWgradColumnsPerWarp = 16;

// dw_wgrad_kernel<K> for an odd K in 1..31 (nullptr otherwise).
const void* wgrad_kernel_for(int K);

// dw[i] += sum over slices s = 0..slices-1 of partial[s][i], in slice order, for i < n
// (the deterministic weight gradient's reduction; n a multiple of 4).
const void* wgrad_reduce_kernel_fn();

}  // namespace dwb
