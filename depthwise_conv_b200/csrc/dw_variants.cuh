// dw_variants.cuh -- the (R, M, ACC) variants compiled for every kernel size.
//   R (columns per thread) in {7, 8, 14, 16} covers the widths 7, 14, 16, 28,
//   32 and 56 without overhang; M (rows per thread) in {1, 2}; ACC 0 = fp32
//   FFMA2, 1 = fp16x2 row partials with fp32 accumulation across rows.
#pragma once
#include "dw_kernel.cuh"

#define DWB_ENTRY(K, R, M, A) {K, R, M, A, reinterpret_cast<const void*>(&::dwb::dw_stream_kernel<K, R, M, A>)}
#define DWB_VARIANTS_ACC(K, A)                                                                      \
  DWB_ENTRY(K, 7, 1, A), DWB_ENTRY(K, 7, 2, A), DWB_ENTRY(K, 8, 1, A), DWB_ENTRY(K, 8, 2, A),     \
      DWB_ENTRY(K, 14, 1, A), DWB_ENTRY(K, 14, 2, A), DWB_ENTRY(K, 16, 1, A), DWB_ENTRY(K, 16, 2, A)
#define DWB_VARIANTS(K) DWB_VARIANTS_ACC(K, 0), DWB_VARIANTS_ACC(K, 1)

#define DWB_DEFINE_TABLE(K)                                                          \
  namespace dwb {                                                                    \
  extern const KernelEntry kTableK##K[] = {DWB_VARIANTS(K)};                         \
  extern const int kCountK##K = static_cast<int>(sizeof(kTableK##K) / sizeof(KernelEntry)); \
  }
