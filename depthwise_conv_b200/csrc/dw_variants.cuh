// dw_variants.cuh -- the (R, M, ACC, PRE) variants compiled for every kernel size.
//   R (columns per thread) in {7, 8, 14, 16} covers the widths 7, 14, 16, 28,
//   32 and 56 without overhang, plus R in {28, 32} for K <= 13, where a wider
//   register block amortises the per-kernel-row overhead over more FMAs;
//   M (rows per thread) in {1, 2}; ACC 0 = fp32 FFMA2, 1 = fp16x2 chains with
//   fp32 accumulation; PRE (load schedule, mixed mode only) 0 or 1.  Each
//   mixed-mode variant with K <= kBandMaxK also has a band-mode kernel.
//   dw_planner.cpp (variant_compiled, band_compiled) mirrors this list.
#pragma once
#include "dw_kernel.cuh"

namespace dwb {
// Band-mode kernels (dw_band_body) are built for the mixed accumulation and
// K <= kBandMaxK, where the two resident K x K weight buffers stay small and
// TMA requests, not FMAs, bound the tile kernel.  dw_planner.cpp mirrors this.
template <int K, int R, int M, int ACC, int PRE>
inline const void* band_entry() {
  if constexpr (ACC == 1 && K <= kBandMaxK) {
    return band_kernel_fn<K, R, M, ACC, PRE>();
  } else {
    return nullptr;
  }
}
}  // namespace dwb

#define DWB_ENTRY(K, R, M, A, P) \
  {K, R, M, A, P, ::dwb::kernel_fn<K, R, M, A, P>(), ::dwb::band_entry<K, R, M, A, P>()}
#define DWB_VARIANTS_AP(K, A, P)                                                                            \
  DWB_ENTRY(K, 7, 1, A, P), DWB_ENTRY(K, 7, 2, A, P), DWB_ENTRY(K, 8, 1, A, P), DWB_ENTRY(K, 8, 2, A, P),   \
      DWB_ENTRY(K, 14, 1, A, P), DWB_ENTRY(K, 14, 2, A, P), DWB_ENTRY(K, 16, 1, A, P), DWB_ENTRY(K, 16, 2, A, P)
#define DWB_WIDE_AP(K, A, P) \
  DWB_ENTRY(K, 28, 1, A, P), DWB_ENTRY(K, 28, 2, A, P), DWB_ENTRY(K, 32, 1, A, P), DWB_ENTRY(K, 32, 2, A, P)
#define DWB_VARIANTS(K) DWB_VARIANTS_AP(K, 0, 0), DWB_VARIANTS_AP(K, 1, 0), DWB_VARIANTS_AP(K, 1, 1)
#define DWB_VARIANTS_WIDE(K) \
  DWB_VARIANTS(K), DWB_WIDE_AP(K, 0, 0), DWB_WIDE_AP(K, 1, 0), DWB_WIDE_AP(K, 1, 1)

#define DWB_DEFINE_TABLE_OF(K, LIST)                                                      \
  namespace dwb {                                                                         \
  extern const KernelEntry kTableK##K[] = {LIST(K)};                                      \
  extern const int kCountK##K = static_cast<int>(sizeof(kTableK##K) / sizeof(KernelEntry)); \
  }
#define DWB_DEFINE_TABLE(K) DWB_DEFINE_TABLE_OF(K, DWB_VARIANTS)
#define DWB_DEFINE_TABLE_WIDE(K) DWB_DEFINE_TABLE_OF(K, DWB_VARIANTS_WIDE)
