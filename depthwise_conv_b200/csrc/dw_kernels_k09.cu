// Compiled variants of the depthwise kernel for K = 9 (see dw_variants.cuh).
#include "dw_variants.cuh"
DWB_DEFINE_TABLE_WIDE(9)
