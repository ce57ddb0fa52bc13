// dw_pointwise_gemm.cu -- the ConvMixer pointwise block as one tensor-core kernel:
//   y[m][n] = act( sum_k x[m][k] * w[n][k] + bias[n] ) * scale[n] + shift[n]
// x: NHWC activations as a [pixels][C_in] row-major matrix, w: the 1x1
// convolution's weight [C_out][C_in] (PyTorch's own layout), y: NHWC
// [pixels][C_out].  This is the 1x1 convolution, its bias, the activation and
// the inference BatchNorm of convmixer/convmixer.py:116-118 (and of the patch
// stem, whose non-overlapping patches form the same kind of matrix) with no
// intermediate tensor in HBM.
//
// One CTA per 128 x BN output tile (BN in kPwTileNs), 6 warps:
//   warp 4 (one lane)  TMA producer: K blocks of 64 channels of x (128 rows)
//                      and w (BN rows) into a ring of `stages` operand stages,
//                      128-byte swizzled, out-of-range rows/columns zero-filled
//                      (two boxes per stage: splitting them into 16-row boxes
//                      issued by parallel lanes measured 1.7x slower);
//   warp 5             allocates BN (rounded up to a power of two) TMEM columns;
//                      one lane issues four 128 x BN x 16 tcgen05.mma per stage
//                      into the fp32 accumulator in TMEM and frees the stage
//                      with tcgen05.commit when those MMAs have read it;
//   warps 0-3          epilogue: warp w reads TMEM lanes 32w..32w+31 (tile rows)
//                      16 columns at a time (tcgen05.ld, double-buffered), adds
//                      the bias, applies the activation and the BN scale/shift in
//                      packed fp32x2 arithmetic and stores 32 contiguous bytes of
//                      its row per 16 columns.
// Measured on B200 (clock64 trace of one CTA): operand stages arrive ahead
// of use; the MMA issuer is the bound, at ~600 clocks per 64-channel K block,
// i.e. ~150 clocks per 128 x N x 16 instruction for N = 96 and N = 256 alike,
// so only 128 x 256 tiles run near the tensor peak (~84%).  The ConvMixer
// batch-1 block (1024 x 1536 x 1536) has 48 such tiles, so the kernel takes
// ~10 us where cuBLAS (2-CTA tiles, 6.3 us) plus the one-pass epilogue
// (3.0 us) take 9.3 us; the ConvMixer modules therefore keep that pair and
// this kernel is the fused alternative (depthwise::pointwise_gemm).
// Every mbarrier wait is bounded; an expired wait records its code in the
// device error word (6 producer, 7 MMA issuer, 8 epilogue) and the kernel
// still reaches its end: the MMA issuer always commits to the accumulator
// barrier, so the epilogue's wait ends once every issued MMA has completed,
// and tensor memory is freed only after that.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "dw_device.cuh"
#include "dw_pointwise_gemm.h"
#include "dw_umma.cuh"

namespace dwb {

template <int BN>
constexpr uint32_t pw_tmem_cols() {
  return BN <= 32 ? 32u : BN <= 64 ? 64u : BN <= 128 ? 128u : 256u;
}

// act(a + bias) * scale + shift on one packed pair of columns.
template <int ACT>
__device__ __forceinline__ uint32_t pw_epilogue_pair(uint32_t lo, uint32_t hi, f32x2 bias, f32x2 scale,
                                                     f32x2 shift) {
  f32x2 a = (static_cast<f32x2>(hi) << 32) | lo;
  fadd2(a, bias);
  if constexpr (ACT == kActGelu) {
    a = gelu_erf2(a);
  } else if constexpr (ACT == kActRelu) {
    const float2 f = bits_f2(a);
    a = f2_bits(make_float2(fmaxf(f.x, 0.0f), fmaxf(f.y, 0.0f)));
  }
  const float2 o = bits_f2(fma2(a, scale, shift));
  const __half2 h = __floats2half2_rn(o.x, o.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int BN, int ACT>
__global__ void __launch_bounds__(kPwThreads, 1)
    pw_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                   const PwGemmParams p) {
  constexpr int A_BYTES = kPwTileM * kPwTileK * 2;
  constexpr int STAGE = pw_stage_bytes(BN);
  constexpr uint32_t TMEM_COLS = pw_tmem_cols<BN>();
  constexpr uint32_t IDESC = f16_f32acc_idesc<kPwTileM, BN>();
  static_assert(A_BYTES % 1024 == 0 && STAGE % 1024 == 0, "stages keep the 1024-byte swizzle-atom alignment");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  float* prm = reinterpret_cast<float*>(tmem_slot + 4);  // bias, scale, shift: BN floats each

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kPwTileM;
  const int n0 = blockIdx.y * BN;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Set-up above overlaps the previous kernel of the stream; global memory
  // (x may be its output, y may alias what it reads) only after the wait.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      RingPos ps;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (kb >= S && !mbar_wait_bounded(&empty[ps.slot], ps.phase ^ 1u, p.err, 6)) break;
        unsigned char* st = smem + ps.slot * STAGE;
        mbar_arrive_expect_tx(&full[ps.slot], STAGE);  // full boxes land, out-of-range parts as zeros
        tma_load_2d(st, &tmap_x, &full[ps.slot], kb * kPwTileK, m0);
        tma_load_2d(st + A_BYTES, &tmap_w, &full[ps.slot], kb * kPwTileK, n0);
        ps.next(S);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      RingPos ps;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait_bounded(&full[ps.slot], ps.phase, p.err, 7)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_addr(smem + ps.slot * STAGE);
        const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < kPwTileK / 16; ++kk)
          umma_f16(tmem, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32), IDESC,
                   (kb | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[ps.slot]);  // the stage is free once these MMAs have read it
        ps.next(S);
      }
      umma_commit(acc_full);  // always: completes when every MMA issued above has
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 0-3, 128 threads) ----------------
    for (int i = threadIdx.x; i < BN; i += 4 * 32) {
      const int n = n0 + i;
      const bool in = n < p.N;
      prm[i] = (in && p.bias) ? __half2float(p.bias[n]) : 0.0f;
      prm[BN + i] = (in && p.scale) ? __half2float(p.scale[n]) : 1.0f;
      prm[2 * BN + i] = (in && p.shift) ? __half2float(p.shift[n]) : 0.0f;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps only
    const bool ok = mbar_wait_bounded<true>(acc_full, 0u, p.err, 8);
    tc_fence_after();
    const int row = m0 + warp * 32 + lane;
    const bool row_ok = ok && row < p.M;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    __half* yrow = p.y + static_cast<long long>(row) * p.N + n0;
    const f32x2* b2 = reinterpret_cast<const f32x2*>(prm);
    const f32x2* s2 = reinterpret_cast<const f32x2*>(prm + BN);
    const f32x2* t2 = reinterpret_cast<const f32x2*>(prm + 2 * BN);
    uint32_t v[2][16];
    tmem_ld16(taddr, v[0]);
#pragma unroll
    for (int c = 0; c < BN / 16; ++c) {
      tmem_ld_wait();
      if (c + 1 < BN / 16) tmem_ld16(taddr + (c + 1) * 16, v[(c + 1) & 1]);  // next chunk in flight
      const uint32_t(&u)[16] = v[c & 1];
      if (row_ok && n0 + c * 16 < p.N) {
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int pc = c * 8 + j;  // column pair within the tile
          o[j] = pw_epilogue_pair<ACT>(u[2 * j], u[2 * j + 1], b2[pc], s2[pc], t2[pc]);
        }
        uint4* dst = reinterpret_cast<uint4*>(yrow + c * 16);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        if (n0 + c * 16 + 8 < p.N) dst[1] = make_uint4(o[4], o[5], o[6], o[7]);  // N is a multiple of 8
      }
    }
    tmem_ld_wait();
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int BN>
static const void* pw_fn_for_act(int act) {
  switch (act) {
    case kActGelu: return reinterpret_cast<const void*>(&pw_gemm_kernel<BN, kActGelu>);
    case kActRelu: return reinterpret_cast<const void*>(&pw_gemm_kernel<BN, kActRelu>);
    default: return reinterpret_cast<const void*>(&pw_gemm_kernel<BN, kActNone>);
  }
}

const void* pw_gemm_kernel_for(int bn, int act) {
  switch (bn) {
    case 64: return pw_fn_for_act<64>(act);
    case 96: return pw_fn_for_act<96>(act);
    case 128: return pw_fn_for_act<128>(act);
    case 256: return pw_fn_for_act<256>(act);
    default: return nullptr;
  }
}

}  // namespace dwb
