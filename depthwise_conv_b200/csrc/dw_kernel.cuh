// dw_kernel.cuh -- the row-streaming depthwise convolution kernel for sm_100a.
//
// Work decomposition
//   CTA  = one output tile: tile_h rows x tile_w columns x 64 channels of one
//          image (channels past C are zero-filled by TMA and never stored).
//   warp = one "slot" of the tile: M consecutive output rows x R consecutive
//          output columns x 64 channels; lane l owns channels (2l, 2l+1), so
//          every shared-memory access of a warp is one contiguous 128-byte row
//          (conflict-free) and every row/column skip is warp-uniform.
//   thread accumulators: acc[M][R] float2 (two channels), fp32 throughout.
//
// Data movement (no multicast, plain per-CTA TMA tile loads)
//   The kernel walks the kernel rows ki (step s).  At step s every output row
//   h of the tile reads input row h - pad + s, so the tile needs the input
//   rows [h0 - pad + s, h0 - pad + s + tile_h): a window that slides one row
//   per step.  A dedicated producer warp streams those rows, and weight row
//   ki, through two shared-memory rings guarded by full/empty mbarriers:
//     input row  : [tile_w + K - 1 columns][64 channels] fp16 (zero padding
//                  comes from TMA out-of-bounds fill)
//     weight row : [K taps][64 channels] fp16
//   Steps whose input rows all fall outside the image are not executed.
//
// Inner loop (weight-stationary per kernel row)
//   The K weights of row ki are converted once to float2 registers; then for
//   each of the M rows the thread slides along R + K - 1 input columns: each
//   input half2 is loaded and converted once and feeds up to R accumulators
//   through packed fp32x2 FMAs (ACC = 0), or fp16x2 HFMA2 into a per-row
//   partial that is added to the fp32 accumulator after the row (ACC = 1).
//
// Epilogue (fused): v = acc + bias; v = act(v); v = v * scale + shift;
//   v += residual; stored as half2, 128 contiguous bytes per warp.
#pragma once

#include "dw_device.cuh"

namespace dwb {

constexpr int kChannelsPerCta = 64;                 // 32 lanes x 2 channels
constexpr int kPixelBytes = kChannelsPerCta * 2;    // one staged pixel = 128 B
constexpr int kPixelH2 = kChannelsPerCta / 2;       // half2 per staged pixel
constexpr int kBarrierBytes = 1024;                 // mbarrier area at smem start

struct DwParams {
  __half* y;
  const __half* bias;      // [C] or nullptr
  const __half* scale;     // [C] or nullptr
  const __half* shift;     // [C] or nullptr
  const __half* residual;  // NHWC like y, or nullptr
  int B, H, W, C;
  int tile_h, tile_w, tile_w_in;
  int tiles_h, tiles_w, cblocks;
  int ncg;                 // column groups (warps across the tile width)
  int consumer_warps;
  int ring_rows, ring_wrows;
  int act;
  uint32_t x_ring_off, w_ring_off;  // byte offsets inside dynamic smem
  int* err;                         // device error word (bounded-wait expiry)
};

template <int K, int R, int M, int ACC>
__global__ void dw_stream_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                 const __grid_constant__ CUtensorMap tmap_w, const DwParams p) {
  constexpr int PAD = K / 2;
  constexpr int NJ = R + K - 1;  // input columns a thread slides over
  extern __shared__ __align__(1024) unsigned char smem[];

  const int RR = p.ring_rows;
  const int RW = p.ring_wrows;
  uint64_t* full_x = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty_x = full_x + RR;
  uint64_t* full_w = empty_x + RR;
  uint64_t* empty_w = full_w + RW;
  unsigned char* xring = smem + p.x_ring_off;
  unsigned char* wring = smem + p.w_ring_off;
  const uint32_t row_bytes = static_cast<uint32_t>(p.tile_w_in) * kPixelBytes;
  constexpr uint32_t wrow_bytes = K * kPixelBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Tile decode: tile-row fastest so consecutive CTAs share halo rows in L2.
  long long t = blockIdx.x;
  const int th = static_cast<int>(t % p.tiles_h);
  t /= p.tiles_h;
  const int tw = static_cast<int>(t % p.tiles_w);
  t /= p.tiles_w;
  const int cbk = static_cast<int>(t % p.cblocks);
  const int b = static_cast<int>(t / p.cblocks);
  const int h0 = th * p.tile_h;
  const int w0 = tw * p.tile_w;
  const int c0 = cbk * kChannelsPerCta;
  const int rows_in_tile = min(p.tile_h, p.H - h0);

  // Kernel-row range with at least one in-image input row for this tile.
  const int s_lo = max(0, PAD - (h0 + rows_in_tile - 1));
  const int s_hi = min(K, p.H + PAD - h0);
  const int nsteps = s_hi - s_lo;
  const int nrows = nsteps + p.tile_h - 1;  // streamed input rows

  if (threadIdx.x == 0) {
    for (int i = 0; i < RR; ++i) {
      mbar_init(&full_x[i], 1);
      mbar_init(&empty_x[i], p.consumer_warps);
    }
    for (int i = 0; i < RW; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&empty_w[i], p.consumer_warps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == p.consumer_warps) {
    // ---------------- producer warp ----------------
    if (lane == 0 && nsteps > 0) {
      prefetch_tmap(&tmap_x);
      prefetch_tmap(&tmap_w);
      int q = 0;  // next input row (sequence number) to issue
      bool ok = true;
      for (int st = 0; st < nsteps && ok; ++st) {
        // weight row (s_lo + st)
        const int ws = st % RW;
        if (st >= RW) ok = mbar_wait_bounded(&empty_w[ws], ((st / RW) - 1) & 1, p.err, 3);
        if (!ok) break;
        mbar_arrive_expect_tx(&full_w[ws], wrow_bytes);
        tma_load_3d(wring + ws * wrow_bytes, &tmap_w, &full_w[ws], c0, 0, s_lo + st);
        // input rows needed by this step: q < st + tile_h
        const int need = min(st + p.tile_h, nrows);
        for (; q < need; ++q) {
          const int slot = q % RR;
          if (q >= RR) ok = mbar_wait_bounded(&empty_x[slot], ((q / RR) - 1) & 1, p.err, 3);
          if (!ok) break;
          const int abs_row = h0 - PAD + s_lo + q;
          if (abs_row >= 0 && abs_row < p.H) {
            mbar_arrive_expect_tx(&full_x[slot], row_bytes);
            tma_load_4d(xring + slot * row_bytes, &tmap_x, &full_x[slot], c0, w0 - PAD, abs_row, b);
          } else {
            mbar_arrive(&full_x[slot]);  // nothing to load: consumers skip this row
          }
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int rg = warp / p.ncg;
  const int cg = warp - rg * p.ncg;
  const int trow0 = rg * M;  // first tile row of this warp
  const int col0 = cg * R;   // first tile column of this warp

  float2 acc[M][R];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[m][r] = make_float2(0.f, 0.f);

  bool ok = true;
  for (int st = 0; st < nsteps; ++st) {
    // Rows [st, st + tile_h) must be resident; earlier ones were waited on.
    if (st == 0) {
      for (int q = 0; q < min(p.tile_h, nrows) && ok; ++q) ok = mbar_wait_bounded(&full_x[q % RR], (q / RR) & 1, p.err, 1);
    } else {
      const int q = st + p.tile_h - 1;
      if (q < nrows) ok = mbar_wait_bounded(&full_x[q % RR], (q / RR) & 1, p.err, 1);
    }
    if (ok) ok = mbar_wait_bounded(&full_w[st % RW], (st / RW) & 1, p.err, 2);
    if (!ok) break;

    const int s = s_lo + st;  // kernel row
    const __half2* wrow = reinterpret_cast<const __half2*>(wring + (st % RW) * wrow_bytes) + lane;

    if constexpr (ACC == 0) {
      float2 wv[K];
#pragma unroll
      for (int kj = 0; kj < K; ++kj) wv[kj] = __half22float2(wrow[kj * kPixelH2]);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int out_row = h0 + trow0 + m;
        const int in_row = out_row - PAD + s;
        if (out_row < p.H && in_row >= 0 && in_row < p.H) {  // warp-uniform
          const int q = st + trow0 + m;
          const __half2* xrow =
              reinterpret_cast<const __half2*>(xring + (q % RR) * row_bytes) + col0 * kPixelH2 + lane;
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const float2 xv = __half22float2(xrow[j * kPixelH2]);
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int kj = j - r;
              if (kj >= 0 && kj < K) ffma2(acc[m][r], xv, wv[kj]);
            }
          }
        }
      }
    } else {
      __half2 wv[K];
#pragma unroll
      for (int kj = 0; kj < K; ++kj) wv[kj] = wrow[kj * kPixelH2];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int out_row = h0 + trow0 + m;
        const int in_row = out_row - PAD + s;
        if (out_row < p.H && in_row >= 0 && in_row < p.H) {
          const int q = st + trow0 + m;
          const __half2* xrow =
              reinterpret_cast<const __half2*>(xring + (q % RR) * row_bytes) + col0 * kPixelH2 + lane;
          __half2 part[R];
#pragma unroll
          for (int r = 0; r < R; ++r) part[r] = __float2half2_rn(0.f);
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const __half2 xv = xrow[j * kPixelH2];
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int kj = j - r;
              if (kj >= 0 && kj < K) part[r] = __hfma2(xv, wv[kj], part[r]);
            }
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float2 f = __half22float2(part[r]);
            acc[m][r].x += f.x;
            acc[m][r].y += f.y;
          }
        }
      }
    }

    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty_x[st % RR]);  // row st is never read again
      mbar_arrive(&empty_w[st % RW]);
    }
  }
  if (!ok) return;  // a bounded wait expired; the error word is set

  // ---------------- fused epilogue ----------------
  const int c = c0 + 2 * lane;
  if (c >= p.C) return;
  float2 bias = make_float2(0.f, 0.f), scale = make_float2(1.f, 1.f), shift = make_float2(0.f, 0.f);
  if (p.bias) bias = __half22float2(*reinterpret_cast<const __half2*>(p.bias + c));
  if (p.scale) scale = __half22float2(*reinterpret_cast<const __half2*>(p.scale + c));
  if (p.shift) shift = __half22float2(*reinterpret_cast<const __half2*>(p.shift + c));
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int h = h0 + trow0 + m;
    if (h >= p.H) continue;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int w = w0 + col0 + r;
      if (w >= p.W) continue;
      const long long off = ((static_cast<long long>(b) * p.H + h) * p.W + w) * p.C + c;
      float vx = apply_act(acc[m][r].x + bias.x, p.act) * scale.x + shift.x;
      float vy = apply_act(acc[m][r].y + bias.y, p.act) * scale.y + shift.y;
      if (p.residual) {
        const float2 res = __half22float2(*reinterpret_cast<const __half2*>(p.residual + off));
        vx += res.x;
        vy += res.y;
      }
      *reinterpret_cast<__half2*>(p.y + off) = __floats2half2_rn(vx, vy);
    }
  }
}

// One compiled variant of the kernel, registered for the launcher.
struct KernelEntry {
  int k, r, m, acc;
  const void* fn;
};

// Variants compiled into this library for kernel size K (nullptr-terminated
// by count).  Defined in dw_kernels_k*.cu.
int kernels_for_k(int K, const KernelEntry** out);

}  // namespace dwb
