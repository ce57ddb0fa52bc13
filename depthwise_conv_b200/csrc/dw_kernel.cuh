// dw_kernel.cuh -- the row-streaming depthwise convolution kernel for sm_100a.
//
// Work decomposition
//   tile = tile_h output rows x tile_w output columns x 64 channels of one
//          image (channels past C are zero-filled by TMA and never stored).
//   CTA  = persistent: it walks the tiles blockIdx.x, blockIdx.x + gridDim.x,
//          ... so the loads of the next tile overlap the last steps and the
//          epilogue of the current one.
//   warp = one "slot" of the tile: M consecutive output rows x R consecutive
//          output columns x 64 channels; lane l owns channels (2l, 2l+1), so
//          every shared-memory access of a warp is one contiguous 128-byte row
//          (conflict-free) and every row/column skip is warp-uniform.
//   thread accumulators: acc[M][R], packed fp32 pairs.
//
// Data movement (no multicast, plain per-CTA TMA tile loads)
//   The kernel walks the kernel rows ki (step s).  At step s every output row
//   h of the tile reads input row h - pad + s, so the tile needs the input
//   rows [h0 - pad + s, h0 - pad + s + tile_h): a window that slides one row
//   per step.  A dedicated producer warp streams the tile through a ring of
//   shared-memory "stages" guarded by one full and one empty mbarrier each;
//   the ring runs continuously across the CTA's tiles.  Stage q of a tile
//   holds staged input row q and, for q >= tile_h - 1, weight row
//   s_lo + q - (tile_h - 1) -- the weights of the step that first needs that
//   input row -- so every step waits for exactly one stage and releases
//   exactly one (stage st: its input row is never read again):
//     input row  : [tile_w + K - 1 columns][64 channels] fp16 (zero padding
//                  comes from TMA out-of-bounds fill)
//     weight row : [K taps][64 channels] fp16
//   Kernel rows whose input rows all fall outside the image are skipped.
//
// Load schedule (PRE): 0 = each input column is read from shared memory
//   right before the FMAs that use it; 1 = the warp first reads its whole
//   input row segment into registers, then runs the FMAs.  The two compile to
//   different instruction schedules; which is faster depends on K, R and M,
//   so both are compiled for the mixed mode and the planner/tuner picks.
//
// Inner loop (weight-stationary per kernel row)
//   The K weights of row ki are held in registers; then the thread slides
//   along R + K - 1 input columns of its M rows at once (the rows are
//   interleaved so each weight register feeds M independent chains): each
//   input half2 is loaded once and feeds up to R outputs.
//     ACC = 0: inputs and weights converted to fp32, packed fp32x2 FMAs
//              (FFMA2) into fp32 accumulators -- every tap in fp32;
//     ACC = 1: fp16x2 HFMA2 into short fp16 chains (one kernel row, or half
//              a row for K >= 25) that are added to the fp32 accumulators
//              when they end -- no conversion in the loop.
//
// Row split (S > 1, for small images where tiles are few)
//   S warps share each output slot; warp group g computes the kernel rows
//   s_lo + g, s_lo + g + S, ... into fp32 accumulators.  At the end of the
//   tile groups 1..S-1 store their accumulators in a shared-memory exchange
//   area and group 0 adds them before the epilogue.  The hand-off is two mbarriers (partials
//   written / area free again) with bounded waits, so a failing warp can
//   never leave the others blocked.  Every warp still waits for and releases
//   every stage in order, which keeps the ring protocol unchanged.
//
// Epilogue (fused): v = acc + bias; v = act(v); v = v * scale + shift;
//   v += residual; stored as half2, 128 contiguous bytes per warp.  When the
//   residual is the input itself (a ConvMixer block) and each CTA runs one
//   tile with a ring deep enough to hold all of its input rows, the residual is
//   read from the staged input rows in shared memory instead of from HBM/L2.
#pragma once

#include "dw_device.cuh"
#include "dw_planner.h"

namespace dwb {

constexpr int kChannelsPerCta = 64;                 // 32 lanes x 2 channels
constexpr int kPixelBytes = kChannelsPerCta * 2;    // one staged pixel = 128 B
constexpr int kPixelH2 = kChannelsPerCta / 2;       // half2 per staged pixel
constexpr int kBarrierBytes = 1024;                 // mbarrier area at smem start
constexpr bool kProducerSleeps = true;              // producer's empty-slot waits may suspend
// Consumers' stage waits spin on try_wait: letting them suspend as the producer does (leaving
// the issue slots to computing warps) measured 0-5% slower on B200.
constexpr bool kConsumerSleeps = false;

struct DwParams {
  __half* y;
  const __half* bias;      // [C] or nullptr
  const __half* scale;     // [C] or nullptr
  const __half* shift;     // [C] or nullptr
  const __half* residual;  // NHWC like y, or nullptr
  int B, H, W, C;
  int tile_h, tile_w, tile_w_in;
  int tiles_h, tiles_w, cblocks;
  uint32_t num_tiles;      // < 2^31 (checked by the launcher)
  int ncg;                 // column groups (warps across the tile width)
  int consumer_warps;                // nsplit * slots
  int slots;                         // warps per split group (ncg * row groups)
  int nsplit;                        // row split S (1 = none)
  int stages;                       // stage ring depth
  int act;
  uint32_t ring_off;                // byte offset of stage 0 inside dynamic smem
  uint32_t stage_bytes;             // (tile_w_in + K) staged pixels
  uint32_t red_off;                 // partial-sum exchange area (S > 1)
  int res_in_ring;                  // residual == input and every CTA keeps its one tile whole in the ring
  // band mode (dw_band_kernel): the CTA streams bands of band_tiles row tiles
  int band_tiles;                   // row tiles per band
  int bands_h;                      // bands per image column strip
  uint32_t num_bands;               // B * cblocks * tiles_w * bands_h
  uint32_t wbuf_off;                // two resident weight buffers of K*K staged pixels
  int* err;                         // device error word (bounded-wait expiry)
};

// Geometry of one tile.
struct TileInfo {
  int b, h0, w0, c0;
  int s_lo;    // first kernel row with an in-image input row
  int nsteps;  // kernel rows executed
  int nrows;   // input rows streamed = nsteps + tile_h - 1
};

template <int K>
__device__ __forceinline__ TileInfo decode_tile(const DwParams& p, uint32_t t) {
  constexpr int PAD = K / 2;
  TileInfo ti;
  // tile-row fastest so CTAs working at the same time share halo rows in L2
  uint32_t q = t / static_cast<uint32_t>(p.tiles_h);
  const int th = static_cast<int>(t - q * static_cast<uint32_t>(p.tiles_h));
  t = q;
  q = t / static_cast<uint32_t>(p.tiles_w);
  const int tw = static_cast<int>(t - q * static_cast<uint32_t>(p.tiles_w));
  t = q;
  q = t / static_cast<uint32_t>(p.cblocks);
  const int cbk = static_cast<int>(t - q * static_cast<uint32_t>(p.cblocks));
  ti.b = static_cast<int>(q);
  ti.h0 = th * p.tile_h;
  ti.w0 = tw * p.tile_w;
  ti.c0 = cbk * kChannelsPerCta;
  const int rows_in_tile = min(p.tile_h, p.H - ti.h0);
  ti.s_lo = max(0, PAD - (ti.h0 + rows_in_tile - 1));
  const int s_hi = min(K, p.H + PAD - ti.h0);
  ti.nsteps = s_hi - ti.s_lo;  // >= 1 because h0 < H
  ti.nrows = ti.nsteps + p.tile_h - 1;
  return ti;
}

// One kernel row for the warp's M rows (row m reads xrow[m]; rows whose
// input row lies outside the image are skipped, warp-uniformly).  In mixed
// mode the fp16 chains live only inside this call: each row's chains start
// with a product and end in the fp32 accumulators before the next row.  (Chains
// spanning two kernel rows halve the flushes of the small kernels but hold the
// chains in registers across the step boundary; measured on B200 that costs
// more than the flushes it saves: k7 and k9 layers 5-7% slower.)
template <int K, int R, int M, int ACC, int PRE>
__device__ __forceinline__ void step_rows(f32x2 (&acc)[M][R], const __half2* __restrict__ wrow,
                                          const __half2* __restrict__ xrow0, const __half2* __restrict__ xrow1,
                                          bool v0, bool v1) {
  constexpr int NJ = R + K - 1;
  constexpr int SPLIT = (ACC == 1 && K >= 25) ? 2 : 1;  // chains of at most 16 taps
  if constexpr (ACC == 0) {
    f32x2 wv[K];
#pragma unroll
    for (int kj = 0; kj < K; ++kj) wv[kj] = h2_to_f32x2(wrow[kj * kPixelH2]);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      if (m == 0 ? v0 : v1) {
        const __half2* xrow = m == 0 ? xrow0 : xrow1;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const f32x2 xv = h2_to_f32x2(xrow[j * kPixelH2]);
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
      if (m == 0 ? v0 : v1) {
        const __half2* xrow = m == 0 ? xrow0 : xrow1;
        __half2 part[SPLIT][R];  // each chain starts with a product (no zero initialisation)
        __half2 xs[PRE ? NJ : 1];
        if constexpr (PRE) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) xs[j] = xrow[j * kPixelH2];
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          __half2 xv;
          if constexpr (PRE) {
            xv = xs[j];
          } else {
            xv = xrow[j * kPixelH2];
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int kj = j - r;
            if (kj >= 0 && kj < K) {
              const int c = (SPLIT == 2 && kj >= K / 2 + 1) ? 1 : 0;
              const bool first = kj == 0 || (SPLIT == 2 && kj == K / 2 + 1);
              part[c][r] = first ? __hmul2(xv, wv[kj]) : __hfma2(xv, wv[kj], part[c][r]);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < SPLIT; ++c)
#pragma unroll
          for (int r = 0; r < R; ++r) add_h2_to_f32x2(acc[m][r], part[c][r]);
      }
    }
  }
}

// Epilogue of one warp slot: y = act(acc + bias) * scale + shift (+ residual).  ACT / RES / FULL are
// resolved once per tile by the caller, so the loop is straight-line code
// (FULL: every row and column of the slot is inside the image).
// The residual of output row m, column r is res_row[m][r * res_col]: rows of
// the residual tensor in global memory, or (a ConvMixer block, residual = the
// input) the staged input rows still resident in the stage ring.
template <int ACT, bool RES, bool FULL, int M, int R>
__device__ __forceinline__ void store_slot(const f32x2 (&acc)[M][R], f32x2 bias, f32x2 scale, f32x2 shift,
                                           __half2* y, const __half2* const (&res_row)[2], int res_col,
                                           long long row_h2, int col_h2, int rows_valid, int cols_valid) {
#pragma unroll
  for (int m = 0; m < M; ++m) {
    if (!FULL && m >= rows_valid) break;
    __half2* yp = y + m * row_h2;
    const __half2* rp = RES ? res_row[m] : nullptr;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (!FULL && r >= cols_valid) break;
      f32x2 a = acc[m][r];
      fadd2(a, bias);
      if (ACT == kActGelu) {
        a = gelu_erf2(a);
      } else if (ACT == kActRelu) {
        const float2 f = bits_f2(a);
        a = f2_bits(make_float2(fmaxf(f.x, 0.0f), fmaxf(f.y, 0.0f)));
      }
      f32x2 v = fma2(a, scale, shift);  // a * scale + shift, both channels in one FFMA2
      if (RES) fadd2(v, h2_to_f32x2(rp[r * res_col]));
      const float2 o = bits_f2(v);
      yp[r * col_h2] = __floats2half2_rn(o.x, o.y);
    }
  }
}

template <int ACT, bool RES, int M, int R>
__device__ __forceinline__ void store_tile_slot(const f32x2 (&acc)[M][R], f32x2 bias, f32x2 scale, f32x2 shift,
                                                __half2* y, const __half2* const (&res_row)[2], int res_col,
                                                long long row_h2, int col_h2, int rows_valid, int cols_valid) {
  if (rows_valid == M && cols_valid == R)
    store_slot<ACT, RES, true>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid);
  else
    store_slot<ACT, RES, false>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid);
}

// Register cap of a variant (dw_regcaps.inc; 255 = none).
struct RegCap {
  int k, r, m, acc, pre, cap;
};
constexpr RegCap kRegCaps[] = {
#include "dw_regcaps.inc"
    {0, 0, 0, 0, 0, 255}};
template <int K, int R, int M, int ACC, int PRE>
constexpr int reg_cap() {
#if defined(DWB_FORCE_CAP)
  return DWB_FORCE_CAP;  // build.py --regcaps: every variant at one cap, to read ptxas's spills
#elif defined(DWB_NO_REGCAPS)
  return 255;
#else
  for (const RegCap& c : kRegCaps)
    if (c.k == K && c.r == R && c.m == M && c.acc == ACC && c.pre == PRE) return c.cap;
  return 255;
#endif
}

// End of a tile for one consumer warp: the row-split hand-off of the fp32
// partial sums (S > 1: groups 1..S-1 store theirs in the exchange area, group 0
// adds them) and the fused epilogue of group 0.  Returns false if a bounded wait
// expired.  rows_end: first output row past the tile's valid rows.  res_ring:
// the residual rows in the stage ring (ConvMixer block, see res_in_ring), or
// null to read the residual tensor from global memory.
template <int M, int R>
__device__ __forceinline__ bool finish_tile(const DwParams& p, unsigned char* smem, uint64_t* red_full,
                                           uint64_t* red_empty, f32x2 (&acc)[M][R], int sg, int slot_id,
                                           uint32_t tile_iter, int lane, int b, int out0, int rows_end, int w0,
                                           int c0, int col0, f32x2 bias, f32x2 scale, f32x2 shift,
                                           const __half2* const (&res_ring)[2]) {
  if (p.nsplit > 1) {
    // exchange area: [group 1..S-1][slot][m][r][lane] packed fp32 pairs, so
    // a warp's access to one (m, r) is 256 contiguous bytes
    f32x2* red = reinterpret_cast<f32x2*>(smem + p.red_off) + lane;
    constexpr int kSlotPairs = M * R * 32;
    if (sg > 0) {
      if (tile_iter > 0) {  // group 0 has read the previous tile's partials
        if (!mbar_wait_bounded(red_empty, (tile_iter - 1) & 1u, p.err, 4)) return false;
      }
      f32x2* dst = red + ((sg - 1) * p.slots + slot_id) * kSlotPairs;
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) dst[(m * R + r) * 32] = acc[m][r];
      mbar_arrive(red_full);  // every lane, after its own stores (release)
      return true;
    }
    if (!mbar_wait_bounded(red_full, tile_iter & 1u, p.err, 4)) return false;
    for (int g = 1; g < p.nsplit; ++g) {
      const f32x2* src = red + ((g - 1) * p.slots + slot_id) * kSlotPairs;
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) fadd2(acc[m][r], src[(m * R + r) * 32]);
    }
    mbar_arrive(red_empty);  // every lane, after its own loads
  }

  // ---------------- fused epilogue ----------------
  const int c = c0 + 2 * lane;
  const int rows_valid = min(M, rows_end - out0);
  const int cols_valid = min(R, p.W - (w0 + col0));
  if (c < p.C && rows_valid > 0 && cols_valid > 0) {
    const long long base = ((static_cast<long long>(b) * p.H + out0) * p.W + w0 + col0) * p.C + c;
    __half2* y = reinterpret_cast<__half2*>(p.y + base);
    const long long row_h2 = static_cast<long long>(p.W) * p.C / 2;
    const int col_h2 = p.C / 2;
    const __half2* res_row[2] = {res_ring[0], res_ring[1]};
    int res_col = kPixelH2;
    if (!res_ring[0]) {
      res_col = col_h2;
      if (p.residual) {
        res_row[0] = reinterpret_cast<const __half2*>(p.residual + base);
        res_row[1] = res_row[0] + row_h2;
      }
    }
    switch (p.act * 2 + (res_row[0] != nullptr)) {  // one branch per tile, then straight-line stores
      case 0: store_tile_slot<kActNone, false>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid); break;
      case 1: store_tile_slot<kActNone, true>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid); break;
      case 2: store_tile_slot<kActRelu, false>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid); break;
      case 3: store_tile_slot<kActRelu, true>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid); break;
      case 4: store_tile_slot<kActGelu, false>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid); break;
      default: store_tile_slot<kActGelu, true>(acc, bias, scale, shift, y, res_row, res_col, row_h2, col_h2, rows_valid, cols_valid); break;
    }
  }
  return true;
}

// Per-channel epilogue parameters of lane's two channels at channel block c0.
__device__ __forceinline__ void load_channel_params(const DwParams& p, int c0, int lane, f32x2& bias, f32x2& scale,
                                                    f32x2& shift) {
  const int c = c0 + 2 * lane;
  float2 b = make_float2(0.f, 0.f), sc = make_float2(1.f, 1.f), sh = make_float2(0.f, 0.f);
  if (c < p.C) {
    if (p.bias) b = __half22float2(*reinterpret_cast<const __half2*>(p.bias + c));
    if (p.scale) sc = __half22float2(*reinterpret_cast<const __half2*>(p.scale + c));
    if (p.shift) sh = __half22float2(*reinterpret_cast<const __half2*>(p.shift + c));
  }
  bias = f2_bits(b);
  scale = f2_bits(sc);
  shift = f2_bits(sh);
}

template <int K, int R, int M, int ACC, int PRE>
__device__ __forceinline__ void dw_stream_body(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const DwParams& p) {
  constexpr int PAD = K / 2;
  extern __shared__ __align__(1024) unsigned char smem[];

  const int NS = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NS;
  uint64_t* red_full = empty + NS;     // row split: partial sums of a tile written
  uint64_t* red_empty = red_full + 1;  // row split: exchange area free again
  unsigned char* ring = smem + p.ring_off;
  const uint32_t row_bytes = static_cast<uint32_t>(p.tile_w_in) * kPixelBytes;  // weight row follows it
  constexpr uint32_t wrow_bytes = K * kPixelBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], p.consumer_warps);
    }
    if (p.nsplit > 1) {
      mbar_init(red_full, (p.nsplit - 1) * p.slots * 32);  // one arrival per thread of groups 1..S-1
      mbar_init(red_empty, p.slots * 32);                  // one arrival per thread of group 0
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Everything above overlaps the previous kernel of the stream (programmatic
  // dependent launch); from here on the kernel reads and writes global memory,
  // and the next kernel may start its own set-up.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == p.consumer_warps) {
    // ---------------- producer warp ----------------
    // Fills the stages in order; a stage is refilled only after every
    // consumer warp released its previous use (empty barrier).  Fill q of a
    // tile: its input row (skipped outside the image) and, for q >= tile_h - 1,
    // the weight row of the step that first needs that input row.
    auto fill = [&](int slot, const TileInfo& ti, int q) {
      const int abs_row = ti.h0 - PAD + ti.s_lo + q;
      unsigned char* dst = ring + slot * p.stage_bytes;
      const bool xrow = abs_row >= 0 && abs_row < p.H;
      const bool wrow = q >= p.tile_h - 1;
      const uint32_t bytes = (xrow ? row_bytes : 0u) + (wrow ? wrow_bytes : 0u);
      if (bytes) {
        mbar_arrive_expect_tx(&full[slot], bytes);
        if (xrow) tma_load_4d(dst, &tmap_x, &full[slot], ti.c0, ti.w0 - PAD, abs_row, ti.b);
        if (wrow) tma_load_3d(dst + row_bytes, &tmap_w, &full[slot], ti.c0, 0, ti.s_lo + q - (p.tile_h - 1));
      } else {
        mbar_arrive(&full[slot]);  // nothing to load (rows above/below the image are skipped)
      }
    };
    // The CTA's first fills find every stage free, so lane q issues fill q of
    // the first tile: one thread issuing TMA loads back to back waits ~100
    // clocks per load, and the first compute step needs tile_h of them.
    int first = 0;
    if (blockIdx.x < p.num_tiles) {
      const TileInfo ti = decode_tile<K>(p, blockIdx.x);
      first = min(min(NS, ti.nrows), 32);
      if (lane < first) fill(lane, ti, lane);
    }
    __syncwarp();
    if (lane == 0) {
      RingPos fr;  // next stage to fill, and the parity of that fill
      for (int i = 0; i < first; ++i) fr.next(NS);
      long long fills = first;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        const TileInfo ti = decode_tile<K>(p, t);
        for (int q = (t == blockIdx.x) ? first : 0; q < ti.nrows; ++q) {
          if (fills >= NS) ok = mbar_wait_bounded<kProducerSleeps>(&empty[fr.slot], fr.phase ^ 1u, p.err, 3);
          if (!ok) break;
          fill(fr.slot, ti, q);
          fr.next(NS);
          ++fills;
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int sg = warp / p.slots;            // split group: kernel rows st = sg (mod nsplit)
  const int slot_id = warp - sg * p.slots;  // output slot within the tile
  const int rg = slot_id / p.ncg;
  const int cg = slot_id - rg * p.ncg;
  const int trow0 = rg * M;  // first tile row of this warp
  const int col0 = cg * R;   // first tile column of this warp
  const int xoff = col0 * kPixelH2 + lane;  // half2 offset of this thread's first input column

  RingPos wait_s;  // next stage to wait for
  RingPos rel_s;   // next stage to release (stage st of the current tile during step st)
  bool ok = true;

  f32x2 bias = 0, scale = 0, shift = 0;
  int bias_c0 = -1;
  uint32_t tile_iter = 0;  // tiles this CTA has finished (phase of the split hand-off)

  for (uint32_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++tile_iter) {
    const TileInfo ti = decode_tile<K>(p, t);

    // per-channel epilogue parameters, reloaded when the tile's channels change
    if (ti.c0 != bias_c0) {
      bias_c0 = ti.c0;
      load_channel_params(p, ti.c0, lane, bias, scale, shift);
    }

    // packed fp32 (channel 2l, channel 2l+1); the bias is added in the epilogue, so the
    // parameter loads above are not waited for before the first step
    f32x2 acc[M][R];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < R; ++r) acc[m][r] = f32x2_zero();
    int turn = sg;  // steps until this warp's next kernel row

    // warps whose columns all lie right of the image have nothing to compute
    const bool any_col = ti.w0 + col0 < p.W;

    // stage of row trow0 of this tile (stage 0 of the tile is at rel_s)
    const int tile_slot0 = rel_s.slot;
    int my_slot = rel_s.slot + trow0;
    if (my_slot >= NS) my_slot -= NS;

    // Stages [0, tile_h - 1) hold input rows that step 0 needs as well.
    for (int q = 0; q < p.tile_h - 1 && ok; ++q) {
      ok = mbar_wait_bounded<kConsumerSleeps>(&full[wait_s.slot], wait_s.phase, p.err, 1);
      wait_s.next(NS);
    }

    bool ready = false;  // this step's stage was found complete during the previous step
    for (int st = 0; st < ti.nsteps && ok; ++st) {
      // stage st + tile_h - 1: the last input row and the weight row of this step
      if (!ready) ok = mbar_wait_bounded<kConsumerSleeps>(&full[wait_s.slot], wait_s.phase, p.err, 2);
      if (!ok) break;
      const __half2* wrow = reinterpret_cast<const __half2*>(ring + wait_s.slot * p.stage_bytes + row_bytes) + lane;
      wait_s.next(NS);
      // probe the next step's stage now; the answer is read after this step's FMAs
      ready = st + 1 < ti.nsteps && mbar_test_wait(&full[wait_s.slot], wait_s.phase);

      const int s = ti.s_lo + st;  // kernel row
      const int slot1 = (my_slot + 1 == NS) ? 0 : my_slot + 1;
      const __half2* xrow0 = reinterpret_cast<const __half2*>(ring + my_slot * p.stage_bytes) + xoff;
      const __half2* xrow1 = reinterpret_cast<const __half2*>(ring + slot1 * p.stage_bytes) + xoff;
      const int out0 = ti.h0 + trow0;
      const int in0 = out0 - PAD + s;
      const bool mine = turn == 0;  // warp-uniform
      turn = mine ? p.nsplit - 1 : turn - 1;
      const bool v0 = mine && any_col && out0 < p.H && in0 >= 0 && in0 < p.H;                        // warp-uniform
      const bool v1 = mine && any_col && M == 2 && out0 + 1 < p.H && in0 + 1 >= 0 && in0 + 1 < p.H;  // warp-uniform

      if (v0 || v1) {
        step_rows<K, R, M, ACC, PRE>(acc, wrow, xrow0, xrow1, v0, v1);
      }

      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[rel_s.slot]);  // input row st of the tile is never read again
      rel_s.next(NS);
      my_slot = slot1;
    }
    if (!ok) break;
    // The last tile_h - 1 stages of the tile are done too.
    __syncwarp();
    for (int q = ti.nsteps; q < ti.nrows; ++q) {
      if (lane == 0) mbar_arrive(&empty[rel_s.slot]);
      rel_s.next(NS);
    }

    const __half2* res_ring[2] = {nullptr, nullptr};
    if (p.res_in_ring) {
      // residual = the input, and this CTA's only tile is still whole in the ring: output row
      // trow0 + m reads input row h0 + trow0 + m, staged at tile position trow0 + m + PAD - s_lo,
      // column col0 + r + PAD of the staged row
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int q = (tile_slot0 + trow0 + m + PAD - ti.s_lo) % NS;
        res_ring[m] = reinterpret_cast<const __half2*>(ring + q * p.stage_bytes) + (col0 + PAD) * kPixelH2 + lane;
      }
    }
    ok = finish_tile<M, R>(p, smem, red_full, red_empty, acc, sg, slot_id, tile_iter, lane, ti.b, ti.h0 + trow0,
                           p.H, ti.w0, ti.c0, col0, bias, scale, shift, res_ring);
  }
}

// ---------------------------------------------------------------------------
// Band mode.  The tile kernel above stages tile_h + K - 1 input rows (and the K
// weight rows) for every tile of tile_h output rows, so a short tile reloads
// its K - 1 halo rows and the weights each time; TMA issues one 128-byte
// request per staged pixel, and on batched layers with small K those
// requests, not the FMAs, set the pace.  In band mode a CTA walks a band of
// band_tiles consecutive row tiles of one column strip (one image, 64
// channels, tile_w columns): every input row of the band enters the ring once
// and stays until the last tile that reads it is done, and the band's K x K
// weights are loaded once into one of two resident buffers (double-buffered
// across bands).
//
// Rows of a band are numbered v = 0 .. nv - 1 (input row h_lo - PAD + v; rows
// outside the image are counted but not loaded, and no FMA reads them).  Tile
// th (output rows h_lo + th * tile_h ...) reads rows [th * tile_h, th * tile_h
// + tile_h + K - 1) and step s of it rows th * tile_h + s + [0, tile_h).  A
// consumer warp waits for the rows in order as the steps need them and
// releases row th * tile_h + s after step s when s < tile_h (no later tile
// reads it), the rest of the tile's first tile_h rows at its end, and all
// remaining rows at the band's end -- each row is waited for and released
// once by every consumer warp, in order, as in the tile kernel.  A ring of
// tile_h + K - 1 or more stages never deadlocks: the oldest row a step can
// need a stage for was released at least K steps earlier.
struct BandInfo {
  int b, c0, w0;
  int h_lo, h_hi;  // output rows of the band
  int ntiles;      // row tiles in the band
  int nv;          // rows streamed: (h_hi - h_lo) + K - 1
};

template <int K>
__device__ __forceinline__ BandInfo decode_band(const DwParams& p, uint32_t j) {
  BandInfo bi;
  // band fastest, then column tile, channel block, image: CTAs working at the same time share
  // the halo rows between neighbouring bands in L2
  uint32_t q = j / static_cast<uint32_t>(p.bands_h);
  const int bh = static_cast<int>(j - q * static_cast<uint32_t>(p.bands_h));
  j = q;
  q = j / static_cast<uint32_t>(p.tiles_w);
  const int tw = static_cast<int>(j - q * static_cast<uint32_t>(p.tiles_w));
  j = q;
  q = j / static_cast<uint32_t>(p.cblocks);
  const int cbk = static_cast<int>(j - q * static_cast<uint32_t>(p.cblocks));
  bi.b = static_cast<int>(q);
  bi.c0 = cbk * kChannelsPerCta;
  bi.w0 = tw * p.tile_w;
  const int band_rows = p.band_tiles * p.tile_h;
  bi.h_lo = bh * band_rows;
  bi.h_hi = min(p.H, bi.h_lo + band_rows);
  bi.ntiles = (bi.h_hi - bi.h_lo + p.tile_h - 1) / p.tile_h;
  bi.nv = bi.h_hi - bi.h_lo + K - 1;
  return bi;
}

template <int K, int R, int M, int ACC, int PRE>
__device__ __forceinline__ void dw_band_body(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const DwParams& p) {
  constexpr int PAD = K / 2;
  constexpr uint32_t kWeightBytes = K * K * kPixelBytes;
  extern __shared__ __align__(1024) unsigned char smem[];

  const int NS = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NS;
  uint64_t* red_full = empty + NS;
  uint64_t* red_empty = red_full + 1;
  uint64_t* wfull = red_empty + 1;  // [2] resident weight buffer loaded
  uint64_t* wempty = wfull + 2;     // [2] resident weight buffer free again
  unsigned char* ring = smem + p.ring_off;
  const uint32_t row_bytes = static_cast<uint32_t>(p.tile_w_in) * kPixelBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], p.consumer_warps);
    }
    if (p.nsplit > 1) {
      mbar_init(red_full, (p.nsplit - 1) * p.slots * 32);
      mbar_init(red_empty, p.slots * 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], p.consumer_warps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();

  if (warp == p.consumer_warps) {
    // ---------------- producer warp ----------------
    auto fill = [&](int slot, const BandInfo& bi, int v) {
      const int row = bi.h_lo - PAD + v;
      if (row >= 0 && row < p.H) {
        mbar_arrive_expect_tx(&full[slot], row_bytes);
        tma_load_4d(ring + slot * p.stage_bytes, &tmap_x, &full[slot], bi.c0, bi.w0 - PAD, row, bi.b);
      } else {
        mbar_arrive(&full[slot]);  // rows above/below the image: nothing to load, never read
      }
    };
    // the CTA's first band: its weights and first rows issued by separate lanes (as in the tile kernel)
    int first = 0;
    if (blockIdx.x < p.num_bands) {
      const BandInfo bi = decode_band<K>(p, blockIdx.x);
      first = min(min(NS, bi.nv), 31);
      if (lane == 31) {
        mbar_arrive_expect_tx(&wfull[0], kWeightBytes);
        tma_load_3d(smem + p.wbuf_off, &tmap_w, &wfull[0], bi.c0, 0, 0);
      } else if (lane < first) {
        fill(lane, bi, lane);
      }
    }
    __syncwarp();
    if (lane == 0) {
      RingPos fr;
      for (int i = 0; i < first; ++i) fr.next(NS);
      long long fills = first;
      bool ok = true;
      uint32_t it = 0;
      for (uint32_t j = blockIdx.x; j < p.num_bands && ok; j += gridDim.x, ++it) {
        const BandInfo bi = decode_band<K>(p, j);
        const int par = static_cast<int>(it & 1u);
        if (it > 0) {
          // the k-th use of weight buffer par waits until every consumer is done with use k - 1
          if (it >= 2) ok = mbar_wait_bounded<kProducerSleeps>(&wempty[par], ((it >> 1) - 1) & 1u, p.err, 3);
          if (!ok) break;
          mbar_arrive_expect_tx(&wfull[par], kWeightBytes);
          tma_load_3d(smem + p.wbuf_off + par * kWeightBytes, &tmap_w, &wfull[par], bi.c0, 0, 0);
        }
        for (int v = (it == 0) ? first : 0; v < bi.nv; ++v) {
          if (fills >= NS) ok = mbar_wait_bounded<kProducerSleeps>(&empty[fr.slot], fr.phase ^ 1u, p.err, 3);
          if (!ok) break;
          fill(fr.slot, bi, v);
          fr.next(NS);
          ++fills;
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int sg = warp / p.slots;
  const int slot_id = warp - sg * p.slots;
  const int rg = slot_id / p.ncg;
  const int cg = slot_id - rg * p.ncg;
  const int trow0 = rg * M;
  const int col0 = cg * R;
  const int xoff = col0 * kPixelH2 + lane;

  RingPos wait_s;  // next row to wait for (continues across bands)
  RingPos rel_s;   // next row to release
  bool ok = true;
  f32x2 bias = 0, scale = 0, shift = 0;
  int bias_c0 = -1;
  uint32_t tile_iter = 0;
  uint32_t it = 0;
  const __half2* const no_ring[2] = {nullptr, nullptr};

  for (uint32_t j = blockIdx.x; j < p.num_bands && ok; j += gridDim.x, ++it) {
    const BandInfo bi = decode_band<K>(p, j);
    const int par = static_cast<int>(it & 1u);
    if (bi.c0 != bias_c0) {
      bias_c0 = bi.c0;
      load_channel_params(p, bi.c0, lane, bias, scale, shift);
    }
    ok = mbar_wait_bounded<kConsumerSleeps>(&wfull[par], (it >> 1) & 1u, p.err, 1);
    if (!ok) break;
    const __half2* wbase = reinterpret_cast<const __half2*>(smem + p.wbuf_off + par * kWeightBytes) + lane;
    const int band_slot0 = wait_s.slot;  // every row of the previous band was waited for and released
    const bool any_col = bi.w0 + col0 < p.W;
    int wait_v = 0, rel_v = 0;

    for (int th = 0; th < bi.ntiles && ok; ++th, ++tile_iter) {
      const int h0rel = th * p.tile_h;
      const int out0 = bi.h_lo + h0rel + trow0;
      f32x2 acc[M][R];
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[m][r] = f32x2_zero();
      int turn = sg;
      int my_slot = (band_slot0 + h0rel + trow0) % NS;

      bool ready = false;  // row wait_v was found complete during the previous step
      for (int s = 0; s < K; ++s) {
        const int need = min(h0rel + s + p.tile_h - 1, bi.nv - 1);
        while (wait_v <= need) {
          if (!ready) ok = mbar_wait_bounded<kConsumerSleeps>(&full[wait_s.slot], wait_s.phase, p.err, 2);
          ready = false;
          if (!ok) break;
          wait_s.next(NS);
          ++wait_v;
        }
        if (!ok) break;
        // probe the row the next step waits for first; the answer is read after this step's FMAs
        ready = wait_v < bi.nv && mbar_test_wait(&full[wait_s.slot], wait_s.phase);
        const int slot1 = (my_slot + 1 == NS) ? 0 : my_slot + 1;
        const __half2* xrow0 = reinterpret_cast<const __half2*>(ring + my_slot * p.stage_bytes) + xoff;
        const __half2* xrow1 = reinterpret_cast<const __half2*>(ring + slot1 * p.stage_bytes) + xoff;
        const __half2* wrow = wbase + s * K * kPixelH2;
        const int in0 = out0 - PAD + s;
        const bool mine = turn == 0;
        turn = mine ? p.nsplit - 1 : turn - 1;
        const bool v0 = mine && any_col && out0 < bi.h_hi && in0 >= 0 && in0 < p.H;
        const bool v1 = mine && any_col && M == 2 && out0 + 1 < bi.h_hi && in0 + 1 >= 0 && in0 + 1 < p.H;
        if (v0 || v1) {
          step_rows<K, R, M, ACC, PRE>(acc, wrow, xrow0, xrow1, v0, v1);
        }
        __syncwarp();
        if (s < p.tile_h && rel_v == h0rel + s && rel_v < bi.nv) {  // no later tile reads this row
          if (lane == 0) mbar_arrive(&empty[rel_s.slot]);
          rel_s.next(NS);
          ++rel_v;
        }
        my_slot = slot1;
      }
      if (!ok) break;
      // rows no later tile of the band reads (all of them after the band's last tile)
      __syncwarp();
      const int rel_to = (th == bi.ntiles - 1) ? bi.nv : min(h0rel + p.tile_h, bi.nv);
      while (rel_v < rel_to) {
        if (lane == 0) mbar_arrive(&empty[rel_s.slot]);
        rel_s.next(NS);
        ++rel_v;
      }
      ok = finish_tile<M, R>(p, smem, red_full, red_empty, acc, sg, slot_id, tile_iter, lane, bi.b, out0, bi.h_hi,
                             bi.w0, bi.c0, col0, bias, scale, shift, no_ring);
    }
    if (!ok) break;
    __syncwarp();
    if (lane == 0) mbar_arrive(&wempty[par]);  // this band's weights are no longer read
  }
}

// The kernel, without and with a register cap.  A variant without an entry
// in dw_regcaps.inc is compiled with no __maxnreg__ at all (ptxas's own
// choice), one with an entry under that cap.
template <int K, int R, int M, int ACC, int PRE>
__global__ void dw_stream_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                 const __grid_constant__ CUtensorMap tmap_w, const DwParams p) {
  dw_stream_body<K, R, M, ACC, PRE>(tmap_x, tmap_w, p);
}
template <int K, int R, int M, int ACC, int PRE, int CAP>
__global__ void __maxnreg__(CAP) dw_stream_kernel_capped(const __grid_constant__ CUtensorMap tmap_x,
                                                         const __grid_constant__ CUtensorMap tmap_w,
                                                         const DwParams p) {
  dw_stream_body<K, R, M, ACC, PRE>(tmap_x, tmap_w, p);
}
template <int K, int R, int M, int ACC, int PRE>
__global__ void dw_band_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                               const DwParams p) {
  dw_band_body<K, R, M, ACC, PRE>(tmap_x, tmap_w, p);
}
template <int K, int R, int M, int ACC, int PRE, int CAP>
__global__ void __maxnreg__(CAP) dw_band_kernel_capped(const __grid_constant__ CUtensorMap tmap_x,
                                                       const __grid_constant__ CUtensorMap tmap_w, const DwParams p) {
  dw_band_body<K, R, M, ACC, PRE>(tmap_x, tmap_w, p);
}
template <int K, int R, int M, int ACC, int PRE>
inline const void* band_kernel_fn() {
  constexpr int cap = reg_cap<K, R, M, ACC, PRE>();
  if constexpr (cap < 255) {
    return reinterpret_cast<const void*>(&dw_band_kernel_capped<K, R, M, ACC, PRE, cap>);
  } else {
    return reinterpret_cast<const void*>(&dw_band_kernel<K, R, M, ACC, PRE>);
  }
}
template <int K, int R, int M, int ACC, int PRE>
inline const void* kernel_fn() {
  constexpr int cap = reg_cap<K, R, M, ACC, PRE>();
  if constexpr (cap < 255) {
    return reinterpret_cast<const void*>(&dw_stream_kernel_capped<K, R, M, ACC, PRE, cap>);
  } else {
    return reinterpret_cast<const void*>(&dw_stream_kernel<K, R, M, ACC, PRE>);
  }
}

// One compiled variant of the kernel, registered for the launcher (band:
// the band-mode kernel of the same variant, or null where none is built).
struct KernelEntry {
  int k, r, m, acc, pre;
  const void* fn;
  const void* band;
};

// Variants compiled into this library for kernel size K.  Defined in
// dw_kernels_k*.cu.
int kernels_for_k(int K, const KernelEntry** out);

}  // namespace dwb
