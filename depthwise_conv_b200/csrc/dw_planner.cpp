// dw_planner.cpp -- choose (R, M, tile, row split, stage ring depth, load
// schedule) for the row-streaming kernel.
//
// The planner enumerates the compiled variants and tile shapes and keeps the
// one with the lowest modelled time on the busiest SM:
//   * work is counted in FMA-pipe clocks per warp: a valid (output row,
//     kernel row) pair costs 2*R*K clocks plus the flush (mixed) or the
//     conversion of the R + K - 1 staged inputs (fp32), and every kernel row
//     costs its K weights; rows whose input falls outside the image are not
//     counted (the kernel skips them);
//   * an SM runs min(ctas_per_sm, ...) CTAs at once over 4 sub-partitions;
//     fewer than one resident warp per sub-partition idles the others;
//   * every CTA streams its stages (input row + weight row) of 128-byte
//     pixels from L2, at about 64 bytes per clock per SM, and pays the load
//     latency once per step it cannot prefetch (ring depth);
//   * a row split S divides a slot's kernel rows over S warps (one warp's
//     critical path shrinks, the partial sums are handed over at the end);
//   * the load schedule is the one measured better for the kernel size
//     (default_load_schedule); the tuner measures both.
#include "dw_planner.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace dwb {

const int kVariantR[kNumVariantR] = {32, 28, 16, 14, 8, 7};

bool variant_compiled(int K, int R, int M, int acc, int pre) {
  if (M != 1 && M != 2) return false;
  if (pre != 0 && !(pre == 1 && acc == DWB_ACCUM_MIXED)) return false;
  if (R == 7 || R == 8 || R == 14 || R == 16) return true;
  return (R == 28 || R == 32) && K <= 13;
}
const int kVariantM[2] = {2, 1};

bool band_compiled(int K, int acc) { return acc == DWB_ACCUM_MIXED && K <= kBandMaxK; }

int default_load_schedule(int K, int R, int M, int acc) {
  (void)R;
  (void)M;
  // measured on B200: reading the row up front wins for the smallest and the
  // middle kernel sizes, the interleaved schedule for K = 9..13 and K >= 29
  if (acc != DWB_ACCUM_MIXED) return 0;
  return (K <= 7 || (K >= 15 && K <= 27)) ? 1 : 0;
}

namespace {
constexpr int kChannelsPerCta = 64;
constexpr int kPixelBytes = 128;
constexpr int kBarrierBytes = 1024;
constexpr int kMaxConsumerWarps = 31;  // a CTA of at most 32 warps (1024 threads) with its producer
constexpr int kMaxBoxDim = 256;  // TMA box limit per dimension
constexpr double kLoadLatency = 2000.0;  // clocks from TMA issue to data (L2/HBM), modelled
// TMA tile loads of 64-channel NHWC pixels: one 128-byte request per staged
// pixel, about 8 clocks each per SM (measured on B200 from the issue times of
// back-to-back row loads), i.e. ~16 bytes per clock per SM
constexpr double kTmaBytesPerClk = 16.0;
constexpr int kNumSplits = 5;
constexpr int kSplits[kNumSplits] = {1, 2, 3, 4, 8};  // row splits the planner considers

inline long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }

// Registers are allocated per warp in units of 256, and a CTA's warps are
// spread round-robin over the SM's 4 sub-partitions, each with a quarter of
// the register file.  Returns how many CTAs of `warps` warps fit on one SM by
// registers (0 = not even one).
inline int ctas_by_registers(int regs_per_thread, int warps, int regs_per_sm) {
  const long long per_warp = ceil_div(static_cast<long long>(regs_per_thread) * 32, 256) * 256;
  const long long warps_per_smsp = (regs_per_sm / 4) / per_warp;  // warps one sub-partition can hold
  const long long cta_warps_per_smsp = (warps + 3) / 4;            // a CTA's share of one sub-partition
  return static_cast<int>(warps_per_smsp / cta_warps_per_smsp);    // conservative
}

// Valid kernel rows for output row h (input rows inside [0, H)).
inline int valid_taps(int h, int H, int K) {
  const int pad = K / 2;
  return std::min(K, H + pad - h) - std::max(0, pad - h);
}
}  // namespace

int estimate_regs(int K, int R, int M, int acc) {
  // accumulators (2 per output) + weights + fp16 chain partials + addressing
  const int w = acc == 0 ? 2 * K : K;
  const int part = acc == 0 ? 0 : (K >= 25 ? 2 * R : R);
  int est = 2 * M * R + w + part + 28;
  return std::min(255, std::max(48, est));
}

long long plan_smem_bytes(int K, int tile_w_in, int stages, int nsplit, int slots, int M, int R, long long* red_off) {
  long long off = kBarrierBytes + static_cast<long long>(stages) * (tile_w_in + K) * kPixelBytes;
  if (red_off) *red_off = off;
  if (nsplit > 1) off += static_cast<long long>(nsplit - 1) * slots * M * R * 32 * 8;
  return off;
}

long long band_smem_bytes(int K, int tile_w_in, int stages, int nsplit, int slots, int M, int R, long long* red_off,
                          long long* wbuf_off) {
  long long off = kBarrierBytes + static_cast<long long>(stages) * tile_w_in * kPixelBytes;
  if (red_off) *red_off = off;
  if (nsplit > 1) off += static_cast<long long>(nsplit - 1) * slots * M * R * 32 * 8;
  off = (off + 127) / 128 * 128;
  if (wbuf_off) *wbuf_off = off;
  return off + 2LL * K * K * kPixelBytes;
}

bool barriers_fit(int stages, bool band) { return (2 * stages + 2 + (band ? 4 : 0)) * 8 <= kBarrierBytes; }

int validate_problem(const dwb_problem& pr) {
  const long long B = pr.batch, H = pr.height, W = pr.width, C = pr.channels;
  const int K = pr.kernel_size;
  if (pr.accum != DWB_ACCUM_F32 && pr.accum != DWB_ACCUM_MIXED) return DWB_ERR_BAD_ARG;
  if (B < 0 || H < 1 || W < 1 || C < 1) return DWB_ERR_BAD_SHAPE;
  if (K < 1 || K > 31 || (K % 2) == 0) return DWB_ERR_BAD_SHAPE;
  if (C % 8 != 0) return DWB_ERR_BAD_SHAPE;
  if (H > (1LL << 30) || W > (1LL << 30) || C > (1LL << 30) || B > (1LL << 30)) return DWB_ERR_BAD_SHAPE;
  return DWB_OK;
}

int enumerate_plans(const dwb_problem& pr, const HwInfo& hw, RegsFn regs, void* ctx, PlanSink sink, void* sink_ctx) {
  const int vst = validate_problem(pr);
  if (vst != DWB_OK) return vst;
  const long long B = pr.batch, H = pr.height, W = pr.width, C = pr.channels;
  const int K = pr.kernel_size;
  const long long cblocks = ceil_div(C, kChannelsPerCta);
  const int pad = K / 2;
  int count = 0;

  for (int ri = 0; ri < kNumVariantR; ++ri) {
    const int R = kVariantR[ri];
    for (int mi = 0; mi < 2; ++mi) {
      const int M = kVariantM[mi];
      const int pre = default_load_schedule(K, R, M, pr.accum);
      if (!variant_compiled(K, R, M, pr.accum, pre)) continue;
      const int rg = regs ? regs(K, R, M, pr.accum, pre, ctx) : estimate_regs(K, R, M, pr.accum);
      if (rg <= 0) continue;  // variant not compiled
      const int ncg_box = (kMaxBoxDim - (K - 1)) / R;
      const int ncg_need = static_cast<int>(ceil_div(std::min<long long>(W, 8LL * R), R));
      const int ncg_hi = std::min({8, ncg_box, ncg_need});
      for (int ncg = 1; ncg <= ncg_hi; ++ncg) {
        const int tile_w = ncg * R;
        const int tile_w_in = tile_w + K - 1;
        const long long tiles_w = ceil_div(W, tile_w);
        for (int nrg = 1; nrg * ncg <= kMaxConsumerWarps; ++nrg) {
          const int tile_h = nrg * M;
          if (tile_h > H + M - 1) break;  // taller tiles only add empty rows
          const int slots = nrg * ncg;
         for (int si = 0; si < kNumSplits; ++si) {
          const int nsplit = kSplits[si];
          if (nsplit * slots > kMaxConsumerWarps || nsplit > K) break;
          const int consumer_warps = nsplit * slots;
          const int threads = (consumer_warps + 1) * 32;
          const int cps_regs = ctas_by_registers(rg, consumer_warps + 1, hw.regs_per_sm);
          if (cps_regs < 1) break;
          // splitting only pays where tiles are too few to fill the device
          const long long tiles_all = B * ceil_div(H, tile_h) * ceil_div(W, tile_w) * cblocks;
          if (nsplit > 1 && tiles_all * slots > 16LL * hw.sm_count) break;
          const long long tiles_h = ceil_div(H, tile_h);
          const long long tiles = B * tiles_h * tiles_w * cblocks;
          if (tiles > (1LL << 40)) continue;

          // Work per CTA, averaged over the tile rows of the image.
          const double row_cost =
              pr.accum == DWB_ACCUM_F32 ? 2.0 * R * K + 4.0 * (R + K - 1) : 2.0 * R * K + 6.0 * R;
          const double wrow_cost = pr.accum == DWB_ACCUM_F32 ? 4.0 * K : 1.0 * K;
          double work_sum = 0.0, bytes_sum = 0.0, steps_sum = 0.0;
          for (long long t = 0; t < tiles_h; ++t) {
            const int h0 = static_cast<int>(t * tile_h);
            const int rows_in = static_cast<int>(std::min<long long>(tile_h, H - h0));
            const int s_lo = std::max(0, pad - (h0 + rows_in - 1));
            const int s_hi = static_cast<int>(std::min<long long>(K, H + pad - h0));
            const int nsteps = std::max(0, s_hi - s_lo);
            double valid = 0.0;
            for (int i = 0; i < rows_in; ++i) valid += valid_taps(h0 + i, static_cast<int>(H), K);
            // per warp column group: every row group walks all steps (the
            // weight conversion is paid by every split group)
            work_sum += ncg * (valid * row_cost + static_cast<double>(nsteps) * nrg * wrow_cost);
            bytes_sum += (static_cast<double>(nsteps + tile_h - 1) * tile_w_in + nsteps * K) * kPixelBytes;
            steps_sum += nsteps;
          }
          // row split: groups 1..S-1 hand M*R fp32 pairs per slot to group 0
          const double red_cost = nsplit > 1 ? static_cast<double>(nsplit) * slots * M * R * 4.0 + 600.0 : 0.0;
          const double work_cta = work_sum / static_cast<double>(tiles_h) + red_cost;
          const double bytes_cta = bytes_sum / static_cast<double>(tiles_h);
          const double steps_cta = steps_sum / static_cast<double>(tiles_h);
          const long long tiles_busiest = ceil_div(tiles, hw.sm_count);  // tiles on the busiest SM

          // Prefetch depth (rows the producer may run ahead of the consumers):
          // deeper rings hide the load latency, shallower ones fit more CTAs.
          // A row split keeps S steps in flight, so its ring is S - 1 stages deeper.
          int last_ring = -1;
          const int depths[4] = {2, 4, 8, K + 64};
          for (int di = 0; di < 4; ++di) {
            const int ring_rows = std::min(tile_h + nsplit - 1 + depths[di], tile_h + K - 1);
            if (ring_rows == last_ring) continue;
            last_ring = ring_rows;
            long long red_off = 0;
            const long long smem = plan_smem_bytes(K, tile_w_in, ring_rows, nsplit, slots, M, R, &red_off);
            if (smem > hw.smem_optin) break;
            if (!barriers_fit(ring_rows)) break;
            const int cps = static_cast<int>(std::min<long long>(
                {hw.smem_per_sm / (smem + hw.smem_reserved), static_cast<long long>(cps_regs),
                 hw.max_threads_sm / threads, hw.max_ctas_sm}));
            if (cps < 1) continue;
            const long long grid = std::min<long long>(tiles, static_cast<long long>(cps) * hw.sm_count);
            const long long resident = std::min<long long>(cps, tiles_busiest);
            const double warps_per_smsp = static_cast<double>(resident * consumer_warps) / 4.0;
            const double util = warps_per_smsp >= 3.0   ? 1.0
                                : warps_per_smsp >= 2.0 ? 0.9
                                : warps_per_smsp >= 1.0 ? 0.65
                                                        : 0.65 * warps_per_smsp;
            const double t_tp = std::max(static_cast<double>(tiles_busiest) * work_cta / (4.0 * util),
                                         static_cast<double>(tiles_busiest) * bytes_cta / kTmaBytesPerClk);
            // a persistent CTA pays the load latency once, then once per step it
            // cannot prefetch far enough ahead
            const double tiles_per_cta = std::ceil(static_cast<double>(tiles) / static_cast<double>(grid));
            const double ahead = static_cast<double>(ring_rows - tile_h + 1);  // steps of lookahead
            const double t_lat = kLoadLatency + tiles_per_cta * (steps_cta * kLoadLatency / ahead + 300.0);
            // critical path of one warp: its share of the slot's kernel rows, serially
            const double t_warp = tiles_per_cta * work_cta / consumer_warps;
            const double cost = std::max({t_tp, t_lat, t_warp}) + tiles_per_cta * 300.0;
          dwb_plan pl;
          std::memset(&pl, 0, sizeof(pl));
          pl.kernel_size = K;
          pl.cols_per_thread = R;
          pl.rows_per_thread = M;
          pl.channel_block = kChannelsPerCta;
          pl.tile_h = tile_h;
          pl.tile_w = tile_w;
          pl.tile_w_in = tile_w_in;
          pl.ring_rows = ring_rows;
          pl.ring_wrows = 0;
          pl.consumer_warps = consumer_warps;
          pl.threads = threads;
          pl.smem_bytes = static_cast<int32_t>(smem);
          pl.ctas_per_sm = cps;
          pl.grid = grid;
          pl.tiles = tiles;
          pl.accum = pr.accum;
          pl.regs_estimate = rg;
          pl.model_cost = cost;
          pl.row_splits = nsplit;
          pl.load_schedule = pre;
          pl.band_tiles = 0;
          ++count;
          if (sink) sink(pl, sink_ctx);
          }

          // Band mode: a CTA streams bands of bt row tiles, every input row once
          // per band and the K x K weights once (mixed accumulation, small K).
          if (band_compiled(K, pr.accum)) {
            const long long bts[4] = {2, 4, 8, tiles_h};
            long long last_bt = -1;
            for (int bi = 0; bi < 4; ++bi) {
              const long long bt = std::min<long long>(bts[bi], tiles_h);
              if (bt == last_bt) continue;
              last_bt = bt;
              const long long bands_h = ceil_div(tiles_h, bt);
              const long long bands = B * cblocks * tiles_w * bands_h;
              if (bands > 0x7fffffffLL || bands < 1) continue;
              const double band_rows = std::min<double>(static_cast<double>(bt * tile_h), static_cast<double>(H));
              const double bytes_band = ((band_rows + K - 1) * tile_w_in + static_cast<double>(K) * K) * kPixelBytes;
              const double work_band = work_cta * static_cast<double>(bt);
              const long long bands_busiest = ceil_div(bands, hw.sm_count);
              for (int extra = 0; extra <= 8; extra += 4) {
                const int ring_rows = tile_h + K - 1 + extra;
                long long red_off = 0, wbuf_off = 0;
                const long long smem = band_smem_bytes(K, tile_w_in, ring_rows, nsplit, slots, M, R, &red_off, &wbuf_off);
                if (smem > hw.smem_optin || !barriers_fit(ring_rows, true)) break;
                const int cps = static_cast<int>(std::min<long long>(
                    {hw.smem_per_sm / (smem + hw.smem_reserved), static_cast<long long>(cps_regs),
                     hw.max_threads_sm / threads, hw.max_ctas_sm}));
                if (cps < 1) continue;
                const long long grid = std::min<long long>(bands, static_cast<long long>(cps) * hw.sm_count);
                const long long resident = std::min<long long>(cps, bands_busiest);
                const double warps_per_smsp = static_cast<double>(resident * consumer_warps) / 4.0;
                const double util = warps_per_smsp >= 3.0   ? 1.0
                                    : warps_per_smsp >= 2.0 ? 0.9
                                    : warps_per_smsp >= 1.0 ? 0.65
                                                            : 0.65 * warps_per_smsp;
                const double t_tp = std::max(static_cast<double>(bands_busiest) * work_band / (4.0 * util),
                                             static_cast<double>(bands_busiest) * bytes_band / kTmaBytesPerClk);
                const double bands_per_cta = std::ceil(static_cast<double>(bands) / static_cast<double>(grid));
                const double ahead = static_cast<double>(extra + 1);  // rows the producer runs ahead of a window
                const double t_lat = kLoadLatency + bands_per_cta * static_cast<double>(bt) *
                                                        (static_cast<double>(K) * kLoadLatency / (ahead * K) + 300.0);
                const double t_warp = bands_per_cta * work_band / consumer_warps;
                const double cost = std::max({t_tp, t_lat, t_warp}) + bands_per_cta * static_cast<double>(bt) * 300.0;
                dwb_plan pl;
                std::memset(&pl, 0, sizeof(pl));
                pl.kernel_size = K;
                pl.cols_per_thread = R;
                pl.rows_per_thread = M;
                pl.channel_block = kChannelsPerCta;
                pl.tile_h = tile_h;
                pl.tile_w = tile_w;
                pl.tile_w_in = tile_w_in;
                pl.ring_rows = ring_rows;
                pl.consumer_warps = consumer_warps;
                pl.threads = threads;
                pl.smem_bytes = static_cast<int32_t>(smem);
                pl.ctas_per_sm = cps;
                pl.grid = grid;
                pl.tiles = bands;
                pl.accum = pr.accum;
                pl.regs_estimate = rg;
                pl.model_cost = cost;
                pl.row_splits = nsplit;
                pl.load_schedule = pre;
                pl.band_tiles = static_cast<int32_t>(bt);
                ++count;
                if (sink) sink(pl, sink_ctx);
              }
            }
          }
         }
        }
      }
    }
  }
  return count > 0 ? DWB_OK : DWB_ERR_UNSUPPORTED;
}

namespace {
struct BestSink {
  dwb_plan best;
  bool found = false;
};
void keep_best(const dwb_plan& p, void* vctx) {
  BestSink* b = static_cast<BestSink*>(vctx);
  if (!b->found || p.model_cost < b->best.model_cost * 0.999) {
    b->best = p;
    b->found = true;
  }
}
}  // namespace

int plan_problem(const dwb_problem& pr, const HwInfo& hw, RegsFn regs, void* ctx, dwb_plan* out) {
  if (!out) return DWB_ERR_NULL_POINTER;
  std::memset(out, 0, sizeof(*out));
  BestSink b;
  const int rc = enumerate_plans(pr, hw, regs, ctx, keep_best, &b);
  if (rc != DWB_OK) return rc;
  if (!b.found) return DWB_ERR_UNSUPPORTED;
  *out = b.best;
  return DWB_OK;
}

// Recompute every derived field of a caller-supplied plan and check it
// against the kernel's requirements.
int check_plan(const dwb_problem& pr, const HwInfo& hw, int regs, dwb_plan* p) {
  const int vst = validate_problem(pr);
  if (vst != DWB_OK) return vst;
  const int K = pr.kernel_size;
  const int R = p->cols_per_thread, M = p->rows_per_thread;
  if (!variant_compiled(K, R, M, p->accum, p->load_schedule) || p->kernel_size != K || p->accum != pr.accum)
    return DWB_ERR_BAD_ARG;
  if (p->tile_w < R || p->tile_w % R != 0 || p->tile_h < M || p->tile_h % M != 0) return DWB_ERR_BAD_ARG;
  if (p->tile_w + K - 1 > kMaxBoxDim) return DWB_ERR_BAD_ARG;
  if (p->row_splits == 0) p->row_splits = 1;  // plans from callers that predate the field
  const int S = p->row_splits;
  if (S < 1 || S > K) return DWB_ERR_BAD_ARG;
  const int slots = (p->tile_w / R) * (p->tile_h / M);
  const int cw = S * slots;
  if (slots < 1 || cw > 31) return DWB_ERR_BAD_ARG;
  const bool band = p->band_tiles > 0;
  if (p->band_tiles < 0 || (band && !band_compiled(K, p->accum))) return DWB_ERR_BAD_ARG;
  if (p->ring_rows < (band ? p->tile_h + K - 1 : p->tile_h)) return DWB_ERR_BAD_ARG;
  if (!barriers_fit(p->ring_rows, band)) return DWB_ERR_BAD_ARG;
  p->ring_wrows = 0;  // weight rows travel in the input-row stages (or stay resident: band mode)
  p->channel_block = kChannelsPerCta;
  p->tile_w_in = p->tile_w + K - 1;
  p->consumer_warps = cw;
  p->threads = 32 * (cw + 1);
  const long long smem = band ? band_smem_bytes(K, p->tile_w_in, p->ring_rows, S, slots, M, R, nullptr, nullptr)
                              : plan_smem_bytes(K, p->tile_w_in, p->ring_rows, S, slots, M, R, nullptr);
  if (smem > hw.smem_optin) return DWB_ERR_BAD_ARG;
  if (regs > 0 && ctas_by_registers(regs, cw + 1, hw.regs_per_sm) < 1) return DWB_ERR_BAD_ARG;
  p->smem_bytes = static_cast<int32_t>(smem);
  const long long tiles_h = ceil_div(pr.height, p->tile_h);
  const long long strips = pr.batch * ceil_div(pr.width, p->tile_w) * ceil_div(pr.channels, kChannelsPerCta);
  // work units the CTAs walk: tiles, or bands of band_tiles row tiles
  p->tiles = strips * (band ? ceil_div(tiles_h, p->band_tiles) : tiles_h);
  if (p->tiles > (1LL << 40) || (band && p->tiles > 0x7fffffffLL)) return DWB_ERR_BAD_SHAPE;
  // grid: < 0 = persistent (sized by the launcher from the occupancy), else
  // the caller's CTA count, at most one per tile (0 = one CTA per tile)
  if (p->grid == 0 || p->grid > p->tiles) p->grid = p->tiles;
  if (p->grid > 0x7fffffffLL) return DWB_ERR_BAD_SHAPE;
  p->regs_estimate = regs;
  return DWB_OK;
}

}  // namespace dwb
