// dw_planner.h -- launch/tiling planner for the row-streaming depthwise kernel.
//
// Pure host arithmetic (no CUDA calls), so it is exercised on machines
// without a GPU through dwb_plan_query().  The launcher calls the same
// function with the real per-variant register counts of the loaded device.
#pragma once

#include <stdint.h>

#include "../../include/dwconv_b200.h"

namespace dwb {

// Band-mode kernels (mixed accumulation) are built for K <= kBandMaxK.
constexpr int kBandMaxK = 17;

struct HwInfo {
  int sm_count = 148;          // B200
  int smem_optin = 232448;     // max dynamic smem per CTA (227 KB)
  int smem_per_sm = 233472;    // 228 KB per SM
  int smem_reserved = 1024;    // per-CTA system reservation
  int regs_per_sm = 65536;
  int max_threads_sm = 2048;
  int max_ctas_sm = 32;
};

// Register count of a compiled variant, or 0 when the variant is not built.
typedef int (*RegsFn)(int K, int R, int M, int acc, int pre, void* ctx);

// Register estimate used when no device is present (matches ptxas within a
// few registers for the variants in dw_variants.cuh).
int estimate_regs(int K, int R, int M, int acc);

// Column-group sizes and row blockings the library compiles (dw_variants.cuh).
constexpr int kNumVariantR = 6;
extern const int kVariantR[kNumVariantR];
extern const int kVariantM[2];
bool variant_compiled(int K, int R, int M, int acc, int pre);
// Whether the variant also has a band-mode kernel (dw_variants.cuh).
bool band_compiled(int K, int acc);

// Load schedule the cost model assumes for a variant (the tuner measures both).
int default_load_schedule(int K, int R, int M, int acc);

// Dynamic shared memory of a plan: mbarriers, the stage ring (each stage =
// one staged input row of tile_w_in pixels + one weight row of K taps), then
// (row split S > 1) the partial-sum exchange area of groups 1..S-1.
// *red_off receives the exchange area's byte offset.
long long plan_smem_bytes(int K, int tile_w_in, int stages, int nsplit, int slots, int M, int R, long long* red_off);

// Dynamic shared memory of a band-mode plan: mbarriers, the stage ring (one
// staged input row per stage), the partial-sum exchange area (S > 1), then the
// two resident K x K weight buffers, whose byte offset goes to *wbuf_off.
long long band_smem_bytes(int K, int tile_w_in, int stages, int nsplit, int slots, int M, int R, long long* red_off,
                          long long* wbuf_off);

// Whether the 1 KB mbarrier area holds the ring's 2 * stages + 2 barriers
// (+ 4 for the band mode's weight buffers).
bool barriers_fit(int stages, bool band = false);

// Range checks shared by every entry point.  Returns a dwb_status.
int validate_problem(const dwb_problem& pr);

// Call `sink` for every feasible plan (with its modelled cost).
typedef void (*PlanSink)(const dwb_plan& plan, void* ctx);
int enumerate_plans(const dwb_problem& pr, const HwInfo& hw, RegsFn regs, void* ctx, PlanSink sink, void* sink_ctx);

// Validate the problem and fill *out with the lowest-cost plan.
int plan_problem(const dwb_problem& pr, const HwInfo& hw, RegsFn regs, void* ctx, dwb_plan* out);

// Check a caller-supplied plan (R, M, tile_h, tile_w, ring sizes, accum) and
// recompute its derived fields.  regs: the variant's registers (0 = unknown).
int check_plan(const dwb_problem& pr, const HwInfo& hw, int regs, dwb_plan* p);

}  // namespace dwb
