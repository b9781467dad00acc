// planner.hpp -- per-problem routing, moduli count and cost model (host only).
//
// Routing rules follow the reference planner (src/planner.h:7-83, src/planner.cpp:286-330) so a
// call routes every problem the same way where a rule decides: EMPTY / K_ZERO / ALPHA_ZERO /
// K_TOO_LARGE / SMALL_K / PRECISION / TINY, and the same moduli count.  Where the reference asks
// its throughput model (AUTO: emulate, or native as UNPROFITABLE), this library asks a model of
// its own B200 kernels (prep, paired / single-CTA residue GEMM, reconstruct) against cuBLAS
// DGEMM, whose constants are fitted on the device by calib/calibrate.py and read from
// calib/b200.json next to the library (or $GGEMM_CALIB_JSON).
#pragma once
#include <cstddef>

#include "ggemm.h"

namespace g2 {

enum Route : int {
  kRouteEmu = 0,
  kRouteEmpty = 1,        // m == 0 || n == 0
  kRouteKZero = 2,        // k == 0: C = beta C, native
  kRouteKTooLarge = 3,    // k > 131040 (int32 accumulation would overflow)
  kRouteTiny = 4,         // m n k below tiny_mnk (AUTO)
  kRouteUnprofitable = 5, // cost model prefers native FP64 (AUTO)
  kRoutePrecision = 6,    // no N <= 20 reaches the target
  kRouteSmallK = 7,       // AUTO and k <= 16
  kRouteAlphaZero = 8     // alpha == 0: C = beta C, native, A and B never read
};
constexpr int kAutoNativeMaxK = 16;
constexpr double kRhoBudgetDefault = 16.0;

// Native routes that are exact by construction do not count as fallbacks in the stats.
inline bool route_is_fallback(int r) {
  return r != kRouteEmu && r != kRouteEmpty && r != kRouteKZero && r != kRouteAlphaZero;
}

struct PlanEntry {
  int route;       // Route
  int num_moduli;  // valid for kRouteEmu
  int tile_cfg;    // always 0 (the reference's tile classes do not exist here)
  double t_emu_s, t_native_s;
};

// Cost model of this library's kernels and of cuBLAS DGEMM on one device (calib/calibrate.py):
//   prep   bytes / prep_bw   + blocks x prep_block_s / num_sms   (blocks: 32 A rows / 8 B cols)
//   gemm   ops / gemm_ops    + tiles x gemm_tile_s / num_sms    (ops over 128-row padded tiles)
//   recon  bytes / recon_bw  + blocks x recon_block_s / num_sms (blocks: 128 rows x 16 cols)
//   native 2 m n k / fp64_flops + native_problem_s
struct DeviceModel {
  int num_sms;
  double prep_bw, prep_block_s, gemm_ops, gemm_tile_s, recon_bw, recon_block_s;
  double fp64_flops, native_problem_s;
  double tiny_mnk;  // AUTO: problems with m n k below it go native (TINY), as in the reference
  int from_file;    // 1 if the constants came from a calibration file
};

// The model for a device with num_sms SMs: the calibration file ($GGEMM_CALIB_JSON, else
// calib/b200.json next to this library) or built-in B200 values, then the reference's override
// variables: GGEMM_FP64_FLOPS (fp64_flops), GGEMM_INT8_OPS (gemm_ops), GGEMM_MEM_BW (prep_bw and
// recon_bw), GGEMM_TINY_MNK.
void device_model_init(DeviceModel* dm, int num_sms);

// Modelled seconds of one problem emulated with N moduli, and natively.
double emu_time(int m, int n, int k, bool beta_nonzero, int N, const DeviceModel& dm);
double native_time(int m, int n, int k, bool beta_nonzero, const DeviceModel& dm);

// Fixed N from cfg, else the normwise choice for (k, target); -1 if unreachable.
int plan_num_moduli(const ggemm_config_t* cfg, int k);

// Plans num problems into out[0..num).  memo: optional int scratch of memo_cap entries
// (>= plan_memo_cap(num)) for planning each distinct shape once.  rho_budget: the AUTO
// componentwise budget.  Returns GGEMM_OK or GGEMM_ERR_UNSAFE.
int plan_group(const ggemm_problem_t* probs, int num, const ggemm_config_t* cfg,
               ggemm_path_t path, const DeviceModel& dm, double rho_budget, PlanEntry* out,
               int* memo, size_t memo_cap);
size_t plan_memo_cap(int num);
double env_rho_budget();

}  // namespace g2
