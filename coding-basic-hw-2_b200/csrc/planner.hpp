// planner.hpp -- per-problem routing, moduli count and cost model (host only).
//
// Decisions follow the reference planner (src/planner.h:7-83, src/planner.cpp:132-330) so that
// a call routes every problem the same way: EMPTY / K_ZERO / ALPHA_ZERO / K_TOO_LARGE /
// SMALL_K / PRECISION by rule, TINY / UNPROFITABLE by a throughput model (AUTO only).  The
// model's constants come from a device model; for a B200 they are this library's own
// measurements (see ggemm.cpp), overridable with the same environment variables.
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
  int tile_cfg;    // cost-model tile class: 0 = 128, 1 = 64, 2 = 32
  double t_emu_s, t_native_s;
};

struct DeviceModel {
  int num_sms;
  double fp64_flops, int8_ops, mem_bw, tiny_mnk;
};

// B200 model: measured or nominal values, then GGEMM_FP64_FLOPS / GGEMM_INT8_OPS / GGEMM_MEM_BW
// / GGEMM_TINY_MNK / GGEMM_CALIB_JSON overrides (same names as the reference).
void device_model_init(DeviceModel* dm, int cc_major, int num_sms);

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
