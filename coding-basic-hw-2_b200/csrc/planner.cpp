// planner.cpp -- see planner.hpp.  Host only; no allocation.
#include "planner.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "crt.hpp"

namespace g2 {
namespace {

inline double kp_of(int k) { return (double)(((size_t)k + 31) / 32 * 32); }
inline double tile_dim(int cfg) { return cfg == 0 ? 128.0 : (cfg == 1 ? 64.0 : 32.0); }
inline double round_up(double x, double t) { return std::ceil(x / t) * t; }
inline double tiles_of(int m, int n, int cfg) {
  const double t = tile_dim(cfg);
  return std::ceil(m / t) * std::ceil(n / t);
}

// Cost-model tile classes, their relative INT8 efficiency, resident tiles per SM and the
// number of FP64 read passes of prep (reference src/planner.cpp:151-172).
constexpr int kTileCfgs = 3;
constexpr double kTileEff[kTileCfgs] = {1.0, 0.63, 0.30};
constexpr double kSlotsPerSm = 2.0;
constexpr double kPrepPasses = 2.0;
constexpr double kWsIntsPerRow = 4.0;

// Largest tile whose padded-area efficiency is >= 0.75, else the most efficient one.
int tile_by_padding(int m, int n) {
  int best = kTileCfgs - 1;
  double best_eff = -1;
  for (int c = 0; c < kTileCfgs; ++c) {
    const double t = tile_dim(c);
    const double eff = (double)m * n / (round_up(m, t) * round_up(n, t));
    if (eff >= 0.75) return c;
    if (eff > best_eff) {
      best_eff = eff;
      best = c;
    }
  }
  return best;
}

// Three dependent stages (prep, residue GEMM, reconstruct) against native DGEMM.
void cost(const ggemm_problem_t& p, int nm, int cfg, const DeviceModel& dm, double* t_emu,
          double* t_nat) {
  const double m = p.m, n = p.n, k = p.k, kp = kp_of(p.k), t = tile_dim(cfg);
  const double c_rw = (p.beta != 0.0) ? 2.0 : 1.0;
  const double np = nm + 1;  // residue planes + abs plane
  const double prep =
      (kPrepPasses * (m * k + k * n) * 8 + np * (m + n) * kp + 4.0 * kWsIntsPerRow * (m + n)) /
      dm.mem_bw;
  const double slots = (double)dm.num_sms * kSlotsPerSm;
  const double per_tile = 2.0 * t * t * kp / (dm.int8_ops * kTileEff[cfg] / slots);
  const double gemm =
      std::ceil(np * tiles_of(p.m, p.n, cfg) / slots) * per_tile + np * m * n * 4 / dm.mem_bw;
  const double recon = (np * m * n * 4 + c_rw * m * n * 8) / dm.mem_bw;
  *t_emu = prep + gemm + recon;
  const double nat_c = 2.0 * m * n * k / dm.fp64_flops;
  const double nat_m = (m * k + k * n + c_rw * m * n) * 8 / dm.mem_bw;
  *t_nat = std::max(nat_c, nat_m);
}

// Wave quantization: shrink the tile of problems whose single tile outweighs a slot's share of
// the group, until stable.  True if any tile class changed.
bool tune_tiles(const ggemm_problem_t* probs, int num, const DeviceModel& dm, PlanEntry* out) {
  const double slots = (double)dm.num_sms * kSlotsPerSm;
  bool any = false;
  for (int pass = 0; pass < kTileCfgs; ++pass) {
    double W = 0;
    for (int g = 0; g < num; ++g) {
      if (out[g].route != kRouteEmu) continue;
      const double t = tile_dim(out[g].tile_cfg);
      W += (out[g].num_moduli + 1) * tiles_of(probs[g].m, probs[g].n, out[g].tile_cfg) * t * t *
           kp_of(probs[g].k);
    }
    if (W <= 0) return any;
    const double per_slot = W / slots;
    bool changed = false;
    for (int g = 0; g < num; ++g) {
      if (out[g].route != kRouteEmu || out[g].tile_cfg >= kTileCfgs - 1) continue;
      const double t = tile_dim(out[g].tile_cfg);
      if (t * t * kp_of(probs[g].k) > per_slot) {
        out[g].tile_cfg++;
        changed = true;
      }
    }
    if (!changed) return any;
    any = true;
  }
  return any;
}

// Everything after the alpha == 0 check depends only on (m, n, k, beta != 0).
int plan_shape(const ggemm_problem_t& p, const ggemm_config_t* cfg, bool autop, int allow_fb,
               double rho_budget, const DeviceModel& dm, PlanEntry& e) {
  if (p.k > kMaxKExact) {
    if (!allow_fb) return GGEMM_ERR_UNSAFE;
    e.route = kRouteKTooLarge;
    return GGEMM_OK;
  }
  if (autop && allow_fb && p.k <= kAutoNativeMaxK) {
    e.route = kRouteSmallK;
    return GGEMM_OK;
  }
  if (autop && !(cfg && cfg->num_moduli > 0)) {
    e.num_moduli = choose_num_moduli_cw(p.k, rho_budget);
    if (e.num_moduli >= 0) e.num_moduli = std::min(std::max(e.num_moduli, 2), kMaxModuli);
  } else {
    e.num_moduli = plan_num_moduli(cfg, p.k);
  }
  if (e.num_moduli < 0) {
    if (!allow_fb) return GGEMM_ERR_UNSAFE;
    e.route = kRoutePrecision;
    e.num_moduli = 0;
    return GGEMM_OK;
  }
  if (!autop) return GGEMM_OK;
  e.tile_cfg = tile_by_padding(p.m, p.n);
  cost(p, e.num_moduli, e.tile_cfg, dm, &e.t_emu_s, &e.t_native_s);
  if (allow_fb) {
    if ((double)p.m * p.n * p.k < dm.tiny_mnk) e.route = kRouteTiny;
    else if (e.t_emu_s > e.t_native_s) e.route = kRouteUnprofitable;
  }
  return GGEMM_OK;
}

inline bool same_shape(const ggemm_problem_t& a, const ggemm_problem_t& b) {
  return a.m == b.m && a.n == b.n && a.k == b.k && (a.beta != 0.0) == (b.beta != 0.0);
}
inline uint32_t shape_hash(const ggemm_problem_t& p) {
  uint64_t h = (uint64_t)(uint32_t)p.m * 0x9E3779B97F4A7C15ull;
  h ^= (uint64_t)(uint32_t)p.n * 0xC2B2AE3D27D4EB4Full;
  h ^= (uint64_t)(uint32_t)p.k * 0x165667B19E3779F9ull;
  h ^= (p.beta != 0.0) ? 0x27D4EB2F165667C5ull : 0;
  h ^= h >> 29;
  h *= 0xBF58476D1CE4E5B9ull;
  return (uint32_t)(h ^ (h >> 32));
}

double env_double(const char* name, double lo, double hi, bool* used) {
  const char* s = std::getenv(name);
  if (!s || !*s) return 0;
  char* end = nullptr;
  const double v = std::strtod(s, &end);
  if (end == s || !(v >= lo && v <= hi)) {
    std::fprintf(stderr, "[ggemm] WARNING: %s=%s outside [%g, %g], ignored\n", name, s, lo, hi);
    return 0;
  }
  *used = true;
  return v;
}

bool json_number(const char* txt, const char* key, double* v) {
  char pat[96];
  std::snprintf(pat, sizeof pat, "\"%s\"", key);
  const char* p = std::strstr(txt, pat);
  if (!p) return false;
  p = std::strchr(p + std::strlen(pat), ':');
  if (!p) return false;
  char* end = nullptr;
  const double x = std::strtod(p + 1, &end);
  if (end == p + 1 || !(x > 0)) return false;
  *v = x;
  return true;
}

}  // namespace

double env_rho_budget() {
  const char* s = std::getenv("GGEMM_RHO_BUDGET");
  if (!s || !*s) return kRhoBudgetDefault;
  char* end = nullptr;
  const double v = std::strtod(s, &end);
  return (end != s && v > 0) ? v : kRhoBudgetDefault;
}

void device_model_init(DeviceModel* dm, int cc_major, int num_sms) {
  double fp64, i8, bw;
  if (cc_major == 10) {
    // B200: native DGEMM ~36 TF/s, this library's INT8 residue GEMM and HBM3e copy bandwidth
    // (measured on this pool's B200s: 6.5 TB/s copy).
    fp64 = 36e12;
    i8 = 2.5e15;
    bw = 6.0e12;
  } else if (cc_major == 9) {
    fp64 = 67e12 * 0.8;
    i8 = 1979e12 * 0.5;
    bw = 3.35e12 * 0.8;
  } else {
    fp64 = 10e12;
    i8 = 200e12;
    bw = 1e12;
  }
  if (const char* path = std::getenv("GGEMM_CALIB_JSON")) {
    if (FILE* f = std::fopen(path, "rb")) {
      static char buf[1 << 16];
      const size_t n = std::fread(buf, 1, sizeof buf - 1, f);
      buf[n] = 0;
      std::fclose(f);
      double v;
      if (json_number(buf, "f64_peak_flops", &v) && v >= 1e11 && v <= 1e16) fp64 = v;
      if (json_number(buf, "i8_peak_ops", &v) && v >= 1e12 && v <= 1e17) i8 = v;
      if (json_number(buf, "bw_Bps", &v) && v >= 1e10 && v <= 1e14) bw = v;
    }
  }
  bool used = false;
  double v = env_double("GGEMM_FP64_FLOPS", 1e11, 1e16, &used);
  if (used) fp64 = v;
  used = false;
  v = env_double("GGEMM_INT8_OPS", 1e12, 1e17, &used);
  if (used) i8 = v;
  used = false;
  v = env_double("GGEMM_MEM_BW", 1e10, 1e14, &used);
  if (used) bw = v;
  dm->num_sms = num_sms > 0 ? num_sms : 1;
  dm->fp64_flops = fp64;
  dm->int8_ops = i8;
  dm->mem_bw = bw;
  dm->tiny_mnk = 32.0 * 32.0 * 32.0;
  if (const char* s = std::getenv("GGEMM_TINY_MNK")) {
    char* end = nullptr;
    const double t = std::strtod(s, &end);
    if (end != s && t >= 0) dm->tiny_mnk = t;
  }
}

int plan_num_moduli(const ggemm_config_t* cfg, int k) {
  int nm;
  if (cfg && cfg->num_moduli > 0) {
    nm = cfg->num_moduli;
  } else {
    const double tgt = (cfg && cfg->target_rel_err > 0) ? cfg->target_rel_err : 1e-15;
    nm = choose_num_moduli(k, tgt);
    if (nm < 0) return -1;
  }
  return std::min(std::max(nm, 2), kMaxModuli);
}

size_t plan_memo_cap(int num) {
  size_t cap = 1;
  while (cap < 2 * (size_t)std::max(num, 1)) cap <<= 1;
  return cap;
}

int plan_group(const ggemm_problem_t* probs, int num, const ggemm_config_t* cfg,
               ggemm_path_t path, const DeviceModel& dm, double rho_budget, PlanEntry* out,
               int* memo, size_t memo_cap) {
  const int allow_fb = cfg ? cfg->allow_fallback : 0;
  const bool autop = (path == GGEMM_PATH_AUTO);
  size_t mask = 0;
  if (memo && num > 0) {
    const size_t cap = plan_memo_cap(num);
    if (cap <= memo_cap) {
      std::fill(memo, memo + cap, -1);
      mask = cap - 1;
    } else {
      memo = nullptr;
    }
  }
  for (int g = 0; g < num; ++g) {
    const ggemm_problem_t& p = probs[g];
    PlanEntry& e = out[g];
    e.route = kRouteEmu;
    e.num_moduli = 0;
    e.tile_cfg = 0;
    e.t_emu_s = e.t_native_s = 0;
    if (p.m == 0 || p.n == 0) { e.route = kRouteEmpty; continue; }
    if (p.k == 0) { e.route = kRouteKZero; continue; }
    if (p.alpha == 0.0) { e.route = kRouteAlphaZero; continue; }
    if (memo) {
      size_t s = shape_hash(p) & mask;
      int rep;
      while ((rep = memo[s]) >= 0 && !same_shape(probs[rep], p)) s = (s + 1) & mask;
      if (rep >= 0) {
        e = out[rep];
        continue;
      }
      memo[s] = g;
    }
    const int r = plan_shape(p, cfg, autop, allow_fb, rho_budget, dm, e);
    if (r) return r;
  }
  if (autop && tune_tiles(probs, num, dm, out)) {
    for (int g = 0; g < num; ++g) {
      PlanEntry& e = out[g];
      if (e.route != kRouteEmu) continue;
      cost(probs[g], e.num_moduli, e.tile_cfg, dm, &e.t_emu_s, &e.t_native_s);
      if (allow_fb && e.t_emu_s > e.t_native_s) e.route = kRouteUnprofitable;
    }
  }
  return GGEMM_OK;
}

}  // namespace g2
