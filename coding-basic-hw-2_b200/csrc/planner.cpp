// planner.cpp -- see planner.hpp.  Host only; no allocation.
#include "planner.hpp"

#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "crt.hpp"

namespace g2 {
namespace {

// Built-in B200 constants: calib/b200.json as fitted on this pool's B200s (used when no file is
// found next to the library).
constexpr DeviceModel kB200Default = {
    148,
    /*prep_bw=*/2.107e+12, /*prep_block_s=*/2.719e-06,
    /*gemm_ops=*/2.785e+15, /*gemm_tile_s=*/1.594e-06,
    /*recon_bw=*/7.89e+12, /*recon_block_s=*/2.822e-06,
    /*fp64_flops=*/3.138e+13, /*native_problem_s=*/1.068e-07,
    /*tiny_mnk=*/32.0 * 32.0 * 32.0, 0};

bool json_number(const char* txt, const char* key, double* v) {
  char pat[96];
  std::snprintf(pat, sizeof pat, "\"%s\"", key);
  const char* p = std::strstr(txt, pat);
  if (!p) return false;
  p = std::strchr(p + std::strlen(pat), ':');
  if (!p) return false;
  char* end = nullptr;
  const double x = std::strtod(p + 1, &end);
  if (end == p + 1 || !(x >= 0)) return false;
  *v = x;
  return true;
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

// calib/b200.json beside the shared library that holds this code.
std::string default_calib_path() {
  Dl_info info;
  if (!dladdr(reinterpret_cast<void*>(&device_model_init), &info) || !info.dli_fname) return {};
  std::string so = info.dli_fname;
  const size_t slash = so.rfind('/');
  const std::string dir = slash == std::string::npos ? "." : so.substr(0, slash);
  return dir + "/calib/b200.json";
}

void load_calibration(DeviceModel* dm) {
  std::string path;
  if (const char* e = std::getenv("GGEMM_CALIB_JSON")) path = e;
  if (path.empty()) path = default_calib_path();
  if (path.empty()) return;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return;
  static char buf[1 << 16];  // the scalar fields come first in the file
  const size_t n = std::fread(buf, 1, sizeof buf - 1, f);
  buf[n] = 0;
  std::fclose(f);
  struct Field {
    const char* key;
    double* dst;
    double lo, hi;
  } fields[] = {{"prep_bw", &dm->prep_bw, 1e10, 1e14},
                {"prep_block_s", &dm->prep_block_s, 0, 1e-3},
                {"gemm_ops", &dm->gemm_ops, 1e12, 1e17},
                {"gemm_tile_s", &dm->gemm_tile_s, 0, 1e-3},
                {"recon_bw", &dm->recon_bw, 1e10, 1e14},
                {"recon_block_s", &dm->recon_block_s, 0, 1e-3},
                {"fp64_flops", &dm->fp64_flops, 1e11, 1e16},
                {"native_problem_s", &dm->native_problem_s, 0, 1e-2}};
  int got = 0;
  for (const Field& fd : fields) {
    double v;
    if (json_number(buf, fd.key, &v) && v >= fd.lo && v <= fd.hi) {
      *fd.dst = v;
      ++got;
    }
  }
  dm->from_file = got == (int)(sizeof fields / sizeof fields[0]);
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

// Everything after the alpha == 0 check depends only on (m, n, k, beta != 0).  Rule routes and
// the moduli count as in the reference (src/planner.cpp:286-330); the AUTO cost decision from
// this library's model.
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
  const bool bnz = p.beta != 0.0;
  e.t_emu_s = emu_time(p.m, p.n, p.k, bnz, e.num_moduli, dm);
  e.t_native_s = native_time(p.m, p.n, p.k, bnz, dm);
  if (allow_fb) {
    if ((double)p.m * p.n * p.k < dm.tiny_mnk) e.route = kRouteTiny;
    else if (e.t_emu_s > e.t_native_s) e.route = kRouteUnprofitable;
  }
  return GGEMM_OK;
}

}  // namespace

double emu_time(int m, int n, int k, bool beta_nonzero, int N, const DeviceModel& dm) {
  const double M = m, Nn = n, kp = (double)(((size_t)k + 31) / 32 * 32), np = N + 1;
  const double sms = std::max(1, dm.num_sms);
  const double prep_bytes = 8.0 * (M * k + (double)k * Nn) + np * (M + Nn) * kp + 16.0 * (M + Nn);
  const double prep_blocks = (double)((m + 31) / 32 + (n + 7) / 8);
  const double ops = 2.0 * (double)((m + 127) / 128 * 128) * (double)((n + 15) / 16 * 16) * kp * np;
  const double tiles = np * (double)((m + 127) / 128) * (double)(n > 128 ? (n + 255) / 256 : 1);
  const double recon_bytes =
      (N + 4.0) * M * Nn + 8.0 * M * Nn * (beta_nonzero ? 2.0 : 1.0) + 16.0 * (M + Nn);
  const double recon_blocks = (double)((n + 15) / 16) * (double)((m + 127) / 128);
  return prep_bytes / dm.prep_bw + prep_blocks * dm.prep_block_s / sms + ops / dm.gemm_ops +
         tiles * dm.gemm_tile_s / sms + recon_bytes / dm.recon_bw +
         recon_blocks * dm.recon_block_s / sms;
}

double native_time(int m, int n, int k, bool beta_nonzero, const DeviceModel& dm) {
  (void)beta_nonzero;
  return 2.0 * (double)m * n * k / dm.fp64_flops + dm.native_problem_s;
}

double env_rho_budget() {
  const char* s = std::getenv("GGEMM_RHO_BUDGET");
  if (!s || !*s) return kRhoBudgetDefault;
  char* end = nullptr;
  const double v = std::strtod(s, &end);
  return (end != s && v > 0) ? v : kRhoBudgetDefault;
}

void device_model_init(DeviceModel* dm, int num_sms) {
  *dm = kB200Default;
  load_calibration(dm);
  bool used = false;
  double v = env_double("GGEMM_FP64_FLOPS", 1e11, 1e16, &used);
  if (used) dm->fp64_flops = v;
  used = false;
  v = env_double("GGEMM_INT8_OPS", 1e12, 1e17, &used);
  if (used) dm->gemm_ops = v;
  used = false;
  v = env_double("GGEMM_MEM_BW", 1e10, 1e14, &used);
  if (used) dm->prep_bw = dm->recon_bw = v;
  dm->num_sms = num_sms > 0 ? num_sms : 1;
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
  return GGEMM_OK;
}

}  // namespace g2
