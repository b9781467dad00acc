// stages.cpp -- ggemm_stage_* entry points (include/ggemm_stages.h): each stage of the
// pipeline as one kernel launch over caller-provided buffers, for parity tests.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.hpp"

using namespace g2;

namespace {

// Host staging for the descriptor copy.  cudaMemcpyAsync from pageable memory returns only
// after the source has been consumed, so the buffer may be reused by the next call.
thread_local std::vector<char> t_stage;

size_t blob_layout(int num, size_t desc_bytes, size_t prefix_elem, size_t* off_prefix) {
  *off_prefix = align_up((size_t)num * desc_bytes, 64);
  return *off_prefix + (size_t)(num + 1) * prefix_elem;
}

int copy_blob(void* scratch, size_t scratch_bytes, size_t bytes, cudaStream_t s) {
  if (bytes > scratch_bytes) return GGEMM_ERR_WORKSPACE;
  return cudaMemcpyAsync(scratch, t_stage.data(), bytes, cudaMemcpyHostToDevice, s) ==
                 cudaSuccess
             ? GGEMM_OK
             : GGEMM_ERR_CUDA;
}

}  // namespace

extern "C" size_t ggemm_stage_scratch_bytes(int num) {
  const size_t d = std::max({sizeof(ggemm_prep_desc_t), sizeof(GemmJob),
                             sizeof(ggemm_recon_desc_t)});
  return align_up((size_t)std::max(num, 1) * d, 64) + (size_t)(num + 2) * 8 + 256;
}

extern "C" int ggemm_stage_prep(const ggemm_prep_desc_t* descs, int num, void* scratch,
                                size_t scratch_bytes, void* counters, cudaStream_t s) {
  if (num < 0 || (num > 0 && (!descs || !scratch || !counters))) return GGEMM_ERR_INVALID;
  if (num == 0) return GGEMM_OK;
  if (upload_tables_current_device()) return GGEMM_ERR_NUMERICS;
  size_t off_p;
  const size_t bytes = blob_layout(num, sizeof(ggemm_prep_desc_t), sizeof(int), &off_p);
  t_stage.assign(bytes, 0);
  // descriptors are independent: sorted by prep instance (launch_prep)
  ggemm_prep_desc_t* sd = reinterpret_cast<ggemm_prep_desc_t*>(t_stage.data());
  std::memcpy(sd, descs, (size_t)num * sizeof(ggemm_prep_desc_t));
  for (int i = 0; i < num; ++i) {
    const ggemm_prep_desc_t& d = descs[i];
    if (d.rows < 0 || d.k < 0 || d.N < 1 || d.N > kMaxModuli || (d.kind & ~(1 | GGEMM_PREP_QSCALED)))
      return GGEMM_ERR_INVALID;
    if (d.rows > 0 && (!d.X || !d.img || !d.ws)) return GGEMM_ERR_INVALID;
    if (((uintptr_t)d.img & 15) || (d.plane_bytes & 15) ||
        (size_t)d.plane_bytes < ggemm_img_plane_bytes(d.rows, d.k))
      return GGEMM_ERR_INVALID;
  }
  long long blocks = 0;
  for (int i = 0; i < num; ++i) {
    blocks += prep_blocks(sd[i]);
    if (blocks > 0x7FFFFFFF) return GGEMM_ERR_INVALID;
  }
  int* pre = reinterpret_cast<int*>(t_stage.data() + off_p);
  PrepSplit sp;
  prep_partition(sd, num, pre, &sp);
  int r = copy_blob(scratch, scratch_bytes, bytes, s);
  if (r) return r;
  const char* db = static_cast<const char*>(scratch);
  return launch_prep(reinterpret_cast<const ggemm_prep_desc_t*>(db),
                     reinterpret_cast<const int*>(db + off_p), sp,
                     static_cast<DevCounters*>(counters), s)
             ? GGEMM_ERR_NUMERICS
             : GGEMM_OK;
}

extern "C" int ggemm_stage_gemm(const ggemm_gemm_desc_t* descs, int num, void* scratch,
                                size_t scratch_bytes, void* counters, cudaStream_t s) {
  if (num < 0 || (num > 0 && (!descs || !scratch || !counters))) return GGEMM_ERR_INVALID;
  if (num == 0) return GGEMM_OK;
  if (upload_tables_current_device()) return GGEMM_ERR_I8GEMM;
  size_t off_p;
  const size_t bytes = blob_layout(num, sizeof(GemmJob), sizeof(long long), &off_p);
  t_stage.assign(bytes, 0);
  GemmJob* jobs = reinterpret_cast<GemmJob*>(t_stage.data());
  long long* pre = reinterpret_cast<long long*>(t_stage.data() + off_p);
  long long tiles = 0;
  for (int i = 0; i < num; ++i) {
    const ggemm_gemm_desc_t& d = descs[i];
    if (d.m < 0 || d.n < 0 || d.k < 0 || d.planes < 0 || d.k > kMaxKExact)
      return GGEMM_ERR_INVALID;
    const bool qscaled = d.layout == GGEMM_PRODUCTS_DIGITS_QSCALED;
    const bool digits = d.layout == GGEMM_PRODUCTS_DIGITS || qscaled;
    if (!digits && d.layout != GGEMM_PRODUCTS_INT32) return GGEMM_ERR_INVALID;
    GemmJob j{};
    j.A = d.A;
    j.B = d.B;
    j.C = d.C;
    j.Y = reinterpret_cast<uint8_t*>(d.C);
    j.a_plane = d.a_plane;
    j.b_plane = d.b_plane;
    j.c_plane = d.c_plane;
    j.y_plane = d.c_plane;
    j.m = d.m;
    j.n = d.n;
    j.ksteps = (d.k + 31) / 32;
    j.planes = (d.m > 0 && d.n > 0 && d.k > 0) ? d.planes : 0;
    j.N = d.N;
    j.y8 = qscaled ? 2 : digits ? 1 : 0;
    set_gemm_tiling(j);
    if (j.planes > 0) {
      if (!d.A || !d.B || !d.C || ((uintptr_t)d.A & 15) || ((uintptr_t)d.B & 15) ||
          ((uintptr_t)d.C & (digits ? 15 : 3)) || (d.a_plane & 15) || (d.b_plane & 15))
        return GGEMM_ERR_INVALID;
      if ((size_t)d.a_plane < ggemm_img_plane_bytes(d.m, d.k) ||
          (size_t)d.b_plane < ggemm_img_plane_bytes(d.n, d.k))
        return GGEMM_ERR_INVALID;
      if (digits ? (d.N < 1 || d.N > kMaxModuli || d.planes > d.N + 1 || (d.c_plane & 15) ||
                    (size_t)d.c_plane < ggemm_digit_plane_bytes(d.m, d.n))
                 : d.c_plane < (long long)d.m * d.n)
        return GGEMM_ERR_INVALID;
    }
    jobs[i] = j;
  }
  // Paired GEMM (GGEMM_GEMM_PAIR: 1 always, 0 never, unset: when gemm_pair_pays).
  const char* env = std::getenv("GGEMM_GEMM_PAIR");
  const int force = env ? std::atoi(env) : -1;
  std::vector<int> pm, pn, pk, pp;
  for (int i = 0; i < num; ++i) {
    const GemmJob& j = jobs[i];
    if (j.planes <= 0) continue;
    pm.push_back(j.m);
    pn.push_back(j.n);
    pk.push_back(j.ksteps);
    pp.push_back(j.planes);
  }
  const bool pair = !pm.empty() && (force == 1 || (force != 0 &&
                                                   gemm_pair_pays(pm.data(), pn.data(), pk.data(),
                                                                  pp.data(), (int)pm.size(),
                                                                  current_device_sms())));
  for (int i = 0; i < num; ++i) {
    if (pair) set_gemm_tiling_pair(jobs[i]);
    pre[i] = tiles;
    tiles += gemm_tiles(jobs[i]);
  }
  pre[num] = tiles;
  int r = copy_blob(scratch, scratch_bytes, bytes, s);
  if (r) return r;
  const char* db = static_cast<const char*>(scratch);
  const GemmJob* dj = reinterpret_cast<const GemmJob*>(db);
  const long long* dp = reinterpret_cast<const long long*>(db + off_p);
  DevCounters* cnt = static_cast<DevCounters*>(counters);
  const int walk = gemm_jobs_ragged(jobs, num) ? kGemmWalkBothEnds : 0;
  const int e = pair ? launch_gemm_pair(dj, dp, num, tiles, cnt, s, walk)
                     : launch_gemm(dj, dp, num, tiles, cnt, s, walk);
  return e ? GGEMM_ERR_I8GEMM : GGEMM_OK;
}

extern "C" int ggemm_stage_recon(const ggemm_recon_desc_t* descs, int num, int repair_mode,
                                 void* scratch, size_t scratch_bytes, void* counters,
                                 cudaStream_t s) {
  if (num < 0 || (num > 0 && (!descs || !scratch || !counters))) return GGEMM_ERR_INVALID;
  if (repair_mode < GGEMM_STAGE_REPAIR_OFF || repair_mode > GGEMM_STAGE_REPAIR_ON)
    return GGEMM_ERR_INVALID;
  if (num == 0) return GGEMM_OK;
  if (upload_tables_current_device()) return GGEMM_ERR_NUMERICS;
  size_t off_p;
  const size_t bytes = blob_layout(num, sizeof(ggemm_recon_desc_t), sizeof(long long), &off_p);
  t_stage.assign(bytes, 0);
  // descriptors are independent: sorted by reconstruct instance (launch_recon)
  ggemm_recon_desc_t* sd = reinterpret_cast<ggemm_recon_desc_t*>(t_stage.data());
  std::memcpy(sd, descs, (size_t)num * sizeof(ggemm_recon_desc_t));
  long long* pre = reinterpret_cast<long long*>(t_stage.data() + off_p);
  for (int i = 0; i < num; ++i) {
    const ggemm_recon_desc_t& d = descs[i];
    if (d.m < 0 || d.n < 0 || d.k < 0 || d.N < 1 || d.N > kMaxModuli) return GGEMM_ERR_INVALID;
    if (d.layout == GGEMM_PRODUCTS_DIGITS) {
      if (((uintptr_t)d.C32 & 15) || (d.c_plane & 15) ||
          (size_t)d.c_plane < ggemm_digit_plane_bytes(d.m, d.n))
        return GGEMM_ERR_INVALID;
    } else if (d.layout != GGEMM_PRODUCTS_INT32) {
      return GGEMM_ERR_INVALID;
    }
  }
  ReconSplit sp;
  recon_partition(sd, num, pre, &sp);
  int r = copy_blob(scratch, scratch_bytes, bytes, s);
  if (r) return r;
  const char* db = static_cast<const char*>(scratch);
  return launch_recon(reinterpret_cast<const ggemm_recon_desc_t*>(db),
                      reinterpret_cast<const long long*>(db + off_p), sp, repair_mode,
                      static_cast<DevCounters*>(counters), s)
             ? GGEMM_ERR_NUMERICS
             : GGEMM_OK;
}

extern "C" int ggemm_stage_wait_probe(void* counters, long long wait_ns, cudaStream_t s) {
  DevCounters* cnt = static_cast<DevCounters*>(counters);
  if (!cnt && noalloc_counters(&cnt) != GGEMM_OK) return GGEMM_ERR_CUDA;
  return launch_wait_probe(cnt, (unsigned long long)(wait_ns > 0 ? wait_ns : 0), s)
             ? GGEMM_ERR_CUDA
             : GGEMM_OK;
}

extern "C" int ggemm_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

extern "C" const char* ggemm_version(void) { return "ggemm-b200 0.1 (sm_100a)"; }

extern "C" int ggemm_stage_plan(const ggemm_problem_t* problems, int num,
                                const ggemm_config_t* cfg, int path, int num_sms,
                                double fp64_flops, double int8_ops, double mem_bw,
                                double tiny_mnk, double rho_budget, int* route,
                                int* num_moduli, int* tile_cfg) {
  if (num < 0 || (num > 0 && (!problems || !route || !num_moduli || !tile_cfg)))
    return GGEMM_ERR_INVALID;
  DeviceModel dm{};
  device_model_init(&dm, num_sms > 0 ? num_sms : 148);  // calibration file, environment
  if (fp64_flops > 0) dm.fp64_flops = fp64_flops;
  if (int8_ops > 0) dm.gemm_ops = int8_ops;
  if (mem_bw > 0) dm.prep_bw = dm.recon_bw = mem_bw;
  if (tiny_mnk >= 0) dm.tiny_mnk = tiny_mnk;
  std::vector<PlanEntry> out((size_t)std::max(num, 1));
  const int r = plan_group(problems, num, cfg, (ggemm_path_t)path, dm,
                           rho_budget > 0 ? rho_budget : env_rho_budget(), out.data(), nullptr,
                           0);
  if (r) return r;
  for (int g = 0; g < num; ++g) {
    route[g] = out[g].route;
    num_moduli[g] = out[g].num_moduli;
    tile_cfg[g] = out[g].tile_cfg;
  }
  return GGEMM_OK;
}

extern "C" int ggemm_stage_reuse(const ggemm_problem_t* problems, int num, const int* nmod,
                                 int policy, int* out) {
  if (num < 0 || !out) return GGEMM_ERR_INVALID;
  ReuseArena ar;
  if (ar.reserve(std::max(num, 1))) return GGEMM_ERR_INVALID;
  const ReuseResult r =
      ar.build(problems, num, nmod, policy == 1 ? kReusePromote : kReuseExactN);
  if (r.status) return r.status == 1 ? GGEMM_ERR_WORKSPACE : GGEMM_ERR_INVALID;
  out[0] = r.num_ua;
  out[1] = r.num_ub;
  out[2] = r.num_promoted;
  int* o = out + 3;
  for (int i = 0; i < num; ++i) o[i] = i < r.num_ua ? r.ua_rep[i] : -1;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = i < r.num_ua ? r.ua_nmod[i] : 0;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = i < r.num_ub ? r.ub_rep[i] : -1;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = i < r.num_ub ? r.ub_nmod[i] : 0;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = r.prob_a[i];
  o += num;
  for (int i = 0; i < num; ++i) o[i] = r.prob_b[i];
  o += num;
  for (int i = 0; i < num; ++i) o[i] = r.eff_nmod[i];
  return GGEMM_OK;
}

extern "C" size_t ggemm_stage_crt_tables(void* out, size_t bytes) {
  int st = 0;
  const CrtTables& t = crt_tables(&st);
  if (st != 0) return 0;
  if (out) std::memcpy(out, &t, bytes < sizeof t ? bytes : sizeof t);
  return sizeof t;
}

extern "C" double ggemm_stage_error_bound(int k, int num_moduli) {
  return error_bound(k, num_moduli);
}
