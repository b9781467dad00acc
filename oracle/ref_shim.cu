// ref_shim.cu -- C entry points over the REFERENCE implementation (moneychen168/Coding-Basic-HW-2),
// compiled together with the reference's own sources (src/*.cu, src/*.cpp, unmodified, read
// from where they lie) into oracle/_ref/libggemm_ref.so by oracle/Makefile.
//
// TEST INFRASTRUCTURE ONLY.  The product never loads this library.  tests/ use it as the
// checker:
//   * on the CPU: the reference's CRT tables (src/moduli.h:124-181), error bound and N choice
//     (src/ozaki2_numerics.cu:639-673), planner (src/planner.cpp:286-330) and operand-reuse pass
//     (src/operand_reuse.cpp:47-141) -- host code, no GPU needed;
//   * on a B200: the reference's own prep / INT8 GEMM / reconstruct kernels built for sm_100a
//     (src/ozaki2_numerics.cu:609-637, src/int8_grouped_gemm.cu:711-735) and its public
//     ggemm_* API, as the device oracle for bit-exact residues, C32 and outputs.
#include <cstring>

#include "int8_grouped_gemm.h"
#include "internal.h"
#include "moduli.h"
#include "operand_reuse.h"
#include "ozaki2_numerics.h"
#include "planner.h"

extern "C" {

size_t ozr_tables_size() { return sizeof(oz2_crt_tables); }
int ozr_build_tables(void* out, size_t bytes) {
  oz2_crt_tables t;
  int r = oz2_build_crt_tables(&t);
  std::memcpy(out, &t, bytes < sizeof t ? bytes : sizeof t);
  return r;
}
double ozr_error_bound(int k, int N) { return oz2_error_bound(k, N); }
int ozr_choose(int k, double target) { return oz2_choose_num_moduli(k, target); }
int ozr_choose_cw(int k, double rho) { return oz2_choose_num_moduli_cw(k, rho); }

size_t ozr_sizeof_problem() { return sizeof(ggemm_problem_t); }
size_t ozr_sizeof_plan_entry() { return sizeof(ggemm_plan_entry_t); }
size_t ozr_sizeof_oz2_problem() { return sizeof(oz2_problem); }
size_t ozr_sizeof_i8_problem() { return sizeof(i8_problem); }

// Planner with an explicit device model (no calibration file, no environment).
int ozr_plan(const ggemm_problem_t* probs, int num, const ggemm_config_t* cfg, int path,
             int num_sms, double fp64_flops, double int8_ops, double mem_bw, double tiny_mnk,
             ggemm_plan_entry_t* out) {
  ggemm_device_model_t dm;
  dm.num_sms = num_sms;
  dm.fp64_flops = fp64_flops;
  dm.int8_ops = int8_ops;
  dm.mem_bw = mem_bw;
  dm.tiny_mnk = tiny_mnk;
  return ggemm_plan(probs, num, cfg, (ggemm_path_t)path, &dm, out);
}

// Operand reuse: out receives, in order, [num_ua, num_ub, num_promoted] then
// ua_rep[num], ua_nmod[num], ub_rep[num], ub_nmod[num], prob_a[num], prob_b[num], eff_nmod[num].
int ozr_reuse(const ggemm_problem_t* probs, int num, const int* nmod, int policy, int* out) {
  reuse_arena ar;
  if (ar.reserve(num > 0 ? num : 1) != REUSE_OK) return -1;
  reuse_plan rp = build_operand_reuse(ar, probs, num, nmod, (reuse_policy)policy);
  if (rp.status != REUSE_OK) return rp.status;
  out[0] = rp.num_ua;
  out[1] = rp.num_ub;
  out[2] = rp.num_promoted;
  int* o = out + 3;
  for (int i = 0; i < num; ++i) o[i] = i < rp.num_ua ? rp.ua_rep[i] : -1;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = i < rp.num_ua ? rp.ua_nmod[i] : 0;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = i < rp.num_ub ? rp.ub_rep[i] : -1;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = i < rp.num_ub ? rp.ub_nmod[i] : 0;
  o += num;
  for (int i = 0; i < num; ++i) o[i] = rp.prob_a[i];
  o += num;
  for (int i = 0; i < num; ++i) o[i] = rp.prob_b[i];
  o += num;
  for (int i = 0; i < num; ++i) o[i] = rp.eff_nmod[i];
  return 0;
}

// ---- device seams (B200 only) ----------------------------------------------------------------
int ozr_init_constants() { return oz2_init_constants(); }
int ozr_prep_grouped(const void* d_probs, int num, int max_m, int max_n, void* stream) {
  return oz2_prep_grouped(static_cast<const oz2_problem*>(d_probs), num, max_m, max_n,
                          static_cast<cudaStream_t>(stream));
}
int ozr_reconstruct_grouped(const void* d_probs, int num, int max_m, int max_n, void* stream,
                            int mode) {
  return oz2_reconstruct_grouped(static_cast<const oz2_problem*>(d_probs), num, max_m, max_n,
                                 static_cast<cudaStream_t>(stream), mode);
}
size_t ozr_i8_sched_ws_bytes(int num) { return i8_grouped_gemm_sched_ws_bytes(num, 0); }
int ozr_i8_grouped_gemm(const void* d_probs, int num, const void* h_probs, void* d_ws,
                        size_t ws_bytes, void* stream) {
  return i8_grouped_gemm(static_cast<const i8_problem*>(d_probs), num,
                         static_cast<const i8_problem*>(h_probs), d_ws, ws_bytes,
                         static_cast<cudaStream_t>(stream));
}
int ozr_read_counters(unsigned long long* out4, int reset, void* stream) {
  oz2_counters c{};
  int r = oz2_read_counters(out4 ? &c : nullptr, reset, static_cast<cudaStream_t>(stream));
  if (out4) {
    out4[0] = c.nonfinite_vectors;
    out4[1] = c.uncertified;
    out4[2] = c.repaired;
    out4[3] = c.safety_fallback;
  }
  return r;
}
void ozr_force_prep_split(int S) { oz2_debug_force_prep_split(S); }

}  // extern "C"
