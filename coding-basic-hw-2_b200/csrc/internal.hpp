// internal.hpp -- handle layout and helpers shared by the host translation units.
#pragma once
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

#include "crt.hpp"
#include "ggemm.h"
#include "ggemm_stages.h"
#include "kernels.cuh"
#include "planner.hpp"
#include "reuse.hpp"

namespace g2 {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline size_t c_plane_elems(int m, int n) { return align_up((size_t)m * (size_t)n, 64); }
// int32 elements of one problem's products in the layout use_y8 picks (kernels.cuh),
// 256-byte aligned.
inline size_t product_elems(int m, int n, int N) {
  return align_up(use_y8(m, n, N) ? y8_bytes(m, n, N) : c32_bytes(m, n, N), kAlign) / 4;
}
inline size_t ws_ints(int rows) { return align_up(4 * (size_t)rows, 64); }
// Bytes of all planes (N residue planes + abs plane) of one operand image.
inline size_t img_bytes(int rows, int k, int N) {
  return (size_t)(N + 1) * align_up(ggemm_img_plane_bytes(rows, k), kAlign);
}

// Native FP64 groups for cublasDgemmGroupedBatched (host arrays, one entry per group).
struct NativeGroups {
  std::vector<cublasOperation_t> ta, tb;
  std::vector<int> m, n, k, lda, ldb, ldc, size;
  std::vector<double> alpha, beta;
  void reserve(size_t P);
};
// Sorts idx[0..cnt) so problems with equal (m, n, k, lda, ldb, ldc, alpha, beta) are adjacent
// and fills one group per run; returns the number of groups.
int group_native(const ggemm_problem_t* probs, int* idx, int cnt, NativeGroups& g);

// One chunk of emulated problems: descriptors live in the device blob at the given offsets.
struct Chunk {
  int first, count;        // range in emu order
  size_t off_prep, off_prep_prefix, off_jobs, off_job_prefix, off_recon, off_recon_prefix;
  int num_prep, prep_blocks;
  size_t base_b, base_c;   // byte offsets of the chunk's B images and products in the pool
  size_t base_wa, base_wb; // ... of its row (A) and column (B) workspace
  PrepSplit prep_split;    // descriptors sorted by prep instance (launch_prep)
  ReconSplit recon_split;  // ... by reconstruct instance (launch_recon)
  bool qscale;  // A images q-scaled (every problem of the chunk in the digit layout)
  bool pair;    // residue GEMM on CTA pairs (launch_gemm_pair)
  bool ragged;  // jobs of different K depth (two-ended tile walk)
  bool plane_outer;  // tiles numbered plane by plane (problems share operands; kGemmWalkPlaneOuter)
  long long tiles, recon_blocks;
};

}  // namespace g2

struct ggemm_handle_s {
  int device = 0, num_sms = 148;
  cudaStream_t stream = nullptr;
  cublasHandle_t cublas = nullptr;
  void* cublas_ws = nullptr;
  size_t cublas_ws_bytes = 0;

  int max_problems = 0;
  size_t max_A = 0, max_B = 0, max_C = 0;
  int min_k = 32;

  // device workspace (allocated at create; every call fits into it, in chunks if needed).
  // One pool per handle holds, per chunk, the A images from offset 0, then the B images, then
  // the products (Chunk::base_b / base_c), so the split follows each call's shapes.
  int8_t* pool = nullptr;
  size_t pool_cap = 0;  // bytes
  g2::DevCounters* counters = nullptr;

  // one pinned, mapped host descriptor blob per slot (h_blob_dev: its device address), copied
  // into the device blob by launch_blob_upload
  char* h_blob[2] = {nullptr, nullptr};
  const void* h_blob_dev[2] = {nullptr, nullptr};
  char* d_blob[2] = {nullptr, nullptr};
  size_t blob_cap = 0;
  cudaEvent_t slot_done[2] = {nullptr, nullptr};
  int next_slot = 0;

  // host scratch, sized at create (no allocation inside calls)
  std::vector<g2::PlanEntry> plan;
  std::vector<int> memo;
  std::vector<int> emu, nat, order;
  std::vector<int> ua_of, ub_of;          // per emulated problem: unique operand ids
  std::vector<int> ua_rep, ub_rep, ua_n, ub_n;
  std::vector<int> ua_chunk, ub_chunk;    // last chunk that placed a unique operand
  std::vector<size_t> ua_img, ub_img, ua_ws, ub_ws;  // ... and where (while chunking)
  // per emulated problem, in its own chunk: image / workspace offsets of its A and B, whether it
  // prepares them there, and the offset of its products
  std::vector<size_t> pa_img, pb_img, pa_ws, pb_ws;
  std::vector<char> pa_new, pb_new;
  std::vector<size_t> c32_off;
  std::vector<int> pair_m, pair_n, pair_k, pair_p;  // gemm_pair_pays arguments of a chunk
  std::vector<g2::Chunk> chunks;
  g2::NativeGroups ngroups;
  std::vector<const void*> nat_ptrs;

  g2::DeviceModel dm{};
  g2::ReuseArena reuse;
  double rho_budget = 16.0;
  int reuse_promote = 0;
  int gemm_pair = -1;  // GGEMM_GEMM_PAIR: -1 chosen per chunk (gemm_pair_pays), 0 never, 1 always
  int stats_repair = 0;
  int ws_diag_printed = 0;
  cudaEvent_t stage_ev[4] = {nullptr, nullptr, nullptr, nullptr};
  bool stage_ev_on = false;
};

namespace g2 {
// Validation shared by direct calls and plans (reference src/ggemm.cu:83-100).
int validate_call(ggemm_handle_t h, const ggemm_problem_t* p, int num);
// Public repair mode -> stage repair mode (-1 if invalid); default ON for AUTO, COUNT else.
int stage_repair_mode(ggemm_path_t path, const ggemm_config_t* cfg);

// Everything a call of the emulated grouped pipeline enqueues, prepared on the host.
struct EmuCall {
  int ne = 0, nn = 0, nprep_total = 0;
  int nmax = 0, nmin = 0;
  int num_ua = 0, num_ub = 0, num_promoted = 0;
  bool reuse = false;
  size_t blob_bytes = 0;
  size_t off_nat_ptrs = 0;
  int nat_groups = 0;
};
// Plans a call and writes every descriptor into host blob `hb`; the device addresses are
// computed against `db`.  Returns GGEMM_OK or an error.
int build_emu_call(ggemm_handle_t h, ggemm_path_t path, const ggemm_config_t* cfg,
                   const ggemm_problem_t* probs, int num, char* hb, const char* db,
                   EmuCall* out);
// Enqueues the launches of a built call on s (descriptors already on the device at db).
// per_plane: EMU_LOOP (one GEMM launch per plane).  record: stage events (ggemm_ext.h).
int enqueue_emu_call(ggemm_handle_t h, const EmuCall& c, const ggemm_problem_t* probs,
                     const char* db, int repair, bool per_plane, bool record, cudaStream_t s,
                     int* launches);
int enqueue_native(ggemm_handle_t h, const ggemm_problem_t* probs, const int* idx, int cnt,
                   bool grouped, int ngroups, const char* d_ptrs, cudaStream_t s, int* launches);
// Device address of the counter block of ggemm_dgemm_noalloc's scratch on the current device
// (noalloc.cu; sets the device up on first use).  Returns GGEMM_OK or an error.
int noalloc_counters(DevCounters** out);
}  // namespace g2
