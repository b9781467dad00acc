// kernels.cuh -- host-visible declarations of the three pipeline kernels and their device data.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include <algorithm>

#include "ggemm_stages.h"

namespace g2 {

// Device counters of a handle (or of a stage call): 64 bytes, zeroed by the owner.
struct DevCounters {
  unsigned long long nonfinite;  // A rows / B columns containing NaN or Inf (prep)
  unsigned long long uncertified;
  unsigned long long repaired;
  unsigned long long safety;
  unsigned int status;  // 0 = ok; otherwise a kStatus* code set by a kernel
  unsigned int pad0;
  unsigned long long safety_ticket;  // work ticket of the safety-fallback blocks (reconstruct)
  unsigned int pad[4];
};
static_assert(sizeof(DevCounters) == 64, "counter block layout");

enum : unsigned int {
  kStatusOk = 0,
  kStatusGemmTimeout = 1,  // a residue-GEMM pipeline wait ran past its deadline
  kStatusPrepTimeout = 2,  // a prep residue-MMA wait ran past its deadline
  kStatusProbeTimeout = 3, // the bounded-wait probe (launch_wait_probe) gave up, as designed
};

// Digit layout ("Y8", GGEMM_PRODUCTS_DIGITS in ggemm_stages.h) of the products handed from the
// GEMM to the reconstruct: 16-byte records (16 digits, or 4 int32 abs products) of one row,
// the records of a column block stored row after row, so that a GEMM epilogue warp (32 rows)
// writes 512 contiguous bytes per store and a reconstruct thread reads 8 columns of one plane
// with one 8-byte load.  Planes are sized for whole 32-column chunks (the epilogue's unit).
inline size_t y8_plane_bytes(int m, int n) { return ggemm_digit_plane_bytes(m, n); }
inline size_t y8_bytes(int m, int n, int N) {
  return (size_t)N * y8_plane_bytes(m, n) + 4 * y8_plane_bytes(m, n);
}
// int32 layout: N + 1 planes of m * n products (column-major), each padded to 64 elements.
inline size_t c32_bytes(int m, int n, int N) {
  return 4 * (size_t)(N + 1) * (((size_t)m * (size_t)n + 63) / 64 * 64);
}
// The digit layout is used whenever it is no larger than the int32 layout (it is larger only
// for n below about 10, where the 32-column records are mostly padding).
inline bool use_y8(int m, int n, int N) { return y8_bytes(m, n, N) <= c32_bytes(m, n, N); }

// One problem of the residue GEMM as the kernel sees it (built on the host).
struct GemmJob {
  const int8_t* A;
  const int8_t* B;
  int32_t* C;            // int32 products (y8 == 0)
  uint8_t* Y;            // digit layout (y8 == 1)
  long long a_plane, b_plane, c_plane, y_plane;
  int m, n, ksteps, planes;
  int rga, rgb, tm, tn;  // row groups of A / B, tile rows / columns
  int bm, bn;            // tile height (128, or 256 on CTA pairs) and width (256, or 128 for
                         // n <= 128 on single CTAs)
  int N, plane0, y8;     // moduli, index of the job's first plane, output layout
};

constexpr int kGemmBM = 128, kGemmBNMax = 256;

// Tile shape of one problem: 128 rows x 256 columns (128 when n <= 128); requires m, n set.
inline void set_gemm_tiling(GemmJob& j) {
  j.bm = kGemmBM;
  j.bn = j.n > 128 ? 256 : 128;
  j.tm = (j.m + kGemmBM - 1) / kGemmBM;
  j.tn = (j.n + j.bn - 1) / j.bn;
  j.rga = (j.m + 7) / 8;
  j.rgb = (j.n + 7) / 8;
}
// Tile shape of the paired GEMM (launch_gemm_pair): 256 x 256 tiles (a CTA pair each).
inline void set_gemm_tiling_pair(GemmJob& j) {
  j.bm = 256;
  j.bn = 256;
  j.tm = (j.m + 255) / 256;
  j.tn = (j.n + 255) / 256;
  j.rga = (j.m + 7) / 8;
  j.rgb = (j.n + 7) / 8;
}
// Whether a set of problems should run on the paired GEMM: its 256-row tiles pad the rows by at
// most 10 % more multiply-adds than gemm_kernel's 128-row tiles, and there are tiles for every
// pair of SMs.  m, n, ksteps, planes per problem.  Measured with the 8-K-step rings: the paired
// kernel took 6.41 against 7.41 ms on one C3 problem, 6.06 against 6.73 ms on one C5 component
// and 1.30 against 1.40 ms on the C2 group (7.4 % more multiply-adds there).
inline bool gemm_pair_pays(const int* m, const int* n, const int* ksteps, const int* planes,
                           int num, int num_sms) {
  double w1 = 0, w2 = 0;
  long long tiles = 0;
  for (int i = 0; i < num; ++i) {
    const double per = (double)n[i] * ksteps[i] * planes[i];
    w1 += (double)((m[i] + 127) / 128 * 128) * per;
    w2 += (double)((m[i] + 255) / 256 * 256) * per;
    tiles += (long long)((m[i] + 255) / 256) * ((n[i] + 255) / 256) * planes[i];
  }
  return w2 <= 1.10 * w1 && tiles >= num_sms;
}
constexpr int kPrepThreads = 256, kReconThreads = 256, kReconPerThread = 4;

// Blocks of one prep descriptor (A: 32 rows per block, B: 8 columns per block).
inline int prep_blocks(const ggemm_prep_desc_t& d) {
  if (d.rows <= 0 || d.k < 0) return 0;
  return (d.kind & 1) == 0 ? (d.rows + 31) / 32 : (d.rows + 7) / 8;
}
inline long long recon_blocks(const ggemm_recon_desc_t& d) {
  const long long mn = (long long)d.m * (long long)d.n;
  const long long per = (long long)kReconThreads * kReconPerThread;
  return (mn + per - 1) / per;
}
// Digit-layout reconstruct: one block per 128 rows x 16 columns (one digit record column).
constexpr int kY8Rows = 128;
inline long long recon_blocks_y8(const ggemm_recon_desc_t& d) {
  if (d.m <= 0 || d.n <= 0) return 0;
  return (long long)((d.n + 15) / 16) * ((d.m + kY8Rows - 1) / kY8Rows);
}
// Blocks of one reconstruct descriptor in its layout.
inline long long recon_job_blocks(const ggemm_recon_desc_t& d) {
  return d.layout == GGEMM_PRODUCTS_DIGITS ? recon_blocks_y8(d) : recon_blocks(d);
}
inline long long gemm_tiles(const GemmJob& j) { return (long long)j.tm * j.tn * j.planes; }

// Uploads the CRT constants to the current device (once per device; thread-safe).
int upload_tables_current_device();
// Streaming multiprocessors of the current device (cached).
int current_device_sms();

// Copies `bytes` from pinned, mapped host memory (src_dev: its device address) to device memory
// d_dst with a kernel (no copy engine, so it does not wait behind other streams' host -> device
// copies).  Both addresses 16-byte aligned.  Returns a cudaError_t.
int launch_blob_upload(void* d_dst, const void* src_dev, size_t bytes, cudaStream_t s);
// Launchers, on `s`: the GEMM one kernel, prep and the reconstruct one kernel per class of
// moduli counts present.  prefix: device array of num+1 exclusive block / tile prefix sums.
// Return the cudaError_t of the launches.
// Prep is compiled per class of moduli counts: N = 14, 15 and 16 (the counts the N selection
// gives for k up to 2^16) each get an instance with their epilogue called directly; the other
// counts share one instance per accumulator mode (N <= 15 / N > 15) that dispatches on N.
__host__ __device__ constexpr inline bool prep_needs_bias(int N) { return N > 15; }
constexpr int kPrepClasses = 5;
inline int prep_class(int N) { return N == 14 ? 0 : N == 15 ? 1 : N <= 15 ? 2 : N == 16 ? 3 : 4; }
// Descriptors sorted by class: class c owns descriptors [first[c], first[c + 1]) and blocks
// [block0[c], block0[c + 1]) of the prefix numbering.
struct PrepSplit {
  int first[kPrepClasses + 1];
  long long block0[kPrepClasses + 1];
};
// Sorts descs[0, num) by class (stable; descriptors are independent), writes the exclusive
// block prefix (num + 1 entries) and the split.
inline void prep_partition(ggemm_prep_desc_t* descs, int num, int* prefix, PrepSplit* sp) {
  std::stable_sort(descs, descs + num, [](const ggemm_prep_desc_t& a, const ggemm_prep_desc_t& b) {
    return prep_class(a.N) < prep_class(b.N);
  });
  long long blocks = 0;
  int x = 0;
  for (int c = 0; c < kPrepClasses; ++c) {
    sp->first[c] = x;
    sp->block0[c] = blocks;
    for (; x < num && prep_class(descs[x].N) == c; ++x) {
      prefix[x] = (int)blocks;
      blocks += prep_blocks(descs[x]);
    }
  }
  sp->first[kPrepClasses] = num;
  sp->block0[kPrepClasses] = blocks;
  prefix[num] = (int)blocks;
}
// One launch per non-empty class; *launches, when given, is increased by their number.
int launch_prep(const ggemm_prep_desc_t* d_descs, const int* d_prefix, const PrepSplit& sp,
                DevCounters* cnt, cudaStream_t s, int* launches = nullptr);
// walk_flags: kGemmWalkBothEnds -- each CTA alternates between the front (deep K) and back
// (shallow K) of the tile order, so that shallow tiles' epilogues overlap deep tiles' MMAs
// (pass it when gemm_jobs_ragged()); kGemmWalkPlaneOuter -- tiles numbered plane by plane over
// all jobs (every job has the same plane count, d_prefix counts one plane's tiles per job and
// total_tiles = planes x d_prefix[num]), for groups whose problems share operands.
constexpr int kGemmWalkBothEnds = 1, kGemmWalkPlaneOuter = 2;
int launch_gemm(const GemmJob* d_jobs, const long long* d_prefix, int num, long long total_tiles,
                DevCounters* cnt, cudaStream_t s, int walk_flags);
// Whether jobs differ in K depth (the alternating walk pays only then).
inline bool gemm_jobs_ragged(const GemmJob* jobs, int num) {
  for (int i = 1; i < num; ++i)
    if (jobs[i].ksteps != jobs[0].ksteps) return true;
  return false;
}
// The paired GEMM (CTA pairs, tcgen05.mma.cta_group::2) over jobs tiled by set_gemm_tiling_pair.
int launch_gemm_pair(const GemmJob* d_jobs, const long long* d_prefix, int num,
                     long long total_tiles, DevCounters* cnt, cudaStream_t s, int walk_flags);
// Reconstruct: compiled per repair mode and per class of moduli counts (N = 14, 15, 16 each, the
// rest together); descriptors sorted by class, class c owning descriptors [first[c],
// first[c + 1]) and blocks [block0[c], block0[c + 1]) (blocks per descriptor: recon_job_blocks).
constexpr int kReconClasses = 4;
inline int recon_class(int N) { return N == 14 ? 0 : N == 15 ? 1 : N == 16 ? 2 : 3; }
struct ReconSplit {
  int first[kReconClasses + 1];
  long long block0[kReconClasses + 1];
};
// Sorts descs[0, num) by class (stable; descriptors are independent), writes the exclusive
// block prefix (num + 1 entries) and the split.
inline void recon_partition(ggemm_recon_desc_t* descs, int num, long long* prefix,
                            ReconSplit* sp) {
  std::stable_sort(descs, descs + num,
                   [](const ggemm_recon_desc_t& a, const ggemm_recon_desc_t& b) {
                     return recon_class(a.N) < recon_class(b.N);
                   });
  long long blocks = 0;
  int x = 0;
  for (int c = 0; c < kReconClasses; ++c) {
    sp->first[c] = x;
    sp->block0[c] = blocks;
    for (; x < num && recon_class(descs[x].N) == c; ++x) {
      prefix[x] = blocks;
      blocks += recon_job_blocks(descs[x]);
    }
  }
  sp->first[kReconClasses] = num;
  sp->block0[kReconClasses] = blocks;
  prefix[num] = blocks;
}
// Bounded-wait probe: one block waits on an mbarrier that nothing arrives on, through the same
// bounded wait (mbar_wait with a %globaltimer deadline) as the pipeline kernels, gives up after
// wait_ns and records kStatusProbeTimeout in cnt->status.  It shows the give-up path ends and
// leaves the context usable, without a fault.  wait_ns is clamped to [1 us, 1 s].
int launch_wait_probe(DevCounters* cnt, unsigned long long wait_ns, cudaStream_t s);
// One launch per non-empty class; the first also carries the safety-fallback blocks (entries of
// NaN / Inf rows and columns, safety_blocks).  *launches, when given, is increased by their
// number.  nonfinite_hint: cnt->nonfinite holds prep's count of non-finite rows / columns for
// these descriptors (0 lets the safety blocks return at once); otherwise they scan every tile's
// shifts.
int launch_recon(const ggemm_recon_desc_t* d_descs, const long long* d_prefix,
                 const ReconSplit& sp, int mode, DevCounters* cnt, cudaStream_t s,
                 int* launches = nullptr, bool nonfinite_hint = false);

}  // namespace g2
