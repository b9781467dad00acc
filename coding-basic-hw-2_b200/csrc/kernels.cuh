// kernels.cuh -- host-visible declarations of the three pipeline kernels and their device data.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "ggemm_stages.h"

namespace g2 {

// Device counters of a handle (or of a stage call): 64 bytes, zeroed by the owner.
struct DevCounters {
  unsigned long long nonfinite;  // A rows / B columns containing NaN or Inf (prep)
  unsigned long long uncertified;
  unsigned long long repaired;
  unsigned long long safety;
  unsigned int status;  // 0 = ok; otherwise a kStatus* code set by a kernel
  unsigned int pad[7];
};
static_assert(sizeof(DevCounters) == 64, "counter block layout");

enum : unsigned int {
  kStatusOk = 0,
  kStatusGemmTimeout = 1,  // a residue-GEMM pipeline wait ran past its deadline
};

// One problem of the residue GEMM as the kernel sees it (built on the host).
struct GemmJob {
  const int8_t* A;
  const int8_t* B;
  int32_t* C;
  long long a_plane, b_plane, c_plane;
  int m, n, ksteps, planes;
  int rga, rgb, tm, tn;  // row groups of A / B, tile rows / columns
  int bn;                // tile width: 256 columns, or 128 for n <= 128
};

constexpr int kGemmBM = 128, kGemmBNMax = 256;

// Tile shape of one problem: 128 rows x 256 columns (128 when n <= 128); requires m, n set.
inline void set_gemm_tiling(GemmJob& j) {
  j.bn = j.n > 128 ? 256 : 128;
  j.tm = (j.m + kGemmBM - 1) / kGemmBM;
  j.tn = (j.n + j.bn - 1) / j.bn;
  j.rga = (j.m + 7) / 8;
  j.rgb = (j.n + 7) / 8;
}
constexpr int kPrepThreads = 256, kReconThreads = 256, kReconPerThread = 4;

// Blocks of one prep descriptor (A: 32 rows per block, B: 8 columns per block).
inline int prep_blocks(const ggemm_prep_desc_t& d) {
  if (d.rows <= 0 || d.k < 0) return 0;
  return d.kind == 0 ? (d.rows + 31) / 32 : (d.rows + 7) / 8;
}
inline long long recon_blocks(const ggemm_recon_desc_t& d) {
  const long long mn = (long long)d.m * (long long)d.n;
  const long long per = (long long)kReconThreads * kReconPerThread;
  return (mn + per - 1) / per;
}
inline long long gemm_tiles(const GemmJob& j) { return (long long)j.tm * j.tn * j.planes; }

// Uploads the CRT constants to the current device (once per device; thread-safe).
int upload_tables_current_device();
// Streaming multiprocessors of the current device (cached).
int current_device_sms();

// Launchers: one kernel each on `s`.  prefix: device array of num+1 exclusive block / tile
// prefix sums.  Return cudaError_t of the launch.
int launch_prep(const ggemm_prep_desc_t* d_descs, const int* d_prefix, int num, int total_blocks,
                DevCounters* cnt, cudaStream_t s);
int launch_gemm(const GemmJob* d_jobs, const long long* d_prefix, int num, long long total_tiles,
                DevCounters* cnt, cudaStream_t s);
int launch_recon(const ggemm_recon_desc_t* d_descs, const long long* d_prefix, int num,
                 long long total_blocks, int mode, DevCounters* cnt, cudaStream_t s);

}  // namespace g2
