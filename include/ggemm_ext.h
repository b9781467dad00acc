/* ggemm_ext.h -- extensions of this library beyond the reference API.
 *
 * Instrumentation: the reference marks its stages with NVTX ranges (src/internal.h:16-34,
 * src/ggemm.cu:622-680); here a caller can additionally ask a handle to record CUDA events on
 * its stream around the stages of every emulated call, so stage times can be measured on the
 * device without a profiler.
 *
 * Device status: kernels that give up on a bounded wait record a status word per handle
 * (no reference counterpart: the reference's kernels never wait on one another).
 *
 * Multi-GPU sharding: the reference runs on one device (README.md:189-190); this partitions a
 * group across several devices by estimated cost, keeping problems that share an A or B operand
 * together and splitting the columns of problems too large for one shard.
 */
#pragma once
#include "ggemm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* events: 4 cudaEvent_t (created by the caller) recorded on the handle's stream at: start of
 * the first prep, end of prep, end of the residue GEMM, end of the reconstruct of each
 * emulated call that runs as a single chunk.  NULL switches recording off. */
int ggemm_set_stage_events(ggemm_handle_t h, cudaEvent_t* events);

/* Synchronizes the handle's stream and returns the device status word of the handle's kernels
 * (0 = ok, 1 = a residue-GEMM pipeline wait ran past its deadline, 2 = a prep residue-MMA
 * wait ran past its deadline); -1 on a CUDA error. */
int ggemm_device_status(ggemm_handle_t h);

/* Partitions `num` problems over `num_shards` devices.  A problem may be split into column
 * blocks (multiples of 128 columns) so that no shard's estimated cost exceeds the average by
 * more than one column block.  Outputs, for up to out_cap sub-problems:
 *   out[i]        the sub-problem (pointers offset into the original A / B / C: B + j0*ldb,
 *                 C + j0*ldc for a column block starting at column j0)
 *   out_shard[i]  its shard (0 .. num_shards-1), out_src[i] its original problem index
 * *num_out receives the number written.  Problems sharing an A or B pointer stay on one shard
 * (column blocks of one problem may spread).  Returns GGEMM_OK, GGEMM_ERR_INVALID or
 * GGEMM_ERR_WORKSPACE (out_cap too small). */
int ggemm_shard_group(const ggemm_problem_t* problems, int num, int num_shards,
                      ggemm_problem_t* out, int* out_shard, int* out_src, int out_cap,
                      int* num_out);

/* One emulated FP64 GEMM, C = alpha*A*B + beta*C (column-major, device pointers on the current
 * device), for callers that cannot allocate device memory: code that owns no CUDA allocator,
 * runs inside another runtime's memory pool, or must not call cudaMalloc / cudaFree.  It has
 * no counterpart in the reference.  The caller passes inputs and outputs; all scratch (residue
 * images, products, workspace, descriptors, counters) lives in one fixed 64 MiB device
 * array compiled into this library, which every GPU that loads the library holds until exit.
 * Nothing is allocated: no cudaMalloc / cudaFree, no allocating library routine.
 *   num_moduli: 0 = adaptive (target 1e-15) or a fixed N in [2, 20];
 *   repair_mode: GGEMM_REPAIR_* (default = COUNT, as GGEMM_PATH_EMU_GROUPED).
 * For alpha != 0 and k > 0, results equal ggemm_grouped_dgemm(GGEMM_PATH_EMU_GROUPED) of the
 * same problem, bit for bit.  For alpha == 0 or k == 0 this computes C = beta C in its own kernel
 * without reading A or B (C = +0, C not read, when beta == 0); the grouped call sends those
 * problems to cuBLAS, which gives the same values but may give zeros of the other sign.
 * A problem whose scratch exceeds 64 MiB (about 1130^3 at N = 15) returns GGEMM_ERR_WORKSPACE
 * with a one-line message on stderr, before anything is enqueued; k > 131040 returns
 * GGEMM_ERR_UNSAFE.
 * The first call on a device does a one-time set-up with that device current (uploads the CRT
 * constants, which synchronizes the device, and looks up the array's device address); make that
 * first call before any stream capture.  Work is enqueued on `stream`.  Every call shares the
 * array and finds the previous call's contents in it: calls that overlap on the GPU (other
 * streams, other host threads) race and must be ordered by the caller. */
int ggemm_dgemm_noalloc(const ggemm_problem_t* problem, int num_moduli, int repair_mode,
                        cudaStream_t stream);

/* Device status of the last ggemm_dgemm_noalloc call enqueued on this device: synchronizes
 * `stream` (the stream of that call), then reads the status word in the fixed scratch (no
 * allocation).  0 = ok; 1 or 2 = a residue-GEMM or prep pipeline wait ran past its deadline, so
 * that call's C is not valid; -1 on a CUDA error.  The next call clears the word when it starts
 * on the GPU, so read it before enqueueing another call. */
int ggemm_dgemm_noalloc_status(cudaStream_t stream);

#ifdef __cplusplus
}
#endif
