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
 * (0 = ok, 1 = a residue-GEMM pipeline wait ran past its deadline); -1 on a CUDA error. */
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

#ifdef __cplusplus
}
#endif
