/* ggemm_stages.h -- stage-level entry points of the emulation pipeline (parity seams).
 *
 * The reference exposes its three stages as internal C++ functions that its own tests call
 * one by one (src/ozaki2_numerics.h:39-105 and src/int8_grouped_gemm.h:34-101).  These are the
 * same seams as a plain C ABI, so a test can run prep, the residue GEMM and the reconstruct
 * separately and compare residues, int32 products and outputs with a checker:
 *   ggemm_stage_prep    replaces oz2_prep_grouped          (src/ozaki2_numerics.cu:609-623)
 *   ggemm_stage_gemm    replaces i8_grouped_gemm / _launch (src/int8_grouped_gemm.cu:711-780)
 *   ggemm_stage_recon   replaces oz2_reconstruct_grouped   (src/ozaki2_numerics.cu:625-637)
 * Counters (oz2_read_counters, src/ozaki2_numerics.cu:675-693) are a caller-owned 64-byte
 * device block, read back by the caller.
 *
 * Residue planes are stored in this library's own layout: each plane is the image of a K-major
 * tensor-core operand with 32-byte swizzle, so the GEMM fetches a tile with one bulk copy per
 * 32-byte K step:
 *   rows are grouped by 8 (row group g = r / 8), K by 32 bytes (step s = q / 32);
 *   atom (s, g) = 256 contiguous bytes at ((s * RG) + g) * 256, RG = ceil(rows / 8);
 *   inside an atom, row r % 8 occupies 32 bytes at (r % 8) * 32, its two 16-byte halves
 *   swapped when bit 2 of (r % 8) is set:  byte (q % 32) lands at
 *   (((q % 32) / 16) ^ ((r % 8) >> 2)) * 16 + (q % 16).
 * Rows r >= rows (up to RG*8) and K positions q >= k (up to ceil(k/32)*32) hold zeros.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include "ggemm.h"

#ifdef __cplusplus
extern "C" {
#endif

#define GGEMM_IMG_GROUP_ROWS 8
#define GGEMM_IMG_KSTEP 32
#define GGEMM_IMG_ATOM 256

/* Bytes of one residue plane of a rows x k operand. */
static inline size_t ggemm_img_plane_bytes(int rows, int k) {
  const size_t rg = ((size_t)rows + 7) / 8, ks = ((size_t)k + 31) / 32;
  return rg * ks * GGEMM_IMG_ATOM;
}
/* Byte offset of element (r, q) inside a plane of an operand with `rows` rows. */
static inline size_t ggemm_img_offset(int rows, int r, int q) {
  const size_t rg = ((size_t)rows + 7) / 8;
  const int rr = r & 7, qq = q & 31;
  return ((size_t)(q >> 5) * rg + (size_t)(r >> 3)) * GGEMM_IMG_ATOM + (size_t)rr * 32 +
         (size_t)(((qq >> 4) ^ (rr >> 2)) * 16 + (qq & 15));
}

/* One operand of one problem for prep.  kind 0: the rows of a column-major A (element (r, q)
 * at X[r + q*ld]); kind 1: the columns of a column-major B (element (r, q) at X[q + r*ld]).
 * kind | GGEMM_PREP_QSCALED (extension): residue plane l holds the symmetric residue of
 * q_l x instead of x, q_l = ((P_N / p_l)^-1 mod p_l) the CRT factor of plane l, so that the
 * residue GEMM's digit epilogue skips one modular product (GGEMM_PRODUCTS_DIGITS_QSCALED).
 * img: N+1 planes (N residue planes, then the abs plane) at stride plane_bytes.
 * ws: 4*rows int32 {shift | abs shift | ||dX_r|| (float bits) | ||X'_r|| (float bits)}. */
typedef struct {
  const double* X;
  long long ld;
  int rows, k, N, kind;
  int8_t* img;
  long long plane_bytes;
  int32_t* ws;
} ggemm_prep_desc_t;

/* Products handed from the residue GEMM to the reconstruct (`layout` below).
 * GGEMM_PRODUCTS_INT32: N+1 planes of m*n int32 products C_l = A_l B_l^T, column-major
 *   (ld = m), at stride c_plane int32 elements.
 * GGEMM_PRODUCTS_DIGITS: for residue plane l < N the CRT digit y_l = (C_l mod p_l) q_l mod p_l
 *   (the value the reconstruct derives from C_l first) as one byte; for the abs plane l = N
 *   the int32 product.  Both in 16-byte records of consecutive columns of one row (16 digits,
 *   or 4 int32 products), the records of one column block stored row after row, c_plane in
 *   bytes:
 *     digit y_l(i, j):   byte  at base + l*c_plane + ((j/16)*m + i)*16 + j%16
 *     abs product (i, j): int32 at ((int32_t*)(base + N*c_plane))[((j/4)*m + i)*4 + j%4]
 *   c_plane >= ggemm_digit_plane_bytes(m, n) and a multiple of 16; the abs plane takes
 *   4 * ggemm_digit_plane_bytes(m, n) bytes.  Columns j >= n, up to the next multiple of 32,
 *   are padding (the GEMM writes whole 32-column chunks).
 *   N + 4 bytes per entry instead of 4 (N + 1). */
#define GGEMM_PRODUCTS_INT32 0
#define GGEMM_PRODUCTS_DIGITS 1
/* Residue GEMM layout only (extension): the digit layout, computed from products of which one
 * operand's images were prepared with GGEMM_PREP_QSCALED (the digits are C'_l mod p_l; the
 * output is byte-identical to GGEMM_PRODUCTS_DIGITS from unscaled images). */
#define GGEMM_PRODUCTS_DIGITS_QSCALED 2
#define GGEMM_PREP_QSCALED 2

/* Bytes of one digit plane of an m x n problem (256-byte multiple). */
static inline size_t ggemm_digit_plane_bytes(int m, int n) {
  const size_t b = (((size_t)n + 31) / 32) * (size_t)m * 32;
  return (b + 255) / 256 * 256;
}

/* One problem of the residue GEMM: for every plane l < planes the exact int32 product
 * C_l(i, j) = sum_q A_l(i, q) * B_l(j, q), A/B in the image layout above (A: m rows, B: n
 * rows, depth k), stored in `layout` at C (int32 layout: C[l*c_plane + i + j*m]).
 * N is the number of moduli (digit layout only; planes <= N + 1 there). */
typedef struct {
  const int8_t* A;
  const int8_t* B;
  int32_t* C;
  long long a_plane, b_plane, c_plane; /* bytes, bytes, int32 elements (digit layout: bytes) */
  int m, n, k, planes;
  int N, layout;
} ggemm_gemm_desc_t;

/* One problem of the reconstruct.  C32: the N+1 products in `layout`, c_plane as above;
 * rs / cs: prep workspaces of A (4m) and B (4n). */
typedef struct {
  int m, n, k, N;
  const double* A; long long lda;
  const double* B; long long ldb;
  double* C; long long ldc;
  double alpha, beta;
  const int32_t* C32; long long c_plane;
  const int32_t* rs;
  const int32_t* cs;
  int layout, reserved;
} ggemm_recon_desc_t;

#define GGEMM_STAGE_REPAIR_OFF 0
#define GGEMM_STAGE_REPAIR_COUNT 1
#define GGEMM_STAGE_REPAIR_ON 2

/* Device scratch a stage call needs for num descriptors (caller-allocated, device memory). */
size_t ggemm_stage_scratch_bytes(int num);
/* Device counters: 4 x uint64 {nonfinite vectors, uncertified, repaired, safety fallback}
 * followed by a uint32 status word (0 = ok); 64 bytes, caller-allocated and zeroed.  Bytes
 * 40-47 are scratch of ggemm_stage_recon (a work ticket it zeroes before each launch). */
#define GGEMM_STAGE_COUNTER_BYTES 64

/* Each enqueues its kernel on `s` (none when there is no work): the GEMM one launch, prep and
 * reconstruct one launch per class of moduli counts present (N = 14, 15, 16 and the others are
 * compiled separately).  Descriptors are HOST arrays; they are copied into `scratch` first.
 * Returns GGEMM_OK or GGEMM_ERR_*. */
int ggemm_stage_prep(const ggemm_prep_desc_t* descs, int num, void* scratch,
                     size_t scratch_bytes, void* counters, cudaStream_t s);
int ggemm_stage_gemm(const ggemm_gemm_desc_t* descs, int num, void* scratch,
                     size_t scratch_bytes, void* counters, cudaStream_t s);
int ggemm_stage_recon(const ggemm_recon_desc_t* descs, int num, int repair_mode, void* scratch,
                      size_t scratch_bytes, void* counters, cudaStream_t s);

/* Bounded-wait probe (no counterpart in the reference, whose kernels never wait on one
 * another): one block waits on an mbarrier that nothing arrives on, through the same bounded
 * wait the pipeline kernels use, gives up after wait_ns (clamped to [1 us, 1 s]) and sets the
 * status word of `counters` to 3 if it was 0.  counters == NULL targets the counter block of the
 * allocation-free entry point (ggemm_dgemm_noalloc, ggemm_ext.h) on the current device.  It lets
 * a test make a wait run out and check that the host reads the status and the context stays
 * usable, without a fault.  Returns GGEMM_OK or GGEMM_ERR_CUDA. */
int ggemm_stage_wait_probe(void* counters, long long wait_ns, cudaStream_t s);

/* Host-only planner seam (replaces ggemm_plan, src/planner.cpp:281-330): plans num problems
 * for the given path, writing route / moduli / tile class (always 0) per problem (route codes of
 * the reference's ggemm_route_t, src/planner.h:7-17).  Rule routes and moduli counts are the
 * reference's; AUTO's cost decision uses this library's calibrated model (calib/b200.json),
 * whose native DGEMM rate, residue-GEMM rate and stage bandwidth are replaced by fp64_flops,
 * int8_ops and mem_bw when those are > 0; tiny_mnk >= 0 replaces the TINY threshold.
 * rho_budget <= 0 uses GGEMM_RHO_BUDGET or 16.  Returns GGEMM_OK or GGEMM_ERR_*. */
int ggemm_stage_plan(const ggemm_problem_t* problems, int num, const ggemm_config_t* cfg,
                     int path, int num_sms, double fp64_flops, double int8_ops, double mem_bw,
                     double tiny_mnk, double rho_budget, int* route, int* num_moduli,
                     int* tile_cfg);
/* Host-only operand-reuse seam (replaces build_operand_reuse, src/operand_reuse.cpp:47-141).
 * nmod[g] <= 0 marks a problem as not emulated; policy 0 = EXACT_N, 1 = PROMOTE.
 * out[0..2] = {unique A, unique B, promoted}, then 7 arrays of num ints: ua_rep, ua_nmod,
 * ub_rep, ub_nmod (unused tails -1 / 0), prob_a, prob_b, eff_nmod. */
int ggemm_stage_reuse(const ggemm_problem_t* problems, int num, const int* nmod, int policy,
                      int* out);

/* Host-only: copies the CRT constant tables (same content and layout as the reference's
 * oz2_crt_tables, src/moduli.h:43-58) into out (up to `bytes`); returns their size, 0 on a
 * table-construction failure.  ggemm_stage_error_bound is the a-priori bound of
 * src/ozaki2_numerics.cu:639-650. */
size_t ggemm_stage_crt_tables(void* out, size_t bytes);
double ggemm_stage_error_bound(int k, int num_moduli);

/* Number of CUDA devices this library can see (0 on a machine without a GPU). */
int ggemm_device_count(void);
/* Version string of this library. */
const char* ggemm_version(void);

#ifdef __cplusplus
}
#endif
