/* oz2_oracle.h -- CPU restatement of the Ozaki-II (CRT, INT8) grouped FP64 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is compared
 * against; it is never linked into, called by or shipped with the product library.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg load it.
 *
 * What it restates (file:line are in the reference project moneychen168/Coding-Basic-HW-2):
 *   - CRT constant tables                       src/moduli.h:124-181
 *   - a-priori error bound, N selection         src/ozaki2_numerics.cu:639-673
 *   - prep (shift, trunc, residues, abs plane,  src/ozaki2_numerics.cu:112-231 (element math),
 *     row/column workspace), with the SAME        :263-364 (A rows: 8 chains k = t mod 8,
 *     floating-point reduction orders               sequential combine),
 *                                                 :368-441 (B cols: 32 lane chains + xor butterfly)
 *   - exact INT8 x INT8 -> INT32 GEMM           src/int8_grouped_gemm.h:4-10
 *   - CRT reconstruct / certificate / repair    src/ozaki2_numerics.cu:445-586
 *   - the naive FP64 triple-loop GEMM used as    tests/test_numerics_standalone.cu:292-299
 *     the reference's host-side FP64 path
 *
 * Parity is pinned by tests/: against the reference's own host code compiled into oracle/_ref
 * (tables, bounds, N choice), against golden vectors produced by the reference's kernels, and
 * against the published tables (log2P, choose(k, 1e-15)).
 */
#ifndef OZ2_ORACLE_H
#define OZ2_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OZO_MAX_MODULI 20
#define OZO_POW2_TABLE 128
#define OZO_S2_BITS 18
#define OZO_SHIFT_NONFINITE (-2147483647 - 1)
#define OZO_SHIFT_ZERO (-2147483647)
#define OZO_REPAIR_OFF 0
#define OZO_REPAIR_COUNT 1
#define OZO_REPAIR_ON 2

/* Same content and field order as the reference's oz2_crt_tables (src/moduli.h:43-58). */
typedef struct {
  int32_t p[OZO_MAX_MODULI];
  uint32_t magic[OZO_MAX_MODULI];
  uint8_t pow2[OZO_MAX_MODULI][OZO_POW2_TABLE];
  uint64_t s1[OZO_MAX_MODULI + 1][OZO_MAX_MODULI];
  uint32_t s2[OZO_MAX_MODULI + 1][OZO_MAX_MODULI];
  int32_t qinv[OZO_MAX_MODULI + 1][OZO_MAX_MODULI];
  int64_t P1[OZO_MAX_MODULI + 1];
  double P2[OZO_MAX_MODULI + 1];
  double inv_Pu[OZO_MAX_MODULI + 1];
  int32_t log2_u1[OZO_MAX_MODULI + 1];
  double T[OZO_MAX_MODULI + 1];
  double log2P[OZO_MAX_MODULI + 1];
} ozo_tables;

size_t ozo_tables_size(void);
/* 0 on success. */
int ozo_build_tables(ozo_tables* t);
double ozo_error_bound(int k, int num_moduli);
int ozo_choose_num_moduli(int k, double target_rel_err);
int ozo_choose_num_moduli_cw(int k, double rho_budget);

/* Prep of the rows of A (column-major m x k, leading dim lda), reduction order of the
 * reference's A blocks.  out: planes [(N+1)][m][kp] int8 (row-major, K contiguous), plane
 * stride m*kp; columns k..kp-1 are zero.  ws: 4*m int32 {s_i | sig_i | ||dA_i|| | ||A'_i||}.
 * nonfinite: incremented once per row containing NaN/Inf (may be NULL). */
void ozo_prep_rows(const double* A, int m, int k, int lda, int N, int kp, int8_t* out,
                   int32_t* ws, uint64_t* nonfinite);
/* Prep of the columns of B (column-major k x n, leading dim ldb), reduction order of the
 * reference's B warps.  out: planes [(N+1)][n][kp] int8; ws: 4*n int32. */
void ozo_prep_cols(const double* B, int n, int k, int ldb, int N, int kp, int8_t* out,
                   int32_t* ws, uint64_t* nonfinite);

/* C[i + j*m] = sum_k A8[i*kp + k] * B8[j*kp + k]; returns 0, or 1 if a sum leaves int32. */
int ozo_i8_gemm(const int8_t* A8, const int8_t* B8, int m, int n, int kp, int32_t* C);

/* CRT reconstruct + alpha/beta + certificate + repair for one problem.
 * C32: planes [(N+1)][m*n] (column-major, ld = m).  rs/cs: prep workspaces.
 * A, B: the FP64 inputs (read only for repaired / non-finite entries).
 * C: in/out, column-major ldc.  cnt[4] += {nonfinite(unused here), uncertified, repaired,
 * safety_fallback}.  mode: OZO_REPAIR_*. */
void ozo_reconstruct(int m, int n, int k, int N, double alpha, double beta, const double* A,
                     int lda, const double* B, int ldb, double* C, int ldc, const int32_t* C32,
                     const int32_t* rs, const int32_t* cs, int mode, uint64_t* cnt);

/* Debug view of the CRT integers of one entry: S1 (exact), S2 (exact), Q, xr = X / u1. */
void ozo_crt_entry(int N, const int32_t* c_planes, size_t plane_stride, uint64_t* S1,
                   uint32_t* S2, double* Q, double* xr);

/* Whole pipeline for one problem (prep rows, prep cols, GEMM of N+1 planes, reconstruct).
 * Returns 0, or nonzero on an int32 overflow in the GEMM.  Scratch is allocated inside. */
int ozo_emulated_dgemm(int m, int n, int k, int N, double alpha, double beta, const double* A,
                       int lda, const double* B, int ldb, double* C, int ldc, int mode,
                       uint64_t* cnt);

/* Naive FP64 triple loop, column-major, sequential k (the reference's host FP64 path).
 * C = alpha*A*B + beta*C.  threads <= 0: one POSIX thread per online CPU.  Columns [j0, j1) only. */
void ozo_dgemm_naive(int m, int n, int k, double alpha, const double* A, int lda,
                     const double* B, int ldb, double beta, double* C, int ldc, int j0, int j1,
                     int threads);
int ozo_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
