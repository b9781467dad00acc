/* ggemm.h -- grouped FP64 GEMM emulated on B200 INT8 tensor cores (Ozaki scheme II, CRT).
 *
 * Drop-in C ABI of the reference library's public header (include/ggemm.h of
 * moneychen168/Coding-Basic-HW-2): identical struct layouts, enum values, macros and entry
 * points, so a caller compiled against the reference header links against this library
 * unchanged.  Column-major, no transpose:  C_g = alpha_g * A_g (m x k) * B_g (k x n) + beta_g C_g.
 *
 * Entry points and the reference interface each one replaces:
 *   ggemm_create          include/ggemm.h:71-72   (src/ggemm.cu:308-311)
 *   ggemm_create_ex       include/ggemm.h:78-80   (src/ggemm.cu:228-341)
 *   ggemm_destroy         include/ggemm.h:81      (src/ggemm.cu:287-306)
 *   ggemm_grouped_dgemm   include/ggemm.h:85-86   (src/ggemm.cu:698-741)
 * Return codes (the reference keeps them in src/internal.h:65-75; they are public here).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int m, n, k;
  const double* A; int lda;   /* device pointers */
  const double* B; int ldb;
  double*       C; int ldc;
  double alpha, beta;
} ggemm_problem_t;

typedef enum {
  GGEMM_PATH_NATIVE_LOOP = 0,        /* cuBLAS DGEMM per problem (native FP64 baseline)     */
  GGEMM_PATH_NATIVE_GROUPED = 1,     /* cublasDgemmGroupedBatched (native FP64 baseline)    */
  GGEMM_PATH_EMU_LOOP = 2,           /* emulation, one prep/GEMM-per-plane/recon per problem */
  GGEMM_PATH_EMU_GROUPED = 3,        /* emulation of the whole group in a fixed launch count */
  GGEMM_PATH_AUTO = 4,               /* EMU_GROUPED + planner (N per problem, fallback)      */
  GGEMM_PATH_EMU_GROUPED_REUSE = 5,  /* EMU_GROUPED with prep once per unique A / B operand  */
  GGEMM_PATH_EMU_LOOP_BATCHED = 6    /* emulation, prep / one GEMM over planes / recon each  */
} ggemm_path_t;

typedef struct {
  int num_moduli;        /* 0 = adaptive per problem; else fixed N in [2, GGEMM_MAX_MODULI]  */
  double target_rel_err; /* adaptive target (normwise), default 1e-15                         */
  int allow_fallback;    /* 1 = route unsafe / unprofitable problems to native FP64           */
  int repair_mode;       /* GGEMM_REPAIR_*, 0 = path default                                  */
} ggemm_config_t;

#define GGEMM_MAX_MODULI 20

#define GGEMM_REPAIR_DEFAULT 0   /* EMU_* paths: COUNT; AUTO: ON                    */
#define GGEMM_REPAIR_OFF     1   /* no certificate                                   */
#define GGEMM_REPAIR_COUNT   2   /* certificate evaluated, failures counted          */
#define GGEMM_REPAIR_ON      3   /* failures recomputed as FP64 dot products         */

typedef struct {
  int num_problems;
  int num_fallback;       /* problems routed to native FP64 for precision / profit reasons */
  int kernel_launches;    /* launches issued by the last call                              */
  int moduli_min, moduli_max;
  int reuse_enabled;
  int num_unique_A;
  int num_unique_B;
  int num_promoted;
  /* Per-handle device counters (read only with env GGEMM_STATS_REPAIR=1, which synchronizes
   * the handle's stream); -1 when not measured. */
  long long num_repaired;
  long long num_uncertified;
  long long num_safety_fallback;
} ggemm_stats_t;

typedef struct ggemm_handle_s* ggemm_handle_t;

enum {
  GGEMM_OK = 0,
  GGEMM_ERR_INVALID = 1,    /* bad arguments / null handle / too many problems              */
  GGEMM_ERR_WORKSPACE = 2,  /* the call exceeds the workspace sized at create time          */
  GGEMM_ERR_UNSAFE = 3,     /* k > GGEMM_MAX_K_EXACT (or target unreachable), no fallback   */
  GGEMM_ERR_CUDA = 4,
  GGEMM_ERR_CUBLAS = 5,
  GGEMM_ERR_NUMERICS = 6,   /* prep / reconstruct launch or device status failure          */
  GGEMM_ERR_I8GEMM = 7,     /* residue GEMM launch or device status failure                */
  GGEMM_ERR_ALLOC = 8       /* only from ggemm_create / plan creation                       */
};

/* All device and pinned workspace is allocated here; calls never allocate.
 * max_problems / max_total_*_elems bound every later call on this handle. */
int  ggemm_create(ggemm_handle_t* h, int max_problems, size_t max_total_A_elems,
                  size_t max_total_B_elems, size_t max_total_C_elems, cudaStream_t stream);
/* As ggemm_create, with min_k = smallest k of any emulated problem (ggemm_create uses 32):
 * the residue workspace is sized for the K padding of such k. */
int  ggemm_create_ex(ggemm_handle_t* h, int max_problems, size_t max_total_A_elems,
                     size_t max_total_B_elems, size_t max_total_C_elems, cudaStream_t stream,
                     int min_k);
void ggemm_destroy(ggemm_handle_t h);

/* problems: HOST array of descriptors whose pointers are device pointers on the handle's
 * device.  Work is enqueued on the handle's stream.  0 on success, GGEMM_ERR_* otherwise. */
int ggemm_grouped_dgemm(ggemm_handle_t h, ggemm_path_t path, const ggemm_config_t* cfg,
                        const ggemm_problem_t* problems, int num_problems, ggemm_stats_t* stats);

#ifdef __cplusplus
}
#endif
