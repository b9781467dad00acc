/* ggemm_graph.h -- plan / execute for repeated calls with frozen shapes (CUDA Graph).
 *
 * Same entry points and contract as the reference's src/ggemm_graph.h:30-47:
 *   ggemm_make_plan / _ex     planning + descriptor upload + stream capture of the launch
 *                             sequence into an instantiated graph (allocates, synchronizes:
 *                             call outside timed regions)      (src/ggemm_graph.cu:259-306)
 *   ggemm_execute_plan        one cudaGraphLaunch, ordered against the handle's stream
 *                                                              (src/ggemm_graph.cu:309-333)
 *   ggemm_plan_update_pointers  new A/B/C device pointers for the same shapes, one small
 *                             H2D of the plan's descriptors    (src/ggemm_graph.cu:335-386)
 *   ggemm_plan_get_stats / ggemm_destroy_plan                  (src/ggemm_graph.cu:388-394)
 * Plans share the handle's scratch and must be destroyed before the handle.
 */
#pragma once
#include "ggemm.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggemm_plan_s* ggemm_plan_t;

/* path: GGEMM_PATH_EMU_GROUPED or GGEMM_PATH_AUTO.  NULL on error (*err = GGEMM_ERR_*). */
ggemm_plan_t ggemm_make_plan(ggemm_handle_t h, ggemm_path_t path, const ggemm_config_t* cfg,
                             const ggemm_problem_t* problems, int num_problems);
ggemm_plan_t ggemm_make_plan_ex(ggemm_handle_t h, ggemm_path_t path, const ggemm_config_t* cfg,
                                const ggemm_problem_t* problems, int num_problems, int* err);
int ggemm_execute_plan(ggemm_plan_t plan, cudaStream_t stream);
/* A/B/C: HOST arrays of num_problems device pointers (NULL array = keep). */
int ggemm_plan_update_pointers(ggemm_plan_t plan, const double* const* A, const double* const* B,
                               double* const* C);
int ggemm_plan_get_stats(ggemm_plan_t plan, ggemm_stats_t* stats);
void ggemm_destroy_plan(ggemm_plan_t plan);

#ifdef __cplusplus
}
#endif
