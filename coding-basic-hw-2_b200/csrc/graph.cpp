// graph.cpp -- plan / execute (include/ggemm_graph.h).
//
// A plan freezes the shapes of a group: the descriptors are built once into plan-owned
// memory (pinned mirror + device blob), the exact launch sequence of a direct call is captured
// into a CUDA graph and instantiated.  Executing runs the same kernels on the same descriptor
// contents, so results equal a direct call bit for bit (reference contract,
// src/ggemm_graph.h:1-18).  Pointers of the problems live in the device descriptors, not in
// kernel parameters, so update_pointers rewrites and re-uploads the descriptors; only a lone
// native fallback problem (plain cublasDgemm, pointers are kernel arguments) forces a
// re-capture and an in-place graph update.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "ggemm_graph.h"
#include "internal.hpp"

using namespace g2;

struct ggemm_plan_s {
  ggemm_handle_t h = nullptr;
  ggemm_path_t path = GGEMM_PATH_EMU_GROUPED;
  ggemm_config_t cfg{};
  int repair = 0;
  std::vector<ggemm_problem_t> probs;
  EmuCall call;
  std::vector<Chunk> chunks;
  std::vector<int> emu, nat;
  std::vector<PlanEntry> plan;
  NativeGroups ngroups;
  char* h_blob = nullptr;
  char* d_blob = nullptr;
  size_t blob_cap = 0;
  cudaStream_t cap = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaEvent_t ev_h = nullptr, ev_p = nullptr, ev_upd = nullptr;
  ggemm_stats_t st{};
};

static void free_plan(ggemm_plan_t p) {
  if (!p) return;
  if (p->h) cudaStreamSynchronize(p->h->stream);
  if (p->exec) cudaGraphExecDestroy(p->exec);
  if (p->graph) cudaGraphDestroy(p->graph);
  if (p->cap) cudaStreamDestroy(p->cap);
  if (p->ev_upd) {
    cudaEventSynchronize(p->ev_upd);
    cudaEventDestroy(p->ev_upd);
  }
  if (p->ev_h) cudaEventDestroy(p->ev_h);
  if (p->ev_p) cudaEventDestroy(p->ev_p);
  cudaFree(p->d_blob);
  if (p->h_blob) cudaFreeHost(p->h_blob);
  delete p;
}

// Builds the plan's descriptors into its own host blob and snapshots the handle scratch the
// launches need (chunks, partition, plan entries, native groups).
static int build_descriptors(ggemm_plan_t p) {
  ggemm_handle_t h = p->h;
  const int r = build_emu_call(h, p->path, &p->cfg, p->probs.data(), (int)p->probs.size(),
                               p->h_blob, p->d_blob, &p->call);
  if (r) return r;
  p->chunks.assign(h->chunks.begin(), h->chunks.end());
  p->emu.assign(h->emu.begin(), h->emu.begin() + p->call.ne);
  p->nat.assign(h->nat.begin(), h->nat.begin() + p->call.nn);
  p->plan.assign(h->plan.begin(), h->plan.begin() + p->probs.size());
  p->ngroups = h->ngroups;
  return GGEMM_OK;
}

// Enqueues the plan's launches on s (only ever called while s is captured).
static int enqueue(ggemm_plan_t p, cudaStream_t s, int* launches) {
  ggemm_handle_t h = p->h;
  // the shared enqueue helpers read the handle's scratch: restore the plan's snapshot
  h->chunks.assign(p->chunks.begin(), p->chunks.end());
  std::copy(p->emu.begin(), p->emu.end(), h->emu.begin());
  std::copy(p->nat.begin(), p->nat.end(), h->nat.begin());
  std::copy(p->plan.begin(), p->plan.end(), h->plan.begin());
  h->ngroups = p->ngroups;
  int r = enqueue_emu_call(h, p->call, p->probs.data(), p->d_blob, p->repair, false, false, s,
                           launches);
  if (!r && p->call.nn > 0)
    r = enqueue_native(h, p->probs.data(), h->nat.data(), p->call.nn, p->call.nn >= 2,
                       p->call.nat_groups, p->d_blob + p->call.off_nat_ptrs, s, launches);
  return r;
}

static int capture(ggemm_plan_t p, cudaGraph_t* out, int* launches) {
  ggemm_handle_t h = p->h;
  *out = nullptr;
  if (cudaStreamBeginCapture(p->cap, cudaStreamCaptureModeRelaxed) != cudaSuccess)
    return GGEMM_ERR_CUDA;
  int r = enqueue(p, p->cap, launches);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(p->cap, &g);
  // cuBLAS goes back to the handle's stream and fixed workspace
  if (cublasSetStream(h->cublas, h->stream) != CUBLAS_STATUS_SUCCESS ||
      cublasSetWorkspace(h->cublas, h->cublas_ws, h->cublas_ws_bytes) != CUBLAS_STATUS_SUCCESS)
    r = r ? r : GGEMM_ERR_CUBLAS;
  if (!r && ce != cudaSuccess) r = GGEMM_ERR_CUDA;
  if (r) {
    if (g) cudaGraphDestroy(g);
    return r;
  }
  *out = g;
  return GGEMM_OK;
}

extern "C" ggemm_plan_t ggemm_make_plan_ex(ggemm_handle_t h, ggemm_path_t path,
                                           const ggemm_config_t* cfg,
                                           const ggemm_problem_t* problems, int num, int* err) {
  int dummy;
  int& e = err ? *err : dummy;
  e = GGEMM_ERR_INVALID;
  if (!h || (path != GGEMM_PATH_EMU_GROUPED && path != GGEMM_PATH_AUTO)) return nullptr;
  if ((e = validate_call(h, problems, num))) return nullptr;
  static const ggemm_config_t kDefault = {0, 1e-15, 1, 0};
  if (!cfg) cfg = &kDefault;
  if (cfg->num_moduli < 0 || cfg->num_moduli == 1 || cfg->num_moduli > GGEMM_MAX_MODULI ||
      stage_repair_mode(path, cfg) < 0) {
    e = GGEMM_ERR_INVALID;
    return nullptr;
  }
  if (cudaSetDevice(h->device) != cudaSuccess) {
    e = GGEMM_ERR_CUDA;
    return nullptr;
  }
  ggemm_plan_t p = new (std::nothrow) ggemm_plan_s();
  if (!p) {
    e = GGEMM_ERR_ALLOC;
    return nullptr;
  }
  p->h = h;
  p->path = path;
  p->cfg = *cfg;
  p->repair = stage_repair_mode(path, cfg);
  try {
    p->probs.assign(problems, problems + num);
  } catch (...) {
    free_plan(p);
    e = GGEMM_ERR_ALLOC;
    return nullptr;
  }
  p->blob_cap = h->blob_cap;
  if (cudaMalloc(&p->d_blob, p->blob_cap) != cudaSuccess ||
      cudaHostAlloc(&p->h_blob, p->blob_cap, cudaHostAllocDefault) != cudaSuccess) {
    free_plan(p);
    e = GGEMM_ERR_ALLOC;
    return nullptr;
  }
  if (cudaStreamCreateWithFlags(&p->cap, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&p->ev_h, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&p->ev_p, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&p->ev_upd, cudaEventDisableTiming) != cudaSuccess) {
    free_plan(p);
    e = GGEMM_ERR_CUDA;
    return nullptr;
  }
  if ((e = build_descriptors(p))) {
    free_plan(p);
    return nullptr;
  }
  ggemm_stats_t& st = p->st;
  st.num_problems = num;
  for (int i = 0; i < p->call.nn; ++i) st.num_fallback += route_is_fallback(p->plan[p->nat[i]].route);
  st.moduli_min = p->call.nmin;
  st.moduli_max = p->call.nmax;
  st.num_unique_A = st.num_unique_B = p->call.ne;
  st.num_repaired = st.num_uncertified = st.num_safety_fallback = -1;
  if (p->call.blob_bytes &&
      cudaMemcpyAsync(p->d_blob, p->h_blob, p->call.blob_bytes, cudaMemcpyHostToDevice,
                      h->stream) != cudaSuccess) {
    free_plan(p);
    e = GGEMM_ERR_CUDA;
    return nullptr;
  }
  cudaEventRecord(p->ev_upd, h->stream);
  if (cudaStreamSynchronize(h->stream) != cudaSuccess) {
    free_plan(p);
    e = GGEMM_ERR_CUDA;
    return nullptr;
  }
  if (p->call.ne == 0 && p->call.nn == 0) {
    e = GGEMM_OK;
    return p;
  }
  int launches = 0;
  if ((e = capture(p, &p->graph, &launches))) {
    free_plan(p);
    return nullptr;
  }
  st.kernel_launches = launches;
  if (cudaGraphInstantiate(&p->exec, p->graph, 0) != cudaSuccess ||
      cudaGraphUpload(p->exec, h->stream) != cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess) {
    free_plan(p);
    e = GGEMM_ERR_CUDA;
    return nullptr;
  }
  e = GGEMM_OK;
  return p;
}

extern "C" ggemm_plan_t ggemm_make_plan(ggemm_handle_t h, ggemm_path_t path,
                                        const ggemm_config_t* cfg,
                                        const ggemm_problem_t* problems, int num) {
  return ggemm_make_plan_ex(h, path, cfg, problems, num, nullptr);
}

extern "C" int ggemm_execute_plan(ggemm_plan_t p, cudaStream_t stream) {
  if (!p) return GGEMM_ERR_INVALID;
  if (!p->exec) return GGEMM_OK;
  ggemm_handle_t h = p->h;
  cudaStream_t hs = h->stream;
  const bool counters = h->stats_repair && p->call.ne > 0;
  if (stream != hs) {
    // join with the handle's stream on both sides: the workspace is shared
    if (cudaEventRecord(p->ev_h, hs) != cudaSuccess ||
        cudaStreamWaitEvent(stream, p->ev_h, 0) != cudaSuccess)
      return GGEMM_ERR_CUDA;
  }
  if (counters && cudaMemsetAsync(h->counters, 0, sizeof(DevCounters), stream) != cudaSuccess)
    return GGEMM_ERR_CUDA;
  if (cudaGraphLaunch(p->exec, stream) != cudaSuccess) return GGEMM_ERR_CUDA;
  if (stream != hs) {
    if (cudaEventRecord(p->ev_p, stream) != cudaSuccess ||
        cudaStreamWaitEvent(hs, p->ev_p, 0) != cudaSuccess)
      return GGEMM_ERR_CUDA;
  }
  if (counters) {
    DevCounters c{};
    if (cudaMemcpyAsync(&c, h->counters, sizeof c, cudaMemcpyDeviceToHost, stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return GGEMM_ERR_CUDA;
    if (c.status != kStatusOk) return GGEMM_ERR_I8GEMM;
    p->st.num_repaired = (long long)c.repaired;
    p->st.num_uncertified = (long long)c.uncertified;
    p->st.num_safety_fallback = (long long)c.safety;
  }
  return GGEMM_OK;
}

extern "C" int ggemm_plan_update_pointers(ggemm_plan_t p, const double* const* A,
                                          const double* const* B, double* const* C) {
  if (!p) return GGEMM_ERR_INVALID;
  const int num = (int)p->probs.size();
  for (int g = 0; g < num; ++g) {
    const ggemm_problem_t& q = p->probs[g];
    if (q.m == 0 || q.n == 0) continue;
    if (C && !C[g]) return GGEMM_ERR_INVALID;
    if (q.k > 0 && ((A && !A[g]) || (B && !B[g]))) return GGEMM_ERR_INVALID;
  }
  for (int g = 0; g < num; ++g) {
    if (A) p->probs[g].A = A[g];
    if (B) p->probs[g].B = B[g];
    if (C) p->probs[g].C = C[g];
  }
  ggemm_handle_t h = p->h;
  if (cudaSetDevice(h->device) != cudaSuccess) return GGEMM_ERR_CUDA;
  // the previous patch copy must have consumed the pinned mirror before it is rewritten
  if (cudaEventSynchronize(p->ev_upd) != cudaSuccess) return GGEMM_ERR_CUDA;
  EmuCall before = p->call;
  int r = build_descriptors(p);  // same shapes: same layout, new pointer values
  if (r) return r;
  if (p->call.blob_bytes != before.blob_bytes) return GGEMM_ERR_INVALID;
  if (p->call.blob_bytes &&
      cudaMemcpyAsync(p->d_blob, p->h_blob, p->call.blob_bytes, cudaMemcpyHostToDevice,
                      h->stream) != cudaSuccess)
    return GGEMM_ERR_CUDA;
  if (cudaEventRecord(p->ev_upd, h->stream) != cudaSuccess) return GGEMM_ERR_CUDA;
  if (p->call.nn == 1 && p->exec) {  // pointers are cuBLAS kernel arguments: re-capture
    cudaGraph_t g = nullptr;
    int launches = 0;
    if ((r = capture(p, &g, &launches))) return r;
    cudaGraphExecUpdateResultInfo info;
    if (cudaGraphExecUpdate(p->exec, g, &info) != cudaSuccess) {
      cudaGetLastError();
      if (cudaStreamSynchronize(h->stream) != cudaSuccess) {
        cudaGraphDestroy(g);
        return GGEMM_ERR_CUDA;
      }
      cudaGraphExecDestroy(p->exec);
      p->exec = nullptr;
      if (cudaGraphInstantiate(&p->exec, g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        return GGEMM_ERR_CUDA;
      }
    }
    cudaGraphDestroy(p->graph);
    p->graph = g;
  }
  return GGEMM_OK;
}

extern "C" int ggemm_plan_get_stats(ggemm_plan_t p, ggemm_stats_t* st) {
  if (!p || !st) return GGEMM_ERR_INVALID;
  *st = p->st;
  return GGEMM_OK;
}

extern "C" void ggemm_destroy_plan(ggemm_plan_t p) { free_plan(p); }
