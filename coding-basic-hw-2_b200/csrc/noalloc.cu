// noalloc.cu -- ggemm_dgemm_noalloc (include/ggemm_ext.h): one emulated FP64 GEMM whose scratch
// lives in a fixed device array compiled into this library, for callers that cannot allocate
// device memory.  Those are callers that own no CUDA allocator (code running inside another
// runtime's device-memory pool, plugins of hosts that forbid cudaMalloc, code paths that must
// not grow the footprint or synchronize the way cudaMalloc / cudaFree can).  They pass inputs
// and outputs; everything else this call needs -- prep workspace, residue images, int32
// products, descriptors, counters -- comes from g_noalloc_scratch below.
//
// Runs the same three kernels as ggemm_grouped_dgemm (prep, tcgen05 residue GEMM,
// reconstruct), preceded by a one-thread set-up kernel that writes the descriptors (passed as a
// kernel argument) into the array and clears the counters.  Nothing here calls cudaMalloc,
// cudaFree, cudaMemcpy or any allocating library routine.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <mutex>

#include "ggemm_ext.h"
#include "internal.hpp"

namespace g2 {

// The scratch: 64 MiB per device.  It is part of this library's device image, so every GPU
// that loads the library holds it until the process exits.
constexpr size_t kNoAllocBytes = 64ull << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

constexpr size_t kOffCounters = 0;
constexpr size_t kOffDescs = 256;
constexpr size_t kOffData = 4096;

struct NoAllocDescs {
  ggemm_prep_desc_t prep[2];
  int prep_prefix[3];
  GemmJob job;
  long long job_prefix[2];
  ggemm_recon_desc_t recon;
  long long recon_prefix[2];
};
static_assert(kOffDescs + sizeof(NoAllocDescs) <= kOffData, "descriptor block too large");

// Device code names the array directly: descriptors in, counters cleared (the array keeps the
// previous call's contents).
__global__ void noalloc_setup_kernel(NoAllocDescs d) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *reinterpret_cast<NoAllocDescs*>(g_noalloc_scratch + kOffDescs) = d;
    DevCounters* c = reinterpret_cast<DevCounters*>(g_noalloc_scratch + kOffCounters);
    c->nonfinite = c->uncertified = c->repaired = c->safety = 0;
    c->status = 0;
  }
}

// C = beta C, not reading C when beta == 0: what ggemm_grouped_dgemm computes for alpha == 0 or
// k == 0 (its native route).  Block 0 also clears the counters, so the status query reports this
// call.
__global__ void noalloc_scale_kernel(double* __restrict__ C, long long ldc, int m, int n,
                                     double beta) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    DevCounters* c = reinterpret_cast<DevCounters*>(g_noalloc_scratch + kOffCounters);
    c->nonfinite = c->uncertified = c->repaired = c->safety = 0;
    c->status = 0;
  }
  const long long total = (long long)m * n;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long j = e / m, i = e - j * m;
    double* c = C + i + j * ldc;
    *c = beta == 0.0 ? 0.0 : beta * *c;
  }
}

std::mutex g_mu;
unsigned char* g_addr[64] = {nullptr};

// Once per device, with that device current: CRT tables + kernel attributes, and the device
// address of the scratch array (in host code its name is only a stand-in for the symbol).
int setup_current_device(unsigned char** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GGEMM_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    if (upload_tables_current_device() != 0) return GGEMM_ERR_NUMERICS;
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      std::fprintf(stderr, "[ggemm] ggemm_dgemm_noalloc: cudaGetSymbolAddress failed: %s\n",
                   cudaGetErrorString(e));
      return GGEMM_ERR_CUDA;
    }
    g_addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_addr[dev];
  return GGEMM_OK;
}

inline size_t up256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

int noalloc_counters(DevCounters** out) {
  unsigned char* base = nullptr;
  if (int r = setup_current_device(&base)) return r;
  *out = reinterpret_cast<DevCounters*>(base + kOffCounters);
  return GGEMM_OK;
}

}  // namespace g2

using namespace g2;

extern "C" int ggemm_dgemm_noalloc(const ggemm_problem_t* p, int num_moduli, int repair_mode,
                                   cudaStream_t stream) {
  if (!p) return GGEMM_ERR_INVALID;
  const ggemm_problem_t q = *p;
  if (q.m < 0 || q.n < 0 || q.k < 0) return GGEMM_ERR_INVALID;
  if (q.lda < (q.m > 1 ? q.m : 1) || q.ldb < (q.k > 1 ? q.k : 1) || q.ldc < (q.m > 1 ? q.m : 1))
    return GGEMM_ERR_INVALID;
  if (num_moduli < 0 || num_moduli == 1 || num_moduli > GGEMM_MAX_MODULI) return GGEMM_ERR_INVALID;
  if (repair_mode < GGEMM_REPAIR_DEFAULT || repair_mode > GGEMM_REPAIR_ON) return GGEMM_ERR_INVALID;
  if (q.m == 0 || q.n == 0) return GGEMM_OK;
  if (!q.C || (q.k > 0 && q.alpha != 0.0 && (!q.A || !q.B))) return GGEMM_ERR_INVALID;
  if (q.k > kMaxKExact) return GGEMM_ERR_UNSAFE;
  int N = num_moduli;
  if (N == 0) {
    N = choose_num_moduli(q.k, 1e-15);
    if (N < 0) return GGEMM_ERR_UNSAFE;
    N = N < 2 ? 2 : N;
  }
  const int mode = repair_mode == GGEMM_REPAIR_DEFAULT ? GGEMM_STAGE_REPAIR_COUNT
                   : repair_mode == GGEMM_REPAIR_OFF   ? GGEMM_STAGE_REPAIR_OFF
                   : repair_mode == GGEMM_REPAIR_COUNT ? GGEMM_STAGE_REPAIR_COUNT
                                                       : GGEMM_STAGE_REPAIR_ON;
  if (q.alpha == 0.0 || q.k == 0) {  // C = beta C without reading A or B
    unsigned char* base = nullptr;
    if (int r = setup_current_device(&base)) return r;
    const long long total = (long long)q.m * q.n;
    const long long blocks = std::min<long long>((total + 255) / 256, 148ll * 8);
    noalloc_scale_kernel<<<(unsigned)blocks, 256, 0, stream>>>(q.C, q.ldc, q.m, q.n, q.beta);
    return cudaGetLastError() == cudaSuccess ? GGEMM_OK : GGEMM_ERR_CUDA;
  }

  // scratch layout: counters | descriptors | ws A | ws B | image A | image B | products
  const size_t pa = up256(ggemm_img_plane_bytes(q.m, q.k));
  const size_t pb = up256(ggemm_img_plane_bytes(q.n, q.k));
  const size_t cp = ((size_t)q.m * q.n + 63) / 64 * 64;
  const bool digits = use_y8(q.m, q.n, N);
  const size_t prod = digits ? y8_bytes(q.m, q.n, N) : c32_bytes(q.m, q.n, N);
  const size_t off_wa = kOffData;
  const size_t off_wb = off_wa + up256(16 * (size_t)q.m);
  const size_t off_ia = off_wb + up256(16 * (size_t)q.n);
  const size_t off_ib = off_ia + (size_t)(N + 1) * pa;
  const size_t off_c = off_ib + (size_t)(N + 1) * pb;
  const size_t need = off_c + prod;
  if (need > kNoAllocBytes) {
    std::fprintf(stderr,
                 "[ggemm] ggemm_dgemm_noalloc: m=%d n=%d k=%d with %d moduli needs %zu bytes of "
                 "scratch; the fixed scratch holds %zu bytes (use ggemm_grouped_dgemm)\n",
                 q.m, q.n, q.k, N, need, kNoAllocBytes);
    return GGEMM_ERR_WORKSPACE;
  }
  unsigned char* base = nullptr;
  if (int r = setup_current_device(&base)) return r;

  NoAllocDescs d{};
  int nprep = 0, prep_blocks_total = 0;
  {
    ggemm_prep_desc_t a{};
    a.X = q.A;
    a.ld = q.lda;
    a.rows = q.m;
    a.k = q.k;
    a.N = N;
    a.kind = digits ? GGEMM_PREP_QSCALED : 0;  // q-scaled residues for the digit epilogue
    a.img = reinterpret_cast<int8_t*>(base + off_ia);
    a.plane_bytes = (long long)pa;
    a.ws = reinterpret_cast<int32_t*>(base + off_wa);
    ggemm_prep_desc_t b = a;
    b.X = q.B;
    b.ld = q.ldb;
    b.rows = q.n;
    b.kind = 1;
    b.img = reinterpret_cast<int8_t*>(base + off_ib);
    b.plane_bytes = (long long)pb;
    b.ws = reinterpret_cast<int32_t*>(base + off_wb);
    d.prep[0] = a;
    d.prep[1] = b;
    d.prep_prefix[0] = 0;
    d.prep_prefix[1] = prep_blocks(a);
    d.prep_prefix[2] = prep_blocks(a) + prep_blocks(b);
    nprep = 2;
    prep_blocks_total = d.prep_prefix[2];
  }
  GemmJob& j = d.job;
  j.A = reinterpret_cast<const int8_t*>(base + off_ia);
  j.B = reinterpret_cast<const int8_t*>(base + off_ib);
  j.C = reinterpret_cast<int32_t*>(base + off_c);
  j.Y = base + off_c;
  j.a_plane = (long long)pa;
  j.b_plane = (long long)pb;
  j.c_plane = (long long)cp;
  j.y_plane = (long long)y8_plane_bytes(q.m, q.n);
  j.N = N;
  j.y8 = digits ? 2 : 0;
  j.m = q.m;
  j.n = q.n;
  j.ksteps = (q.k + 31) / 32;
  j.planes = N + 1;
  set_gemm_tiling(j);
  d.job_prefix[0] = 0;
  d.job_prefix[1] = gemm_tiles(j);
  ggemm_recon_desc_t& rc = d.recon;
  rc.m = q.m;
  rc.n = q.n;
  rc.k = q.k;
  rc.N = N;
  rc.A = q.A;
  rc.lda = q.lda;
  rc.B = q.B;
  rc.ldb = q.ldb;
  rc.C = q.C;
  rc.ldc = q.ldc;
  rc.alpha = q.alpha;
  rc.beta = q.beta;
  rc.C32 = reinterpret_cast<const int32_t*>(base + off_c);
  rc.c_plane = digits ? (long long)y8_plane_bytes(q.m, q.n) : (long long)cp;
  rc.layout = digits ? GGEMM_PRODUCTS_DIGITS : GGEMM_PRODUCTS_INT32;
  rc.rs = reinterpret_cast<const int32_t*>(base + off_wa);
  rc.cs = reinterpret_cast<const int32_t*>(base + off_wb);
  d.recon_prefix[0] = 0;
  d.recon_prefix[1] = recon_job_blocks(rc);

  const unsigned char* db = base + kOffDescs;
  DevCounters* cnt = reinterpret_cast<DevCounters*>(base + kOffCounters);
  noalloc_setup_kernel<<<1, 32, 0, stream>>>(d);
  if (cudaGetLastError() != cudaSuccess) return GGEMM_ERR_CUDA;
  PrepSplit sp;  // both descriptors have N moduli: one prep instance
  for (int c = 0; c <= kPrepClasses; ++c) {
    const bool after = c > prep_class(N);
    sp.first[c] = after ? nprep : 0;
    sp.block0[c] = after ? prep_blocks_total : 0;
  }
  if (nprep &&
      launch_prep(reinterpret_cast<const ggemm_prep_desc_t*>(db + offsetof(NoAllocDescs, prep)),
                  reinterpret_cast<const int*>(db + offsetof(NoAllocDescs, prep_prefix)), sp, cnt,
                  stream))
    return GGEMM_ERR_NUMERICS;
  if (d.job_prefix[1] > 0 &&
      launch_gemm(reinterpret_cast<const GemmJob*>(db + offsetof(NoAllocDescs, job)),
                  reinterpret_cast<const long long*>(db + offsetof(NoAllocDescs, job_prefix)), 1,
                  d.job_prefix[1], cnt, stream, 0))
    return GGEMM_ERR_I8GEMM;
  ReconSplit rsp;  // one descriptor: one reconstruct instance
  for (int c = 0; c <= kReconClasses; ++c) {
    const bool after = c > recon_class(N);
    rsp.first[c] = after ? 1 : 0;
    rsp.block0[c] = after ? d.recon_prefix[1] : 0;
  }
  if (launch_recon(reinterpret_cast<const ggemm_recon_desc_t*>(db + offsetof(NoAllocDescs, recon)),
                   reinterpret_cast<const long long*>(db + offsetof(NoAllocDescs, recon_prefix)),
                   rsp, mode, cnt, stream, nullptr, /*nonfinite_hint=*/true))
    return GGEMM_ERR_NUMERICS;
  return GGEMM_OK;
}

extern "C" int ggemm_dgemm_noalloc_status(cudaStream_t stream) {
  DevCounters c{};
  if (cudaMemcpyFromSymbolAsync(&c, g_noalloc_scratch, sizeof c, kOffCounters,
                                cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return -1;
  return (int)c.status;
}
