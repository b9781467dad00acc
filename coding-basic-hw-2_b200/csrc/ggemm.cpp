// ggemm.cpp -- handle, workspace and the seven call paths of the public C ABI (include/ggemm.h).
//
// Reference behaviour preserved (src/ggemm.cu:228-741): all allocation at create, validation
// and element budgets, per-problem routing by the planner, operand reuse on path 5, one
// pinned host->device copy of a descriptor blob per call, a launch count independent of the
// group size for the grouped paths, native FP64 (cuBLAS) for k == 0 / alpha == 0 / fallbacks,
// stats and the opt-in synchronizing repair counters.
//
// What differs (B200 design): residues are written in the tensor-core operand image layout,
// the residue GEMM is a tcgen05 kernel, counters are per handle, and a group whose workspace
// exceeds the handle's capacity runs in consecutive chunks (prep, GEMM, reconstruct per chunk)
// instead of failing, so one B200 can hold groups whose int32 products alone exceed its HBM.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "ggemm_ext.h"
#include "ggemm_graph.h"
#include "internal.hpp"

namespace g2 {

#define G2_CU(x)                                 \
  do {                                           \
    if ((x) != cudaSuccess) return GGEMM_ERR_CUDA; \
  } while (0)

constexpr size_t kCublasWsBytes = 64ull << 20;
constexpr int kPlanesMax = kMaxModuli + 1;

void NativeGroups::reserve(size_t P) {
  ta.resize(P);
  tb.resize(P);
  for (auto* v : {&m, &n, &k, &lda, &ldb, &ldc, &size}) v->resize(P);
  alpha.resize(P);
  beta.resize(P);
}

static inline uint64_t bits_of(double x) {
  uint64_t u;
  std::memcpy(&u, &x, sizeof u);
  return u;
}

int group_native(const ggemm_problem_t* probs, int* idx, int cnt, NativeGroups& g) {
  auto key_less = [probs](int x, int y) {
    const ggemm_problem_t &a = probs[x], &b = probs[y];
    if (a.m != b.m) return a.m < b.m;
    if (a.n != b.n) return a.n < b.n;
    if (a.k != b.k) return a.k < b.k;
    if (a.lda != b.lda) return a.lda < b.lda;
    if (a.ldb != b.ldb) return a.ldb < b.ldb;
    if (a.ldc != b.ldc) return a.ldc < b.ldc;
    if (bits_of(a.alpha) != bits_of(b.alpha)) return bits_of(a.alpha) < bits_of(b.alpha);
    if (bits_of(a.beta) != bits_of(b.beta)) return bits_of(a.beta) < bits_of(b.beta);
    return x < y;
  };
  std::sort(idx, idx + cnt, key_less);
  int ng = 0;
  for (int i = 0; i < cnt; ++i) {
    const ggemm_problem_t& p = probs[idx[i]];
    if (i > 0) {
      const ggemm_problem_t& q = probs[idx[i - 1]];
      if (q.m == p.m && q.n == p.n && q.k == p.k && q.lda == p.lda && q.ldb == p.ldb &&
          q.ldc == p.ldc && bits_of(q.alpha) == bits_of(p.alpha) &&
          bits_of(q.beta) == bits_of(p.beta)) {
        ++g.size[ng - 1];
        continue;
      }
    }
    g.ta[ng] = CUBLAS_OP_N;
    g.tb[ng] = CUBLAS_OP_N;
    g.m[ng] = p.m;
    g.n[ng] = p.n;
    g.k[ng] = p.k;
    g.lda[ng] = p.lda;
    g.ldb[ng] = p.ldb;
    g.ldc[ng] = p.ldc;
    g.alpha[ng] = p.alpha;
    g.beta[ng] = p.beta;
    g.size[ng] = 1;
    ++ng;
  }
  return ng;
}

int validate_call(ggemm_handle_t h, const ggemm_problem_t* p, int num) {
  if (num < 0 || num > h->max_problems || (num > 0 && !p)) return GGEMM_ERR_INVALID;
  size_t ta = 0, tb = 0, tc = 0;
  for (int g = 0; g < num; ++g) {
    const ggemm_problem_t& q = p[g];
    if (q.m < 0 || q.n < 0 || q.k < 0) return GGEMM_ERR_INVALID;
    if (q.lda < std::max(1, q.m) || q.ldb < std::max(1, q.k) || q.ldc < std::max(1, q.m))
      return GGEMM_ERR_INVALID;
    if (q.m > 0 && q.n > 0) {
      if (!q.C) return GGEMM_ERR_INVALID;
      if (q.k > 0 && (!q.A || !q.B)) return GGEMM_ERR_INVALID;
    }
    ta += (size_t)q.m * q.k;
    tb += (size_t)q.k * q.n;
    tc += (size_t)q.m * q.n;
  }
  if (ta > h->max_A || tb > h->max_B || tc > h->max_C) return GGEMM_ERR_WORKSPACE;
  return GGEMM_OK;
}

int stage_repair_mode(ggemm_path_t path, const ggemm_config_t* cfg) {
  const int m = cfg ? cfg->repair_mode : GGEMM_REPAIR_DEFAULT;
  switch (m) {
    case GGEMM_REPAIR_DEFAULT:
      return path == GGEMM_PATH_AUTO ? GGEMM_STAGE_REPAIR_ON : GGEMM_STAGE_REPAIR_COUNT;
    case GGEMM_REPAIR_OFF: return GGEMM_STAGE_REPAIR_OFF;
    case GGEMM_REPAIR_COUNT: return GGEMM_STAGE_REPAIR_COUNT;
    case GGEMM_REPAIR_ON: return GGEMM_STAGE_REPAIR_ON;
    default: return -1;
  }
}

// ------------------------------------------------------------------------ call construction
namespace {

struct BlobWriter {
  char* hb;
  size_t off = 0, cap;
  bool overflow = false;
  size_t take(size_t bytes, size_t align = 16) {
    off = align_up(off, align);
    const size_t at = off;
    off += bytes;
    if (off > cap) overflow = true;
    return at;
  }
  template <typename T>
  T* at(size_t o) {
    return reinterpret_cast<T*>(hb + o);
  }
};

void print_ws_diag(ggemm_handle_t h, const ggemm_problem_t& p, int N) {
  if (h->ws_diag_printed) return;
  h->ws_diag_printed = 1;
  std::fprintf(stderr,
               "[ggemm] GGEMM_ERR_WORKSPACE: one problem (m=%d n=%d k=%d, %d moduli) needs "
               "%zu + %zu residue bytes and %zu product bytes; the handle's pool holds %zu "
               "bytes (create with larger budgets or min_k <= %d)\n",
               p.m, p.n, p.k, N, img_bytes(p.m, p.k, N), img_bytes(p.n, p.k, N),
               4 * product_elems(p.m, p.n, N), h->pool_cap, p.k);
}

}  // namespace

int build_emu_call(ggemm_handle_t h, ggemm_path_t path, const ggemm_config_t* cfg,
                   const ggemm_problem_t* probs, int num, char* hb, const char* db,
                   EmuCall* out) {
  EmuCall c;
  const bool loop = path == GGEMM_PATH_EMU_LOOP;
  const bool lbat = path == GGEMM_PATH_EMU_LOOP_BATCHED;
  c.reuse = path == GGEMM_PATH_EMU_GROUPED_REUSE;
  const ggemm_path_t plan_path = c.reuse ? GGEMM_PATH_EMU_GROUPED
                                 : lbat  ? GGEMM_PATH_EMU_LOOP
                                         : path;
  PlanEntry* plan = h->plan.data();
  int r = plan_group(probs, num, cfg, plan_path, h->dm, h->rho_budget, plan, h->memo.data(),
                     h->memo.size());
  if (r) return r;

  ReuseResult rr{};
  if (c.reuse) {
    int* nm = h->order.data();  // scratch
    for (int g = 0; g < num; ++g) nm[g] = plan[g].route == kRouteEmu ? plan[g].num_moduli : 0;
    rr = h->reuse.build(probs, num, nm, h->reuse_promote ? kReusePromote : kReuseExactN);
    if (rr.status) return rr.status == 1 ? GGEMM_ERR_WORKSPACE : GGEMM_ERR_INVALID;
    if (h->reuse_promote)
      for (int g = 0; g < num; ++g)
        if (plan[g].route == kRouteEmu) plan[g].num_moduli = rr.eff_nmod[g];
  }

  // partition
  int* emu = h->emu.data();
  int* nat = h->nat.data();
  for (int g = 0; g < num; ++g) {
    const PlanEntry& e = plan[g];
    if (e.route == kRouteEmpty) continue;
    if (e.route == kRouteEmu) emu[c.ne++] = g;
    else nat[c.nn++] = g;
  }
  c.nmin = c.ne ? kMaxModuli : 0;
  for (int j = 0; j < c.ne; ++j) {
    const int N = plan[emu[j]].num_moduli;
    c.nmax = std::max(c.nmax, N);
    c.nmin = std::min(c.nmin, N);
  }

  // unique operands
  if (c.reuse) {
    c.num_ua = rr.num_ua;
    c.num_ub = rr.num_ub;
    c.num_promoted = rr.num_promoted;
    for (int u = 0; u < rr.num_ua; ++u) {
      h->ua_rep[u] = rr.ua_rep[u];
      h->ua_n[u] = rr.ua_nmod[u];
    }
    for (int u = 0; u < rr.num_ub; ++u) {
      h->ub_rep[u] = rr.ub_rep[u];
      h->ub_n[u] = rr.ub_nmod[u];
    }
    for (int j = 0; j < c.ne; ++j) {
      h->ua_of[j] = rr.prob_a[emu[j]];
      h->ub_of[j] = rr.prob_b[emu[j]];
    }
  } else {
    c.num_ua = c.num_ub = c.ne;
    for (int j = 0; j < c.ne; ++j) {
      h->ua_rep[j] = h->ub_rep[j] = emu[j];
      h->ua_n[j] = h->ub_n[j] = plan[emu[j]].num_moduli;
      h->ua_of[j] = h->ub_of[j] = j;
    }
  }
  for (int u = 0; u < c.num_ua; ++u) h->ua_chunk[u] = -1;
  for (int u = 0; u < c.num_ub; ++u) h->ub_chunk[u] = -1;

  // chunks: consecutive emulated problems whose residue images, products and row / column
  // workspace fit the pool.  Chunk layout: A images from offset 0, then B images, products,
  // row workspace and column workspace, each region 256-byte aligned.  A unique operand is
  // prepared once per chunk that uses it; each problem records where its operands' images and
  // workspace lie in its own chunk (pa_* / pb_*), and whether it is the problem that prepares
  // them there (pa_new / pb_new).
  h->chunks.clear();
  {
    size_t ia = 0, ib = 0, wa = 0, wb = 0, cc = 0;
    Chunk cur{};
    cur.first = 0;
    cur.count = 0;
    auto close = [&](Chunk& ch) {
      ch.base_b = align_up(ia, kAlign);
      ch.base_c = align_up(ch.base_b + ib, kAlign);
      ch.base_wa = align_up(ch.base_c + 4 * cc, kAlign);
      ch.base_wb = align_up(ch.base_wa + 4 * wa, kAlign);
    };
    for (int j = 0; j < c.ne; ++j) {
      const int g = emu[j];
      const ggemm_problem_t& p = probs[g];
      const int N = plan[g].num_moduli;
      const int ua = h->ua_of[j], ub = h->ub_of[j];
      const bool chunk_per_problem = loop || lbat;
      for (int attempt = 0; attempt < 2; ++attempt) {
        const int cid = (int)h->chunks.size();  // id of the open chunk (changes on a retry)
        const bool new_a = h->ua_chunk[ua] != cid;
        const bool new_b = h->ub_chunk[ub] != cid;
        const size_t na = new_a ? img_bytes(p.m, p.k, h->ua_n[ua]) : 0;
        const size_t nb = new_b ? img_bytes(p.n, p.k, h->ub_n[ub]) : 0;
        const size_t nwa = new_a ? ws_ints(p.m) : 0;
        const size_t nwb = new_b ? ws_ints(p.n) : 0;
        const size_t ncc = product_elems(p.m, p.n, N);
        const size_t bytes = align_up(ia + na, kAlign) + align_up(ib + nb, kAlign) +
                             align_up(4 * (cc + ncc), kAlign) + align_up(4 * (wa + nwa), kAlign) +
                             4 * (wb + nwb);
        if (bytes <= h->pool_cap && !(chunk_per_problem && cur.count > 0)) {
          if (new_a) {
            h->ua_chunk[ua] = cid;
            h->ua_img[ua] = ia;
            h->ua_ws[ua] = wa;
            ia += na;
            wa += nwa;
          }
          if (new_b) {
            h->ub_chunk[ub] = cid;
            h->ub_img[ub] = ib;
            h->ub_ws[ub] = wb;
            ib += nb;
            wb += nwb;
          }
          h->pa_new[j] = new_a;
          h->pb_new[j] = new_b;
          h->pa_img[j] = h->ua_img[ua];
          h->pa_ws[j] = h->ua_ws[ua];
          h->pb_img[j] = h->ub_img[ub];
          h->pb_ws[j] = h->ub_ws[ub];
          h->c32_off[j] = cc;
          cc += ncc;
          ++cur.count;
          break;
        }
        if (cur.count == 0) {  // does not fit even alone
          print_ws_diag(h, p, N);
          return GGEMM_ERR_WORKSPACE;
        }
        close(cur);  // close the chunk and retry in a fresh one
        h->chunks.push_back(cur);
        cur = Chunk{};
        cur.first = j;
        cur.count = 0;
        ia = ib = wa = wb = cc = 0;
        if (h->chunks.size() >= (size_t)h->max_problems) return GGEMM_ERR_WORKSPACE;
        (void)attempt;
      }
    }
    if (cur.count > 0) {
      close(cur);
      h->chunks.push_back(cur);
    }
  }

  // descriptors
  BlobWriter bw{hb, 0, h->blob_cap};
  int* order = h->order.data();
  for (Chunk& ch : h->chunks) {
    // The A images of a chunk are q-scaled (GGEMM_PREP_QSCALED) when every problem of the chunk
    // takes the digit layout and has its A image's moduli count: the GEMM epilogue then
    // skips the modular product by q_l.
    ch.qscale = true;
    for (int j = ch.first; j < ch.first + ch.count; ++j) {
      const ggemm_problem_t& p = probs[emu[j]];
      const int N = plan[emu[j]].num_moduli;
      if (!use_y8(p.m, p.n, N) || h->ua_n[h->ua_of[j]] != N) ch.qscale = false;
    }
    int32_t* wsa = reinterpret_cast<int32_t*>(h->pool + ch.base_wa);
    int32_t* wsb = reinterpret_cast<int32_t*>(h->pool + ch.base_wb);
    // prep descriptors: the unique A / B operands this chunk prepares
    int np = 0;
    for (int j = ch.first; j < ch.first + ch.count; ++j) np += h->pa_new[j] + h->pb_new[j];
    ch.num_prep = np;
    ch.off_prep = bw.take((size_t)np * sizeof(ggemm_prep_desc_t), 64);
    ch.off_prep_prefix = bw.take((size_t)(np + 1) * sizeof(int), 16);
    if (bw.overflow) return GGEMM_ERR_WORKSPACE;
    ggemm_prep_desc_t* pd = bw.at<ggemm_prep_desc_t>(ch.off_prep);
    int* pp = bw.at<int>(ch.off_prep_prefix);
    int q = 0, blocks = 0;
    for (int j = ch.first; j < ch.first + ch.count; ++j) {
      const int ua = h->ua_of[j], ub = h->ub_of[j];
      if (h->pa_new[j]) {
        const ggemm_problem_t& p = probs[h->ua_rep[ua]];
        ggemm_prep_desc_t& d = pd[q];
        d.X = p.A;
        d.ld = p.lda;
        d.rows = p.m;
        d.k = p.k;
        d.N = h->ua_n[ua];
        d.kind = ch.qscale ? GGEMM_PREP_QSCALED : 0;
        d.img = h->pool + h->pa_img[j];
        d.plane_bytes = (long long)align_up(ggemm_img_plane_bytes(p.m, p.k), kAlign);
        d.ws = wsa + h->pa_ws[j];
        ++q;
      }
      if (h->pb_new[j]) {
        const ggemm_problem_t& p = probs[h->ub_rep[ub]];
        ggemm_prep_desc_t& d = pd[q];
        d.X = p.B;
        d.ld = p.ldb;
        d.rows = p.n;
        d.k = p.k;
        d.N = h->ub_n[ub];
        d.kind = 1;
        d.img = h->pool + ch.base_b + h->pb_img[j];
        d.plane_bytes = (long long)align_up(ggemm_img_plane_bytes(p.n, p.k), kAlign);
        d.ws = wsb + h->pb_ws[j];
        ++q;
      }
    }
    // descriptors sorted by prep instance (launch_prep)
    prep_partition(pd, q, pp, &ch.prep_split);
    blocks = (int)ch.prep_split.block0[kPrepClasses];
    ch.prep_blocks = blocks;

    // residue GEMM jobs: one per problem (EMU_LOOP: one per plane), heaviest tiles first
    int nj = 0;
    for (int j = ch.first; j < ch.first + ch.count; ++j)
      nj += loop ? (plan[emu[j]].num_moduli + 1) : 1;
    ch.off_jobs = bw.take((size_t)nj * sizeof(GemmJob), 64);
    ch.off_job_prefix = bw.take((size_t)(loop ? 2 * nj : nj + 1) * sizeof(long long), 16);
    ch.off_recon = bw.take((size_t)ch.count * sizeof(ggemm_recon_desc_t), 64);
    ch.off_recon_prefix = bw.take((size_t)(ch.count + 1) * sizeof(long long), 16);
    if (bw.overflow) return GGEMM_ERR_WORKSPACE;
    GemmJob* jobs = bw.at<GemmJob>(ch.off_jobs);
    long long* jp = bw.at<long long>(ch.off_job_prefix);
    ggemm_recon_desc_t* rd = bw.at<ggemm_recon_desc_t>(ch.off_recon);
    long long* rp = bw.at<long long>(ch.off_recon_prefix);
    for (int x = 0; x < ch.count; ++x) order[x] = ch.first + x;
    if (!loop && !lbat)  // LPT: deepest K (heaviest tiles) first, then most tiles
      std::sort(order, order + ch.count, [&](int a, int b) {
        const ggemm_problem_t &pa = probs[emu[a]], &pb = probs[emu[b]];
        if (pa.k != pb.k) return pa.k > pb.k;
        const long long ta = (long long)((pa.m + 127) / 128) * ((pa.n + 255) / 256) *
                             (plan[emu[a]].num_moduli + 1);
        const long long tb = (long long)((pb.m + 127) / 128) * ((pb.n + 255) / 256) *
                             (plan[emu[b]].num_moduli + 1);
        if (ta != tb) return ta > tb;
        return a < b;
      });
    // problems of the chunk that share an operand (tiles numbered plane-outer, below)
    bool shared = false;
    for (int j = ch.first; j < ch.first + ch.count; ++j)
      shared = shared || !h->pa_new[j] || !h->pb_new[j];
    // the paired GEMM (256 x 256 tiles on CTA pairs) when its row padding costs little
    // (gemm_pair_pays); GGEMM_GEMM_PAIR forces either kernel
    ch.pair = false;
    if (!loop && !lbat && h->gemm_pair != 0) {
      if (h->gemm_pair == 1) {
        ch.pair = true;
      } else {
        int* mm = h->pair_m.data();
        int* nn = h->pair_n.data();
        int* kk = h->pair_k.data();
        int* pl = h->pair_p.data();
        for (int x = 0; x < ch.count; ++x) {
          const ggemm_problem_t& p = probs[emu[ch.first + x]];
          mm[x] = p.m;
          nn[x] = p.n;
          kk[x] = (p.k + 31) / 32;
          pl[x] = plan[emu[ch.first + x]].num_moduli + 1;
        }
        ch.pair = gemm_pair_pays(mm, nn, kk, pl, ch.count, h->num_sms);
      }
    }
    long long tiles = 0;
    int jq = 0;
    for (int x = 0; x < ch.count; ++x) {
      const int j = order[x];
      const int g = emu[j];
      const ggemm_problem_t& p = probs[g];
      const int N = plan[g].num_moduli;
      GemmJob base{};
      base.A = h->pool + h->pa_img[j];
      base.B = h->pool + ch.base_b + h->pb_img[j];
      base.C = reinterpret_cast<int32_t*>(h->pool + ch.base_c) + h->c32_off[j];
      base.Y = reinterpret_cast<uint8_t*>(base.C);
      base.a_plane = (long long)align_up(ggemm_img_plane_bytes(p.m, p.k), kAlign);
      base.b_plane = (long long)align_up(ggemm_img_plane_bytes(p.n, p.k), kAlign);
      base.c_plane = (long long)c_plane_elems(p.m, p.n);
      base.y_plane = (long long)y8_plane_bytes(p.m, p.n);
      base.N = N;
      base.y8 = use_y8(p.m, p.n, N) ? (ch.qscale ? 2 : 1) : 0;
      base.m = p.m;
      base.n = p.n;
      base.ksteps = (p.k + 31) / 32;
      if (ch.pair) set_gemm_tiling_pair(base);
      else set_gemm_tiling(base);
      if (loop) {
        for (int l = 0; l <= N; ++l) {
          GemmJob jb = base;
          jb.A += l * base.a_plane;
          jb.B += l * base.b_plane;
          if (base.y8) jb.plane0 = l;
          else jb.C += l * base.c_plane;
          jb.planes = 1;
          jobs[jq] = jb;
          jp[2 * jq] = 0;
          jp[2 * jq + 1] = gemm_tiles(jb);
          tiles += gemm_tiles(jb);
          ++jq;
        }
      } else {
        base.planes = N + 1;
        jobs[jq] = base;
        jp[jq] = tiles;
        tiles += gemm_tiles(base);
        ++jq;
      }
    }
    if (!loop) jp[jq] = tiles;
    ch.tiles = tiles;
    ch.ragged = gemm_jobs_ragged(jobs, jq);
    // plane-outer tile numbering when problems of the chunk share an operand and every job has
    // the same plane count: the prefix then counts one plane's tiles per job
    ch.plane_outer = false;
    if (!loop && jq > 1) {
      bool same_planes = true;
      for (int x = 1; x < jq; ++x) same_planes = same_planes && jobs[x].planes == jobs[0].planes;
      if (shared && same_planes) {
        ch.plane_outer = true;
        long long tp = 0;
        for (int x = 0; x < jq; ++x) {
          jp[x] = tp;
          tp += (long long)jobs[x].tm * jobs[x].tn;
        }
        jp[jq] = tp;
        ch.tiles = tp * jobs[0].planes;
      }
    }
    for (int x = 0; x < ch.count; ++x) {
      const int j = ch.first + x;
      const int g = emu[j];
      const ggemm_problem_t& p = probs[g];
      const bool y8 = use_y8(p.m, p.n, plan[g].num_moduli);
      ggemm_recon_desc_t& d = rd[x];
      d = ggemm_recon_desc_t{};
      d.layout = y8 ? GGEMM_PRODUCTS_DIGITS : GGEMM_PRODUCTS_INT32;
      d.m = p.m;
      d.n = p.n;
      d.k = p.k;
      d.N = plan[g].num_moduli;
      d.A = p.A;
      d.lda = p.lda;
      d.B = p.B;
      d.ldb = p.ldb;
      d.C = p.C;
      d.ldc = p.ldc;
      d.alpha = p.alpha;
      d.beta = p.beta;
      d.C32 = reinterpret_cast<int32_t*>(h->pool + ch.base_c) + h->c32_off[j];
      d.c_plane = y8 ? (long long)y8_plane_bytes(p.m, p.n) : (long long)c_plane_elems(p.m, p.n);
      d.rs = wsa + h->pa_ws[j];
      d.cs = wsb + h->pb_ws[j];
    }
    // descriptors sorted by reconstruct instance (launch_recon)
    recon_partition(rd, ch.count, rp, &ch.recon_split);
    ch.recon_blocks = ch.recon_split.block0[kReconClasses];
    c.nprep_total += np;
  }

  // native problems: pointer arrays for the grouped cuBLAS call
  if (c.nn >= 2) {
    c.nat_groups = group_native(probs, nat, c.nn, h->ngroups);
    c.off_nat_ptrs = bw.take((size_t)3 * c.nn * sizeof(void*), 16);
    if (bw.overflow) return GGEMM_ERR_WORKSPACE;
    const void** P = bw.at<const void*>(c.off_nat_ptrs);
    for (int i = 0; i < c.nn; ++i) {
      const ggemm_problem_t& p = probs[nat[i]];
      P[i] = p.A;
      P[c.nn + i] = p.B;
      P[2 * c.nn + i] = p.C;
    }
  }
  c.blob_bytes = bw.off;
  (void)db;
  *out = c;
  return GGEMM_OK;
}

int enqueue_native(ggemm_handle_t h, const ggemm_problem_t* probs, const int* idx, int cnt,
                   bool grouped, int ngroups, const char* d_ptrs, cudaStream_t s,
                   int* launches) {
  if (cnt == 0) return GGEMM_OK;
  if (cublasSetStream(h->cublas, s) != CUBLAS_STATUS_SUCCESS ||
      cublasSetWorkspace(h->cublas, h->cublas_ws, h->cublas_ws_bytes) != CUBLAS_STATUS_SUCCESS)
    return GGEMM_ERR_CUBLAS;
  if (!grouped || cnt == 1) {
    for (int i = 0; i < cnt; ++i) {
      const ggemm_problem_t& p = probs[idx[i]];
      if (cublasDgemm(h->cublas, CUBLAS_OP_N, CUBLAS_OP_N, p.m, p.n, p.k, &p.alpha, p.A, p.lda,
                      p.B, p.ldb, &p.beta, p.C, p.ldc) != CUBLAS_STATUS_SUCCESS)
        return GGEMM_ERR_CUBLAS;
      ++*launches;
    }
    return GGEMM_OK;
  }
  const void* const* base = reinterpret_cast<const void* const*>(d_ptrs);
  NativeGroups& g = h->ngroups;
  if (cublasDgemmGroupedBatched(
          h->cublas, g.ta.data(), g.tb.data(), g.m.data(), g.n.data(), g.k.data(),
          g.alpha.data(), reinterpret_cast<const double* const*>(base), g.lda.data(),
          reinterpret_cast<const double* const*>(base + cnt), g.ldb.data(), g.beta.data(),
          reinterpret_cast<double* const*>(const_cast<void* const*>(base + 2 * cnt)),
          g.ldc.data(), ngroups, g.size.data()) != CUBLAS_STATUS_SUCCESS)
    return GGEMM_ERR_CUBLAS;
  ++*launches;
  return GGEMM_OK;
}

int enqueue_emu_call(ggemm_handle_t h, const EmuCall& c, const ggemm_problem_t* probs,
                     const char* db, int repair, bool per_plane, bool record, cudaStream_t s,
                     int* launches) {
  (void)c;
  record = record && h->stage_ev_on && h->chunks.size() == 1;
  auto mark = [&](int i) { return !record || cudaEventRecord(h->stage_ev[i], s) == cudaSuccess; };
  // prep counts this call's non-finite rows / columns from zero: the reconstruct's safety
  // blocks read the count to know whether any entry needs them
  if (!h->chunks.empty() &&
      cudaMemsetAsync(&h->counters->nonfinite, 0, sizeof(h->counters->nonfinite), s) !=
          cudaSuccess)
    return GGEMM_ERR_CUDA;
  for (const Chunk& ch : h->chunks) {
    if (!mark(0)) return GGEMM_ERR_CUDA;
    if (ch.prep_blocks > 0) {
      if (launch_prep(reinterpret_cast<const ggemm_prep_desc_t*>(db + ch.off_prep),
                      reinterpret_cast<const int*>(db + ch.off_prep_prefix), ch.prep_split,
                      h->counters, s, launches))
        return GGEMM_ERR_NUMERICS;
    }
    if (!mark(1)) return GGEMM_ERR_CUDA;
    const GemmJob* jobs = reinterpret_cast<const GemmJob*>(db + ch.off_jobs);
    const long long* jp = reinterpret_cast<const long long*>(db + ch.off_job_prefix);
    if (per_plane) {
      // EMU_LOOP: one problem per chunk, one GEMM launch per plane (own 2-entry prefix)
      const ggemm_problem_t& p = probs[h->emu[ch.first]];
      const int planes = h->plan[h->emu[ch.first]].num_moduli + 1;
      GemmJob shape{};
      shape.m = p.m;
      shape.n = p.n;
      set_gemm_tiling(shape);
      const long long tiles = (long long)shape.tm * shape.tn;
      for (int q = 0; q < planes && tiles > 0; ++q) {
        if (launch_gemm(jobs + q, jp + 2 * q, 1, tiles, h->counters, s, 0))
          return GGEMM_ERR_I8GEMM;
        ++*launches;
      }
    } else if (ch.tiles > 0) {
      const int walk = (ch.ragged ? kGemmWalkBothEnds : 0) |
                       (ch.plane_outer ? kGemmWalkPlaneOuter : 0);
      const int e = ch.pair ? launch_gemm_pair(jobs, jp, ch.count, ch.tiles, h->counters, s, walk)
                            : launch_gemm(jobs, jp, ch.count, ch.tiles, h->counters, s, walk);
      if (e) return GGEMM_ERR_I8GEMM;
      ++*launches;
    }
    if (!mark(2)) return GGEMM_ERR_CUDA;
    if (ch.recon_blocks > 0) {
      if (launch_recon(reinterpret_cast<const ggemm_recon_desc_t*>(db + ch.off_recon),
                       reinterpret_cast<const long long*>(db + ch.off_recon_prefix),
                       ch.recon_split, repair, h->counters, s, launches,
                       /*nonfinite_hint=*/true))
        return GGEMM_ERR_NUMERICS;
    }
    if (!mark(3)) return GGEMM_ERR_CUDA;
  }
  return GGEMM_OK;
}

}  // namespace g2

using namespace g2;

static int counters_reset(ggemm_handle_t h) {
  if (!h->stats_repair) return GGEMM_OK;
  return cudaMemsetAsync(h->counters, 0, sizeof(DevCounters), h->stream) == cudaSuccess
             ? GGEMM_OK
             : GGEMM_ERR_CUDA;
}

static int counters_read(ggemm_handle_t h, ggemm_stats_t* st) {
  st->num_repaired = st->num_uncertified = st->num_safety_fallback = -1;
  if (!h->stats_repair) return GGEMM_OK;
  DevCounters c{};
  if (cudaMemcpyAsync(&c, h->counters, sizeof c, cudaMemcpyDeviceToHost, h->stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess)
    return GGEMM_ERR_CUDA;
  if (c.status != kStatusOk) return GGEMM_ERR_I8GEMM;
  st->num_repaired = (long long)c.repaired;
  st->num_uncertified = (long long)c.uncertified;
  st->num_safety_fallback = (long long)c.safety;
  return GGEMM_OK;
}

static int acquire_slot(ggemm_handle_t h, int* slot) {
  const int s = h->next_slot;
  h->next_slot ^= 1;
  if (cudaEventSynchronize(h->slot_done[s]) != cudaSuccess) return GGEMM_ERR_CUDA;
  *slot = s;
  return GGEMM_OK;
}

static int path_native(ggemm_handle_t h, bool grouped, const ggemm_problem_t* probs, int num,
                       ggemm_stats_t* st) {
  int cnt = 0;
  int* nat = h->nat.data();
  for (int g = 0; g < num; ++g)
    if (probs[g].m > 0 && probs[g].n > 0) nat[cnt++] = g;
  if (!grouped || cnt < 2)
    return enqueue_native(h, probs, nat, cnt, false, 0, nullptr, h->stream,
                          &st->kernel_launches);
  int slot, r;
  if ((r = acquire_slot(h, &slot))) return r;
  char* hb = h->h_blob[slot];
  const int ng = group_native(probs, nat, cnt, h->ngroups);
  const void** P = reinterpret_cast<const void**>(hb);
  for (int i = 0; i < cnt; ++i) {
    P[i] = probs[nat[i]].A;
    P[cnt + i] = probs[nat[i]].B;
    P[2 * cnt + i] = probs[nat[i]].C;
  }
  if (launch_blob_upload(h->d_blob[0], h->h_blob_dev[slot], 3 * cnt * sizeof(void*), h->stream))
    return GGEMM_ERR_CUDA;
  r = enqueue_native(h, probs, nat, cnt, true, ng, h->d_blob[0], h->stream,
                     &st->kernel_launches);
  const int r2 = cudaEventRecord(h->slot_done[slot], h->stream) == cudaSuccess ? 0 : GGEMM_ERR_CUDA;
  return r ? r : r2;
}

static int path_emu(ggemm_handle_t h, ggemm_path_t path, const ggemm_config_t* cfg,
                    const ggemm_problem_t* probs, int num, ggemm_stats_t* st, int repair) {
  int slot, r;
  if ((r = acquire_slot(h, &slot))) return r;
  char* hb = h->h_blob[slot];
  char* db = h->d_blob[0];
  EmuCall c;
  r = build_emu_call(h, path, cfg, probs, num, hb, db, &c);
  if (r) return r;
  st->num_fallback = 0;
  for (int i = 0; i < c.nn; ++i) st->num_fallback += route_is_fallback(h->plan[h->nat[i]].route);
  st->moduli_min = c.nmin;
  st->moduli_max = c.nmax;
  st->reuse_enabled = c.reuse ? 1 : 0;
  st->num_unique_A = c.reuse ? c.num_ua : c.ne;
  st->num_unique_B = c.reuse ? c.num_ub : c.ne;
  st->num_promoted = c.reuse ? c.num_promoted : 0;
  if (launch_blob_upload(db, h->h_blob_dev[slot], c.blob_bytes, h->stream))
    return GGEMM_ERR_CUDA;
  r = enqueue_emu_call(h, c, probs, db, repair, path == GGEMM_PATH_EMU_LOOP, true, h->stream,
                       &st->kernel_launches);
  if (!r && c.nn > 0)
    r = enqueue_native(h, probs, h->nat.data(), c.nn, c.nn >= 2, c.nat_groups,
                       db + c.off_nat_ptrs, h->stream, &st->kernel_launches);
  const int r2 = cudaEventRecord(h->slot_done[slot], h->stream) == cudaSuccess ? 0 : GGEMM_ERR_CUDA;
  return r ? r : r2;
}

// ============================================================================ public C ABI
extern "C" void ggemm_destroy(ggemm_handle_t h) {
  if (!h) return;
  cudaStreamSynchronize(h->stream);
  for (int s = 0; s < 2; ++s) {
    if (h->slot_done[s]) cudaEventDestroy(h->slot_done[s]);
    if (h->h_blob[s]) cudaFreeHost(h->h_blob[s]);
    if (h->d_blob[s]) cudaFree(h->d_blob[s]);
  }
  if (h->cublas) cublasDestroy(h->cublas);
  cudaFree(h->cublas_ws);
  cudaFree(h->pool);
  cudaFree(h->counters);
  delete h;
}

extern "C" int ggemm_create(ggemm_handle_t* out, int max_problems, size_t max_A, size_t max_B,
                            size_t max_C, cudaStream_t stream) {
  return ggemm_create_ex(out, max_problems, max_A, max_B, max_C, stream, 32);
}

static double k_inflation(int min_k) {
  double f = 1.0;
  for (int k = min_k; k < min_k + 32; ++k) f = std::max(f, (double)align_up((size_t)k, 32) / k);
  return f;
}

extern "C" int ggemm_create_ex(ggemm_handle_t* out, int max_problems, size_t max_A,
                               size_t max_B, size_t max_C, cudaStream_t stream, int min_k) {
  if (!out || max_problems <= 0 || min_k < 1) return GGEMM_ERR_INVALID;
  *out = nullptr;
  ggemm_handle_t h = new (std::nothrow) ggemm_handle_s();
  if (!h) return GGEMM_ERR_ALLOC;
#define FAIL(code)     \
  do {                 \
    ggemm_destroy(h);  \
    return (code);     \
  } while (0)
#define CUA(x)                                       \
  do {                                               \
    if ((x) != cudaSuccess) FAIL(GGEMM_ERR_ALLOC);   \
  } while (0)
  h->stream = stream;
  h->max_problems = max_problems;
  h->max_A = max_A;
  h->max_B = max_B;
  h->max_C = max_C;
  h->min_k = min_k;
  const size_t P = (size_t)max_problems;

  cudaDeviceProp prop;
  if (cudaGetDevice(&h->device) != cudaSuccess ||
      cudaGetDeviceProperties(&prop, h->device) != cudaSuccess)
    FAIL(GGEMM_ERR_CUDA);
  h->num_sms = prop.multiProcessorCount;
  device_model_init(&h->dm, h->num_sms);
  h->rho_budget = env_rho_budget();
  if (upload_tables_current_device() != 0) FAIL(GGEMM_ERR_NUMERICS);

  if (cublasCreate(&h->cublas) != CUBLAS_STATUS_SUCCESS) FAIL(GGEMM_ERR_CUBLAS);
  h->cublas_ws_bytes = kCublasWsBytes;
  CUA(cudaMalloc(&h->cublas_ws, h->cublas_ws_bytes));
  if (cublasSetStream(h->cublas, stream) != CUBLAS_STATUS_SUCCESS ||
      cublasSetWorkspace(h->cublas, h->cublas_ws, h->cublas_ws_bytes) != CUBLAS_STATUS_SUCCESS ||
      cublasSetPointerMode(h->cublas, CUBLAS_POINTER_MODE_HOST) != CUBLAS_STATUS_SUCCESS ||
      cublasSetMathMode(h->cublas, CUBLAS_DEFAULT_MATH) != CUBLAS_STATUS_SUCCESS)
    FAIL(GGEMM_ERR_CUBLAS);

  // Workspace: the reference's sizing (21 planes, K padding inflation, per-problem slack) as
  // one pool, capped at a fraction of device memory; calls that need more run in chunks.
  const double infl = std::max(2.0, k_inflation(min_k));
  double want = kPlanesMax * (std::ceil(infl * (double)max_A) + (double)P * 2048) +
                kPlanesMax * (std::ceil(infl * (double)max_B) + (double)P * 2048) +
                4.0 * kPlanesMax * ((double)max_C + (double)P * 64);
  {
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    double frac = 0.55;
    if (const char* e = std::getenv("GGEMM_WORKSPACE_FRACTION")) {
      const double v = std::atof(e);
      if (v > 0.0 && v <= 0.95) frac = v;
    }
    want = std::min(want, frac * (double)total_b);
  }
  h->pool_cap = align_up(std::max<size_t>((size_t)want, 1 << 18), kAlign);
  CUA(cudaMalloc(&h->pool, h->pool_cap));
  CUA(cudaMalloc(&h->counters, sizeof(DevCounters)));
  CUA(cudaMemsetAsync(h->counters, 0, sizeof(DevCounters), stream));

  // Descriptor blob: worst case per problem (2 prep descriptors, 21 per-plane jobs for
  // EMU_LOOP, 1 reconstruct descriptor, prefixes, native pointers), plus alignment.
  const size_t per_prob = 2 * sizeof(ggemm_prep_desc_t) + kPlanesMax * sizeof(GemmJob) +
                          sizeof(ggemm_recon_desc_t) + (2 + 2 * kPlanesMax + 2) * 8 +
                          3 * sizeof(void*) + 4 * 64;
  h->blob_cap = align_up(P * per_prob + 64 * 1024, kAlign);
  for (int s = 0; s < 2; ++s) {
    CUA(cudaHostAlloc(&h->h_blob[s], h->blob_cap, cudaHostAllocMapped | cudaHostAllocPortable));
    void* dev_view = nullptr;
    CUA(cudaHostGetDevicePointer(&dev_view, h->h_blob[s], 0));
    h->h_blob_dev[s] = dev_view;
    CUA(cudaEventCreateWithFlags(&h->slot_done[s], cudaEventDisableTiming));
    CUA(cudaEventRecord(h->slot_done[s], stream));
  }
  CUA(cudaMalloc(&h->d_blob[0], h->blob_cap));

  try {
    h->plan.resize(P);
    h->memo.resize(plan_memo_cap(max_problems));
    for (auto* v : {&h->emu, &h->nat, &h->order, &h->ua_of, &h->ub_of, &h->ua_rep, &h->ub_rep,
                    &h->ua_n, &h->ub_n, &h->ua_chunk, &h->ub_chunk})
      v->resize(P);
    for (auto* v : {&h->ua_img, &h->ub_img, &h->ua_ws, &h->ub_ws, &h->c32_off, &h->pa_img,
                    &h->pb_img, &h->pa_ws, &h->pb_ws})
      v->resize(P);
    h->pa_new.resize(P);
    for (auto* v : {&h->pair_m, &h->pair_n, &h->pair_k, &h->pair_p}) v->resize(P);
    h->pb_new.resize(P);
    h->chunks.reserve(P + 1);
    h->ngroups.reserve(P);
    if (h->reuse.reserve(max_problems) != 0) FAIL(GGEMM_ERR_INVALID);
  } catch (...) {
    FAIL(GGEMM_ERR_ALLOC);
  }
  if (const char* e = std::getenv("GGEMM_REUSE_PROMOTE")) h->reuse_promote = std::atoi(e) == 1;
  if (const char* e = std::getenv("GGEMM_STATS_REPAIR")) h->stats_repair = std::atoi(e) == 1;
  if (const char* e = std::getenv("GGEMM_GEMM_PAIR")) {
    const int v = std::atoi(e);
    h->gemm_pair = (v == 0 || v == 1) ? v : -1;
  }
  if (cudaStreamSynchronize(stream) != cudaSuccess) FAIL(GGEMM_ERR_CUDA);
#undef CUA
#undef FAIL
  *out = h;
  return GGEMM_OK;
}

extern "C" int ggemm_grouped_dgemm(ggemm_handle_t h, ggemm_path_t path,
                                   const ggemm_config_t* cfg, const ggemm_problem_t* problems,
                                   int num_problems, ggemm_stats_t* stats) {
  ggemm_stats_t local;
  ggemm_stats_t* st = stats ? stats : &local;
  std::memset(st, 0, sizeof(*st));
  st->num_problems = num_problems;
  st->num_repaired = st->num_uncertified = st->num_safety_fallback = -1;
  if (!h) return GGEMM_ERR_INVALID;
  int r = validate_call(h, problems, num_problems);
  if (r) return r;
  static const ggemm_config_t kDefault = {0, 1e-15, 1, 0};
  if (!cfg) cfg = &kDefault;
  if (cfg->num_moduli < 0 || cfg->num_moduli == 1 || cfg->num_moduli > GGEMM_MAX_MODULI)
    return GGEMM_ERR_INVALID;
  const int repair = stage_repair_mode(path, cfg);
  if (repair < 0) return GGEMM_ERR_INVALID;
  if (cudaSetDevice(h->device) != cudaSuccess) return GGEMM_ERR_CUDA;
  switch (path) {
    case GGEMM_PATH_NATIVE_LOOP: return path_native(h, false, problems, num_problems, st);
    case GGEMM_PATH_NATIVE_GROUPED: return path_native(h, true, problems, num_problems, st);
    case GGEMM_PATH_EMU_LOOP:
    case GGEMM_PATH_EMU_GROUPED:
    case GGEMM_PATH_AUTO:
    case GGEMM_PATH_EMU_GROUPED_REUSE:
    case GGEMM_PATH_EMU_LOOP_BATCHED:
      if ((r = counters_reset(h))) return r;
      r = path_emu(h, path, cfg, problems, num_problems, st, repair);
      if (!r) r = counters_read(h, st);
      return r;
    default: return GGEMM_ERR_INVALID;
  }
}

extern "C" int ggemm_set_stage_events(ggemm_handle_t h, cudaEvent_t* events) {
  if (!h) return GGEMM_ERR_INVALID;
  if (!events) {
    h->stage_ev_on = false;
    return GGEMM_OK;
  }
  for (int i = 0; i < 4; ++i) {
    if (!events[i]) return GGEMM_ERR_INVALID;
    h->stage_ev[i] = events[i];
  }
  h->stage_ev_on = true;
  return GGEMM_OK;
}

extern "C" int ggemm_device_status(ggemm_handle_t h) {
  if (!h) return -1;
  DevCounters c{};
  if (cudaSetDevice(h->device) != cudaSuccess ||
      cudaMemcpyAsync(&c, h->counters, sizeof c, cudaMemcpyDeviceToHost, h->stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess)
    return -1;
  return (int)c.status;
}
