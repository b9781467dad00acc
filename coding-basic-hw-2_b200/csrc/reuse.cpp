// reuse.cpp -- see reuse.hpp.
//
// Design: unique operands are the runs of equal keys in the emulated problems sorted by
// (key, problem index); a run's first problem is its representative, and runs are numbered by
// their representative's position, which is the order of first appearance.  PROMOTE then labels
// the connected components of the bipartite graph "unique A -- problem -- unique B" with a
// breadth-first walk over an adjacency list in compressed (offset / edge) form, and gives every
// operand and problem of a component the component's largest moduli count.  All scratch is sized
// in reserve(); build() allocates nothing.
#include "reuse.hpp"

#include <algorithm>

namespace g2 {
namespace {

// Operand key of problem p: (pointer, leading dimension, rows, k) and, under EXACT_N, N.
struct KeyA {
  static const void* ptr(const ggemm_problem_t& p) { return p.A; }
  static int ld(const ggemm_problem_t& p) { return p.lda; }
  static int rows(const ggemm_problem_t& p) { return p.m; }
};
struct KeyB {
  static const void* ptr(const ggemm_problem_t& p) { return p.B; }
  static int ld(const ggemm_problem_t& p) { return p.ldb; }
  static int rows(const ggemm_problem_t& p) { return p.n; }
};

template <typename K>
bool key_less(const ggemm_problem_t& a, int na, const ggemm_problem_t& b, int nb) {
  const uintptr_t pa = (uintptr_t)K::ptr(a), pb = (uintptr_t)K::ptr(b);
  if (pa != pb) return pa < pb;
  if (K::ld(a) != K::ld(b)) return K::ld(a) < K::ld(b);
  if (K::rows(a) != K::rows(b)) return K::rows(a) < K::rows(b);
  if (a.k != b.k) return a.k < b.k;
  return na < nb;
}

// Numbers the unique operands of kind K among the `ne` emulated problems emu[0..ne):
// prob_id[g] receives the id, rep[id] the first problem, nmod[id] the largest N of its problems.
// key_n[g] is the N that takes part in the key (0 when N is not part of it).  Returns the count.
template <typename K>
int number_operands(const ggemm_problem_t* probs, const int* nmod_in, const int* key_n,
                    const int* emu, int ne, int* order, int* run_first, int* prob_id, int* rep,
                    int* nmod) {
  std::copy(emu, emu + ne, order);
  std::sort(order, order + ne, [&](int x, int y) {
    if (key_less<K>(probs[x], key_n[x], probs[y], key_n[y])) return true;
    if (key_less<K>(probs[y], key_n[y], probs[x], key_n[x])) return false;
    return x < y;
  });
  // run_first[g]: the first (smallest-index) problem with g's key
  for (int i = 0; i < ne; ++i) {
    const int g = order[i];
    const bool starts = i == 0 || key_less<K>(probs[order[i - 1]], key_n[order[i - 1]], probs[g],
                                              key_n[g]);
    run_first[g] = starts ? g : run_first[order[i - 1]];
  }
  // ids in order of first appearance
  int count = 0;
  for (int i = 0; i < ne; ++i) {
    const int g = emu[i];
    if (run_first[g] == g) {
      rep[count] = g;
      nmod[count] = 0;
      prob_id[g] = count++;
    }
  }
  for (int i = 0; i < ne; ++i) {
    const int g = emu[i];
    const int id = prob_id[run_first[g]];
    prob_id[g] = id;
    nmod[id] = std::max(nmod[id], nmod_in[g]);
  }
  return count;
}

}  // namespace

int ReuseArena::reserve(int max_problems) {
  if (max_problems < 1) max_problems = 1;
  if (max_problems > (1 << 29)) {
    cap_ = 0;
    return 1;
  }
  cap_ = max_problems;
  const size_t P = (size_t)cap_;
  for (auto* v : {&ua_rep_, &ua_nmod_, &ub_rep_, &ub_nmod_, &prob_a_, &prob_b_, &eff_, &emu_,
                  &order_, &run_first_, &key_n_})
    v->assign(P, 0);
  offs_.assign(2 * P + 1, 0);
  edges_.assign(2 * P, 0);
  comp_.assign(2 * P, 0);
  queue_.assign(2 * P, 0);
  cmax_.assign(2 * P, 0);
  return 0;
}

ReuseResult ReuseArena::build(const ggemm_problem_t* probs, int num, const int* nmod,
                              ReusePolicy policy) {
  ReuseResult r{};
  if (num < 0 || (num > 0 && (!probs || !nmod))) {
    r.status = 2;
    return r;
  }
  if (num > cap_) {
    r.status = 1;
    return r;
  }
  const bool exact = policy == kReuseExactN;
  int ne = 0;
  for (int g = 0; g < num; ++g) {
    if (nmod[g] > 0) {
      emu_[ne++] = g;
      eff_[g] = nmod[g];
      key_n_[g] = exact ? nmod[g] : 0;
    } else {
      prob_a_[g] = prob_b_[g] = -1;
      eff_[g] = 0;
    }
  }
  const int ua = number_operands<KeyA>(probs, nmod, key_n_.data(), emu_.data(), ne, order_.data(),
                                       run_first_.data(), prob_a_.data(), ua_rep_.data(),
                                       ua_nmod_.data());
  const int ub = number_operands<KeyB>(probs, nmod, key_n_.data(), emu_.data(), ne, order_.data(),
                                       run_first_.data(), prob_b_.data(), ub_rep_.data(),
                                       ub_nmod_.data());
  int promoted = 0;
  if (!exact && ne > 0) {
    // Graph nodes: unique A ids [0, ua), unique B ids [ua, ua + ub); one edge per problem.
    const int V = ua + ub;
    int* off = offs_.data();
    int* adj = edges_.data();
    std::fill(off, off + V + 1, 0);
    for (int i = 0; i < ne; ++i) {
      const int g = emu_[i];
      ++off[prob_a_[g] + 1];
      ++off[ua + prob_b_[g] + 1];
    }
    for (int v = 0; v < V; ++v) off[v + 1] += off[v];
    int* fill = queue_.data();  // insertion cursors (the queue is free until the walk)
    std::copy(off, off + V, fill);
    for (int i = 0; i < ne; ++i) {
      const int g = emu_[i];
      const int a = prob_a_[g], b = ua + prob_b_[g];
      adj[fill[a]++] = b;
      adj[fill[b]++] = a;
    }
    int* comp = comp_.data();
    int* best = cmax_.data();
    std::fill(comp, comp + V, -1);
    int ncomp = 0;
    for (int s = 0; s < V; ++s) {
      if (comp[s] >= 0) continue;
      int head = 0, tail = 0, m = 0;
      queue_[tail++] = s;
      comp[s] = ncomp;
      while (head < tail) {
        const int v = queue_[head++];
        m = std::max(m, v < ua ? ua_nmod_[v] : ub_nmod_[v - ua]);
        for (int e = off[v]; e < off[v + 1]; ++e)
          if (comp[adj[e]] < 0) {
            comp[adj[e]] = ncomp;
            queue_[tail++] = adj[e];
          }
      }
      best[ncomp++] = m;
    }
    for (int u = 0; u < ua; ++u) ua_nmod_[u] = best[comp[u]];
    for (int u = 0; u < ub; ++u) ub_nmod_[u] = best[comp[ua + u]];
    for (int i = 0; i < ne; ++i) {
      const int g = emu_[i];
      const int N = ua_nmod_[prob_a_[g]];
      promoted += N > eff_[g];
      eff_[g] = N;
    }
  }
  r.status = 0;
  r.num_ua = ua;
  r.num_ub = ub;
  r.num_emu = ne;
  r.num_promoted = promoted;
  r.ua_rep = ua_rep_.data();
  r.ua_nmod = ua_nmod_.data();
  r.ub_rep = ub_rep_.data();
  r.ub_nmod = ub_nmod_.data();
  r.prob_a = prob_a_.data();
  r.prob_b = prob_b_.data();
  r.eff_nmod = eff_.data();
  return r;
}

}  // namespace g2
