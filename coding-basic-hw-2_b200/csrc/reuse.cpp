// reuse.cpp -- see reuse.hpp.
#include "reuse.hpp"

#include <algorithm>

namespace g2 {
namespace {

inline uint64_t mix(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
inline uint32_t key_hash(const void* p, int ld, int rows, int k, int n_key, uint64_t salt) {
  uint64_t h = mix((uint64_t)(uintptr_t)p ^ salt);
  h = mix(h ^ (((uint64_t)(uint32_t)ld << 32) | (uint32_t)rows));
  h = mix(h ^ (((uint64_t)(uint32_t)k << 32) | (uint32_t)n_key));
  return (uint32_t)h;
}
inline int root(int* par, int x) {
  while (par[x] != x) {
    par[x] = par[par[x]];
    x = par[x];
  }
  return x;
}

}  // namespace

int ReuseArena::reserve(int max_problems) {
  if (max_problems < 1) max_problems = 1;
  if (max_problems > (1 << 30)) {
    cap_ = 0;
    return 1;
  }
  cap_ = max_problems;
  uint32_t sz = 1;
  while (sz < 2u * (uint32_t)max_problems) sz <<= 1;
  mask_ = sz - 1;
  gen_ = 0;
  a_stamp_.assign(sz, 0);
  b_stamp_.assign(sz, 0);
  a_slot_.assign(sz, -1);
  b_slot_.assign(sz, -1);
  for (auto* v : {&ua_rep_, &ua_nmod_, &ub_rep_, &ub_nmod_, &prob_a_, &prob_b_, &eff_})
    v->assign(cap_, 0);
  parent_.assign(2 * (size_t)cap_, 0);
  cmax_.assign(2 * (size_t)cap_, 0);
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
  if (++gen_ == 0) {
    std::fill(a_stamp_.begin(), a_stamp_.end(), 0u);
    std::fill(b_stamp_.begin(), b_stamp_.end(), 0u);
    gen_ = 1;
  }
  const bool exact = policy == kReuseExactN;
  int ua = 0, ub = 0, ne = 0;
  for (int g = 0; g < num; ++g) {
    const int N = nmod[g];
    if (N <= 0) {
      prob_a_[g] = prob_b_[g] = -1;
      eff_[g] = 0;
      continue;
    }
    ++ne;
    const ggemm_problem_t& p = probs[g];
    const int nkey = exact ? N : 0;
    // unique A
    for (uint32_t s = key_hash(p.A, p.lda, p.m, p.k, nkey, 0) & mask_;; s = (s + 1) & mask_) {
      if (a_stamp_[s] != gen_) {
        a_stamp_[s] = gen_;
        a_slot_[s] = ua;
        ua_rep_[ua] = g;
        ua_nmod_[ua] = N;
        prob_a_[g] = ua++;
        break;
      }
      const int c = a_slot_[s];
      const ggemm_problem_t& q = probs[ua_rep_[c]];
      if (q.A == p.A && q.lda == p.lda && q.m == p.m && q.k == p.k &&
          (!exact || ua_nmod_[c] == N)) {
        ua_nmod_[c] = std::max(ua_nmod_[c], N);
        prob_a_[g] = c;
        break;
      }
    }
    // unique B
    for (uint32_t s = key_hash(p.B, p.ldb, p.n, p.k, nkey, 0x5BD1E995ull) & mask_;;
         s = (s + 1) & mask_) {
      if (b_stamp_[s] != gen_) {
        b_stamp_[s] = gen_;
        b_slot_[s] = ub;
        ub_rep_[ub] = g;
        ub_nmod_[ub] = N;
        prob_b_[g] = ub++;
        break;
      }
      const int c = b_slot_[s];
      const ggemm_problem_t& q = probs[ub_rep_[c]];
      if (q.B == p.B && q.ldb == p.ldb && q.n == p.n && q.k == p.k &&
          (!exact || ub_nmod_[c] == N)) {
        ub_nmod_[c] = std::max(ub_nmod_[c], N);
        prob_b_[g] = c;
        break;
      }
    }
    eff_[g] = N;
  }
  int promoted = 0;
  if (!exact && ne > 0) {
    int* par = parent_.data();
    int* mx = cmax_.data();
    const int ob = cap_;  // B nodes follow the A nodes
    for (int u = 0; u < ua; ++u) { par[u] = u; mx[u] = ua_nmod_[u]; }
    for (int u = 0; u < ub; ++u) { par[ob + u] = ob + u; mx[ob + u] = ub_nmod_[u]; }
    for (int g = 0; g < num; ++g) {
      if (prob_a_[g] < 0) continue;
      int x = root(par, prob_a_[g]), y = root(par, ob + prob_b_[g]);
      if (x == y) continue;
      if (x > y) std::swap(x, y);
      par[y] = x;
      mx[x] = std::max(mx[x], mx[y]);
    }
    for (int u = 0; u < ua; ++u) ua_nmod_[u] = mx[root(par, u)];
    for (int u = 0; u < ub; ++u) ub_nmod_[u] = mx[root(par, ob + u)];
    for (int g = 0; g < num; ++g) {
      if (prob_a_[g] < 0) continue;
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
