// reuse.hpp -- detection of shared A / B operands across a group (host only, no allocation
// after reserve()).  Semantics of the reference pass (src/operand_reuse.h:1-85,
// src/operand_reuse.cpp:47-141):
//   A key = (A pointer, lda, m, k), B key = (B pointer, ldb, n, k); under EXACT_N the moduli
//   count is part of the key.  Unique operands are numbered in order of first appearance.
//   PROMOTE treats problems that share an operand as connected and runs every problem of a
//   connected component with the component's largest N (the prep shift depends on N through
//   T_N).  The implementation (reuse.cpp) sorts keys and walks components breadth-first.
#pragma once
#include <cstdint>
#include <vector>

#include "ggemm.h"

namespace g2 {

enum ReusePolicy { kReuseExactN = 0, kReusePromote = 1 };

struct ReuseResult {
  int status;  // 0 ok, 1 capacity, 2 invalid
  int num_ua, num_ub, num_emu, num_promoted;
  const int* ua_rep;   // [num_ua] first problem carrying unique A u
  const int* ua_nmod;  // [num_ua] moduli to prep A u with
  const int* ub_rep;
  const int* ub_nmod;
  const int* prob_a;    // [num] unique-A id of problem g (-1: not emulated)
  const int* prob_b;
  const int* eff_nmod;  // [num] moduli problem g runs with
};

class ReuseArena {
 public:
  int reserve(int max_problems);  // 0 ok
  ReuseResult build(const ggemm_problem_t* probs, int num, const int* nmod, ReusePolicy policy);
  int capacity() const { return cap_; }

 private:
  int cap_ = 0;
  std::vector<int> ua_rep_, ua_nmod_, ub_rep_, ub_nmod_, prob_a_, prob_b_, eff_;
  std::vector<int> emu_, order_, run_first_, key_n_;     // per problem
  std::vector<int> offs_, edges_, comp_, queue_, cmax_;  // operand graph (PROMOTE)
};

}  // namespace g2
