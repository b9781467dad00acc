// crt.hpp -- moduli and CRT constants of the Ozaki-II emulation (host side), plus the compact
// per-device copy the kernels read from __constant__ memory.
//
// The moduli list and every derived constant must equal the reference's
// (src/moduli.h:39-58, 124-181): the residues, CRT integers and FP64 outputs are compared bit
// for bit.  The derivation here is this library's own (a small fixed-width big integer).
#pragma once
#include <cstddef>
#include <cstdint>

namespace g2 {

constexpr int kMaxModuli = 20;
constexpr int kS2Bits = 18;
constexpr int kShiftNonfinite = -2147483647 - 1;  // row / column contains NaN or Inf
constexpr int kShiftZero = -2147483647;           // row / column is all zero (abs shift)
constexpr int kByteDigits = 12;                   // bytes of trunc(2^s a) as 96-bit integer

// Host tables, field for field the content of the reference's oz2_crt_tables.
struct CrtTables {
  int32_t p[kMaxModuli];
  uint32_t magic[kMaxModuli];
  uint8_t pow2[kMaxModuli][128];
  uint64_t s1[kMaxModuli + 1][kMaxModuli];
  uint32_t s2[kMaxModuli + 1][kMaxModuli];
  int32_t qinv[kMaxModuli + 1][kMaxModuli];
  int64_t P1[kMaxModuli + 1];
  double P2[kMaxModuli + 1];
  double inv_Pu[kMaxModuli + 1];
  int32_t log2_u1[kMaxModuli + 1];
  double T[kMaxModuli + 1];
  double log2P[kMaxModuli + 1];
};

// What the kernels use.
struct DevTables {
  // prep: residues of a byte-digit expansion (tensor-core dot, then an FP32 rounding step)
  float pf[kMaxModuli];
  float invpf[kMaxModuli];
  int8_t wb[kMaxModuli][kByteDigits];  // 2^(8 i) mod p_l, symmetric representative
  int8_t wbq[kMaxModuli + 1][kMaxModuli][kByteDigits];  // q_l 2^(8 i) mod p_l (N moduli)
  double T[kMaxModuli + 1];
  // reconstruct
  uint32_t p[kMaxModuli];
  uint32_t magic[kMaxModuli];
  uint32_t qinv[kMaxModuli + 1][kMaxModuli];
  uint64_t s1[kMaxModuli + 1][kMaxModuli];
  uint32_t s2[kMaxModuli + 1][kMaxModuli];
  int64_t P1[kMaxModuli + 1];
  double P2[kMaxModuli + 1];
  double inv_Pu[kMaxModuli + 1];
  int32_t log2_u1[kMaxModuli + 1];
};

// Built once per process (thread-safe); status 0 on success.
const CrtTables& crt_tables(int* status = nullptr);
void make_dev_tables(const CrtTables& t, DevTables* d);

// A-priori normwise bound of one entry relative to ||a_i|| ||b_j|| (reference
// src/ozaki2_numerics.cu:639-650) and the two N selections (:652-673).
double error_bound(int k, int num_moduli);
int choose_num_moduli(int k, double target_rel_err);
int choose_num_moduli_cw(int k, double rho_budget);

constexpr int kMaxKExact = 131040;  // kp * 128^2 < 2^31 for exact int32 accumulation

}  // namespace g2
