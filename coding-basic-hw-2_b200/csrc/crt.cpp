// crt.cpp -- host construction of the CRT constants (see crt.hpp).
#include "crt.hpp"

#include <array>
#include <cmath>
#include <cstring>
#include <mutex>

namespace g2 {
namespace {

// Moduli: the 16 INT8 moduli of Ozaki scheme II (Ozaki, Uchino, Imamura 2025, eq. 19) and the
// primes 181, 179, 173, 167; identical to the reference list (src/moduli.h:39-41).
constexpr int kModuli[kMaxModuli] = {256, 255, 253, 251, 247, 239, 233, 229, 227, 223,
                                     217, 211, 199, 197, 193, 191, 181, 179, 173, 167};

// Unsigned integer of 256 bits as eight 32-bit limbs, least significant first.
struct Wide {
  std::array<uint32_t, 8> w{};
  static Wide of(uint64_t v) {
    Wide r;
    r.w[0] = (uint32_t)v;
    r.w[1] = (uint32_t)(v >> 32);
    return r;
  }
  void mul(uint32_t m) {
    uint64_t c = 0;
    for (auto& x : w) {
      const uint64_t t = (uint64_t)x * m + c;
      x = (uint32_t)t;
      c = t >> 32;
    }
  }
  uint32_t divmod(uint32_t d, Wide* q) const {
    uint64_t r = 0;
    Wide out;
    for (int i = 7; i >= 0; --i) {
      const uint64_t cur = (r << 32) | w[i];
      out.w[i] = (uint32_t)(cur / d);
      r = cur % d;
    }
    if (q) *q = out;
    return (uint32_t)r;
  }
  int bit(int i) const { return (i < 0 || i >= 256) ? 0 : (int)((w[i >> 5] >> (i & 31)) & 1u); }
  int bits() const {
    for (int i = 255; i >= 0; --i)
      if (bit(i)) return i + 1;
    return 0;
  }
  Wide shr(int s) const {  // floor(x / 2^s); s < 0 shifts left
    Wide r;
    for (int i = 0; i < 256; ++i)
      if (bit(i + s)) r.w[i >> 5] |= 1u << (i & 31);
    return r;
  }
  Wide low(int s) const {  // x mod 2^s
    Wide r;
    for (int i = 0; i < s && i < 256; ++i)
      if (bit(i)) r.w[i >> 5] |= 1u << (i & 31);
    return r;
  }
  uint64_t u64() const { return (uint64_t)w[0] | ((uint64_t)w[1] << 32); }
  // Horner from the top 32-bit limb in x87 extended precision, then one rounding to double:
  // the same evaluation as the reference (src/moduli.h:108-111), so P2 and T round identically.
  double to_double() const {
    long double v = 0;
    int top = 7;
    while (top > 0 && w[top] == 0) --top;
    for (int i = top; i >= 0; --i) v = v * 4294967296.0L + (long double)w[i];
    return (double)v;
  }
};

int build(CrtTables* t) {
  std::memset(t, 0, sizeof(*t));
  for (int a = 0; a < kMaxModuli; ++a)
    for (int b = a + 1; b < kMaxModuli; ++b) {
      int x = kModuli[a], y = kModuli[b];
      while (y) { const int r = x % y; x = y; y = r; }
      if (x != 1) return 1;
    }
  for (int l = 0; l < kMaxModuli; ++l) {
    const uint32_t p = (uint32_t)kModuli[l];
    t->p[l] = (int32_t)p;
    t->magic[l] = (uint32_t)((1ull << 32) / p);
    uint32_t v = 1u % p;
    for (int e = 0; e < 128; ++e) {
      t->pow2[l][e] = (uint8_t)v;
      v = (v << 1) % p;
    }
  }
  for (int N = 1; N <= kMaxModuli; ++N) {
    Wide P = Wide::of(1);
    for (int l = 0; l < N; ++l) P.mul((uint32_t)kModuli[l]);
    Wide M[kMaxModuli];
    int maxbits = 0;
    for (int l = 0; l < N; ++l) {
      const uint32_t p = (uint32_t)kModuli[l];
      if (P.divmod(p, &M[l]) != 0) return 3;
      const uint32_t mr = M[l].divmod(p, nullptr);
      int inv = -1;
      for (uint32_t x = 0; x < p && inv < 0; ++x)
        if ((mr * x) % p == 1u % p) inv = (int)x;
      if (inv < 0) return 4;
      t->qinv[N][l] = inv;
      if (M[l].bits() > maxbits) maxbits = M[l].bits();
    }
    const int sh = maxbits - 49;  // u1 = 2^sh keeps every M_l / u1 below 2^49
    t->log2_u1[N] = sh;
    for (int l = 0; l < N; ++l) {
      const uint64_t s1 = M[l].shr(sh).u64();
      uint64_t s2 = 0;
      if (sh >= kS2Bits) {
        const Wide lo = M[l].low(sh);
        s2 = lo.shr(sh - kS2Bits).u64() + (uint64_t)lo.bit(sh - kS2Bits - 1);  // half up
      } else if (sh >= 0) {
        s2 = M[l].low(sh).u64() << (kS2Bits - sh);
      }
      if (s2 > (1u << kS2Bits)) return 5;
      if (s1 >= (1ull << 49)) return 6;
      t->s1[N][l] = s1;
      t->s2[N][l] = (uint32_t)s2;
    }
    const Wide P1 = P.shr(sh);
    if (P1.bits() > 57) return 7;
    t->P1[N] = (int64_t)P1.u64();
    t->P2[N] = sh > 0 ? std::ldexp(P.low(sh).to_double(), -sh) : 0.0;
    t->inv_Pu[N] = 1.0 / ((double)t->P1[N] + t->P2[N]);
    const double Pd = P.to_double();
    t->log2P[N] = std::log2(Pd);
    t->T[N] = std::sqrt(Pd * 0.5 * (1.0 - std::ldexp(1.0, -20))) * (1.0 - std::ldexp(1.0, -40));
  }
  return 0;
}

}  // namespace

const CrtTables& crt_tables(int* status) {
  static CrtTables tab;
  static int st = -1;
  static std::once_flag once;
  std::call_once(once, [] { st = build(&tab); });
  if (status) *status = st;
  return tab;
}

void make_dev_tables(const CrtTables& t, DevTables* d) {
  std::memset(d, 0, sizeof(*d));
  for (int l = 0; l < kMaxModuli; ++l) {
    const uint32_t p = (uint32_t)t.p[l];
    d->pf[l] = (float)p;
    d->invpf[l] = 1.0f / (float)p;
    uint32_t w = 1u % p;
    for (int i = 0; i < kByteDigits; ++i) {
      d->wb[l][i] = (int8_t)(2 * w > p ? (int)w - (int)p : (int)w);
      w = (w << 8) % p;
    }
    d->p[l] = p;
    d->magic[l] = t.magic[l];
  }
  for (int N = 0; N <= kMaxModuli; ++N) {
    d->T[N] = t.T[N];
    for (int l = 0; l < kMaxModuli; ++l) {
      d->qinv[N][l] = (uint32_t)t.qinv[N][l];
      const uint32_t p = (uint32_t)t.p[l];
      for (int i = 0; i < kByteDigits; ++i) {
        const uint32_t w = (uint32_t)(d->wb[l][i] < 0 ? d->wb[l][i] + (int)p : d->wb[l][i]);
        const uint32_t s = (uint32_t)((uint64_t)w * (uint32_t)t.qinv[N][l] % p);
        d->wbq[N][l][i] = (int8_t)(2 * s > p ? (int)s - (int)p : (int)s);
      }
      d->s1[N][l] = t.s1[N][l];
      d->s2[N][l] = t.s2[N][l];
    }
    d->P1[N] = t.P1[N];
    d->P2[N] = t.P2[N];
    d->inv_Pu[N] = t.inv_Pu[N];
    d->log2_u1[N] = t.log2_u1[N];
  }
}

double error_bound(int k, int num_moduli) {
  int st;
  const CrtTables& t = crt_tables(&st);
  if (st != 0 || num_moduli < 1 || num_moduli > kMaxModuli || k < 0) return INFINITY;
  const double T = t.T[num_moduli];
  const double T2 = T * T;
  const double kk = (double)k;
  const double u = std::ldexp(1.0, -53);
  const double u1 = std::ldexp(1.0, t.log2_u1[num_moduli]);
  return 4.0 * std::sqrt(kk) / T + 4.0 * kk / T2 +
         4.0 * u1 * (num_moduli * 255.0 * std::ldexp(1.0, -19) + std::ldexp(1.0, -10)) / T2 + u;
}

int choose_num_moduli(int k, double target_rel_err) {
  if (k < 0 || k > kMaxKExact) return -1;
  for (int N = 2; N <= kMaxModuli; ++N)
    if (error_bound(k, N) <= target_rel_err) return N;
  return -1;
}

int choose_num_moduli_cw(int k, double rho_budget) {
  if (k < 0 || k > kMaxKExact) return -1;
  if (rho_budget < 1.0) rho_budget = 1.0;
  const double u = std::ldexp(1.0, -53);
  const double budget = 0.5 * (k > 2 ? (double)(k - 2) : 1.0) * u;
  for (int N = 2; N <= kMaxModuli; ++N)
    if ((error_bound(k, N) - u) * rho_budget <= budget) return N;
  return kMaxModuli;
}

}  // namespace g2
