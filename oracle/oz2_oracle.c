/* oz2_oracle.c -- CPU restatement of the Ozaki-II grouped FP64 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): see oz2_oracle.h.
 * Every routine cites the reference function it restates (paths relative to the reference
 * project).  The floating-point operations are spelled out one by one (explicit fma() where
 * the reference computes a fused multiply-add) because the CUDA path must reproduce them bit
 * for bit; the integer parts (residues, CRT sums) are restated from the mathematics.
 */
#include "oz2_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* Moduli of the reference (src/moduli.h:39-41): the 16 INT8 moduli of Ozaki scheme II,
 * extended by the primes 181, 179, 173, 167.  This list is data the two implementations must
 * share exactly (the CRT integers depend on it). */
static const int kModuli[OZO_MAX_MODULI] = {256, 255, 253, 251, 247, 239, 233, 229, 227, 223,
                                            217, 211, 199, 197, 193, 191, 181, 179, 173, 167};

/* ------------------------------------------------------------------ fixed-size big integers
 * Non-negative integers up to 8 x 32 bits (P_20 < 2^155), little-endian 32-bit limbs. */
#define BN_LIMBS 8
typedef struct {
  uint32_t w[BN_LIMBS];
} bn;

static void bn_set(bn* a, uint64_t v) {
  memset(a, 0, sizeof(*a));
  a->w[0] = (uint32_t)v;
  a->w[1] = (uint32_t)(v >> 32);
}
static void bn_mul_u32(bn* a, uint32_t m) {
  uint64_t carry = 0;
  for (int i = 0; i < BN_LIMBS; ++i) {
    uint64_t t = (uint64_t)a->w[i] * m + carry;
    a->w[i] = (uint32_t)t;
    carry = t >> 32;
  }
}
/* q = a / d, returns a mod d. */
static uint32_t bn_divmod_u32(const bn* a, uint32_t d, bn* q) {
  uint64_t r = 0;
  bn out;
  memset(&out, 0, sizeof(out));
  for (int i = BN_LIMBS - 1; i >= 0; --i) {
    uint64_t cur = (r << 32) | a->w[i];
    out.w[i] = (uint32_t)(cur / d);
    r = cur % d;
  }
  if (q) *q = out;
  return (uint32_t)r;
}
static int bn_bitlen(const bn* a) {
  for (int i = BN_LIMBS - 1; i >= 0; --i)
    if (a->w[i]) {
      int b = 0;
      uint32_t t = a->w[i];
      while (t) { ++b; t >>= 1; }
      return i * 32 + b;
    }
  return 0;
}
static int bn_bit(const bn* a, int i) {
  if (i < 0 || i >= 32 * BN_LIMBS) return 0;
  return (int)((a->w[i / 32] >> (i % 32)) & 1u);
}
/* floor(a / 2^s) (s >= 0) or a * 2^-s (s < 0). */
static void bn_shift_right(const bn* a, int s, bn* out) {
  bn r;
  memset(&r, 0, sizeof(r));
  for (int i = 0; i < 32 * BN_LIMBS; ++i) {
    int src = i + s;
    if (bn_bit(a, src)) r.w[i / 32] |= 1u << (i % 32);
  }
  *out = r;
}
/* a mod 2^s, s >= 0. */
static void bn_low_bits(const bn* a, int s, bn* out) {
  bn r;
  memset(&r, 0, sizeof(r));
  for (int i = 0; i < s && i < 32 * BN_LIMBS; ++i)
    if (bn_bit(a, i)) r.w[i / 32] |= 1u << (i % 32);
  *out = r;
}
static uint64_t bn_u64(const bn* a) { return (uint64_t)a->w[0] | ((uint64_t)a->w[1] << 32); }
/* Conversion used for P, P mod u1: Horner evaluation from the most significant 32-bit limb in
 * x87 extended precision, then one rounding to double.  The CRT constants P2 and T inherit
 * these roundings, so the evaluation order must be the reference's (src/moduli.h:108-111). */
static double bn_to_double(const bn* a) {
  long double v = 0;
  int top = BN_LIMBS - 1;
  while (top > 0 && a->w[top] == 0) --top;
  for (int i = top; i >= 0; --i) v = v * 4294967296.0L + (long double)a->w[i];
  return (double)v;
}
static int gcd_int(int a, int b) {
  while (b) { int t = a % b; a = b; b = t; }
  return a;
}

size_t ozo_tables_size(void) { return sizeof(ozo_tables); }

/* Restates oz2_build_crt_tables (src/moduli.h:124-181). */
int ozo_build_tables(ozo_tables* t) {
  memset(t, 0, sizeof(*t));
  for (int a = 0; a < OZO_MAX_MODULI; ++a)
    for (int b = a + 1; b < OZO_MAX_MODULI; ++b)
      if (gcd_int(kModuli[a], kModuli[b]) != 1) return 1;
  for (int l = 0; l < OZO_MAX_MODULI; ++l) {
    const int p = kModuli[l];
    if (p < 2 || p > 256) return 2;
    t->p[l] = p;
    t->magic[l] = (uint32_t)((1ull << 32) / (uint64_t)p);
    for (int e = 0; e < OZO_POW2_TABLE; ++e) {
      /* 2^e mod p */
      uint32_t v = 1u % (uint32_t)p;
      for (int q = 0; q < e; ++q) v = (v * 2u) % (uint32_t)p;
      t->pow2[l][e] = (uint8_t)v;
    }
  }
  for (int N = 1; N <= OZO_MAX_MODULI; ++N) {
    bn P;
    bn_set(&P, 1);
    for (int l = 0; l < N; ++l) bn_mul_u32(&P, (uint32_t)kModuli[l]);
    bn M[OZO_MAX_MODULI];
    int maxbits = 0;
    for (int l = 0; l < N; ++l) {
      const uint32_t p = (uint32_t)kModuli[l];
      if (bn_divmod_u32(&P, p, &M[l]) != 0) return 3;
      const uint32_t mr = bn_divmod_u32(&M[l], p, NULL);
      int inv = -1;
      for (uint32_t x = 0; x < p; ++x)
        if ((mr * x) % p == 1u % p) { inv = (int)x; break; }
      if (inv < 0) return 4;
      t->qinv[N][l] = inv;
      const int b = bn_bitlen(&M[l]);
      if (b > maxbits) maxbits = b;
    }
    const int sh = maxbits - 49; /* u1 = 2^sh so that every M_l / u1 < 2^49 */
    t->log2_u1[N] = sh;
    for (int l = 0; l < N; ++l) {
      bn hi;
      bn_shift_right(&M[l], sh, &hi);
      uint64_t s1 = bn_u64(&hi);
      uint64_t s2 = 0;
      if (sh >= OZO_S2_BITS) {
        bn low, top;
        bn_low_bits(&M[l], sh, &low);
        bn_shift_right(&low, sh - OZO_S2_BITS, &top);
        /* round half up on the first dropped bit */
        s2 = bn_u64(&top) + (uint64_t)bn_bit(&low, sh - OZO_S2_BITS - 1);
      } else if (sh >= 0) {
        bn low;
        bn_low_bits(&M[l], sh, &low);
        s2 = bn_u64(&low) << (OZO_S2_BITS - sh);
      }
      if (s2 > (1u << OZO_S2_BITS)) return 5;
      if (s1 >= (1ull << 49)) return 6;
      t->s1[N][l] = s1;
      t->s2[N][l] = (uint32_t)s2;
    }
    bn P1;
    bn_shift_right(&P, sh, &P1);
    if (bn_bitlen(&P1) > 57) return 7;
    t->P1[N] = (int64_t)bn_u64(&P1);
    if (sh > 0) {
      bn low;
      bn_low_bits(&P, sh, &low);
      t->P2[N] = ldexp(bn_to_double(&low), -sh);
    } else {
      t->P2[N] = 0.0;
    }
    t->inv_Pu[N] = 1.0 / ((double)t->P1[N] + t->P2[N]);
    const double Pd = bn_to_double(&P);
    t->log2P[N] = log2(Pd);
    t->T[N] = sqrt(Pd * 0.5 * (1.0 - ldexp(1.0, -20))) * (1.0 - ldexp(1.0, -40));
  }
  return 0;
}

static const ozo_tables* tables(void) {
  static ozo_tables tab;
  static int built = 0;
  if (!built) {
    ozo_build_tables(&tab);
    built = 1;
  }
  return &tab;
}

/* Restates oz2_error_bound (src/ozaki2_numerics.cu:639-650). */
double ozo_error_bound(int k, int num_moduli) {
  const ozo_tables* t = tables();
  if (num_moduli < 1 || num_moduli > OZO_MAX_MODULI || k < 0) return INFINITY;
  const double T = t->T[num_moduli];
  const double T2 = T * T;
  const double kk = (double)k;
  const double u = ldexp(1.0, -53);
  const double u1 = ldexp(1.0, t->log2_u1[num_moduli]);
  return 4.0 * sqrt(kk) / T + 4.0 * kk / T2 +
         4.0 * u1 * (num_moduli * 255.0 * ldexp(1.0, -19) + ldexp(1.0, -10)) / T2 + u;
}

/* Restates oz2_choose_num_moduli (src/ozaki2_numerics.cu:652-657). */
int ozo_choose_num_moduli(int k, double target_rel_err) {
  if (k < 0 || k > 131040) return -1;
  for (int N = 2; N <= OZO_MAX_MODULI; ++N)
    if (ozo_error_bound(k, N) <= target_rel_err) return N;
  return -1;
}

/* Restates oz2_choose_num_moduli_cw (src/ozaki2_numerics.cu:665-673). */
int ozo_choose_num_moduli_cw(int k, double rho_budget) {
  if (k < 0 || k > 131040) return -1;
  if (rho_budget < 1.0) rho_budget = 1.0;
  const double u = ldexp(1.0, -53);
  const double budget = 0.5 * (k > 2 ? (double)(k - 2) : 1.0) * u;
  for (int N = 2; N <= OZO_MAX_MODULI; ++N)
    if ((ozo_error_bound(k, N) - u) * rho_budget <= budget) return N;
  return OZO_MAX_MODULI;
}

/* ----------------------------------------------------------------------- element-level math
 * These follow src/ozaki2_numerics.cu:112-231 operation by operation. */

/* x * 2^e, one multiplication when |e| <= 1000, else three clamped steps (:112-122). */
static double mul_pow2(double x, int e) {
  if (e >= -1000 && e <= 1000) return x * ldexp(1.0, e);
  for (int r = 0; r < 3; ++r) {
    int ee = e < -1000 ? -1000 : (e > 1000 ? 1000 : e);
    x *= ldexp(1.0, ee);
    e -= ee;
  }
  return x;
}

/* Largest s with 2^s * nub <= T (:133-140). */
static int choose_shift(double nrm, int nrm_exp_add, double T) {
  int g, G;
  const double f = frexp(nrm, &g);
  const double F = frexp(T, &G);
  g += nrm_exp_add;
  return G - g - (f > F ? 1 : 0);
}

/* (:146-153) */
static int shift_from_norm(double maxabs, double ssq, int rescaled, double T) {
  if (isinf(maxabs) || isnan(ssq)) return OZO_SHIFT_NONFINITE;
  if (!(maxabs > 0.0)) return 0;
  const double margin = 1.0 + ldexp(1.0, -30);
  const double nm = sqrt(ssq * margin);
  const int add = rescaled ? ilogb(maxabs) : 0;
  return choose_shift(nm, add, T);
}

/* (:156-160) */
static int abs_shift(double maxabs, int sh) {
  if (sh == OZO_SHIFT_NONFINITE) return 0;
  if (!(maxabs > 0.0)) return OZO_SHIFT_ZERO;
  return 6 - ilogb(maxabs);
}

static int needs_rescale(double maxabs) {
  return maxabs > 0.0 && (maxabs > ldexp(1.0, 400) || maxabs < ldexp(1.0, -400));
}

/* Symmetric residue of the integer-valued double xt (|xt| < 2^81) modulo p, computed from the
 * exact binary expansion |xt| = M * 2^E: r = (M mod p) * (2^E mod p) mod p, negated for
 * xt < 0, mapped to [-(p-1)/2, (p-1)/2] for odd p and to [-128, 127] for p = 256. */
static int8_t sym_residue(double xt, int p) {
  const double ax = fabs(xt);
  uint64_t M;
  int E;
  if (ax < 9007199254740992.0) {
    M = (uint64_t)ax;
    E = 0;
  } else {
    int ex;
    const double fr = frexp(ax, &ex); /* ax = fr * 2^ex, fr in [0.5, 1) */
    M = (uint64_t)ldexp(fr, 53);
    E = ex - 53;
  }
  uint64_t r = M % (uint64_t)p;
  uint64_t w = 1 % (uint64_t)p;
  for (int q = 0; q < E; ++q) w = (w * 2) % (uint64_t)p;
  r = (r * w) % (uint64_t)p;
  if (xt < 0.0 && r) r = (uint64_t)p - r;
  int ri = (int)r;
  if (ri > (p - 1) / 2) ri -= p;
  return (int8_t)ri;
}

/* float upper bound of sqrt(x) (:225-227): correctly rounded sqrt, then round up to float. */
static int32_t norm_ub_bits(double x) {
  const double d = sqrt(x * (1.0 + ldexp(1.0, -30)));
  float f = (float)d;
  if ((double)f < d) f = nextafterf(f, INFINITY);
  int32_t bits;
  memcpy(&bits, &f, sizeof bits);
  return bits;
}

/* One element of prep (:207-222): residues of trunc(2^sh a) into planes 0..N-1 at byte
 * offset `off` (plane stride pst), abs plane value into plane N, norm contributions. */
static void prep_elem(double a, int sh, int sg, int N, int8_t* out, size_t off, size_t pst,
                      double* da2, double* na2) {
  const ozo_tables* t = tables();
  if (sh == OZO_SHIFT_NONFINITE) {
    for (int l = 0; l <= N; ++l) out[(size_t)l * pst + off] = 0;
    return;
  }
  const double xs = mul_pow2(a, sh);
  const double xt = trunc(xs);
  const double fr = xs - xt;
  *da2 = fma(fr, fr, *da2);
  *na2 = fma(xt, xt, *na2);
  for (int l = 0; l < N; ++l) out[(size_t)l * pst + off] = sym_residue(xt, t->p[l]);
  const int8_t absv = (sg == OZO_SHIFT_ZERO)
                          ? (int8_t)0
                          : (int8_t)(int)fmin(127.0, trunc(mul_pow2(fabs(a), sg)));
  out[(size_t)N * pst + off] = absv;
}

/* Rows of A.  Reduction orders of the reference's A blocks (:263-364): per row, eight chains
 * over k = t, t+8, t+16, ... (t = 0..7) for max / sum of squares and for the two norms, the
 * chains combined sequentially t = 0..7 starting from 0.0. */
void ozo_prep_rows(const double* A, int m, int k, int lda, int N, int kp, int8_t* out,
                   int32_t* ws, uint64_t* nonfinite) {
  const ozo_tables* t = tables();
  const double T = t->T[N];
  const size_t pst = (size_t)m * (size_t)kp;
  for (int i = 0; i < m; ++i) {
    double mx[8], ss[8];
    for (int c = 0; c < 8; ++c) {
      mx[c] = 0.0;
      ss[c] = 0.0;
      for (int q = c; q < k; q += 8) {
        const double a = A[i + (size_t)q * lda];
        mx[c] = fmax(mx[c], fabs(a));
        ss[c] = fma(a, a, ss[c]);
      }
    }
    double rowmax = 0.0;
    for (int c = 0; c < 8; ++c) rowmax = fmax(rowmax, mx[c]);
    const int resc = needs_rescale(rowmax);
    if (resc) {
      const int e = -ilogb(rowmax);
      for (int c = 0; c < 8; ++c) {
        ss[c] = 0.0;
        for (int q = c; q < k; q += 8) {
          const double a = mul_pow2(A[i + (size_t)q * lda], e);
          ss[c] = fma(a, a, ss[c]);
        }
      }
    }
    double S = 0.0;
    for (int c = 0; c < 8; ++c) S += ss[c];
    const int sh = shift_from_norm(rowmax, S, resc, T);
    const int sg = abs_shift(rowmax, sh);
    ws[i] = sh;
    ws[m + i] = sg;
    if (sh == OZO_SHIFT_NONFINITE && nonfinite) ++*nonfinite;
    double da[8] = {0, 0, 0, 0, 0, 0, 0, 0}, na[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int q = 0; q < kp; ++q) {
      const double a = q < k ? A[i + (size_t)q * lda] : 0.0;
      prep_elem(a, sh, sg, N, out, (size_t)i * kp + q, pst, &da[q & 7], &na[q & 7]);
    }
    double D = 0.0, Nn = 0.0;
    for (int c = 0; c < 8; ++c) {
      D += da[c];
      Nn += na[c];
    }
    ws[2 * m + i] = norm_ub_bits(D);
    ws[3 * m + i] = norm_ub_bits(Nn);
  }
}

/* The reference's warp reduction `v += shfl_xor(v, o)` for o = 16, 8, 4, 2, 1; every lane ends
 * with the same value, returned here (lane 0). */
static double butterfly_sum(double v[32]) {
  for (int o = 16; o; o >>= 1) {
    double nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
    memcpy(v, nv, sizeof nv);
  }
  return v[0];
}

/* Columns of B.  Reduction orders of the reference's B warps (:368-441): max / sum of
 * squares over 32 lane chains k = lane, lane+32, ...; the norms over lane chains
 * k = 4*lane + 128*c + e (c ascending, e = 0..3); each combined by the xor butterfly. */
void ozo_prep_cols(const double* B, int n, int k, int ldb, int N, int kp, int8_t* out,
                   int32_t* ws, uint64_t* nonfinite) {
  const ozo_tables* t = tables();
  const double T = t->T[N];
  const size_t pst = (size_t)n * (size_t)kp;
  for (int j = 0; j < n; ++j) {
    const double* b = B + (size_t)j * ldb;
    double mx[32], ss[32];
    for (int l = 0; l < 32; ++l) {
      mx[l] = 0.0;
      ss[l] = 0.0;
      for (int q = l; q < k; q += 32) {
        mx[l] = fmax(mx[l], fabs(b[q]));
        ss[l] = fma(b[q], b[q], ss[l]);
      }
    }
    double cmax = 0.0;
    for (int l = 0; l < 32; ++l) cmax = fmax(cmax, mx[l]);
    const int resc = needs_rescale(cmax);
    if (resc) {
      const int e = -ilogb(cmax);
      for (int l = 0; l < 32; ++l) {
        ss[l] = 0.0;
        for (int q = l; q < k; q += 32) {
          const double a = mul_pow2(b[q], e);
          ss[l] = fma(a, a, ss[l]);
        }
      }
    }
    const double S = butterfly_sum(ss);
    const int sh = shift_from_norm(cmax, S, resc, T);
    const int sg = abs_shift(cmax, sh);
    ws[j] = sh;
    ws[n + j] = sg;
    if (sh == OZO_SHIFT_NONFINITE && nonfinite) ++*nonfinite;
    double da[32], na[32];
    for (int l = 0; l < 32; ++l) {
      da[l] = 0.0;
      na[l] = 0.0;
      for (int k0 = 4 * l; k0 < kp; k0 += 128)
        for (int e = 0; e < 4; ++e) {
          const int q = k0 + e;
          const double a = q < k ? b[q] : 0.0;
          prep_elem(a, sh, sg, N, out, (size_t)j * kp + q, pst, &da[l], &na[l]);
        }
    }
    const double D = butterfly_sum(da);
    const double Nn = butterfly_sum(na);
    ws[2 * n + j] = norm_ub_bits(D);
    ws[3 * n + j] = norm_ub_bits(Nn);
  }
}

/* Exact INT8 GEMM, C = A * B^T with K-contiguous operands (src/int8_grouped_gemm.h:4-10). */
int ozo_i8_gemm(const int8_t* A8, const int8_t* B8, int m, int n, int kp, int32_t* C) {
  int bad = 0;
  for (int j = 0; j < n; ++j)
    for (int i = 0; i < m; ++i) {
      int64_t acc = 0;
      const int8_t* a = A8 + (size_t)i * kp;
      const int8_t* b = B8 + (size_t)j * kp;
      for (int q = 0; q < kp; ++q) acc += (int32_t)a[q] * (int32_t)b[q];
      if (acc > INT32_MAX || acc < INT32_MIN) bad = 1;
      C[(size_t)j * m + i] = (int32_t)acc;
    }
  return bad;
}

/* CRT integers of one entry (:507-520): y_l = (c_l mod p_l) q_l mod p_l, S1 = sum s1_l y_l,
 * S2 = sum s2_l y_l, Q = rint((S1 + S2 2^-18) u1/P), xr = (S1 - Q P1) + (S2 2^-18 - Q P2). */
void ozo_crt_entry(int N, const int32_t* c_planes, size_t plane_stride, uint64_t* S1o,
                   uint32_t* S2o, double* Qo, double* xro) {
  const ozo_tables* t = tables();
  uint64_t S1 = 0;
  uint32_t S2 = 0;
  for (int l = 0; l < N; ++l) {
    const int64_t p = t->p[l];
    const int64_t c = c_planes[(size_t)l * plane_stride];
    int64_t r = c % p;
    if (r < 0) r += p;
    const uint64_t y = (uint64_t)((r * t->qinv[N][l]) % p);
    S1 += t->s1[N][l] * y;
    S2 += t->s2[N][l] * (uint32_t)y;
  }
  const double s2d = (double)S2 * (1.0 / (double)(1u << OZO_S2_BITS));
  const double Q = rint(((double)S1 + s2d) * t->inv_Pu[N]);
  const int64_t X1 = (int64_t)S1 - (int64_t)Q * t->P1[N];
  const double xr = (double)X1 + fma(-Q, t->P2[N], s2d);
  *S1o = S1;
  *S2o = S2;
  *Qo = Q;
  *xro = xr;
}

/* Sequential FP64 fma dot (:445-452). */
static double fp64_dot(const double* A, int lda, const double* B, int ldb, int k, int i, int j) {
  double s = 0.0;
  const double* a = A + i;
  const double* b = B + (size_t)j * ldb;
  for (int q = 0; q < k; ++q) s = fma(a[(size_t)q * lda], b[q], s);
  return s;
}

/* Restates one problem of oz2_reconstruct_kernel (src/ozaki2_numerics.cu:454-563). */
void ozo_reconstruct(int m, int n, int k, int N, double alpha, double beta, const double* A,
                     int lda, const double* B, int ldb, double* C, int ldc, const int32_t* C32,
                     const int32_t* rs, const int32_t* cs, int mode, uint64_t* cnt) {
  const ozo_tables* t = tables();
  const size_t mn = (size_t)m * (size_t)n;
  const double aalpha = fabs(alpha);
  const int lu1 = t->log2_u1[N];
  const double inv_u1 = ldexp(1.0, -lu1);
  const double crt_u = N * 255.0 * ldexp(1.0, -19) + ldexp(1.0, -10);
  const double u = ldexp(1.0, -53);
  const double nt = (double)k + (alpha != 1.0 ? 1.0 : 0.0) + (beta != 0.0 ? 1.0 : 0.0);
  const double ntu = nt * u;
  const double gam = (ntu / fma(-nt, u, 1.0) - 2.0 * u) * (1.0 - ldexp(1.0, -40));
  for (int j = 0; j < n; ++j)
    for (int i = 0; i < m; ++i) {
      const size_t idx = (size_t)j * m + i;
      double* cp = C + i + (size_t)j * ldc;
      const double c0 = (beta == 0.0) ? 0.0 : *cp;
      if (alpha == 0.0) {
        *cp = (beta == 0.0) ? 0.0 : beta * c0;
        continue;
      }
      const int rsh = rs[i], csh = cs[j];
      if (rsh == OZO_SHIFT_NONFINITE || csh == OZO_SHIFT_NONFINITE) {
        const double d = fp64_dot(A, lda, B, ldb, k, i, j);
        *cp = (beta == 0.0) ? alpha * d : fma(alpha, d, beta * c0);
        if (cnt) ++cnt[3];
        continue;
      }
      const int sig = rs[m + i], tau = cs[n + j];
      if (sig == OZO_SHIFT_ZERO || tau == OZO_SHIFT_ZERO) {
        *cp = (beta == 0.0) ? alpha * 0.0 : fma(alpha, 0.0, beta * c0);
        continue;
      }
      uint64_t S1;
      uint32_t S2;
      double Q, xr;
      ozo_crt_entry(N, C32 + idx, mn, &S1, &S2, &Q, &xr);
      const int esc = lu1 - rsh - csh;
      const double v = mul_pow2(xr, esc);
      const double emu = (beta == 0.0) ? alpha * v : fma(alpha, v, beta * c0);
      if (mode == OZO_REPAIR_OFF || (beta != 0.0 && !isfinite(c0))) {
        *cp = emu;
        continue;
      }
      float fda, fna, fdb, fnb;
      memcpy(&fda, &rs[2 * m + i], 4);
      memcpy(&fna, &rs[3 * m + i], 4);
      memcpy(&fdb, &cs[2 * n + j], 4);
      memcpy(&fnb, &cs[3 * n + j], 4);
      const double da = fda, na = fna, db = fdb, nb = fnb;
      const double et = fma(da, nb, fma(na, db, da * db)) * (1.0 + ldexp(1.0, -40));
      const double Eu =
          fma(4.0 * u, fabs(xr), fma(et, inv_u1, crt_u)) * (1.0 + ldexp(1.0, -40));
      const double E = mul_pow2(Eu, esc);
      const double L = (double)C32[(size_t)N * mn + idx];
      double lab = mul_pow2(L, -(sig + tau));
      lab = fmax(lab, fabs(v) - E) * (1.0 - ldexp(1.0, -40));
      if (lab < ldexp(1.0, -1000)) lab = 0.0;
      const double lhs = aalpha * E * (1.0 + ldexp(1.0, -40));
      const double rhs = gam * fma(aalpha, lab, fabs(beta * c0)) * (1.0 - ldexp(1.0, -40));
      const int cert = gam > 0.0 && E >= ldexp(1.0, -1000) && isfinite(lhs) && isfinite(v) &&
                       lhs <= rhs;
      if (cert) {
        *cp = emu;
      } else if (mode == OZO_REPAIR_COUNT) {
        *cp = emu;
        if (cnt) ++cnt[1];
      } else {
        const double d = fp64_dot(A, lda, B, ldb, k, i, j);
        *cp = (beta == 0.0) ? alpha * d : fma(alpha, d, beta * c0);
        if (cnt) ++cnt[2];
      }
    }
}

int ozo_emulated_dgemm(int m, int n, int k, int N, double alpha, double beta, const double* A,
                       int lda, const double* B, int ldb, double* C, int ldc, int mode,
                       uint64_t* cnt) {
  if (m <= 0 || n <= 0) return 0;
  const int kp = (k + 31) / 32 * 32;
  const int P = N + 1;
  int8_t* A8 = (int8_t*)calloc((size_t)P * m * kp + 1, 1);
  int8_t* B8 = (int8_t*)calloc((size_t)P * n * kp + 1, 1);
  int32_t* C32 = (int32_t*)calloc((size_t)P * m * n + 1, 4);
  int32_t* rs = (int32_t*)calloc((size_t)4 * m + 1, 4);
  int32_t* cs = (int32_t*)calloc((size_t)4 * n + 1, 4);
  int bad = 0;
  if (alpha != 0.0) {
    ozo_prep_rows(A, m, k, lda, N, kp, A8, rs, cnt ? &cnt[0] : NULL);
    ozo_prep_cols(B, n, k, ldb, N, kp, B8, cs, cnt ? &cnt[0] : NULL);
    for (int l = 0; l < P; ++l)
      bad |= ozo_i8_gemm(A8 + (size_t)l * m * kp, B8 + (size_t)l * n * kp, m, n, kp,
                         C32 + (size_t)l * m * n);
  }
  ozo_reconstruct(m, n, k, N, alpha, beta, A, lda, B, ldb, C, ldc, C32, rs, cs, mode, cnt);
  free(A8);
  free(B8);
  free(C32);
  free(rs);
  free(cs);
  return bad;
}

int ozo_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

typedef struct {
  int m, k, j0, j1;
  double alpha, beta;
  const double *A, *B;
  double* C;
  int lda, ldb, ldc;
} naive_job;

/* The reference's host FP64 path: s += a*b over k in order (test_numerics_standalone.cu:
 * 292-299), then alpha/beta.  Columns [j0, j1) of one worker; each dot stays sequential. */
static void* naive_worker(void* arg) {
  const naive_job* jb = (const naive_job*)arg;
  for (int j = jb->j0; j < jb->j1; ++j) {
    const double* b = jb->B + (size_t)j * jb->ldb;
    for (int i = 0; i < jb->m; ++i) {
      double s = 0.0;
      for (int q = 0; q < jb->k; ++q) s += jb->A[i + (size_t)q * jb->lda] * b[q];
      double* cp = jb->C + i + (size_t)j * jb->ldc;
      *cp = (jb->beta == 0.0) ? jb->alpha * s : jb->alpha * s + jb->beta * *cp;
    }
  }
  return NULL;
}

/* Columns [j0, j1) split over `threads` POSIX threads (<= 0: one per online CPU). */
void ozo_dgemm_naive(int m, int n, int k, double alpha, const double* A, int lda,
                     const double* B, int ldb, double beta, double* C, int ldc, int j0, int j1,
                     int threads) {
  (void)n;
  int nt = threads > 0 ? threads : ozo_max_threads();
  if (nt > 256) nt = 256;
  const int cols = j1 - j0;
  if (cols <= 0) return;
  if (nt > cols) nt = cols;
  pthread_t tid[256];
  naive_job jobs[256];
  for (int t = 0; t < nt; ++t) {
    naive_job jb = {m, k, j0 + (int)((long)cols * t / nt), j0 + (int)((long)cols * (t + 1) / nt),
                    alpha, beta, A, B, C, lda, ldb, ldc};
    jobs[t] = jb;
  }
  for (int t = 1; t < nt; ++t) pthread_create(&tid[t], NULL, naive_worker, &jobs[t]);
  naive_worker(&jobs[0]);
  for (int t = 1; t < nt; ++t) pthread_join(tid[t], NULL);
}
