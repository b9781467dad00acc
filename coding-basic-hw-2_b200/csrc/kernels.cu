// kernels.cu -- the three sm_100a kernels of the emulated grouped FP64 GEMM:
//   prep_kernel   FP64 operands -> per-row power-of-two shifts, N int8 residue planes + the
//                 abs plane, written directly in the tensor-core operand image layout
//                 (ggemm_stages.h); the residues of all planes come from one tcgen05.mma of
//                 byte digits against block-diagonal weights; HBM bound.
//   gemm_kernel   persistent tcgen05.mma.kind::i8 GEMM over every (problem, plane, tile):
//                 bulk copies -> shared-memory ring (mbarriers) -> TMEM int32 accumulators ->
//                 epilogue warps write CRT digit bytes (or int32 products); tensor-core bound.
//   recon_kernel  CRT reconstruction from digit bytes (or int32 products), unscaling,
//                 alpha/beta, componentwise certificate and FP64 repair; HBM bound.
// The numerical definitions (what is computed, bit for bit) are those of the reference
// src/ozaki2_numerics.cu:8-76 and :112-586; the work decomposition is this library's own.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <vector>

#include "crt.hpp"
#include "kernels.cuh"
#include "ptx.cuh"

namespace g2 {

__constant__ DevTables c_tab;

// =============================================================================== shared math
// x * 2^e: one multiplication for |e| <= 1000, else three clamped steps (the reference's
// mul_pow2, src/ozaki2_numerics.cu:112-122; exact unless the result is subnormal).
__device__ __forceinline__ double mul_pow2(double x, int e) {
  if (e >= -1000 && e <= 1000) return x * __longlong_as_double((long long)(e + 1023) << 52);
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int ee = max(-1000, min(1000, e));
    x *= __longlong_as_double((long long)(ee + 1023) << 52);
    e -= ee;
  }
  return x;
}
// The same product without the branch: three clamped steps always (for |e| <= 1000 the second
// and third multiply by 1.0), so a warp whose lanes straddle the bound does not diverge.
__device__ __forceinline__ double mul_pow2_nb(double x, int e) {
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const int ee = max(-1000, min(1000, e));
    x *= __longlong_as_double((long long)(ee + 1023) << 52);
    e -= ee;
  }
  return x;
}

// max(m, |a|) on the bit patterns: non-negative doubles order like their unsigned bits, so
// for finite and infinite |a| this is fmax(m, |a|).  A NaN element wins instead of being skipped;
// every row / column with a NaN ends with the non-finite shift either way (its sum of squares
// is NaN), so the shifts, the abs shifts and everything after are unchanged.  (FP64 fmax costs
// several instructions for its NaN rules.)
__device__ __forceinline__ unsigned long long absmax_bits(unsigned long long m, double a) {
  return max(m, (unsigned long long)__double_as_longlong(a) & 0x7FFFFFFFFFFFFFFFull);
}

__device__ __forceinline__ bool needs_rescale(double maxabs) {
  return maxabs > 0.0 && (maxabs > 0x1p400 || maxabs < 0x1p-400);
}

// Largest s with 2^s * ||x|| <= T (src/ozaki2_numerics.cu:133-153).
__device__ __forceinline__ int shift_from_norm(double maxabs, double ssq, bool rescaled,
                                               double T) {
  if (isinf(maxabs) || isnan(ssq)) return kShiftNonfinite;
  if (!(maxabs > 0.0)) return 0;
  const double nm = sqrt(ssq * (1.0 + 0x1p-30));
  int g, G;
  const double f = frexp(nm, &g);
  const double F = frexp(T, &G);
  g += rescaled ? ilogb(maxabs) : 0;
  return G - g - (f > F ? 1 : 0);
}

// Abs-plane exponent: maxabs * 2^sig in [64, 128) (src/ozaki2_numerics.cu:156-160).
__device__ __forceinline__ int abs_shift(double maxabs, int sh) {
  if (sh == kShiftNonfinite) return 0;
  if (!(maxabs > 0.0)) return kShiftZero;
  return 6 - ilogb(maxabs);
}

// Float upper bound of sqrt(x) as bits (src/ozaki2_numerics.cu:225-227).
__device__ __forceinline__ int32_t norm_ub_bits(double x) {
  return __float_as_int(__double2float_ru(sqrt(x * (1.0 + 0x1p-30))));
}

// ============================================================================== prep kernel
// Residues through the tensor cores.  x = trunc(2^s a) is an integer-valued double with
// |x| < 2^80.  Read as a 96-bit two's complement integer, its bytes u_i (i < 12) give signed
// bytes s_i = u_i - 256 c_i with carries c_i = u_i >> 7, and
//     x = sum_{i<12} s_i 2^(8i) + sum_{i<11} c_i 2^(8(i+1))
// (the top carry c_11 is the sign bit and cancels the 2^96 of the two's complement).  These 23
// small integers, plus the abs-plane byte, form a 32-byte int8 "digit slot" per element.  For
// a modulus p, t = sum_d slot_d W_p[d] with W_p[d] the symmetric residue of the digit's weight
// (2^(8i) or 2^(8(i+1)) mod p) satisfies t = x (mod p) and |t| <= 12*128*127 + 11*127 < 2^18.
// One tcgen05.mma (kind::i8, exact int32) computes t for every plane: an MMA row carries the
// slots of 4 consecutive K positions of one row of the operand (K = 4 x 32 bytes), and the
// weight matrix is block diagonal, column 4 l + e holding plane l's weights against slot e.
// The epilogue turns t into the residue byte: with M = 1.5 * 2^23, the float M + t is exact,
// fma(t, fl(1/p), M) = M + round(t / p) (|t| / p < 2^11, and t / p is at least 1/(2p) away from
// a half-integer for odd p), and the low byte of bits(M + t) - bits(M + q) p is (t - q p) mod 256
// because bits(M) = 0x4B400000 is a multiple of 256: the symmetric residue as int8.  For
// p = 256 the weights reduce t to the low byte of x; the abs plane's weights select its byte.
// The result is identical to the reference's Barrett / table evaluation
// (src/ozaki2_numerics.cu:174-205): a residue class has exactly one symmetric representative.
constexpr int kPrepTileBytes = 4 * 16 * 256;  // 4 slots (K steps) x 16 row groups x 256 B
constexpr int kPrepMaxCols = 96;              // 4 (N + 1) rounded up to 16, N <= 20
constexpr int kPrepWBytes = 4 * (kPrepMaxCols / 8) * 256;

// A CTA is two independent halves of 4 warps.  Each half owns one tile of 128 MMA rows per
// round (its own slot buffers, mbarriers and TMEM accumulators) and synchronizes only its own
// 128 threads (barrier 1 + half), so one half's MMA and memory waits overlap the other's
// work.  Rounds are pipelined: for N <= 15 the accumulators are double buffered and round i's
// MMA runs while the half turns round i - 1's accumulators into residue bytes; for N > 15 (wider
// accumulators) the half finishes round i - 1 first and round i's MMA overlaps the next round's
// digit slots.
struct PrepSmem {
  uint8_t adig[2][2][kPrepTileBytes];  // [half][buffer] digit slots (1024-byte aligned)
  uint8_t wts[kPrepWBytes];            // block-diagonal weights, K-major, 32-byte swizzle
  double a[8][32];
  double b[8][32];
  double rowmax[32];
  int sh[32], sg[32];
  uint64_t bar[2][2];    // [half][buffer]: MMAs of a round complete
  uint64_t ready[2][2];  // [half][buffer]: the half's 4 warps wrote the round's slots
  uint32_t tmem;
  // per half: gave up after a timed-out wait.  Only the half's own threads write it, before
  // they arrive at the half's next barrier, so every thread of the half reads the same value
  // after that barrier and the half leaves its rounds together.
  int abort[2];
  int issued[2], waited[2];  // per half: rounds whose MMAs were issued / seen complete
};
constexpr size_t kPrepSmem = 1024 + sizeof(PrepSmem);
constexpr int kPrepTmemCols = 256;
// TMEM column stride of one accumulator: n_cols rounded up to a power of two (>= 32).
__host__ __device__ constexpr int prep_acc_stride(int n_cols) {
  return n_cols <= 32 ? 32 : n_cols <= 64 ? 64 : 128;
}
// Double-buffered accumulators fit (2 halves x 2 buffers x stride <= 256 columns) exactly
// for N <= 15; above, each half has one accumulator of stride 128 (kBias below: the kernel is
// compiled once per case).
// TMEM column of the accumulator of (half, buffer).
template <bool kBias>
__device__ __forceinline__ uint32_t prep_region(int n_cols, int half, int bf) {
  return kBias ? (uint32_t)(half * 128) : (uint32_t)((2 * half + bf) * prep_acc_stride(n_cols));
}

// Abs-plane value floor(2^sg |a|) in [0, 127] (0 for an all-zero row).  2^sg |a| < 128 for
// every element of a finite row (sg puts the row maximum in [64, 128)), so the truncating
// conversion is exact; the reference's clamp at 127 is kept as an integer min.
__device__ __forceinline__ uint32_t abs_byte(double a, int sg) {
  if (sg == kShiftZero) return 0u;
  return min(__double2uint_rz(mul_pow2(fabs(a), sg)), 127u);
}

// x = trunc(xs) and the three 32-bit words of x as a 96-bit two's complement integer.
// narrow: |xs| < 2^63 (every N <= 16, as |x| <= T[N] < 2^62.1): one truncating conversion
// gives x as an int64.  Otherwise (|x| < 2^80) the words come from an exact FP64 split.
__device__ __forceinline__ void trunc_words(double xs, bool narrow, double& xt, uint32_t& w0,
                                            uint32_t& w1, uint32_t& w2) {
  if (narrow) {
    const long long xi = __double2ll_rz(xs);
    xt = (double)xi;  // exact: xi came from a double
    w0 = (uint32_t)xi;
    w1 = (uint32_t)((unsigned long long)xi >> 32);
    w2 = (uint32_t)(xi >> 63);
  } else {
    xt = trunc(xs);
    const double xh = floor(xt * 0x1p-32);
    const double xl = fma(-xh, 0x1p32, xt);  // in [0, 2^32), exact
    w0 = (uint32_t)__double_as_longlong(xl + 0x1p52);
    const long long h = __double_as_longlong(xh + 0x1.8p52) - __double_as_longlong(0x1.8p52);
    w1 = (uint32_t)h;
    w2 = (uint32_t)((unsigned long long)h >> 32);
  }
}

// Digit slot of the words of x and the abs byte ab:
//   bytes 0..11  s_i (x as 96-bit two's complement), bytes 12..22 c_0..c_10, byte 23 ab.
__device__ __forceinline__ void digit_slot(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t ab,
                                           uint4& lo, uint4& hi) {
  lo = make_uint4(w0, w1, w2, (w0 >> 7) & 0x01010101u);
  hi = make_uint4((w1 >> 7) & 0x01010101u, ((w2 >> 7) & 0x00010101u) | (ab << 24), 0u, 0u);
}

// Slot e of MMA row rho of the tile of `half` in buffer bf (K-major image, 32-byte swizzle:
// slot e is K step e).
__device__ __forceinline__ void put_slot(PrepSmem& sm, int half, int bf, int rho, int e,
                                         const uint4& lo, const uint4& hi) {
  const int rr = rho & 7, sw = (rr >> 2) << 4;
  uint8_t* base = sm.adig[half][bf] + (e * 16 + (rho >> 3)) * 256 + rr * 32;
  *reinterpret_cast<uint4*>(base + sw) = lo;
  *reinterpret_cast<uint4*>(base + (16 ^ sw)) = hi;
}

// Block-diagonal weights (the MMA's B operand, K-major, 32-byte swizzle), one image per
// (qscale, N) built on the host (make_prep_weight_images) and copied to shared memory by every
// block: row n = 4 l + e holds plane l's weights in K step (slot) e and zeros elsewhere; planes
// l > N are zero.  qscale (GGEMM_PREP_QSCALED): the weights of plane l < N are q_l 2^(8 i) mod p_l
// (symmetric), so that the plane holds the residue of q_l x instead of x (q_l the CRT factor the
// reconstruct applies to plane l's digits).
__device__ uint8_t g_prep_wts[2][kMaxModuli + 1][kPrepWBytes];

__device__ __forceinline__ void load_weights(PrepSmem& sm, int N, int n_cols, bool qscale) {
  const uint4* src = reinterpret_cast<const uint4*>(g_prep_wts[qscale ? 1 : 0][N]);
  uint4* dst = reinterpret_cast<uint4*>(sm.wts);
  for (int c = threadIdx.x; c < 8 * n_cols; c += blockDim.x) dst[c] = src[c];
}

// With single-buffered accumulators (N > 15) they start from kPrepBias = bits(1.5 * 2^23)
// instead of zero, so the MMA yields tm = bits(M + t) directly (|t| < 2^22) and the epilogue
// saves one integer add per residue; the low byte of tm is t's low byte (the bias is a multiple
// of 256), which the p = 256 plane and the abs plane keep as they are.  With double-buffered
// accumulators (N <= 15) the refill of one accumulator while the MMA writes the other cost more
// than it saved (measured), so they start from zero and the epilogue adds the bias.
constexpr uint32_t kPrepBias = 0x4B400000u;

// Residue bytes of t0, t1 for odd p from tm = kPrepBias + t (low byte of each result; see
// above): per residue r = fmaf(float(tm) - M, 1/p, M) (the subtraction exact, one rounding to
// nearest, so bits(r) = bits(M) + rint(t / p)), then tm - bits(r) * p; the two FP32 steps run as
// packed f32x2 instructions for both residues.
__device__ __forceinline__ void residue_byte2(uint32_t tm0, uint32_t tm1, float invp, uint32_t p,
                                              uint32_t& b0, uint32_t& b1) {
  uint64_t x, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "r"(tm0), "r"(tm1));
  const uint64_t neg_m = 0xCB400000CB400000ull;  // (-1.5 * 2^23, -1.5 * 2^23)
  const uint64_t m2 = 0x4B4000004B400000ull;     // (1.5 * 2^23, 1.5 * 2^23)
  const uint32_t iv = __float_as_uint(invp);
  uint64_t inv2;
  asm("mov.b64 %0, {%1, %1};" : "=l"(inv2) : "r"(iv));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(x) : "l"(x), "l"(neg_m));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(inv2), "l"(m2));
  uint32_t r0, r1;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(r0), "=r"(r1) : "l"(r));
  b0 = tm0 - r0 * p;
  b1 = tm1 - r1 * p;
}

// Sets the n_cols columns of this thread's lane of the accumulator at `acc` to kPrepBias.
__device__ __forceinline__ void prep_bias_acc(uint32_t acc, int n_cols) {
  const uint32_t taddr = acc + ((uint32_t)(((threadIdx.x >> 5) & 3) * 32) << 16);
  for (int c = 0; c < n_cols; c += 16) tmem_fill_32x32b_x16(taddr + (uint32_t)c, kPrepBias);
}

__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Bounded wait (every thread of a half) for the MMAs of one of its buffers; on a timeout the
// block gives up.
__device__ __forceinline__ bool prep_wait(PrepSmem& sm, int half, int bf, uint32_t parity,
                                          DevCounters* cnt) {
  if (mbar_try_wait(&sm.bar[half][bf], parity) ||
      mbar_wait(&sm.bar[half][bf], parity, global_timer_ns() + 4000000000ull, &sm.abort[half])) {
    if ((threadIdx.x & 127) == 0) ++sm.waited[half];
    return true;
  }
  sm.abort[half] = 1;
  atomicCAS(&cnt->status, 0u, (unsigned)kStatusPrepTimeout);
  return false;
}

// Barrier of the 128 threads of one half (ids 1 and 2; 0 is __syncthreads).
__device__ __forceinline__ void half_sync(int half) {
  if (half) asm volatile("bar.sync 2, 128;" ::: "memory");
  else asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Bounded wait of the issuing thread of a half for the 4 warps' arrivals of round i.
__device__ __forceinline__ bool prep_wait_ready(PrepSmem& sm, int half, int i, DevCounters* cnt) {
  uint64_t* b = &sm.ready[half][i & 1];
  const uint32_t parity = (uint32_t)(i >> 1) & 1u;
  if (mbar_try_wait(b, parity) || mbar_wait(b, parity, global_timer_ns() + 4000000000ull, &sm.abort[half]))
    return true;
  sm.abort[half] = 1;
  atomicCAS(&cnt->status, 0u, (unsigned)kStatusPrepTimeout);
  return false;
}

// Issues round i's MMAs of a half (one thread), committed to bar[half][i & 1].
template <bool kBias>
__device__ __forceinline__ void prep_issue(PrepSmem& sm, uint32_t tmem, int n_cols, int half,
                                           int i) {
  const int bf = i & 1;
  const uint32_t idesc = idesc_i8(128, n_cols);
  const uint32_t wb = smem_addr(sm.wts);
  const uint32_t ab = smem_addr(sm.adig[half][bf]);
  const uint32_t d = tmem + prep_region<kBias>(n_cols, half, bf);
  const uint32_t acc0 = kBias ? 1u : 0u;  // biased accumulators add to their start value
#pragma unroll
  for (int e = 0; e < 4; ++e)
    mma_i8(d, smem_desc_sw32(ab + e * 16 * 256, 256),
           smem_desc_sw32(wb + e * (n_cols / 8) * 256, 256), idesc, e > 0 ? 1u : acc0);
  mma_commit(&sm.bar[half][bf]);
  ++sm.issued[half];
}

// Second half of round i of this thread's half (its slots are written to buffer i & 1): issues
// round i's MMAs (thread 0 of the half, committed to bar[half][i & 1]) and turns round i - 1's
// accumulators into residue bytes (epi(col), col = their TMEM column; when prev).  Returns
// false once the block has given up.
template <bool kBias, typename Epi>
__device__ __forceinline__ bool prep_round(PrepSmem& sm, uint32_t tmem, int n_cols, int i,
                                           bool prev, Epi&& epi, DevCounters* cnt) {
  const int half = threadIdx.x >> 7;
  constexpr bool dbuf = !kBias;
  const int pb = (i - 1) & 1;
  const uint32_t pp = (uint32_t)((i - 1) >> 1) & 1u;
  fence_proxy_async_smem();
  if (!dbuf && prev && prep_wait(sm, half, pb, pp, cnt)) {
    epi(prep_region<kBias>(n_cols, half, 0));
    prep_bias_acc(tmem + prep_region<kBias>(n_cols, half, 0), n_cols);
  }
  if (!dbuf) tmem_st_wait();  // this thread's accumulator reset precedes the MMAs
  // slots of round i written and the accumulator the MMAs overwrite read.  Single-buffered
  // (kBias): each warp arrives on ready[half][i & 1] and only the issuing thread waits, so the
  // warps of a half are not held in lock step (measured faster there); double-buffered: a
  // barrier of the half (measured faster there: fewer registers live across the round).
  tc_fence_before();
  if constexpr (kBias) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.ready[half][i & 1]);
    if ((threadIdx.x & 127) == 0 && prep_wait_ready(sm, half, i, cnt)) {
      tc_fence_after();
      prep_issue<kBias>(sm, tmem, n_cols, half, i);
    }
    // warp-uniform: the next round's __syncwarp needs every lane
    if (__any_sync(0xFFFFFFFFu, *(volatile int*)&sm.abort[half] != 0)) return false;
  } else {
    half_sync(half);
    tc_fence_after();
    if (sm.abort[half]) return false;
    if ((threadIdx.x & 127) == 0) prep_issue<kBias>(sm, tmem, n_cols, half, i);
  }
  if (dbuf && prev && prep_wait(sm, half, pb, pp, cnt)) epi(prep_region<kBias>(n_cols, half, pb));
  return true;
}

// Epilogue of a round for one thread (after its MMAs completed), compiled per moduli count N
// so that every plane index, constant and branch is resolved at compile time: its MMA row
// (TMEM lane 32 (warp % 4) + lane of the accumulator) holds t for 4 consecutive K positions of
// one row, column 4 l + e for plane l, element e (t, or kPrepBias + t when prep_needs_bias(N)); it
// writes one 32-bit word
// (4 residue bytes) per plane at dst + l * pb.  Groups of 4 planes (16 columns) are loaded from
// TMEM; the load of group g + 1 overlaps the bytes of group g.  (The caller resets the
// accumulator to the bias afterwards; doing it here, in a function that is not inlined, would
// cost the caller registers.)
template <int N>
__device__ __forceinline__ void prep_epilogue_n(uint32_t taddr, int8_t* dst, long long pb,
                                                bool store) {
  constexpr int G = (N + 4) / 4;
  uint32_t v[2][16];
  tmem_ld_32x32b_x16(taddr, v[0]);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    tmem_ld_wait(v[g & 1]);
    if (g + 1 < G) tmem_ld_32x32b_x16(taddr + (uint32_t)((g + 1) * 16), v[(g + 1) & 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int l = 4 * g + i;
      if (l > N) break;
      uint32_t b[4];
      if (l == 0 || l == N) {
#pragma unroll
        for (int e = 0; e < 4; ++e) b[e] = v[g & 1][4 * i + e];
      } else {
        constexpr uint32_t bias = prep_needs_bias(N) ? 0u : kPrepBias;
#pragma unroll
        for (int e = 0; e < 4; e += 2)
          residue_byte2(v[g & 1][4 * i + e] + bias, v[g & 1][4 * i + e + 1] + bias,
                        c_tab.invpf[l], c_tab.p[l], b[e], b[e + 1]);
      }
      if (store) *reinterpret_cast<uint32_t*>(dst + l * pb) = pack4(b[0], b[1], b[2], b[3]);
    }
  }

}

// Dispatch on N (one copy of the per-N bodies, not inlined into every caller).
__device__ __noinline__ void prep_epilogue(uint32_t acc, int N, int8_t* dst, long long pb,
                                           bool store) {
  tc_fence_after();  // the TMEM reads follow the completion seen on the mbarrier
  const uint32_t taddr = acc + ((uint32_t)(((threadIdx.x >> 5) & 3) * 32) << 16);
  switch (N) {
#define G2_EPI(n) \
  case n: prep_epilogue_n<n>(taddr, dst, pb, store); break;
    G2_EPI(1) G2_EPI(2) G2_EPI(3) G2_EPI(4) G2_EPI(5) G2_EPI(6) G2_EPI(7) G2_EPI(8) G2_EPI(9)
    G2_EPI(10) G2_EPI(11) G2_EPI(12) G2_EPI(13) G2_EPI(14) G2_EPI(15) G2_EPI(16) G2_EPI(17)
    G2_EPI(18) G2_EPI(19) G2_EPI(20)
#undef G2_EPI
    default: break;
  }
}

// The epilogue of an instance compiled for one moduli count kN, called directly (measured
// faster than the dispatch above); kN = 0: any N, through the dispatch.
template <int kN>
__device__ __noinline__ void prep_epilogue_fixed(uint32_t acc, int8_t* dst, long long pb,
                                                 bool store) {
  tc_fence_after();  // the TMEM reads follow the completion seen on the mbarrier
  const uint32_t taddr = acc + ((uint32_t)(((threadIdx.x >> 5) & 3) * 32) << 16);
  prep_epilogue_n<kN>(taddr, dst, pb, store);
}
template <int kN>
__device__ __forceinline__ void prep_epilogue_of(uint32_t acc, int N, int8_t* dst, long long pb,
                                                 bool store) {
  if constexpr (kN > 0) prep_epilogue_fixed<kN>(acc, dst, pb, store);
  else prep_epilogue(acc, N, dst, pb, store);
}

// Image byte offset of (row r, K position q) inside a plane (ggemm_stages.h).
__device__ __forceinline__ long long img_off(int rg, int r, int q) {
  const int rr = r & 7, qq = q & 31;
  return ((long long)(q >> 5) * rg + (r >> 3)) * 256 + rr * 32 + (((qq >> 4) ^ (rr >> 2)) << 4) +
         (qq & 15);
}

// Rows of a column-major A: 32 rows per block, 8 warps.  Reduction orders (the reference's,
// src/ozaki2_numerics.cu:263-364): for every row, 8 chains over K positions q = t (mod 8),
// ascending, for the max / sum of squares and for ||dA||^2, ||A'||^2; chains combined
// t = 0..7 from 0.0.  In a round (32 K positions) thread (warp w, lane r) takes the chain
// positions k0 + w + 8 j, j = 0..3, of row r: they lie in the K quads g = (w / 4) + 2 j, so
// half w / 4 (chains 4 (w / 4) .. +3) owns the 4 quads of its parity.  MMA row
// 32 (r / 8) + 8 j + r % 8 of the half's tile holds quad (w / 4) + 2 j of row r, so the epilogue
// thread (warp w, lane L) owns row 8 (w % 4) + L % 8 and quad (w / 4) + 2 (L / 8): a warp's
// store of a plane then covers the 4 quads of its parity of 8 rows in one 256-byte image atom
// (8 sectors) instead of one quad of 32 rows (32 sectors); the latter took 1.21 ms against the
// column path's 0.69 ms on an 8192 x 8192 operand.
template <bool kBias, int kN>
__device__ void prep_rows_block(const ggemm_prep_desc_t& d, int blk, DevCounters* cnt,
                                PrepSmem& sm, uint32_t tmem, int n_cols) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rows = d.rows, K = d.k, N = d.N;
  const int r = blk * 32 + lane;
  const bool valid = r < rows;
  const double* __restrict__ X = d.X;
  const long long ld = d.ld;
  const double T = c_tab.T[N];

  unsigned long long mxb = 0;
  double ss = 0.0;
  if (valid) {
#pragma unroll 16
    for (int q = w; q < K; q += 8) {
      const double a = X[r + q * ld];
      mxb = absmax_bits(mxb, a);
      ss = fma(a, a, ss);
    }
  }
  sm.a[w][lane] = __longlong_as_double((long long)mxb);
  __syncthreads();
  if (w == 0) {
    unsigned long long M = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) M = absmax_bits(M, sm.a[t][lane]);
    sm.rowmax[lane] = __longlong_as_double((long long)M);
  }
  __syncthreads();
  const double rowmax = sm.rowmax[lane];
  const bool resc = valid && needs_rescale(rowmax);
  if (resc) {  // rare: sum of squares of a * 2^-ilogb(rowmax)
    const int e = -ilogb(rowmax);
    ss = 0.0;
    for (int q = w; q < K; q += 8) {
      const double a = mul_pow2(X[r + q * ld], e);
      ss = fma(a, a, ss);
    }
  }
  sm.b[w][lane] = ss;
  __syncthreads();
  if (w == 0) {
    double S = 0.0;
#pragma unroll
    for (int t = 0; t < 8; ++t) S += sm.b[t][lane];
    const int sh = valid ? shift_from_norm(rowmax, S, resc, T) : 0;
    const int sg = valid ? abs_shift(rowmax, sh) : kShiftZero;
    sm.sh[lane] = sh;
    sm.sg[lane] = sg;
    if (valid) {
      d.ws[r] = sh;
      d.ws[rows + r] = sg;
    }
    const unsigned nf = __ballot_sync(0xFFFFFFFFu, valid && sh == kShiftNonfinite);
    if (lane == 0 && nf) atomicAdd(&cnt->nonfinite, (unsigned long long)__popc(nf));
  }
  __syncthreads();
  const int sh = sm.sh[lane], sg = sm.sg[lane];
  const bool finite = sh != kShiftNonfinite;
  const bool narrow = N <= 16;
  const int ksteps = (K + 31) >> 5;
  const int rg = (rows + 7) >> 3;
  const int half = w >> 2;
  const int re = blk * 32 + 8 * (w & 3) + (lane & 7);  // row and K quad of the epilogue thread
  const int qe = half + 2 * (lane >> 3);
  const bool in_image = (re >> 3) < rg;

  double da = 0.0, na = 0.0;  // chain t = w
  // operands of the next two rounds are in flight while a round is processed
  double cur[4], nx1[4], nx2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = w + 8 * j;
    cur[j] = (valid && q < K) ? X[r + q * ld] : 0.0;
    nx1[j] = (valid && q + 32 < K) ? X[r + (q + 32) * ld] : 0.0;
  }
  int i = 0;
  for (; i < ksteps; ++i) {
    const int k0 = 32 * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = k0 + 64 + w + 8 * j;
      nx2[j] = (valid && q < K) ? X[r + q * ld] : 0.0;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w0 = 0u, w1 = 0u, w2 = 0u, ab = 0u;
      if (finite) {
        const double xs = mul_pow2(cur[j], sh);
        double xt;
        trunc_words(xs, narrow, xt, w0, w1, w2);
        const double fr = xs - xt;
        da = fma(fr, fr, da);
        na = fma(xt, xt, na);
        ab = abs_byte(cur[j], sg);
      }
      uint4 lo, hi;
      digit_slot(w0, w1, w2, ab, lo, hi);
      put_slot(sm, half, i & 1, 32 * (lane >> 3) + 8 * j + (lane & 7), w & 3, lo, hi);
    }
    int8_t* prev_dst = d.img + img_off(rg, re, k0 - 32 + 4 * qe);
    if (!prep_round<kBias>(sm, tmem, n_cols, i, i > 0,
                    [&](uint32_t col) {
                      prep_epilogue_of<kN>(tmem + col, N, prev_dst, d.plane_bytes, in_image);
                    },
                    cnt))
      break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      cur[j] = nx1[j];
      nx1[j] = nx2[j];
    }
  }
  if (i == ksteps && ksteps > 0 &&
      prep_wait(sm, half, (i - 1) & 1, (uint32_t)((i - 1) >> 1) & 1u, cnt))
    prep_epilogue_of<kN>(tmem + prep_region<kBias>(n_cols, half, kBias ? 0 : (i - 1) & 1), N,
                  d.img + img_off(rg, re, 32 * (i - 1) + 4 * qe), d.plane_bytes, in_image);
  __syncthreads();
  sm.a[w][lane] = da;
  sm.b[w][lane] = na;
  __syncthreads();
  if (w == 0 && valid) {
    double D = 0.0, Nn = 0.0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      D += sm.a[t][lane];
      Nn += sm.b[t][lane];
    }
    d.ws[2 * rows + r] = norm_ub_bits(D);
    d.ws[3 * rows + r] = norm_ub_bits(Nn);
  }
}

// Columns of a column-major B: one warp per column, 8 columns (one image row group) per
// block.  Reduction orders (src/ozaki2_numerics.cu:368-441): max / sum of squares over lane
// chains q = lane (mod 32); norms over lane chains q = 4 lane + 128 c + e; both combined by the
// xor butterfly.  In a round (128 K positions) lane L of warp w takes positions c0 + 4 L + e,
// e = 0..3, of its column: its own MMA row (32 (w % 4) + L of tile w / 4), so the same thread
// writes the slots and reads back the residues.
template <bool kBias, int kN>
__device__ void prep_cols_block(const ggemm_prep_desc_t& d, int blk, DevCounters* cnt,
                                PrepSmem& sm, uint32_t tmem, int n_cols) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rows = d.rows, K = d.k, N = d.N;
  const int col = blk * 8 + w;
  const bool valid = col < rows;
  const double* __restrict__ b = d.X + (long long)(valid ? col : 0) * d.ld;
  const double T = c_tab.T[N];

  unsigned long long mxb = 0;
  double ss = 0.0;
  if (valid) {
#pragma unroll 16
    for (int q = lane; q < K; q += 32) {
      const double a = b[q];
      mxb = absmax_bits(mxb, a);
      ss = fma(a, a, ss);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
    mxb = max(mxb, (unsigned long long)__shfl_xor_sync(0xFFFFFFFFu, (long long)mxb, o));
  const double mx = __longlong_as_double((long long)mxb);
  const bool resc = valid && needs_rescale(mx);
  if (resc) {
    const int e = -ilogb(mx);
    ss = 0.0;
    for (int q = lane; q < K; q += 32) {
      const double a = mul_pow2(b[q], e);
      ss = fma(a, a, ss);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  const int sh = valid ? shift_from_norm(mx, ss, resc, T) : 0;
  const int sg = valid ? abs_shift(mx, sh) : kShiftZero;
  if (valid && lane == 0) {
    d.ws[col] = sh;
    d.ws[rows + col] = sg;
    if (sh == kShiftNonfinite) atomicAdd(&cnt->nonfinite, 1ull);
  }
  const bool finite = sh != kShiftNonfinite;
  const bool narrow = N <= 16;
  const int ksteps = (K + 31) >> 5;
  const int rg = (rows + 7) >> 3;

  double da = 0.0, na = 0.0;
  const int rounds = (ksteps + 3) >> 2;  // 128 K positions per round
  double cur[4], nx1[4], nx2[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int q = 4 * lane + e;
    cur[e] = (valid && q < K) ? b[q] : 0.0;
    nx1[e] = (valid && q + 128 < K) ? b[q + 128] : 0.0;
  }
  int i = 0;
  for (; i < rounds; ++i) {
    const int q0 = 128 * i + 4 * lane;
    const bool in_k = (q0 >> 5) < ksteps;
#pragma unroll
    for (int e = 0; e < 4; ++e) nx2[e] = (valid && q0 + 256 + e < K) ? b[q0 + 256 + e] : 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint32_t w0 = 0u, w1 = 0u, w2 = 0u, ab = 0u;
      if (finite && in_k) {
        const double xs = mul_pow2(cur[e], sh);
        double xt;
        trunc_words(xs, narrow, xt, w0, w1, w2);
        const double fr = xs - xt;
        da = fma(fr, fr, da);
        na = fma(xt, xt, na);
        ab = abs_byte(cur[e], sg);
      }
      uint4 lo, hi;
      digit_slot(w0, w1, w2, ab, lo, hi);
      put_slot(sm, w >> 2, i & 1, 32 * (w & 3) + lane, e, lo, hi);
    }
    const int qp = q0 - 128;
    const bool in_kp = qp >= 0 && (qp >> 5) < ksteps;
    int8_t* prev_dst = d.img + img_off(rg, col, in_kp ? qp : 0);
    if (!prep_round<kBias>(sm, tmem, n_cols, i, i > 0,
                    [&](uint32_t c) { prep_epilogue_of<kN>(tmem + c, N, prev_dst, d.plane_bytes, in_kp); },
                    cnt))
      break;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      cur[e] = nx1[e];
      nx1[e] = nx2[e];
    }
  }
  if (i == rounds && rounds > 0 &&
      prep_wait(sm, w >> 2, (i - 1) & 1, (uint32_t)((i - 1) >> 1) & 1u, cnt)) {
    const int qp = 128 * (i - 1) + 4 * lane;
    const bool in_kp = (qp >> 5) < ksteps;
    prep_epilogue_of<kN>(tmem + prep_region<kBias>(n_cols, w >> 2, kBias ? 0 : (i - 1) & 1), N,
                  d.img + img_off(rg, col, in_kp ? qp : 0), d.plane_bytes, in_kp);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    da += __shfl_xor_sync(0xFFFFFFFFu, da, o);
    na += __shfl_xor_sync(0xFFFFFFFFu, na, o);
  }
  if (valid && lane == 0) {
    d.ws[2 * rows + col] = norm_ub_bits(da);
    d.ws[3 * rows + col] = norm_ub_bits(na);
  }
}

// Owner of x in an exclusive prefix array (prefix[0] = 0 <= x, non-decreasing): the largest
// i < num with prefix[i] <= x.  Found by one warp (every warp of a block computes the same
// value): up to 256 entries, lane L counts the
// entries i = L (mod 32) with prefix[i] <= x, all loads in flight at once (one memory round trip
// instead of one per bisection step).  Above 256 entries, a 32-way search: each round the lanes
// probe 32 evenly spaced entries of the remaining range (ceil(log32 num) round trips).  Call by
// all 32 lanes.
template <typename P>
__device__ __forceinline__ int find_owner_warp(const P* __restrict__ prefix, int num, P x) {
  const int lane = threadIdx.x & 31;
  if (num <= 256) {
    int c = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = lane + 32 * k;
      c += (i < num && prefix[i] <= x) ? 1 : 0;
    }
    return __reduce_add_sync(0xFFFFFFFFu, c) - 1;
  }
  int lo = 0, hi = num;  // prefix[lo] <= x; the answer lies in [lo, hi)
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) >> 5;
    const int pos = lo + lane * step;
    const unsigned ok = __ballot_sync(0xFFFFFFFFu, pos < hi && prefix[pos] <= x);
    lo += (31 - __clz(ok)) * step;  // lane 0 probes lo itself, so ok != 0
    hi = min(hi, lo + step);
  }
  return lo;
}

// Compiled per class of moduli counts (prep_class): kN = 14, 15, 16 for that count only, kN = 0
// for the other counts with kBias = prep_needs_bias(N).  The host launches each on its own range
// of the descriptor array; prefix values are absolute and the grid's blocks start at block
// block0 of that numbering.
template <bool kBias, int kN>
__global__ void __launch_bounds__(kPrepThreads, 2)
    prep_kernel(const ggemm_prep_desc_t* __restrict__ descs, const int* __restrict__ prefix,
                int num, int block0, DevCounters* cnt) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int bl = block0 + (int)blockIdx.x;
  const int owner = find_owner_warp(prefix, num, bl);
  const ggemm_prep_desc_t d = descs[owner];
  if (d.N < 1 || d.N > kMaxModuli || d.rows <= 0 || prep_needs_bias(d.N) != kBias ||
      (kN > 0 && d.N != kN))
    return;
  const int n_cols = (4 * (d.N + 1) + 15) / 16 * 16;
  load_weights(sm, d.N, n_cols, (d.kind & GGEMM_PREP_QSCALED) != 0);
  if (threadIdx.x == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(&sm.bar[h][0], 1);
      mbar_init(&sm.bar[h][1], 1);
      mbar_init(&sm.ready[h][0], 4);
      mbar_init(&sm.ready[h][1], 4);
      sm.issued[h] = 0;
      sm.waited[h] = 0;
    }
    sm.abort[0] = 0;
    sm.abort[1] = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(&sm.tmem, kPrepTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  if (kBias) {  // the half's accumulator starts from the bias (ordered before the
                           // first MMA by the round's fence / barrier)
    prep_bias_acc(tmem + prep_region<kBias>(n_cols, threadIdx.x >> 7, 0), n_cols);
    tmem_st_wait();
  }
  const int blk = bl - prefix[owner];
  if ((d.kind & 1) == 0) prep_rows_block<kBias, kN>(d, blk, cnt, sm, tmem, n_cols);
  else prep_cols_block<kBias, kN>(d, blk, cnt, sm, tmem, n_cols);
  // a half that gave up may still have MMAs in flight (at most its last two rounds, since
  // every round waits for the one before): let them finish (bounded) first
  __syncthreads();
  if ((threadIdx.x & 127) == 0) {
    const int h = threadIdx.x >> 7;
    int dummy = 0;
    for (int j = max(sm.waited[h], sm.issued[h] - 2); j < sm.issued[h]; ++j)
      if (!mbar_wait(&sm.bar[h][j & 1], (uint32_t)(j >> 1) & 1u,
                     global_timer_ns() + 4000000000ull, &dummy))
        break;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, kPrepTmemCols);
}

// ============================================================================== GEMM kernel
// Tile 128 x 256 (128 x 128 for n <= 128) x (8 x 32-byte K steps) per pipeline stage.
// Warp roles:
//   warp 0: TMEM allocation + bulk-copy producer (lanes [0, kKS) copy A, [kKS, 2 kKS) copy B)
//   warp 1: tcgen05.mma issuer (one lane)
//   warps 2..5: epilogue (TMEM -> registers -> CRT digit bytes and int32 abs products, or int32
//   products); warp w reads TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31, i.e. tile rows.
// Two TMEM accumulators (2 x 256 columns, all of TMEM) let the epilogue of one tile overlap the
// MMAs of the next.  The 256-column tile halves the operand bytes fetched per MAC of the
// B side, which (with 128 x 128 tiles) bound the kernel by L2 -> SM traffic.  Tiles come from a
// host-side LPT order; each CTA walks it from both ends when the jobs differ in depth (TileWalk)
// and keeps its walk's tile
// coordinates in shared memory (the schedule below).
// Stages of 8 K steps: a ring of fewer, larger stages measured faster than more, smaller ones of
// the same bytes (4 x 4 steps: 7.79 ms, 2 x 8: 7.52 ms, one 8192^3 problem at N = 16).
constexpr int kKS = 8;      // 32-byte K steps per pipeline stage
constexpr int kStages = 2;  // kStages * kKS * 12 KB of operands in flight
constexpr int kStepBytesA = 16 * 256;                     // one 32-byte K step of 128 rows
constexpr int kStepBytesB = 32 * 256;                     // ... of 256 rows
constexpr int kStageBytes = kKS * (kStepBytesA + kStepBytesB);  // kKS K steps of A and B
constexpr int kGemmThreads = 192;
constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s per wait

struct GemmSmemCtl {
  uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2], drain;
  uint32_t tmem_base;
  int abort;
};
// Tile schedule of a CTA in shared memory: {job, plane, tm, tn} of each tile of its walk, built
// once at kernel start (bisection over the job prefix staged in the still unused operand ring),
// so that no role decodes a tile on its critical path.  Used when the CTA walks at most
// kSchedMax tiles and the call has at most kSchedJobs jobs; otherwise every role decodes each
// tile itself (warp-parallel search).
constexpr int kSchedMax = 1024;
constexpr int kSchedJobs = 4096;
static_assert((kSchedJobs + 1) * 8 <= kStages * kStageBytes, "prefix staging");
constexpr size_t kGemmSmem =
    1024 + kStages * kStageBytes + sizeof(GemmSmemCtl) + 64 + kSchedMax * sizeof(int4);

struct TileInfo {
  const GemmJob* job;
  int plane, tm, tn;
};

// Order in which CTA b walks the tiles (all three roles walk the same order).  The host sorts
// the jobs by tile cost (deepest K first), so the first half of the tile numbering holds the
// heavy tiles and the second half the light ones; CTA b alternates between a front walk
// (tiles t < T/2 with t = b mod G, heaviest first) and a back walk (tiles t >= T/2 with
// T - 1 - t = b mod G, lightest first), so that the epilogue of a light tile overlaps the MMAs of
// a heavy one.  Every tile is visited by exactly one CTA.
struct TileWalk {
  long long T, nf, nb;
  int b, G;
  __device__ __forceinline__ long long count() const { return nf + nb; }
  __device__ __forceinline__ long long at(long long i) const {
    const long long m = nf < nb ? nf : nb;
    bool front;
    long long k;
    if (i < 2 * m) {
      front = (i & 1) == 0;
      k = i >> 1;
    } else {
      front = nf > nb;
      k = m + (i - 2 * m);
    }
    return front ? b + k * G : T - 1 - b - k * G;
  }
};

// Walk b of G over T tiles.  both_ends: alternate between the heavy front and the light back
// (groups whose jobs differ in depth); otherwise the front walk covers every tile in order, so
// the tiles in flight at any time are consecutive (one band: shared operand panels in L2).
__device__ __forceinline__ TileWalk tile_walk(long long T, int b, int G, bool both_ends) {
  TileWalk w;
  w.T = T;
  w.b = b;
  w.G = G;
  const long long mid = both_ends ? T / 2 : T;
  w.nf = mid > w.b ? (mid - 1 - w.b) / w.G + 1 : 0;
  w.nb = T - 1 - w.b >= mid ? (T - 1 - w.b - mid) / w.G + 1 : 0;
  return w;
}

// Coordinates of a job's local tile: plane-major; inside a plane, bands of kBandRows rows of
// row tiles (2048 operand rows), each walked column tile after column tile with the row tile
// fastest.  The CTAs that run at the same time then share a band's A row panels and its
// column tiles' B panels in L2 (row tile fastest over a whole plane made them share B but spread
// over all of A: about ten times the operand bytes read from DRAM, measured).
constexpr int kBandRows = 2048;
// (tm, tn) of the local tile `local` inside one plane of a job.
__device__ __forceinline__ void band_tile(int local, const GemmJob& jb, int& tm, int& tn) {
  const int tmc = jb.tm, tnc = jb.tn;
  const int band = max(1, kBandRows / jb.bm);
  const int g = local / (band * tnc);
  const int within = local - g * band * tnc;
  const int rows = min(band, tmc - g * band);
  tn = within / rows;
  tm = g * band + (within - tn * rows);
}
__device__ __forceinline__ void job_tile(int local, const GemmJob& jb, int& plane, int& tm,
                                         int& tn) {
  const int per_plane = jb.tm * jb.tn;
  plane = local / per_plane;
  band_tile(local - plane * per_plane, jb, tm, tn);
}

// Walk flags (kGemmWalk*, host-chosen per launch): alternate both ends of the tile order, and
// plane-outer numbering.  Plane-outer (groups whose problems share operands, every job with the
// same plane count): tile t is tile t % T_p of plane t / T_p, with T_p the tiles of one plane
// over all jobs and prefix[] counting one plane's tiles per job, so that one plane of an operand
// shared by many problems (a reuse component's A) stays in L2 while those problems stream past
// it (job-major numbering read the shared A images once per problem: 5x the image bytes from
// DRAM, measured).
// Tile t of the call: its job (warp-parallel owner search, so call by all 32 lanes), plane and
// tile coordinates (a job has fewer than 2^31 tiles).
__device__ __forceinline__ TileInfo decode_tile(const GemmJob* __restrict__ jobs,
                                                const long long* __restrict__ prefix, int num,
                                                long long t, bool plane_outer) {
  TileInfo ti;
  if (plane_outer) {
    const long long tp = prefix[num];
    ti.plane = (int)(t / tp);
    const long long r = t - (long long)ti.plane * tp;
    const int j = find_owner_warp(prefix, num, r);
    ti.job = jobs + j;
    band_tile((int)(r - prefix[j]), *ti.job, ti.tm, ti.tn);
    return ti;
  }
  const int j = find_owner_warp(prefix, num, t);
  ti.job = jobs + j;
  job_tile((int)(t - prefix[j]), *ti.job, ti.plane, ti.tm, ti.tn);
  return ti;
}

// Builds a CTA's tile schedule {job, plane, tm, tn} in shared memory (sched), staging the job
// prefix in `staged` (the still unused operand ring); whole block.
__device__ __forceinline__ void build_schedule(const GemmJob* __restrict__ jobs,
                                               const long long* __restrict__ prefix, int num,
                                               const TileWalk& walk, bool plane_outer,
                                               long long* staged, int4* sched) {
  for (int x = threadIdx.x; x < num; x += blockDim.x) staged[x] = prefix[x];
  __syncthreads();
  const long long tp = plane_outer ? prefix[num] : 1;
  for (int x = threadIdx.x; x < (int)walk.count(); x += blockDim.x) {
    long long t = walk.at(x);
    const int pl = plane_outer ? (int)(t / tp) : 0;
    if (plane_outer) t -= (long long)pl * tp;
    int lo = 0, hi = num - 1;  // largest j with staged[j] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (staged[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    int plane, tm, tn;
    if (plane_outer) {
      plane = pl;
      band_tile((int)(t - staged[lo]), jobs[lo], tm, tn);
    } else {
      job_tile((int)(t - staged[lo]), jobs[lo], plane, tm, tn);
    }
    sched[x] = make_int4(lo, plane, tm, tn);
  }
  __syncthreads();  // the staged prefix in the operand ring is no longer read
}
__device__ __forceinline__ TileInfo sched_tile(const GemmJob* jobs, int4 r) {
  TileInfo ti;
  ti.job = jobs + r.x;
  ti.plane = r.y;
  ti.tm = r.z;
  ti.tn = r.w;
  return ti;
}

__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, GemmSmemCtl* ctl,
                                             DevCounters* cnt) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = global_timer_ns() + kWaitNs;
  if (mbar_wait(bar, parity, deadline, &ctl->abort)) return true;
  ctl->abort = 1;
  atomicCAS(&cnt->status, 0u, (unsigned)kStatusGemmTimeout);
  return false;
}

// CRT digit of an int32 product for one residue plane (the reference computes the same digit
// inside its reconstruct, src/ozaki2_numerics.cu:509-517).  With u = c + 2^31 (unsigned),
// magic = floor(2^32 / p) and p odd or 256:
//   r = u - umulhi(u, magic) p            in [0, 2p), r = c + 2^31 (mod p)
//   x = r q + corr                        < 2^17, corr = (p - 2^31 mod p) q mod p, x = c q (mod p)
//   y = x - umulhi(x, magic) p            in [0, 2p), then min(y, y - p) (unsigned) in [0, p)
// umulhi(u, magic) undershoots floor(u / p) by at most one for every u < 2^32.
struct DigitCtx {
  uint32_t p, magic, q, corr;
  bool digit;  // false: the abs plane (int32 output)
};

// qscaled: the A images hold residues of q_l a (GGEMM_PREP_QSCALED), corr is then the multiple
// of p_l that crt_digit_q adds.
__device__ __forceinline__ DigitCtx digit_ctx(int plane, int N, bool qscaled) {
  DigitCtx dc{1u, 0u, 0u, 0u, plane < N};
  if (dc.digit) {
    dc.p = c_tab.p[plane];
    dc.magic = c_tab.magic[plane];
    dc.q = c_tab.qinv[N][plane];
    dc.corr = qscaled ? (0x80000000u + dc.p - 1u) / dc.p * dc.p
                      : (dc.p - 0x80000000u % dc.p) % dc.p * dc.q % dc.p;
  }
  return dc;
}

__device__ __forceinline__ uint32_t crt_digit(uint32_t c, const DigitCtx& dc) {
  const uint32_t u = c ^ 0x80000000u;
  const uint32_t r = u - __umulhi(u, dc.magic) * dc.p;
  const uint32_t x = r * dc.q + dc.corr;
  const uint32_t y = x - __umulhi(x, dc.magic) * dc.p;
  return min(y, y - dc.p);
}

// Digit of a product of q-scaled residues: c = C'_l = q_l C_l (mod p_l), so y_l = c mod p_l.
// u = c + corr (corr = p ceil(2^31 / p)) lies in [0, 2^32) because |c| <= kMaxKExact 127^2
// for odd p (for p = 256 only u's low byte matters and a wrap is harmless); the quotient
// estimate umulhi(u, floor(2^32 / p)) is low by at most one, so r < 2p.
__device__ __forceinline__ uint32_t crt_digit_q(uint32_t c, const DigitCtx& dc) {
  const uint32_t u = c + dc.corr;
  const uint32_t r = u - __umulhi(u, dc.magic) * dc.p;
  return min(r, r - dc.p);
}

template <bool kQ>
__device__ __forceinline__ uint32_t digit_of(uint32_t c, const DigitCtx& dc) {
  return kQ ? crt_digit_q(c, dc) : crt_digit(c, dc);
}

// 32 columns of one row: two 16-digit records (16 bytes each, at ydst and ydst + dstep) or eight
// 4-product records (at ldst + g * lstep).  Consecutive rows' records are adjacent, so a warp
// (32 consecutive rows) writes 512 contiguous bytes per store instruction.
template <bool kQ>
__device__ __forceinline__ void emit_record(const uint32_t (&v)[32], const DigitCtx& dc,
                                            uint8_t* ydst, long long dstep, int32_t* ldst,
                                            long long lstep) {
  if (dc.digit) {
    uint32_t w[8];
#pragma unroll
    for (int g = 0; g < 8; ++g)
      w[g] = pack4(digit_of<kQ>(v[4 * g], dc), digit_of<kQ>(v[4 * g + 1], dc),
                   digit_of<kQ>(v[4 * g + 2], dc), digit_of<kQ>(v[4 * g + 3], dc));
    *reinterpret_cast<uint4*>(ydst) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(ydst + dstep) = make_uint4(w[4], w[5], w[6], w[7]);
  } else {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      *reinterpret_cast<int4*>(ldst + g * lstep) =
          make_int4((int)v[4 * g], (int)v[4 * g + 1], (int)v[4 * g + 2], (int)v[4 * g + 3]);
  }
}

// Digit-layout epilogue of one tile for one thread (TMEM lane = row of the tile): nch chunks of
// 32 columns.  kQ: the job's A images are q-scaled (GemmJob::y8 == 2).
template <bool kQ>
__device__ __forceinline__ void gemm_digit_records(const GemmJob& jb, const TileInfo& ti, int row,
                                                   uint32_t taddr, int nch) {
  const int pl = jb.plane0 + ti.plane;
  const DigitCtx dc = digit_ctx(pl, jb.N, kQ);
  // digit records of 16 columns, abs records of 4: column j of this row at record j / 16 (j / 4)
  const long long c0 = (long long)ti.tn * jb.bn;  // the tile's first column
  uint8_t* ydst = jb.Y + (long long)pl * jb.y_plane + ((c0 / 16) * jb.m + row) * 16;
  int32_t* ldst = reinterpret_cast<int32_t*>(jb.Y + (long long)jb.N * jb.y_plane) +
                  ((c0 / 4) * jb.m + row) * 4;
  const long long dstep = (long long)jb.m * 16;  // next 16-column digit record (bytes)
  const long long lstep = (long long)jb.m * 4;   // next 4-column abs record (int32)
  const long long cstep = 2 * dstep;             // 32 columns further (bytes)
  const long long lcstep = 8 * lstep;            // ... (int32)
  const bool live = row < jb.m;
  // two register buffers: the TMEM load of chunk c + 1 overlaps the digits of chunk c
  uint32_t va[32], vb[32];
  tmem_ld_32x32b_x32(taddr, va);
  tmem_ld_wait(va);
#pragma unroll 1
  for (int c = 0; c < nch; c += 2) {
    if (c + 1 < nch) tmem_ld_32x32b_x32(taddr + (uint32_t)((c + 1) * 32), vb);
    if (live) emit_record<kQ>(va, dc, ydst + c * cstep, dstep, ldst + c * lcstep, lstep);
    if (c + 1 < nch) {
      tmem_ld_wait(vb);
      if (c + 2 < nch) tmem_ld_32x32b_x32(taddr + (uint32_t)((c + 2) * 32), va);
      if (live)
        emit_record<kQ>(vb, dc, ydst + (c + 1) * cstep, dstep, ldst + (c + 1) * lcstep, lstep);
      if (c + 2 < nch) tmem_ld_wait(va);
    }
  }
}

// Epilogue of one tile for one thread: TMEM lane = row of the tile at taddr (columns from 0),
// products written in the job's layout (digits: gemm_digit_records; int32: column-major planes).
__device__ __forceinline__ void gemm_tile_epilogue(const GemmJob& jb, const TileInfo& ti, int row,
                                                   uint32_t taddr) {
  // record columns of this tile that lie inside the problem
  const int nch = min(jb.bn, jb.n - ti.tn * jb.bn + 31) / 32;
  if (jb.y8 == 2) {
    gemm_digit_records<true>(jb, ti, row, taddr, nch);
  } else if (jb.y8) {
    gemm_digit_records<false>(jb, ti, row, taddr, nch);
  } else {
    int32_t* C = jb.C + (long long)ti.plane * jb.c_plane;
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), v);
      tmem_ld_wait(v);
      const int col0 = ti.tn * jb.bn + c * 32;
      if (row < jb.m) {
        int32_t* cp = C + row + (long long)col0 * jb.m;
        const int ncol = min(32, jb.n - col0);
#pragma unroll
        for (int x = 0; x < 32; ++x)
          if (x < ncol) cp[(long long)x * jb.m] = (int32_t)v[x];
      }
    }
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const GemmJob* __restrict__ jobs, const long long* __restrict__ prefix, int num,
                long long total_tiles, DevCounters* cnt, int walk_flags) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  GemmSmemCtl* ctl = reinterpret_cast<GemmSmemCtl*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], 4);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const TileWalk walk = tile_walk(total_tiles, (int)blockIdx.x, (int)gridDim.x,
                                  (walk_flags & kGemmWalkBothEnds) != 0);
  const bool plane_outer = (walk_flags & kGemmWalkPlaneOuter) != 0;
  int4* sched = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(ctl) +
                                        ((sizeof(GemmSmemCtl) + 63) & ~size_t(63)));
  const bool cached = walk.count() <= kSchedMax && num <= kSchedJobs;  // block-uniform
  if (cached) build_schedule(jobs, prefix, num, walk, plane_outer,
                              reinterpret_cast<long long*>(smem), sched);
  // tile `it` of this CTA's walk (warp-collective when not cached)
  auto tile_of = [&](long long it) -> TileInfo {
    if (cached) return sched_tile(jobs, sched[it]);
    return decode_tile(jobs, prefix, num, walk.at(it), plane_outer);
  };

  if (warp == 0) {
    // --------------------------------------------------------------------- producer
    // Lane 0 waits for a free stage and arms its barrier; lanes [0, kKS) then copy the stage's K
    // steps of A and lanes [kKS, 2 kKS) those of B (parallel issue of the bulk copies).
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, last_par = 0;  // per stage: ever armed / parity of the last arming
    // the abort flag is read warp-uniformly (the tile decode is a warp collective)
    for (long long it = 0;
         it < walk.count() && !__any_sync(0xFFFFFFFFu, *(volatile int*)&ctl->abort); ++it) {
      const TileInfo ti = tile_of(it);
      const GemmJob& jb = *ti.job;
      const int g0a = ti.tm * 16, ga = min(16, jb.rga - g0a);
      const int gbt = jb.bn / 8;
      const int g0b = ti.tn * gbt, gb = min(gbt, jb.rgb - g0b);
      const int8_t* A = jb.A + (long long)ti.plane * jb.a_plane + (long long)g0a * 256;
      const int8_t* B = jb.B + (long long)ti.plane * jb.b_plane + (long long)g0b * 256;
      const long long astep = (long long)jb.rga * 256, bstep = (long long)jb.rgb * 256;
      bool ok = true;
      for (int ks = 0; ks < jb.ksteps; ks += kKS) {
        const int nst = min(kKS, jb.ksteps - ks);
        if (lane == 0) {
          ok = bounded_wait(&ctl->empty[stage], phase ^ 1u, ctl, cnt);
          if (ok) mbar_arrive_expect_tx(&ctl->full[stage], (uint32_t)(nst * (ga + gb) * 256));
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        if (!ok) break;
        armed |= 1u << stage;
        last_par = (last_par & ~(1u << stage)) | (phase << stage);
        uint8_t* sa = smem + stage * kStageBytes;
        uint8_t* sb = sa + kKS * kStepBytesA;
        if (lane < nst)
          bulk_g2s(sa + lane * kStepBytesA, A + (long long)(ks + lane) * astep,
                   (uint32_t)(ga * 256), &ctl->full[stage]);
        else if (lane >= kKS && lane < kKS + nst)
          bulk_g2s(sb + (lane - kKS) * kStepBytesB, B + (long long)(ks + lane - kKS) * bstep,
                   (uint32_t)(gb * 256), &ctl->full[stage]);
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
    // every issued copy has landed before the CTA may exit
    if (lane == 0)
      for (int s = 0; s < kStages; ++s)
        if (armed & (1u << s)) {
          const uint64_t deadline = global_timer_ns() + kWaitNs;
          int dummy_abort = 0;
          mbar_wait(&ctl->full[s], (last_par >> s) & 1u, deadline, &dummy_abort);
        }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the tiles (the tile decode is warp-parallel); lane 0 waits and issues.
    int stage = 0;
    uint32_t phase = 0;
    int buf = 0;
    uint32_t acc_phase = 0;
    bool issued = false;
    // the abort flag is read warp-uniformly (the tile decode is a warp collective)
    for (long long it = 0;
         it < walk.count() && !__any_sync(0xFFFFFFFFu, *(volatile int*)&ctl->abort); ++it) {
      const TileInfo ti = tile_of(it);
      const int ksteps = ti.job->ksteps;
      // MMA width: the tile's columns inside the problem, rounded up to 16 (edge tiles of a
      // ragged n skip the padding columns; the epilogue never reads past the problem's n)
      const int nrem = ti.job->n - ti.tn * ti.job->bn;
      const uint32_t idesc = idesc_i8(kGemmBM, min(ti.job->bn, (nrem + 15) & ~15));
      bool ok = true;
      if (lane == 0) {
        ok = bounded_wait(&ctl->acc_empty[buf], acc_phase ^ 1u, ctl, cnt);
        if (ok) {
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)(buf * kGemmBNMax);
          for (int ks = 0; ks < ksteps; ks += kKS) {
            const int nst = min(kKS, ksteps - ks);
            if (!bounded_wait(&ctl->full[stage], phase, ctl, cnt)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem_addr(smem + stage * kStageBytes);
            const uint32_t sb = sa + kKS * kStepBytesA;
            for (int j = 0; j < nst; ++j) {
              const uint64_t ad = smem_desc_sw32(sa + j * kStepBytesA, 256);
              const uint64_t bd = smem_desc_sw32(sb + j * kStepBytesB, 256);
              mma_i8(d_tmem, ad, bd, idesc, (ks > 0 || j > 0) ? 1u : 0u);
            }
            issued = true;
            mma_commit(&ctl->empty[stage]);
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (ok) mma_commit(&ctl->acc_full[buf]);
        }
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      if (++buf == 2) {
        buf = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0 && issued) {  // all MMAs of this CTA complete before TMEM is released
      mma_commit(&ctl->drain);
      const uint64_t deadline = global_timer_ns() + kWaitNs;
      int dummy_abort = 0;
      mbar_wait(&ctl->drain, 0, deadline, &dummy_abort);
    }
  } else {
    // ------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    int buf = 0;
    uint32_t acc_phase = 0;
    for (long long it = 0; it < walk.count(); ++it) {
      const TileInfo ti = tile_of(it);
      const GemmJob& jb = *ti.job;
      bool ok = true;
      if (lane == 0) ok = bounded_wait(&ctl->acc_full[buf], acc_phase, ctl, cnt);
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row = ti.tm * kGemmBM + quad * 32 + lane;
      const uint32_t taddr = tmem + (uint32_t)(buf * kGemmBNMax) + ((uint32_t)(quad * 32) << 16);
      gemm_tile_epilogue(jb, ti, row, taddr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->acc_empty[buf]);
      if (++buf == 2) {
        buf = 0;
        acc_phase ^= 1u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ======================================================== paired residue GEMM (CTA pairs)
// A cluster of two CTAs computes 256 x 256 tiles with tcgen05.mma.cta_group::2.  CTA r holds the
// tile's A rows [128 r, 128 r + 128) and B rows (tile columns) [r W / 2, (r + 1) W / 2) of the
// tile's MMA width W, in the same shared-memory image layout as gemm_kernel; one thread of CTA 0
// issues the MMAs, and each CTA's TMEM receives its 128 rows x W columns.  Per SM and 32-byte K
// step that is 4 KB of A and 4 KB of B copied into shared memory, against 4 + 8 KB for
// gemm_kernel's 128 x 256 tile.
// Each CTA's producer bulk-copies its own valid row groups into its own shared memory, counted
// on its own stage barrier (the same data path as gemm_kernel; 2D tensor copies of this layout
// measured 1.7x slower).  Warp 1 of CTA 1, idle otherwise, relays each of its stages that landed
// to CTA 0 with one remote arrival on CTA 0's stage barrier, which therefore completes once both
// CTAs' copies of the stage have landed (two arrivals there, one in CTA 1).  MMA commits
// multicast to both CTAs' stage-free and accumulator-full barriers; the epilogue warps of both
// CTAs arrive on CTA 0's accumulator-free barrier.  No load uses cluster multicast.
// Three stages of 8 K steps (64 KB each): on one C5 reuse component the GEMM took 7.44 ms with
// six stages of 4 steps, 6.63 ms with four of 6, 6.07-6.29 ms with three of 8 and 6.41 ms with
// two of 12 (the same 192 KB in every case).
// Every wait is bounded (kWaitNs).  Copies in flight when a CTA gives up land within
// microseconds, long before the partner's own bounded waits end and the CTAs pass the final
// cluster barrier, so neither CTA exits while the other can still touch its shared memory.
constexpr int kStages2 = 3;
constexpr int kKS2 = 8;                                // 32-byte K steps per stage
constexpr int kStepBytes2 = 16 * 256;                  // one K step of 128 rows
constexpr int kStageBytes2 = kKS2 * 2 * kStepBytes2;   // kKS2 K steps of A and of B
constexpr int kGemm2Rows = 256, kGemm2Cols = 256;
struct GemmSmemCtl2 {
  uint64_t full[kStages2], empty[kStages2], acc_full[2], acc_empty[2], drain;
  uint32_t tmem_base;
  int abort;
};
static_assert((kSchedJobs + 1) * 8 <= kStages2 * kStageBytes2, "prefix staging");
constexpr size_t kGemm2Smem =
    1024 + kStages2 * kStageBytes2 + sizeof(GemmSmemCtl2) + 64 + kSchedMax * sizeof(int4);

__device__ __forceinline__ bool bounded_wait_pair(uint64_t* bar, uint32_t parity,
                                                  GemmSmemCtl2* ctl, DevCounters* cnt) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = global_timer_ns() + kWaitNs;
  if (mbar_wait(bar, parity, deadline, &ctl->abort)) return true;
  ctl->abort = 1;
  atomicCAS(&cnt->status, 0u, (unsigned)kStatusGemmTimeout);
  return false;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const GemmJob* __restrict__ jobs, const long long* __restrict__ prefix,
                     int num, long long total_tiles, DevCounters* cnt, int walk_flags) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  GemmSmemCtl2* ctl = reinterpret_cast<GemmSmemCtl2*>(smem + kStages2 * kStageBytes2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      // this CTA's producer arms it and its copies complete it; in CTA 0 also CTA 1's relay
      mbar_init(&ctl->full[s], rank == 0 ? 2 : 1);
      mbar_init(&ctl->empty[s], 1);      // one multicast commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);   // one multicast commit
      mbar_init(&ctl->acc_empty[b], 8);  // 4 epilogue warps of each CTA (used in CTA 0)
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(&ctl->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  // the pair's walk: pair b of G pairs (both CTAs of a pair walk the same tiles)
  const TileWalk walk =
      tile_walk(total_tiles, (int)(blockIdx.x >> 1), (int)(gridDim.x >> 1),
                (walk_flags & kGemmWalkBothEnds) != 0);
  const bool plane_outer = (walk_flags & kGemmWalkPlaneOuter) != 0;
  int4* sched = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(ctl) +
                                        ((sizeof(GemmSmemCtl2) + 63) & ~size_t(63)));
  const bool cached = walk.count() <= kSchedMax && num <= kSchedJobs;  // block-uniform
  if (cached) build_schedule(jobs, prefix, num, walk, plane_outer,
                              reinterpret_cast<long long*>(smem), sched);
  auto tile_of = [&](long long it) -> TileInfo {
    if (cached) return sched_tile(jobs, sched[it]);
    return decode_tile(jobs, prefix, num, walk.at(it), plane_outer);
  };
  // MMA width of a tile: its columns inside the problem, rounded up to 32 (each CTA then holds
  // a multiple of 16 B rows)
  auto width_of = [](const GemmJob& jb, int tn) {
    return min(kGemm2Cols, (jb.n - tn * kGemm2Cols + 31) & ~31);
  };

  if (warp == 0) {
    // --------------------------------------------------------------------- producer
    // valid row groups of this CTA: A rows [256 tm + 128 r, + 128), B rows (tile columns)
    // [256 tn + r W / 2, + W / 2); groups past the image are not copied (their accumulator rows /
    // columns are never stored)
    int stage = 0;
    uint32_t phase = 0;
    for (long long it = 0;
         it < walk.count() && !__any_sync(0xFFFFFFFFu, *(volatile int*)&ctl->abort); ++it) {
      const TileInfo ti = tile_of(it);
      const GemmJob& jb = *ti.job;
      const int W = width_of(jb, ti.tn);
      const int g0a = ti.tm * 32 + (int)rank * 16;
      const int g0b = ti.tn * 32 + (int)rank * (W / 16);
      const int ga = max(0, min(16, jb.rga - g0a));
      const int gb = max(0, min(W / 16, jb.rgb - g0b));
      const int8_t* A = jb.A + (long long)ti.plane * jb.a_plane + (long long)g0a * 256;
      const int8_t* B = jb.B + (long long)ti.plane * jb.b_plane + (long long)g0b * 256;
      const long long astep = (long long)jb.rga * 256, bstep = (long long)jb.rgb * 256;
      bool ok = true;
      for (int ks = 0; ks < jb.ksteps; ks += kKS2) {
        const int nst = min(kKS2, jb.ksteps - ks);
        if (lane == 0) {
          ok = bounded_wait_pair(&ctl->empty[stage], phase ^ 1u, ctl, cnt);
          if (ok) mbar_arrive_expect_tx(&ctl->full[stage], (uint32_t)(nst * (ga + gb) * 256));
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        if (!ok) break;
        uint8_t* sa = smem + stage * kStageBytes2;
        uint8_t* sb = sa + kKS2 * kStepBytes2;
        if (lane < nst) {
          if (ga > 0)
            bulk_g2s(sa + lane * kStepBytes2, A + (long long)(ks + lane) * astep,
                     (uint32_t)(ga * 256), &ctl->full[stage]);
        } else if (lane >= kKS2 && lane < kKS2 + nst) {
          if (gb > 0)
            bulk_g2s(sb + (lane - kKS2) * kStepBytes2, B + (long long)(ks + lane - kKS2) * bstep,
                     (uint32_t)(gb * 256), &ctl->full[stage]);
        }
        __syncwarp();
        if (++stage == kStages2) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else if (warp == 1 && rank == 0) {
    // ------------------------------------------------------- MMA issuer (CTA 0, one lane)
    int stage = 0;
    uint32_t phase = 0;
    int buf = 0;
    uint32_t acc_phase = 0;
    for (long long it = 0;
         it < walk.count() && !__any_sync(0xFFFFFFFFu, *(volatile int*)&ctl->abort); ++it) {
      const TileInfo ti = tile_of(it);
      const int ksteps = ti.job->ksteps;
      const uint32_t idesc = idesc_i8(kGemm2Rows, width_of(*ti.job, ti.tn));
      bool ok = true;
      if (lane == 0) {
        ok = bounded_wait_pair(&ctl->acc_empty[buf], acc_phase ^ 1u, ctl, cnt);
        if (ok) {
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)(buf * kGemm2Cols);
          for (int ks = 0; ks < ksteps; ks += kKS2) {
            const int nst = min(kKS2, ksteps - ks);
            if (!bounded_wait_pair(&ctl->full[stage], phase, ctl, cnt)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_addr(smem + stage * kStageBytes2);
            const uint32_t sb = sa + kKS2 * kStepBytes2;
            for (int j = 0; j < nst; ++j) {
              const uint64_t ad = smem_desc_sw32(sa + j * kStepBytes2, 256);
              const uint64_t bd = smem_desc_sw32(sb + j * kStepBytes2, 256);
              mma_i8_pair(d_tmem, ad, bd, idesc, (ks > 0 || j > 0) ? 1u : 0u);
            }
            mma_commit_pair(&ctl->empty[stage], 3);
            if (++stage == kStages2) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (ok) mma_commit_pair(&ctl->acc_full[buf], 3);
        }
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      if (++buf == 2) {
        buf = 0;
        acc_phase ^= 1u;
      }
    }
    // both CTAs' drain barriers complete once every MMA issued above has completed
    if (lane == 0) mma_commit_pair(&ctl->drain, 3);
  } else if (warp == 1) {
    // ------------------------------------------------------------- relay (CTA 1, one lane)
    int stage = 0;
    uint32_t phase = 0;
    for (long long it = 0;
         it < walk.count() && !__any_sync(0xFFFFFFFFu, *(volatile int*)&ctl->abort); ++it) {
      const int ksteps = tile_of(it).job->ksteps;
      bool ok = true;
      if (lane == 0) {
        for (int ks = 0; ks < ksteps; ks += kKS2) {
          if (!bounded_wait_pair(&ctl->full[stage], phase, ctl, cnt)) {
            ok = false;
            break;
          }
          mbar_arrive_cluster(mapa_shared(smem_addr(&ctl->full[stage]), 0));
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    int buf = 0;
    uint32_t acc_phase = 0;
    for (long long it = 0; it < walk.count(); ++it) {
      const TileInfo ti = tile_of(it);
      const GemmJob& jb = *ti.job;
      bool ok = true;
      if (lane == 0) ok = bounded_wait_pair(&ctl->acc_full[buf], acc_phase, ctl, cnt);
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row = ti.tm * kGemm2Rows + (int)rank * 128 + quad * 32 + lane;
      const uint32_t taddr = tmem + (uint32_t)(buf * kGemm2Cols) + ((uint32_t)(quad * 32) << 16);
      gemm_tile_epilogue(jb, ti, row, taddr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&ctl->acc_empty[buf]), 0));
      if (++buf == 2) {
        buf = 0;
        acc_phase ^= 1u;
      }
    }
  }
  // every MMA of the pair has completed before TMEM is released, and neither CTA exits before
  // the other is done with the pair's barriers and shared memory
  if (threadIdx.x == 0) {
    int no_abort = 0;
    mbar_wait(&ctl->drain, 0, global_timer_ns() + kWaitNs, &no_abort);
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 0) tmem_dealloc_pair(tmem, 512);
}

// ================================================================== bounded-wait probe
__global__ void __launch_bounds__(32, 1)
    wait_probe_kernel(DevCounters* __restrict__ cnt, unsigned long long wait_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    // phase 0 never completes: no thread arrives on `bar`
    if (!mbar_wait(&bar, 0, global_timer_ns() + wait_ns, &abort))
      atomicCAS(&cnt->status, 0u, (unsigned)kStatusProbeTimeout);
  }
  __syncwarp();
}

// ======================================================================= reconstruct kernel
// y mod p for 0 <= y < 2^32, magic = floor(2^32 / p): the estimate undershoots by at most one.
__device__ __forceinline__ uint32_t mod_p(uint32_t y, uint32_t p, uint32_t magic) {
  const uint32_t q = __umulhi(y, magic);
  const uint32_t r = y - q * p;
  return r >= p ? r - p : r;
}

// Sequential fma dot product over k (src/ozaki2_numerics.cu:445-452): the same rounding as a
// native FP64 dot, used for repairs and for rows / columns containing NaN or Inf.
__device__ __forceinline__ double fp64_dot(const ggemm_recon_desc_t& d, int i, int j) {
  const double* a = d.A + i;
  const double* b = d.B + (long long)j * d.ldb;
  double s = 0.0;
  for (int q = 0; q < d.k; ++q) s = fma(a[(long long)q * d.lda], b[q], s);
  return s;
}

// Per-problem constants of the reconstruct (hoisted out of the entry loop).
struct ReconCtx {
  double gam, crt_u, inv_u1;
  int N, lu1;
};

__device__ __forceinline__ ReconCtx recon_ctx(const ggemm_recon_desc_t& d) {
  ReconCtx cx;
  const double u = 0x1p-53;
  const double nt = (double)d.k + (d.alpha != 1.0 ? 1.0 : 0.0) + (d.beta != 0.0 ? 1.0 : 0.0);
  cx.gam = (nt * u / fma(-nt, u, 1.0) - 2.0 * u) * (1.0 - 0x1p-40);
  cx.N = d.N;
  cx.lu1 = c_tab.log2_u1[d.N];
  cx.crt_u = d.N * 255.0 * 0x1p-19 + 0x1p-10;
  cx.inv_u1 = __longlong_as_double((long long)(1023 - cx.lu1) << 52);
  return cx;
}

// S1 = sum s1_l y_l, S2 = sum s2_l y_l with y_l = (c_l mod p_l) q_l mod p_l (exact integers).
__device__ __forceinline__ void crt_sums(const int32_t (&v)[kMaxModuli + 1], int N, uint64_t& S1,
                                         uint32_t& S2) {
  S1 = 0;
  S2 = 0;
#pragma unroll
  for (int l = 0; l < kMaxModuli; ++l) {
    if (l >= N) break;
    const uint32_t p = c_tab.p[l], mg = c_tab.magic[l];
    const int32_t c = v[l];
    const uint32_t uc = c < 0 ? 0u - (uint32_t)c : (uint32_t)c;
    uint32_t r = mod_p(uc, p, mg);
    if (c < 0 && r) r = p - r;
    const uint32_t y = mod_p(r * c_tab.qinv[N][l], p, mg);
    S1 += c_tab.s1[N][l] * (uint64_t)y;
    S2 += c_tab.s2[N][l] * y;
  }
}

// Replaces *cp by alpha * r + beta * c0, r the sequential FP64 dot of row i and column j.
__device__ __forceinline__ void dot_entry(const ggemm_recon_desc_t& d, int i, int j, double* cp,
                                          double c0) {
  const double r = fp64_dot(d, i, j);
  *cp = (d.beta == 0.0) ? d.alpha * r : fma(d.alpha, r, d.beta * c0);
}

// Everything after the CRT sums for one entry (src/ozaki2_numerics.cu:519-563).  Returns true
// for an uncertified entry in REPAIR_ON mode, which is left unwritten: the caller repairs it
// with dot_entry (kept out of this function so that its loop is not inlined per entry).
__device__ __forceinline__ bool recon_finish(const ggemm_recon_desc_t& d, const ReconCtx& cx,
                                             int mode, double* cp, double c0, uint64_t S1,
                                             uint32_t S2, int32_t L32, int rsh, int csh, int sig,
                                             int tau, double da, double na, double db, double nb,
                                             unsigned& n_unc) {
  const double alpha = d.alpha, beta = d.beta;
  const int N = cx.N;
  const double s2d = (double)S2 * 0x1p-18;
  const double Q = rint(((double)S1 + s2d) * c_tab.inv_Pu[N]);
  const long long X1 = (long long)S1 - (long long)Q * c_tab.P1[N];
  const double xr = (double)X1 + fma(-Q, c_tab.P2[N], s2d);
  const int esc = cx.lu1 - rsh - csh;
  const double v = mul_pow2_nb(xr, esc);
  const double emu = (beta == 0.0) ? alpha * v : fma(alpha, v, beta * c0);
  if (mode == GGEMM_STAGE_REPAIR_OFF || (beta != 0.0 && !(fabs(c0) < INFINITY))) {
    *cp = emu;
    return false;
  }
  const double u = 0x1p-53;
  const double et = fma(da, nb, fma(na, db, da * db)) * (1.0 + 0x1p-40);
  const double Eu = fma(4.0 * u, fabs(xr), fma(et, cx.inv_u1, cx.crt_u)) * (1.0 + 0x1p-40);
  const double E = mul_pow2_nb(Eu, esc);
  double lab = mul_pow2_nb((double)L32, -(sig + tau));
  // fmax(lab, |v| - E): lab is never NaN, and a NaN difference keeps lab, as fmax does; the
  // sign of a zero result is erased below
  const double dv = fabs(v) - E;
  lab = (dv > lab ? dv : lab) * (1.0 - 0x1p-40);
  if (lab < 0x1p-1000) lab = 0.0;
  const double aalpha = fabs(alpha);
  const double lhs = aalpha * E * (1.0 + 0x1p-40);
  const double rhs = cx.gam * fma(aalpha, lab, fabs(beta * c0)) * (1.0 - 0x1p-40);
  const bool cert = cx.gam > 0.0 && E >= 0x1p-1000 && fabs(lhs) < INFINITY &&
                    fabs(v) < INFINITY && lhs <= rhs;
  if (cert || mode == GGEMM_STAGE_REPAIR_COUNT) {
    *cp = emu;
    n_unc += cert ? 0u : 1u;
    return false;
  }
  return true;
}

// The cases that never read the products (src/ozaki2_numerics.cu:492-504).  Returns 0 for an
// ordinary entry, 1 when the entry is done, 2 for a row or column containing NaN or Inf: the
// entry is left unwritten and the caller computes it with dot_entry (the safety fallback).
__device__ __forceinline__ int recon_special(const ggemm_recon_desc_t& d, double* cp, double c0,
                                             int rsh, int csh, int sig, int tau) {
  const double alpha = d.alpha, beta = d.beta;
  if (alpha == 0.0) {
    *cp = (beta == 0.0) ? 0.0 : beta * c0;
    return 1;
  }
  if (rsh == kShiftNonfinite || csh == kShiftNonfinite) return 2;
  if (sig == kShiftZero || tau == kShiftZero) {
    *cp = (beta == 0.0) ? alpha * 0.0 : fma(alpha, 0.0, beta * c0);
    return 1;
  }
  return 0;
}

// One entry, scalar loads (any m).
__device__ __forceinline__ void recon_entry(const ggemm_recon_desc_t& d, const ReconCtx& cx,
                                            int mode, long long idx, int i, int j,
                                            unsigned& n_unc, unsigned& n_rep, unsigned& n_saf) {
  double* cp = d.C + i + (long long)j * d.ldc;
  const double c0 = (d.beta == 0.0) ? 0.0 : *cp;
  const int rsh = d.alpha == 0.0 ? 0 : d.rs[i], csh = d.alpha == 0.0 ? 0 : d.cs[j];
  const int sig = d.alpha == 0.0 ? 0 : d.rs[d.m + i], tau = d.alpha == 0.0 ? 0 : d.cs[d.n + j];
  if (const int sp = recon_special(d, cp, c0, rsh, csh, sig, tau)) {
    n_saf += sp == 2 ? 1u : 0u;  // computed by the safety blocks
    return;
  }
  int32_t v[kMaxModuli + 1];
  const int32_t* __restrict__ C32 = d.C32 + idx;
#pragma unroll
  for (int l = 0; l <= kMaxModuli; ++l)
    if (l <= cx.N) v[l] = __ldg(C32 + l * d.c_plane);
  uint64_t S1;
  uint32_t S2;
  crt_sums(v, cx.N, S1, S2);
  int32_t L = 0;
#pragma unroll
  for (int l = 0; l <= kMaxModuli; ++l)
    if (l == cx.N) L = v[l];
  if (recon_finish(d, cx, mode, cp, c0, S1, S2, L, rsh, csh, sig, tau,
                   __int_as_float(d.rs[2 * d.m + i]), __int_as_float(d.rs[3 * d.m + i]),
                   __int_as_float(d.cs[2 * d.n + j]), __int_as_float(d.cs[3 * d.n + j]), n_unc)) {
    dot_entry(d, i, j, cp, c0);
    ++n_rep;
  }
}

// Two consecutive rows i0, i0+1 of column j with 8-byte loads of every plane (m even): all
// N+1 loads are issued before any arithmetic, so each thread keeps (N+1) x 8 bytes in flight.
__device__ __forceinline__ void recon_pair(const ggemm_recon_desc_t& d, const ReconCtx& cx,
                                           int mode, long long e0, int i0, int j,
                                           unsigned& n_unc, unsigned& n_rep, unsigned& n_saf) {
  const int N = cx.N;
  int2 c2[kMaxModuli + 1];
  const int2* __restrict__ src = reinterpret_cast<const int2*>(d.C32 + e0);
  const long long pst = d.c_plane >> 1;
  const bool need_planes = d.alpha != 0.0 && d.k > 0;  // k == 0: every entry is special
  if (need_planes) {
#pragma unroll
    for (int l = 0; l <= kMaxModuli; ++l)
      if (l <= N) c2[l] = __ldg(src + l * pst);
  }
  const double beta = d.beta;
  double* cbase = d.C + i0 + (long long)j * d.ldc;
  int2 rsh2 = make_int2(0, 0), sig2 = rsh2, da2 = rsh2, na2 = rsh2;
  int csh = 0, tau = 0;
  float fdb = 0.f, fnb = 0.f;
  if (need_planes) {
    rsh2 = __ldg(reinterpret_cast<const int2*>(d.rs + i0));
    sig2 = __ldg(reinterpret_cast<const int2*>(d.rs + d.m + i0));
    da2 = __ldg(reinterpret_cast<const int2*>(d.rs + 2 * d.m + i0));
    na2 = __ldg(reinterpret_cast<const int2*>(d.rs + 3 * d.m + i0));
    csh = __ldg(d.cs + j);
    tau = __ldg(d.cs + d.n + j);
    fdb = __int_as_float(__ldg(d.cs + 2 * d.n + j));
    fnb = __int_as_float(__ldg(d.cs + 3 * d.n + j));
  }
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    double* cp = cbase + x;
    const double c0 = (beta == 0.0) ? 0.0 : *cp;
    const int rsh = x ? rsh2.y : rsh2.x, sig = x ? sig2.y : sig2.x;
    if (const int sp = recon_special(d, cp, c0, rsh, csh, sig, tau)) {
      n_saf += sp == 2 ? 1u : 0u;  // computed by the safety blocks
      continue;
    }
    int32_t v[kMaxModuli + 1];
#pragma unroll
    for (int l = 0; l <= kMaxModuli; ++l) v[l] = x ? c2[l].y : c2[l].x;
    uint64_t S1;
    uint32_t S2;
    crt_sums(v, N, S1, S2);
    int32_t L = 0;
#pragma unroll
    for (int l = 0; l <= kMaxModuli; ++l)
      if (l == N) L = v[l];
    if (recon_finish(d, cx, mode, cp, c0, S1, S2, L, rsh, csh, sig, tau,
                     __int_as_float(x ? da2.y : da2.x), __int_as_float(x ? na2.y : na2.x), fdb,
                     fnb, n_unc)) {
      dot_entry(d, i0 + x, j, cp, c0);
      ++n_rep;
    }
  }
}

// Block-level reduction of the three counters: at most one atomic per counter per block.
// Every thread of the block calls it.
__device__ __forceinline__ void flush_counters(unsigned n_unc, unsigned n_rep, unsigned n_saf,
                                               DevCounters* cnt) {
  unsigned long long cu = n_unc, cr = n_rep, cf = n_saf;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    cu += __shfl_xor_sync(0xFFFFFFFFu, cu, o);
    cr += __shfl_xor_sync(0xFFFFFFFFu, cr, o);
    cf += __shfl_xor_sync(0xFFFFFFFFu, cf, o);
  }
  __shared__ unsigned long long s_cnt[3][kReconThreads / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    s_cnt[0][w] = cu;
    s_cnt[1][w] = cr;
    s_cnt[2][w] = cf;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    unsigned long long t = 0;
    for (int x = 0; x < kReconThreads / 32; ++x) t += s_cnt[threadIdx.x][x];
    if (t) {
      unsigned long long* dst = threadIdx.x == 0 ? &cnt->uncertified
                                : threadIdx.x == 1 ? &cnt->repaired
                                                   : &cnt->safety;
      atomicAdd(dst, t);
    }
  }
}

// Reconstruct from int32 products: block `local` of the problem takes 1024 consecutive
// column-major entries, 4 per thread (two pairs when m is even).
// Not inlined: the digit-layout body then keeps all 128 registers for itself (the int32 body
// is the rare layout, used only for narrow problems).
__device__ __noinline__ void recon_c32_block(const ggemm_recon_desc_t* __restrict__ dp,
                                             long long local, int mode, unsigned& n_unc,
                                             unsigned& n_rep, unsigned& n_saf) {
  const ggemm_recon_desc_t d = *dp;
  if (d.N >= 1 && d.N <= kMaxModuli && d.m > 0 && d.n > 0) {
    const ReconCtx cx = recon_ctx(d);
    const long long mn = (long long)d.m * d.n;
    const long long base = local * (kReconThreads * kReconPerThread);
    const bool vec = (d.m & 1) == 0 && (d.c_plane & 1) == 0 &&
                     ((uintptr_t)d.C32 & 7) == 0 && ((uintptr_t)d.rs & 7) == 0;
    if (vec) {
#pragma unroll 1
      for (int e = 0; e < kReconPerThread / 2; ++e) {
        const long long e0 = base + 2 * ((long long)e * kReconThreads + threadIdx.x);
        if (e0 >= mn) break;
        const int j = (int)(e0 / d.m);
        recon_pair(d, cx, mode, e0, (int)(e0 - (long long)j * d.m), j, n_unc, n_rep, n_saf);
      }
    } else {
#pragma unroll 1
      for (int e = 0; e < kReconPerThread; ++e) {
        const long long idx = base + e * kReconThreads + threadIdx.x;
        if (idx >= mn) break;
        const int j = (int)(idx / d.m);
        const int i = (int)(idx - (long long)j * d.m);
        recon_entry(d, cx, mode, idx, i, j, n_unc, n_rep, n_saf);
      }
    }
  }
}

// Reconstruct from the digit layout.  Block: kY8Rows rows x one 16-column digit record; thread t
// takes row kY8Rows b + t / 2 and the 8 columns 8 (t % 2) .. 8 (t % 2) + 7 of the record, so
// that a warp reads 256 contiguous bytes of each digit plane per load.  The digit and abs-plane
// loads of a thread (8 bytes per digit plane, 32 bytes of the abs plane) are all issued before
// its first arithmetic.  The CRT sums run plane by plane over the thread's 8 entries, so each
// plane's weights are read once per thread instead of once per entry.  Column statistics are
// read per entry (L1 hits).  Every thread of the block calls it.
template <int kN>
__device__ __forceinline__ void recon_y8_block(const ggemm_recon_desc_t& d, long long local,
                                               int mode, unsigned& n_unc, unsigned& n_rep,
                                               unsigned& n_saf) {
  // block: kY8Rows rows x one 16-column digit record; thread: row i, columns j0 .. j0 + 7 (half
  // cg of the record).  A warp (16 rows) reads 256 contiguous bytes of a digit plane.
  const bool ok_desc = d.N >= 1 && d.N <= kMaxModuli && d.m > 0 && d.n > 0;
  const long long rblocks = ok_desc ? (d.m + kY8Rows - 1) / kY8Rows : 1;
  const int ch = ok_desc ? (int)(local / rblocks) : 0;
  const int i = (int)(local - ch * rblocks) * kY8Rows + (threadIdx.x >> 1);
  const int cg = threadIdx.x & 1;
  const bool planes = ok_desc && d.alpha != 0.0 && d.k > 0;
  if (!ok_desc || i >= d.m) return;
  ReconCtx cx = recon_ctx(d);
  if constexpr (kN > 0) cx.N = kN;  // an instance for this moduli count only (host-sorted)
  const int N = cx.N;
  const int j0 = ch * 16 + cg * 8;
  const int ncol = min(8, d.n - j0);
  // columns j0 .. j0 + 7: half cg of digit record ch, abs records 4 ch + 2 cg and the next one
  const long long rec = ((long long)ch * d.m + i) * 16 + cg * 8;
  const long long lrec = ((long long)(4 * ch + 2 * cg) * d.m + i) * 4;
  const uint8_t* Y = reinterpret_cast<const uint8_t*>(d.C32);
  uint2 yv[kMaxModuli];
  int4 l0 = make_int4(0, 0, 0, 0), l1 = l0;
  if (planes) {
#pragma unroll
    for (int l = 0; l < kMaxModuli; ++l)
      if (l < N) yv[l] = __ldg(reinterpret_cast<const uint2*>(Y + l * d.c_plane + rec));
    const int32_t* lp = reinterpret_cast<const int32_t*>(Y + (long long)N * d.c_plane) + lrec;
    l0 = __ldg(reinterpret_cast<const int4*>(lp));
    l1 = __ldg(reinterpret_cast<const int4*>(lp + 4LL * d.m));
  }
  int rsh = 0, sig = 0;
  double da = 0.0, na = 0.0;
  if (d.alpha != 0.0) {
    rsh = __ldg(d.rs + i);
    sig = __ldg(d.rs + d.m + i);
    da = (double)__int_as_float(__ldg(d.rs + 2 * d.m + i));
    na = (double)__int_as_float(__ldg(d.rs + 3 * d.m + i));
  }
  double* crow = d.C + i + (long long)j0 * d.ldc;
  double c8[8];  // the thread's 8 entries of C
#pragma unroll
  for (int x = 0; x < 8; ++x) c8[x] = (d.beta != 0.0 && x < ncol) ? crow[x * d.ldc] : 0.0;
  // CRT sums of the 8 entries, plane by plane
  uint64_t S1[8];
  uint32_t S2[8];
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    S1[x] = 0;
    S2[x] = 0;
  }
  if (planes) {
#pragma unroll
    for (int l = 0; l < kMaxModuli; ++l) {
      if (l >= N) break;
      const uint64_t w1 = c_tab.s1[N][l];
      const uint32_t w2 = c_tab.s2[N][l];
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const uint32_t y = __byte_perm(x < 4 ? yv[l].x : yv[l].y, 0u, 0x4440u + (x & 3));
        S1[x] += w1 * y;
        S2[x] += w2 * y;
      }
    }
  }
  // two halves of four entries (unrolled: the finishing code of the second half overlaps the
  // first's, measured faster than one copy); entries that need an FP64 dot (safety fallback,
  // repair) are only marked here
  unsigned need_saf = 0, need_rep = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int xb = 4 * h;
    if (xb >= ncol) break;
    const int4 lq = h ? l1 : l0;
    const double* c0 = c8 + xb;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      if (xb + x >= ncol) break;
      double* cp = crow + (xb + x) * d.ldc;
      // the column's shifts and norms, read per entry (L1 hits: every row of the block reads
      // the same 16 columns) instead of staged in shared memory behind a block barrier
      const int jx = j0 + xb + x;
      const bool av = d.alpha != 0.0;
      const int csh = av ? __ldg(d.cs + jx) : 0, tau = av ? __ldg(d.cs + d.n + jx) : 0;
      if (const int sp = recon_special(d, cp, c0[x], rsh, csh, sig, tau)) {
        need_saf |= (sp == 2 ? 1u : 0u) << (xb + x);
        continue;
      }
      const int32_t L = x == 0 ? lq.x : x == 1 ? lq.y : x == 2 ? lq.z : lq.w;
      if (recon_finish(d, cx, mode, cp, c0[x], h ? S1[4 + x] : S1[x], h ? S2[4 + x] : S2[x], L,
                       rsh, csh, sig, tau, da, na,
                       (double)__int_as_float(__ldg(d.cs + 2 * d.n + jx)),
                       (double)__int_as_float(__ldg(d.cs + 3 * d.n + jx)), n_unc))
        need_rep |= 1u << (xb + x);
    }
  }
  n_saf += __popc(need_saf);  // computed by the safety blocks
  n_rep += __popc(need_rep);
  for (unsigned need = need_rep; need; need &= need - 1) {
    const int x = __ffs(need) - 1;
    double* cp = crow + x * d.ldc;
    dot_entry(d, i, j0 + x, cp, d.beta != 0.0 ? *cp : 0.0);
  }
}

// ======================================================================= safety fallback
// Entries in a row of A or a column of B that holds NaN or Inf (prep's non-finite shift) are not
// emulated: each becomes alpha * dot + beta * C(i, j), dot the sequential FP64 fma chain over
// q = 0 .. k-1 from 0.0 (the reference's per-entry loop, src/ozaki2_numerics.cu:445-452, 492-497).
// The reconstruct only counts them; this kernel computes them in tiles of up to 64 x 64 entries,
// 4 x 4 per thread, the operands staged in shared memory kSafeK K positions at a time.  Every
// entry's chain is the same sequence of fma operations (same operands, same order, no padding
// steps) as the per-entry loop, so the values are the same bit for bit, NaN and Inf included.
// Work items of a problem (alpha != 0): side R, the poisoned rows of a 64-row tile against a
// 64-column tile, all written; side C, the poisoned columns of a 64-column tile against a 64-row
// tile, written only in rows that are not poisoned (side R writes the others).
constexpr int kSafeTile = 64, kSafeK = 32, kSafeThreads = 256;
constexpr int kSafeLdB = kSafeTile + 2;  // b rows padded (16-byte aligned, fewer store conflicts)

struct SafeSmem {
  double a[kSafeK][kSafeTile];  // a[q][r] = A(rows[r], k0 + q)
  double b[kSafeK][kSafeLdB];   // b[q][c] = B(k0 + q, cols[c])
  int rows[kSafeTile], cols[kSafeTile];
  unsigned char write_row[kSafeTile];
  int nr, nc;
};

__device__ __forceinline__ long long safety_items(const ggemm_recon_desc_t& d) {
  if (d.N < 1 || d.N > kMaxModuli || d.m <= 0 || d.n <= 0 || d.k <= 0 || d.alpha == 0.0)
    return 0;
  return 2LL * ((d.m + kSafeTile - 1) / kSafeTile) * ((d.n + kSafeTile - 1) / kSafeTile);
}

// Compacts the indices [i0, i0 + 64) ∩ [0, len) of one side into list[]: with `poisoned` the
// ones whose shift is non-finite, otherwise all of them (write[], when given, marks the clean
// ones).  Called by one warp; returns the count.
__device__ __forceinline__ int safety_list(const int32_t* __restrict__ shift, int i0, int len,
                                           bool poisoned, int* list, unsigned char* write) {
  const int lane = threadIdx.x & 31;
  int n = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = i0 + 32 * h + lane;
    const bool in = i < len;
    const bool bad = in && __ldg(shift + i) == kShiftNonfinite;
    const bool take = poisoned ? bad : in;
    const unsigned msk = __ballot_sync(0xFFFFFFFFu, take);
    if (take) {
      const int pos = n + __popc(msk & ((1u << lane) - 1u));
      list[pos] = i;
      if (write) write[pos] = bad ? 0 : 1;
    }
    n += __popc(msk);
  }
  return n;
}

// Work item t of problem d (every thread of the block calls it).
__device__ void safety_item(const ggemm_recon_desc_t& d, long long t, SafeSmem& sm) {
  const int RT = (d.m + kSafeTile - 1) / kSafeTile, CT = (d.n + kSafeTile - 1) / kSafeTile;
  const long long per = (long long)RT * CT;
  const bool side_c = t >= per;
  const long long u = side_c ? t - per : t;
  const int rt = (int)(u / CT), ct = (int)(u - (long long)rt * CT);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (w == 0) {
    const int n = safety_list(d.rs, rt * kSafeTile, d.m, !side_c, sm.rows,
                              side_c ? sm.write_row : nullptr);
    if (!side_c) {
      sm.write_row[lane] = 1;
      sm.write_row[lane + 32] = 1;
    }
    if (lane == 0) sm.nr = n;
  } else if (w == 1) {
    const int n = safety_list(d.cs, ct * kSafeTile, d.n, side_c, sm.cols, nullptr);
    if (lane == 0) sm.nc = n;
  }
  __syncthreads();
  const int nr = sm.nr, nc = sm.nc;  // block-uniform
  if (nr > 0 && nc > 0) {
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // columns 4 tx .., rows 4 ty ..
    const bool live = 4 * ty < nr && 4 * tx < nc;
    double acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
    // the operands of chunk k0 + kSafeK are loaded into registers while chunk k0 is computed
    constexpr int kPer = kSafeK * kSafeTile / kSafeThreads;
    double ra[kPer], rb[kPer];
    auto fetch = [&](int k0) {
      const int kq = min(kSafeK, d.k - k0);
      // A: element e -> row slot e % 64, K position e / 64 (a warp reads consecutive rows of one
      // column); slots past nr repeat the last row (read, never used)
#pragma unroll
      for (int x = 0; x < kPer; ++x) {
        const int e = threadIdx.x + kSafeThreads * x;
        const int r = e & (kSafeTile - 1), q = e / kSafeTile;
        const int row = sm.rows[min(r, nr - 1)];
        ra[x] = q < kq ? __ldg(d.A + row + (long long)(k0 + q) * d.lda) : 0.0;
      }
      // B: element e -> K position e % 32, column slot e / 32 (a warp reads 32 consecutive K
      // positions of one column)
#pragma unroll
      for (int x = 0; x < kPer; ++x) {
        const int e = threadIdx.x + kSafeThreads * x;
        const int q = e & (kSafeK - 1), c = e / kSafeK;
        const int col = sm.cols[min(c, nc - 1)];
        rb[x] = q < kq ? __ldg(d.B + (k0 + q) + (long long)col * d.ldb) : 0.0;
      }
    };
    fetch(0);
    for (int k0 = 0; k0 < d.k; k0 += kSafeK) {
      const int kq = min(kSafeK, d.k - k0);
#pragma unroll
      for (int x = 0; x < kPer; ++x) {
        const int e = threadIdx.x + kSafeThreads * x;
        sm.a[e / kSafeTile][e & (kSafeTile - 1)] = ra[x];
        sm.b[e & (kSafeK - 1)][e / kSafeK] = rb[x];
      }
      __syncthreads();
      if (k0 + kSafeK < d.k) fetch(k0 + kSafeK);
      if (live) {
#pragma unroll 4
        for (int q = 0; q < kq; ++q) {  // exactly the chain's steps k0 .. k0 + kq - 1
          const double2 a01 = *reinterpret_cast<const double2*>(&sm.a[q][4 * ty]);
          const double2 a23 = *reinterpret_cast<const double2*>(&sm.a[q][4 * ty + 2]);
          const double2 b01 = *reinterpret_cast<const double2*>(&sm.b[q][4 * tx]);
          const double2 b23 = *reinterpret_cast<const double2*>(&sm.b[q][4 * tx + 2]);
          const double av[4] = {a01.x, a01.y, a23.x, a23.y};
          const double bv[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
      }
      __syncthreads();
    }
    if (live) {
      const double alpha = d.alpha, beta = d.beta;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * ty + i;
        if (r >= nr || !sm.write_row[r]) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = 4 * tx + j;
          if (c >= nc) continue;
          double* cp = d.C + sm.rows[r] + (long long)sm.cols[c] * d.ldc;
          *cp = (beta == 0.0) ? alpha * acc[i][j] : fma(alpha, acc[i][j], beta * *cp);
        }
      }
    }
  }
  __syncthreads();  // the next item rebuilds the lists
}

// The safety blocks of a reconstruct launch (the first blocks of the first class's grid, so that
// they run beside the reconstruct blocks).  Work items are numbered by concatenating the
// descriptors' items (safety_items), which every warp derives the same way, 32 descriptors at a
// time; a block takes the next unclaimed item from *ticket (zeroed before the launch), so the
// uneven items (K from 1 to many thousands) balance across the blocks.  hint: prep's count of
// non-finite rows / columns of this call (0: nothing to do), or nullptr.
__device__ __noinline__ void safety_blocks(const ggemm_recon_desc_t* __restrict__ descs, int num,
                                           const unsigned long long* hint,
                                           unsigned long long* ticket) {
  if (hint && *reinterpret_cast<const volatile unsigned long long*>(hint) == 0) return;
  __shared__ SafeSmem sm;
  __shared__ long long s_next;
  auto claim = [&]() -> long long {
    __syncthreads();
    if (threadIdx.x == 0) s_next = (long long)atomicAdd(ticket, 1ull);
    __syncthreads();
    return s_next;
  };
  const int lane = threadIdx.x & 31;
  long long base = 0, next = claim();
  for (int p0 = 0; p0 < num; p0 += 32) {
    const int p = p0 + lane;
    const long long cnt = p < num ? safety_items(descs[p]) : 0;
    long long incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += v;
    }
    const long long total = __shfl_sync(0xFFFFFFFFu, incl, 31);
    while (next < base + total) {
      // the owner is the first lane whose range ends after `next` (its count is > 0)
      const int owner = __popc(__ballot_sync(0xFFFFFFFFu, base + incl <= next));
      const long long start = base + __shfl_sync(0xFFFFFFFFu, incl - cnt, owner);
      safety_item(descs[p0 + owner], next - start, sm);
      next = claim();
    }
    base += total;
  }
}

// One launch per class of moduli counts over its problems (recon_class; prefix values are
// absolute, the grid starts at block block0); the layout is chosen per problem (block-uniform).
// Compiled per repair mode (GGEMM_STAGE_REPAIR_*), so the digit-layout body carries only its
// mode's certificate / repair branches, and per moduli count kN = 14, 15, 16 (kN = 0: any N), so
// that its CRT loops and constant-table offsets are resolved at compile time.
template <int kMode, int kN>
__global__ void __launch_bounds__(kReconThreads, 2)
    recon_kernel(const ggemm_recon_desc_t* __restrict__ descs,
                 const long long* __restrict__ prefix, int num, long long block0,
                 DevCounters* cnt, const ggemm_recon_desc_t* __restrict__ all_descs, int all_num,
                 int n_safety, const unsigned long long* hint) {
  if ((int)blockIdx.x < n_safety) {
    safety_blocks(all_descs, all_num, hint, &cnt->safety_ticket);
    return;
  }
  const long long bl = block0 + (long long)blockIdx.x - n_safety;
  const int owner = find_owner_warp(prefix, num, bl);
  const ggemm_recon_desc_t d = descs[owner];
  const long long local = bl - prefix[owner];
  unsigned n_unc = 0, n_rep = 0, n_saf = 0;
  if (d.layout == GGEMM_PRODUCTS_DIGITS) {
    if (kN > 0 && d.N != kN) return;  // not this instance's (the host never launches it so)
    recon_y8_block<kN>(d, local, kMode, n_unc, n_rep, n_saf);
  }
  else recon_c32_block(descs + owner, local, kMode, n_unc, n_rep, n_saf);
  flush_counters(n_unc, n_rep, n_saf, cnt);
}

// ============================================================ descriptor upload
// Copies the per-call descriptor blob from pinned, mapped host memory into device memory with the
// SMs instead of a copy engine.  A cudaMemcpyAsync of the blob queues on the copy engine behind
// whatever host -> device copies other streams have queued there: in a pipelined caller that copies
// the next step's inputs (tens of GB) while this step computes, the call's kernels would wait for
// that whole copy before they could start.  16-byte words, then the tail bytes.
__global__ void __launch_bounds__(256) blob_upload_kernel(uint4* __restrict__ dst,
                                                          const uint4* __restrict__ src,
                                                          long long n16, int tail) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride)
    dst[i] = src[i];
  if (blockIdx.x == 0 && threadIdx.x < tail)
    reinterpret_cast<uint8_t*>(dst + n16)[threadIdx.x] =
        reinterpret_cast<const uint8_t*>(src + n16)[threadIdx.x];
}

// ===================================================================================== host
namespace {
std::mutex g_dev_mu;
uint64_t g_uploaded = 0;  // bit per device ordinal (< 64)
int g_sms[64] = {0};
bool g_gemm_attr[64] = {false};
}  // namespace

// Host copy of the prep weight images g_prep_wts[qscale][N] (layout above).
static std::vector<uint8_t> make_prep_weight_images(const DevTables& dt) {
  std::vector<uint8_t> out(sizeof(g_prep_wts), 0);
  for (int qs = 0; qs < 2; ++qs)
    for (int N = 1; N <= kMaxModuli; ++N) {
      uint8_t* img = out.data() + ((size_t)qs * (kMaxModuli + 1) + N) * kPrepWBytes;
      const int n_cols = (4 * (N + 1) + 15) / 16 * 16, rg = n_cols / 8;
      for (int c = 0; c < 8 * n_cols; ++c) {
        const int half = c & 1, n = (c >> 1) % n_cols, e = (c >> 1) / n_cols;
        const int l = n >> 2, rr = n & 7;
        uint8_t* dst = img + (e * rg + (n >> 3)) * 256 + rr * 32 + ((half ^ (rr >> 2)) << 4);
        if ((n & 3) != e || l > N) continue;
        const int8_t* wl = qs ? dt.wbq[N][l] : dt.wb[l];
        for (int b = 0; b < 16; ++b) {
          const int dd = 16 * half + b;
          int v = 0;
          if (l == N) v = dd == 23 ? 1 : 0;
          else if (dd < 12) v = wl[dd];
          else if (dd < 23) v = wl[dd - 11];
          dst[b] = (uint8_t)(v & 255);
        }
      }
    }
  return out;
}

int upload_tables_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_uploaded & (1ull << dev)) return 0;
  int st = 0;
  const CrtTables& t = crt_tables(&st);
  if (st != 0) return 100 + st;
  static DevTables dt;
  make_dev_tables(t, &dt);
  if (cudaMemcpyToSymbol(c_tab, &dt, sizeof(dt)) != cudaSuccess) return 2;
  static std::vector<uint8_t> wts;
  if (wts.empty()) wts = make_prep_weight_images(dt);
  if (cudaMemcpyToSymbol(g_prep_wts, wts.data(), wts.size()) != cudaSuccess) return 2;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  g_sms[dev] = sms > 0 ? sms : 148;
  if (cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kGemmSmem) != cudaSuccess ||
      cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kGemm2Smem) != cudaSuccess)
    return 3;
  if (cudaFuncSetAttribute(prep_kernel<false, 14>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kPrepSmem) != cudaSuccess ||
      cudaFuncSetAttribute(prep_kernel<false, 15>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kPrepSmem) != cudaSuccess ||
      cudaFuncSetAttribute(prep_kernel<false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kPrepSmem) != cudaSuccess ||
      cudaFuncSetAttribute(prep_kernel<true, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kPrepSmem) != cudaSuccess ||
      cudaFuncSetAttribute(prep_kernel<true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kPrepSmem) != cudaSuccess)
    return 3;
  g_gemm_attr[dev] = true;
  if (cudaDeviceSynchronize() != cudaSuccess) return 4;
  g_uploaded |= 1ull << dev;
  return 0;
}

int current_device_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  return g_sms[dev] > 0 ? g_sms[dev] : 148;
}

int launch_blob_upload(void* d_dst, const void* src_dev, size_t bytes, cudaStream_t s) {
  if (bytes == 0) return 0;
  if ((((uintptr_t)d_dst | (uintptr_t)src_dev) & 15) != 0) return (int)cudaErrorInvalidValue;
  const long long n16 = (long long)(bytes / 16);
  const int tail = (int)(bytes % 16);
  const long long want = (n16 + 255) / 256;
  const unsigned grid = (unsigned)std::max(1LL, std::min(want, 4LL * current_device_sms()));
  blob_upload_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<uint4*>(d_dst),
                                          reinterpret_cast<const uint4*>(src_dev), n16, tail);
  return (int)cudaGetLastError();
}

int launch_prep(const ggemm_prep_desc_t* d_descs, const int* d_prefix, const PrepSplit& sp,
                DevCounters* cnt, cudaStream_t s, int* launches) {
  int n = 0;
  for (int c = 0; c < kPrepClasses; ++c) {
    const int f = sp.first[c], num = sp.first[c + 1] - f;
    const long long blocks = sp.block0[c + 1] - sp.block0[c];
    if (num <= 0 || blocks <= 0) continue;
    const ggemm_prep_desc_t* dd = d_descs + f;
    const int* pp = d_prefix + f;
    const int b0 = (int)sp.block0[c];
    const unsigned g = (unsigned)blocks;
    switch (c) {
      case 0: prep_kernel<false, 14><<<g, kPrepThreads, kPrepSmem, s>>>(dd, pp, num, b0, cnt); break;
      case 1: prep_kernel<false, 15><<<g, kPrepThreads, kPrepSmem, s>>>(dd, pp, num, b0, cnt); break;
      case 2: prep_kernel<false, 0><<<g, kPrepThreads, kPrepSmem, s>>>(dd, pp, num, b0, cnt); break;
      case 3: prep_kernel<true, 16><<<g, kPrepThreads, kPrepSmem, s>>>(dd, pp, num, b0, cnt); break;
      default: prep_kernel<true, 0><<<g, kPrepThreads, kPrepSmem, s>>>(dd, pp, num, b0, cnt); break;
    }
    ++n;
  }
  if (launches) *launches += n;
  return (int)cudaGetLastError();
}

int launch_gemm(const GemmJob* d_jobs, const long long* d_prefix, int num, long long total_tiles,
                DevCounters* cnt, cudaStream_t s, int walk_flags) {
  if (num <= 0 || total_tiles <= 0) return 0;
  const long long grid = std::min<long long>(total_tiles, (long long)current_device_sms());
  gemm_kernel<<<(unsigned)grid, kGemmThreads, kGemmSmem, s>>>(d_jobs, d_prefix, num, total_tiles,
                                                              cnt, walk_flags);
  return (int)cudaGetLastError();
}

int launch_gemm_pair(const GemmJob* d_jobs, const long long* d_prefix, int num,
                     long long total_tiles, DevCounters* cnt, cudaStream_t s, int walk_flags) {
  if (num <= 0 || total_tiles <= 0) return 0;
  const long long pairs = std::min<long long>(total_tiles, (long long)current_device_sms() / 2);
  gemm_pair_kernel<<<(unsigned)(2 * pairs), kGemmThreads, kGemm2Smem, s>>>(
      d_jobs, d_prefix, num, total_tiles, cnt, walk_flags);
  return (int)cudaGetLastError();
}

int launch_wait_probe(DevCounters* cnt, unsigned long long wait_ns, cudaStream_t s) {
  wait_ns = std::min<unsigned long long>(std::max<unsigned long long>(wait_ns, 1000ull),
                                         1000000000ull);
  wait_probe_kernel<<<1, 32, 0, s>>>(cnt, wait_ns);
  return (int)cudaGetLastError();
}

struct SafetyArgs {
  const ggemm_recon_desc_t* descs;
  int num, blocks;
  const unsigned long long* hint;
};

template <int kMode>
static void launch_recon_mode(int c, const ggemm_recon_desc_t* dd, const long long* pp, int num,
                              unsigned grid, long long b0, DevCounters* cnt, const SafetyArgs& sa,
                              cudaStream_t s) {
#define G2_RECON(n)                                                                         \
  recon_kernel<kMode, n><<<grid, kReconThreads, 0, s>>>(dd, pp, num, b0, cnt, sa.descs, sa.num, \
                                                        sa.blocks, sa.hint)
  switch (c) {
    case 0: G2_RECON(14); break;
    case 1: G2_RECON(15); break;
    case 2: G2_RECON(16); break;
    default: G2_RECON(0); break;
  }
#undef G2_RECON
}

int launch_recon(const ggemm_recon_desc_t* d_descs, const long long* d_prefix,
                 const ReconSplit& sp, int mode, DevCounters* cnt, cudaStream_t s,
                 int* launches, bool nonfinite_hint) {
  int n = 0;
  // the safety blocks ride in the first launch, ahead of its reconstruct blocks; their work
  // ticket starts from 0
  SafetyArgs sa{d_descs, sp.first[kReconClasses], 2 * current_device_sms(),
                nonfinite_hint ? &cnt->nonfinite : nullptr};
  if (sa.num > 0 &&
      cudaMemsetAsync(&cnt->safety_ticket, 0, sizeof(cnt->safety_ticket), s) != cudaSuccess)
    return (int)cudaGetLastError();
  for (int c = 0; c < kReconClasses; ++c) {
    const int f = sp.first[c], num = sp.first[c + 1] - f;
    const long long blocks = sp.block0[c + 1] - sp.block0[c];
    if (num <= 0 || blocks <= 0) continue;
    if (blocks + sa.blocks > 0x7FFFFFFFLL) return (int)cudaErrorInvalidConfiguration;
    const unsigned grid = (unsigned)(blocks + sa.blocks);
    if (mode == GGEMM_STAGE_REPAIR_OFF)
      launch_recon_mode<GGEMM_STAGE_REPAIR_OFF>(c, d_descs + f, d_prefix + f, num, grid,
                                                sp.block0[c], cnt, sa, s);
    else if (mode == GGEMM_STAGE_REPAIR_COUNT)
      launch_recon_mode<GGEMM_STAGE_REPAIR_COUNT>(c, d_descs + f, d_prefix + f, num, grid,
                                                  sp.block0[c], cnt, sa, s);
    else
      launch_recon_mode<GGEMM_STAGE_REPAIR_ON>(c, d_descs + f, d_prefix + f, num, grid,
                                               sp.block0[c], cnt, sa, s);
    sa.blocks = 0;
    ++n;
  }
  if (launches) *launches += n;
  return (int)cudaGetLastError();
}

}  // namespace g2
