// Exact CRT reconstruction on the FP64 pipe (host and device).
//
// The GEMM leaves, per output element, P balanced residues r_t in [-128, 127]
// (r_t = x mod p_t, x the exact integer dot product) and a correction c.  The
// reference recombines them by balanced Garner digits and 128-bit integer
// arithmetic (fp64_emu.cu:854-952): V, the unique representative of x modulo
// M = prod p_t in the balanced mixed-radix range [L, L + M), then
// RN(V + c * 2^cshift) as a double, then the row and column scaling.
//
// This form computes the same V with exact double-precision arithmetic, so
// the work runs on the FP64 pipe instead of the integer multiply pipe:
//
//   u_t = r_t + 128 in [0, 255] (the stored byte with its top bit flipped);
//   S   = sum_t u_t E_t,  E_t = (M / p_t) * ((M / p_t)^-1 mod p_t) < M;
//   S   = Z + V + q M  with Z = 128 * sum_t E_t mod M (a constant).
//
// E_t is split into three 40-bit limbs, so with M < 2^120 every limb sum
// a_l = -z_l + sum_t u_t e_{t,l} is an integer below 2^53 in magnitude and
// every partial sum is exact in double (P <= 32).  q = floor((S - Z - L) / M)
// comes from a double estimate with error below 2^-38; when the estimate lies
// within 2^-20 of an integer the candidate is checked exactly against
// [L, L + M).  V's limbs v_l = a_l - q m_l are exact (one fused multiply-add
// each, |v_l| < 2^53), the correction is added as two exact limbs, a carry
// pass leaves v_0, v_1 in [0, 2^40), and RN(V + c 2^cshift) is one fused
// multiply-add (exact partial sums make its single rounding the correct one;
// from 2^93 on the low limb only decides a sticky half).  The result equals the
// Garner form bit for bit.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

#ifdef __CUDACC__
#define F64E_HD __host__ __device__ __forceinline__
#define F64E_HD_NOINLINE __host__ __device__ __noinline__
#else
#define F64E_HD inline
#define F64E_HD_NOINLINE inline
#endif

namespace f64e {

constexpr int kCrt64MaxP = 20;

struct Crt64Tables {
  int P;
  int ok;                       // M < 2^120: this form applies
  float log2M;                  // as ModTables::log2M (the width rule's input)
  double e[kCrt64MaxP][3];      // 40-bit limbs of E_t, each times 2^-32 (u_t enters as u_t * 2^32)
  double z[3];                  // -(40-bit limbs of Z): the limb sums' starting values
  double m[3];                  // 40-bit limbs of M
  double lam[3];                // L = lam0 + lam1 2^40 + lam2 2^80, lam0, lam1 in [0, 2^40)
  double k[3];                  // 2^(40 l) / M
  double cl;                    // -L / M
  // Constants of the common path, kept in the parameter block so the
  // instructions read them from the constant bank instead of registers.
  double clh;                   // -L / M - 1/2
  double two40, twom40, half, thr13, tie;   // 2^40, 2^-40, 1/2, 2^13, 1/2 - 2^-20
};

F64E_HD uint64_t crt64_bits(double x) {
#ifdef __CUDA_ARCH__
  return (uint64_t)__double_as_longlong(x);
#else
  uint64_t b;
  std::memcpy(&b, &x, 8);
  return b;
#endif
}

F64E_HD double crt64_from_bits(uint64_t b) {
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)b);
#else
  double x;
  std::memcpy(&x, &b, 8);
  return x;
#endif
}

F64E_HD_NOINLINE double crt64_ldexp(double x, int e) {
#ifdef __CUDA_ARCH__
  return ldexp(x, e);
#else
  return std::ldexp(x, e);
#endif
}

// x * 2^e exactly as ldexp: an exponent add while the result stays normal.
F64E_HD double crt64_scale2(double x, int e) {
  const uint64_t b = crt64_bits(x);
  const int ex = (int)((b >> 52) & 0x7FF);
  const int ne = ex + e;
  if (ex != 0 && ex != 0x7FF && ne > 0 && ne < 0x7FF) return crt64_from_bits(b + ((uint64_t)(int64_t)e << 52));
  return crt64_ldexp(x, e);
}

// 2^e for -1022 <= e <= 1023.
F64E_HD double crt64_pow2(int e) { return crt64_from_bits((uint64_t)(1023 + e) << 52); }

// Sign of w0 + w1 2^40 + w2 2^80 for integers |w_l| < 2^53 - 2^14: carries
// move the low limbs into [0, 2^40), then the top limb carries the sign.
F64E_HD bool crt64_negative(double w0, double w1, double w2) {
  double c = floor(w0 * 0x1p-40);
  w1 += c;
  c = floor(w1 * 0x1p-40);
  w2 += c;
  return w2 < 0.0;
}

// The quotient estimate q lies within one of the true one; return the q
// whose remainder S - Z - q M lies in [L, L + M).  (Limbs of M and L by
// value: a rarely taken out-of-line call that copies no tables.)
F64E_HD double crt64_fix_q(double a0, double a1, double a2, double q, double m0, double m1, double m2,
                                    double l0, double l1, double l2) {
  const double v0 = fma(-q, m0, a0), v1 = fma(-q, m1, a1), v2 = fma(-q, m2, a2);
  const double w0 = v0 - l0, w1 = v1 - l1, w2 = v2 - l2;
  if (crt64_negative(w0, w1, w2)) return q - 1.0;
  if (!crt64_negative(w0 - m0, w1 - m1, w2 - m2)) return q + 1.0;
  return q;
}

// The common case of crt64_finish: false when the quotient estimate lies
// within 2^-20 of an integer or the scaled result would not be a normal
// double (zero, subnormal, overflow); crt64_finish handles those.  The
// estimate is shifted down by 1/2 so that q is its nearest integer and the
// distance to the tie is one subtraction.
F64E_HD bool crt64_finish_fast(const Crt64Tables& T, double a0, double a1, double a2, double c, double csc, int sh,
                               double* out) {
  const double h = fma(a2, T.k[2], fma(a1, T.k[1], fma(a0, T.k[0], T.clh)));   // (S - Z - L) / M - 1/2
  const double q = rint(h);
  const bool near_tie = fabs(h - q) > T.tie;
  double v0 = fma(-q, T.m[0], a0), v1 = fma(-q, T.m[1], a1), v2 = fma(-q, T.m[2], a2);
  // c 2^cshift = ch 2^40 + cl with cl in [0, 2^40)
  const double y = c * csc;
  const double ch = floor(y);
  v0 = fma(y - ch, T.two40, v0);
  v1 += ch;
  // carries: v0, v1 into [0, 2^40)
  const double c0 = floor(v0 * T.twom40);
  v0 = fma(-c0, T.two40, v0);
  v1 += c0;
  const double c1 = floor(v1 * T.twom40);
  v1 = fma(-c1, T.two40, v1);
  v2 += c1;
  // rounding (see crt64_finish)
  const bool big = fabs(v2 + T.half) >= T.thr13;
  const double r = big ? fma(v2, T.two40, v1 + fmin(v0, T.half)) : fma(fma(v2, T.two40, v1), T.two40, v0);
  const int e = big ? sh + 40 : sh;
  const uint64_t b = crt64_bits(r);
  const int ex = (int)((b >> 52) & 0x7FF);
  *out = crt64_from_bits(b + ((uint64_t)(int64_t)e << 52));
  return !near_tie && ex != 0 && (unsigned)(ex + e - 1) < 0x7FEu;
}

// From the limb sums a_l (with -Z folded in), the correction c (an integer,
// |c| < 2^53) scaled by csc = 2^(cshift - 40), and the output exponent sh:
// ldexp(RN(V + c 2^cshift), sh).
F64E_HD double crt64_finish(const Crt64Tables& T, double a0, double a1, double a2, double c, double csc, int sh) {
  const double est = fma(a2, T.k[2], fma(a1, T.k[1], fma(a0, T.k[0], T.cl)));
  double q = floor(est);
  const double fr = est - q;
  if (fr < 0x1p-20 || fr > 1.0 - 0x1p-20)
    q = crt64_fix_q(a0, a1, a2, q, T.m[0], T.m[1], T.m[2], T.lam[0], T.lam[1], T.lam[2]);
  double v0 = fma(-q, T.m[0], a0), v1 = fma(-q, T.m[1], a1), v2 = fma(-q, T.m[2], a2);
  // c 2^cshift = ch 2^40 + cl with cl in [0, 2^40)
  const double y = c * csc;
  const double ch = floor(y);
  v0 += (y - ch) * 0x1p40;
  v1 += ch;
  // carries: v0, v1 into [0, 2^40)
  const double c0 = floor(v0 * 0x1p-40);
  v0 = fma(-c0, 0x1p40, v0);
  v1 += c0;
  const double c1 = floor(v1 * 0x1p-40);
  v1 = fma(-c1, 0x1p40, v1);
  v2 += c1;
  // X = T 2^40 + v0 with T = v2 2^40 + v1.  For -2^53 <= T < 2^53 (v2 in
  // [-2^13, 2^13)) T is exact and one fused multiply-add rounds X.  Otherwise
  // every double in [T, T + 1] is at least 2^53 in magnitude, so neither a
  // double nor a rounding tie lies strictly between T and T + 1: v0 < 2^40
  // only decides whether X / 2^40 sits at T or strictly inside, which T + 1/2
  // stands for, and X / 2^40 rounds in one fused multiply-add.
  const bool big = v2 >= 0x1p13 || v2 < -0x1p13;
  const double t = fma(v2, 0x1p40, v1);
  const double small_r = fma(t, 0x1p40, v0);
  const double big_r = fma(v2, 0x1p40, v1 + fmin(v0, 0.5));
  return crt64_scale2(big ? big_r : small_r, big ? sh + 40 : sh);
}

// Host: the device kernel's scaling of built tables.  The kernel feeds u_t
// as the subnormal u_t 2^-1042 (its byte in the high word of a double with a
// zero exponent field: no conversion, no subtraction), so the limbs are
// scaled by 2^978 (below 2^1018) and each product is u_t e_{t,l} 2^-64; the
// starting sums take the same 2^-64, and the kernel multiplies the sums by
// 2^64 (exact) before crt64_finish.
inline void crt64_device_scale(Crt64Tables* T) {
  for (int t = 0; t < T->P; t++)
    for (int l = 0; l < 3; l++) T->e[t][l] = std::ldexp(T->e[t][l], 32 + 978);
  for (int l = 0; l < 3; l++) T->z[l] = std::ldexp(T->z[l], -64);
}

// Host: the tables of a modulus list; false (ok = 0) when M >= 2^120 or the
// moduli are not pairwise coprime.
inline bool crt64_build(const int32_t* primes, int P, float log2M, Crt64Tables* T) {
  using u128 = unsigned __int128;
  std::memset(T, 0, sizeof(*T));
  T->P = P;
  T->log2M = log2M;
  if (P < 1 || P > kCrt64MaxP) return false;
  u128 M = 1;
  for (int t = 0; t < P; t++) {
    if (primes[t] < 2 || M > ((u128)1 << 120) / (u128)primes[t]) return false;
    M *= (u128)primes[t];
  }
  if (M >= ((u128)1 << 120)) return false;
  const u128 mask = ((u128)1 << 40) - 1;
  auto limb = [&](u128 v, int l) { return (double)(uint64_t)((v >> (40 * l)) & mask); };
  u128 Z = 0;
  for (int t = 0; t < P; t++) {
    const u128 Mt = M / (u128)primes[t];
    const int64_t pt = primes[t];
    const int64_t mt = (int64_t)(Mt % (u128)pt);
    int64_t y = 0;
    for (int64_t x = 1; x < pt; x++)
      if (mt * x % pt == 1) {
        y = x;
        break;
      }
    if (y == 0 && pt > 1) return false;
    const u128 E = Mt * (u128)y;  // < M
    for (int l = 0; l < 3; l++) T->e[t][l] = std::ldexp(limb(E, l), -32);
    Z = (Z + (E % M) * 128) % M;
  }
  for (int l = 0; l < 3; l++) {
    T->z[l] = -limb(Z, l);
    T->m[l] = limb(M, l);
    T->k[l] = (double)(std::ldexp(1.0L, 40 * l) / (long double)M);
  }
  // L = -sum_t floor(p_t / 2) (p_0 ... p_{t-1}): the low end of the balanced
  // mixed-radix digit range; -L < M.
  u128 run = 1, negL = 0;
  for (int t = 0; t < P; t++) {
    negL += (u128)(primes[t] / 2) * run;
    run *= (u128)primes[t];
  }
  // L = -negL = lam0 + lam1 2^40 + lam2 2^80 with lam0, lam1 in [0, 2^40)
  const u128 Lp = ((u128)1 << 120) - negL;   // L + 2^120, in [0, 2^120)
  T->lam[0] = limb(Lp, 0);
  T->lam[1] = limb(Lp, 1);
  T->lam[2] = limb(Lp, 2) - 1099511627776.0;  // - 2^40
  T->cl = (double)((long double)negL / (long double)M);
  T->clh = T->cl - 0.5;
  T->two40 = 0x1p40;
  T->twom40 = 0x1p-40;
  T->half = 0.5;
  T->thr13 = 0x1p13;
  T->tie = 0.5 - 0x1p-20;
  T->ok = 1;
  return true;
}

}  // namespace f64e
