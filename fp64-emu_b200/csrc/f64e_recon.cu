// Balanced-Garner reconstruction, quantization correction and rescale
// (reference: fp64_emu.cu:854-952).
//
// For each output element the P balanced residues r_t give mixed-radix digits
//   d_t = bal( (r_t - sum_{u<t} d_u * (M_u mod p_t)) * (M_t mod p_t)^-1 mod p_t )
// (M_u = p_0 ... p_{u-1}); the factors are int8 and packed four per word, so
// the inner products are dp4a, and only the words holding u < t are visited.
// The digits are unique, hence so is V = sum d_t M_t in [-M/2, M/2), which is
// recombined by grouped Horner (7 moduli per int64 group) and one 128-bit
// combine, plus the correction (Ahi.Bq + Aq.Bhi) * 2^(b-15); exact mode
// rounds the 128-bit value once to double, the fast mode combines in fp64 with
// the reference's fused multiply-adds.  The result is scaled by
// 2^-(sA_i + sB_j).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include <map>
#include <mutex>
#include <vector>

#include "f64e_crt64.cuh"
#include "f64e_device.cuh"
#include "f64e_kernels.h"

namespace f64e {

namespace {

// x * 2^e, exact: adds to the exponent field when the result stays normal,
// otherwise defers to ldexp (subnormal / overflow / zero), so the bits are
// ldexp's in every case.
__device__ __noinline__ double ldexp_slow(double x, int e) { return ldexp(x, e); }

__device__ __forceinline__ double scale2(double x, int e) {
  const uint64_t b = (uint64_t)__double_as_longlong(x);
  const int ex = (int)((b >> 52) & 0x7FF);
  const int ne = ex + e;
  if (ex != 0 && ex != 0x7FF && ne > 0 && ne < 0x7FF)
    return __longlong_as_double((long long)(b + ((uint64_t)(int64_t)e << 52)));
  return ldexp_slow(x, e);  // zero, subnormal or overflowing results: ldexp's rounding
}

// Signed 128-bit integer as two 64-bit halves.
struct I128 {
  uint64_t lo;
  int64_t hi;
};

__device__ __forceinline__ I128 i128_of(int64_t v) {
  I128 r;
  r.lo = (uint64_t)v;
  r.hi = v >> 63;
  return r;
}

// a * m + d for 0 < m < 2^63 (a group product of moduli), signed d.
__device__ __forceinline__ I128 i128_mul_add(I128 a, uint64_t m, int64_t d) {
  const uint64_t lo = a.lo * m;
  const uint64_t hi = __umul64hi(a.lo, m) + (uint64_t)a.hi * m;
  I128 r;
  r.lo = lo + (uint64_t)d;
  r.hi = (int64_t)(hi + (r.lo < lo ? 1ULL : 0ULL) + (d < 0 ? ~0ULL : 0ULL));
  return r;
}

// a * m + d for signed 64-bit a, 0 < m < 2^63, signed d: the unsigned
// product of a's bit pattern from four 32 x 32 -> 64 partial products, then
// -m * 2^64 when a < 0.
__device__ __forceinline__ I128 i128_mul_add_s64(int64_t a, uint64_t m, int64_t d) {
  const uint64_t au = (uint64_t)a;
  const uint32_t al = (uint32_t)au, ah = (uint32_t)(au >> 32), ml = (uint32_t)m, mh = (uint32_t)(m >> 32);
  const uint64_t p00 = (uint64_t)al * ml, p01 = (uint64_t)al * mh, p10 = (uint64_t)ah * ml, p11 = (uint64_t)ah * mh;
  const uint64_t mid = (p00 >> 32) + (uint32_t)p01 + (uint32_t)p10;
  const uint64_t lo = (mid << 32) | (uint32_t)p00;
  const uint64_t hi = p11 + (p01 >> 32) + (p10 >> 32) + (mid >> 32) - (a < 0 ? m : 0ULL);
  I128 r;
  r.lo = lo + (uint64_t)d;
  r.hi = (int64_t)(hi + (r.lo < lo ? 1ULL : 0ULL) + (uint64_t)(d >> 63));
  return r;
}

// a + c * 2^s for 0 < s < 64.
__device__ __forceinline__ I128 i128_add_shl(I128 a, int64_t c, int s) {
  const uint64_t clo = (uint64_t)c << s;
  const uint64_t chi = (uint64_t)(c >> (64 - s));
  I128 r;
  r.lo = a.lo + clo;
  r.hi = (int64_t)((uint64_t)a.hi + chi + (r.lo < clo ? 1ULL : 0ULL));
  return r;
}

// Correctly rounded (RNE) conversion: keep the top 64 significant bits, fold
// the dropped tail into a sticky bit far below the rounding position.
__device__ __forceinline__ double i128_to_double(I128 v) {
  const bool neg = v.hi < 0;
  uint64_t lo = v.lo, hi = (uint64_t)v.hi;
  if (neg) {
    lo = ~lo + 1ULL;
    hi = ~hi + (lo == 0ULL ? 1ULL : 0ULL);
  }
  double m;
  if (hi == 0) {
    m = __ull2double_rn(lo);
  } else {
    const int sh = 64 - __clzll((long long)hi);  // 1..64
    const uint64_t top = (sh == 64) ? hi : ((hi << (64 - sh)) | (lo >> sh));
    const uint64_t tail = (sh == 64) ? lo : (lo & ((1ULL << sh) - 1ULL));
    m = scale2(__ull2double_rn(top | (tail ? 1ULL : 0ULL)), sh);
  }
  return neg ? -m : m;
}

// RNE(v) * 2^e in one step: the top 64 significant bits with the dropped
// tail folded into a sticky bit convert with one rounding; the power of two
// of that conversion and e are applied together (exact for normal results,
// ldexp's rounding otherwise).
__device__ __forceinline__ double i128_to_double_scaled(I128 v, int e) {
  const uint64_t sg = (uint64_t)(v.hi >> 63);
  uint64_t lo = v.lo ^ sg, hi = (uint64_t)v.hi ^ sg;
  lo -= sg;                                  // two's complement magnitude: + 1 when negative
  hi += (sg & (lo == 0ULL ? 1ULL : 0ULL));
  uint64_t top = lo;
  int sh = 0;
  if (hi != 0) {
    const int lz = __clzll((long long)hi);  // 0..63
    sh = 64 - lz;
    top = lz ? ((hi << lz) | (lo >> sh)) : hi;
    top |= ((lz ? (lo << lz) : lo) != 0ULL) ? 1ULL : 0ULL;
  }
  const double m = __ull2double_rn(top);
  return scale2(sg ? -m : m, sh + e);
}

template <int CM>
__device__ __forceinline__ void load_corr(const ReconArgs& a, int64_t off, int64_t plane, int64_t (&cr)[4]) {
  if (CM == 0) {
#pragma unroll
    for (int e = 0; e < 4; e++) cr[e] = 0;
  } else if (CM == 1) {
    const int4 v = *reinterpret_cast<const int4*>(static_cast<const int32_t*>(a.corr) + off);
    cr[0] = v.x; cr[1] = v.y; cr[2] = v.z; cr[3] = v.w;
  } else if (CM == 2) {
    const int32_t* c = static_cast<const int32_t*>(a.corr);
    const int4 v = *reinterpret_cast<const int4*>(c + off);
    const int4 w = *reinterpret_cast<const int4*>(c + plane + off);
    cr[0] = (int64_t)v.x + w.x; cr[1] = (int64_t)v.y + w.y; cr[2] = (int64_t)v.z + w.z; cr[3] = (int64_t)v.w + w.w;
  } else {
    const int64_t* c = static_cast<const int64_t*>(a.corr) + off;
    const longlong2 v0 = *reinterpret_cast<const longlong2*>(c);
    const longlong2 v1 = *reinterpret_cast<const longlong2*>(c + 2);
    cr[0] = v0.x; cr[1] = v0.y; cr[2] = v1.x; cr[3] = v1.y;
  }
}

// Debug bounds build: the reads and the write of one four-column group (the
// first and the last residue plane bound the planes between them).  False,
// with the site recorded, when any lies outside its launcher's range; the
// caller then skips the group.  Always true in the release build.
template <int CM>
__device__ __forceinline__ bool recon_group_in_span(const ReconArgs& a, int64_t off, int64_t plane, int P,
                                                    int64_t i, int64_t j0) {
#ifdef F64E_DEBUG_BOUNDS
  bool ok = in_span(a.res + off, 4, a.res_span, a.status, kBoundsReconLoad) &&
            in_span(a.res + (int64_t)(P - 1) * plane + off, 4, a.res_span, a.status, kBoundsReconLoad);
  if (CM == 1) ok = ok && in_span(static_cast<const int32_t*>(a.corr) + off, 16, a.corr_span, a.status,
                                  kBoundsReconLoad);
  if (CM == 2) ok = ok && in_span(static_cast<const int32_t*>(a.corr) + off, 16, a.corr_span, a.status,
                                  kBoundsReconLoad) &&
                    in_span(static_cast<const int32_t*>(a.corr) + plane + off, 16, a.corr_span, a.status,
                            kBoundsReconLoad);
  if (CM == 3) ok = ok && in_span(static_cast<const int64_t*>(a.corr) + off, 32, a.corr_span, a.status,
                                  kBoundsReconLoad);
  const int64_t nc = a.N - j0 < 4 ? a.N - j0 : 4;
  return ok && in_span(a.C + i * a.ldc + j0, 8 * (size_t)nc, a.out_span, a.status, kBoundsReconStore);
#else
  (void)a; (void)off; (void)plane; (void)P; (void)i; (void)j0;
  return true;
#endif
}

}  // namespace

// General form (any moduli): balanced digits, reduction with one correction.
// Block (64, 4): x spans 64 four-column chunks of a row, y four rows.
template <int CM>
__global__ void __launch_bounds__(256) reconstruct_kernel(const ReconArgs a, const ModTables T) {
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int cshift = gn.bits_eff - 15;
  const int P = T.P;
  const int ng = (P + 6) / 7;
  const int64_t nq = (a.N + 3) >> 2;
  const int64_t plane = a.MF * a.ldn;
  const bool vec_out = ((a.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.C) & 15) == 0);
  for (int64_t i = (int64_t)blockIdx.y * 4 + threadIdx.y; i < a.MF; i += (int64_t)gridDim.y * 4) {
    const int sa = (int)a.sftA[i] + gn.g;
    const int16_t* __restrict__ sB = a.sftB + (i / a.M) * a.N;
    for (int64_t jq = (int64_t)blockIdx.x * 64 + threadIdx.x; jq < nq; jq += (int64_t)gridDim.x * 64) {
      const int64_t j0 = jq << 2;
      const int64_t off = i * a.ldn + j0;
      if (!recon_group_in_span<CM>(a, off, plane, P, i, j0)) continue;
      int32_t dp[4][kGroups];
#pragma unroll
      for (int e = 0; e < 4; e++)
#pragma unroll
        for (int g = 0; g < kGroups; g++) dp[e][g] = 0;
#pragma unroll
      for (int t = 0; t < kMaxP; t++) {
        if (t >= P) break;
        const uint32_t rw = *reinterpret_cast<const uint32_t*>(a.res + t * plane + off);
        const uint32_t p = T.p[t], md = T.mdiv[t];
        const int mi = T.minv[t];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int rt = (int)(int8_t)(uint8_t)(rw >> (8 * e));
          int acc = 0;
#pragma unroll
          for (int g = 0; g < (t + 3) / 4; g++) acc = __dp4a(dp[e][g], T.mp[t][g], acc);
          // |y| < 2^27; the bias p * 2^21 makes it non-negative and below 2^30.
          const int y = (rt - acc) * mi;
          const int d = balance(mod_small((uint32_t)(y + (int)(p << 21)), p, md), p);
          dp[e][t >> 2] |= (int32_t)((uint32_t)(uint8_t)(int8_t)d << (8 * (t & 3)));
        }
      }
      int64_t cr[4];
      load_corr<CM>(a, off, plane, cr);
      double outv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        int64_t a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
        for (int t = kMaxP - 1; t >= 0; t--) {
          if (t >= P) continue;
          const int64_t d = (int64_t)(int8_t)(uint8_t)((uint32_t)dp[e][t >> 2] >> (8 * (t & 3)));
          if (t >= 14) a2 = a2 * (int64_t)T.p[t] + d;
          else if (t >= 7) a1 = a1 * (int64_t)T.p[t] + d;
          else a0 = a0 * (int64_t)T.p[t] + d;
        }
        const int64_t j = j0 + e;
        const int sh = -sa - (j < a.N ? (int)sB[j] + gn.g : 0);
        if (a.exact) {
          I128 v = i128_of(ng == 3 ? a2 : (ng == 2 ? a1 : a0));
          if (ng == 3) v = i128_mul_add(v, (uint64_t)T.m64[1], a1);
          if (ng >= 2) v = i128_mul_add(v, (uint64_t)T.m64[0], a0);
          v = i128_add_shl(v, cr[e], cshift);
          outv[e] = scale2(i128_to_double(v), sh);
        } else {
          double v = (double)((ng == 3) ? a2 : ((ng == 2) ? a1 : a0));
          if (ng == 3) v = fma(v, (double)T.m64[1], (double)a1);
          if (ng >= 2) v = fma(v, (double)T.m64[0], (double)a0);
          v += ldexp((double)cr[e], cshift);
          outv[e] = ldexp(v, sh);
        }
      }
      double* crow = a.C + i * a.ldc;
      if (vec_out && j0 + 4 <= a.N) {
        *reinterpret_cast<double2*>(crow + j0) = make_double2(outv[0], outv[1]);
        *reinterpret_cast<double2*>(crow + j0 + 2) = make_double2(outv[2], outv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (j0 + e < a.N) crow[j0 + e] = outv[e];
      }
    }
  }
}

// byte_perm selector writing the low byte of the second operand into byte k.
__host__ __device__ constexpr uint32_t insert_sel(int k) {
  return (0x3210u & ~(0xFu << (4 * k))) | (4u << (4 * k));
}

// Fast form (every modulus > 128): digits kept offset, d' = d + h in [0, p),
// exact quotients, no correction steps (constants: ModTables fast forms).
// NP > 0 fixes the modulus count at compile time (the default plans' 14 and
// 15): no branch inside the digit loop; NP = 0 takes T.P.
template <int CM, bool EXACT, int NP>
__global__ void __launch_bounds__(256, 2) reconstruct_fast_kernel(const ReconArgs a, const ModTables T) {
  constexpr int PMAX = NP > 0 ? NP : kMaxP;
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int cshift = gn.bits_eff - 15;
  const int P = NP > 0 ? NP : T.P;
  const int ng = (P + 6) / 7;
  const int64_t nq = (a.N + 3) >> 2;
  const int64_t plane = a.MF * a.ldn;
  const bool vec_out = ((a.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.C) & 15) == 0);
  for (int64_t i = (int64_t)blockIdx.y * 4 + threadIdx.y; i < a.MF; i += (int64_t)gridDim.y * 4) {
    const int sa = (int)a.sftA[i] + gn.g;
    const int16_t* __restrict__ sB = a.sftB + (a.M == a.MF ? 0 : (i / a.M) * a.N);
    for (int64_t jq = (int64_t)blockIdx.x * 64 + threadIdx.x; jq < nq; jq += (int64_t)gridDim.x * 64) {
      const int64_t j0 = jq << 2;
      const int64_t off = i * a.ldn + j0;
      if (!recon_group_in_span<CM>(a, off, plane, P, i, j0)) continue;
      uint32_t rw[PMAX];
#pragma unroll
      for (int t = 0; t < PMAX; t++)
        rw[t] = (NP > 0 || t < P) ? __ldg(reinterpret_cast<const unsigned int*>(a.res + t * plane + off)) : 0u;
      int64_t cr[4];
      load_corr<CM>(a, off, plane, cr);
      uint32_t dp[4][kGroups];
      // Group values as digit-weighted sums, accumulated as the digits come:
      // the first four digits of a group (weights < 2^24) in 32 bits, the
      // rest in 64; unused digit positions hold 0 and add nothing.
      uint32_t glo[4][3];
      uint64_t ghi[4][3];
#pragma unroll
      for (int e = 0; e < 4; e++) {
#pragma unroll
        for (int g = 0; g < kGroups; g++) dp[e][g] = 0;
#pragma unroll
        for (int g = 0; g < 3; g++) {
          glo[e][g] = 0;
          ghi[e][g] = 0;
        }
      }
#pragma unroll
      for (int t = 0; t < PMAX; t++) {
        if (NP == 0 && t >= P) break;
        const uint32_t p = T.p[t], mr = T.mrec[t], kr = T.krec[t];
        const int mi = T.minv[t];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int rt = (int)(int8_t)(uint8_t)(rw[t] >> (8 * e));
          uint32_t acc = 0;
#pragma unroll
          for (int g = 0; g < (t + 3) / 4; g++) acc = __dp4a(dp[e][g], T.cu[t][g], acc);
          const uint32_t X = (uint32_t)((rt - (int)acc) * mi) + kr;   // in [0, 2^31)
          const uint32_t d = X - (__umulhi(X, mr) >> 7) * p;          // d + h in [0, p)
          dp[e][t >> 2] = __byte_perm(dp[e][t >> 2], d, insert_sel(t & 3));
          if (t % 7 < 4) glo[e][t / 7] += d * (uint32_t)T.wgrp[t];
          else ghi[e][t / 7] += (uint64_t)d * T.wgrp[t];
        }
      }
      double outv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int64_t a0 = (int64_t)(ghi[e][0] + glo[e][0]) - T.hoff[0];
        const int64_t a1 = (ng >= 2) ? (int64_t)(ghi[e][1] + glo[e][1]) - T.hoff[1] : 0;
        const int64_t a2 = (ng == 3) ? (int64_t)(ghi[e][2] + glo[e][2]) - T.hoff[2] : 0;
        const int64_t j = j0 + e;
        const int sh = -sa - (j < a.N ? (int)sB[j] + gn.g : 0);
        if (EXACT) {
          I128 v;
          if (ng == 3) {
            v = i128_mul_add_s64(a2, (uint64_t)T.m64[1], a1);
            v = i128_mul_add(v, (uint64_t)T.m64[0], a0);
          } else if (ng == 2) {
            v = i128_mul_add_s64(a1, (uint64_t)T.m64[0], a0);
          } else {
            v = i128_of(a0);
          }
          if (CM != 0) v = i128_add_shl(v, cr[e], cshift);
          outv[e] = i128_to_double_scaled(v, sh);
        } else {
          double v = (double)((ng == 3) ? a2 : ((ng == 2) ? a1 : a0));
          if (ng == 3) v = fma(v, (double)T.m64[1], (double)a1);
          if (ng >= 2) v = fma(v, (double)T.m64[0], (double)a0);
          v += ldexp((double)cr[e], cshift);
          outv[e] = ldexp(v, sh);
        }
      }
      double* crow = a.C + i * a.ldc;
      if (vec_out && j0 + 4 <= a.N) {
        *reinterpret_cast<double2*>(crow + j0) = make_double2(outv[0], outv[1]);
        *reinterpret_cast<double2*>(crow + j0 + 2) = make_double2(outv[2], outv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (j0 + e < a.N) crow[j0 + e] = outv[e];
      }
    }
  }
}


// Direct CRT form (exact mode, every modulus set with M < 2^121).  With u_t
// the canonical residue (the stored balanced residue plus p_t when negative),
// S = sum_t u_t E_t is the sum of four 32-bit limb products per modulus, and
// the balanced Garner value is the representative V = S - q M in [L, L + M)
// (L the low end of the balanced mixed-radix range, for every modulus
// order).  q = floor(S / M - L / M) comes from a double estimate whose error
// is below 2^-40; when the estimate lies within 2^-20 of an integer, V is
// moved into [L, L + M) by exact 128-bit comparisons.  The value is the
// Garner value bit for bit, so the rounding that follows is unchanged.
__device__ __noinline__ I128 crt_fix(I128 v, uint64_t Llo, uint64_t Lhi, uint64_t Mlo, uint64_t Mhi) {
  // w = v - L
  const uint64_t wlo = v.lo - Llo;
  const int64_t whi = (int64_t)((uint64_t)v.hi - Lhi - (v.lo < Llo ? 1ULL : 0ULL));
  if (whi < 0) {   // v < L: one M up
    const uint64_t lo = v.lo + Mlo;
    v.hi = (int64_t)((uint64_t)v.hi + Mhi + (lo < Mlo ? 1ULL : 0ULL));
    v.lo = lo;
  } else if ((uint64_t)whi > Mhi || ((uint64_t)whi == Mhi && wlo >= Mlo)) {   // v >= L + M: one M down
    const uint64_t lo = v.lo - Mlo;
    v.hi = (int64_t)((uint64_t)v.hi - Mhi - (v.lo < Mlo ? 1ULL : 0ULL));
    v.lo = lo;
  }
  return v;
}

template <int CM>
__global__ void __launch_bounds__(256, 4) reconstruct_crt_kernel(const ReconArgs a, const ModTables T) {
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int cshift = gn.bits_eff - 15;
  const int P = T.P;
  const int64_t nq = (a.N + 3) >> 2;
  const int64_t plane = a.MF * a.ldn;
  const bool vec_out = ((a.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.C) & 15) == 0);
  const uint64_t Mlo = ((uint64_t)T.crtM[1] << 32) | T.crtM[0], Mhi = ((uint64_t)T.crtM[3] << 32) | T.crtM[2];
  for (int64_t i = (int64_t)blockIdx.y * 4 + threadIdx.y; i < a.MF; i += (int64_t)gridDim.y * 4) {
    const int sa = (int)a.sftA[i] + gn.g;
    const int16_t* __restrict__ sB = a.sftB + (a.M == a.MF ? 0 : (i / a.M) * a.N);
    for (int64_t jq = (int64_t)blockIdx.x * 64 + threadIdx.x; jq < nq; jq += (int64_t)gridDim.x * 64) {
      const int64_t j0 = jq << 2;
      const int64_t off = i * a.ldn + j0;
      if (!recon_group_in_span<CM>(a, off, plane, P, i, j0)) continue;
      uint32_t rw[kMaxP];
#pragma unroll
      for (int t = 0; t < kMaxP; t++)
        rw[t] = (t < P) ? __ldg(reinterpret_cast<const unsigned int*>(a.res + t * plane + off)) : 0u;
      int64_t cr[4];
      load_corr<CM>(a, off, plane, cr);
      double outv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int t = 0; t < kMaxP; t++) {
          if (t >= P) break;
          const uint32_t p = T.p[t];
          const int r = (int)(int8_t)(uint8_t)(rw[t] >> (8 * e));
          const uint32_t u = (uint32_t)r + ((uint32_t)(r >> 31) & p);
#pragma unroll
          for (int l = 0; l < 4; l++) acc[l] += (uint64_t)u * T.crtE[t][l];
        }
        // S in five 32-bit limbs
        const uint32_t s0 = (uint32_t)acc[0];
        const uint64_t t1 = acc[1] + (acc[0] >> 32);
        const uint64_t t2 = acc[2] + (t1 >> 32);
        const uint64_t t3 = acc[3] + (t2 >> 32);
        const uint32_t s1 = (uint32_t)t1, s2 = (uint32_t)t2, s3 = (uint32_t)t3, s4 = (uint32_t)(t3 >> 32);
        const double x = __ull2double_rn(((uint64_t)s4 << 32) | s3) * T.crtK96 +
                         __ull2double_rn(((uint64_t)s2 << 32) | s1) * T.crtK32 + (double)s0 * T.crtK0 + T.crt_c;
        const double fq = floor(x);
        const uint32_t q = (uint32_t)fq;
        const double fr = x - fq;
        // V = S - q M modulo 2^128 (the true V lies in [L, L + M), |V| < 2^121)
        const uint64_t qm0 = (uint64_t)q * T.crtM[0];
        const uint64_t qm1 = (uint64_t)q * T.crtM[1] + (qm0 >> 32);
        const uint64_t qm2 = (uint64_t)q * T.crtM[2] + (qm1 >> 32);
        const uint64_t qm3 = (uint64_t)q * T.crtM[3] + (qm2 >> 32);
        const uint64_t Slo = ((uint64_t)s1 << 32) | s0, Shi = ((uint64_t)s3 << 32) | s2;
        const uint64_t QMlo = (qm1 << 32) | (uint32_t)qm0, QMhi = (qm3 << 32) | (uint32_t)qm2;
        I128 v;
        v.lo = Slo - QMlo;
        v.hi = (int64_t)(Shi - QMhi - (Slo < QMlo ? 1ULL : 0ULL));
        if (fr < 0x1p-20 || fr > 1.0 - 0x1p-20) v = crt_fix(v, T.crtL[0], T.crtL[1], Mlo, Mhi);
        const int64_t j = j0 + e;
        const int sh = -sa - (j < a.N ? (int)sB[j] + gn.g : 0);
        if (CM != 0) v = i128_add_shl(v, cr[e], cshift);
        outv[e] = i128_to_double_scaled(v, sh);
      }
      double* crow = a.C + i * a.ldc;
      if (vec_out && j0 + 4 <= a.N) {
        *reinterpret_cast<double2*>(crow + j0) = make_double2(outv[0], outv[1]);
        *reinterpret_cast<double2*>(crow + j0 + 2) = make_double2(outv[2], outv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (j0 + e < a.N) crow[j0 + e] = outv[e];
      }
    }
  }
}


// FP64-pipe CRT form (exact mode, M < 2^120; f64e_crt64.cuh): the limb sums
// sum_t u_t e_{t,l} as fused multiply-adds of exact doubles.  u_t enters
// without a conversion: one byte_perm places the byte, top bit flipped
// (u_t = r_t + 128), in the high word of a double whose exponent field is 0,
// i.e. the subnormal u_t * 2^-1042 (FP64 arithmetic keeps subnormals exact
// and at full rate); the table limbs are scaled by 2^978 (crt64_device_tables),
// so every product is u_t e_{t,l} 2^-64 exactly and the sums are the integer
// limb sums times 2^-64.  Block (64, 4): x spans 64 four-column chunks of a
// row, y four rows; each thread reads one 32-bit word (four columns) per
// residue plane.  NP > 0 fixes the modulus count at compile time (the default
// plans' 13, 14 and 15), so the modulus loop has no branches and its loads
// and multiply-adds interleave freely; NP = 0 takes T.P.
template <int CM, int MINB, int NP>
__global__ void __launch_bounds__(256, MINB) reconstruct_f64_kernel(const ReconArgs a, const Crt64Tables T) {
  constexpr int PMAX = NP > 0 ? NP : kMaxP;
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const double csc = crt64_pow2(gn.bits_eff - 15 - 40);
  const int P = NP > 0 ? NP : T.P;
  const int64_t nq = (a.N + 3) >> 2;
  const int64_t plane = a.MF * a.ldn;
  const bool vec_out = ((a.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.C) & 15) == 0);
  for (int64_t i = (int64_t)blockIdx.y * 4 + threadIdx.y; i < a.MF; i += (int64_t)gridDim.y * 4) {
    const int sa = (int)a.sftA[i] + gn.g;
    const int16_t* __restrict__ sB = a.sftB + (a.M == a.MF ? 0 : (i / a.M) * a.N);
    for (int64_t jq = (int64_t)blockIdx.x * 64 + threadIdx.x; jq < nq; jq += (int64_t)gridDim.x * 64) {
      const int64_t j0 = jq << 2;
      const int64_t off = i * a.ldn + j0;
      if (!recon_group_in_span<CM>(a, off, plane, P, i, j0)) continue;
      const int8_t* rp = a.res + off;
      uint32_t rw[PMAX];
#pragma unroll
      for (int t = 0; t < PMAX; t++)
        rw[t] = (NP > 0 || t < P) ? __ldg(reinterpret_cast<const unsigned int*>(rp + t * plane)) ^ 0x80808080u : 0u;
      int64_t cr[4];
      load_corr<CM>(a, off, plane, cr);
      double outv[4];
      uint32_t slow = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        double a0 = T.z[0], a1 = T.z[1], a2 = T.z[2];
#pragma unroll
        for (int t = 0; t < PMAX; t++) {
          if (NP == 0 && t >= P) break;
          const double du = __hiloint2double((int)__byte_perm(rw[t], 0u, 0x4440u | (uint32_t)e), 0);
          a0 = fma(du, T.e[t][0], a0);
          a1 = fma(du, T.e[t][1], a1);
          a2 = fma(du, T.e[t][2], a2);
        }
        const int64_t j = j0 + e;
        const int sh = -sa - (j < a.N ? (int)sB[j] + gn.g : 0);
        double r;
        if (!crt64_finish_fast(T, a0 * 0x1p64, a1 * 0x1p64, a2 * 0x1p64, (double)cr[e], csc, sh, &r))
          slow |= 1u << e;
        outv[e] = r;
      }
      double* crow = a.C + i * a.ldc;
      if (vec_out && j0 + 4 <= a.N) {
        *reinterpret_cast<double2*>(crow + j0) = make_double2(outv[0], outv[1]);
        *reinterpret_cast<double2*>(crow + j0 + 2) = make_double2(outv[2], outv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (j0 + e < a.N) crow[j0 + e] = outv[e];
      }
      if (slow) {
        // Rare: a quotient estimate near a tie, or a result that is zero,
        // subnormal or overflows.  Recompute those elements with the exact
        // tie check and ldexp's rounding, from the residues in memory, and
        // overwrite what the common path stored for them.
#pragma unroll 1
        for (int e = 0; e < 4; e++) {
          if (!((slow >> e) & 1) || j0 + e >= a.N) continue;
          double a0 = T.z[0], a1 = T.z[1], a2 = T.z[2];
#pragma unroll 1
          for (int t = 0; t < P; t++) {
            const double du = (double)((uint32_t)(uint8_t)rp[t * plane + e] ^ 0x80u) * 0x1p-1042;
            a0 = fma(du, T.e[t][0], a0);
            a1 = fma(du, T.e[t][1], a1);
            a2 = fma(du, T.e[t][2], a2);
          }
          const int sh = -sa - ((int)sB[j0 + e] + gn.g);
          const int64_t ce = e == 0 ? cr[0] : (e == 1 ? cr[1] : (e == 2 ? cr[2] : cr[3]));
          crow[j0 + e] = crt64_finish(T, a0 * 0x1p64, a1 * 0x1p64, a2 * 0x1p64, (double)ce, csc, sh);
        }
      }
    }
  }
}

// Tables of the FP64 CRT form for a modulus set, built once per set, in the
// device kernel's scaling: limbs e_{t,l} times 2^978 (u_t enters as the
// subnormal u_t 2^-1042, so each product is u_t e_{t,l} 2^-64) and the
// starting sums -z_l times 2^-64.
const Crt64Tables& crt64_device_tables(const ModTables& T) {
  static std::mutex mtx;
  static std::map<std::vector<int32_t>, Crt64Tables> cache;
  std::vector<int32_t> key(T.p, T.p + T.P);
  std::lock_guard<std::mutex> lk(mtx);
  auto it = cache.find(key);
  if (it == cache.end()) {
    Crt64Tables C;
    if (crt64_build(key.data(), T.P, T.log2M, &C)) crt64_device_scale(&C);
    it = cache.emplace(key, C).first;
  }
  return it->second;
}

void launch_reconstruct(const ReconArgs& a, const ModTables& T, cudaStream_t s, bool beside_gemm, int sms) {
  if (a.MF <= 0 || a.N <= 0) return;
  const int64_t nq = (a.N + 3) >> 2;
  dim3 grid((unsigned)std::min<int64_t>((nq + 63) / 64, 1 << 20), (unsigned)std::min<int64_t>((a.MF + 3) / 4, 65535));
  const dim3 block(64, 4);
  // F64E_RECON_FORM selects the exact-mode form for A/B checks (read per
  // call): "f64" (default where M < 2^120), "crt" (direct CRT on the integer
  // pipe), "garner" (digit by digit).  F64E_RECON_BESIDE chooses the form
  // beside a resident GEMM chunk: "garner" (default), "f64", or n = the FP64
  // form with its grid capped at n blocks per SM (the grid-stride loops cover
  // the rest).
  const char* fv = std::getenv("F64E_RECON_FORM");
  const char* gv = std::getenv("F64E_RECON_GARNER");
  const char* bv = std::getenv("F64E_RECON_BESIDE");
  bool want_garner = (gv && gv[0] == '1') || (fv && fv[0] == 'g');
  const bool want_crt = fv && fv[0] == 'c';
  // Beside a resident GEMM chunk the digit-by-digit form is the default:
  // there the FP64 form's blocks crowd out the extraction of the next chunk
  // (measured on row-chunked 8192^3 products: 157 against 154 TFLOP/s).
  if (beside_gemm && !(bv && (bv[0] == 'f' || (bv[0] >= '1' && bv[0] <= '9')))) want_garner = true;
  if (beside_gemm && bv && bv[0] >= '1' && bv[0] <= '9' && sms > 0) {
    const int64_t cap = (int64_t)std::atoi(bv) * sms;
    grid.y = (unsigned)std::max<int64_t>(1, std::min<int64_t>(grid.y, cap / std::max<unsigned>(grid.x, 1u)));
  }
  if (a.exact && !want_garner && !want_crt) {
    const Crt64Tables& C = crt64_device_tables(T);
    if (C.ok) {
      const int np = (T.P == 13 || T.P == 14 || T.P == 15) ? T.P : 0;
#define F64E_RF64_NP(CMV, MB, NPV) reconstruct_f64_kernel<CMV, MB, NPV><<<grid, block, 0, s>>>(a, C)
#define F64E_RF64_CM(CMV, MB)                  \
  do {                                         \
    if (np == 14) F64E_RF64_NP(CMV, MB, 14);      \
    else if (np == 15) F64E_RF64_NP(CMV, MB, 15); \
    else if (np == 13) F64E_RF64_NP(CMV, MB, 13); \
    else F64E_RF64_NP(CMV, MB, 0);             \
  } while (0)
      // three blocks per SM (80 registers); the int64 deep-K correction
      // layout, rare, takes the generic modulus count only
      switch (a.corr_mode) {
        case 0: F64E_RF64_CM(0, 3); break;
        case 1: F64E_RF64_CM(1, 3); break;
        case 2: F64E_RF64_CM(2, 3); break;
        default: F64E_RF64_NP(3, 3, 0); break;
      }
#undef F64E_RF64_CM
#undef F64E_RF64_NP
      return;
    }
  }
  // The direct CRT kernel is the faster one alone (64 registers, four blocks
  // per SM); beside a resident GEMM chunk the Garner kernel (112 registers: one
  // block beside the GEMM CTA) takes less from the GEMM, and the product is
  // faster with it there (measured on row-chunked 8192^3 products).
  if (a.exact && T.crt_ok && (want_crt || !beside_gemm) && !want_garner) {
    switch (a.corr_mode) {
      case 0: reconstruct_crt_kernel<0><<<grid, block, 0, s>>>(a, T); break;
      case 1: reconstruct_crt_kernel<1><<<grid, block, 0, s>>>(a, T); break;
      case 2: reconstruct_crt_kernel<2><<<grid, block, 0, s>>>(a, T); break;
      default: reconstruct_crt_kernel<3><<<grid, block, 0, s>>>(a, T); break;
    }
    return;
  }
  if (T.fast_recon) {
    // the default plans' common layouts (exact, one correction plane, 14 or
    // 15 moduli) with the modulus count fixed at compile time
    if (a.exact && a.corr_mode == 1 && T.P == 14) {
      reconstruct_fast_kernel<1, true, 14><<<grid, block, 0, s>>>(a, T);
      return;
    }
    if (a.exact && a.corr_mode == 1 && T.P == 15) {
      reconstruct_fast_kernel<1, true, 15><<<grid, block, 0, s>>>(a, T);
      return;
    }
    if (a.exact) {
      switch (a.corr_mode) {
        case 0: reconstruct_fast_kernel<0, true, 0><<<grid, block, 0, s>>>(a, T); break;
        case 1: reconstruct_fast_kernel<1, true, 0><<<grid, block, 0, s>>>(a, T); break;
        case 2: reconstruct_fast_kernel<2, true, 0><<<grid, block, 0, s>>>(a, T); break;
        default: reconstruct_fast_kernel<3, true, 0><<<grid, block, 0, s>>>(a, T); break;
      }
    } else {
      switch (a.corr_mode) {
        case 0: reconstruct_fast_kernel<0, false, 0><<<grid, block, 0, s>>>(a, T); break;
        case 1: reconstruct_fast_kernel<1, false, 0><<<grid, block, 0, s>>>(a, T); break;
        case 2: reconstruct_fast_kernel<2, false, 0><<<grid, block, 0, s>>>(a, T); break;
        default: reconstruct_fast_kernel<3, false, 0><<<grid, block, 0, s>>>(a, T); break;
      }
    }
    return;
  }
  switch (a.corr_mode) {
    case 0: reconstruct_kernel<0><<<grid, block, 0, s>>>(a, T); break;
    case 1: reconstruct_kernel<1><<<grid, block, 0, s>>>(a, T); break;
    case 2: reconstruct_kernel<2><<<grid, block, 0, s>>>(a, T); break;
    default: reconstruct_kernel<3><<<grid, block, 0, s>>>(a, T); break;
  }
}

}  // namespace f64e
