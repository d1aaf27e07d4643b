// Parameter blocks shared by the host orchestration and the fp64-emu kernels.
// Everything a kernel needs about the modulus set travels by value in
// ModTables (under 3 KB of kernel-parameter space), so no call ever uploads
// tables or keeps per-device caches: every launch is capture-safe.
#pragma once

#include <cstdint>

namespace f64e {

constexpr int kMaxP = 20;   // largest modulus count (reference: fp64_emu.cu:27)
constexpr int kGroups = 5;  // packed Garner factor words, four int8 factors each

struct ModTables {
  int P;                       // number of moduli
  float log2M;                 // CRT range in bits, capped at 126 (float sum, as the reference)
  uint32_t p[kMaxP];           // moduli
  uint32_t mdiv[kMaxP];        // floor(2^32 / p): residue quotient estimate
  uint32_t off[kMaxP];         // largest multiple of p not above 2^31 (signed-residue bias)
  uint32_t mu2[kMaxP];         // 2 * floor(2^31 / p): limb-sum Barrett multiplier
  uint32_t c36[kMaxP];         // 2^36 mod p
  uint32_t c18[kMaxP];         // 2^18 mod p
  uint8_t pow2mod[kMaxP][38];  // 2^b mod p for b = 16..53 (undoing the 2^b extraction bias)
  int32_t mp[kMaxP][kGroups];  // balanced (M_u mod p_t), u < t, four per word
  int32_t minv[kMaxP];         // (M_t mod p_t)^-1
  int64_t m64[2];              // products of moduli 0..6 and 7..13

  // Fast forms (exact quotients, no correction steps).  Extraction: the
  // residue pre-sum of a biased integer u < 2^56 is two dp4a over its seven
  // bytes with the weights 2^(8i) mod p; its quotient by p is umulhi(v, mex)
  // exactly for v < 2^24.  The stored residue is ((v + 128) mod p) - 128.
  uint32_t kl[kMaxP];          // bytes 2^0, 2^8, 2^16, 2^24 mod p
  uint32_t kh[kMaxP];          // bytes 2^32, 2^40, 2^48 mod p (top byte 0)
  uint32_t mex[kMaxP];         // ceil(2^32 / p)
  // Reconstruction with digits stored offset, d' = d + h in [0, p): the
  // Garner sum uses unsigned factors cu = M_u mod p_t, and the offset terms
  // fold into one constant per digit, krec = ((sum_u h_u cu) * minv + h_t)
  // mod p_t plus a multiple of p_t >= 2^29 keeping the argument positive;
  // the quotient is (umulhi(X, mrec) >> 7) exactly for X < 2^31 (p > 128).
  uint32_t cu[kMaxP][kGroups]; // unsigned (M_u mod p_t), u < t, four per word
  uint32_t krec[kMaxP];
  uint32_t mrec[kMaxP];        // ceil(2^39 / p)
  int64_t hoff[3];             // Horner value of the offsets h per 7-modulus group
  uint64_t wgrp[kMaxP];        // radix weight of digit t inside its 7-modulus group
  int fast_recon;              // every modulus > 128

  // Direct CRT form (M = prod p_t < 2^121): V = S - q M with S = sum u_t E_t,
  // u_t the canonical residue, E_t = (M / p_t) * ((M / p_t)^-1 mod p_t) in
  // four 32-bit limbs, q = floor(S / M + crt_c) from a double estimate (exact
  // away from ties; ties take the digit-by-digit path).  crt_c = -L / M for
  // L, the low end of the balanced mixed-radix range of this modulus order.
  int crt_ok;
  uint32_t crtE[kMaxP][4];
  uint32_t crtM[4];
  double crtK96, crtK32, crtK0;  // 2^96 / M, 2^32 / M, 1 / M
  double crt_c;
  uint64_t crtL[2];            // L as a 128-bit two's complement (lo, hi)
};

// Byte range [lo, hi) a kernel may touch through one pointer.  Filled by the
// launchers in every build; only a library built with F64E_DEBUG_BOUNDS checks
// accesses against it (in_span, f64e_device.cuh).
struct Span {
  uintptr_t lo = 0, hi = 0;
};

// Device-resident scalars at the head of every workspace.  maxlg holds the
// operand maxima of the per-row / per-column log2 norms; in a partitioned
// multi-GPU run they are MAX-all-reduced between the sizing and compute
// phases, so every rank derives the same operand width.
struct WsHead {
  float maxlg[2];
  int32_t status;    // first bounded wait that timed out (0 = none)
  uint32_t counter;  // CTAs done in the current sizing launch (zeroed with status)
};

}  // namespace f64e
