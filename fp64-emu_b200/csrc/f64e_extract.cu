// Residue extraction: fp64 operands -> K-major int8 planes that the modular
// GEMM reads through TMA.
//
// Per element (reference: fp64_emu.cu:249-397): the scaled integer
// T = RNE(|x| * 2^s) is taken from the raw IEEE bits with integer arithmetic
// only; the biased value T +- 2^b splits into three 18-bit limbs whose
// weighted sum is reduced once per modulus with a 32-bit Barrett step to a
// residue; the two correction digits are hi = clamp(RNE(T*2^(7-b))) and
// q = clamp(RNE(resid*2^8)).  The integer sequence (including its wrap on
// non-finite rows) is the reference's, so every plane holds, element by
// element, the reference's residue modulo its p (and the correction planes
// the reference's digits bit for bit).
//
// Differences from the reference: the residue byte of the common path is
// ((v + 128) mod p) - 128, in [-128, p - 129], instead of the symmetric
// balanced residue: the same value modulo p and within int8, one multiply
// cheaper to form.  The GEMM needs only |residue| <= 128 (so that K terms of
// at most 2^14 stay inside int32 for K < 2^17) and everything after it works
// modulo p, so the products are bit-identical.  Planes are K-major with a
// 16-byte row pitch (TMA-legal for any K, pad columns zero), and an operand
// given as [K, N] is transposed inside the extraction through shared memory
// instead of by a separate fp64 transpose copy (fp64_emu.cu:1233-1235).
#include "f64e_device.cuh"
#include "f64e_kernels.h"

namespace f64e {

namespace {

__device__ __forceinline__ uint64_t rne_shr(uint64_t mag, int s) {
  if (s <= 0) return (-s < 64) ? (mag << (-s)) : 0ULL;
  if (s > 63) return 0ULL;
  const uint64_t keep = mag >> s;
  const uint64_t rem = mag & ((1ULL << s) - 1ULL);
  const uint64_t half = 1ULL << (s - 1);
  return keep + ((rem > half || (rem == half && (keep & 1ULL))) ? 1ULL : 0ULL);
}

// Same value as rne_shr for v < 2^62: adding 2^(s-1) - 1 plus the kept
// low bit carries into the kept part exactly when the dropped part is above
// half, or equal to half with an odd kept part.
__device__ __forceinline__ uint64_t rne_shr_small(uint64_t v, int s) {
  if (s <= 0) return (-s < 64) ? (v << (-s)) : 0ULL;
  if (s > 63) return 0ULL;
  const uint64_t lsb = (v >> s) & 1ULL;
  return (v + ((1ULL << (s - 1)) - 1ULL) + lsb) >> s;
}

// Out-of-line copy for the rare wide operand (rows whose maximum is not
// finite), so the common path is not predicated through it.
__device__ __noinline__ uint64_t rne_shr_wide(uint64_t v, int s) { return rne_shr(v, s); }

__device__ __forceinline__ int clamp127(int64_t v) { return v > 127 ? 127 : (v < -127 ? -127 : (int)v); }

// Biased scaled integer u = T*sign + 2^b (two's complement, mod 2^64) and
// the two correction digits of one element.
struct Split {
  uint64_t u;
  int h, q;
};

__device__ __forceinline__ Split split_elem(double x, int s, int be, bool corr) {
  const uint64_t xb = (uint64_t)__double_as_longlong(x);
  const bool neg = (int64_t)xb < 0;
  const int e = (int)((xb >> 52) & 0x7FF);
  const uint64_t m = xb & 0xFFFFFFFFFFFFFULL;
  const uint64_t mag = e ? ((1ULL << 52) | m) : m;
  const int t = (e ? e : 1) - 1075 + s + 52;
  const uint64_t Tu = rne_shr_small(mag, 52 - t);  // mag < 2^53
  const uint64_t td = neg ? (0ULL - Tu) : Tu;  // two's complement of the signed value
  Split S;
  if (corr) {
    const uint64_t r8 = rne_shr_small(mag, 44 - t) - (Tu << 8);
    const uint64_t h8 = (Tu >> 62) ? rne_shr_wide(Tu, be - 7) : rne_shr_small(Tu, be - 7);
    S.h = clamp127((int64_t)(neg ? (0ULL - h8) : h8));
    S.q = clamp127((int64_t)(neg ? (0ULL - r8) : r8));
  } else {
    S.h = S.q = 0;
  }
  S.u = td + (1ULL << be);
  return S;
}

// Same split in FP64 for finite x with 2^s a normal double and
// y = |x| 2^s < 2^53 (every element of a row with a finite maximum): y is
// exact (products below 2^-1022 round, but such y give T = q = 0 either way);
// T = RNE(y) from the 2^52 magic add (ulp 1 on [2^52, 2^53), ties to even;
// y >= 2^52 is an integer already and adds 0); q = RNE(256 y) - 256 T =
// RNE(256 (y - T)) since 256 T is an even integer; hi = RNE(T 2^(7-b)).
// Both last roundings take the sign of x into their factor (RNE is odd-
// symmetric) and use the 1.5 * 2^52 magic, whose low word is the signed
// result.  bias = 2^b.  Returns false when the conditions fail.
__device__ __forceinline__ bool split_fast(double x, double p2s, double p2h, uint64_t bias, bool corr, Split& S) {
  const uint64_t xb = (uint64_t)__double_as_longlong(x);
  const double y = __longlong_as_double((long long)(xb & 0x7FFFFFFFFFFFFFFFULL)) * p2s;
  if (!(y < 9007199254740992.0)) return false;  // y >= 2^53, inf or NaN
  const bool big = y >= 4503599627370496.0;     // [2^52, 2^53): y is an integer
  const double c = big ? 0.0 : 4503599627370496.0;
  const double z = y + c;
  const uint64_t Tu = (uint64_t)__double_as_longlong(z) - (big ? 0x4320000000000000ULL : 0x4330000000000000ULL);
  // sign * Tu + 2^b in two's complement: (Tu ^ m) + 2^b + (m & 1), m = 0 or ~0
  const uint64_t m = (uint64_t)((int64_t)xb >> 63);
  S.u = (Tu ^ m) + bias + (m & 1ULL);
  if (corr) {
    const uint64_t sb = xb & 0x8000000000000000ULL;
    const double Td = z - c;
    const double s256 = __longlong_as_double((long long)(0x4070000000000000ULL | sb));   // +-256
    const double sp2h = __longlong_as_double((long long)((uint64_t)__double_as_longlong(p2h) | sb));
    const int r8 = (int)(uint32_t)__double_as_longlong(fma(y - Td, s256, 6755399441055744.0));
    const int h8 = (int)(uint32_t)__double_as_longlong(fma(Td, sp2h, 6755399441055744.0));
    S.h = max(min(h8, 127), -127);
    S.q = max(min(r8, 127), -127);
  } else {
    S.h = S.q = 0;
  }
  return true;
}

__device__ __noinline__ Split split_slow(double x, int s, int be, bool corr) { return split_elem(x, s, be, corr); }

// 2^e as a double for -1022 <= e <= 1023.
__device__ __forceinline__ double pow2d(int e) { return __longlong_as_double((long long)(e + 1023) << 52); }

// Reference form of one residue (fp64_emu.cu:278-287): three 18-bit limbs,
// 32-bit Barrett with one correction.  Exact whenever u < 2^56; kept for
// elements beyond that (rows whose maximum is not finite), where the
// reference's wrap-around arithmetic defines the bits.
__device__ __forceinline__ uint32_t residue_ref(uint64_t u, uint32_t p, uint32_t c36, uint32_t c18, uint32_t cb,
                                                uint32_t mu2) {
  const uint32_t a = (uint32_t)(u >> 36), b = (uint32_t)((u >> 18) & 0x3FFFFu), c = (uint32_t)(u & 0x3FFFFu);
  const uint32_t v = a * c36 + b * c18 + c + cb;
  const uint32_t q = __umulhi(v, mu2);
  uint32_t r = v - q * p;
  if (r >= p) r -= p;
  int rb = (int)r;
  if (rb > ((int)p - 1) / 2) rb -= (int)p;
  return (uint32_t)(uint8_t)(int8_t)rb;
}

// Fast form for u < 2^56: v = u + cb + 128 folded to under 2^20 by two dp4a
// over the seven bytes of u (cb undoes the 2^b bias modulo p); r = v mod p is
// v - umulhi(v, mex) p exactly (v < 2^24, p <= 256).  The caller stores
// r - 128 = r ^ 0x80 per byte: congruent to u - 2^b, in [-128, p - 129].
__device__ __forceinline__ uint32_t residue_fast(uint32_t lo, uint32_t hi, uint32_t kl, uint32_t kh, uint32_t cb128,
                                                 uint32_t mex, uint32_t p) {
  const uint32_t v = __dp4a(lo, kl, __dp4a(hi, kh, cb128));
  return v - __umulhi(v, mex) * p;
}

__device__ __forceinline__ uint32_t pack4(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}
__device__ __forceinline__ uint32_t pack4i(int b0, int b1, int b2, int b3) {
  return pack4((uint32_t)b0, (uint32_t)b1, (uint32_t)b2, (uint32_t)b3);
}

// Packed residue words (4 elements per word) of plane t, fast form.
template <int NE>
__device__ __forceinline__ void residue_words(const Split (&S)[NE], const ModTables& T, int t, int be,
                                              uint32_t (&w)[NE / 4]) {
  const uint32_t p = T.p[t];
  const uint32_t cb128 = p + 128u - (uint32_t)T.pow2mod[t][be - 16];
  const uint32_t kl = T.kl[t], kh = T.kh[t], mex = T.mex[t];
#pragma unroll
  for (int i = 0; i < NE / 4; i++) {
    uint32_t r[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const uint64_t u = S[4 * i + e].u;
      r[e] = residue_fast((uint32_t)u, (uint32_t)(u >> 32), kl, kh, cb128, mex, p);
    }
    w[i] = pack4(r[0], r[1], r[2], r[3]) ^ 0x80808080u;
  }
}

// Reference form for one 4-element word of plane t (rare: elements of rows
// whose maximum is not finite).  Out of line, so the fast path is not
// predicated through it.
__device__ __noinline__ uint32_t residue_word_ref(uint64_t u0, uint64_t u1, uint64_t u2, uint64_t u3, uint32_t p,
                                                  uint32_t c36, uint32_t c18, uint32_t cb, uint32_t mu2) {
  return pack4(residue_ref(u0, p, c36, c18, cb, mu2), residue_ref(u1, p, c36, c18, cb, mu2),
               residue_ref(u2, p, c36, c18, cb, mu2), residue_ref(u3, p, c36, c18, cb, mu2));
}

}  // namespace

__device__ __forceinline__ void store_corr(const Split (&S)[8], bool corr, const ExtractArgs& a, int8_t* dst) {
  if (corr) {
    *reinterpret_cast<uint2*>(dst + a.hi_plane * a.pstride) =
        make_uint2(pack4i(S[0].h, S[1].h, S[2].h, S[3].h), pack4i(S[4].h, S[5].h, S[6].h, S[7].h));
    *reinterpret_cast<uint2*>(dst + a.q_plane * a.pstride) =
        make_uint2(pack4i(S[0].q, S[1].q, S[2].q, S[3].q), pack4i(S[4].q, S[5].q, S[6].q, S[7].q));
  }
}

// Eight k-consecutive elements of one row of the operand (shift s; fast: the
// row's maximum is finite and 2^s a normal double, p2s = 2^s): split, and
// their 8 bytes written to every plane at dst + t * pstride.  CORR_FIRST
// stores the two correction planes before the residues, which frees their
// registers for the residue loop (64 registers in extract_cols: four blocks
// per SM).  The row kernel keeps them last: beside a resident GEMM chunk its
// measured products were faster that way.
// NP > 0 fixes the modulus count at compile time (the default plans' 14 and
// 15): the plane loop then has no branches and the planes' arithmetic and
// stores interleave; NP = 0 takes T.P.
template <bool CORR_FIRST, int NP>
__device__ __forceinline__ void extract8(const double (&x)[8], int s, bool fast, double p2s, double p2h, int be,
                                         bool corr, const ExtractArgs& a, const ModTables& T, int8_t* dst) {
  constexpr int PMAX = NP > 0 ? NP : kMaxP;
  const int P = NP > 0 ? NP : T.P;
  const int64_t pstride = a.pstride;
  // Debug bounds build: the group's first and last plane bound every store
  // (planes ascend with their index); on a miss no plane is written.
  if (!in_span(dst, 8, a.dst, a.status, kBoundsExtractStore) ||
      !in_span(dst + (int64_t)max(P - 1, corr ? max(a.hi_plane, a.q_plane) : 0) * pstride, 8, a.dst, a.status,
               kBoundsExtractStore))
    return;
  Split S[8];
  const uint64_t bias = 1ULL << be;
  uint32_t top = 0;
#pragma unroll
  for (int u = 0; u < 8; u++) {
    if (!(fast && split_fast(x[u], p2s, p2h, bias, corr, S[u]))) S[u] = split_slow(x[u], s, be, corr);
    top |= (uint32_t)(S[u].u >> 32);
  }
  if (CORR_FIRST) store_corr(S, corr, a, dst);
  // The reference form only for groups holding an element of a row with a
  // non-finite maximum (u >= 2^56).
  if ((top >> 24) == 0) {
#pragma unroll
    for (int t = 0; t < PMAX; t++) {
      if (NP == 0 && t >= P) break;
      uint32_t w[2];
      residue_words<8>(S, T, t, be, w);
      *reinterpret_cast<uint2*>(dst + t * pstride) = make_uint2(w[0], w[1]);
    }
  } else {
    for (int t = 0; t < P; t++) {
      const uint32_t p = T.p[t], cb = p - (uint32_t)T.pow2mod[t][be - 16];
      *reinterpret_cast<uint2*>(dst + t * pstride) =
          make_uint2(residue_word_ref(S[0].u, S[1].u, S[2].u, S[3].u, p, T.c36[t], T.c18[t], cb, T.mu2[t]),
                     residue_word_ref(S[4].u, S[5].u, S[6].u, S[7].u, p, T.c36[t], T.c18[t], cb, T.mu2[t]));
    }
  }
  if (!CORR_FIRST) store_corr(S, corr, a, dst);
}

// [rows, K] operand: thread (tx, ty) of a 256-thread block (32 x 8) handles
// 8 consecutive columns of one row; a warp covers 256 columns (2 KB read,
// 256 B written per plane, both contiguous).  (bx, by) of a (gdx, gdy) grid,
// with grid-stride loops over the K chunks and the rows.
template <bool VEC, int NP>
__device__ __forceinline__ void extract_rows_body(const ExtractArgs& a, const ModTables& T, int bx, int by, int gdx,
                                                  int gdy, int tx, int ty) {
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int be = gn.bits_eff;
  const bool corr = a.use_corr != 0;
  const int64_t nch = a.Kp >> 3;
  for (int64_t r = (int64_t)by * 8 + ty; r < a.rows; r += (int64_t)gdy * 8) {
    const int s = (int)a.sft[r] + gn.g;
    const bool row_fast = (s >= -960) && (s <= 960);
    const double p2s = pow2d(row_fast ? s : 0), p2h = pow2d(7 - be);
    const double* __restrict__ xr = a.X + r * a.ld + a.koff;
    for (int64_t ch = (int64_t)bx * 32 + tx; ch < nch; ch += (int64_t)gdx * 32) {
      const int64_t k0 = ch << 3;
      if (k0 < a.K && !in_span(xr + k0, 8 * (size_t)(a.K - k0 < 8 ? a.K - k0 : 8), a.src, a.status,
                               kBoundsExtractLoad))
        continue;
      double x[8];
      if (VEC && k0 + 8 <= a.K) {
        const double2* p2 = reinterpret_cast<const double2*>(xr + k0);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const double2 v = __ldg(p2 + u);
          x[2 * u] = v.x;
          x[2 * u + 1] = v.y;
        }
      } else {
#pragma unroll
        for (int u = 0; u < 8; u++) x[u] = (k0 + u < a.K) ? __ldg(xr + k0 + u) : 0.0;
      }
      extract8<false, NP>(x, s, row_fast, p2s, p2h, be, corr, a, T, a.planes + r * a.Kp + k0);
    }
  }
}

// PAIR: two [rows, K] operands in one launch, blockIdx.z selecting the
// arguments (small products, where launches dominate).  Three blocks per SM
// (79 registers, no spills): the kernel waits on its loads, and the third
// block hides more of that than the register cap costs (measured: 8192^2
// operands extract in 0.92-0.95 ms against 1.03-1.07 ms at two blocks).
template <bool VEC, bool PAIR, int NP>
__global__ void __launch_bounds__(256, 3) extract_rows_kernel(const ExtractPair ap, const ModTables T) {
  extract_rows_body<VEC, NP>(ap.a[PAIR ? blockIdx.z : 0], T, (int)blockIdx.x, (int)blockIdx.y, (int)gridDim.x,
                             (int)gridDim.y, (int)threadIdx.x, (int)threadIdx.y);
}

// [batch, K, N] operand: a block takes a 64 (k) x 32 (n) tile.  Warp w reads
// the rows k0 + w + 8 i (32 consecutive n, 256 B each) and parks the doubles
// transposed in shared memory, 66 per n (16.5 KB); thread (n, kg) then splits
// the eight k-consecutive elements kg of its n exactly as extract_rows does
// and writes 8 bytes per plane.  A warp takes 8 n x 4 k-groups: each plane
// store is 32 contiguous bytes in each of 8 plane rows, and each 8-lane phase
// of its 16-byte shared loads reads 8 different n, whose pitch of 33 16-byte
// chunks puts them in 8 different bank groups.
constexpr int kColTileK = 64, kColTileN = 32, kColPitch = 66;

// Tile (bx: n tiles, by: K tiles, bz: batch member) of a [batch, K, N]
// operand, by a 256-thread block with xs[kColTileN * kColPitch] of shared
// memory.  One barrier, reached by every thread of the block.
template <int NP>
__device__ __forceinline__ void extract_cols_body(const ExtractArgs& a, const ModTables& T, int bx, int by, int bz,
                                                  double* xs) {
  const int64_t b = bz;
  const int64_t n0 = (int64_t)bx * kColTileN, k0 = (int64_t)by * kColTileK;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  {
    const int64_t n = n0 + lane;
    const bool nin = n < a.N;
    const double* __restrict__ xb = a.X + b * a.K * a.ld + n;   // row pitch a.ld (>= a.N)
    double v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int64_t k = k0 + w + 8 * i;
      v[i] = (nin && k < a.K && in_span(xb + k * a.ld, 8, a.src, a.status, kBoundsExtractLoad)) ? __ldg(xb + k * a.ld)
                                                                                                 : 0.0;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) xs[lane * kColPitch + w + 8 * i] = v[i];
  }
  __syncthreads();
  const int nl = 8 * (w & 3) + (lane & 7), kg = 4 * (w >> 2) + (lane >> 3);
  const int64_t n = n0 + nl, kk = k0 + 8 * kg;
  if (n >= a.N || kk >= a.Kp) return;
  double x[8];
  const double2* src = reinterpret_cast<const double2*>(xs + nl * kColPitch + 8 * kg);
#pragma unroll
  for (int u = 0; u < 4; u++) {
    const double2 d = src[u];
    x[2 * u] = d.x;
    x[2 * u + 1] = d.y;
  }
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int be = gn.bits_eff;
  const int s = (int)a.sft[b * a.N + n] + gn.g;
  const bool fast = (s >= -960) && (s <= 960);
  extract8<true, NP>(x, s, fast, pow2d(fast ? s : 0), pow2d(7 - be), be, a.use_corr != 0, a, T,
                 a.planes + (b * a.N + n) * a.Kp + kk);
}

template <int NP>
__global__ void __launch_bounds__(256, 2) extract_cols_kernel(const ExtractArgs a, const ModTables T) {
  __shared__ __align__(16) double xs[kColTileN * kColPitch];
  extract_cols_body<NP>(a, T, (int)blockIdx.x, (int)blockIdx.y, (int)blockIdx.z, xs);
}

// A [rows, K] operand and a [batch, K, N] operand in one launch (small nt
// products, where launches dominate): blocks [0, na) take the first as a
// (gxa, na / gxa) grid, the rest the second's (gxb, gyb, batch) tiles.
template <bool VEC>
__global__ void __launch_bounds__(256, 2) extract_nt_pair_kernel(const ExtractArgs ra, const ExtractArgs cb,
                                                                 const ModTables T, int gxa, int na, int gxb,
                                                                 int gyb) {
  __shared__ __align__(16) double xs[kColTileN * kColPitch];
  const int i = (int)blockIdx.x;
  if (i < na) {
    extract_rows_body<VEC, 0>(ra, T, i % gxa, i / gxa, gxa, na / gxa, (int)(threadIdx.x & 31),
                              (int)(threadIdx.x >> 5));
  } else {
    const int j = i - na, per = gxb * gyb;
    const int bz = j / per, r = j - bz * per;
    extract_cols_body<0>(cb, T, r % gxb, r / gxb, bz, xs);
  }
}

namespace {
bool rows_vec(const ExtractArgs& a) {
  return (a.ld % 2 == 0) && (a.koff % 2 == 0) && ((reinterpret_cast<uintptr_t>(a.X) & 15) == 0);
}
}  // namespace

void launch_extract_rows(const ExtractArgs& a, const ModTables& T, cudaStream_t s) {
  if (a.rows <= 0 || a.Kp <= 0) return;
  const int64_t nch = a.Kp >> 3;
  const unsigned gx = (unsigned)std::min<int64_t>((nch + 31) / 32, 1 << 20);
  const unsigned gy = (unsigned)std::min<int64_t>((a.rows + 7) / 8, 65535);
  ExtractPair ap;
  ap.a[0] = a;
  ap.a[1] = a;
  const dim3 grid(gx, gy), block(32, 8);
  if (rows_vec(a)) {
    if (T.P == 14) extract_rows_kernel<true, false, 14><<<grid, block, 0, s>>>(ap, T);
    else if (T.P == 15) extract_rows_kernel<true, false, 15><<<grid, block, 0, s>>>(ap, T);
    else extract_rows_kernel<true, false, 0><<<grid, block, 0, s>>>(ap, T);
  } else {
    extract_rows_kernel<false, false, 0><<<grid, block, 0, s>>>(ap, T);
  }
}

void launch_extract_rows_pair(const ExtractArgs& a0, const ExtractArgs& a1, const ModTables& T, cudaStream_t s) {
  if (a0.rows <= 0 || a1.rows <= 0 || a0.Kp <= 0) {
    launch_extract_rows(a0, T, s);
    launch_extract_rows(a1, T, s);
    return;
  }
  const int64_t nch = a0.Kp >> 3;
  const unsigned gx = (unsigned)std::min<int64_t>((nch + 31) / 32, 1 << 20);
  const unsigned gy = (unsigned)std::min<int64_t>((std::max(a0.rows, a1.rows) + 7) / 8, 65535);
  ExtractPair ap;
  ap.a[0] = a0;
  ap.a[1] = a1;
  if (rows_vec(a0) && rows_vec(a1)) extract_rows_kernel<true, true, 0><<<dim3(gx, gy, 2), dim3(32, 8), 0, s>>>(ap, T);
  else extract_rows_kernel<false, true, 0><<<dim3(gx, gy, 2), dim3(32, 8), 0, s>>>(ap, T);
}

void launch_extract_nt_pair(const ExtractArgs& ra, const ExtractArgs& cb, const ModTables& T, cudaStream_t s) {
  if (ra.rows <= 0 || ra.Kp <= 0 || cb.N <= 0 || cb.batch <= 0) {
    launch_extract_rows(ra, T, s);
    launch_extract_cols(cb, T, s);
    return;
  }
  const int64_t nch = ra.Kp >> 3;
  const int64_t gxa = std::min<int64_t>((nch + 31) / 32, 1 << 20);
  const int64_t gya = std::min<int64_t>((ra.rows + 7) / 8, 65535);
  const int64_t gxb = (cb.N + kColTileN - 1) / kColTileN, gyb = (cb.Kp + kColTileK - 1) / kColTileK;
  const int64_t na = gxa * gya, nb = gxb * gyb * cb.batch;
  if (na + nb > INT32_MAX) {
    launch_extract_rows(ra, T, s);
    launch_extract_cols(cb, T, s);
    return;
  }
  const unsigned grid = (unsigned)(na + nb);
  if (rows_vec(ra))
    extract_nt_pair_kernel<true><<<grid, 256, 0, s>>>(ra, cb, T, (int)gxa, (int)na, (int)gxb, (int)gyb);
  else
    extract_nt_pair_kernel<false><<<grid, 256, 0, s>>>(ra, cb, T, (int)gxa, (int)na, (int)gxb, (int)gyb);
}

void launch_extract_cols(const ExtractArgs& a, const ModTables& T, cudaStream_t s) {
  if (a.N <= 0 || a.Kp <= 0 || a.batch <= 0) return;
  const dim3 grid((unsigned)((a.N + kColTileN - 1) / kColTileN), (unsigned)((a.Kp + kColTileK - 1) / kColTileK),
                  (unsigned)a.batch);
  if (T.P == 14) extract_cols_kernel<14><<<grid, 256, 0, s>>>(a, T);
  else if (T.P == 15) extract_cols_kernel<15><<<grid, 256, 0, s>>>(a, T);
  else extract_cols_kernel<0><<<grid, 256, 0, s>>>(a, T);
}

}  // namespace f64e
