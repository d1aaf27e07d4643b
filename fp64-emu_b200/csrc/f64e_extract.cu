// Residue extraction: fp64 operands -> K-major int8 planes that the modular
// GEMM reads through TMA.
//
// Per element (reference: fp64_emu.cu:249-397): the scaled integer
// T = RNE(|x| * 2^s) is taken from the raw IEEE bits with integer arithmetic
// only; the biased value T +- 2^b splits into three 18-bit limbs whose
// weighted sum is reduced once per modulus with a 32-bit Barrett step to a
// balanced residue; the two correction digits are hi = clamp(RNE(T*2^(7-b)))
// and q = clamp(RNE(resid*2^8)).  The integer sequence (including its wrap on
// non-finite rows) is the reference's, so the planes are bit-identical for
// every input.
//
// Layout differences from the reference: planes are K-major with a 16-byte
// row pitch (TMA-legal for any K, pad columns zero), and an operand given as
// [K, N] is transposed inside the extraction through shared memory instead of
// by a separate fp64 transpose copy (fp64_emu.cu:1233-1235).
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

__device__ __forceinline__ int clamp127(int64_t v) { return v > 127 ? 127 : (v < -127 ? -127 : (int)v); }

// Limbs of the biased scaled integer and the two correction digits of x.
struct Limbs {
  uint32_t a, b, c;
  int h, q;
};

__device__ __forceinline__ Limbs split_elem(double x, int s, int be, bool corr) {
  const uint64_t xb = (uint64_t)__double_as_longlong(x);
  const bool neg = (int64_t)xb < 0;
  const int e = (int)((xb >> 52) & 0x7FF);
  const uint64_t m = xb & 0xFFFFFFFFFFFFFULL;
  const uint64_t mag = e ? ((1ULL << 52) | m) : m;
  const int t = (e ? e : 1) - 1075 + s + 52;
  const uint64_t Tu = rne_shr(mag, 52 - t);
  const uint64_t td = neg ? (0ULL - Tu) : Tu;  // two's complement of the signed value
  Limbs L;
  if (corr) {
    const uint64_t r8 = rne_shr(mag, 44 - t) - (Tu << 8);
    const uint64_t h8 = rne_shr(Tu, be - 7);
    L.h = clamp127((int64_t)(neg ? (0ULL - h8) : h8));
    L.q = clamp127((int64_t)(neg ? (0ULL - r8) : r8));
  } else {
    L.h = L.q = 0;
  }
  const uint64_t uu = td + (1ULL << be);
  L.a = (uint32_t)(uu >> 36);
  L.b = (uint32_t)((uu >> 18) & 0x3FFFFu);
  L.c = (uint32_t)(uu & 0x3FFFFu);
  return L;
}

// Balanced residue byte of one element for modulus index t; cb undoes the
// 2^b bias (cb = p - (2^b mod p)).
__device__ __forceinline__ uint32_t residue_byte(const Limbs& L, uint32_t p, uint32_t c36, uint32_t c18,
                                                 uint32_t cb, uint32_t mu2) {
  const uint32_t v = L.a * c36 + L.b * c18 + L.c + cb;
  const uint32_t q = __umulhi(v, mu2);
  uint32_t r = v - q * p;
  if (r >= p) r -= p;
  int rb = (int)r;
  if (rb > ((int)p - 1) / 2) rb -= (int)p;
  return (uint32_t)(uint8_t)(int8_t)rb;
}

__device__ __forceinline__ uint32_t pack4(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  return b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
}
__device__ __forceinline__ uint32_t pack4i(int b0, int b1, int b2, int b3) {
  return pack4((uint32_t)(uint8_t)b0, (uint32_t)(uint8_t)b1, (uint32_t)(uint8_t)b2, (uint32_t)(uint8_t)b3);
}

}  // namespace

// [rows, K] operand: thread (x, y) of a (32, 8) block handles 8 consecutive
// columns of one row; a warp covers 256 columns (2 KB read, 256 B written per
// plane, both contiguous).
template <bool VEC>
__global__ void __launch_bounds__(256) extract_rows_kernel(const ExtractArgs a, const ModTables T) {
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int be = gn.bits_eff;
  const bool corr = a.use_corr != 0;
  const int P = T.P;
  const int64_t nch = a.Kp >> 3;
  const int64_t pstride = a.rows * a.Kp;
  for (int64_t r = (int64_t)blockIdx.y * 8 + threadIdx.y; r < a.rows; r += (int64_t)gridDim.y * 8) {
    const int s = (int)a.sft[r] + gn.g;
    const double* __restrict__ xr = a.X + r * a.ld + a.koff;
    for (int64_t ch = (int64_t)blockIdx.x * 32 + threadIdx.x; ch < nch; ch += (int64_t)gridDim.x * 32) {
      const int64_t k0 = ch << 3;
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
      Limbs L[8];
#pragma unroll
      for (int u = 0; u < 8; u++) L[u] = split_elem(x[u], s, be, corr);
      int8_t* dst = a.planes + r * a.Kp + k0;
      for (int t = 0; t < P; t++) {
        const uint32_t p = T.p[t], c36 = T.c36[t], c18 = T.c18[t], mu2 = T.mu2[t];
        const uint32_t cb = p - (uint32_t)T.pow2mod[t][be - 16];
        uint32_t by[8];
#pragma unroll
        for (int u = 0; u < 8; u++) by[u] = residue_byte(L[u], p, c36, c18, cb, mu2);
        *reinterpret_cast<uint2*>(dst + t * pstride) =
            make_uint2(pack4(by[0], by[1], by[2], by[3]), pack4(by[4], by[5], by[6], by[7]));
      }
      if (corr) {
        *reinterpret_cast<uint2*>(dst + a.hi_plane * pstride) =
            make_uint2(pack4i(L[0].h, L[1].h, L[2].h, L[3].h), pack4i(L[4].h, L[5].h, L[6].h, L[7].h));
        *reinterpret_cast<uint2*>(dst + a.q_plane * pstride) =
            make_uint2(pack4i(L[0].q, L[1].q, L[2].q, L[3].q), pack4i(L[4].q, L[5].q, L[6].q, L[7].q));
      }
    }
  }
}

// [batch, K, N] operand: a block transposes a 64 (k) x 32 (n) tile.  Thread
// (n = lane, warp w) reads columns coalesced along n for the k quads w and
// w + 8, packs four k-consecutive residues per plane into one word in shared
// memory (row pitch 17 words: conflict-free writes), then the block writes
// each plane's 32 x 64-byte tile as 16-byte vectors along K.
constexpr int kColTileK = 64, kColTileN = 32, kColPitch = 17;

__global__ void __launch_bounds__(256) extract_cols_kernel(const ExtractArgs a, const ModTables T) {
  __shared__ uint32_t sw[kMaxP + 2][kColTileN][kColPitch];
  const Gain gn = pick_gain(a.maxlg[0], a.maxlg[1], T.log2M, a.bits);
  const int be = gn.bits_eff;
  const bool corr = a.use_corr != 0;
  const int P = T.P;
  const int64_t b = blockIdx.z;
  const int64_t n0 = (int64_t)blockIdx.x * kColTileN, k0 = (int64_t)blockIdx.y * kColTileK;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t n = n0 + tx;
  const bool nin = n < a.N;
  const int s = nin ? (int)a.sft[b * a.N + n] + gn.g : 0;
  const double* __restrict__ xb = a.X + b * a.K * a.N + n;
#pragma unroll
  for (int qi = 0; qi < 2; qi++) {
    const int qd = ty + 8 * qi;
    const int64_t kb = k0 + 4 * qd;
    Limbs L[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int64_t k = kb + u;
      const double x = (nin && k < a.K) ? __ldg(xb + k * a.N) : 0.0;
      L[u] = split_elem(x, s, be, corr);
    }
    for (int t = 0; t < P; t++) {
      const uint32_t p = T.p[t], c36 = T.c36[t], c18 = T.c18[t], mu2 = T.mu2[t];
      const uint32_t cb = p - (uint32_t)T.pow2mod[t][be - 16];
      sw[t][tx][qd] = pack4(residue_byte(L[0], p, c36, c18, cb, mu2), residue_byte(L[1], p, c36, c18, cb, mu2),
                            residue_byte(L[2], p, c36, c18, cb, mu2), residue_byte(L[3], p, c36, c18, cb, mu2));
    }
    if (corr) {
      sw[a.hi_plane][tx][qd] = pack4i(L[0].h, L[1].h, L[2].h, L[3].h);
      sw[a.q_plane][tx][qd] = pack4i(L[0].q, L[1].q, L[2].q, L[3].q);
    }
  }
  __syncthreads();
  const int G = P + (corr ? 2 : 0);
  const int64_t pstride = a.rows * a.Kp;
  for (int i = threadIdx.x; i < G * 128; i += 256) {
    const int t = i >> 7, rem = i & 127, row = rem >> 2, part = rem & 3;
    const int64_t nn = n0 + row, kk = k0 + part * 16;
    if (nn < a.N && kk < a.Kp) {
      const uint4 v = make_uint4(sw[t][row][part * 4 + 0], sw[t][row][part * 4 + 1], sw[t][row][part * 4 + 2],
                                 sw[t][row][part * 4 + 3]);
      *reinterpret_cast<uint4*>(a.planes + t * pstride + (b * a.N + nn) * a.Kp + kk) = v;
    }
  }
}

void launch_extract_rows(const ExtractArgs& a, const ModTables& T, cudaStream_t s) {
  if (a.rows <= 0 || a.Kp <= 0) return;
  const int64_t nch = a.Kp >> 3;
  const unsigned gx = (unsigned)std::min<int64_t>((nch + 31) / 32, 1 << 20);
  const unsigned gy = (unsigned)std::min<int64_t>((a.rows + 7) / 8, 65535);
  const bool vec = (a.ld % 2 == 0) && (a.koff % 2 == 0) && ((reinterpret_cast<uintptr_t>(a.X) & 15) == 0);
  if (vec) extract_rows_kernel<true><<<dim3(gx, gy), dim3(32, 8), 0, s>>>(a, T);
  else extract_rows_kernel<false><<<dim3(gx, gy), dim3(32, 8), 0, s>>>(a, T);
}

void launch_extract_cols(const ExtractArgs& a, const ModTables& T, cudaStream_t s) {
  if (a.N <= 0 || a.Kp <= 0 || a.batch <= 0) return;
  const dim3 grid((unsigned)((a.N + kColTileN - 1) / kColTileN), (unsigned)((a.Kp + kColTileK - 1) / kColTileK),
                  (unsigned)a.batch);
  extract_cols_kernel<<<grid, 256, 0, s>>>(a, T);
}

}  // namespace f64e
