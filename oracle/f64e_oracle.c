/*
 * f64e_oracle.c -- CPU restatement of the fp64-emu RARE emulated-FP64 matrix
 * product (reference: fp64_emu_cuda/fp64_emu.cu of CharlesCNorton/fp64-emu).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker: the tests, the
 * smoke check and bench.py's cpu_baseline leg call it; the product (the CUDA
 * library under fp64-emu_b200/csrc) never links, loads or falls back to it.
 *
 * Every stage follows the reference's arithmetic step for step where the
 * result depends on the order of floating-point operations (the sizing sums,
 * the float Cauchy-Schwarz rule, the fp64 recombine), and restates the exact
 * integer stages (residues, modular dot products, Garner digits, int128
 * recombine) by their mathematical definition, which the reference's Barrett
 * forms reproduce exactly (their reduction bounds are checked in the comments
 * below).
 *
 * Floating-point contraction: nvcc contracts `s += v * v` and
 * `acc * m + a` into fused multiply-adds by default (-fmad=true).  `contract`
 * selects fma() for exactly those expressions, so the oracle can model either
 * compilation; 1 is what the reference's default build does.
 *
 * Build: oracle/Makefile (gcc -O3 -mavx2 -mfma -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_MAXP 20
#define ORC_GROUPS 5 /* packed Garner factor words: four int8 factors per word */

/* ---------------------------------------------------------------- sizing -- */

/* Shift and log2-norm from a row/column max |x| and sum of squares
 * (fp64_emu.cu:136-145 and 184-188). */
static void shift_from_stats(double m, double s2, int bits, int16_t* sft, float* lg) {
  const int e = (m > 0.0 && isfinite(m)) ? ilogb(m) : 0;
  const int sh = (bits - 1) - e;
  *lg = (s2 > 0.0 && isfinite(s2)) ? (float)(0.5 * log2(s2) + sh)
                                   : (m > 0.0 ? INFINITY : -INFINITY);
  *sft = (int16_t)sh;
}

static inline double sq_acc(double ss, double v, int contract) {
  return contract ? fma(v, v, ss) : ss + v * v;
}

/* Per-row statistics, one row at a time, in the reference's order
 * (fp64_emu.cu:111-146): 256 thread-strided partials, then the 128..1
 * pairwise tree. */
void orc_row_stats(const double* X, int64_t rows, int64_t cols, int bits, int contract,
                   int16_t* sft, float* lg) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    const double* x = X + r * cols;
    double pm[256], ps[256];
    for (int t = 0; t < 256; t++) {
      double mx = 0.0, ss = 0.0;
      for (int64_t c = t; c < cols; c += 256) {
        const double v = x[c];
        mx = fmax(mx, fabs(v));
        ss = sq_acc(ss, v, contract);
      }
      pm[t] = mx;
      ps[t] = ss;
    }
    for (int s = 128; s > 0; s >>= 1)
      for (int t = 0; t < s; t++) {
        pm[t] = fmax(pm[t], pm[t + s]);
        ps[t] += ps[t + s];
      }
    shift_from_stats(pm[0], ps[0], bits, &sft[r], &lg[r]);
  }
}

/* Slab count for the column statistics (fp64_emu.cu:1159-1162). */
void orc_col_slabs(int64_t NF, int64_t K, int64_t* kslab, int64_t* nslab) {
  int64_t nsl0 = 131072 / (NF > 1 ? NF : 1);
  if (nsl0 < 1) nsl0 = 1;
  if (nsl0 > 128) nsl0 = 128;
  *kslab = (K + nsl0 - 1) / nsl0;
  *nslab = (*kslab > 0) ? (K + *kslab - 1) / *kslab : 0;
}

/* Per-column statistics of an operand given as [batch, K, N]
 * (fp64_emu.cu:152-189): each column sums its K slabs sequentially, then the
 * slab partials are combined in slab order. */
void orc_col_stats_ex(const double* X, int64_t batch, int64_t K, int64_t N, int64_t slab_cols,
                      int bits, int contract, int16_t* sft, float* lg);

void orc_col_stats(const double* X, int64_t batch, int64_t K, int64_t N, int bits,
                   int contract, int16_t* sft, float* lg) {
  orc_col_stats_ex(X, batch, K, N, 0, bits, contract, sft, lg);
}

/* slab_cols > 0 orders the column sums as the slab rule does for that many
 * columns (a rank holding a slice of the columns reproduces the full run). */
void orc_col_stats_ex(const double* X, int64_t batch, int64_t K, int64_t N, int64_t slab_cols,
                      int bits, int contract, int16_t* sft, float* lg) {
  const int64_t NF = batch * N;
  int64_t kslab, nslab;
  orc_col_slabs(slab_cols > 0 ? slab_cols : NF, K, &kslab, &nslab);
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < NF; j++) {
    const int64_t b = j / N, n = j - b * N;
    const double* base = X + b * K * N + n;
    double MX = 0.0, SS = 0.0;
    for (int64_t s = 0; s < nslab; s++) {
      const int64_t k0 = s * kslab;
      const int64_t k1 = (k0 + kslab < K) ? k0 + kslab : K;
      double mx = 0.0, ss = 0.0;
      for (int64_t k = k0; k < k1; k++) {
        const double v = base[k * N];
        mx = fmax(mx, fabs(v));
        ss = sq_acc(ss, v, contract);
      }
      MX = fmax(MX, mx);
      SS += ss;
    }
    shift_from_stats(MX, SS, bits, &sft[j], &lg[j]);
  }
}

/* CRT range in bits as the reference's table cache sums it: float
 * accumulation of log2 p (fp64_emu.cu:1052), capped at 126 (call site
 * fp64_emu.cu:1182-1185). */
float orc_log2M(const int32_t* primes, int P) {
  float s = 0.0f;
  for (int i = 0; i < P; i++) s += (float)log2((double)primes[i]);
  return s < 126.0f ? s : 126.0f;
}

int orc_pick_bits_from_max(float a, float b, float log2M, int bits, int* g_out);

/* Cauchy-Schwarz width rule (fp64_emu.cu:193-231).  Returns bits_eff and the
 * gain g folded into every shift.  max over floats is order independent. */
int orc_pick_bits(const float* lgA, int64_t m, const float* lgB, int64_t n, float log2M,
                  int bits, int* g_out) {
  float a = -INFINITY, b = -INFINITY;
  for (int64_t i = 0; i < m; i++) a = fmaxf(a, lgA[i]);
  for (int64_t j = 0; j < n; j++) b = fmaxf(b, lgB[j]);
  return orc_pick_bits_from_max(a, b, log2M, bits, g_out);
}

int orc_pick_bits_from_max(float a, float b, float log2M, int bits, int* g_out) {
  const float need = a + b + 0.5f;
  int g = 0;
  if (isfinite(need)) g = (int)floorf((log2M - 1.0f - need) * 0.5f);
  if (g > 53 - bits) g = 53 - bits;
  int be = bits + g;
  if (be < 16) be = 16;
  *g_out = be - bits;
  return be;
}

/* ------------------------------------------------------------ extraction -- */

/* Round-to-nearest-even of mag * 2^(-s) (fp64_emu.cu:292-299). */
static inline uint64_t rne_shr(uint64_t mag, int s) {
  if (s <= 0) return (-s < 64) ? (mag << (-s)) : 0ULL;
  if (s > 63) return 0ULL;
  const uint64_t keep = mag >> s;
  const uint64_t rem = mag & ((1ULL << s) - 1ULL);
  const uint64_t half = 1ULL << (s - 1);
  return keep + ((rem > half || (rem == half && (keep & 1ULL))) ? 1ULL : 0ULL);
}

/* Integer split of the raw IEEE encoding (fp64_emu.cu:300-321): returns the
 * signed scaled integer round(x * 2^srow) and the correction digits
 * hi = clamp(round(T * 2^(7-bits))) and q = clamp(round(resid * 2^8)). */
static inline int64_t split_x(double x, int srow, int bits, int8_t* h, int8_t* q) {
  int64_t xb;
  memcpy(&xb, &x, 8);
  const int neg = xb < 0;
  const int e = (int)((xb >> 52) & 0x7FF);
  const uint64_t m = (uint64_t)xb & 0xFFFFFFFFFFFFFULL;
  const uint64_t mag = e ? ((1ULL << 52) | m) : m;
  const int t = (e ? e : 1) - 1075 + srow + 52;
  const uint64_t Tu = rne_shr(mag, 52 - t);
  const int64_t r8 = (int64_t)rne_shr(mag, 44 - t) - (int64_t)(Tu << 8);
  const int64_t h8 = (int64_t)rne_shr(Tu, bits - 7);
  const int64_t hs = neg ? -h8 : h8;
  const int64_t qs = neg ? -r8 : r8;
  *h = (int8_t)(hs > 127 ? 127 : (hs < -127 ? -127 : hs));
  *q = (int8_t)(qs > 127 ? 127 : (qs < -127 ? -127 : qs));
  return neg ? -(int64_t)Tu : (int64_t)Tu;
}

/* Balanced residue: the unique r == v (mod p) in [-floor(p/2), floor((p-1)/2)].
 * The reference's 32-bit Barrett forms (fp64_emu.cu:278-287 on the biased limb
 * sum v < 2^28, fp64_emu.cu:613-620 on |v| < 2^31, fp64_emu.cu:42-51 on the
 * Garner digits) all return exactly this value: their quotient estimates fall
 * short by at most the number of correction subtractions they perform. */
static inline int bal_mod(int64_t v, int p) {
  int64_t r = v % p;
  if (r < 0) r += p;
  if (r > (p - 1) / 2) r -= p;
  return (int)r;
}

/* Residue and correction planes of rows x [rows, K] with per-row or per-element
 * shifts.  planes: [P][rows][K] balanced residues; hi, q: [rows][K] (may be
 * NULL when use_corr is off).  `srow[r]` is the (already widened) shift of row
 * r; for operands shifted per column, `scol` gives the per-k shift and srow is
 * ignored. */
void orc_extract(const double* X, int64_t rows, int64_t K, const int16_t* srow,
                 const int16_t* scol, int bits, const int32_t* primes, int P, int8_t* planes,
                 int8_t* hi, int8_t* q) {
  const int64_t total = rows * K;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t k = 0; k < K; k++) {
      int8_t h, qq;
      const int s = scol ? scol[k] : srow[r];
      const int64_t td = split_x(X[r * K + k], s, bits, &h, &qq);
      const int64_t o = r * K + k;
      if (hi) hi[o] = h;
      if (q) q[o] = qq;
      for (int t = 0; t < P; t++) planes[(int64_t)t * total + o] = (int8_t)bal_mod(td, primes[t]);
    }
  }
}

/* ---------------------------------------------------------- modular GEMM -- */

/* Exact dot product of two int8 rows; int32 partial sums over 65536-long
 * chunks (each < 2^30 in magnitude) folded into int64. */
static inline int64_t dot_i8(const int8_t* a, const int8_t* b, int64_t K) {
  int64_t tot = 0;
  for (int64_t k0 = 0; k0 < K; k0 += 65536) {
    const int64_t k1 = (k0 + 65536 < K) ? k0 + 65536 : K;
    int32_t s = 0;
    for (int64_t k = k0; k < k1; k++) s += (int32_t)a[k] * (int32_t)b[k];
    tot += s;
  }
  return tot;
}

/* res[t][b*M+m][n] = balanced residue of (A_t B_t^T)[m,n] mod p_t;
 * corr[b*M+m][n] = Ahi.Bq^T + Aq.Bhi^T (int64), the two first-order
 * correction products (plane pairing at fp64_emu.cu:1246-1268). */
void orc_residue_gemm(const int8_t* Apl, const int8_t* Bpl, const int8_t* Ahi,
                      const int8_t* Aq, const int8_t* Bhi, const int8_t* Bq, int64_t batch,
                      int64_t M, int64_t N, int64_t K, const int32_t* primes, int P, int8_t* res,
                      int64_t* corr) {
  const int64_t MF = batch * M, NF = batch * N;
  const int64_t tA = MF * K, tB = NF * K, tC = MF * N;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t i = 0; i < MF; i++) {
    const int64_t b = i / M;
    for (int64_t n = 0; n < N; n++) {
      const int64_t j = b * N + n;
      for (int t = 0; t < P; t++) {
        const int64_t d = dot_i8(Apl + t * tA + i * K, Bpl + t * tB + j * K, K);
        res[t * tC + i * N + n] = (int8_t)bal_mod(d, primes[t]);
      }
      if (corr)
        corr[i * N + n] = dot_i8(Ahi + i * K, Bq + j * K, K) + dot_i8(Aq + i * K, Bhi + j * K, K);
    }
  }
}

/* -------------------------------------------------------- reconstruction -- */

static int modinv_small(int a, int m) {
  a %= m;
  if (a < 0) a += m;
  for (int x = 1; x < m; x++)
    if ((int64_t)a * x % m == 1) return x;
  return 0;
}

/* Garner tables (fp64_emu.cu:969-993): c[t][u] = balanced (M_u mod p_t) for
 * u < t with M_u = p_0 ... p_{u-1}; minv[t] = (M_t mod p_t)^{-1}; m64[g] =
 * product of moduli 7g..7g+6. */
void orc_tables(const int32_t* primes, int P, int32_t* cfac /*[P][P]*/, int32_t* minv,
                int64_t* m64) {
  memset(cfac, 0, sizeof(int32_t) * P * P);
  m64[0] = m64[1] = 1;
  for (int g = 0; g < 2; g++) {
    int64_t prod = 1;
    for (int t = g * 7; t < g * 7 + 7 && t < P; t++) prod *= primes[t];
    m64[g] = prod;
  }
  for (int t = 0; t < P; t++) {
    const int64_t pt = primes[t];
    int64_t run = 1 % pt;
    for (int u = 0; u < P; u++) {
      if (u == t) minv[t] = modinv_small((int)run, (int)pt);
      if (u < t) {
        int bal = (int)run;
        if (bal > ((int)pt - 1) / 2) bal -= (int)pt;
        cfac[t * P + u] = bal;
      }
      run = run * (primes[u] % pt) % pt;
    }
  }
}

/* Correctly rounded int128 -> double with the sticky-tail fold
 * (fp64_emu.cu:94-105). */
static double s128_to_double(__int128 v) {
  const int neg = v < 0;
  const unsigned __int128 u = neg ? (unsigned __int128)0 - (unsigned __int128)v
                                  : (unsigned __int128)v;
  const uint64_t hi = (uint64_t)(u >> 64), lo = (uint64_t)u;
  if (hi == 0) {
    const double m = (double)lo;
    return neg ? -m : m;
  }
  const int sh = 64 - __builtin_clzll(hi);
  uint64_t top, tail;
  if (sh == 64) {
    top = hi;
    tail = lo;
  } else {
    top = (hi << (64 - sh)) | (lo >> sh);
    tail = lo & ((1ULL << sh) - 1ULL);
  }
  const double m = ldexp((double)(top | (tail != 0ULL ? 1ULL : 0ULL)), sh);
  return neg ? -m : m;
}

/* Balanced-Garner reconstruction, correction and rescale
 * (fp64_emu.cu:854-952).  res: [P][MF][N]; corr: [MF][N] int64 or NULL;
 * sftA: [MF]; sftB: [batch*N] (already widened by g). */
void orc_reconstruct(const int8_t* res, const int64_t* corr, int64_t batch, int64_t M,
                     int64_t N, const int32_t* primes, int P, const int16_t* sftA,
                     const int16_t* sftB, int bits_eff, int exact, int contract, double* C) {
  int32_t cfac[ORC_MAXP * ORC_MAXP], minv[ORC_MAXP];
  int64_t m64[2];
  orc_tables(primes, P, cfac, minv, m64);
  const int64_t MF = batch * M, total = MF * N;
  const int cshift = bits_eff - 15;
  const int ng = (P + 6) / 7;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < MF; i++) {
    const int64_t b = i / M;
    for (int64_t j = 0; j < N; j++) {
      const int64_t idx = i * N + j;
      int d[ORC_MAXP];
      for (int t = 0; t < P; t++) {
        int acc = 0;
        for (int u = 0; u < t; u++) acc += d[u] * cfac[t * P + u];
        d[t] = bal_mod((int64_t)(res[(int64_t)t * total + idx] - acc) * minv[t], primes[t]);
      }
      int64_t a0 = 0, a1 = 0, a2 = 0;
      for (int t = P - 1; t >= 0; t--) {
        if (t >= 14) a2 = a2 * primes[t] + d[t];
        else if (t >= 7) a1 = a1 * primes[t] + d[t];
        else a0 = a0 * primes[t] + d[t];
      }
      const int64_t cr = corr ? corr[idx] : 0;
      const int sh = -(int)sftA[i] - (int)sftB[b * N + j];
      if (exact) {
        __int128 acc = (ng == 3) ? a2 : ((ng == 2) ? a1 : a0);
        if (ng == 3) acc = acc * (__int128)m64[1] + a1;
        if (ng >= 2) acc = acc * (__int128)m64[0] + a0;
        acc += (__int128)cr * ((__int128)1 << cshift);
        C[idx] = ldexp(s128_to_double(acc), sh);
      } else {
        double acc = (double)((ng == 3) ? a2 : ((ng == 2) ? a1 : a0));
        if (ng == 3)
          acc = contract ? fma(acc, (double)m64[1], (double)a1) : acc * (double)m64[1] + (double)a1;
        if (ng >= 2)
          acc = contract ? fma(acc, (double)m64[0], (double)a0) : acc * (double)m64[0] + (double)a0;
        acc += ldexp((double)cr, cshift);
        C[idx] = ldexp(acc, sh);
      }
    }
  }
}

/* ------------------------------------------------------------ top level -- */

/* Whole product in the reference's pipeline order (run_crt,
 * fp64_emu.cu:1127-1477, and the deep-K form run_crt_bigk, 1485-1579, which
 * computes the same residues of the full-depth dot products).
 *   A: [batch, M, K];  B: [batch, N, K] (b_nt = 0) or [batch, K, N] (b_nt = 1)
 *   C: [batch, M, N]
 * Optional outputs (NULL to skip): bits_eff_out, sftA_out [batch*M],
 * sftB_out [batch*N] (shifts after the widening fold).
 * Returns 0, or -1 on bad arguments / allocation failure. */
int orc_emu_ex(const double* A, const double* B, double* C, int64_t batch, int64_t M, int64_t N,
               int64_t K, int b_nt, const int32_t* primes, int P, int exact, int bits, int use_corr,
               int contract, int32_t* bits_eff_out, int16_t* sftA_out, int16_t* sftB_out,
               int64_t slab_cols, float* maxlg_out, const float* maxlg_in);

int orc_emu(const double* A, const double* B, double* C, int64_t batch, int64_t M, int64_t N,
            int64_t K, int b_nt, const int32_t* primes, int P, int exact, int bits, int use_corr,
            int contract, int32_t* bits_eff_out, int16_t* sftA_out, int16_t* sftB_out) {
  return orc_emu_ex(A, B, C, batch, M, N, K, b_nt, primes, P, exact, bits, use_corr, contract,
                    bits_eff_out, sftA_out, sftB_out, 0, NULL, NULL);
}

/* Extended form for the partitioned protocol: maxlg_out (float[2]) receives
 * this operand pair's maxima of the log2 norms; maxlg_in, when given, replaces
 * them in the width rule (the all-reduced maxima); with C == NULL only the
 * sizing runs. */
int orc_emu_ex(const double* A, const double* B, double* C, int64_t batch, int64_t M, int64_t N,
               int64_t K, int b_nt, const int32_t* primes, int P, int exact, int bits, int use_corr,
               int contract, int32_t* bits_eff_out, int16_t* sftA_out, int16_t* sftB_out,
               int64_t slab_cols, float* maxlg_out, const float* maxlg_in) {
  if (P < 1 || P > ORC_MAXP || bits < 16 || bits > 53 || batch < 0 || M < 0 || N < 0 || K < 0)
    return -1;
  const int64_t MF = batch * M, NF = batch * N;
  if (MF == 0 || NF == 0) return 0;
  if (K == 0) {
    if (C) memset(C, 0, sizeof(double) * MF * N);
    return 0;
  }
  int rc = -1;
  int16_t *sA = malloc(sizeof(int16_t) * MF), *sB = malloc(sizeof(int16_t) * NF);
  float *lA = malloc(sizeof(float) * MF), *lB = malloc(sizeof(float) * NF);
  double* Bn = NULL;
  int8_t *pa = NULL, *pb = NULL, *res = NULL;
  int64_t* corr = NULL;
  if (!sA || !sB || !lA || !lB) goto out;

  orc_row_stats(A, MF, K, bits, contract, sA, lA);
  if (b_nt) orc_col_stats_ex(B, batch, K, N, slab_cols, bits, contract, sB, lB);
  else orc_row_stats(B, NF, K, bits, contract, sB, lB);
  float ma = -INFINITY, mb = -INFINITY;
  for (int64_t i = 0; i < MF; i++) ma = fmaxf(ma, lA[i]);
  for (int64_t j = 0; j < NF; j++) mb = fmaxf(mb, lB[j]);
  if (maxlg_out) {
    maxlg_out[0] = ma;
    maxlg_out[1] = mb;
  }
  if (!C) {
    rc = 0;
    goto out;
  }
  if (maxlg_in) {
    ma = maxlg_in[0];
    mb = maxlg_in[1];
  }
  int g = 0;
  const int be = orc_pick_bits_from_max(ma, mb, orc_log2M(primes, P), bits, &g);
  for (int64_t i = 0; i < MF; i++) sA[i] = (int16_t)(sA[i] + g);
  for (int64_t j = 0; j < NF; j++) sB[j] = (int16_t)(sB[j] + g);

  /* B as [batch, N, K] rows for the extraction. */
  const double* Brow = B;
  if (b_nt) {
    Bn = malloc(sizeof(double) * NF * K);
    if (!Bn) goto out;
    for (int64_t b = 0; b < batch; b++)
      for (int64_t k = 0; k < K; k++)
        for (int64_t n = 0; n < N; n++) Bn[(b * N + n) * K + k] = B[(b * K + k) * N + n];
    Brow = Bn;
  }
  const int G = P + (use_corr ? 2 : 0);
  pa = malloc((size_t)G * MF * K);
  pb = malloc((size_t)G * NF * K);
  res = malloc((size_t)P * MF * N);
  if (use_corr) corr = malloc(sizeof(int64_t) * MF * N);
  if (!pa || !pb || !res || (use_corr && !corr)) goto out;
  int8_t* Ahi = use_corr ? pa + (int64_t)P * MF * K : NULL;
  int8_t* Aq = use_corr ? pa + (int64_t)(P + 1) * MF * K : NULL;
  int8_t* Bhi = use_corr ? pb + (int64_t)P * NF * K : NULL;
  int8_t* Bq = use_corr ? pb + (int64_t)(P + 1) * NF * K : NULL;
  orc_extract(A, MF, K, sA, NULL, be, primes, P, pa, Ahi, Aq);
  orc_extract(Brow, NF, K, sB, NULL, be, primes, P, pb, Bhi, Bq);
  orc_residue_gemm(pa, pb, Ahi, Aq, Bhi, Bq, batch, M, N, K, primes, P, res, corr);
  orc_reconstruct(res, corr, batch, M, N, primes, P, sA, sB, be, exact, contract, C);
  if (bits_eff_out) *bits_eff_out = be;
  if (sftA_out) memcpy(sftA_out, sA, sizeof(int16_t) * MF);
  if (sftB_out) memcpy(sftB_out, sB, sizeof(int16_t) * NF);
  rc = 0;
out:
  free(sA); free(sB); free(lA); free(lB); free(Bn); free(pa); free(pb); free(res); free(corr);
  return rc;
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
