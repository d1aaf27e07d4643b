// Host orchestration and C ABI of libf64e (declared in include/f64e.h).
//
// One call runs (reference pipeline run_crt, fp64_emu.cu:1127-1477):
//   sizing      row / column shifts and log2 norms, operand maxima
//   extraction  K-major int8 residue + correction planes
//   GEMM        one persistent tcgen05 launch over every plane-batch slot
//   rebuild     Garner reconstruction, correction, rescale
// Deep K (> 131071, mm / bmm only) runs the extraction and GEMM per 65536-deep
// segment and accumulates residues (int32) and corrections (int64) before one
// fold and one reconstruction (reference run_crt_bigk, fp64_emu.cu:1485-1579).
//
// Differences from the reference that do not change results: the modulus
// tables travel by value as kernel parameters (no per-device cache, no
// uploads), the width rule is evaluated where it is used instead of rewriting
// the shifts, and there is a single GEMM engine, so there is no first-call
// probe and no host synchronisation anywhere on the product path.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "f64e.h"
#include "f64e_kernels.h"

namespace f64e {
void launch_deepk_accum(const int8_t* res, int32_t* racc, int64_t nres, const int32_t* corr, int64_t* cacc,
                        int64_t ncorr, int first, cudaStream_t s);
void launch_deepk_fold(const int32_t* racc, int8_t* res, int64_t per_plane, const ModTables& T, cudaStream_t s);
}  // namespace f64e

using namespace f64e;

namespace {

thread_local std::string g_err;
std::atomic<uint64_t> g_wait_limit{2000000000ULL};

constexpr int64_t kNtMaxK = 131071;              // single-launch int32 bound (fp64_emu.cu:1596-1599)
constexpr int64_t kSegK = 65536;                 // deep-K segment depth
constexpr int64_t kMaxK = 128 * kSegK;           // 8,388,608
constexpr int64_t kFusedCorrMaxK = 65536;        // 2 K 127^2 < 2^31
constexpr int64_t kB200Sms = 148;                 // CTAs of one wave of the GEMM kernels

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

// F64E_GEMM_SINGLE=1 keeps every product on the one-CTA GEMM (A/B checks of
// the CTA-pair kernel); read per call.
bool gemm_force_single() {
  const char* v = std::getenv("F64E_GEMM_SINGLE");
  return v && v[0] == '1';
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(F64E_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int modinv_small(int a, int m) {
  a %= m;
  if (a < 0) a += m;
  for (int x = 1; x < m; x++)
    if ((int64_t)a * x % m == 1) return x;
  return 0;
}

// Host-built modulus tables (reference: build_recon_tables, fp64_emu.cu:969-993,
// and the extraction constants of fp64_emu.cu:264-273), cached per modulus list.
int get_tables(const int32_t* primes, int P, ModTables* out) {
  static std::mutex mtx;
  static std::map<std::vector<int32_t>, ModTables> cache;
  std::vector<int32_t> key(primes, primes + P);
  std::lock_guard<std::mutex> lk(mtx);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return F64E_OK;
  }
  ModTables T;
  std::memset(&T, 0, sizeof(T));
  T.P = P;
  float l2 = 0.0f;
  for (int i = 0; i < P; i++) l2 += (float)std::log2((double)primes[i]);
  T.log2M = std::min(l2, 126.0f);
  for (int t = 0; t < P; t++) {
    const uint32_t p = (uint32_t)primes[t];
    T.p[t] = p;
    T.mdiv[t] = (uint32_t)((1ULL << 32) / p);
    T.off[t] = (0x80000000u / p) * p;
    T.mu2[t] = 2u * ((1u << 31) / p);
    T.c36[t] = (uint32_t)((1ULL << 36) % p);
    T.c18[t] = (uint32_t)((1ULL << 18) % p);
    for (int b = 16; b <= 53; b++) T.pow2mod[t][b - 16] = (uint8_t)((1ULL << b) % p);
  }
  for (int g = 0; g < 2; g++) {
    int64_t prod = 1;
    for (int t = g * 7; t < std::min(g * 7 + 7, P); t++) prod *= primes[t];
    T.m64[g] = prod;
  }
  for (int t = 0; t < P; t++) {
    const int64_t pt = primes[t];
    int64_t run = 1 % pt;  // M_u mod p_t
    for (int u = 0; u < P; u++) {
      if (u == t) {
        T.minv[t] = modinv_small((int)run, (int)pt);
        if (T.minv[t] == 0 && pt > 1)
          return fail(F64E_ERR_ARGUMENT, "moduli must be pairwise coprime (modulus %d)", (int)pt);
      }
      if (u < t) {
        int bal = (int)run;
        if (bal > ((int)pt - 1) / 2) bal -= (int)pt;
        T.mp[t][u >> 2] |= (int32_t)((uint32_t)(uint8_t)(int8_t)bal << (8 * (u & 3)));
      }
      run = run * (primes[u] % pt) % pt;
    }
  }
  // Fast-form constants (see ModTables).
  T.fast_recon = 1;
  for (int t = 0; t < P; t++) {
    const uint64_t p = (uint64_t)primes[t];
    uint32_t kl = 0, kh = 0;
    for (int i = 0; i < 4; i++) kl |= (uint32_t)(((1ULL << (8 * i)) % p) & 0xFF) << (8 * i);
    for (int i = 0; i < 3; i++) kh |= (uint32_t)(((1ULL << (8 * (i + 4))) % p) & 0xFF) << (8 * i);
    T.kl[t] = kl;
    T.kh[t] = kh;
    T.mex[t] = (uint32_t)(((1ULL << 32) + p - 1) / p);
    if (p <= 128) T.fast_recon = 0;
    T.mrec[t] = (p > 128) ? (uint32_t)(((1ULL << 39) + p - 1) / p) : 0;
  }
  for (int t = 0; t < P; t++) {
    const int64_t pt = primes[t];
    int64_t run = 1 % pt;
    int64_t csum = 0;  // sum_u h_u * (M_u mod p_t)
    for (int u = 0; u < t; u++) {
      T.cu[t][u >> 2] |= (uint32_t)(run & 0xFF) << (8 * (u & 3));
      csum += (int64_t)(primes[u] / 2) * run;
      run = run * (primes[u] % pt) % pt;
    }
    const int64_t kc = ((csum % pt) * T.minv[t] + pt / 2) % pt;
    const int64_t B = pt * (((1LL << 29) + pt - 1) / pt);
    T.krec[t] = (uint32_t)(kc + B);
  }
  for (int t = 0; t < P; t++) {
    uint64_t w = 1;
    for (int u = (t / 7) * 7; u < t; u++) w *= (uint64_t)primes[u];
    T.wgrp[t] = w;
  }
  for (int g = 0; g < 3; g++) {
    int64_t hv = 0;
    for (int t = std::min(g * 7 + 6, P - 1); t >= g * 7; t--) hv = hv * primes[t] + primes[t] / 2;
    T.hoff[g] = hv;
  }
  // Direct CRT constants (see ModTables), for products of the moduli below 2^121.
  {
    using u128 = unsigned __int128;
    u128 M = 1;
    bool ok = true;
    for (int t = 0; t < P && ok; t++) {
      if (M > ((u128)1 << 121) / (u128)primes[t]) ok = false;
      else M *= (u128)primes[t];
    }
    T.crt_ok = ok ? 1 : 0;
    if (ok) {
      for (int t = 0; t < P; t++) {
        const u128 Mt = M / (u128)primes[t];
        const int y = modinv_small((int)(Mt % (u128)primes[t]), primes[t]);
        const u128 E = Mt * (u128)y;   // < M
        for (int i = 0; i < 4; i++) T.crtE[t][i] = (uint32_t)(E >> (32 * i));
      }
      for (int i = 0; i < 4; i++) T.crtM[i] = (uint32_t)(M >> (32 * i));
      const long double Md = (long double)M;
      T.crtK96 = (double)(std::ldexp(1.0L, 96) / Md);
      T.crtK32 = (double)(std::ldexp(1.0L, 32) / Md);
      T.crtK0 = (double)(1.0L / Md);
      // low end of the balanced mixed-radix range: sum_t dmin_t * (p_0 ... p_{t-1}),
      // dmin_t = -floor(p_t / 2) (the digit range of a balanced residue)
      u128 run = 1, negL = 0;
      for (int t = 0; t < P; t++) {
        negL += (u128)(primes[t] / 2) * run;
        run *= (u128)primes[t];
      }
      T.crt_c = (double)((long double)negL / Md);
      const u128 L = (u128)0 - negL;
      T.crtL[0] = (uint64_t)L;
      T.crtL[1] = (uint64_t)(L >> 64);
    }
  }
  cache.emplace(key, T);
  *out = T;
  return F64E_OK;
}

struct Plan {
  int64_t batch, M, N, K, MF, NF;
  int nt, P, G, exact, bits, use_corr;
  bool deep;
  int64_t Kseg, Kp, ldn;
  int nseg;
  int gemm_corr;   // 0 none, 1 fused int32, 2 two int32 planes
  int recon_corr;  // 0 none, 1 int32, 2 two int32 planes, 3 int64
  int64_t kslab;
  int nslab;
  size_t o_sftA, o_sftB, o_lgA, o_lgB, o_pmax, o_pss, o_pA, o_pB, o_res, o_corr, o_racc, o_cacc, total;
};

int make_plan(const f64e_problem* p, Plan* L) {
  if (!p) return fail(F64E_ERR_ARGUMENT, "null problem");
  if (p->nprimes > kMaxP) return fail(F64E_ERR_ARGUMENT, "too many primes");
  if (p->nprimes < 1) return fail(F64E_ERR_ARGUMENT, "nprimes must be at least 1");
  if (!p->primes) return fail(F64E_ERR_ARGUMENT, "primes must be a host array");
  for (int i = 0; i < p->nprimes; i++)
    if (p->primes[i] < 2 || p->primes[i] > 256)
      return fail(F64E_ERR_ARGUMENT, "moduli must lie in [2, 256] (balanced int8 residues)");
  if (p->batch < 0 || p->M < 0 || p->N < 0 || p->K < 0) return fail(F64E_ERR_ARGUMENT, "negative dimension");
  if (p->b_layout != F64E_B_NK && p->b_layout != F64E_B_KN) return fail(F64E_ERR_ARGUMENT, "bad b_layout");
  const bool nt = p->b_layout == F64E_B_KN;
  if (nt && p->K > kNtMaxK) return fail(F64E_ERR_ARGUMENT, "K bound for int32 modular GEMM");
  if (!nt && p->K > kMaxK) return fail(F64E_ERR_ARGUMENT, "K bound: 128 segments of 65536");
  if (p->bits < 16 || p->bits > 53) return fail(F64E_ERR_ARGUMENT, "bits must be in [16, 53]");
  if (p->M > INT32_MAX / 2 || p->N > INT32_MAX / 2 || p->batch > INT32_MAX / 64)
    return fail(F64E_ERR_ARGUMENT, "dimension too large");
  Plan& l = *L;
  l.batch = p->batch;
  l.M = p->M;
  l.N = p->N;
  l.K = p->K;
  l.MF = p->batch * p->M;
  l.NF = p->batch * p->N;
  l.nt = nt ? 1 : 0;
  l.P = p->nprimes;
  l.use_corr = p->use_corr ? 1 : 0;
  l.G = l.P + (l.use_corr ? 2 : 0);
  l.exact = p->exact ? 1 : 0;
  l.bits = p->bits;
  l.deep = p->K > kNtMaxK;
  l.Kseg = l.deep ? kSegK : p->K;
  l.nseg = l.deep ? (int)((p->K + kSegK - 1) / kSegK) : 1;
  l.Kp = round_up(std::max<int64_t>(l.Kseg, 1), 16);
  l.ldn = round_up(std::max<int64_t>(l.N, 1), 16);
  if (!l.use_corr) {
    l.gemm_corr = 0;
  } else if (l.Kseg > kFusedCorrMaxK) {
    l.gemm_corr = 2;
  } else {
    // The fused correction slot runs a K loop twice as long as a residue
    // slot.  When the whole GEMM is one wave of tiles (one per CTA, or per
    // CTA pair) that slot alone sets the kernel's time, so such products
    // keep the two correction products as separate planes: the same integers,
    // summed by the reconstruction.  (The deep-K accumulation takes one
    // fused plane per segment.)
    const bool pair = gemm_use_pair((int)std::min<int64_t>(l.M, INT32_MAX));
    const int64_t bm = pair ? 2 * gemm_pair_block_rows() : gemm_block_rows_a();
    const int64_t fused_tiles = ((l.M + bm - 1) / bm) * ((l.N + 255) / 256) * (l.P + 1) * l.batch;
    l.gemm_corr = (!l.deep && fused_tiles <= (pair ? kB200Sms / 2 : kB200Sms)) ? 2 : 1;
  }
  if (!l.use_corr) l.recon_corr = 0;
  else l.recon_corr = l.deep ? 3 : l.gemm_corr;
  l.kslab = 0;
  l.nslab = 0;
  if (nt) col_slabs(p->slab_cols > 0 ? p->slab_cols : l.NF, l.K, &l.kslab, &l.nslab);
  size_t o = 256;  // WsHead
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 255) / 256 * 256;
    return at;
  };
  l.o_sftA = take(sizeof(int16_t) * l.MF);
  l.o_sftB = take(sizeof(int16_t) * l.NF);
  l.o_lgA = take(sizeof(float) * l.MF);
  l.o_lgB = take(sizeof(float) * l.NF);
  l.o_pmax = take(nt ? sizeof(double) * l.nslab * l.NF : 0);
  l.o_pss = take(nt ? sizeof(double) * l.nslab * l.NF : 0);
  l.o_pA = take((size_t)l.G * l.MF * l.Kp);
  l.o_pB = take((size_t)l.G * l.NF * l.Kp);
  l.o_res = take((size_t)l.P * l.MF * l.ldn);
  const int ncorr = l.gemm_corr == 2 ? 2 : (l.gemm_corr == 1 ? 1 : 0);
  l.o_corr = take(sizeof(int32_t) * ncorr * l.MF * l.ldn);
  l.o_racc = take(l.deep ? sizeof(int32_t) * l.P * l.MF * l.ldn : 0);
  l.o_cacc = take(l.deep && l.use_corr ? sizeof(int64_t) * l.MF * l.ldn : 0);
  l.total = o;
  return F64E_OK;
}

struct Dev {
  int dev = 0;
  int sms = 0;
  bool ok = false;
};

int device_info(Dev* d) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  static std::mutex mtx;
  static std::map<int, Dev> cache;
  std::lock_guard<std::mutex> lk(mtx);
  auto it = cache.find(dev);
  if (it == cache.end()) {
    Dev v;
    v.dev = dev;
    int major = 0, minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&v.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    v.ok = (major == 10 && minor == 0);
    it = cache.emplace(dev, v).first;
  }
  *d = it->second;
  if (!d->ok) return fail(F64E_ERR_UNSUPPORTED, "fp64-emu B200 kernels need an sm_100 device");
  return F64E_OK;
}

template <typename T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

int run_sizing(const Plan& l, const double* A, const double* B, void* ws, cudaStream_t s) {
  WsHead* head = at<WsHead>(ws, 0);
  // status word and the CTA counter of the launch that takes the operand maxima
  cudaError_t e = cudaMemsetAsync(&head->status, 0, 2 * sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  if (l.nt) {
    launch_nt_stats_maxlg(A, l.MF, B, l.batch, l.K, l.N, l.kslab, l.nslab, l.bits, at<int16_t>(ws, l.o_sftA),
                          at<float>(ws, l.o_lgA), at<int16_t>(ws, l.o_sftB), at<float>(ws, l.o_lgB),
                          at<double>(ws, l.o_pmax), at<double>(ws, l.o_pss), head->maxlg, &head->counter, s);
  } else {
    launch_rows_stats_both(A, l.MF, B, l.NF, l.K, l.bits, at<int16_t>(ws, l.o_sftA), at<float>(ws, l.o_lgA),
                           at<int16_t>(ws, l.o_sftB), at<float>(ws, l.o_lgB), head->maxlg, &head->counter, s);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sizing launch");
  return F64E_OK;
}

// A view of the product: the whole problem, or one chunk of it (a block of
// rows of A and C, a block of rows and columns of the first row block, or a
// block of members of a batch).  Each chunk owns a contiguous share of the
// residue buffers and of A's planes in the chunk's own layout
// ([G][members][rows][Kp] planes, [P][members * rows][ldn] residues), so the
// kernels see it as a product of its own.  B's planes stay in the whole
// product's layout for row and column blocks (a column block addresses a
// band of rows of every plane) and are per chunk for member blocks.
struct View {
  int64_t batch, M, N;         // members, rows of A / C, columns of C in this view
  int64_t ldn;                 // row pitch of this view's residues
  int64_t ldc;                 // row pitch of C
  int64_t b_zrows;             // rows from one B plane slice (plane, member) to the next
  const double* A;             // [batch][M][K]
  const double* B;             // first of this view's rows ([N][K] layout) or columns ([K][N] layout)
  const int16_t* sftA;         // [batch * M]
  const int16_t* sftB;         // [batch * N]
  int8_t* pA;                  // [G][batch][M][Kp]
  int8_t* pB;                  // B planes: slice z at pB + z * b_zrows * Kp
  int8_t* res;                 // [P][batch * M][ldn]
  int32_t* corr;               // [ncorr][batch * M][ldn]
  double* C;                   // [batch * M] rows of pitch ldc
};

int ncorr_planes(const Plan& l) { return l.gemm_corr == 2 ? 2 : (l.gemm_corr == 1 ? 1 : 0); }

View full_view(const Plan& l, const double* A, const double* B, void* ws, double* out) {
  View v;
  v.batch = l.batch;
  v.M = l.M;
  v.N = l.N;
  v.ldn = l.ldn;
  v.ldc = l.N;
  v.b_zrows = l.N;
  v.A = A;
  v.B = B;
  v.sftA = at<int16_t>(ws, l.o_sftA);
  v.sftB = at<int16_t>(ws, l.o_sftB);
  v.pA = at<int8_t>(ws, l.o_pA);
  v.pB = at<int8_t>(ws, l.o_pB);
  v.res = at<int8_t>(ws, l.o_res);
  v.corr = at<int32_t>(ws, l.o_corr);
  v.C = out;
  return v;
}

// Rows [r0, r1) of a single product (B's planes shared by every chunk).
View row_chunk(const Plan& l, const View& f, int64_t r0, int64_t r1) {
  View v = f;
  v.M = r1 - r0;
  v.A = f.A + r0 * l.K;
  v.sftA = f.sftA + r0;
  v.pA = f.pA + (int64_t)l.G * r0 * l.Kp;
  v.res = f.res + (int64_t)l.P * r0 * l.ldn;
  v.corr = f.corr + (int64_t)ncorr_planes(l) * r0 * l.ldn;
  v.C = f.C + r0 * l.N;
  return v;
}

// Columns [c0, c1) of a row chunk r of a single product; `before` is the sum
// of the residue pitches of the chunk's earlier column blocks, so the blocks
// tile the chunk's residue share.
View col_block(const Plan& l, const View& r, int64_t c0, int64_t c1, int64_t before) {
  View v = r;
  v.N = c1 - c0;
  v.ldn = round_up(v.N, 16);
  v.B = r.B + (l.nt ? c0 : c0 * l.K);
  v.sftB = r.sftB + c0;
  v.pB = r.pB + c0 * l.Kp;
  v.res = r.res + (int64_t)l.P * r.M * before;
  v.corr = r.corr + (int64_t)ncorr_planes(l) * r.M * before;
  v.C = r.C + c0;
  return v;
}

// Members [b0, b1) of a batch (both operands per chunk).
View batch_chunk(const Plan& l, const View& f, int64_t b0, int64_t b1) {
  View v = f;
  v.batch = b1 - b0;
  v.A = f.A + b0 * l.M * l.K;
  v.B = f.B + b0 * l.N * l.K;
  v.sftA = f.sftA + b0 * l.M;
  v.sftB = f.sftB + b0 * l.N;
  v.pA = f.pA + (int64_t)l.G * b0 * l.M * l.Kp;
  v.pB = f.pB + (int64_t)l.G * b0 * l.N * l.Kp;
  v.res = f.res + (int64_t)l.P * b0 * l.M * l.ldn;
  v.corr = f.corr + (int64_t)ncorr_planes(l) * b0 * l.M * l.ldn;
  v.C = f.C + b0 * l.M * l.N;
  return v;
}

int64_t env_int(const char* name);

// [base + off, base + off + bytes) as a Span (debug bounds build).
Span span_of(const void* base, size_t off, size_t bytes) {
  Span sp;
  sp.lo = reinterpret_cast<uintptr_t>(base) + off;
  sp.hi = sp.lo + bytes;
  return sp;
}

ExtractArgs extract_args(const Plan& l, void* ws, int64_t k0, int64_t kw) {
  ExtractArgs ea{};
  ea.K = kw;
  ea.Kp = l.Kp;
  ea.ld = l.K;
  ea.koff = k0;
  ea.maxlg = at<WsHead>(ws, 0)->maxlg;
  ea.bits = l.bits;
  ea.use_corr = l.use_corr;
  ea.status = &at<WsHead>(ws, 0)->status;
  return ea;
}

// Extraction of one K window [k0, k0 + kw) of A (planes [residues, hi, q]).
ExtractArgs extract_A_args(const Plan& l, const View& v, void* ws, int64_t k0, int64_t kw) {
  ExtractArgs ea = extract_args(l, ws, k0, kw);
  ea.X = v.A;
  ea.rows = v.batch * v.M;
  ea.batch = v.batch;
  ea.N = v.N;
  ea.sft = v.sftA;
  ea.hi_plane = l.P;
  ea.q_plane = l.P + 1;
  ea.planes = v.pA;
  ea.pstride = ea.rows * l.Kp;
  ea.src = span_of(v.A, 0, sizeof(double) * (size_t)ea.rows * (size_t)ea.ld);
  ea.dst = span_of(ws, l.o_pA, (size_t)l.G * l.MF * l.Kp);
  return ea;
}

void extract_A(const Plan& l, const ModTables& T, const View& v, void* ws, int64_t k0, int64_t kw, cudaStream_t s) {
  launch_extract_rows(extract_A_args(l, v, ws, k0, kw), T, s);
}

// Extraction of one K window of B (planes [residues, q, hi]).
ExtractArgs extract_B_args(const Plan& l, const View& v, void* ws, int64_t k0, int64_t kw) {
  ExtractArgs eb = extract_args(l, ws, k0, kw);
  eb.X = v.B;
  eb.rows = v.batch * v.N;
  eb.batch = v.batch;
  eb.N = v.N;
  if (l.nt) eb.ld = l.N;   // [K][N]: row pitch of the whole operand
  eb.sft = v.sftB;
  eb.q_plane = l.P;
  eb.hi_plane = l.P + 1;
  eb.planes = v.pB;
  eb.pstride = v.batch * v.b_zrows * l.Kp;
  // [K][N] layout: member b's element (k, n) at X[(b K + k) ld + n]; [N][K]: rows of pitch ld
  const size_t nel = l.nt ? (size_t)((v.batch * eb.K - 1) * eb.ld + v.N) : (size_t)eb.rows * (size_t)eb.ld;
  eb.src = span_of(v.B, 0, (v.batch > 0 && v.N > 0 && eb.K > 0) ? sizeof(double) * nel : 0);
  eb.dst = span_of(ws, l.o_pB, (size_t)l.G * l.NF * l.Kp);
  return eb;
}

void extract_B(const Plan& l, const ModTables& T, const View& v, void* ws, int64_t k0, int64_t kw, cudaStream_t s) {
  const ExtractArgs eb = extract_B_args(l, v, ws, k0, kw);
  if (l.nt) launch_extract_cols(eb, T, s);
  else launch_extract_rows(eb, T, s);
}

// Both operands of a view; one launch for both operands of a small product
// (where launch latency, not the extraction, dominates).
void extract_AB(const Plan& l, const ModTables& T, const View& v, void* ws, int64_t k0, int64_t kw, cudaStream_t s) {
  constexpr int64_t kPairMaxElems = int64_t(1) << 22;
  if ((v.batch * v.M + v.batch * v.N) * kw <= kPairMaxElems) {
    if (l.nt) launch_extract_nt_pair(extract_A_args(l, v, ws, k0, kw), extract_B_args(l, v, ws, k0, kw), T, s);
    else launch_extract_rows_pair(extract_A_args(l, v, ws, k0, kw), extract_B_args(l, v, ws, k0, kw), T, s);
    return;
  }
  extract_A(l, T, v, ws, k0, kw, s);
  extract_B(l, T, v, ws, k0, kw, s);
}

GemmArgs gemm_args(const Plan& l, const View& v, void* ws) {
  GemmArgs g{};
  g.M = (int)v.M;
  g.N = (int)v.N;
  g.batch = (int)v.batch;
  g.P = l.P;
  g.Kp = (int)l.Kp;
  g.nkb = (int)((l.Kp + 127) / 128);
  g.corr_mode = l.gemm_corr;
  g.ldn = (int)v.ldn;
  g.res = v.res;
  g.corr = v.corr;
  g.status = &at<WsHead>(ws, 0)->status;
  g.wait_limit_ns = g_wait_limit.load();
  g.res_span = span_of(ws, l.o_res, (size_t)l.P * l.MF * l.ldn);
  g.corr_span = span_of(ws, l.o_corr, sizeof(int32_t) * ncorr_planes(l) * l.MF * l.ldn);
  return g;
}

// Tensor maps of one view's planes for the kernel gemm_use_pair picks.
int gemm_maps(const Plan& l, const View& v, CUtensorMap* tA, CUtensorMap* tB) {
  const bool pair = gemm_use_pair((int)v.M) && !gemm_force_single();
  const int rows_a = pair ? gemm_pair_block_rows() : gemm_block_rows_a();
  const int rows_b = pair ? gemm_pair_block_rows() : gemm_block_rows_b();
  if (!encode_plane_map(tA, v.pA, (int64_t)l.G * v.batch, v.M, l.Kp, rows_a) ||
      !encode_plane_map(tB, v.pB, (int64_t)l.G * v.batch, v.N, l.Kp, rows_b, v.b_zrows))
    return fail(F64E_ERR_CUDA, "cuTensorMapEncodeTiled rejected the plane layout");
  return F64E_OK;
}

int launch_gemm_view(const Plan& l, const ModTables& T, const View& v, const CUtensorMap& tA, const CUtensorMap& tB,
                     void* ws, const Dev& d, cudaStream_t s) {
  const GemmArgs g = gemm_args(l, v, ws);
  const bool pair = gemm_use_pair(g.M) && !gemm_force_single();
  cudaError_t e = pair ? launch_residue_gemm_pair(tA, tB, g, T, d.sms, s) : launch_residue_gemm(tA, tB, g, T, d.sms, s);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "modular GEMM launch");
  return F64E_OK;
}

int run_gemm(const Plan& l, const ModTables& T, const View& v, void* ws, const Dev& d, bool checked, cudaStream_t s) {
  if (checked) {
    const GemmArgs g = gemm_args(l, v, ws);
    launch_residue_gemm_check(v.pA, v.pB, v.batch * v.M, v.batch * v.N, g, T, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "modular GEMM launch");
    return F64E_OK;
  }
  CUtensorMap tA, tB;
  const int rc = gemm_maps(l, v, &tA, &tB);
  if (rc) return rc;
  return launch_gemm_view(l, T, v, tA, tB, ws, d, s);
}

void run_reconstruct(const Plan& l, const ModTables& T, const View& v, void* ws, int corr_mode, const void* corr,
                     cudaStream_t s, bool beside_gemm = false, int sms = 0) {
  ReconArgs r{};
  r.res = v.res;
  r.corr_mode = corr_mode;
  r.corr = corr;
  r.MF = v.batch * v.M;
  r.M = v.M;
  r.N = v.N;
  r.ldn = v.ldn;
  r.sftA = v.sftA;
  r.sftB = v.sftB;
  r.maxlg = at<WsHead>(ws, 0)->maxlg;
  r.bits = l.bits;
  r.exact = l.exact;
  r.C = v.C;
  r.ldc = v.ldc;
  r.status = &at<WsHead>(ws, 0)->status;
  r.res_span = span_of(ws, l.o_res, (size_t)l.P * l.MF * l.ldn);
  r.corr_span = corr_mode == 3 ? span_of(ws, l.o_cacc, sizeof(int64_t) * l.MF * l.ldn)
                               : span_of(ws, l.o_corr, sizeof(int32_t) * ncorr_planes(l) * l.MF * l.ldn);
  r.out_span = span_of(v.C, 0, r.MF > 0 ? sizeof(double) * (size_t)((r.MF - 1) * v.ldc + v.N) : 0);
#ifdef F64E_DEBUG_BOUNDS
  // Self-test hook of the checking build: F64E_DEBUG_SHRINK_OUT_BYTES=n moves
  // the end of the output range n bytes in, so the writes of the last
  // elements are reported (site 20) and skipped.  Those elements lie inside
  // the caller's output, so no access leaves the real buffers either way.
  const int64_t shrink = env_int("F64E_DEBUG_SHRINK_OUT_BYTES");
  if (shrink > 0) r.out_span.hi -= std::min<uintptr_t>((uintptr_t)shrink, r.out_span.hi - r.out_span.lo);
#endif
  launch_reconstruct(r, T, s, beside_gemm, sms);
}

// Device-to-host copy of one view's block of C (rows of pitch ldc) to the
// same place in a host array shaped like C.
cudaError_t copy_out(const View& v, const View& f, double* host, cudaStream_t s) {
  double* dst = host + (v.C - f.C);
  return cudaMemcpy2DAsync(dst, sizeof(double) * v.ldc, v.C, sizeof(double) * v.ldc, sizeof(double) * v.N,
                           (size_t)(v.batch * v.M), cudaMemcpyDeviceToHost, s);
}

// ------------------------------------------------------------ pipelining --
// A product whose three compute phases run in one call is cut into chunks.
// A single product is cut into row blocks, and its first row block again
// into column blocks, so the first GEMM needs only a slice of each operand
// extracted: the extraction exposed before the pipeline fills is one row
// block of A and one column block of B.  A batch is cut into member blocks.
// GEMM chunks run on two high-priority library streams in turn (chunk c + 1
// takes each SM as soon as chunk c's CTA there exits), the extraction of
// later chunks on a low-priority library stream and the reconstruction of
// earlier ones on the caller's stream: the persistent GEMM holds one CTA per
// SM and leaves registers and shared memory for one block of either kernel
// beside it.  Results are the same bits as the unchunked product: every
// element's arithmetic is independent of the chunking and the sizing covers
// the whole product.
constexpr int kPipeMaxChunks = 16;
constexpr int kPipeMaxCols = 4;
constexpr int kPipeEvents = 4 * (kPipeMaxChunks + kPipeMaxCols) + 8;

struct PipeRes {
  cudaStream_t hi[2] = {nullptr, nullptr}, aux = nullptr, cp = nullptr;   // cp: device-to-host copies
  cudaEvent_t ev[kPipeEvents] = {};
  std::mutex mtx;
};

// Per-device streams and events, created on first use and kept for the
// process.  Returns nullptr (and the product runs unchunked) while the
// caller's stream is being captured and they do not exist yet.
PipeRes* pipe_res(int dev, cudaStream_t s, int* rc) {
  static std::mutex mtx;
  static std::map<int, PipeRes*> all;
  *rc = F64E_OK;
  std::lock_guard<std::mutex> lk(mtx);
  auto it = all.find(dev);
  if (it != all.end()) return it->second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
  int lo = 0, hi = 0;
  cudaError_t e = cudaDeviceGetStreamPriorityRange(&lo, &hi);
  PipeRes* r = new PipeRes;
  for (int i = 0; i < 2 && e == cudaSuccess; i++) e = cudaStreamCreateWithPriority(&r->hi[i], cudaStreamNonBlocking, hi);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&r->aux, cudaStreamNonBlocking, lo);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&r->cp, cudaStreamNonBlocking, lo);
  for (int i = 0; i < kPipeEvents && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&r->ev[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    *rc = cuda_fail(e, "pipeline streams");
    return nullptr;
  }
  all.emplace(dev, r);
  return r;
}

// F64E_PIPE_CHUNK=<n> sets the chunk extent (rows of a single product,
// members of a batch) and F64E_PIPE_CHUNK=0 turns chunking off;
// F64E_PIPE_COLS=<n> sets the column block of the first row block (0: none).
// Read per call (A/B checks of the chunked path against the unchunked one).
int64_t env_int(const char* name) {
  const char* v = std::getenv(name);
  if (!v || !*v) return -1;
  return std::max<int64_t>(0, std::atoll(v));
}

struct Chunking {
  bool by_batch = false;
  int64_t per = 0;    // rows (or members) per chunk; 0 = unchunked
  int64_t cols = 0;   // columns per block of the first row chunk; 0 = whole
  int head = 1;       // row chunks of A extracted before the first GEMM (single products)
  std::vector<int64_t> bounds;   // chunk boundaries 0 = b_0 < b_1 < ... < b_C = extent
};

Chunking pipe_chunking(const Plan& l) {
  Chunking c;
  c.by_batch = l.batch > 1;
  const int64_t extent = c.by_batch ? l.batch : l.M;
  const int64_t ov = env_int("F64E_PIPE_CHUNK");
  if (ov >= 0) {
    c.per = ov;
  } else if (c.by_batch) {
    // member blocks of 2048 or more rows in all, eight chunks at most
    if (l.MF >= 2048 && l.batch >= 4) c.per = (l.batch + 7) / 8;
  } else if (l.M >= 2048) {
    // row chunks of about 2048 rows (at least two, eight at most): shorter
    // chunks leave the extraction of the next one less GEMM time to hide in
    const int64_t n = std::min<int64_t>(8, std::max<int64_t>(2, l.M / 2048));
    c.per = round_up((l.M + n - 1) / n, 256);
  }
  if (c.per <= 0 || c.per >= extent) {
    c.per = 0;
    return c;
  }
  if ((extent + c.per - 1) / c.per > kPipeMaxChunks) c.per = (extent + kPipeMaxChunks - 1) / kPipeMaxChunks;
  if (!c.by_batch) {
    // Column blocks of the first row chunk shorten the exposed extraction,
    // but their GEMMs are too short to hide the next block's extraction on
    // B200 (measured: net loss at 8192^3), so they stay off unless asked for.
    const int64_t cv = env_int("F64E_PIPE_COLS");
    if (cv >= 0) c.cols = cv;
    if (c.cols > 0) c.cols = std::max<int64_t>(c.cols, (l.N + kPipeMaxCols - 1) / kPipeMaxCols);
    if (c.cols > 0) c.cols = round_up(c.cols, 16);
    if (c.cols >= l.N) c.cols = 0;
  }
  // Row chunks of A extracted in the head: F64E_PIPE_HEAD = n (0: all of A).
  if (!c.by_batch) {
    const int64_t hv = env_int("F64E_PIPE_HEAD");
    if (hv >= 0) c.head = hv == 0 ? kPipeMaxChunks : (int)std::min<int64_t>(hv, kPipeMaxChunks);
  }
  // Boundaries.  Single products of at least three chunks start and end with
  // half-size chunks (the first one's extraction and the last one's
  // reconstruction are the parts no GEMM runs beside); F64E_PIPE_ENDS=0 keeps
  // every chunk the same size.
  c.bounds.assign(1, 0);
  const int64_t ends = env_int("F64E_PIPE_ENDS");
  const int64_t half = round_up((c.per + 1) / 2, 256);
  if (!c.by_batch && ends != 0 && c.per >= 1024 && extent >= 3 * c.per) {
    int64_t at = half;
    c.bounds.push_back(at);
    while (extent - at > c.per + half) {
      at += c.per;
      c.bounds.push_back(at);
    }
    if (extent - at > half) c.bounds.push_back(extent - half);
    c.bounds.push_back(extent);
  } else {
    for (int64_t at = c.per; at < extent; at += c.per) c.bounds.push_back(at);
    c.bounds.push_back(extent);
  }
  if ((int64_t)c.bounds.size() - 1 > kPipeMaxChunks) {   // fall back to equal chunks within the limit
    const int64_t per = (extent + kPipeMaxChunks - 1) / kPipeMaxChunks;
    c.bounds.assign(1, 0);
    for (int64_t at = per; at < extent; at += per) c.bounds.push_back(at);
    c.bounds.push_back(extent);
  }
  return c;
}

int run_pipelined(const Plan& l, const ModTables& T, const View& f, void* ws, const Dev& d, PipeRes* pr,
                  const Chunking& ch, cudaStream_t s, void* const* gev, int ngev, int* launches, double* out_host) {
  const int C = (int)ch.bounds.size() - 1;
  // GEMM units in launch order: the column blocks of row chunk 0, then row chunks 1.. (or member chunks).
  std::vector<View> rows(C), units;
  for (int c = 0; c < C; c++) {
    const int64_t a0 = ch.bounds[c], a1 = ch.bounds[c + 1];
    rows[c] = ch.by_batch ? batch_chunk(l, f, a0, a1) : row_chunk(l, f, a0, a1);
  }
  const int J = ch.cols > 0 ? (int)((l.N + ch.cols - 1) / ch.cols) : 1;
  std::vector<View> bcols(J, f);   // B column blocks (their extraction views)
  if (J > 1) {
    int64_t before = 0;
    for (int j = 0; j < J; j++) {
      const int64_t c0 = j * ch.cols, c1 = std::min(l.N, c0 + ch.cols);
      units.push_back(col_block(l, rows[0], c0, c1, before));
      bcols[j] = units.back();
      before += round_up(c1 - c0, 16);
    }
  } else {
    units.push_back(rows[0]);
  }
  for (int c = 1; c < C; c++) units.push_back(rows[c]);
  const int U = (int)units.size();
  std::vector<CUtensorMap> tA(U), tB(U);
  for (int u = 0; u < U; u++) {
    const int rc = gemm_maps(l, units[u], &tA[u], &tB[u]);   // all host-side failures before the first launch
    if (rc) return rc;
  }
  // need[u]: index of the extraction event GEMM unit u waits for (-1: extracted before the fork)
  std::vector<int> need(U, -1);
  std::lock_guard<std::mutex> lk(pr->mtx);
  cudaEvent_t* E = pr->ev;
  int ne = 1;   // E[0] = fork
  // Head, on the caller's stream: everything the first GEMM unit reads (and
  // the first H row chunks of A).
  const int H = (ch.by_batch || J > 1) ? 1 : std::max(1, std::min(C, ch.head));
  for (int c = 0; c < H; c++) extract_A(l, T, rows[c], ws, 0, l.K, s);
  if (ch.by_batch) extract_B(l, T, rows[0], ws, 0, l.K, s);
  else extract_B(l, T, J > 1 ? bcols[0] : f, ws, 0, l.K, s);
  cudaError_t e = cudaEventRecord(E[0], s);
  for (int i = 0; i < 2 && e == cudaSuccess; i++) e = cudaStreamWaitEvent(pr->hi[i], E[0], 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pr->aux, E[0], 0);
  if (e != cudaSuccess) return cuda_fail(e, "pipeline fork");
  // The rest of the extraction, in the order the GEMM units need it.
  for (int j = 1; j < J; j++) {
    extract_B(l, T, bcols[j], ws, 0, l.K, pr->aux);
    cudaEventRecord(E[ne], pr->aux);
    need[j] = ne++;
  }
  for (int c = H; c < C; c++) {
    extract_A(l, T, rows[c], ws, 0, l.K, pr->aux);
    if (ch.by_batch) extract_B(l, T, rows[c], ws, 0, l.K, pr->aux);
    cudaEventRecord(E[ne], pr->aux);
    need[(J > 1 ? J : 1) + c - 1] = ne++;
  }
  const int e_aux = ne++;
  cudaEventRecord(E[e_aux], pr->aux);
  int rc = F64E_OK;
  // F64E_PIPE_GEMM_STREAMS=1: every GEMM chunk on one stream, so no two GEMM
  // launches are ever resident at once (A/B checks).
  const bool one_gemm_stream = env_int("F64E_PIPE_GEMM_STREAMS") == 1;
  const int e_gemm = ne;
  for (int u = 0; u < U; u++) {
    cudaStream_t h = pr->hi[one_gemm_stream ? 0 : (u & 1)];
    if (need[u] >= 0) cudaStreamWaitEvent(h, E[need[u]], 0);
    if (2 * u + 1 < ngev) cudaEventRecord(static_cast<cudaEvent_t>(gev[2 * u]), h);
    if (rc == F64E_OK) rc = launch_gemm_view(l, T, units[u], tA[u], tB[u], ws, d, h);
    if (2 * u + 1 < ngev) cudaEventRecord(static_cast<cudaEvent_t>(gev[2 * u + 1]), h);
    cudaEventRecord(E[e_gemm + u], h);
  }
  const int e_done = e_gemm + U;
  cudaError_t ec = cudaSuccess;
  for (int u = 0; u < U; u++) {
    cudaStreamWaitEvent(s, E[e_gemm + u], 0);   // joins both GEMM streams
    // row chunks of a single product: every reconstruction but the last runs beside a GEMM chunk
    run_reconstruct(l, T, units[u], ws, l.recon_corr, units[u].corr, s, !ch.by_batch && u + 1 < U, d.sms);
    if (out_host) {   // this block's copy to the host overlaps the later blocks' work
      cudaEventRecord(E[e_done + u], s);
      cudaStreamWaitEvent(pr->cp, E[e_done + u], 0);
      if (ec == cudaSuccess) ec = copy_out(units[u], f, out_host, pr->cp);
    }
  }
  if (out_host) {
    cudaEventRecord(E[e_done + U], pr->cp);
    cudaStreamWaitEvent(s, E[e_done + U], 0);   // joins the copy stream
  }
  e = cudaStreamWaitEvent(s, E[e_aux], 0);      // joins the extraction stream
  if (e == cudaSuccess) e = ec;
  if (launches) *launches = U;
  if (rc) return rc;
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "pipelined launch");
  return F64E_OK;
}

int run(const f64e_problem* p, const double* A, const double* B, double* out, void* ws, size_t ws_bytes,
        void* stream, int phases, bool checked, cudaEvent_t* ev, void* const* gev = nullptr, int ngev = 0,
        int* launches = nullptr, double* out_host = nullptr) {
  if (launches) *launches = 0;
  Plan l;
  int rc = make_plan(p, &l);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (l.MF == 0 || l.NF == 0) return F64E_OK;
  if (!out) return fail(F64E_ERR_ARGUMENT, "null output pointer");
  if (l.K == 0) {   // empty inner dimension: C = 0 (the operands hold no elements, their pointers may be null)
    if (phases & F64E_PHASE_COMPUTE) {
      cudaError_t e = cudaMemsetAsync(out, 0, sizeof(double) * l.MF * l.N, s);
      if (e == cudaSuccess && out_host)
        e = cudaMemcpyAsync(out_host, out, sizeof(double) * l.MF * l.N, cudaMemcpyDeviceToHost, s);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
    return F64E_OK;
  }
  if (!A || !B) return fail(F64E_ERR_ARGUMENT, "null operand pointer");
  if (!ws || ws_bytes < l.total) return fail(F64E_ERR_WORKSPACE, "workspace of %zu bytes is below the %zu needed",
                                             ws_bytes, l.total);
  if (reinterpret_cast<uintptr_t>(ws) & 255) return fail(F64E_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  Dev d;
  rc = device_info(&d);
  if (rc) return rc;
  ModTables T;
  rc = get_tables(p->primes, p->nprimes, &T);
  if (rc) return rc;

  if (ev) cudaEventRecord(ev[0], s);
  if (phases & F64E_PHASE_SIZING) {
    rc = run_sizing(l, A, B, ws, s);
    if (rc) return rc;
  }
  if (!(phases & F64E_PHASE_COMPUTE)) return F64E_OK;
  const View f = full_view(l, A, B, ws, out);
  if (!ev && !checked && !l.deep && (phases & F64E_PHASE_COMPUTE) == F64E_PHASE_COMPUTE) {
    const Chunking ch = pipe_chunking(l);
    if (ch.per > 0) {
      PipeRes* pr = pipe_res(d.dev, s, &rc);
      if (rc) return rc;
      if (pr) return run_pipelined(l, T, f, ws, d, pr, ch, s, gev, ngev, launches, out_host);
    }
  }
  if (!l.deep) {
    if (phases & F64E_PHASE_EXTRACT) extract_AB(l, T, f, ws, 0, l.K, s);
    if (ev) cudaEventRecord(ev[1], s);
    if (phases & F64E_PHASE_GEMM) {
      if (ngev >= 2) cudaEventRecord(static_cast<cudaEvent_t>(gev[0]), s);
      rc = run_gemm(l, T, f, ws, d, checked, s);
      if (rc) return rc;
      if (ngev >= 2) cudaEventRecord(static_cast<cudaEvent_t>(gev[1]), s);
      if (launches) *launches = 1;
    }
  } else if (phases & (F64E_PHASE_EXTRACT | F64E_PHASE_GEMM)) {
    if ((phases & (F64E_PHASE_EXTRACT | F64E_PHASE_GEMM)) != (F64E_PHASE_EXTRACT | F64E_PHASE_GEMM))
      return fail(F64E_ERR_ARGUMENT, "deep-K products run EXTRACT and GEMM together");
    const int64_t nres = (int64_t)l.P * l.MF * l.ldn, ncorr = l.use_corr ? l.MF * l.ldn : 0;
    for (int sgi = 0; sgi < l.nseg; sgi++) {
      const int64_t k0 = (int64_t)sgi * l.Kseg, kw = std::min(l.Kseg, l.K - k0);
      extract_A(l, T, f, ws, k0, kw, s);
      extract_B(l, T, f, ws, k0, kw, s);
      if (2 * sgi + 1 < ngev) cudaEventRecord(static_cast<cudaEvent_t>(gev[2 * sgi]), s);
      rc = run_gemm(l, T, f, ws, d, checked, s);
      if (rc) return rc;
      if (2 * sgi + 1 < ngev) cudaEventRecord(static_cast<cudaEvent_t>(gev[2 * sgi + 1]), s);
      launch_deepk_accum(at<int8_t>(ws, l.o_res), at<int32_t>(ws, l.o_racc), nres, at<int32_t>(ws, l.o_corr),
                         at<int64_t>(ws, l.o_cacc), ncorr, sgi == 0, s);
    }
    if (launches) *launches = l.nseg;
    launch_deepk_fold(at<int32_t>(ws, l.o_racc), at<int8_t>(ws, l.o_res), l.MF * l.ldn, T, s);
    if (ev) cudaEventRecord(ev[1], s);
  }
  if (ev) {
    cudaEventRecord(ev[2], s);
    cudaEventRecord(ev[3], s);
  }
  if (phases & F64E_PHASE_RECON) {
    const void* corr = l.recon_corr == 3 ? (const void*)at<int64_t>(ws, l.o_cacc) : (const void*)f.corr;
    run_reconstruct(l, T, f, ws, l.recon_corr, corr, s);
  }
  if (ev) cudaEventRecord(ev[4], s);
  if (out_host && (phases & F64E_PHASE_RECON)) {
    const cudaError_t e = copy_out(f, f, out_host, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return F64E_OK;
}

f64e_problem make_problem(int64_t batch, int64_t M, int64_t N, int64_t K, int32_t layout, const int32_t* primes,
                          int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr) {
  f64e_problem p;
  p.batch = batch;
  p.M = M;
  p.N = N;
  p.K = K;
  p.b_layout = layout;
  p.nprimes = nprimes;
  p.primes = primes;
  p.exact = exact;
  p.bits = (bits < INT32_MIN || bits > INT32_MAX) ? 0 : (int32_t)bits;
  p.use_corr = use_corr;
  p.slab_cols = 0;
  return p;
}

int check_batch(int64_t batch, int32_t nprimes, int32_t use_corr) {
  const int64_t NP = (int64_t)nprimes + (use_corr ? 2 : 0);
  if (nprimes <= kMaxP && NP * batch > 65535)
    return fail(F64E_ERR_ARGUMENT, "(nprimes + 2) * batch exceeds the launch z-extent");
  return F64E_OK;
}

}  // namespace

namespace f64e {

// Internal entry for other translation units of the library (the
// allocation-free entry point): the generic product on a given workspace.
int run_problem(const f64e_problem* p, const double* A, const double* B, double* out, void* ws, size_t ws_bytes,
                void* stream, int phases) {
  g_err.clear();
  return run(p, A, B, out, ws, ws_bytes, stream, phases, false, nullptr);
}

int report_error(int code, const char* msg) { return fail(code, "%s", msg); }

}  // namespace f64e

extern "C" {

int64_t f64e_maxp(void) { return kMaxP; }

size_t f64e_workspace_size(const f64e_problem* p) {
  Plan l;
  if (make_plan(p, &l)) return 0;
  return l.total;
}

int f64e_gemm(const f64e_problem* p, const double* A, const double* B, double* out, void* ws, size_t ws_bytes,
              void* stream, int phases) {
  g_err.clear();
  return run(p, A, B, out, ws, ws_bytes, stream, phases, false, nullptr);
}

int f64e_gemm_ev(const f64e_problem* p, const double* A, const double* B, double* out, void* ws, size_t ws_bytes,
                 void* stream, int phases, void* const* events, int32_t n_events, int32_t* launches) {
  g_err.clear();
  if (n_events > 0 && !events) return fail(F64E_ERR_ARGUMENT, "null event array");
  int nl = 0;
  const int rc = run(p, A, B, out, ws, ws_bytes, stream, phases, false, nullptr, events, std::max(0, n_events), &nl);
  if (launches) *launches = nl;
  return rc;
}

int f64e_gemm_host(const f64e_problem* p, const double* A_host, const double* B_host, double* out_host,
                   double* A_dev, double* B_dev, double* out_dev, void* ws, size_t ws_bytes, void* stream) {
  g_err.clear();
  Plan l;
  int rc = make_plan(p, &l);
  if (rc) return rc;
  if (l.MF == 0 || l.NF == 0) return F64E_OK;
  if (!A_host || !B_host || !out_host || !A_dev || !B_dev || !out_dev)
    return fail(F64E_ERR_ARGUMENT, "null operand pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(A_dev, A_host, sizeof(double) * l.MF * l.K, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(B_dev, B_host, sizeof(double) * l.NF * l.K, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync");
  return run(p, A_dev, B_dev, out_dev, ws, ws_bytes, stream, F64E_PHASE_ALL, false, nullptr, nullptr, 0, nullptr,
             out_host);
}

int f64e_gemm_checked(const f64e_problem* p, const double* A, const double* B, double* out, void* ws,
                      size_t ws_bytes, void* stream) {
  g_err.clear();
  return run(p, A, B, out, ws, ws_bytes, stream, F64E_PHASE_ALL, true, nullptr);
}

int f64e_mm(double* out, const double* A, const double* B, int64_t M, int64_t N, int64_t K, const int32_t* primes,
            int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr, void* ws, size_t ws_bytes,
            void* stream) {
  g_err.clear();
  const f64e_problem p = make_problem(1, M, N, K, F64E_B_NK, primes, nprimes, exact, bits, use_corr);
  return run(&p, A, B, out, ws, ws_bytes, stream, F64E_PHASE_ALL, false, nullptr);
}

int f64e_mm_nt(double* out, const double* A, const double* Bt, int64_t M, int64_t N, int64_t K,
               const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr, void* ws,
               size_t ws_bytes, void* stream) {
  g_err.clear();
  const f64e_problem p = make_problem(1, M, N, K, F64E_B_KN, primes, nprimes, exact, bits, use_corr);
  return run(&p, A, Bt, out, ws, ws_bytes, stream, F64E_PHASE_ALL, false, nullptr);
}

int f64e_bmm(double* out, const double* A, const double* B, int64_t batch, int64_t M, int64_t N, int64_t K,
             const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr, void* ws,
             size_t ws_bytes, void* stream) {
  g_err.clear();
  int rc = check_batch(batch, nprimes, use_corr);
  if (rc) return rc;
  const f64e_problem p = make_problem(batch, M, N, K, F64E_B_NK, primes, nprimes, exact, bits, use_corr);
  return run(&p, A, B, out, ws, ws_bytes, stream, F64E_PHASE_ALL, false, nullptr);
}

int f64e_bmm_nt(double* out, const double* A, const double* Bt, int64_t batch, int64_t M, int64_t N, int64_t K,
                const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr, void* ws,
                size_t ws_bytes, void* stream) {
  g_err.clear();
  int rc = check_batch(batch, nprimes, use_corr);
  if (rc) return rc;
  const f64e_problem p = make_problem(batch, M, N, K, F64E_B_KN, primes, nprimes, exact, bits, use_corr);
  return run(&p, A, Bt, out, ws, ws_bytes, stream, F64E_PHASE_ALL, false, nullptr);
}

int f64e_mm_timed(double* out, float* times, const double* A, const double* B, int64_t M, int64_t N, int64_t K,
                  const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr, void* ws,
                  size_t ws_bytes, void* stream) {
  g_err.clear();
  if (K > kNtMaxK) return fail(F64E_ERR_ARGUMENT, "K bound for int32 modular GEMM");
  if (!times) return fail(F64E_ERR_ARGUMENT, "times must be a host float[4]");
  const f64e_problem p = make_problem(1, M, N, K, F64E_B_NK, primes, nprimes, exact, bits, use_corr);
  cudaEvent_t ev[5];
  for (int i = 0; i < 5; i++) {
    const cudaError_t e = cudaEventCreate(&ev[i]);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; j++) cudaEventDestroy(ev[j]);
      return cuda_fail(e, "cudaEventCreate");
    }
  }
  int rc = run(&p, A, B, out, ws, ws_bytes, stream, F64E_PHASE_ALL, false, ev);
  if (rc == F64E_OK) {
    if (M * N == 0 || K == 0) {
      for (int i = 0; i < 4; i++) times[i] = 0.0f;
    } else {
      const cudaError_t e = cudaEventSynchronize(ev[4]);
      if (e != cudaSuccess) rc = cuda_fail(e, "cudaEventSynchronize");
      for (int i = 0; i < 4 && rc == F64E_OK; i++) cudaEventElapsedTime(&times[i], ev[i], ev[i + 1]);
    }
  }
  for (int i = 0; i < 5; i++) cudaEventDestroy(ev[i]);
  return rc;
}

int f64e_status(const void* ws, void* stream, int32_t* status) {
  g_err.clear();
  if (!ws || !status) return fail(F64E_ERR_ARGUMENT, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WsHead* head = static_cast<const WsHead*>(ws);
  cudaError_t e = cudaMemcpyAsync(status, &head->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  return F64E_OK;
}

void f64e_set_wait_limit_ns(uint64_t ns) { g_wait_limit.store(ns ? ns : 1); }

int f64e_wait_selftest(void* ws, size_t ws_bytes, uint64_t limit_ns, void* stream, int32_t* status) {
  g_err.clear();
  if (!ws || !status || ws_bytes < sizeof(WsHead)) return fail(F64E_ERR_ARGUMENT, "workspace of a WsHead at least");
  if (limit_ns == 0 || limit_ns > 10000000000ULL) return fail(F64E_ERR_ARGUMENT, "limit must be in (0, 10 s]");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  WsHead* head = static_cast<WsHead*>(ws);
  cudaError_t e = cudaMemsetAsync(&head->status, 0, sizeof(int32_t), s);
  if (e == cudaSuccess) e = launch_wait_selftest(&head->status, limit_ns, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(status, &head->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "wait self-test");
  return F64E_OK;
}

const char* f64e_last_error(void) { return g_err.c_str(); }

int f64e_debug_fetch(const f64e_problem* p, const void* ws, int which, void* host, size_t cap, size_t* nbytes,
                     void* stream) {
  g_err.clear();
  Plan l;
  int rc = make_plan(p, &l);
  if (rc) return rc;
  size_t off = 0, n = 0;
  const int ncorr = l.gemm_corr == 2 ? 2 : (l.gemm_corr == 1 ? 1 : 0);
  switch (which) {
    case 0: off = l.o_pA; n = (size_t)l.G * l.MF * l.Kp; break;
    case 1: off = l.o_pB; n = (size_t)l.G * l.NF * l.Kp; break;
    case 2: off = l.o_res; n = (size_t)l.P * l.MF * l.ldn; break;
    case 3: off = l.o_corr; n = sizeof(int32_t) * ncorr * l.MF * l.ldn; break;
    case 4: off = l.o_sftA; n = sizeof(int16_t) * l.MF; break;
    case 5: off = l.o_sftB; n = sizeof(int16_t) * l.NF; break;
    case 6: off = 0; n = 2 * sizeof(float); break;
    default: return fail(F64E_ERR_ARGUMENT, "unknown buffer %d", which);
  }
  n = std::min(n, cap);
  if (nbytes) *nbytes = n;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(host, static_cast<const char*>(ws) + off, n, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "debug fetch");
  return F64E_OK;
}

}  // extern "C"
