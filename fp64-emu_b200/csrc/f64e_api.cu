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
    T.hh[t] = (uint32_t)(p / 2);
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
  if (!l.use_corr) l.gemm_corr = 0;
  else l.gemm_corr = (l.Kseg <= kFusedCorrMaxK) ? 1 : 2;
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
  cudaError_t e = cudaMemsetAsync(&head->status, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  launch_row_stats(A, l.MF, l.K, l.bits, at<int16_t>(ws, l.o_sftA), at<float>(ws, l.o_lgA), s);
  if (l.nt)
    launch_col_stats(B, l.batch, l.K, l.N, l.kslab, l.nslab, l.bits, at<int16_t>(ws, l.o_sftB),
                     at<float>(ws, l.o_lgB), at<double>(ws, l.o_pmax), at<double>(ws, l.o_pss), s);
  else
    launch_row_stats(B, l.NF, l.K, l.bits, at<int16_t>(ws, l.o_sftB), at<float>(ws, l.o_lgB), s);
  launch_maxlg(at<float>(ws, l.o_lgA), l.MF, at<float>(ws, l.o_lgB), l.NF, head->maxlg, s);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sizing launch");
  return F64E_OK;
}

// Extraction of one K window [k0, k0 + kw) of both operands.
void run_extract(const Plan& l, const ModTables& T, const double* A, const double* B, void* ws, int64_t k0,
                 int64_t kw, cudaStream_t s) {
  WsHead* head = at<WsHead>(ws, 0);
  ExtractArgs ea{};
  ea.X = A;
  ea.rows = l.MF;
  ea.K = kw;
  ea.Kp = l.Kp;
  ea.ld = l.K;
  ea.koff = k0;
  ea.batch = l.batch;
  ea.N = l.N;
  ea.sft = at<int16_t>(ws, l.o_sftA);
  ea.maxlg = head->maxlg;
  ea.bits = l.bits;
  ea.use_corr = l.use_corr;
  ea.hi_plane = l.P;      // A planes: [residues, hi, q]
  ea.q_plane = l.P + 1;
  ea.planes = at<int8_t>(ws, l.o_pA);
  launch_extract_rows(ea, T, s);
  ExtractArgs eb = ea;
  eb.X = B;
  eb.rows = l.NF;
  eb.sft = at<int16_t>(ws, l.o_sftB);
  eb.q_plane = l.P;       // B planes: [residues, q, hi]
  eb.hi_plane = l.P + 1;
  eb.planes = at<int8_t>(ws, l.o_pB);
  if (l.nt) launch_extract_cols(eb, T, s);
  else launch_extract_rows(eb, T, s);
}

GemmArgs gemm_args(const Plan& l, void* ws) {
  GemmArgs g{};
  g.M = (int)l.M;
  g.N = (int)l.N;
  g.batch = (int)l.batch;
  g.P = l.P;
  g.Kp = (int)l.Kp;
  g.nkb = (int)((l.Kp + 127) / 128);
  g.corr_mode = l.gemm_corr;
  g.ldn = (int)l.ldn;
  g.res = at<int8_t>(ws, l.o_res);
  g.corr = at<int32_t>(ws, l.o_corr);
  g.status = &at<WsHead>(ws, 0)->status;
  g.wait_limit_ns = g_wait_limit.load();
  return g;
}

int run_gemm(const Plan& l, const ModTables& T, void* ws, const Dev& d, bool checked, cudaStream_t s) {
  const GemmArgs g = gemm_args(l, ws);
  if (checked) {
    launch_residue_gemm_check(at<int8_t>(ws, l.o_pA), at<int8_t>(ws, l.o_pB), l.MF, l.NF, g, T, s);
  } else {
    CUtensorMap tA, tB;
    const bool pair = gemm_use_pair(g.M) && !gemm_force_single();
    const int rows_a = pair ? gemm_pair_block_rows() : gemm_block_rows_a();
    const int rows_b = pair ? gemm_pair_block_rows() : gemm_block_rows_b();
    if (!encode_plane_map(&tA, at<int8_t>(ws, l.o_pA), (int64_t)l.G * l.batch, l.M, l.Kp, rows_a) ||
        !encode_plane_map(&tB, at<int8_t>(ws, l.o_pB), (int64_t)l.G * l.batch, l.N, l.Kp, rows_b))
      return fail(F64E_ERR_CUDA, "cuTensorMapEncodeTiled rejected the plane layout");
    const cudaError_t e = pair ? launch_residue_gemm_pair(tA, tB, g, T, d.sms, s)
                               : launch_residue_gemm(tA, tB, g, T, d.sms, s);
    if (e != cudaSuccess) return cuda_fail(e, "modular GEMM launch");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "modular GEMM launch");
  return F64E_OK;
}

void run_reconstruct(const Plan& l, const ModTables& T, void* ws, double* out, cudaStream_t s) {
  ReconArgs r{};
  r.res = at<int8_t>(ws, l.o_res);
  r.corr_mode = l.recon_corr;
  r.corr = l.recon_corr == 3 ? (const void*)at<int64_t>(ws, l.o_cacc) : (const void*)at<int32_t>(ws, l.o_corr);
  r.MF = l.MF;
  r.M = l.M;
  r.N = l.N;
  r.ldn = l.ldn;
  r.sftA = at<int16_t>(ws, l.o_sftA);
  r.sftB = at<int16_t>(ws, l.o_sftB);
  r.maxlg = at<WsHead>(ws, 0)->maxlg;
  r.bits = l.bits;
  r.exact = l.exact;
  r.C = out;
  launch_reconstruct(r, T, s);
}

int run(const f64e_problem* p, const double* A, const double* B, double* out, void* ws, size_t ws_bytes,
        void* stream, int phases, bool checked, cudaEvent_t* ev) {
  Plan l;
  int rc = make_plan(p, &l);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (l.MF == 0 || l.NF == 0) return F64E_OK;
  if (!A || !B || !out) return fail(F64E_ERR_ARGUMENT, "null operand pointer");
  if (l.K == 0) {
    if (phases & F64E_PHASE_COMPUTE) {
      const cudaError_t e = cudaMemsetAsync(out, 0, sizeof(double) * l.MF * l.N, s);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
    return F64E_OK;
  }
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
  if (!l.deep) {
    if (phases & F64E_PHASE_EXTRACT) run_extract(l, T, A, B, ws, 0, l.K, s);
    if (ev) cudaEventRecord(ev[1], s);
    if (phases & F64E_PHASE_GEMM) {
      rc = run_gemm(l, T, ws, d, checked, s);
      if (rc) return rc;
    }
  } else if (phases & (F64E_PHASE_EXTRACT | F64E_PHASE_GEMM)) {
    if ((phases & (F64E_PHASE_EXTRACT | F64E_PHASE_GEMM)) != (F64E_PHASE_EXTRACT | F64E_PHASE_GEMM))
      return fail(F64E_ERR_ARGUMENT, "deep-K products run EXTRACT and GEMM together");
    const int64_t nres = (int64_t)l.P * l.MF * l.ldn, ncorr = l.use_corr ? l.MF * l.ldn : 0;
    for (int sgi = 0; sgi < l.nseg; sgi++) {
      const int64_t k0 = (int64_t)sgi * l.Kseg;
      run_extract(l, T, A, B, ws, k0, std::min(l.Kseg, l.K - k0), s);
      rc = run_gemm(l, T, ws, d, checked, s);
      if (rc) return rc;
      launch_deepk_accum(at<int8_t>(ws, l.o_res), at<int32_t>(ws, l.o_racc), nres, at<int32_t>(ws, l.o_corr),
                         at<int64_t>(ws, l.o_cacc), ncorr, sgi == 0, s);
    }
    launch_deepk_fold(at<int32_t>(ws, l.o_racc), at<int8_t>(ws, l.o_res), l.MF * l.ldn, T, s);
    if (ev) cudaEventRecord(ev[1], s);
  }
  if (ev) {
    cudaEventRecord(ev[2], s);
    cudaEventRecord(ev[3], s);
  }
  if (phases & F64E_PHASE_RECON) run_reconstruct(l, T, ws, out, s);
  if (ev) cudaEventRecord(ev[4], s);
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
