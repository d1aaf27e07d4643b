/*
 * f64e.h -- C ABI of the B200-native fp64-emu library (libf64e.so).
 *
 * Emulated FP64 matrix products on INT8 tensor cores (RARE / Ozaki-II CRT):
 * operands are scaled per row / column to exact integers, reduced to balanced
 * INT8 residues modulo up to 20 pairwise-coprime moduli, multiplied with one
 * tcgen05 INT8 GEMM per modulus (plus the two first-order correction GEMMs),
 * and rebuilt by balanced-Garner reconstruction.
 *
 * Each product entry point replaces one op of the reference's torch binding
 * (CharlesCNorton/fp64-emu, torch-ext/torch_binding.cpp:7-12, implemented in
 * fp64_emu_cuda/fp64_emu.cu) with the same argument meaning and the same
 * argument checks, expressed with plain pointers and sizes:
 *   - pointers A, B, out are device pointers to contiguous float64 data;
 *   - primes is a HOST array of nprimes moduli (the reference's primes_cpu);
 *     the reference's inv_cpu / mu_cpu tables are ignored by the reference
 *     itself (fp64_emu.cu:1137-1140) and have no counterpart here;
 *   - workspace is device memory of at least f64e_workspace_size() bytes,
 *     256-byte aligned, owned by the caller; nothing is allocated inside;
 *   - stream is a cudaStream_t (NULL = legacy default stream); every kernel
 *     is enqueued on it and no call synchronizes, except f64e_mm_timed (which
 *     returns host timings, like the reference) and f64e_status.
 * Return value: F64E_OK or an F64E_ERR_* code; f64e_last_error() gives the
 * message of the last failure on the calling thread.  Nothing throws.
 */
#ifndef F64E_H
#define F64E_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define F64E_API __attribute__((visibility("default")))
#else
#define F64E_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  F64E_OK = 0,
  F64E_ERR_ARGUMENT = 1,    /* shape / parameter rejected (the reference's TORCH_CHECKs) */
  F64E_ERR_WORKSPACE = 2,   /* workspace missing, too small or misaligned */
  F64E_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  F64E_ERR_UNSUPPORTED = 4, /* current device is not an sm_100 part */
  F64E_ERR_TIMEOUT = 5      /* a bounded device wait ran out (see f64e_status) */
};

/* Layout of the second operand. */
enum {
  F64E_B_NK = 0, /* B is [batch, N, K]: mm, bmm   (out = A @ B^T) */
  F64E_B_KN = 1  /* B is [batch, K, N]: mm_nt, bmm_nt (out = A @ B) */
};

/* Phases of f64e_gemm, run in this order on the caller's stream:
 *   SIZING   per-row / per-column shifts and the two operand maxima of the
 *            log2 norms (float[2] at workspace offset 0);
 *   EXTRACT  residue and correction planes;
 *   GEMM     the modular tensor-core GEMMs;
 *   RECON    reconstruction into out.
 * A partitioned multi-GPU caller MAX-all-reduces the two floats between
 * SIZING and the rest, so every rank uses the single-GPU operand width.
 * Deep-K problems (K > 131071) interleave EXTRACT and GEMM per segment and
 * need both bits in the same call.
 * A call that runs EXTRACT, GEMM and RECON together may cut the product into
 * chunks (rows of A and C, or batch members) and overlap the chunks' phases
 * on two library-owned streams forked from and joined back to the caller's
 * stream; the result is the same bits.  The intermediate planes it leaves in
 * the workspace are then in the chunks' own layout, so a later call that runs
 * GEMM or RECON alone needs the preceding phases run as separate calls.  The
 * first such call on a device creates those streams; a call made while the
 * caller's stream is being captured before that runs unchunked. */
enum {
  F64E_PHASE_SIZING = 1,
  F64E_PHASE_EXTRACT = 2,
  F64E_PHASE_GEMM = 4,
  F64E_PHASE_RECON = 8,
  F64E_PHASE_COMPUTE = 14,
  F64E_PHASE_ALL = 15
};

/* Largest modulus count (reference: fp64_emu_maxp, fp64_emu.cu:956). */
F64E_API int64_t f64e_maxp(void);

/* Full problem description used by the generic entry points. */
typedef struct f64e_problem {
  int64_t batch;         /* >= 1 (1 for mm / mm_nt) */
  int64_t M, N, K;       /* per batch member */
  int32_t b_layout;      /* F64E_B_NK or F64E_B_KN */
  int32_t nprimes;       /* 1..20 */
  const int32_t* primes; /* host array, each modulus in [2, 256] */
  int32_t exact;         /* int128 recombine (1) or fp64 recombine (0) */
  int32_t bits;          /* operand width before widening, 16..53 */
  int32_t use_corr;      /* the two first-order correction GEMMs */
  int64_t slab_cols;     /* F64E_B_KN only: column count whose slab rule orders the
                            column sums (fp64_emu.cu:1159-1162); 0 = batch * N.  A
                            rank holding a slice of the columns passes the full
                            count to reproduce the single-GPU sums exactly. */
} f64e_problem;

/* Bytes of workspace the problem needs (0 when the arguments are invalid;
 * f64e_last_error() then says why). */
F64E_API size_t f64e_workspace_size(const f64e_problem* p);

/* Generic product: out[b] = A[b] @ op(B[b]) for the layout in p.  phases is a
 * mask of F64E_PHASE_*; both phases must see the same arguments and the same
 * workspace. */
F64E_API int f64e_gemm(const f64e_problem* p, const double* A, const double* B, double* out, void* workspace,
              size_t workspace_bytes, void* stream, int phases);

/* f64e_gemm that also brackets every modular-GEMM launch with two caller
 * events (cudaEvent_t, created with timing): launch i records events[2i]
 * before and events[2i + 1] after it, on the stream the launch runs on, for
 * i < n_events / 2.  *launches receives the number of GEMM launches (chunks,
 * or K segments).  Measurement aid with no reference counterpart. */
F64E_API int f64e_gemm_ev(const f64e_problem* p, const double* A, const double* B, double* out, void* workspace,
                 size_t workspace_bytes, void* stream, int phases, void* const* events, int32_t n_events,
                 int32_t* launches);

/* out[M,N] = A[M,K] @ B[N,K]^T.  Replaces fp64_emu_mm (fp64_emu.cu:1583-1608):
 * K <= 8,388,608 (deep K runs K-segmented), bits in [16, 53]. */
F64E_API int f64e_mm(double* out, const double* A, const double* B, int64_t M, int64_t N, int64_t K,
            const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr,
            void* workspace, size_t workspace_bytes, void* stream);

/* out[M,N] = A[M,K] @ Bt[K,N], Bt consumed in place.  Replaces fp64_emu_mm_nt
 * (fp64_emu.cu:1613-1632): K <= 131071. */
F64E_API int f64e_mm_nt(double* out, const double* A, const double* Bt, int64_t M, int64_t N, int64_t K,
               const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits, int32_t use_corr,
               void* workspace, size_t workspace_bytes, void* stream);

/* out[b] = A[b] @ B[b]^T, B as [batch, N, K].  Replaces fp64_emu_bmm
 * (fp64_emu.cu:1637-1662): (nprimes + 2*use_corr) * batch <= 65535. */
F64E_API int f64e_bmm(double* out, const double* A, const double* B, int64_t batch, int64_t M, int64_t N,
             int64_t K, const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits,
             int32_t use_corr, void* workspace, size_t workspace_bytes, void* stream);

/* out[b] = A[b] @ Bt[b], Bt as [batch, K, N].  Replaces fp64_emu_bmm_nt
 * (fp64_emu.cu:1665-1686). */
F64E_API int f64e_bmm_nt(double* out, const double* A, const double* Bt, int64_t batch, int64_t M, int64_t N,
                int64_t K, const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits,
                int32_t use_corr, void* workspace, size_t workspace_bytes, void* stream);

/* mm plus phase timings in ms, written to the HOST array times[4] =
 * {sizing + extraction, modular GEMMs, 0 (marker), reconstruction}.
 * Replaces fp64_emu_mm_timed (fp64_emu.cu:1688-1704); synchronizes the
 * stream.  K <= 131071. */
F64E_API int f64e_mm_timed(double* out, float* times, const double* A, const double* B, int64_t M, int64_t N,
                  int64_t K, const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits,
                  int32_t use_corr, void* workspace, size_t workspace_bytes, void* stream);

/* Device status word of a workspace: 0, or the site code of the first bounded
 * wait that ran out in the last product run with it.  Synchronizes the
 * stream.  Returns F64E_OK / F64E_ERR_*.
 * In the checking build (libf64e_debug.so, compiled with F64E_DEBUG_BOUNDS;
 * same ABI) the word also takes the first out-of-range access, which the
 * kernel skipped instead of performing: 16 extraction read, 17 extraction
 * write, 18 GEMM epilogue write, 19 reconstruction read, 20 reconstruction
 * write.  The reference has no such build; it stands in for the device-side
 * bounds checks a sanitizer would give. */
F64E_API int f64e_status(const void* workspace, void* stream, int32_t* status);

/* Limit, in nanoseconds, on every device-side wait of the GEMM (default
 * 2e9).  Process-wide. */
F64E_API void f64e_set_wait_limit_ns(uint64_t ns);

/* Failure-detection self-test: one device thread waits, with the GEMM's
 * bounded wait, on a barrier that nothing arrives at, so the wait runs out
 * after limit_ns (0 < limit_ns <= 1e10) and records its site code (9) in the
 * workspace status word; *status receives the word.  The context stays
 * usable.  Synchronizes the stream.  Returns F64E_OK / F64E_ERR_*. */
F64E_API int f64e_wait_selftest(void* workspace, size_t workspace_bytes, uint64_t limit_ns, void* stream,
                                int32_t* status);

/* Message of the last failed call on this thread ("" if none). */
F64E_API const char* f64e_last_error(void);

/* The whole product with operands and result in host memory: copies A and B
 * into the caller's device buffers (A_dev: batch*M*K doubles, B_dev:
 * batch*N*K, out_dev: batch*M*N), runs every phase, and copies each finished
 * block of the result back to out_host while later blocks are still being
 * computed, all on `stream`.  Host buffers should be page-locked for the
 * copies to overlap the computation; the result is in out_host once the
 * stream reaches this call's end.  No reference counterpart (the reference's
 * ops take device tensors; a caller there copies around the call). */
F64E_API int f64e_gemm_host(const f64e_problem* p, const double* A_host, const double* B_host, double* out_host,
                   double* A_dev, double* B_dev, double* out_dev, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Self-check aid: the same product as f64e_gemm with the modular GEMM done by
 * a plain dp4a kernel instead of the tensor-core kernel (slow; for tests). */
F64E_API int f64e_gemm_checked(const f64e_problem* p, const double* A, const double* B, double* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Test aid: copy intermediate device buffers of the last run with this
 * workspace to host memory.  which: 0 = A planes, 1 = B planes, 2 = residue
 * planes, 3 = correction planes, 4 = sftA (int16), 5 = sftB (int16),
 * 6 = maxlg (float[2]).  Writes at most cap bytes; returns the byte count
 * via *nbytes.  Synchronizes the stream. */
F64E_API int f64e_debug_fetch(const f64e_problem* p, const void* workspace, int which, void* host, size_t cap,
                     size_t* nbytes, void* stream);

/* Size of the device scratch array behind f64e_mm_nt_noalloc: 64 MiB, enough
 * for products up to roughly M = N = K = 1100 at the default plan. */
#define F64E_NOALLOC_SCRATCH_BYTES (64ull << 20)

/* f64e_mm_nt for callers that cannot allocate device memory (code inside
 * another framework's memory arena, plugin hosts and real-time paths that may
 * not call cudaMalloc / cudaFree, sandboxed deployments without an allocator).
 * No counterpart in the reference.  Same arguments and result as f64e_mm_nt,
 * minus the workspace: the product runs in a file-scope device array of
 * F64E_NOALLOC_SCRATCH_BYTES, held until the process exits on every GPU whose
 * context loaded this library's device code -- under CUDA's default lazy
 * module loading, the GPUs where the library has run a kernel; with
 * CUDA_MODULE_LOADING=EAGER, every GPU the process opens.  Problems needing
 * more scratch are rejected with F64E_ERR_WORKSPACE.  Nothing is allocated.
 * All calls on a device share the one array (it keeps the last call's
 * contents; nothing in it needs to start at zero): calls whose work overlaps
 * on the GPU race and must be serialized by the caller.  The first call in
 * each CUDA context looks up the array's device address
 * (cudaGetSymbolAddress, cached under the context's id, so a reset or a
 * caller-made context gets a fresh lookup) and should come before any
 * stream capture. */
F64E_API int f64e_mm_nt_noalloc(double* out, const double* A, const double* Bt, int64_t M, int64_t N, int64_t K,
                                const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits,
                                int32_t use_corr, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* F64E_H */
