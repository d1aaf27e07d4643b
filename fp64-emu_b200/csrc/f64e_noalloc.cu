// Allocation-free form of f64e_mm_nt.
//
// Some callers cannot allocate device memory: code running inside another
// framework's device-memory arena (which owns every byte and forbids side
// allocations), plugin hosts and real-time paths that may not call
// cudaMalloc / cudaFree (both can synchronize the device), and embedded or
// sandboxed deployments whose allocator is not reachable.  They cannot pass
// the workspace the other entry points take.  This entry point runs the same
// product with its workspace in a file-scope device array of fixed size
// (F64E_NOALLOC_SCRATCH_BYTES), so the caller supplies only inputs, outputs
// and a stream, and nothing is allocated.
//
// Limits and sharing:
//   * the array occupies F64E_NOALLOC_SCRATCH_BYTES on every GPU whose
//     context loads this library's device code: with CUDA's default lazy
//     module loading that is every GPU where this entry point (or another
//     kernel of the library) has run; with CUDA_MODULE_LOADING=EAGER it is
//     every GPU the process creates a context on.  It is held until the
//     context is destroyed (process exit or cudaDeviceReset);
//   * problems whose workspace exceeds it are rejected (F64E_ERR_WORKSPACE);
//   * every call on a device uses the same array, which keeps whatever the
//     last call left there; calls whose work overlaps on the GPU (different
//     streams, or host threads without ordering) race on it and must be
//     serialized by the caller.  Nothing needs to start at zero: the product
//     writes every scratch byte it reads before reading it, and it clears
//     its status word itself.
//   * the array's host-side name is only a stand-in for the device copy, so
//     the entry point looks up the device address with cudaGetSymbolAddress
//     (with the caller's device current) the first time it runs in a CUDA
//     context, and caches it under that context's unique id (cuCtxGetId):
//     a new context -- after cudaDeviceReset, or a context the caller made
//     with cuCtxCreate -- gets a fresh lookup instead of a stale address.
//     That first call in a context should come before any stream capture.
#include <mutex>

#include "f64e.h"
#include "f64e_kernels.h"

namespace f64e {
int run_problem(const f64e_problem* p, const double* A, const double* B, double* out, void* ws, size_t ws_bytes,
                void* stream, int phases);
int report_error(int code, const char* msg);
}  // namespace f64e

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[F64E_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mtx;
struct ScratchSlot {
  unsigned long long ctx_id;  // unique id of the context the address belongs to
  void* addr;                 // device address of the array there; null until set up
};
ScratchSlot g_scratch[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the current CUDA context (driver entry points fetched through
// the runtime, so the library links no libcuda).  0 when unavailable or when
// no context is current yet (cudaGetSymbolAddress then creates the device's
// primary context, and the next call caches under its id).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the scratch array in the current device's current
// context (looked up once per context, with that device current).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return f64e::report_error(F64E_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return f64e::report_error(F64E_ERR_UNSUPPORTED, "device index out of range");
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_scratch_mtx);
  ScratchSlot& s = g_scratch[dev];
  if (!s.addr || ctx == 0 || s.ctx_id != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return f64e::report_error(F64E_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc scratch failed");
    s.addr = p;
    s.ctx_id = ctx;
  }
  *out = s.addr;
  return F64E_OK;
}

}  // namespace

extern "C" int f64e_mm_nt_noalloc(double* out, const double* A, const double* Bt, int64_t M, int64_t N, int64_t K,
                                  const int32_t* primes, int32_t nprimes, int32_t exact, int64_t bits,
                                  int32_t use_corr, void* stream) {
  f64e_problem p;
  p.batch = 1;
  p.M = M;
  p.N = N;
  p.K = K;
  p.b_layout = F64E_B_KN;
  p.nprimes = nprimes;
  p.primes = primes;
  p.exact = exact;
  p.bits = (bits < 0 || bits > 64) ? 0 : (int32_t)bits;
  p.use_corr = use_corr;
  p.slab_cols = 0;
  const size_t need = f64e_workspace_size(&p);
  if (need == 0) return F64E_ERR_ARGUMENT;  // message already set by the size query
  if (need > (size_t)F64E_NOALLOC_SCRATCH_BYTES)
    return f64e::report_error(F64E_ERR_WORKSPACE,
                              "problem needs more scratch than the no-alloc entry point holds "
                              "(F64E_NOALLOC_SCRATCH_BYTES); use f64e_mm_nt with a caller workspace");
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != F64E_OK) return rc;
  return f64e::run_problem(&p, A, Bt, out, ws, (size_t)F64E_NOALLOC_SCRATCH_BYTES, stream, F64E_PHASE_ALL);
}
