// torch op binding of the B200 fp64-emu library, namespace fp64_emu_b200.
//
// The five product ops keep the reference's schemas exactly
// (torch-ext/torch_binding.cpp:7-12 of CharlesCNorton/fp64-emu) and its
// argument checks and messages (fp64_emu_cuda/fp64_emu.cu:1583-1704); the
// work is done by the C ABI in include/f64e.h with a workspace from torch's
// caching allocator on the current stream.  A few extra ops expose the
// two-phase form used by the partitioned multi-GPU path and test aids.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <vector>

#include "f64e.h"

namespace {

std::vector<int32_t> host_primes(const at::Tensor& primes_cpu) {
  auto pc = primes_cpu.to(at::kCPU, at::kInt).contiguous();
  return std::vector<int32_t>(pc.data_ptr<int32_t>(), pc.data_ptr<int32_t>() + pc.numel());
}

void check(int rc) { TORCH_CHECK(rc == F64E_OK, "fp64_emu: ", f64e_last_error()); }

at::Tensor make_ws(const f64e_problem& p, const at::Tensor& like) {
  const size_t n = f64e_workspace_size(&p);
  TORCH_CHECK(n > 0, "fp64_emu: ", f64e_last_error());
  return at::empty({(int64_t)n}, like.options().dtype(at::kByte));
}

void* stream_of() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_out(const at::Tensor& out, const at::Tensor& A, at::IntArrayRef shape, const char* msg) {
  TORCH_CHECK(out.dtype() == at::kDouble && out.sizes() == shape && out.is_contiguous(), msg);
  TORCH_CHECK(out.is_cuda() && out.device() == A.device(), "out must be on the device of A");
}

f64e_problem problem(int64_t batch, int64_t M, int64_t N, int64_t K, bool b_kn, const std::vector<int32_t>& pr,
                     bool exact, int64_t bits, bool use_corr) {
  f64e_problem p;
  p.batch = batch;
  p.M = M;
  p.N = N;
  p.K = K;
  p.b_layout = b_kn ? F64E_B_KN : F64E_B_NK;
  p.nprimes = (int32_t)pr.size();
  p.primes = pr.data();
  p.exact = exact ? 1 : 0;
  p.bits = (int32_t)bits;
  p.use_corr = use_corr ? 1 : 0;
  p.slab_cols = 0;
  return p;
}

int64_t maxp() { return f64e_maxp(); }

// out[m,n] = A[m,k] @ B[n,k]^T (reference fp64_emu_mm, fp64_emu.cu:1583-1608).
void mm(at::Tensor& out, const at::Tensor& A, const at::Tensor& B, const at::Tensor& primes_cpu,
        const at::Tensor& inv_cpu, const at::Tensor& mu_cpu, bool exact, int64_t bits, bool use_corr) {
  (void)inv_cpu;
  (void)mu_cpu;
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.dtype() == at::kDouble && B.dtype() == at::kDouble,
              "A,B must be f64 CUDA");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.is_contiguous() && B.is_contiguous(), "2D contig");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "expect B as [N, K]");
  check_out(out, A, {M, N}, "out f64 [M,N]");
  TORCH_CHECK((int)primes_cpu.numel() <= f64e_maxp(), "too many primes");
  TORCH_CHECK(K <= (int64_t)128 * 65536, "K bound: 128 segments of 65536");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  const c10::cuda::CUDAGuard guard(A.device());
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem(1, M, N, K, false, pr, exact, bits, use_corr);
  at::Tensor ws = make_ws(p, A);
  check(f64e_mm(out.data_ptr<double>(), A.data_ptr<double>(), B.data_ptr<double>(), M, N, K, pr.data(),
                (int32_t)pr.size(), exact, bits, use_corr, ws.data_ptr(), ws.numel(), stream_of()));
}

// out[m,n] = A[m,k] @ Bt[k,n] (reference fp64_emu_mm_nt, fp64_emu.cu:1613-1632).
void mm_nt(at::Tensor& out, const at::Tensor& A, const at::Tensor& Bt, const at::Tensor& primes_cpu,
           const at::Tensor& inv_cpu, const at::Tensor& mu_cpu, bool exact, int64_t bits, bool use_corr) {
  (void)inv_cpu;
  (void)mu_cpu;
  TORCH_CHECK(A.is_cuda() && Bt.is_cuda() && A.dtype() == at::kDouble && Bt.dtype() == at::kDouble,
              "A,Bt must be f64 CUDA");
  TORCH_CHECK(A.dim() == 2 && Bt.dim() == 2 && A.is_contiguous() && Bt.is_contiguous(), "2D contig");
  const int64_t M = A.size(0), K = A.size(1), N = Bt.size(1);
  TORCH_CHECK(Bt.size(0) == K, "expect Bt as [K, N]");
  check_out(out, A, {M, N}, "out f64 [M,N]");
  TORCH_CHECK((int)primes_cpu.numel() <= f64e_maxp(), "too many primes");
  TORCH_CHECK(K <= 131071, "K bound for int32 modular GEMM");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  const c10::cuda::CUDAGuard guard(A.device());
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem(1, M, N, K, true, pr, exact, bits, use_corr);
  at::Tensor ws = make_ws(p, A);
  check(f64e_mm_nt(out.data_ptr<double>(), A.data_ptr<double>(), Bt.data_ptr<double>(), M, N, K, pr.data(),
                   (int32_t)pr.size(), exact, bits, use_corr, ws.data_ptr(), ws.numel(), stream_of()));
}

// out[b] = A[b] @ B[b]^T (reference fp64_emu_bmm, fp64_emu.cu:1637-1662).
void bmm(at::Tensor& out, const at::Tensor& A, const at::Tensor& B, const at::Tensor& primes_cpu,
         const at::Tensor& inv_cpu, const at::Tensor& mu_cpu, bool exact, int64_t bits, bool use_corr) {
  (void)inv_cpu;
  (void)mu_cpu;
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.dtype() == at::kDouble && B.dtype() == at::kDouble,
              "A,B must be f64 CUDA");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3 && A.is_contiguous() && B.is_contiguous(), "3D contig");
  const int64_t batch = A.size(0), M = A.size(1), K = A.size(2), N = B.size(1);
  TORCH_CHECK(B.size(0) == batch && B.size(2) == K, "expect B as [batch, N, K]");
  check_out(out, A, {batch, M, N}, "out f64 [batch,M,N]");
  const int64_t NP = primes_cpu.numel() + (use_corr ? 2 : 0);
  TORCH_CHECK((int)primes_cpu.numel() <= f64e_maxp(), "too many primes");
  TORCH_CHECK(NP * batch <= 65535, "(nprimes + 2) * batch exceeds the launch z-extent");
  TORCH_CHECK(K <= (int64_t)128 * 65536, "K bound: 128 segments of 65536");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  const c10::cuda::CUDAGuard guard(A.device());
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem(batch, M, N, K, false, pr, exact, bits, use_corr);
  at::Tensor ws = make_ws(p, A);
  check(f64e_bmm(out.data_ptr<double>(), A.data_ptr<double>(), B.data_ptr<double>(), batch, M, N, K, pr.data(),
                 (int32_t)pr.size(), exact, bits, use_corr, ws.data_ptr(), ws.numel(), stream_of()));
}

// out[b] = A[b] @ Bt[b] (reference fp64_emu_bmm_nt, fp64_emu.cu:1665-1686).
void bmm_nt(at::Tensor& out, const at::Tensor& A, const at::Tensor& Bt, const at::Tensor& primes_cpu,
            const at::Tensor& inv_cpu, const at::Tensor& mu_cpu, bool exact, int64_t bits, bool use_corr) {
  (void)inv_cpu;
  (void)mu_cpu;
  TORCH_CHECK(A.is_cuda() && Bt.is_cuda() && A.dtype() == at::kDouble && Bt.dtype() == at::kDouble,
              "A,Bt must be f64 CUDA");
  TORCH_CHECK(A.dim() == 3 && Bt.dim() == 3 && A.is_contiguous() && Bt.is_contiguous(), "3D contig");
  const int64_t batch = A.size(0), M = A.size(1), K = A.size(2), N = Bt.size(2);
  TORCH_CHECK(Bt.size(0) == batch && Bt.size(1) == K, "expect Bt as [batch, K, N]");
  check_out(out, A, {batch, M, N}, "out f64 [batch,M,N]");
  const int64_t NP = primes_cpu.numel() + (use_corr ? 2 : 0);
  TORCH_CHECK((int)primes_cpu.numel() <= f64e_maxp(), "too many primes");
  TORCH_CHECK(NP * batch <= 65535, "(nprimes + 2) * batch exceeds the launch z-extent");
  TORCH_CHECK(K <= 131071, "K bound for int32 modular GEMM");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  const c10::cuda::CUDAGuard guard(A.device());
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem(batch, M, N, K, true, pr, exact, bits, use_corr);
  at::Tensor ws = make_ws(p, A);
  check(f64e_bmm_nt(out.data_ptr<double>(), A.data_ptr<double>(), Bt.data_ptr<double>(), batch, M, N, K,
                    pr.data(), (int32_t)pr.size(), exact, bits, use_corr, ws.data_ptr(), ws.numel(), stream_of()));
}

// mm with phase timings (reference fp64_emu_mm_timed, fp64_emu.cu:1688-1704).
void mm_timed(at::Tensor& out, at::Tensor& times, const at::Tensor& A, const at::Tensor& B,
              const at::Tensor& primes_cpu, const at::Tensor& inv_cpu, const at::Tensor& mu_cpu, bool exact,
              int64_t bits, bool use_corr) {
  (void)inv_cpu;
  (void)mu_cpu;
  TORCH_CHECK(A.size(1) <= 131071, "K bound for int32 modular GEMM");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.dtype() == at::kDouble && B.dtype() == at::kDouble,
              "A,B must be f64 CUDA");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.is_contiguous() && B.is_contiguous(), "2D contig");
  TORCH_CHECK(B.size(1) == A.size(1), "expect B as [N, K]");
  TORCH_CHECK(times.device().is_cpu() && times.dtype() == at::kFloat && times.numel() >= 4 &&
                  times.is_contiguous(),
              "times must be a CPU float32 tensor of 4");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  check_out(out, A, {M, N}, "out f64 [M,N]");
  const c10::cuda::CUDAGuard guard(A.device());
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem(1, M, N, K, false, pr, exact, bits, use_corr);
  at::Tensor ws = make_ws(p, A);
  check(f64e_mm_timed(out.data_ptr<double>(), times.data_ptr<float>(), A.data_ptr<double>(), B.data_ptr<double>(),
                      M, N, K, pr.data(), (int32_t)pr.size(), exact, bits, use_corr, ws.data_ptr(), ws.numel(),
                      stream_of()));
}

// ---- two-phase and test-aid ops ----

f64e_problem problem_of(const at::Tensor& A, const at::Tensor& B, bool b_kn, const std::vector<int32_t>& pr,
                        bool exact, int64_t bits, bool use_corr) {
  TORCH_CHECK(A.dim() == B.dim() && (A.dim() == 2 || A.dim() == 3), "A and B must both be 2-D or 3-D");
  const bool batched = A.dim() == 3;
  const int64_t batch = batched ? A.size(0) : 1;
  const int64_t M = A.size(-2), K = A.size(-1);
  const int64_t N = b_kn ? B.size(-1) : B.size(-2);
  TORCH_CHECK((b_kn ? B.size(-2) : B.size(-1)) == K, "inner dimensions differ");
  TORCH_CHECK(!batched || B.size(0) == batch, "batch sizes differ");
  return problem(batch, M, N, K, b_kn, pr, exact, bits, use_corr);
}

int64_t workspace_bytes(const at::Tensor& A, const at::Tensor& B, const at::Tensor& primes_cpu, bool b_kn,
                        bool use_corr, int64_t slab_cols) {
  const auto pr = host_primes(primes_cpu);
  f64e_problem p = problem_of(A, B, b_kn, pr, true, 53, use_corr);
  p.slab_cols = slab_cols;
  const size_t n = f64e_workspace_size(&p);
  TORCH_CHECK(n > 0, "fp64_emu: ", f64e_last_error());
  return (int64_t)n;
}

void gemm_phase(at::Tensor& out, at::Tensor& ws, const at::Tensor& A, const at::Tensor& B,
                const at::Tensor& primes_cpu, bool b_kn, bool exact, int64_t bits, bool use_corr, int64_t phases,
                bool checked, int64_t slab_cols, const std::vector<int64_t>* events = nullptr,
                int32_t* launches = nullptr) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.dtype() == at::kDouble && B.dtype() == at::kDouble,
              "A,B must be f64 CUDA");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && out.is_contiguous() && ws.is_contiguous(), "contig");
  TORCH_CHECK(ws.is_cuda() && ws.device() == A.device() && out.device() == A.device(), "same device");
  const auto pr = host_primes(primes_cpu);
  f64e_problem p = problem_of(A, B, b_kn, pr, exact, bits, use_corr);
  p.slab_cols = slab_cols;
  TORCH_CHECK(out.dtype() == at::kDouble && out.numel() == p.batch * p.M * p.N, "out f64 of batch*M*N");
  const c10::cuda::CUDAGuard guard(A.device());
  const size_t nb = (size_t)ws.numel() * ws.element_size();
  if (checked)
    check(f64e_gemm_checked(&p, A.data_ptr<double>(), B.data_ptr<double>(), out.data_ptr<double>(), ws.data_ptr(),
                            nb, stream_of()));
  else if (events) {
    std::vector<void*> ev(events->size());
    for (size_t i = 0; i < ev.size(); i++) ev[i] = reinterpret_cast<void*>((*events)[i]);
    check(f64e_gemm_ev(&p, A.data_ptr<double>(), B.data_ptr<double>(), out.data_ptr<double>(), ws.data_ptr(), nb,
                       stream_of(), (int)phases, ev.data(), (int32_t)ev.size(), launches));
  } else {
    check(f64e_gemm(&p, A.data_ptr<double>(), B.data_ptr<double>(), out.data_ptr<double>(), ws.data_ptr(), nb,
                    stream_of(), (int)phases));
  }
}

void gemm_ws(at::Tensor& out, at::Tensor& ws, const at::Tensor& A, const at::Tensor& B,
             const at::Tensor& primes_cpu, bool b_kn, bool exact, int64_t bits, bool use_corr, int64_t phases,
             int64_t slab_cols) {
  gemm_phase(out, ws, A, B, primes_cpu, b_kn, exact, bits, use_corr, phases, false, slab_cols);
}

// gemm_ws that brackets each modular-GEMM launch with two of the given CUDA
// events (raw cudaEvent_t handles, e.g. torch.cuda.Event.cuda_event) and
// returns the number of GEMM launches.
int64_t gemm_ws_ev(at::Tensor& out, at::Tensor& ws, const at::Tensor& A, const at::Tensor& B,
                   const at::Tensor& primes_cpu, bool b_kn, bool exact, int64_t bits, bool use_corr, int64_t phases,
                   int64_t slab_cols, at::IntArrayRef events) {
  for (const int64_t e : events) TORCH_CHECK(e != 0, "events must be created (record them once first)");
  const std::vector<int64_t> ev(events.begin(), events.end());
  int32_t launches = 0;
  gemm_phase(out, ws, A, B, primes_cpu, b_kn, exact, bits, use_corr, phases, false, slab_cols, &ev, &launches);
  return launches;
}

// Host-resident product: A, B and out are CPU tensors (page-locked for the
// copies to overlap); the device buffers and workspace come from torch's
// caching allocator on the current device and stream.  The result blocks are
// copied back while later blocks compute; the call returns once out holds
// the product.
void gemm_host(at::Tensor& out, const at::Tensor& A, const at::Tensor& B, const at::Tensor& primes_cpu, bool b_kn,
               bool exact, int64_t bits, bool use_corr) {
  TORCH_CHECK(!A.is_cuda() && !B.is_cuda() && !out.is_cuda(), "host product: A, B and out must be CPU tensors");
  TORCH_CHECK(A.dtype() == at::kDouble && B.dtype() == at::kDouble && out.dtype() == at::kDouble, "f64 tensors");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && out.is_contiguous(), "contig");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem_of(A, B, b_kn, pr, exact, bits, use_corr);
  TORCH_CHECK(out.numel() == p.batch * p.M * p.N, "out f64 of batch*M*N");
  const auto dev = at::TensorOptions().device(at::kCUDA, c10::cuda::current_device()).dtype(at::kDouble);
  at::Tensor Ad = at::empty(A.sizes(), dev), Bd = at::empty(B.sizes(), dev), Cd = at::empty(out.sizes(), dev);
  const size_t nb = f64e_workspace_size(&p);
  TORCH_CHECK(nb > 0, "fp64_emu: ", f64e_last_error());
  at::Tensor ws = at::empty({(int64_t)nb}, dev.dtype(at::kByte));
  check(f64e_gemm_host(&p, A.data_ptr<double>(), B.data_ptr<double>(), out.data_ptr<double>(), Ad.data_ptr<double>(),
                       Bd.data_ptr<double>(), Cd.data_ptr<double>(), ws.data_ptr(), nb, stream_of()));
  const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_of()));
  TORCH_CHECK(e == cudaSuccess, "fp64_emu: ", cudaGetErrorString(e));
}

// One product of fp64_emu.HostStream, queued without a host wait: the
// operand copies on streams[0], the product on streams[1], the result copy on
// streams[2] (raw cudaStream_t handles of the slot's device).  events (raw
// cudaEvent_t, created): [caller, loaded, computed, done]; the three streams
// first wait for what the caller's current stream queued before the call,
// and when the slot held an earlier product (used) the copies into its
// device operands wait until that product has read them and the product
// waits until its result has left the device.
void host_submit(at::Tensor& out, const at::Tensor& A, const at::Tensor& B, at::Tensor& Ad, at::Tensor& Bd,
                 at::Tensor& Cd, at::Tensor& ws, const at::Tensor& primes_cpu, bool b_kn, bool exact, int64_t bits,
                 bool use_corr, at::IntArrayRef streams, at::IntArrayRef events, bool used) {
  TORCH_CHECK(!A.is_cuda() && !B.is_cuda() && !out.is_cuda(), "host submit: A, B and out must be CPU tensors");
  TORCH_CHECK(Ad.is_cuda() && Bd.is_cuda() && Cd.is_cuda() && ws.is_cuda(), "host submit: device buffers");
  TORCH_CHECK(Bd.device() == Ad.device() && Cd.device() == Ad.device() && ws.device() == Ad.device(),
              "host submit: device buffers on one device");
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&out, &A, &B, &Ad, &Bd, &Cd})
    TORCH_CHECK(t->dtype() == at::kDouble && t->is_contiguous(), "host submit: contiguous f64 tensors");
  TORCH_CHECK(A.sizes() == Ad.sizes() && B.sizes() == Bd.sizes() && out.sizes() == Cd.sizes(),
              "host submit: host and device shapes differ");
  TORCH_CHECK(ws.is_contiguous(), "host submit: contiguous workspace");
  TORCH_CHECK(streams.size() == 3 && events.size() == 4, "host submit: 3 streams and 4 events");
  for (const int64_t e : events) TORCH_CHECK(e != 0, "events must be created (record them once first)");
  TORCH_CHECK(bits >= 16 && bits <= 53, "bits must be in [16, 53]");
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem_of(Ad, Bd, b_kn, pr, exact, bits, use_corr);
  const c10::cuda::CUDAGuard guard(Ad.device());
  cudaStream_t h2d = reinterpret_cast<cudaStream_t>(streams[0]), comp = reinterpret_cast<cudaStream_t>(streams[1]),
               d2h = reinterpret_cast<cudaStream_t>(streams[2]);
  cudaEvent_t caller = reinterpret_cast<cudaEvent_t>(events[0]), loaded = reinterpret_cast<cudaEvent_t>(events[1]),
              computed = reinterpret_cast<cudaEvent_t>(events[2]), done = reinterpret_cast<cudaEvent_t>(events[3]);
  cudaError_t e = cudaEventRecord(caller, static_cast<cudaStream_t>(stream_of()));
  for (cudaStream_t st : {h2d, comp, d2h})
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, caller, 0);
  if (used && e == cudaSuccess) e = cudaStreamWaitEvent(h2d, computed, 0);
  if (used && e == cudaSuccess) e = cudaStreamWaitEvent(comp, done, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(Ad.data_ptr(), A.data_ptr(), (size_t)A.numel() * 8, cudaMemcpyHostToDevice, h2d);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(Bd.data_ptr(), B.data_ptr(), (size_t)B.numel() * 8, cudaMemcpyHostToDevice, h2d);
  if (e == cudaSuccess) e = cudaEventRecord(loaded, h2d);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(comp, loaded, 0);
  TORCH_CHECK(e == cudaSuccess, "fp64_emu: ", cudaGetErrorString(e));
  check(f64e_gemm(&p, Ad.data_ptr<double>(), Bd.data_ptr<double>(), Cd.data_ptr<double>(), ws.data_ptr(),
                  (size_t)ws.numel() * ws.element_size(), comp, F64E_PHASE_ALL));
  e = cudaEventRecord(computed, comp);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(d2h, computed, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out.data_ptr(), Cd.data_ptr(), (size_t)out.numel() * 8, cudaMemcpyDeviceToHost, d2h);
  if (e == cudaSuccess) e = cudaEventRecord(done, d2h);
  TORCH_CHECK(e == cudaSuccess, "fp64_emu: ", cudaGetErrorString(e));
}

void gemm_checked(at::Tensor& out, at::Tensor& ws, const at::Tensor& A, const at::Tensor& B,
                  const at::Tensor& primes_cpu, bool b_kn, bool exact, int64_t bits, bool use_corr) {
  gemm_phase(out, ws, A, B, primes_cpu, b_kn, exact, bits, use_corr, F64E_PHASE_ALL, true, 0);
}

int64_t status(const at::Tensor& ws) {
  TORCH_CHECK(ws.is_cuda(), "workspace must be CUDA");
  const c10::cuda::CUDAGuard guard(ws.device());
  int32_t st = 0;
  check(f64e_status(ws.data_ptr(), stream_of(), &st));
  return st;
}

at::Tensor debug_fetch(const at::Tensor& ws, const at::Tensor& A, const at::Tensor& B, const at::Tensor& primes_cpu,
                       bool b_kn, bool use_corr, int64_t which) {
  const auto pr = host_primes(primes_cpu);
  const f64e_problem p = problem_of(A, B, b_kn, pr, true, 53, use_corr);
  const c10::cuda::CUDAGuard guard(ws.device());
  const size_t cap = (size_t)ws.numel();
  at::Tensor host = at::empty({(int64_t)cap}, at::TensorOptions().dtype(at::kByte));
  size_t n = 0;
  check(f64e_debug_fetch(&p, ws.data_ptr(), (int)which, host.data_ptr(), cap, &n, stream_of()));
  return host.narrow(0, 0, (int64_t)n).clone();
}

void set_wait_limit_ns(int64_t ns) { f64e_set_wait_limit_ns((uint64_t)ns); }

int64_t wait_selftest(at::Tensor& ws, int64_t limit_ns) {
  TORCH_CHECK(ws.is_cuda() && ws.is_contiguous(), "workspace must be a contiguous CUDA tensor");
  TORCH_CHECK(limit_ns > 0, "limit must be positive");
  const c10::cuda::CUDAGuard guard(ws.device());
  int32_t st = 0;
  check(f64e_wait_selftest(ws.data_ptr(), (size_t)ws.numel() * ws.element_size(), (uint64_t)limit_ns, stream_of(),
                           &st));
  return st;
}

}  // namespace

TORCH_LIBRARY(fp64_emu_b200, ops) {
  ops.def("fp64_emu_maxp() -> int");
  ops.def(
      "fp64_emu_mm(Tensor! out, Tensor A, Tensor B, Tensor primes_cpu, Tensor inv_cpu, Tensor mu_cpu, bool exact, "
      "int bits=53, bool use_corr=True) -> ()");
  ops.def(
      "fp64_emu_bmm(Tensor! out, Tensor A, Tensor B, Tensor primes_cpu, Tensor inv_cpu, Tensor mu_cpu, bool exact, "
      "int bits=53, bool use_corr=True) -> ()");
  ops.def(
      "fp64_emu_mm_nt(Tensor! out, Tensor A, Tensor Bt, Tensor primes_cpu, Tensor inv_cpu, Tensor mu_cpu, bool "
      "exact, int bits=53, bool use_corr=True) -> ()");
  ops.def(
      "fp64_emu_bmm_nt(Tensor! out, Tensor A, Tensor Bt, Tensor primes_cpu, Tensor inv_cpu, Tensor mu_cpu, bool "
      "exact, int bits=53, bool use_corr=True) -> ()");
  ops.def(
      "fp64_emu_mm_timed(Tensor! out, Tensor! times, Tensor A, Tensor B, Tensor primes_cpu, Tensor inv_cpu, Tensor "
      "mu_cpu, bool exact, int bits=53, bool use_corr=True) -> ()");
  ops.def(
      "fp64_emu_workspace_bytes(Tensor A, Tensor B, Tensor primes_cpu, bool b_kn, bool use_corr, int slab_cols=0) "
      "-> int");
  ops.def(
      "fp64_emu_gemm_ws(Tensor! out, Tensor! ws, Tensor A, Tensor B, Tensor primes_cpu, bool b_kn, bool exact, "
      "int bits, bool use_corr, int phases, int slab_cols=0) -> ()");
  ops.def(
      "fp64_emu_gemm_ws_ev(Tensor! out, Tensor! ws, Tensor A, Tensor B, Tensor primes_cpu, bool b_kn, bool exact, "
      "int bits, bool use_corr, int phases, int slab_cols, int[] events) -> int");
  ops.def(
      "fp64_emu_gemm_host(Tensor! out, Tensor A, Tensor B, Tensor primes_cpu, bool b_kn, bool exact, int bits, "
      "bool use_corr) -> ()");
  ops.def(
      "fp64_emu_host_submit(Tensor! out, Tensor A, Tensor B, Tensor! Ad, Tensor! Bd, Tensor! Cd, Tensor! ws, "
      "Tensor primes_cpu, bool b_kn, bool exact, int bits, bool use_corr, int[] streams, int[] events, bool used) "
      "-> ()");
  ops.def(
      "fp64_emu_gemm_checked(Tensor! out, Tensor! ws, Tensor A, Tensor B, Tensor primes_cpu, bool b_kn, bool "
      "exact, int bits, bool use_corr) -> ()");
  ops.def("fp64_emu_status(Tensor ws) -> int");
  ops.def(
      "fp64_emu_debug_fetch(Tensor ws, Tensor A, Tensor B, Tensor primes_cpu, bool b_kn, bool use_corr, int which) "
      "-> Tensor");
  ops.def("fp64_emu_set_wait_limit_ns(int ns) -> ()");
  ops.def("fp64_emu_wait_selftest(Tensor! ws, int limit_ns) -> int");
  ops.impl("fp64_emu_maxp", &maxp);
  ops.impl("fp64_emu_workspace_bytes", &workspace_bytes);
  ops.impl("fp64_emu_set_wait_limit_ns", &set_wait_limit_ns);
}

// The host product's tensors live on the CPU; its work runs on the current CUDA device.
TORCH_LIBRARY_IMPL(fp64_emu_b200, CPU, ops) { ops.impl("fp64_emu_gemm_host", &gemm_host); }

TORCH_LIBRARY_IMPL(fp64_emu_b200, CUDA, ops) {
  ops.impl("fp64_emu_mm", &mm);
  ops.impl("fp64_emu_bmm", &bmm);
  ops.impl("fp64_emu_mm_nt", &mm_nt);
  ops.impl("fp64_emu_bmm_nt", &bmm_nt);
  ops.impl("fp64_emu_mm_timed", &mm_timed);
  ops.impl("fp64_emu_gemm_ws", &gemm_ws);
  ops.impl("fp64_emu_gemm_ws_ev", &gemm_ws_ev);
  ops.impl("fp64_emu_gemm_checked", &gemm_checked);
  ops.impl("fp64_emu_host_submit", &host_submit);   // CPU operands, CUDA buffers: the CUDA key
  ops.impl("fp64_emu_status", &status);
  ops.impl("fp64_emu_debug_fetch", &debug_fetch);
  ops.impl("fp64_emu_wait_selftest", &wait_selftest);
}
