// Operand sizing: per-row (and per-column, for operands consumed in their
// [K, N] layout) power-of-two shifts and log2 2-norms, and the operand maxima
// of those norms that feed the Cauchy-Schwarz width rule.
//
// The shifts depend only on max |x|; the norms feed one float comparison per
// call (the width rule), so they are reduced in exactly the reference's order
// to keep the chosen width identical on every input:
//   rows:    fp64_emu.cu:111-146 (256 thread-strided partials, then a 128..1
//            pairwise tree),
//   columns: fp64_emu.cu:152-189 with the slab count of fp64_emu.cu:1159-1162.
// `s += v * v` is a fused multiply-add, as nvcc contracts it in the reference.
#include "f64e_kernels.h"
#include "f64e_device.cuh"

namespace f64e {

__device__ __forceinline__ void finish_stats(double m, double s2, int bits, int16_t* sft, float* lg) {
  const int e = (m > 0.0 && isfinite(m)) ? ilogb(m) : 0;
  const int sh = (bits - 1) - e;
  *lg = (s2 > 0.0 && isfinite(s2)) ? (float)(0.5 * log2(s2) + sh) : (m > 0.0 ? INFINITY : -INFINITY);
  *sft = (int16_t)sh;
}

// Statistics of one row by one CTA of 256 threads.  Loads are issued four
// ahead; the accumulation order per thread is the plain strided order.
__device__ __forceinline__ void row_stats_one(const double* __restrict__ x, int64_t cols, int bits,
                                              int16_t* __restrict__ sft, float* __restrict__ lg) {
  double mx = 0.0, ss = 0.0;
  int64_t c = threadIdx.x;
  for (; c + 768 < cols; c += 1024) {
    const double v0 = __ldg(x + c), v1 = __ldg(x + c + 256), v2 = __ldg(x + c + 512), v3 = __ldg(x + c + 768);
    mx = fmax(mx, fabs(v0));
    ss = fma(v0, v0, ss);
    mx = fmax(mx, fabs(v1));
    ss = fma(v1, v1, ss);
    mx = fmax(mx, fabs(v2));
    ss = fma(v2, v2, ss);
    mx = fmax(mx, fabs(v3));
    ss = fma(v3, v3, ss);
  }
  for (; c < cols; c += 256) {
    const double v = __ldg(x + c);
    mx = fmax(mx, fabs(v));
    ss = fma(v, v, ss);
  }
  __shared__ double sm[256], sq[256];
  const int t = threadIdx.x;
  sm[t] = mx;
  sq[t] = ss;
  __syncthreads();
#pragma unroll
  for (int s = 128; s >= 32; s >>= 1) {
    if (t < s) {
      sm[t] = fmax(sm[t], sm[t + s]);
      sq[t] += sq[t + s];
    }
    __syncthreads();
  }
  if (t < 32) {
    double m = sm[t], q = sq[t];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      const double mo = __shfl_down_sync(0xFFFFFFFFu, m, s);
      const double qo = __shfl_down_sync(0xFFFFFFFFu, q, s);
      m = fmax(m, mo);
      q += qo;
    }
    if (t == 0) finish_stats(m, q, bits, sft, lg);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) row_stats_kernel(const double* __restrict__ X, int64_t rows,
                                                        int64_t cols, int bits, int16_t* __restrict__ sft,
                                                        float* __restrict__ lg) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) row_stats_one(X + r * cols, cols, bits, &sft[r], &lg[r]);
}

// Operand maxima of lg over both operands by one CTA of 256 threads (max is
// order independent), written to out[0..1].
__device__ __forceinline__ void maxlg_block(const float* lgA, int64_t m, const float* lgB, int64_t n, float* out) {
  float a = -INFINITY, b = -INFINITY;
  for (int64_t i = threadIdx.x; i < m; i += blockDim.x) a = fmaxf(a, __ldcg(lgA + i));
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) b = fmaxf(b, __ldcg(lgB + j));
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) {
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, s));
    b = fmaxf(b, __shfl_xor_sync(0xFFFFFFFFu, b, s));
  }
  __shared__ float sa[32], sb[32];
  if ((threadIdx.x & 31) == 0) {
    sa[threadIdx.x >> 5] = a;
    sb[threadIdx.x >> 5] = b;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    a = threadIdx.x < nw ? sa[threadIdx.x] : -INFINITY;
    b = threadIdx.x < nw ? sb[threadIdx.x] : -INFINITY;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, s));
      b = fmaxf(b, __shfl_xor_sync(0xFFFFFFFFu, b, s));
    }
    if (threadIdx.x == 0) {
      out[0] = a;
      out[1] = b;
    }
  }
}

// True in every thread of the CTA that finishes last among gridDim.x CTAs
// (counter zeroed before the launch).  The caller's results are published by
// the fence before the count, so the last CTA sees every CTA's writes.
__device__ __forceinline__ bool last_block_done(unsigned* counter) {
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last) __threadfence();
  return last;
}

// Both operands in the [rows, K] layout in one launch: CTAs take A's rows,
// then B's; the last CTA to finish takes the operand maxima.
__global__ void __launch_bounds__(256) rows_stats_both_kernel(const double* __restrict__ A, int64_t ra,
                                                              const double* __restrict__ B, int64_t rb,
                                                              int64_t cols, int bits, int16_t* __restrict__ sftA,
                                                              float* __restrict__ lgA, int16_t* __restrict__ sftB,
                                                              float* __restrict__ lgB, float* __restrict__ maxlg,
                                                              unsigned* __restrict__ counter) {
  for (int64_t r = blockIdx.x; r < ra + rb; r += gridDim.x) {
    if (r < ra) row_stats_one(A + r * cols, cols, bits, &sftA[r], &lgA[r]);
    else row_stats_one(B + (r - ra) * cols, cols, bits, &sftB[r - ra], &lgB[r - ra]);
  }
  if (last_block_done(counter)) maxlg_block(lgA, ra, lgB, rb, maxlg);
}

// Column partials over K slab `slab`: thread j of column block bx owns global
// column j of a [batch, K, N] operand (member j / N), reads coalesced across
// columns.  No barrier.
__device__ __forceinline__ void col_partial_one(const double* __restrict__ X, int64_t totalcols, int64_t K,
                                                int64_t N, int64_t kslab, int64_t bx, int64_t slab,
                                                double* __restrict__ pmax, double* __restrict__ pss) {
  const int64_t j = bx * 256 + threadIdx.x;
  if (j >= totalcols) return;
  const int64_t b = j / N, n = j - b * N;
  const int64_t k0 = slab * kslab;
  const int64_t k1 = min(k0 + kslab, K);
  const double* __restrict__ base = X + b * K * N + n;
  double mx = 0.0, ss = 0.0;
  int64_t k = k0;
  // eight loads in flight, accumulated in k order
  for (; k + 7 < k1; k += 8) {
    double v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) v[u] = __ldg(base + (k + u) * N);
#pragma unroll
    for (int u = 0; u < 8; u++) {
      mx = fmax(mx, fabs(v[u]));
      ss = fma(v[u], v[u], ss);
    }
  }
  for (; k < k1; k++) {
    const double v = __ldg(base + k * N);
    mx = fmax(mx, fabs(v));
    ss = fma(v, v, ss);
  }
  pmax[slab * totalcols + j] = mx;
  pss[slab * totalcols + j] = ss;
}

__global__ void __launch_bounds__(256) col_partial_kernel(const double* __restrict__ X, int64_t totalcols,
                                                          int64_t K, int64_t N, int64_t kslab,
                                                          double* __restrict__ pmax, double* __restrict__ pss) {
  col_partial_one(X, totalcols, K, N, kslab, blockIdx.x, blockIdx.y, pmax, pss);
}

// A's row statistics and B's column partials in one launch (the operands of
// an nt product): CTAs [0, ncb) take the (column block, K slab) pairs of B,
// gx column blocks per slab (each thread a long sequential chain, so they
// start first), the rest A's rows (stride nrb).
__global__ void __launch_bounds__(256) nt_stats_kernel(const double* __restrict__ A, int64_t rows, int64_t cols,
                                                       int bits, int16_t* __restrict__ sftA, float* __restrict__ lgA,
                                                       int64_t nrb, const double* __restrict__ B, int64_t totalcols,
                                                       int64_t K, int64_t N, int64_t kslab, int64_t gx, int64_t ncb,
                                                       double* __restrict__ pmax, double* __restrict__ pss) {
  const int64_t i = blockIdx.x;
  if (i < ncb) {
    col_partial_one(B, totalcols, K, N, kslab, i % gx, i / gx, pmax, pss);
  } else {
    for (int64_t r = i - ncb; r < rows; r += nrb) row_stats_one(A + r * cols, cols, bits, &sftA[r], &lgA[r]);
  }
}

// Column finalize of B plus the operand maxima by the last CTA to finish.
// One warp per column: lane l loads the partials of slabs l, l + 32, ...,
// and the warp adds them in slab order s = 0, 1, ... from shuffles (every
// lane runs the same chain; lane 0 writes).  Narrow operands have up to 128
// slabs, which a thread per column would walk one dependent load at a time.
__global__ void __launch_bounds__(256) col_finalize_maxlg_kernel(const double* __restrict__ pmax,
                                                                 const double* __restrict__ pss, int64_t totalcols,
                                                                 int nslab, int bits, int16_t* __restrict__ sft,
                                                                 float* __restrict__ lg, const float* lgA,
                                                                 int64_t ra, float* __restrict__ maxlg,
                                                                 unsigned* __restrict__ counter) {
  const int lane = threadIdx.x & 31;
  const int64_t j = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (j < totalcols) {
    double mx = 0.0, ss = 0.0;
    for (int s0 = 0; s0 < nslab; s0 += 32) {
      const int s = s0 + lane;
      const double pm = s < nslab ? __ldcg(pmax + (int64_t)s * totalcols + j) : 0.0;
      const double ps = s < nslab ? __ldcg(pss + (int64_t)s * totalcols + j) : 0.0;
      const int n = min(32, nslab - s0);
#pragma unroll
      for (int u = 0; u < 32; u++) {
        const double a = __shfl_sync(0xFFFFFFFFu, pm, u);
        const double b = __shfl_sync(0xFFFFFFFFu, ps, u);
        if (u < n) {
          mx = fmax(mx, a);
          ss += b;
        }
      }
    }
    if (lane == 0) finish_stats(mx, ss, bits, &sft[j], &lg[j]);
  }
  if (last_block_done(counter)) maxlg_block(lgA, ra, lg, totalcols, maxlg);
}

void col_slabs(int64_t NF, int64_t K, int64_t* kslab, int* nslab) {
  int64_t nsl0 = 131072 / std::max<int64_t>(NF, 1);
  nsl0 = std::min<int64_t>(std::max<int64_t>(nsl0, 1), 128);
  *kslab = (K + nsl0 - 1) / nsl0;
  *nslab = *kslab > 0 ? (int)((K + *kslab - 1) / *kslab) : 0;
}

void launch_rows_stats_both(const double* A, int64_t ra, const double* B, int64_t rb, int64_t cols, int bits,
                            int16_t* sftA, float* lgA, int16_t* sftB, float* lgB, float* maxlg, unsigned* counter,
                            cudaStream_t s) {
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ra + rb, 1 << 30));
  rows_stats_both_kernel<<<grid, 256, 0, s>>>(A, ra, B, rb, cols, bits, sftA, lgA, sftB, lgB, maxlg, counter);
}

void launch_nt_stats_maxlg(const double* A, int64_t ra, const double* X, int64_t batch, int64_t K, int64_t N,
                           int64_t kslab, int nslab, int bits, int16_t* sftA, float* lgA, int16_t* sft, float* lg,
                           double* pmax, double* pss, float* maxlg, unsigned* counter, cudaStream_t s) {
  const int64_t NF = batch * N;
  const int64_t gx = std::max<int64_t>(1, (NF + 255) / 256);
  const int64_t nrb = std::min<int64_t>(ra, 1 << 30);
  const int64_t ncb = (nslab > 0 && NF > 0) ? gx * nslab : 0;
  if (nrb + ncb > 0) {
    if (nrb + ncb <= INT32_MAX) {
      nt_stats_kernel<<<(unsigned)(nrb + ncb), 256, 0, s>>>(A, ra, K, bits, sftA, lgA, nrb, X, NF, K, N, kslab, gx,
                                                            ncb, pmax, pss);
    } else {
      if (ra > 0) row_stats_kernel<<<(unsigned)nrb, 256, 0, s>>>(A, ra, K, bits, sftA, lgA);
      if (ncb > 0) col_partial_kernel<<<dim3((unsigned)gx, nslab), 256, 0, s>>>(X, NF, K, N, kslab, pmax, pss);
    }
  }
  const unsigned gf = (unsigned)std::max<int64_t>(1, (NF + 7) / 8);   // a warp per column
  col_finalize_maxlg_kernel<<<gf, 256, 0, s>>>(pmax, pss, NF, nslab, bits, sft, lg, lgA, ra, maxlg, counter);
}

}  // namespace f64e
