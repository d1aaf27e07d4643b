// K-segmented accumulation for depths past the single-launch int32 bound
// (reference: accum_res_kernel / accum_corr_kernel / reduce_planes_kernel and
// run_crt_bigk, fp64_emu.cu:815-847, 1485-1579).  Balanced residues of each
// 65536-deep segment sum into int32 (at most 128 segments of |r| <= 128),
// correction products into int64; one fold returns the balanced residue of
// the full-depth dot product, identical to a single-pass result.
#include "f64e_device.cuh"
#include "f64e_kernels.h"

namespace f64e {

__global__ void deepk_accum_kernel(const int8_t* __restrict__ res, int32_t* __restrict__ racc, int64_t nres,
                                   const int32_t* __restrict__ corr, int64_t* __restrict__ cacc, int64_t ncorr,
                                   int first) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nres; i += stride)
    racc[i] = (first ? 0 : racc[i]) + (int32_t)res[i];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < ncorr; i += stride)
    cacc[i] = (first ? 0 : cacc[i]) + (int64_t)corr[i];
}

__global__ void deepk_fold_kernel(const int32_t* __restrict__ racc, int8_t* __restrict__ res, int64_t per_plane,
                                  const ModTables T) {
  for (int t = blockIdx.y; t < T.P; t += gridDim.y) {
    const uint32_t p = T.p[t], md = T.mdiv[t], off = T.off[t];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per_plane;
         i += (int64_t)gridDim.x * blockDim.x)
      res[t * per_plane + i] = (int8_t)bal_mod_s32(racc[t * per_plane + i], p, md, off);
  }
}

void launch_deepk_accum(const int8_t* res, int32_t* racc, int64_t nres, const int32_t* corr, int64_t* cacc,
                        int64_t ncorr, int first, cudaStream_t s) {
  const int64_t n = std::max(nres, ncorr);
  if (n <= 0) return;
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 8192);
  deepk_accum_kernel<<<grid, 256, 0, s>>>(res, racc, nres, corr, cacc, ncorr, first);
}

void launch_deepk_fold(const int32_t* racc, int8_t* res, int64_t per_plane, const ModTables& T, cudaStream_t s) {
  if (per_plane <= 0) return;
  const dim3 grid((unsigned)std::min<int64_t>((per_plane + 255) / 256, 2048), (unsigned)T.P);
  deepk_fold_kernel<<<grid, 256, 0, s>>>(racc, res, per_plane, T);
}

}  // namespace f64e
