// Plain dp4a form of the modular GEMM with the tensor-core kernel's inputs,
// outputs and epilogue (one thread per output element).  Used only by the
// self-check entry point f64e_gemm_checked to localise a parity failure to the
// GEMM stage; it is never on the product path.
#include "f64e_device.cuh"
#include "f64e_kernels.h"

namespace f64e {

__global__ void residue_gemm_check_kernel(const int8_t* __restrict__ Apl, const int8_t* __restrict__ Bpl,
                                          const GemmArgs g, const ModTables T) {
  const int ncs = g.corr_mode == 1 ? g.batch : (g.corr_mode == 2 ? 2 * g.batch : 0);
  const int64_t nslots = (int64_t)g.P * g.batch + ncs;
  const int64_t per = (int64_t)g.M * g.N;
  const int64_t total = nslots * per;
  const int64_t kw = g.Kp / 4;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slot = idx / per, r = idx - slot * per;
    const int m = (int)(r / g.N), n = (int)(r - (int64_t)m * g.N);
    int z0, z1, nh, kind, t = 0;
    int64_t out;
    const int64_t slot_elems = (int64_t)g.M * g.ldn;
    if (slot < ncs) {
      kind = 1;
      if (g.corr_mode == 1) {
        z0 = g.P * g.batch + (int)slot;
        z1 = (g.P + 1) * g.batch + (int)slot;
        nh = 2;
        out = slot * slot_elems;
      } else {
        const int h = (int)slot / g.batch, b = (int)slot - h * g.batch;
        z0 = z1 = (g.P + h) * g.batch + b;
        nh = 1;
        out = (int64_t)(h * g.batch + b) * slot_elems;
      }
    } else {
      const int s = (int)(slot - ncs);
      kind = 0;
      t = s / g.batch;
      z0 = z1 = s;
      nh = 1;
      out = (int64_t)s * slot_elems;
    }
    int acc = 0;
    for (int h = 0; h < nh; h++) {
      const int z = h ? z1 : z0;
      const int* a = reinterpret_cast<const int*>(Apl + ((int64_t)z * g.M + m) * g.Kp);
      const int* b = reinterpret_cast<const int*>(Bpl + ((int64_t)z * g.N + n) * g.Kp);
      for (int64_t k = 0; k < kw; k++) acc = __dp4a(a[k], b[k], acc);
    }
    if (kind == 0)
      g.res[out + (int64_t)m * g.ldn + n] = (int8_t)bal_mod_s32(acc, T.p[t], T.mdiv[t], T.off[t]);
    else
      g.corr[out + (int64_t)m * g.ldn + n] = acc;
  }
}

void launch_residue_gemm_check(const int8_t* Apl, const int8_t* Bpl, int64_t, int64_t, const GemmArgs& g,
                               const ModTables& T, cudaStream_t s) {
  const int ncs = g.corr_mode == 1 ? g.batch : (g.corr_mode == 2 ? 2 * g.batch : 0);
  const int64_t total = ((int64_t)g.P * g.batch + ncs) * g.M * g.N;
  if (total <= 0) return;
  const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 1 << 20);
  residue_gemm_check_kernel<<<grid, 256, 0, s>>>(Apl, Bpl, g, T);
}

}  // namespace f64e
