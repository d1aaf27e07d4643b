// Host build of the FP64-pipe CRT reconstruction (fp64-emu_b200/csrc/
// f64e_crt64.cuh) for the CPU tests: the same arithmetic as the device kernel
// on host doubles (IEEE fused multiply-add), driven from Python through
// ctypes and compared with exact integer arithmetic.
#include <cstdint>

#include "f64e_crt64.cuh"

extern "C" {

// Tables of a modulus list; returns 1 when the form applies (M < 2^120).
int crt64_check_tables(const int32_t* primes, int P, f64e::Crt64Tables* out) {
  if (!f64e::crt64_build(primes, P, 0.0f, out)) return 0;
  f64e::crt64_device_scale(out);   // the device kernel's scaling
  return 1;
}

int crt64_check_size() { return (int)sizeof(f64e::Crt64Tables); }

// out[i] = ldexp(RN(V_i + corr[i] 2^cshift), sh[i]) for the balanced residues
// res[i * P + t] of element i, as the device kernel computes it (u_t as the
// subnormal u_t 2^-1042 from the biased byte, three limb sums in the device
// scaling, crt64_finish_fast with crt64_finish for the elements it declines).
// Also counts the declined elements (*slow) so the tests can see both paths.
void crt64_check_run(const f64e::Crt64Tables* T, const int8_t* res, const double* corr, const int32_t* sh,
                     int cshift, int64_t n, double* out, int64_t* slow) {
  if (slow) *slow = 0;
  const double csc = f64e::crt64_pow2(cshift - 40);
  for (int64_t i = 0; i < n; i++) {
    double a0 = T->z[0], a1 = T->z[1], a2 = T->z[2];
    for (int t = 0; t < T->P; t++) {
      const uint32_t u = (uint32_t)(uint8_t)res[i * T->P + t] ^ 0x80u;
      const double du = f64e::crt64_from_bits((uint64_t)u << 32);   // the subnormal u 2^-1042
      a0 = std::fma(du, T->e[t][0], a0);
      a1 = std::fma(du, T->e[t][1], a1);
      a2 = std::fma(du, T->e[t][2], a2);
    }
    a0 *= 0x1p64;
    a1 *= 0x1p64;
    a2 *= 0x1p64;
    // as the device kernel: the common path, else the exact side path
    double r;
    if (!f64e::crt64_finish_fast(*T, a0, a1, a2, corr[i], csc, sh[i], &r)) {
      r = f64e::crt64_finish(*T, a0, a1, a2, corr[i], csc, sh[i]);
      if (slow) ++*slow;
    }
    out[i] = r;
  }
}
}
