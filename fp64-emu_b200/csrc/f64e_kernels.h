// Host-side launchers of the fp64-emu B200 kernels (one translation unit per
// stage).  All launches go to the caller's stream; none allocates memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "f64e_params.h"

namespace f64e {

// ---- sizing (f64e_sizing.cu) ----
void col_slabs(int64_t NF, int64_t K, int64_t* kslab, int* nslab);
// Both operands as [rows, K] in one launch, operand maxima included (counter
// zeroed before the launch).
void launch_rows_stats_both(const double* A, int64_t ra, const double* B, int64_t rb, int64_t cols, int bits,
                            int16_t* sftA, float* lgA, int16_t* sftB, float* lgB, float* maxlg, unsigned* counter,
                            cudaStream_t s);
// A's row statistics, B's column statistics ([batch, K, N]) and the operand
// maxima: one launch for the row statistics and column partials, one for the
// column finalize (whose last CTA takes the maxima; counter zeroed before).
void launch_nt_stats_maxlg(const double* A, int64_t ra, const double* X, int64_t batch, int64_t K, int64_t N,
                           int64_t kslab, int nslab, int bits, int16_t* sftA, float* lgA, int16_t* sft, float* lg,
                           double* pmax, double* pss, float* maxlg, unsigned* counter, cudaStream_t s);

// ---- extraction (f64e_extract.cu) ----
// Planes are K-major int8: plane t lives at planes + t * pstride (rows * Kp
// for an operand's own planes; more for a block of rows of larger planes),
// row r at + r * Kp, Kp = K rounded up to 16 (the pad columns are written as
// zeros).  Plane order: residues 0..P-1, then the two
// correction planes at P and P + 1, whose roles (hi or q) the caller picks.
struct ExtractArgs {
  const double* X;      // operand
  int64_t rows;         // rows of the K-major planes (batch * M, or batch * N)
  int64_t K, Kp;        // extracted K window and plane pitch
  int64_t ld, koff;     // [rows, K] layout: element (r, k) at X[r * ld + koff + k];
                        // [K, N] layout: element (k, n) of member b at X[(b * K + k) * ld + n]
  int64_t batch, N;     // [K, N] layout only: members and columns per member
  const int16_t* sft;   // per-row (or per-column) shifts before widening
  const float* maxlg;   // operand maxima of lg (WsHead::maxlg)
  int bits;             // requested operand width
  int use_corr;
  int hi_plane, q_plane;  // plane indices of the correction digits
  int8_t* planes;
  int64_t pstride;      // bytes from one plane to the next
  Span src, dst;        // the operand's elements, the planes' bytes (debug bounds build)
  int* status;          // status word (debug bounds build)
};
struct ExtractPair {
  ExtractArgs a[2];
};
void launch_extract_rows(const ExtractArgs& a, const ModTables& T, cudaStream_t s);  // X is [rows, K]
// Two [rows, K] operands with the same Kp in one launch.
void launch_extract_rows_pair(const ExtractArgs& a0, const ExtractArgs& a1, const ModTables& T, cudaStream_t s);
void launch_extract_cols(const ExtractArgs& a, const ModTables& T, cudaStream_t s);  // X is [batch, K, N]
// A [rows, K] operand (ra) and a [batch, K, N] operand (cb) in one launch.
void launch_extract_nt_pair(const ExtractArgs& ra, const ExtractArgs& cb, const ModTables& T, cudaStream_t s);

// ---- modular GEMM (f64e_gemm.cu) ----
struct GemmArgs {
  int M, N, batch, P;
  int Kp;              // plane pitch (bytes); the K extent seen by TMA
  int nkb;             // 128-wide K blocks per slot
  int corr_mode;       // 0 none, 1 one fused int32 plane (Ahi.Bq + Aq.Bhi), 2 two int32 planes
  int ldn;             // row pitch (elements) of the residue / correction outputs
  int8_t* res;         // [P * batch][M][ldn]
  int32_t* corr;       // [1 or 2][batch][M][ldn]
  int* status;
  uint64_t wait_limit_ns;
  Span res_span, corr_span;   // output ranges (debug bounds build)
};
// 3-D map (Kp, rows, zdim) of K-major int8 planes; consecutive z-slices are
// zrows * Kp bytes apart (zrows = rows when 0).
bool encode_plane_map(CUtensorMap* map, const void* base, int64_t zdim, int64_t rows, int64_t Kp, int box_rows,
                      int64_t zrows = 0);
int gemm_block_rows_a();
int gemm_block_rows_b();
int gemm_pair_block_rows();   // box rows of both operands in the CTA-pair kernel
bool gemm_use_pair(int M);    // CTA-pair kernel for tall problems
// A bounded wait that runs out on purpose (one thread, no copies in flight).
cudaError_t launch_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t s);
cudaError_t launch_residue_gemm(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& g, const ModTables& T,
                                int num_sms, cudaStream_t s);
cudaError_t launch_residue_gemm_pair(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& g,
                                     const ModTables& T, int num_sms, cudaStream_t s);

// ---- reference-form modular GEMM for validation (f64e_gemm_check.cu) ----
// Plain dp4a kernel with the same inputs and outputs as the tcgen05 kernel;
// used only by the library's self-check entry point.
void launch_residue_gemm_check(const int8_t* Apl, const int8_t* Bpl, int64_t MF, int64_t NF, const GemmArgs& g,
                               const ModTables& T, cudaStream_t s);

// ---- reconstruction (f64e_recon.cu) ----
struct ReconArgs {
  const int8_t* res;     // [P][batch * M][ldn]
  const void* corr;      // see corr_mode
  int corr_mode;         // 0 none, 1 int32 [MF][ldn], 2 two int32 planes, 3 int64 [MF][ldn]
  int64_t MF, M, N, ldn;
  const int16_t* sftA;   // [batch * M], before widening
  const int16_t* sftB;   // [batch * N], before widening
  const float* maxlg;
  int bits, exact;
  double* C;             // [batch * M][N], row pitch ldc
  int64_t ldc;
  Span res_span, corr_span, out_span;   // debug bounds build
  int* status;                          // debug bounds build
};
// beside_gemm: the launch runs beside a resident GEMM chunk (picks the form
// that takes less from it).
void launch_reconstruct(const ReconArgs& a, const ModTables& T, cudaStream_t s, bool beside_gemm = false,
                        int sms = 0);

}  // namespace f64e
