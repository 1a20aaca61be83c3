// Parameters and dispatch of the fused small-grid 2D Hyena kernels (fused.cu).
#pragma once

#include <cuda_runtime.h>

namespace hyfft {

struct Fused2DParams {
  const void* q;
  const void* k;
  const void* v;
  long long in_bst, in_pst;
  void* y;
  const void* dy;
  void* dq;
  void* dk;
  void* dv;
  long long out_bst, out_pst;
  const float* w;     // [3C][SK*SK]
  const float* bias;  // [3C] or null
  const float* D;     // [C]
  const float* filt;  // [C][K0][K1] (kspec)
  float2* Kbr;        // [C][F0][F1] bit-reversed spectrum of the rolled filter
  float2* G;          // [C][F0][F1] dK spectrum accumulator (backward)
  float* dfilt;       // [C][K0][K1]
  float* dD;          // [C]
  float* dw;          // [3C][SK*SK]
  float* db;          // [3C]
  int B, C, half;
  int K0, K1;
  int gate1, gate2;
  int* status;        // set non-zero by a kernel whose bounded wait timed out (workspace word)
  void* qs;           // short-conv outputs q', k', v' [B][N0*N1][C] (activation dtype): written by
  void* ks;           //   the FFT forward and read back by its backward instead of recomputing
  void* vs;           //   the three stencils; null: not kept
};

// Tensor-core (tcgen05) Toeplitz path for bf16 grids with both sides <= 16 (toeplitz.cu).
enum TpOp { TP_FWD = 0, TP_BWD = 1, TP_PROBE = 2 };
int tp2d_dispatch(int op, int N0, int N1, int SK, const Fused2DParams* p, cudaStream_t st);

// ops of fused2d_dispatch
enum FusedOp { FOP_KSPEC = 0, FOP_FWD = 1, FOP_BWD = 2, FOP_DFILT = 3, FOP_PROBE = 4 };

// Returns HYFFT_OK (launched, or supported for FOP_PROBE), HYFFT_ERR_UNSUPPORTED (not
// compiled for this shape: use the general engine) or HYFFT_ERR_CUDA.
int fused2d_dispatch(int op, int dtype, int N0, int N1, int F0, int F1, int SK, const Fused2DParams* p,
                     cudaStream_t st);

}  // namespace hyfft
