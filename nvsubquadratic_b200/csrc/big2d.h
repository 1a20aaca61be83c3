// Parameters and dispatch of the fused large-grid 2D FFT convolution (big2d.cu):
// 2D, centred ("same") linear convolution with F0 = F1 = F in {192, 256}, N0, N1 <= 128,
// one filter shared by the batch.
#pragma once

#include <cuda_runtime.h>

namespace hyfft {

constexpr int kB2F = 256;             // longest FFT length per axis
constexpr int kB2FShort = 192;        // shorter length, where N + ceil(K/2) - 1 <= 192 on both axes
constexpr int kB2MaxN = 128;          // largest spatial extent

struct Big2DView {  // element (b, c, i0, i1) at b*bst + c*cst + i0*s0 + i1*s1
  const void* ptr;
  long long bst, cst, s0, s1;
};

struct Big2DParams {
  Big2DView x;        // conv input (x; dy for the adjoint); first input of the dK kernel
  Big2DView x2;       // second input of the dK kernel (dy)
  Big2DView y;        // conv output (y; dx for the adjoint)
  const float* D;     // [C] skip scale or null: out = round(round(conv) + round(D * x))
  Big2DView filt;     // float32 filter taps (b unused)
  Big2DView dfilt;    // float32 filter gradient (b unused)
  float2* Kh;         // [C][F/2+1][F] spectrum of the rolled filter (column bins outer)
  float2* T;          // [C][F][F/2+1] row-transform scratch of the filter / its gradient
  float2* G;          // [C][F/2+1][F] filter-gradient spectrum accumulator (zeroed by the host)
  int F;              // FFT length of both axes: 192 or 256
  int B, C, N0, N1, K0, K1;
  int conj;           // 1: multiply by conj(Kh) (the adjoint, dx = corr(dy, k))
  // Column spectra of the conv input, [B][C][F/2+1][F]: with zs_mode 1 the conv kernel
  // stores each column's forward transform there (the mixer's forward keeps z's); with
  // zs_mode 2 the adjoint conv kernel adds conj(Zs) * (its own input's column spectrum)
  // into G, the filter-gradient spectrum, so no separate dK kernel recomputes both.
  float2* Zs;
  int zs_mode;
};

enum Big2DOp { B2_KSPEC = 0, B2_CONV = 1, B2_DK = 2, B2_DFILT = 3 };

// Launch one step (HYFFT_OK, or HYFFT_ERR_CUDA). dtype: HYFFT_F32 / BF16 / F16 of x, x2, y.
int big2d_dispatch(int op, int dtype, const Big2DParams& p, cudaStream_t st);

}  // namespace hyfft
