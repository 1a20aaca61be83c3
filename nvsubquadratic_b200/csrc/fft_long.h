// Host interface of the long 1D (four-step) channel-innermost passes (fft_long.cu).
#pragma once

#include <cuda_runtime.h>

#include "fft_pass.cuh"

namespace hyfft {

// Whether launch_long_pass takes this pass, and its launch (HYFFT_ERR_UNSUPPORTED: nothing
// launched, the caller falls back to another pass kernel).
bool long_pass_applies(const PassDesc& d, int im, int om, int tin, int tout);
int launch_long_pass(const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st);

// Backward product pass over the second four-step axis (see fft_long_bwd_kernel).
struct LongBwdDesc {
  const float2* sx;
  float2* sdy;
  const float2* kh;
  float2* dkh;
  long long pst, tst, ost;  // spectrum strides of the pair, the point (n_b / k_b) and the line's k_a
  long long k_pst;          // filter pair stride (0: one filter for every pair)
  long long nlines;         // (P / pl) * Fa * C
  int C, Fa, pl;            // channels, first-axis extent, pairs summed per line
  int tw_logF;              // inverse post-twiddle e^{+2 pi i n_b k_a / 2^tw_logF}
  float scale;              // 1 / F of the second axis
};

int launch_long_bwd(const LongBwdDesc& d, int fb, cudaStream_t st);

}  // namespace hyfft
