// Spectral pointwise kernels and small reductions of the general engine.
#pragma once

#include "common.cuh"

namespace hyfft {

// S[p, f, c] *= Kh[kb(p), f, c]  over the full spectrum (channels innermost).
// kb(p) = 0 for a shared kernel, p for per-sample kernels (unpacked pairs).
__global__ void spec_mul_kernel(float2* __restrict__ S, const float2* __restrict__ Kh, long long per_pair,
                                int P, int shared_kernel) {
  const long long n = per_pair * P;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / per_pair, r = i - p * per_pair;
    const float2 k = Kh[(shared_kernel ? 0 : p) * per_pair + r];
    S[i] = cmul(S[i], k);
  }
}

// Backward spectra: dKh[kb, f, c] = sum_{p in kb} Sdy[p, f, c] * conj(Sx[p, f, c]),
// then Sdy *= conj(Kh). With packed pairs the real part of the inverse of the sum is
// sum_b corr(dy_b, x_b); with a shared kernel the sum runs over all pairs.
__global__ void spec_bwd_kernel(float2* __restrict__ Sdy, const float2* __restrict__ Sx,
                                const float2* __restrict__ Kh, float2* __restrict__ dKh,
                                long long per_pair, int P, int shared_kernel) {
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < per_pair; r += (long long)gridDim.x * blockDim.x) {
    if (shared_kernel) {
      const float2 k = Kh[r];
      float2 acc = make_float2(0.f, 0.f);
      for (int p = 0; p < P; ++p) {
        const long long i = (long long)p * per_pair + r;
        const float2 g = Sdy[i];
        const float2 x = Sx[i];
        acc = cadd(acc, cmulc(g, x));
        Sdy[i] = cmulc(g, k);
      }
      dKh[r] = acc;
    } else {
      for (int p = 0; p < P; ++p) {
        const long long i = (long long)p * per_pair + r;
        const float2 g = Sdy[i];
        dKh[i] = cmulc(g, Sx[i]);
        Sdy[i] = cmulc(g, Kh[i]);
      }
    }
  }
}

// dD[c] = sum_{b, s} dy[b, c, s] * x[b, c, s] for layout BHL (cst = S) or BLH (cst = 1),
// accumulated with one atomic per channel per CTA into `out` (zeroed by the host).
// BLH: grid (ceil(C / 32), row blocks), lanes over channels, warps over (b, s) rows.
// BHL: grid (C, B), the CTA sums one contiguous (b, c) line of S elements.
template <typename T>
__global__ void dshortcut_kernel(const T* __restrict__ dy, const T* __restrict__ x, float* __restrict__ out,
                                 int B, int C, long long S, int blh) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;  // 256 threads: 8 warps
  if (blh) {
    const int c = blockIdx.x * 32 + lane;
    float acc = 0.f;
    if (c < C) {
      for (long long r = (long long)blockIdx.y * 8 + w; r < (long long)B * S; r += (long long)gridDim.y * 8) {
        const long long i = r * C + c;
        acc = fmaf(DT<T>::load(dy + i), DT<T>::load(x + i), acc);
      }
    }
    red[w][lane] = acc;
    __syncthreads();
    if (w == 0) {
      float s = 0.f;
      for (int j = 0; j < 8; ++j) s += red[j][lane];
      if (c < C) atomicAdd(out + c, s);
    }
  } else {
    const int c = blockIdx.x, b = blockIdx.y;
    const long long base = ((long long)b * C + c) * S;
    float a = 0.f;
    for (long long s = threadIdx.x; s < S; s += blockDim.x) a = fmaf(DT<T>::load(dy + base + s), DT<T>::load(x + base + s), a);
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) red[w][0] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int j = 0; j < 8; ++j) s += red[j][0];
      atomicAdd(out + c, s);
    }
  }
}

}  // namespace hyfft
