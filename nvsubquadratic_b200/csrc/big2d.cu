// Fused large-grid 2D FFT convolution: y = crop(IFFT2(FFT2(x) * Kh)) (+ D-skip), its
// adjoint and its filter gradient, for F0 = F1 = 256 and N0, N1 <= 128 (e.g. the
// 128x128 HyenaND grid), one CTA per (batch item, channel).
//
// Data path of one CTA: the rows of x (real, read once from HBM through any strided
// view, BHL or channels-last) are transformed two at a time as one complex 256-point
// FFT and split into their half spectra (129 bins), which stay in shared memory
// (N0 x 129 complex float32, 132 KB); each of the 129 columns is transformed (256
// points, rows >= N0 are zero), multiplied by the filter spectrum, inverted and
// cropped back in place; the rows are inverted two at a time and written once.
// Every activation crosses HBM once per pass; only the filter spectrum (read from
// L2) is shared between CTAs.
//
// The filter is rolled by its crop offset (tap (a, b) at ((a - K0/2) mod 256,
// (b - K1/2) mod 256)), so the reference's centred crop
// (nvsubquadratic/ops/fftconv.py:714-725) becomes the window [0, N) of every axis and
// the adjoint is the same kernel with conj(Kh). 256 >= N + K/2 on each axis keeps the
// circular convolution equal to the linear one on that window.
//
// FFT primitive: a 256-point complex transform by 16 lanes (half a warp), lane l
// holding points l + 16 m in registers (m = 0..15), as two radix-16 register stages
// around one transpose through a padded per-group shared-memory tile; input and
// output use the same lane/register distribution.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "big2d.h"
#include "common.cuh"
#include "fft_pass.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;

namespace {

constexpr int kThreads = 256;                // filter-spectrum / filter-gradient kernels
constexpr int kGroups = kThreads / 16;
constexpr int kBigThreads = 512;             // per-image kernels (one CTA per SM, 16 warps)
constexpr int kBigGroups = kBigThreads / 16;
constexpr int kScLd = 17;                    // padded row of the 16 x 16 transpose tile
constexpr int kScSize = 16 * kScLd;          // float2 per group

// 16-point DFT (natural order in and out) with compile-time pruning: ZIN = inputs
// 8..15 are zero; HOUT = only outputs 0..7 are needed (the others are left unset).
template <bool ZIN, bool HOUT>
__device__ __forceinline__ void dft16p(float2 (&v)[16], float dir) {
  constexpr float c1 = 0.92387953251128674f, s1 = 0.38268343236508978f, h = 0.70710678118654752f;
#pragma unroll
  for (int n2 = 0; n2 < 4; ++n2) {
    if constexpr (ZIN) {
      const float2 a = v[n2], b = v[n2 + 4];
      const float2 jb = make_float2(-dir * b.y, dir * b.x);
      v[n2] = cadd(a, b);
      v[n2 + 4] = cadd(a, jb);
      v[n2 + 8] = csub(a, b);
      v[n2 + 12] = csub(a, jb);
    } else {
      dft4(v[n2], v[n2 + 4], v[n2 + 8], v[n2 + 12], dir);
    }
  }
  const float2 w1 = make_float2(c1, dir * s1), w2 = make_float2(h, dir * h), w3 = make_float2(s1, dir * c1);
  const float2 w6 = make_float2(-h, dir * h), w9 = make_float2(-c1, -dir * s1);
  v[5] = cmul(v[5], w1);
  v[9] = cmul(v[9], w2);
  v[13] = cmul(v[13], w3);
  v[6] = cmul(v[6], w2);
  v[10] = make_float2(-dir * v[10].y, dir * v[10].x);
  v[14] = cmul(v[14], w6);
  v[7] = cmul(v[7], w3);
  v[11] = cmul(v[11], w6);
  v[15] = cmul(v[15], w9);
  float2 o[16];
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1) {
    const float2 a0 = v[4 * k1], a1 = v[4 * k1 + 1], a2 = v[4 * k1 + 2], a3 = v[4 * k1 + 3];
    const float2 t0 = cadd(a0, a2), t1 = csub(a0, a2), t2 = cadd(a1, a3), t3 = csub(a1, a3);
    const float2 jt3 = make_float2(-dir * t3.y, dir * t3.x);
    o[k1] = cadd(t0, t2);
    o[k1 + 4] = cadd(t1, jt3);
    if constexpr (!HOUT) {
      o[k1 + 8] = csub(t0, t2);
      o[k1 + 12] = csub(t1, jt3);
    }
  }
#pragma unroll
  for (int k = 0; k < (HOUT ? 8 : 16); ++k) v[k] = o[k];
}

__device__ __forceinline__ void init_tw(float2* tw) {
  for (int j = threadIdx.x; j < kB2F; j += blockDim.x) {
    float s, c;
    sincospif(2.0f * (float)j / (float)kB2F, &s, &c);
    tw[j] = make_float2(c, s);
  }
}

// In place: v[m] = x[l + 16 m] -> v[m] = X[l + 16 m], X[k] = sum_n x[n] e^{dir 2 pi i n k / 256}.
// ZIN: x[n] = 0 for n >= 128 (registers 8..15 hold zeros); HOUT: only X[k], k < 128
// (registers 0..7) are produced. Called by all 32 lanes of the warp together.
template <bool ZIN = false, bool HOUT = false>
__device__ __forceinline__ void fft256(float2 (&v)[16], float2* sc, const float2* tw, int l, float dir) {
  dft16p<ZIN, false>(v, dir);
#pragma unroll
  for (int k2 = 1; k2 < 16; ++k2) {
    const float2 w = tw[l * k2];
    v[k2] = cmul(v[k2], make_float2(w.x, dir * w.y));
  }
  __syncwarp();
#pragma unroll
  for (int k2 = 0; k2 < 16; ++k2) sc[l * kScLd + k2] = v[k2];
  __syncwarp();
#pragma unroll
  for (int n1 = 0; n1 < 16; ++n1) v[n1] = sc[n1 * kScLd + l];
  dft16p<false, HOUT>(v, dir);
}

// After fft256 of u = a + i b (a, b real lines): the half spectra A[j], B[j] for the
// bins j = l + 16 m <= 128, from U[j] and U[256 - j] (held by lane (16 - l) & 15).
// All lanes of the warp must call it.
__device__ __forceinline__ void split_pair(const float2 (&v)[16], int l, float2 (&A)[9], float2 (&Bv)[9]) {
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const float2 s = (l == 0) ? v[(16 - m) & 15] : v[15 - m];
    float2 p;
    p.x = __shfl_sync(0xffffffffu, s.x, (16 - l) & 15, 16);
    p.y = __shfl_sync(0xffffffffu, s.y, (16 - l) & 15, 16);
    if (m <= 8) {
      const float2 u = v[m];
      // A = (U + conj(P)) / 2, B = (U - conj(P)) / (2i)
      A[m] = make_float2(0.5f * (u.x + p.x), 0.5f * (u.y - p.y));
      Bv[m] = make_float2(0.5f * (u.y + p.y), -0.5f * (u.x - p.x));
    }
  }
}

template <typename T>
__device__ __forceinline__ float ldv(const Big2DView& v, int b, int c, int i0, int i1) {
  return DT<T>::load(reinterpret_cast<const T*>(v.ptr) + (long long)b * v.bst + (long long)c * v.cst +
                     (long long)i0 * v.s0 + (long long)i1 * v.s1);
}

// ---------------------------------------------------------------- filter spectrum
// Row transforms of the rolled filter: T[c][r][j], r < 256, j <= 128. grid (C, 8).
__global__ void __launch_bounds__(kThreads) b2_kspec_rows(const Big2DParams p) {
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[kB2F];
  init_tw(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int r0 = 2 * (blockIdx.y * kGroups + g);
  const int h0 = p.K0 / 2, h1 = p.K1 / 2;
  const int a0 = (r0 + h0) & (kB2F - 1), a1 = (r0 + 1 + h0) & (kB2F - 1);
  const float* f = reinterpret_cast<const float*>(p.filt.ptr) + (long long)c * p.filt.cst;
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int bb = (l + 16 * m + h1) & (kB2F - 1);
    const bool inb = bb < p.K1;
    v[m].x = (inb && a0 < p.K0) ? f[a0 * p.filt.s0 + bb * p.filt.s1] : 0.f;
    v[m].y = (inb && a1 < p.K0) ? f[a1 * p.filt.s0 + bb * p.filt.s1] : 0.f;
  }
  fft256(v, sc + g * kScSize, tw, l, -1.f);
  float2 A[9], Bv[9];
  split_pair(v, l, A, Bv);
  float2* t0 = p.T + ((long long)c * kB2F + r0) * kB2H;
#pragma unroll
  for (int m = 0; m <= 8; ++m) {
    const int j = l + 16 * m;
    if (j < kB2H) {
      t0[j] = A[m];
      t0[kB2H + j] = Bv[m];
    }
  }
}

// Column transforms: Kh[c][j][i] = sum_r T[c][r][j] e^{-2 pi i r i / 256}. grid (C, 9).
__global__ void __launch_bounds__(kThreads) b2_kspec_cols(const Big2DParams p) {
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[kB2F];
  init_tw(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int j = blockIdx.y * kGroups + g;
  const bool act = j < kB2H;
  const float2* t = p.T + (long long)c * kB2F * kB2H + (act ? j : 0);
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) v[m] = act ? t[(long long)(l + 16 * m) * kB2H] : make_float2(0.f, 0.f);
  fft256(v, sc + g * kScSize, tw, l, -1.f);
  if (act) {
    float2* o = p.Kh + ((long long)c * kB2H + j) * kB2F;
#pragma unroll
    for (int m = 0; m < 16; ++m) o[l + 16 * m] = v[m];
  }
}

// ---------------------------------------------------------------- row pass helpers
// Lane l's points of rows [2 pr, 2 pr + 1] of image (b, c): v[m] = x[r0][l + 16 m] +
// i x[r1][l + 16 m] for m < 8 (positions >= 128 >= N1 are zero), zeros for a pair past N0.
template <typename T>
__device__ __forceinline__ void rows_load(const Big2DView& in, int b, int c, int N0, int N1, int pr, int l,
                                          float2 (&v)[8]) {
  const int npairs = (N0 + 1) >> 1;
  const bool act = pr < npairs;
  const int r0 = 2 * pr, r1 = r0 + 1;
  const bool has1 = act && r1 < N0;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int n = l + 16 * m;
    v[m] = make_float2(0.f, 0.f);
    if (act && n < N1) {
      v[m].x = ldv<T>(in, b, c, r0, n);
      if (has1) v[m].y = ldv<T>(in, b, c, r1, n);
    }
  }
}

// Forward row transforms of rows [2 pr, 2 pr + 1] of input view `in` for image (b, c):
// bins j in [jlo, jlo + jn) go to dst[r * ld + j - jlo]. All threads of the CTA call it.
// The next round's rows are loaded before this round's transform, so their global-memory
// latency overlaps the arithmetic.
template <typename T>
__device__ __forceinline__ void rows_forward(const Big2DView& in, int b, int c, int N0, int N1, float2* dst, int ld,
                                             int jlo, int jn, float2* sc, const float2* tw) {
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int npairs = (N0 + 1) >> 1;
  const int rounds = (npairs + kBigGroups - 1) / kBigGroups;
  float2 nxt[8];
  rows_load<T>(in, b, c, N0, N1, g, l, nxt);
  for (int rb = 0; rb < rounds; ++rb) {
    const int pr = rb * kBigGroups + g;
    const bool act = pr < npairs;
    const int r0 = 2 * pr, r1 = r0 + 1;
    const bool has1 = act && r1 < N0;
    float2 v[16];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      v[m] = nxt[m];
      v[m + 8] = make_float2(0.f, 0.f);
    }
    if (rb + 1 < rounds) rows_load<T>(in, b, c, N0, N1, pr + kBigGroups, l, nxt);
    fft256<true, false>(v, sc, tw, l, -1.f);
    float2 A[9], Bv[9];
    split_pair(v, l, A, Bv);
    if (act) {
#pragma unroll
      for (int m = 0; m <= 8; ++m) {
        const int j = l + 16 * m - jlo;
        if (j >= 0 && j < jn && j + jlo < kB2H) {
          dst[r0 * ld + j] = A[m];
          if (has1) dst[r1 * ld + j] = Bv[m];
        }
      }
    }
  }
}

// ---------------------------------------------------------------- convolution
template <typename T>
__global__ void __launch_bounds__(kBigThreads) b2_conv(const Big2DParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float2* A = reinterpret_cast<float2*>(smem);                  // [128][129]
  float2* sc = A + kB2MaxN * kB2H;                               // [32][272]
  float2* tw = sc + kBigGroups * kScSize;                           // [256]
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  // channels-last inputs: neighbouring channels of one image run together (shared
  // sectors); channel-major: the batch items of one channel do (shared filter spectrum)
  const bool cfast = p.x.cst == 1;
  const int c = cfast ? blockIdx.x : blockIdx.y, b = cfast ? blockIdx.y : blockIdx.x;
  const int N0 = p.N0, N1 = p.N1;
  float2* mysc = sc + g * kScSize;
  init_tw(tw);
  __syncthreads();

  rows_forward<T>(p.x, b, c, N0, N1, A, kB2H, 0, kB2H, mysc, tw);
  __syncthreads();

  // columns: transform, * Kh (or conj), inverse, keep rows [0, N0); each round's
  // filter-spectrum column (an L2 read) is loaded one round ahead, right after the
  // previous column has consumed its own, so the load overlaps an inverse and a forward
  // transform
  const float2* kh = p.Kh + (long long)c * kB2H * kB2F;
  const float cj = p.conj ? -1.f : 1.f;
  constexpr int kColRounds = (kB2H + kBigGroups - 1) / kBigGroups;
  float2 kv[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) kv[m] = g < kB2H ? __ldg(kh + (long long)g * kB2F + l + 16 * m) : make_float2(0.f, 0.f);
  for (int rb = 0; rb < kColRounds; ++rb) {
    const int j = rb * kBigGroups + g;
    const bool act = j < kB2H;
    float2 v[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int r = l + 16 * m;
      v[m] = (m < 8 && act && r < N0) ? A[r * kB2H + j] : make_float2(0.f, 0.f);
    }
    fft256<true, false>(v, mysc, tw, l, -1.f);
    if (p.zs_mode != 0 && act) {
      float2* zc = p.Zs + (((long long)b * p.C + c) * kB2H + j) * kB2F + l;
      if (p.zs_mode == 1) {
#pragma unroll
        for (int m = 0; m < 16; ++m) zc[16 * m] = v[m];
      } else {
        // G[c][j][i] += conj(Z[b][c][j][i]) * DY[j][i] (the per-image term of the filter gradient)
        float2* gc = p.G + ((long long)c * kB2H + j) * kB2F + l;
        float2 z[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) z[m] = __ldcs(zc + 16 * m);
#pragma unroll
        for (int m = 0; m < 16; ++m) atomicAdd(gc + 16 * m, cmulc(v[m], z[m]));
      }
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      float2 k = kv[m];
      k.y *= cj;
      v[m] = cmul(v[m], k);
    }
    const int jn = j + kBigGroups;
    if (rb + 1 < kColRounds) {
#pragma unroll
      for (int m = 0; m < 16; ++m) kv[m] = jn < kB2H ? __ldg(kh + (long long)jn * kB2F + l + 16 * m) : make_float2(0.f, 0.f);
    }
    fft256<false, true>(v, mysc, tw, l, 1.f);
    if (act) {
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int r = l + 16 * m;
        if (r < N0) A[r * kB2H + j] = v[m];
      }
    }
  }
  __syncthreads();

  // inverse rows two at a time, epilogue
  const float scale = 1.0f / (float)(kB2F * kB2F);
  const int npairs = (N0 + 1) >> 1;
  const float Dc = p.D ? p.D[c] : 0.f;
  T* yo = reinterpret_cast<T*>(const_cast<void*>(p.y.ptr)) + (long long)b * p.y.bst + (long long)c * p.y.cst;
  for (int rb = 0; rb < (npairs + kBigGroups - 1) / kBigGroups; ++rb) {
    const int pr = rb * kBigGroups + g;
    const bool act = pr < npairs;
    const int r0 = 2 * pr, r1 = r0 + 1;
    const bool has1 = act && r1 < N0;
    float2 v[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int j = l + 16 * m;
      float2 a = make_float2(0.f, 0.f), bb = make_float2(0.f, 0.f);
      if (act) {
        if (j < kB2H) {
          a = A[r0 * kB2H + j];
          if (has1) bb = A[r1 * kB2H + j];
        } else {
          a = A[r0 * kB2H + (kB2F - j)];
          a.y = -a.y;
          if (has1) {
            bb = A[r1 * kB2H + (kB2F - j)];
            bb.y = -bb.y;
          }
        }
      }
      v[m] = make_float2(a.x - bb.y, a.y + bb.x);  // a + i b
    }
    // the D-skip inputs of these two rows, loaded before the transform
    float2 xs[8];
    if (p.D) rows_load<T>(p.x, b, c, N0, N1, pr, l, xs);
    fft256<false, true>(v, mysc, tw, l, 1.f);
    if (act) {
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int n = l + 16 * m;
        if (n < N1) {
          float o0 = DT<T>::round(v[m].x * scale), o1 = DT<T>::round(v[m].y * scale);
          if (p.D) {
            o0 = DT<T>::round(o0 + DT<T>::round(Dc * xs[m].x));
            if (has1) o1 = DT<T>::round(o1 + DT<T>::round(Dc * xs[m].y));
          }
          DT<T>::store(yo + (long long)r0 * p.y.s0 + (long long)n * p.y.s1, o0);
          if (has1) DT<T>::store(yo + (long long)r1 * p.y.s0 + (long long)n * p.y.s1, o1);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- filter gradient
// G[c][j][i] += conj(X[i][j]) * DY[i][j] for one image, in two halves of the column
// bins (j < 65, then j >= 65) so that both row-transformed inputs fit in shared memory.
template <typename T>
__global__ void __launch_bounds__(kBigThreads) b2_dk(const Big2DParams p) {
  constexpr int HALF = 65;
  extern __shared__ __align__(16) unsigned char smem[];
  float2* Ax = reinterpret_cast<float2*>(smem);                 // [128][65]
  float2* Ay = Ax + kB2MaxN * HALF;                              // [128][65]
  float2* sc = Ay + kB2MaxN * HALF;
  float2* tw = sc + kBigGroups * kScSize;
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  // channel fastest: concurrent CTAs accumulate into different channels' spectra
  const int c = blockIdx.x, b = blockIdx.y;
  const int N0 = p.N0, N1 = p.N1;
  float2* mysc = sc + g * kScSize;
  init_tw(tw);
  __syncthreads();
  float2* G = p.G + (long long)c * kB2H * kB2F;
  for (int h = 0; h < 2; ++h) {
    const int jlo = h ? HALF : 0, jn = h ? kB2H - HALF : HALF;
    rows_forward<T>(p.x, b, c, N0, N1, Ax, HALF, jlo, jn, mysc, tw);
    rows_forward<T>(p.x2, b, c, N0, N1, Ay, HALF, jlo, jn, mysc, tw);
    __syncthreads();
    for (int rb = 0; rb < (jn + kBigGroups - 1) / kBigGroups; ++rb) {
      const int jj = rb * kBigGroups + g;
      const bool act = jj < jn;
      float2 x[16], y[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int r = l + 16 * m;
        const bool in = m < 8 && act && r < N0;
        x[m] = in ? Ax[r * HALF + jj] : make_float2(0.f, 0.f);
        y[m] = in ? Ay[r * HALF + jj] : make_float2(0.f, 0.f);
      }
      fft256<true, false>(x, mysc, tw, l, -1.f);
      fft256<true, false>(y, mysc, tw, l, -1.f);
      if (act) {
        float2* gc = G + (long long)(jlo + jj) * kB2F;
#pragma unroll
        for (int m = 0; m < 16; ++m) atomicAdd(gc + l + 16 * m, cmulc(y[m], x[m]));
      }
    }
    __syncthreads();
  }
}

// Inverse of G along axis 0: T[c][r][j] = sum_i G[c][j][i] e^{+2 pi i r i / 256}. grid (C, 9).
__global__ void __launch_bounds__(kThreads) b2_dfilt_cols(const Big2DParams p) {
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[kB2F];
  init_tw(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int j = blockIdx.y * kGroups + g;
  const bool act = j < kB2H;
  const float2* gc = p.G + ((long long)c * kB2H + (act ? j : 0)) * kB2F;
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) v[m] = act ? gc[l + 16 * m] : make_float2(0.f, 0.f);
  fft256(v, sc + g * kScSize, tw, l, 1.f);
  if (act) {
    float2* t = p.T + (long long)c * kB2F * kB2H + j;
#pragma unroll
    for (int m = 0; m < 16; ++m) t[(long long)(l + 16 * m) * kB2H] = v[m];
  }
}

// Inverse along axis 1 (two rows at a time as one complex line), un-roll, crop to the
// filter taps: dfilt[c][a][b]. grid (C, 8).
__global__ void __launch_bounds__(kThreads) b2_dfilt_rows(const Big2DParams p) {
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[kB2F];
  init_tw(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int r0 = 2 * (blockIdx.y * kGroups + g), r1 = r0 + 1;
  const float2* t0 = p.T + ((long long)c * kB2F + r0) * kB2H;
  const float2* t1 = t0 + kB2H;
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = l + 16 * m;
    float2 a, bb;
    if (j < kB2H) {
      a = t0[j];
      bb = t1[j];
    } else {
      a = t0[kB2F - j];
      bb = t1[kB2F - j];
      a.y = -a.y;
      bb.y = -bb.y;
    }
    v[m] = make_float2(a.x - bb.y, a.y + bb.x);
  }
  fft256(v, sc + g * kScSize, tw, l, 1.f);
  const float scale = 1.0f / (float)(kB2F * kB2F);
  const int h0 = p.K0 / 2, h1 = p.K1 / 2;
  const int a0 = (r0 + h0) & (kB2F - 1), a1 = (r1 + h0) & (kB2F - 1);
  float* d = reinterpret_cast<float*>(const_cast<void*>(p.dfilt.ptr)) + (long long)c * p.dfilt.cst;
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int bb = (l + 16 * m + h1) & (kB2F - 1);
    if (bb < p.K1) {
      if (a0 < p.K0) d[a0 * p.dfilt.s0 + bb * p.dfilt.s1] = v[m].x * scale;
      if (a1 < p.K0) d[a1 * p.dfilt.s0 + bb * p.dfilt.s1] = v[m].y * scale;
    }
  }
}

constexpr size_t kConvSmem = sizeof(float2) * ((size_t)kB2MaxN * kB2H + kBigGroups * kScSize + kB2F);
constexpr size_t kDkSmem = sizeof(float2) * ((size_t)2 * kB2MaxN * 65 + kBigGroups * kScSize + kB2F);
static_assert(kConvSmem <= 227 * 1024 && kDkSmem <= 227 * 1024, "shared memory per CTA");

template <typename T>
int run_t(int op, const Big2DParams& p, cudaStream_t st) {
  if (op == B2_CONV) {
    if (!kernel_smem_once((const void*)b2_conv<T>, kConvSmem)) return HYFFT_ERR_CUDA;
    b2_conv<T><<<p.x.cst == 1 ? dim3(p.C, p.B) : dim3(p.B, p.C), kBigThreads, kConvSmem, st>>>(p);
  } else {
    if (!kernel_smem_once((const void*)b2_dk<T>, kDkSmem)) return HYFFT_ERR_CUDA;
    b2_dk<T><<<dim3(p.C, p.B), kBigThreads, kDkSmem, st>>>(p);
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
}

}  // namespace

int big2d_dispatch(int op, int dtype, const Big2DParams& p, cudaStream_t st) {
  if (op == B2_KSPEC) {
    b2_kspec_rows<<<dim3(p.C, kB2F / 2 / kGroups), kThreads, 0, st>>>(p);
    b2_kspec_cols<<<dim3(p.C, (kB2H + kGroups - 1) / kGroups), kThreads, 0, st>>>(p);
    g_launches.fetch_add(2, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  if (op == B2_DFILT) {
    b2_dfilt_cols<<<dim3(p.C, (kB2H + kGroups - 1) / kGroups), kThreads, 0, st>>>(p);
    b2_dfilt_rows<<<dim3(p.C, kB2F / 2 / kGroups), kThreads, 0, st>>>(p);
    g_launches.fetch_add(2, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  if (dtype == HYFFT_F32) return run_t<float>(op, p, st);
  if (dtype == HYFFT_BF16) return run_t<__nv_bfloat16>(op, p, st);
  return run_t<__half>(op, p, st);
}

}  // namespace hyfft
