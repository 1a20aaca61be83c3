// Fused large-grid 2D FFT convolution: y = crop(IFFT2(FFT2(x) * Kh)) (+ D-skip), its
// adjoint and its filter gradient, for F0 = F1 = F in {192, 256} and N0, N1 <= 128
// (e.g. the 128x128 HyenaND grid), one CTA per (batch item, channel).
//
// Data path of one CTA: the rows of x (real, read once from HBM through any strided
// view, BHL or channels-last) are transformed two at a time as one complex F-point
// FFT and split into their half spectra (F/2 + 1 bins), which stay in shared memory
// (N0 x (F/2 + 1) complex float32: 99 KB for F = 192, 132 KB for 256); each column is
// transformed (F points, rows >= N0 are zero), multiplied by the filter spectrum,
// inverted and cropped back in place; the rows are inverted two at a time and written
// once. Bins 0 and F/2 of a real row are real, so columns 0 and F/2 travel as one
// complex column (real part column 0, imaginary part column F/2): their spectra are
// separated by conjugate symmetry before the product and both inverse columns are real,
// so the column phase is F/2 transforms each way, a whole number of rounds of the
// CTA's 32 transform groups. Every activation crosses HBM once per pass; only the
// filter spectrum (read from L2) is shared between CTAs.
//
// The filter is rolled by its crop offset (tap (a, b) at ((a - K0/2) mod F,
// (b - K1/2) mod F)), so the reference's centred crop
// (nvsubquadratic/ops/fftconv.py:714-725) becomes the window [0, N) of every axis and
// the adjoint is the same kernel with conj(Kh). F >= N + ceil(K/2) - 1 on each axis
// keeps the circular convolution (and correlation) equal to the linear one on that
// window; the host picks F = 192 where that holds (the 128 x 128 grid with a 128 x 128
// filter needs 191) and F = 256 otherwise.
//
// FFT primitives, by 16 lanes (half a warp) per transform. Spatial side: lane l holds
// points l + 16 m (m < F/16). Spectral side: lane l < R = F/16 holds bins l + R b
// (b < 16). F = 256 (R = 16): two radix-16 register stages around one transpose
// through a padded per-group shared-memory tile. F = 192 (R = 12): forward = 12-point
// DFT over m per lane (3 x 4), twiddle W_192^{l a}, transpose, 16-point DFT over l on
// lanes a < 12; inverse = the same steps in reverse order.
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
constexpr int kSc12 = 13;                    // padded row of the 16 x 12 tile (F = 192)

template <int F>
struct B2 {
  static_assert(F == 192 || F == 256, "large-grid FFT length");
  static constexpr int H = F / 2 + 1;   // half-spectrum bins along axis 1
  static constexpr int R = F / 16;      // lanes holding spectral values; spatial points per lane
  static constexpr int TASKS = F / 2;   // column transforms per image (columns 0 and F/2 packed)
  static constexpr int HALF = (H + 1) / 2;  // column split of the dK kernel
  // x mod F for 0 <= x < 2F
  static __device__ __forceinline__ int wrap(int x) { return (F & (F - 1)) == 0 ? (x & (F - 1)) : (x >= F ? x - F : x); }
};

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

// 12-point DFT of v[0..11], natural order in and out: n = 3 n1 + n2, k = k1 + 4 k2
// (four-point DFTs over n1, twiddles W_12^{n2 k1}, three-point DFTs over n2).
// HOUT: only outputs 0..7 are needed.
template <bool HOUT>
__device__ __forceinline__ void dft12(float2 (&v)[16], float dir) {
  constexpr float h3 = 0.86602540378443865f;  // sqrt(3) / 2
  float2 t[3][4];
#pragma unroll
  for (int n2 = 0; n2 < 3; ++n2) {
    float2 a0 = v[n2], a1 = v[n2 + 3], a2 = v[n2 + 6], a3 = v[n2 + 9];
    dft4(a0, a1, a2, a3, dir);
    t[n2][0] = a0;
    t[n2][1] = a1;
    t[n2][2] = a2;
    t[n2][3] = a3;
  }
  t[1][1] = cmul(t[1][1], make_float2(h3, dir * 0.5f));
  t[1][2] = cmul(t[1][2], make_float2(0.5f, dir * h3));
  t[1][3] = make_float2(-dir * t[1][3].y, dir * t[1][3].x);
  t[2][1] = cmul(t[2][1], make_float2(0.5f, dir * h3));
  t[2][2] = cmul(t[2][2], make_float2(-0.5f, dir * h3));
  t[2][3] = make_float2(-t[2][3].x, -t[2][3].y);
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1) {
    const float2 a = t[0][k1], s = cadd(t[1][k1], t[2][k1]), d = csub(t[1][k1], t[2][k1]);
    const float2 m = make_float2(fmaf(-0.5f, s.x, a.x), fmaf(-0.5f, s.y, a.y));
    const float2 jd = make_float2(-dir * h3 * d.y, dir * h3 * d.x);
    v[k1] = cadd(a, s);
    v[k1 + 4] = cadd(m, jd);
    if constexpr (!HOUT) v[k1 + 8] = csub(m, jd);
  }
}

template <int F>
__device__ __forceinline__ void init_tw(float2* tw) {
  for (int j = threadIdx.x; j < F; j += blockDim.x) {
    float s, c;
    sincospif(2.0f * (float)j / (float)F, &s, &c);
    tw[j] = make_float2(c, s);
  }
}

// Forward transform, spatial -> spectral side: v[m] = x[l + 16 m] (m < F/16) ->
// v[b] = X[l + R b] (b < 16; lanes l < R), X[k] = sum_n x[n] e^{dir 2 pi i n k / F}.
// ZIN: x[n] = 0 for n >= 128 (registers 8.. hold zeros). Called by all 32 lanes of
// the warp together (both half-warps run a transform).
template <int F, bool ZIN>
__device__ __forceinline__ void fwdT(float2 (&v)[16], float2* sc, const float2* tw, int l, float dir) {
  if constexpr (F == 256) {
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
    dft16p<false, false>(v, dir);
  } else {
    dft12<false>(v, dir);  // v[a] = sum_m x[l + 16 m] W_12^{m a}
#pragma unroll
    for (int a = 1; a < 12; ++a) {
      const float2 w = tw[l * a];
      v[a] = cmul(v[a], make_float2(w.x, dir * w.y));
    }
    __syncwarp();
#pragma unroll
    for (int a = 0; a < 12; ++a) sc[l * kSc12 + a] = v[a];
    __syncwarp();
    const int la = l < 12 ? l : 11;  // lanes 12..15 carry no spectral values
#pragma unroll
    for (int n = 0; n < 16; ++n) v[n] = sc[n * kSc12 + la];
    dft16p<false, false>(v, dir);  // v[b] = X[la + 12 b]
  }
}

// Inverse-direction transform, spectral -> spatial side: v[b] = X[l + R b] (lanes
// l < R; the other lanes' values are ignored) -> v[m] = x[l + 16 m],
// x[n] = sum_k X[k] e^{dir 2 pi i n k / F}. HOUT: only x[n], n < 128 (m < 8), are needed.
template <int F, bool HOUT>
__device__ __forceinline__ void invT(float2 (&v)[16], float2* sc, const float2* tw, int l, float dir) {
  if constexpr (F == 256) {
    dft16p<false, false>(v, dir);
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
  } else {
    const int la = l < 12 ? l : 11;
    dft16p<false, false>(v, dir);  // v[n] = sum_b X[la + 12 b] W_16^{n b}
#pragma unroll
    for (int n = 1; n < 16; ++n) {
      const float2 w = tw[la * n];
      v[n] = cmul(v[n], make_float2(w.x, dir * w.y));
    }
    __syncwarp();
    if (l < 12) {
#pragma unroll
      for (int n = 0; n < 16; ++n) sc[n * kSc12 + l] = v[n];
    }
    __syncwarp();
#pragma unroll
    for (int a = 0; a < 12; ++a) v[a] = sc[l * kSc12 + a];
    dft12<HOUT>(v, dir);  // v[m] = x[l + 16 m]
  }
}

// Source lane and register of the partner bin F - k of bin k = l + R m on the spectral
// side: lane (R - l) mod R, register 15 - m (or (16 - m) mod 16 on lane 0).
template <int R>
__device__ __forceinline__ int partner_lane(int l) {
  return l < R ? (R - l) % R : l;
}

// After fwdT of u = a + i b (a, b real lines): the half spectra A[j], B[j] for the
// bins j = l + R m <= F/2 (m <= 8), from U[j] and U[F - j]. All lanes of the warp must
// call it.
template <int R>
__device__ __forceinline__ void split_pair(const float2 (&v)[16], int l, float2 (&A)[9], float2 (&Bv)[9]) {
  const int src = partner_lane<R>(l);
#pragma unroll
  for (int m = 0; m <= 8; ++m) {
    const float2 s = (l == 0) ? v[(16 - m) & 15] : v[15 - m];
    float2 p;
    p.x = __shfl_sync(0xffffffffu, s.x, src, 16);
    p.y = __shfl_sync(0xffffffffu, s.y, src, 16);
    const float2 u = v[m];
    // A = (U + conj(P)) / 2, B = (U - conj(P)) / (2i)
    A[m] = make_float2(0.5f * (u.x + p.x), 0.5f * (u.y - p.y));
    Bv[m] = make_float2(0.5f * (u.y + p.y), -0.5f * (u.x - p.x));
  }
}

// ---------------------------------------------------------------- filter spectrum
// Row transforms of the rolled filter: T[c][r][j], r < F, j <= F/2. grid (C, F/2/16).
template <int F>
__global__ void __launch_bounds__(kThreads) b2_kspec_rows(const Big2DParams p) {
  using G = B2<F>;
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[F];
  init_tw<F>(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int r0 = 2 * (blockIdx.y * kGroups + g);
  const int h0 = p.K0 / 2, h1 = p.K1 / 2;
  const int a0 = G::wrap(r0 + h0), a1 = G::wrap(r0 + 1 + h0);
  const float* f = reinterpret_cast<const float*>(p.filt.ptr) + (long long)c * p.filt.cst;
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    v[m] = make_float2(0.f, 0.f);
    if (m < G::R) {
      const int bb = G::wrap(l + 16 * m + h1);
      const bool inb = bb < p.K1;
      v[m].x = (inb && a0 < p.K0) ? f[a0 * p.filt.s0 + bb * p.filt.s1] : 0.f;
      v[m].y = (inb && a1 < p.K0) ? f[a1 * p.filt.s0 + bb * p.filt.s1] : 0.f;
    }
  }
  fwdT<F, false>(v, sc + g * kScSize, tw, l, -1.f);
  float2 A[9], Bv[9];
  split_pair<G::R>(v, l, A, Bv);
  float2* t0 = p.T + ((long long)c * F + r0) * G::H;
  if (l < G::R) {
#pragma unroll
    for (int m = 0; m <= 8; ++m) {
      const int j = l + G::R * m;
      if (j < G::H) {
        t0[j] = A[m];
        t0[G::H + j] = Bv[m];
      }
    }
  }
}

// Column transforms: Kh[c][j][i] = sum_r T[c][r][j] e^{-2 pi i r i / F}. grid (C, ceil(H/16)).
template <int F>
__global__ void __launch_bounds__(kThreads) b2_kspec_cols(const Big2DParams p) {
  using G = B2<F>;
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[F];
  init_tw<F>(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int j = blockIdx.y * kGroups + g;
  const bool act = j < G::H;
  const float2* t = p.T + (long long)c * F * G::H + (act ? j : 0);
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m)
    v[m] = (act && m < G::R) ? t[(long long)(l + 16 * m) * G::H] : make_float2(0.f, 0.f);
  fwdT<F, false>(v, sc + g * kScSize, tw, l, -1.f);
  if (act && l < G::R) {
    float2* o = p.Kh + ((long long)c * G::H + j) * F;
#pragma unroll
    for (int m = 0; m < 16; ++m) o[l + G::R * m] = v[m];
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
  const T* row0 = reinterpret_cast<const T*>(in.ptr) + (long long)b * in.bst + (long long)c * in.cst +
                  (long long)r0 * in.s0;
  const T* row1 = row0 + in.s0;
  if (in.s1 == 1) {  // unit-stride rows (channel-major activations): constant offsets from one base
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int n = l + 16 * m;
      v[m] = make_float2(0.f, 0.f);
      if (act && n < N1) {
        v[m].x = DT<T>::load(row0 + n);
        if (has1) v[m].y = DT<T>::load(row1 + n);
      }
    }
  } else {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int n = l + 16 * m;
      v[m] = make_float2(0.f, 0.f);
      if (act && n < N1) {
        v[m].x = DT<T>::load(row0 + (long long)n * in.s1);
        if (has1) v[m].y = DT<T>::load(row1 + (long long)n * in.s1);
      }
    }
  }
}

// Forward row transforms of the row pairs pr0 .. pr0 + npr - 1 (rows 2 pr, 2 pr + 1) of
// input view `in` for image (b, c), NG transform groups: bins j in [jlo, jlo + jn) of row
// r go to dst[(r - 2 pr0) * ld + j - jlo]. All threads of the CTA call it. The next
// round's rows are loaded before this round's transform, so their global-memory latency
// overlaps the arithmetic.
template <typename T, int F, int NG>
__device__ __forceinline__ void rows_forward(const Big2DView& in, int b, int c, int N0, int N1, float2* dst, int ld,
                                             int jlo, int jn, float2* sc, const float2* tw, int pr0 = 0,
                                             int npr = kB2MaxN / 2) {
  using G = B2<F>;
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int npairs = (N0 + 1) >> 1;
  const int rounds = (npr + NG - 1) / NG;
  float2 nxt[8];
  rows_load<T>(in, b, c, N0, N1, g < npr ? pr0 + g : npairs, l, nxt);
  for (int rb = 0; rb < rounds; ++rb) {
    const int pl = rb * NG + g, pr = pr0 + pl;
    const bool act = pl < npr && pr < npairs;
    const int r0 = 2 * pr, r1 = r0 + 1;
    const bool has1 = act && r1 < N0;
    float2 v[16];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      v[m] = nxt[m];
      v[m + 8] = make_float2(0.f, 0.f);
    }
    if (rb + 1 < rounds) rows_load<T>(in, b, c, N0, N1, pl + NG < npr ? pr + NG : npairs, l, nxt);
    fwdT<F, true>(v, sc, tw, l, -1.f);
    float2 A[9], Bv[9];
    split_pair<G::R>(v, l, A, Bv);
    if (act && l < G::R) {
      float2* d0 = dst + (r0 - 2 * pr0) * ld - jlo;
#pragma unroll
      for (int m = 0; m <= 8; ++m) {
        const int j = l + G::R * m;
        if (j >= jlo && j < jlo + jn && j < G::H) {
          d0[j] = A[m];
          if (has1) d0[ld + j] = Bv[m];
        }
      }
    }
  }
}

// ---------------------------------------------------------------- convolution
// Per-group transpose scratch of the conv kernels (float2): the 16 x 13 tile of the
// 192-point transforms, the 16 x 17 tile of the 256-point ones.
template <int F>
constexpr int conv_sc() {
  return F == 192 ? 16 * kSc12 : kScSize;
}
template <int F>
constexpr int conv_ld() {
  return F == 192 ? kSc12 : kScLd;
}
// zs_mode 2 stages every round's kept Zs column in shared memory one round ahead
// (where it fits: F = 192).
template <int F>
constexpr bool conv_zstage() {
  return F == 192;
}

__device__ __forceinline__ void cp16(void* s, const void* g) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// One group's copy of an F-point complex column (F * 8 bytes, 16-byte aligned) to shared memory.
template <int F>
__device__ __forceinline__ void stage_col(float2* dst, const float2* src, int l) {
#pragma unroll
  for (int i = l; i < F / 2; i += 16) cp16(dst + 2 * i, src + 2 * i);
}

// Shared-memory layout behind the row half-spectra of a conv CTA (NG groups):
// sc [NG][conv_sc] | tw [F] | ext [3][F] | zb [NG][F] (zs_mode 2 staging, F = 192 only).
// ext holds the packed task's extra operands: the filter-spectrum column F/2 and, with
// zs_mode 2, the image's kept Zs columns 0 and F/2.
template <int F, int NG>
constexpr size_t conv_tail_floats2(bool zstage) {
  return (size_t)NG * conv_sc<F>() + 4 * F + (zstage ? (size_t)NG * F : 0);
}

// Prologue copies (cp.async, one commit group): the packed task's extra operands when this
// CTA runs task 0, and with zstage the kept Zs column of this group's first task.
template <int F, int NT>
__device__ __forceinline__ void conv_prologue(const Big2DParams& p, int b, int c, float2* ext, float2* myzb,
                                              int first_task, bool has_packed, bool zstage) {
  using G = B2<F>;
  const float2* kh = p.Kh + (long long)c * G::H * F;
  const float2* zimg = p.Zs + ((long long)b * p.C + c) * G::H * F;
  if (has_packed) {
    for (int i = threadIdx.x; i < F / 2; i += NT) cp16(ext + 2 * i, kh + (long long)(F / 2) * F + 2 * i);
    if (p.zs_mode == 2) {
      for (int i = threadIdx.x; i < F / 2; i += NT) {
        cp16(ext + F + 2 * i, zimg + 2 * i);
        cp16(ext + 2 * F + 2 * i, zimg + (long long)(F / 2) * F + 2 * i);
      }
    }
  }
  if (zstage && first_task > 0) stage_col<F>(myzb, zimg + (long long)first_task * F, threadIdx.x & 15);
  cp_commit();
}

// Column phase: tasks t0 .. t0 + ntask - 1 (task t: column t; task 0: columns 0 and F/2,
// both real along the rows, as one complex column) by NG groups, ntask / NG rounds.
// Row r of the half-spectra is at (r < 64 ? Alo : Ahi)[(r & 63) * H + j]. Each column: transform, * Kh (or conj), inverse,
// keep rows [0, N0). Each round's filter-spectrum column (an L2 read) is loaded one round
// ahead, right after the previous column has consumed its own, so the load overlaps an
// inverse and a forward transform; with zs_mode 2 the next round's kept Zs column is
// copied to shared memory at the same point.
template <int F, int NG>
__device__ __forceinline__ void column_phase(const Big2DParams& p, float2* Alo, float2* Ahi, int t0, int ntask, int b,
                                             int c, float2* mysc, float2* myzb, const float2* ext, const float2* tw,
                                             bool zstage) {
  using G = B2<F>;
  constexpr int H = G::H, R = G::R, LD = conv_ld<F>();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const bool sl = l < R;  // lane holds spectral values
  const int N0 = p.N0;
  const float2* kh = p.Kh + (long long)c * H * F;
  const float2* zimg = p.Zs + ((long long)b * p.C + c) * H * F;
  const float cj = p.conj ? -1.f : 1.f;
  const int rounds = ntask / NG;
  float2 kv[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) kv[m] = sl ? __ldg(kh + (long long)(t0 + g) * F + l + R * m) : make_float2(0.f, 0.f);
  for (int rb = 0; rb < rounds; ++rb) {
    const int j = t0 + rb * NG + g;
    const bool packed = j == 0;
    float2 v[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int r = l + 16 * m;
      v[m] = make_float2(0.f, 0.f);
      if (m < 8 && r < N0) {
        const float2* row = (m < 4 ? Alo : Ahi) + (r & 63) * H;
        if (packed) v[m] = make_float2(row[0].x, row[F / 2].x);
        else v[m] = row[j];
      }
    }
    fwdT<F, true>(v, mysc, tw, l, -1.f);
    if (zstage) {  // this round's staged column (copied a round ago) is complete and visible
      cp_wait_all();
      __syncwarp();
    }
    if (!packed) {
      if (p.zs_mode != 0 && sl) {
        float2* zc = p.Zs + (((long long)b * p.C + c) * H + j) * F + l;
        if (p.zs_mode == 1) {
#pragma unroll
          for (int m = 0; m < 16; ++m) zc[R * m] = v[m];
        } else {
          // G[c][j][i] += conj(Z[b][c][j][i]) * DY[j][i] (the per-image term of the filter gradient)
          float2* gc = p.G + ((long long)c * H + j) * F + l;
          if (zstage) {
#pragma unroll
            for (int m = 0; m < 16; ++m) atomicAdd(gc + R * m, cmulc(v[m], myzb[l + R * m]));
          } else {
            float2 z[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) z[m] = __ldcs(zc + R * m);
#pragma unroll
            for (int m = 0; m < 16; ++m) atomicAdd(gc + R * m, cmulc(v[m], z[m]));
          }
        }
      }
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        float2 k = kv[m];
        k.y *= cj;
        v[m] = cmul(v[m], k);
      }
    } else {
      // separate the spectra of column 0 (Z0) and column F/2 (ZH) of the packed column
      // u = c0 + i cH: Z0[i] = (U[i] + conj(U[F - i])) / 2, ZH[i] = (U[i] - conj(U[F - i])) / (2i).
      // Only this half-warp takes the branch: its own 16 lanes synchronise.
      const unsigned half = 0xffffu << (threadIdx.x & 16);
      __syncwarp(half);
      if (sl) {
#pragma unroll
        for (int m = 0; m < 16; ++m) mysc[m * LD + l] = v[m];
      }
      __syncwarp(half);
      const int src = partner_lane<R>(l);
      float2* zc0 = p.Zs + (((long long)b * p.C + c) * H) * F + l;
      float2* zcH = zc0 + (long long)(F / 2) * F;
      float2* gc0 = p.G + ((long long)c * H) * F + l;
      float2* gcH = gc0 + (long long)(F / 2) * F;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float2 u = v[m];
        const int i = l + R * m;
        const float2 q = sl ? mysc[((l == 0) ? ((16 - m) & 15) : (15 - m)) * LD + src] : make_float2(0.f, 0.f);
        const float2 z0 = make_float2(0.5f * (u.x + q.x), 0.5f * (u.y - q.y));
        const float2 zh = make_float2(0.5f * (u.y + q.y), -0.5f * (u.x - q.x));
        if (sl) {
          if (p.zs_mode == 1) {
            zc0[R * m] = z0;
            zcH[R * m] = zh;
          } else if (p.zs_mode == 2) {
            atomicAdd(gc0 + R * m, cmulc(z0, ext[F + i]));
            atomicAdd(gcH + R * m, cmulc(zh, ext[2 * F + i]));
          }
        }
        float2 k0 = kv[m], kH = sl ? ext[i] : make_float2(0.f, 0.f);
        k0.y *= cj;
        kH.y *= cj;
        const float2 p0 = cmul(z0, k0), pH = cmul(zh, kH);
        v[m] = make_float2(p0.x - pH.y, p0.y + pH.x);  // p0 + i pH
      }
    }
    const int jn = j + NG;
    if (rb + 1 < rounds) {
#pragma unroll
      for (int m = 0; m < 16; ++m) kv[m] = sl ? __ldg(kh + (long long)jn * F + l + R * m) : make_float2(0.f, 0.f);
      if (zstage) {  // every lane of the group is done with this round's staged column
        __syncwarp();
        stage_col<F>(myzb, zimg + (long long)jn * F, l);
        cp_commit();
      }
    }
    invT<F, true>(v, mysc, tw, l, 1.f);
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int r = l + 16 * m;
      if (r < N0) {
        float2* row = (m < 4 ? Alo : Ahi) + (r & 63) * H;
        if (packed) {
          row[0] = make_float2(v[m].x, 0.f);
          row[F / 2] = make_float2(v[m].y, 0.f);
        } else {
          row[j] = v[m];
        }
      }
    }
  }
}

// Inverse row transforms of the row pairs pr0 .. pr0 + npr - 1, two rows as one complex
// line, and the epilogue (scale, D-skip, dtype rounding, store). Row r's half spectrum is
// at A[(r - 2 pr0) * H].
template <typename T, int F, int NG>
__device__ __forceinline__ void rows_inverse(const Big2DParams& p, const float2* A, int b, int c, int pr0, int npr,
                                             float2* mysc, const float2* tw) {
  using G = B2<F>;
  constexpr int H = G::H, R = G::R;
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const bool sl = l < R;
  const int N0 = p.N0, N1 = p.N1;
  const float scale = 1.0f / (float)(F * F);
  const int npairs = (N0 + 1) >> 1;
  const float Dc = p.D ? p.D[c] : 0.f;
  T* yo = reinterpret_cast<T*>(const_cast<void*>(p.y.ptr)) + (long long)b * p.y.bst + (long long)c * p.y.cst;
  for (int rb = 0; rb < (npr + NG - 1) / NG; ++rb) {
    const int pl = rb * NG + g, pr = pr0 + pl;
    const bool act = pl < npr && pr < npairs;
    const int r0 = 2 * pr, r1 = r0 + 1;
    const bool has1 = act && r1 < N0;
    const float2* a0 = A + (r0 - 2 * pr0) * H;
    T* y0 = yo + (long long)r0 * p.y.s0;
    float2 v[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int j = l + R * m;
      float2 a = make_float2(0.f, 0.f), bb = make_float2(0.f, 0.f);
      if (act && sl) {
        if (j < H) {
          a = a0[j];
          if (has1) bb = a0[H + j];
        } else {
          a = a0[F - j];
          a.y = -a.y;
          if (has1) {
            bb = a0[H + F - j];
            bb.y = -bb.y;
          }
        }
      }
      v[m] = make_float2(a.x - bb.y, a.y + bb.x);  // a + i b
    }
    // the D-skip inputs of these two rows, loaded before the transform
    float2 xs[8];
    if (p.D) rows_load<T>(p.x, b, c, N0, N1, act ? pr : npairs, l, xs);
    invT<F, true>(v, mysc, tw, l, 1.f);
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
          const long long on = p.y.s1 == 1 ? n : (long long)n * p.y.s1;
          DT<T>::store(y0 + on, o0);
          if (has1) DT<T>::store(y0 + p.y.s0 + on, o1);
        }
      }
    }
  }
}

// One CTA per image (b, c): all 128 rows of the half spectra in shared memory, 32 groups.
template <typename T, int F>
__global__ void __launch_bounds__(kBigThreads) b2_conv(const Big2DParams p) {
  using G = B2<F>;
  constexpr int H = G::H;
  extern __shared__ __align__(16) unsigned char smem[];
  float2* A = reinterpret_cast<float2*>(smem);                  // [128][H]
  float2* sc = A + kB2MaxN * H;                                  // [32][conv_sc]
  float2* tw = sc + kBigGroups * conv_sc<F>();                   // [F]
  float2* ext = tw + F;                                          // [3][F]
  float2* zb = ext + 3 * F;                                      // [32][F]
  const int g = threadIdx.x >> 4;
  // channels-last inputs: neighbouring channels of one image run together (shared
  // sectors); channel-major: the batch items of one channel do (shared filter spectrum)
  const bool cfast = p.x.cst == 1;
  const int c = cfast ? blockIdx.x : blockIdx.y, b = cfast ? blockIdx.y : blockIdx.x;
  const bool zstage = conv_zstage<F>() && p.zs_mode == 2;
  float2* mysc = sc + g * conv_sc<F>();
  float2* myzb = zb + g * F;
  conv_prologue<F, kBigThreads>(p, b, c, ext, myzb, g, true, zstage);
  init_tw<F>(tw);
  __syncthreads();
  rows_forward<T, F, kBigGroups>(p.x, b, c, p.N0, p.N1, A, H, 0, H, mysc, tw);
  cp_wait_all();
  __syncthreads();
  column_phase<F, kBigGroups>(p, A, A + 64 * H, 0, G::TASKS, b, c, mysc, myzb, ext, tw, zstage);
  __syncthreads();
  rows_inverse<T, F, kBigGroups>(p, A, b, c, 0, kB2MaxN / 2, mysc, tw);
}

// ---------------------------------------------------------------- filter gradient
// G[c][j][i] += conj(X[i][j]) * DY[i][j] for one image, in two halves of the column
// bins (j < HALF, then j >= HALF) so that both row-transformed inputs fit in shared memory.
template <typename T, int F>
__global__ void __launch_bounds__(kBigThreads) b2_dk(const Big2DParams p) {
  using G = B2<F>;
  constexpr int H = G::H, R = G::R, HALF = G::HALF;
  extern __shared__ __align__(16) unsigned char smem[];
  float2* Ax = reinterpret_cast<float2*>(smem);                 // [128][HALF]
  float2* Ay = Ax + kB2MaxN * HALF;                              // [128][HALF]
  float2* sc = Ay + kB2MaxN * HALF;
  float2* tw = sc + kBigGroups * kScSize;
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  // channel fastest: concurrent CTAs accumulate into different channels' spectra
  const int c = blockIdx.x, b = blockIdx.y;
  const int N0 = p.N0, N1 = p.N1;
  float2* mysc = sc + g * kScSize;
  init_tw<F>(tw);
  __syncthreads();
  float2* Gc = p.G + (long long)c * H * F;
  for (int h = 0; h < 2; ++h) {
    const int jlo = h ? HALF : 0, jn = h ? H - HALF : HALF;
    rows_forward<T, F, kBigGroups>(p.x, b, c, N0, N1, Ax, HALF, jlo, jn, mysc, tw);
    rows_forward<T, F, kBigGroups>(p.x2, b, c, N0, N1, Ay, HALF, jlo, jn, mysc, tw);
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
      fwdT<F, true>(x, mysc, tw, l, -1.f);
      fwdT<F, true>(y, mysc, tw, l, -1.f);
      if (act && l < R) {
        float2* gc = Gc + (long long)(jlo + jj) * F;
#pragma unroll
        for (int m = 0; m < 16; ++m) atomicAdd(gc + l + R * m, cmulc(y[m], x[m]));
      }
    }
    __syncthreads();
  }
}

// Inverse of G along axis 0: T[c][r][j] = sum_i G[c][j][i] e^{+2 pi i r i / F}. grid (C, ceil(H/16)).
template <int F>
__global__ void __launch_bounds__(kThreads) b2_dfilt_cols(const Big2DParams p) {
  using G = B2<F>;
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[F];
  init_tw<F>(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int j = blockIdx.y * kGroups + g;
  const bool act = j < G::H;
  const float2* gc = p.G + ((long long)c * G::H + (act ? j : 0)) * F;
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) v[m] = (act && l < G::R) ? gc[l + G::R * m] : make_float2(0.f, 0.f);
  invT<F, false>(v, sc + g * kScSize, tw, l, 1.f);
  if (act) {
    float2* t = p.T + (long long)c * F * G::H + j;
#pragma unroll
    for (int m = 0; m < G::R; ++m) t[(long long)(l + 16 * m) * G::H] = v[m];
  }
}

// Inverse along axis 1 (two rows at a time as one complex line), un-roll, crop to the
// filter taps: dfilt[c][a][b]. grid (C, F/2/16).
template <int F>
__global__ void __launch_bounds__(kThreads) b2_dfilt_rows(const Big2DParams p) {
  using G = B2<F>;
  __shared__ float2 sc[kGroups * kScSize];
  __shared__ float2 tw[F];
  init_tw<F>(tw);
  __syncthreads();
  const int g = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int c = blockIdx.x;
  const int r0 = 2 * (blockIdx.y * kGroups + g), r1 = r0 + 1;
  const float2* t0 = p.T + ((long long)c * F + r0) * G::H;
  const float2* t1 = t0 + G::H;
  float2 v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = l + G::R * m;
    float2 a = make_float2(0.f, 0.f), bb = make_float2(0.f, 0.f);
    if (l < G::R) {
      if (j < G::H) {
        a = t0[j];
        bb = t1[j];
      } else {
        a = t0[F - j];
        bb = t1[F - j];
        a.y = -a.y;
        bb.y = -bb.y;
      }
    }
    v[m] = make_float2(a.x - bb.y, a.y + bb.x);
  }
  invT<F, false>(v, sc + g * kScSize, tw, l, 1.f);
  const float scale = 1.0f / (float)(F * F);
  const int h0 = p.K0 / 2, h1 = p.K1 / 2;
  const int a0 = G::wrap(r0 + h0), a1 = G::wrap(r1 + h0);
  float* d = reinterpret_cast<float*>(const_cast<void*>(p.dfilt.ptr)) + (long long)c * p.dfilt.cst;
#pragma unroll
  for (int m = 0; m < G::R; ++m) {
    const int bb = G::wrap(l + 16 * m + h1);
    if (bb < p.K1) {
      if (a0 < p.K0) d[a0 * p.dfilt.s0 + bb * p.dfilt.s1] = v[m].x * scale;
      if (a1 < p.K0) d[a1 * p.dfilt.s0 + bb * p.dfilt.s1] = v[m].y * scale;
    }
  }
}

template <int F>
constexpr size_t conv_smem(bool zstage) {
  return sizeof(float2) * ((size_t)kB2MaxN * B2<F>::H + conv_tail_floats2<F, kBigGroups>(zstage));
}
template <int F>
constexpr size_t dk_smem() {
  return sizeof(float2) * ((size_t)2 * kB2MaxN * B2<F>::HALF + kBigGroups * kScSize + F);
}
static_assert(conv_smem<256>(conv_zstage<256>()) <= 227 * 1024 && conv_smem<192>(conv_zstage<192>()) <= 227 * 1024 &&
                  dk_smem<256>() <= 227 * 1024,
              "shared memory per CTA");
static_assert(kSc12 * 16 <= kScSize, "F = 192 transpose tile fits a group's scratch");

template <typename T, int F>
int run_t(int op, const Big2DParams& p, cudaStream_t st) {
  if (op == B2_CONV) {
    const size_t sm = conv_smem<F>(conv_zstage<F>() && p.zs_mode == 2);
    if (!kernel_smem_once((const void*)b2_conv<T, F>, conv_smem<F>(conv_zstage<F>()))) return HYFFT_ERR_CUDA;
    b2_conv<T, F><<<p.x.cst == 1 ? dim3(p.C, p.B) : dim3(p.B, p.C), kBigThreads, sm, st>>>(p);
  } else {
    if (!kernel_smem_once((const void*)b2_dk<T, F>, dk_smem<F>())) return HYFFT_ERR_CUDA;
    b2_dk<T, F><<<dim3(p.C, p.B), kBigThreads, dk_smem<F>(), st>>>(p);
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
}

template <int F>
int dispatch_f(int op, int dtype, const Big2DParams& p, cudaStream_t st) {
  using G = B2<F>;
  if (op == B2_KSPEC) {
    b2_kspec_rows<F><<<dim3(p.C, F / 2 / kGroups), kThreads, 0, st>>>(p);
    b2_kspec_cols<F><<<dim3(p.C, (G::H + kGroups - 1) / kGroups), kThreads, 0, st>>>(p);
    g_launches.fetch_add(2, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  if (op == B2_DFILT) {
    b2_dfilt_cols<F><<<dim3(p.C, (G::H + kGroups - 1) / kGroups), kThreads, 0, st>>>(p);
    b2_dfilt_rows<F><<<dim3(p.C, F / 2 / kGroups), kThreads, 0, st>>>(p);
    g_launches.fetch_add(2, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  if (dtype == HYFFT_F32) return run_t<float, F>(op, p, st);
  if (dtype == HYFFT_BF16) return run_t<__nv_bfloat16, F>(op, p, st);
  return run_t<__half, F>(op, p, st);
}

}  // namespace

int big2d_dispatch(int op, int dtype, const Big2DParams& p, cudaStream_t st) {
  if (p.F == 192) return dispatch_f<192>(op, dtype, p, st);
  if (p.F == 256) return dispatch_f<256>(op, dtype, p, st);
  return HYFFT_ERR_UNSUPPORTED;
}

}  // namespace hyfft
