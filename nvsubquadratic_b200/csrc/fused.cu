// Fused single-pass Hyena kernels for small 2D grids (e.g. the 14x14 ViT token
// grid): one CTA owns 8 channels x (a few) batch pairs and does everything on
// chip — channels-last loads of q, k, v (16-byte vectors, read in place from the
// [B, *S, 3C] projection output), depthwise short conv, gate 1, the padded 2D
// FFT long conv with its D-skip, gate 2 and the channels-last store — so every
// activation crosses HBM once.
//
// The 2D transforms are the pruned register FFTs of fftreg.cuh (one thread per
// row / column, radix 2, compile-time zero-padding and crop pruning). Spectra
// stay in bit-reversed order end to end. The filter is rolled by its crop offset
// (tap (a, b) placed at ((a - K0/2) mod F0, (b - K1/2) mod F1)) before its FFT, so
// both the forward and the adjoint transforms read and write the window [0, N)
// of every axis; the reference's centred crop (nvsubquadratic/ops/fftconv.py:714-725)
// becomes a phase ramp folded into the filter spectrum.
//
// Two batch items share one complex signal (real part item p, imaginary part item
// p + ceil(B/2)); the filter is real, so one complex transform carries both.
//
// Backward: dK accumulates sum_pairs DH * conj(Z) (its real inverse is
// sum_b corr(dh_b, z_b)) with float2 atomics into a [C][F0][F1] spectrum that a
// small kernel inverts; dD and the short-conv weight gradients use per-CTA
// reductions plus atomics.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstring>

#include "common.cuh"
#include "fftreg.cuh"
#include "fused2d.h"

namespace hyfft {

extern std::atomic<long long> g_launches;



constexpr int kCG = 8;  // channels per CTA (one 16-byte bf16 vector)

// ------------------------------------------------------------------ 8-channel vectors
template <typename T>
struct V8;
template <>
struct V8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&o)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
  static __device__ __forceinline__ void copy(__nv_bfloat16* d, const __nv_bfloat16* s) {
    *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s);
  }
  static __device__ __forceinline__ void zero(__nv_bfloat16* d) { *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0); }
};
template <>
struct V8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&o)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&o)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
  static __device__ __forceinline__ void copy(float* d, const float* s) {
    reinterpret_cast<float4*>(d)[0] = reinterpret_cast<const float4*>(s)[0];
    reinterpret_cast<float4*>(d)[1] = reinterpret_cast<const float4*>(s)[1];
  }
  static __device__ __forceinline__ void zero(float* d) {
    reinterpret_cast<float4*>(d)[0] = make_float4(0, 0, 0, 0);
    reinterpret_cast<float4*>(d)[1] = make_float4(0, 0, 0, 0);
  }
};

template <typename T>
__device__ __forceinline__ void round8(float (&o)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = DT<T>::round(o[i]);
}

// Copy of one position's 8 channels (16 bytes for 16-bit types, 32 for float) from global
// to shared memory, left in flight (cp.async, L2 only); !valid writes zeros and reads
// nothing. All copies of a load phase are issued before one wait, so their latencies
// overlap instead of adding up.
template <typename T>
__device__ __forceinline__ void cp_v8(T* sdst, const T* gsrc, bool valid) {
  constexpr int kChunks = (int)(8 * sizeof(T)) / 16;
#pragma unroll
  for (int h = 0; h < kChunks; ++h) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(reinterpret_cast<char*>(sdst) + 16 * h);
    const char* g = reinterpret_cast<const char*>(gsrc) + (valid ? 16 * h : 0);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(g), "r"(valid ? 16 : 0) : "memory");
  }
}
__device__ __forceinline__ void cp_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// two neighbouring channels of one position (4- or 8-byte aligned)
template <typename T>
__device__ __forceinline__ float2 ld2ch(const T* p);
template <>
__device__ __forceinline__ float2 ld2ch<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <>
__device__ __forceinline__ float2 ld2ch<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}

// weight of channel c at tap j from a tap-major [taps][8] table, read as two 16-byte vectors
__device__ __forceinline__ float wtap8(const float* w, int j, int c) {
  const float4 v = reinterpret_cast<const float4*>(w + j * 8)[c >> 2];
  const int r = c & 3;
  return r == 0 ? v.x : (r == 1 ? v.y : (r == 2 ? v.z : v.w));
}

// Depthwise SKxSK cross-correlation ("same" padding) of 8 channels of one image tile
// [N0*N1][8] at (n0, n1); w: [SK*SK][8] (16-byte aligned), bias: [8] or null. SK == 0: identity.
template <typename T, int N0, int N1, int SK>
__device__ __forceinline__ void stencil8(const T* tile, const float* w, const float* bias, int n0, int n1,
                                         float (&o)[8]) {
  if constexpr (SK == 0) {
    V8<T>::load(tile + (n0 * N1 + n1) * kCG, o);
  } else {
    constexpr int OFF = (SK - 1) / 2;
#pragma unroll
    for (int c = 0; c < 8; ++c) o[c] = bias ? bias[c] : 0.f;
#pragma unroll
    for (int a = 0; a < SK; ++a) {
      const int i0 = n0 + a - OFF;
      if (i0 < 0 || i0 >= N0) continue;
#pragma unroll
      for (int b = 0; b < SK; ++b) {
        const int i1 = n1 + b - OFF;
        if (i1 < 0 || i1 >= N1) continue;
        float x[8];
        V8<T>::load(tile + (i0 * N1 + i1) * kCG, x);
#pragma unroll
        for (int c = 0; c < 8; ++c) o[c] = fmaf(wtap8(w, a * SK + b, c), x[c], o[c]);
      }
    }
  }
}

// Transposed stencil at the two neighbouring outputs (n0, n1) and (n0, n1 + 1) of one row:
// they share SK of their SK + 1 input columns, so each input vector is loaded once.
// o1 is left zero when n1 + 1 == N1.
template <int N0, int N1, int SK, typename S>
__device__ __forceinline__ void stencil8_t2(const S* tile, const float* w, int n0, int n1, float (&o0)[8],
                                            float (&o1)[8]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) o0[c] = o1[c] = 0.f;
  const bool two = n1 + 1 < N1;
  if constexpr (SK == 0) {
    V8<S>::load(tile + (n0 * N1 + n1) * kCG, o0);
    if (two) V8<S>::load(tile + (n0 * N1 + n1 + 1) * kCG, o1);
  } else {
    constexpr int OFF = (SK - 1) / 2;
#pragma unroll
    for (int a = 0; a < SK; ++a) {
      const int i0 = n0 - a + OFF;
      if (i0 < 0 || i0 >= N0) continue;
      float x[SK + 1][8];  // input columns n1 + OFF - SK + 1 + m, m = 0..SK
#pragma unroll
      for (int m = 0; m <= SK; ++m) {
        const int i1 = n1 + OFF - SK + 1 + m;
        if (i1 >= 0 && i1 < N1) {
          V8<S>::load(tile + (i0 * N1 + i1) * kCG, x[m]);
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) x[m][c] = 0.f;
        }
      }
#pragma unroll
      for (int b = 0; b < SK; ++b) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float wv = wtap8(w, a * SK + b, c);
          o0[c] = fmaf(wv, x[SK - 1 - b][c], o0[c]);
          o1[c] = fmaf(wv, x[SK - b][c], o1[c]);
        }
      }
    }
  }
}

__host__ __device__ constexpr size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }

// ------------------------------------------------------------------ filter spectrum
// Kbr[c] = bit-reversed 2D DFT of the filter rolled by (K0/2, K1/2). One CTA per channel.
template <int F0, int F1>
__global__ void __launch_bounds__(64) kspec2d_kernel(const Fused2DParams p) {
  constexpr int LD = F1 + 1;
  __shared__ float2 S[F0 * LD];
  const int c = blockIdx.x;
  const int c0 = p.K0 / 2, c1 = p.K1 / 2;
  const float* f = p.filt + (long long)c * p.K0 * p.K1;
  for (int i = threadIdx.x; i < F0 * F1; i += blockDim.x) {
    const int r = i / F1, s = i % F1;
    // rolled position (r, s) holds tap ((r + c0) mod F0, (s + c1) mod F1) if inside the kernel
    const int a = (r + c0) % F0, b = (s + c1) % F1;
    const float val = (a < p.K0 && b < p.K1) ? f[a * p.K1 + b] : 0.f;
    S[r * LD + s] = make_float2(val, 0.f);
  }
  __syncthreads();
  if (threadIdx.x < F0) {  // rows
    float2 v[F1];
#pragma unroll
    for (int i = 0; i < F1; ++i) v[i] = S[threadIdx.x * LD + i];
    reg::fft_dif<F1, F1, -1>(v);
#pragma unroll
    for (int i = 0; i < F1; ++i) S[threadIdx.x * LD + i] = v[i];
  }
  __syncthreads();
  if (threadIdx.x < F1) {  // columns
    float2 v[F0];
#pragma unroll
    for (int i = 0; i < F0; ++i) v[i] = S[i * LD + threadIdx.x];
    reg::fft_dif<F0, F0, -1>(v);
    float2* out = p.Kbr + (long long)c * F0 * F1 + threadIdx.x;
#pragma unroll
    for (int i = 0; i < F0; ++i) out[i * F1] = v[i];
  }
}

// dfilt[c] = crop of the real inverse of G[c] (bit-reversed), un-rolled. One CTA per channel.
template <int F0, int F1>
__global__ void __launch_bounds__(64) dfilt2d_kernel(const Fused2DParams p) {
  constexpr int LD = F1 + 1;
  __shared__ float2 S[F0 * LD];
  const int c = blockIdx.x;
  const float2* g = p.G + (long long)c * F0 * F1;
  if (threadIdx.x < F1) {  // columns: bit-reversed along axis 0 -> natural
    float2 v[F0];
#pragma unroll
    for (int i = 0; i < F0; ++i) v[i] = g[i * F1 + threadIdx.x];
    reg::fft_dit<F0, F0, +1>(v);
#pragma unroll
    for (int i = 0; i < F0; ++i) S[i * LD + threadIdx.x] = v[i];
  }
  __syncthreads();
  if (threadIdx.x < F0) {  // rows
    float2 v[F1];
#pragma unroll
    for (int i = 0; i < F1; ++i) v[i] = S[threadIdx.x * LD + i];
    reg::fft_dit<F1, F1, +1>(v);
#pragma unroll
    for (int i = 0; i < F1; ++i) S[threadIdx.x * LD + i] = v[i];
  }
  __syncthreads();
  const float scale = 1.0f / (float)(F0 * F1);
  const int c0 = p.K0 / 2, c1 = p.K1 / 2;
  float* out = p.dfilt + (long long)c * p.K0 * p.K1;
  for (int i = threadIdx.x; i < p.K0 * p.K1; i += blockDim.x) {
    const int a = i / p.K1, b = i % p.K1;
    const int r = ((a - c0) % F0 + F0) % F0, s = ((b - c1) % F1 + F1) % F1;
    out[i] = S[r * LD + s].x * scale;
  }
}

// ------------------------------------------------------------------ forward
template <typename T, int N0, int N1, int SK, int PG>
struct FwdSmem {
  static constexpr int NP = N0 * N1, NIMG = 2 * PG, NT = SK > 0 ? SK * SK : 1;
  static constexpr size_t stage = al16(sizeof(T) * 3 * NIMG * NP * kCG);
  template <int F1>
  static constexpr size_t W() { return al16(sizeof(float2) * kCG * PG * N0 * (F1 + 1)); }
  static constexpr size_t small = al16(sizeof(float) * (3 * kCG * NT + 3 * kCG + kCG));
  static constexpr size_t zbuf = al16(sizeof(T) * NIMG * NP * kCG);  // z = q' * g1(k'), reused by the epilogue
  template <int F1>
  static constexpr size_t total() { return stage + W<F1>() + small + zbuf; }
};

template <typename T, int N0, int N1, int F0, int F1, int SK, int PG>
__global__ void __launch_bounds__(256, (F0 <= 24 && F1 <= 24) ? 4 : 1) hyena2d_fwd_kernel(const Fused2DParams p) {
  using L = FwdSmem<T, N0, N1, SK, PG>;
  constexpr int NP = L::NP, NIMG = L::NIMG, NT = L::NT, LD = F1 + 1, NPAIR = kCG * PG;
  extern __shared__ __align__(16) unsigned char smem[];
  T* stage = reinterpret_cast<T*>(smem);                                       // [3][NIMG][NP][8]
  float2* W = reinterpret_cast<float2*>(smem + L::stage);                       // [NPAIR][N0][LD]
  float* wts = reinterpret_cast<float*>(smem + L::stage + L::template W<F1>());  // [3][NT][8]
  float* bsm = wts + 3 * kCG * NT;                                               // [3][8]
  float* Dsm = bsm + 3 * kCG;                                                    // [8]
  T* zs = reinterpret_cast<T*>(smem + L::stage + L::template W<F1>() + L::small);  // [NIMG][NP][8]
  const int tid = threadIdx.x;
  const int c0 = blockIdx.x * kCG;
  const int p0 = blockIdx.y * PG;

  for (int i = tid; i < 3 * kCG * NT; i += blockDim.x) {  // tap-major: the 8 channels of a tap are one vector
    const int t = i / (kCG * NT), r = i % (kCG * NT), tap = r / kCG, cc = r % kCG;
    wts[i] = SK > 0 ? p.w[((long long)t * p.C + c0 + cc) * NT + tap] : 1.f;
  }
  for (int i = tid; i < 3 * kCG; i += blockDim.x) {
    const int t = i / kCG, cc = i % kCG;
    bsm[i] = p.bias ? p.bias[t * p.C + c0 + cc] : 0.f;
  }
  if (tid < kCG) Dsm[tid] = p.D[c0 + tid];
  const T* src[3] = {reinterpret_cast<const T*>(p.q), reinterpret_cast<const T*>(p.k), reinterpret_cast<const T*>(p.v)};
  for (int i = tid; i < 3 * NIMG * NP; i += blockDim.x) {
    const int t = i / (NIMG * NP), r = i % (NIMG * NP), s = r / NP, pos = r % NP;
    const int pp = p0 + (s % PG);
    const int b = s < PG ? pp : pp + p.half;
    T* dst = stage + ((t * NIMG + s) * NP + pos) * kCG;
    const bool ok = pp < p.half && b < p.B;
    cp_v8<T>(dst, ok ? src[t] + (long long)b * p.in_bst + (long long)pos * p.in_pst + c0 : src[t], ok);
  }
  cp_wait_all();
  __syncthreads();

  const bool has_bias = p.bias != nullptr;
  // z = q' * g1(k') for both images of each pair -> W (re, im)
  for (int i = tid; i < PG * NP; i += blockDim.x) {
    const int ps = i / NP, pos = i % NP, n0 = pos / N1, n1 = pos % N1;
    float z[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int s = h * PG + ps;
      float qv[8], kv[8];
      stencil8<T, N0, N1, SK>(stage + (0 * NIMG + s) * NP * kCG, wts, has_bias ? bsm : nullptr, n0, n1, qv);
      stencil8<T, N0, N1, SK>(stage + (1 * NIMG + s) * NP * kCG, wts + kCG * NT, has_bias ? bsm + kCG : nullptr,
                              n0, n1, kv);
      round8<T>(qv);
      round8<T>(kv);
      if (p.qs) {  // keep q', k' for the backward
        const int pp = p0 + ps, b = h == 0 ? pp : pp + p.half;
        if (pp < p.half && b < p.B) {
          const long long o = ((long long)b * NP + pos) * p.C + c0;
          V8<T>::store(reinterpret_cast<T*>(p.qs) + o, qv);
          V8<T>::store(reinterpret_cast<T*>(p.ks) + o, kv);
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) z[h][c] = DT<T>::round(qv[c] * DT<T>::round(gate_f(p.gate1, kv[c])));
      V8<T>::store(zs + (s * NP + pos) * kCG, z[h]);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) W[((c * PG + ps) * N0 + n0) * LD + n1] = make_float2(z[0][c], z[1][c]);
  }
  __syncthreads();

  // rows: forward DIF along axis 1 (N1 -> F1, bit-reversed)
  for (int t = tid; t < NPAIR * N0; t += blockDim.x) {
    float2* row = W + t * LD;
    float2 v[F1];
#pragma unroll
    for (int i = 0; i < F1; ++i) v[i] = i < N1 ? row[i] : make_float2(0.f, 0.f);
    reg::fft_dif<F1, N1, -1>(v);
#pragma unroll
    for (int i = 0; i < F1; ++i) row[i] = v[i];
  }
  __syncthreads();

  // columns: DIF along axis 0, * filter spectrum, DIT back, keep rows [0, N0)
  const float inv = 1.0f / (float)(F0 * F1);
  for (int l = tid; l < NPAIR * F1; l += blockDim.x) {
    const int pi = l / F1, i1 = l % F1, c = c0 + pi / PG;
    float2* col = W + pi * N0 * LD + i1;
    float2 v[F0];
#pragma unroll
    for (int i = 0; i < F0; ++i) v[i] = i < N0 ? col[i * LD] : make_float2(0.f, 0.f);
    reg::fft_dif<F0, N0, -1>(v);
    const float2* kh = p.Kbr + (long long)c * F0 * F1 + i1;
#pragma unroll
    for (int i = 0; i < F0; ++i) v[i] = cmul(v[i], __ldg(kh + i * F1));
    reg::fft_dit<F0, N0, +1>(v);
#pragma unroll
    for (int i = 0; i < N0; ++i) col[i * LD] = cscale(v[i], inv);
  }
  __syncthreads();

  // rows: inverse DIT along axis 1, keep [0, N1)
  for (int t = tid; t < NPAIR * N0; t += blockDim.x) {
    float2* row = W + t * LD;
    float2 v[F1];
#pragma unroll
    for (int i = 0; i < F1; ++i) v[i] = row[i];
    reg::fft_dit<F1, N1, +1>(v);
#pragma unroll
    for (int i = 0; i < N1; ++i) row[i] = v[i];
  }
  __syncthreads();

  // epilogue: h = round(conv) + round(D z); y = h * g2(v')
  T* yout = reinterpret_cast<T*>(p.y);
  for (int i = tid; i < NIMG * NP; i += blockDim.x) {
    const int s = i / NP, pos = i % NP, n0 = pos / N1, n1 = pos % N1;
    const int ps = s % PG, h = s / PG;
    const int pp = p0 + ps;
    const int b = h == 0 ? pp : pp + p.half;
    if (pp >= p.half || b >= p.B) continue;
    float zv[8], vv[8], out[8];
    V8<T>::load(zs + (s * NP + pos) * kCG, zv);
    stencil8<T, N0, N1, SK>(stage + (2 * NIMG + s) * NP * kCG, wts + 2 * kCG * NT, has_bias ? bsm + 2 * kCG : nullptr,
                            n0, n1, vv);
    round8<T>(vv);
    if (p.vs) V8<T>::store(reinterpret_cast<T*>(p.vs) + ((long long)b * NP + pos) * p.C + c0, vv);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float2 cv = W[((c * PG + ps) * N0 + n0) * LD + n1];
      const float conv = h == 0 ? cv.x : cv.y;
      const float z = zv[c];
      const float hv = DT<T>::round(DT<T>::round(conv) + DT<T>::round(wtap8(Dsm, 0, c) * z));
      out[c] = hv * DT<T>::round(gate_f(p.gate2, vv[c]));
    }
    V8<T>::store(yout + (long long)b * p.out_bst + (long long)pos * p.out_pst + c0, out);
  }
}

// ------------------------------------------------------------------ backward
template <typename T, int N0, int N1, int SK>
struct BwdSmem {
  static constexpr int NP = N0 * N1, NIMG = 2, NT = SK > 0 ? SK * SK : 1;
  static constexpr size_t stage = al16(sizeof(T) * 4 * NIMG * NP * kCG);  // q, k, v, dy
  template <int F1>
  static constexpr size_t W() { return al16(sizeof(float2) * kCG * N0 * (F1 + 1)); }
  static constexpr size_t dgrad = al16(sizeof(T) * 3 * NIMG * NP * kCG);  // dq', dk', dv'
  static constexpr size_t qkv = al16(sizeof(T) * 3 * NIMG * NP * kCG);    // q', k', v' (short conv outputs)
  static constexpr size_t small = al16(sizeof(float) * (3 * kCG * NT + 3 * kCG + kCG + kCG + 3 * kCG * (NT + 1)));
  template <int F1>
  static constexpr size_t total() { return stage + 2 * W<F1>() + dgrad + qkv + small; }
};

template <typename T, int N0, int N1, int F0, int F1, int SK>
__global__ void __launch_bounds__(256, 2) hyena2d_bwd_kernel(const Fused2DParams p) {
  using L = BwdSmem<T, N0, N1, SK>;
  constexpr int NP = L::NP, NIMG = 2, NT = L::NT, LD = F1 + 1, NPAIR = kCG;
  extern __shared__ __align__(16) unsigned char smem[];
  T* stage = reinterpret_cast<T*>(smem);                                          // [4][2][NP][8]
  float2* W1 = reinterpret_cast<float2*>(smem + L::stage);                         // z -> h
  float2* W2 = reinterpret_cast<float2*>(smem + L::stage + L::template W<F1>());   // dh -> dz
  T* dgr = reinterpret_cast<T*>(smem + L::stage + 2 * L::template W<F1>());        // [3][2][NP][8]
  T* qkv = reinterpret_cast<T*>(smem + L::stage + 2 * L::template W<F1>() + L::dgrad);  // [3][2][NP][8]
  float* wts = reinterpret_cast<float*>(smem + L::stage + 2 * L::template W<F1>() + L::dgrad + L::qkv);
  float* bsm = wts + 3 * kCG * NT;
  float* Dsm = bsm + 3 * kCG;
  float* dDsm = Dsm + kCG;
  float* dwsm = dDsm + kCG;  // [3][8][NT + 1] short-conv weight (and bias) gradient of this CTA
  const int tid = threadIdx.x;
  const int c0 = blockIdx.x * kCG;
  const int pp = blockIdx.y;  // pair index: items pp and pp + half
  for (int i = tid; i < 3 * kCG * (NT + 1); i += blockDim.x) dwsm[i] = 0.f;

  for (int i = tid; i < 3 * kCG * NT; i += blockDim.x) {  // tap-major: the 8 channels of a tap are one vector
    const int t = i / (kCG * NT), r = i % (kCG * NT), tap = r / kCG, cc = r % kCG;
    wts[i] = SK > 0 ? p.w[((long long)t * p.C + c0 + cc) * NT + tap] : 1.f;
  }
  for (int i = tid; i < 3 * kCG; i += blockDim.x) {
    const int t = i / kCG, cc = i % kCG;
    bsm[i] = p.bias ? p.bias[t * p.C + c0 + cc] : 0.f;
  }
  if (tid < kCG) {
    Dsm[tid] = p.D[c0 + tid];
    dDsm[tid] = 0.f;
  }
  const T* src[4] = {reinterpret_cast<const T*>(p.q), reinterpret_cast<const T*>(p.k), reinterpret_cast<const T*>(p.v),
                     reinterpret_cast<const T*>(p.dy)};
  for (int i = tid; i < 4 * NIMG * NP; i += blockDim.x) {
    const int t = i / (NIMG * NP), r = i % (NIMG * NP), s = r / NP, pos = r % NP;
    const int b = s == 0 ? pp : pp + p.half;
    T* dst = stage + ((t * NIMG + s) * NP + pos) * kCG;
    const long long bst = t == 3 ? p.out_bst : p.in_bst, pst = t == 3 ? p.out_pst : p.in_pst;
    cp_v8<T>(dst, b < p.B ? src[t] + (long long)b * bst + (long long)pos * pst + c0 : src[t], b < p.B);
  }
  const bool kept = p.qs != nullptr;  // q', k', v' saved by the forward
  if (kept) {
    const T* sv[3] = {reinterpret_cast<const T*>(p.qs), reinterpret_cast<const T*>(p.ks),
                      reinterpret_cast<const T*>(p.vs)};
    for (int i = tid; i < 3 * NIMG * NP; i += blockDim.x) {
      const int t = i / (NIMG * NP), r = i % (NIMG * NP), s = r / NP, pos = r % NP;
      const int b = s == 0 ? pp : pp + p.half;
      T* dst = qkv + ((t * NIMG + s) * NP + pos) * kCG;
      cp_v8<T>(dst, b < p.B ? sv[t] + ((long long)b * NP + pos) * p.C + c0 : sv[t], b < p.B);
    }
  }
  cp_wait_all();
  __syncthreads();

  const bool has_bias = p.bias != nullptr;
  // z and dh = dy * g2(v') for both images -> W1, W2
  for (int pos = tid; pos < NP; pos += blockDim.x) {
    const int n0 = pos / N1, n1 = pos % N1;
    float z[2][8], dh[2][8];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      float qv[8], kv[8], vv[8], g[8];
      if (kept) {
        V8<T>::load(qkv + ((0 * NIMG + s) * NP + pos) * kCG, qv);
        V8<T>::load(qkv + ((1 * NIMG + s) * NP + pos) * kCG, kv);
        V8<T>::load(qkv + ((2 * NIMG + s) * NP + pos) * kCG, vv);
      } else {
        stencil8<T, N0, N1, SK>(stage + (0 * NIMG + s) * NP * kCG, wts, has_bias ? bsm : nullptr, n0, n1, qv);
        stencil8<T, N0, N1, SK>(stage + (1 * NIMG + s) * NP * kCG, wts + kCG * NT, has_bias ? bsm + kCG : nullptr,
                                n0, n1, kv);
        stencil8<T, N0, N1, SK>(stage + (2 * NIMG + s) * NP * kCG, wts + 2 * kCG * NT,
                                has_bias ? bsm + 2 * kCG : nullptr, n0, n1, vv);
        round8<T>(qv);
        round8<T>(kv);
        round8<T>(vv);
        V8<T>::store(qkv + ((0 * NIMG + s) * NP + pos) * kCG, qv);
        V8<T>::store(qkv + ((1 * NIMG + s) * NP + pos) * kCG, kv);
        V8<T>::store(qkv + ((2 * NIMG + s) * NP + pos) * kCG, vv);
      }
      V8<T>::load(stage + ((3 * NIMG + s) * NP + pos) * kCG, g);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        z[s][c] = DT<T>::round(qv[c] * DT<T>::round(gate_f(p.gate1, kv[c])));
        dh[s][c] = DT<T>::round(g[c] * DT<T>::round(gate_f(p.gate2, vv[c])));
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      W1[(c * N0 + n0) * LD + n1] = make_float2(z[0][c], z[1][c]);
      W2[(c * N0 + n0) * LD + n1] = make_float2(dh[0][c], dh[1][c]);
    }
  }
  __syncthreads();

  // rows: forward DIF of both buffers
  for (int t = tid; t < 2 * NPAIR * N0; t += blockDim.x) {
    float2* row = (t < NPAIR * N0 ? W1 : W2) + (t % (NPAIR * N0)) * LD;
    float2 v[F1];
#pragma unroll
    for (int i = 0; i < F1; ++i) v[i] = i < N1 ? row[i] : make_float2(0.f, 0.f);
    reg::fft_dif<F1, N1, -1>(v);
#pragma unroll
    for (int i = 0; i < F1; ++i) row[i] = v[i];
  }
  __syncthreads();

  // columns: spectra of z and dh; dK += DH conj(Z); H = K Z; DZ = DH conj(K); inverse
  const float inv = 1.0f / (float)(F0 * F1);
  for (int l = tid; l < NPAIR * F1; l += blockDim.x) {
    const int cc = l / F1, i1 = l % F1, c = c0 + cc;
    float2* colz = W1 + cc * N0 * LD + i1;
    float2* cold = W2 + cc * N0 * LD + i1;
    float2 vz[F0], vd[F0];
#pragma unroll
    for (int i = 0; i < F0; ++i) vd[i] = i < N0 ? cold[i * LD] : make_float2(0.f, 0.f);
    reg::fft_dif<F0, N0, -1>(vd);
#pragma unroll
    for (int i = 0; i < F0; ++i) vz[i] = i < N0 ? colz[i * LD] : make_float2(0.f, 0.f);
    reg::fft_dif<F0, N0, -1>(vz);
    const float2* kh = p.Kbr + (long long)c * F0 * F1 + i1;
    float2* gacc = p.G + (long long)c * F0 * F1 + i1;
#pragma unroll
    for (int i = 0; i < F0; ++i) {
      const float2 kk = __ldg(kh + i * F1);
      atomicAdd(gacc + i * F1, cmulc(vd[i], vz[i]));
      vz[i] = cmul(vz[i], kk);
      vd[i] = cmulc(vd[i], kk);
    }
    reg::fft_dit<F0, N0, +1>(vz);
    reg::fft_dit<F0, N0, +1>(vd);
#pragma unroll
    for (int i = 0; i < N0; ++i) {
      colz[i * LD] = cscale(vz[i], inv);
      cold[i * LD] = cscale(vd[i], inv);
    }
  }
  __syncthreads();

  // rows: inverse DIT of both buffers
  for (int t = tid; t < 2 * NPAIR * N0; t += blockDim.x) {
    float2* row = (t < NPAIR * N0 ? W1 : W2) + (t % (NPAIR * N0)) * LD;
    float2 v[F1];
#pragma unroll
    for (int i = 0; i < F1; ++i) v[i] = row[i];
    reg::fft_dit<F1, N1, +1>(v);
#pragma unroll
    for (int i = 0; i < N1; ++i) row[i] = v[i];
  }
  __syncthreads();

  // elementwise backward: gate 2, D-skip, gate 1 -> dq', dk', dv' (activation dtype, as
  // autograd produces them) in shared memory; dD partial sums
  float dDp[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) dDp[c] = 0.f;
  for (int i = tid; i < NIMG * NP; i += blockDim.x) {
    const int s = i / NP, pos = i % NP, n0 = pos / N1, n1 = pos % N1;
    float qv[8], kv[8], vv[8], g[8], oq[8], ok[8], ov[8];
    V8<T>::load(qkv + ((0 * NIMG + s) * NP + pos) * kCG, qv);
    V8<T>::load(qkv + ((1 * NIMG + s) * NP + pos) * kCG, kv);
    V8<T>::load(qkv + ((2 * NIMG + s) * NP + pos) * kCG, vv);
    V8<T>::load(stage + ((3 * NIMG + s) * NP + pos) * kCG, g);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float2 ch = W1[(c * N0 + n0) * LD + n1];
      const float2 cd = W2[(c * N0 + n0) * LD + n1];
      const float conv_h = s == 0 ? ch.x : ch.y;
      const float conv_d = s == 0 ? cd.x : cd.y;
      const float g1k = DT<T>::round(gate_f(p.gate1, kv[c]));
      const float z = DT<T>::round(qv[c] * g1k);
      const float g2v = DT<T>::round(gate_f(p.gate2, vv[c]));
      const float hv = DT<T>::round(DT<T>::round(conv_h) + DT<T>::round(wtap8(Dsm, 0, c) * z));
      const float dh = DT<T>::round(g[c] * g2v);
      ov[c] = g[c] * hv * gate_df(p.gate2, vv[c]);
      const float dz = DT<T>::round(DT<T>::round(conv_d) + DT<T>::round(wtap8(Dsm, 0, c) * dh));
      oq[c] = dz * g1k;
      ok[c] = dz * qv[c] * gate_df(p.gate1, kv[c]);
      dDp[c] = fmaf(dh, z, dDp[c]);
    }
    V8<T>::store(dgr + ((0 * NIMG + s) * NP + pos) * kCG, oq);
    V8<T>::store(dgr + ((1 * NIMG + s) * NP + pos) * kCG, ok);
    V8<T>::store(dgr + ((2 * NIMG + s) * NP + pos) * kCG, ov);
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float vsum = dDp[c];
    for (int o = 16; o > 0; o >>= 1) vsum += __shfl_xor_sync(0xffffffffu, vsum, o);
    if ((tid & 31) == 0) atomicAdd(dDsm + c, vsum);
  }
  __syncthreads();
  if (tid < kCG) atomicAdd(p.dD + c0 + tid, dDsm[tid]);

  // short conv input gradients (transposed stencil) -> dq, dk, dv (channels-last)
  T* outs[3] = {reinterpret_cast<T*>(p.dq), reinterpret_cast<T*>(p.dk), reinterpret_cast<T*>(p.dv)};
  constexpr int NH = (N1 + 1) / 2;  // output pairs per row
  for (int i = tid; i < 3 * NIMG * N0 * NH; i += blockDim.x) {
    const int t = i / (NIMG * N0 * NH), r = i % (NIMG * N0 * NH), s = r / (N0 * NH), rr = r % (N0 * NH);
    const int n0 = rr / NH, n1 = (rr % NH) * 2, pos = n0 * N1 + n1;
    const int b = s == 0 ? pp : pp + p.half;
    if (b >= p.B) continue;
    float o0[8], o1[8];
    stencil8_t2<N0, N1, SK, T>(dgr + (t * NIMG + s) * NP * kCG, wts + t * kCG * NT, n0, n1, o0, o1);
    T* dst = outs[t] + (long long)b * p.in_bst + (long long)pos * p.in_pst + c0;  // dq, dk, dv mirror q, k, v
    V8<T>::store(dst, o0);
    if (n1 + 1 < N1) V8<T>::store(dst + p.in_pst, o1);
  }
  // short conv weight / bias gradients: one task per (tensor, image, output row, channel)
  // slides a SK x SK window of the input along the row, accumulates all taps (and the
  // bias) in registers and adds them into the CTA's shared accumulator
  if constexpr (SK > 0) {
    constexpr int OFF = (SK - 1) / 2;
    for (int i = tid; i < 3 * NIMG * N0 * kCG; i += blockDim.x) {
      const int cc = i % kCG, n0 = (i / kCG) % N0, s = (i / (kCG * N0)) % NIMG, t = i / (kCG * N0 * NIMG);
      const T* go = dgr + (t * NIMG + s) * NP * kCG + cc;
      const T* in = stage + (t * NIMG + s) * NP * kCG + cc;
      float acc[NT + 1];
#pragma unroll
      for (int j = 0; j <= NT; ++j) acc[j] = 0.f;
      float win[SK][SK];  // win[a][e] = in[n0 + a - OFF][n1 + e - OFF]
      auto ld = [&](int r, int c) -> float {
        return (r >= 0 && r < N0 && c >= 0 && c < N1) ? DT<T>::load(in + (r * N1 + c) * kCG) : 0.f;
      };
#pragma unroll
      for (int a = 0; a < SK; ++a)
#pragma unroll
        for (int e = 1; e < SK; ++e) win[a][e] = ld(n0 + a - OFF, e - 1 - OFF);
#pragma unroll 2
      for (int n1 = 0; n1 < N1; ++n1) {
#pragma unroll
        for (int a = 0; a < SK; ++a) {
#pragma unroll
          for (int e = 0; e + 1 < SK; ++e) win[a][e] = win[a][e + 1];
          win[a][SK - 1] = ld(n0 + a - OFF, n1 + SK - 1 - OFF);
        }
        const float g = DT<T>::load(go + (n0 * N1 + n1) * kCG);
#pragma unroll
        for (int a = 0; a < SK; ++a)
#pragma unroll
          for (int e = 0; e < SK; ++e) acc[a * SK + e] = fmaf(g, win[a][e], acc[a * SK + e]);
        acc[NT] += g;
      }
      if constexpr ((N0 % 2) == 0) {
        // the task count is a multiple of 32 and a warp never spans two tensors: lanes l, l + 8,
        // l + 16, l + 24 hold the same (tensor, channel), so sum them before one atomic per value
#pragma unroll
        for (int j = 0; j <= NT; ++j) {
          acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], 8);
          acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], 16);
        }
        if ((tid & 31) < 8) {
#pragma unroll
          for (int j = 0; j <= NT; ++j) atomicAdd(dwsm + (t * kCG + cc) * (NT + 1) + j, acc[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j <= NT; ++j) atomicAdd(dwsm + (t * kCG + cc) * (NT + 1) + j, acc[j]);
      }
    }
    __syncthreads();
    for (int i = tid; i < 3 * kCG * (NT + 1); i += blockDim.x) {
      const int t = i / (kCG * (NT + 1)), r = i % (kCG * (NT + 1)), cc = r / (NT + 1), tap = r % (NT + 1);
      if (tap < NT) atomicAdd(p.dw + ((long long)t * p.C + c0 + cc) * NT + tap, dwsm[i]);
      else if (p.db) atomicAdd(p.db + (long long)t * p.C + c0 + cc, dwsm[i]);
    }
  }
}

// ------------------------------------------------------------------ dispatch
struct Shape2D {
  int N0, N1, F0, F1;
};

template <typename T, int N0, int N1, int F0, int F1, int SK>
struct Fused2D {
  static constexpr int PG = 1;
  static size_t fwd_smem() { return FwdSmem<T, N0, N1, SK, PG>::template total<F1>(); }
  static size_t bwd_smem() { return BwdSmem<T, N0, N1, SK>::template total<F1>(); }

  static int launch_kspec(const Fused2DParams& p, cudaStream_t st) {
    kspec2d_kernel<F0, F1><<<p.C, 64, 0, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  static int fwd(const Fused2DParams& p, cudaStream_t st) {
    auto kern = hyena2d_fwd_kernel<T, N0, N1, F0, F1, SK, PG>;
    const size_t sm = fwd_smem();
    if (!kernel_smem_once((const void*)kern, sm, true)) return HYFFT_ERR_CUDA;
    dim3 grid(p.C / kCG, (p.half + PG - 1) / PG);
    kern<<<grid, 256, sm, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  static int bwd(const Fused2DParams& p, cudaStream_t st) {
    auto kern = hyena2d_bwd_kernel<T, N0, N1, F0, F1, SK>;
    const size_t sm = bwd_smem();
    if (!kernel_smem_once((const void*)kern, sm, true)) return HYFFT_ERR_CUDA;
    dim3 grid(p.C / kCG, p.half);
    kern<<<grid, 256, sm, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
  static int dfilt(const Fused2DParams& p, cudaStream_t st) {
    dfilt2d_kernel<F0, F1><<<p.C, 64, 0, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? HYFFT_OK : HYFFT_ERR_CUDA;
  }
};

// Every (grid, FFT size, short-conv size) the fused path is compiled for.
#define HYFFT_FUSED2D_SHAPES(X) \
  X(14, 14, 24, 24)             \
  X(16, 16, 24, 24)             \
  X(14, 14, 32, 32)             \
  X(16, 16, 32, 32)             \
  X(12, 10, 32, 32)             \
  X(6, 6, 16, 16)               \
  X(7, 5, 16, 16)               \
  X(8, 8, 16, 16)


template <typename T, int N0, int N1, int F0, int F1, int SK>
static int fused_run(int op, const Fused2DParams& p, cudaStream_t st) {
  using X = Fused2D<T, N0, N1, F0, F1, SK>;
  switch (op) {
    case FOP_KSPEC: return X::launch_kspec(p, st);
    case FOP_FWD: return X::fwd(p, st);
    case FOP_BWD: return X::bwd(p, st);
    case FOP_DFILT: return X::dfilt(p, st);
    default: return (X::fwd_smem() <= 227 * 1024 && X::bwd_smem() <= 227 * 1024) ? HYFFT_OK : HYFFT_ERR_UNSUPPORTED;
  }
}

template <typename T>
static int fused_dispatch_t(int op, int N0, int N1, int F0, int F1, int SK, const Fused2DParams& p, cudaStream_t st) {
#define HYFFT_TRY_SHAPE(a, b, c, d)                                          \
  if (N0 == a && N1 == b && F0 == c && F1 == d) {                           \
    if (SK == 3) return fused_run<T, a, b, c, d, 3>(op, p, st);             \
    if (SK == 0) return fused_run<T, a, b, c, d, 0>(op, p, st);             \
  }
  HYFFT_FUSED2D_SHAPES(HYFFT_TRY_SHAPE)
#undef HYFFT_TRY_SHAPE
  return HYFFT_ERR_UNSUPPORTED;
}

// Returns HYFFT_OK (launched / supported), HYFFT_ERR_UNSUPPORTED (not compiled for
// this shape: caller uses the general engine) or HYFFT_ERR_CUDA.
int fused2d_dispatch(int op, int dtype, int N0, int N1, int F0, int F1, int SK, const Fused2DParams* p,
                     cudaStream_t st) {
  int rc;
  if (dtype == HYFFT_BF16) rc = fused_dispatch_t<__nv_bfloat16>(op, N0, N1, F0, F1, SK, *p, st);
  else if (dtype == HYFFT_F32) rc = fused_dispatch_t<float>(op, N0, N1, F0, F1, SK, *p, st);
  else rc = HYFFT_ERR_UNSUPPORTED;
  if (rc == HYFFT_OK && op != FOP_PROBE) g_launches.fetch_add(1, std::memory_order_relaxed);
  return rc;
}

}  // namespace hyfft
