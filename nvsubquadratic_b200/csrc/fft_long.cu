// Channel-innermost passes of the long 1D transform (the four-step decomposition
// F = Fa * Fb of a causal / linear 1D convolution whose FFT length exceeds one CTA's line
// tile): each pass transforms lines of Fa or Fb = 64 .. 4096 points whose neighbours are
// neighbouring channels (the spectra are stored [pair][k_a][n_b or k_b][C], channels-last
// activations [b][pos][C]).
//
// One CTA owns NL = min(32, 16384 / F) neighbouring lines (a run of channels) and 512
// threads. The line transform is a three-level decomposition F = R1 * R2 * R3 with every
// level's radix in registers and two transposes through shared memory:
//   t = j + M r             (M = R2 R3, r < R1)      level 1 over r, twiddle W_F^(j k1)
//   j = i + R3 s            (s < R2)                 level 2 over s, twiddle W_M^(i k2)
//   k = k1 + R1 k2 + R1 R2 k3                         level 3 over i
// Level 1 reads its R1 points of a line straight from global memory (the lanes of a warp
// cover the NL lines, so every access is NL neighbouring channels), level 3 writes straight
// to global memory. Every global read of a CTA happens before its first barrier and every
// CTA only writes the points of its own lines, so a pass may run in place.
//
// The four-step twiddle W_{2^tw}^(t m) (m = the line's other-axis index) is applied on the
// store from two 4096-entry tables (high and low 12 bits of the exponent in units of
// 2^-24 of a turn), filled once per device from double precision.
//
// MID != 0 (product pass of a convolution): forward transform, product with the filter
// spectrum at the same index (MID == 2: its conjugate), then the adjoint levels in reverse
// order (level 3 inverse in the same registers, level 2 and level 1 inverse with the
// conjugate twiddles) and the store of the inverse pass, post-twiddle included.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "../../include/hyfft.h"
#include "fft_long.h"
#include "fft_pass.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;

#ifndef HYFFT_LONG_THREADS
#define HYFFT_LONG_THREADS 512
#define HYFFT_LONG_POINTS 16384
#define HYFFT_LONG_MINB 1
#endif
constexpr int kLongThreads = HYFFT_LONG_THREADS;
constexpr int kLongPoints = HYFFT_LONG_POINTS;  // F * NL per CTA
constexpr int kLongMinBlocks = HYFFT_LONG_MINB;

// e^{-2 pi i e / 4096} and e^{-2 pi i e / 2^24}, e < 4096
static __device__ float2 g_long_tw_hi[4096];
static __device__ float2 g_long_tw_lo[4096];

template <int F>
__host__ __device__ constexpr int long_lines() { return kLongPoints / F < 32 ? kLongPoints / F : 32; }
template <int F>
__host__ __device__ constexpr int long_bwd_lines() { return long_lines<F>() / 2; }

// Shared-memory layout of a CTA's lines: point p of line l at (p + p / R3) * NL + l (one pad
// row of NL slots after every R3 points, so that the level-3 reads, lanes on consecutive
// k2 and points R3 apart, spread over the banks). Every level reads and writes its R points
// at compile-time offsets from one per-item base:
//   level 1 (l, j):      p = k1 M + j             -> base (j + j / R3) NL + l,         k1 * C1
//   level 2 (l, i, k1):  p = k1 M + i + R3 s      -> base (k1 M' + i) NL + l,          s * C2
//   level 3 (l, k1, k2): p = k1 M + k2 R3 + i     -> base (k1 M' + k2 (R3 + 1)) NL + l, i * NL
// with M' = M + M / R3, C1 = M' NL, C2 = (R3 + 1) NL.
template <int R1, int R2, int R3, int NL>
struct LongIdx {
  static constexpr int M = R2 * R3, MP = M + M / R3, C1 = MP * NL, C2 = (R3 + 1) * NL;
  static __device__ __forceinline__ int b1(int l, int j) { return (j + j / R3) * NL + l; }
  static __device__ __forceinline__ int b2(int l, int i, int k1) { return (k1 * MP + i) * NL + l; }
  static __device__ __forceinline__ int b3(int l, int k1, int k2) { return (k1 * MP + k2 * (R3 + 1)) * NL + l; }
};

// Twiddles of the line transform in shared memory, laid out so that a level's per-item base
// plus a compile-time offset addresses them and neighbouring lanes read neighbouring entries:
//   T1[k1 M + j] = W_F^(j k1)  (F entries),   T2[k2 R3 + i] = W_M^(i k2)  (M entries).
template <int R1, int R2, int R3>
__host__ __device__ constexpr int long_twn() { return R1 * R2 * R3 + R2 * R3; }

template <int R1, int R2, int R3, int NSETS = 1>
__host__ __device__ constexpr size_t long_smem_bytes() {
  constexpr int F = R1 * R2 * R3, NL = NSETS == 1 ? long_lines<F>() : long_bwd_lines<F>();
  return sizeof(float2) * ((size_t)NSETS * (F + F / R3) * NL + long_twn<R1, R2, R3>() + F) +
         5 * sizeof(long long) * NL + 3 * sizeof(int) * NL;
}

template <int R1, int R2, int R3>
__device__ __forceinline__ void long_fill_twiddles(float2* tw) {
  constexpr int F = R1 * R2 * R3, M = R2 * R3;
  for (int e = threadIdx.x; e < F + M; e += kLongThreads) {
    int x;
    if (e < F) x = (e % M) * (e / M);               // j k1
    else x = R1 * ((e - F) % R3) * ((e - F) / R3);  // R1 i k2 (W_M = W_F^R1)
    tw[e] = __ldg(&g_long_tw_hi[x * (4096 / F)]);
  }
}

__device__ __forceinline__ float2 conj_if(float2 w, float dir) {
  if (dir > 0.f) w.y = -w.y;
  return w;
}

// e^{dir 2 pi i ex / 2^tw_logF} for 0 <= ex < 2^tw_logF <= 2^24
__device__ __forceinline__ float2 four_step_twiddle(unsigned ex, int tw_logF, float dir) {
  const unsigned e24 = ex << (24 - tw_logF);
  return conj_if(cmul(__ldg(&g_long_tw_hi[e24 >> 12]), __ldg(&g_long_tw_lo[e24 & 4095u])), dir);
}

// Scale and four-step twiddle of the run of points t0 + S q (q = 0, 1, ...) of a line with
// multiplier m: w_q = scale e^{dir 2 pi i m (t0 + S q) / 2^tw_logF} = w * s^q, both factors
// exact from the tables, the powers by recurrence (at most 15 products, relative error
// below 2e-6).
struct TwRun {
  float2 w, s;
};
__device__ __forceinline__ TwRun tw_run(int m, int t0, int S, int tw_logF, float scale, float dir) {
  TwRun r;
  if (tw_logF == 0 || m == 0) {
    r.w = make_float2(scale, 0.f);
    r.s = make_float2(1.f, 0.f);
    return r;
  }
  const unsigned mask = (1u << tw_logF) - 1u;  // m, t0, S < 2^12: the products fit 32 bits
  r.w = cscale(four_step_twiddle(((unsigned)m * (unsigned)t0) & mask, tw_logF, dir), scale);
  r.s = four_step_twiddle(((unsigned)m * (unsigned)S) & mask, tw_logF, dir);
  return r;
}

// Store-side twiddle table of a CTA whose lines share one four-step multiplier m (the channel
// count is a multiple of the lines per CTA): T4[e] = scale e^{dir 2 pi i m t(e) / 2^tw_logF}
// for the F output points, in the order the storing level walks them, so that an item's
// points sit at compile-time offsets and neighbouring lanes read neighbouring entries:
//   level-3 store (k1, k2; k3):  e = (k1 R3 + k3) R2 + k2,  t = k1 + R1 k2 + R1 R2 k3
//   adjoint level-1 store (j; r): e = r M + j,              t = j + M r
template <int R1, int R2, int R3, bool L1ORDER>
__device__ __forceinline__ void long_fill_store_twiddles(float2* t4, int m, int tw_logF, float scale, float dir) {
  constexpr int F = R1 * R2 * R3, M = R2 * R3;
  const unsigned mask = (1u << tw_logF) - 1u;
  for (int e = threadIdx.x; e < F; e += kLongThreads) {
    int t;
    if constexpr (L1ORDER) {
      t = e % M + M * (e / M);
    } else {
      const int k2 = e % R2, k3 = (e / R2) % R3, k1 = e / (R2 * R3);
      t = k1 + R1 * k2 + R1 * R2 * k3;
    }
    t4[e] = cscale(four_step_twiddle(((unsigned)m * (unsigned)t) & mask, tw_logF, dir), scale);
  }
}

// Per-line bookkeeping of a CTA's lines in shared memory.
struct LongLines {
  long long *cb_in, *cb_out, *im_in, *im_out, *kbase;
  int *chan, *twm, *pos0;
};
template <int NL>
__device__ __forceinline__ LongLines long_lines_at(void* p) {
  LongLines L;
  L.cb_in = reinterpret_cast<long long*>(p);
  L.cb_out = L.cb_in + NL;
  L.im_in = L.cb_out + NL;
  L.im_out = L.im_in + NL;
  L.kbase = L.im_out + NL;
  L.chan = reinterpret_cast<int*>(L.kbase + NL);
  L.twm = L.chan + NL;
  L.pos0 = L.twm + NL;
  return L;
}

// The R points of a run t0 + S q of line l, forward-ordered, scaled, twiddled and stored
// with the output window, dtype rounding and D-skip of the pass (fft_pass_kernel semantics).
// full: every point of the run lies inside the output window (complex output).
// D * skip of the real item of a run (rounded to the activation dtype), loaded ahead
template <int R, typename TO>
__device__ __forceinline__ void long_skip_run(const PassDesc& d, const LongLines& L, int l, int t0, int S,
                                              float (&sre)[R]) {
  const int pb = t0 * d.pos_mul + L.pos0[l] - d.out_lo, ps = S * d.pos_mul;
  const long long step = (long long)ps * d.ro_tst;
  const TO* sk = reinterpret_cast<const TO*>(d.skip) + L.cb_out[l] + (long long)pb * d.ro_tst;
  const float Dc = reinterpret_cast<const float*>(d.Dv)[L.chan[l]];
#pragma unroll
  for (int q = 0; q < R; ++q) {
    const int pos = pb + ps * q;
    sre[q] = (pos >= 0 && pos < d.n_out) ? DT<TO>::round(Dc * DT<TO>::load(sk + q * step)) : 0.f;
  }
}

// pre: D * skip of the real item from long_skip_run (OUT_REAL_SKIP)
// tt: this run's entries of the store twiddle table (stride TS), or null (factors from tw_run)
template <int R, int TS, int OM, typename TO>
__device__ __forceinline__ void long_store_run(const PassDesc& d, const LongLines& L, int l, int t0, int S, float sd,
                                               bool full, float2 (&v)[R], const float (&pre)[R], const float2* tt) {
  TwRun tr;
  if (!tt) tr = tw_run(L.twm[l], t0, S, d.tw_logF, d.scale, sd);
  auto wq = [&](int q) {
    if (tt) return tt[q * TS];
    const float2 w = tr.w;
    tr.w = cmul(tr.w, tr.s);
    return w;
  };
  if constexpr (OM == OUT_CPLX) {
    float2* dst = d.cout + L.cb_out[l] + (long long)(t0 - d.out_lo) * d.co_tst;
    const long long step = (long long)S * d.co_tst;
    if (full) {
#pragma unroll
      for (int q = 0; q < R; ++q) dst[q * step] = cmul(v[q], wq(q));
    } else {
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const int bo = t0 + S * q - d.out_lo;
        const float2 w = wq(q);
        if (bo >= 0 && bo < d.n_out) dst[q * step] = cmul(v[q], w);
      }
    }
  } else {
    const int pb = t0 * d.pos_mul + L.pos0[l] - d.out_lo, ps = S * d.pos_mul;
    const long long off0 = (long long)pb * d.ro_tst, step = (long long)ps * d.ro_tst;
    TO* dst = reinterpret_cast<TO*>(d.rout) + L.cb_out[l] + off0;
    const long long ri = L.im_out[l];
    TO* dsti = reinterpret_cast<TO*>(d.rout) + ri + off0;
    float sim[R];  // D * skip of the imaginary item, loaded ahead of the stores (which may alias it)
    if constexpr (OM == OUT_REAL_SKIP) {
      const TO* ski = reinterpret_cast<const TO*>(d.skip) + ri + off0;
      const float Dc = reinterpret_cast<const float*>(d.Dv)[L.chan[l]];
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const int pos = pb + ps * q;
        sim[q] = (ri >= 0 && pos >= 0 && pos < d.n_out) ? DT<TO>::round(Dc * DT<TO>::load(ski + q * step)) : 0.f;
      }
    }
#pragma unroll
    for (int q = 0; q < R; ++q) {
      const int pos = pb + ps * q;
      const float2 val = cmul(v[q], wq(q));
      if (pos < 0 || pos >= d.n_out) continue;
      float re = DT<TO>::round(val.x), im = DT<TO>::round(val.y);
      if constexpr (OM == OUT_REAL_SKIP) {
        re = re + pre[q];
        im = im + sim[q];
      }
      DT<TO>::store(dst + q * step, re);
      if (ri >= 0) DT<TO>::store(dsti + q * step, im);
    }
  }
}

template <int R1, int R2, int R3, int MID, int DIR, int IM, int OM, typename TI, typename TO>
__global__ void __launch_bounds__(kLongThreads, kLongMinBlocks) fft_long_cl_kernel(const PassDesc d) {
  constexpr int F = R1 * R2 * R3, M = R2 * R3, S3 = R1 * R2;
  constexpr int NL = long_lines<F>();
  constexpr int T = kLongThreads;
  constexpr int N1 = NL * M, N2 = NL * R1 * R3, N3 = NL * R1 * R2;  // items per level
  constexpr int IT1 = (N1 + T - 1) / T, IT2 = (N2 + T - 1) / T, IT3 = (N3 + T - 1) / T;
  using X = LongIdx<R1, R2, R3, NL>;
  constexpr float D1 = MID ? -1.f : (float)DIR;  // direction of the forward levels
  constexpr float SD = MID ? 1.f : (float)DIR;   // direction of the store-side twiddle
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float2* sm = reinterpret_cast<float2*>(smem_raw);  // [(F + F / R3)][NL]
  float2* tw = sm + (size_t)(F + F / R3) * NL;       // T1 then T2
  const float2* T1 = tw;
  const float2* T2 = tw + F;
  float2* T4 = tw + long_twn<R1, R2, R3>();  // [F] store twiddles (uniform multiplier)
  const LongLines L = long_lines_at<NL>(T4 + F);
  const long long line0 = (long long)blockIdx.x * NL;
  long_fill_twiddles<R1, R2, R3>(tw);
  for (int l = threadIdx.x; l < NL; l += T) {
    const long long lid = line0 + l;
    if (lid >= d.nlines) {
      L.cb_in[l] = -1;
      continue;
    }
    const int c = (int)(lid % d.C);
    long long rest = lid / d.C;
    int o[2] = {0, 0};
    for (int a = d.n_oth - 1; a >= 0; --a) {
      o[a] = (int)(rest % d.oth_ext[a]);
      rest /= d.oth_ext[a];
    }
    const long long p = rest;
    const bool has_im = d.packed && p + d.half < d.B;
    L.chan[l] = c;
    L.twm[l] = o[0];
    L.pos0[l] = o[0] * d.pos_oth;
    if (IM == IN_CPLX) {
      L.cb_in[l] = p * d.ci_pst + (long long)o[0] * d.ci_ost[0] + (long long)o[1] * d.ci_ost[1] + c;
    } else {
      L.cb_in[l] = p * d.ri_bst + (long long)c * d.ri_cst + (long long)o[0] * d.ri_ost[0] + (long long)o[1] * d.ri_ost[1];
      L.im_in[l] = has_im ? L.cb_in[l] + (long long)d.half * d.ri_bst : -1;
    }
    if (OM == OUT_CPLX) {
      L.cb_out[l] = p * d.co_pst + (long long)o[0] * d.co_ost[0] + (long long)o[1] * d.co_ost[1] + c;
    } else {
      L.cb_out[l] = p * d.ro_bst + (long long)c * d.ro_cst + (long long)o[0] * d.ro_ost[0] + (long long)o[1] * d.ro_ost[1];
      L.im_out[l] = has_im ? L.cb_out[l] + (long long)d.half * d.ro_bst : -1;
    }
    if (MID) L.kbase[l] = (d.k_shared ? 0 : p) * d.k_pst + (long long)o[0] * d.k_ost[0] + (long long)o[1] * d.k_ost[1] + c;
  }
  __syncthreads();
  const bool full_out = OM == OUT_CPLX && d.out_lo == 0 && d.n_out >= F;
  // the CTA's lines share one four-step multiplier when the channel count is a multiple of NL
  const float2* t4 = (d.tw_logF > 0 && d.C % NL == 0) ? T4 : nullptr;

  // level 1: R1-point transforms over r of x[j + M r], twiddle W_F^(j k1) -> A[k1 M + j];
  // the loads of all of a thread's items are issued before the first transform
  {
    float2 v[IT1][R1];
#pragma unroll
    for (int u = 0; u < IT1; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, j = it / NL;
      if (N1 % T != 0 && it >= N1) continue;
      const long long base = L.cb_in[l];
      if constexpr (IM == IN_CPLX) {
        const int b0 = j - d.in_off;
        const float2* src = d.cin + base + (long long)b0 * d.ci_tst;
        const long long step = (long long)M * d.ci_tst;
        if (base >= 0 && d.in_off == 0 && d.n_in >= F) {
#pragma unroll
          for (int r = 0; r < R1; ++r) v[u][r] = src[r * step];
        } else {
#pragma unroll
          for (int r = 0; r < R1; ++r) {
            const int bi = b0 + M * r;
            v[u][r] = (base >= 0 && bi >= 0 && bi < d.n_in) ? src[r * step] : make_float2(0.f, 0.f);
          }
        }
      } else {
        const long long ri = base >= 0 ? L.im_in[l] : -1;
        const int p0 = j * d.pos_mul + (base >= 0 ? L.pos0[l] : 0) - d.in_off, ps = M * d.pos_mul;
        const long long off0 = (long long)p0 * d.ri_tst, step = (long long)ps * d.ri_tst;
        const TI* s0 = reinterpret_cast<const TI*>(d.rin) + base + off0;
        const TI* s1 = reinterpret_cast<const TI*>(d.rin) + ri + off0;
        if (ri < 0) {  // no second item packed into the imaginary part
#pragma unroll
          for (int r = 0; r < R1; ++r) {
            const int pos = p0 + ps * r;
            v[u][r] = make_float2((base >= 0 && pos >= 0 && pos < d.n_in) ? DT<TI>::load(s0 + r * step) : 0.f, 0.f);
          }
        } else {
#pragma unroll
          for (int r = 0; r < R1; ++r) {
            const int pos = p0 + ps * r;
            const bool ok = pos >= 0 && pos < d.n_in;
            v[u][r] = make_float2(ok ? DT<TI>::load(s0 + r * step) : 0.f, ok ? DT<TI>::load(s1 + r * step) : 0.f);
          }
        }
      }
    }
    // (while the loads are in flight) the store twiddle table, read after two barriers
    if (t4) long_fill_store_twiddles<R1, R2, R3, MID != 0>(T4, L.twm[0], d.tw_logF, d.scale, SD);
#pragma unroll
    for (int u = 0; u < IT1; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, j = it / NL;
      if (N1 % T != 0 && it >= N1) continue;
      dftR<R1>(v[u], D1);
      float2* o = sm + X::b1(l, j);
      const float2* t1 = T1 + j;
      o[0] = v[u][0];
#pragma unroll
      for (int k1 = 1; k1 < R1; ++k1) o[k1 * X::C1] = cmul(v[u][k1], conj_if(t1[k1 * M], D1));
    }
  }
  __syncthreads();

  // filter spectrum of the product pass, fetched for every level-3 item ahead of level 2
  float2 kreg[MID ? IT3 : 1][MID ? R3 : 1];
  if constexpr (MID) {
#pragma unroll
    for (int u = 0; u < IT3; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, k2 = (it / NL) % R2, k1 = it / (NL * R2);
      if (N3 % T != 0 && it >= N3) continue;
      const bool ok = L.cb_in[l] >= 0;
      const float2* kp = d.kin + (ok ? L.kbase[l] : 0) + (long long)(k1 + R1 * k2) * d.k_tst;
      const long long ks = (long long)S3 * d.k_tst;
#pragma unroll
      for (int k3 = 0; k3 < R3; ++k3) kreg[u][k3] = ok ? __ldg(kp + k3 * ks) : make_float2(0.f, 0.f);
    }
  }

  // D * skip of every level-3 item's points (inverse passes with the skip epilogue), likewise
  constexpr bool PRE = !MID && OM == OUT_REAL_SKIP;
  float pre[PRE ? IT3 : 1][PRE ? R3 : 1];
  if constexpr (PRE) {
#pragma unroll
    for (int u = 0; u < IT3; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, k2 = (it / NL) % R2, k1 = it / (NL * R2);
      if (N3 % T != 0 && it >= N3) continue;
      if (L.cb_in[l] >= 0) long_skip_run<R3, TO>(d, L, l, k1 + R1 * k2, S3, pre[u]);
    }
  }

  // level 2 (in place per item): R2-point transforms over s of A[k1 M + i + R3 s], twiddle
  // W_M^(i k2) -> B[k1 M + k2 R3 + i]
#pragma unroll
  for (int u = 0; u < IT2; ++u) {
    const int it = threadIdx.x + u * T, l = it % NL, i = (it / NL) % R3, k1 = it / (NL * R3);
    if (N2 % T != 0 && it >= N2) continue;
    float2* o = sm + X::b2(l, i, k1);
    const float2* t2 = T2 + i;
    float2 v[R2];
#pragma unroll
    for (int s = 0; s < R2; ++s) v[s] = o[s * X::C2];
    dftR<R2>(v, D1);
    o[0] = v[0];
#pragma unroll
    for (int k2 = 1; k2 < R2; ++k2) o[k2 * X::C2] = cmul(v[k2], conj_if(t2[k2 * R3], D1));
  }
  __syncthreads();

  // level 3: R3-point transforms over i -> X[k1 + R1 k2 + R1 R2 k3]
#pragma unroll
  for (int u = 0; u < IT3; ++u) {
    const int it = threadIdx.x + u * T, l = it % NL, k2 = (it / NL) % R2, k1 = it / (NL * R2);
    if (N3 % T != 0 && it >= N3) continue;
    float2* o = sm + X::b3(l, k1, k2);
    float2 v[R3];
#pragma unroll
    for (int i = 0; i < R3; ++i) v[i] = o[i * NL];
    dftR<R3>(v, D1);
    if constexpr (MID) {
#pragma unroll
      for (int k3 = 0; k3 < R3; ++k3) {
        float2 kv = kreg[u][k3];
        if (MID == 2) kv.y = -kv.y;
        v[k3] = cmul(v[k3], kv);
      }
      dftR<R3>(v, 1.f);  // inverse over k3 -> i, back into the same points
#pragma unroll
      for (int i = 0; i < R3; ++i) o[i * NL] = v[i];
    } else {
      const float2* tt = t4 ? t4 + k1 * R3 * R2 + k2 : nullptr;
      if constexpr (PRE) {
        if (L.cb_in[l] >= 0) long_store_run<R3, R2, OM, TO>(d, L, l, k1 + R1 * k2, S3, SD, full_out, v, pre[u], tt);
      } else {
        const float none[R3] = {};
        if (L.cb_in[l] >= 0) long_store_run<R3, R2, OM, TO>(d, L, l, k1 + R1 * k2, S3, SD, full_out, v, none, tt);
      }
    }
  }
  if constexpr (MID) {
    __syncthreads();
    // inverse level 2 (in place per item): conj twiddle, R2-point inverse over k2 -> s
#pragma unroll
    for (int u = 0; u < IT2; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, i = (it / NL) % R3, k1 = it / (NL * R3);
      if (N2 % T != 0 && it >= N2) continue;
      float2* o = sm + X::b2(l, i, k1);
      const float2* t2 = T2 + i;
      float2 v[R2];
      v[0] = o[0];
#pragma unroll
      for (int k2 = 1; k2 < R2; ++k2) v[k2] = cmul(o[k2 * X::C2], conj_if(t2[k2 * R3], 1.f));
      dftR<R2>(v, 1.f);
#pragma unroll
      for (int s = 0; s < R2; ++s) o[s * X::C2] = v[s];
    }
    __syncthreads();
    // inverse level 1: conj twiddle, R1-point inverse over k1 -> x[j + M r], stored
#pragma unroll
    for (int u = 0; u < IT1; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, j = it / NL;
      if (N1 % T != 0 && it >= N1) continue;
      const float2* o = sm + X::b1(l, j);
      const float2* t1 = T1 + j;
      float2 v[R1];
      v[0] = o[0];
#pragma unroll
      for (int k1 = 1; k1 < R1; ++k1) v[k1] = cmul(o[k1 * X::C1], conj_if(t1[k1 * M], 1.f));
      dftR<R1>(v, 1.f);
      const float none[R1] = {};
      if (L.cb_in[l] >= 0) long_store_run<R1, M, OM, TO>(d, L, l, j, M, SD, full_out, v, none, t4 ? t4 + j : nullptr);
    }
  }
}

// Backward product pass of the long 1D transform, on the lines (k_a, c) of the second
// four-step axis: it finishes the forward transforms of x (sx) and dy (sdy) from their
// partial spectra (after the first axis), forms
//   dX = dY conj(K)   and   dK = sum_p conj(X_p) dY_p   (per item p with per-sample filters),
// and runs the adjoint levels of both with the inverse pass's post-twiddle: dX back into
// sdy (in place), dK into dkh. It replaces two forward passes, the elementwise spectral
// backward and two inverse passes (five sweeps over the spectra) by one. dK is accumulated
// over the pairs after its inverse (the transform is linear), so that no spectrum stays in
// registers from one pair to the next.
template <int R1, int R2, int R3>
__global__ void __launch_bounds__(kLongThreads, kLongMinBlocks) fft_long_bwd_kernel(const LongBwdDesc d) {
  constexpr int F = R1 * R2 * R3, M = R2 * R3, S3 = R1 * R2;
  constexpr int NL = long_bwd_lines<F>();
  constexpr int T = kLongThreads;
  constexpr int N1 = NL * M, N2 = NL * R1 * R3, N3 = NL * R1 * R2;  // items per level
  constexpr int IT1 = (N1 + T - 1) / T, IT2 = (N2 + T - 1) / T, IT3 = (N3 + T - 1) / T;
  using X = LongIdx<R1, R2, R3, NL>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float2* smx = reinterpret_cast<float2*>(smem_raw);  // [(F + F / R3)][NL], x then dK
  float2* smy = smx + (size_t)(F + F / R3) * NL;       // dy then dX
  float2* tw = smy + (size_t)(F + F / R3) * NL;        // T1 then T2
  const float2* T1 = tw;
  const float2* T2 = tw + F;
  float2* T4 = tw + long_twn<R1, R2, R3>();  // [F] store twiddles (uniform multiplier)
  long long* sb = reinterpret_cast<long long*>(T4 + F);  // [NL] spectrum base (-1: past the end)
  long long* kb = sb + NL;                                                    // [NL] filter base
  int* twm = reinterpret_cast<int*>(kb + NL);                                 // [NL] k_a
  const long long line0 = (long long)blockIdx.x * NL;
  long_fill_twiddles<R1, R2, R3>(tw);
  for (int l = threadIdx.x; l < NL; l += T) {
    const long long lid = line0 + l;
    if (lid >= d.nlines) {
      sb[l] = -1;
      continue;
    }
    const int c = (int)(lid % d.C);
    const long long rest = lid / d.C;
    const int ka = (int)(rest % d.Fa);
    const long long po = (rest / d.Fa) * d.pl;
    sb[l] = po * d.pst + (long long)ka * d.ost + c;
    kb[l] = po * d.k_pst + (long long)ka * d.ost + c;
    twm[l] = ka;
  }
  __syncthreads();
  const float2* t4 = d.C % NL == 0 ? T4 : nullptr;
  if (t4) long_fill_store_twiddles<R1, R2, R3, true>(T4, twm[0], d.tw_logF, d.scale, 1.f);

  // forward level 1 of one line set (g: partial spectrum, pair offset qoff) into sm
  auto forward1 = [&](const float2* g, float2* sm, long long qoff) {
    float2 v[IT1][R1];
#pragma unroll
    for (int u = 0; u < IT1; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, j = it / NL;
      const bool ok = it < N1 && sb[l] >= 0;
      const float2* src = g + (ok ? sb[l] + qoff : 0) + (long long)j * d.tst;
      const long long step = (long long)M * d.tst;
#pragma unroll
      for (int r = 0; r < R1; ++r) v[u][r] = ok ? src[r * step] : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < IT1; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, j = it / NL;
      if (it >= N1) continue;
      dftR<R1>(v[u], -1.f);
      float2* o = sm + X::b1(l, j);
      const float2* t1 = T1 + j;
      o[0] = v[u][0];
#pragma unroll
      for (int k1 = 1; k1 < R1; ++k1) o[k1 * X::C1] = cmul(v[u][k1], t1[k1 * M]);
    }
  };
  auto level2 = [&](float2* sm, float dir) {  // forward (dir -1) or adjoint (+1) level 2, in place per item
#pragma unroll
    for (int u = 0; u < IT2; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, i = (it / NL) % R3, k1 = it / (NL * R3);
      if (it >= N2) continue;
      float2* o = sm + X::b2(l, i, k1);
      const float2* t2 = T2 + i;
      float2 v[R2];
      if (dir < 0.f) {
#pragma unroll
        for (int s = 0; s < R2; ++s) v[s] = o[s * X::C2];
        dftR<R2>(v, -1.f);
        o[0] = v[0];
#pragma unroll
        for (int k2 = 1; k2 < R2; ++k2) o[k2 * X::C2] = cmul(v[k2], t2[k2 * R3]);
      } else {
        v[0] = o[0];
#pragma unroll
        for (int k2 = 1; k2 < R2; ++k2) v[k2] = cmulc(o[k2 * X::C2], t2[k2 * R3]);
        dftR<R2>(v, 1.f);
#pragma unroll
        for (int s = 0; s < R2; ++s) o[s * X::C2] = v[s];
      }
    }
  };
  // adjoint level 1 and the store with the inverse pass's twiddle and scale (add: accumulate
  // into what the previous pairs stored)
  auto inverse1_store = [&](const float2* sm, float2* g, const long long* gb, long long qoff, bool add) {
#pragma unroll
    for (int u = 0; u < IT1; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, j = it / NL;
      if (it >= N1) continue;
      const float2* o = sm + X::b1(l, j);
      const float2* t1 = T1 + j;
      float2 v[R1];
      v[0] = o[0];
#pragma unroll
      for (int k1 = 1; k1 < R1; ++k1) v[k1] = cmulc(o[k1 * X::C1], t1[k1 * M]);
      dftR<R1>(v, 1.f);
      if (sb[l] < 0) continue;
      float2* gl = g + gb[l] + qoff + (long long)j * d.tst;
      const long long step = (long long)M * d.tst;
      TwRun tr;
      if (!t4) tr = tw_run(twm[l], j, M, d.tw_logF, d.scale, 1.f);
#pragma unroll
      for (int r = 0; r < R1; ++r) {
        float2 w;
        if (t4) {
          w = t4[r * M + j];
        } else {
          w = tr.w;
          tr.w = cmul(tr.w, tr.s);
        }
        float2 val = cmul(v[r], w);
        if (add) val = cadd(val, gl[r * step]);
        gl[r * step] = val;
      }
    }
  };

  for (int q = 0; q < d.pl; ++q) {
    const long long qoff = (long long)q * d.pst;
    forward1(d.sx, smx, qoff);
    forward1(d.sdy, smy, qoff);
    // the filter spectrum of the level-3 items, fetched ahead of level 2
    float2 kreg[IT3][R3];
#pragma unroll
    for (int u = 0; u < IT3; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, k2 = (it / NL) % R2, k1 = it / (NL * R2);
      const bool ok = it < N3 && sb[l] >= 0;
      const float2* kp = d.kh + (ok ? kb[l] + (long long)q * d.k_pst : 0) + (long long)(k1 + R1 * k2) * d.tst;
      const long long ks = (long long)S3 * d.tst;
#pragma unroll
      for (int k3 = 0; k3 < R3; ++k3) kreg[u][k3] = ok ? __ldg(kp + k3 * ks) : make_float2(0.f, 0.f);
    }
    __syncthreads();
    level2(smx, -1.f);
    level2(smy, -1.f);
    __syncthreads();
    // level 3 of both, the products, adjoint level 3 of dX (into smy) and dK (into smx)
#pragma unroll
    for (int u = 0; u < IT3; ++u) {
      const int it = threadIdx.x + u * T, l = it % NL, k2 = (it / NL) % R2, k1 = it / (NL * R2);
      if (it >= N3) continue;
      float2* ox = smx + X::b3(l, k1, k2);
      float2* oy = smy + X::b3(l, k1, k2);
      float2 vx[R3], vy[R3];
#pragma unroll
      for (int i = 0; i < R3; ++i) {
        vx[i] = ox[i * NL];
        vy[i] = oy[i * NL];
      }
      dftR<R3>(vx, -1.f);
      dftR<R3>(vy, -1.f);
#pragma unroll
      for (int k3 = 0; k3 < R3; ++k3) {
        vx[k3] = cmulc(vy[k3], vx[k3]);
        vy[k3] = cmulc(vy[k3], kreg[u][k3]);
      }
      dftR<R3>(vx, 1.f);
      dftR<R3>(vy, 1.f);
#pragma unroll
      for (int i = 0; i < R3; ++i) {
        ox[i * NL] = vx[i];
        oy[i * NL] = vy[i];
      }
    }
    __syncthreads();
    level2(smx, 1.f);
    level2(smy, 1.f);
    __syncthreads();
    inverse1_store(smy, d.sdy, sb, qoff, false);
    inverse1_store(smx, d.dkh, kb, (long long)q * d.k_pst, d.k_pst == 0 && q > 0);
    __syncthreads();  // smx / smy are refilled by the next pair
  }
}

namespace {

// Fill the twiddle tables of the current device once (double precision, rounded to float).
int ensure_long_tables() {
  static std::mutex mu;
  static unsigned long long ready = 0;  // bit per device
  static float2 hi[4096], lo[4096];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return HYFFT_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (ready >> dev & 1ull) return HYFFT_OK;
  if (!ready) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int e = 0; e < 4096; ++e) {
      const double a = two_pi * e / 4096.0, b = two_pi * e / 16777216.0;
      hi[e] = make_float2((float)std::cos(a), (float)-std::sin(a));
      lo[e] = make_float2((float)std::cos(b), (float)-std::sin(b));
    }
  }
  if (cudaMemcpyToSymbol(g_long_tw_hi, hi, sizeof(hi)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_long_tw_lo, lo, sizeof(lo)) != cudaSuccess)
    return HYFFT_ERR_CUDA;
  ready |= 1ull << dev;
  return HYFFT_OK;
}

template <int R1, int R2, int R3, int MID, int DIR, int IM, int OM, typename TI, typename TO>
int launch_t(const PassDesc& d, cudaStream_t st) {
  constexpr int F = R1 * R2 * R3;
  const long long grid = (d.nlines + long_lines<F>() - 1) / long_lines<F>();
  if (grid <= 0) return HYFFT_OK;
  if (grid > 0x7fffffffLL) return HYFFT_ERR_UNSUPPORTED;
  const int rc = ensure_long_tables();
  if (rc != HYFFT_OK) return rc;
  constexpr size_t smem = long_smem_bytes<R1, R2, R3>();
  auto kern = fft_long_cl_kernel<R1, R2, R3, MID, DIR, IM, OM, TI, TO>;
  if (!kernel_smem_once((const void*)kern, smem, true)) return HYFFT_ERR_CUDA;
  kern<<<(unsigned)grid, kLongThreads, smem, st>>>(d);
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

template <int R1, int R2, int R3>
int launch_f(const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st) {
  using bf = __nv_bfloat16;
  if (im == IN_CPLX && om == OUT_CPLX) {
    if (d.mid == 1) return launch_t<R1, R2, R3, 1, -1, IN_CPLX, OUT_CPLX, float, float>(d, st);
    if (d.mid == 2) return launch_t<R1, R2, R3, 2, -1, IN_CPLX, OUT_CPLX, float, float>(d, st);
    if (d.dir < 0) return launch_t<R1, R2, R3, 0, -1, IN_CPLX, OUT_CPLX, float, float>(d, st);
    return launch_t<R1, R2, R3, 0, 1, IN_CPLX, OUT_CPLX, float, float>(d, st);
  }
  if (im == IN_REAL) {  // forward transform of a channels-last activation or filter
    if (tin == HYFFT_BF16) return launch_t<R1, R2, R3, 0, -1, IN_REAL, OUT_CPLX, bf, float>(d, st);
    return launch_t<R1, R2, R3, 0, -1, IN_REAL, OUT_CPLX, float, float>(d, st);
  }
  if (om == OUT_REAL) {  // inverse transform into a channels-last activation
    if (tout == HYFFT_BF16) return launch_t<R1, R2, R3, 0, 1, IN_CPLX, OUT_REAL, float, bf>(d, st);
    return launch_t<R1, R2, R3, 0, 1, IN_CPLX, OUT_REAL, float, float>(d, st);
  }
  if (tout == HYFFT_BF16) return launch_t<R1, R2, R3, 0, 1, IN_CPLX, OUT_REAL_SKIP, float, bf>(d, st);
  return launch_t<R1, R2, R3, 0, 1, IN_CPLX, OUT_REAL_SKIP, float, float>(d, st);
}

template <int R1, int R2, int R3>
int launch_bwd_t(const LongBwdDesc& d, cudaStream_t st) {
  constexpr int F = R1 * R2 * R3;
  const long long grid = (d.nlines + long_bwd_lines<F>() - 1) / long_bwd_lines<F>();
  if (grid <= 0) return HYFFT_OK;
  if (grid > 0x7fffffffLL) return HYFFT_ERR_UNSUPPORTED;
  const int rc = ensure_long_tables();
  if (rc != HYFFT_OK) return rc;
  constexpr size_t smem = long_smem_bytes<R1, R2, R3, 2>();
  if (!kernel_smem_once((const void*)fft_long_bwd_kernel<R1, R2, R3>, smem, true)) return HYFFT_ERR_CUDA;
  fft_long_bwd_kernel<R1, R2, R3><<<(unsigned)grid, kLongThreads, smem, st>>>(d);
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

}  // namespace

// Whether launch_long_pass takes this pass: F = 128 .. 4096, complex spectra with
// channel-innermost lines, real sides channels-last (unit channel stride) in float32 or
// bfloat16, product passes complex to complex over a full (not half) filter spectrum.
bool long_pass_applies(const PassDesc& d, int im, int om, int tin, int tout) {
  if (d.F < 128 || d.F > 4096 || getenv("HYFFT_DISABLE_LONG_PASS")) return false;
  if (im == IN_CPLX && om == OUT_CPLX) return !d.k_half;
  if (d.mid) return false;
  if (im == IN_REAL) return om == OUT_CPLX && d.dir < 0 && d.ri_cst == 1 && (tin == HYFFT_F32 || tin == HYFFT_BF16);
  return im == IN_CPLX && d.dir > 0 && d.ro_cst == 1 && (tout == HYFFT_F32 || tout == HYFFT_BF16);
}

int launch_long_pass(const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st) {
  switch (d.F) {
    case 128: return launch_f<8, 4, 4>(d, im, om, tin, tout, st);
    case 256: return launch_f<16, 4, 4>(d, im, om, tin, tout, st);
    case 512: return launch_f<16, 8, 4>(d, im, om, tin, tout, st);
    case 1024: return launch_f<16, 16, 4>(d, im, om, tin, tout, st);
    case 2048: return launch_f<16, 16, 8>(d, im, om, tin, tout, st);
    case 4096: return launch_f<16, 16, 16>(d, im, om, tin, tout, st);
    default: return HYFFT_ERR_UNSUPPORTED;
  }
}

// The backward product pass of a long 1D transform whose second axis has fb points
// (HYFFT_ERR_UNSUPPORTED for lengths without a long-pass form: nothing launched).
int launch_long_bwd(const LongBwdDesc& d, int fb, cudaStream_t st) {
  if (getenv("HYFFT_DISABLE_LONG_PASS") || getenv("HYFFT_DISABLE_BWD_PASS")) return HYFFT_ERR_UNSUPPORTED;
  switch (fb) {
    case 128: return launch_bwd_t<8, 4, 4>(d, st);
    case 256: return launch_bwd_t<16, 4, 4>(d, st);
    case 512: return launch_bwd_t<16, 8, 4>(d, st);
    case 1024: return launch_bwd_t<16, 16, 4>(d, st);
    case 2048: return launch_bwd_t<16, 16, 8>(d, st);
    default: return HYFFT_ERR_UNSUPPORTED;
  }
}

}  // namespace hyfft
