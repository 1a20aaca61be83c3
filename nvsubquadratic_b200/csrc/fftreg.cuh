// Fully unrolled register FFTs (one thread per transform) for short axes of length
// 2^m or 3 * 2^m.
//
// fft_dif<N, NIN, SIGN>: natural-order input with v[NIN..N) known to be zero,
//   decimation in frequency; the output is in bit-reversed order.
// fft_dit<N, NOUT, SIGN>: bit-reversed input, decimation in time; only the
//   natural-order outputs v[0..NOUT) are computed.
//
// Which butterflies can be skipped or reduced (known-zero inputs of the zero
// padding, outputs outside the kept window) is decided at compile time from
// bit masks, so the padding and the crop of the linear convolution cost
// nothing. Twiddles W = exp(SIGN * 2*pi*i * j / n) are compile-time constants
// evaluated in double precision from their Taylor series (exact for the
// multiples of pi/2). A forward DIF followed by an inverse DIT needs no
// bit-reversal permutation: spectra simply stay in bit-reversed order.
#pragma once

#include <stdint.h>

namespace hyfft {
namespace reg {

constexpr double kPi = 3.141592653589793238462643383279502884;

__host__ __device__ constexpr double cx_sin(double x) {  // |x| <= pi
  double x2 = x * x, term = x, sum = x;
  for (int n = 1; n <= 16; ++n) {
    term *= -x2 / ((2.0 * n) * (2.0 * n + 1.0));
    sum += term;
  }
  return sum;
}
__host__ __device__ constexpr double cx_cos(double x) {  // |x| <= pi
  double x2 = x * x, term = 1.0, sum = 1.0;
  for (int n = 1; n <= 16; ++n) {
    term *= -x2 / ((2.0 * n - 1.0) * (2.0 * n));
    sum += term;
  }
  return sum;
}

template <int J, int NN, int SIGN>
struct Tw {
  static constexpr int jj = ((J % NN) + NN) % NN;
  static constexpr bool one = (jj == 0);
  static constexpr bool half = (2 * jj == NN);
  static constexpr bool quarter = (4 * jj == NN);
  static constexpr bool three = (4 * jj == 3 * NN);
  static constexpr double ang = SIGN * 2.0 * kPi * (double)(2 * jj > NN ? jj - NN : jj) / (double)NN;
  static constexpr float re = (float)cx_cos(ang);
  static constexpr float im = (float)cx_sin(ang);
};

template <int J, int NN, int SIGN>
__device__ __forceinline__ float2 twmul(float2 a) {
  using T = Tw<J, NN, SIGN>;
  if constexpr (T::one) {
    return a;
  } else if constexpr (T::half) {
    return make_float2(-a.x, -a.y);
  } else if constexpr (T::quarter) {  // * (SIGN * i)
    return SIGN > 0 ? make_float2(-a.y, a.x) : make_float2(a.y, -a.x);
  } else if constexpr (T::three) {  // * (-SIGN * i)
    return SIGN > 0 ? make_float2(a.y, -a.x) : make_float2(-a.y, a.x);
  } else {
    return make_float2(fmaf(a.x, T::re, -a.y * T::im), fmaf(a.x, T::im, a.y * T::re));
  }
}

__host__ __device__ constexpr uint64_t low_mask(int n) { return n >= 64 ? ~0ull : ((1ull << n) - 1ull); }

// ---------------------------------------------------------------- DIF (zero-input pruning)
// zero mask of the stage output given its input zero mask Z (butterfly span 2H)
__host__ __device__ constexpr uint64_t dif_zero_after(uint64_t Z, int N, int H) {
  uint64_t out = 0;
  for (int i = 0; i < N; ++i) {
    const int lo = (i % (2 * H) < H) ? i : i - H;
    const bool za = (Z >> lo) & 1ull, zc = (Z >> (lo + H)) & 1ull;
    if (za && zc) out |= 1ull << i;
  }
  return out;
}

template <int N, int H, int LO, uint64_t Z, int SIGN>
struct DifBfly {
  static __device__ __forceinline__ void run(float2* v) {
    if constexpr (LO < N) {
      if constexpr ((LO % (2 * H)) < H) {
        constexpr int j = LO % (2 * H);
        constexpr bool za = (Z >> LO) & 1ull;
        constexpr bool zc = (Z >> (LO + H)) & 1ull;
        if constexpr (za && zc) {
        } else if constexpr (zc) {
          v[LO + H] = twmul<j, 2 * H, SIGN>(v[LO]);
        } else if constexpr (za) {
          const float2 c = v[LO + H];
          v[LO] = c;
          v[LO + H] = twmul<j, 2 * H, SIGN>(make_float2(-c.x, -c.y));
        } else {
          const float2 a = v[LO], c = v[LO + H];
          v[LO] = make_float2(a.x + c.x, a.y + c.y);
          v[LO + H] = twmul<j, 2 * H, SIGN>(make_float2(a.x - c.x, a.y - c.y));
        }
      }
      DifBfly<N, H, LO + 1, Z, SIGN>::run(v);
    }
  }
};

template <int N, int H, uint64_t Z, int SIGN>
struct DifStage {
  static __device__ __forceinline__ void run(float2* v) {
    if constexpr (H >= 1) {
      DifBfly<N, H, 0, Z, SIGN>::run(v);
      DifStage<N, H / 2, dif_zero_after(Z, N, H), SIGN>::run(v);
    }
  }
};

__host__ __device__ constexpr bool is_pow2(int n) { return n >= 1 && (n & (n - 1)) == 0; }
__host__ __device__ constexpr int imin(int a, int b) { return a < b ? a : b; }

// 3-point DFT in place, X_k = sum_n x_n exp(SIGN 2 pi i n k / 3); ZB / ZC: b / c known zero.
template <int SIGN, bool ZB, bool ZC>
__device__ __forceinline__ void dft3(float2& a, float2& b, float2& c) {
  constexpr float h = 0.86602540378443864676f;  // sqrt(3) / 2
  if constexpr (ZB && ZC) {
    b = a;
    c = a;
  } else {
    const float2 s = ZC ? b : (ZB ? c : make_float2(b.x + c.x, b.y + c.y));        // b + c
    const float2 d = ZC ? b : (ZB ? make_float2(-c.x, -c.y) : make_float2(b.x - c.x, b.y - c.y));  // b - c
    const float2 m = make_float2(fmaf(-0.5f, s.x, a.x), fmaf(-0.5f, s.y, a.y));
    const float2 r = make_float2(-SIGN * h * d.y, SIGN * h * d.x);  // SIGN * (sqrt(3)/2) * i * (b - c)
    a = make_float2(a.x + s.x, a.y + s.y);
    b = make_float2(m.x + r.x, m.y + r.y);
    c = make_float2(m.x - r.x, m.y - r.y);
  }
}

// ---------------------------------------------------------------- N = 3 * M (M a power of two)
// With n = n1 + M n2 and k = 3 k1 + k2: forward = 3-point DFTs over n2, twiddles
// W_N^(n1 k2), then M-point DIFs over n1 on the contiguous segments v[M k2 .. M k2 + M).
// The spectrum is left as v[M k2 + j] = X[3 bitrev_M(j) + k2]; the inverse (DIT) below
// consumes exactly that order and returns natural order.
template <int M, int NIN, int SIGN, int N1>
struct Mix3Dif {
  static __device__ __forceinline__ void run(float2* v) {
    if constexpr (N1 < M && N1 < NIN) {  // columns n1 >= NIN are all zero and stay zero
      constexpr bool zb = N1 + M >= NIN, zc = N1 + 2 * M >= NIN;
      dft3<SIGN, zb, zc>(v[N1], v[N1 + M], v[N1 + 2 * M]);
      v[N1 + M] = twmul<N1, 3 * M, SIGN>(v[N1 + M]);
      v[N1 + 2 * M] = twmul<2 * N1, 3 * M, SIGN>(v[N1 + 2 * M]);
      Mix3Dif<M, NIN, SIGN, N1 + 1>::run(v);
    }
  }
};
template <int M, int NOUT, int SIGN, int N1>
struct Mix3Dit {
  static __device__ __forceinline__ void run(float2* v) {
    if constexpr (N1 < M && N1 < NOUT) {  // outputs n = n1 + M n2 >= n1: columns n1 >= NOUT are not needed
      v[N1 + M] = twmul<N1, 3 * M, SIGN>(v[N1 + M]);
      v[N1 + 2 * M] = twmul<2 * N1, 3 * M, SIGN>(v[N1 + 2 * M]);
      dft3<SIGN, false, false>(v[N1], v[N1 + M], v[N1 + 2 * M]);
      Mix3Dit<M, NOUT, SIGN, N1 + 1>::run(v);
    }
  }
};

template <int N, int NIN, int SIGN>
__device__ __forceinline__ void fft_dif(float2* v) {
  static_assert(NIN >= 1 && NIN <= N, "bad NIN");
  if constexpr (is_pow2(N)) {
    static_assert(N <= 64, "N must be <= 64");
    DifStage<N, N / 2, ~low_mask(NIN) & low_mask(N), SIGN>::run(v);
  } else {
    static_assert(N % 3 == 0 && is_pow2(N / 3) && N / 3 <= 32, "N must be 2^m or 3 * 2^m");
    constexpr int M = N / 3;
    Mix3Dif<M, NIN, SIGN, 0>::run(v);
    constexpr int NS = imin(NIN, M);  // segment inputs n1 >= NIN are zero
    DifStage<M, M / 2, ~low_mask(NS) & low_mask(M), SIGN>::run(v);
    DifStage<M, M / 2, ~low_mask(NS) & low_mask(M), SIGN>::run(v + M);
    DifStage<M, M / 2, ~low_mask(NS) & low_mask(M), SIGN>::run(v + 2 * M);
  }
}

// ---------------------------------------------------------------- DIT (output pruning)
// mask of stage-H inputs needed given the mask M of its needed outputs
__host__ __device__ constexpr uint64_t dit_need_before(uint64_t M, int N, int H) {
  uint64_t out = 0;
  for (int i = 0; i < N; ++i) {
    const int lo = (i % (2 * H) < H) ? i : i - H;
    if (((M >> lo) & 1ull) || ((M >> (lo + H)) & 1ull)) out |= 1ull << i;
  }
  return out;
}
// needed outputs of stage H when the final outputs needed are [0, NOUT)
__host__ __device__ constexpr uint64_t dit_need_after(int N, int NOUT, int H) {
  uint64_t M = low_mask(NOUT);
  for (int h = N / 2; h > H; h /= 2) M = dit_need_before(M, N, h);
  return M;
}

template <int N, int H, int LO, uint64_t M, int SIGN>
struct DitBfly {
  static __device__ __forceinline__ void run(float2* v) {
    if constexpr (LO < N) {
      if constexpr ((LO % (2 * H)) < H) {
        constexpr int j = LO % (2 * H);
        constexpr bool nt = (M >> LO) & 1ull;
        constexpr bool nb = (M >> (LO + H)) & 1ull;
        if constexpr (nt || nb) {
          const float2 a = v[LO];
          const float2 c = twmul<j, 2 * H, SIGN>(v[LO + H]);
          if constexpr (nt) v[LO] = make_float2(a.x + c.x, a.y + c.y);
          if constexpr (nb) v[LO + H] = make_float2(a.x - c.x, a.y - c.y);
        }
      }
      DitBfly<N, H, LO + 1, M, SIGN>::run(v);
    }
  }
};

template <int N, int NOUT, int H, int SIGN>
struct DitStage {
  static __device__ __forceinline__ void run(float2* v) {
    if constexpr (H < N) {
      DitBfly<N, H, 0, dit_need_after(N, NOUT, H), SIGN>::run(v);
      DitStage<N, NOUT, H * 2, SIGN>::run(v);
    }
  }
};

template <int N, int NOUT, int SIGN>
__device__ __forceinline__ void fft_dit(float2* v) {
  static_assert(NOUT >= 1 && NOUT <= N, "bad NOUT");
  if constexpr (is_pow2(N)) {
    static_assert(N <= 64, "N must be <= 64");
    DitStage<N, NOUT, 1, SIGN>::run(v);
  } else {
    static_assert(N % 3 == 0 && is_pow2(N / 3) && N / 3 <= 32, "N must be 2^m or 3 * 2^m");
    constexpr int M = N / 3;
    constexpr int NS = imin(NOUT, M);  // segment outputs n1 >= NOUT are not needed
    DitStage<M, NS, 1, SIGN>::run(v);
    DitStage<M, NS, 1, SIGN>::run(v + M);
    DitStage<M, NS, 1, SIGN>::run(v + 2 * M);
    Mix3Dit<M, NOUT, SIGN, 0>::run(v);
  }
}

__host__ __device__ constexpr int bitrev(int i, int n) {
  int r = 0;
  for (int b = 1; b < n; b <<= 1) {
    r = (r << 1) | (i & 1);
    i >>= 1;
  }
  return r;
}

}  // namespace reg
}  // namespace hyfft
