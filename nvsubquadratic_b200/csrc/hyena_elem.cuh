// Elementwise / stencil kernels of the general Hyena path: depthwise short conv,
// gate 1 (z = q' * g1(k')), gate 2 (y = h * g2(v')) and their backward.
// Activations are channels-last [B, *S, C] with a per-position element stride,
// so q, k, v may be strided views into one [B, *S, 3C] projection output.
//
// Work split: a CTA owns a group of 64 channels (two per lane: one 2-element vector)
// and a run of rows (b, position); each warp walks rows, so a warp-wide access is
// 32 consecutive channel pairs of one position (128 B for bf16). Row -> (b, p0, p1, p2)
// uses 32-bit division once per row. The stencil extents are template parameters for
// the shapes the reference uses (1D 3/4/7, 2D 3x3, 3D 3x3x3; K0 = 0 means no short
// conv, K0 = -1 the runtime-shaped fallback), so the tap loops unroll and the
// short-conv weights of the CTA's channels sit in shared memory as [tensor][tap][64].
#pragma once

#include "common.cuh"

namespace hyfft {

struct StencilGeom {
  int nd;
  int n[3];      // spatial extents (1 for unused axes)
  int k[3];      // short conv extents (1 for unused axes)
  int off[3];    // left padding per axis ("same": (k-1)/2, causal: k-1)
  int ntaps;     // k0*k1*k2
  int has_conv;  // 0: identity (no short conv)
  int has_bias;
};

constexpr int kElemCG = 64;       // channels per CTA (32 lanes x 2)
constexpr int kElemThreads = 256;  // 8 warps
constexpr int kMaxTaps = 27;

// 2-channel vectors of the activation dtype
template <typename T> struct V2;
template <> struct V2<float> {
  static __device__ __forceinline__ float2 load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void store(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
  static __device__ __forceinline__ float2 round(float2 v) { return v; }
};
template <> struct V2<__nv_bfloat16> {
  static __device__ __forceinline__ float2 load(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float2 v) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __float22bfloat162_rn(v);
  }
  static __device__ __forceinline__ float2 round(float2 v) { return __bfloat1622float2(__float22bfloat162_rn(v)); }
};
template <> struct V2<__half> {
  static __device__ __forceinline__ float2 load(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
  }
  static __device__ __forceinline__ void store(__half* p, float2 v) {
    *reinterpret_cast<__half2*>(p) = __float22half2_rn(v);
  }
  static __device__ __forceinline__ float2 round(float2 v) { return __half22float2(__float22half2_rn(v)); }
};

// Geometry of one thread's row.
struct RowPos {
  int b, p0, p1, p2;
  long long pos;  // flat position
};
__device__ __forceinline__ RowPos row_pos(long long r, const StencilGeom& g, long long Ntot) {
  RowPos o;
  if (r < (1LL << 31) && Ntot < (1LL << 31)) {  // 32-bit division: far cheaper than 64-bit
    const unsigned ur = (unsigned)r, un = (unsigned)Ntot;
    const unsigned b = ur / un;
    const unsigned p = ur - b * un;
    const unsigned n2 = (unsigned)g.n[2], n1 = (unsigned)g.n[1];
    const unsigned q2 = p / n2;
    const unsigned q1 = q2 / n1;
    o.b = (int)b;
    o.pos = p;
    o.p2 = (int)(p - q2 * n2);
    o.p1 = (int)(q2 - q1 * n1);
    o.p0 = (int)q1;
  } else {
    o.b = (int)(r / Ntot);
    o.pos = r - (long long)o.b * Ntot;
    o.p2 = (int)(o.pos % g.n[2]);
    const long long q2 = o.pos / g.n[2];
    o.p1 = (int)(q2 % g.n[1]);
    o.p0 = (int)(q2 / g.n[1]);
  }
  return o;
}

// (b, position) of row r without the stencil coordinates.
__device__ __forceinline__ void row_bp(long long r, long long Ntot, long long& b, long long& pos) {
  if (r < (1LL << 31) && Ntot < (1LL << 31)) {
    const unsigned ur = (unsigned)r, un = (unsigned)Ntot;
    const unsigned ub = ur / un;
    b = ub;
    pos = ur - ub * un;
  } else {
    b = r / Ntot;
    pos = r - b * Ntot;
  }
}

// Runtime or compile-time stencil extents.
template <int K> __device__ __forceinline__ int kext(int rt) { return K > 0 ? K : rt; }

// Visit every in-range tap of a stencil around (p0,p1,p2): f(tap_index, flat_neighbour).
// SIGN = +1: neighbour = p + tap - off (correlation, forward); -1: p - tap + off (transpose).
template <int K0, int K1, int K2, int SIGN, typename F>
__device__ __forceinline__ void for_taps(const StencilGeom& g, const RowPos& rp, F&& f) {
  if constexpr (K0 > 0 && K1 > 0 && K2 > 0) {
#pragma unroll
    for (int a = 0; a < K0; ++a) {
      const int i0 = rp.p0 + SIGN * (a - g.off[0]);
      if (i0 < 0 || i0 >= g.n[0]) continue;
#pragma unroll
      for (int bq = 0; bq < K1; ++bq) {
        const int i1 = rp.p1 + SIGN * (bq - g.off[1]);
        if (i1 < 0 || i1 >= g.n[1]) continue;
#pragma unroll
        for (int e = 0; e < K2; ++e) {
          const int i2 = rp.p2 + SIGN * (e - g.off[2]);
          if (i2 < 0 || i2 >= g.n[2]) continue;
          f((a * K1 + bq) * K2 + e, ((long long)i0 * g.n[1] + i1) * g.n[2] + i2);
        }
      }
    }
  } else {
    int tap = 0;
#pragma unroll 1
    for (int a = 0; a < g.k[0]; ++a) {
      const int i0 = rp.p0 + SIGN * (a - g.off[0]);
#pragma unroll 1
      for (int bq = 0; bq < g.k[1]; ++bq) {
        const int i1 = rp.p1 + SIGN * (bq - g.off[1]);
#pragma unroll 1
        for (int e = 0; e < g.k[2]; ++e, ++tap) {
          const int i2 = rp.p2 + SIGN * (e - g.off[2]);
          if (i0 < 0 || i0 >= g.n[0] || i1 < 0 || i1 >= g.n[1] || i2 < 0 || i2 >= g.n[2]) continue;
          f(tap, ((long long)i0 * g.n[1] + i1) * g.n[2] + i2);
        }
      }
    }
  }
}

// Two consecutive channels: one vector access when PAIR (even channel count, even
// strides, aligned bases), else two scalar accesses with the second guarded by `two`.
template <typename T, bool PAIR>
__device__ __forceinline__ float2 ld2(const T* p, bool two) {
  if constexpr (PAIR) return V2<T>::load(p);
  else return make_float2(DT<T>::load(p), two ? DT<T>::load(p + 1) : 0.f);
}
template <typename T, bool PAIR>
__device__ __forceinline__ void st2(T* p, float2 v, bool two) {
  if constexpr (PAIR) {
    V2<T>::store(p, v);
  } else {
    DT<T>::store(p, v.x);
    if (two) DT<T>::store(p + 1, v.y);
  }
}
template <bool PAIR>
__device__ __forceinline__ float2 ld2f(const float* p, bool two) {
  if constexpr (PAIR) return *reinterpret_cast<const float2*>(p);
  else return make_float2(p[0], two ? p[1] : 0.f);
}
template <bool PAIR>
__device__ __forceinline__ void st2f(float* p, float2 v, bool two) {
  if constexpr (PAIR) {
    *reinterpret_cast<float2*>(p) = v;
  } else {
    p[0] = v.x;
    if (two) p[1] = v.y;
  }
}

// Stage the short-conv weights (and biases) of channels [c0, c0 + 64) of q, k and v:
// sw[(t * ntaps + tap) * 64 + j] = w[(t * C + c0 + j) * ntaps + tap].
__device__ __forceinline__ void stage_weights(float* sw, float* sb, const float* __restrict__ w,
                                              const float* __restrict__ bias, int C, int c0, int ntaps,
                                              bool has_bias) {
  for (int i = threadIdx.x; i < 3 * ntaps * kElemCG; i += blockDim.x) {
    const int j = i % kElemCG;
    const int tt = i / kElemCG;  // t * ntaps + tap
    const int t = tt / ntaps, tap = tt - t * ntaps;
    const int c = c0 + j;
    sw[i] = (w && c < C) ? w[((long long)t * C + c) * ntaps + tap] : 0.f;
  }
  for (int i = threadIdx.x; i < 3 * kElemCG; i += blockDim.x) {
    const int t = i / kElemCG, c = c0 + (i % kElemCG);
    sb[i] = (has_bias && bias && c < C) ? bias[(long long)t * C + c] : 0.f;
  }
}

// Forward prologue: q', k', v' (saved, dtype-rounded) and z = q' * g1(k').
// grid: (ceil(C / 64), row blocks); warp w of CTA y walks rows y * 8 + w + j * (gridDim.y * 8).
template <typename T, bool PAIR, int K0, int K1, int K2>
__global__ void __launch_bounds__(kElemThreads) hyena_pre_fwd_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, long long in_bst, long long in_pst,
    StencilGeom g, int B, int C, const float* __restrict__ w, const float* __restrict__ bias, int gate1,
    T* __restrict__ qs, T* __restrict__ ks, T* __restrict__ vs, T* __restrict__ z) {
  __shared__ float sw[3 * kMaxTaps * kElemCG];
  __shared__ float sb[3 * kElemCG];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * kElemCG;
  const int c = c0 + 2 * lane;
  const bool two = c + 1 < C;
  if constexpr (K0 != 0) {
    stage_weights(sw, sb, w, bias, C, c0, g.ntaps, g.has_bias);
    __syncthreads();
  }
  if (c >= C) return;
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long rows = (long long)B * Ntot;
  const long long rstride = (long long)gridDim.y * (kElemThreads / 32);
  for (long long r = (long long)blockIdx.y * (kElemThreads / 32) + warp; r < rows; r += rstride) {
    const RowPos rp = row_pos(r, g, Ntot);
    const long long bb = (long long)rp.b * in_bst + c;
    float2 a[3];
    if constexpr (K0 == 0) {
      const long long o = bb + rp.pos * in_pst;
      a[0] = ld2<T, PAIR>(q + o, two);
      a[1] = ld2<T, PAIR>(k + o, two);
      a[2] = ld2<T, PAIR>(v + o, two);
    } else {
#pragma unroll
      for (int t = 0; t < 3; ++t) a[t] = make_float2(sb[t * kElemCG + 2 * lane], sb[t * kElemCG + 2 * lane + 1]);
      for_taps<K0, K1, K2, 1>(g, rp, [&](int tap, long long pl) {
        const long long o = bb + pl * in_pst;
        const float2 xq = ld2<T, PAIR>(q + o, two), xk = ld2<T, PAIR>(k + o, two), xv = ld2<T, PAIR>(v + o, two);
        const float2 wq = *reinterpret_cast<const float2*>(&sw[(0 * g.ntaps + tap) * kElemCG + 2 * lane]);
        const float2 wk = *reinterpret_cast<const float2*>(&sw[(1 * g.ntaps + tap) * kElemCG + 2 * lane]);
        const float2 wv = *reinterpret_cast<const float2*>(&sw[(2 * g.ntaps + tap) * kElemCG + 2 * lane]);
        a[0].x = fmaf(wq.x, xq.x, a[0].x); a[0].y = fmaf(wq.y, xq.y, a[0].y);
        a[1].x = fmaf(wk.x, xk.x, a[1].x); a[1].y = fmaf(wk.y, xk.y, a[1].y);
        a[2].x = fmaf(wv.x, xv.x, a[2].x); a[2].y = fmaf(wv.y, xv.y, a[2].y);
      });
    }
    const float2 qv = V2<T>::round(a[0]), kv = V2<T>::round(a[1]), vv = V2<T>::round(a[2]);
    const float2 g1 = V2<T>::round(make_float2(gate_f(gate1, kv.x), gate_f(gate1, kv.y)));
    const long long i = r * C + c;
    st2<T, PAIR>(qs + i, qv, two);
    st2<T, PAIR>(ks + i, kv, two);
    st2<T, PAIR>(vs + i, vv, two);
    st2<T, PAIR>(z + i, make_float2(qv.x * g1.x, qv.y * g1.y), two);
  }
}

// Forward epilogue: y = h * g2(v')   (h, v' contiguous [B, N, C]; y strided)
template <typename T, bool PAIR>
__global__ void __launch_bounds__(kElemThreads) hyena_post_fwd_kernel(
    const T* __restrict__ h, const T* __restrict__ vs, int gate2, long long Ntot, int B, int C, T* __restrict__ y,
    long long out_bst, long long out_pst) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * kElemCG + 2 * lane;
  const bool two = c + 1 < C;
  if (c >= C) return;
  const long long rows = (long long)B * Ntot;
  const long long rstride = (long long)gridDim.y * (kElemThreads / 32);
  for (long long r = (long long)blockIdx.y * (kElemThreads / 32) + warp; r < rows; r += rstride) {
    long long b, pos;
    row_bp(r, Ntot, b, pos);
    const long long i = r * C + c;
    const float2 hv = ld2<T, PAIR>(h + i, two), vv = ld2<T, PAIR>(vs + i, two);
    const float2 g2 = V2<T>::round(make_float2(gate_f(gate2, vv.x), gate_f(gate2, vv.y)));
    st2<T, PAIR>(y + b * out_bst + pos * out_pst + c, make_float2(hv.x * g2.x, hv.y * g2.y), two);
  }
}

// Backward through gate 2: dh = dy * g2(v'), dv' = dy * h * g2'(v') (activation dtype, as
// autograd produces them).
template <typename T, bool PAIR>
__global__ void __launch_bounds__(kElemThreads) hyena_bwd_gate2_kernel(
    const T* __restrict__ dy, long long out_bst, long long out_pst, const T* __restrict__ h,
    const T* __restrict__ vs, int gate2, long long Ntot, int B, int C, T* __restrict__ dh, T* __restrict__ dvp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * kElemCG + 2 * lane;
  const bool two = c + 1 < C;
  if (c >= C) return;
  const long long rows = (long long)B * Ntot;
  const long long rstride = (long long)gridDim.y * (kElemThreads / 32);
  for (long long r = (long long)blockIdx.y * (kElemThreads / 32) + warp; r < rows; r += rstride) {
    long long b, pos;
    row_bp(r, Ntot, b, pos);
    const long long i = r * C + c;
    const float2 gd = ld2<T, PAIR>(dy + b * out_bst + pos * out_pst + c, two);
    const float2 vv = ld2<T, PAIR>(vs + i, two), hv = ld2<T, PAIR>(h + i, two);
    const float2 g2 = V2<T>::round(make_float2(gate_f(gate2, vv.x), gate_f(gate2, vv.y)));
    st2<T, PAIR>(dh + i, make_float2(gd.x * g2.x, gd.y * g2.y), two);
    st2<T, PAIR>(dvp + i, make_float2(gd.x * hv.x * gate_df(gate2, vv.x), gd.y * hv.y * gate_df(gate2, vv.y)), two);
  }
}

// Backward through gate 1: dq' = dz * g1(k'), dk' = dz * q' * g1'(k') (activation dtype);
// all contiguous [B, N, C], same (row, channel-pair) split as the other kernels.
template <typename T, bool PAIR>
__global__ void __launch_bounds__(kElemThreads) hyena_bwd_gate1_kernel(
    const T* __restrict__ dz, const T* __restrict__ qs, const T* __restrict__ ks, int gate1, long long rows, int C,
    T* __restrict__ dqp, T* __restrict__ dkp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * kElemCG + 2 * lane;
  const bool two = c + 1 < C;
  if (c >= C) return;
  const long long rstride = (long long)gridDim.y * (kElemThreads / 32);
  for (long long r = (long long)blockIdx.y * (kElemThreads / 32) + warp; r < rows; r += rstride) {
    const long long i = r * C + c;
    const float2 gd = ld2<T, PAIR>(dz + i, two), kv = ld2<T, PAIR>(ks + i, two), qv = ld2<T, PAIR>(qs + i, two);
    const float2 g1 = V2<T>::round(make_float2(gate_f(gate1, kv.x), gate_f(gate1, kv.y)));
    st2<T, PAIR>(dqp + i, make_float2(gd.x * g1.x, gd.y * g1.y), two);
    st2<T, PAIR>(dkp + i, make_float2(gd.x * qv.x * gate_df(gate1, kv.x), gd.y * qv.y * gate_df(gate1, kv.y)), two);
  }
}

// Backward of the depthwise short conv w.r.t. its input (transposed stencil):
//   din[pos] = sum_tap w[ch, tap] * dout[pos - tap + off]
// dout: contiguous [B, N, C] for each of q/k/v (three pointers); din strided.
template <typename T, bool PAIR, int K0, int K1, int K2>
__global__ void __launch_bounds__(kElemThreads) hyena_short_dgrad_kernel(
    const T* __restrict__ dqp, const T* __restrict__ dkp, const T* __restrict__ dvp, StencilGeom g, int B,
    int C, const float* __restrict__ w, T* __restrict__ dq, T* __restrict__ dk, T* __restrict__ dv, long long out_bst,
    long long out_pst) {
  __shared__ float sw[3 * kMaxTaps * kElemCG];
  __shared__ float sb[3 * kElemCG];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * kElemCG;
  const int c = c0 + 2 * lane;
  const bool two = c + 1 < C;
  if constexpr (K0 != 0) {
    stage_weights(sw, sb, w, nullptr, C, c0, g.ntaps, false);
    __syncthreads();
  }
  if (c >= C) return;
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long rows = (long long)B * Ntot;
  const long long rstride = (long long)gridDim.y * (kElemThreads / 32);
  for (long long r = (long long)blockIdx.y * (kElemThreads / 32) + warp; r < rows; r += rstride) {
    const RowPos rp = row_pos(r, g, Ntot);
    const long long o = (long long)rp.b * out_bst + rp.pos * out_pst + c;
    float2 a[3] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    if constexpr (K0 == 0) {
      const long long i = r * C + c;
      a[0] = ld2<T, PAIR>(dqp + i, two);
      a[1] = ld2<T, PAIR>(dkp + i, two);
      a[2] = ld2<T, PAIR>(dvp + i, two);
    } else {
      const long long bb = (long long)rp.b * Ntot * C + c;
      for_taps<K0, K1, K2, -1>(g, rp, [&](int tap, long long pl) {
        const long long j = bb + pl * C;
        const float2 xq = ld2<T, PAIR>(dqp + j, two), xk = ld2<T, PAIR>(dkp + j, two), xv = ld2<T, PAIR>(dvp + j, two);
        const float2 wq = *reinterpret_cast<const float2*>(&sw[(0 * g.ntaps + tap) * kElemCG + 2 * lane]);
        const float2 wk = *reinterpret_cast<const float2*>(&sw[(1 * g.ntaps + tap) * kElemCG + 2 * lane]);
        const float2 wv = *reinterpret_cast<const float2*>(&sw[(2 * g.ntaps + tap) * kElemCG + 2 * lane]);
        a[0].x = fmaf(wq.x, xq.x, a[0].x); a[0].y = fmaf(wq.y, xq.y, a[0].y);
        a[1].x = fmaf(wk.x, xk.x, a[1].x); a[1].y = fmaf(wk.y, xk.y, a[1].y);
        a[2].x = fmaf(wv.x, xv.x, a[2].x); a[2].y = fmaf(wv.y, xv.y, a[2].y);
      });
    }
    st2<T, PAIR>(dq + o, a[0], two);
    st2<T, PAIR>(dk + o, a[1], two);
    st2<T, PAIR>(dv + o, a[2], two);
  }
}

// Weight / bias gradient of the short conv:
//   dw[ch, tap] = sum_{b,pos} dout[b,pos,c] * in[b, pos + tap - off, c],  db[ch] = sum dout
// grid: (ceil(C / 64), 3 tensors, row blocks). Each thread keeps its two channels' taps
// in registers over its rows (compile-time stencils), the CTA reduces its 8 warps in
// shared memory, and one atomic per (channel, tap) goes to dw / db (zeroed by the host).
// The runtime-shaped fallback accumulates straight into shared memory instead.
template <typename T, bool PAIR, int K0, int K1, int K2>
__global__ void __launch_bounds__(kElemThreads) hyena_short_wgrad_kernel(
    const T* __restrict__ dqp, const T* __restrict__ dkp, const T* __restrict__ dvp,
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, long long in_bst, long long in_pst,
    StencilGeom g, int B, int C, float* __restrict__ dw, float* __restrict__ db) {
  constexpr bool CT = K0 > 0 && K1 > 0 && K2 > 0;
  constexpr int NT = CT ? K0 * K1 * K2 : 1;
  constexpr int NW = kElemThreads / 32;
  __shared__ float red[NW][kElemCG + 1];
  __shared__ float sacc[CT ? 1 : (kMaxTaps + 1) * kElemCG];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.y;  // 0 q, 1 k, 2 v
  const int c = blockIdx.x * kElemCG + 2 * lane;
  const bool ok = c < C;
  const bool two = c + 1 < C;
  const T* dout = t == 0 ? dqp : (t == 1 ? dkp : dvp);
  const T* in = t == 0 ? q : (t == 1 ? k : v);
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long rows = (long long)B * Ntot;
  if constexpr (!CT) {
    for (int i = threadIdx.x; i < (kMaxTaps + 1) * kElemCG; i += blockDim.x) sacc[i] = 0.f;
    __syncthreads();
  }
  float2 acc[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i] = make_float2(0.f, 0.f);
  float2 bacc = make_float2(0.f, 0.f);
  if (ok) {
    // a contiguous run of rows per CTA, so stencil neighbours are mostly L1 hits
    const long long per = (rows + gridDim.z - 1) / gridDim.z;
    const long long r0 = (long long)blockIdx.z * per, r1 = min(rows, r0 + per);
#pragma unroll 4
    for (long long r = r0 + warp; r < r1; r += NW) {
      const RowPos rp = row_pos(r, g, Ntot);
      const float2 go = ld2<T, PAIR>(dout + r * C + c, two);
      bacc.x += go.x;
      bacc.y += go.y;
      const long long bb = (long long)rp.b * in_bst + c;
      for_taps<K0, K1, K2, 1>(g, rp, [&](int tap, long long pl) {
        const float2 xin = ld2<T, PAIR>(in + bb + pl * in_pst, two);
        if constexpr (CT) {
          acc[tap].x = fmaf(go.x, xin.x, acc[tap].x);
          acc[tap].y = fmaf(go.y, xin.y, acc[tap].y);
        } else {
          atomicAdd(&sacc[tap * kElemCG + 2 * lane], go.x * xin.x);
          atomicAdd(&sacc[tap * kElemCG + 2 * lane + 1], go.y * xin.y);
        }
      });
    }
  }
  const int ntaps = g.ntaps;
  for (int tap = 0; tap <= ntaps; ++tap) {
    float2 val = make_float2(0.f, 0.f);
    if (tap == ntaps) {
      val = bacc;
    } else if constexpr (CT) {
#pragma unroll
      for (int u = 0; u < NT; ++u)
        if (u == tap) val = acc[u];
    }
    red[warp][2 * lane] = val.x;
    red[warp][2 * lane + 1] = val.y;
    __syncthreads();
    if (threadIdx.x < kElemCG) {
      const int cc = blockIdx.x * kElemCG + threadIdx.x;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < NW; ++j) s += red[j][threadIdx.x];
      if constexpr (!CT) {
        if (tap < ntaps) s = sacc[tap * kElemCG + threadIdx.x];
      }
      if (cc < C) {
        const long long ch = (long long)t * C + cc;
        if (tap < ntaps) atomicAdd(dw + ch * ntaps + tap, s);
        else if (g.has_bias) atomicAdd(db + ch, s);
      }
    }
    __syncthreads();
  }
}

// Line geometry of the sliding-window stencil kernels: a "line" is one run of positions
// along the innermost spatial axis (axis ND-1) at fixed batch item and outer coordinates;
// KA x KB outer stencil rows (axes 0 and 1 of a 3D stencil, axis 0 of a 2D one, none in
// 1D) and KI taps along the line.
template <int ND>
__device__ __forceinline__ int line_len(const StencilGeom& g) { return g.n[ND - 1]; }
template <int ND>
__device__ __forceinline__ long long lines_per_item(const StencilGeom& g) {
  return ND == 3 ? (long long)g.n[0] * g.n[1] : (ND == 2 ? (long long)g.n[0] : 1LL);
}

// Short-conv weight / bias gradient, sliding-window form for the compile-time stencils:
// a warp walks SEG consecutive positions of one line for its 64 channels, keeping the
// KA*KB x KI input window in registers (one new column of KA*KB loads per position
// instead of all taps). grid (ceil(C/64), 3 tensors, item blocks). Same result layout
// and reduction as hyena_short_wgrad_kernel.
template <typename T, bool PAIR, int ND, int KA, int KB, int KI, bool SPLIT = false>
__global__ void __launch_bounds__(kElemThreads) hyena_short_wgrad_line_kernel(
    const T* __restrict__ dqp, const T* __restrict__ dkp, const T* __restrict__ dvp, const T* __restrict__ q,
    const T* __restrict__ k, const T* __restrict__ v, long long in_bst, long long in_pst, StencilGeom g, int B, int C,
    float* __restrict__ dw, float* __restrict__ db) {
  // SPLIT: this CTA covers only the outer stencil rows a = blockIdx.y / 3 (KB rows), so a
  // 3D stencil keeps 9 taps per thread in registers instead of 27 (grid.y = 3 * KA)
  constexpr int NA = (SPLIT ? 1 : KA) * KB, NT = NA * KI, NTG = KA * KB * KI, NW = kElemThreads / 32, SEG = 64;
  __shared__ float red[NW][kElemCG + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = SPLIT ? blockIdx.y % 3 : blockIdx.y;
  const int a0 = SPLIT ? blockIdx.y / 3 : 0;
  const int c = blockIdx.x * kElemCG + 2 * lane;
  const bool ok = c < C, two = c + 1 < C;
  const T* dout = t == 0 ? dqp : (t == 1 ? dkp : dvp);
  const T* in = t == 0 ? q : (t == 1 ? k : v);
  const int nl = line_len<ND>(g);
  const int offI = g.off[ND - 1];
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const int nseg = (nl + SEG - 1) / SEG;
  const long long lpi = lines_per_item<ND>(g);
  const long long items = (long long)B * lpi * nseg;
  float2 acc[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i] = make_float2(0.f, 0.f);
  float2 bacc = make_float2(0.f, 0.f);
  if (ok) {
    for (long long it = (long long)blockIdx.z * NW + warp; it < items; it += (long long)gridDim.z * NW) {
      const long long li = it / nseg;
      const int sg = (int)(it - li * nseg);
      const int b = (int)(li / lpi);
      const long long lo = li - (long long)b * lpi;  // outer line index
      int o0 = 0, o1 = 0;
      if (ND == 3) { o0 = (int)(lo / g.n[1]); o1 = (int)(lo - (long long)o0 * g.n[1]); }
      if (ND == 2) o0 = (int)lo;
      const int pa = sg * SEG, pb = min(nl, pa + SEG);
      long long rb[NA];
      bool rok[NA];
#pragma unroll
      for (int ai = 0; ai < (SPLIT ? 1 : KA); ++ai) {
        const int a = a0 + ai;
#pragma unroll
        for (int bq = 0; bq < KB; ++bq) {
          const int j = ai * KB + bq;
          long long rowpos;  // flat position of (outer neighbour, 0)
          bool okr = true;
          if (ND == 3) {
            const int i0 = o0 + a - g.off[0], i1 = o1 + bq - g.off[1];
            okr = i0 >= 0 && i0 < g.n[0] && i1 >= 0 && i1 < g.n[1];
            rowpos = ((long long)i0 * g.n[1] + i1) * g.n[2];
          } else if (ND == 2) {
            const int i0 = o0 + a - g.off[0];
            okr = i0 >= 0 && i0 < g.n[0];
            rowpos = (long long)i0 * g.n[1];
          } else {
            rowpos = 0;
          }
          rok[j] = okr;
          rb[j] = (long long)b * in_bst + c + rowpos * in_pst;
        }
      }
      const long long lb = (long long)b * Ntot + (ND == 3 ? ((long long)o0 * g.n[1] + o1) * g.n[2]
                                                          : (ND == 2 ? (long long)o0 * g.n[1] : 0LL));
      float2 w[NA][KI];
      auto ldin = [&](int j, int pi) -> float2 {
        if (!rok[j] || pi < 0 || pi >= nl) return make_float2(0.f, 0.f);
        return ld2<T, PAIR>(in + rb[j] + (long long)pi * in_pst, two);
      };
#pragma unroll
      for (int j = 0; j < NA; ++j) {
#pragma unroll
        for (int e = 1; e < KI; ++e) w[j][e] = ldin(j, pa - 1 + e - offI);
      }
      for (int p = pa; p < pb; ++p) {
#pragma unroll
        for (int j = 0; j < NA; ++j) {
#pragma unroll
          for (int e = 0; e + 1 < KI; ++e) w[j][e] = w[j][e + 1];
          w[j][KI - 1] = ldin(j, p + KI - 1 - offI);
        }
        const float2 go = ld2<T, PAIR>(dout + (lb + p) * C + c, two);
        bacc.x += go.x;
        bacc.y += go.y;
#pragma unroll
        for (int j = 0; j < NA; ++j) {
#pragma unroll
          for (int e = 0; e < KI; ++e) {
            acc[j * KI + e].x = fmaf(go.x, w[j][e].x, acc[j * KI + e].x);
            acc[j * KI + e].y = fmaf(go.y, w[j][e].y, acc[j * KI + e].y);
          }
        }
      }
    }
  }
  for (int tap = 0; tap <= NT; ++tap) {
    float2 val = bacc;
#pragma unroll
    for (int u = 0; u < NT; ++u)
      if (u == tap) val = acc[u];
    red[warp][2 * lane] = val.x;
    red[warp][2 * lane + 1] = val.y;
    __syncthreads();
    if (threadIdx.x < kElemCG) {
      const int cc = blockIdx.x * kElemCG + threadIdx.x;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < NW; ++j) sum += red[j][threadIdx.x];
      if (cc < C) {
        const long long ch = (long long)t * C + cc;
        if (tap < NT) atomicAdd(dw + ch * NTG + a0 * KB * KI + tap, sum);
        else if (g.has_bias && a0 == 0) atomicAdd(db + ch, sum);
      }
    }
    __syncthreads();
  }
}

// Short conv forward (MODE 0: q', k', v' and z = q' * g1(k')) and input gradient
// (MODE 1: the transposed stencil of dq', dk', dv'), sliding-window form for the
// compile-time stencils. A warp takes SEG positions of one line for its 64 channels and
// sweeps q, k, v one after the other with a KA*KB x KI register window of the input
// (one new column per position); the CTA's weights sit in shared memory.
// MODE 0: in = q/k/v (strided), out = qs/ks/vs (+ z) contiguous [B, N, C].
// MODE 1: in = dq'/dk'/dv' contiguous, out = dq/dk/dv strided.
// grid (ceil(C/64), item blocks).
template <typename T, bool PAIR, int ND, int KA, int KB, int KI, int MODE>
__global__ void __launch_bounds__(kElemThreads, (KA * KB * KI > 9) ? 2 : 3) hyena_line_stencil_kernel(
    const T* __restrict__ in0, const T* __restrict__ in1, const T* __restrict__ in2, long long in_bst,
    long long in_pst, T* __restrict__ out0, T* __restrict__ out1, T* __restrict__ out2, long long out_bst,
    long long out_pst, T* __restrict__ z, StencilGeom g, int B, int C, const float* __restrict__ w,
    const float* __restrict__ bias, int gate1) {
  constexpr int NA = KA * KB, NT = NA * KI, NW = kElemThreads / 32, SEG = 64;
  __shared__ float sw[3 * NT * kElemCG];
  __shared__ float sb[3 * kElemCG];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * kElemCG;
  const int c = c0 + 2 * lane;
  const bool two = c + 1 < C;
  stage_weights(sw, sb, w, bias, C, c0, NT, MODE == 0 && g.has_bias);
  __syncthreads();
  if (c >= C) return;
  const int nl = line_len<ND>(g);
  // forward: input position p + e - off; transposed: p - e + off = p + (KI-1-off) - (KI-1-e)
  const int offI = MODE == 0 ? g.off[ND - 1] : KI - 1 - g.off[ND - 1];
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const int nseg = (nl + SEG - 1) / SEG;
  const long long lpi = lines_per_item<ND>(g);
  const long long items = (long long)B * lpi * nseg;
  const T* ins[3] = {in0, in1, in2};
  T* outs[3] = {out0, out1, out2};
  for (long long it = (long long)blockIdx.y * NW + warp; it < items; it += (long long)gridDim.y * NW) {
    const long long li = it / nseg;
    const int sg = (int)(it - li * nseg);
    const int b = (int)(li / lpi);
    const long long lo = li - (long long)b * lpi;
    int o0 = 0, o1 = 0;
    if (ND == 3) { o0 = (int)(lo / g.n[1]); o1 = (int)(lo - (long long)o0 * g.n[1]); }
    if (ND == 2) o0 = (int)lo;
    const int pa = sg * SEG, pb = min(nl, pa + SEG);
    const long long lpos = ND == 3 ? ((long long)o0 * g.n[1] + o1) * g.n[2] : (ND == 2 ? (long long)o0 * g.n[1] : 0LL);
    // input row bases for the outer stencil rows (j = a * KB + bq), in the input's layout
    long long rb[NA];
    bool rok[NA];
#pragma unroll
    for (int a = 0; a < KA; ++a) {
#pragma unroll
      for (int bq = 0; bq < KB; ++bq) {
        const int j = a * KB + bq;
        const int da = MODE == 0 ? a - g.off[0] : g.off[0] - a;
        const int dbq = MODE == 0 ? bq - g.off[1] : g.off[1] - bq;
        long long rowpos = 0;
        bool okr = true;
        if (ND == 3) {
          const int i0 = o0 + da, i1 = o1 + dbq;
          okr = i0 >= 0 && i0 < g.n[0] && i1 >= 0 && i1 < g.n[1];
          rowpos = ((long long)i0 * g.n[1] + i1) * g.n[2];
        } else if (ND == 2) {
          const int i0 = o0 + da;
          okr = i0 >= 0 && i0 < g.n[0];
          rowpos = (long long)i0 * g.n[1];
        }
        rok[j] = okr;
        rb[j] = MODE == 0 ? (long long)b * in_bst + c + rowpos * in_pst : ((long long)b * Ntot + rowpos) * C + c;
      }
    }
    const long long ps = MODE == 0 ? in_pst : (long long)C;
#pragma unroll 1
    for (int t = 0; t < 3; ++t) {
      const T* in = ins[t];
      auto ldin = [&](int j, int pi) -> float2 {
        if (!rok[j] || pi < 0 || pi >= nl) return make_float2(0.f, 0.f);
        return ld2<T, PAIR>(in + rb[j] + (long long)pi * ps, two);
      };
      // weights of this tensor: tap (j, e) for the forward; (j, KI-1-u) for window slot u in
      // MODE 1. Up to 9 taps they stay in registers; larger (3D) stencils read them from
      // shared memory at each use, so the window and the weights do not both hold ~54
      // registers and the kernel keeps two CTAs per SM.
      constexpr bool WREG = NT <= 9;
      auto wsm = [&](int j, int u) -> float2 {
        const int e = MODE == 0 ? u : KI - 1 - u;
        return *reinterpret_cast<const float2*>(&sw[(t * NT + j * KI + e) * kElemCG + 2 * lane]);
      };
      float2 wr[WREG ? NT : 1];
      if constexpr (WREG) {
#pragma unroll
        for (int j = 0; j < NA; ++j) {
#pragma unroll
          for (int u = 0; u < KI; ++u) wr[j * KI + u] = wsm(j, u);
        }
      }
      const float2 bs = MODE == 0 ? make_float2(sb[t * kElemCG + 2 * lane], sb[t * kElemCG + 2 * lane + 1])
                                  : make_float2(0.f, 0.f);
      float2 win[NA][KI];
#pragma unroll
      for (int j = 0; j < NA; ++j) {
#pragma unroll
        for (int u = 1; u < KI; ++u) win[j][u] = ldin(j, pa - 1 + u - offI);
      }
      for (int p = pa; p < pb; ++p) {
        float2 acc = bs;
#pragma unroll
        for (int j = 0; j < NA; ++j) {
#pragma unroll
          for (int u = 0; u + 1 < KI; ++u) win[j][u] = win[j][u + 1];
          win[j][KI - 1] = ldin(j, p + KI - 1 - offI);
#pragma unroll
          for (int u = 0; u < KI; ++u) {
            float2 wv;
            if constexpr (WREG) wv = wr[j * KI + u];
            else wv = wsm(j, u);
            acc.x = fmaf(wv.x, win[j][u].x, acc.x);
            acc.y = fmaf(wv.y, win[j][u].y, acc.y);
          }
        }
        if constexpr (MODE == 0) {
          const long long o = ((long long)b * Ntot + lpos + p) * C + c;
          const float2 r = V2<T>::round(acc);
          st2<T, PAIR>(outs[t] + o, r, two);
          if (t == 1) {  // z = q' * g1(k'); q' was written by this warp in the previous sweep
            const float2 qv = ld2<T, PAIR>(outs[0] + o, two);
            const float2 g1 = V2<T>::round(make_float2(gate_f(gate1, r.x), gate_f(gate1, r.y)));
            st2<T, PAIR>(z + o, make_float2(qv.x * g1.x, qv.y * g1.y), two);
          }
        } else {
          st2<T, PAIR>(outs[t] + (long long)b * out_bst + (lpos + p) * out_pst + c, acc, two);
        }
      }
    }
  }
}

// dD[c] = sum_{b, pos} dh[b, pos, c] * z[b, pos, c] (contiguous [B, N, C]); grid
// (ceil(C / 64), row blocks), one atomic per channel per CTA (dD zeroed by the host).
template <typename T, bool PAIR>
__global__ void __launch_bounds__(kElemThreads) hyena_dskip_kernel(const T* __restrict__ dh, const T* __restrict__ z,
                                                                    long long rows, int C, float* __restrict__ dD) {
  constexpr int NW = kElemThreads / 32;
  __shared__ float red[NW][kElemCG + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * kElemCG + 2 * lane;
  const bool two = c + 1 < C;
  float2 acc = make_float2(0.f, 0.f);
  if (c < C) {
    for (long long r = (long long)blockIdx.y * NW + warp; r < rows; r += (long long)gridDim.y * NW) {
      const long long i = r * C + c;
      const float2 a = ld2<T, PAIR>(dh + i, two), b = ld2<T, PAIR>(z + i, two);
      acc.x = fmaf(a.x, b.x, acc.x);
      acc.y = fmaf(a.y, b.y, acc.y);
    }
  }
  red[warp][2 * lane] = acc.x;
  red[warp][2 * lane + 1] = acc.y;
  __syncthreads();
  if (threadIdx.x < kElemCG) {
    const int cc = blockIdx.x * kElemCG + threadIdx.x;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NW; ++j) s += red[j][threadIdx.x];
    if (cc < C) atomicAdd(dD + cc, s);
  }
}

// Layout change between channels-last [B][N][C] and channel-major [B][C][N] (both
// contiguous) through 32 x 32 shared-memory tiles, so both sides are read and written
// along their unit stride. TO_CM: channels-last -> channel-major. grid (ceil(N/32),
// ceil(C/32), B), 256 threads.
template <typename T, bool TO_CM>
__global__ void __launch_bounds__(256) cl_cm_transpose_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                              long long N, int C) {
  __shared__ T tile[32][33];
  const long long n0 = (long long)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  const long long base = (long long)blockIdx.z * N * C;
  const T* sp = src + base;
  T* dp = dst + base;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if constexpr (TO_CM) {
    for (int i = ty; i < 32; i += 8) {
      const long long n = n0 + i;
      const int c = c0 + tx;
      if (n < N && c < C) tile[i][tx] = sp[n * C + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int c = c0 + i;
      const long long n = n0 + tx;
      if (n < N && c < C) dp[(long long)c * N + n] = tile[tx][i];
    }
  } else {
    for (int i = ty; i < 32; i += 8) {
      const int c = c0 + i;
      const long long n = n0 + tx;
      if (n < N && c < C) tile[i][tx] = sp[(long long)c * N + n];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const long long n = n0 + i;
      const int c = c0 + tx;
      if (n < N && c < C) dp[n * C + c] = tile[tx][i];
    }
  }
}

// ---------------------------------------------------------------- transposes fused with the gates
// The large-grid kernels read and write channel-major [B][C][N] tensors; the gates around
// them are elementwise over channels-last [B][N][C] ones. These kernels do a gate and the
// layout change in one pass over a 64-position x 64-channel tile (256 threads, 16-byte
// chunks of 8 channels or 8 positions, the tile in shared memory with its 16-byte chunks
// XOR-swizzled by (row / 8) so both the row-wise and the column-wise accesses are free of
// bank conflicts), with the rounding of the separate kernels they replace:
//   GATE_POST_FWD:  in hc (cm) -> hb = hc (cl), y = h * round(g2(v'))           (hyena_post_fwd_kernel)
//   GATE_BWD2:      dy, hb, v' (cl) -> dv' = dy * h * g2'(v') (cl),
//                                      dh = dy * round(g2(v')) written cm      (hyena_bwd_gate2_kernel)
//   GATE_BWD1:      in dz (cm), q', k' (cl) -> dq' = dz * round(g1(k')),
//                                             dk' = dz * q' * g1'(k') (cl)      (hyena_bwd_gate1_kernel)
// All tensors contiguous; N and C multiples of 64; grid (N / 64, C / 64, B).
enum GateXMode { GATE_POST_FWD = 0, GATE_BWD2 = 1, GATE_BWD1 = 2 };

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = DT<T>::load(e + i);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) DT<T>::store(e + i, f[i]);
  return u;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(256) cl_cm_gate_kernel(const T* __restrict__ a, const T* __restrict__ b1,
                                                         const T* __restrict__ b2, T* __restrict__ o1,
                                                         T* __restrict__ o2, int gate, long long N, int C) {
  static_assert(sizeof(T) == 2, "16-bit activations");
  __shared__ __align__(16) T tile[64 * 64];  // [channel][position], 16-byte chunks swizzled
  const long long n0 = (long long)blockIdx.x * 64;
  const int c0 = blockIdx.y * 64;
  const long long base = (long long)blockIdx.z * N * C;
  const int t = threadIdx.x;
  // swizzled element offset of (channel row r, position p) in the tile
  auto at = [](int r, int p) { return r * 64 + ((((p >> 3) ^ (r >> 3)) & 7) << 3) + (p & 7); };
  if constexpr (MODE != GATE_BWD2) {
    // channel-major input rows: chunk (row r, positions 8k..8k+7)
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int q = t + 256 * it, r = q >> 3, k = q & 7;
      const uint4 u = *reinterpret_cast<const uint4*>(a + base + (long long)(c0 + r) * N + n0 + 8 * k);
      *reinterpret_cast<uint4*>(tile + at(r, 8 * k)) = u;
    }
    __syncthreads();
  }
  // channels-last chunks: (position p, channels 8g..8g+7); a warp covers 4 positions x 64 channels
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int q = t + 256 * it, p = q >> 3, g8 = q & 7;
    const long long off = base + (n0 + p) * C + c0 + 8 * g8;
    if constexpr (MODE == GATE_POST_FWD) {
      float h[8], v[8], y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = DT<T>::load(tile + at(8 * g8 + i, p));
      unpack8<T>(*reinterpret_cast<const uint4*>(b1 + off), v);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = h[i] * DT<T>::round(gate_f(gate, v[i]));
      *reinterpret_cast<uint4*>(o1 + off) = pack8<T>(h);  // hb: the same bits as hc
      *reinterpret_cast<uint4*>(o2 + off) = pack8<T>(y);
    } else if constexpr (MODE == GATE_BWD2) {
      float dy[8], h[8], v[8], dv[8], dh[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(a + off), dy);
      unpack8<T>(*reinterpret_cast<const uint4*>(b1 + off), h);
      unpack8<T>(*reinterpret_cast<const uint4*>(b2 + off), v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dh[i] = dy[i] * DT<T>::round(gate_f(gate, v[i]));
        dv[i] = dy[i] * h[i] * gate_df(gate, v[i]);
      }
      *reinterpret_cast<uint4*>(o1 + off) = pack8<T>(dv);
#pragma unroll
      for (int i = 0; i < 8; ++i) DT<T>::store(tile + at(8 * g8 + i, p), dh[i]);
    } else {
      float dz[8], kk[8], qq[8], dq[8], dk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) dz[i] = DT<T>::load(tile + at(8 * g8 + i, p));
      unpack8<T>(*reinterpret_cast<const uint4*>(b1 + off), qq);
      unpack8<T>(*reinterpret_cast<const uint4*>(b2 + off), kk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dq[i] = dz[i] * DT<T>::round(gate_f(gate, kk[i]));
        dk[i] = dz[i] * qq[i] * gate_df(gate, kk[i]);
      }
      *reinterpret_cast<uint4*>(o1 + off) = pack8<T>(dq);
      *reinterpret_cast<uint4*>(o2 + off) = pack8<T>(dk);
    }
  }
  if constexpr (MODE == GATE_BWD2) {
    __syncthreads();
    // dh channel-major rows
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int q = t + 256 * it, r = q >> 3, k = q & 7;
      *reinterpret_cast<uint4*>(o2 + base + (long long)(c0 + r) * N + n0 + 8 * k) =
          *reinterpret_cast<const uint4*>(tile + at(r, 8 * k));
    }
  }
}

}  // namespace hyfft
