// Elementwise / stencil kernels of the general Hyena path: depthwise short conv,
// gate 1 (z = q' * g1(k')), gate 2 (y = h * g2(v')) and their backward.
// Activations are channels-last [B, *S, C] with a per-position element stride,
// so q, k, v may be strided views into one [B, *S, 3C] projection output.
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

__device__ __forceinline__ void unflatten3(long long pos, const StencilGeom& g, int& p0, int& p1, int& p2) {
  p2 = (int)(pos % g.n[2]);
  long long r = pos / g.n[2];
  p1 = (int)(r % g.n[1]);
  p0 = (int)(r / g.n[1]);
}

// Depthwise cross-correlation of channel `ch` (of 3C) at position (p0,p1,p2):
//   out = sum_tap w[ch, tap] * in[pos + tap - off] (+ bias[ch])
template <typename T>
__device__ __forceinline__ float short_conv_at(const T* __restrict__ in, long long bbase, long long pstride, int c,
                                               int ch, int p0, int p1, int p2, const StencilGeom& g,
                                               const float* __restrict__ w, const float* __restrict__ bias) {
  if (!g.has_conv) return DT<T>::load(in + bbase + ((long long)(p0 * g.n[1] + p1) * g.n[2] + p2) * pstride + c);
  float acc = g.has_bias ? bias[ch] : 0.f;
  const float* wc = w + (long long)ch * g.ntaps;
  int tap = 0;
  for (int a = 0; a < g.k[0]; ++a) {
    const int i0 = p0 + a - g.off[0];
    for (int b = 0; b < g.k[1]; ++b) {
      const int i1 = p1 + b - g.off[1];
      for (int e = 0; e < g.k[2]; ++e, ++tap) {
        const int i2 = p2 + e - g.off[2];
        if (i0 < 0 || i0 >= g.n[0] || i1 < 0 || i1 >= g.n[1] || i2 < 0 || i2 >= g.n[2]) continue;
        const long long pl = ((long long)i0 * g.n[1] + i1) * g.n[2] + i2;
        acc = fmaf(wc[tap], DT<T>::load(in + bbase + pl * pstride + c), acc);
      }
    }
  }
  return acc;
}

// Forward prologue: q', k', v' (saved, dtype-rounded) and z = q' * g1(k').
template <typename T>
__global__ void hyena_pre_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                     long long in_bst, long long in_pst, StencilGeom g, int B, int C,
                                     const float* __restrict__ w, const float* __restrict__ bias, int gate1,
                                     T* __restrict__ qs, T* __restrict__ ks, T* __restrict__ vs, T* __restrict__ z) {
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long total = (long long)B * Ntot * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long r = i / C;
    const long long pos = r % Ntot;
    const int b = (int)(r / Ntot);
    int p0, p1, p2;
    unflatten3(pos, g, p0, p1, p2);
    const long long bb = (long long)b * in_bst;
    const float qv = DT<T>::round(short_conv_at(q, bb, in_pst, c, c, p0, p1, p2, g, w, bias));
    const float kv = DT<T>::round(short_conv_at(k, bb, in_pst, c, C + c, p0, p1, p2, g, w, bias));
    const float vv = DT<T>::round(short_conv_at(v, bb, in_pst, c, 2 * C + c, p0, p1, p2, g, w, bias));
    const float zv = qv * DT<T>::round(gate_f(gate1, kv));
    DT<T>::store(qs + i, qv);
    DT<T>::store(ks + i, kv);
    DT<T>::store(vs + i, vv);
    DT<T>::store(z + i, zv);
  }
}

// Forward epilogue: y = h * g2(v')   (h, v' contiguous [B, N, C]; y strided)
template <typename T>
__global__ void hyena_post_fwd_kernel(const T* __restrict__ h, const T* __restrict__ vs, int gate2, long long Ntot,
                                      int B, int C, T* __restrict__ y, long long out_bst, long long out_pst) {
  const long long total = (long long)B * Ntot * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long r = i / C;
    const long long pos = r % Ntot;
    const long long b = r / Ntot;
    const float val = DT<T>::load(h + i) * DT<T>::round(gate_f(gate2, DT<T>::load(vs + i)));
    DT<T>::store(y + b * out_bst + pos * out_pst + c, val);
  }
}

// Backward through gate 2: dh = dy * g2(v') (dtype), dv' = dy * h * g2'(v') (fp32).
template <typename T>
__global__ void hyena_bwd_gate2_kernel(const T* __restrict__ dy, long long out_bst, long long out_pst,
                                       const T* __restrict__ h, const T* __restrict__ vs, int gate2, long long Ntot,
                                       int B, int C, T* __restrict__ dh, float* __restrict__ dvp) {
  const long long total = (long long)B * Ntot * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long r = i / C;
    const long long pos = r % Ntot;
    const long long b = r / Ntot;
    const float g = DT<T>::load(dy + b * out_bst + pos * out_pst + c);
    const float vv = DT<T>::load(vs + i);
    DT<T>::store(dh + i, g * DT<T>::round(gate_f(gate2, vv)));
    dvp[i] = g * DT<T>::load(h + i) * gate_df(gate2, vv);
  }
}

// Backward through gate 1: dq' = dz * g1(k'), dk' = dz * q' * g1'(k') (fp32).
template <typename T>
__global__ void hyena_bwd_gate1_kernel(const T* __restrict__ dz, const T* __restrict__ qs, const T* __restrict__ ks,
                                       int gate1, long long total, float* __restrict__ dqp, float* __restrict__ dkp) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const float g = DT<T>::load(dz + i);
    const float kv = DT<T>::load(ks + i);
    dqp[i] = g * DT<T>::round(gate_f(gate1, kv));
    dkp[i] = g * DT<T>::load(qs + i) * gate_df(gate1, kv);
  }
}

// Backward of the depthwise short conv w.r.t. its input (transposed stencil):
//   din[pos] = sum_tap w[ch, tap] * dout[pos - tap + off]
// dout: fp32 contiguous [B, N, C] for each of q/k/v (three pointers); din strided.
template <typename T>
__global__ void hyena_short_dgrad_kernel(const float* __restrict__ dqp, const float* __restrict__ dkp,
                                         const float* __restrict__ dvp, StencilGeom g, int B, int C,
                                         const float* __restrict__ w, T* __restrict__ dq, T* __restrict__ dk,
                                         T* __restrict__ dv, long long out_bst, long long out_pst) {
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long total = (long long)B * Ntot * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long r = i / C;
    const long long pos = r % Ntot;
    const int b = (int)(r / Ntot);
    const long long o = (long long)b * out_bst + pos * out_pst + c;
    if (!g.has_conv) {
      DT<T>::store(dq + o, dqp[i]);
      DT<T>::store(dk + o, dkp[i]);
      DT<T>::store(dv + o, dvp[i]);
      continue;
    }
    int p0, p1, p2;
    unflatten3(pos, g, p0, p1, p2);
    const long long bb = (long long)b * Ntot * C;
    float aq = 0.f, ak = 0.f, av = 0.f;
    const float* wq = w + (long long)c * g.ntaps;
    const float* wk = w + (long long)(C + c) * g.ntaps;
    const float* wv = w + (long long)(2 * C + c) * g.ntaps;
    int tap = 0;
    for (int a = 0; a < g.k[0]; ++a) {
      const int i0 = p0 - a + g.off[0];
      for (int bq = 0; bq < g.k[1]; ++bq) {
        const int i1 = p1 - bq + g.off[1];
        for (int e = 0; e < g.k[2]; ++e, ++tap) {
          const int i2 = p2 - e + g.off[2];
          if (i0 < 0 || i0 >= g.n[0] || i1 < 0 || i1 >= g.n[1] || i2 < 0 || i2 >= g.n[2]) continue;
          const long long j = bb + (((long long)i0 * g.n[1] + i1) * g.n[2] + i2) * C + c;
          aq = fmaf(wq[tap], dqp[j], aq);
          ak = fmaf(wk[tap], dkp[j], ak);
          av = fmaf(wv[tap], dvp[j], av);
        }
      }
    }
    DT<T>::store(dq + o, aq);
    DT<T>::store(dk + o, ak);
    DT<T>::store(dv + o, av);
  }
}

// Weight / bias gradient of the short conv:
//   dw[ch, tap] = sum_{b,pos} dout[b,pos,c] * in[b, pos + tap - off, c],  db[ch] = sum dout
// grid.x: channel blocks of 32 (over 3C), grid.y: slices of (b, pos); atomics into
// dw/db (zeroed by the host first).
template <typename T>
__global__ void hyena_short_wgrad_kernel(const float* __restrict__ dqp, const float* __restrict__ dkp,
                                         const float* __restrict__ dvp, const T* __restrict__ q,
                                         const T* __restrict__ k, const T* __restrict__ v, long long in_bst,
                                         long long in_pst, StencilGeom g, int B, int C, float* __restrict__ dw,
                                         float* __restrict__ db) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int ch = blockIdx.x * 32 + lane;  // channel of the 3C concatenation
  const bool ok = ch < 3 * C;
  const int which = ok ? ch / C : 0;
  const int c = ok ? ch - which * C : 0;
  const float* dout = which == 0 ? dqp : (which == 1 ? dkp : dvp);
  const T* in = which == 0 ? q : (which == 1 ? k : v);
  const long long Ntot = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long rows = (long long)B * Ntot;
  float acc[27];
#pragma unroll
  for (int t = 0; t < 27; ++t) acc[t] = 0.f;
  float bacc = 0.f;
  if (ok) {
    for (long long r = (long long)blockIdx.y * nw + warp; r < rows; r += (long long)gridDim.y * nw) {
      const long long pos = r % Ntot;
      const int b = (int)(r / Ntot);
      int p0, p1, p2;
      unflatten3(pos, g, p0, p1, p2);
      const float go = dout[r * C + c];
      bacc += go;
      int tap = 0;
      for (int a = 0; a < g.k[0]; ++a) {
        const int i0 = p0 + a - g.off[0];
        for (int bq = 0; bq < g.k[1]; ++bq) {
          const int i1 = p1 + bq - g.off[1];
          for (int e = 0; e < g.k[2]; ++e, ++tap) {
            const int i2 = p2 + e - g.off[2];
            if (i0 < 0 || i0 >= g.n[0] || i1 < 0 || i1 >= g.n[1] || i2 < 0 || i2 >= g.n[2]) continue;
            const long long pl = ((long long)i0 * g.n[1] + i1) * g.n[2] + i2;
            const float xin = DT<T>::load(in + (long long)b * in_bst + pl * in_pst + c);
#pragma unroll
            for (int t = 0; t < 27; ++t)
              if (t == tap) acc[t] = fmaf(go, xin, acc[t]);
          }
        }
      }
    }
  }
  // reduce over warps through shared memory, then one atomic per (ch, tap)
  __shared__ float red[32][33];
  for (int t = 0; t < g.ntaps + 1; ++t) {
    float val = (t < g.ntaps) ? 0.f : bacc;
#pragma unroll
    for (int u = 0; u < 27; ++u)
      if (u == t) val = acc[u];
    if (t == g.ntaps) val = bacc;
    red[warp][lane] = val;
    __syncthreads();
    if (warp == 0 && ok) {
      float s = 0.f;
      for (int j = 0; j < nw; ++j) s += red[j][lane];
      if (t < g.ntaps) atomicAdd(dw + (long long)ch * g.ntaps + t, s);
      else if (g.has_bias) atomicAdd(db + ch, s);
    }
    __syncthreads();
  }
}

}  // namespace hyfft
