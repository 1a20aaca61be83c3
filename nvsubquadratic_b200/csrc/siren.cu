// Implicit filter generation: the SIREN kernel network with the exponential modulation
// mask, forward and backward, in float32 on the CUDA cores.
//
//   x(p)   = grid coordinates of point p (per-axis coordinate vectors, row-major points)
//   h_0    = sin(W_pe x + b_pe)                       [E]
//   h_l    = sin(W_l h_{l-1} + b_l), l = 1 .. NH      [H]   (W_1 is H x E, the others H x H)
//   k[p,c] = mask(p, c) * (W_out h_NH + b_out)[c],  mask(p, c) = exp(-sum_d |x_d| |w_m[d, c]|)
//
// the network of nvsubquadratic/modules/kernels_nd.py (SIRENPositionalEmbeddingND :818-874,
// SIRENKernelND :1149-1199, no FiLM) and the window of nvsubquadratic/modules/masks_nd.py
// (ExponentialModulationND :229-255). The filter is written channels-last [G, C] (the
// reference's layout) or channel-major [C, G] (what the mixer's long convolution reads),
// so no copy or transpose sits between the generator and the filter transform.
//
// Kernels: the network on tiles of 16 points (256 threads over (point, unit) pairs, each
// layer's weights staged in shared memory) writes h_NH [G, H]; the readout is a tiled SGEMM
// (64 x 64 tile, 4 x 4 per thread) whose epilogue adds the bias, applies the mask and stores
// in the requested layout. The backward forms dh = (dk * mask) W_out and
// dW_out = (dk * mask)^T h, db_out as tiled SGEMMs (the latter split over point chunks,
// float atomics), then walks the network backwards tile by tile (recomputing the
// pre-activations), with each CTA's weight-gradient sums kept in shared memory across a
// grid-stride loop and added once per CTA (per tile when they do not fit). The mask's decay rates get no gradient: the
// reference describes them as fixed (masks_nd.py:150-156).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "../../include/hyfft.h"
#include "common.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;
int set_error(int code, const char* msg);  // engine.cu: the message hyfft_last_error returns

namespace {

constexpr int kMaxWidth = 128;  // embedding / hidden widths the kernels take

struct Net {
  const float* pe_w;  // [E][D]
  const float* pe_b;  // [E] or null
  const float* hw;    // hidden layers, concatenated: [H][E], then NH - 1 times [H][H]
  const float* hb;    // [NH][H] or null
  int D, E, H, NH;
};
struct Coords {
  const float* c[3];  // per-axis coordinate vectors
  int n[3];
  int D;
};

__device__ __forceinline__ const float* layer_w(const Net& n, int l) {
  return n.hw + (l == 0 ? 0 : (size_t)n.H * n.E + (size_t)(l - 1) * n.H * n.H);
}

__device__ __forceinline__ void point_coords(const Coords& co, long long p, float (&x)[3]) {
  long long r = p;
  x[0] = x[1] = x[2] = 0.f;
  for (int d = co.D - 1; d >= 0; --d) {
    const int i = (int)(r % co.n[d]);
    r /= co.n[d];
    x[d] = __ldg(co.c[d] + i);
  }
}

// The network on a tile of kNetP points, by all kNetThreads threads of the CTA over
// (point, unit) pairs: pre-activations pre[(l * kNetP + p) * W + u] and activations
// act = sin(pre) likewise (l = 0: the embedding; W the wider of E and H). Each hidden layer's
// weights are staged in shared memory first (rows padded by one, so that the lanes of a
// warp, on neighbouring units of one point, read different banks). xs: [kNetP][3] coordinates.
constexpr int kNetThreads = 256;
constexpr int kNetP = 16;

__device__ __forceinline__ void stage_layer(const Net& net, int l, float* wsm) {
  const int in = l == 0 ? net.E : net.H;
  const float* w = layer_w(net, l);
  for (int q = threadIdx.x; q < net.H * in; q += kNetThreads) {
    const int j = q / in, i = q - j * in;
    wsm[j * (in + 1) + i] = __ldg(w + q);
  }
}

__device__ __forceinline__ void net_forward_tile(const Net& net, const float* xs, float* pre, float* act, float* wsm,
                                                 int W) {
  for (int q = threadIdx.x; q < kNetP * net.E; q += kNetThreads) {
    const int p = q / net.E, e = q - p * net.E;
    float acc = net.pe_b ? __ldg(net.pe_b + e) : 0.f;
    for (int d = 0; d < net.D; ++d) acc = fmaf(__ldg(net.pe_w + e * net.D + d), xs[p * 3 + d], acc);
    pre[p * W + e] = acc;
    act[p * W + e] = sinf(acc);
  }
  int in = net.E;
  for (int l = 0; l < net.NH; ++l) {
    __syncthreads();  // the previous layer's activations, and wsm free again
    stage_layer(net, l, wsm);
    __syncthreads();
    const float* src = act + (size_t)l * kNetP * W;
    float* dp = pre + (size_t)(l + 1) * kNetP * W;
    float* da = act + (size_t)(l + 1) * kNetP * W;
    for (int q = threadIdx.x; q < kNetP * net.H; q += kNetThreads) {
      const int p = q / net.H, j = q - p * net.H;
      float acc = net.hb ? __ldg(net.hb + l * net.H + j) : 0.f;
      const float* wr = wsm + j * (in + 1);
      const float* ar = src + p * W;
      for (int i = 0; i < in; ++i) acc = fmaf(wr[i], ar[i], acc);
      dp[p * W + j] = acc;
      da[p * W + j] = sinf(acc);
    }
    in = net.H;
  }
  __syncthreads();
}

__device__ __forceinline__ void tile_coords(const Coords& co, long long p0, long long G, float* xs) {
  if (threadIdx.x < kNetP) {
    float x[3];
    point_coords(co, p0 + threadIdx.x < G ? p0 + threadIdx.x : G - 1, x);
    for (int d = 0; d < 3; ++d) xs[threadIdx.x * 3 + d] = x[d];
  }
  __syncthreads();
}

__host__ __device__ inline size_t net_smem_bytes(int NH, int E, int H) {
  const int W = E > H ? E : H, in = W;
  return sizeof(float) * (2 * (size_t)(NH + 1) * kNetP * W + (size_t)H * (in + 1) + 3 * kNetP);
}

// h_NH of every point: [G][H]
__global__ void __launch_bounds__(kNetThreads) siren_hidden_kernel(const Net net, const Coords co, long long G,
                                                                   float* __restrict__ hout) {
  extern __shared__ float smem[];
  const int W = max(net.E, net.H);
  float* pre = smem;                                 // [NH + 1][kNetP][W]
  float* act = pre + (size_t)(net.NH + 1) * kNetP * W;  // sin(pre)
  float* wsm = act + (size_t)(net.NH + 1) * kNetP * W;  // one layer's weights, rows padded
  float* xs = wsm + (size_t)net.H * (W + 1);          // [kNetP][3]
  for (long long p0 = (long long)blockIdx.x * kNetP; p0 < G; p0 += (long long)gridDim.x * kNetP) {
    tile_coords(co, p0, G, xs);
    net_forward_tile(net, xs, pre, act, wsm, W);
    const float* last = act + (size_t)net.NH * kNetP * W;
    for (int q = threadIdx.x; q < kNetP * net.H; q += kNetThreads) {
      const int p = q / net.H, j = q - p * net.H;
      if (p0 + p < G) hout[(p0 + p) * net.H + j] = last[p * W + j];
    }
    __syncthreads();
  }
}

// k[p][c] (layout 1: [G][C]; 0: [C][G]) = mask(p, c) * (sum_j h[p][j] wo[c][j] + bo[c])
__global__ void __launch_bounds__(256) siren_out_kernel(const float* __restrict__ h, const float* __restrict__ wo,
                                                        const float* __restrict__ bo, const float* __restrict__ mw,
                                                        const Coords co, long long G, int C, int H, int cl,
                                                        float* __restrict__ out) {
  __shared__ float As[16][68];  // [j][p]
  __shared__ float Bs[16][68];  // [j][c]
  __shared__ float Xs[3][64];   // |x_d| of the tile's points
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const long long p0 = (long long)blockIdx.x * 64;
  const int c0 = blockIdx.y * 64;
  if (mw && tid < 64) {
    float x[3];
    point_coords(co, p0 + tid < G ? p0 + tid : G - 1, x);
    for (int d = 0; d < 3; ++d) Xs[d][tid] = fabsf(x[d]);
  }
  float acc[4][4] = {};
  for (int k0 = 0; k0 < H; k0 += 16) {
    for (int e = tid; e < 64 * 16; e += 256) {
      const int r = e >> 4, j = e & 15;
      const long long p = p0 + r;
      const int c = c0 + r;
      As[j][r] = (p < G && k0 + j < H) ? __ldg(h + p * H + k0 + j) : 0.f;
      Bs[j][r] = (c < C && k0 + j < H) ? __ldg(wo + (long long)c * H + k0 + j) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float4 a = *reinterpret_cast<const float4*>(&As[j][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[j][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const long long p = p0 + ty * 4 + u;
    if (p >= G) continue;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int c = c0 + tx * 4 + v;
      if (c >= C) continue;
      float val = acc[u][v] + (bo ? __ldg(bo + c) : 0.f);
      if (mw) {
        float m = 1.f;
        for (int d = 0; d < co.D; ++d) m *= expf(-Xs[d][ty * 4 + u] * fabsf(__ldg(mw + (long long)d * C + c)));
        val *= m;
      }
      if (cl) out[p * C + c] = val;
      else out[(long long)c * G + p] = val;
    }
  }
}

// dk * mask at (p, c) for the backward's loaders (layout as the forward's output)
__device__ __forceinline__ float masked_dk(const float* __restrict__ dk, const float* __restrict__ mw, const float* ax,
                                           long long p, int c, long long G, int C, int D, int cl) {
  float v = cl ? __ldg(dk + p * C + c) : __ldg(dk + (long long)c * G + p);
  if (mw) {
    float m = 1.f;
    for (int d = 0; d < D; ++d) m *= expf(-ax[d] * fabsf(__ldg(mw + (long long)d * C + c)));
    v *= m;
  }
  return v;
}

// dh[p][j] = sum_c (dk * mask)[p][c] wo[c][j]: 64 x 64 tiles of [G][H], the sum over C in the CTA
__global__ void __launch_bounds__(256) siren_dh_kernel(const float* __restrict__ dk, const float* __restrict__ wo,
                                                       const float* __restrict__ mw, const Coords co, long long G,
                                                       int C, int H, int cl, float* __restrict__ dh) {
  __shared__ float As[16][68];  // [c][p]
  __shared__ float Bs[16][68];  // [c][j]
  __shared__ float Xs[64][3];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const long long p0 = (long long)blockIdx.x * 64;
  const int j0 = blockIdx.y * 64;
  if (tid < 64) {
    float x[3];
    point_coords(co, p0 + tid < G ? p0 + tid : G - 1, x);
    for (int d = 0; d < 3; ++d) Xs[tid][d] = fabsf(x[d]);
  }
  __syncthreads();
  float acc[4][4] = {};
  for (int k0 = 0; k0 < C; k0 += 16) {
    for (int e = tid; e < 64 * 16; e += 256) {
      // channels-last dk: neighbouring threads on neighbouring channels; channel-major: on points
      const int r = cl ? (e >> 4) : (e & 63), k = cl ? (e & 15) : (e >> 6);
      const long long p = p0 + r;
      As[k][r] = (p < G && k0 + k < C) ? masked_dk(dk, mw, Xs[r], p, k0 + k, G, C, co.D, cl) : 0.f;
    }
    for (int e = tid; e < 64 * 16; e += 256) {
      const int k = e >> 6, j = e & 63;
      Bs[k][j] = (k0 + k < C && j0 + j < H) ? __ldg(wo + (long long)(k0 + k) * H + j0 + j) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const long long p = p0 + ty * 4 + u;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int j = j0 + tx * 4 + v;
      if (p < G && j < H) dh[p * H + j] = acc[u][v];
    }
  }
}

// dwo[c][j] += sum_p (dk * mask)[p][c] h[p][j] and dbo[c] += sum_p (dk * mask)[p][c] over the
// CTA's chunk of points (grid z), one float atomic per output and CTA
__global__ void __launch_bounds__(256) siren_dwo_kernel(const float* __restrict__ dk, const float* __restrict__ h,
                                                        const float* __restrict__ mw, const Coords co, long long G,
                                                        int C, int H, int cl, long long chunk,
                                                        float* __restrict__ dwo, float* __restrict__ dbo) {
  __shared__ float As[16][68];  // [p][c]
  __shared__ float Bs[16][68];  // [p][j]
  __shared__ float Xs[16][3];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int c0 = blockIdx.x * 64, j0 = blockIdx.y * 64;
  const long long pa = (long long)blockIdx.z * chunk, pb = min(G, pa + chunk);
  float acc[4][4] = {};
  float bsum = 0.f;  // thread tid < 64: dbo of channel c0 + tid
  for (long long q0 = pa; q0 < pb; q0 += 16) {
    if (tid < 16) {
      float x[3];
      point_coords(co, q0 + tid < pb ? q0 + tid : pb - 1, x);
      for (int d = 0; d < 3; ++d) Xs[tid][d] = fabsf(x[d]);
    }
    __syncthreads();
    for (int e = tid; e < 16 * 64; e += 256) {
      const int k = cl ? (e >> 6) : (e & 15), c = cl ? (e & 63) : (e >> 4);
      const long long p = q0 + k;
      As[k][c] = (p < pb && c0 + c < C) ? masked_dk(dk, mw, Xs[k], p, c0 + c, G, C, co.D, cl) : 0.f;
      const int kk = e >> 6, j = e & 63;
      Bs[kk][j] = (q0 + kk < pb && j0 + j < H) ? __ldg(h + (q0 + kk) * H + j0 + j) : 0.f;
    }
    __syncthreads();
    if (blockIdx.y == 0 && tid < 64) {
#pragma unroll
      for (int k = 0; k < 16; ++k) bsum += As[k][tid];
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = c0 + ty * 4 + u;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int j = j0 + tx * 4 + v;
      if (c < C && j < H) atomicAdd(dwo + (long long)c * H + j, acc[u][v]);
    }
  }
  if (dbo && blockIdx.y == 0 && tid < 64 && c0 + tid < C) atomicAdd(dbo + c0 + tid, bsum);
}

// Backward through the network for every point (pre-activations recomputed), from
// dh = dL/dh_NH [G][H]: gradients of the hidden layers and the embedding, summed per CTA in
// shared memory over a grid-stride loop of point tiles and added to the outputs once.
struct NetGrad {
  float* pe_w;  // [E][D]
  float* pe_b;  // [E] or null
  float* hw;    // as Net::hw
  float* hb;    // [NH][H] or null
};

__host__ __device__ inline size_t grad_floats(int D, int E, int H, int NH) {
  return (size_t)E * D + E + (size_t)H * E + (size_t)(NH - 1) * H * H + (size_t)NH * H;
}

__global__ void __launch_bounds__(kNetThreads) siren_hidden_bwd_kernel(const Net net, const Coords co, long long G,
                                                                       const float* __restrict__ dh, NetGrad g,
                                                                       int acc_smem) {
  extern __shared__ float smem[];
  const int W = max(net.E, net.H);
  float* pre = smem;                                    // [NH + 1][kNetP][W]
  float* act = pre + (size_t)(net.NH + 1) * kNetP * W;  // sin(pre)
  float* wsm = act + (size_t)(net.NH + 1) * kNetP * W;  // one layer's weights, rows padded
  float* xs = wsm + (size_t)net.H * (W + 1);            // [kNetP][3]
  float* gA = xs + 3 * kNetP;                           // dL/dpre of the current layer [kNetP][W]
  float* gB = gA + (size_t)kNetP * W;                   // dL/dact of the layer below
  float* acc = gB + (size_t)kNetP * W;                  // the CTA's gradient sums (grad_floats)
  // accumulator offsets: pe_w, pe_b, then per hidden layer its weight, then the hidden biases
  const size_t o_pe_b = (size_t)net.E * net.D, o_hw = o_pe_b + net.E;
  const size_t o_hb = o_hw + (size_t)net.H * net.E + (size_t)(net.NH - 1) * net.H * net.H;
  const size_t nacc = grad_floats(net.D, net.E, net.H, net.NH);
  auto dst_of = [&](size_t i) -> float* {
    if (i < o_pe_b) return g.pe_w + i;
    if (i < o_hw) return g.pe_b ? g.pe_b + (i - o_pe_b) : nullptr;
    if (i < o_hb) return g.hw + (i - o_hw);
    return g.hb ? g.hb + (i - o_hb) : nullptr;
  };
  // the CTA's sums in shared memory when they fit, else added to the outputs per tile
  auto add = [&](size_t i, float v) {
    if (acc_smem) {
      acc[i] += v;
    } else if (float* d = dst_of(i)) {
      atomicAdd(d, v);
    }
  };
  if (acc_smem)
    for (size_t i = threadIdx.x; i < nacc; i += kNetThreads) acc[i] = 0.f;
  for (long long p0 = (long long)blockIdx.x * kNetP; p0 < G; p0 += (long long)gridDim.x * kNetP) {
    tile_coords(co, p0, G, xs);
    net_forward_tile(net, xs, pre, act, wsm, W);
    // dL/dact of the last layer (zero for points past the end)
    for (int q = threadIdx.x; q < kNetP * net.H; q += kNetThreads) {
      const int p = q / net.H, j = q - p * net.H;
      gB[p * W + j] = (p0 + p < G) ? __ldg(dh + (p0 + p) * net.H + j) : 0.f;
    }
    __syncthreads();
    for (int l = net.NH; l >= 0; --l) {
      const int width = l == 0 ? net.E : net.H;
      const float* pl = pre + (size_t)l * kNetP * W;
      for (int q = threadIdx.x; q < kNetP * width; q += kNetThreads) {
        const int p = q / width, u = q - p * width;
        gA[p * W + u] = gB[p * W + u] * cosf(pl[p * W + u]);
      }
      if (l > 0) stage_layer(net, l - 1, wsm);  // the weights of hidden layer l (index l - 1)
      __syncthreads();
      if (l == 0) {  // embedding: dW_pe[e][d] += sum_p gA[p][e] x_d[p], db_pe[e] += sum_p gA[p][e]
        for (int q = threadIdx.x; q < net.E * (net.D + 1); q += kNetThreads) {
          const int e = q / (net.D + 1), d = q - e * (net.D + 1);
          float sacc = 0.f;
          for (int p = 0; p < kNetP; ++p) sacc = fmaf(gA[p * W + e], d < net.D ? xs[p * 3 + d] : 1.f, sacc);
          add(d < net.D ? (size_t)e * net.D + d : o_pe_b + e, sacc);
        }
      } else {  // hidden layer l: input act[l - 1]
        const int in = l == 1 ? net.E : net.H;
        const float* a_in = act + (size_t)(l - 1) * kNetP * W;
        const size_t o_w = o_hw + (l == 1 ? 0 : (size_t)net.H * net.E + (size_t)(l - 2) * net.H * net.H);
        // neighbouring threads on neighbouring inputs i of one unit j
        for (int q = threadIdx.x; q < net.H * (in + 1); q += kNetThreads) {
          const int j = q / (in + 1), i = q - j * (in + 1);
          float sacc = 0.f;
          for (int p = 0; p < kNetP; ++p) sacc = fmaf(gA[p * W + j], i < in ? a_in[p * W + i] : 1.f, sacc);
          add(i < in ? o_w + (size_t)j * in + i : o_hb + (size_t)(l - 1) * net.H + j, sacc);
        }
        // dL/dact of the layer below: gB[p][i] = sum_j W[j][i] gA[p][j]
        for (int q = threadIdx.x; q < kNetP * in; q += kNetThreads) {
          const int p = q / in, i = q - p * in;
          float sacc = 0.f;
          for (int j = 0; j < net.H; ++j) sacc = fmaf(wsm[j * (in + 1) + i], gA[p * W + j], sacc);
          gB[p * W + i] = sacc;
        }
      }
      __syncthreads();
    }
  }
  if (!acc_smem) return;
  __syncthreads();
  for (size_t i = threadIdx.x; i < nacc; i += kNetThreads)
    if (float* d = dst_of(i)) atomicAdd(d, acc[i]);
}

}  // namespace
}  // namespace hyfft

namespace hyfft {
namespace {

struct SirenPlan {
  long long G = 1;
  Coords co;
  Net net;
  int C = 0, cl = 1, W = 0;
  int acc_smem = 1;  // backward sums in shared memory
  size_t smem_fwd = 0, smem_bwd = 0;
};

constexpr size_t kSmemMax = 227 * 1024;

int siren_plan(const hyfft_siren_desc* d, const float* coords, const float* pe_w, const float* pe_b, const float* hw,
               const float* hb, SirenPlan& s) {
  if (!d || !coords || !pe_w || !hw) return set_error(HYFFT_ERR_INVALID, "siren: null descriptor or parameter");
  if (d->ndim < 1 || d->ndim > 3 || d->embedding < 1 || d->hidden < 1 || d->num_hidden < 1 || d->channels < 1)
    return set_error(HYFFT_ERR_INVALID, "siren: ndim must be 1..3 and every width positive");
  if (d->layout != HYFFT_LAYOUT_BHL && d->layout != HYFFT_LAYOUT_BLH) return set_error(HYFFT_ERR_INVALID, "siren: bad layout");
  if (d->embedding > kMaxWidth || d->hidden > kMaxWidth)
    return set_error(HYFFT_ERR_UNSUPPORTED, "siren: embedding and hidden widths above 128 are not covered");
  s.co.D = d->ndim;
  long long off = 0;
  for (int a = 0; a < 3; ++a) {
    s.co.n[a] = a < d->ndim ? d->n[a] : 1;
    if (s.co.n[a] < 1) return set_error(HYFFT_ERR_INVALID, "siren: grid extents must be positive");
    s.co.c[a] = coords + off;
    if (a < d->ndim) off += s.co.n[a];
    s.G *= s.co.n[a];
  }
  s.net = Net{pe_w, pe_b, hw, hb, d->ndim, d->embedding, d->hidden, d->num_hidden};
  s.C = d->channels;
  s.cl = d->layout == HYFFT_LAYOUT_BLH ? 1 : 0;
  s.W = std::max(d->embedding, d->hidden);
  // the backward keeps its gradient sums in shared memory when they fit beside the tile
  const size_t nacc = grad_floats(d->ndim, d->embedding, d->hidden, d->num_hidden);
  s.smem_fwd = net_smem_bytes(d->num_hidden, d->embedding, d->hidden);
  const size_t bwd_base = s.smem_fwd + sizeof(float) * 2 * (size_t)kNetP * s.W;
  s.acc_smem = bwd_base + sizeof(float) * nacc <= kSmemMax ? 1 : 0;
  s.smem_bwd = bwd_base + (s.acc_smem ? sizeof(float) * nacc : 0);
  if (s.smem_fwd > kSmemMax || s.smem_bwd > kSmemMax)
    return set_error(HYFFT_ERR_UNSUPPORTED, "siren: the network's activations do not fit a CTA's shared memory");
  return HYFFT_OK;
}

int grid_stride_ctas(long long G) {
  return (int)std::max<long long>(1, std::min<long long>((G + kNetP - 1) / kNetP, 4 * 148));
}

int launched() {
  if (cudaGetLastError() != cudaSuccess) return set_error(HYFFT_ERR_CUDA, "siren: kernel launch failed");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

}  // namespace
}  // namespace hyfft

using namespace hyfft;

extern "C" {

int hyfft_siren_sizes(const hyfft_siren_desc* d, size_t* saved_bytes, size_t* workspace_bytes) {
  if (!d || d->ndim < 1 || d->ndim > 3 || d->hidden < 1) return set_error(HYFFT_ERR_INVALID, "siren: bad descriptor");
  long long G = 1;
  for (int a = 0; a < d->ndim; ++a) {
    if (d->n[a] < 1) return set_error(HYFFT_ERR_INVALID, "siren: grid extents must be positive");
    G *= d->n[a];
  }
  if (saved_bytes) *saved_bytes = sizeof(float) * (size_t)G * d->hidden;      // h of the last hidden layer
  if (workspace_bytes) *workspace_bytes = sizeof(float) * (size_t)G * d->hidden;  // its gradient
  return HYFFT_OK;
}

int hyfft_siren_forward(const hyfft_siren_desc* d, const float* coords, const float* pe_w, const float* pe_b,
                        const float* hid_w, const float* hid_b, const float* out_w, const float* out_b,
                        const float* mask_w, float* kernel, void* saved, size_t saved_bytes, void* stream) {
  SirenPlan s;
  int rc = siren_plan(d, coords, pe_w, pe_b, hid_w, hid_b, s);
  if (rc != HYFFT_OK) return rc;
  if (!out_w || !kernel || !saved) return set_error(HYFFT_ERR_INVALID, "siren: null output or saved buffer");
  if (saved_bytes < sizeof(float) * (size_t)s.G * s.net.H) return set_error(HYFFT_ERR_WORKSPACE, "siren: saved buffer too small");
  if (bind_device_of(kernel) != HYFFT_OK) return HYFFT_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* h = static_cast<float*>(saved);
  if (!kernel_smem_once((const void*)siren_hidden_kernel, s.smem_fwd)) return HYFFT_ERR_CUDA;
  siren_hidden_kernel<<<grid_stride_ctas(s.G), kNetThreads, s.smem_fwd, st>>>(s.net, s.co, s.G, h);
  if ((rc = launched()) != HYFFT_OK) return rc;
  const dim3 og((unsigned)((s.G + 63) / 64), (unsigned)((s.C + 63) / 64));
  siren_out_kernel<<<og, 256, 0, st>>>(h, out_w, out_b, mask_w, s.co, s.G, s.C, s.net.H, s.cl, kernel);
  return launched();
}

int hyfft_siren_backward(const hyfft_siren_desc* d, const float* coords, const float* pe_w, const float* pe_b,
                         const float* hid_w, const float* hid_b, const float* out_w, const float* mask_w,
                         const float* dkernel, const void* saved, float* d_pe_w, float* d_pe_b, float* d_hid_w,
                         float* d_hid_b, float* d_out_w, float* d_out_b, void* workspace, size_t workspace_bytes,
                         void* stream) {
  SirenPlan s;
  int rc = siren_plan(d, coords, pe_w, pe_b, hid_w, hid_b, s);
  if (rc != HYFFT_OK) return rc;
  if (!out_w || !dkernel || !saved || !d_pe_w || !d_hid_w || !d_out_w || !workspace)
    return set_error(HYFFT_ERR_INVALID, "siren: null tensor in the backward");
  if ((pe_b != nullptr) != (d_pe_b != nullptr) || (hid_b != nullptr) != (d_hid_b != nullptr))
    return set_error(HYFFT_ERR_INVALID, "siren: bias gradients must match the biases given");
  if (workspace_bytes < sizeof(float) * (size_t)s.G * s.net.H) return set_error(HYFFT_ERR_WORKSPACE, "siren: workspace too small");
  if (bind_device_of(dkernel) != HYFFT_OK) return HYFFT_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int D = s.net.D, E = s.net.E, H = s.net.H, NH = s.net.NH;
  // every gradient is overwritten: zero, then the kernels add their per-CTA sums
  const size_t nhw = (size_t)H * E + (size_t)(NH - 1) * H * H;
  if (cudaMemsetAsync(d_pe_w, 0, sizeof(float) * E * D, st) != cudaSuccess ||
      (d_pe_b && cudaMemsetAsync(d_pe_b, 0, sizeof(float) * E, st) != cudaSuccess) ||
      cudaMemsetAsync(d_hid_w, 0, sizeof(float) * nhw, st) != cudaSuccess ||
      (d_hid_b && cudaMemsetAsync(d_hid_b, 0, sizeof(float) * NH * H, st) != cudaSuccess) ||
      cudaMemsetAsync(d_out_w, 0, sizeof(float) * (size_t)s.C * H, st) != cudaSuccess ||
      (d_out_b && cudaMemsetAsync(d_out_b, 0, sizeof(float) * s.C, st) != cudaSuccess))
    return HYFFT_ERR_CUDA;
  const float* h = static_cast<const float*>(saved);
  float* dh = static_cast<float*>(workspace);
  const dim3 hg((unsigned)((s.G + 63) / 64), (unsigned)((H + 63) / 64));
  siren_dh_kernel<<<hg, 256, 0, st>>>(dkernel, out_w, mask_w, s.co, s.G, s.C, H, s.cl, dh);
  if ((rc = launched()) != HYFFT_OK) return rc;
  // dW_out: point chunks sized for about four waves of 148 SMs
  const long long tiles = (long long)((s.C + 63) / 64) * ((H + 63) / 64);
  const long long nz = std::max<long long>(1, std::min<long long>((s.G + 255) / 256, (4 * 148 + tiles - 1) / tiles));
  const long long chunk = ((s.G + nz - 1) / nz + 15) / 16 * 16;
  const dim3 wg((unsigned)((s.C + 63) / 64), (unsigned)((H + 63) / 64), (unsigned)((s.G + chunk - 1) / chunk));
  siren_dwo_kernel<<<wg, 256, 0, st>>>(dkernel, h, mask_w, s.co, s.G, s.C, H, s.cl, chunk, d_out_w, d_out_b);
  if ((rc = launched()) != HYFFT_OK) return rc;
  if (!kernel_smem_once((const void*)siren_hidden_bwd_kernel, s.smem_bwd)) return HYFFT_ERR_CUDA;
  siren_hidden_bwd_kernel<<<grid_stride_ctas(s.G), kNetThreads, s.smem_bwd, st>>>(
      s.net, s.co, s.G, dh, NetGrad{d_pe_w, d_pe_b, d_hid_w, d_hid_b}, s.acc_smem);
  return launched();
}

}  // extern "C"
