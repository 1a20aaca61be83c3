// Plane-marching kernels for the 3D depthwise short convolution of the Hyena mixer
// (KX x KY x KZ taps, 16-bit activations, channels-last): the forward stencil on q, k, v
// (with z = q' * g1(k')), its transpose for dq, dk, dv, and the weight / bias gradients.
//
// A CTA owns 64 channels (two per lane, one 128-byte row of a position per warp access),
// a tile of TY x TZ output positions of the (y, z) plane and a run of x planes. It marches
// along x with a ring of four input planes in shared memory: the KX planes the current
// output plane reads and the next one, which cp.async fetches (16-byte chunks, halo and
// out-of-range positions zero-filled by the copy itself) while the current plane is
// computed. Each warp computes one y row of 16 z positions, four at a time: per stencil
// row (a, b) it reads 4 + KZ - 1 neighbouring positions from shared memory and applies
// the KZ taps of that row, so the KX * KY * KZ weights (or, for the weight gradient, the
// accumulators) stay in registers.
//
// A 2D grid (Y, Z) with Z >= 96 runs the same kernels as a march along Y: each "plane" is
// one row of up to 128 positions (tile 1 x 128, KY = 1), so a CTA streams a run of rows
// through the four-slot ring, every input row is read from HBM once per run (plus two
// halo rows), and the CTA's weight-gradient partial sums cover the whole run.
//
// Reference: the depthwise short conv applied to q, k, v before the long convolution,
// nvsubquadratic Hyena mixer (hyena_nd.py:530-546); cross-correlation with left padding
// off = (k - 1) / 2 ("same") or k - 1 (causal) per axis.
#pragma once

#include "hyena_elem.cuh"

namespace hyfft {

constexpr int kS3TY = 4;    // output rows (y) per tile of a 3D plane: two warps per row
constexpr int kS3TZ = 32;   // output positions (z) per tile row: 16 per warp
constexpr int kS3Buf = 4;   // ring of input planes
constexpr int kS3ZU = 4;    // z positions a warp computes per step
// A 2D grid marches along its first axis as x with one-row "planes" (y extent 1) of up to
// 128 positions: tile 1 x 128, eight warps side by side along z.
constexpr int kS2TZ = 128;

template <int KY, int KZ, int TY = kS3TY, int TZ = kS3TZ>
__host__ __device__ constexpr int s3_plane_positions() {
  return (TY + KY - 1) * (TZ + KZ - 1);
}
// ring depth: four planes for a 3D stencil, one for a 2D stencil run as one x plane
template <int KX>
__host__ __device__ constexpr int s3_ring() {
  return KX == 1 ? 1 : kS3Buf;
}
template <int KX, int KY, int KZ, int TY = kS3TY, int TZ = kS3TZ>
__host__ __device__ constexpr size_t s3_smem_bytes() {
  return (size_t)s3_ring<KX>() * s3_plane_positions<KY, KZ, TY, TZ>() * kElemCG * 2;  // 16-bit elements
}
// the weight-gradient kernel reuses its ring for the CTA reduction [8 warps][taps + 1][64]
template <int KX, int KY, int KZ, int TY = kS3TY, int TZ = kS3TZ>
__host__ __device__ constexpr size_t s3_wgrad_smem_bytes() {
  return s3_smem_bytes<KX, KY, KZ, TY, TZ>() > (size_t)8 * (KX * KY * KZ + 1) * kElemCG * 4
             ? s3_smem_bytes<KX, KY, KZ, TY, TZ>()
             : (size_t)8 * (KX * KY * KZ + 1) * kElemCG * 4;
}

struct S3Tile {
  int c0, y0, z0, b, xa, xb;
};

// Tile of this CTA: grid (ceil(C / 64), y tiles * z tiles, B * x chunks).
template <int TY, int TZ>
__device__ __forceinline__ S3Tile s3_tile(const StencilGeom& g, int xchunk) {
  S3Tile t;
  const int nzt = (g.n[2] + TZ - 1) / TZ;
  const int nxc = (g.n[0] + xchunk - 1) / xchunk;
  t.c0 = blockIdx.x * kElemCG;
  t.y0 = (blockIdx.y / nzt) * TY;
  t.z0 = (blockIdx.y % nzt) * TZ;
  t.b = blockIdx.z / nxc;
  t.xa = (blockIdx.z % nxc) * xchunk;
  t.xb = min(g.n[0], t.xa + xchunk);
  return t;
}

// cp.async of input plane xin of the tile (positions y0 - oy .. , z0 - oz ..) into a ring slot.
template <typename T, int KY, int KZ, int TY, int TZ>
__device__ __forceinline__ void s3_load_plane(T* slot, const T* src, long long bst, long long pst,
                                              const StencilGeom& g, const S3Tile& t, int C, int xin, int oy,
                                              int oz) {
  constexpr int ZW = TZ + KZ - 1, NPOS = s3_plane_positions<KY, KZ, TY, TZ>();
  const bool xok = xin >= 0 && xin < g.n[0];
  for (int q = threadIdx.x; q < NPOS * 8; q += blockDim.x) {
    const int pos = q >> 3, part = q & 7;
    const int yy = pos / ZW, zz = pos - yy * ZW;
    const int gy = t.y0 - oy + yy, gz = t.z0 - oz + zz, c = t.c0 + part * 8;
    const bool ok = xok && gy >= 0 && gy < g.n[1] && gz >= 0 && gz < g.n[2] && c < C;
    const T* s = ok ? src + (long long)t.b * bst + (((long long)xin * g.n[1] + gy) * g.n[2] + gz) * pst + c : src;
    const unsigned d = (unsigned)__cvta_generic_to_shared(slot + pos * kElemCG + part * 8);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(s), "r"(ok ? 16 : 0) : "memory");
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// One-row planes (the 2D march, KY = 1): a thread's 16-byte chunks sit at the same offsets
// in every plane, so their in-plane offsets (int: the host keeps a row of positions times
// the position stride below 2^31) and range checks are computed once per kernel.
template <int KZ, int TZ>
struct RowChunks {
  static constexpr int NCH = (TZ + KZ - 1) * 8, IT = (NCH + kElemThreads - 1) / kElemThreads;
  int off[IT];
  unsigned okm;
  __device__ __forceinline__ RowChunks(const StencilGeom& g, const S3Tile& t, int C, long long pst, int oz) {
    okm = 0;
#pragma unroll
    for (int i = 0; i < IT; ++i) {
      const int q = threadIdx.x + i * kElemThreads;
      const int gz = t.z0 - oz + (q >> 3), c = t.c0 + (q & 7) * 8;
      const bool ok = q < NCH && gz >= 0 && gz < g.n[2] && c < C;
      off[i] = ok ? (int)((long long)gz * pst + c) : 0;
      okm |= (ok ? 1u : 0u) << i;
    }
  }
  // cp.async of row plane xin (one commit group)
  template <typename T>
  __device__ __forceinline__ void load(T* slot, const T* src, long long bst, long long pst, const StencilGeom& g,
                                       const S3Tile& t, int xin) const {
    const bool xok = xin >= 0 && xin < g.n[0];
    const T* base = src + (long long)t.b * bst + (long long)xin * g.n[2] * pst;
#pragma unroll
    for (int i = 0; i < IT; ++i) {
      const int q = threadIdx.x + i * kElemThreads;
      if (q < NCH) {
        const bool ok = xok && ((okm >> i) & 1u);
        const T* sp = ok ? base + off[i] : src;
        const unsigned d = (unsigned)__cvta_generic_to_shared(slot + q * 8);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(sp), "r"(ok ? 16 : 0)
                     : "memory");
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
};

template <typename T>
__device__ __forceinline__ float2 s3_ld(const T* p) {
  return V2<T>::load(p);
}

// A 2D stencil runs as KX = 1 over a single x plane (n[0] = 1): one ring slot, no prefetch.
// Forward stencil (MODE 0) or its transpose (MODE 1) over q, k, v in turn.
// MODE 0: in = q/k/v (batch stride in_bst, position stride in_pst), out = q'/k'/v'
//   contiguous [B, N, C] (dtype-rounded) and z = q' * g1(k').
// MODE 1: in = dq'/dk'/dv' contiguous, out = dq/dk/dv (out_bst, out_pst):
//   out[p] = sum_tap w[tap] in[p - tap + off], a forward stencil with flipped taps and
//   left padding k - 1 - off.
template <typename T, int KX, int KY, int KZ, int MODE, int TY = kS3TY, int TZ = kS3TZ>
__global__ void __launch_bounds__(kElemThreads, (KX == 1 || KY == 1) ? 3 : 2) hyena_plane_stencil_kernel(
    const T* __restrict__ in0, const T* __restrict__ in1, const T* __restrict__ in2, long long in_bst,
    long long in_pst, T* __restrict__ out0, T* __restrict__ out1, T* __restrict__ out2, long long out_bst,
    long long out_pst, T* __restrict__ z, StencilGeom g, int C, const float* __restrict__ w,
    const float* __restrict__ bias, int gate1, int xchunk) {
  constexpr int NT = KX * KY * KZ, ZW = TZ + KZ - 1, NPOS = s3_plane_positions<KY, KZ, TY, TZ>(), NB = s3_ring<KX>();
  constexpr int WPR = TZ / 16;  // warps per tile row, 16 z positions each
  static_assert(TY * WPR == kElemThreads / 32, "one warp per 16 positions of the tile");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  const S3Tile t = s3_tile<TY, TZ>(g, xchunk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int yl = warp / WPR, zw = (warp % WPR) * 16;
  const int c = t.c0 + 2 * lane;
  const bool cok = c < C;
  const int ox = MODE == 0 ? g.off[0] : KX - 1 - g.off[0];
  const int oy = MODE == 0 ? g.off[1] : KY - 1 - g.off[1];
  const int oz = MODE == 0 ? g.off[2] : KZ - 1 - g.off[2];
  const long long N = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long ps = MODE == 0 ? in_pst : (long long)C;
  const long long bs = MODE == 0 ? in_bst : N * C;
  const int gy = t.y0 + yl;
  const RowChunks<KZ, TZ> rows(g, t, C, ps, oz);  // used by one-row planes only
  auto load_plane = [&](T* slot, const T* src, int xin) {
    if constexpr (KY == 1 && TY == 1) rows.template load<T>(slot, src, bs, ps, g, t, xin);
    else s3_load_plane<T, KY, KZ, TY, TZ>(slot, src, bs, ps, g, t, C, xin, oy, oz);
  };

#pragma unroll 1
  for (int ti = 0; ti < 3; ++ti) {
    // weights of this tensor for channels c, c + 1 (MODE 1: flipped taps)
    float2 wr[NT];
#pragma unroll
    for (int a = 0; a < KX; ++a)
#pragma unroll
      for (int bq = 0; bq < KY; ++bq)
#pragma unroll
        for (int e = 0; e < KZ; ++e) {
          const int tap = MODE == 0 ? (a * KY + bq) * KZ + e
                                    : ((KX - 1 - a) * KY + (KY - 1 - bq)) * KZ + (KZ - 1 - e);
          const long long wi = ((long long)ti * C + c) * NT + tap;
          wr[(a * KY + bq) * KZ + e] = cok ? make_float2(__ldg(w + wi), __ldg(w + wi + NT)) : make_float2(0.f, 0.f);
        }
    const float2 bs2 = (MODE == 0 && g.has_bias && bias && cok)
                           ? make_float2(__ldg(bias + (long long)ti * C + c), __ldg(bias + (long long)ti * C + c + 1))
                           : make_float2(0.f, 0.f);
    // (pointers picked by value: an array indexed by ti would live in local memory)
    const T* src = ti == 0 ? in0 : (ti == 1 ? in1 : in2);
    T* dst = ti == 0 ? out0 : (ti == 1 ? out1 : out2);
    // prologue: the KX planes of the first output plane
#pragma unroll 1
    for (int a = 0; a < KX; ++a) {
      const int xin = t.xa - ox + a;
      load_plane(ring + ((xin + 256) % NB) * NPOS * kElemCG, src, xin);
    }
#pragma unroll 1
    for (int x = t.xa; x < t.xb; ++x) {
      const bool pre = x + 1 < t.xb;
      if (pre) {
        const int xin = x - ox + KX;
        load_plane(ring + ((xin + 256) % NB) * NPOS * kElemCG, src, xin);
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      }
      __syncthreads();
      if (cok && gy < g.n[1]) {
#pragma unroll 1
        for (int zb = 0; zb < 16; zb += kS3ZU) {
          float2 acc[kS3ZU];
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) acc[i] = bs2;
          // z = q' * g1(k') needs q' of these positions (written by this thread in the q sweep):
          // load it before the stencil so the load latency hides behind the taps
          float2 qpre[kS3ZU];
          if (MODE == 0 && ti == 1) {
#pragma unroll
            for (int i = 0; i < kS3ZU; ++i) {
              const int gz = t.z0 + zw + zb + i;
              const long long o = ((long long)t.b * N + ((long long)x * g.n[1] + gy) * g.n[2] + gz) * C + c;
              qpre[i] = gz < g.n[2] ? V2<T>::load(out0 + o) : make_float2(0.f, 0.f);
            }
          }
#pragma unroll
          for (int a = 0; a < KX; ++a) {
            const T* sl = ring + ((x - ox + a + 256) % NB) * NPOS * kElemCG;
#pragma unroll
            for (int bq = 0; bq < KY; ++bq) {
              const T* row = sl + ((yl + bq) * ZW + zw + zb) * kElemCG + 2 * lane;
              float2 v[kS3ZU + KZ - 1];
#pragma unroll
              for (int m = 0; m < kS3ZU + KZ - 1; ++m) v[m] = s3_ld<T>(row + m * kElemCG);
#pragma unroll
              for (int i = 0; i < kS3ZU; ++i)
#pragma unroll
                for (int e = 0; e < KZ; ++e) {
                  const float2 wv = wr[(a * KY + bq) * KZ + e];
                  acc[i] = ffma2(wv, v[i + e], acc[i]);
                }
            }
          }
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) {
            const int gz = t.z0 + zw + zb + i;
            if (gz >= g.n[2]) break;
            const long long pos = ((long long)x * g.n[1] + gy) * g.n[2] + gz;
            if constexpr (MODE == 0) {
              const long long o = ((long long)t.b * N + pos) * C + c;
              const float2 r = V2<T>::round(acc[i]);
              V2<T>::store(dst + o, r);
              if (ti == 1) {  // z = q' * g1(k')
                const float2 qv = qpre[i];
                const float2 g1 = V2<T>::round(make_float2(gate_f(gate1, r.x), gate_f(gate1, r.y)));
                V2<T>::store(z + o, make_float2(qv.x * g1.x, qv.y * g1.y));
              }
            } else {
              V2<T>::store(dst + (long long)t.b * out_bst + pos * out_pst + c, acc[i]);
            }
          }
        }
      }
      __syncthreads();  // the next prefetch overwrites the oldest plane read here
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
  }
}

// Transposed stencil and weight / bias gradients in one march over the same ring of dout
// planes (dq'/dk'/dv', contiguous): for output position p the ring holds the neighbourhood
// dout[p - tap + off] of every tap, so
//   dq[p]     = sum_tap w[tap] dout[p - tap + off]                (as MODE 1 above)
//   dW[tap]  += in[p] dout[p - tap + off]  (= sum_p' dout[p'] in[p' + tap - off])
//   db       += dout[p]                     (the centre tap's neighbour)
// with in = q/k/v read at p only (in_bst, in_pst): the gradient pass needs no ring of its
// own, and every ring value is unpacked once for both products. Per-thread accumulators, a
// shared-memory reduction over the CTA's warps and one atomic per channel and tap per CTA
// (dw, db zeroed by the host).
template <typename T, int KX, int KY, int KZ, int TY, int TZ>
__global__ void __launch_bounds__(kElemThreads, 2) hyena_plane_bwd_kernel(
    const T* __restrict__ d0, const T* __restrict__ d1, const T* __restrict__ d2, const T* __restrict__ in0,
    const T* __restrict__ in1, const T* __restrict__ in2, long long in_bst, long long in_pst, T* __restrict__ out0,
    T* __restrict__ out1, T* __restrict__ out2, StencilGeom g, int C, const float* __restrict__ w,
    float* __restrict__ dw, float* __restrict__ db, int xchunk) {
  constexpr int NT = KX * KY * KZ, ZW = TZ + KZ - 1, NPOS = s3_plane_positions<KY, KZ, TY, TZ>(), NB = s3_ring<KX>();
  constexpr int NW = kElemThreads / 32;
  constexpr int WPR = TZ / 16;  // warps per tile row, 16 z positions each
  static_assert(TY * WPR == NW, "one warp per 16 positions of the tile");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw);  // [NW][NT + 1][64] after the march
  const S3Tile t = s3_tile<TY, TZ>(g, xchunk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int yl = warp / WPR, zw = (warp % WPR) * 16;
  const int c = t.c0 + 2 * lane;
  const bool cok = c < C;
  // ring offsets of the transposed stencil (flipped taps, left padding k - 1 - off)
  const int ox = KX - 1 - g.off[0], oy = KY - 1 - g.off[1], oz = KZ - 1 - g.off[2];
  // neighbourhood index of the centre tap (tap == off on every axis)
  const int ac = KX - 1 - g.off[0], bc = KY - 1 - g.off[1], ec = KZ - 1 - g.off[2];
  const long long N = (long long)g.n[0] * g.n[1] * g.n[2];
  const long long ps = C, bs = N * C;
  const int gy = t.y0 + yl;
  const RowChunks<KZ, TZ> rows(g, t, C, ps, oz);  // used by one-row planes only
  auto load_plane = [&](T* slot, const T* src, int xin) {
    if constexpr (KY == 1 && TY == 1) rows.template load<T>(slot, src, bs, ps, g, t, xin);
    else s3_load_plane<T, KY, KZ, TY, TZ>(slot, src, bs, ps, g, t, C, xin, oy, oz);
  };

#pragma unroll 1
  for (int ti = 0; ti < 3; ++ti) {
    float2 wr[NT], dacc[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int a = j / (KY * KZ), bq = (j / KZ) % KY, e = j % KZ;
      const int tap = ((KX - 1 - a) * KY + (KY - 1 - bq)) * KZ + (KZ - 1 - e);
      const long long wi = ((long long)ti * C + c) * NT + tap;
      wr[j] = cok ? make_float2(__ldg(w + wi), __ldg(w + wi + NT)) : make_float2(0.f, 0.f);
      dacc[j] = make_float2(0.f, 0.f);
    }
    float2 accb = make_float2(0.f, 0.f);
    const T* src = ti == 0 ? d0 : (ti == 1 ? d1 : d2);
    const T* xin_t = ti == 0 ? in0 : (ti == 1 ? in1 : in2);
    T* dst = ti == 0 ? out0 : (ti == 1 ? out1 : out2);
#pragma unroll 1
    for (int a = 0; a < KX; ++a) {
      const int xin = t.xa - ox + a;
      load_plane(ring + ((xin + 256) % NB) * NPOS * kElemCG, src, xin);
    }
#pragma unroll 1
    for (int x = t.xa; x < t.xb; ++x) {
      const bool pre = x + 1 < t.xb;
      if (pre) {
        const int xin = x - ox + KX;
        load_plane(ring + ((xin + 256) % NB) * NPOS * kElemCG, src, xin);
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      }
      __syncthreads();
      if (cok && gy < g.n[1]) {
        // in[p] of the next step loaded one step ahead, behind the current step's taps
        auto ld_in = [&](int zb, float2 (&iv)[kS3ZU]) {
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) {
            const int gz = t.z0 + zw + zb + i;
            const long long pos = ((long long)x * g.n[1] + gy) * g.n[2] + gz;
            iv[i] = (zb < 16 && gz < g.n[2]) ? V2<T>::load(xin_t + (long long)t.b * in_bst + pos * in_pst + c)
                                             : make_float2(0.f, 0.f);
          }
        };
        float2 inext[kS3ZU];
        ld_in(0, inext);
#pragma unroll 1
        for (int zb = 0; zb < 16; zb += kS3ZU) {
          float2 iv[kS3ZU], acc[kS3ZU];
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) {
            iv[i] = inext[i];
            acc[i] = make_float2(0.f, 0.f);
          }
          ld_in(zb + kS3ZU, inext);
#pragma unroll
          for (int a = 0; a < KX; ++a) {
            const T* sl = ring + ((x - ox + a + 256) % NB) * NPOS * kElemCG;
#pragma unroll
            for (int bq = 0; bq < KY; ++bq) {
              const T* row = sl + ((yl + bq) * ZW + zw + zb) * kElemCG + 2 * lane;
              float2 v[kS3ZU + KZ - 1];
#pragma unroll
              for (int m = 0; m < kS3ZU + KZ - 1; ++m) v[m] = s3_ld<T>(row + m * kElemCG);
#pragma unroll
              for (int e = 0; e < KZ; ++e) {
                const int j = (a * KY + bq) * KZ + e;
                const bool centre = a == ac && bq == bc && e == ec;  // (v indexed statically only)
#pragma unroll
                for (int i = 0; i < kS3ZU; ++i) {
                  acc[i] = ffma2(wr[j], v[i + e], acc[i]);
                  dacc[j] = ffma2(iv[i], v[i + e], dacc[j]);
                  if (centre) {
                    accb.x += v[i + e].x;
                    accb.y += v[i + e].y;
                  }
                }
              }
            }
          }
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) {
            const int gz = t.z0 + zw + zb + i;
            if (gz >= g.n[2]) {  // positions past the grid add nothing to the gradients either
              break;
            }
            const long long pos = ((long long)x * g.n[1] + gy) * g.n[2] + gz;
            V2<T>::store(dst + (long long)t.b * in_bst + pos * in_pst + c, acc[i]);
          }
        }
      }
      __syncthreads();  // the next prefetch overwrites the oldest plane read here
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
    // CTA reduction over the warps through the (now idle) ring; dacc[j] belongs to tap
    // flip(j), the bias sum to the last slot
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      red[(warp * (NT + 1) + j) * kElemCG + 2 * lane] = dacc[j].x;
      red[(warp * (NT + 1) + j) * kElemCG + 2 * lane + 1] = dacc[j].y;
    }
    red[(warp * (NT + 1) + NT) * kElemCG + 2 * lane] = accb.x;
    red[(warp * (NT + 1) + NT) * kElemCG + 2 * lane + 1] = accb.y;
    __syncthreads();
    for (int i = threadIdx.x; i < (NT + 1) * kElemCG; i += blockDim.x) {
      const int j = i / kElemCG, cc = i - j * kElemCG, ch = t.c0 + cc;
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < NW; ++q) sum += red[(q * (NT + 1) + j) * kElemCG + cc];
      if (ch < C) {
        if (j < NT) {
          const int a = j / (KY * KZ), bq = (j / KZ) % KY, e = j % KZ;
          const int tap = ((KX - 1 - a) * KY + (KY - 1 - bq)) * KZ + (KZ - 1 - e);
          atomicAdd(dw + ((long long)ti * C + ch) * NT + tap, sum);
        } else if (db) {
          atomicAdd(db + (long long)ti * C + ch, sum);
        }
      }
    }
    __syncthreads();  // the ring is refilled for the next tensor
  }
}

// Weight and bias gradients: dW[t][c][tap] = sum_{b, p} dout[b, p, c] * in[b, p + tap - off, c]
// with in = q/k/v (in_bst, in_pst) and dout = dq'/dk'/dv' contiguous; db[t][c] = sum dout.
// Per-thread accumulators for all taps, a shared-memory reduction over the CTA's warps,
// one atomic per channel and tap per CTA (dw, db zeroed by the host).
template <typename T, int KX, int KY, int KZ, int TY = kS3TY, int TZ = kS3TZ>
__global__ void __launch_bounds__(kElemThreads, (KX == 1 || KY == 1) ? 3 : 2) hyena_plane_wgrad_kernel(
    const T* __restrict__ d0, const T* __restrict__ d1, const T* __restrict__ d2, const T* __restrict__ in0,
    const T* __restrict__ in1, const T* __restrict__ in2, long long in_bst, long long in_pst, StencilGeom g, int C,
    float* __restrict__ dw, float* __restrict__ db, int xchunk) {
  constexpr int NT = KX * KY * KZ, ZW = TZ + KZ - 1, NPOS = s3_plane_positions<KY, KZ, TY, TZ>(), NB = s3_ring<KX>();
  constexpr int NW = kElemThreads / 32;
  constexpr int WPR = TZ / 16;  // warps per tile row, 16 z positions each
  static_assert(TY * WPR == NW, "one warp per 16 positions of the tile");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw);  // [NW][NT + 1][64] after the march
  const S3Tile t = s3_tile<TY, TZ>(g, xchunk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int yl = warp / WPR, zw = (warp % WPR) * 16;
  const int c = t.c0 + 2 * lane;
  const bool cok = c < C;
  const int ox = g.off[0], oy = g.off[1], oz = g.off[2];
  const long long N = (long long)g.n[0] * g.n[1] * g.n[2];
  const int gy = t.y0 + yl;
  const RowChunks<KZ, TZ> rows(g, t, C, in_pst, oz);  // used by one-row planes only
  auto load_plane = [&](T* slot, const T* src, int xin) {
    if constexpr (KY == 1 && TY == 1) rows.template load<T>(slot, src, in_bst, in_pst, g, t, xin);
    else s3_load_plane<T, KY, KZ, TY, TZ>(slot, src, in_bst, in_pst, g, t, C, xin, oy, oz);
  };

#pragma unroll 1
  for (int ti = 0; ti < 3; ++ti) {
    float2 acc[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j] = make_float2(0.f, 0.f);
    float2 accb = make_float2(0.f, 0.f);
    const T* src = ti == 0 ? in0 : (ti == 1 ? in1 : in2);
    const T* dsrc = ti == 0 ? d0 : (ti == 1 ? d1 : d2);
#pragma unroll 1
    for (int a = 0; a < KX; ++a) {
      const int xin = t.xa - ox + a;
      load_plane(ring + ((xin + 256) % NB) * NPOS * kElemCG, src, xin);
    }
#pragma unroll 1
    for (int x = t.xa; x < t.xb; ++x) {
      const bool pre = x + 1 < t.xb;
      if (pre) {
        const int xin = x - ox + KX;
        load_plane(ring + ((xin + 256) % NB) * NPOS * kElemCG, src, xin);
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      }
      __syncthreads();
      if (cok && gy < g.n[1]) {
        // dout of the next step is loaded one step ahead, behind the current step's taps
        auto ld_dout = [&](int zb, float2 (&dv)[kS3ZU]) {
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) {
            const int gz = t.z0 + zw + zb + i;
            const long long pos = ((long long)x * g.n[1] + gy) * g.n[2] + gz;
            dv[i] = (zb < 16 && gz < g.n[2]) ? V2<T>::load(dsrc + ((long long)t.b * N + pos) * C + c)
                                                    : make_float2(0.f, 0.f);
          }
        };
        float2 dnext[kS3ZU];
        ld_dout(0, dnext);
#pragma unroll 1
        for (int zb = 0; zb < 16; zb += kS3ZU) {
          float2 dv[kS3ZU];
#pragma unroll
          for (int i = 0; i < kS3ZU; ++i) {
            dv[i] = dnext[i];
            accb.x += dv[i].x;
            accb.y += dv[i].y;
          }
          ld_dout(zb + kS3ZU, dnext);
#pragma unroll
          for (int a = 0; a < KX; ++a) {
            const T* sl = ring + ((x - ox + a + 256) % NB) * NPOS * kElemCG;
#pragma unroll
            for (int bq = 0; bq < KY; ++bq) {
              const T* row = sl + ((yl + bq) * ZW + zw + zb) * kElemCG + 2 * lane;
              float2 v[kS3ZU + KZ - 1];
#pragma unroll
              for (int m = 0; m < kS3ZU + KZ - 1; ++m) v[m] = s3_ld<T>(row + m * kElemCG);
#pragma unroll
              for (int e = 0; e < KZ; ++e) {
                float2& ac = acc[(a * KY + bq) * KZ + e];
#pragma unroll
                for (int i = 0; i < kS3ZU; ++i) {
                  ac = ffma2(dv[i], v[i + e], ac);
                }
              }
            }
          }
        }
      }
      __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
    // CTA reduction over the warps through the (now idle) ring
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      red[(warp * (NT + 1) + j) * kElemCG + 2 * lane] = acc[j].x;
      red[(warp * (NT + 1) + j) * kElemCG + 2 * lane + 1] = acc[j].y;
    }
    red[(warp * (NT + 1) + NT) * kElemCG + 2 * lane] = accb.x;
    red[(warp * (NT + 1) + NT) * kElemCG + 2 * lane + 1] = accb.y;
    __syncthreads();
    for (int i = threadIdx.x; i < (NT + 1) * kElemCG; i += blockDim.x) {
      const int j = i / kElemCG, cc = i - j * kElemCG, ch = t.c0 + cc;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < NW; ++q) s += red[(q * (NT + 1) + j) * kElemCG + cc];
      if (ch < C) {
        if (j < NT) atomicAdd(dw + ((long long)ti * C + ch) * NT + j, s);
        else if (db) atomicAdd(db + (long long)ti * C + ch, s);
      }
    }
    __syncthreads();  // the ring is refilled for the next tensor
  }
}

}  // namespace hyfft
