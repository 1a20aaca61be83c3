// Tensor-core Hyena kernels for small 2D grids (both sides <= 16, bf16 I/O), e.g.
// the 14x14 ViT token grid: the long convolution runs on tcgen05 as a dense
// Toeplitz GEMM instead of an FFT.
//
// Why: for an N0 x N1 grid the "same" linear convolution with a (<= 2N-1)-tap
// filter is, per channel, the product of a (N0*N1) x (N0*N1) block-Toeplitz
// matrix T (blocks T1_d[c_out][c_in] = k[d + K0/2][c_out - c_in + K1/2], d = r_out -
// r_in) with the images of that channel. At 196 positions that is 77 kFLOP per
// image on the tensor cores (~2.25 PFLOP/s) versus ~30 kFLOP per image of
// pruned FFT on the fp32 pipes (~70 TFLOP/s), so the dense form is ~10x cheaper
// in time and leaves the kernel bound by HBM.
//
// Layout tricks:
//  * Columns are padded to a pitch of 16, so a 128-row M tile covers 8 grid rows
//    and one K step covers one input row. Every 128x16 A tile of T is then 8
//    consecutive 16x16 blocks T1_d, T1_{d+1}, ..., so all A tiles are sliding
//    windows (descriptor start address + 512 B per block) into one buffer of
//    N0-1+16 blocks per channel (~15 KB), never a materialised N^2 matrix.
//  * The D-skip is folded into the filter's centre tap (h = conv(z, k + D*delta)),
//    so the GEMM produces h directly and dD is the centre tap of the filter
//    gradient.
//  * z and dh live in one shared-memory layout per row [c/8][img/8][img%8][c%8]
//    that is a K-major operand (N = images, K = columns) for the convolution GEMMs
//    and an MN-major operand (M/N = positions, K = images) for the filter-gradient
//    GEMM G = DH * Z^T.
//
// Forward (per CTA: CG channels x NB images): depthwise 3x3 short conv + gate 1
// from channels-last q, k (16-byte vectors read in place from the projection
// output) -> z; per channel: Toeplitz blocks -> tcgen05.mma into TMEM; epilogue:
// gate 2 with v' -> y (channels-last vector stores).
// Backward: z and dh -> SMEM; per channel H = T z, DZ = T^T dh (TMEM); gate
// backward -> dq', dk', dv' (SMEM); per channel G = DH Z^T (TMEM, 448 columns),
// reduced along its Toeplitz diagonals into dK; transposed short conv -> dq, dk,
// dv; weight / bias gradient reductions.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <atomic>

#include "common.cuh"
#include "fused2d.h"
#include "umma.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;

namespace tp {

using bf16 = __nv_bfloat16;

template <int CG>
struct VG;
template <>
struct VG<8> {
  static __device__ __forceinline__ void load(const bf16* p, float (&o)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(bf16* p, const float (&o)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct VG<4> {
  static __device__ __forceinline__ void load(const bf16* p, float (&o)[4]) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(bf16* p, const float (&o)[4]) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 2; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    *reinterpret_cast<uint2*>(p) = u;
  }
  // shared-memory variants (plain loads)
  static __device__ __forceinline__ void lds(const bf16* p, float (&o)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
};

__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Depthwise SKxSK "same" cross-correlation of CG channels at (n0, n1) of one image,
// read from global memory (channels-last, position stride pst, channel offset applied).
template <int N0, int N1, int SK, int CG>
__device__ __forceinline__ void gstencil(const bf16* img, long long pst, const float* w, const float* bias, int n0,
                                         int n1, float (&o)[CG]) {
  if constexpr (SK == 0) {
    VG<CG>::load(img + (long long)(n0 * N1 + n1) * pst, o);
  } else {
    constexpr int OFF = (SK - 1) / 2, NT = SK * SK;
#pragma unroll
    for (int c = 0; c < CG; ++c) o[c] = bias ? bias[c] : 0.f;
#pragma unroll
    for (int a = 0; a < SK; ++a) {
      const int i0 = n0 + a - OFF;
      if (i0 < 0 || i0 >= N0) continue;
#pragma unroll
      for (int b = 0; b < SK; ++b) {
        const int i1 = n1 + b - OFF;
        if (i1 < 0 || i1 >= N1) continue;
        float x[CG];
        VG<CG>::load(img + (long long)(i0 * N1 + i1) * pst, x);
#pragma unroll
        for (int c = 0; c < CG; ++c) o[c] = fmaf(w[c * NT + a * SK + b], x[c], o[c]);
      }
    }
  }
}

template <int N0>
struct Geo {
  static constexpr int MT = (N0 + 7) / 8;        // 128-row M tiles (8 grid rows each)
  static constexpr int NR = 8 * MT;              // grid rows incl. padding rows
  static constexpr int NBLK = (N0 - 1) + 8 * MT;  // 16x16 Toeplitz blocks per table
  static constexpr int BLKB = 512;               // bytes per block
};

// Fill one table of Toeplitz blocks for a channel (all threads). Block b holds, for
// d = b - (N0 - 1):  forward  T1_d[m = c_out][k = c_in]  = k'[d + K0/2][c_out - c_in + K1/2]
//                    adjoint  U_d[m = c_in][k = c_out]   = k'[K0/2 - d][c_out - c_in + K1/2]
// with k' = k + D at the centre tap; stored K-major [m/8][k/8][m%8][k%8] (bf16).
// f: the channel's K0 x K1 taps (shared memory).
template <int N0, int N1, bool ADJ>
__device__ __forceinline__ void gen_blocks(unsigned char* dst, const float* f, int K0, int K1, float Dc) {
  constexpr int NBLK = Geo<N0>::NBLK;
  const int ck0 = K0 / 2, ck1 = K1 / 2;
  for (int it = threadIdx.x; it < NBLK * 32; it += blockDim.x) {
    const int b = it >> 5, m = (it >> 1) & 15, kc = it & 1;
    const int d = b - (N0 - 1);
    const int row = ADJ ? ck0 - d : d + ck0;
    const bool row_ok = row >= 0 && row < K0 && m < N1;
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float v2[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int k = kc * 8 + e + u;
        const int co = ADJ ? k : m, ci = ADJ ? m : k;
        const int col = co - ci + ck1;
        float val = 0.f;
        if (row_ok && k < N1 && col >= 0 && col < K1) {
          val = f[row * K1 + col];
          if (row == ck0 && col == ck1) val += Dc;
        }
        v2[u] = val;
      }
      const __nv_bfloat162 h = __floats2bfloat162_rn(v2[0], v2[1]);
      pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(dst + b * 512 + (m >> 3) * 256 + kc * 128 + (m & 7) * 16) =
        make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int n) {
  return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}

// offset (bytes) of (image, grid position (r, c)) in the z / dh operand layout of a channel
template <int NB>
__device__ __forceinline__ int zoff(int img, int r, int c) {
  return r * (32 * NB) + (c >> 3) * (16 * NB) + (img >> 3) * 128 + (img & 7) * 16 + (c & 7) * 2;
}

__device__ __forceinline__ void set_status(int* st) {
  if (st) atomicExch(st, 1);
}

// ------------------------------------------------------------------ shared-memory helpers
template <int CG>
struct VS;
template <>
struct VS<4> {
  using Raw = uint2;
  static __device__ __forceinline__ void load(const bf16* p, float (&o)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
  static __device__ __forceinline__ void store(bf16* p, const float (&o)[4]) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(o[0], o[1]);
    h[1] = __floats2bfloat162_rn(o[2], o[3]);
    *reinterpret_cast<uint2*>(p) = u;
  }
};
template <>
struct VS<8> {
  using Raw = uint4;
  static __device__ __forceinline__ void load(const bf16* p, float (&o)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(bf16* p, const float (&o)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};

// cp.async copy of one position's CG channels (8 or 16 bytes) from global to shared
// memory, left in flight; !valid zero-fills and reads nothing.
template <int CG>
__device__ __forceinline__ void cp_async_vec(void* sdst, const void* gsrc, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(sdst);
  if constexpr (CG * 2 == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc), "r"(valid ? 16 : 0)
                 : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(gsrc), "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_f32(float* sdst, const float* gsrc) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(sdst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Up to four channels-last bf16 sources with their batch / position strides (channel
// offset already applied).
struct TileSrc {
  const bf16* p[4];
  long long bst[4], pst[4];
};

// Stage CG channels of NT_ tensors x HB images x NP positions (channels-last global, one
// vector per position) into shared memory [tensor][image][position][CG] with cp.async:
// every copy of the stage is in flight at once (one commit group; the caller waits);
// zeros past B.
template <int NP, int CG, int HB, int NT_>
__device__ __forceinline__ void stage_async(bf16* R, const TileSrc& s, int b_first, int B) {
#pragma unroll
  for (int t = 0; t < NT_; ++t) {
    for (int i = threadIdx.x; i < HB * NP; i += blockDim.x) {
      const int j = i / NP, pos = i - j * NP;
      const int b = b_first + j;
      const bool ok = b < B;
      const bf16* src = s.p[t] + (ok ? (long long)b * s.bst[t] + (long long)pos * s.pst[t] : 0LL);
      cp_async_vec<CG>(R + ((long long)(t * HB + j) * NP + pos) * CG, src, ok);
    }
  }
  cp_async_commit();
}

// The CTA's CG channels of the filter, [CG][K0 * K1] float, into shared memory (cp.async,
// committed with the next stage).
__device__ __forceinline__ void stage_filter_async(float* fsm, const float* filt, int c0, int CG, int KK) {
  const float* src = filt + (long long)c0 * KK;
  for (int i = threadIdx.x; i < CG * KK; i += blockDim.x) cp_async_f32(fsm + i, src + i);
}

// Depthwise SKxSK "same" cross-correlation of CG channels at (n0, n1) of a staged
// image tile [NP][CG] (bf16, shared memory). SK == 0: identity.
template <int N0, int N1, int SK, int CG>
__device__ __forceinline__ void sstencil(const bf16* tile, const float* w, const float* bias, int n0, int n1,
                                         float (&o)[CG]) {
  if constexpr (SK == 0) {
    VS<CG>::load(tile + (n0 * N1 + n1) * CG, o);
  } else {
    constexpr int OFF = (SK - 1) / 2, NT = SK * SK;
#pragma unroll
    for (int c = 0; c < CG; ++c) o[c] = bias ? bias[c] : 0.f;
#pragma unroll
    for (int a = 0; a < SK; ++a) {
      const int i0 = n0 + a - OFF;
      if (i0 < 0 || i0 >= N0) continue;
#pragma unroll
      for (int b = 0; b < SK; ++b) {
        const int i1 = n1 + b - OFF;
        if (i1 < 0 || i1 >= N1) continue;
        float x[CG];
        VS<CG>::load(tile + (i0 * N1 + i1) * CG, x);
#pragma unroll
        for (int c = 0; c < CG; ++c) o[c] = fmaf(w[c * NT + a * SK + b], x[c], o[c]);
      }
    }
  }
}

// ------------------------------------------------------------------ forward
template <int N0, int N1, int SK, int CG, int NB>
struct FwdLayout {
  using G = Geo<N0>;
  static constexpr int NT = SK > 0 ? SK * SK : 1;
  static constexpr int RB = 32 * NB, HB = 8, NP = N0 * N1;
  static constexpr size_t z = 0;
  static constexpr size_t r = z + (size_t)CG * G::NR * RB;                     // [3][HB][NP][CG] bf16
  static constexpr size_t rsz = ((size_t)3 * HB * NP * CG * 2 + 127) / 128 * 128;
  static constexpr size_t tsz = 2 * (size_t)G::NBLK * G::BLKB;                // block tables (alias r)
  static constexpr size_t t = r;
  static constexpr size_t w = r + (rsz > tsz ? rsz : tsz);
  static constexpr size_t bar = w + ((4 * (3 * CG * NT + 3 * CG + CG) + 15) / 16) * 16;
  static constexpr size_t fk = bar + 32;  // [CG][K0 * K1] filter taps (size set at launch)
  static constexpr uint32_t tcols = tmem_cols_for(CG * G::MT * NB);
  static size_t bytes(int K0, int K1) { return fk + ((size_t)CG * K0 * K1 * 4 + 15) / 16 * 16; }
};

// Forward, per CTA CG channels x NB images (two CTAs per SM):
//  1. cp.async: the CTA's filter taps and q, k of the first 8 images; while they fly, the
//     z operand is cleared and the short-conv weights loaded;
//  2. per 8 images: short conv + gate 1 -> z (operand layout), v' (bf16) kept in v_s for
//     the epilogue... computed there from the staged v instead (re-staged by cp.async);
//  3. per channel: Toeplitz blocks from the shared-memory filter (double-buffered tables,
//     aliasing the staging area) and tcgen05 MMAs into TMEM;
//  4. epilogue per 8 images: v staged by cp.async, y = round(h) * round(g2(v')).
template <int N0, int N1, int SK, int CG, int NB>
__global__ void __launch_bounds__(256, 2) tp2d_fwd_kernel(const Fused2DParams p) {
  using G = Geo<N0>;
  using L = FwdLayout<N0, N1, SK, CG, NB>;
  constexpr int MT = G::MT, NR = G::NR, RB = L::RB, NT = L::NT, NP = L::NP, HB = L::HB;
  constexpr uint32_t IDESC = umma::idesc_bf16(128, NB, 0, 0);
  static_assert(MT <= 2, "8 warps cover at most two 128-row tiles");
  static_assert(NB % HB == 0 && HB == 8, "images are staged 8 at a time");
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* Zt = smem + L::z;
  bf16* R = reinterpret_cast<bf16*>(smem + L::r);
  unsigned char* Tb = smem + L::t;
  float* wts = reinterpret_cast<float*>(smem + L::w);
  float* bsm = wts + 3 * CG * NT;
  float* Dsm = bsm + 3 * CG;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + L::bar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::bar + 16);
  float* fsm = reinterpret_cast<float*>(smem + L::fk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = blockIdx.x * CG, b0 = blockIdx.y * NB;
  const int KK = p.K0 * p.K1;

  TileSrc src;
  src.p[0] = reinterpret_cast<const bf16*>(p.q) + c0;
  src.p[1] = reinterpret_cast<const bf16*>(p.k) + c0;
  src.p[2] = reinterpret_cast<const bf16*>(p.v) + c0;
  src.p[3] = src.p[0];
  for (int i = 0; i < 4; ++i) {
    src.bst[i] = p.in_bst;
    src.pst[i] = p.in_pst;
  }
  TileSrc vsrc = src;
  vsrc.p[0] = src.p[2];
  stage_filter_async(fsm, p.filt, c0, CG, KK);
  stage_async<NP, CG, HB, 2>(R, src, b0, p.B);  // q, k of the first images (with the filter)

  if (warp == 0) umma::tmem_alloc(tslot, L::tcols);
  if (tid == 0) {
    umma::mbar_init(&mbar[0], 1);
    umma::mbar_init(&mbar[1], 1);
    umma::fence_mbar_init();
  }
  for (int i = tid; i < 3 * CG * NT; i += blockDim.x) {
    const int t = i / (CG * NT), r = i % (CG * NT), cc = r / NT, tap = r % NT;
    wts[i] = SK > 0 ? p.w[((long long)t * p.C + c0 + cc) * NT + tap] : 1.f;
  }
  for (int i = tid; i < 3 * CG; i += blockDim.x) bsm[i] = p.bias ? p.bias[(i / CG) * p.C + c0 + i % CG] : 0.f;
  for (int i = tid; i < CG; i += blockDim.x) Dsm[i] = p.D[c0 + i];
  for (int i = tid; i < CG * NR * RB / 16; i += blockDim.x) reinterpret_cast<uint4*>(Zt)[i] = make_uint4(0, 0, 0, 0);

  const float* bq = p.bias ? bsm : nullptr;
  const float* bk = p.bias ? bsm + CG : nullptr;
  const float* bv = p.bias ? bsm + 2 * CG : nullptr;

  // ---- z = q' * g1(k') into the operand layout, 8 staged images at a time
  for (int h0 = 0; h0 < NB; h0 += HB) {
    if (h0 > 0) {
      __syncthreads();  // the previous images' stencils are done with R
      stage_async<NP, CG, HB, 2>(R, src, b0 + h0, p.B);
    }
    cp_async_wait_all();
    __syncthreads();
    for (int it = tid; it < HB * NP; it += blockDim.x) {
      const int j = it / NP, pos = it - j * NP, r = pos / N1, c = pos - r * N1;
      if (b0 + h0 + j >= p.B) continue;
      float qv[CG], kv[CG];
      sstencil<N0, N1, SK, CG>(R + (long long)j * NP * CG, wts, bq, r, c, qv);
      sstencil<N0, N1, SK, CG>(R + (long long)(HB + j) * NP * CG, wts + CG * NT, bk, r, c, kv);
      const int off = zoff<NB>(h0 + j, r, c);
#pragma unroll
      for (int ch = 0; ch < CG; ++ch) {
        const float z = rbf(rbf(qv[ch]) * rbf(gate_f(p.gate1, rbf(kv[ch]))));
        *reinterpret_cast<bf16*>(Zt + ch * NR * RB + off) = __float2bfloat16_rn(z);
      }
    }
  }
  umma::fence_async_smem();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;

  // ---- per channel: Toeplitz blocks + MMAs (double-buffered block tables over the staging area)
  bool ok = true;
  for (int ch = 0; ch < CG; ++ch) {
    const int buf = ch & 1;
    if (ch >= 2) ok &= umma::mbar_wait(&mbar[buf], ((ch - 2) >> 1) & 1);
    unsigned char* tb = Tb + buf * G::NBLK * G::BLKB;
    gen_blocks<N0, N1, false>(tb, fsm + ch * KK, p.K0, p.K1, Dsm[ch]);
    umma::fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      umma::fence_after_sync();
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        for (int ri = 0; ri < N0; ++ri) {
          const uint64_t da = umma::sdesc(umma::su32(tb + (8 * mt - ri + N0 - 1) * G::BLKB), 128, 256);
          const uint64_t db = umma::sdesc(umma::su32(Zt + ch * NR * RB + ri * RB), 16 * NB, 128);
          umma::mma(tmem + (uint32_t)((ch * MT + mt) * NB), da, db, IDESC, ri > 0 ? 1u : 0u);
        }
      }
      umma::commit(&mbar[buf]);
    }
  }
  // the staging area holds the block tables until every MMA has read them
  if (CG >= 2) ok &= umma::mbar_wait(&mbar[(CG - 2) & 1], ((CG - 2) >> 1) & 1);
  ok &= umma::mbar_wait(&mbar[(CG - 1) & 1], ((CG - 1) >> 1) & 1);
  umma::fence_after_sync();

  // ---- epilogue: y = round(h) * round(g2(v')), v staged 8 images at a time
  const int mt = warp >> 2, q4 = warp & 3;
  const int m = q4 * 32 + lane, r = mt * 8 + (m >> 4), c = m & 15;
  bf16* y = reinterpret_cast<bf16*>(p.y) + c0;
  const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
  for (int h0 = 0; h0 < NB; h0 += HB) {
    __syncthreads();
    stage_async<NP, CG, HB, 1>(R, vsrc, b0 + h0, p.B);
    cp_async_wait_all();
    __syncthreads();
    if (mt < MT) {
      const bool valid = ok && r < N0 && c < N1;
      float h[CG][8];
#pragma unroll
      for (int ch = 0; ch < CG; ++ch) umma::tmem_ld8(lane_base + (uint32_t)((ch * MT + mt) * NB + h0), h[ch]);
      if (valid) {
#pragma unroll
        for (int j = 0; j < HB; ++j) {
          const int b = b0 + h0 + j;
          if (b >= p.B) break;
          float vv[CG], out[CG];
          sstencil<N0, N1, SK, CG>(R + (long long)j * NP * CG, wts + 2 * CG * NT, bv, r, c, vv);
#pragma unroll
          for (int ch = 0; ch < CG; ++ch) out[ch] = rbf(h[ch][j]) * rbf(gate_f(p.gate2, rbf(vv[ch])));
          VG<CG>::store(y + (long long)b * p.out_bst + (long long)(r * N1 + c) * p.out_pst, out);
        }
      }
    }
  }
  if (!ok && tid == 0) set_status(p.status);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, L::tcols);
}

// ------------------------------------------------------------------ backward
template <int N0, int N1, int SK, int CG, int NB>
struct BwdLayout {
  using G = Geo<N0>;
  static constexpr int NT = SK > 0 ? SK * SK : 1;
  static constexpr int RB = 32 * NB, HB = 8, NP = N0 * N1;
  static constexpr size_t z = 0;
  static constexpr size_t dh = z + (size_t)CG * G::NR * RB;
  static constexpr size_t rsz = ((size_t)4 * HB * NP * CG * 2 + 127) / 128 * 128;
  static constexpr size_t tsz = 2 * (size_t)G::NBLK * G::BLKB;  // forward + adjoint tables (aliased with R)
  static constexpr size_t r = dh + (size_t)CG * G::NR * RB;      // [4][HB][NP][CG] bf16
  static constexpr size_t ds = r + (rsz > tsz ? rsz : tsz);       // [3][HB][NP][CG] bf16
  static constexpr size_t w = ds + ((size_t)3 * HB * NP * CG * 2 + 15) / 16 * 16;
  static constexpr size_t dw = w + ((4 * (3 * CG * NT + 3 * CG + CG) + 15) / 16) * 16;  // [3][CG][NT+1]
  static constexpr size_t bar = dw + ((4 * 3 * CG * (NT + 1) + 15) / 16) * 16;
  static constexpr size_t dk = bar + 48;  // [CG][K0][kpitch(K1)] dK accumulators, then [CG][K0*K1] filter
  // dK row pitch: 16 or 48 floats, so the two grid rows a warp covers land in disjoint banks
  static __host__ __device__ int kpitch(int K1) { return K1 <= 16 ? 16 : 48; }
  static __host__ __device__ size_t fk(int K0, int K1) { return dk + (size_t)CG * K0 * kpitch(K1) * 4; }
  static size_t bytes(int K0, int K1) { return fk(K0, K1) + ((size_t)CG * K0 * K1 * 4 + 15) / 16 * 16; }
};

template <int N0, int N1, int SK, int CG, int NB>
__global__ void __launch_bounds__(256) tp2d_bwd_kernel(const Fused2DParams p) {
  using G = Geo<N0>;
  using L = BwdLayout<N0, N1, SK, CG, NB>;
  constexpr int MT = G::MT, NR = G::NR, RB = L::RB, NT = L::NT, NP = L::NP, HB = L::HB;
  constexpr uint32_t IDESC = umma::idesc_bf16(128, NB, 0, 0);
  constexpr uint32_t IDESC_G = umma::idesc_bf16(128, 16 * N0, 1, 1);
  constexpr uint32_t TCOLS = 512;
  static_assert(MT <= 2, "8 warps cover at most two 128-row tiles");
  static_assert(2 * CG * MT * NB <= 512 && MT * 16 * N0 <= 512, "TMEM budget");
  static_assert(NB == 16, "the filter-gradient GEMM uses one K step of 16 images");
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* Zt = smem + L::z;
  unsigned char* DHt = smem + L::dh;
  bf16* R = reinterpret_cast<bf16*>(smem + L::r);
  unsigned char* Tf = smem + L::r;  // block tables alias the staging area (phase 2 only)
  unsigned char* Tt = Tf + G::NBLK * G::BLKB;
  bf16* ds = reinterpret_cast<bf16*>(smem + L::ds);
  float* dkacc = reinterpret_cast<float*>(smem + L::dk);
  float* wts = reinterpret_cast<float*>(smem + L::w);
  float* bsm = wts + 3 * CG * NT;
  float* Dsm = bsm + 3 * CG;
  float* dwacc = reinterpret_cast<float*>(smem + L::dw);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + L::bar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::bar + 32);
  float* fsm = reinterpret_cast<float*>(smem + L::fk(p.K0, p.K1));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = blockIdx.x * CG, b0 = blockIdx.y * NB;
  const int ck0 = p.K0 / 2, ck1 = p.K1 / 2;
  const int KK = p.K0 * p.K1, KP = L::kpitch(p.K1);

  TileSrc src;
  src.p[0] = reinterpret_cast<const bf16*>(p.q) + c0;
  src.p[1] = reinterpret_cast<const bf16*>(p.k) + c0;
  src.p[2] = reinterpret_cast<const bf16*>(p.v) + c0;
  src.p[3] = reinterpret_cast<const bf16*>(p.dy) + c0;
  src.bst[0] = src.bst[1] = src.bst[2] = p.in_bst;
  src.pst[0] = src.pst[1] = src.pst[2] = p.in_pst;
  src.bst[3] = p.out_bst;
  src.pst[3] = p.out_pst;
  stage_filter_async(fsm, p.filt, c0, CG, KK);
  stage_async<NP, CG, HB, 4>(R, src, b0, p.B);  // q, k, v, dy of the first images (with the filter)

  if (warp == 0) umma::tmem_alloc(tslot, TCOLS);
  if (tid == 0) {
    umma::mbar_init(&mbar[0], 1);
    umma::mbar_init(&mbar[1], 1);
    umma::fence_mbar_init();
  }
  for (int i = tid; i < 3 * CG * NT; i += blockDim.x) {
    const int t = i / (CG * NT), r = i % (CG * NT), cc = r / NT, tap = r % NT;
    wts[i] = SK > 0 ? p.w[((long long)t * p.C + c0 + cc) * NT + tap] : 1.f;
  }
  for (int i = tid; i < 3 * CG; i += blockDim.x) bsm[i] = p.bias ? p.bias[(i / CG) * p.C + c0 + i % CG] : 0.f;
  for (int i = tid; i < CG; i += blockDim.x) Dsm[i] = p.D[c0 + i];
  for (int i = tid; i < 2 * CG * NR * RB / 16; i += blockDim.x) reinterpret_cast<uint4*>(Zt)[i] = make_uint4(0, 0, 0, 0);
  for (int i = tid; i < CG * p.K0 * KP; i += blockDim.x) dkacc[i] = 0.f;
  for (int i = tid; i < 3 * CG * (NT + 1); i += blockDim.x) dwacc[i] = 0.f;

  const float* bias3[3] = {p.bias ? bsm : nullptr, p.bias ? bsm + CG : nullptr, p.bias ? bsm + 2 * CG : nullptr};

  // ---- z and dh into the operand layouts, 8 staged images at a time
  for (int h0 = 0; h0 < NB; h0 += HB) {
    if (h0 > 0) {
      __syncthreads();  // the previous images' stencils are done with R
      stage_async<NP, CG, HB, 4>(R, src, b0 + h0, p.B);
    }
    cp_async_wait_all();
    __syncthreads();
    for (int it = tid; it < HB * NP; it += blockDim.x) {
      const int j = it / NP, pos = it - j * NP, r = pos / N1, c = pos - r * N1;
      if (b0 + h0 + j >= p.B) continue;
      float qv[CG], kv[CG], vv[CG], g[CG];
      sstencil<N0, N1, SK, CG>(R + (long long)(0 * HB + j) * NP * CG, wts, bias3[0], r, c, qv);
      sstencil<N0, N1, SK, CG>(R + (long long)(1 * HB + j) * NP * CG, wts + CG * NT, bias3[1], r, c, kv);
      sstencil<N0, N1, SK, CG>(R + (long long)(2 * HB + j) * NP * CG, wts + 2 * CG * NT, bias3[2], r, c, vv);
      VS<CG>::load(R + ((long long)(3 * HB + j) * NP + pos) * CG, g);
      const int off = zoff<NB>(h0 + j, r, c);
#pragma unroll
      for (int ch = 0; ch < CG; ++ch) {
        const float z = rbf(rbf(qv[ch]) * rbf(gate_f(p.gate1, rbf(kv[ch]))));
        const float dh = rbf(g[ch] * rbf(gate_f(p.gate2, rbf(vv[ch]))));
        *reinterpret_cast<bf16*>(Zt + ch * NR * RB + off) = __float2bfloat16_rn(z);
        *reinterpret_cast<bf16*>(DHt + ch * NR * RB + off) = __float2bfloat16_rn(dh);
      }
    }
  }
  __syncthreads();
  const uint32_t tmem = *tslot;
  const uint32_t DZ0 = (uint32_t)(CG * MT * NB);

  // ---- per channel: H = T z and DZ = T^T dh (one pair of block tables, reused per channel)
  bool ok = true;
  for (int ch = 0; ch < CG; ++ch) {
    if (ch >= 1) ok &= umma::mbar_wait(&mbar[0], (ch - 1) & 1);
    const float* fch = fsm + ch * KK;
    gen_blocks<N0, N1, false>(Tf, fch, p.K0, p.K1, Dsm[ch]);
    gen_blocks<N0, N1, true>(Tt, fch, p.K0, p.K1, Dsm[ch]);
    umma::fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      umma::fence_after_sync();
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        for (int s = 0; s < N0; ++s) {
          const uint32_t blk = (uint32_t)((8 * mt - s + N0 - 1) * G::BLKB);
          const uint64_t dz = umma::sdesc(umma::su32(Zt + ch * NR * RB + s * RB), 16 * NB, 128);
          const uint64_t dd = umma::sdesc(umma::su32(DHt + ch * NR * RB + s * RB), 16 * NB, 128);
          umma::mma(tmem + (uint32_t)((ch * MT + mt) * NB), umma::sdesc(umma::su32(Tf) + blk, 128, 256), dz, IDESC,
                    s > 0 ? 1u : 0u);
          umma::mma(tmem + DZ0 + (uint32_t)((ch * MT + mt) * NB), umma::sdesc(umma::su32(Tt) + blk, 128, 256), dd,
                    IDESC, s > 0 ? 1u : 0u);
        }
      }
      umma::commit(&mbar[0]);
    }
  }
  ok &= umma::mbar_wait(&mbar[0], (CG - 1) & 1);
  umma::fence_after_sync();

  // ---- gate backward + transposed short conv + weight gradients, 8 staged images at a time
  const int mt = warp >> 2, q4 = warp & 3;
  const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
  bf16* outs[3] = {reinterpret_cast<bf16*>(p.dq) + c0, reinterpret_cast<bf16*>(p.dk) + c0,
                   reinterpret_cast<bf16*>(p.dv) + c0};
  constexpr int OFF = SK > 0 ? (SK - 1) / 2 : 0;
  for (int h0 = 0; h0 < NB; h0 += HB) {
    __syncthreads();
    stage_async<NP, CG, HB, 4>(R, src, b0 + h0, p.B);
    cp_async_wait_all();
    __syncthreads();
    umma::fence_after_sync();
    if (mt < MT) {
      const int m = q4 * 32 + lane, r = mt * 8 + (m >> 4), c = m & 15;
      const bool valid = ok && r < N0 && c < N1;
      const int pos = r * N1 + c;
      float hacc[CG][8], dacc[CG][8];
#pragma unroll
      for (int ch = 0; ch < CG; ++ch) {
        umma::tmem_ld8(lane_base + (uint32_t)((ch * MT + mt) * NB + h0), hacc[ch]);
        umma::tmem_ld8(lane_base + DZ0 + (uint32_t)((ch * MT + mt) * NB + h0), dacc[ch]);
      }
      if (valid) {
#pragma unroll
        for (int j = 0; j < HB; ++j) {
          if (b0 + h0 + j >= p.B) break;
          float qv[CG], kv[CG], vv[CG], g[CG], oq[CG], ok_[CG], ov[CG];
          sstencil<N0, N1, SK, CG>(R + (long long)(0 * HB + j) * NP * CG, wts, bias3[0], r, c, qv);
          sstencil<N0, N1, SK, CG>(R + (long long)(1 * HB + j) * NP * CG, wts + CG * NT, bias3[1], r, c, kv);
          sstencil<N0, N1, SK, CG>(R + (long long)(2 * HB + j) * NP * CG, wts + 2 * CG * NT, bias3[2], r, c, vv);
          VS<CG>::load(R + ((long long)(3 * HB + j) * NP + pos) * CG, g);
#pragma unroll
          for (int ch = 0; ch < CG; ++ch) {
            const float qr = rbf(qv[ch]), kr = rbf(kv[ch]), vr = rbf(vv[ch]);
            const float hv = rbf(hacc[ch][j]);
            const float dz = rbf(dacc[ch][j]);
            ov[ch] = g[ch] * hv * gate_df(p.gate2, vr);
            oq[ch] = dz * rbf(gate_f(p.gate1, kr));
            ok_[ch] = dz * qr * gate_df(p.gate1, kr);
          }
          bf16* dsi = ds + ((long long)j * NP + pos) * CG;
          VS<CG>::store(dsi, oq);
          VS<CG>::store(dsi + (long long)HB * NP * CG, ok_);
          VS<CG>::store(dsi + 2LL * HB * NP * CG, ov);
        }
      }
    }
    __syncthreads();
#pragma unroll 1
    for (int t = 0; t < 3; ++t) {
      float wacc[CG][NT + 1];
#pragma unroll
      for (int ch = 0; ch < CG; ++ch)
#pragma unroll
        for (int u = 0; u <= NT; ++u) wacc[ch][u] = 0.f;
      const float* wt = wts + t * CG * NT;
      for (int it = tid; it < HB * NP; it += blockDim.x) {
        const int j = it / NP, pos = it - j * NP, r = pos / N1, c = pos - r * N1;
        const int b = b0 + h0 + j;
        if (b >= p.B) continue;
        const bf16* dimg = ds + (long long)(t * HB + j) * NP * CG;
        float o[CG];
        if constexpr (SK == 0) {
          VS<CG>::load(dimg + pos * CG, o);
        } else {
#pragma unroll
          for (int ch = 0; ch < CG; ++ch) o[ch] = 0.f;
#pragma unroll
          for (int a = 0; a < SK; ++a) {
            const int i0 = r - a + OFF;
            if (i0 < 0 || i0 >= N0) continue;
#pragma unroll
            for (int bq = 0; bq < SK; ++bq) {
              const int i1 = c - bq + OFF;
              if (i1 < 0 || i1 >= N1) continue;
              float x[CG];
              VS<CG>::load(dimg + (i0 * N1 + i1) * CG, x);
#pragma unroll
              for (int ch = 0; ch < CG; ++ch) o[ch] = fmaf(wt[ch * NT + a * SK + bq], x[ch], o[ch]);
            }
          }
          float d0[CG];
          VS<CG>::load(dimg + pos * CG, d0);
          const bf16* inimg = R + (long long)(t * HB + j) * NP * CG;
#pragma unroll
          for (int a = 0; a < SK; ++a) {
            const int i0 = r + a - OFF;
            if (i0 < 0 || i0 >= N0) continue;
#pragma unroll
            for (int bq = 0; bq < SK; ++bq) {
              const int i1 = c + bq - OFF;
              if (i1 < 0 || i1 >= N1) continue;
              float x[CG];
              VS<CG>::load(inimg + (i0 * N1 + i1) * CG, x);
#pragma unroll
              for (int ch = 0; ch < CG; ++ch) wacc[ch][a * SK + bq] = fmaf(d0[ch], x[ch], wacc[ch][a * SK + bq]);
            }
          }
#pragma unroll
          for (int ch = 0; ch < CG; ++ch) wacc[ch][NT] += d0[ch];
        }
        VG<CG>::store(outs[t] + (long long)b * p.in_bst + (long long)pos * p.in_pst, o);  // dq, dk, dv mirror q, k, v
      }
      if constexpr (SK > 0) {
#pragma unroll
        for (int ch = 0; ch < CG; ++ch)
#pragma unroll
          for (int u = 0; u <= NT; ++u) {
            float s = wacc[ch][u];
            for (int o2 = 16; o2 > 0; o2 >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o2);
            if (lane == 0) atomicAdd(dwacc + (t * CG + ch) * (NT + 1) + u, s);
          }
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();

  // ---- per channel: G = DH Z^T (positions x positions), reduced along Toeplitz diagonals
  for (int ch = 0; ch < CG; ++ch) {
    if (tid == 0) {
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const uint64_t da = umma::sdesc(umma::su32(DHt + ch * NR * RB + t * 8 * RB), 128, 16 * NB);
        const uint64_t db = umma::sdesc(umma::su32(Zt + ch * NR * RB), 128, 16 * NB);
        umma::mma(tmem + (uint32_t)(t * 16 * N0), da, db, IDESC_G, 0u);
      }
      umma::commit(&mbar[1]);
    }
    ok &= umma::mbar_wait(&mbar[1], ch & 1);
    umma::fence_after_sync();
    if (mt < MT) {
      const int m = q4 * 32 + lane, ro = mt * 8 + (m >> 4), co = m & 15;
      const bool valid = ok && ro < N0 && co < N1;
      float* acc = dkacc + ch * p.K0 * KP;
#pragma unroll 1
      for (int ri = 0; ri < N0; ++ri) {
        float gv[16];
        umma::tmem_ld16(lane_base + (uint32_t)(mt * 16 * N0 + ri * 16), gv);
        const int a = ro - ri + ck0;
        if (!valid || a < 0 || a >= p.K0) continue;
#pragma unroll
        for (int ci = 0; ci < N1; ++ci) {
          const int bb = co - ci + ck1;
          if (bb >= 0 && bb < p.K1) atomicAdd(acc + a * KP + bb, gv[ci]);
        }
      }
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
  }
  if (!ok && tid == 0) set_status(p.status);
  if constexpr (SK > 0) {
    for (int i = tid; i < 3 * CG * (NT + 1); i += blockDim.x) {
      const int t = i / (CG * (NT + 1)), rr = i % (CG * (NT + 1)), ch = rr / (NT + 1), u = rr % (NT + 1);
      const long long chg = (long long)t * p.C + c0 + ch;
      if (u < NT) atomicAdd(p.dw + chg * NT + u, dwacc[i]);
      else if (p.db) atomicAdd(p.db + chg, dwacc[i]);
    }
  }
  // filter gradient (of k' = k + D*delta): dfilt = dk', dD = dk' at the centre tap
  for (int i = tid; i < CG * p.K0 * p.K1; i += blockDim.x) {
    const int ch = i / (p.K0 * p.K1), rr = i % (p.K0 * p.K1), a = rr / p.K1, bb = rr % p.K1;
    const float v = dkacc[(ch * p.K0 + a) * KP + bb];
    atomicAdd(p.dfilt + ((long long)(c0 + ch) * p.K0 + a) * p.K1 + bb, v);
    if (a == ck0 && bb == ck1) atomicAdd(p.dD + c0 + ch, v);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, TCOLS);
}

// ------------------------------------------------------------------ dispatch
constexpr int kFwdCG = 4, kBwdCG = 4, kNB = 16;

template <int N0, int N1, int SK>
static int tp_run(int op, const Fused2DParams* pp, cudaStream_t st) {
  using LF = FwdLayout<N0, N1, SK, kFwdCG, kNB>;
  using LB = BwdLayout<N0, N1, SK, kBwdCG, kNB>;
  // the largest filter the kernels take (31 x 31 taps) fixes the shared-memory bound
  if (op == TP_PROBE)
    return (LF::bytes(31, 31) <= 227 * 1024 && LB::bytes(31, 31) <= 227 * 1024) ? HYFFT_OK : HYFFT_ERR_UNSUPPORTED;
  const Fused2DParams& p = *pp;
  if (p.C % kFwdCG != 0 || p.C % kBwdCG != 0) return HYFFT_ERR_UNSUPPORTED;
  if (p.K0 > 2 * N0 - 1 + 1 || p.K1 > 2 * N1 - 1 + 1 || p.K0 > 31 || p.K1 > 31) return HYFFT_ERR_UNSUPPORTED;
  if (op == TP_FWD) {
    auto kern = tp2d_fwd_kernel<N0, N1, SK, kFwdCG, kNB>;
    const size_t sm = LF::bytes(p.K0, p.K1);
    if (!kernel_smem_once((const void*)kern, sm, true)) return HYFFT_ERR_CUDA;
    dim3 grid(p.C / kFwdCG, (p.B + kNB - 1) / kNB);
    kern<<<grid, 256, sm, st>>>(p);
  } else {
    auto kern = tp2d_bwd_kernel<N0, N1, SK, kBwdCG, kNB>;
    const size_t sm = LB::bytes(p.K0, p.K1);
    if (!kernel_smem_once((const void*)kern, sm, true)) return HYFFT_ERR_CUDA;
    dim3 grid(p.C / kBwdCG, (p.B + kNB - 1) / kNB);
    kern<<<grid, 256, sm, st>>>(p);
  }
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

}  // namespace tp

#define HYFFT_TP_SHAPES(X) \
  X(14, 14)                \
  X(16, 16)                \
  X(8, 8)

int tp2d_dispatch(int op, int N0, int N1, int SK, const Fused2DParams* p, cudaStream_t st) {
#define HYFFT_TP_TRY(a, b)                                        \
  if (N0 == a && N1 == b) {                                       \
    if (SK == 3) return tp::tp_run<a, b, 3>(op, p, st);           \
    if (SK == 0) return tp::tp_run<a, b, 0>(op, p, st);           \
  }
  HYFFT_TP_SHAPES(HYFFT_TP_TRY)
#undef HYFFT_TP_TRY
  return HYFFT_ERR_UNSUPPORTED;
}

}  // namespace hyfft
