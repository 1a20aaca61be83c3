// Batched, strided, pruned 1D FFT pass over one axis of a multi-dimensional
// array: the building block of the general (any-shape) FFT-conv engine.
//
// One CTA owns a tile of TL "lines" (1D signals along the FFT axis), stages
// them in shared memory, runs a radix-4/2 Stockham FFT on all of them, and
// writes them back. Loads and stores use independent thread mappings so that
// both sides are coalesced: the spectrum buffers keep channels innermost
// ([pair][axes...][C]), so consecutive lines of a tile are consecutive
// channels; real activation tensors are read along whichever axis has unit
// stride.
//
// Zero padding (input pruning), cropping (output pruning), the four-step
// twiddle of long 1D transforms, packing two real batch items into one complex
// signal (real part = item p, imaginary part = item p + half) and the
// D-skip / dtype-rounding epilogue of the reference op are fused into the
// load / store phases.
#pragma once

#include "common.cuh"

namespace hyfft {

constexpr int kPassThreads = 256;
constexpr int kPassPoints = 4096;  // max TL * F per CTA (32 KB of float2)
constexpr int kPassMaxLines = 128;

enum InMode { IN_CPLX = 0, IN_REAL = 1 };
enum OutMode { OUT_CPLX = 0, OUT_REAL = 1, OUT_REAL_SKIP = 2 };

struct PassDesc {
  int F, logF;   // FFT length along the line (power of two, <= kPassPoints)
  float dir;     // -1 forward, +1 inverse
  float scale;   // applied to every output element (1/F for inverse passes)
  int TL;        // lines per CTA
  int P, C;      // pair groups, channels
  int n_oth;     // number of "other" axes (0..2) iterated per pair/channel
  int oth_ext[2];
  long long nlines;  // P * prod(oth_ext) * C

  // complex buffers: element (p, oth, t, c) at p*c_pst + sum oth*c_ost + t*c_tst + c
  const float2* cin;
  float2* cout;
  long long ci_pst, ci_tst, ci_ost[2];
  long long co_pst, co_tst, co_ost[2];

  // signal ranges: input holds positions [in_off, in_off+n_in); keep outputs
  // at positions [out_lo, out_lo+n_out). For complex IO the position is the
  // FFT index t and the buffer index is position - offset. For real IO the
  // position is t*pos_mul + oth0*pos_oth (four-step) and the real index along
  // the axis is position - offset.
  int in_off, n_in, out_lo, n_out;
  int pos_mul, pos_oth;

  // post-FFT twiddle e^{dir * 2*pi*i * t * oth0 / 2^tw_logF} (four-step); 0 = off
  int tw_logF;

  // real tensors: element (b, c, pos, oth) at b*bst + c*cst + pos*tst + sum oth*ost
  const void* rin;
  long long ri_bst, ri_cst, ri_tst, ri_ost[2];
  // fused product pass (mid != 0): after the forward transform (dir -1) every point t of
  // a line is multiplied by the kernel spectrum kin[k_base + t * k_tst] (mid == 2: its
  // conjugate), then transformed back (+1) before the store; k_base = (k_shared ? 0 : p)
  // * k_pst + sum oth * k_ost + c.
  int mid;
  const float2* kin;
  long long k_pst, k_tst, k_ost[2];
  int k_shared;
  // k_half: kin holds only bins [0, ext/2] of the last "other" axis (the spectrum of a real
  // filter); a line whose last-axis bin is above ext/2 reads the conjugate of the mirrored
  // line (every other-axis index and the point index t negated modulo their extents)
  int k_half;

  void* rout;
  long long ro_bst, ro_cst, ro_tst, ro_ost[2];
  const void* skip;  // same layout as rout (OUT_REAL_SKIP): y = round(round(v) + round(D*skip))
  const void* Dv;    // [C] float32 skip scale (values of the activation dtype)
  int B, half, packed;  // pair p -> items p and p+half (if packed and p+half < B)

  int load_t_fastest;   // 1: load mapping walks t fastest (source contiguous along t)
  int store_t_fastest;  // 1: store mapping walks t fastest
};

// Radix-4 / radix-2 butterflies (dir = -1 forward, +1 inverse).
__device__ __forceinline__ void dft4(float2& a0, float2& a1, float2& a2, float2& a3, float dir) {
  float2 t0 = cadd(a0, a2), t1 = csub(a0, a2), t2 = cadd(a1, a3), t3 = csub(a1, a3);
  float2 jt3 = make_float2(-dir * t3.y, dir * t3.x);  // (dir * i) * t3
  a0 = cadd(t0, t2);
  a2 = csub(t0, t2);
  a1 = cadd(t1, jt3);
  a3 = csub(t1, jt3);
}

// e^{dir * 2*pi*i * j / F} for 0 <= j < F from a table of the first half turn,
// tw[j] = (cos(2 pi j / F), sin(2 pi j / F)) for j < F/2.
__device__ __forceinline__ float2 twiddle(const float2* tw, int j, int half, float dir) {
  float2 w = tw[j & (half - 1)];
  if (j >= half) w = make_float2(-w.x, -w.y);
  return make_float2(w.x, dir * w.y);
}

// Shared-memory index of point t of a line: one pad slot every 16 points, so the
// stride-16 writes of a radix-16 Stockham stage fall into distinct banks.
__device__ __forceinline__ int padi(int t) { return t + (t >> 4); }
__host__ __device__ constexpr int pass_ld(int F) { return F + (F >> 4) + 1; }

// 16-point DFT in registers, natural order in, natural order out (two radix-4 layers).
__device__ __forceinline__ void dft16(float2 (&v)[16], float dir) {
  constexpr float c1 = 0.92387953251128674f, s1 = 0.38268343236508978f, h = 0.70710678118654752f;
#pragma unroll
  for (int n2 = 0; n2 < 4; ++n2) dft4(v[n2], v[n2 + 4], v[n2 + 8], v[n2 + 12], dir);
  // v[n2 + 4 k1] *= W16^(n2 k1), W16 = e^{dir 2 pi i / 16}
  const float2 w1 = make_float2(c1, dir * s1), w2 = make_float2(h, dir * h), w3 = make_float2(s1, dir * c1);
  const float2 w6 = make_float2(-h, dir * h), w9 = make_float2(-c1, -dir * s1);
  v[5] = cmul(v[5], w1);
  v[9] = cmul(v[9], w2);
  v[13] = cmul(v[13], w3);
  v[6] = cmul(v[6], w2);
  v[10] = make_float2(-dir * v[10].y, dir * v[10].x);  // * W16^4 = dir * i
  v[14] = cmul(v[14], w6);
  v[7] = cmul(v[7], w3);
  v[11] = cmul(v[11], w6);
  v[15] = cmul(v[15], w9);
  float2 o[16];
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1) {
    float2 a0 = v[4 * k1], a1 = v[4 * k1 + 1], a2 = v[4 * k1 + 2], a3 = v[4 * k1 + 3];
    dft4(a0, a1, a2, a3, dir);
    o[k1] = a0;
    o[k1 + 4] = a1;
    o[k1 + 8] = a2;
    o[k1 + 12] = a3;
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = o[k];
}

// 8-point DFT in registers, natural order in and out (two 4-point DFTs of the even
// and odd points, combined with W8^k).
__device__ __forceinline__ void dft8(float2 (&v)[8], float dir) {
  constexpr float h = 0.70710678118654752f;
  float2 e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6];
  float2 o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
  dft4(e0, e1, e2, e3, dir);
  dft4(o0, o1, o2, o3, dir);
  o1 = cmul(o1, make_float2(h, dir * h));
  o2 = make_float2(-dir * o2.y, dir * o2.x);
  o3 = cmul(o3, make_float2(-h, dir * h));
  v[0] = cadd(e0, o0);
  v[4] = csub(e0, o0);
  v[1] = cadd(e1, o1);
  v[5] = csub(e1, o1);
  v[2] = cadd(e2, o2);
  v[6] = csub(e2, o2);
  v[3] = cadd(e3, o3);
  v[7] = csub(e3, o3);
}

template <int R>
__device__ __forceinline__ void dftR(float2 (&v)[R], float dir) {
  if constexpr (R == 16) {
    dft16(v, dir);
  } else if constexpr (R == 8) {
    dft8(v, dir);
  } else if constexpr (R == 4) {
    dft4(v[0], v[1], v[2], v[3], dir);
  } else {
    const float2 a = v[0], b = v[1];
    v[0] = cadd(a, b);
    v[1] = csub(a, b);
  }
}

// One radix-R Stockham stage over TL lines of length F = 2^logF (sub-transform
// length Ns = 2^lgNs so far). IPT items of R points per thread are held in
// registers between the two barriers.
template <int R, int LGR, int IPT>
__device__ __forceinline__ void stockham_stage(float2* sm, const float2* tw, int TL, int logF, int ld, int lgNs,
                                               float dir) {
  const int F = 1 << logF, halfF = F >> 1;
  const int lgpl = logF - LGR, per_line = 1 << lgpl;
  const int total = TL << lgpl;
  const int Ns = 1 << lgNs;
  float2 v[IPT][R];
#pragma unroll
  for (int it = 0; it < IPT; ++it) {
    const int item = threadIdx.x + it * kPassThreads;
    if (item < total) {
      const int l = item >> lgpl, j = item & (per_line - 1);
      const int k = j & (Ns - 1);
      const float2* src = sm + l * ld;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float2 a = src[padi(r * per_line + j)];
        if (r > 0 && k > 0) a = cmul(a, twiddle(tw, (r * k) << (logF - lgNs - LGR), halfF, dir));
        v[it][r] = a;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < IPT; ++it) {
    const int item = threadIdx.x + it * kPassThreads;
    if (item < total) {
      const int l = item >> lgpl, j = item & (per_line - 1);
      const int k = j & (Ns - 1);
      dftR<R>(v[it], dir);
      float2* dst = sm + l * ld;
      const int base = ((j >> lgNs) << (lgNs + LGR)) + k;
#pragma unroll
      for (int r = 0; r < R; ++r) dst[padi(base + r * Ns)] = v[it][r];
    }
  }
  __syncthreads();
}

// In-place Stockham autosort FFT of TL lines of length F stored at
// sm[l * ld + padi(t)] (TL * F <= kPassPoints). All threads of the CTA take part;
// radix-16 stages while at least four factors of two remain, then one radix 8 / 4 / 2.
// Twiddles come from the half-turn table tw (F/2 entries).
static __device__ void stockham_tile(float2* sm, const float2* tw, int TL, int F, int logF, int ld, float dir) {
  int lgNs = 0;
  while (logF - lgNs >= 4) {
    stockham_stage<16, 4, kPassPoints / (16 * kPassThreads)>(sm, tw, TL, logF, ld, lgNs, dir);
    lgNs += 4;
  }
  // one final stage for the remaining 1..3 factors of two
  const int rem = logF - lgNs;
  if (rem == 3) stockham_stage<8, 3, kPassPoints / (8 * kPassThreads)>(sm, tw, TL, logF, ld, lgNs, dir);
  else if (rem == 2) stockham_stage<4, 2, kPassPoints / (4 * kPassThreads)>(sm, tw, TL, logF, ld, lgNs, dir);
  else if (rem == 1) stockham_stage<2, 1, kPassPoints / (2 * kPassThreads)>(sm, tw, TL, logF, ld, lgNs, dir);
}

struct LineInfo {
  long long cin_base, cout_base;  // complex buffer base of the line (t = 0)
  long long r_re_in, r_im_in;     // real input base of the two packed items (-1: none)
  long long r_re_out, r_im_out;   // real output base
  int pos0;                       // oth0 * pos_oth
  int tw_m;                       // twiddle multiplier (oth0)
  int c;                          // channel
  int valid;
};

// The per-line bookkeeping lives in shared memory as separate arrays per field, so that
// threads reading consecutive lines hit consecutive words (no bank conflicts).
struct LineSoA {
  long long *cin, *cout, *rri, *rii, *rro, *rio, *kb;
  int *pos0, *twm, *ch, *valid;
};
constexpr int kLineBytes = (7 * 8 + 4 * 4) * kPassMaxLines;  // shared-memory bytes of the bookkeeping
__device__ __forceinline__ LineSoA line_soa(unsigned char* base) {
  LineSoA s;
  long long* q = reinterpret_cast<long long*>(base);
  s.cin = q;
  s.cout = q + kPassMaxLines;
  s.rri = q + 2 * kPassMaxLines;
  s.rii = q + 3 * kPassMaxLines;
  s.rro = q + 4 * kPassMaxLines;
  s.rio = q + 5 * kPassMaxLines;
  s.kb = q + 6 * kPassMaxLines;
  int* r = reinterpret_cast<int*>(q + 7 * kPassMaxLines);
  s.pos0 = r;
  s.twm = r + kPassMaxLines;
  s.ch = r + 2 * kPassMaxLines;
  s.valid = r + 3 * kPassMaxLines;
  return s;
}
__device__ __forceinline__ void put_line(const LineSoA& s, int l, const LineInfo& L) {
  s.cin[l] = L.cin_base;
  s.cout[l] = L.cout_base;
  s.rri[l] = L.r_re_in;
  s.rii[l] = L.r_im_in;
  s.rro[l] = L.r_re_out;
  s.rio[l] = L.r_im_out;
  s.pos0[l] = L.pos0;
  s.twm[l] = L.tw_m;
  s.ch[l] = L.c;
  s.valid[l] = L.valid;
}
__device__ __forceinline__ LineInfo get_line(const LineSoA& s, int l) {
  LineInfo L;
  L.cin_base = s.cin[l];
  L.cout_base = s.cout[l];
  L.r_re_in = s.rri[l];
  L.r_im_in = s.rii[l];
  L.r_re_out = s.rro[l];
  L.r_im_out = s.rio[l];
  L.pos0 = s.pos0[l];
  L.tw_m = s.twm[l];
  L.c = s.ch[l];
  L.valid = s.valid[l];
  return L;
}

template <int IN_MODE, int OUT_MODE, typename TI, typename TO>
__global__ void __launch_bounds__(kPassThreads, 3) fft_pass_kernel(const PassDesc d) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const LineSoA ls = line_soa(smem_raw);
  float2* sm = reinterpret_cast<float2*>(smem_raw + kLineBytes);
  const int TL = d.TL, F = d.F;
  const int ld = pass_ld(F);  // padded line stride (odd, spreads lines over banks)
  float2* tw = sm + (size_t)TL * ld;
  const int logF = d.logF, logTL = 31 - __clz(TL);  // TL and F are powers of two
  const long long line0 = (long long)blockIdx.x * TL;
  for (int j = threadIdx.x; j < (F >> 1); j += blockDim.x) {
    float sn, cs;
    sincospif(2.0f * (float)j / (float)F, &sn, &cs);
    tw[j] = make_float2(cs, sn);
  }

  // ---- per-line bookkeeping
  for (int l = threadIdx.x; l < TL; l += blockDim.x) {
    LineInfo L;
    long long lid = line0 + l;
    L.valid = lid < d.nlines;
    if (!L.valid) lid = 0;
    const int c = (int)(lid % d.C);
    long long rest = lid / d.C;
    int o[2] = {0, 0};
    for (int a = d.n_oth - 1; a >= 0; --a) {
      o[a] = (int)(rest % d.oth_ext[a]);
      rest /= d.oth_ext[a];
    }
    const int p = (int)rest;
    L.c = c;
    L.cin_base = (long long)p * d.ci_pst + (long long)o[0] * d.ci_ost[0] + (long long)o[1] * d.ci_ost[1] + c;
    L.cout_base = (long long)p * d.co_pst + (long long)o[0] * d.co_ost[0] + (long long)o[1] * d.co_ost[1] + c;
    const int b_im = p + d.half;
    const bool has_im = d.packed && b_im < d.B;
    L.r_re_in = (long long)p * d.ri_bst + (long long)c * d.ri_cst + (long long)o[0] * d.ri_ost[0] + (long long)o[1] * d.ri_ost[1];
    L.r_im_in = has_im ? L.r_re_in + (long long)d.half * d.ri_bst : -1;
    L.r_re_out = (long long)p * d.ro_bst + (long long)c * d.ro_cst + (long long)o[0] * d.ro_ost[0] + (long long)o[1] * d.ro_ost[1];
    L.r_im_out = has_im ? L.r_re_out + (long long)d.half * d.ro_bst : -1;
    L.pos0 = o[0] * d.pos_oth;
    L.tw_m = o[0];
    if (d.mid)
      ls.kb[l] = (long long)(d.k_shared ? 0 : p) * d.k_pst + (long long)o[0] * d.k_ost[0] +
                 (long long)o[1] * d.k_ost[1] + c;
    put_line(ls, l, L);
  }
  __syncthreads();

  // ---- load
  const int npts = TL * F;
#pragma unroll 4
  for (int e = threadIdx.x; e < npts; e += blockDim.x) {
    int l, t;
    if (d.load_t_fastest) { l = e >> logF; t = e & (F - 1); }
    else { t = e >> logTL; l = e & (TL - 1); }
    if constexpr (IN_MODE == IN_CPLX) {
      // asynchronous 8-byte copy straight into shared memory; out-of-range points are
      // zero-filled by the copy itself (source size 0, the source is not read)
      const int bi = t - d.in_off;
      const bool in = ls.valid[l] && bi >= 0 && bi < d.n_in;
      const float2* g = in ? d.cin + ls.cin[l] + (long long)bi * d.ci_tst : d.cin;
      const unsigned sa = (unsigned)__cvta_generic_to_shared(sm + l * ld + padi(t));
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(sa), "l"(g), "r"(in ? 8 : 0) : "memory");
      continue;
    }
    const LineInfo L = get_line(ls, l);
    float2 val = make_float2(0.f, 0.f);
    if (L.valid) {
      {
        const int pos = t * d.pos_mul + L.pos0 - d.in_off;
        if (pos >= 0 && pos < d.n_in) {
          const TI* src = reinterpret_cast<const TI*>(d.rin);
          const long long off = (long long)pos * d.ri_tst;
          val.x = DT<TI>::load(src + L.r_re_in + off);
          if (L.r_im_in >= 0) val.y = DT<TI>::load(src + L.r_im_in + off);
        }
      }
    }
    sm[l * ld + padi(t)] = val;
  }
  if constexpr (IN_MODE == IN_CPLX) asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();

  stockham_tile(sm, tw, TL, F, d.logF, ld, d.dir);

  if (d.mid) {  // product with the kernel spectrum, then the inverse transform
    const float cj = d.mid == 2 ? -1.f : 1.f;
#pragma unroll 4
    for (int e = threadIdx.x; e < npts; e += blockDim.x) {
      const int t = e >> logTL, l = e & (TL - 1);  // neighbouring lines are neighbouring channels
      if (!ls.valid[l]) continue;
      float2 k = __ldg(d.kin + ls.kb[l] + (long long)t * d.k_tst);
      k.y *= cj;
      float2* v = sm + l * ld + padi(t);
      *v = cmul(*v, k);
    }
    __syncthreads();
    stockham_tile(sm, tw, TL, F, d.logF, ld, 1.f);
  }
  const float sdir = d.mid ? 1.f : d.dir;  // direction of the store-side twiddle

  // ---- store
#pragma unroll 4
  for (int e = threadIdx.x; e < npts; e += blockDim.x) {
    int l, t;
    if (d.store_t_fastest) { l = e >> logF; t = e & (F - 1); }
    else { t = e >> logTL; l = e & (TL - 1); }
    const LineInfo L = get_line(ls, l);
    if (!L.valid) continue;
    float2 val = cscale(sm[l * ld + padi(t)], d.scale);
    if (d.tw_logF > 0 && L.tw_m != 0) {
      // e^{dir*2*pi*i*t*m/2^tw_logF}; reduce the exponent mod 2^tw_logF first
      // ex < 2^tw_logF <= 2^24 is exact in float, and so is the power-of-two scaling
      const long long ex = ((long long)t * L.tw_m) & ((1LL << d.tw_logF) - 1);
      val = cmul(val, expipi(sdir * ldexpf((float)ex, 1 - d.tw_logF)));
    }
    if (OUT_MODE == OUT_CPLX) {
      const int bo = t - d.out_lo;
      if (bo >= 0 && bo < d.n_out) d.cout[L.cout_base + (long long)bo * d.co_tst] = val;
    } else {
      const int pos = t * d.pos_mul + L.pos0 - d.out_lo;
      if (pos >= 0 && pos < d.n_out) {
        TO* dst = reinterpret_cast<TO*>(d.rout);
        const long long off = (long long)pos * d.ro_tst;
        float re = DT<TO>::round(val.x), im = DT<TO>::round(val.y);
        if (OUT_MODE == OUT_REAL_SKIP) {
          const TO* sk = reinterpret_cast<const TO*>(d.skip);
          const float Dc = reinterpret_cast<const float*>(d.Dv)[L.c];
          re = re + DT<TO>::round(Dc * DT<TO>::load(sk + L.r_re_out + off));
          if (L.r_im_out >= 0) im = im + DT<TO>::round(Dc * DT<TO>::load(sk + L.r_im_out + off));
        }
        DT<TO>::store(dst + L.r_re_out + off, re);
        if (L.r_im_out >= 0) DT<TO>::store(dst + L.r_im_out + off, im);
      }
    }
  }
}

// ---------------------------------------------------------------- channel-innermost passes
// Pass over lines whose neighbours are neighbouring channels (the channel index has unit
// stride in every spectrum buffer, and in channels-last activations), F = R1 * R2 <= 256
// and no four-step twiddle: the middle passes of 2D / 3D transforms, and the first /
// last pass of a transform from / into a channels-last activation. Each lane of a warp
// owns one of 32 consecutive lines, so every global access of a warp covers 32
// neighbouring channels. The transform is a two-level decomposition, t = j + R2 r and
// k = k1 + R1 k2:
//   X[k1 + R1 k2] = sum_j W_R2^(j k2) W_F^(j k1) sum_r W_R1^(r k1) x[j + R2 r],
// level one in registers straight from global memory, the transposition through shared
// memory laid out [point][line] (conflict-free: a warp touches 32 neighbouring words),
// level two in registers straight to global memory. All reads of global memory happen
// before the first barrier, so the pass may run in place.
// MID != 0 (product pass): forward transform, product with the kernel spectrum (MID == 2:
// its conjugate), inverse transform, mirrored through shared memory a second time.
// DIR: direction of a plain pass (-1 forward, +1 inverse); MID passes are forward first.
// IM / OM: complex or real (packed pair: real part item p, imaginary part item p + half)
// input / output with the same semantics as fft_pass_kernel (OUT_REAL_SKIP adds the
// dtype-rounded D-skip term).
constexpr int kClWarps = 8;

template <int F>
__host__ __device__ constexpr int cl_lines_per_cta() { return F >= 128 ? 32 : 32 * (128 / F); }

// shared-memory pitch of one point across the CTA's lines (odd: the staged t-major
// transposes of TMAJ passes stay conflict-light)
template <int F>
__host__ __device__ constexpr int cl_pitch() { return cl_lines_per_cta<F>() + 1; }

template <int F>
__host__ __device__ constexpr size_t cl_smem_bytes() {
  return sizeof(float2) * ((size_t)F * cl_pitch<F>() + F) + 6 * sizeof(long long) * cl_lines_per_cta<F>() +
         sizeof(int) * cl_lines_per_cta<F>();
}

template <int R1, int R2, int MID, int DIR, int IM, int OM, typename TI, typename TO, bool TMAJ = false>
__global__ void __launch_bounds__(kClWarps * 32) fft_lines_cl_kernel(const PassDesc d) {
  constexpr int F = R1 * R2;
  constexpr int NL = cl_lines_per_cta<F>();  // lines per CTA
  constexpr int NP = cl_pitch<F>();          // shared-memory pitch of one point
  constexpr int G = NL / 32;                 // groups of 32 lines
  constexpr float D1 = MID ? -1.f : (float)DIR;
  static_assert(!TMAJ || (!MID && (IM == IN_REAL) != (OM != OUT_CPLX)), "t-major staging: one real side");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float2* sm = reinterpret_cast<float2*>(smem_raw);        // [F][NP]
  float2* tw = sm + F * NP;                                 // [F] e^{-2 pi i m / F}
  long long* cb_in = reinterpret_cast<long long*>(tw + F);  // [NL] line bases, -1: past the end
  long long* cb_out = cb_in + NL;                           // complex output / real output (item p)
  long long* kbase = cb_out + NL;
  long long* im_in = kbase + NL;    // real input of item p + half (-1: none)
  long long* im_out = im_in + NL;   // real output of item p + half (-1: none)
  long long* pad = im_out + NL;
  int* chan = reinterpret_cast<int*>(pad + NL);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long line0 = (long long)blockIdx.x * NL;
  for (int m = threadIdx.x; m < F; m += blockDim.x) {
    float sn, cs;
    sincospif(2.0f * (float)m / (float)F, &sn, &cs);
    tw[m] = make_float2(cs, -sn);
  }
  for (int l = threadIdx.x; l < NL; l += blockDim.x) {
    const long long lid = line0 + l;
    if (lid >= d.nlines) {
      cb_in[l] = -1;
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
    chan[l] = c;
    if (IM == IN_CPLX) {
      cb_in[l] = p * d.ci_pst + (long long)o[0] * d.ci_ost[0] + (long long)o[1] * d.ci_ost[1] + c;
    } else {
      cb_in[l] = p * d.ri_bst + (long long)c * d.ri_cst + (long long)o[0] * d.ri_ost[0] + (long long)o[1] * d.ri_ost[1];
      im_in[l] = has_im ? cb_in[l] + (long long)d.half * d.ri_bst : -1;
    }
    if (OM == OUT_CPLX) {
      cb_out[l] = p * d.co_pst + (long long)o[0] * d.co_ost[0] + (long long)o[1] * d.co_ost[1] + c;
    } else {
      cb_out[l] = p * d.ro_bst + (long long)c * d.ro_cst + (long long)o[0] * d.ro_ost[0] + (long long)o[1] * d.ro_ost[1];
      im_out[l] = has_im ? cb_out[l] + (long long)d.half * d.ro_bst : -1;
    }
    if (MID) {
      int mo[2] = {o[0], o[1]};
      const bool mir = d.k_half && 2 * o[d.n_oth - 1] > d.oth_ext[d.n_oth - 1];
      if (mir)
        for (int a = 0; a < d.n_oth; ++a) mo[a] = (d.oth_ext[a] - o[a]) % d.oth_ext[a];
      kbase[l] = (d.k_shared ? 0 : p) * d.k_pst + (long long)mo[0] * d.k_ost[0] + (long long)mo[1] * d.k_ost[1] + c;
      pad[l] = mir ? 1 : 0;
    }
  }
  __syncthreads();

  // store of point t of line l (value before scaling)
  auto store = [&](int l, int t, float2 v) {
    const int bo = t - d.out_lo;
    if (bo < 0 || bo >= d.n_out) return;
    const float2 val = cscale(v, d.scale);
    if constexpr (OM == OUT_CPLX) {
      d.cout[cb_out[l] + (long long)bo * d.co_tst] = val;
    } else {
      TO* dst = reinterpret_cast<TO*>(d.rout);
      const long long off = (long long)bo * d.ro_tst;
      const long long ri = im_out[l];
      float re = DT<TO>::round(val.x), im = DT<TO>::round(val.y);
      if constexpr (OM == OUT_REAL_SKIP) {
        const TO* sk = reinterpret_cast<const TO*>(d.skip);
        const float Dc = reinterpret_cast<const float*>(d.Dv)[chan[l]];
        re = re + DT<TO>::round(Dc * DT<TO>::load(sk + cb_out[l] + off));
        if (ri >= 0) im = im + DT<TO>::round(Dc * DT<TO>::load(sk + ri + off));
      }
      DT<TO>::store(dst + cb_out[l] + off, re);
      if (ri >= 0) DT<TO>::store(dst + ri + off, im);
    }
  };

  if constexpr (TMAJ && IM == IN_REAL) {
    // t-major source (unit stride along the line, lines far apart): stage every line
    // t-fastest into sm[t][line] first, zeros outside the input window
    const TI* src = reinterpret_cast<const TI*>(d.rin);
    for (int e = threadIdx.x; e < NL * F; e += blockDim.x) {
      const int l = e / F, t = e - l * F;
      const long long base = cb_in[l];
      const int bi = t - d.in_off;
      float2 v = make_float2(0.f, 0.f);
      if (base >= 0 && bi >= 0 && bi < d.n_in) {
        const long long off = (long long)bi * d.ri_tst;
        v.x = DT<TI>::load(src + base + off);
        if (im_in[l] >= 0) v.y = DT<TI>::load(src + im_in[l] + off);
      }
      sm[t * NP + l] = v;
    }
    __syncthreads();
  }
  // level one: R1-point transforms over r of x[j + R2 r], twiddle W_F^(j k1) -> sm[k1 R2 + j]
  // (a TMAJ item reads its points {j + R2 r} from shared memory and writes the same set)
  for (int it = warp; it < G * R2; it += kClWarps) {
    const int g = it / R2, j = it % R2, l = g * 32 + lane;
    const long long base = cb_in[l];
    float2 v[R1];
    if constexpr (TMAJ && IM == IN_REAL) {
#pragma unroll
      for (int r = 0; r < R1; ++r) v[r] = sm[(j + R2 * r) * NP + l];
    } else if constexpr (IM == IN_CPLX) {
      const float2* src = d.cin + base + (long long)(j - d.in_off) * d.ci_tst;
      const long long step = (long long)R2 * d.ci_tst;
#pragma unroll
      for (int r = 0; r < R1; ++r) {
        const int bi = j + R2 * r - d.in_off;
        v[r] = (base >= 0 && bi >= 0 && bi < d.n_in) ? src[r * step] : make_float2(0.f, 0.f);
      }
    } else {
      const TI* src = reinterpret_cast<const TI*>(d.rin);
      const long long ri = base >= 0 ? im_in[l] : -1;
#pragma unroll
      for (int r = 0; r < R1; ++r) {
        const int bi = j + R2 * r - d.in_off;
        const bool ok = base >= 0 && bi >= 0 && bi < d.n_in;
        const long long off = (long long)bi * d.ri_tst;
        v[r] = make_float2(ok ? DT<TI>::load(src + base + off) : 0.f, (ok && ri >= 0) ? DT<TI>::load(src + ri + off) : 0.f);
      }
    }
    dftR<R1>(v, D1);
#pragma unroll
    for (int k1 = 0; k1 < R1; ++k1) {
      float2 a = v[k1];
      if (k1 > 0 && j > 0) {
        float2 w = tw[j * k1];
        if (D1 > 0.f) w.y = -w.y;
        a = cmul(a, w);
      }
      sm[(k1 * R2 + j) * NP + l] = a;
    }
  }
  __syncthreads();

  if constexpr (TMAJ && OM != OUT_CPLX) {
    // t-major destination: all level-two items in registers, then natural order into
    // shared memory, then every line stored t-fastest
    constexpr int ITEMS = (G * R1 + kClWarps - 1) / kClWarps;
    float2 res[ITEMS][R2];
#pragma unroll
    for (int ii = 0; ii < ITEMS; ++ii) {
      const int it = warp + ii * kClWarps;
      if (it < G * R1) {
        const int g = it / R1, k1 = it % R1, l = g * 32 + lane;
#pragma unroll
        for (int j = 0; j < R2; ++j) res[ii][j] = sm[(k1 * R2 + j) * NP + l];
        dftR<R2>(res[ii], D1);
      }
    }
    __syncthreads();
#pragma unroll
    for (int ii = 0; ii < ITEMS; ++ii) {
      const int it = warp + ii * kClWarps;
      if (it < G * R1) {
        const int g = it / R1, k1 = it % R1, l = g * 32 + lane;
#pragma unroll
        for (int k2 = 0; k2 < R2; ++k2) sm[(k1 + R1 * k2) * NP + l] = res[ii][k2];
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < NL * d.n_out; e += blockDim.x) {
      const int l = e / d.n_out, t = d.out_lo + (e - l * d.n_out);
      if (cb_in[l] >= 0 && t < F) store(l, t, sm[t * NP + l]);
    }
    return;
  }
  // level two: R2-point transforms over j -> X[k1 + R1 k2]
  for (int it = warp; it < G * R1; it += kClWarps) {
    const int g = it / R1, k1 = it % R1, l = g * 32 + lane;
    float2 v[R2];
#pragma unroll
    for (int j = 0; j < R2; ++j) v[j] = sm[(k1 * R2 + j) * NP + l];
    dftR<R2>(v, D1);
    if constexpr (MID) {
      if (cb_in[l] >= 0) {
        const long long kb = kbase[l];
        const bool mir = pad[l] != 0;
#pragma unroll
        for (int k2 = 0; k2 < R2; ++k2) {
          const int kk = k1 + R1 * k2;
          float2 kv = __ldg(d.kin + kb + (long long)(mir ? ((F - kk) & (F - 1)) : kk) * d.k_tst);
          if (mir != (MID == 2)) kv.y = -kv.y;
          v[k2] = cmul(v[k2], kv);
        }
      }
      dftR<R2>(v, 1.f);  // inverse over k2 -> j, then W_F^(-j k1)
#pragma unroll
      for (int j = 0; j < R2; ++j) {
        float2 a = v[j];
        if (k1 > 0 && j > 0) {
          const float2 w = tw[j * k1];
          a = cmul(a, make_float2(w.x, -w.y));
        }
        sm[(k1 * R2 + j) * NP + l] = a;
      }
    } else {
      if (cb_in[l] >= 0) {
#pragma unroll
        for (int k2 = 0; k2 < R2; ++k2) store(l, k1 + R1 * k2, v[k2]);
      }
    }
  }
  if constexpr (MID) {
    __syncthreads();
    // inverse level one: R1-point transforms over k1 -> x[j + R2 r]
    for (int it = warp; it < G * R2; it += kClWarps) {
      const int g = it / R2, j = it % R2, l = g * 32 + lane;
      float2 v[R1];
#pragma unroll
      for (int k1 = 0; k1 < R1; ++k1) v[k1] = sm[(k1 * R2 + j) * NP + l];
      dftR<R1>(v, 1.f);
      if (cb_in[l] >= 0) {
#pragma unroll
        for (int r = 0; r < R1; ++r) store(l, j + R2 * r, v[r]);
      }
    }
  }
}

// Backward product pass on the same two-level channel-innermost structure: for every
// line along the last forward axis it transforms the partial spectra of x (fx) and dy
// (fdy), forms DX = DY * conj(Kh) and DK = DY * conj(X) point by point, and inverse
// transforms both, storing DX into the dx chain's buffer (idx: crop of the first inverse
// pass) and DK into the kernel-gradient buffer (idk). With a kernel shared by the batch
// (pl = number of pairs > 1) the CTA loops over the pairs of its lines and adds the
// per-pair DK lines (the inverse transform is linear). With packed pairs the real part
// of the inverse of DY * conj(X) is the sum of both items' correlations.
// Kh: fx.kin with fx.k_* strides (k_shared: one kernel for all pairs).
template <int R1, int R2>
__host__ __device__ constexpr size_t cl_bwd_smem_bytes() {
  return sizeof(float2) * (2 * (size_t)R1 * R2 * cl_lines_per_cta<R1 * R2>() + R1 * R2) +
         6 * sizeof(long long) * cl_lines_per_cta<R1 * R2>();
}

template <int R1, int R2>
__global__ void __launch_bounds__(kClWarps * 32, 3) fft_lines_cl_bwd_kernel(const PassDesc fx, const PassDesc fdy,
                                                                         const PassDesc idx, const PassDesc idk,
                                                                         int pl) {
  constexpr int F = R1 * R2;
  constexpr int NL = cl_lines_per_cta<F>();
  constexpr int G = NL / 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float2* sa = reinterpret_cast<float2*>(smem_raw);  // [F][NL]: X, then DK
  float2* sb = sa + F * NL;                           // [F][NL]: DY, then DX
  float2* tw = sb + F * NL;                           // [F] e^{-2 pi i m / F}
  long long* bx = reinterpret_cast<long long*>(tw + F);
  long long* bdy = bx + NL;
  long long* bdx = bdy + NL;
  long long* bdk = bdx + NL;
  long long* bkh = bdk + NL;
  long long* bmir = bkh + NL;  // 1: the filter line is read mirrored and conjugated (k_half)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long nl = fx.nlines / pl;
  const long long line0 = (long long)blockIdx.x * NL;
  for (int m = threadIdx.x; m < F; m += blockDim.x) {
    float sn, cs;
    sincospif(2.0f * (float)m / (float)F, &sn, &cs);
    tw[m] = make_float2(cs, -sn);
  }
  for (int l = threadIdx.x; l < NL; l += blockDim.x) {
    const long long lid = line0 + l;
    if (lid >= nl) {
      bx[l] = -1;
      continue;
    }
    const int c = (int)(lid % fx.C);
    long long rest = lid / fx.C;
    int o[2] = {0, 0};
    for (int a = fx.n_oth - 1; a >= 0; --a) {
      o[a] = (int)(rest % fx.oth_ext[a]);
      rest /= fx.oth_ext[a];
    }
    const long long p = rest;  // 0 when the CTA loops over the pairs
    const long long ks = fx.k_shared ? 0 : p;
    bx[l] = p * fx.ci_pst + (long long)o[0] * fx.ci_ost[0] + (long long)o[1] * fx.ci_ost[1] + c;
    bdy[l] = p * fdy.ci_pst + (long long)o[0] * fdy.ci_ost[0] + (long long)o[1] * fdy.ci_ost[1] + c;
    bdx[l] = p * idx.co_pst + (long long)o[0] * idx.co_ost[0] + (long long)o[1] * idx.co_ost[1] + c;
    bdk[l] = ks * idk.co_pst + (long long)o[0] * idk.co_ost[0] + (long long)o[1] * idk.co_ost[1] + c;
    int mo[2] = {o[0], o[1]};
    const bool mir = fx.k_half && 2 * o[fx.n_oth - 1] > fx.oth_ext[fx.n_oth - 1];
    if (mir)
      for (int a = 0; a < fx.n_oth; ++a) mo[a] = (fx.oth_ext[a] - o[a]) % fx.oth_ext[a];
    bkh[l] = ks * fx.k_pst + (long long)mo[0] * fx.k_ost[0] + (long long)mo[1] * fx.k_ost[1] + c;
    bmir[l] = mir ? 1 : 0;
  }
  __syncthreads();

#pragma unroll 1
  for (int pp = 0; pp < pl; ++pp) {
    // forward level one of X (into sa) and DY (into sb), one signal at a time
    for (int it = warp; it < 2 * G * R2; it += kClWarps) {
      const int sig = it / (G * R2), ir = it % (G * R2);
      const int g = ir / R2, j = ir % R2, l = g * 32 + lane;
      const bool ok = bx[l] >= 0;
      const PassDesc& f = sig ? fdy : fx;
      float2 u[R1];
      const float2* sx = f.cin + (ok ? (sig ? bdy[l] : bx[l]) : 0) + pp * f.ci_pst + (long long)(j - f.in_off) * f.ci_tst;
      const long long stx = (long long)R2 * f.ci_tst;
#pragma unroll
      for (int r = 0; r < R1; ++r) {
        const int bix = j + R2 * r - f.in_off;
        u[r] = (ok && bix >= 0 && bix < f.n_in) ? sx[r * stx] : make_float2(0.f, 0.f);
      }
      dftR<R1>(u, -1.f);
      float2* dst = sig ? sb : sa;
#pragma unroll
      for (int k1 = 0; k1 < R1; ++k1) {
        float2 a = u[k1];
        if (k1 > 0 && j > 0) a = cmul(a, tw[j * k1]);
        dst[(k1 * R2 + j) * NL + l] = a;
      }
    }
    __syncthreads();
    // level two, products, inverse level two
    for (int it = warp; it < G * R1; it += kClWarps) {
      const int g = it / R1, k1 = it % R1, l = g * 32 + lane;
      float2 u[R2], v[R2];
#pragma unroll
      for (int j = 0; j < R2; ++j) {
        u[j] = sa[(k1 * R2 + j) * NL + l];
        v[j] = sb[(k1 * R2 + j) * NL + l];
      }
      dftR<R2>(u, -1.f);
      dftR<R2>(v, -1.f);
      const long long kb = bkh[l];
      if (bx[l] >= 0) {
        const bool mir = bmir[l] != 0;
#pragma unroll
        for (int k2 = 0; k2 < R2; ++k2) {
          const int kk = k1 + R1 * k2;
          float2 kv = __ldg(fx.kin + kb + (long long)(mir ? ((F - kk) & (F - 1)) : kk) * fx.k_tst);
          if (mir) kv.y = -kv.y;
          const float2 dk = cmulc(v[k2], u[k2]);  // DY * conj(X)
          v[k2] = cmulc(v[k2], kv);               // DY * conj(Kh)
          u[k2] = dk;
        }
      }
      dftR<R2>(u, 1.f);
      dftR<R2>(v, 1.f);
#pragma unroll
      for (int j = 0; j < R2; ++j) {
        float2 a = u[j], b = v[j];
        if (k1 > 0 && j > 0) {
          const float2 w = tw[j * k1];
          const float2 wc = make_float2(w.x, -w.y);
          a = cmul(a, wc);
          b = cmul(b, wc);
        }
        sa[(k1 * R2 + j) * NL + l] = a;
        sb[(k1 * R2 + j) * NL + l] = b;
      }
    }
    __syncthreads();
    // inverse level one; DX into the dx chain, DK (accumulated over the pairs) into dKh
    for (int it = warp; it < 2 * G * R2; it += kClWarps) {
      const int sig = it / (G * R2), ir = it % (G * R2);
      const int g = ir / R2, j = ir % R2, l = g * 32 + lane;
      if (bx[l] < 0) continue;
      float2 u[R1];
      const float2* src = sig ? sb : sa;
#pragma unroll
      for (int k1 = 0; k1 < R1; ++k1) u[k1] = src[(k1 * R2 + j) * NL + l];
      dftR<R1>(u, 1.f);
      if (sig) {
        float2* ox = idx.cout + bdx[l] + pp * idx.co_pst;
#pragma unroll
        for (int r = 0; r < R1; ++r) {
          const int bo = j + R2 * r - idx.out_lo;
          if (bo >= 0 && bo < idx.n_out) ox[(long long)bo * idx.co_tst] = cscale(u[r], idx.scale);
        }
      } else {
        float2* ok = idk.cout + bdk[l];
#pragma unroll
        for (int r = 0; r < R1; ++r) {
          const int bk = j + R2 * r - idk.out_lo;
          if (bk >= 0 && bk < idk.n_out) {
            float2* q = ok + (long long)bk * idk.co_tst;
            const float2 val = cscale(u[r], idk.scale);
            *q = pp == 0 ? val : cadd(*q, val);
          }
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace hyfft
