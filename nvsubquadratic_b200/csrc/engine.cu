// General FFT-conv engine: host-side planning of the pass sequence and the
// C-ABI entry points for the op contract and the fused Hyena mixer.
//
// Spectra live in caller-provided workspace as complex float32 arrays laid
// out [pair][F_0]...[F_{D-1}][C] (channels innermost). Two real batch items
// that share a kernel are packed into one complex signal (real part = item p,
// imaginary part = item p + ceil(B/2)); because the kernel is real its
// spectrum multiplies both halves independently, so one complex transform
// carries two convolutions and no Hermitian post-processing is needed.
//
// FFT length per axis: the smallest power of two that is >= K and that
// leaves no wrap-around inside the kept window (>= N + ceil(K/2) - 1 for the
// centred "same" conv, >= L + K - 1 for causal). The linear result is
// identical to the reference's F = min(N + (K+1)//2, 2N) / min(L+K, 2L)
// (nvsubquadratic/ops/fftconv.py:580, :627, :699-702, :773-777); the one case
// where the reference wraps around (causal with K > L + 1) is remapped by the
// Python wrapper to an equivalent centred kernel before it reaches here.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <type_traits>
#include <string>

#include "common.cuh"
#include "fft_pass.cuh"
#include "fft_long.h"
#include "big2d.h"
#include "hyena_elem.cuh"
#include "stencil3d.cuh"
#include "pointwise.cuh"
#include "fused2d.h"

namespace hyfft {

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

// for the other translation units: record msg as this thread's last error, return code
int set_error(int code, const char* msg) { return fail(code, "%s", msg); }

std::atomic<long long> g_launches{0};

static int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HYFFT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

#define HY_TRY(expr)              \
  do {                            \
    int _rc = (expr);             \
    if (_rc != HYFFT_OK) return _rc; \
  } while (0)

static int ilog2(long long v) {
  int r = 0;
  while ((1LL << r) < v) ++r;
  return r;
}
static long long next_pow2(long long v) { return v <= 1 ? 1 : (1LL << ilog2(v)); }

// ------------------------------------------------------------------ geometry
struct Geo {
  int D = 1;
  int N[3] = {1, 1, 1};
  int K[3] = {1, 1, 1};
  int F[3] = {1, 1, 1};
  int crop[3] = {0, 0, 0};  // forward output window start per axis
  bool four = false;        // 1D four-step decomposition F = Fa * Fb
  int Fa = 1, Fb = 1;
  long long vol_F = 1;      // prod F
  // circular (periodic) axes: bit d set = axis d has FFT length N[d] (no padding) and its
  // "same" alignment is a roll by rshift[d] = (K[d] - 1) / 2, applied as a phase ramp on
  // the filter spectrum (ops/circular_fftconv.py:310-404, ops/mixed_fftconv.py:295-342)
  int periodic = 0;
  int rshift[3] = {0, 0, 0};
};

static int make_geo(int nd, const int* n, const int* k, int causal, int periodic, Geo& g) {
  if (nd < 1 || nd > 3) return fail(HYFFT_ERR_INVALID, "ndim must be 1..3 (got %d)", nd);
  if (causal && nd != 1) return fail(HYFFT_ERR_INVALID, "causal convolution is 1D only");
  if (periodic & ~((1 << nd) - 1)) return fail(HYFFT_ERR_INVALID, "periodic mask 0x%x names axes beyond %d", periodic, nd);
  if (periodic && causal) return fail(HYFFT_ERR_INVALID, "causal convolution has no periodic axis");
  g.D = nd;
  g.vol_F = 1;
  g.periodic = periodic;
  for (int d = 0; d < nd; ++d) {
    if (n[d] < 1 || k[d] < 1) return fail(HYFFT_ERR_INVALID, "extents must be positive");
    if (k[d] > 2 * n[d]) return fail(HYFFT_ERR_INVALID, "kernel extent %d > 2 * input extent %d", k[d], n[d]);
    g.N[d] = n[d];
    g.K[d] = k[d];
    if (periodic & (1 << d)) {
      if (k[d] > n[d]) return fail(HYFFT_ERR_INVALID, "kernel extent %d > input extent %d on periodic axis %d", k[d], n[d], d);
      if (next_pow2(n[d]) != n[d])
        return fail(HYFFT_ERR_UNSUPPORTED, "periodic axis %d of length %d: circular FFT lengths must be powers of two", d, n[d]);
      g.F[d] = n[d];
      g.crop[d] = 0;
      g.rshift[d] = (k[d] - 1) / 2;
      if (nd > 1 && g.F[d] > kPassPoints) return fail(HYFFT_ERR_UNSUPPORTED, "multi-D axis FFT length %d > %d", g.F[d], kPassPoints);
      g.vol_F *= g.F[d];
      continue;
    }
    long long need;
    if (causal) {
      if (k[d] > n[d] + 1)
        return fail(HYFFT_ERR_UNSUPPORTED, "causal kernel longer than L+1 wraps around; remap it to a centred kernel first");
      need = (long long)n[d] + k[d] - 1;
      g.crop[d] = 0;
    } else {
      need = (long long)n[d] + (k[d] + 1) / 2 - 1;
      g.crop[d] = k[d] / 2;
    }
    need = std::max<long long>(need, k[d]);
    g.F[d] = (int)next_pow2(need);
    if (g.F[d] > (1 << 24)) return fail(HYFFT_ERR_UNSUPPORTED, "FFT length %d too large", g.F[d]);
    if (nd > 1 && g.F[d] > kPassPoints) return fail(HYFFT_ERR_UNSUPPORTED, "multi-D axis FFT length %d > %d", g.F[d], kPassPoints);
    g.vol_F *= g.F[d];
  }
  g.four = (nd == 1 && g.F[0] > kPassPoints);
  if (g.four) {
    const int lf = ilog2(g.F[0]);
    // the second axis takes the larger factor: the first axis carries the real activation
    // side, whose channel runs (lines per CTA of the long passes) are then the longer ones
    g.Fb = 1 << ((lf + 1) / 2);
    g.Fa = g.F[0] / g.Fb;
  }
  return HYFFT_OK;
}

// A strided real tensor (element strides), viewed as [b][c][s0][s1][s2].
struct RealView {
  const void* ptr = nullptr;
  long long bst = 0, cst = 0, sst[3] = {0, 0, 0};
};

static RealView real_view(const void* p, int layout, int B, int C, const int* ext, int nd) {
  RealView v;
  v.ptr = p;
  long long vol = 1;
  for (int d = 0; d < nd; ++d) vol *= ext[d];
  if (layout == HYFFT_LAYOUT_BHL) {
    v.bst = (long long)C * vol;
    v.cst = vol;
    long long s = 1;
    for (int d = nd - 1; d >= 0; --d) { v.sst[d] = s; s *= ext[d]; }
  } else {
    v.bst = (long long)C * vol;
    v.cst = 1;
    long long s = C;
    for (int d = nd - 1; d >= 0; --d) { v.sst[d] = s; s *= ext[d]; }
  }
  (void)B;
  return v;
}

static RealView offset_channels(RealView v, int c0, int elem_bytes) {
  v.ptr = static_cast<const char*>(v.ptr) + (long long)c0 * v.cst * elem_bytes;
  return v;
}

static int dtype_bytes(int dt) { return dt == HYFFT_F32 ? 4 : 2; }

// ------------------------------------------------------------------ pass launch
template <int IM, int OM, typename TI, typename TO>
static int launch_pass_t(const PassDesc& d, cudaStream_t st) {
  const long long grid = (d.nlines + d.TL - 1) / d.TL;
  if (grid <= 0) return HYFFT_OK;
  if (grid > 0x7fffffffLL) return fail(HYFFT_ERR_UNSUPPORTED, "too many FFT lines");
  const size_t smem =
      (size_t)kLineBytes + sizeof(float2) * ((size_t)d.TL * pass_ld(d.F) + (size_t)(d.F / 2));
  if (smem > 48 * 1024 && !kernel_smem_once((const void*)fft_pass_kernel<IM, OM, TI, TO>, smem))
    return fail(HYFFT_ERR_CUDA, "fft_pass_kernel: cannot allow %zu bytes of shared memory", smem);
  fft_pass_kernel<IM, OM, TI, TO><<<(unsigned)grid, kPassThreads, smem, st>>>(d);
  return check_launch("fft_pass_kernel");
}

template <int IM, int OM>
static int launch_pass_dt(const PassDesc& d, int tin, int tout, cudaStream_t st) {
  // only the real side's dtype matters; complex-only passes use float
  if (IM == IN_REAL && OM != OUT_CPLX) {  // fused product pass from a real source to a real output
    if (tin == HYFFT_F32) return launch_pass_t<IM, OM, float, float>(d, st);
    if (tin == HYFFT_BF16) return launch_pass_t<IM, OM, __nv_bfloat16, __nv_bfloat16>(d, st);
    return launch_pass_t<IM, OM, __half, __half>(d, st);
  }
  if (IM == IN_REAL) {
    if (tin == HYFFT_F32) return launch_pass_t<IM, OM, float, float>(d, st);
    if (tin == HYFFT_BF16) return launch_pass_t<IM, OM, __nv_bfloat16, float>(d, st);
    return launch_pass_t<IM, OM, __half, float>(d, st);
  }
  if (OM != OUT_CPLX) {
    if (tout == HYFFT_F32) return launch_pass_t<IM, OM, float, float>(d, st);
    if (tout == HYFFT_BF16) return launch_pass_t<IM, OM, float, __nv_bfloat16>(d, st);
    return launch_pass_t<IM, OM, float, __half>(d, st);
  }
  return launch_pass_t<IM, OM, float, float>(d, st);
}

// Passes with F = 32 .. 256, no four-step twiddle and channel-innermost lines (complex
// spectra, channels-last activations) run on the two-level kernel (fft_lines_cl_kernel).
template <int R1, int R2, int MID, int DIR, int IM, int OM, typename TI, typename TO, bool TMAJ = false>
static int launch_cl_t(const PassDesc& d, cudaStream_t st) {
  constexpr int F = R1 * R2;
  const long long grid = (d.nlines + cl_lines_per_cta<F>() - 1) / cl_lines_per_cta<F>();
  if (grid <= 0) return HYFFT_OK;
  if (grid > 0x7fffffffLL) return fail(HYFFT_ERR_UNSUPPORTED, "too many FFT lines");
  constexpr size_t smem = cl_smem_bytes<F>();
  auto kern = fft_lines_cl_kernel<R1, R2, MID, DIR, IM, OM, TI, TO, TMAJ>;
  if (smem > 48 * 1024 && !kernel_smem_once((const void*)kern, smem))
    return fail(HYFFT_ERR_CUDA, "fft_lines_cl_kernel: cannot allow %zu bytes of shared memory", smem);
  kern<<<(unsigned)grid, kClWarps * 32, smem, st>>>(d);
  return check_launch("fft_lines_cl_kernel");
}
template <int R1, int R2>
static int launch_cl_f(const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st) {
  using bf = __nv_bfloat16;
  if (im == IN_CPLX && om == OUT_CPLX) {
    if (d.mid == 1) return launch_cl_t<R1, R2, 1, -1, IN_CPLX, OUT_CPLX, float, float>(d, st);
    if (d.mid == 2) return launch_cl_t<R1, R2, 2, -1, IN_CPLX, OUT_CPLX, float, float>(d, st);
    if (d.dir < 0) return launch_cl_t<R1, R2, 0, -1, IN_CPLX, OUT_CPLX, float, float>(d, st);
    return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_CPLX, float, float>(d, st);
  }
  if (im == IN_REAL) {  // forward transform of an activation or filter
    if (d.ri_cst != 1) {  // channel-major source: lines staged t-fastest
      if (tin == HYFFT_BF16) return launch_cl_t<R1, R2, 0, -1, IN_REAL, OUT_CPLX, bf, float, true>(d, st);
      return launch_cl_t<R1, R2, 0, -1, IN_REAL, OUT_CPLX, float, float, true>(d, st);
    }
    if (tin == HYFFT_BF16) return launch_cl_t<R1, R2, 0, -1, IN_REAL, OUT_CPLX, bf, float>(d, st);
    return launch_cl_t<R1, R2, 0, -1, IN_REAL, OUT_CPLX, float, float>(d, st);
  }
  if (d.ro_cst != 1) {  // channel-major destination: lines stored t-fastest
    if (om == OUT_REAL) {
      if (tout == HYFFT_BF16) return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL, float, bf, true>(d, st);
      return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL, float, float, true>(d, st);
    }
    if (tout == HYFFT_BF16) return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL_SKIP, float, bf, true>(d, st);
    return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL_SKIP, float, float, true>(d, st);
  }
  if (om == OUT_REAL) {  // inverse transform into an activation
    if (tout == HYFFT_BF16) return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL, float, bf>(d, st);
    return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL, float, float>(d, st);
  }
  if (tout == HYFFT_BF16) return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL_SKIP, float, bf>(d, st);
  return launch_cl_t<R1, R2, 0, 1, IN_CPLX, OUT_REAL_SKIP, float, float>(d, st);
}
static int launch_cl(const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st) {
  switch (d.F) {
    case 32: return launch_cl_f<8, 4>(d, im, om, tin, tout, st);
    case 64: return launch_cl_f<16, 4>(d, im, om, tin, tout, st);
    case 128: return launch_cl_f<16, 8>(d, im, om, tin, tout, st);
    default: return launch_cl_f<16, 16>(d, im, om, tin, tout, st);
  }
}
static bool cl_pass_applies(const PassDesc& d, int im, int om, int tin, int tout) {
  if (d.tw_logF != 0 || !(d.F == 32 || d.F == 64 || d.F == 128 || d.F == 256) || getenv("HYFFT_DISABLE_CL_PASS"))
    return false;
  if (im == IN_CPLX && om == OUT_CPLX) return true;
  if (d.mid || d.pos_mul != 1 || d.pos_oth != 0 || getenv("HYFFT_DISABLE_CL_REAL")) return false;
  // real side: channels-last (neighbouring lines are neighbouring channels) or channel-major
  // with unit stride along the line (staged t-fastest through shared memory)
  if (im == IN_REAL)
    return om == OUT_CPLX && d.dir < 0 && (d.ri_cst == 1 || (d.ri_tst == 1 && !getenv("HYFFT_DISABLE_CL_TMAJ"))) &&
           (tin == HYFFT_F32 || tin == HYFFT_BF16);
  return im == IN_CPLX && d.dir > 0 && (d.ro_cst == 1 || (d.ro_tst == 1 && !getenv("HYFFT_DISABLE_CL_TMAJ"))) &&
         (tout == HYFFT_F32 || tout == HYFFT_BF16);
}

template <int R1, int R2>
static int launch_cl_bwd_t(const PassDesc& fx, const PassDesc& fdy, const PassDesc& idx, const PassDesc& idk, int pl,
                           cudaStream_t st) {
  constexpr int F = R1 * R2;
  const long long nl = fx.nlines / pl;
  const long long grid = (nl + cl_lines_per_cta<F>() - 1) / cl_lines_per_cta<F>();
  if (grid <= 0) return HYFFT_OK;
  if (grid > 0x7fffffffLL) return fail(HYFFT_ERR_UNSUPPORTED, "too many FFT lines");
  constexpr size_t smem = cl_bwd_smem_bytes<R1, R2>();
  if (smem > 48 * 1024 && !kernel_smem_once((const void*)fft_lines_cl_bwd_kernel<R1, R2>, smem))
    return fail(HYFFT_ERR_CUDA, "fft_lines_cl_bwd_kernel: cannot allow %zu bytes of shared memory", smem);
  fft_lines_cl_bwd_kernel<R1, R2><<<(unsigned)grid, kClWarps * 32, smem, st>>>(fx, fdy, idx, idk, pl);
  return check_launch("fft_lines_cl_bwd_kernel");
}
static int launch_cl_bwd(const PassDesc& fx, const PassDesc& fdy, const PassDesc& idx, const PassDesc& idk, int pl,
                         cudaStream_t st) {
  switch (fx.F) {
    case 32: return launch_cl_bwd_t<8, 4>(fx, fdy, idx, idk, pl, st);
    case 64: return launch_cl_bwd_t<16, 4>(fx, fdy, idx, idk, pl, st);
    case 128: return launch_cl_bwd_t<16, 8>(fx, fdy, idx, idk, pl, st);
    default: return launch_cl_bwd_t<16, 16>(fx, fdy, idx, idk, pl, st);
  }
}

// Long-line channel-innermost passes (fft_long.cu) take the four-step passes and every pass
// longer than the two-level kernel's 256 points.
static int launch_pass(const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st) {
  if ((d.tw_logF != 0 || d.F > 256) && long_pass_applies(d, im, om, tin, tout)) {
    const int rc = launch_long_pass(d, im, om, tin, tout, st);
    if (rc != HYFFT_ERR_UNSUPPORTED) return rc == HYFFT_OK ? rc : fail(rc, "fft_long_cl_kernel launch failed");
  }
  if (cl_pass_applies(d, im, om, tin, tout)) return launch_cl(d, im, om, tin, tout, st);
  if (im == IN_REAL && om == OUT_CPLX) return launch_pass_dt<IN_REAL, OUT_CPLX>(d, tin, tout, st);
  if (im == IN_REAL && om == OUT_REAL) return launch_pass_dt<IN_REAL, OUT_REAL>(d, tin, tout, st);
  if (im == IN_REAL && om == OUT_REAL_SKIP) return launch_pass_dt<IN_REAL, OUT_REAL_SKIP>(d, tin, tout, st);
  if (im == IN_CPLX && om == OUT_CPLX) return launch_pass_dt<IN_CPLX, OUT_CPLX>(d, tin, tout, st);
  if (im == IN_CPLX && om == OUT_REAL) return launch_pass_dt<IN_CPLX, OUT_REAL>(d, tin, tout, st);
  if (im == IN_CPLX && om == OUT_REAL_SKIP) return launch_pass_dt<IN_CPLX, OUT_REAL_SKIP>(d, tin, tout, st);
  return fail(HYFFT_ERR_INVALID, "unsupported pass mode");
}

static void base_desc(PassDesc& d, int F, float dir, int P, int C) {
  memset(&d, 0, sizeof(d));
  d.F = F;
  d.logF = ilog2(F);
  d.dir = dir;
  d.scale = dir > 0 ? 1.0f / (float)F : 1.0f;
  d.TL = std::min(kPassMaxLines, std::max(1, kPassPoints / F));
  d.P = P;
  d.C = C;
  d.pos_mul = 1;
  d.pos_oth = 0;
  d.oth_ext[0] = d.oth_ext[1] = 1;
}

static void finish_lines(PassDesc& d) {
  long long n = (long long)d.P * d.C;
  for (int a = 0; a < d.n_oth; ++a) n *= d.oth_ext[a];
  d.nlines = n;
}

// Spectrum strides for [pair][F_0..F_{D-1}][C].
struct SpecStrides {
  long long st[3];
  long long pst;
};
static SpecStrides spec_strides(const Geo& g, int C, bool half = false) {
  SpecStrides s;
  long long acc = C;
  for (int d = g.D - 1; d >= 0; --d) {
    s.st[d] = acc;
    acc *= (half && d == g.D - 1) ? g.F[d] / 2 + 1 : g.F[d];
  }
  s.pst = acc;
  return s;
}

struct Pairing {
  int P;       // number of complex signals per channel
  int B;       // number of real items
  int half;    // item p pairs with p + half
  int packed;
};
static Pairing pairing(int B, bool pack) {
  Pairing pr;
  pr.B = B;
  pr.packed = pack ? 1 : 0;
  pr.half = pack ? (B + 1) / 2 : B;
  pr.P = pr.half;
  return pr;
}

static void set_real_in(PassDesc& d, const RealView& v, const Pairing& pr) {
  d.rin = v.ptr;
  d.ri_bst = v.bst;
  d.ri_cst = v.cst;
  d.B = pr.B;
  d.half = pr.half;
  d.packed = pr.packed;
}
static void set_real_out(PassDesc& d, const RealView& v, const Pairing& pr) {
  d.rout = const_cast<void*>(v.ptr);
  d.ro_bst = v.bst;
  d.ro_cst = v.cst;
  d.B = pr.B;
  d.half = pr.half;
  d.packed = pr.packed;
}

// A chain of passes can be recorded instead of launched, so that the last forward pass
// and the first inverse pass of a convolution can be merged into one product pass.
struct PassRec {
  PassDesc d;
  int im, om, tin, tout;
};
struct PassList {
  PassRec r[4];
  int n = 0;
};
static int emit_pass(PassList* rec, const PassDesc& d, int im, int om, int tin, int tout, cudaStream_t st) {
  if (!rec) return launch_pass(d, im, om, tin, tout, st);
  if (rec->n >= 4) return fail(HYFFT_ERR_INVALID, "pass list overflow");
  rec->r[rec->n++] = PassRec{d, im, om, tin, tout};
  return HYFFT_OK;
}

// Forward transform of a real source (extents E, placed at offsets off) into the
// full spectrum S. Channels [0, C) of the view.
// half (a real filter, D >= 2): keep only bins [0, F/2] of the last axis (Hermitian symmetry).
static int fwd_chain(const Geo& g, int C, const RealView& src, int tdt, const Pairing& pr, const int* E,
                     const int* off, float2* S, cudaStream_t st, PassList* rec = nullptr, bool half = false) {
  const SpecStrides ss = spec_strides(g, C, half);
  const int FL = half ? g.F[g.D - 1] / 2 + 1 : g.F[g.D - 1];  // stored bins of the last axis
  if (g.four) {
    // pass A: along n_a (stride Fb*C in S), lines (p, n_b, c); twiddle e^{-2 pi i k_a n_b / F}
    PassDesc a;
    base_desc(a, g.Fa, -1.f, pr.P, C);
    a.n_oth = 1;
    a.oth_ext[0] = g.Fb;
    a.cout = S;
    a.co_pst = ss.pst;
    a.co_tst = (long long)g.Fb * C;
    a.co_ost[0] = C;
    set_real_in(a, src, pr);
    a.ri_tst = src.sst[0];
    a.pos_mul = g.Fb;
    a.pos_oth = 1;
    a.in_off = off[0];
    a.n_in = E[0];
    a.out_lo = 0;
    a.n_out = g.Fa;
    a.tw_logF = ilog2(g.F[0]);
    a.load_t_fastest = 0;
    a.store_t_fastest = 0;
    finish_lines(a);
    HY_TRY(emit_pass(rec, a, IN_REAL, OUT_CPLX, tdt, HYFFT_F32, st));
    // pass B: along n_b (stride C), lines (p, k_a, c)
    PassDesc b;
    base_desc(b, g.Fb, -1.f, pr.P, C);
    b.n_oth = 1;
    b.oth_ext[0] = g.Fa;
    b.cin = S;
    b.cout = S;
    b.ci_pst = b.co_pst = ss.pst;
    b.ci_tst = b.co_tst = C;
    b.ci_ost[0] = b.co_ost[0] = (long long)g.Fb * C;
    b.in_off = 0;
    b.n_in = g.Fb;
    b.out_lo = 0;
    b.n_out = g.Fb;
    finish_lines(b);
    return emit_pass(rec, b, IN_CPLX, OUT_CPLX, tdt, HYFFT_F32, st);
  }
  const int D = g.D;
  // last axis from the real source
  {
    PassDesc a;
    base_desc(a, g.F[D - 1], -1.f, pr.P, C);
    a.n_oth = D - 1;
    for (int e = 0; e < D - 1; ++e) {
      a.oth_ext[e] = E[e];
      a.co_ost[e] = ss.st[e];
      a.ri_ost[e] = src.sst[e];
    }
    a.cout = S;
    a.co_pst = ss.pst;
    a.co_tst = ss.st[D - 1];
    set_real_in(a, src, pr);
    a.ri_tst = src.sst[D - 1];
    a.in_off = off[D - 1];
    a.n_in = E[D - 1];
    a.out_lo = 0;
    a.n_out = FL;
    a.load_t_fastest = (src.sst[D - 1] == 1) ? 1 : 0;
    a.store_t_fastest = 0;
    finish_lines(a);
    HY_TRY(emit_pass(rec, a, IN_REAL, OUT_CPLX, tdt, HYFFT_F32, st));
  }
  for (int d = D - 2; d >= 0; --d) {
    PassDesc a;
    base_desc(a, g.F[d], -1.f, pr.P, C);
    a.n_oth = D - 1;
    int j = 0;
    for (int e = 0; e < D; ++e) {
      if (e == d) continue;
      a.oth_ext[j] = e < d ? E[e] : (e == D - 1 ? FL : g.F[e]);
      a.ci_ost[j] = a.co_ost[j] = ss.st[e];
      ++j;
    }
    a.cin = S;
    a.cout = S;
    a.ci_pst = a.co_pst = ss.pst;
    a.ci_tst = a.co_tst = ss.st[d];
    a.in_off = off[d];
    a.n_in = E[d];
    a.out_lo = 0;
    a.n_out = g.F[d];
    finish_lines(a);
    HY_TRY(emit_pass(rec, a, IN_CPLX, OUT_CPLX, HYFFT_F32, HYFFT_F32, st));
  }
  return HYFFT_OK;
}

struct Epilogue {
  int mode = OUT_REAL;     // OUT_REAL or OUT_REAL_SKIP
  const void* skip = nullptr;
  const float* Dv = nullptr;
};

// Inverse transform of the full spectrum S into a real destination, keeping the
// window [lo[d], lo[d] + cnt[d]) of every axis.
static int inv_chain(const Geo& g, int C, float2* S, const RealView& dst, int tdt, const Pairing& pr, const int* lo,
                     const int* cnt, const Epilogue& ep, cudaStream_t st, PassList* rec = nullptr) {
  const SpecStrides ss = spec_strides(g, C);
  if (g.four) {
    PassDesc b;  // along k_b with twiddle e^{+2 pi i n_b k_a / F}
    base_desc(b, g.Fb, +1.f, pr.P, C);
    b.n_oth = 1;
    b.oth_ext[0] = g.Fa;
    b.cin = S;
    b.cout = S;
    b.ci_pst = b.co_pst = ss.pst;
    b.ci_tst = b.co_tst = C;
    b.ci_ost[0] = b.co_ost[0] = (long long)g.Fb * C;
    b.in_off = 0;
    b.n_in = g.Fb;
    b.out_lo = 0;
    b.n_out = g.Fb;
    b.tw_logF = ilog2(g.F[0]);
    finish_lines(b);
    HY_TRY(emit_pass(rec, b, IN_CPLX, OUT_CPLX, HYFFT_F32, HYFFT_F32, st));
    PassDesc a;  // along k_a into the real output, position n_a * Fb + n_b
    base_desc(a, g.Fa, +1.f, pr.P, C);
    a.n_oth = 1;
    a.oth_ext[0] = g.Fb;
    a.cin = S;
    a.ci_pst = ss.pst;
    a.ci_tst = (long long)g.Fb * C;
    a.ci_ost[0] = C;
    a.in_off = 0;
    a.n_in = g.Fa;
    set_real_out(a, dst, pr);
    a.ro_tst = dst.sst[0];
    a.pos_mul = g.Fb;
    a.pos_oth = 1;
    a.out_lo = lo[0];
    a.n_out = cnt[0];
    a.skip = ep.skip;
    a.Dv = ep.Dv;
    a.load_t_fastest = 0;
    a.store_t_fastest = 0;
    finish_lines(a);
    return emit_pass(rec, a, IN_CPLX, ep.mode, HYFFT_F32, tdt, st);
  }
  const int D = g.D;
  for (int d = 0; d < D - 1; ++d) {
    PassDesc a;
    base_desc(a, g.F[d], +1.f, pr.P, C);
    a.n_oth = D - 1;
    int j = 0;
    for (int e = 0; e < D; ++e) {
      if (e == d) continue;
      a.oth_ext[j] = e < d ? cnt[e] : g.F[e];
      a.ci_ost[j] = a.co_ost[j] = ss.st[e];
      ++j;
    }
    a.cin = S;
    a.cout = S;
    a.ci_pst = a.co_pst = ss.pst;
    a.ci_tst = a.co_tst = ss.st[d];
    a.in_off = 0;
    a.n_in = g.F[d];
    a.out_lo = lo[d];
    a.n_out = cnt[d];
    finish_lines(a);
    HY_TRY(emit_pass(rec, a, IN_CPLX, OUT_CPLX, HYFFT_F32, HYFFT_F32, st));
  }
  PassDesc a;
  base_desc(a, g.F[D - 1], +1.f, pr.P, C);
  a.n_oth = D - 1;
  for (int e = 0; e < D - 1; ++e) {
    a.oth_ext[e] = cnt[e];
    a.ci_ost[e] = ss.st[e];
    a.ro_ost[e] = dst.sst[e];
  }
  a.cin = S;
  a.ci_pst = ss.pst;
  a.ci_tst = ss.st[D - 1];
  a.in_off = 0;
  a.n_in = g.F[D - 1];
  set_real_out(a, dst, pr);
  a.ro_tst = dst.sst[D - 1];
  a.out_lo = lo[D - 1];
  a.n_out = cnt[D - 1];
  a.skip = ep.skip;
  a.Dv = ep.Dv;
  a.load_t_fastest = 0;
  a.store_t_fastest = (dst.sst[D - 1] == 1) ? 1 : 0;
  finish_lines(a);
  return emit_pass(rec, a, IN_CPLX, ep.mode, HYFFT_F32, tdt, st);
}

static int grid_for(long long n, int threads = 256) {
  long long g = (n + threads - 1) / threads;
  return (int)std::max<long long>(1, std::min<long long>(g, 148LL * 16));
}

// ------------------------------------------------------------------ conv plan
struct ConvPlan {
  Geo g;
  int B = 0, C = 0, kB = 1, dt = HYFFT_F32, layout = HYFFT_LAYOUT_BHL;
  bool shared = true;
  Pairing px, pk;
  int Cc = 0;  // channels per chunk
  long long spec_x_bytes_per_ch = 0, spec_k_bytes_per_ch = 0;
  bool big2d = false;  // fused large-grid 2D kernels (big2d.cu) instead of the pass chain
  int b2F = 0;         // their FFT length per axis (192 or 256)
  bool khalf = false;  // the filter spectrum keeps bins [0, F/2] of the last axis only (product passes
                       // of 2D / 3D convolutions read the other half mirrored and conjugated)
};

static size_t ws_budget() {
  const char* e = getenv("HYFFT_WS_BUDGET_MB");
  long long mb = e ? atoll(e) : 16384;
  if (mb < 64) mb = 64;
  return (size_t)mb << 20;
}

// allow_big2d = false plans the pass chain even for shapes the large-grid 2D kernels
// would take (the static-scratch forward runs only the chunked pass chain).
static int make_conv_plan(const hyfft_conv_desc* d, ConvPlan& p, bool allow_big2d = true) {
  if (!d) return fail(HYFFT_ERR_INVALID, "null descriptor");
  HY_TRY(make_geo(d->ndim, d->n, d->k, d->causal, d->periodic, p.g));
  if (d->batch < 1 || d->channels < 1) return fail(HYFFT_ERR_INVALID, "batch and channels must be positive");
  if (d->kernel_batch != 1 && d->kernel_batch != d->batch)
    return fail(HYFFT_ERR_INVALID, "kernel_batch must be 1 or batch (%d), got %d", d->batch, d->kernel_batch);
  if (d->dtype < HYFFT_F32 || d->dtype > HYFFT_F16) return fail(HYFFT_ERR_INVALID, "bad dtype");
  if (d->layout != HYFFT_LAYOUT_BHL && d->layout != HYFFT_LAYOUT_BLH) return fail(HYFFT_ERR_INVALID, "bad layout");
  p.B = d->batch;
  p.C = d->channels;
  p.kB = d->kernel_batch;
  p.dt = d->dtype;
  p.layout = d->layout;
  p.shared = (p.kB == 1);
  p.px = pairing(p.B, p.shared);
  p.pk = pairing(p.kB, false);
  p.spec_x_bytes_per_ch = (long long)p.px.P * p.g.vol_F * 8;
  p.spec_k_bytes_per_ch = (long long)p.pk.P * p.g.vol_F * 8;
  // bwd holds 2 activation spectra + 2 kernel spectra per channel
  const long long per_ch = 2 * (p.spec_x_bytes_per_ch + p.spec_k_bytes_per_ch);
  long long cc = (long long)(ws_budget() / (size_t)std::max<long long>(per_ch, 1));
  p.Cc = (int)std::max<long long>(1, std::min<long long>(cc, p.C));
  p.big2d = allow_big2d && !p.g.periodic && p.g.D == 2 && !d->causal && p.g.F[0] == kB2F && p.g.F[1] == kB2F && p.g.N[0] <= kB2MaxN &&
            p.g.N[1] <= kB2MaxN && p.kB == 1 && !getenv("HYFFT_DISABLE_BIG2D");
  if (p.big2d) {
    // the circular convolution of length F equals the linear one on the output window
    // [0, N) while F >= N + ceil(K/2) - 1 (no tap offset of another output wraps onto a
    // tap): 192 covers the 128 x 128 grid with a 128 x 128 filter
    bool short_ok = !getenv("HYFFT_B2_F256");
    for (int a = 0; a < 2; ++a)
      short_ok = short_ok && p.g.N[a] + (p.g.K[a] + 1) / 2 - 1 <= kB2FShort && p.g.K[a] <= kB2FShort;
    p.b2F = short_ok ? kB2FShort : kB2F;
  }
  const int F0 = p.g.F[0];
  p.khalf = p.g.D >= 2 && !p.g.four && !p.big2d && (F0 == 32 || F0 == 64 || F0 == 128 || F0 == 256) &&
            p.g.F[p.g.D - 1] % 2 == 0 && !getenv("HYFFT_DISABLE_CL_PASS") && !getenv("HYFFT_DISABLE_PRODUCT_PASS") &&
            !getenv("HYFFT_FULL_KSPEC");
  return HYFFT_OK;
}

static size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

// One [C][F/2+1][F] complex spectrum of the large-grid 2D kernels.
static size_t big2d_spec_bytes(const ConvPlan& p) {
  return align_up((size_t)p.C * (p.b2F / 2 + 1) * p.b2F * sizeof(float2));
}

static void conv_ws_sizes(const ConvPlan& p, size_t& fwd, size_t& bwd) {
  if (p.big2d) {  // Kh, T (+ G for the backward), then the float shortcut vector
    const size_t spec = big2d_spec_bytes(p), dvec = align_up((size_t)p.C * 4);
    fwd = 2 * spec + dvec;
    bwd = 3 * spec + dvec;
    return;
  }
  const size_t sx = align_up((size_t)p.spec_x_bytes_per_ch * p.Cc);
  const size_t sk = align_up((size_t)p.spec_k_bytes_per_ch * p.Cc);
  const size_t dvec = align_up((size_t)p.C * 4);
  fwd = sx + sk + dvec;
  bwd = 2 * sx + 2 * sk + dvec;
}

template <typename T>
__global__ void to_float_kernel(const T* __restrict__ s, float* __restrict__ d, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) d[i] = DT<T>::load(s + i);
}

static int to_float(const void* src, int dt, float* dst, int n, cudaStream_t st) {
  const int gr = (n + 255) / 256;
  if (dt == HYFFT_F32) to_float_kernel<float><<<gr, 256, 0, st>>>((const float*)src, dst, n);
  else if (dt == HYFFT_BF16) to_float_kernel<__nv_bfloat16><<<gr, 256, 0, st>>>((const __nv_bfloat16*)src, dst, n);
  else to_float_kernel<__half><<<gr, 256, 0, st>>>((const __half*)src, dst, n);
  return check_launch("to_float_kernel");
}

// Forward transform of x, product with the kernel spectrum Kh (conjugated if conj) and
// inverse transform into y, with the last forward pass and the first inverse pass (both
// along the same axis, over the same lines) merged into one product pass, so the full
// spectrum is neither written by the one nor re-read by the other. Returns
// HYFFT_ERR_UNSUPPORTED (nothing launched) if the two passes do not line up.
static int fused_conv_chain(const Geo& g, int Cc, const RealView& xc, int tin, const Pairing& px, const int* E,
                            const int* off, float2* S, const float2* Kh, bool shared, int conj, const RealView& yc,
                            int tout, const int* lo, const int* cnt, const Epilogue& ep, cudaStream_t st,
                            bool khalf = false) {
  PassList fl, il;
  HY_TRY(fwd_chain(g, Cc, xc, tin, px, E, off, S, st, &fl));
  HY_TRY(inv_chain(g, Cc, S, yc, tout, px, lo, cnt, ep, st, &il));
  if (fl.n < 1 || il.n < 1) return HYFFT_ERR_UNSUPPORTED;
  const PassRec& f = fl.r[fl.n - 1];
  const PassRec& v = il.r[0];
  bool same = f.d.F == v.d.F && f.d.TL == v.d.TL && f.d.n_oth == v.d.n_oth && f.d.nlines == v.d.nlines &&
              f.d.P == v.d.P && f.d.C == v.d.C;
  for (int j = 0; j < f.d.n_oth; ++j) same = same && f.d.oth_ext[j] == v.d.oth_ext[j];
  if (f.im == IN_REAL && v.om != OUT_CPLX) same = same && f.d.pos_mul == v.d.pos_mul && f.d.pos_oth == v.d.pos_oth;
  if (!same) return HYFFT_ERR_UNSUPPORTED;
  for (int i = 0; i + 1 < fl.n; ++i) HY_TRY(launch_pass(fl.r[i].d, fl.r[i].im, fl.r[i].om, fl.r[i].tin, fl.r[i].tout, st));
  PassDesc m = f.d;  // load side of the last forward pass
  m.cout = v.d.cout;  // store side of the first inverse pass
  m.co_pst = v.d.co_pst;
  m.co_tst = v.d.co_tst;
  m.co_ost[0] = v.d.co_ost[0];
  m.co_ost[1] = v.d.co_ost[1];
  m.out_lo = v.d.out_lo;
  m.n_out = v.d.n_out;
  m.tw_logF = v.d.tw_logF;
  m.rout = v.d.rout;
  m.ro_bst = v.d.ro_bst;
  m.ro_cst = v.d.ro_cst;
  m.ro_tst = v.d.ro_tst;
  m.ro_ost[0] = v.d.ro_ost[0];
  m.ro_ost[1] = v.d.ro_ost[1];
  m.skip = v.d.skip;
  m.Dv = v.d.Dv;
  m.store_t_fastest = v.d.store_t_fastest;
  m.scale = v.d.scale;
  m.mid = conj ? 2 : 1;
  m.kin = Kh;
  m.k_shared = shared ? 1 : 0;
  m.k_pst = spec_strides(g, Cc, khalf).pst;
  if (f.im == IN_CPLX && khalf) {  // 2D / 3D lines along axis 0; the other axes 1 .. D-1 in order
    const SpecStrides ks = spec_strides(g, Cc, true);
    m.k_tst = ks.st[0];
    m.k_ost[0] = g.D > 1 ? ks.st[1] : 0;
    m.k_ost[1] = g.D > 2 ? ks.st[2] : 0;
    m.k_half = 1;
  } else if (f.im == IN_CPLX) {  // the filter spectrum has the signal spectrum's layout
    m.k_tst = f.d.ci_tst;
    m.k_ost[0] = f.d.ci_ost[0];
    m.k_ost[1] = f.d.ci_ost[1];
  } else {
    m.k_tst = f.d.co_tst;
    m.k_ost[0] = f.d.co_ost[0];
    m.k_ost[1] = f.d.co_ost[1];
  }
  HY_TRY(launch_pass(m, f.im, v.om, f.tin, v.tout, st));
  for (int i = 1; i < il.n; ++i) HY_TRY(launch_pass(il.r[i].d, il.r[i].im, il.r[i].om, il.r[i].tin, il.r[i].tout, st));
  return HYFFT_OK;
}

// One forward convolution over channels [c0, c0 + Cc) of already-prepared views.
// Phase ramp of the periodic axes on a filter spectrum stored [pair][F...][C] (last axis
// F/2 + 1 bins when half; 1D four-step layout [pair][k_a][k_b][C], k = k_a + Fa k_b):
// S *= prod_d exp(sign * 2 pi i k_d rshift[d] / F[d]). sign +1 aligns the convolution
// output like the reference's roll by -rshift; sign -1 (the conjugate) maps the gradient
// of the rolled filter back to the filter's own taps.
struct RampDesc {
  int D, half, four, Fa, Fb;
  int F[3], r[3];
  long long C;
  float sign;
};

__global__ void spec_ramp_kernel(float2* __restrict__ S, const RampDesc d, long long total) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long rest = i / d.C;
    float2 w = make_float2(1.f, 0.f);
    if (d.four) {
      const long long kb = rest % d.Fb;
      const long long ka = (rest / d.Fb) % d.Fa;
      const long long F = (long long)d.Fa * d.Fb;
      const long long m = ((ka + (long long)d.Fa * kb) % F) * d.r[0] % F;
      float sn, cs;
      sincospif(2.0f * (float)m / (float)F, &sn, &cs);
      w = make_float2(cs, d.sign * sn);
    } else {
      for (int ax = d.D - 1; ax >= 0; --ax) {
        const int ext = (d.half && ax == d.D - 1) ? d.F[ax] / 2 + 1 : d.F[ax];
        const long long k = rest % ext;
        rest /= ext;
        if (d.r[ax] == 0) continue;
        const long long m = k * d.r[ax] % d.F[ax];
        float sn, cs;
        sincospif(2.0f * (float)m / (float)d.F[ax], &sn, &cs);
        w = cmul(w, make_float2(cs, d.sign * sn));
      }
    }
    S[i] = cmul(S[i], w);
  }
}

// Apply the periodic axes' phase ramp to a filter(-gradient) spectrum of Cc channels.
static int apply_ramp(const ConvPlan& p, float2* S, int Cc, bool half, float sign, cudaStream_t st) {
  if (!p.g.periodic) return HYFFT_OK;
  RampDesc d;
  d.D = p.g.D;
  d.half = half ? 1 : 0;
  d.four = p.g.four ? 1 : 0;
  d.Fa = p.g.Fa;
  d.Fb = p.g.Fb;
  bool any = false;
  long long vol = 1;
  for (int a = 0; a < 3; ++a) {
    d.F[a] = p.g.F[a];
    d.r[a] = (p.g.periodic & (1 << a)) ? p.g.rshift[a] : 0;
    any = any || d.r[a] != 0;
  }
  if (!any) return HYFFT_OK;
  for (int a = 0; a < p.g.D; ++a) vol *= (half && a == p.g.D - 1) ? p.g.F[a] / 2 + 1 : p.g.F[a];
  d.C = Cc;
  d.sign = sign;
  const long long total = (long long)p.pk.P * vol * Cc;
  spec_ramp_kernel<<<grid_for(total), 256, 0, st>>>(S, d, total);
  return check_launch("spec_ramp_kernel");
}

template <typename T>
static int cl_cm(const T* src, T* dst, int B, long long N, int C, bool to_cm, cudaStream_t st);

// The long 1D (four-step) passes read and write channels-last real tensors with coalesced
// runs of channels. A channel-major filter chunk [kB][C][K] (float32) is therefore
// transposed to [kB][K][Cc] in a free spectrum buffer before its transform, and its
// gradient is written channels-last there and transposed back after the inverse.
static bool four_step_cl_filter(const ConvPlan& p, const RealView& kv) {
  return p.g.four && kv.cst != 1 && !getenv("HYFFT_DISABLE_LONG_PASS") && p.g.Fa >= 128 && p.g.Fa <= 4096;
}
static int filter_to_cl(const ConvPlan& p, const RealView& kc, int Cc, float* T, RealView& out, cudaStream_t st) {
  const long long K = p.g.K[0];
  for (int b = 0; b < p.kB; ++b)
    HY_TRY(cl_cm<float>((const float*)kc.ptr + b * kc.bst, T + (size_t)b * K * Cc, 1, K, Cc, false, st));
  out = real_view(T, HYFFT_LAYOUT_BLH, p.kB, Cc, p.g.K, 1);
  return HYFFT_OK;
}
static int filter_from_cl(const ConvPlan& p, const float* T, int Cc, const RealView& dkc, cudaStream_t st) {
  const long long K = p.g.K[0];
  for (int b = 0; b < p.kB; ++b)
    HY_TRY(cl_cm<float>(T + (size_t)b * K * Cc, (float*)const_cast<void*>(dkc.ptr) + b * dkc.bst, 1, K, Cc, true, st));
  return HYFFT_OK;
}

static int conv_forward_chunk(const ConvPlan& p, int c0, int Cc, const RealView& xv, const RealView& kv,
                              const float* Dfull, const RealView& yv, float2* S, float2* Kh, cudaStream_t st) {
  const int eb = dtype_bytes(p.dt);
  const RealView xc = offset_channels(xv, c0, eb);
  RealView kc = offset_channels(kv, c0, 4);
  const RealView yc = offset_channels(yv, c0, eb);
  const int zero[3] = {0, 0, 0};
  if (four_step_cl_filter(p, kv)) HY_TRY(filter_to_cl(p, kc, Cc, (float*)S, kc, st));  // S is free until z's pass
  HY_TRY(fwd_chain(p.g, Cc, kc, HYFFT_F32, p.pk, p.g.K, zero, Kh, st, nullptr, p.khalf));
  HY_TRY(apply_ramp(p, Kh, Cc, p.khalf, 1.f, st));
  Epilogue ep;
  if (Dfull) {
    ep.mode = OUT_REAL_SKIP;
    ep.skip = xc.ptr;
    ep.Dv = Dfull + c0;
  }
  const int rc = getenv("HYFFT_DISABLE_PRODUCT_PASS")
                     ? HYFFT_ERR_UNSUPPORTED
                     : fused_conv_chain(p.g, Cc, xc, p.dt, p.px, p.g.N, zero, S, Kh, p.shared, 0, yc, p.dt, p.g.crop,
                                        p.g.N, ep, st, p.khalf);
  if (rc != HYFFT_ERR_UNSUPPORTED) return rc;
  // the elementwise product below reads the full filter spectrum
  if (p.khalf) {
    HY_TRY(fwd_chain(p.g, Cc, kc, HYFFT_F32, p.pk, p.g.K, zero, Kh, st));
    HY_TRY(apply_ramp(p, Kh, Cc, false, 1.f, st));
  }
  HY_TRY(fwd_chain(p.g, Cc, xc, p.dt, p.px, p.g.N, zero, S, st));
  const long long per_pair = p.g.vol_F * Cc;
  spec_mul_kernel<<<grid_for(per_pair * p.px.P), 256, 0, st>>>(S, Kh, per_pair, p.px.P, p.shared ? 1 : 0);
  HY_TRY(check_launch("spec_mul_kernel"));
  return inv_chain(p.g, Cc, S, yc, p.dt, p.px, p.g.crop, p.g.N, ep, st);
}

// Backward with the last forward passes of x and dy, the spectral products and the first
// inverse passes of dx and dK merged into one backward product pass (complex passes of
// 32..256 points along the first axis, 2D / 3D). Returns HYFFT_ERR_UNSUPPORTED (nothing
// launched) when the passes do not line up.
static int fused_bwd_chain(const ConvPlan& p, int Cc, const RealView& xc, const RealView& dyc, const RealView& dxc,
                           const RealView& dkc, const Epilogue& ep, float2* S1, float2* S2, const float2* Kh,
                           float2* dKh, cudaStream_t st) {
  const int zero[3] = {0, 0, 0};
  if (getenv("HYFFT_DISABLE_BWD_PASS") || p.g.four || p.g.D < 2) return HYFFT_ERR_UNSUPPORTED;
  PassList fx, fy, ix, ik;
  HY_TRY(fwd_chain(p.g, Cc, xc, p.dt, p.px, p.g.N, zero, S1, st, &fx));
  HY_TRY(fwd_chain(p.g, Cc, dyc, p.dt, p.px, p.g.N, p.g.crop, S2, st, &fy));
  HY_TRY(inv_chain(p.g, Cc, S2, dxc, p.dt, p.px, zero, p.g.N, ep, st, &ix));
  Epilogue none;
  HY_TRY(inv_chain(p.g, Cc, dKh, dkc, HYFFT_F32, p.pk, zero, p.g.K, none, st, &ik));
  if (fx.n < 2 || fy.n < 2 || ix.n < 2 || ik.n < 2) return HYFFT_ERR_UNSUPPORTED;
  PassDesc a = fx.r[fx.n - 1].d;
  const PassDesc& b = fy.r[fy.n - 1].d;
  const PassDesc& c = ix.r[0].d;
  const PassDesc& k = ik.r[0].d;
  const bool cplx = fx.r[fx.n - 1].im == IN_CPLX && fy.r[fy.n - 1].im == IN_CPLX && ix.r[0].om == OUT_CPLX &&
                    ik.r[0].om == OUT_CPLX;
  bool same = cplx && a.F == b.F && a.F == c.F && a.F == k.F && a.n_oth == c.n_oth && a.n_oth == k.n_oth &&
              a.nlines == b.nlines && a.nlines == c.nlines && a.tw_logF == 0 && c.tw_logF == 0 &&
              (a.F == 32 || a.F == 64 || a.F == 128 || a.F == 256);
  for (int j = 0; j < a.n_oth; ++j)
    same = same && a.oth_ext[j] == b.oth_ext[j] && a.oth_ext[j] == c.oth_ext[j] && a.oth_ext[j] == k.oth_ext[j];
  if (!same) return HYFFT_ERR_UNSUPPORTED;
  // Kh shares S's per-axis strides (the same [pair][F...][C] layout)
  a.kin = Kh;
  a.k_shared = p.shared ? 1 : 0;
  {
    const SpecStrides ks = spec_strides(p.g, Cc, p.khalf);
    a.k_pst = ks.pst;
    a.k_tst = ks.st[0];
    a.k_ost[0] = p.g.D > 1 ? ks.st[1] : 0;
    a.k_ost[1] = p.g.D > 2 ? ks.st[2] : 0;
    a.k_half = p.khalf ? 1 : 0;
  }
  const int pl = p.shared ? p.px.P : 1;
  for (int i = 0; i + 1 < fx.n; ++i) HY_TRY(launch_pass(fx.r[i].d, fx.r[i].im, fx.r[i].om, fx.r[i].tin, fx.r[i].tout, st));
  for (int i = 0; i + 1 < fy.n; ++i) HY_TRY(launch_pass(fy.r[i].d, fy.r[i].im, fy.r[i].om, fy.r[i].tin, fy.r[i].tout, st));
  HY_TRY(launch_cl_bwd(a, b, c, k, pl, st));
  for (int i = 1; i < ix.n; ++i) HY_TRY(launch_pass(ix.r[i].d, ix.r[i].im, ix.r[i].om, ix.r[i].tin, ix.r[i].tout, st));
  for (int i = 1; i < ik.n; ++i) HY_TRY(launch_pass(ik.r[i].d, ik.r[i].im, ik.r[i].om, ik.r[i].tin, ik.r[i].tout, st));
  return HYFFT_OK;
}

// Backward of a long 1D (four-step) convolution with the second-axis forward passes of x and
// dy, the spectral products and the second-axis inverse passes of dx and dK merged into one
// backward product pass (fft_long_bwd_kernel). fcl: the filter gradient is written
// channels-last into S1 (free once the merged pass has read it) and transposed into dkc.
// Returns HYFFT_ERR_UNSUPPORTED (nothing launched) when the lengths have no such pass.
static int long_bwd_chain(const ConvPlan& p, int Cc, const RealView& xc, const RealView& dyc, const RealView& dxc,
                          const RealView& dkc, const Epilogue& ep, float2* S1, float2* S2, const float2* Kh,
                          float2* dKh, bool fcl, cudaStream_t st) {
  const int zero[3] = {0, 0, 0};
  if (!p.g.four || p.g.periodic || p.g.Fb < 128 || p.g.Fb > 2048 || getenv("HYFFT_DISABLE_LONG_PASS") ||
      getenv("HYFFT_DISABLE_BWD_PASS"))
    return HYFFT_ERR_UNSUPPORTED;
  PassList fx, fy, ix, ik;
  HY_TRY(fwd_chain(p.g, Cc, xc, p.dt, p.px, p.g.N, zero, S1, st, &fx));
  HY_TRY(fwd_chain(p.g, Cc, dyc, p.dt, p.px, p.g.N, p.g.crop, S2, st, &fy));
  HY_TRY(inv_chain(p.g, Cc, S2, dxc, p.dt, p.px, zero, p.g.N, ep, st, &ix));
  Epilogue none;
  const RealView dk_dst = fcl ? real_view(S1, HYFFT_LAYOUT_BLH, p.kB, Cc, p.g.K, 1) : dkc;
  HY_TRY(inv_chain(p.g, Cc, dKh, dk_dst, HYFFT_F32, p.pk, zero, p.g.K, none, st, &ik));
  if (fx.n != 2 || fy.n != 2 || ix.n != 2 || ik.n != 2) return HYFFT_ERR_UNSUPPORTED;
  const PassDesc& b = fx.r[1].d;  // x's second-axis pass: lines (pair, k_a, c) along n_b
  LongBwdDesc d;
  d.sx = S1;
  d.sdy = S2;
  d.kh = Kh;
  d.dkh = dKh;
  d.pst = b.ci_pst;
  d.tst = b.ci_tst;
  d.ost = b.ci_ost[0];
  d.k_pst = p.shared ? 0 : b.ci_pst;
  d.pl = p.shared ? p.px.P : 1;
  d.nlines = (long long)(p.px.P / d.pl) * p.g.Fa * Cc;
  d.C = Cc;
  d.Fa = p.g.Fa;
  d.tw_logF = ix.r[0].d.tw_logF;
  d.scale = ix.r[0].d.scale;
  HY_TRY(launch_pass(fx.r[0].d, fx.r[0].im, fx.r[0].om, fx.r[0].tin, fx.r[0].tout, st));
  HY_TRY(launch_pass(fy.r[0].d, fy.r[0].im, fy.r[0].om, fy.r[0].tin, fy.r[0].tout, st));
  const int rc = launch_long_bwd(d, p.g.Fb, st);
  if (rc != HYFFT_OK) return fail(rc == HYFFT_ERR_UNSUPPORTED ? HYFFT_ERR_CUDA : rc, "fft_long_bwd_kernel launch failed");
  HY_TRY(launch_pass(ix.r[1].d, ix.r[1].im, ix.r[1].om, ix.r[1].tin, ix.r[1].tout, st));
  HY_TRY(launch_pass(ik.r[1].d, ik.r[1].im, ik.r[1].om, ik.r[1].tin, ik.r[1].tout, st));
  if (fcl) HY_TRY(filter_from_cl(p, (const float*)S1, Cc, dkc, st));
  return HYFFT_OK;
}

static int conv_backward_chunk(const ConvPlan& p, int c0, int Cc, const RealView& xv, const RealView& kv,
                               const float* Dfull, const RealView& dyv, const RealView& dxv, const RealView& dkv,
                               float2* S1, float2* S2, float2* Kh, float2* dKh, cudaStream_t st,
                               bool kh_ready = false) {
  const int eb = dtype_bytes(p.dt);
  const RealView xc = offset_channels(xv, c0, eb);
  RealView kc = offset_channels(kv, c0, 4);
  const RealView dyc = offset_channels(dyv, c0, eb);
  const int zero[3] = {0, 0, 0};
  const bool fcl = four_step_cl_filter(p, kv);
  if (!kh_ready) {
    if (fcl) HY_TRY(filter_to_cl(p, kc, Cc, (float*)S1, kc, st));  // S1 is free until x's pass
    HY_TRY(fwd_chain(p.g, Cc, kc, HYFFT_F32, p.pk, p.g.K, zero, Kh, st, nullptr, p.khalf));
    HY_TRY(apply_ramp(p, Kh, Cc, p.khalf, 1.f, st));
  }
  // (periodic axes: the filter gradient needs the conjugate ramp before its inverse, so
  // the merged backward pass, which inverts it in place, is not used)
  if (dxv.ptr && dkv.ptr && !p.g.periodic) {
    Epilogue ep;
    if (Dfull) {
      ep.mode = OUT_REAL_SKIP;
      ep.skip = dyc.ptr;
      ep.Dv = Dfull + c0;
    }
    const int rc = p.g.four ? long_bwd_chain(p, Cc, xc, dyc, offset_channels(dxv, c0, eb), offset_channels(dkv, c0, 4),
                                             ep, S1, S2, Kh, dKh, fcl, st)
                            : fused_bwd_chain(p, Cc, xc, dyc, offset_channels(dxv, c0, eb),
                                              offset_channels(dkv, c0, 4), ep, S1, S2, Kh, dKh, st);
    if (rc != HYFFT_ERR_UNSUPPORTED) return rc;
  }
  // the elementwise backward below reads the full filter spectrum
  if (p.khalf) {
    HY_TRY(fwd_chain(p.g, Cc, kc, HYFFT_F32, p.pk, p.g.K, zero, Kh, st));
    HY_TRY(apply_ramp(p, Kh, Cc, false, 1.f, st));
  }
  HY_TRY(fwd_chain(p.g, Cc, xc, p.dt, p.px, p.g.N, zero, S1, st));
  HY_TRY(fwd_chain(p.g, Cc, dyc, p.dt, p.px, p.g.N, p.g.crop, S2, st));
  const long long per_pair = p.g.vol_F * Cc;
  spec_bwd_kernel<<<grid_for(per_pair), 256, 0, st>>>(S2, S1, Kh, dKh, per_pair, p.px.P, p.shared ? 1 : 0);
  HY_TRY(check_launch("spec_bwd_kernel"));
  HY_TRY(apply_ramp(p, dKh, Cc, false, -1.f, st));
  if (dxv.ptr) {
    const RealView dxc = offset_channels(dxv, c0, eb);
    Epilogue ep;
    if (Dfull) {
      ep.mode = OUT_REAL_SKIP;
      ep.skip = dyc.ptr;
      ep.Dv = Dfull + c0;
    }
    HY_TRY(inv_chain(p.g, Cc, S2, dxc, p.dt, p.px, zero, p.g.N, ep, st));
  }
  if (dkv.ptr) {
    const RealView dkc = offset_channels(dkv, c0, 4);
    Epilogue ep;
    if (fcl) {  // channels-last into S1 (free since the spectral products), then transposed
      HY_TRY(inv_chain(p.g, Cc, dKh, real_view(S1, HYFFT_LAYOUT_BLH, p.kB, Cc, p.g.K, 1), HYFFT_F32, p.pk, zero,
                       p.g.K, ep, st));
      return filter_from_cl(p, (const float*)S1, Cc, dkc, st);
    }
    HY_TRY(inv_chain(p.g, Cc, dKh, dkc, HYFFT_F32, p.pk, zero, p.g.K, ep, st));
  }
  return HYFFT_OK;
}

static int run_dshortcut(int dt, int layout, const void* dy, const void* x, float* out, int B, int C, long long S,
                         cudaStream_t st) {
  const int blh = layout == HYFFT_LAYOUT_BLH;
  if (cudaMemsetAsync(out, 0, sizeof(float) * (size_t)C, st) != cudaSuccess) return fail(HYFFT_ERR_CUDA, "memset dshortcut");
  const dim3 gr = blh ? dim3((unsigned)((C + 31) / 32),
                             (unsigned)std::max<long long>(1, std::min<long long>(1200 / ((C + 31) / 32) + 1,
                                                                                  ((long long)B * S + 63) / 64)),
                             1)
                      : dim3((unsigned)C, (unsigned)B, 1);
  if (dt == HYFFT_F32) dshortcut_kernel<float><<<gr, 256, 0, st>>>((const float*)dy, (const float*)x, out, B, C, S, blh);
  else if (dt == HYFFT_BF16)
    dshortcut_kernel<__nv_bfloat16><<<gr, 256, 0, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, out, B, C, S, blh);
  else dshortcut_kernel<__half><<<gr, 256, 0, st>>>((const __half*)dy, (const __half*)x, out, B, C, S, blh);
  return check_launch("dshortcut_kernel");
}

// ---- large-grid 2D path: workspace = [Kh | T | G], all [C][F/2+1][F]-sized
static Big2DView b2view(const RealView& v) {
  Big2DView o;
  o.ptr = v.ptr;
  o.bst = v.bst;
  o.cst = v.cst;
  o.s0 = v.sst[0];
  o.s1 = v.sst[1];
  return o;
}

static void big2d_params(const ConvPlan& p, const RealView& kv, const float* D, char* ws, Big2DParams& b) {
  memset(&b, 0, sizeof(b));
  const size_t spec = big2d_spec_bytes(p);
  b.filt = b2view(kv);
  b.D = D;
  b.Kh = (float2*)ws;
  b.T = (float2*)(ws + spec);
  b.G = (float2*)(ws + 2 * spec);
  b.F = p.b2F;
  b.B = p.B;
  b.C = p.C;
  b.N0 = p.g.N[0];
  b.N1 = p.g.N[1];
  b.K0 = p.g.K[0];
  b.K1 = p.g.K[1];
}

// [B][C][F/2+1][F] column spectra of a conv input (the mixer keeps z's for its backward).
static size_t big2d_zs_bytes(const ConvPlan& p) {
  return align_up((size_t)p.B * p.C * (p.b2F / 2 + 1) * p.b2F * sizeof(float2));
}

// A second stream per device for work off the mixer's critical path (the large-grid
// filter-spectrum and filter-gradient transforms, which depend only on the filter or on the
// accumulated gradient spectrum): forked from the caller's stream and joined back into it
// with events, so it overlaps the stencils and gates. Created on the first call on a device
// (before any stream capture); the record/wait pairs are serialised per device, so calls
// from several host threads stay ordered. HYFFT_NO_SIDE_STREAM keeps everything on the
// caller's stream.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex mu;
};
static SideStream* side_stream() {
  if (getenv("HYFFT_NO_SIDE_STREAM")) return nullptr;
  static std::mutex mu;
  static std::map<int, SideStream> m;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  SideStream& ss = m[dev];
  if (!ss.s) {
    if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      ss.s = nullptr;
      return nullptr;
    }
  }
  return &ss;
}
// the side stream waits for everything issued on st so far
static int fork_side(SideStream* ss, cudaStream_t st) {
  std::lock_guard<std::mutex> lock(ss->mu);
  if (cudaEventRecord(ss->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss->s, ss->fork, 0) != cudaSuccess)
    return fail(HYFFT_ERR_CUDA, "fork to the side stream failed");
  return HYFFT_OK;
}
// st waits for everything issued on the side stream so far
static int join_side(SideStream* ss, cudaStream_t st) {
  std::lock_guard<std::mutex> lock(ss->mu);
  if (cudaEventRecord(ss->join, ss->s) != cudaSuccess || cudaStreamWaitEvent(st, ss->join, 0) != cudaSuccess)
    return fail(HYFFT_ERR_CUDA, "join from the side stream failed");
  return HYFFT_OK;
}

// The rolled filter's spectrum into kh (workspace T scratch as in big2d_forward).
static int big2d_kspec(const ConvPlan& p, const RealView& kv, char* ws, float2* kh, cudaStream_t st) {
  Big2DParams b;
  big2d_params(p, kv, nullptr, ws, b);
  b.Kh = kh;
  if (big2d_dispatch(B2_KSPEC, p.dt, b, st) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "big2d filter spectrum launch failed");
  return HYFFT_OK;
}

// zs_out: if set, the conv stores its input's column spectra there (zs_mode 1).
// kh: if set, the filter spectrum goes there (the mixer keeps it for its backward).
// kspec_done: kh already holds the filter spectrum (computed on the side stream).
static int big2d_forward(const ConvPlan& p, const RealView& xv, const RealView& kv, const float* D, const RealView& yv,
                         char* ws, cudaStream_t st, float2* zs_out = nullptr, float2* kh = nullptr,
                         bool kspec_done = false) {
  Big2DParams b;
  big2d_params(p, kv, D, ws, b);
  b.x = b2view(xv);
  b.y = b2view(yv);
  if (zs_out) {
    b.Zs = zs_out;
    b.zs_mode = 1;
  }
  if (kh) b.Kh = kh;
  if (!kspec_done && big2d_dispatch(B2_KSPEC, p.dt, b, st) != HYFFT_OK)
    return fail(HYFFT_ERR_CUDA, "big2d filter spectrum launch failed");
  if (big2d_dispatch(B2_CONV, p.dt, b, st) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "big2d conv launch failed");
  return HYFFT_OK;
}

// zs_in: the forward input's column spectra (kept by big2d_forward); with them the
// adjoint conv also accumulates the filter-gradient spectrum and the dK kernel is skipped.
// kh_in: the filter spectrum the forward kept (else it is recomputed).
// side: with the fused filter gradient, its inverse transforms run there (forked after the
// adjoint; the caller joins).
static int big2d_backward(const ConvPlan& p, const RealView& xv, const RealView& kv, const float* D,
                          const RealView& dyv, const RealView& dxv, const RealView& dkv, char* ws, cudaStream_t st,
                          float2* zs_in = nullptr, float2* kh_in = nullptr, SideStream* side = nullptr) {
  Big2DParams b;
  big2d_params(p, kv, D, ws, b);
  if (kh_in) b.Kh = kh_in;
  else if (big2d_dispatch(B2_KSPEC, p.dt, b, st) != HYFFT_OK)
    return fail(HYFFT_ERR_CUDA, "big2d filter spectrum launch failed");
  const bool fused_dk = zs_in && dxv.ptr && dkv.ptr;
  if (fused_dk && cudaMemsetAsync(b.G, 0, big2d_spec_bytes(p), st) != cudaSuccess)
    return fail(HYFFT_ERR_CUDA, "memset G");
  if (dxv.ptr) {  // dx = corr(dy, k) + D * dy
    b.x = b2view(dyv);
    b.y = b2view(dxv);
    b.conj = 1;
    if (fused_dk) {
      b.Zs = zs_in;
      b.zs_mode = 2;
    }
    if (big2d_dispatch(B2_CONV, p.dt, b, st) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "big2d adjoint launch failed");
    b.Zs = nullptr;
    b.zs_mode = 0;
  }
  if (fused_dk) {
    b.dfilt = b2view(dkv);
    if (side) HY_TRY(fork_side(side, st));
    if (big2d_dispatch(B2_DFILT, p.dt, b, side ? side->s : st) != HYFFT_OK)
      return fail(HYFFT_ERR_CUDA, "big2d dfilt launch failed");
    return HYFFT_OK;
  }
  if (dkv.ptr) {
    if (cudaMemsetAsync(b.G, 0, big2d_spec_bytes(p), st) != cudaSuccess) return fail(HYFFT_ERR_CUDA, "memset G");
    b.x = b2view(xv);
    b.x2 = b2view(dyv);
    b.dfilt = b2view(dkv);
    if (big2d_dispatch(B2_DK, p.dt, b, st) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "big2d dK launch failed");
    if (big2d_dispatch(B2_DFILT, p.dt, b, st) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "big2d dfilt launch failed");
  }
  return HYFFT_OK;
}

}  // namespace hyfft

using namespace hyfft;

// ===================================================================== C ABI
extern "C" {

const char* hyfft_last_error(void) { return g_last_error.c_str(); }
const char* hyfft_version(void) { return "hyfft 0.1 (sm_100a)"; }
long long hyfft_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int hyfft_conv_workspace_size(const hyfft_conv_desc* d, size_t* fwd_bytes, size_t* bwd_bytes) {
  ConvPlan p;
  HY_TRY(make_conv_plan(d, p));
  size_t f, b;
  conv_ws_sizes(p, f, b);
  if (fwd_bytes) *fwd_bytes = f;
  if (bwd_bytes) *bwd_bytes = b;
  return HYFFT_OK;
}

int hyfft_conv_forward(const hyfft_conv_desc* d, const void* x, const float* kernel, const void* shortcut, void* y,
                       void* workspace, size_t workspace_bytes, void* stream) {
  ConvPlan p;
  HY_TRY(make_conv_plan(d, p));
  if (!x || !kernel || !y) return fail(HYFFT_ERR_INVALID, "null tensor pointer");
  if (bind_device_of(x) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "cannot make the device of the inputs current");
  size_t need, nb;
  conv_ws_sizes(p, need, nb);
  if (!workspace || workspace_bytes < need) return fail(HYFFT_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  if (p.big2d) {
    float* Dv = (float*)((char*)workspace + 2 * big2d_spec_bytes(p));
    if (shortcut) HY_TRY(to_float(shortcut, p.dt, Dv, p.C, st));
    return big2d_forward(p, real_view(x, p.layout, p.B, p.C, p.g.N, p.g.D),
                         real_view(kernel, p.layout, p.kB, p.C, p.g.K, p.g.D), shortcut ? Dv : nullptr,
                         real_view(y, p.layout, p.B, p.C, p.g.N, p.g.D), (char*)workspace, st);
  }
  char* w = (char*)workspace;
  float2* S = (float2*)w;
  w += align_up((size_t)p.spec_x_bytes_per_ch * p.Cc);
  float2* Kh = (float2*)w;
  w += align_up((size_t)p.spec_k_bytes_per_ch * p.Cc);
  float* Dv = (float*)w;
  if (shortcut) HY_TRY(to_float(shortcut, p.dt, Dv, p.C, st));
  const RealView xv = real_view(x, p.layout, p.B, p.C, p.g.N, p.g.D);
  const RealView kv = real_view(kernel, p.layout, p.kB, p.C, p.g.K, p.g.D);
  const RealView yv = real_view(y, p.layout, p.B, p.C, p.g.N, p.g.D);
  for (int c0 = 0; c0 < p.C; c0 += p.Cc) {
    const int cc = std::min(p.Cc, p.C - c0);
    HY_TRY(conv_forward_chunk(p, c0, cc, xv, kv, shortcut ? Dv : nullptr, yv, S, Kh, st));
  }
  return HYFFT_OK;
}

int hyfft_conv_backward(const hyfft_conv_desc* d, const void* x, const float* kernel, const void* shortcut,
                        const void* dy, void* dx, float* dkernel, float* dshortcut, void* workspace,
                        size_t workspace_bytes, void* stream) {
  ConvPlan p;
  HY_TRY(make_conv_plan(d, p));
  if (!x || !kernel || !dy) return fail(HYFFT_ERR_INVALID, "null tensor pointer");
  if (bind_device_of(x) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "cannot make the device of the inputs current");
  size_t nf, need;
  conv_ws_sizes(p, nf, need);
  if (!workspace || workspace_bytes < need) return fail(HYFFT_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  if (p.big2d) {
    float* Dv = (float*)((char*)workspace + 3 * big2d_spec_bytes(p));
    if (shortcut) HY_TRY(to_float(shortcut, p.dt, Dv, p.C, st));
    HY_TRY(big2d_backward(p, real_view(x, p.layout, p.B, p.C, p.g.N, p.g.D),
                          real_view(kernel, p.layout, p.kB, p.C, p.g.K, p.g.D), shortcut ? Dv : nullptr,
                          real_view(dy, p.layout, p.B, p.C, p.g.N, p.g.D), real_view(dx, p.layout, p.B, p.C, p.g.N, p.g.D),
                          real_view(dkernel, p.layout, p.kB, p.C, p.g.K, p.g.D), (char*)workspace, st));
    if (shortcut && dshortcut) {
      long long S = 1;
      for (int i = 0; i < p.g.D; ++i) S *= p.g.N[i];
      HY_TRY(run_dshortcut(p.dt, p.layout, dy, x, dshortcut, p.B, p.C, S, st));
    }
    return HYFFT_OK;
  }
  char* w = (char*)workspace;
  const size_t sx = align_up((size_t)p.spec_x_bytes_per_ch * p.Cc);
  const size_t sk = align_up((size_t)p.spec_k_bytes_per_ch * p.Cc);
  float2* S1 = (float2*)w;
  float2* S2 = (float2*)(w + sx);
  float2* Kh = (float2*)(w + 2 * sx);
  float2* dKh = (float2*)(w + 2 * sx + sk);
  float* Dv = (float*)(w + 2 * sx + 2 * sk);
  if (shortcut) HY_TRY(to_float(shortcut, p.dt, Dv, p.C, st));
  const RealView xv = real_view(x, p.layout, p.B, p.C, p.g.N, p.g.D);
  const RealView kv = real_view(kernel, p.layout, p.kB, p.C, p.g.K, p.g.D);
  const RealView dyv = real_view(dy, p.layout, p.B, p.C, p.g.N, p.g.D);
  const RealView dxv = real_view(dx, p.layout, p.B, p.C, p.g.N, p.g.D);
  const RealView dkv = real_view(dkernel, p.layout, p.kB, p.C, p.g.K, p.g.D);
  for (int c0 = 0; c0 < p.C; c0 += p.Cc) {
    const int cc = std::min(p.Cc, p.C - c0);
    HY_TRY(conv_backward_chunk(p, c0, cc, xv, kv, shortcut ? Dv : nullptr, dyv, dxv, dkv, S1, S2, Kh, dKh, st));
  }
  if (shortcut && dshortcut) {
    long long S = 1;
    for (int i = 0; i < p.g.D; ++i) S *= p.g.N[i];
    HY_TRY(run_dshortcut(p.dt, p.layout, dy, x, dshortcut, p.B, p.C, S, st));
  }
  return HYFFT_OK;
}

}  // extern "C"

// ------------------------------------------------ forward on a fixed device scratch
// The scratch of hyfft_conv_forward_static_scratch: one array per device, part of the
// library's device image, so using it allocates nothing. Host code never uses the
// name as a device address; it asks the runtime for the address once per device.
static __device__ __align__(256) unsigned char g_conv_scratch[HYFFT_CONV_SCRATCH_MAX_BYTES];

namespace {
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxScratchDevices] = {};

// With the target device current: the device address of g_conv_scratch on it, looked
// up on the first call for that device and cached afterwards.
int conv_scratch_address(void** out) {
  int dev = -1;
  const cudaError_t ge = cudaGetDevice(&dev);
  if (ge != cudaSuccess) return fail(HYFFT_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(ge));
  if (dev < 0 || dev >= kMaxScratchDevices)
    return fail(HYFFT_ERR_UNSUPPORTED, "device ordinal %d beyond the %d the static scratch tracks", dev,
                kMaxScratchDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_conv_scratch);
    if (e != cudaSuccess || !p)
      return fail(HYFFT_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return HYFFT_OK;
}
}  // namespace

extern "C" {

int hyfft_conv_forward_static_scratch(const hyfft_conv_desc* d, const void* x, const float* kernel,
                                      const void* shortcut, void* y, void* stream) {
  ConvPlan p;
  HY_TRY(make_conv_plan(d, p, /*allow_big2d=*/false));
  if (!x || !kernel || !y) return fail(HYFFT_ERR_INVALID, "null tensor pointer");
  // Chunk the channels so that one chunk's spectra, the float shortcut vector and the
  // 256-byte alignment padding of the two spectrum buffers fit the scratch.
  const size_t cap = HYFFT_CONV_SCRATCH_MAX_BYTES;
  const size_t dvec = align_up((size_t)p.C * 4);
  const size_t per_ch = (size_t)(p.spec_x_bytes_per_ch + p.spec_k_bytes_per_ch);
  if (dvec + 512 + per_ch > cap)
    return fail(HYFFT_ERR_WORKSPACE,
                "one channel needs %zu bytes of scratch (spectra %zu + shortcut %zu); the static scratch holds %zu "
                "bytes: use hyfft_conv_forward with a caller workspace",
                dvec + 512 + per_ch, per_ch, dvec, cap);
  p.Cc = (int)std::min<size_t>((size_t)p.C, (cap - dvec - 512) / per_ch);
  size_t need, nb;
  conv_ws_sizes(p, need, nb);
  if (need > cap) return fail(HYFFT_ERR_WORKSPACE, "static scratch plan needs %zu > %zu bytes", need, cap);
  if (bind_device_of(x) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "cannot make the device of the inputs current");
  void* scratch = nullptr;
  HY_TRY(conv_scratch_address(&scratch));
  cudaStream_t st = (cudaStream_t)stream;
  char* w = (char*)scratch;
  float2* S = (float2*)w;
  w += align_up((size_t)p.spec_x_bytes_per_ch * p.Cc);
  float2* Kh = (float2*)w;
  w += align_up((size_t)p.spec_k_bytes_per_ch * p.Cc);
  float* Dv = (float*)w;
  if (shortcut) HY_TRY(to_float(shortcut, p.dt, Dv, p.C, st));
  const RealView xv = real_view(x, p.layout, p.B, p.C, p.g.N, p.g.D);
  const RealView kv = real_view(kernel, p.layout, p.kB, p.C, p.g.K, p.g.D);
  const RealView yv = real_view(y, p.layout, p.B, p.C, p.g.N, p.g.D);
  for (int c0 = 0; c0 < p.C; c0 += p.Cc) {
    const int cc = std::min(p.Cc, p.C - c0);
    HY_TRY(conv_forward_chunk(p, c0, cc, xv, kv, shortcut ? Dv : nullptr, yv, S, Kh, st));
  }
  return HYFFT_OK;
}

}  // extern "C"

// ===================================================================== Hyena (general path)
namespace hyfft {

struct HyenaPlan {
  hyfft_hyena_desc d;
  ConvPlan cp;          // the long conv on z (channels-last contiguous [B, *S, C])
  StencilGeom sg;
  long long Ntot = 1;   // prod n
  long long E = 0;      // B * Ntot * C
  int eb = 2;
  bool fused = false;   // single-pass fused FFT kernels (fused.cu) apply
  bool tp = false;      // tensor-core Toeplitz kernels (toeplitz.cu) apply (takes precedence)
  int SK = 0;
  int fF[2] = {0, 0};   // FFT sizes of the fused kernels (2^m or 3 * 2^m per axis)
  bool cache_kh = false;  // general engine: the forward keeps the filter spectrum of every channel
                          // chunk in the saved state (chunk c0's block at c0 * spec_k_bytes_per_ch)
                          // and the backward reuses it
};

// Smallest FFT length of the fused kernels (2^m or 3 * 2^m, at most 64) for an axis of
// n points and a k-tap centred filter rolled by its crop offset k/2: the circular
// convolution equals the linear one on [0, n) when F >= n + k/2 and F >= n + ceil(k/2) - 1,
// and the filter fits when F >= k.
static int fused_fft_len(int n, int k) {
  const int need = std::max(std::max(n + k / 2, n + (k + 1) / 2 - 1), k);
  int best = 1 << 30;
  for (int p = 1; p <= 64; p <<= 1) {
    if (p >= need) best = std::min(best, p);
    if (3 * p >= need && 3 * p <= 48) best = std::min(best, 3 * p);
  }
  return best;
}


static int make_hyena_plan(const hyfft_hyena_desc* d, HyenaPlan& h) {
  if (!d) return fail(HYFFT_ERR_INVALID, "null descriptor");
  h.d = *d;
  hyfft_conv_desc cd;
  memset(&cd, 0, sizeof(cd));
  cd.ndim = d->ndim;
  cd.batch = d->batch;
  cd.channels = d->channels;
  for (int i = 0; i < 3; ++i) {
    cd.n[i] = i < d->ndim ? d->n[i] : 1;
    cd.k[i] = i < d->ndim ? d->k[i] : 1;
  }
  cd.kernel_batch = 1;
  cd.causal = d->causal;
  cd.dtype = d->dtype;
  cd.layout = HYFFT_LAYOUT_BLH;
  cd.periodic = d->periodic;
  HY_TRY(make_conv_plan(&cd, h.cp));
  if (d->gate1 < 0 || d->gate1 > 2 || d->gate2 < 0 || d->gate2 > 2) return fail(HYFFT_ERR_INVALID, "bad gate");
  StencilGeom& g = h.sg;
  g.nd = d->ndim;
  g.has_conv = d->short_k[0] > 0 ? 1 : 0;
  g.has_bias = (g.has_conv && d->short_bias) ? 1 : 0;
  g.ntaps = 1;
  h.Ntot = 1;
  for (int i = 0; i < 3; ++i) {
    const bool used = i < d->ndim;
    g.n[i] = used ? d->n[i] : 1;
    g.k[i] = (used && g.has_conv) ? d->short_k[i] : 1;
    if (g.k[i] < 1) return fail(HYFFT_ERR_INVALID, "short conv extents must be positive");
    if (d->short_causal && g.has_conv) {
      if (d->ndim != 1) return fail(HYFFT_ERR_INVALID, "causal short conv is 1D only");
      g.off[i] = g.k[i] - 1;
    } else {
      g.off[i] = (g.k[i] - 1) / 2;
    }
    g.ntaps *= g.k[i];
    h.Ntot *= g.n[i];
  }
  if (g.ntaps > 27) return fail(HYFFT_ERR_UNSUPPORTED, "short conv with more than 27 taps");
  h.E = (long long)d->batch * h.Ntot * d->channels;
  h.eb = dtype_bytes(d->dtype);
  if (d->in_pos_stride < d->channels || d->out_pos_stride < d->channels)
    return fail(HYFFT_ERR_INVALID, "position strides must be >= channels");
  // fused single-pass path: 2D, "same" 3x3 (or no) short conv, 8-channel vectors
  const bool sq3 = g.has_conv && g.k[0] == 3 && g.k[1] == 3 && !d->short_causal;
  h.SK = sq3 ? 3 : 0;
  if (!getenv("HYFFT_DISABLE_FUSED") && !d->periodic && d->ndim == 2 && !d->causal && (sq3 || !g.has_conv) &&
      (d->dtype == HYFFT_BF16 || d->dtype == HYFFT_F32) && d->channels % 8 == 0 && d->in_pos_stride % 8 == 0 &&
      d->in_batch_stride % 8 == 0 && d->out_pos_stride % 8 == 0 && d->out_batch_stride % 8 == 0) {
    // the shortest compiled transform first (e.g. 24 = 3 * 8 for a 14-point axis and a 14-tap
    // filter), else the power-of-two length of the general plan
    const int f0 = fused_fft_len(h.cp.g.N[0], h.cp.g.K[0]), f1 = fused_fft_len(h.cp.g.N[1], h.cp.g.K[1]);
    if (!getenv("HYFFT_FUSED_POW2") && fused2d_dispatch(FOP_PROBE, d->dtype, h.cp.g.N[0], h.cp.g.N[1], f0, f1, h.SK,
                                                        nullptr, nullptr) == HYFFT_OK) {
      h.fused = true;
      h.fF[0] = f0;
      h.fF[1] = f1;
    } else if (fused2d_dispatch(FOP_PROBE, d->dtype, h.cp.g.N[0], h.cp.g.N[1], h.cp.g.F[0], h.cp.g.F[1], h.SK,
                                nullptr, nullptr) == HYFFT_OK) {
      h.fused = true;
      h.fF[0] = h.cp.g.F[0];
      h.fF[1] = h.cp.g.F[1];
    }
    // bf16 grids with both sides <= 16: the long conv as a tcgen05 Toeplitz GEMM
    const int N0 = h.cp.g.N[0], N1 = h.cp.g.N[1], K0 = h.cp.g.K[0], K1 = h.cp.g.K[1];
    // (opt-in while its CUDA-core stencil / reduction phases are slower than the fused FFT kernels)
    h.tp = getenv("HYFFT_USE_TP") && !getenv("HYFFT_DISABLE_TP") && d->dtype == HYFFT_BF16 && K0 <= 31 && K1 <= 31 &&
           K0 <= 2 * N0 &&
           K1 <= 2 * N1 && tp2d_dispatch(TP_PROBE, N0, N1, h.SK, nullptr, nullptr) == HYFFT_OK;
    if (h.tp) h.fused = false;
  }
  // (kept when it fits the workspace budget: the backward then skips one filter transform per chunk)
  h.cache_kh = !h.fused && !h.tp && !h.cp.big2d && !getenv("HYFFT_NO_KH_CACHE") &&
               (size_t)h.cp.spec_k_bytes_per_ch * h.cp.C <= ws_budget();
  return HYFFT_OK;
}

static void hyena_sizes(const HyenaPlan& h, size_t& fwd, size_t& bwd, size_t& saved) {
  if (h.tp) {  // nothing kept between passes; the workspace holds a status word
    saved = 0;
    fwd = 256;
    bwd = 256;
    return;
  }
  if (h.fused) {
    const size_t spec = align_up((size_t)h.d.channels * h.fF[0] * h.fF[1] * sizeof(float2));
    saved = spec + 3 * align_up((size_t)h.E * h.eb);  // filter spectrum and q', k', v', reused by the backward
    fwd = 256;
    bwd = spec;    // dK spectrum accumulator
    return;
  }
  size_t cf, cb;
  conv_ws_sizes(h.cp, cf, cb);
  const size_t act = align_up((size_t)h.E * h.eb);
  saved = 5 * act;                 // q', k', v', z, h
  if (h.cache_kh) saved += align_up((size_t)h.cp.spec_k_bytes_per_ch * h.cp.C);  // filter spectrum
  if (h.cp.big2d) saved += big2d_zs_bytes(h.cp) + big2d_spec_bytes(h.cp);  // z's column spectra, filter spectrum
  fwd = cf + align_up((size_t)h.d.channels * 4);
  bwd = cb + 5 * act + align_up((size_t)h.d.channels * 4);  // dh, dz, dv', dq', dk'
  if (h.cp.big2d) {  // channel-major copies around the large-grid kernels: z, h | z, dh, dz
    fwd += 2 * act;
    bwd += 3 * act;
  }
}

// channels-last [B][N][C] <-> channel-major [B][C][N] (contiguous)
int cl_cm_tma(const void* src, void* dst, int B, long long N, int C, bool to_cm, int* status, cudaStream_t st);

template <typename T>
static int cl_cm(const T* src, T* dst, int B, long long N, int C, bool to_cm, cudaStream_t st) {
  if (sizeof(T) == 2) {  // 64 x 64 tiles moved by TMA (transpose_tma.cu) where the shape allows
    const int rc = cl_cm_tma(src, dst, B, N, C, to_cm, nullptr, st);
    if (rc == HYFFT_OK) return HYFFT_OK;
    if (rc != HYFFT_ERR_UNSUPPORTED) return fail(rc, "cl_cm_tma_kernel launch failed");
  }
  const dim3 grid((unsigned)((N + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)B);
  if (to_cm) cl_cm_transpose_kernel<T, true><<<grid, 256, 0, st>>>(src, dst, N, C);
  else cl_cm_transpose_kernel<T, false><<<grid, 256, 0, st>>>(src, dst, N, C);
  return check_launch("cl_cm_transpose_kernel");
}

// The gates fused with the layout change around the large-grid kernels (cl_cm_gate_kernel),
// where the shape and the pointers allow: 16-bit activations, C and N multiples of 64,
// every tensor contiguous and 16-byte aligned.
static bool gate_x_ok(int eb, int C, long long N, std::initializer_list<const void*> ps) {
  if (eb != 2 || C % 64 || N % 64 || getenv("HYFFT_DISABLE_GATE_FUSION")) return false;
  for (const void* q : ps)
    if (((uintptr_t)q % 16) != 0) return false;
  return true;
}
template <typename T, int MODE>
static int gate_x(const T* a, const T* b1, const T* b2, T* o1, T* o2, int gate, int B, long long N, int C,
                  cudaStream_t st) {
  if constexpr (sizeof(T) != 2) {
    return fail(HYFFT_ERR_UNSUPPORTED, "cl_cm_gate_kernel: 16-bit activations only");
  } else {
    const dim3 grid((unsigned)(N / 64), (unsigned)(C / 64), (unsigned)B);
    cl_cm_gate_kernel<T, MODE><<<grid, 256, 0, st>>>(a, b1, b2, o1, o2, gate, N, C);
    return check_launch("cl_cm_gate_kernel");
  }
}

// ---- launch helpers of the elementwise / stencil kernels (hyena_elem.cuh)
template <int V> using IC = std::integral_constant<int, V>;

// Call f(IC<K0>, IC<K1>, IC<K2>) with the compile-time stencil of g when it is one of the
// shapes the reference uses, else with the runtime-shaped fallback (-1).
template <bool PAIR, typename F>
static void with_stencil(const StencilGeom& g, F&& f) {
  const int a = g.k[0], b = g.k[1], c = g.k[2];
  if (!g.has_conv) f(IC<0>{}, IC<0>{}, IC<0>{});
  else if constexpr (!PAIR) f(IC<-1>{}, IC<-1>{}, IC<-1>{});
  else if (a == 3 && b == 1 && c == 1) f(IC<3>{}, IC<1>{}, IC<1>{});
  else if (a == 4 && b == 1 && c == 1) f(IC<4>{}, IC<1>{}, IC<1>{});
  else if (a == 7 && b == 1 && c == 1) f(IC<7>{}, IC<1>{}, IC<1>{});
  else if (a == 3 && b == 3 && c == 1) f(IC<3>{}, IC<3>{}, IC<1>{});
  else if (a == 3 && b == 3 && c == 3) f(IC<3>{}, IC<3>{}, IC<3>{});
  else f(IC<-1>{}, IC<-1>{}, IC<-1>{});
}

// ------------------------------------------------------------------ 3D plane-marching stencils
// 3x3x3 short convs of 16-bit channels-last activations run on the plane-marching kernels
// (stencil3d.cuh) when every 16-byte chunk of 8 channels is aligned.
template <typename T>
static bool plane_stencil_ok(const HyenaPlan& h, std::initializer_list<const void*> ps) {
  const hyfft_hyena_desc& d = h.d;
  const bool s3 = d.ndim == 3 && h.sg.k[0] == 3 && h.sg.k[1] == 3 && h.sg.k[2] == 3;
  const bool s2 = d.ndim == 2 && h.sg.k[0] == 3 && h.sg.k[1] == 3;
  if (sizeof(T) != 2 || !h.sg.has_conv || !(s3 || s2) || getenv("HYFFT_DISABLE_PLANE_STENCIL")) return false;
  if (d.channels % 8 || d.in_batch_stride % 8 || d.in_pos_stride % 8) return false;
  // one-row planes keep a thread's in-row chunk offsets as int
  if ((long long)h.sg.n[d.ndim - 1] * std::max<long long>(d.in_pos_stride, d.channels) + d.channels >= (1LL << 31))
    return false;
  for (const void* p : ps)
    if (p && ((uintptr_t)p % 16) != 0) return false;
  return true;
}

struct PlaneLaunch {
  dim3 grid;
  int xchunk;
  StencilGeom g;  // 3D geometry of the kernels
};
// A 2D grid whose last axis has at least 96 positions marches along its first axis (as x)
// with one-row planes of up to 128 positions; a smaller one runs as one x plane of 4 x 32
// tiles.
static bool plane_march2d(const HyenaPlan& h) { return h.d.ndim == 2 && h.sg.n[1] >= 96; }
// x runs per CTA such that the grid fills about two waves of two CTAs per SM (3D), or one
// wave of three CTAs per SM (2D march: the halo rows re-read per run stay few).
static PlaneLaunch plane_launch(const HyenaPlan& h, int march_ctas_per_sm = 3) {
  StencilGeom g = h.sg;
  const bool march = plane_march2d(h);
  int TY = kS3TY, TZ = kS3TZ;
  if (march) {  // (n0, n1) -> (x = n0, y = 1, z = n1)
    g.nd = 3;
    g.n[2] = g.n[1];
    g.n[1] = 1;
    g.k[2] = g.k[1];
    g.k[1] = 1;
    g.off[2] = g.off[1];
    g.off[1] = 0;
    TY = 1;
    TZ = kS2TZ;
  } else if (h.d.ndim == 2) {  // (n0, n1) -> (x = 1, y = n0, z = n1)
    g.nd = 3;
    g.n[2] = g.n[1];
    g.n[1] = g.n[0];
    g.n[0] = 1;
    g.k[2] = g.k[1];
    g.k[1] = g.k[0];
    g.k[0] = 1;
    g.off[2] = g.off[1];
    g.off[1] = g.off[0];
    g.off[0] = 0;
  }
  const long long base = (long long)((h.d.channels + kElemCG - 1) / kElemCG) * ((g.n[1] + TY - 1) / TY) *
                         ((g.n[2] + TZ - 1) / TZ) * h.d.batch;
  const long long target = march ? (long long)march_ctas_per_sm * 148 : 4 * 148;
  const long long nxc = march ? std::max<long long>(1, std::min<long long>(g.n[0], target / base))
                              : std::max<long long>(1, std::min<long long>(g.n[0], (target + base - 1) / base));
  PlaneLaunch pl;
  pl.xchunk = (int)((g.n[0] + nxc - 1) / nxc);
  const long long chunks = (g.n[0] + pl.xchunk - 1) / pl.xchunk;
  pl.grid = dim3((unsigned)((h.d.channels + kElemCG - 1) / kElemCG),
                 (unsigned)(((g.n[1] + TY - 1) / TY) * ((g.n[2] + TZ - 1) / TZ)),
                 (unsigned)(h.d.batch * chunks));
  pl.g = g;
  return pl;
}

// Rows of (b, position) per CTA column so that a warp walks about `per_warp` rows.
static dim3 elem_grid(int C, long long rows, long long per_warp) {
  const long long gy = std::max<long long>(1, std::min<long long>(65535, (rows + 8 * per_warp - 1) / (8 * per_warp)));
  return dim3((unsigned)((C + kElemCG - 1) / kElemCG), (unsigned)gy, 1);
}

// Two-channel vector accesses need an even channel count, even element strides and
// bases aligned to two elements.
static bool elem_pairs_ok(const HyenaPlan& h, std::initializer_list<const void*> ps) {
  const hyfft_hyena_desc& d = h.d;
  if (d.channels % 2 || d.in_batch_stride % 2 || d.in_pos_stride % 2 || d.out_batch_stride % 2 ||
      d.out_pos_stride % 2)
    return false;
  for (const void* p : ps)
    if (p && ((uintptr_t)p % (2 * h.eb)) != 0) return false;
  return true;
}

// dD[c] = dfilt[c][K0 / 2][K1 / 2]: for a centred filter the D-skip acts at the tap whose
// gradient is sum_n dh[n] z[n], so the two gradients coincide.
__global__ void centre_tap_kernel(const float* __restrict__ dfilt, float* __restrict__ dD, int C, int K0, int K1) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < C) dD[c] = dfilt[((long long)c * K0 + K0 / 2) * K1 + K1 / 2];
}

template <typename T>
static int hyena_forward_body(const HyenaPlan& h, const T* q, const T* k, const T* v, const float* filt,
                              const float* D, const float* sw, const float* sb, T* y, char* saved, char* ws,
                              cudaStream_t st, SideStream* side) {
  const hyfft_hyena_desc& d = h.d;
  const size_t act = align_up((size_t)h.E * h.eb);
  T* qs = (T*)(saved);
  T* ks = (T*)(saved + act);
  T* vs = (T*)(saved + 2 * act);
  T* z = (T*)(saved + 3 * act);
  T* hb = (T*)(saved + 4 * act);
  if (side) {  // large grid: the filter spectrum on the side stream, overlapping the short conv
    HY_TRY(fork_side(side, st));
    HY_TRY(big2d_kspec(h.cp, real_view(filt, HYFFT_LAYOUT_BHL, 1, h.cp.C, h.cp.g.K, h.cp.g.D), ws,
                       (float2*)(saved + 5 * act + big2d_zs_bytes(h.cp)), side->s));
  }
  const long long rows = (long long)d.batch * h.Ntot;
  const bool pair = elem_pairs_ok(h, {q, k, v, y});
  auto pre = [&](auto pr) {
    constexpr bool P = decltype(pr)::value;
    with_stencil<P>(h.sg, [&](auto a, auto b, auto c) {
      constexpr int K0 = decltype(a)::value, K1 = decltype(b)::value, K2 = decltype(c)::value;
      if constexpr (K0 > 0 && K1 > 0 && K2 > 0) {
        constexpr int ND = K2 > 1 ? 3 : (K1 > 1 ? 2 : 1);
        constexpr int KA = ND == 1 ? 1 : K0, KB = ND == 3 ? K1 : 1, KI = ND == 3 ? K2 : (ND == 2 ? K1 : K0);
        if constexpr ((ND == 3 || ND == 2) && P && sizeof(T) == 2 && KA == 3 && KI == 3 && (ND == 2 || KB == 3)) {
          constexpr int PX = ND == 3 ? 3 : 1;
          constexpr size_t sm = s3_smem_bytes<PX, 3, 3>();
          if constexpr (ND == 2) {
            constexpr size_t sm2 = s3_smem_bytes<3, 1, 3, 1, kS2TZ>();
            if (plane_march2d(h) && plane_stencil_ok<T>(h, {q, k, v}) &&
                kernel_smem_once((const void*)hyena_plane_stencil_kernel<T, 3, 1, 3, 0, 1, kS2TZ>, sm2)) {
              const PlaneLaunch pl = plane_launch(h);
              hyena_plane_stencil_kernel<T, 3, 1, 3, 0, 1, kS2TZ><<<pl.grid, kElemThreads, sm2, st>>>(
                  q, k, v, d.in_batch_stride, d.in_pos_stride, qs, ks, vs, 0, 0, z, pl.g, d.channels, sw, sb,
                  d.gate1, pl.xchunk);
              return;
            }
          }
          // (the line kernels below take over if the shared-memory size cannot be granted)
          if (!plane_march2d(h) && plane_stencil_ok<T>(h, {q, k, v}) &&
              kernel_smem_once((const void*)hyena_plane_stencil_kernel<T, PX, 3, 3, 0>, sm)) {
            const PlaneLaunch pl = plane_launch(h);
            hyena_plane_stencil_kernel<T, PX, 3, 3, 0><<<pl.grid, kElemThreads, sm, st>>>(
                q, k, v, d.in_batch_stride, d.in_pos_stride, qs, ks, vs, 0, 0, z, pl.g, d.channels, sw, sb, d.gate1,
                pl.xchunk);
            return;
          }
        }
        if (d.ndim == ND) {
          const long long nl = h.sg.n[ND - 1];
          const long long items = (long long)d.batch * (h.Ntot / nl) * ((nl + 63) / 64);
          const dim3 lg((unsigned)((d.channels + kElemCG - 1) / kElemCG),
                        (unsigned)std::max<long long>(1, std::min<long long>(65535, (items + 7) / 8)), 1);
          hyena_line_stencil_kernel<T, P, ND, KA, KB, KI, 0><<<lg, kElemThreads, 0, st>>>(
              q, k, v, d.in_batch_stride, d.in_pos_stride, qs, ks, vs, 0, 0, z, h.sg, d.batch, d.channels, sw, sb,
              d.gate1);
          return;
        }
      }
      hyena_pre_fwd_kernel<T, P, K0, K1, K2><<<elem_grid(d.channels, rows, 4), kElemThreads, 0, st>>>(
          q, k, v, d.in_batch_stride, d.in_pos_stride, h.sg, d.batch, d.channels, sw, sb, d.gate1, qs, ks, vs, z);
    });
  };
  if (pair) pre(std::true_type{});
  else pre(std::false_type{});
  HY_TRY(check_launch("hyena_pre_fwd_kernel"));
  // long conv with D-skip: h = round(conv(z)) + round(D * z)
  const ConvPlan& p = h.cp;
  size_t cf, cb;
  conv_ws_sizes(p, cf, cb);
  float2* S = (float2*)ws;
  float2* Kh = h.cache_kh ? (float2*)(saved + 5 * act) : (float2*)(ws + align_up((size_t)p.spec_x_bytes_per_ch * p.Cc));
  const RealView zv = real_view(z, HYFFT_LAYOUT_BLH, p.B, p.C, p.g.N, p.g.D);
  const RealView kv = real_view(filt, HYFFT_LAYOUT_BHL, 1, p.C, p.g.K, p.g.D);
  const RealView hv = real_view(hb, HYFFT_LAYOUT_BLH, p.B, p.C, p.g.N, p.g.D);
  if (p.big2d) {
    float2* zs = (float2*)(saved + 5 * act);
    float2* khs = (float2*)(saved + 5 * act + big2d_zs_bytes(p));
    // channel-major z and h around the large-grid kernels (unit-stride rows; reading the
    // channels-last tensors in place with 2-byte strided accesses measured 1.5x slower)
    T* zc = (T*)(ws + cf + align_up((size_t)d.channels * 4));
    T* hc = (T*)((char*)zc + align_up((size_t)h.E * h.eb));
    HY_TRY(cl_cm<T>(z, zc, d.batch, h.Ntot, d.channels, true, st));
    if (side) HY_TRY(join_side(side, st));
    HY_TRY(big2d_forward(p, real_view(zc, HYFFT_LAYOUT_BHL, p.B, p.C, p.g.N, p.g.D), kv, D,
                         real_view(hc, HYFFT_LAYOUT_BHL, p.B, p.C, p.g.N, p.g.D), ws, st, zs, khs, side != nullptr));
    // h back to channels-last and gate 2 in one pass where the output is contiguous
    if (d.out_pos_stride == d.channels && d.out_batch_stride == h.Ntot * d.channels &&
        gate_x_ok(sizeof(T), d.channels, h.Ntot, {hc, hb, vs, y}))
      return gate_x<T, GATE_POST_FWD>(hc, vs, nullptr, hb, y, d.gate2, d.batch, h.Ntot, d.channels, st);
    HY_TRY(cl_cm<T>(hc, hb, d.batch, h.Ntot, d.channels, false, st));
  } else {
    for (int c0 = 0; c0 < p.C; c0 += p.Cc) {
      const int cc = std::min(p.Cc, p.C - c0);
      float2* khc = h.cache_kh ? Kh + (size_t)c0 * (p.spec_k_bytes_per_ch / sizeof(float2)) : Kh;
      HY_TRY(conv_forward_chunk(p, c0, cc, zv, kv, D, hv, S, khc, st));
    }
  }
  if (pair)
    hyena_post_fwd_kernel<T, true><<<elem_grid(d.channels, rows, 8), kElemThreads, 0, st>>>(
        hb, vs, d.gate2, h.Ntot, d.batch, d.channels, y, d.out_batch_stride, d.out_pos_stride);
  else
    hyena_post_fwd_kernel<T, false><<<elem_grid(d.channels, rows, 8), kElemThreads, 0, st>>>(
        hb, vs, d.gate2, h.Ntot, d.batch, d.channels, y, d.out_batch_stride, d.out_pos_stride);
  return check_launch("hyena_post_fwd_kernel");
}

template <typename T>
static int hyena_backward_body(const HyenaPlan& h, const T* q, const T* k, const T* v, const float* filt,
                               const float* D, const float* sw, const T* dy, T* dq, T* dk, T* dv, float* dfilt,
                               float* dD, float* dsw, float* dsb, const char* saved, char* ws, cudaStream_t st,
                               SideStream* side) {
  const hyfft_hyena_desc& d = h.d;
  const size_t act = align_up((size_t)h.E * h.eb);
    const T* qs = (const T*)(saved);
  const T* ks = (const T*)(saved + act);
  const T* vs = (const T*)(saved + 2 * act);
  const T* z = (const T*)(saved + 3 * act);
  const T* hb = (const T*)(saved + 4 * act);
  const ConvPlan& p = h.cp;
  size_t cf, cb;
  conv_ws_sizes(p, cf, cb);
  char* w = ws + cb;
  T* dh = (T*)w;
  w += act;
  T* dz = (T*)w;
  w += act;
  T* dvp = (T*)w;
  w += act;
  T* dqp = (T*)w;
  w += act;
  T* dkp = (T*)w;
  const long long rows = (long long)d.batch * h.Ntot;
  const bool pair = elem_pairs_ok(h, {q, k, v, dy, dq, dk, dv});
  const dim3 eg = elem_grid(d.channels, rows, 8);
  // reductions (dD, short-conv weights): about 1200 CTAs in all, one atomic per channel each
  auto red_rows = [&](int cols) {
    return std::max<long long>(1, std::min<long long>(65535, 1200 / std::max(1, cols)));
  };
  // large grid: channel-major copies of z, dh, dz around the large-grid kernels; the gates
  // on either side of them are fused with the layout changes where gate_x_ok allows (gate 2
  // only when the adjoint also forms the filter gradient, the path that needs no
  // channels-last dh)
  T* zc = p.big2d ? (T*)(ws + cb + 5 * act + align_up((size_t)d.channels * 4)) : nullptr;
  T* dhc = p.big2d ? (T*)((char*)zc + act) : nullptr;
  T* dzc = p.big2d ? (T*)((char*)dhc + act) : nullptr;
  const bool fuse2 = p.big2d && dfilt != nullptr && d.out_pos_stride == d.channels &&
                     d.out_batch_stride == h.Ntot * d.channels &&
                     gate_x_ok(sizeof(T), d.channels, h.Ntot, {dy, hb, vs, dvp, dhc});
  const bool fuse1 = p.big2d && gate_x_ok(sizeof(T), d.channels, h.Ntot, {dzc, qs, ks, dqp, dkp});
  if (fuse2) {
    HY_TRY((gate_x<T, GATE_BWD2>(dy, hb, vs, dvp, dhc, d.gate2, d.batch, h.Ntot, d.channels, st)));
  } else {
    if (pair)
      hyena_bwd_gate2_kernel<T, true><<<eg, kElemThreads, 0, st>>>(dy, d.out_batch_stride, d.out_pos_stride, hb,
                                                                   vs, d.gate2, h.Ntot, d.batch, d.channels, dh, dvp);
    else
      hyena_bwd_gate2_kernel<T, false><<<eg, kElemThreads, 0, st>>>(dy, d.out_batch_stride, d.out_pos_stride, hb,
                                                                    vs, d.gate2, h.Ntot, d.batch, d.channels, dh, dvp);
    HY_TRY(check_launch("hyena_bwd_gate2_kernel"));
  }
  // long conv backward: dz = convT(dh) + D*dh, dfilt, dD
  {
    const size_t sx = align_up((size_t)p.spec_x_bytes_per_ch * p.Cc);
    const size_t sk = align_up((size_t)p.spec_k_bytes_per_ch * p.Cc);
    float2* S1 = (float2*)ws;
    float2* S2 = (float2*)(ws + sx);
    float2* Kh = h.cache_kh ? (float2*)const_cast<char*>(saved + 5 * act) : (float2*)(ws + 2 * sx);
    float2* dKh = (float2*)(ws + 2 * sx + sk);
    const RealView zv = real_view(z, HYFFT_LAYOUT_BLH, p.B, p.C, p.g.N, p.g.D);
    const RealView kv = real_view(filt, HYFFT_LAYOUT_BHL, 1, p.C, p.g.K, p.g.D);
    const RealView dhv = real_view(dh, HYFFT_LAYOUT_BLH, p.B, p.C, p.g.N, p.g.D);
    const RealView dzv = real_view(dz, HYFFT_LAYOUT_BLH, p.B, p.C, p.g.N, p.g.D);
    const RealView dkv = real_view(dfilt, HYFFT_LAYOUT_BHL, 1, p.C, p.g.K, p.g.D);
    // large grid with a filter gradient: the adjoint conv accumulates it from z's column
    // spectra kept by the forward, so z itself is not transformed again, and dD is the
    // gradient's centre tap (the rolled filter's tap (0, 0) is where the D-skip acts)
    const bool zs = p.big2d && dfilt != nullptr;
    if (p.big2d) {
      float2* zsp = zs ? (float2*)const_cast<char*>(saved + 5 * act) : nullptr;
      float2* khs = (float2*)const_cast<char*>(saved + 5 * act + big2d_zs_bytes(p));
      if (!zs) HY_TRY(cl_cm<T>(z, zc, d.batch, h.Ntot, d.channels, true, st));
      if (!fuse2) HY_TRY(cl_cm<T>(dh, dhc, d.batch, h.Ntot, d.channels, true, st));
      HY_TRY(big2d_backward(p, real_view(zc, HYFFT_LAYOUT_BHL, p.B, p.C, p.g.N, p.g.D), kv, D,
                            real_view(dhc, HYFFT_LAYOUT_BHL, p.B, p.C, p.g.N, p.g.D),
                            real_view(dzc, HYFFT_LAYOUT_BHL, p.B, p.C, p.g.N, p.g.D), dkv, ws, st, zsp, khs,
                            zs ? side : nullptr));
      if (!fuse1) HY_TRY(cl_cm<T>(dzc, dz, d.batch, h.Ntot, d.channels, false, st));
      if (zs && dD) {
        // after the filter gradient, on the stream that computes it
        centre_tap_kernel<<<(d.channels + 255) / 256, 256, 0, side ? side->s : st>>>(dfilt, dD, d.channels,
                                                                                       p.g.K[0], p.g.K[1]);
        HY_TRY(check_launch("centre_tap_kernel"));
      }
    } else {
      for (int c0 = 0; c0 < p.C; c0 += p.Cc) {
        const int cc = std::min(p.Cc, p.C - c0);
        float2* khc = h.cache_kh ? Kh + (size_t)c0 * (p.spec_k_bytes_per_ch / sizeof(float2)) : Kh;
        HY_TRY(conv_backward_chunk(p, c0, cc, zv, kv, D, dhv, dzv, dkv, S1, S2, khc, dKh, st, h.cache_kh));
      }
    }
    if (dD && !zs) {
      if (cudaMemsetAsync(dD, 0, sizeof(float) * (size_t)d.channels, st) != cudaSuccess)
        return fail(HYFFT_ERR_CUDA, "memset dD");
      const dim3 rg(eg.x, (unsigned)red_rows((int)eg.x), 1);
      if (pair) hyena_dskip_kernel<T, true><<<rg, kElemThreads, 0, st>>>(dh, z, rows, d.channels, dD);
      else hyena_dskip_kernel<T, false><<<rg, kElemThreads, 0, st>>>(dh, z, rows, d.channels, dD);
      HY_TRY(check_launch("hyena_dskip_kernel"));
    }
  }
  if (fuse1) {  // dz back to channels-last and gate 1 in one pass
    HY_TRY((gate_x<T, GATE_BWD1>(dzc, qs, ks, dqp, dkp, d.gate1, d.batch, h.Ntot, d.channels, st)));
  } else {
    if (pair)
      hyena_bwd_gate1_kernel<T, true><<<eg, kElemThreads, 0, st>>>(dz, qs, ks, d.gate1, rows, d.channels, dqp, dkp);
    else
      hyena_bwd_gate1_kernel<T, false><<<eg, kElemThreads, 0, st>>>(dz, qs, ks, d.gate1, rows, d.channels, dqp, dkp);
    HY_TRY(check_launch("hyena_bwd_gate1_kernel"));
  }
  // 2D march with short-conv weight gradients: the weight gradient runs inside the
  // transposed-stencil kernel (HYFFT_DISABLE_FUSED_WGRAD keeps the two kernels)
  const bool fuse_wgrad = h.sg.has_conv && dsw != nullptr && !getenv("HYFFT_DISABLE_FUSED_WGRAD");
  bool wgrad_done = false;
  int launch_rc = HYFFT_OK;
  auto dgrad = [&](auto pr) {
    constexpr bool P = decltype(pr)::value;
    with_stencil<P>(h.sg, [&](auto a, auto b, auto c) {
      constexpr int K0 = decltype(a)::value, K1 = decltype(b)::value, K2 = decltype(c)::value;
      if constexpr (K0 > 0 && K1 > 0 && K2 > 0) {
        constexpr int ND = K2 > 1 ? 3 : (K1 > 1 ? 2 : 1);
        constexpr int KA = ND == 1 ? 1 : K0, KB = ND == 3 ? K1 : 1, KI = ND == 3 ? K2 : (ND == 2 ? K1 : K0);
        if constexpr ((ND == 3 || ND == 2) && P && sizeof(T) == 2 && KA == 3 && KI == 3 && (ND == 2 || KB == 3)) {
          constexpr int PX = ND == 3 ? 3 : 1;
          constexpr size_t sm = s3_smem_bytes<PX, 3, 3>();
          if constexpr (ND == 2) {
            // transposed stencil and weight / bias gradients in one march (two CTAs per SM)
            constexpr size_t smb = s3_wgrad_smem_bytes<3, 1, 3, 1, kS2TZ>();
            if (fuse_wgrad && plane_march2d(h) && plane_stencil_ok<T>(h, {q, k, v, dqp, dkp, dvp, dq, dk, dv}) &&
                kernel_smem_once((const void*)hyena_plane_bwd_kernel<T, 3, 1, 3, 1, kS2TZ>, smb)) {
              if (cudaMemsetAsync(dsw, 0, sizeof(float) * 3 * (size_t)d.channels * h.sg.ntaps, st) != cudaSuccess ||
                  (dsb && h.sg.has_bias &&
                   cudaMemsetAsync(dsb, 0, sizeof(float) * 3 * (size_t)d.channels, st) != cudaSuccess)) {
                launch_rc = fail(HYFFT_ERR_CUDA, "memset short-conv gradients");
                return;
              }
              const PlaneLaunch pl = plane_launch(h, 2);
              hyena_plane_bwd_kernel<T, 3, 1, 3, 1, kS2TZ><<<pl.grid, kElemThreads, smb, st>>>(
                  dqp, dkp, dvp, q, k, v, d.in_batch_stride, d.in_pos_stride, dq, dk, dv, pl.g, d.channels, sw, dsw,
                  h.sg.has_bias ? dsb : nullptr, pl.xchunk);
              wgrad_done = true;
              return;
            }
            constexpr size_t sm2 = s3_smem_bytes<3, 1, 3, 1, kS2TZ>();
            if (plane_march2d(h) && plane_stencil_ok<T>(h, {dqp, dkp, dvp, dq, dk, dv}) &&
                kernel_smem_once((const void*)hyena_plane_stencil_kernel<T, 3, 1, 3, 1, 1, kS2TZ>, sm2)) {
              const PlaneLaunch pl = plane_launch(h);
              hyena_plane_stencil_kernel<T, 3, 1, 3, 1, 1, kS2TZ><<<pl.grid, kElemThreads, sm2, st>>>(
                  dqp, dkp, dvp, 0, 0, dq, dk, dv, d.in_batch_stride, d.in_pos_stride, nullptr, pl.g, d.channels,
                  sw, nullptr, 0, pl.xchunk);
              return;
            }
          }
          if (!plane_march2d(h) && plane_stencil_ok<T>(h, {dqp, dkp, dvp, dq, dk, dv}) &&
              kernel_smem_once((const void*)hyena_plane_stencil_kernel<T, PX, 3, 3, 1>, sm)) {
            const PlaneLaunch pl = plane_launch(h);
            hyena_plane_stencil_kernel<T, PX, 3, 3, 1><<<pl.grid, kElemThreads, sm, st>>>(
                dqp, dkp, dvp, 0, 0, dq, dk, dv, d.in_batch_stride, d.in_pos_stride, nullptr, pl.g, d.channels, sw,
                nullptr, 0, pl.xchunk);
            return;
          }
        }
        if (d.ndim == ND) {
          const long long nl = h.sg.n[ND - 1];
          const long long items = (long long)d.batch * (h.Ntot / nl) * ((nl + 63) / 64);
          const dim3 lg((unsigned)((d.channels + kElemCG - 1) / kElemCG),
                        (unsigned)std::max<long long>(1, std::min<long long>(65535, (items + 7) / 8)), 1);
          hyena_line_stencil_kernel<T, P, ND, KA, KB, KI, 1><<<lg, kElemThreads, 0, st>>>(
              dqp, dkp, dvp, 0, 0, dq, dk, dv, d.in_batch_stride, d.in_pos_stride, nullptr, h.sg, d.batch,
              d.channels, sw, nullptr, 0);
          return;
        }
      }
      hyena_short_dgrad_kernel<T, P, K0, K1, K2><<<elem_grid(d.channels, rows, 4), kElemThreads, 0, st>>>(
          dqp, dkp, dvp, h.sg, d.batch, d.channels, sw, dq, dk, dv, d.in_batch_stride, d.in_pos_stride);
    });
  };
  if (pair) dgrad(std::true_type{});
  else dgrad(std::false_type{});
  HY_TRY(check_launch("hyena_short_dgrad_kernel"));
  HY_TRY(launch_rc);
  if (h.sg.has_conv && dsw && !wgrad_done) {
    if (cudaMemsetAsync(dsw, 0, sizeof(float) * 3 * (size_t)d.channels * h.sg.ntaps, st) != cudaSuccess)
      return fail(HYFFT_ERR_CUDA, "memset dshort_w");
    if (dsb && h.sg.has_bias && cudaMemsetAsync(dsb, 0, sizeof(float) * 3 * (size_t)d.channels, st) != cudaSuccess)
      return fail(HYFFT_ERR_CUDA, "memset dshort_b");
    const unsigned gx = (unsigned)((d.channels + kElemCG - 1) / kElemCG);
    // about 16 rows per warp (at least ~4 waves of CTAs); one atomic per channel and tap per CTA
    const long long wz = std::max<long long>(1, std::min<long long>(65535, rows / (8 * 16)));
    const dim3 wg(gx, 3, (unsigned)std::max<long long>(std::min<long long>(wz, std::max<long long>(1, 24000 / (3 * gx))),
                                                       (long long)red_rows(3 * (int)gx)));
    auto wgrad = [&](auto pr) {
      constexpr bool P = decltype(pr)::value;
      with_stencil<P>(h.sg, [&](auto a, auto b, auto c) {
        constexpr int K0 = decltype(a)::value, K1 = decltype(b)::value, K2 = decltype(c)::value;
        if constexpr (K0 > 0 && K1 > 0 && K2 > 0) {
          // sliding-window form: 1D (k,1,1), 2D (k0,k1,1), 3D (k0,k1,k2) along the innermost axis
          constexpr int ND = K2 > 1 ? 3 : (K1 > 1 ? 2 : 1);
          constexpr int KA = ND == 1 ? 1 : K0, KB = ND == 3 ? K1 : 1, KI = ND == 3 ? K2 : (ND == 2 ? K1 : K0);
          if constexpr ((ND == 3 || ND == 2) && P && sizeof(T) == 2 && KA == 3 && KI == 3 && (ND == 2 || KB == 3)) {
            constexpr int PX = ND == 3 ? 3 : 1;
            constexpr size_t sm = s3_wgrad_smem_bytes<PX, 3, 3>();
            if constexpr (ND == 2) {
              constexpr size_t sm2 = s3_wgrad_smem_bytes<3, 1, 3, 1, kS2TZ>();
              if (plane_march2d(h) && plane_stencil_ok<T>(h, {q, k, v, dqp, dkp, dvp}) &&
                  kernel_smem_once((const void*)hyena_plane_wgrad_kernel<T, 3, 1, 3, 1, kS2TZ>, sm2)) {
                const PlaneLaunch pl = plane_launch(h);
                hyena_plane_wgrad_kernel<T, 3, 1, 3, 1, kS2TZ><<<pl.grid, kElemThreads, sm2, st>>>(
                    dqp, dkp, dvp, q, k, v, d.in_batch_stride, d.in_pos_stride, pl.g, d.channels, dsw,
                    h.sg.has_bias ? dsb : nullptr, pl.xchunk);
                return;
              }
            }
            if (!plane_march2d(h) && plane_stencil_ok<T>(h, {q, k, v, dqp, dkp, dvp}) &&
                kernel_smem_once((const void*)hyena_plane_wgrad_kernel<T, PX, 3, 3>, sm)) {
              const PlaneLaunch pl = plane_launch(h);
              hyena_plane_wgrad_kernel<T, PX, 3, 3><<<pl.grid, kElemThreads, sm, st>>>(
                  dqp, dkp, dvp, q, k, v, d.in_batch_stride, d.in_pos_stride, pl.g, d.channels, dsw,
                  h.sg.has_bias ? dsb : nullptr, pl.xchunk);
              return;
            }
          }
          if (d.ndim == ND) {
            const long long nl = h.sg.n[ND - 1];
            const long long items = (long long)d.batch * (h.Ntot / nl) * ((nl + 63) / 64);
            const long long gz = std::max<long long>(1, std::min<long long>(65535, std::min<long long>(
                                                             (items + 7) / 8, 4800 / (3 * (long long)gx))));
            if constexpr (ND == 3)  // one CTA per outer stencil row: 9 taps per thread in registers
              hyena_short_wgrad_line_kernel<T, P, ND, KA, KB, KI, true>
                  <<<dim3(gx, 3 * KA, (unsigned)gz), kElemThreads, 0, st>>>(dqp, dkp, dvp, q, k, v, d.in_batch_stride,
                                                                            d.in_pos_stride, h.sg, d.batch, d.channels,
                                                                            dsw, dsb);
            else
              hyena_short_wgrad_line_kernel<T, P, ND, KA, KB, KI><<<dim3(gx, 3, (unsigned)gz), kElemThreads, 0, st>>>(
                  dqp, dkp, dvp, q, k, v, d.in_batch_stride, d.in_pos_stride, h.sg, d.batch, d.channels, dsw, dsb);
            return;
          }
        }
        hyena_short_wgrad_kernel<T, P, K0, K1, K2><<<wg, kElemThreads, 0, st>>>(
            dqp, dkp, dvp, q, k, v, d.in_batch_stride, d.in_pos_stride, h.sg, d.batch, d.channels, dsw, dsb);
      });
    };
    if (pair) wgrad(std::true_type{});
    else wgrad(std::false_type{});
    HY_TRY(check_launch("hyena_short_wgrad_kernel"));
  }
  return HYFFT_OK;
}

// The mixer passes with the large-grid filter transforms on the side stream; every path
// joins it back into the caller's stream before returning (also after a failure).
template <typename T>
static int hyena_forward_t(const HyenaPlan& h, const T* q, const T* k, const T* v, const float* filt, const float* D,
                           const float* sw, const float* sb, T* y, char* saved, char* ws, cudaStream_t st) {
  SideStream* side = h.cp.big2d ? side_stream() : nullptr;
  const int rc = hyena_forward_body<T>(h, q, k, v, filt, D, sw, sb, y, saved, ws, st, side);
  if (side) {
    const int jc = join_side(side, st);
    if (rc == HYFFT_OK) return jc;
  }
  return rc;
}
template <typename T>
static int hyena_backward_t(const HyenaPlan& h, const T* q, const T* k, const T* v, const float* filt,
                            const float* D, const float* sw, const T* dy, T* dq, T* dk, T* dv, float* dfilt,
                            float* dD, float* dsw, float* dsb, const char* saved, char* ws, cudaStream_t st) {
  SideStream* side = h.cp.big2d ? side_stream() : nullptr;
  const int rc = hyena_backward_body<T>(h, q, k, v, filt, D, sw, dy, dq, dk, dv, dfilt, dD, dsw, dsb, saved, ws, st,
                                        side);
  if (side) {
    const int jc = join_side(side, st);
    if (rc == HYFFT_OK) return jc;
  }
  return rc;
}

static bool aligned16(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p && ((uintptr_t)p % 16) != 0) return false;
  return true;
}

static void fused_params(const HyenaPlan& h, Fused2DParams& p, const void* q, const void* k, const void* v,
                         const float* filt, const float* D, const float* sw, const float* sb) {
  const hyfft_hyena_desc& d = h.d;
  memset(&p, 0, sizeof(p));
  p.q = q;
  p.k = k;
  p.v = v;
  p.in_bst = d.in_batch_stride;
  p.in_pst = d.in_pos_stride;
  p.out_bst = d.out_batch_stride;
  p.out_pst = d.out_pos_stride;
  p.w = sw;
  p.bias = h.sg.has_bias ? sb : nullptr;
  p.D = D;
  p.filt = filt;
  p.B = d.batch;
  p.C = d.channels;
  p.half = (d.batch + 1) / 2;
  p.K0 = h.cp.g.K[0];
  p.K1 = h.cp.g.K[1];
  p.gate1 = d.gate1;
  p.gate2 = d.gate2;
}

// q', k', v' of the fused path sit after the filter spectrum in the saved state
static void fused_saved_acts(const HyenaPlan& h, Fused2DParams& p, const void* saved) {
  char* base = const_cast<char*>(static_cast<const char*>(saved)) +
               align_up((size_t)h.d.channels * h.fF[0] * h.fF[1] * sizeof(float2));
  const size_t act = align_up((size_t)h.E * h.eb);
  p.qs = base;
  p.ks = base + act;
  p.vs = base + 2 * act;
}

static int fused_op(const HyenaPlan& h, int op, const Fused2DParams& p, cudaStream_t st, const char* what) {
  const Geo& g = h.cp.g;
  const int rc = fused2d_dispatch(op, h.d.dtype, g.N[0], g.N[1], h.fF[0], h.fF[1], h.SK, &p, st);
  if (rc != HYFFT_OK) return fail(rc == HYFFT_ERR_UNSUPPORTED ? rc : HYFFT_ERR_CUDA, "%s launch failed", what);
  return HYFFT_OK;
}

static int hyena_fused_forward(const HyenaPlan& h, const void* q, const void* k, const void* v, const float* filt,
                               const float* D, const float* sw, const float* sb, void* y, void* saved,
                               cudaStream_t st) {
  if (!aligned16({q, k, v, y, saved}))
    return fail(HYFFT_ERR_INVALID, "q, k, v, y and saved must be 16-byte aligned");
  Fused2DParams p;
  fused_params(h, p, q, k, v, filt, D, sw, sb);
  p.y = y;
  p.Kbr = static_cast<float2*>(saved);
  fused_saved_acts(h, p, saved);
  HY_TRY(fused_op(h, FOP_KSPEC, p, st, "kspec2d_kernel"));
  return fused_op(h, FOP_FWD, p, st, "hyena2d_fwd_kernel");
}

static int hyena_fused_backward(const HyenaPlan& h, const void* q, const void* k, const void* v, const float* filt,
                                const float* D, const float* sw, const float* sb, const void* dy, void* dq, void* dk,
                                void* dv, float* dfilt, float* dD, float* dsw, float* dsb, const void* saved,
                                void* ws, cudaStream_t st) {
  if (!aligned16({q, k, v, dy, dq, dk, dv, saved, ws}))
    return fail(HYFFT_ERR_INVALID, "q, k, v, dy, dq, dk, dv, saved and workspace must be 16-byte aligned");
  if (!dD || (h.sg.has_conv && !dsw) || (h.sg.has_bias && !dsb))
    return fail(HYFFT_ERR_INVALID, "dD, dshort_w (and dshort_b with a bias) are required");
  const hyfft_hyena_desc& d = h.d;
  Fused2DParams p;
  fused_params(h, p, q, k, v, filt, D, sw, sb);
  p.dy = dy;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.Kbr = const_cast<float2*>(static_cast<const float2*>(saved));
  fused_saved_acts(h, p, saved);
  p.G = static_cast<float2*>(ws);
  p.dfilt = dfilt;
  p.dD = dD;
  p.dw = h.sg.has_conv ? dsw : nullptr;
  p.db = h.sg.has_bias ? dsb : nullptr;
  cudaMemsetAsync(p.G, 0, sizeof(float2) * (size_t)d.channels * h.fF[0] * h.fF[1], st);
  cudaMemsetAsync(dD, 0, sizeof(float) * d.channels, st);
  if (p.dw) cudaMemsetAsync(p.dw, 0, sizeof(float) * 3 * (size_t)d.channels * h.sg.ntaps, st);
  if (p.db) cudaMemsetAsync(p.db, 0, sizeof(float) * 3 * (size_t)d.channels, st);
  HY_TRY(fused_op(h, FOP_BWD, p, st, "hyena2d_bwd_kernel"));
  return fused_op(h, FOP_DFILT, p, st, "dfilt2d_kernel");
}

static int hyena_tp_forward(const HyenaPlan& h, const void* q, const void* k, const void* v, const float* filt,
                            const float* D, const float* sw, const float* sb, void* y, void* ws, cudaStream_t st) {
  if (!aligned16({q, k, v, y, ws})) return fail(HYFFT_ERR_INVALID, "q, k, v and y must be 16-byte aligned");
  Fused2DParams p;
  fused_params(h, p, q, k, v, filt, D, sw, sb);
  p.y = y;
  p.status = static_cast<int*>(ws);
  cudaMemsetAsync(ws, 0, sizeof(int), st);
  const int rc = tp2d_dispatch(TP_FWD, h.cp.g.N[0], h.cp.g.N[1], h.SK, &p, st);
  if (rc != HYFFT_OK) return fail(rc, "tp2d_fwd_kernel launch failed");
  return HYFFT_OK;
}

static int hyena_tp_backward(const HyenaPlan& h, const void* q, const void* k, const void* v, const float* filt,
                             const float* D, const float* sw, const float* sb, const void* dy, void* dq, void* dk,
                             void* dv, float* dfilt, float* dD, float* dsw, float* dsb, void* ws, cudaStream_t st) {
  if (!aligned16({q, k, v, dy, dq, dk, dv, ws}))
    return fail(HYFFT_ERR_INVALID, "q, k, v, dy, dq, dk and dv must be 16-byte aligned");
  if (!dD || (h.sg.has_conv && !dsw) || (h.sg.has_bias && !dsb))
    return fail(HYFFT_ERR_INVALID, "dD, dshort_w (and dshort_b with a bias) are required");
  const hyfft_hyena_desc& d = h.d;
  Fused2DParams p;
  fused_params(h, p, q, k, v, filt, D, sw, sb);
  p.dy = dy;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.dfilt = dfilt;
  p.dD = dD;
  p.dw = h.sg.has_conv ? dsw : nullptr;
  p.db = h.sg.has_bias ? dsb : nullptr;
  p.status = static_cast<int*>(ws);
  cudaMemsetAsync(ws, 0, sizeof(int), st);
  cudaMemsetAsync(dfilt, 0, sizeof(float) * (size_t)d.channels * h.cp.g.K[0] * h.cp.g.K[1], st);
  cudaMemsetAsync(dD, 0, sizeof(float) * d.channels, st);
  if (p.dw) cudaMemsetAsync(p.dw, 0, sizeof(float) * 3 * (size_t)d.channels * h.sg.ntaps, st);
  if (p.db) cudaMemsetAsync(p.db, 0, sizeof(float) * 3 * (size_t)d.channels, st);
  const int rc = tp2d_dispatch(TP_BWD, h.cp.g.N[0], h.cp.g.N[1], h.SK, &p, st);
  if (rc != HYFFT_OK) return fail(rc, "tp2d_bwd_kernel launch failed");
  return HYFFT_OK;
}

}  // namespace hyfft

extern "C" {

int hyfft_hyena_workspace_size(const hyfft_hyena_desc* d, size_t* fwd_bytes, size_t* bwd_bytes, size_t* saved_bytes) {
  HyenaPlan h;
  HY_TRY(make_hyena_plan(d, h));
  size_t f, b, s;
  hyena_sizes(h, f, b, s);
  if (fwd_bytes) *fwd_bytes = f;
  if (bwd_bytes) *bwd_bytes = b;
  if (saved_bytes) *saved_bytes = s;
  return HYFFT_OK;
}

int hyfft_hyena_forward(const hyfft_hyena_desc* d, const void* q, const void* k, const void* v, const float* filt,
                        const float* D, const float* short_w, const float* short_b, void* y, void* saved,
                        void* workspace, size_t workspace_bytes, void* stream) {
  HyenaPlan h;
  HY_TRY(make_hyena_plan(d, h));
  if (!q || !k || !v || !filt || !D || !y) return fail(HYFFT_ERR_INVALID, "null tensor pointer");
  if (bind_device_of(q) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "cannot make the device of the inputs current");
  if (h.sg.has_conv && !short_w) return fail(HYFFT_ERR_INVALID, "short conv weight missing");
  if (h.sg.has_bias && !short_b) return fail(HYFFT_ERR_INVALID, "short conv bias missing");
  size_t f, b, s;
  hyena_sizes(h, f, b, s);
  if (!workspace || workspace_bytes < f) return fail(HYFFT_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, f);
  if (!saved && s > 0) return fail(HYFFT_ERR_WORKSPACE, "saved buffer of %zu bytes required", s);
  cudaStream_t st = (cudaStream_t)stream;
  if (h.tp) return hyena_tp_forward(h, q, k, v, filt, D, short_w, short_b, y, workspace, st);
  if (h.fused) return hyena_fused_forward(h, q, k, v, filt, D, short_w, short_b, y, saved, st);
  if (d->dtype == HYFFT_BF16)
    return hyena_forward_t<__nv_bfloat16>(h, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                                          filt, D, short_w, short_b, (__nv_bfloat16*)y, (char*)saved, (char*)workspace, st);
  if (d->dtype == HYFFT_F16)
    return hyena_forward_t<__half>(h, (const __half*)q, (const __half*)k, (const __half*)v, filt, D, short_w, short_b,
                                   (__half*)y, (char*)saved, (char*)workspace, st);
  return hyena_forward_t<float>(h, (const float*)q, (const float*)k, (const float*)v, filt, D, short_w, short_b,
                                (float*)y, (char*)saved, (char*)workspace, st);
}

int hyfft_hyena_backward(const hyfft_hyena_desc* d, const void* q, const void* k, const void* v, const float* filt,
                         const float* D, const float* short_w, const float* short_b, const void* dy, void* dq, void* dk,
                         void* dv, float* dfilt, float* dD, float* dshort_w, float* dshort_b, const void* saved,
                         void* workspace, size_t workspace_bytes, void* stream) {
  (void)short_b;
  HyenaPlan h;
  HY_TRY(make_hyena_plan(d, h));
  if (!q || !k || !v || !filt || !D || !dy || !dq || !dk || !dv || !dfilt)
    return fail(HYFFT_ERR_INVALID, "null tensor pointer");
  if (bind_device_of(q) != HYFFT_OK) return fail(HYFFT_ERR_CUDA, "cannot make the device of the inputs current");
  if (h.sg.has_conv && !short_w) return fail(HYFFT_ERR_INVALID, "short conv weight missing");
  size_t f, b, s;
  hyena_sizes(h, f, b, s);
  if (!workspace || workspace_bytes < b) return fail(HYFFT_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, b);
  if (!saved && s > 0) return fail(HYFFT_ERR_WORKSPACE, "saved buffer required");
  cudaStream_t st = (cudaStream_t)stream;
  if (h.tp)
    return hyena_tp_backward(h, q, k, v, filt, D, short_w, short_b, dy, dq, dk, dv, dfilt, dD, dshort_w, dshort_b,
                             workspace, st);
  if (h.fused)
    return hyena_fused_backward(h, q, k, v, filt, D, short_w, short_b, dy, dq, dk, dv, dfilt, dD, dshort_w, dshort_b,
                                saved, workspace, st);
  if (d->dtype == HYFFT_BF16)
    return hyena_backward_t<__nv_bfloat16>(h, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                                           filt, D, short_w, (const __nv_bfloat16*)dy, (__nv_bfloat16*)dq,
                                           (__nv_bfloat16*)dk, (__nv_bfloat16*)dv, dfilt, dD, dshort_w, dshort_b,
                                           (const char*)saved, (char*)workspace, st);
  if (d->dtype == HYFFT_F16)
    return hyena_backward_t<__half>(h, (const __half*)q, (const __half*)k, (const __half*)v, filt, D, short_w,
                                    (const __half*)dy, (__half*)dq, (__half*)dk, (__half*)dv, dfilt, dD, dshort_w,
                                    dshort_b, (const char*)saved, (char*)workspace, st);
  return hyena_backward_t<float>(h, (const float*)q, (const float*)k, (const float*)v, filt, D, short_w,
                                 (const float*)dy, (float*)dq, (float*)dk, (float*)dv, dfilt, dD, dshort_w, dshort_b,
                                 (const char*)saved, (char*)workspace, st);
}

}  // extern "C"
