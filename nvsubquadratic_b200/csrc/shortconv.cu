// Direct depthwise causal 1D convolution (no FFT), forward and backward, channel-major
// [B, C, L] activations:
//
//   pre[b, c, t] = sum_{k < K} w[c, k] * x[b, c, t - (K - 1) + k] + bias[c]   (x = 0 before t = 0)
//   y = act(pre),  act = identity or SiLU
//
// i.e. F.conv1d(F.pad(x, (K - 1, 0)), w[:, None, :], bias, groups=C), the semantics the
// reference op causal_conv1d pins (nvsubquadratic/ops/causal_conv1d_custom.py:81-98, its
// test tests/ops/test_causal_conv1d_custom.py:62-68). The conv is rounded to the
// activation dtype before the activation, and the activation's result again, as the
// reference's two dtype-preserving torch ops round.
//
// One CTA owns a segment of kSeg outputs of one (b, c) row: the segment's inputs plus the
// K - 1 samples before it are staged in shared memory as float (neighbouring threads read
// neighbouring samples), each thread computes 4 neighbouring outputs from a register
// window. The backward CTA recomputes pre over its segment plus the K - 1 samples after
// it, forms dpre = dy * act'(pre), and produces dx for the segment (the transposed
// stencil) and its share of dw / dbias (per-CTA sums, one float atomic per tap).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "../../include/hyfft.h"
#include "common.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;

namespace {

constexpr int kScThreads = 256;
constexpr int kScPer = 4;                         // outputs per thread
constexpr int kSeg = kScThreads * kScPer;         // outputs per CTA
constexpr int kScMaxK = 1024;                     // longest filter the kernels take

__device__ __forceinline__ float silu_f(float v) { return v / (1.f + expf(-v)); }
__device__ __forceinline__ float silu_df(float v) {
  const float s = 1.f / (1.f + expf(-v));
  return s * (1.f + v * (1.f - s));
}

// row[i] = x[t0 - halo + i] for i < n (zero outside [0, L)), float.
template <typename T>
__device__ __forceinline__ void load_row(float* row, const T* __restrict__ xr, long long L, long long t0, int halo,
                                         int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const long long t = t0 - halo + i;
    row[i] = (t >= 0 && t < L) ? DT<T>::load(xr + t) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kScThreads) causal_conv1d_fwd_kernel(const T* __restrict__ x,
                                                                       const float* __restrict__ w,
                                                                       const float* __restrict__ bias, T* __restrict__ y,
                                                                       int C, long long L, int K, int act) {
  extern __shared__ float sm[];
  float* ws = sm;          // [K]
  float* row = sm + K;     // [K - 1 + kSeg]
  const int c = blockIdx.y, b = blockIdx.z;
  const long long t0 = (long long)blockIdx.x * kSeg;
  const long long rb = ((long long)b * C + c) * L;
  for (int k = threadIdx.x; k < K; k += blockDim.x) ws[k] = w[(long long)c * K + k];
  load_row<T>(row, x + rb, L, t0, K - 1, K - 1 + kSeg);
  __syncthreads();
  const float bc = bias ? bias[c] : 0.f;
  const int i0 = threadIdx.x * kScPer;  // outputs t0 + i0 .. t0 + i0 + 3; row index i + k
  float acc[kScPer];
#pragma unroll
  for (int u = 0; u < kScPer; ++u) acc[u] = bc;
  float win[kScPer];
#pragma unroll
  for (int u = 0; u < kScPer - 1; ++u) win[u + 1] = row[i0 + u];
  for (int k = 0; k < K; ++k) {
    // window of row[i0 + k .. i0 + k + 3]
#pragma unroll
    for (int u = 0; u < kScPer - 1; ++u) win[u] = win[u + 1];
    win[kScPer - 1] = row[i0 + k + kScPer - 1];
    const float wk = ws[k];
#pragma unroll
    for (int u = 0; u < kScPer; ++u) acc[u] = fmaf(wk, win[u], acc[u]);
  }
  T* yr = y + rb;
#pragma unroll
  for (int u = 0; u < kScPer; ++u) {
    const long long t = t0 + i0 + u;
    if (t < L) {
      float v = DT<T>::round(acc[u]);
      if (act) v = silu_f(v);
      DT<T>::store(yr + t, v);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kScThreads) causal_conv1d_bwd_kernel(
    const T* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias, const T* __restrict__ dy,
    T* __restrict__ dx, float* __restrict__ dw, float* __restrict__ db, int C, long long L, int K, int act) {
  extern __shared__ float sm[];
  const int n = kSeg + K - 1;     // dpre over [t0, t0 + kSeg + K - 1)
  float* ws = sm;                 // [K]
  float* xrow = ws + K;           // x over [t0 - (K - 1), t0 + kSeg + K - 1): 2 (K - 1) + kSeg
  float* dp = xrow + n + K - 1;   // dpre over [t0, t0 + n)
  const int c = blockIdx.y, b = blockIdx.z;
  const long long t0 = (long long)blockIdx.x * kSeg;
  const long long rb = ((long long)b * C + c) * L;
  for (int k = threadIdx.x; k < K; k += blockDim.x) ws[k] = w[(long long)c * K + k];
  load_row<T>(xrow, x + rb, L, t0, K - 1, n + K - 1);
  __syncthreads();
  const float bc = bias ? bias[c] : 0.f;
  const T* dyr = dy + rb;
  // dpre[i] for position t0 + i (zero past L)
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const long long t = t0 + i;
    float g = 0.f;
    if (t < L) {
      g = DT<T>::load(dyr + t);
      if (act) {
        float pre = bc;
        for (int k = 0; k < K; ++k) pre = fmaf(ws[k], xrow[i + k], pre);
        g = DT<T>::round(g * silu_df(DT<T>::round(pre)));
      }
    }
    dp[i] = g;
  }
  __syncthreads();
  // dx[t] = sum_k w[k] dpre[t + (K - 1) - k] for t in the segment
  const int i0 = threadIdx.x * kScPer;
  float acc[kScPer] = {0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < K; ++k) {
    const float wk = ws[K - 1 - k];
#pragma unroll
    for (int u = 0; u < kScPer; ++u) acc[u] = fmaf(wk, dp[i0 + u + k], acc[u]);
  }
  T* dxr = dx + rb;
#pragma unroll
  for (int u = 0; u < kScPer; ++u) {
    const long long t = t0 + i0 + u;
    if (t < L) DT<T>::store(dxr + t, acc[u]);
  }
  // dw[k] += sum_{t in segment} dpre[t] x[t - (K - 1) + k]: row index of x is (t - t0) + k
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg_n = (int)min((long long)kSeg, L - t0);
  for (int k = warp; k < K + 1; k += kScThreads / 32) {
    float s = 0.f;
    if (k < K) {
      for (int i = lane; i < seg_n; i += 32) s = fmaf(dp[i], xrow[i + k], s);
    } else {
      for (int i = lane; i < seg_n; i += 32) s += dp[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      if (k < K) atomicAdd(dw + (long long)c * K + k, s);
      else if (db) atomicAdd(db + c, s);
    }
  }
}

template <typename T>
int launch_fwd(const void* x, const float* w, const float* bias, void* y, long long B, long long C, long long L, int K,
               int act, cudaStream_t st) {
  const size_t sm = sizeof(float) * ((size_t)K + K - 1 + kSeg);
  auto kern = causal_conv1d_fwd_kernel<T>;
  if (!kernel_smem_once((const void*)kern, sm)) return HYFFT_ERR_CUDA;
  const dim3 grid((unsigned)((L + kSeg - 1) / kSeg), (unsigned)C, (unsigned)B);
  kern<<<grid, kScThreads, sm, st>>>((const T*)x, w, bias, (T*)y, (int)C, L, K, act);
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

template <typename T>
int launch_bwd(const void* x, const float* w, const float* bias, const void* dy, void* dx, float* dw, float* db,
               long long B, long long C, long long L, int K, int act, cudaStream_t st) {
  const int n = kSeg + K - 1;
  const size_t sm = sizeof(float) * ((size_t)K + (n + K - 1) + n);
  auto kern = causal_conv1d_bwd_kernel<T>;
  if (!kernel_smem_once((const void*)kern, sm)) return HYFFT_ERR_CUDA;
  const dim3 grid((unsigned)((L + kSeg - 1) / kSeg), (unsigned)C, (unsigned)B);
  kern<<<grid, kScThreads, sm, st>>>((const T*)x, w, bias, (const T*)dy, (T*)dx, dw, db, (int)C, L, K, act);
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

int check_args(const void* x, const float* w, long long B, long long C, long long L, int K, int act, int dtype) {
  if (!x || !w) return HYFFT_ERR_INVALID;
  if (B < 1 || C < 1 || L < 1 || K < 1 || C > 65535 || B > 65535) return HYFFT_ERR_INVALID;
  if (act != 0 && act != 1) return HYFFT_ERR_INVALID;
  if (dtype < HYFFT_F32 || dtype > HYFFT_F16) return HYFFT_ERR_INVALID;
  if (K > kScMaxK) return HYFFT_ERR_UNSUPPORTED;
  if ((L + kSeg - 1) / kSeg > 0x7fffffffLL) return HYFFT_ERR_UNSUPPORTED;
  return HYFFT_OK;
}

}  // namespace
}  // namespace hyfft

using namespace hyfft;

extern "C" {

int hyfft_causal_conv1d_forward(const void* x, const float* weight, const float* bias, void* y, int64_t B, int64_t C,
                                int64_t L, int32_t K, int32_t activation, int32_t dtype, void* stream) {
  const int rc = check_args(x, weight, B, C, L, K, activation, dtype);
  if (rc != HYFFT_OK) return rc;
  if (!y) return HYFFT_ERR_INVALID;
  if (bind_device_of(x) != HYFFT_OK) return HYFFT_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == HYFFT_F32) return launch_fwd<float>(x, weight, bias, y, B, C, L, K, activation, st);
  if (dtype == HYFFT_BF16) return launch_fwd<__nv_bfloat16>(x, weight, bias, y, B, C, L, K, activation, st);
  return launch_fwd<__half>(x, weight, bias, y, B, C, L, K, activation, st);
}

int hyfft_causal_conv1d_backward(const void* x, const float* weight, const float* bias, const void* dy, void* dx,
                                 float* dweight, float* dbias, int64_t B, int64_t C, int64_t L, int32_t K,
                                 int32_t activation, int32_t dtype, void* stream) {
  const int rc = check_args(x, weight, B, C, L, K, activation, dtype);
  if (rc != HYFFT_OK) return rc;
  if (!dy || !dx || !dweight) return HYFFT_ERR_INVALID;
  if (bind_device_of(x) != HYFFT_OK) return HYFFT_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(dweight, 0, sizeof(float) * (size_t)C * K, st) != cudaSuccess) return HYFFT_ERR_CUDA;
  if (dbias && cudaMemsetAsync(dbias, 0, sizeof(float) * (size_t)C, st) != cudaSuccess) return HYFFT_ERR_CUDA;
  if (dtype == HYFFT_F32)
    return launch_bwd<float>(x, weight, bias, dy, dx, dweight, dbias, B, C, L, K, activation, st);
  if (dtype == HYFFT_BF16)
    return launch_bwd<__nv_bfloat16>(x, weight, bias, dy, dx, dweight, dbias, B, C, L, K, activation, st);
  return launch_bwd<__half>(x, weight, bias, dy, dx, dweight, dbias, B, C, L, K, activation, st);
}

}  // extern "C"
