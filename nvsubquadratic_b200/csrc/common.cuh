// Shared device helpers for the B200 Hyena FFT-conv kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/hyfft.h"

namespace hyfft {

// The library links its own (static) CUDA runtime, whose current device is independent
// of the caller's: make the device that owns `p` current before launching anything.
inline int bind_device_of(const void* p) {
  if (!p) return HYFFT_OK;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return HYFFT_OK;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != a.device && cudaSetDevice(a.device) != cudaSuccess) return HYFFT_ERR_CUDA;
  }
  return HYFFT_OK;
}

// Raise a kernel's dynamic shared-memory limit (and, with max_carveout, ask for the
// largest shared-memory carveout) once per kernel and device: the attribute calls are
// driver round trips that would otherwise sit on every launch.
inline bool kernel_smem_once(const void* fn, size_t bytes, bool max_carveout = false) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({fn, dev});
  if (it != done.end() && it->second >= bytes) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) return false;
  if (max_carveout && cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return false;
  done[{fn, dev}] = bytes;
  return true;
}

// ---------------------------------------------------------------- complex
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
// a * conj(b)
__device__ __forceinline__ float2 cmulc(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, a.y * b.y), fmaf(a.y, b.x, -a.x * b.y));
}
// Complex add / subtract as one packed two-lane fp32 instruction on sm_100a (add.rn.f32x2 /
// sub.rn.f32x2: IEEE round-to-nearest per lane, so the results equal two scalar adds) —
// the radix butterflies of every FFT kernel are mostly these, and the kernels are bound by
// instruction issue.
__device__ __forceinline__ float2 cadd(float2 a, float2 b) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  float2 r;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nadd.rn.f32x2 rd, ra, rb;\n"
      "mov.b64 {%0, %1}, rd;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
#else
  return make_float2(a.x + b.x, a.y + b.y);
#endif
}
__device__ __forceinline__ float2 csub(float2 a, float2 b) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  float2 r;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nsub.rn.f32x2 rd, ra, rb;\n"
      "mov.b64 {%0, %1}, rd;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
#else
  return make_float2(a.x - b.x, a.y - b.y);
#endif
}
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }
// (a.x * b.x + c.x, a.y * b.y + c.y), each lane one fused multiply-add rounded to nearest
// (fma.rn.f32x2 on sm_100a: the results equal two fmaf calls)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  float2 r;
  asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
#else
  return make_float2(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y));
#endif
}

// e^{i*pi*x}
__device__ __forceinline__ float2 expipi(float x) {
  float s, c;
  sincospif(x, &s, &c);
  return make_float2(c, s);
}

// ---------------------------------------------------------------- dtypes
template <typename T> struct DT;
template <> struct DT<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct DT<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct DT<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float v) { *p = __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

// ---------------------------------------------------------------- gates
// 0 identity, 1 sigmoid, 2 silu (the activations Hyena.forward applies at
// hyena_nd.py:546 and :570).
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

__device__ __forceinline__ float gate_f(int g, float x) {
  if (g == HYFFT_GATE_SIGMOID) return sigmoidf_(x);
  if (g == HYFFT_GATE_SILU) return x * sigmoidf_(x);
  return x;
}
// derivative of the gate
__device__ __forceinline__ float gate_df(int g, float x) {
  if (g == HYFFT_GATE_SIGMOID) { float s = sigmoidf_(x); return s * (1.0f - s); }
  if (g == HYFFT_GATE_SILU) { float s = sigmoidf_(x); return s * (1.0f + x * (1.0f - s)); }
  return 1.0f;
}

}  // namespace hyfft
