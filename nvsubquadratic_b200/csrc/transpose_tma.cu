// Channels-last <-> channel-major transposes of 2-byte activations with TMA.
//
//   to_cm:   src [B][N][C] -> dst [B][C][N]
//   !to_cm:  src [B][C][N] -> dst [B][N][C]
//
// One CTA moves one 64 x 64 tile (64 positions x 64 channels, 8 KB): a tiled TMA load
// (cp.async.bulk.tensor, 128-byte swizzle, completion on an mbarrier) brings the tile into
// shared memory, each of the 64 threads transposes one 8 x 8 block of 2-byte elements in
// registers (32 byte permutes), writes it to the output tile (same swizzle), and one TMA
// store writes the tile back. The two tensor maps view the tensors as 2D matrices
// ([B*N][C] and [B*C][N]) over this GPU's own memory, and every copy is CTA-local.
//
// Lane mapping: thread t handles block (a, j) = (t % 8, (t % 8 + t / 8) % 8) of the 8 x 8
// grid of blocks: the 8 threads of a quarter-warp (one 16-byte shared-memory phase) then
// touch 8 different rows and 8 different 16-byte chunks on both the load side (rows 8a+i,
// chunk j ^ i) and the store side (rows 8j+i, chunk a ^ i), so neither side has bank
// conflicts under the 128-byte swizzle (chunk c of row r sits at chunk c ^ (r & 7)).
//
// Applies when C and N are multiples of 64 and both pointers are 16-byte aligned (tiles never
// straddle two images); the caller falls back to the shared-memory tile kernel otherwise.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/hyfft.h"
#include "common.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;

namespace {

constexpr int kTile = 64;                       // positions x channels per tile
constexpr int kTileBytes = kTile * kTile * 2;   // 8 KB

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile of 128-byte rows
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__global__ void __launch_bounds__(64) cl_cm_tma_kernel(const __grid_constant__ CUtensorMap tin,
                                                       const __grid_constant__ CUtensorMap tout, int B, int N, int C,
                                                       int to_cm, int* status) {
  __shared__ __align__(1024) unsigned char tile_in[kTileBytes];
  __shared__ __align__(1024) unsigned char tile_out[kTileBytes];
  __shared__ __align__(8) uint64_t bar;
  const int t = threadIdx.x;
  const int nt = blockIdx.x, ct = blockIdx.y, b = blockIdx.z;
  // input tile coordinates {inner, row}: positions x channels (to_cm) or channels x positions
  const int in_x = to_cm ? ct * kTile : nt * kTile;
  const int in_y = to_cm ? b * N + nt * kTile : b * C + ct * kTile;
  const int out_x = to_cm ? nt * kTile : ct * kTile;
  const int out_y = to_cm ? b * C + ct * kTile : b * N + nt * kTile;
  const uint32_t mb = smem_u32(&bar);
  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mb) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(kTileBytes) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(tile_in)), "l"(&tin), "r"(in_x), "r"(in_y), "r"(mb)
        : "memory");
  }
  __syncthreads();
  // bounded wait for the tile (about a second of clocks), then an error flag instead of a hang
  bool ok = false;
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(mb)
        : "memory");
    if (done) {
      ok = true;
      break;
    }
    if (clock64() - t0 > (1ll << 31)) break;
  }
  if (!ok) {
    if (t == 0 && status) atomicExch(status, 1);
    return;  // nothing was stored; the caller reads the status word
  }
  // 8 x 8 block (a, j): rows 8a..8a+7 of the input tile, 16-byte chunk j of each
  const int a = t & 7, j = (a + (t >> 3)) & 7;
  uint4 R[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) R[i] = *reinterpret_cast<const uint4*>(tile_in + swz(8 * a + i, j));
  uint32_t O[8][4];
#pragma unroll
  for (int ip = 0; ip < 4; ++ip) {
    const uint32_t* lo = reinterpret_cast<const uint32_t*>(&R[2 * ip]);
    const uint32_t* hi = reinterpret_cast<const uint32_t*>(&R[2 * ip + 1]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      O[2 * k][ip] = __byte_perm(lo[k], hi[k], 0x5410);      // element 2k of rows 2ip, 2ip+1
      O[2 * k + 1][ip] = __byte_perm(lo[k], hi[k], 0x7632);  // element 2k+1
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<uint4*>(tile_out + swz(8 * j + i, a)) = make_uint4(O[i][0], O[i][1], O[i][2], O[i][3]);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async proxy
  __syncthreads();
  if (t == 0) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
                 ::"l"(&tout), "r"(out_x), "r"(out_y), "r"(smem_u32(tile_out))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // tile_out must outlive the read
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D map over rows x cols 2-byte elements (cols innermost), 64 x 64 boxes, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {kTile, kTile};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// HYFFT_OK when launched; HYFFT_ERR_UNSUPPORTED (nothing launched) when the shape, the
// alignment or the driver does not allow the TMA form.
int cl_cm_tma(const void* src, void* dst, int B, long long N, int C, bool to_cm, int* status, cudaStream_t st) {
  if (getenv("HYFFT_DISABLE_TMA")) return HYFFT_ERR_UNSUPPORTED;
  if (B < 1 || N % kTile != 0 || C % kTile != 0 || (long long)B * N >= (1LL << 31) ||
      (long long)B * C >= (1LL << 31) || ((uintptr_t)src % 16) != 0 || ((uintptr_t)dst % 16) != 0)
    return HYFFT_ERR_UNSUPPORTED;
  CUtensorMap tin, tout;
  const long long rows_cl = (long long)B * N, rows_cm = (long long)B * C;
  const bool made = to_cm ? (make_map(&tin, src, rows_cl, C) && make_map(&tout, dst, rows_cm, N))
                          : (make_map(&tin, src, rows_cm, N) && make_map(&tout, dst, rows_cl, C));
  if (!made) return HYFFT_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)(N / kTile), (unsigned)(C / kTile), (unsigned)B);
  cl_cm_tma_kernel<<<grid, 64, 0, st>>>(tin, tout, B, (int)N, C, to_cm ? 1 : 0, status);
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

}  // namespace hyfft
