// Context-parallel redistribution: the local permutations around the NCCL
// all-to-all that moves a tensor between the sequence-sharded layout
// [B, C, L/P, *rest] (rank r holding zigzag chunks r and 2P-1-r of 2P) and the
// channel-sharded layout [B, C/P, L, *rest] (natural order). The reference
// does each direction as reshape/permute + contiguous + index_select (three
// full copies, nvsubquadratic/parallel/a2a_comms.py:171-282); here each side
// is one gather kernel that moves contiguous runs with 16-byte accesses.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/hyfft.h"
#include "common.cuh"

namespace hyfft {

extern std::atomic<long long> g_launches;

// BHL modes ([B, C, seq, rest]) and channels-last modes ([B, seq*rest, G, C]: positions
// outer, G channel groups, channels innermost; l, L, h count positions incl. rest).
enum CpMode {
  PACK_S2F = 0, UNPACK_S2F = 1, PACK_F2S = 2, UNPACK_F2S = 3,
  CL_PACK_S2F = 4, CL_UNPACK_S2F = 5, CL_PACK_F2S = 6, CL_UNPACK_F2S = 7
};

struct CpDesc {
  int mode;
  long long B, C, d, l, L, h, rest;  // h = chunk length (l / 2 with zigzag)
  int P, zigzag;
  long long rows, run;                // rows of `run` contiguous elements
  long long G;                        // channel groups (channels-last modes)
  // channels-last pack (seq -> chan) / unpack (chan -> seq) on the full-C side: rank j's
  // channels start at j * cblk + coff of the C channels (cblk = d, coff = 0 for the whole block)
  long long cblk, coff;
};

__device__ __forceinline__ void cp_row(const CpDesc& c, long long row, long long& so, long long& dof) {
  switch (c.mode) {
    case PACK_S2F: {  // row = (j, b, cc): dst[j,b,cc,:] = src[b, j*d+cc, :]
      const long long cc = row % c.d, r = row / c.d, b = r % c.B, j = r / c.B;
      so = ((b * c.C + j * c.d + cc) * c.l) * c.rest;
      dof = (((j * c.B + b) * c.d + cc) * c.l) * c.rest;
      break;
    }
    case UNPACK_S2F: {
      if (c.zigzag) {  // row = (b, cc, i) natural chunk i of 2P (length h)
        const long long i = row % (2 * c.P), r = row / (2 * c.P), cc = r % c.d, b = r / c.d;
        const long long j = i < c.P ? i : 2 * c.P - 1 - i;
        const long long half = i < c.P ? 0 : 1;
        dof = ((b * c.d + cc) * c.L + i * c.h) * c.rest;
        so = (((j * c.B + b) * c.d + cc) * c.l + half * c.h) * c.rest;
      } else {  // row = (b, cc, j)
        const long long j = row % c.P, r = row / c.P, cc = r % c.d, b = r / c.d;
        dof = ((b * c.d + cc) * c.L + j * c.l) * c.rest;
        so = (((j * c.B + b) * c.d + cc) * c.l) * c.rest;
      }
      break;
    }
    case PACK_F2S: {
      if (c.zigzag) {  // row = (j, b, cc, half): rank j gets natural chunks j, 2P-1-j
        const long long half = row & 1, r0 = row >> 1, cc = r0 % c.d, r = r0 / c.d, b = r % c.B, j = r / c.B;
        const long long chunk = half ? 2 * c.P - 1 - j : j;
        so = ((b * c.d + cc) * c.L + chunk * c.h) * c.rest;
        dof = (((j * c.B + b) * c.d + cc) * c.l + half * c.h) * c.rest;
      } else {
        const long long cc = row % c.d, r = row / c.d, b = r % c.B, j = r / c.B;
        so = ((b * c.d + cc) * c.L + j * c.l) * c.rest;
        dof = (((j * c.B + b) * c.d + cc) * c.l) * c.rest;
      }
      break;
    }
    case UNPACK_F2S: {  // row = (j, b, cc): dst[b, j*d+cc, :] = src[j, b, cc, :]
      const long long cc = row % c.d, r = row / c.d, b = r % c.B, j = r / c.B;
      dof = ((b * c.P * c.d + j * c.d + cc) * c.l) * c.rest;
      so = (((j * c.B + b) * c.d + cc) * c.l) * c.rest;
      break;
    }
    case CL_PACK_S2F: {  // row = (j, b, t, g): dst[j,b,t,g,:] = src[b,t,g, j*d : (j+1)*d]
      const long long g = row % c.G, r1 = row / c.G, t = r1 % c.l, r2 = r1 / c.l, b = r2 % c.B, j = r2 / c.B;
      so = ((b * c.l + t) * c.G + g) * c.C + j * c.cblk + c.coff;
      dof = (((j * c.B + b) * c.l + t) * c.G + g) * c.d;
      break;
    }
    case CL_UNPACK_S2F: {
      if (c.zigzag) {  // row = (r, b, half): rank r's chunk r (half 0) / 2P-1-r (half 1) -> natural place
        const long long half = row & 1, r1 = row >> 1, b = r1 % c.B, r = r1 / c.B;
        const long long chunk = half ? 2 * c.P - 1 - r : r;
        so = ((r * c.B + b) * c.l + half * c.h) * c.G * c.d;
        dof = (b * c.L + chunk * c.h) * c.G * c.d;
      } else {  // row = (r, b)
        const long long b = row % c.B, r = row / c.B;
        so = (r * c.B + b) * c.l * c.G * c.d;
        dof = (b * c.L + r * c.l) * c.G * c.d;
      }
      break;
    }
    case CL_PACK_F2S: {
      if (c.zigzag) {  // row = (j, b, half): rank j gets natural chunks j, 2P-1-j
        const long long half = row & 1, r1 = row >> 1, b = r1 % c.B, j = r1 / c.B;
        const long long chunk = half ? 2 * c.P - 1 - j : j;
        so = (b * c.L + chunk * c.h) * c.G * c.d;
        dof = ((j * c.B + b) * c.l + half * c.h) * c.G * c.d;
      } else {
        const long long b = row % c.B, j = row / c.B;
        so = (b * c.L + j * c.l) * c.G * c.d;
        dof = (j * c.B + b) * c.l * c.G * c.d;
      }
      break;
    }
    default: {  // CL_UNPACK_F2S: row = (r, b, t, g): dst[b,t,g, r*d : (r+1)*d] = src[r,b,t,g,:]
      const long long g = row % c.G, r1 = row / c.G, t = r1 % c.l, r2 = r1 / c.l, b = r2 % c.B, r = r2 / c.B;
      so = (((r * c.B + b) * c.l + t) * c.G + g) * c.d;
      dof = ((b * c.l + t) * c.G + g) * c.C + r * c.cblk + c.coff;
      break;
    }
  }
}

// Rows are cut into segments of kCpSeg elements (a multiple of 16 bytes) and one warp
// copies one segment at a time, so a few very long rows (whole zigzag chunks) spread over
// the grid as well as many short ones; 16-byte vectors when the run and both offsets
// allow it.
constexpr long long kCpSeg = 4096;

template <typename E>
__global__ void cp_copy_kernel(const E* __restrict__ src, E* __restrict__ dst, CpDesc c, int vec_ok) {
  const int lane = threadIdx.x & 31;
  const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long nseg = (c.run + kCpSeg - 1) / kCpSeg;
  for (long long w = warp; w < c.rows * nseg; w += nwarps) {
    const long long row = w / nseg, sg = w - row * nseg;
    long long so, dof;
    cp_row(c, row, so, dof);
    const long long e0 = sg * kCpSeg, e1 = min(c.run, e0 + kCpSeg);
    if (vec_ok) {
      constexpr int V = 16 / sizeof(E);
      const uint4* s4 = reinterpret_cast<const uint4*>(src + so + e0);
      uint4* d4 = reinterpret_cast<uint4*>(dst + dof + e0);
      const long long nv = (e1 - e0) / V;
      for (long long i = lane; i < nv; i += 32) d4[i] = s4[i];
    } else {
      for (long long i = e0 + lane; i < e1; i += 32) dst[dof + i] = src[so + i];
    }
  }
}

static int cp_launch(CpDesc c, const void* src, void* dst, int eb, cudaStream_t st) {
  if (c.rows <= 0 || c.run <= 0) return HYFFT_OK;
  const bool aligned = ((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0);
  // every row offset is a multiple of `run` or of h*rest; require those to be 16-byte multiples
  int vec_ok;
  if (c.mode >= CL_PACK_S2F) {  // every offset is a multiple of d, C or cblk elements (plus coff)
    vec_ok = aligned && ((c.d * eb) % 16 == 0) && ((c.C * eb) % 16 == 0) && ((c.run * eb) % 16 == 0) &&
             ((c.cblk * eb) % 16 == 0) && ((c.coff * eb) % 16 == 0);
  } else {
    const long long unit = c.zigzag && (c.mode == UNPACK_S2F || c.mode == PACK_F2S) ? c.h * c.rest : c.run;
    vec_ok = aligned && ((c.run * eb) % 16 == 0) && ((unit * eb) % 16 == 0) && ((c.l * c.rest * eb) % 16 == 0) &&
             ((c.L * c.rest * eb) % 16 == 0);
  }
  const long long items = c.rows * ((c.run + kCpSeg - 1) / kCpSeg);
  long long blocks = (items * 32 + 255) / 256;
  if (blocks > 148LL * 32) blocks = 148LL * 32;
  if (blocks < 1) blocks = 1;
  if (eb == 2)
    cp_copy_kernel<uint16_t><<<(unsigned)blocks, 256, 0, st>>>((const uint16_t*)src, (uint16_t*)dst, c, vec_ok);
  else if (eb == 4)
    cp_copy_kernel<uint32_t><<<(unsigned)blocks, 256, 0, st>>>((const uint32_t*)src, (uint32_t*)dst, c, vec_ok);
  else
    return HYFFT_ERR_INVALID;
  if (cudaGetLastError() != cudaSuccess) return HYFFT_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return HYFFT_OK;
}

}  // namespace hyfft

using namespace hyfft;

extern "C" {

int hyfft_cp_pack_split_to_full(const void* src, void* dst, int64_t B, int64_t C, int64_t l, int64_t rest, int32_t P,
                                int32_t elem_bytes, void* stream) {
  if (P < 1 || C % P != 0 || !src || !dst) return HYFFT_ERR_INVALID;
  if (bind_device_of(src) != HYFFT_OK) return HYFFT_ERR_CUDA;
  CpDesc c{};
  c.mode = PACK_S2F;
  c.B = B; c.C = C; c.d = C / P; c.l = l; c.L = l * P; c.h = l; c.rest = rest; c.P = P; c.zigzag = 0;
  c.rows = (long long)P * B * c.d;
  c.run = l * rest;
  return cp_launch(c, src, dst, elem_bytes, (cudaStream_t)stream);
}

int hyfft_cp_unpack_split_to_full(const void* src, void* dst, int64_t B, int64_t d, int64_t l, int64_t rest, int32_t P,
                                  int32_t zigzag, int32_t elem_bytes, void* stream) {
  if (P < 1 || !src || !dst) return HYFFT_ERR_INVALID;
  if (zigzag && (l % 2 != 0)) return HYFFT_ERR_INVALID;
  if (bind_device_of(src) != HYFFT_OK) return HYFFT_ERR_CUDA;
  CpDesc c{};
  c.mode = UNPACK_S2F;
  c.B = B; c.d = d; c.C = d * P; c.l = l; c.L = l * P; c.h = zigzag ? l / 2 : l; c.rest = rest; c.P = P;
  c.zigzag = zigzag ? 1 : 0;
  c.rows = zigzag ? B * d * 2 * P : B * d * P;
  c.run = c.h * rest;
  return cp_launch(c, src, dst, elem_bytes, (cudaStream_t)stream);
}

int hyfft_cp_pack_full_to_split(const void* src, void* dst, int64_t B, int64_t d, int64_t L, int64_t rest, int32_t P,
                                int32_t zigzag, int32_t elem_bytes, void* stream) {
  if (P < 1 || !src || !dst) return HYFFT_ERR_INVALID;
  if (zigzag ? (L % (2 * P) != 0) : (L % P != 0)) return HYFFT_ERR_INVALID;
  if (bind_device_of(src) != HYFFT_OK) return HYFFT_ERR_CUDA;
  CpDesc c{};
  c.mode = PACK_F2S;
  c.B = B; c.d = d; c.C = d * P; c.L = L; c.l = L / P; c.h = zigzag ? L / (2 * P) : L / P; c.rest = rest; c.P = P;
  c.zigzag = zigzag ? 1 : 0;
  c.rows = zigzag ? (long long)P * B * d * 2 : (long long)P * B * d;
  c.run = c.h * rest;
  return cp_launch(c, src, dst, elem_bytes, (cudaStream_t)stream);
}

int hyfft_cp_permute_cl(const void* src, void* dst, int32_t op, int64_t B, int64_t l_rows, int64_t rest, int64_t G,
                        int64_t C, int32_t P, int32_t zigzag, int32_t elem_bytes, void* stream) {
  if (P < 1 || !src || !dst || B < 1 || l_rows < 1 || rest < 1 || G < 1 || C < 1 || C % P != 0)
    return HYFFT_ERR_INVALID;
  if (zigzag && (l_rows % 2 != 0)) return HYFFT_ERR_INVALID;
  if (bind_device_of(src) != HYFFT_OK) return HYFFT_ERR_CUDA;
  CpDesc c{};
  c.B = B; c.C = C; c.d = C / P; c.G = G; c.P = P; c.zigzag = zigzag ? 1 : 0; c.rest = 1;
  c.cblk = c.d; c.coff = 0;
  c.l = l_rows * rest;                        // positions per rank
  c.L = c.l * P;                              // positions of the full sequence
  c.h = zigzag ? (l_rows / 2) * rest : c.l;   // positions per zigzag chunk
  switch (op) {
    case HYFFT_CP_PACK_SEQ_TO_CHAN: c.mode = CL_PACK_S2F; c.rows = (long long)P * B * c.l * G; c.run = c.d; break;
    case HYFFT_CP_UNPACK_SEQ_TO_CHAN:
      c.mode = CL_UNPACK_S2F;
      c.rows = zigzag ? (long long)P * B * 2 : (long long)P * B;
      c.run = (zigzag ? c.h : c.l) * G * c.d;
      break;
    case HYFFT_CP_PACK_CHAN_TO_SEQ:
      c.mode = CL_PACK_F2S;
      c.rows = zigzag ? (long long)P * B * 2 : (long long)P * B;
      c.run = (zigzag ? c.h : c.l) * G * c.d;
      break;
    case HYFFT_CP_UNPACK_CHAN_TO_SEQ: c.mode = CL_UNPACK_F2S; c.rows = (long long)P * B * c.l * G; c.run = c.d; break;
    default: return HYFFT_ERR_INVALID;
  }
  return cp_launch(c, src, dst, elem_bytes, (cudaStream_t)stream);
}

int hyfft_cp_permute_cl_window(const void* src, void* dst, int32_t op, int64_t B, int64_t l_rows, int64_t rest,
                               int64_t G, int64_t C, int32_t P, int64_t c_off, int64_t c_cnt, int32_t elem_bytes,
                               void* stream) {
  if (P < 1 || !src || !dst || B < 1 || l_rows < 1 || rest < 1 || G < 1 || C < 1 || C % P != 0)
    return HYFFT_ERR_INVALID;
  const long long d = C / P;
  if (c_off < 0 || c_cnt < 1 || c_off + c_cnt > d) return HYFFT_ERR_INVALID;
  if (op != HYFFT_CP_PACK_SEQ_TO_CHAN && op != HYFFT_CP_UNPACK_CHAN_TO_SEQ) return HYFFT_ERR_INVALID;
  if (bind_device_of(src) != HYFFT_OK) return HYFFT_ERR_CUDA;
  CpDesc c{};
  c.B = B; c.C = C; c.d = c_cnt; c.G = G; c.P = P; c.zigzag = 0; c.rest = 1;
  c.cblk = d; c.coff = c_off;
  c.l = l_rows * rest;
  c.L = c.l * P;
  c.h = c.l;
  c.mode = op == HYFFT_CP_PACK_SEQ_TO_CHAN ? CL_PACK_S2F : CL_UNPACK_F2S;
  c.rows = (long long)P * B * c.l * G;
  c.run = c_cnt;
  return cp_launch(c, src, dst, elem_bytes, (cudaStream_t)stream);
}

int hyfft_cp_unpack_full_to_split(const void* src, void* dst, int64_t B, int64_t d, int64_t l, int64_t rest, int32_t P,
                                  int32_t elem_bytes, void* stream) {
  if (P < 1 || !src || !dst) return HYFFT_ERR_INVALID;
  if (bind_device_of(src) != HYFFT_OK) return HYFFT_ERR_CUDA;
  CpDesc c{};
  c.mode = UNPACK_F2S;
  c.B = B; c.d = d; c.C = d * P; c.l = l; c.L = l * P; c.h = l; c.rest = rest; c.P = P; c.zigzag = 0;
  c.rows = (long long)P * B * d;
  c.run = l * rest;
  return cp_launch(c, src, dst, elem_bytes, (cudaStream_t)stream);
}

}  // extern "C"
