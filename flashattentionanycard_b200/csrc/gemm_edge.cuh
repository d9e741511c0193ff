// Tensor-core edge path for GEMM shapes TMA cannot describe: a row stride
// that is not a multiple of 16 bytes (K % 8 or N % 8 != 0) or a pointer that
// is not 16-byte aligned, e.g. the 37 x 77 x 93, 1 x 1 x 1 and 127 x 193 x 257
// shapes of the reference's tests (tests/test_correctness.py:83-104), whose
// Triton kernel runs them on tensor cores with masked loads
// (kernels/gemm.py:33-38).
//
// One CTA (8 warps) per 128 x 64 output tile, tcgen05.mma.cta_group::1 with
// M = 128, N = 64 accumulating in 64 TMEM columns.  Per 64-wide k-block the
// CTA's threads load the A tile (128 rows x 64 k) and the B tile (64 k x 64
// columns) element by element with bounds checks (zero outside the matrix)
// into registers, then write them into the 128-byte-swizzled shared-memory
// layouts the TMA path produces, so the MMA uses the same descriptors; one
// elected thread issues the four K = 16 MMAs and commits them to an mbarrier
// that every thread waits on (bounded) before the tile buffers are refilled,
// while the next k-block's loads are already in flight.  The epilogue
// reads TMEM (warp w: tile rows 32 (w % 4) .. +31, the lane quadrant it may
// access, and columns 32 (w / 4) .. +31) and stores every element inside the
// matrix, rounded to the element type.
//
// Same semantics as the main path: fp32 accumulation, every covered element
// written, rows outside the experts' ranges (grouped) left alone.
#pragma once

#include "bokt_device.cuh"

namespace bokt {

constexpr int kEdgeBM = 128;
constexpr int kEdgeBN = 64;
constexpr int kEdgeBK = 64;
constexpr int kEdgeThreads = 256;
constexpr int kEdgeRowStep = kEdgeThreads / 64;  // rows a thread skips between its loads
constexpr int kEdgeABytes = kEdgeBM * kEdgeBK * 2;  // 16 KB
constexpr int kEdgeBBytes = kEdgeBK * kEdgeBN * 2;  // 8 KB
constexpr int kEdgeSmemBytes = 1024 + kEdgeABytes + kEdgeBBytes + 64;

// Offset of element (row, col) in a 128-byte-swizzled tile whose rows are 64
// 16-bit elements (128 bytes): the 16-byte chunk index is XORed with row % 8.
__device__ __forceinline__ uint32_t sw128_offset(int row, int col) {
  return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

// Rows [start, start + count) of expert e, offsets clamped to [0, rows].
__device__ __forceinline__ void edge_expert_rows(const void* offsets, int offsets_i64, int e,
                                                 int rows, int* start, int* count) {
  long long s, t;
  if (offsets_i64) {
    s = reinterpret_cast<const long long*>(offsets)[e];
    t = reinterpret_cast<const long long*>(offsets)[e + 1];
  } else {
    s = reinterpret_cast<const int*>(offsets)[e];
    t = reinterpret_cast<const int*>(offsets)[e + 1];
  }
  s = s < 0 ? 0 : (s > rows ? rows : s);
  t = t < s ? s : (t > rows ? rows : t);
  *start = static_cast<int>(s);
  *count = static_cast<int>(t - s);
}

// grid: one CTA per tile.  Dense (experts == 0): cdiv(rows, 128) x cdiv(N, 64)
// tiles, n fastest.  Grouped: the tiles of expert 0, then expert 1, ...
// (cdiv(c_e, 128) x cdiv(N, 64) each); CTAs past the last tile exit.
template <typename T>
__global__ void __launch_bounds__(kEdgeThreads) gemm_tc_edge_kernel(
    const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, int rows, int N, int K,
    const void* offsets, int offsets_i64, int experts, uint32_t idesc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kEdgeABytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + kEdgeBBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* tile_info = reinterpret_cast<int*>(tmem_holder + 2);  // a_row, rows_valid, n0, expert

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nn = (N + kEdgeBN - 1) / kEdgeBN;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, kEdgeBN);
    tmem_relinquish();
  }
  pdl_allow_next();
  pdl_wait();
  if (threadIdx.x == 0) {
    int t = blockIdx.x, a_row = -1, valid = 0, n0 = 0, expert = 0;
    if (experts == 0) {
      const int mb = t / nn;
      a_row = mb * kEdgeBM;
      n0 = (t - mb * nn) * kEdgeBN;
      valid = min(kEdgeBM, rows - a_row);
    } else {
      for (int e = 0; e < experts; ++e) {
        int start, count;
        edge_expert_rows(offsets, offsets_i64, e, rows, &start, &count);
        const int tiles = ((count + kEdgeBM - 1) / kEdgeBM) * nn;
        if (t < tiles) {
          const int mb = t / nn;
          a_row = start + mb * kEdgeBM;
          n0 = (t - mb * nn) * kEdgeBN;
          valid = min(kEdgeBM, count - mb * kEdgeBM);
          expert = e;
          break;
        }
        t -= tiles;
      }
    }
    tile_info[0] = a_row;
    tile_info[1] = valid;
    tile_info[2] = n0;
    tile_info[3] = expert;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int a_row = tile_info[0];
  const int valid = tile_info[1];
  const int n0 = tile_info[2];
  const T* Bp = B + static_cast<size_t>(tile_info[3]) * K * N;
  const T zero = Pack2<T>::from_float(0.f);

  bool ok = a_row >= 0 && valid > 0;  // uniform: CTA past the last grouped tile does nothing
  const int nkb = (K + kEdgeBK - 1) / kEdgeBK;
  // Thread t loads column c = t % 64 of the tiles (k for A, n for B) in rows
  // r0, r0 + 4, ... (r0 = t / 64): a warp reads 32 consecutive elements of a
  // row.  Each k-block's elements are loaded into registers first (all loads
  // in flight together), then written to shared memory; the next k-block's
  // loads are issued while the tensor cores work on the current one.
  const int c = threadIdx.x & 63;
  const int r0 = threadIdx.x >> 6;
  const bool n_ok = n0 + c < N;
  constexpr int kAPer = kEdgeBM / kEdgeRowStep, kBPer = kEdgeBK / kEdgeRowStep;
  T va[kAPer], vb[kBPer];
  const T* a_col = A + static_cast<size_t>(a_row + r0) * K + c;
  const T* b_col = Bp + static_cast<size_t>(r0) * N + n0 + c;
  const size_t a_step = static_cast<size_t>(kEdgeRowStep) * K;
  const size_t b_step = static_cast<size_t>(kEdgeRowStep) * N;
  auto load_block = [&](int kb) {
    const int k0 = kb * kEdgeBK;
    const bool k_ok = k0 + c < K;
    const T* pa = a_col + k0;
#pragma unroll
    for (int j = 0; j < kAPer; ++j)
      va[j] = (k_ok && r0 + kEdgeRowStep * j < valid) ? pa[j * a_step] : zero;
    const T* pb = b_col + static_cast<size_t>(k0) * N;
#pragma unroll
    for (int j = 0; j < kBPer; ++j)
      vb[j] = (n_ok && k0 + r0 + kEdgeRowStep * j < K) ? pb[j * b_step] : zero;
  };
  if (ok && nkb > 0) load_block(0);
  for (int kb = 0; ok && kb < nkb; ++kb) {
#pragma unroll
    for (int j = 0; j < kAPer; ++j)
      *reinterpret_cast<T*>(sA + sw128_offset(r0 + kEdgeRowStep * j, c)) = va[j];
#pragma unroll
    for (int j = 0; j < kBPer; ++j)
      *reinterpret_cast<T*>(sB + sw128_offset(r0 + kEdgeRowStep * j, c)) = vb[j];
    // The tensor cores read shared memory through the async proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      tc_fence_after();
      const uint32_t a_addr = smem_addr(sA);
      const uint32_t b_addr = smem_addr(sB);
#pragma unroll
      for (int k = 0; k < kEdgeBK / 16; ++k) {
        const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
        const uint64_t b_desc = smem_desc_sw128(b_addr + k * 2048, 64 * 128, 1024);
        umma_f16_ss(tmem_base, a_desc, b_desc, idesc, (kb | k) != 0 ? 1u : 0u);
      }
      umma_commit(bar);
    }
    if (kb + 1 < nkb) load_block(kb + 1);
    ok = mbar_wait(bar, static_cast<uint32_t>(kb & 1), abort_flag, 31);
    ok = __syncthreads_and(ok);
    tc_fence_after();
  }
  const int q = warp & 3;         // TMEM lane quadrant: tile rows 32 q .. 32 q + 31
  const int half = warp >> 2;     // columns 32 half .. 32 half + 31
  const int r = q * 32 + lane;
  const int col0 = half * 32;
  if (ok && nkb > 0) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                           static_cast<uint32_t>(col0), v);
    tmem_ld_wait();
    if (r < valid) {
      T* crow = C + static_cast<size_t>(a_row + r) * N + n0 + col0;
      const int ncols = min(32, N - n0 - col0);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) crow[j] = Pack2<T>::from_float(__uint_as_float(v[j]));
    }
  } else if (ok && valid > 0 && r < valid) {
    // K == 0: C = 0 for the tile.
    for (int j = 0; j < 32 && n0 + col0 + j < N; ++j)
      C[static_cast<size_t>(a_row + r) * N + n0 + col0 + j] = zero;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kEdgeBN);
  }
}

}  // namespace bokt
