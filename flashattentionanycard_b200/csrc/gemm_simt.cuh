// Edge path for GEMM shapes the TMA path cannot describe: a row stride that is
// not a multiple of 16 bytes (K % 8 or N % 8 != 0) or a pointer that is not
// 16-byte aligned, e.g. the 37 x 77 x 93 and 1 x 1 x 1 shapes of the
// reference's tests (tests/test_correctness.py:553).  Plain fp32 FMA, one
// output element per thread, A row staged in shared memory.  Same semantics as
// the tcgen05 path: fp32 accumulation, round on store, every covered element
// written, rows outside the experts' ranges left alone.
#pragma once

#include "bokt_device.cuh"

namespace bokt {

constexpr int kSimtCols = 128;
constexpr int kSimtKChunk = 256;

// grid: (cdiv(N, 128), min(rows, 65535)); rows are strided by gridDim.y.
// Dense: experts == 0, rows = M.  Grouped: rows = T; row r belongs to the
// expert e with clamp(off[e]) <= r < clamp(off[e+1]).
template <typename T>
__global__ void __launch_bounds__(kSimtCols) gemm_simt_kernel(const T* __restrict__ A,
                                                               const T* __restrict__ B,
                                                               T* __restrict__ C, int rows, int N,
                                                               int K, const void* offsets,
                                                               int offsets_i64, int experts) {
  __shared__ float a_row[kSimtKChunk];
  pdl_allow_next();
  pdl_wait();
  const int col = blockIdx.x * kSimtCols + threadIdx.x;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const T* Bp = B;
    if (experts > 0) {
      int found = -1;
      for (int e = 0; e < experts; ++e) {
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
        if (row >= s && row < t) {
          found = e;
          break;
        }
      }
      if (found < 0) continue;  // uniform across the block: same row for all threads
      Bp = B + static_cast<size_t>(found) * K * N;
    }
    float acc = 0.f;
    for (int k0 = 0; k0 < K; k0 += kSimtKChunk) {
      const int kn = min(kSimtKChunk, K - k0);
      __syncthreads();
      for (int k = threadIdx.x; k < kn; k += blockDim.x)
        a_row[k] = Pack2<T>::to_float(A[static_cast<size_t>(row) * K + k0 + k]);
      __syncthreads();
      if (col < N) {
        const T* bcol = Bp + static_cast<size_t>(k0) * N + col;
        for (int k = 0; k < kn; ++k) acc = fmaf(a_row[k], Pack2<T>::to_float(bcol[static_cast<size_t>(k) * N]), acc);
      }
    }
    if (col < N) C[static_cast<size_t>(row) * N + col] = Pack2<T>::from_float(acc);
  }
}

}  // namespace bokt
