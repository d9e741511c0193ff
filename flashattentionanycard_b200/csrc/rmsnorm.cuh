// Fused RMSNorm, y = x * rsqrt(sum(x^2) / N + eps) * w, fp32 arithmetic,
// cast on store.  Same contract as kernels/rmsnorm.py:7-26 (ROWS_PER_CTA rows
// per CTA, whole row processed by one CTA slice, masked tails).
//
// Vector path (N % 8 == 0, 16-byte aligned pointers): every thread keeps its
// share of the row in registers as 16-byte vectors, so X is read from HBM
// exactly once; the sum of squares is reduced with warp shuffles and, when a
// row spans several warps, through shared memory.  HBM-bound: per row it moves
// 2 * N * sizeof(T) bytes (+ W, which stays in L2/L1).
//
// Generic path (any N / alignment): two passes over the row, the second one
// served from L1/L2.
#pragma once

#include "bokt_device.cuh"

namespace bokt {

template <typename T>
__device__ __forceinline__ float row_reduce_sum(float v, int tpr_log2, float* red) {
  // tpr = threads per row, a power of two.  Rows occupy consecutive threads.
  const int tpr = 1 << tpr_log2;
  if (tpr <= 32) {
    for (int o = tpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  }
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  const int wpr = tpr >> 5;  // warps per row
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  const int first = (warp / wpr) * wpr;
  float s = 0.f;
  for (int w = 0; w < wpr; ++w) s += red[first + w];
  __syncthreads();  // red[] is reused by the caller's next reduction
  return s;
}

template <typename T, int VPT>
__global__ void rmsnorm_vec_kernel(const T* __restrict__ X, const T* __restrict__ W,
                                   T* __restrict__ Y, int M, int N, float eps, int rows_per_cta,
                                   int tpr_log2) {
  __shared__ float red[32];
  pdl_allow_next();
  pdl_wait();
  const int tpr = 1 << tpr_log2;
  const int slot = threadIdx.x >> tpr_log2;
  const int tid = threadIdx.x & (tpr - 1);
  const int row = blockIdx.x * rows_per_cta + slot;
  const bool active = (slot < rows_per_cta) && (row < M);
  const int nvec = N >> 3;

  uint4 xv[VPT];
  float ss = 0.f;
  const uint4* xr = reinterpret_cast<const uint4*>(X + static_cast<size_t>(active ? row : 0) * N);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * tpr;
    if (active && v < nvec) {
      xv[j] = __ldg(xr + v);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&xv[j]);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = Pack2<T>::unpack(u[h]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    } else {
      xv[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  ss = row_reduce_sum<T>(ss, tpr_log2, red);
  const float scale = rsqrtf(ss / static_cast<float>(N) + eps);
  if (!active) return;
  const uint4* wr = reinterpret_cast<const uint4*>(W);
  uint4* yr = reinterpret_cast<uint4*>(Y + static_cast<size_t>(row) * N);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * tpr;
    if (v < nvec) {
      const uint4 wv = __ldg(wr + v);
      const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv[j]);
      const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv);
      uint4 out;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 xf = Pack2<T>::unpack(xu[h]);
        const float2 wf = Pack2<T>::unpack(wu[h]);
        ou[h] = Pack2<T>::pack((xf.x * scale) * wf.x, (xf.y * scale) * wf.y);
      }
      yr[v] = out;
    }
  }
}

template <typename T>
__global__ void rmsnorm_generic_kernel(const T* __restrict__ X, const T* __restrict__ W,
                                       T* __restrict__ Y, int M, int N, float eps,
                                       int rows_per_cta, int tpr_log2) {
  __shared__ float red[32];
  pdl_allow_next();
  pdl_wait();
  const int tpr = 1 << tpr_log2;
  const int slot = threadIdx.x >> tpr_log2;
  const int tid = threadIdx.x & (tpr - 1);
  const int row = blockIdx.x * rows_per_cta + slot;
  const bool active = (slot < rows_per_cta) && (row < M);
  const T* xr = X + static_cast<size_t>(active ? row : 0) * N;
  float ss = 0.f;
  if (active)
    for (int c = tid; c < N; c += tpr) {
      const float f = Pack2<T>::to_float(xr[c]);
      ss = fmaf(f, f, ss);
    }
  ss = row_reduce_sum<T>(ss, tpr_log2, red);
  const float scale = rsqrtf(ss / static_cast<float>(N) + eps);
  if (!active) return;
  T* yr = Y + static_cast<size_t>(row) * N;
  for (int c = tid; c < N; c += tpr)
    yr[c] = Pack2<T>::from_float((Pack2<T>::to_float(xr[c]) * scale) * Pack2<T>::to_float(W[c]));
}

}  // namespace bokt
