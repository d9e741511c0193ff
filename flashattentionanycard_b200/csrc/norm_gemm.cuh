// Fused RMSNorm -> GEMM support kernels (sm_100a).
//
// The chain the reference runs as two operators,
//   xn = x * rsqrt(mean(x^2, -1) + eps) * w      (kernels/rmsnorm.py:22-25)
//   out = xn @ B                                 (kernels/gemm.py:7-40)
// is computed as out[m, :] = s[m] * (x[m, :] @ B'), with
//   B'[k, n] = w[k] * B[k, n]                    (folded once per weight pair)
//   s[m] = rsqrt(sum_k x[m, k]^2 / K + eps)      (one HBM-bound pass over x)
// and s applied to the fp32 accumulator in the GEMM epilogue (ROWSCALE
// variants of gemm_tc_kernel / gemm_tc2_kernel), so the normalised
// activations never reach HBM and the GEMM's operand path is untouched.
#pragma once

#include "bokt_device.cuh"

namespace bokt {

constexpr int kRowScaleThreads = 256;

// One warp per row, 16-byte loads (K % 8 == 0), fp32 sum of squares, eight
// loads in flight per lane.
template <typename T>
__global__ void __launch_bounds__(kRowScaleThreads)
    rmsnorm_row_scale_kernel(const T* __restrict__ X, float* __restrict__ scale, int M, int K,
                             float eps) {
  pdl_allow_next();
  pdl_wait();
  const int warps = kRowScaleThreads / 32;
  const int lane = threadIdx.x & 31;
  const int nvec = K / 8;
  const float inv_k = 1.f / static_cast<float>(K);
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const uint4* p = reinterpret_cast<const uint4*>(X + static_cast<size_t>(row) * K);
    float ss = 0.f;
    int i = lane;
    for (; i + 224 < nvec; i += 256) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(p + i + 32 * u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&v[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = Pack2<T>::unpack(w[j]);
          ss = fmaf(x.x, x.x, ss);
          ss = fmaf(x.y, x.y, ss);
        }
      }
    }
    for (; i < nvec; i += 32) {
      const uint4 v = __ldg(p + i);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = Pack2<T>::unpack(w[j]);
        ss = fmaf(x.x, x.x, ss);
        ss = fmaf(x.y, x.y, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) scale[row] = rsqrtf(ss * inv_k + eps);
  }
}

// B'[k, n] = round(w[k] * B[k, n]) over 8-element vectors (N % 8 == 0).
template <typename T>
__global__ void __launch_bounds__(256)
    fold_norm_weight_kernel(const T* __restrict__ w, const T* __restrict__ B, T* __restrict__ Bf,
                            int K, int N) {
  pdl_allow_next();
  pdl_wait();
  const long long nv = static_cast<long long>(N / 8);
  const long long total = nv * K;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i / nv);
    const float g = Pack2<T>::to_float(w[k]);
    uint4 v = __ldg(reinterpret_cast<const uint4*>(B) + i);
    uint32_t* u = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = Pack2<T>::unpack(u[j]);
      u[j] = Pack2<T>::pack(x.x * g, x.y * g);
    }
    reinterpret_cast<uint4*>(Bf)[i] = v;
  }
}

}  // namespace bokt
