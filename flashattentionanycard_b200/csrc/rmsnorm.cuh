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

namespace bokt {

// Persistent TMA-staged RMSNorm (N % 8 == 0, 16-byte aligned rows).
//   grid: one CTA per SM; CTA c handles rows c, c + grid, c + 2 grid, ...
//   warp `consumers` (the last): producer; its lane 0 streams whole rows into
//     a ring of `slots` row buffers with cp.async.bulk (one mbarrier per slot)
//   warps 0 .. consumers-1: consumer w takes the CTA's rows w, w + consumers,
//     ...: sum of squares from shared memory (warp shuffles only), then
//     y = (x * r) * w with w staged once per CTA in shared memory, 16-byte
//     coalesced stores straight to HBM, then frees the slot.
// Up to `slots` rows per SM are in flight regardless of how fast rows are
// consumed, and no CTA-wide barrier sits on the per-row path.
// slots must be a multiple of the consumer warps: then every use of a slot is
// consumed by the same warp, in order, so a parity wait on the slot's barrier
// can never be satisfied by the completion of an older use of the slot.  The
// host enforces it.  Before the CTA exits, the producer also waits until every
// copy it issued has landed.
template <typename T>
__global__ void __launch_bounds__(1024, 1)
    rmsnorm_ring_kernel(const T* __restrict__ X, const T* __restrict__ W, T* __restrict__ Y, int M,
                        int N, float eps, int slots) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  const int row_bytes = N * static_cast<int>(sizeof(T));
  const int nvec = row_bytes / 16;
  uint4* w_s = reinterpret_cast<uint4*>(smem);
  uint8_t* ring = smem + ((row_bytes + 127) & ~127);
  const int slot_stride = (row_bytes + 127) & ~127;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(slots) * slot_stride);
  uint64_t* empty = full + slots;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + slots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int consumers = (blockDim.x >> 5) - 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  pdl_allow_next();
  pdl_wait();
  const uint4* wg = reinterpret_cast<const uint4*>(W);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) w_s[v] = __ldg(wg + v);
  __syncthreads();

  const int my_rows = M > static_cast<int>(blockIdx.x)
                          ? (M - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x
                          : 0;
  if (warp == consumers) {
    if (lane == 0) {
      int issued = 0;
      for (int k = 0; k < my_rows; ++k) {
        const int s = k % slots;
        const uint32_t phase = static_cast<uint32_t>(k / slots) & 1u;
        if (!mbar_wait(&empty[s], phase ^ 1u, abort_flag, 21)) break;
        const long long row = static_cast<long long>(blockIdx.x) + static_cast<long long>(k) * gridDim.x;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(row_bytes));
        bulk_load(ring + static_cast<size_t>(s) * slot_stride, X + row * N,
                  static_cast<uint32_t>(row_bytes), &full[s]);
        ++issued;
      }
      // Every issued copy has landed before this CTA may exit (bounded waits).
      for (int k = issued - slots > 0 ? issued - slots : 0; k < issued; ++k) {
        const int s = k % slots;
        const uint32_t phase = static_cast<uint32_t>(k / slots) & 1u;
        if (!mbar_wait(&full[s], phase, abort_flag, 23)) break;
      }
    }
  } else {
    for (int k = warp; k < my_rows; k += consumers) {
      const int s = k % slots;
      const uint32_t phase = static_cast<uint32_t>(k / slots) & 1u;
      const bool ok = mbar_wait(&full[s], phase, abort_flag, 22);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint4* xs = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(s) * slot_stride);
      float ss = 0.f;
      for (int v = lane; v < nvec; v += 32) {
        const uint4 xv = xs[v];
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&xv);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = Pack2<T>::unpack(u[h]);
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float scale = rsqrtf(ss / static_cast<float>(N) + eps);
      const long long row = static_cast<long long>(blockIdx.x) + static_cast<long long>(k) * gridDim.x;
      uint4* yr = reinterpret_cast<uint4*>(Y + row * N);
      for (int v = lane; v < nvec; v += 32) {
        const uint4 xv = xs[v];
        const uint4 wv = w_s[v];
        const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv);
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
}

__host__ __device__ inline int rmsnorm_ring_smem_bytes(int n, int elem_bytes, int slots) {
  const int row = ((n * elem_bytes) + 127) & ~127;
  return 128 + row * (slots + 1) + slots * 16 + 16;
}

}  // namespace bokt

namespace bokt {

// Persistent RMSNorm with two register buffers per thread (N % 8 == 0, aligned):
// grid = SMs x resident CTAs; CTA c handles rows c, c + grid, ...  The loads
// of the CTA's next row are issued before the current row is reduced and
// stored, so every SM keeps a row per CTA in flight continuously, and whole
// SMs carry equal row counts (no partial last wave).
template <typename T, int VPT>
__global__ void rmsnorm_pipe_kernel(const T* __restrict__ X, const T* __restrict__ W,
                                    T* __restrict__ Y, int M, int N, float eps, int tpr_log2) {
  __shared__ float red[32];
  pdl_allow_next();
  pdl_wait();
  const int tpr = 1 << tpr_log2;  // == blockDim.x: one row per CTA at a time
  const int tid = threadIdx.x;
  const int nvec = N >> 3;
  uint4 wv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * tpr;
    wv[j] = v < nvec ? __ldg(reinterpret_cast<const uint4*>(W) + v) : make_uint4(0, 0, 0, 0);
  }
  uint4 cur[VPT], nxt[VPT];
  int row = blockIdx.x;
  auto load_row = [&](int r, uint4 (&buf)[VPT]) {
    const uint4* xr = reinterpret_cast<const uint4*>(X + static_cast<size_t>(r) * N);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = tid + j * tpr;
      buf[j] = (r < M && v < nvec) ? __ldg(xr + v) : make_uint4(0, 0, 0, 0);
    }
  };
  load_row(row, cur);
  for (; row < M; row += gridDim.x) {
    load_row(row + gridDim.x, nxt);  // in flight while this row is reduced and stored
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const float2 a = Pack2<T>::unpack(cur[j].x), b = Pack2<T>::unpack(cur[j].y);
      const float2 c = Pack2<T>::unpack(cur[j].z), d = Pack2<T>::unpack(cur[j].w);
      ss = fmaf(a.x, a.x, ss); ss = fmaf(a.y, a.y, ss); ss = fmaf(b.x, b.x, ss); ss = fmaf(b.y, b.y, ss);
      ss = fmaf(c.x, c.x, ss); ss = fmaf(c.y, c.y, ss); ss = fmaf(d.x, d.x, ss); ss = fmaf(d.y, d.y, ss);
    }
    ss = row_reduce_sum<T>(ss, tpr_log2, red);
    const float scale = rsqrtf(ss / static_cast<float>(N) + eps);
    uint4* yr = reinterpret_cast<uint4*>(Y + static_cast<size_t>(row) * N);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = tid + j * tpr;
      if (v < nvec) {
        const float2 xa = Pack2<T>::unpack(cur[j].x), xb = Pack2<T>::unpack(cur[j].y);
        const float2 xc = Pack2<T>::unpack(cur[j].z), xd = Pack2<T>::unpack(cur[j].w);
        const float2 wa = Pack2<T>::unpack(wv[j].x), wb = Pack2<T>::unpack(wv[j].y);
        const float2 wc = Pack2<T>::unpack(wv[j].z), wd = Pack2<T>::unpack(wv[j].w);
        uint4 o;
        o.x = Pack2<T>::pack((xa.x * scale) * wa.x, (xa.y * scale) * wa.y);
        o.y = Pack2<T>::pack((xb.x * scale) * wb.x, (xb.y * scale) * wb.y);
        o.z = Pack2<T>::pack((xc.x * scale) * wc.x, (xc.y * scale) * wc.y);
        o.w = Pack2<T>::pack((xd.x * scale) * wd.x, (xd.y * scale) * wd.y);
        yr[v] = o;
      }
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) cur[j] = nxt[j];
  }
}

}  // namespace bokt
