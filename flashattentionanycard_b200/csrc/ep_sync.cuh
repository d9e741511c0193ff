// Device-side exchange and synchronisation of the expert-parallel step over
// NVLink peer memory (CUDA IPC mappings of the other ranks' buffers), so that
// a step contains no host collective and can be captured in a CUDA graph.
//
// ep_put_kernel     : copies this rank's chunk into the same offset of every
//                     rank's buffer (the all-gather of the routing ids).
// ep_barrier_kernel : every rank stores its barrier epoch into slot `me` of
//                     every rank's flag array (release, system scope), then
//                     waits until all slots of its own array have reached the
//                     epoch (acquire).  The epoch is a counter in this rank's
//                     device memory advanced by the kernel itself, so graph
//                     replays need no host input; all ranks run the same
//                     sequence of barriers, so their epochs agree.  A slot
//                     may already hold a later epoch (a fast peer moved on):
//                     the wait is ">=".  Waits are bounded: on timeout the
//                     kernel records kStatusWaitTimeout (detail 4000 + peer)
//                     and returns.
//
// Only plain loads and stores to peer memory: no multicast, no NVLS.  The
// ranks must each run on their own GPU (a barrier waits for kernels on the
// other GPUs; ranks sharing one GPU would be separate launches waiting on each
// other, which nothing schedules together).
#pragma once

#include "bokt_device.cuh"

namespace bokt {

constexpr int kEpMaxWorld = 32;

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// dst_ptrs[d] + offset_vecs <- src[0, vecs) for every rank d (16-byte vectors).
__global__ void ep_put_kernel(const uint4* __restrict__ src, long long vecs,
                              uint4* const* __restrict__ dst_ptrs, long long offset_vecs,
                              int world) {
  pdl_allow_next();
  pdl_wait();
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (int d = 0; d < world; ++d) {
    uint4* dst = dst_ptrs[d] + offset_vecs;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < vecs;
         i += stride)
      dst[i] = src[i];
  }
  __threadfence_system();  // the puts are visible system-wide before the next barrier
}

// One warp: lane d signals and then watches rank d.
__global__ void ep_barrier_kernel(int32_t* const* __restrict__ flag_ptrs,
                                  int32_t* __restrict__ epoch, int world, int me,
                                  long long timeout_ns) {
  pdl_allow_next();
  pdl_wait();
  const int lane = threadIdx.x;
  int32_t e = 0;
  if (lane == 0) {
    e = *epoch + 1;
    *epoch = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  __threadfence_system();  // this rank's earlier writes (previous kernels) precede the signal
  if (lane < world) st_release_sys(flag_ptrs[lane] + me, e);
  if (lane < world) {
    const int32_t* mine = flag_ptrs[me] + lane;
    const uint64_t start = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      const uint32_t seen = static_cast<uint32_t>(ld_acquire_sys(mine));
      if (static_cast<int32_t>(seen - static_cast<uint32_t>(e)) >= 0) break;  // ">=", wrap-safe
      if ((it & 63u) == 63u &&
          globaltimer_ns() - start > static_cast<uint64_t>(timeout_ns)) {
        report_status(kStatusWaitTimeout, 4000 + lane);
        break;
      }
    }
  }
  __syncwarp();
}

}  // namespace bokt
