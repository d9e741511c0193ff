// Split-K / stream-K work decomposition for the tcgen05 GEMM kernels.
//
// The reference's kernel (kernels/gemm.py:31-39) gives every output tile one
// program that runs the whole K loop.  With SPLIT_K = S > 1 the K loop of
// every tile is cut into S slices of (nearly) equal k-block counts, the
// (tile, slice) work units are laid out tile-major and the U = tiles * S units
// are dealt out in G contiguous runs, one per worker (CTA, or CTA pair):
// worker w owns units [w U / G, (w + 1) U / G).  Inside its run a worker sees
// maximal stretches of units of one tile, "segments" (tile, k-blocks
// [kb0, kb1)), and accumulates each segment in TMEM as an ordinary tile.
// S equal to the number of k-blocks is stream-K: every worker gets the same
// number of k-block iterations whatever the tile count.
//
// Fix-up.  The segment that starts at k-block 0 owns the tile: its epilogue
// adds the fp32 partial sums of the tile's other segments and writes the
// output.  A segment that starts after k-block 0 is always the FIRST segment
// of its worker's run (every later segment of a run starts a new tile), so
//   * a worker writes at most one partial, into its own workspace slot, and
//     it does so before anything else; it never waits for another worker;
//   * an owner waits only for those first segments, of the workers right
//     after it (their runs start inside the owner's tile).
// No wait depends on a waiting worker, so the schedule cannot deadlock once
// every worker is resident (grid <= one CTA per SM), and every wait is
// bounded anyway.  The owner adds the partials in worker order, so the result
// is deterministic run to run.  Each epilogue warp publishes and consumes the
// 32 rows it holds on its own (one flag per warp and slot): no barrier across
// the epilogue warps, so a warp that gives up cannot leave the others stuck.
//
// Workspace (caller-owned device memory, zero-filled once when allocated):
//   [0, 256)      header: word 0 = launch sequence number, word 1 = count of
//                 CTAs that finished the current launch
//   [256, ...)    four 32-bit ready flags per CTA slot, one per epilogue warp
//                 (rows 32 q .. 32 q + 31 of the slot), padded to 256 bytes
//   then          one fp32 partial tile per CTA slot: 128 rows x BN columns,
//                 stored as [BN / 4][128 rows][4 columns] so that a warp's 32
//                 consecutive rows of one 4-column group are 512 contiguous bytes.
// Separate reduction (dense GEMMs with S >= kSplitKReduceMin): with many slices
// per tile the owner's serial fix-up dominates, so instead every segment that
// does not cover its whole tile stores its fp32 partial -- a worker's first
// segment into its slot 2 c, its last into 2 c + 1 (c = CTA slot) -- without
// flags or waits, and splitk_reduce_kernel, launched right after on the same
// stream, sums each split tile's partials in worker order across all SMs and
// writes C.  Tiles a single worker covers are written by the GEMM directly.
//
// A flag holds the sequence number (+1) of the launch that filled the slot, so
// no flag has to be cleared between launches: each launch reads the sequence
// number when it starts and the last CTA to finish advances it.  Launches that
// share one workspace must therefore not overlap on the GPU (one stream, or
// one workspace per stream).
#pragma once

#include "bokt_device.cuh"

namespace bokt {

constexpr int kSplitKMax = 128;
// Dense GEMMs with at least this many slices use the separate reduction.
constexpr int kSplitKReduceMin = 4;
constexpr int kSplitKHeaderBytes = 256;
constexpr uint64_t kSplitKWaitNs = 2000000000ull;

__host__ __device__ inline int64_t splitk_flags_bytes(int slots) {
  return ((int64_t(slots) * 4 * 4 + 255) / 256) * 256;
}

// Two partial tiles per CTA slot: the owner fix-up uses the first; the
// separate reduction uses both (a worker's first and last segments).
__host__ __device__ inline int64_t splitk_workspace_bytes(int slots, int bn) {
  return kSplitKHeaderBytes + splitk_flags_bytes(slots) + 2 * int64_t(slots) * 128 * bn * 4;
}

// A stretch of one tile's k-blocks processed by one worker.
struct Segment {
  int tile;
  int kb0;  // first k-block
  int kb1;  // one past the last k-block
};

// Walks one worker's segments.  split == 1: the plain persistent schedule
// (tiles worker, worker + G, ...).  split > 1: the contiguous run of units.
// `workers` must be splitk_workers(): with more workers than units some runs
// would be empty, and an empty run never publishes the partial an owner
// counts on.
struct SegmentCursor {
  long long u;
  long long u_end;
  int stride;
};

__host__ __device__ inline int splitk_workers(int launched, int ntiles, int split) {
  if (split <= 1) return launched;
  const long long units = static_cast<long long>(ntiles) * split;
  return units < launched ? static_cast<int>(units) : launched;
}

__host__ __device__ inline long long splitk_run_start(int worker, int workers, long long units) {
  return units * worker / workers;
}

__host__ __device__ inline int splitk_slice_begin(int j, int split, int nkb) {
  return static_cast<int>(static_cast<long long>(j) * nkb / split);
}

__host__ __device__ inline SegmentCursor segment_cursor(int worker, int workers, int ntiles,
                                                        int split) {
  SegmentCursor c;
  if (split <= 1) {
    c.u = worker;
    c.u_end = ntiles;
    c.stride = workers;
  } else {
    const long long units = static_cast<long long>(ntiles) * split;
    if (worker >= workers) {  // idle: more CTAs than units
      c.u = c.u_end = 0;
    } else {
      c.u = splitk_run_start(worker, workers, units);
      c.u_end = splitk_run_start(worker + 1, workers, units);
    }
    c.stride = 0;
  }
  return c;
}

__host__ __device__ inline bool segment_next(SegmentCursor& c, int split, int nkb, Segment& s) {
  if (c.u >= c.u_end) return false;
  if (split <= 1) {
    s.tile = static_cast<int>(c.u);
    s.kb0 = 0;
    s.kb1 = nkb;
    c.u += c.stride;
    return true;
  }
  const long long t = c.u / split;
  const long long tile_end = (t + 1) * split;
  const long long e = c.u_end < tile_end ? c.u_end : tile_end;
  s.tile = static_cast<int>(t);
  s.kb0 = splitk_slice_begin(static_cast<int>(c.u - t * split), split, nkb);
  s.kb1 = splitk_slice_begin(static_cast<int>(e - t * split), split, nkb);
  c.u = e;
  return true;
}

// Workers whose runs start strictly inside `tile` after `worker`'s: the
// contributors of an owner segment, [first, first + count).
__host__ __device__ inline int splitk_contributors(int worker, int workers, int ntiles, int split,
                                                   int tile, int* first) {
  const long long units = static_cast<long long>(ntiles) * split;
  const long long tile_end = static_cast<long long>(tile + 1) * split;
  int n = 0;
  for (int w = worker + 1; w < workers; ++w) {
    if (splitk_run_start(w, workers, units) >= tile_end) break;
    ++n;
  }
  *first = worker + 1;
  return n;
}

struct SplitKView {
  uint32_t* header;  // [0] sequence, [1] finished CTAs
  uint32_t* flags;
  float* partials;
};

__device__ __forceinline__ SplitKView splitk_view(void* ws, int slots, int bn) {
  SplitKView v;
  uint8_t* b = static_cast<uint8_t*>(ws);
  v.header = reinterpret_cast<uint32_t*>(b);
  v.flags = reinterpret_cast<uint32_t*>(b + kSplitKHeaderBytes);
  v.partials = reinterpret_cast<float*>(b + kSplitKHeaderBytes + splitk_flags_bytes(slots));
  (void)bn;
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until flag(slot) == expected for the `count` contributor slots
// first_slot, first_slot + 1, ...; flag(slot) = flags[slot * 4 + quad].
// Returns false (after recording kStatusWaitTimeout with `where`) if a flag
// does not arrive within the bound.
__device__ __forceinline__ bool splitk_wait_flags(const uint32_t* flags, int first_slot,
                                                  int slot_step, int count, int quad,
                                                  uint32_t expected, int where) {
  const uint64_t start = globaltimer_ns();
  for (int j = 0; j < count; ++j) {
    const uint32_t* f = flags + static_cast<size_t>(first_slot + j * slot_step) * 4 + quad;
    for (uint32_t it = 0;; ++it) {
      if (ld_acquire_gpu(f) == expected) break;
      if ((it & 63u) == 63u && globaltimer_ns() - start > kSplitKWaitNs) {
        report_status(kStatusWaitTimeout, where);
        return false;
      }
    }
  }
  return true;
}

// The epilogue warp `quad` of a non-owner segment publishes its 32 partial
// rows: every lane's stores are fenced, then lane 0 releases the flag.
__device__ __forceinline__ void splitk_publish(uint32_t* flags, int slot, int quad,
                                               uint32_t expected, int lane) {
  __threadfence();
  __syncwarp();
  if (lane == 0) st_release_gpu(flags + static_cast<size_t>(slot) * 4 + quad, expected);
}

// The epilogue warp `quad` of an owner segment waits for its contributors'
// rows (lane 0 polls, the warp agrees on the outcome) and fences before the
// partial loads.  Returns the number of partials to add (0 after a timeout).
__device__ __forceinline__ int splitk_acquire(const uint32_t* flags, int first_slot, int slot_step,
                                              int count, int quad, uint32_t expected, int lane,
                                              int where) {
  if (count == 0) return 0;
  int ok = 1;
  if (lane == 0) ok = splitk_wait_flags(flags, first_slot, slot_step, count, quad, expected, where);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __threadfence();
  return ok ? count : 0;
}

// One epilogue warp stores its 32 accumulator rows (TMEM lanes of the warp,
// columns [0, cols) of the accumulator at `taddr`) as fp32 partial sums:
// slot row `row0 + lane`, slot column `col0 + c`.
template <int COLS>
__device__ __forceinline__ void epilogue_store_partial(uint32_t taddr, float* slot, int row0,
                                                       int col0, int lane) {
  float4* base = reinterpret_cast<float4*>(slot);
  const int row = row0 + lane;
#pragma unroll 1
  for (int c = 0; c < COLS; c += 64) {
    uint32_t v0[32], v1[32];
    tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c), v0);
    tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c + 32), v1);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t* v = j < 8 ? v0 : v1;
      const int b = (j & 7) * 4;
      const float4 f = make_float4(__uint_as_float(v[b]), __uint_as_float(v[b + 1]),
                                   __uint_as_float(v[b + 2]), __uint_as_float(v[b + 3]));
      __stcg(base + static_cast<size_t>((col0 + c) / 4 + j) * 128 + row, f);
    }
  }
}

// Adds the partial sums of `count` slots (slot pointers first, first + step,
// ...) to 64 accumulator columns held as fp32 bits in v0 (columns c..c+31)
// and v1 (c+32..c+63), for slot row `row`, slot columns starting at `col`.
__device__ __forceinline__ void splitk_add_partials(uint32_t (&v0)[32], uint32_t (&v1)[32],
                                                    const float* first, int64_t step_floats,
                                                    int count, int row, int col) {
  for (int p = 0; p < count; ++p) {
    const float4* base = reinterpret_cast<const float4*>(first + step_floats * p);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float4 f = __ldcg(base + static_cast<size_t>(col / 4 + j) * 128 + row);
      uint32_t* v = j < 8 ? v0 : v1;
      const int b = (j & 7) * 4;
      v[b] = __float_as_uint(__uint_as_float(v[b]) + f.x);
      v[b + 1] = __float_as_uint(__uint_as_float(v[b + 1]) + f.y);
      v[b + 2] = __float_as_uint(__uint_as_float(v[b + 2]) + f.z);
      v[b + 3] = __float_as_uint(__uint_as_float(v[b + 3]) + f.w);
    }
  }
}

// End-of-launch bookkeeping, one thread per CTA after the CTA's last
// workspace access: the last CTA of the grid to get here resets the finished
// count and advances the sequence number for the next launch.
__device__ __forceinline__ void splitk_finish(uint32_t* header, uint32_t expected) {
  __threadfence();
  const uint32_t done = atomicAdd(&header[1], 1u);
  if (done == gridDim.x - 1) {
    header[1] = 0;
    __threadfence();
    atomicExch(&header[0], expected);  // expected = sequence + 1
  }
}

// Tile origin of output tile t in the GROUP_M raster of kernels/gemm.py:20-26
// (the order both dense kernels walk), tiles of tile_rows x bn.
__device__ __forceinline__ void raster_origin(int t, int M, int tile_rows, int nn, int group_m,
                                              int bn, int* row0, int* col0) {
  const int nm = (M + tile_rows - 1) / tile_rows;
  const int per_group = group_m * nn;
  const int group = t / per_group;
  const int first_m = group * group_m;
  const int gm = min(nm - first_m, group_m);
  const int local = t - group * per_group;
  *row0 = (first_m + local % gm) * tile_rows;
  *col0 = (local / gm) * bn;
}

// Worker whose run contains unit u: the largest w with
// floor(units w / workers) <= u, i.e. units w < (u + 1) workers.
__host__ __device__ inline int splitk_worker_of(long long u, int workers, long long units) {
  const long long w = ((u + 1) * workers - 1) / units;
  return w < workers ? static_cast<int>(w) : workers - 1;
}

// Separate reduction: the workers [*wa, *wb) whose runs hold units of tile t,
// and which of wa's two partial slots holds the tile (*first_which: 1 when the
// tile is the last segment of a run that started in an earlier tile, else 0;
// every later worker's run starts inside the tile, so the tile is its first
// segment, slot 0).  *wb - *wa < 2: one worker covered the tile, no partials.
__host__ __device__ inline void splitk_tile_workers(int t, int split, int workers, int ntiles,
                                                    int* wa, int* wb, int* first_which) {
  const long long units = static_cast<long long>(ntiles) * split;
  const long long u0 = static_cast<long long>(t) * split;
  *wa = splitk_worker_of(u0, workers, units);
  *wb = splitk_worker_of(u0 + split - 1, workers, units) + 1;
  *first_which = splitk_run_start(*wa, workers, units) < u0 ? 1 : 0;
}

// The separate split-K reduction.  CTA (tile t, CTA row half h, chunk c):
// rows 128 h .. 128 h + 127 of the tile (h = 0 for single-CTA tiles) and the
// G = 8 / LANES 4-column groups of chunk c.  Thread (lane p, row r) sums, in
// worker order, the partials of workers wa + p, wa + p + LANES, ... of the
// tile for each of the chunk's groups (independent accumulators: many loads
// in flight); lane 0 adds the lanes' sums in lane order, rounds once and
// stores the row's 4 G outputs.  LANES splits the workers of tiles that many
// workers share (tall K: few tiles, so also narrow chunks for more CTAs); with
// few workers per tile one lane keeps 8 groups.  The order depends only on the shape and the launch, so repeated
// runs are bit-identical.  Tiles a single worker covered are skipped (the GEMM
// wrote them).  One thread derives the tile's workers and origin (schedule
// arithmetic, no memory reads) before the wait on the GEMM.
template <typename T, int LANES>
__global__ void __launch_bounds__(128 * LANES) splitk_reduce_kernel(
    const float* __restrict__ partials, T* __restrict__ C, int M, int N, int split, int workers,
    int ntiles, int pair, int bn, int group_m) {
  constexpr int G = 8 / LANES;  // 4-column groups per CTA
  __shared__ float4 lane_sum[LANES > 1 ? LANES - 1 : 1][LANES > 1 ? G : 1][128];
  __shared__ int info[5];  // wa, wb, first_which, row0, col0
  pdl_allow_next();
  const int halves = pair ? 2 : 1;
  const int chunks = bn / (4 * G);
  int id = blockIdx.x;
  const int c = id % chunks;
  id /= chunks;
  const int h = id % halves;
  const int t = id / halves;
  if (threadIdx.x == 0) {
    splitk_tile_workers(t, split, workers, ntiles, &info[0], &info[1], &info[2]);
    raster_origin(t, M, pair ? 256 : 128, (N + bn - 1) / bn, group_m, bn, &info[3], &info[4]);
  }
  __syncthreads();
  const int wa = info[0], wb = info[1], first_which = info[2];
  // Every CTA waits, also one that has nothing to do: the next kernel's wait
  // covers this grid only, so this grid must not finish before the GEMM.
  pdl_wait();
  if (wb - wa < 2) return;  // whole tile on one worker
  const int r = threadIdx.x & 127;
  const int p = threadIdx.x >> 7;
  const int64_t slot_vecs = static_cast<int64_t>(32) * bn;  // float4s per partial tile
  const float4* base =
      reinterpret_cast<const float4*>(partials) + static_cast<size_t>(c) * G * 128 + r;
  float4 acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int w = wa + p; w < wb; w += LANES) {
    const int cta = pair ? 2 * w + h : w;
    const float4* src = base + slot_vecs * (2 * cta + (w == wa ? first_which : 0));
    float4 f[G];
#pragma unroll
    for (int g = 0; g < G; ++g) f[g] = __ldcg(src + g * 128);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      acc[g].x += f[g].x;
      acc[g].y += f[g].y;
      acc[g].z += f[g].z;
      acc[g].w += f[g].w;
    }
  }
  if constexpr (LANES > 1) {
    if (p > 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) lane_sum[p - 1][g][r] = acc[g];
    }
    __syncthreads();
    if (p > 0) return;
    for (int j = 1; j < LANES; ++j) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 f = lane_sum[j - 1][g][r];
        acc[g].x += f.x;
        acc[g].y += f.y;
        acc[g].z += f.z;
        acc[g].w += f.w;
      }
    }
  }
  const int row = info[3] + 128 * h + r;
  const int col = info[4] + 4 * G * c;
  if (row >= M) return;
  T* out = C + static_cast<size_t>(row) * N + col;
  if constexpr (G == 1) {
    if (col < N) {  // N is a multiple of 8 on this path, col of 4
      uint2 o;
      o.x = Pack2<T>::pack(acc[0].x, acc[0].y);
      o.y = Pack2<T>::pack(acc[0].z, acc[0].w);
      *reinterpret_cast<uint2*>(out) = o;
    }
  } else {
    // 8 columns (16 bytes) at a time; N is a multiple of 8 on this path.
#pragma unroll
    for (int g = 0; g < G; g += 2) {
      if (col + 4 * g < N) {
        uint4 o;
        o.x = Pack2<T>::pack(acc[g].x, acc[g].y);
        o.y = Pack2<T>::pack(acc[g].z, acc[g].w);
        o.z = Pack2<T>::pack(acc[g + 1].x, acc[g + 1].y);
        o.w = Pack2<T>::pack(acc[g + 1].z, acc[g + 1].w);
        *reinterpret_cast<uint4*>(out + 4 * g) = o;
      }
    }
  }
}

}  // namespace bokt
