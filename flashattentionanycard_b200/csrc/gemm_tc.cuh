// tcgen05 GEMM for sm_100a: C = A * B with A [rows, K] K-major and B [K, N]
// N-major (both row-major in HBM), fp16/bf16 operands, fp32 accumulation in
// TMEM, rounded to the operand type on store.
//
// One kernel body serves both operators of the reference:
//   dense   : kernels/gemm.py:7-40            (GROUP_M raster, masked edges)
//   grouped : kernels/moe_grouped_gemm.py:11-58 (ragged experts, one persistent
//             launch, empty experts cost nothing, every output tile has one writer)
//
// CTA = 6 warps, persistent over a static tile schedule (tile += gridDim.x):
//   warp 0    : TMA producer (one lane) filling a `stages`-deep smem ring
//   warp 1    : TMEM allocator + MMA issuer (one lane), 128 x BN x 16 per MMA
//   warps 2-5 : epilogue; warp w drains TMEM lanes 32*(w%4)..+31 (= tile rows)
// Two TMEM accumulators (2 x BN fp32 columns) let the epilogue of tile i
// overlap the main loop of tile i+1.  Operand tiles use the 128-byte swizzle:
// A tile = 128 rows x 64 K (16 KB), B tile = 64 K rows x BN (BN/64 boxes of
// 64 x 64).  No cluster launch; every CTA loads its own tiles.
#pragma once

#include "bokt_device.cuh"
#include "splitk.cuh"

namespace bokt {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kGemmABytes = kGemmBM * kGemmBK * 2;  // 16 KB per stage
constexpr int kGemmMaxExperts = 4096;

struct GemmTcArgs {
  void* C;
  int M;        // dense: rows of A/C.  grouped: T (rows of X/Y)
  int N;
  int K;
  int group_m;  // dense raster width (tiles of M per group)
  int stages;
  uint32_t idesc;
  uint32_t idesc_half;  // grouped CTA pairs: M = 128 (64 rows per CTA) for short tails
  const void* offsets;  // grouped only: E+1 offsets
  int offsets_i64;
  int E;
  // Scatter epilogue (expert-parallel combine): packed row l goes to row
  // rowmap[l] - o * rows_per_owner of out_ptrs[o], o = rowmap[l] / rows_per_owner;
  // out_ptrs[o] may be a peer GPU's buffer (NVLink stores).
  const int32_t* rowmap;
  void* const* out_ptrs;
  int rows_per_owner;
  int owners;
  // Dense only, or null: C row m is scaled by row_scale[m] in the fp32
  // epilogue before rounding (the RMSNorm row factor of the fused
  // RMSNorm -> GEMM, whose norm weight is folded into B).
  const float* row_scale;
  // Grouped tile order: kRasterExpert walks experts in index order (M fastest
  // inside an expert); kRasterBalanced spreads the tiles of low-reuse experts
  // (at most kLowReuseMBlocks row blocks) evenly between the others.
  int raster;
  // Split-K (splitk.cuh): split_k k-slices per tile, dealt out in contiguous
  // runs; the fp32 partials of non-owner segments go through splitk_ws, a
  // workspace of splitk_slots CTA slots.  split_k == 1: whole tiles.
  int split_k;
  void* splitk_ws;
  int splitk_slots;
  // Nonzero (dense only): every segment that does not cover its whole tile
  // stores its partial (slot 2 c for a run's first segment, 2 c + 1 for its
  // last; c = CTA slot) and splitk_reduce_kernel writes those tiles.
  int splitk_reduce;
};

constexpr int kRasterExpert = 1;
constexpr int kRasterBalanced = 2;
constexpr int kLowReuseMBlocks = 2;
// Rows of an expert walked together across its weight column blocks (the
// grouped tile order); 4096 rows of X are 32 MB at K = 4096.
constexpr int kExpertRowGroup = 4096;

template <int BN>
struct GemmTcShape {
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kGemmABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
};

// Epilogue staging: per epilogue warp, 32 rows x 64 columns of 16-bit output
// (4 KB) plus the 32 destination row pointers.
constexpr int kEpiWarps = 4;
constexpr int kEpiStageBytes = 32 * 128;
constexpr int kEpiBytes = kEpiWarps * (kEpiStageBytes + 32 * 8);

// Dynamic shared memory the kernel needs (host and device agree on this).
__host__ __device__ inline int gemm_tc_smem_bytes(int bn, int stages, bool grouped, int experts) {
  int bytes = 1024 /* alignment slack */ + stages * (kGemmABytes + bn * kGemmBK * 2) +
              kEpiBytes + (2 * stages + 4) * 8 + 16;
  if (grouped) bytes += (4 * experts + 4) * 4;
  return bytes;
}

// One epilogue warp writes its 32 accumulator rows (TMEM lanes of this warp,
// columns [0, BN) of the accumulator at `taddr`) to rows rowptr[0..31] (null:
// row outside the problem), columns [n0, min(n0 + BN, N)).  Each 64-column
// chunk goes TMEM -> registers -> round -> XOR-swizzled staging buffer, then
// is written back with every group of 8 lanes storing one full 128-byte row
// segment: coalesced HBM writes, and full-line NVLink writes when a row
// pointer is a peer GPU's memory.
//
// Split-K owners: `pcount` fp32 partial tiles (the first at `pfirst`, the next
// `pstep` floats apart; splitk.cuh layout, slot row `prow`) are added to the
// accumulator before scaling and rounding, in slot order.
template <int BN, typename OutT, bool SCALED = false>
__device__ __forceinline__ void epilogue_store_tile(uint32_t taddr, uint8_t* stage,
                                                    OutT* const* rowptr, int n0, int N,
                                                    int lane, float scale = 1.f,
                                                    const float* pfirst = nullptr,
                                                    int64_t pstep = 0, int pcount = 0,
                                                    int prow = 0) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 64) {
    uint32_t v0[32], v1[32];
    tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c), v0);
    tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c + 32), v1);
    tmem_ld_wait();
    if (pcount > 0) splitk_add_partials(v0, v1, pfirst, pstep, pcount, prow, c);
    uint8_t* my_row = stage + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t* v = j < 4 ? v0 : v1;
      const int b = (j & 3) * 8;
      if constexpr (SCALED) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[b + e] = __float_as_uint(__uint_as_float(v[b + e]) * scale);
      }
      uint4 pk;
      pk.x = Pack2<OutT>::pack(__uint_as_float(v[b + 0]), __uint_as_float(v[b + 1]));
      pk.y = Pack2<OutT>::pack(__uint_as_float(v[b + 2]), __uint_as_float(v[b + 3]));
      pk.z = Pack2<OutT>::pack(__uint_as_float(v[b + 4]), __uint_as_float(v[b + 5]));
      pk.w = Pack2<OutT>::pack(__uint_as_float(v[b + 6]), __uint_as_float(v[b + 7]));
      *reinterpret_cast<uint4*>(my_row + ((j ^ (lane & 7)) << 4)) = pk;
    }
    __syncwarp();
    const int cc = lane & 7;
    const int col = n0 + c + cc * 8;
    // All eight staged segments and row pointers are read before the first
    // global store: a shared-memory load after a store through a generic
    // pointer would otherwise wait for that store, one round trip per row.
    uint4 d[8];
    OutT* rp[8];
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = it * 4 + (lane >> 3);
      d[it] = *reinterpret_cast<const uint4*>(stage + r * 128 + ((cc ^ (r & 7)) << 4));
      rp[it] = rowptr[r];
    }
#pragma unroll
    for (int it = 0; it < 8; ++it)
      if (rp[it] != nullptr && col < N) *reinterpret_cast<uint4*>(rp[it] + c + cc * 8) = d[it];
    __syncwarp();
  }
}

struct TileCoord {
  int a_row;       // first row of the A / X box
  int n0;          // first column of the tile
  int expert;      // grouped only
  int c_row;       // first row of C / Y written by this tile
  int rows_valid;  // rows of this tile inside the problem (<= 128)
};

// K-loop direction of a tile.  Consecutive waves of the persistent raster
// share operand rows (dense: the same A rows in the GROUP_M order; grouped:
// an expert's X rows, re-read for each of its weight column blocks), so a
// tile that starts on the k-blocks another tile has just finished finds them
// still in L2.  Dense: a worker's odd tiles (odd waves) run their k-blocks
// last to first.  Grouped: tiles of odd weight column blocks run last to
// first, a property of the tile itself, so a row's result does not depend on
// the grid (expert-parallel paths with different grids stay bit-identical).
// The MMA issuer consumes stages in ring order either way; only the fp32
// summation order of the tile changes.  Split-K segments keep one order.
template <bool GROUPED>
__device__ __forceinline__ bool k_reversed_for(int i, int split, int n0, int bn) {
  if (split > 1) return false;
  return GROUPED ? ((n0 / bn) & 1) != 0 : (i & 1) != 0;
}

__device__ __forceinline__ TileCoord dense_tile(int t, int M, int nn, int group_m, int bn) {
  // GROUP_M rasterisation, same mapping as kernels/gemm.py:20-26.
  const int nm = (M + kGemmBM - 1) / kGemmBM;
  const int per_group = group_m * nn;
  const int group = t / per_group;
  const int first_m = group * group_m;
  const int gm = min(nm - first_m, group_m);
  const int local = t - group * per_group;
  const int pm = first_m + local % gm;
  const int pn = local / gm;
  TileCoord c;
  c.a_row = pm * kGemmBM;
  c.n0 = pn * bn;
  c.expert = 0;
  c.c_row = c.a_row;
  c.rows_valid = min(kGemmBM, M - c.a_row);
  return c;
}

// Grouped schedule in shared memory, built once per CTA from the device offsets.
// Experts are listed in schedule order (pos): the high-reuse experts first, in
// index order, then the low-reuse ones; pre[pos] is the first tile of that
// entry in the concatenated tile sequence.  With kRasterExpert every expert is
// high-reuse, so the sequence is the plain index order.
struct GroupedSchedule {
  int* pre;      // [E+1] tile prefix over schedule positions
  int* pstart;   // [E]   first packed row of the entry's expert
  int* pcount;   // [E]   rows of the entry's expert
  int* pexp;     // [E]   expert index of the entry
  int* totals;   // [3]   all tiles, low-reuse tiles, high-reuse entries
};

// Rows [start, start + count) of expert e (offsets clamped to [0, T]).
__device__ __forceinline__ void expert_rows(const GemmTcArgs& args, int e, int* start, int* count) {
  long long s, t;
  if (args.offsets_i64) {
    s = reinterpret_cast<const long long*>(args.offsets)[e];
    t = reinterpret_cast<const long long*>(args.offsets)[e + 1];
  } else {
    s = reinterpret_cast<const int*>(args.offsets)[e];
    t = reinterpret_cast<const int*>(args.offsets)[e + 1];
  }
  const long long T = args.M;
  s = s < 0 ? 0 : (s > T ? T : s);
  t = t < s ? s : (t > T ? T : t);
  *start = static_cast<int>(s);
  *count = static_cast<int>(t - s);
}

// Exclusive warp scan (lanes in order) of v; *total = sum over the warp.
__device__ __forceinline__ int warp_exclusive_scan(int v, int lane, int* total) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  *total = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

// Build the grouped schedule; every thread of the CTA calls this.  Expert
// order (the default): every thread loads its experts' offsets once (one
// round of global loads in parallel), then warp 0 turns the per-expert tile
// counts into the prefix with a chunked warp scan.  Balanced order: warp 0
// alone sorts the experts into the two reuse classes while it scans.  Ends
// without a barrier: the caller's barrier publishes the schedule.
__device__ __forceinline__ void build_grouped_schedule(const GemmTcArgs& args, int nn,
                                                       const GroupedSchedule& g,
                                                       int tile_rows = kGemmBM) {
  const int lane = threadIdx.x & 31;
  const bool warp0 = threadIdx.x < 32;
  const int E = args.E;
  const int per = (E + 31) / 32;
  const int e0 = min(E, lane * per);
  const int e1 = min(E, e0 + per);
  if (args.raster != kRasterBalanced) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int st, c;
      expert_rows(args, e, &st, &c);
      g.pstart[e] = st;
      g.pcount[e] = c;
      g.pexp[e] = e;
      g.pre[e] = ((c + tile_rows - 1) / tile_rows) * nn;  // tiles, turned into the prefix below
    }
    __syncthreads();
    if (warp0) {
      int sum = 0;
      for (int e = e0; e < e1; ++e) sum += g.pre[e];
      int total;
      int run = warp_exclusive_scan(sum, lane, &total);
      for (int e = e0; e < e1; ++e) {
        const int tiles = g.pre[e];
        g.pre[e] = run;
        run += tiles;
      }
      if (lane == 0) {
        g.pre[E] = total;
        g.totals[0] = total;
        g.totals[1] = 0;
        g.totals[2] = E;
      }
    }
    return;
  }
  if (!warp0) return;
  int he = 0, le = 0, ht = 0, lt = 0;
  for (int e = e0; e < e1; ++e) {
    int st, c;
    expert_rows(args, e, &st, &c);
    const int mb = (c + tile_rows - 1) / tile_rows;
    if (mb <= kLowReuseMBlocks) {
      ++le;
      lt += mb * nn;
    } else {
      ++he;
      ht += mb * nn;
    }
  }
  int n_he, n_le, n_ht, n_lt;
  int hpos = warp_exclusive_scan(he, lane, &n_he);
  int lpos = warp_exclusive_scan(le, lane, &n_le) + n_he;
  int htile = warp_exclusive_scan(ht, lane, &n_ht);
  int ltile = warp_exclusive_scan(lt, lane, &n_lt) + n_ht;
  if (lane == 0) {
    g.totals[0] = n_ht + n_lt;
    g.totals[1] = n_lt;
    g.totals[2] = n_he;
    g.pre[E] = n_ht + n_lt;
  }
  for (int e = e0; e < e1; ++e) {
    int st, c;
    expert_rows(args, e, &st, &c);
    const int mb = (c + tile_rows - 1) / tile_rows;
    int pos;
    if (mb <= kLowReuseMBlocks) {
      pos = lpos++;
      g.pre[pos] = ltile;
      ltile += mb * nn;
    } else {
      pos = hpos++;
      g.pre[pos] = htile;
      htile += mb * nn;
    }
    g.pstart[pos] = st;
    g.pcount[pos] = c;
    g.pexp[pos] = e;
  }
}

__device__ __forceinline__ TileCoord grouped_tile(int t, const GroupedSchedule& g, int E, int nn,
                                                  int bn, int raster, int tile_rows = kGemmBM) {
  const int total = g.totals[0];
  const int nlow = g.totals[1];
  int u = t;
  if (raster == kRasterBalanced && nlow > 0) {
    // Position t of the sequence is a low-reuse tile iff floor((t+1) nlow / total)
    // steps up there: the nlow low-reuse tiles are spread evenly, both
    // subsequences keep their order.
    const int f0 = static_cast<int>(static_cast<long long>(t) * nlow / total);
    const int f1 = static_cast<int>(static_cast<long long>(t + 1) * nlow / total);
    u = f1 > f0 ? (total - nlow) + f0 : t - f0;
  }
  // Largest pos with pre[pos] <= u (pre is non-decreasing, u < pre[E]); empty
  // experts share their successor's prefix and are skipped by taking the last.
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.pre[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  const int rel = u - g.pre[lo];
  const int count = g.pcount[lo];
  const int mblocks = (count + tile_rows - 1) / tile_rows;
  // M fastest inside a group of row blocks: all row blocks of the group run
  // together on one weight column block, so W[e][:, n-block] is fetched from
  // HBM once per group and reused from L2.  Groups span kExpertRowGroup rows,
  // so that the group's X rows stay in L2 while it walks the expert's column
  // blocks; an expert with more rows (a hot expert) is split into groups.
  const int gsize = kExpertRowGroup / tile_rows;  // row blocks per group
  const int per_group = gsize * nn;
  const int grp = rel / per_group;
  const int gfirst = grp * gsize;
  const int gm = min(mblocks - gfirst, gsize);
  const int local = rel - grp * per_group;
  const int mb = gfirst + local % gm;
  const int nb = local / gm;
  TileCoord c;
  c.a_row = g.pstart[lo] + mb * tile_rows;
  c.n0 = nb * bn;
  c.expert = g.pexp[lo];
  c.c_row = c.a_row;
  c.rows_valid = min(tile_rows, count - mb * tile_rows);
  return c;
}

template <int BN, bool GROUPED, typename OutT, bool SCATTER = false, bool ROWSCALE = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   GemmTcArgs args) {
  using Shape = GemmTcShape<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int stages = args.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * kGemmABytes;
  uint8_t* sEpi = sB + stages * Shape::kBBytes;  // kEpiWarps x (staging + row pointers)
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + kEpiBytes);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  GroupedSchedule sched;  // grouped only: [E+1] + 3 x [E] + [3] ints
  sched.pre = reinterpret_cast<int*>(tmem_holder + 4);
  sched.pstart = sched.pre + (args.E + 1);
  sched.pcount = sched.pstart + args.E;
  sched.pexp = sched.pcount + args.E;
  sched.totals = sched.pexp + args.E;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int N = args.N;
  const int nn = (N + BN - 1) / BN;
  const int nkb = (args.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4 * 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Shape::kTmemCols);
    tmem_relinquish();
  }
  // Prologue above overlaps the previous kernel; global memory only after this.
  pdl_allow_next();
  pdl_wait();

  int ntiles;
  if constexpr (GROUPED) {
    build_grouped_schedule(args, nn, sched);
  }
  const int split = args.split_k > 1 ? args.split_k : 1;
  SplitKView sk = {};
  const bool fixup = split > 1 && !args.splitk_reduce;  // owner fix-up with flags
  if (split > 1) {
    sk = splitk_view(args.splitk_ws, args.splitk_slots, BN);
    // Sequence number of this launch (+1): the value the partial flags carry.
    if (fixup && threadIdx.x == 0) tmem_holder[2] = ld_acquire_gpu(sk.header) + 1u;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t expected = tmem_holder[2];
  if constexpr (GROUPED) {
    ntiles = sched.totals[0];
  } else {
    ntiles = ((args.M + kGemmBM - 1) / kGemmBM) * nn;
  }
  const int workers = splitk_workers(gridDim.x, ntiles, split);
  const int worker = blockIdx.x;

  auto tile_at = [&](int t) -> TileCoord {
    if constexpr (GROUPED) {
      return grouped_tile(t, sched, args.E, nn, BN, args.raster);
    } else {
      return dense_tile(t, args.M, nn, args.group_m, BN);
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      SegmentCursor cur = segment_cursor(worker, workers, ntiles, split);
      Segment sg;
      for (int i = 0; ok && segment_next(cur, split, nkb, sg); ++i) {
        const TileCoord tc = tile_at(sg.tile);
        const bool rev = k_reversed_for<GROUPED>(i, split, tc.n0, BN);
        for (int kk = sg.kb0; kk < sg.kb1; ++kk) {
          const int kb = rev ? sg.kb1 - 1 - (kk - sg.kb0) : kk;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Shape::kStageBytes);
          uint8_t* a_dst = sA + stage * kGemmABytes;
          uint8_t* b_dst = sB + stage * Shape::kBBytes;
          tma_load_2d(a_dst, &tmA, &full[stage], kb * kGemmBK, tc.a_row);
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            if constexpr (GROUPED) {
              tma_load_3d(b_dst + c * 8192, &tmB, &full[stage], tc.n0 + c * 64, kb * kGemmBK,
                          tc.expert);
            } else {
              tma_load_2d(b_dst + c * 8192, &tmB, &full[stage], tc.n0 + c * 64, kb * kGemmBK);
            }
          }
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      bool ok = true;
      SegmentCursor cur = segment_cursor(worker, workers, ntiles, split);
      Segment sg;
      for (; ok && segment_next(cur, split, nkb, sg); ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (static_cast<uint32_t>(i) >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(sA + stage * kGemmABytes);
          const uint32_t b_addr = smem_addr(sB + stage * Shape::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            // A: K-major, 128-byte rows; a K16 step is 32 bytes along the row.
            const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            // B: N-major; a K16 step is two 8-row groups (2 x 1024 bytes);
            // 64-column boxes sit 64 rows x 128 bytes apart.
            const uint64_t b_desc = smem_desc_sw128(b_addr + k * 2048, 64 * 128, 1024);
            umma_f16_ss(d_tmem, a_desc, b_desc, args.idesc,
                        (kb != sg.kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    OutT* C = reinterpret_cast<OutT*>(args.C);
    uint8_t* stage = sEpi + (warp - 2) * kEpiStageBytes;
    OutT** rowptr = reinterpret_cast<OutT**>(sEpi + kEpiWarps * kEpiStageBytes) + (warp - 2) * 32;
    const int64_t slot_floats = static_cast<int64_t>(kGemmBM) * BN;
    int i = 0;
    SegmentCursor cur = segment_cursor(worker, workers, ntiles, split);
    Segment sg;
    for (; segment_next(cur, split, nkb, sg); ++i) {
      const TileCoord tc = tile_at(sg.tile);
      const int acc = i & 1;
      const uint32_t acc_phase = (static_cast<uint32_t>(i) >> 1) & 1u;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, 4);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (args.splitk_reduce && (sg.kb0 > 0 || sg.kb1 < nkb)) {
        // Separate reduction: only the partial; no flags, no waits.
        epilogue_store_partial<BN>(taddr, sk.partials + slot_floats * (2 * worker + (i > 0)),
                                   q * 32, 0, lane);
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        continue;
      }
      if (sg.kb0 > 0) {
        // Split-K non-owner: this worker's first segment; publish the fp32
        // partial rows of this warp into the CTA's slot.
        epilogue_store_partial<BN>(taddr, sk.partials + slot_floats * worker, q * 32, 0, lane);
        splitk_publish(sk.flags, worker, q, expected, lane);
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        continue;
      }
      int first = 0, count = 0;
      if (sg.kb1 < nkb) {
        count = splitk_contributors(worker, workers, ntiles, split, sg.tile, &first);
        count = splitk_acquire(sk.flags, first, 1, count, q, expected, lane, 21);
      }
      bool row_ok = r < tc.rows_valid;
      OutT* crow = C + static_cast<size_t>(tc.c_row + (row_ok ? r : 0)) * N + tc.n0;
      if constexpr (SCATTER) {
        if (row_ok) {
          const int a = args.rowmap[tc.c_row + r];
          const int o = a / args.rows_per_owner;
          if (a < 0 || o >= args.owners) {
            report_status(kStatusBadExpertId, tc.c_row + r);
            row_ok = false;
          } else {
            crow = reinterpret_cast<OutT*>(args.out_ptrs[o]) +
                   static_cast<size_t>(a - o * args.rows_per_owner) * N + tc.n0;
          }
        }
      }
      rowptr[lane] = row_ok ? crow : nullptr;
      float scale = 1.f;
      if constexpr (ROWSCALE) scale = row_ok ? args.row_scale[tc.c_row + r] : 1.f;
      __syncwarp();
      epilogue_store_tile<BN, OutT, ROWSCALE>(taddr, stage, rowptr, tc.n0, N, lane, scale,
                                              sk.partials + slot_floats * first, slot_floats,
                                              count, r);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    if constexpr (SCATTER) __threadfence_system();  // peer stores visible before the barrier
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (fixup && threadIdx.x == 0) splitk_finish(sk.header, expected);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Shape::kTmemCols);
  }
}

}  // namespace bokt
