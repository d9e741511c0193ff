// MoE routing front end: expert histogram -> offsets (exclusive prefix sum) ->
// stable permutation of assignments by expert -> inverse permutation (combine
// indices), plus the row gather that packs token activations in expert order.
//
// The reference builds offsets on the host (tuner/worker.py:81-86) and leaves
// routing outside the operator (kernels/moe_grouped_gemm.py:3).  Here the
// whole front end is device resident so the grouped GEMM reads offsets that a
// kernel produced (no host round trip, graph-capturable).  Integer work,
// bit-exact against a stable counting sort:
//   counts[e]   = #{i : id[i] == e}
//   offsets[e]  = sum_{e' < e} counts[e']
//   perm[j]     = i  such that i is the (j - offsets[e])-th assignment of expert e
//   inv_perm[i] = j
//
// Three launches over chunks of kRouteChunk assignments:
//   1. route_count   : per-chunk expert histogram (shared-memory atomics; order
//                      independent, so deterministic)
//   2. route_scan    : one CTA; column prefix over chunks + exclusive scan over
//                      experts -> counts, offsets, per-(chunk, expert) base rows
//   3. route_scatter : each chunk walks its assignments in order, 256 at a time;
//                      rank inside a warp from __match_any_sync, across warps from
//                      a per-warp count table -> stable destinations
#pragma once

#include "bokt_device.cuh"
#include "ep_sync.cuh"

namespace bokt {

constexpr int kRouteChunk = 4096;
constexpr int kRouteThreads = 256;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kRouteMaxExperts = 1024;

__global__ void __launch_bounds__(kRouteThreads) route_count_kernel(const int32_t* __restrict__ ids,
                                                                     int A, int E,
                                                                     int32_t* __restrict__ chunk_counts) {
  __shared__ int hist[kRouteMaxExperts];
  pdl_allow_next();
  pdl_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int begin = blockIdx.x * kRouteChunk;
  const int end = min(A, begin + kRouteChunk);
  for (int i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
    else report_status(kStatusBadExpertId, i);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    chunk_counts[static_cast<size_t>(blockIdx.x) * E + e] = hist[e];
}

// One CTA of 1024 threads.  chunk_counts[c][e] is replaced by the first packed
// row of chunk c's assignments to expert e.
__global__ void __launch_bounds__(1024) route_scan_kernel(int32_t* __restrict__ chunk_counts,
                                                          int chunks, int E,
                                                          int32_t* __restrict__ counts,
                                                          int32_t* __restrict__ offsets,
                                                          long long* __restrict__ offsets64) {
  __shared__ int totals[kRouteMaxExperts];
  __shared__ int warp_sums[32];
  __shared__ int carry;
  pdl_allow_next();
  pdl_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < chunks; ++c) {
      const int v = chunk_counts[static_cast<size_t>(c) * E + e];
      chunk_counts[static_cast<size_t>(c) * E + e] = run;  // exclusive column prefix
      run += v;
    }
    totals[e] = run;
    counts[e] = run;
  }
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  // Exclusive scan of totals over experts, 1024 at a time.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < E; base += blockDim.x) {
    const int e = base + threadIdx.x;
    const int v = e < E ? totals[e] : 0;
    int incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - v;
    if (e < E) {
      offsets[e] = excl;
      if (offsets64) offsets64[e] = excl;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[E] = carry;
    if (offsets64) offsets64[E] = carry;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int off = offsets[e];
    for (int c = 0; c < chunks; ++c) chunk_counts[static_cast<size_t>(c) * E + e] += off;
  }
}

__global__ void __launch_bounds__(kRouteThreads) route_scatter_kernel(
    const int32_t* __restrict__ ids, int A, int E, const int32_t* __restrict__ chunk_base,
    int32_t* __restrict__ perm, int32_t* __restrict__ inv_perm) {
  __shared__ int running[kRouteMaxExperts];
  __shared__ int wcnt[kRouteWarps][kRouteMaxExperts];
  pdl_allow_next();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    running[e] = chunk_base[static_cast<size_t>(blockIdx.x) * E + e];
    for (int w = 0; w < kRouteWarps; ++w) wcnt[w][e] = 0;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  const int begin = blockIdx.x * kRouteChunk;
  const int end = min(A, begin + kRouteChunk);
  for (int base = begin; base < end; base += kRouteThreads) {
    const int i = base + threadIdx.x;
    int e = (i < end) ? ids[i] : -1;
    if (e < 0 || e >= E) e = -1;  // invalid ids were reported by route_count
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    const bool leader = (peers & lt_mask) == 0;
    if (e >= 0 && leader) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    int dest = 0;
    if (e >= 0) {
      int pre = 0;
      for (int w = 0; w < warp; ++w) pre += wcnt[w][e];
      dest = running[e] + pre + rank;
    }
    __syncthreads();
    if (e >= 0 && leader) {
      atomicAdd(&running[e], __popc(peers));
      wcnt[warp][e] = 0;
    }
    if (e >= 0) {
      perm[dest] = i;
      inv_perm[i] = dest;
    }
    __syncthreads();
  }
}

// dst[j, :] = src[index[j] / divisor, :]; one CTA slice per row, 16-byte
// vectors when the row length and both bases allow it.
template <typename V>
__global__ void gather_rows_kernel(const V* __restrict__ src, long long src_rows, V* __restrict__ dst,
                                   const int32_t* __restrict__ index, int rows, int row_vecs,
                                   int divisor) {
  pdl_allow_next();
  pdl_wait();
  for (int j = blockIdx.x; j < rows; j += gridDim.x) {
    const int raw = index[j];
    const long long s = raw / divisor;
    if (raw < 0 || s >= src_rows) {
      if (threadIdx.x == 0) report_status(kStatusBadExpertId, j);
      continue;
    }
    const V* sr = src + s * row_vecs;
    V* dr = dst + static_cast<long long>(j) * row_vecs;
    for (int c = threadIdx.x; c < row_vecs; c += blockDim.x) dr[c] = sr[c];
  }
}

}  // namespace bokt

namespace bokt {

constexpr int kStatusPlanMismatch = 3;

// dst[j, :] = src[inner[outer ? outer[j] : j] / divisor - base, :]: the
// two-level row gathers of expert-parallel dispatch and combine (compose a
// routing permutation with a per-rank order without materialising the
// composed index).  Rows whose source falls outside src are reported and
// left unwritten.
template <typename V>
__global__ void gather_rows_indirect_kernel(const V* __restrict__ src, long long src_rows,
                                            V* __restrict__ dst,
                                            const int32_t* __restrict__ inner,
                                            const int32_t* __restrict__ outer, long long inner_len,
                                            int rows, int row_vecs, int divisor, long long base) {
  pdl_allow_next();
  pdl_wait();
  for (int j = blockIdx.x; j < rows; j += gridDim.x) {
    const long long o = outer ? static_cast<long long>(outer[j]) : j;
    if (o < 0 || o >= inner_len) {
      if (threadIdx.x == 0) report_status(kStatusBadExpertId, j);
      continue;
    }
    const long long raw = inner[o];
    const long long s = (raw < 0 ? -1 : raw / divisor) - base;
    if (raw < 0 || s < 0 || s >= src_rows) {
      if (threadIdx.x == 0) report_status(kStatusBadExpertId, j);
      continue;
    }
    const V* sr = src + s * row_vecs;
    V* dr = dst + static_cast<long long>(j) * row_vecs;
    for (int c = threadIdx.x; c < row_vecs; c += blockDim.x) dr[c] = sr[c];
  }
}

// Expert-parallel keys of every packed row p of the global routing (one rank's view).
//   a = perm[p] (assignment, token-major), e = ids[a], q = p - offsets[e],
//   replica j = q * R_e / c_e, virtual expert v = vbase[e] + j, dest d = v_rank[v],
//   owner o = (a / topk) / tokens_per_rank.
//   key_send[p]  = o == me ? d : world          (stable sort -> send order by destination)
//   key_recv[p]  = d == me ? o : world          (-> receive order by source)
//   key_local[p] = d == me ? v_local[v] : n_local (-> local grouped-GEMM order and offsets)
__global__ void ep_keys_kernel(const int32_t* __restrict__ perm, const int32_t* __restrict__ ids,
                               const int32_t* __restrict__ offsets,
                               const int32_t* __restrict__ counts,
                               const int32_t* __restrict__ replicas,
                               const int32_t* __restrict__ vbase,
                               const int32_t* __restrict__ v_rank,
                               const int32_t* __restrict__ v_local, int A, int E, int topk,
                               int tokens_per_rank, int me, int world, int n_local,
                               int32_t* __restrict__ key_send, int32_t* __restrict__ key_recv,
                               int32_t* __restrict__ key_local) {
  pdl_allow_next();
  pdl_wait();
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < A; p += gridDim.x * blockDim.x) {
    const int a = perm[p];
    const int e = (a >= 0 && a < A) ? ids[a] : -1;
    if (e < 0 || e >= E) {
      report_status(kStatusBadExpertId, p);
      key_send[p] = world;
      key_recv[p] = world;
      key_local[p] = n_local;
      continue;
    }
    const long long q = p - offsets[e];
    const int c = counts[e];
    const int j = c > 0 ? static_cast<int>((q * replicas[e]) / c) : 0;
    const int v = vbase[e] + j;
    const int d = v_rank[v];
    const int o = (a / topk) / tokens_per_rank;
    key_send[p] = o == me ? d : world;
    key_recv[p] = d == me ? o : world;
    key_local[p] = d == me ? v_local[v] : n_local;
  }
}

// Flags kStatusPlanMismatch when counts[0..n) differs from the planned sizes
// (the NCCL split sizes were fixed when the plan was made).
__global__ void check_counts_kernel(const int32_t* __restrict__ counts,
                                    const int32_t* __restrict__ expected, int n, int tag) {
  pdl_allow_next();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    if (counts[i] != expected[i]) report_status(kStatusPlanMismatch, tag * 65536 + i);
}

}  // namespace bokt

namespace bokt {

constexpr int kStatusCapacity = 4;

// Per-step expert-parallel layout from the global routing.  Virtual expert v =
// (expert e, replica j) serves the contiguous packed rows
// [v_plo[v], v_plo[v] + v_size[v]) of the global routing; on its rank it is
// stored at rows [v_lbase[v], v_lbase[v] + v_size[v]) of the packed buffer,
// virtual experts in ascending v.  loffs = the local grouped-GEMM offsets of
// rank `me` (n_local + 1 entries).  rank_rows[r] = rows rank r serves; a rank
// over its buffer capacity is reported (kStatusCapacity).
//
// One CTA: the inputs are loaded into shared memory by all threads, one
// thread runs the two short serial passes there (E experts, V virtual
// experts: a few hundred shared-memory operations), and all threads write
// the results back.  Dynamic shared memory: ep_plan_smem_bytes(E, V, world).
__host__ __device__ inline int ep_plan_smem_bytes(int E, int V, int world) {
  return (3 * E + 5 * V + world + 2) * 4;
}

__global__ void __launch_bounds__(256, 1) ep_plan_kernel(const int32_t* __restrict__ counts,
                               const int32_t* __restrict__ offsets,
                               const int32_t* __restrict__ replicas, int E,
                               const int32_t* __restrict__ v_rank, int V, int world, int me,
                               const int32_t* __restrict__ capacity,
                               int32_t* __restrict__ v_plo, int32_t* __restrict__ v_size,
                               int32_t* __restrict__ v_lbase, int32_t* __restrict__ loffs,
                               int32_t* __restrict__ rank_rows) {
  extern __shared__ int32_t plan_smem[];
  int32_t* s_cnt = plan_smem;
  int32_t* s_off = s_cnt + E;
  int32_t* s_rep = s_off + E;
  int32_t* s_vrank = s_rep + E;
  int32_t* s_vsize = s_vrank + V;
  int32_t* s_vplo = s_vsize + V;
  int32_t* s_vlbase = s_vplo + V;
  int32_t* s_loffs = s_vlbase + V;  // V + 1 entries
  int32_t* s_rrows = s_loffs + V + 1;
  __shared__ int s_nl;
  pdl_allow_next();
  pdl_wait();
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    s_cnt[i] = counts[i];
    s_off[i] = offsets[i];
    s_rep[i] = replicas[i];
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) s_vrank[i] = v_rank[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    int v = 0;
    for (int e = 0; e < E; ++e) {
      const long long c = s_cnt[e];
      const int R = s_rep[e];
      for (int j = 0; j < R && v < V; ++j, ++v) {
        const long long lo = (static_cast<long long>(j) * c + R - 1) / R;  // ceil(j c / R)
        const long long hi = (static_cast<long long>(j + 1) * c + R - 1) / R;
        s_vplo[v] = s_off[e] + static_cast<int>(lo);
        s_vsize[v] = static_cast<int>(hi - lo);
      }
    }
    for (; v < V; ++v) s_vplo[v] = s_vsize[v] = 0;  // replicas inconsistent with V
    for (int r = 0; r < world; ++r) s_rrows[r] = 0;
    int nl = 0;
    s_loffs[0] = 0;
    for (v = 0; v < V; ++v) {
      const int r = s_vrank[v];
      if (r < 0 || r >= world) {
        report_status(kStatusPlanMismatch, v);
        s_vlbase[v] = 0;
        continue;
      }
      s_vlbase[v] = s_rrows[r];
      s_rrows[r] += s_vsize[v];
      if (r == me) s_loffs[++nl] = s_rrows[r];
    }
    s_nl = nl;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    v_plo[i] = s_vplo[i];
    v_size[i] = s_vsize[i];
    v_lbase[i] = s_vlbase[i];
  }
  for (int i = threadIdx.x; i <= s_nl; i += blockDim.x) loffs[i] = s_loffs[i];
  for (int r = threadIdx.x; r < world; r += blockDim.x) {
    rank_rows[r] = s_rrows[r];
    if (s_rrows[r] > capacity[r]) report_status(kStatusCapacity, r);
  }
}

__device__ __forceinline__ int ep_virtual_expert(int p, int e, const int32_t* offsets,
                                                 const int32_t* counts, const int32_t* replicas,
                                                 const int32_t* vbase) {
  const long long q = p - offsets[e];
  const int c = counts[e];
  const int j = c > 0 ? static_cast<int>((q * replicas[e]) / c) : 0;
  return vbase[e] + j;
}

// Dispatch over NVLink: every local assignment a_loc of this rank copies its
// token's row into the packed buffer of the rank serving it (xpk[d] may be a
// peer GPU's memory), at that rank's local position.  One warp per row,
// 16-byte vectors.  Positions beyond the destination's capacity are reported
// and skipped.
__global__ void ep_dispatch_kernel(const uint4* __restrict__ x_local, int row_vecs,
                                   const int32_t* __restrict__ ids,
                                   const int32_t* __restrict__ inv_perm,
                                   const int32_t* __restrict__ offsets,
                                   const int32_t* __restrict__ counts,
                                   const int32_t* __restrict__ replicas,
                                   const int32_t* __restrict__ vbase,
                                   const int32_t* __restrict__ v_rank,
                                   const int32_t* __restrict__ v_plo,
                                   const int32_t* __restrict__ v_lbase,
                                   uint4* const* __restrict__ xpk,
                                   const int32_t* __restrict__ capacity, int a_local,
                                   int topk, int me, int E) {
  pdl_allow_next();
  pdl_wait();
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < a_local; i += warps) {
    const int a = me * a_local + i;
    const int e = ids[a];
    if (e < 0 || e >= E) {
      if (lane == 0) report_status(kStatusBadExpertId, a);
      continue;
    }
    const int p = inv_perm[a];
    const int v = ep_virtual_expert(p, e, offsets, counts, replicas, vbase);
    const int d = v_rank[v];
    const int pos = v_lbase[v] + (p - v_plo[v]);
    if (pos < 0 || pos >= capacity[d]) {
      if (lane == 0) report_status(kStatusCapacity, a);
      continue;
    }
    const uint4* src = x_local + static_cast<long long>(i / topk) * row_vecs;
    uint4* dst = xpk[d] + static_cast<long long>(pos) * row_vecs;
    for (int c = lane; c < row_vecs; c += 32) dst[c] = src[c];
  }
  __threadfence_system();  // peer stores visible system-wide before the next barrier
}

// For every packed row this rank serves: rowmap[local row] = global assignment
// index (the grouped GEMM's scatter epilogue sends the row to that
// assignment's owner).
__global__ void ep_rowmap_kernel(const int32_t* __restrict__ perm,
                                 const int32_t* __restrict__ ids,
                                 const int32_t* __restrict__ offsets,
                                 const int32_t* __restrict__ counts,
                                 const int32_t* __restrict__ replicas,
                                 const int32_t* __restrict__ vbase,
                                 const int32_t* __restrict__ v_rank,
                                 const int32_t* __restrict__ v_plo,
                                 const int32_t* __restrict__ v_lbase, int A, int E, int me,
                                 int capacity, int32_t* __restrict__ rowmap) {
  pdl_allow_next();
  pdl_wait();
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < A; p += gridDim.x * blockDim.x) {
    const int a = perm[p];
    const int e = (a >= 0 && a < A) ? ids[a] : -1;
    if (e < 0 || e >= E) continue;  // reported by the routing kernels
    const int v = ep_virtual_expert(p, e, offsets, counts, replicas, vbase);
    if (v_rank[v] != me) continue;
    const int l = v_lbase[v] + (p - v_plo[v]);
    if (l >= 0 && l < capacity) rowmap[l] = a;
  }
}

}  // namespace bokt

namespace bokt {

constexpr int kTopkMax = 8;
constexpr int kGateMaxExperts = 1024;

template <typename T>
__device__ __forceinline__ float load_logit(const T* p) {
  return Pack2<T>::to_float(*p);
}
template <>
__device__ __forceinline__ float load_logit<float>(const float* p) {
  return *p;
}

// Top-k softmax gate: one warp per token.  p = softmax(logits[t, :]) in fp32;
// ids[t, j] = index of the j-th largest p (ties: lower expert index first);
// gates[t, j] = p[ids[t, j]], divided by their sum when `renormalize`.
template <typename T>
__global__ void __launch_bounds__(256) moe_topk_gate_kernel(const T* __restrict__ logits, int tokens,
                                                            int E, int k, int renormalize,
                                                            int32_t* __restrict__ ids,
                                                            float* __restrict__ gates) {
  pdl_allow_next();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < tokens; t += warps) {
    const T* row = logits + static_cast<long long>(t) * E;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, load_logit(row + e));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) sum += expf(load_logit(row + e) - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    // k rounds of a warp-wide arg-max over the logits not yet taken.
    int taken[kTopkMax];
    float picked = 0.f;
    float vals[kTopkMax];
    for (int j = 0; j < k; ++j) {
      float best = -INFINITY;
      int best_e = E;
      for (int e = lane; e < E; e += 32) {
        bool used = false;
        for (int i = 0; i < j; ++i) used |= (taken[i] == e);
        const float v = load_logit(row + e);
        if (!used && (v > best || (v == best && e < best_e))) {
          best = v;
          best_e = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
        if (ov > best || (ov == best && oe < best_e)) {
          best = ov;
          best_e = oe;
        }
      }
      taken[j] = best_e;
      vals[j] = expf(best - mx) / sum;
      picked += vals[j];
    }
    if (lane == 0) {
      for (int j = 0; j < k; ++j) {
        ids[static_cast<long long>(t) * k + j] = taken[j];
        gates[static_cast<long long>(t) * k + j] = renormalize ? vals[j] / picked : vals[j];
      }
    }
  }
}

// out[t] = sum_j gates[t k + j] * y[row(t k + j)] for one token, fp32 FMAs in
// slot order j = 0..k-1, 16-byte vectors spread over the CTA's threads;
// row(a) = rows[a] when rows is given, else a.  Rows outside [0, y_rows) set
// *bad and are skipped.
template <typename T>
__device__ __forceinline__ void combine_token(const T* __restrict__ y, long long y_rows,
                                              const int32_t* __restrict__ rows,
                                              const float* __restrict__ gates,
                                              T* __restrict__ out, int t, int k, int N,
                                              bool* bad) {
  const int nvec = N / 8;
  const uint4* yv4 = reinterpret_cast<const uint4*>(y);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int j = 0; j < k; ++j) {
      const int a = t * k + j;
      const long long r = rows ? static_cast<long long>(rows[a]) : static_cast<long long>(a);
      if (r < 0 || r >= y_rows) {
        *bad = true;
        continue;
      }
      const float g = gates[a];
      const uint4 yv = yv4[r * nvec + v];
      const float2 f0 = Pack2<T>::unpack(yv.x), f1 = Pack2<T>::unpack(yv.y);
      const float2 f2 = Pack2<T>::unpack(yv.z), f3 = Pack2<T>::unpack(yv.w);
      acc[0] = fmaf(g, f0.x, acc[0]);
      acc[1] = fmaf(g, f0.y, acc[1]);
      acc[2] = fmaf(g, f1.x, acc[2]);
      acc[3] = fmaf(g, f1.y, acc[3]);
      acc[4] = fmaf(g, f2.x, acc[4]);
      acc[5] = fmaf(g, f2.y, acc[5]);
      acc[6] = fmaf(g, f3.x, acc[6]);
      acc[7] = fmaf(g, f3.y, acc[7]);
    }
    uint4 o;
    o.x = Pack2<T>::pack(acc[0], acc[1]);
    o.y = Pack2<T>::pack(acc[2], acc[3]);
    o.z = Pack2<T>::pack(acc[4], acc[5]);
    o.w = Pack2<T>::pack(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + static_cast<long long>(t) * N)[v] = o;
  }
}

// Gate-weighted combine back to token order:
//   out[t, :] = sum_j gates[t, j] * y[row(t, j), :],  row = rows ? rows[t*k + j] : t*k + j
// fp32 accumulation, rounded on store; one CTA slice per token, 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(256) moe_combine_kernel(const T* __restrict__ y, long long y_rows,
                                                          const int32_t* __restrict__ rows,
                                                          const float* __restrict__ gates,
                                                          T* __restrict__ out, int tokens, int k,
                                                          int N) {
  pdl_allow_next();
  pdl_wait();
  bool bad = false;
  for (int t = blockIdx.x; t < tokens; t += gridDim.x)
    combine_token(y, y_rows, rows, gates, out, t, k, N, &bad);
  if (bad) report_status(kStatusBadExpertId, blockIdx.x);
}

// The expert-parallel step's last barrier with the combine fused into it (the
// receive side of the peer-store combine).  Every CTA signals this rank's
// epoch to every rank (flag_ptrs as in ep_barrier_kernel; the stores are
// idempotent, so no CTA depends on another being scheduled), waits until all
// ranks have signalled it -- i.e. every peer's grouped GEMM has stored its
// result rows into this rank's slot buffer y [tokens * k, N] -- and then
// reduces its share of this rank's tokens: out[t] = sum_j gates[t k + j] *
// y[t k + j] (combine_token, the arithmetic of moe_combine_kernel).  epoch[0]
// is the barrier epoch, epoch[1] counts CTAs that finished; the last CTA
// resets the count and advances the epoch.  On a timeout the CTA records
// kStatusWaitTimeout (detail 4000 + silent rank) and skips its tokens.
template <typename T>
__global__ void __launch_bounds__(256) ep_barrier_combine_kernel(
    int32_t* const* __restrict__ flag_ptrs, int32_t* __restrict__ epoch, int world, int me,
    long long timeout_ns, const T* __restrict__ y, long long y_rows,
    const float* __restrict__ gates, T* __restrict__ out, int tokens, int k, int N) {
  pdl_allow_next();
  pdl_wait();
  __shared__ int32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int32_t e = 0;
    if (lane == 0) e = epoch[0] + 1;
    e = __shfl_sync(0xffffffffu, e, 0);
    __threadfence_system();
    int ok = 1;
    if (lane < world) {
      st_release_sys(flag_ptrs[lane] + me, e);
      const int32_t* mine = flag_ptrs[me] + lane;
      const uint64_t start = globaltimer_ns();
      for (uint32_t it = 0;; ++it) {
        const uint32_t seen = static_cast<uint32_t>(ld_acquire_sys(mine));
        if (static_cast<int32_t>(seen - static_cast<uint32_t>(e)) >= 0) break;
        if ((it & 63u) == 63u &&
            globaltimer_ns() - start > static_cast<uint64_t>(timeout_ns)) {
          report_status(kStatusWaitTimeout, 4000 + lane);
          ok = 0;
          break;
        }
      }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (lane == 0) {
      s_epoch = e;
      s_ok = ok;
    }
  }
  __syncthreads();
  bool bad = false;
  if (s_ok) {
    for (int t = blockIdx.x; t < tokens; t += gridDim.x)
      combine_token(y, y_rows, static_cast<const int32_t*>(nullptr), gates, out, t, k, N, &bad);
  }
  if (bad) report_status(kStatusBadExpertId, blockIdx.x);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    uint32_t* done = reinterpret_cast<uint32_t*>(epoch + 1);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      __threadfence();
      epoch[0] = s_epoch;
    }
  }
}

}  // namespace bokt
