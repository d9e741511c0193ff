/*
 * bokt.h - C ABI of the sm_100a (B200) kernels behind the bo-kernel-tuner
 * operator interface: dense GEMM, fused RMSNorm, MoE grouped GEMM and the
 * device-side MoE routing front end (expert histogram, offsets, stable token
 * permutation, combine indices).
 *
 * Every entry point takes plain device pointers, integer sizes and an opaque
 * CUDA stream (cudaStream_t passed as void*; NULL = legacy default stream).
 * Nothing here allocates device memory, synchronises the stream or reads a
 * result back, so every compute call can be captured in a CUDA graph once the
 * first call for a given configuration has run (the first call sets kernel
 * attributes).  Return value: 0 on success, a BOKT_ERR_* code otherwise; the
 * message is available from bokt_last_error() on the calling thread.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   bokt_gemm               <- bo_kernel_tuner/kernels/gemm.py:43-48  launch(a, b, out, params)
 *   bokt_rmsnorm            <- bo_kernel_tuner/kernels/rmsnorm.py:29-33 launch(x, weight, out, params, epsilon)
 *   bokt_moe_grouped_gemm   <- bo_kernel_tuner/kernels/moe_grouped_gemm.py:61-65
 *                              launch(x, weights, offsets, out, params, sm_count)
 *   bokt_moe_route          <- bo_kernel_tuner/tuner/worker.py:81-86 (host prefix sum of
 *                              expert token counts -> offsets); the permutation and combine
 *                              indices have no counterpart in the reference
 *                              (kernels/moe_grouped_gemm.py:3 leaves routing outside)
 *   bokt_rmsnorm_gemm       <- the two calls rmsnorm.launch(x, w, xn) then gemm.launch(xn, b, out)
 *   (+ _fold_weight,           (kernels/rmsnorm.py:29-33 followed by kernels/gemm.py:43-48),
 *    _row_scale,               fused: the normalised activations never reach HBM
 *    bokt_gemm_row_scaled)
 *   bokt_gather_rows        <- no counterpart (packing tokens in expert order)
 *   bokt_kernel_attrs       <- the Triton compiled-kernel metadata read by
 *                              bo_kernel_tuner/tuner/worker.py:193,203-204
 *                              (metadata.shared, n_regs, n_spills)
 */
#ifndef BOKT_H_
#define BOKT_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BOKT_ABI_VERSION 1

/* element types (values match the tcgen05 kind::f16 operand format codes) */
#define BOKT_FP16 0
#define BOKT_BF16 1
#define BOKT_FP32 2 /* router logits only */

/* status codes */
#define BOKT_OK 0
#define BOKT_ERR_INVALID 1     /* bad argument: null pointer, negative size, ... */
#define BOKT_ERR_UNSUPPORTED 2 /* legal request the library does not implement */
#define BOKT_ERR_CONFIG 3      /* launch parameters outside the kernel's domain */
#define BOKT_ERR_CUDA 4        /* a CUDA runtime/driver call failed */
#define BOKT_ERR_DEVICE 5      /* a kernel reported a timeout through the device status word */

/* kernel identifiers for bokt_kernel_attrs */
#define BOKT_KERNEL_GEMM 0
#define BOKT_KERNEL_RMSNORM 1
#define BOKT_KERNEL_MOE_GROUPED_GEMM 2
#define BOKT_KERNEL_RMSNORM_GEMM 3

/*
 * Launch parameters: the CUDA counterpart of the Triton meta-parameters the
 * reference tunes (configs/search_spaces.py:48-75).  A field left at 0 takes
 * the kernel's default.
 *   GEMM / grouped GEMM : block_m (128), block_n (64|128|256), block_k (64),
 *                         stages (2..8, bounded by shared memory), group_m
 *                         (grouped-M raster width), cta_multiplier (grouped GEMM
 *                         persistent grid = sm_count * cta_multiplier),
 *                         num_warps (6: TMA, MMA and four epilogue warps)
 *   RMSNorm             : rows_per_cta, num_warps; stages >= 2 selects the persistent
 *                         ring kernel (stages row buffers, num_warps consumer warps)
 *   GEMM                : cta_group 2 runs CTA pairs (tcgen05 cta_group::2, 256-row tiles)
 *   grouped GEMM        : raster 1 (the default) runs the tiles expert by expert;
 *                         raster 2 spreads the tiles of experts with at most two
 *                         row blocks evenly between the others, so their
 *                         once-read weights stream while other tiles compute
 */
typedef struct bokt_params {
  int32_t block_m;
  int32_t block_n;
  int32_t block_k;
  int32_t stages;
  int32_t group_m;
  int32_t cta_multiplier;
  int32_t num_warps;
  int32_t rows_per_cta;
  int32_t split_k;   /* 0/1: one worker runs a tile's whole K loop; 2..128: split-K /
                        stream-K (see bokt_gemm_ex); needs a workspace */
  int32_t cta_group; /* 0/1: one CTA per tile; 2: CTA pairs (dense GEMM) */
  int32_t raster;    /* grouped GEMM tile order: 0/1 expert order, 2 balanced
                        (low-reuse experts spread between the others) */
  int32_t reserved[5];
} bokt_params;

typedef struct bokt_attrs {
  int32_t shared_bytes;   /* static + dynamic shared memory per CTA */
  int32_t registers;      /* registers per thread */
  int32_t local_bytes;    /* local memory per thread (spill indicator) */
  int32_t threads;        /* threads per CTA */
  int32_t max_threads;    /* cudaFuncAttributes.maxThreadsPerBlock */
  int32_t path; /* 0 tcgen05/TMA, 1 tcgen05 edge, 2 vector, 3 scalar, 4 ring, 5 pipelined */
} bokt_attrs;

/* ABI version and the sm architecture the library was built for (100). */
int bokt_abi_version(void);
int bokt_built_sm(void);

/* Message of the last failing call on this thread ("" when none). */
const char* bokt_last_error(void);

/*
 * C[M,N] = A[M,K] * B[K,N]; all row-major, contiguous, same element type;
 * fp32 accumulation, result rounded to the element type on store.  Every
 * element of C is written.  Replaces kernels/gemm.py:43-48.
 * Shapes with K % 8, N % 8 or a pointer not 16-byte aligned (row strides TMA
 * cannot describe) take the tcgen05 edge kernel: masked element loads into the
 * swizzled shared-memory tiles, 128 x 64 tiles, still on tensor cores; everything
 * else runs on the TMA-fed tcgen05 kernels.
 */
int bokt_gemm(const void* A, const void* B, void* C, int M, int N, int K, int dtype,
              const bokt_params* params, void* stream);

/*
 * bokt_gemm with a split-K workspace.  params->split_k = S > 1 cuts every
 * tile's K loop into S slices of nearly equal k-block counts (S is clamped to
 * the number of 64-wide k-blocks) and deals the (tile, slice) units out to the
 * persistent CTAs (or CTA pairs) in contiguous runs, so every worker gets the
 * same number of k-block iterations even when the tile count is not a multiple
 * of the SM count; S = number of k-blocks is stream-K.  S in [1, 128].  For
 * S < 4 the worker that holds a tile's first slice adds the other workers'
 * fp32 partial tiles (read from the workspace, in worker order:
 * deterministic) and writes C.  For S >= 4 (without a row scale) every worker
 * stores the partials of the tiles it does not cover whole and a second
 * kernel, launched on the same stream right after, sums each split tile's
 * partials (fixed order: deterministic) and writes C.  The K loop being
 * split is the one of kernels/gemm.py:31-39 in the reference; the parameter is
 * the split-K entry of the redefined search space (configs/search_spaces.py:48-75).
 *
 * workspace: device memory of bokt_gemm_workspace_bytes(BOKT_KERNEL_GEMM,
 * params) bytes (about 39 MB at block_n 256 on a 148-SM B200), 256-byte
 * aligned and zero-filled ONCE when it is allocated; the library keeps a
 * launch sequence number in it, so it is not cleared between calls.  Calls
 * that share a workspace must not overlap on the GPU (use one per stream).
 * With split_k <= 1 the workspace may be NULL and the call equals bokt_gemm.
 */
int bokt_gemm_ex(const void* A, const void* B, void* C, int M, int N, int K, int dtype,
                 const bokt_params* params, void* workspace, int64_t workspace_bytes,
                 void* stream);

/* Workspace bytes for a split-K launch of `kernel` (BOKT_KERNEL_GEMM or
 * BOKT_KERNEL_MOE_GROUPED_GEMM) with `params` on the current device; 0 when
 * params->split_k <= 1, -1 on error. */
int64_t bokt_gemm_workspace_bytes(int kernel, const bokt_params* params);

/*
 * Inspection of the split-K schedule (host only, no GPU work): for `ntiles`
 * output tiles of `nkb` k-blocks, split_k slices per tile and `launched`
 * workers, writes one record of 6 int32 per segment into out[6 * i ..]:
 * {worker, tile, first k-block, one past the last k-block, first contributor
 * worker, contributor count} (contributors only for a tile's owner segment).
 * Returns the number of segments (records beyond `capacity` are not written),
 * or a negative status.  Exposes the exact arithmetic the kernels run.
 */
int bokt_splitk_schedule(int ntiles, int split_k, int nkb, int launched, int32_t* out,
                         int capacity);

/*
 * Sources of the separate split-K reduction (dense GEMMs with split_k >= 4):
 * for every tile split across workers, in tile order and then in the order
 * the reduction adds them, the triple (tile, worker, which) -- the partial in
 * workspace slot 2 c + which of the worker's CTA slot c (a pair worker p owns
 * CTA slots 2 p and 2 p + 1).  Same arguments and return convention as
 * bokt_splitk_schedule; the kernels' own arithmetic, run on the host.
 */
int bokt_splitk_reduce_sources(int ntiles, int split_k, int nkb, int launched, int32_t* out,
                               int capacity);

/*
 * Y[M,N] = X * rsqrt(mean(X^2, -1) + eps) * W, fp32 arithmetic, one pass over X.
 * Replaces kernels/rmsnorm.py:29-33.
 */
int bokt_rmsnorm(const void* X, const void* W, void* Y, int M, int N, float eps, int dtype,
                 const bokt_params* params, void* stream);

/*
 * Fused RMSNorm -> GEMM.  The reference chain rmsnorm.launch(x, w, xn) then
 * gemm.launch(xn, B, out) is computed as
 *   out[m, :] = s[m] * (X[m, :] @ B_folded),   B_folded[k, n] = w[k] * B[k, n],
 *   s[m] = rsqrt(sum_k X[m, k]^2 / K + eps),
 * with s applied to the fp32 accumulator in the tcgen05 GEMM epilogue: the
 * normalised activations never reach HBM.  The fold is done once per (w, B)
 * pair with bokt_rmsnorm_fold_weight; each call of bokt_rmsnorm_gemm runs the
 * one-pass row-scale kernel (reads X once; scales into the caller's row_scale
 * workspace of M floats) and the row-scaled GEMM (same params as bokt_gemm).
 * Needs K and N multiples of 8 and 16-byte aligned pointers (else
 * BOKT_ERR_UNSUPPORTED).
 */
int bokt_rmsnorm_fold_weight(const void* norm_weight, const void* B, void* B_folded, int K, int N,
                             int dtype, void* stream);
int bokt_rmsnorm_row_scale(const void* X, float* row_scale, int M, int K, float eps, int dtype,
                           void* stream);
int bokt_gemm_row_scaled(const void* A, const void* B, void* C, const float* row_scale, int M,
                         int N, int K, int dtype, const bokt_params* params, void* stream);
int bokt_rmsnorm_gemm(const void* X, const void* B_folded, void* C, float* row_scale, int M,
                      int N, int K, float eps, int dtype, const bokt_params* params,
                      void* stream);

/*
 * For each expert e: Y[off[e]:off[e+1]] = X[off[e]:off[e+1]] * W[e], W of shape
 * [E,K,N]; X and Y have T rows.  offsets has E+1 entries, int32
 * (offsets_is_i64 = 0) or int64 (1), resident on the device and read by the
 * kernel (no host copy, no per-expert launch).  Rows outside [off[0], off[E])
 * are not written, as in the reference.  Replaces
 * kernels/moe_grouped_gemm.py:61-65 (T is x.shape[0] there).
 */
int bokt_moe_grouped_gemm(const void* X, const void* W, const void* offsets, int offsets_is_i64,
                          void* Y, int T, int E, int N, int K, int dtype, int sm_count,
                          const bokt_params* params, void* stream);

/* bokt_moe_grouped_gemm with a split-K workspace (bokt_gemm_ex semantics;
 * split_k > 1 with single-CTA tiles only, cta_group 1). */
int bokt_moe_grouped_gemm_ex(const void* X, const void* W, const void* offsets,
                             int offsets_is_i64, void* Y, int T, int E, int N, int K, int dtype,
                             int sm_count, const bokt_params* params, void* workspace,
                             int64_t workspace_bytes, void* stream);

/*
 * Routing front end for A = tokens * topk assignments given as expert ids
 * (int32, flattened token-major, values in [0, E)).  Outputs (all int32, device):
 *   counts[E]      tokens per expert
 *   offsets[E+1]   exclusive prefix sum of counts (offsets[E] = A)
 *   perm[A]        stable sort of assignments by expert: perm[j] = assignment index
 *                  placed at packed row j
 *   inv_perm[A]    combine index: inv_perm[i] = packed row of assignment i
 * offsets64 (optional, may be NULL) receives the same offsets as int64.
 * workspace: device scratch of bokt_moe_route_workspace_bytes(A, E) bytes.
 * Ids outside [0, E) are an error: the kernel sets the device status word and
 * the outputs are unspecified.
 */
int64_t bokt_moe_route_workspace_bytes(int A, int E);
int bokt_moe_route(const int32_t* expert_ids, int A, int E, int32_t* counts, int32_t* offsets,
                   int64_t* offsets64, int32_t* perm, int32_t* inv_perm, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * bokt_moe_route without a workspace argument, for callers that cannot
 * allocate device memory at all: code running where every byte of device
 * memory is owned by another allocator (a framework's caching pool, a
 * serving engine's pre-partitioned arena), a foreign runtime bound through
 * this C ABI with no device allocator of its own, or a real-time loop where
 * cudaMalloc's implicit synchronisation is not allowed.  No counterpart in the
 * reference (its offsets are a host prefix sum, tuner/worker.py:83-86).
 *
 * Scratch is a fixed 256 KiB device array inside the library (every GPU that
 * loads the library holds it until the process exits).  Limit:
 * ceil(A / 4096) * E <= bokt_moe_route_noalloc_max_words() (65536), e.g.
 * 32768 assignments x 1024 experts or 1,048,576 x 256; larger requests fail
 * with BOKT_ERR_UNSUPPORTED and a message, nothing is launched.  The first call
 * on each device, and again in any new CUDA context on it (after a device
 * reset, or with a context of the caller's own), looks the array's device
 * address up (cudaGetSymbolAddress), so make that first call outside stream
 * capture.  All calls on a device share
 * the one array: calls that overlap on the GPU (different streams, no ordering
 * between them) race and give wrong results; calls in one stream are fine.
 * Outputs are identical to bokt_moe_route's.  Allocates nothing.
 */
int64_t bokt_moe_route_noalloc_max_words(void);
int bokt_moe_route_noalloc(const int32_t* expert_ids, int A, int E, int32_t* counts,
                           int32_t* offsets, int64_t* offsets64, int32_t* perm, int32_t* inv_perm,
                           void* stream);

/*
 * Row gather: dst[j, :] = src[index[j] / divisor, :] for j < rows; row length
 * `cols` elements of `elem_bytes` bytes; src has src_rows rows.  Packs token
 * activations into expert order (divisor = topk, index = perm).  An index
 * outside src sets the device status word and leaves that row unwritten.
 */
int bokt_gather_rows(const void* src, int64_t src_rows, void* dst, const int32_t* index, int rows,
                     int cols, int elem_bytes, int divisor, void* stream);

/*
 * Two-level row gather for expert-parallel dispatch / combine:
 *   dst[j, :] = src[inner[outer[j]] / divisor - base, :]   (outer == NULL: inner[j])
 * inner has inner_len entries, src has src_rows rows of cols elements.  A
 * source outside src sets the device status word; the row is left unwritten.
 * No counterpart in the reference (single GPU only).
 */
int bokt_gather_rows_indirect(const void* src, int64_t src_rows, void* dst, const int32_t* inner,
                              int64_t inner_len, const int32_t* outer, int rows, int cols,
                              int elem_bytes, int divisor, int64_t base, void* stream);

/*
 * Expert-parallel sort keys of every packed row p of the global routing, as
 * seen by rank `me` of `world` (tokens owned in contiguous blocks of
 * tokens_per_rank).  Expert e is served by replicas[e] virtual experts
 * vbase[e] .. vbase[e] + replicas[e] - 1 that split its packed rows
 * contiguously (row q of the expert goes to replica q * replicas[e] / counts[e]);
 * v_rank[v] is the rank serving virtual expert v and v_local[v] its index
 * among that rank's virtual experts.  Outputs (int32[A]):
 *   key_send[p]  = destination rank if this rank owns the token, else world
 *   key_recv[p]  = owning rank if this rank serves the row, else world
 *   key_local[p] = local virtual-expert index if this rank serves it, else n_local
 * Sorting each key with bokt_moe_route gives the send order, the receive order
 * and the local grouped-GEMM order.  No counterpart in the reference.
 */
int bokt_ep_keys(const int32_t* perm, const int32_t* ids, const int32_t* offsets,
                 const int32_t* counts, const int32_t* replicas, const int32_t* vbase,
                 const int32_t* v_rank, const int32_t* v_local, int A, int E, int topk,
                 int tokens_per_rank, int me, int world, int n_local, int32_t* key_send,
                 int32_t* key_recv, int32_t* key_local, void* stream);

/*
 * Sets the device status word (code 3, detail tag * 65536 + i) where
 * counts[i] != expected[i]: the split sizes an expert-parallel plan fixed for
 * NCCL no longer match the routing.  No counterpart in the reference.
 */
int bokt_check_counts(const int32_t* counts, const int32_t* expected, int n, int tag,
                      void* stream);

/*
 * Expert-parallel combine fused into the grouped GEMM: like
 * bokt_moe_grouped_gemm, but packed output row l is not written to a local Y:
 * with a = rowmap[l] and o = a / rows_per_owner it is stored at row
 * a - o * rows_per_owner of out_ptrs[o] (a device array of `owners` pointers,
 * each [rows_per_owner, N]; entries may be peer GPUs' buffers mapped through
 * CUDA IPC, written with NVLink stores from the epilogue while later tiles
 * compute).  tcgen05 path only.  No counterpart in the reference.
 */
int bokt_moe_grouped_gemm_scatter(const void* X, const void* W, const void* offsets,
                                  int offsets_is_i64, int T, int E, int N, int K, int dtype,
                                  int sm_count, const int32_t* rowmap, void* const* out_ptrs,
                                  int rows_per_owner, int owners, const bokt_params* params,
                                  void* stream);

/*
 * Per-step expert-parallel layout (one CTA): virtual expert v serves the
 * global packed rows [v_plo[v], v_plo[v] + v_size[v]) and is stored at local
 * rows [v_lbase[v], ...) of its rank's packed buffer (virtual experts in
 * ascending v).  loffs: rank `me`'s grouped-GEMM offsets; rank_rows: rows per
 * rank; a rank above capacity[r] sets the device status word (code 4).
 * No counterpart in the reference.
 */
int bokt_ep_plan(const int32_t* counts, const int32_t* offsets, const int32_t* replicas, int E,
                 const int32_t* v_rank, int V, int world, int me, const int32_t* capacity,
                 int32_t* v_plo, int32_t* v_size, int32_t* v_lbase, int32_t* loffs,
                 int32_t* rank_rows, void* stream);

/*
 * Expert-parallel dispatch over NVLink: each of this rank's a_local
 * assignments copies its token row (x_local row a_local_index / topk) into the
 * packed buffer xpk_ptrs[d] of the serving rank d at its local position
 * (xpk_ptrs: device array of per-rank pointers, peers' buffers mapped through
 * CUDA IPC).  Rows must be 16-byte multiples.  Positions beyond capacity[d]
 * are reported (code 4) and skipped.  No counterpart in the reference.
 */
int bokt_ep_dispatch(const void* x_local, int cols, int elem_bytes, const int32_t* ids,
                     const int32_t* inv_perm, const int32_t* offsets, const int32_t* counts,
                     const int32_t* replicas, const int32_t* vbase, const int32_t* v_rank,
                     const int32_t* v_plo, const int32_t* v_lbase, void* const* xpk_ptrs,
                     const int32_t* capacity, int a_local, int topk, int me, int E,
                     void* stream);

/*
 * rowmap[l] = global assignment index of local packed row l of rank `me`
 * (input of the scatter epilogue).  No counterpart in the reference.
 */
int bokt_ep_rowmap(const int32_t* perm, const int32_t* ids, const int32_t* offsets,
                   const int32_t* counts, const int32_t* replicas, const int32_t* vbase,
                   const int32_t* v_rank, const int32_t* v_plo, const int32_t* v_lbase, int A,
                   int E, int me, int capacity, int32_t* rowmap, void* stream);

/*
 * Expert-parallel step synchronisation without a host collective (plain
 * NVLink peer loads and stores; each rank on its own GPU).
 * bokt_ep_put: copies `bytes` from src into dst_ptrs[d] + dst_offset_bytes for
 * every rank d (dst_ptrs: device array of `world` pointers, peers' buffers
 * mapped through CUDA IPC); 16-byte aligned sizes and offsets.  The
 * all-gather of the routing ids.
 * bokt_ep_barrier: every rank advances the device counter `epoch` (its own
 * memory, zero-initialised) and stores the new epoch into slot `me` of every
 * rank's flag array flag_ptrs[d] (int32[world] per rank, zero-initialised,
 * peers' through CUDA IPC); then waits until every slot of flag_ptrs[me] has
 * reached the epoch.  All ranks must call the same sequence of barriers.  A
 * wait longer than timeout_ns records a timeout in the device status word
 * (detail 4000 + the silent rank) and returns.  Capturable in a CUDA graph
 * (the epoch lives on the device).  No counterpart in the reference (its
 * worker runs one GPU).
 */
int bokt_ep_put(const void* src, int64_t bytes, void* const* dst_ptrs, int64_t dst_offset_bytes,
                int world, void* stream);
int bokt_ep_barrier(int32_t* const* flag_ptrs, int32_t* epoch, int world, int me,
                    int64_t timeout_ns, void* stream);

/*
 * The step's last barrier with the gate-weighted combine fused into it (the
 * receive side of the scatter combine): the barrier of bokt_ep_barrier, after
 * which -- every peer's grouped GEMM having stored its result rows into this
 * rank's slot buffer y [tokens * k, N], row t * k + j for token t's j-th
 * expert -- the same kernel writes out[t] = sum_j gates[t k + j] * y[t k + j]
 * for this rank's `tokens` tokens (fp32, slot order; bit-identical to
 * bokt_moe_combine with rows = NULL).  epoch: int32[2] (barrier epoch, CTA
 * count), zero-initialised, shared with bokt_ep_barrier.  A timeout skips the
 * combine and is recorded as in bokt_ep_barrier.  The combine of the MoE layer
 * (the reference leaves it outside its operator, kernels/moe_grouped_gemm.py:3).
 */
int bokt_ep_barrier_combine(int32_t* const* flag_ptrs, int32_t* epoch, int world, int me,
                            int64_t timeout_ns, const void* y, const float* gates, void* out,
                            int tokens, int k, int N, int dtype, void* stream);

/*
 * CUDA IPC plumbing for the expert-parallel peer buffers.  bokt_ipc_export
 * writes the 64-byte IPC handle of the allocation containing `ptr` and the
 * offset of `ptr` inside it (works for sub-allocations of a caching
 * allocator); bokt_ipc_import opens a peer process's handle on the current
 * device (peer access enabled lazily) and returns the mapping base (for
 * bokt_ipc_close) and base + offset.  No counterpart in the reference.
 */
int bokt_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int bokt_ipc_import(const void* handle, int64_t offset, void** base_out, void** ptr_out);
int bokt_ipc_close(void* base);

/*
 * Top-k softmax gate (routing front end): per token t, p = softmax(logits[t, :])
 * in fp32; ids[t, j] (int32 [tokens, k]) = the j-th largest p, ties to the
 * lower expert index; gates[t, j] (fp32) = p of that expert, divided by the sum
 * of the k picked when renormalize != 0.  logits: [tokens, E] fp16/bf16/fp32.
 * k <= 8, E <= 1024.  No counterpart in the reference (routing is outside
 * kernels/moe_grouped_gemm.py:3).
 */
int bokt_moe_topk_gate(const void* logits, int logits_dtype, int tokens, int E, int k,
                       int renormalize, int32_t* ids, float* gates, void* stream);

/*
 * Gate-weighted combine: out[t, :] = sum_j gates[t, j] * y[row, :] with
 * row = rows[t * k + j] (e.g. the routing's inv_perm when y is packed by
 * expert) or t * k + j when rows is NULL (y in assignment order); fp32
 * accumulation, rounded to dtype.  N % 8 == 0.  A row outside y sets the
 * device status word.  No counterpart in the reference.
 */
int bokt_moe_combine(const void* y, int64_t y_rows, const int32_t* rows, const float* gates,
                     void* out, int tokens, int k, int N, int dtype, void* stream);

/*
 * Failure-detection self-test: launches one CTA that waits on an mbarrier
 * nothing will complete, with the same bounded wait every pipelined kernel
 * uses.  After timeout_ns (<= 10 s) the wait gives up, the kernel writes 1 to
 * the device int *gave_up, records code 1 / detail 99 in the device status
 * word and returns; the CUDA context stays usable.  No counterpart in the
 * reference.
 */
int bokt_selftest_bounded_wait(int64_t timeout_ns, int* gave_up, void* stream);

/* Resource usage of the kernel a call with these arguments would launch. */
int bokt_kernel_attrs(int kernel, int dtype, int n, int k, const bokt_params* params,
                      bokt_attrs* out);

/*
 * Device status word of the current device: 0 when no kernel has reported a
 * bounded-wait timeout or an out-of-range routing id since the last reset.
 * Synchronises the device.  reset != 0 clears it.
 */
int bokt_device_status(int* code, int* detail, int reset);

#ifdef __cplusplus
}
#endif

#endif /* BOKT_H_ */
