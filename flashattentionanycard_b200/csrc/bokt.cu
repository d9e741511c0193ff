// C ABI of the sm_100a kernel library (declarations and reference citations in
// include/bokt.h).  Host side: argument checks, path selection, TMA tensor-map
// encoding, launch configuration.  No allocation, no synchronisation and no
// host read-back on any compute entry point.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/bokt.h"
#include "bokt_device.cuh"
#include "ep_sync.cuh"
#include "gemm_edge.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "moe_route.cuh"
#include "norm_gemm.cuh"
#include "rmsnorm.cuh"

namespace {

thread_local char g_err[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(BOKT_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int param_or(int v, int dflt) { return v > 0 ? v : dflt; }

// Programmatic dependent launch for every kernel (each kernel waits with
// griddepcontrol.wait before touching global memory).  BOKT_DISABLE_PDL=1
// turns the attribute off, e.g. to compare timings.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("BOKT_DISABLE_PDL");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

cudaLaunchConfig_t launch_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                 cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cfg;
}

// Typed launch: kernel<<<grid, block, smem, s>>>(args...) with PDL.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   Args... args) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_config(grid, block, smem, s, attr);
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Untyped launch through a kernel pointer and an argument array, with PDL.
cudaError_t launch_ptr(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       void** args) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_config(grid, block, smem, s, attr);
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// ----------------------------------------------------------------- device info
struct DeviceInfo {
  int sm_count = 0;
  int smem_optin = 0;
};
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(BOKT_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sm_count == 0) {
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    if (major != 10)
      return fail(BOKT_ERR_UNSUPPORTED, "library built for sm_100a; device %d is sm_%d.x", dev,
                  major);
    e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  }
  *out = d;
  return BOKT_OK;
}

// Raise a kernel's dynamic shared-memory limit once per (device, kernel, size).
// The first call for a configuration happens outside graph capture (warm-up).
struct SmemAttr {
  int dev;
  const void* fn;
  int bytes;
};
SmemAttr g_smem_attr[512];
int g_smem_attr_n = 0;
std::mutex g_smem_mu;

int ensure_smem(const void* fn, int bytes) {
  if (bytes <= 48 * 1024) return BOKT_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_smem_mu);
  for (int i = 0; i < g_smem_attr_n; ++i)
    if (g_smem_attr[i].dev == dev && g_smem_attr[i].fn == fn && g_smem_attr[i].bytes >= bytes)
      return BOKT_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  if (g_smem_attr_n < 512) g_smem_attr[g_smem_attr_n++] = {dev, fn, bytes};
  return BOKT_OK;
}

// ----------------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(BOKT_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  return BOKT_OK;
}

// Row-major [outer..., rows, cols] 16-bit tensor, box {64 cols, box_rows, 1...},
// 128-byte swizzle, zero fill outside the tensor.
int encode_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, bool fp16) {
  (void)fp16;
  int rc = get_encoder();
  if (rc) return rc;
  uint32_t elem_strides[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, rank, const_cast<void*>(base), dims,
                        strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BOKT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return BOKT_OK;
}

// ----------------------------------------------------------------- GEMM dispatch
using bokt::GemmTcArgs;

template <int BN, bool GROUPED, typename T, bool SCATTER, bool ROWSCALE = false>
const void* tc_kernel_ptr() {
  return reinterpret_cast<const void*>(&bokt::gemm_tc_kernel<BN, GROUPED, T, SCATTER, ROWSCALE>);
}

template <bool GROUPED, typename T, bool SCATTER, bool ROWSCALE = false>
const void* tc_kernel_for(int bn) {
  switch (bn) {
    case 64: return tc_kernel_ptr<64, GROUPED, T, SCATTER, ROWSCALE>();
    case 128: return tc_kernel_ptr<128, GROUPED, T, SCATTER, ROWSCALE>();
    case 256: return tc_kernel_ptr<256, GROUPED, T, SCATTER, ROWSCALE>();
  }
  return nullptr;
}

const void* tc_kernel(bool grouped, int dtype, int bn, bool scatter = false,
                      bool rowscale = false) {
  if (rowscale)
    return dtype == BOKT_BF16 ? tc_kernel_for<false, __nv_bfloat16, false, true>(bn)
                              : tc_kernel_for<false, __half, false, true>(bn);
  if (scatter)
    return dtype == BOKT_BF16 ? tc_kernel_for<true, __nv_bfloat16, true>(bn)
                              : tc_kernel_for<true, __half, true>(bn);
  if (grouped)
    return dtype == BOKT_BF16 ? tc_kernel_for<true, __nv_bfloat16, false>(bn)
                              : tc_kernel_for<true, __half, false>(bn);
  return dtype == BOKT_BF16 ? tc_kernel_for<false, __nv_bfloat16, false>(bn)
                            : tc_kernel_for<false, __half, false>(bn);
}

struct TcConfig {
  int bn, stages, group_m, smem, cta_group, raster, split_k;
};

int resolve_tc_config(const bokt_params* p, bool grouped, int experts, int smem_optin,
                      TcConfig* out) {
  const bokt_params zero = {};
  if (!p) p = &zero;
  const int bm = param_or(p->block_m, 128);
  const int bk = param_or(p->block_k, 64);
  const int bn = param_or(p->block_n, 256);
  const int warps = param_or(p->num_warps, 6);
  if (bm != 128) return fail(BOKT_ERR_CONFIG, "block_m must be 128 (tcgen05 cta_group::1 M)");
  if (bk != 64) return fail(BOKT_ERR_CONFIG, "block_k must be 64 (one 128-byte swizzle row)");
  if (bn != 64 && bn != 128 && bn != 256)
    return fail(BOKT_ERR_CONFIG, "block_n must be 64, 128 or 256 (got %d)", bn);
  if (warps != 6) return fail(BOKT_ERR_CONFIG, "num_warps must be 6 (TMA, MMA, 4 epilogue)");
  const int split_k = param_or(p->split_k, 1);
  if (split_k < 1 || split_k > bokt::kSplitKMax)
    return fail(BOKT_ERR_CONFIG, "split_k must be in [1, %d] (got %d)", bokt::kSplitKMax, split_k);
  const int cta_group = param_or(p->cta_group, 1);
  if (cta_group != 1 && cta_group != 2) return fail(BOKT_ERR_CONFIG, "cta_group must be 1 or 2");
  if (split_k > 1 && cta_group == 2 && grouped)
    return fail(BOKT_ERR_CONFIG,
                "split_k > 1 applies to the dense GEMM (single CTAs or pairs) and the "
                "single-CTA grouped GEMM, not to grouped CTA pairs");
  if (cta_group == 2 && bn == 64)
    return fail(BOKT_ERR_CONFIG, "cta_group 2 needs block_n 128 or 256");
  const int raster = param_or(p->raster, bokt::kRasterExpert);
  if (raster != bokt::kRasterExpert && raster != bokt::kRasterBalanced)
    return fail(BOKT_ERR_CONFIG, "raster must be 1 (expert order) or 2 (balanced)");
  if (raster == bokt::kRasterBalanced && !grouped)
    return fail(BOKT_ERR_CONFIG, "raster 2 applies to the grouped GEMM (dense: group_m)");
  const int stages = param_or(p->stages, cta_group == 2 ? (bn == 256 ? 6 : 8) : (bn == 256 ? 4 : 6));
  if (stages < 2 || stages > 8) return fail(BOKT_ERR_CONFIG, "stages must be in [2, 8]");
  int smem = cta_group == 2 ? bokt::gemm_tc2_smem_bytes(bn, stages, grouped ? experts : 0)
                            : bokt::gemm_tc_smem_bytes(bn, stages, grouped, experts);
  if (smem > smem_optin)
    return fail(BOKT_ERR_CONFIG, "block_n=%d stages=%d needs %d bytes of shared memory (max %d)",
                bn, stages, smem, smem_optin);
  // One CTA per SM: the persistent schedule assumes it and two CTAs would
  // contend for the 512 TMEM columns.
  const int one_per_sm = smem_optin / 2 + 1024;
  if (smem < one_per_sm) smem = one_per_sm;
  out->bn = bn;
  out->stages = stages;
  out->group_m = param_or(p->group_m, 8);
  out->smem = smem;
  out->cta_group = cta_group;
  out->raster = raster;
  out->split_k = split_k;
  return BOKT_OK;
}

// Split-K workspace of the current device: one slot per SM (no launch of a
// split-K kernel uses more CTAs), sized for the configuration's BN.
int64_t splitk_bytes_for(const DeviceInfo& dev, int bn) {
  return bokt::splitk_workspace_bytes(dev.sm_count, bn);
}

// Attach the workspace to `args` for a split-K launch; checks size and alignment.
int attach_splitk(const TcConfig& cfg, const DeviceInfo& dev, int nkb, void* ws, int64_t ws_bytes,
                  GemmTcArgs* args) {
  int split = cfg.split_k < nkb ? cfg.split_k : nkb;
  if (split < 1) split = 1;
  args->split_k = split;
  if (split == 1) return BOKT_OK;
  const int64_t need = splitk_bytes_for(dev, cfg.bn);
  if (!ws)
    return fail(BOKT_ERR_INVALID,
                "split_k > 1 needs a workspace of %lld bytes (zero-filled once when allocated); "
                "pass it to the _ex entry point", (long long)need);
  if (ws_bytes < need)
    return fail(BOKT_ERR_INVALID, "split-K workspace too small: %lld bytes, need %lld",
                (long long)ws_bytes, (long long)need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(BOKT_ERR_INVALID, "split-K workspace must be 256-byte aligned");
  args->splitk_ws = ws;
  args->splitk_slots = dev.sm_count;
  return BOKT_OK;
}

template <typename T, bool ROWSCALE, bool GROUPED, bool SCATTER = false>
const void* tc2_kernel_for(int bn) {
  return bn == 256
             ? reinterpret_cast<const void*>(&bokt::gemm_tc2_kernel<256, T, ROWSCALE, GROUPED, SCATTER>)
             : reinterpret_cast<const void*>(&bokt::gemm_tc2_kernel<128, T, ROWSCALE, GROUPED, SCATTER>);
}

const void* tc2_kernel(int dtype, int bn, bool rowscale = false, bool grouped = false,
                       bool scatter = false) {
  const bool bf = dtype == BOKT_BF16;
  if (scatter)
    return bf ? tc2_kernel_for<__nv_bfloat16, false, true, true>(bn)
              : tc2_kernel_for<__half, false, true, true>(bn);
  if (grouped)
    return bf ? tc2_kernel_for<__nv_bfloat16, false, true>(bn)
              : tc2_kernel_for<__half, false, true>(bn);
  if (rowscale)
    return bf ? tc2_kernel_for<__nv_bfloat16, true, false>(bn)
              : tc2_kernel_for<__half, true, false>(bn);
  return bf ? tc2_kernel_for<__nv_bfloat16, false, false>(bn)
            : tc2_kernel_for<__half, false, false>(bn);
}

// Dense GEMM on CTA pairs: cluster of 2 along x, PDL as every other launch.
int launch_tc2(int dtype, const TcConfig& cfg, const CUtensorMap& ma, const CUtensorMap& mb,
               const GemmTcArgs& args, int pairs, cudaStream_t s, bool grouped = false,
               bool scatter = false, const CUtensorMap* ma64 = nullptr) {
  const void* fn = tc2_kernel(dtype, cfg.bn, args.row_scale != nullptr, grouped, scatter);
  int rc = ensure_smem(fn, cfg.smem);
  if (rc) return rc;
  // Third map: 64-row A boxes for grouped half-height tiles (unused by dense launches).
  void* kargs[] = {const_cast<CUtensorMap*>(&ma), const_cast<CUtensorMap*>(&mb),
                   const_cast<CUtensorMap*>(ma64 ? ma64 : &ma), const_cast<GemmTcArgs*>(&args)};
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t lc = launch_config(
      dim3(2 * pairs), dim3(bokt::kGemmThreads), cfg.smem, s,
      attr);
  attr[lc.numAttrs].id = cudaLaunchAttributeClusterDimension;
  attr[lc.numAttrs].val.clusterDim.x = 2;
  attr[lc.numAttrs].val.clusterDim.y = 1;
  attr[lc.numAttrs].val.clusterDim.z = 1;
  lc.numAttrs += 1;
  cudaError_t e = cudaLaunchKernelExC(&lc, fn, kargs);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_tc2 launch");
  return BOKT_OK;
}

int launch_tc(bool grouped, int dtype, const TcConfig& cfg, const CUtensorMap& ma,
              const CUtensorMap& mb, const GemmTcArgs& args, int grid, cudaStream_t s,
              bool scatter = false) {
  const void* fn = tc_kernel(grouped, dtype, cfg.bn, scatter, args.row_scale != nullptr);
  int rc = ensure_smem(fn, cfg.smem);
  if (rc) return rc;
  void* kargs[] = {const_cast<CUtensorMap*>(&ma), const_cast<CUtensorMap*>(&mb),
                   const_cast<GemmTcArgs*>(&args)};
  cudaError_t e = launch_ptr(fn, dim3(grid), dim3(bokt::kGemmThreads), cfg.smem, s, kargs);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_tc launch");
  return BOKT_OK;
}

// Edge shapes (row strides TMA cannot describe): the tcgen05 edge kernel, one
// CTA per 128 x 64 tile.  Dense: experts == 0, rows = M; grouped: rows = T.
template <typename T>
int launch_edge(const void* A, const void* B, void* C, int rows, int N, int K,
                const void* offsets, int offsets_i64, int experts, int dtype, cudaStream_t s) {
  const long long nn = (N + bokt::kEdgeBN - 1) / bokt::kEdgeBN;
  const long long mtiles = (rows + bokt::kEdgeBM - 1) / bokt::kEdgeBM + (experts > 0 ? experts : 0);
  const long long tiles = mtiles * nn;
  if (tiles > 0x7fffffffLL) return fail(BOKT_ERR_UNSUPPORTED, "edge path: too many tiles");
  const uint32_t idesc = bokt::make_idesc_f16(uint32_t(dtype), bokt::kEdgeBM, bokt::kEdgeBN);
  cudaError_t e = launch(bokt::gemm_tc_edge_kernel<T>, dim3(unsigned(tiles)),
                         dim3(bokt::kEdgeThreads), bokt::kEdgeSmemBytes, s,
                         static_cast<const T*>(A), static_cast<const T*>(B), static_cast<T*>(C),
                         rows, N, K, offsets, offsets_i64, experts, idesc);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_tc_edge launch");
  return BOKT_OK;
}

// The separate split-K reduction after a dense launch with args.splitk_reduce
// set: one CTA per (tile, CTA row half, 8 / lanes column groups of 4),
// 128 rows x `lanes` worker lanes; lanes grows with the workers one tile can
// span (about four partials per lane, at most 8 lanes).
int launch_splitk_reduce(int dtype, const TcConfig& cfg, const GemmTcArgs& args, int launched,
                         bool pair, cudaStream_t s) {
  const int tile_rows = pair ? 256 : 128;
  const long long nt = (long long)((args.M + tile_rows - 1) / tile_rows) *
                       ((args.N + cfg.bn - 1) / cfg.bn);
  const int ntiles = int(nt);
  const int workers = bokt::splitk_workers(launched, ntiles, args.split_k);
  const int span = (workers + ntiles - 1) / ntiles + 1;  // workers one tile can touch
  int lanes = 1;
  while (lanes * 4 < span && lanes < 8) lanes *= 2;
  const long long blocks = nt * (pair ? 2 : 1) * (cfg.bn / (32 / lanes));
  if (blocks > 0x7fffffffLL) return fail(BOKT_ERR_UNSUPPORTED, "split-K reduction: too many tiles");
  const float* partials = reinterpret_cast<const float*>(
      static_cast<const uint8_t*>(args.splitk_ws) + bokt::kSplitKHeaderBytes +
      bokt::splitk_flags_bytes(args.splitk_slots));
  const int p = pair ? 1 : 0;
  cudaError_t e = cudaSuccess;
  auto go = [&](auto kernel, auto* c) {
    e = launch(kernel, dim3(unsigned(blocks)), dim3(128 * lanes), 0, s, partials, c, args.M,
               args.N, args.split_k, workers, ntiles, p, cfg.bn, args.group_m);
  };
  if (dtype == BOKT_BF16) {
    auto* c = static_cast<__nv_bfloat16*>(args.C);
    if (lanes == 1) go(bokt::splitk_reduce_kernel<__nv_bfloat16, 1>, c);
    else if (lanes == 2) go(bokt::splitk_reduce_kernel<__nv_bfloat16, 2>, c);
    else if (lanes == 4) go(bokt::splitk_reduce_kernel<__nv_bfloat16, 4>, c);
    else go(bokt::splitk_reduce_kernel<__nv_bfloat16, 8>, c);
  } else {
    auto* c = static_cast<__half*>(args.C);
    if (lanes == 1) go(bokt::splitk_reduce_kernel<__half, 1>, c);
    else if (lanes == 2) go(bokt::splitk_reduce_kernel<__half, 2>, c);
    else if (lanes == 4) go(bokt::splitk_reduce_kernel<__half, 4>, c);
    else go(bokt::splitk_reduce_kernel<__half, 8>, c);
  }
  if (e != cudaSuccess) return cuda_fail(e, "splitk_reduce launch");
  return BOKT_OK;
}

bool tc_eligible(const void* A, const void* B, const void* C, int N, int K) {
  return K > 0 && (K % 8) == 0 && (N % 8) == 0 && aligned16(A) && aligned16(B) && aligned16(C);
}

// Dense GEMM entry body.  row_scale != nullptr scales C row m by row_scale[m]
// in the epilogue (the fused RMSNorm -> GEMM; tcgen05 path only).
int dense_gemm_impl(const void* A, const void* B, void* C, int M, int N, int K, int dtype,
                    const bokt_params* params, void* stream, const float* row_scale,
                    void* workspace = nullptr, int64_t workspace_bytes = 0) {
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (M < 0 || N < 0 || K < 0) return fail(BOKT_ERR_INVALID, "negative size");
  if (M == 0 || N == 0) return BOKT_OK;
  if (!A || !B || !C) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  if (!tc_eligible(A, B, C, N, K)) {
    if (row_scale)
      return fail(BOKT_ERR_UNSUPPORTED,
                  "fused RMSNorm-GEMM needs K > 0, K and N multiples of 8 and 16-byte aligned "
                  "operands (got M=%d N=%d K=%d)", M, N, K);
    return dtype == BOKT_BF16
               ? launch_edge<__nv_bfloat16>(A, B, C, M, N, K, nullptr, 0, 0, dtype, s)
               : launch_edge<__half>(A, B, C, M, N, K, nullptr, 0, 0, dtype, s);
  }
  TcConfig cfg;
  rc = resolve_tc_config(params, false, 0, dev.smem_optin, &cfg);
  if (rc) return rc;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {uint64_t(K), uint64_t(M)};
  const uint64_t sa[1] = {uint64_t(K) * 2};
  const uint32_t ba[2] = {64, 128};
  rc = encode_map(&ma, A, 2, da, sa, ba, dtype == BOKT_FP16);
  if (rc) return rc;
  const uint64_t db[2] = {uint64_t(N), uint64_t(K)};
  const uint64_t sb[1] = {uint64_t(N) * 2};
  const uint32_t bb[2] = {64, 64};
  rc = encode_map(&mb, B, 2, db, sb, bb, dtype == BOKT_FP16);
  if (rc) return rc;
  GemmTcArgs args = {};
  args.C = C;
  args.M = M;
  args.N = N;
  args.K = K;
  args.group_m = cfg.group_m;
  args.stages = cfg.stages;
  args.row_scale = row_scale;
  rc = attach_splitk(cfg, dev, (K + bokt::kGemmBK - 1) / bokt::kGemmBK, workspace,
                     workspace_bytes, &args);
  if (rc) return rc;
  const long long split = args.split_k;
  // Many slices per tile: partials summed by a separate, fully parallel
  // kernel instead of the owner's serial fix-up (not with the fused row scale,
  // which the owner's epilogue applies).
  args.splitk_reduce = split >= bokt::kSplitKReduceMin && !row_scale ? 1 : 0;
  if (cfg.cta_group == 2) {
    args.idesc = bokt::make_idesc_f16(uint32_t(dtype), 256, uint32_t(cfg.bn));
    const long long units = (long long)((M + 255) / 256) * ((N + cfg.bn - 1) / cfg.bn) * split;
    const long long max_pairs = dev.sm_count / 2;
    const int pairs = int(units < max_pairs ? units : max_pairs);
    rc = launch_tc2(dtype, cfg, ma, mb, args, pairs, s);
    if (rc || !args.splitk_reduce) return rc;
    return launch_splitk_reduce(dtype, cfg, args, pairs, true, s);
  }
  args.idesc = bokt::make_idesc_f16(uint32_t(dtype), 128, uint32_t(cfg.bn));
  const long long units = (long long)((M + 127) / 128) * ((N + cfg.bn - 1) / cfg.bn) * split;
  const int grid = int(units < dev.sm_count ? units : dev.sm_count);
  rc = launch_tc(false, dtype, cfg, ma, mb, args, grid, s);
  if (rc || !args.splitk_reduce) return rc;
  return launch_splitk_reduce(dtype, cfg, args, grid, false, s);
}

// ----------------------------------------------------------------- RMSNorm dispatch
struct NormConfig {
  int rows_per_cta, threads, tpr_log2, vpt;  // vpt 0 = generic kernel
  int ring_slots;                            // > 0: persistent TMA-staged ring kernel
};

int resolve_norm_config(const bokt_params* p, int N, bool vec_ok, NormConfig* out) {
  const bokt_params zero = {};
  if (!p) p = &zero;
  const int rows = param_or(p->rows_per_cta, 1);
  const int warps = param_or(p->num_warps, 4);
  if (warps != 1 && warps != 2 && warps != 4 && warps != 8 && warps != 16 && warps != 32)
    return fail(BOKT_ERR_CONFIG, "num_warps must be a power of two <= 32 (got %d)", warps);
  if (rows != 1 && rows != 2 && rows != 4 && rows != 8 && rows != 16)
    return fail(BOKT_ERR_CONFIG, "rows_per_cta must be 1, 2, 4, 8 or 16 (got %d)", rows);
  const int threads = warps * 32;
  if (rows > threads) return fail(BOKT_ERR_CONFIG, "rows_per_cta exceeds threads per CTA");
  const int tpr = threads / rows;
  int lg = 0;
  while ((1 << lg) < tpr) ++lg;
  int vpt = 0;
  if (vec_ok) {
    const int nvec = N / 8;
    const int need = (nvec + tpr - 1) / tpr;
    int v = 1;
    while (v < need) v <<= 1;
    if (v <= 16) vpt = v;
  }
  const int stages = param_or(p->stages, 1);
  if (stages < 1 || stages > 32) return fail(BOKT_ERR_CONFIG, "stages must be in [1, 32]");
  // The ring kernel streams whole rows with cp.async.bulk (16-byte multiples,
  // 16-byte aligned); odd or unaligned rows take the per-row kernels instead,
  // as odd GEMM shapes take the edge GEMM kernel.
  int ring = 0;
  if (stages == 2 && vec_ok && rows == 1 && vpt > 0 && vpt <= 8) {
    // Two register buffers: the persistent software-pipelined kernel (one row
    // per CTA at a time).  Other shapes keep the per-row kernels.
    *out = {rows, threads, lg, vpt, -1};
    return BOKT_OK;
  }
  if (stages >= 4 && vec_ok) {
    if (warps > 31) return fail(BOKT_ERR_CONFIG, "ring kernel: num_warps must be <= 31");
    if (stages % warps != 0)
      return fail(BOKT_ERR_CONFIG,
                  "ring kernel: stages (%d) must be a multiple of num_warps (%d) so each ring "
                  "slot is consumed by one warp",
                  stages, warps);
    ring = stages;
  }
  *out = {rows, threads, lg, vpt, ring};
  return BOKT_OK;
}

// The three routing launches, scratch = ceil(A / 4096) * E int32 words.
int launch_route(const int32_t* ids, int A, int E, int32_t* scratch, int32_t* counts,
                 int32_t* offsets, int64_t* offsets64, int32_t* perm, int32_t* inv_perm,
                 cudaStream_t s, const char* what) {
  const int chunks = (A + bokt::kRouteChunk - 1) / bokt::kRouteChunk;
  cudaError_t e = cudaSuccess;
  if (chunks > 0)
    e = launch(bokt::route_count_kernel, dim3(chunks), dim3(bokt::kRouteThreads), 0, s, ids, A, E,
               scratch);
  if (e == cudaSuccess)
    e = launch(bokt::route_scan_kernel, dim3(1), dim3(1024), 0, s, scratch, chunks, E, counts,
               offsets, reinterpret_cast<long long*>(offsets64));
  if (e == cudaSuccess && chunks > 0)
    e = launch(bokt::route_scatter_kernel, dim3(chunks), dim3(bokt::kRouteThreads), 0, s, ids, A,
               E, static_cast<const int32_t*>(scratch), perm, inv_perm);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return BOKT_OK;
}

template <typename T>
const void* pipe_kernel(int vpt) {
  switch (vpt) {
    case 1: return reinterpret_cast<const void*>(&bokt::rmsnorm_pipe_kernel<T, 1>);
    case 2: return reinterpret_cast<const void*>(&bokt::rmsnorm_pipe_kernel<T, 2>);
    case 4: return reinterpret_cast<const void*>(&bokt::rmsnorm_pipe_kernel<T, 4>);
    case 8: return reinterpret_cast<const void*>(&bokt::rmsnorm_pipe_kernel<T, 8>);
  }
  return nullptr;
}

template <typename T>
const void* norm_kernel(int vpt) {
  switch (vpt) {
    case 0: return reinterpret_cast<const void*>(&bokt::rmsnorm_generic_kernel<T>);
    case 1: return reinterpret_cast<const void*>(&bokt::rmsnorm_vec_kernel<T, 1>);
    case 2: return reinterpret_cast<const void*>(&bokt::rmsnorm_vec_kernel<T, 2>);
    case 4: return reinterpret_cast<const void*>(&bokt::rmsnorm_vec_kernel<T, 4>);
    case 8: return reinterpret_cast<const void*>(&bokt::rmsnorm_vec_kernel<T, 8>);
    case 16: return reinterpret_cast<const void*>(&bokt::rmsnorm_vec_kernel<T, 16>);
  }
  return nullptr;
}

}  // namespace

// =================================================================== C ABI
extern "C" {

int bokt_abi_version(void) { return BOKT_ABI_VERSION; }

int bokt_built_sm(void) { return 100; }

const char* bokt_last_error(void) { return g_err; }

int bokt_gemm(const void* A, const void* B, void* C, int M, int N, int K, int dtype,
              const bokt_params* params, void* stream) {
  g_err[0] = 0;
  return dense_gemm_impl(A, B, C, M, N, K, dtype, params, stream, nullptr);
}

int bokt_gemm_ex(const void* A, const void* B, void* C, int M, int N, int K, int dtype,
                 const bokt_params* params, void* workspace, int64_t workspace_bytes,
                 void* stream) {
  g_err[0] = 0;
  return dense_gemm_impl(A, B, C, M, N, K, dtype, params, stream, nullptr, workspace,
                         workspace_bytes);
}

int64_t bokt_gemm_workspace_bytes(int kernel, const bokt_params* params) {
  g_err[0] = 0;
  if (kernel != BOKT_KERNEL_GEMM && kernel != BOKT_KERNEL_MOE_GROUPED_GEMM) return 0;
  const bokt_params zero = {};
  const bokt_params* p = params ? params : &zero;
  if (param_or(p->split_k, 1) <= 1) return 0;
  DeviceInfo dev;
  if (device_info(&dev)) return -1;
  return splitk_bytes_for(dev, param_or(p->block_n, 256));
}

int bokt_rmsnorm_fold_weight(const void* norm_weight, const void* B, void* B_folded, int K, int N,
                             int dtype, void* stream) {
  g_err[0] = 0;
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (K < 0 || N < 0) return fail(BOKT_ERR_INVALID, "negative size");
  if (K == 0 || N == 0) return BOKT_OK;
  if (!norm_weight || !B || !B_folded) return fail(BOKT_ERR_INVALID, "null pointer");
  if (N % 8 != 0 || !aligned16(B) || !aligned16(B_folded))
    return fail(BOKT_ERR_UNSUPPORTED, "fold needs N %% 8 == 0 and 16-byte aligned B, B_folded");
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  const long long vecs = (long long)K * (N / 8);
  long long blocks = (vecs + 255) / 256;
  if (blocks > 8LL * dev.sm_count) blocks = 8LL * dev.sm_count;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = dtype == BOKT_BF16
      ? launch(bokt::fold_norm_weight_kernel<__nv_bfloat16>, dim3(unsigned(blocks)), dim3(256), 0, s,
               static_cast<const __nv_bfloat16*>(norm_weight),
               static_cast<const __nv_bfloat16*>(B), static_cast<__nv_bfloat16*>(B_folded), K, N)
      : launch(bokt::fold_norm_weight_kernel<__half>, dim3(unsigned(blocks)), dim3(256), 0, s,
               static_cast<const __half*>(norm_weight), static_cast<const __half*>(B),
               static_cast<__half*>(B_folded), K, N);
  if (e != cudaSuccess) return cuda_fail(e, "fold_norm_weight launch");
  return BOKT_OK;
}

int bokt_rmsnorm_row_scale(const void* X, float* scale, int M, int K, float eps, int dtype,
                           void* stream) {
  g_err[0] = 0;
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (M < 0 || K <= 0) return fail(BOKT_ERR_INVALID, "bad size");
  if (M == 0) return BOKT_OK;
  if (!X || !scale) return fail(BOKT_ERR_INVALID, "null pointer");
  if (!(eps >= 0.f) || !(eps < 3.0e38f)) return fail(BOKT_ERR_INVALID, "eps must be finite >= 0");
  if (K % 8 != 0 || !aligned16(X))
    return fail(BOKT_ERR_UNSUPPORTED, "row scale needs K %% 8 == 0 and a 16-byte aligned X");
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  const int warps = bokt::kRowScaleThreads / 32;
  long long blocks = ((long long)M + warps - 1) / warps;
  if (blocks > 16LL * dev.sm_count) blocks = 16LL * dev.sm_count;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = dtype == BOKT_BF16
      ? launch(bokt::rmsnorm_row_scale_kernel<__nv_bfloat16>, dim3(unsigned(blocks)),
               dim3(bokt::kRowScaleThreads), 0, s, static_cast<const __nv_bfloat16*>(X), scale, M,
               K, eps)
      : launch(bokt::rmsnorm_row_scale_kernel<__half>, dim3(unsigned(blocks)),
               dim3(bokt::kRowScaleThreads), 0, s, static_cast<const __half*>(X), scale, M, K, eps);
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm_row_scale launch");
  return BOKT_OK;
}

int bokt_gemm_row_scaled(const void* A, const void* B, void* C, const float* row_scale, int M,
                         int N, int K, int dtype, const bokt_params* params, void* stream) {
  g_err[0] = 0;
  if (!row_scale) return fail(BOKT_ERR_INVALID, "null row_scale");
  return dense_gemm_impl(A, B, C, M, N, K, dtype, params, stream, row_scale);
}

int bokt_rmsnorm_gemm(const void* X, const void* B_folded, void* C, float* row_scale, int M,
                      int N, int K, float eps, int dtype, const bokt_params* params,
                      void* stream) {
  g_err[0] = 0;
  if (!row_scale) return fail(BOKT_ERR_INVALID, "null row_scale workspace");
  if (M > 0 && N > 0 && !tc_eligible(X, B_folded, C, N, K))
    return fail(BOKT_ERR_UNSUPPORTED,
                "fused RMSNorm-GEMM needs K > 0, K and N multiples of 8 and 16-byte aligned "
                "operands (got M=%d N=%d K=%d)", M, N, K);
  int rc = bokt_rmsnorm_row_scale(X, row_scale, M, K, eps, dtype, stream);
  if (rc) return rc;
  return dense_gemm_impl(X, B_folded, C, M, N, K, dtype, params, stream, row_scale);
}

}  // extern "C"

namespace {

// Shared body of the grouped GEMM entry points; scatter != nullptr selects the
// expert-parallel epilogue that sends each packed row to its owner's buffer.
struct ScatterArgs {
  const int32_t* rowmap;
  void* const* out_ptrs;
  int rows_per_owner;
  int owners;
};

int grouped_gemm_impl(const void* X, const void* W, const void* offsets, int offsets_is_i64,
                      void* Y, int T, int E, int N, int K, int dtype, int sm_count,
                      const bokt_params* params, void* stream, const ScatterArgs* scatter,
                      void* workspace = nullptr, int64_t workspace_bytes = 0) {
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (T < 0 || E < 0 || N < 0 || K < 0) return fail(BOKT_ERR_INVALID, "negative size");
  if (E > bokt::kGemmMaxExperts)
    return fail(BOKT_ERR_UNSUPPORTED, "at most %d experts", bokt::kGemmMaxExperts);
  if (T == 0 || E == 0 || N == 0) return BOKT_OK;
  if (!X || !W || !Y || !offsets) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  if (!tc_eligible(X, W, Y, N, K)) {
    if (scatter)
      return fail(BOKT_ERR_UNSUPPORTED,
                  "scatter epilogue needs the tcgen05 path (K, N multiples of 8, aligned)");
    return dtype == BOKT_BF16
               ? launch_edge<__nv_bfloat16>(X, W, Y, T, N, K, offsets, offsets_is_i64, E, dtype, s)
               : launch_edge<__half>(X, W, Y, T, N, K, offsets, offsets_is_i64, E, dtype, s);
  }
  const bokt_params zero = {};
  TcConfig cfg;
  rc = resolve_tc_config(params, true, E, dev.smem_optin, &cfg);
  if (rc) return rc;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {uint64_t(K), uint64_t(T)};
  const uint64_t sa[1] = {uint64_t(K) * 2};
  const uint32_t ba[2] = {64, 128};
  rc = encode_map(&ma, X, 2, da, sa, ba, dtype == BOKT_FP16);
  if (rc) return rc;
  const uint64_t db[3] = {uint64_t(N), uint64_t(K), uint64_t(E)};
  const uint64_t sb[2] = {uint64_t(N) * 2, uint64_t(K) * uint64_t(N) * 2};
  const uint32_t bb[3] = {64, 64, 1};
  rc = encode_map(&mb, W, 3, db, sb, bb, dtype == BOKT_FP16);
  if (rc) return rc;
  GemmTcArgs args = {};
  args.C = Y;
  args.M = T;
  args.N = N;
  args.K = K;
  args.group_m = 1;
  args.stages = cfg.stages;
  args.idesc = bokt::make_idesc_f16(uint32_t(dtype), 128, uint32_t(cfg.bn));
  args.offsets = offsets;
  args.offsets_i64 = offsets_is_i64 ? 1 : 0;
  args.E = E;
  args.raster = cfg.raster;
  if (scatter) {
    args.rowmap = scatter->rowmap;
    args.out_ptrs = scatter->out_ptrs;
    args.rows_per_owner = scatter->rows_per_owner;
    args.owners = scatter->owners;
  }
  const int mult = param_or((params ? params : &zero)->cta_multiplier, 1);
  const int sms = sm_count > 0 ? sm_count : dev.sm_count;
  const long long nn = (N + cfg.bn - 1) / cfg.bn;
  if (cfg.cta_group == 2) {
    // CTA pairs: 256-row tiles per expert, a last block of <= 128 rows as a
    // half-height tile (M = 128, 64 rows per CTA, A boxes of 64 rows).
    CUtensorMap ma64;
    const uint32_t ba64[2] = {64, 64};
    rc = encode_map(&ma64, X, 2, da, sa, ba64, dtype == BOKT_FP16);
    if (rc) return rc;
    GemmTcArgs pa = args;
    pa.idesc = bokt::make_idesc_f16(uint32_t(dtype), 256, uint32_t(cfg.bn));
    pa.idesc_half = bokt::make_idesc_f16(uint32_t(dtype), 128, uint32_t(cfg.bn));
    const long long max_pair_tiles = ((long long)(T + 255) / 256 + E) * nn;
    long long pairs = sms / 2;
    if (pairs > max_pair_tiles) pairs = max_pair_tiles;
    if (pairs < 1) pairs = 1;
    return launch_tc2(dtype, cfg, ma, mb, pa, int(pairs), s, /*grouped=*/true, scatter != nullptr,
                      &ma64);
  }
  rc = attach_splitk(cfg, dev, (K + bokt::kGemmBK - 1) / bokt::kGemmBK, workspace,
                     workspace_bytes, &args);
  if (rc) return rc;
  // Upper bound on tiles without reading offsets: sum_e cdiv(c_e, 128) <= cdiv(T, 128) + E.
  const long long max_tiles = ((long long)(T + 127) / 128 + E) * nn;
  long long grid = (long long)sms * mult;
  if (args.split_k > 1 && grid > dev.sm_count) grid = dev.sm_count;  // one slot per CTA
  if (grid > max_tiles * args.split_k) grid = max_tiles * args.split_k;
  if (grid < 1) grid = 1;
  return launch_tc(true, dtype, cfg, ma, mb, args, int(grid), s, scatter != nullptr);
}

}  // namespace

extern "C" {

int bokt_moe_grouped_gemm(const void* X, const void* W, const void* offsets, int offsets_is_i64,
                          void* Y, int T, int E, int N, int K, int dtype, int sm_count,
                          const bokt_params* params, void* stream) {
  g_err[0] = 0;
  return grouped_gemm_impl(X, W, offsets, offsets_is_i64, Y, T, E, N, K, dtype, sm_count, params,
                           stream, nullptr);
}

int bokt_moe_grouped_gemm_ex(const void* X, const void* W, const void* offsets,
                             int offsets_is_i64, void* Y, int T, int E, int N, int K, int dtype,
                             int sm_count, const bokt_params* params, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  return grouped_gemm_impl(X, W, offsets, offsets_is_i64, Y, T, E, N, K, dtype, sm_count, params,
                           stream, nullptr, workspace, workspace_bytes);
}

int bokt_moe_grouped_gemm_scatter(const void* X, const void* W, const void* offsets,
                                  int offsets_is_i64, int T, int E, int N, int K, int dtype,
                                  int sm_count, const int32_t* rowmap, void* const* out_ptrs,
                                  int rows_per_owner, int owners, const bokt_params* params,
                                  void* stream) {
  g_err[0] = 0;
  if (!rowmap || !out_ptrs || rows_per_owner <= 0 || owners <= 0)
    return fail(BOKT_ERR_INVALID, "scatter needs rowmap, out_ptrs, rows_per_owner, owners");
  const ScatterArgs sc = {rowmap, out_ptrs, rows_per_owner, owners};
  // Y is unused by the scatter epilogue; any valid aligned pointer satisfies the path checks.
  return grouped_gemm_impl(X, W, offsets, offsets_is_i64, const_cast<void*>(X), T, E, N, K,
                           dtype, sm_count, params, stream, &sc);
}

int bokt_ep_plan(const int32_t* counts, const int32_t* offsets, const int32_t* replicas, int E,
                 const int32_t* v_rank, int V, int world, int me, const int32_t* capacity,
                 int32_t* v_plo, int32_t* v_size, int32_t* v_lbase, int32_t* loffs,
                 int32_t* rank_rows, void* stream) {
  g_err[0] = 0;
  if (E <= 0 || V <= 0 || world <= 0 || me < 0 || me >= world)
    return fail(BOKT_ERR_INVALID, "bad size");
  if (!counts || !offsets || !replicas || !v_rank || !capacity || !v_plo || !v_size ||
      !v_lbase || !loffs || !rank_rows)
    return fail(BOKT_ERR_INVALID, "null pointer");
  const int smem = bokt::ep_plan_smem_bytes(E, V, world);
  if (smem > 200 * 1024) return fail(BOKT_ERR_UNSUPPORTED, "ep_plan: E, V or world too large");
  int rc = ensure_smem(reinterpret_cast<const void*>(&bokt::ep_plan_kernel), smem);
  if (rc) return rc;
  cudaError_t e = launch(bokt::ep_plan_kernel, dim3(1), dim3(256), smem,
                         static_cast<cudaStream_t>(stream), counts, offsets, replicas, E, v_rank,
                         V, world, me, capacity, v_plo, v_size, v_lbase, loffs, rank_rows);
  if (e != cudaSuccess) return cuda_fail(e, "ep_plan launch");
  return BOKT_OK;
}

int bokt_ep_dispatch(const void* x_local, int cols, int elem_bytes, const int32_t* ids,
                     const int32_t* inv_perm, const int32_t* offsets, const int32_t* counts,
                     const int32_t* replicas, const int32_t* vbase, const int32_t* v_rank,
                     const int32_t* v_plo, const int32_t* v_lbase, void* const* xpk_ptrs,
                     const int32_t* capacity, int a_local, int topk, int me, int E,
                     void* stream) {
  g_err[0] = 0;
  if (cols <= 0 || elem_bytes <= 0 || a_local < 0 || topk <= 0 || me < 0 || E <= 0)
    return fail(BOKT_ERR_INVALID, "bad size");
  if (a_local == 0) return BOKT_OK;
  const long long row_bytes = (long long)cols * elem_bytes;
  if (row_bytes % 16 != 0 || !aligned16(x_local))
    return fail(BOKT_ERR_UNSUPPORTED, "dispatch rows must be 16-byte multiples, 16-byte aligned");
  if (!ids || !inv_perm || !offsets || !counts || !replicas || !vbase || !v_rank || !v_plo ||
      !v_lbase || !xpk_ptrs || !capacity)
    return fail(BOKT_ERR_INVALID, "null pointer");
  const int warps_per_block = 8;
  int grid = (a_local + warps_per_block - 1) / warps_per_block;
  if (grid > 148 * 16) grid = 148 * 16;
  cudaError_t e = launch(bokt::ep_dispatch_kernel, dim3(grid), dim3(32 * warps_per_block), 0,
                         static_cast<cudaStream_t>(stream), static_cast<const uint4*>(x_local),
                         int(row_bytes / 16), ids, inv_perm, offsets, counts, replicas, vbase,
                         v_rank, v_plo, v_lbase, reinterpret_cast<uint4* const*>(xpk_ptrs),
                         capacity, a_local, topk, me, E);
  if (e != cudaSuccess) return cuda_fail(e, "ep_dispatch launch");
  return BOKT_OK;
}

int bokt_ep_put(const void* src, int64_t bytes, void* const* dst_ptrs, int64_t dst_offset_bytes,
                int world, void* stream) {
  g_err[0] = 0;
  if (bytes < 0 || dst_offset_bytes < 0 || world <= 0 || world > bokt::kEpMaxWorld)
    return fail(BOKT_ERR_INVALID, "bad size");
  if (bytes == 0) return BOKT_OK;
  if (!src || !dst_ptrs) return fail(BOKT_ERR_INVALID, "null pointer");
  if (bytes % 16 != 0 || dst_offset_bytes % 16 != 0 || !aligned16(src))
    return fail(BOKT_ERR_UNSUPPORTED, "put needs 16-byte aligned source, size and offset");
  const long long vecs = bytes / 16;
  long long grid = (vecs + 255) / 256;
  if (grid > 148 * 4) grid = 148 * 4;
  cudaError_t e = launch(bokt::ep_put_kernel, dim3(unsigned(grid)), dim3(256), 0,
                         static_cast<cudaStream_t>(stream), static_cast<const uint4*>(src),
                         (long long)vecs, reinterpret_cast<uint4* const*>(dst_ptrs),
                         (long long)(dst_offset_bytes / 16), world);
  if (e != cudaSuccess) return cuda_fail(e, "ep_put launch");
  return BOKT_OK;
}

int bokt_ep_barrier(int32_t* const* flag_ptrs, int32_t* epoch, int world, int me,
                    int64_t timeout_ns, void* stream) {
  g_err[0] = 0;
  if (world <= 0 || world > bokt::kEpMaxWorld || me < 0 || me >= world)
    return fail(BOKT_ERR_INVALID, "bad world/rank");
  if (timeout_ns <= 0 || timeout_ns > 60000000000ll)
    return fail(BOKT_ERR_INVALID, "timeout must be in (0, 60 s]");
  if (!flag_ptrs || !epoch) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaError_t e = launch(bokt::ep_barrier_kernel, dim3(1), dim3(32), 0,
                         static_cast<cudaStream_t>(stream), flag_ptrs, epoch, world, me,
                         (long long)timeout_ns);
  if (e != cudaSuccess) return cuda_fail(e, "ep_barrier launch");
  return BOKT_OK;
}

int bokt_ep_barrier_combine(int32_t* const* flag_ptrs, int32_t* epoch, int world, int me,
                            int64_t timeout_ns, const void* y, const float* gates, void* out,
                            int tokens, int k, int N, int dtype, void* stream) {
  g_err[0] = 0;
  if (world <= 0 || world > bokt::kEpMaxWorld || me < 0 || me >= world)
    return fail(BOKT_ERR_INVALID, "bad world/rank");
  if (timeout_ns <= 0 || timeout_ns > 60000000000ll)
    return fail(BOKT_ERR_INVALID, "timeout must be in (0, 60 s]");
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (tokens < 0 || k <= 0 || N <= 0) return fail(BOKT_ERR_INVALID, "bad size");
  if (!flag_ptrs || !epoch || (tokens > 0 && (!y || !gates || !out)))
    return fail(BOKT_ERR_INVALID, "null pointer");
  if (N % 8 != 0 || (tokens > 0 && (!aligned16(y) || !aligned16(out))))
    return fail(BOKT_ERR_UNSUPPORTED, "combine needs N %% 8 == 0 and 16-byte aligned rows");
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  // Every CTA waits for the peers, so keep the grid within one wave.
  long long grid = tokens < 1 ? 1 : tokens;
  if (grid > 4LL * dev.sm_count) grid = 4LL * dev.sm_count;
  const int threads = N / 8 < 256 ? ((N / 8 + 31) / 32) * 32 : 256;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long y_rows = (long long)tokens * k;
  cudaError_t e =
      dtype == BOKT_BF16
          ? launch(bokt::ep_barrier_combine_kernel<__nv_bfloat16>, dim3(unsigned(grid)),
                   dim3(threads), 0, s, flag_ptrs, epoch, world, me, (long long)timeout_ns,
                   static_cast<const __nv_bfloat16*>(y), y_rows, gates,
                   static_cast<__nv_bfloat16*>(out), tokens, k, N)
          : launch(bokt::ep_barrier_combine_kernel<__half>, dim3(unsigned(grid)), dim3(threads),
                   0, s, flag_ptrs, epoch, world, me, (long long)timeout_ns,
                   static_cast<const __half*>(y), y_rows, gates, static_cast<__half*>(out),
                   tokens, k, N);
  if (e != cudaSuccess) return cuda_fail(e, "ep_barrier_combine launch");
  return BOKT_OK;
}

int bokt_ep_rowmap(const int32_t* perm, const int32_t* ids, const int32_t* offsets,
                   const int32_t* counts, const int32_t* replicas, const int32_t* vbase,
                   const int32_t* v_rank, const int32_t* v_plo, const int32_t* v_lbase, int A,
                   int E, int me, int capacity, int32_t* rowmap, void* stream) {
  g_err[0] = 0;
  if (A < 0 || E <= 0 || me < 0 || capacity < 0) return fail(BOKT_ERR_INVALID, "bad size");
  if (A == 0) return BOKT_OK;
  if (!perm || !ids || !offsets || !counts || !replicas || !vbase || !v_rank || !v_plo ||
      !v_lbase || !rowmap)
    return fail(BOKT_ERR_INVALID, "null pointer");
  const int grid = (A + 255) / 256 < 4096 ? (A + 255) / 256 : 4096;
  cudaError_t e = launch(bokt::ep_rowmap_kernel, dim3(grid), dim3(256), 0,
                         static_cast<cudaStream_t>(stream), perm, ids, offsets, counts, replicas,
                         vbase, v_rank, v_plo, v_lbase, A, E, me, capacity, rowmap);
  if (e != cudaSuccess) return cuda_fail(e, "ep_rowmap launch");
  return BOKT_OK;
}

int bokt_rmsnorm(const void* X, const void* W, void* Y, int M, int N, float eps, int dtype,
                 const bokt_params* params, void* stream) {
  g_err[0] = 0;
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (M < 0 || N < 0) return fail(BOKT_ERR_INVALID, "negative size");
  if (M == 0 || N == 0) return BOKT_OK;
  if (!X || !W || !Y) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec_ok = (N % 8) == 0 && aligned16(X) && aligned16(W) && aligned16(Y);
  NormConfig cfg;
  int rc = resolve_norm_config(params, N, vec_ok, &cfg);
  if (rc) return rc;
  if (cfg.ring_slots < 0) {
    DeviceInfo dev;
    rc = device_info(&dev);
    if (rc) return rc;
    const void* pfn = dtype == BOKT_BF16 ? pipe_kernel<__nv_bfloat16>(cfg.vpt)
                                         : pipe_kernel<__half>(cfg.vpt);
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pfn, cfg.threads, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (per_sm < 1) per_sm = 1;
    long long grid = (long long)dev.sm_count * per_sm;
    if (grid > M) grid = M;
    void* pargs[] = {const_cast<void**>(&X), const_cast<void**>(&W), &Y, &M, &N, &eps,
                     &cfg.tpr_log2};
    e = launch_ptr(pfn, dim3(unsigned(grid)), dim3(cfg.threads), 0, s, pargs);
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm pipe launch");
    return BOKT_OK;
  }
  if (cfg.ring_slots > 0) {
    DeviceInfo dev;
    rc = device_info(&dev);
    if (rc) return rc;
    const int smem = bokt::rmsnorm_ring_smem_bytes(N, 2, cfg.ring_slots);
    if (smem > dev.smem_optin)
      return fail(BOKT_ERR_CONFIG, "ring kernel: %d slots of %d-element rows need %d bytes of "
                                   "shared memory (max %d)", cfg.ring_slots, N, smem,
                  dev.smem_optin);
    const void* rfn = dtype == BOKT_BF16
                          ? reinterpret_cast<const void*>(&bokt::rmsnorm_ring_kernel<__nv_bfloat16>)
                          : reinterpret_cast<const void*>(&bokt::rmsnorm_ring_kernel<__half>);
    rc = ensure_smem(rfn, smem);
    if (rc) return rc;
    int per_sm = (228 * 1024) / (smem + 1024);
    if (per_sm < 1) per_sm = 1;
    if (per_sm > 4) per_sm = 4;
    long long grid = (long long)dev.sm_count * per_sm;
    if (grid > M) grid = M;
    int slots = cfg.ring_slots;
    void* rargs[] = {const_cast<void**>(&X), const_cast<void**>(&W), &Y, &M, &N, &eps, &slots};
    cudaError_t e = launch_ptr(rfn, dim3(unsigned(grid)), dim3(cfg.threads + 32), smem, s, rargs);
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm ring launch");
    return BOKT_OK;
  }
  const int grid = (M + cfg.rows_per_cta - 1) / cfg.rows_per_cta;
  const void* fn = dtype == BOKT_BF16 ? norm_kernel<__nv_bfloat16>(cfg.vpt)
                                      : norm_kernel<__half>(cfg.vpt);
  void* kargs[] = {const_cast<void**>(&X), const_cast<void**>(&W), &Y, &M, &N, &eps,
                   &cfg.rows_per_cta, &cfg.tpr_log2};
  cudaError_t e = launch_ptr(fn, dim3(grid), dim3(cfg.threads), 0, s, kargs);
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
  return BOKT_OK;
}

int64_t bokt_moe_route_workspace_bytes(int A, int E) {
  if (A < 0 || E <= 0) return 0;
  const int64_t chunks = (A + bokt::kRouteChunk - 1) / bokt::kRouteChunk;
  return (chunks > 0 ? chunks : 1) * int64_t(E) * 4;
}

int bokt_moe_route(const int32_t* expert_ids, int A, int E, int32_t* counts, int32_t* offsets,
                   int64_t* offsets64, int32_t* perm, int32_t* inv_perm, void* workspace,
                   int64_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  if (A < 0 || E <= 0) return fail(BOKT_ERR_INVALID, "need A >= 0 and E > 0");
  if (E > bokt::kRouteMaxExperts)
    return fail(BOKT_ERR_UNSUPPORTED, "at most %d experts", bokt::kRouteMaxExperts);
  if (!counts || !offsets || (A > 0 && (!expert_ids || !perm || !inv_perm)))
    return fail(BOKT_ERR_INVALID, "null pointer");
  if (workspace_bytes < bokt_moe_route_workspace_bytes(A, E) || !workspace)
    return fail(BOKT_ERR_INVALID, "workspace too small: need %lld bytes",
                (long long)bokt_moe_route_workspace_bytes(A, E));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* ws = static_cast<int32_t*>(workspace);
  return launch_route(expert_ids, A, E, ws, counts, offsets, offsets64, perm, inv_perm, s,
                      "moe_route launch");
}

int bokt_gather_rows(const void* src, int64_t src_rows, void* dst, const int32_t* index, int rows,
                     int cols, int elem_bytes, int divisor, void* stream) {
  g_err[0] = 0;
  if (rows < 0 || cols < 0 || src_rows < 0 || divisor <= 0 || elem_bytes <= 0)
    return fail(BOKT_ERR_INVALID, "bad size");
  if (rows == 0 || cols == 0) return BOKT_OK;
  if (!src || !dst || !index) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long row_bytes = (long long)cols * elem_bytes;
  const int grid = rows < 65535 * 4 ? rows : 65535 * 4;
  cudaError_t e;
  if (row_bytes % 16 == 0 && aligned16(src) && aligned16(dst)) {
    const int vecs = int(row_bytes / 16);
    e = launch(bokt::gather_rows_kernel<uint4>, dim3(grid), dim3(128), 0, s,
               static_cast<const uint4*>(src), (long long)src_rows, static_cast<uint4*>(dst), index,
               rows, vecs, divisor);
  } else {
    e = launch(bokt::gather_rows_kernel<uint8_t>, dim3(grid), dim3(128), 0, s,
               static_cast<const uint8_t*>(src), (long long)src_rows, static_cast<uint8_t*>(dst),
               index, rows, int(row_bytes), divisor);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gather_rows launch");
  return BOKT_OK;
}

int bokt_gather_rows_indirect(const void* src, int64_t src_rows, void* dst, const int32_t* inner,
                               int64_t inner_len, const int32_t* outer, int rows, int cols,
                               int elem_bytes, int divisor, int64_t base, void* stream) {
  g_err[0] = 0;
  if (rows < 0 || cols < 0 || src_rows < 0 || divisor <= 0 || elem_bytes <= 0 || inner_len < 0)
    return fail(BOKT_ERR_INVALID, "bad size");
  if (rows == 0 || cols == 0) return BOKT_OK;
  if (!src || !dst || !inner) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long row_bytes = (long long)cols * elem_bytes;
  const int grid = rows < 65535 * 4 ? rows : 65535 * 4;
  cudaError_t e;
  if (row_bytes % 16 == 0 && aligned16(src) && aligned16(dst)) {
    e = launch(bokt::gather_rows_indirect_kernel<uint4>, dim3(grid), dim3(128), 0, s,
               static_cast<const uint4*>(src), (long long)src_rows, static_cast<uint4*>(dst),
               inner, outer, (long long)inner_len, rows, int(row_bytes / 16), divisor,
               (long long)base);
  } else {
    e = launch(bokt::gather_rows_indirect_kernel<uint8_t>, dim3(grid), dim3(128), 0, s,
               static_cast<const uint8_t*>(src), (long long)src_rows, static_cast<uint8_t*>(dst),
               inner, outer, (long long)inner_len, rows, int(row_bytes), divisor,
               (long long)base);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gather_rows_indirect launch");
  return BOKT_OK;
}

int bokt_ep_keys(const int32_t* perm, const int32_t* ids, const int32_t* offsets,
                 const int32_t* counts, const int32_t* replicas, const int32_t* vbase,
                 const int32_t* v_rank, const int32_t* v_local, int A, int E, int topk,
                 int tokens_per_rank, int me, int world, int n_local, int32_t* key_send,
                 int32_t* key_recv, int32_t* key_local, void* stream) {
  g_err[0] = 0;
  if (A < 0 || E <= 0 || topk <= 0 || tokens_per_rank <= 0 || world <= 0 || me < 0 ||
      me >= world || n_local < 0)
    return fail(BOKT_ERR_INVALID, "bad size");
  if (A == 0) return BOKT_OK;
  if (!perm || !ids || !offsets || !counts || !replicas || !vbase || !v_rank || !v_local ||
      !key_send || !key_recv || !key_local)
    return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = (A + 255) / 256 < 4096 ? (A + 255) / 256 : 4096;
  cudaError_t e = launch(bokt::ep_keys_kernel, dim3(grid), dim3(256), 0, s, perm, ids, offsets,
                         counts, replicas, vbase, v_rank, v_local, A, E, topk, tokens_per_rank,
                         me, world, n_local, key_send, key_recv, key_local);
  if (e != cudaSuccess) return cuda_fail(e, "ep_keys launch");
  return BOKT_OK;
}

int bokt_check_counts(const int32_t* counts, const int32_t* expected, int n, int tag,
                      void* stream) {
  g_err[0] = 0;
  if (n < 0) return fail(BOKT_ERR_INVALID, "bad size");
  if (n == 0) return BOKT_OK;
  if (!counts || !expected) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaError_t e = launch(bokt::check_counts_kernel, dim3(1), dim3(256), 0,
                         static_cast<cudaStream_t>(stream), counts, expected, n, tag);
  if (e != cudaSuccess) return cuda_fail(e, "check_counts launch");
  return BOKT_OK;
}

int bokt_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  g_err[0] = 0;
  if (!ptr || !handle_out || !offset_out) return fail(BOKT_ERR_INVALID, "null pointer");
  static PFN_cuMemGetAddressRange_v3020 get_range = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!get_range) return fail(BOKT_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(BOKT_ERR_CUDA, "cuMemGetAddressRange failed (%d)", int(r));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return BOKT_OK;
}

int bokt_ipc_import(const void* handle, int64_t offset, void** base_out, void** ptr_out) {
  g_err[0] = 0;
  if (!handle || !base_out || !ptr_out || offset < 0) return fail(BOKT_ERR_INVALID, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return BOKT_OK;
}

int bokt_ipc_close(void* base) {
  g_err[0] = 0;
  if (!base) return BOKT_OK;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return BOKT_OK;
}

int bokt_moe_topk_gate(const void* logits, int logits_dtype, int tokens, int E, int k,
                       int renormalize, int32_t* ids, float* gates, void* stream) {
  g_err[0] = 0;
  if (tokens < 0 || E <= 0 || k <= 0) return fail(BOKT_ERR_INVALID, "bad size");
  if (k > bokt::kTopkMax || k > E)
    return fail(BOKT_ERR_UNSUPPORTED, "k must be <= %d and <= E", bokt::kTopkMax);
  if (E > bokt::kGateMaxExperts)
    return fail(BOKT_ERR_UNSUPPORTED, "at most %d experts", bokt::kGateMaxExperts);
  if (tokens == 0) return BOKT_OK;
  if (!logits || !ids || !gates) return fail(BOKT_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int grid = (tokens + 7) / 8;
  if (grid > 148 * 32) grid = 148 * 32;
  cudaError_t e;
  if (logits_dtype == BOKT_BF16)
    e = launch(bokt::moe_topk_gate_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s,
               static_cast<const __nv_bfloat16*>(logits), tokens, E, k, renormalize, ids, gates);
  else if (logits_dtype == BOKT_FP16)
    e = launch(bokt::moe_topk_gate_kernel<__half>, dim3(grid), dim3(256), 0, s,
               static_cast<const __half*>(logits), tokens, E, k, renormalize, ids, gates);
  else if (logits_dtype == BOKT_FP32)
    e = launch(bokt::moe_topk_gate_kernel<float>, dim3(grid), dim3(256), 0, s,
               static_cast<const float*>(logits), tokens, E, k, renormalize, ids, gates);
  else
    return fail(BOKT_ERR_INVALID, "logits dtype %d", logits_dtype);
  if (e != cudaSuccess) return cuda_fail(e, "moe_topk_gate launch");
  return BOKT_OK;
}

int bokt_moe_combine(const void* y, int64_t y_rows, const int32_t* rows, const float* gates,
                     void* out, int tokens, int k, int N, int dtype, void* stream) {
  g_err[0] = 0;
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  if (tokens < 0 || k <= 0 || N < 0 || y_rows < 0) return fail(BOKT_ERR_INVALID, "bad size");
  if (tokens == 0 || N == 0) return BOKT_OK;
  if (!y || !gates || !out) return fail(BOKT_ERR_INVALID, "null pointer");
  if (N % 8 != 0 || !aligned16(y) || !aligned16(out))
    return fail(BOKT_ERR_UNSUPPORTED, "combine needs N %% 8 == 0 and 16-byte aligned rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = tokens < 148 * 64 ? tokens : 148 * 64;
  const int threads = N / 8 < 256 ? ((N / 8 + 31) / 32) * 32 : 256;
  cudaError_t e =
      dtype == BOKT_BF16
          ? launch(bokt::moe_combine_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), 0, s,
                   static_cast<const __nv_bfloat16*>(y), (long long)y_rows, rows, gates,
                   static_cast<__nv_bfloat16*>(out), tokens, k, N)
          : launch(bokt::moe_combine_kernel<__half>, dim3(grid), dim3(threads), 0, s,
                   static_cast<const __half*>(y), (long long)y_rows, rows, gates,
                   static_cast<__half*>(out), tokens, k, N);
  if (e != cudaSuccess) return cuda_fail(e, "moe_combine launch");
  return BOKT_OK;
}

int bokt_selftest_bounded_wait(int64_t timeout_ns, int* gave_up, void* stream) {
  g_err[0] = 0;
  if (timeout_ns <= 0 || timeout_ns > 10000000000ll || !gave_up)
    return fail(BOKT_ERR_INVALID, "timeout must be in (0, 10 s] and gave_up non-null");
  cudaError_t e = launch(bokt::selftest_bounded_wait_kernel, dim3(1), dim3(32), 0,
                         static_cast<cudaStream_t>(stream), uint64_t(timeout_ns), gave_up);
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return BOKT_OK;
}

int bokt_kernel_attrs(int kernel, int dtype, int n, int k, const bokt_params* params,
                      bokt_attrs* out) {
  g_err[0] = 0;
  if (!out) return fail(BOKT_ERR_INVALID, "null output");
  if (dtype != BOKT_FP16 && dtype != BOKT_BF16) return fail(BOKT_ERR_INVALID, "dtype %d", dtype);
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  const void* fn = nullptr;
  int dyn = 0, threads = 0, path = 0;
  if (kernel == BOKT_KERNEL_GEMM || kernel == BOKT_KERNEL_MOE_GROUPED_GEMM ||
      kernel == BOKT_KERNEL_RMSNORM_GEMM) {
    const bool grouped = kernel == BOKT_KERNEL_MOE_GROUPED_GEMM;
    const bool norm = kernel == BOKT_KERNEL_RMSNORM_GEMM;
    if ((n % 8) == 0 && (k % 8) == 0 && k > 0) {
      TcConfig cfg;
      rc = resolve_tc_config(params, grouped, grouped ? 64 : 0, dev.smem_optin, &cfg);
      if (rc) return rc;
      fn = cfg.cta_group == 2 ? tc2_kernel(dtype, cfg.bn, norm, grouped)
                              : tc_kernel(grouped, dtype, cfg.bn, false, norm);
      dyn = cfg.smem;
      threads = bokt::kGemmThreads;
      path = 0;
    } else if (norm) {
      return fail(BOKT_ERR_UNSUPPORTED, "fused RMSNorm-GEMM needs K and N multiples of 8");
    } else {
      fn = dtype == BOKT_BF16
               ? reinterpret_cast<const void*>(&bokt::gemm_tc_edge_kernel<__nv_bfloat16>)
               : reinterpret_cast<const void*>(&bokt::gemm_tc_edge_kernel<__half>);
      threads = bokt::kEdgeThreads;
      dyn = bokt::kEdgeSmemBytes;
      path = 1;
    }
  } else if (kernel == BOKT_KERNEL_RMSNORM) {
    NormConfig cfg;
    rc = resolve_norm_config(params, n, (n % 8) == 0, &cfg);
    if (rc) return rc;
    if (cfg.ring_slots < 0) {
      fn = dtype == BOKT_BF16 ? pipe_kernel<__nv_bfloat16>(cfg.vpt) : pipe_kernel<__half>(cfg.vpt);
      threads = cfg.threads;
      path = 5;
    } else if (cfg.ring_slots > 0) {
      fn = dtype == BOKT_BF16
               ? reinterpret_cast<const void*>(&bokt::rmsnorm_ring_kernel<__nv_bfloat16>)
               : reinterpret_cast<const void*>(&bokt::rmsnorm_ring_kernel<__half>);
      threads = cfg.threads + 32;
      dyn = bokt::rmsnorm_ring_smem_bytes(n, 2, cfg.ring_slots);
      path = 4;
    } else {
      fn = dtype == BOKT_BF16 ? norm_kernel<__nv_bfloat16>(cfg.vpt) : norm_kernel<__half>(cfg.vpt);
      threads = cfg.threads;
      path = cfg.vpt ? 2 : 3;
    }
  } else {
    return fail(BOKT_ERR_INVALID, "unknown kernel id %d", kernel);
  }
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, fn);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
  out->shared_bytes = int(a.sharedSizeBytes) + dyn;
  out->registers = a.numRegs;
  out->local_bytes = int(a.localSizeBytes);
  out->threads = threads;
  out->max_threads = a.maxThreadsPerBlock;
  out->path = path;
  return BOKT_OK;
}

int bokt_splitk_schedule(int ntiles, int split_k, int nkb, int launched, int32_t* out,
                         int capacity) {
  g_err[0] = 0;
  if (ntiles < 0 || split_k < 1 || nkb < 1 || launched < 1 || capacity < 0 || (!out && capacity))
    return -fail(BOKT_ERR_INVALID, "bad argument");
  const int split = split_k < nkb ? split_k : nkb;
  const int workers = bokt::splitk_workers(launched, ntiles, split);
  int n = 0;
  for (int w = 0; w < launched; ++w) {
    bokt::SegmentCursor cur = bokt::segment_cursor(w, workers, ntiles, split);
    bokt::Segment sg;
    while (bokt::segment_next(cur, split, nkb, sg)) {
      int first = 0, count = 0;
      if (split > 1 && sg.kb0 == 0 && sg.kb1 < nkb)
        count = bokt::splitk_contributors(w, workers, ntiles, split, sg.tile, &first);
      if (n < capacity) {
        int32_t* r = out + 6 * static_cast<int64_t>(n);
        r[0] = w;
        r[1] = sg.tile;
        r[2] = sg.kb0;
        r[3] = sg.kb1;
        r[4] = first;
        r[5] = count;
      }
      ++n;
    }
  }
  return n;
}

int bokt_splitk_reduce_sources(int ntiles, int split_k, int nkb, int launched, int32_t* out,
                               int capacity) {
  g_err[0] = 0;
  if (ntiles < 0 || split_k < 1 || nkb < 1 || launched < 1 || capacity < 0 || (!out && capacity))
    return -fail(BOKT_ERR_INVALID, "bad argument");
  const int split = split_k < nkb ? split_k : nkb;
  if (split <= 1) return 0;
  const int workers = bokt::splitk_workers(launched, ntiles, split);
  int n = 0;
  for (int t = 0; t < ntiles; ++t) {
    int wa, wb, first_which;
    bokt::splitk_tile_workers(t, split, workers, ntiles, &wa, &wb, &first_which);
    if (wb - wa < 2) continue;
    for (int w = wa; w < wb; ++w, ++n) {
      if (n >= capacity) continue;
      int32_t* r = out + 3 * static_cast<int64_t>(n);
      r[0] = t;
      r[1] = w;
      r[2] = w == wa ? first_which : 0;
    }
  }
  return n;
}

int bokt_device_status(int* code, int* detail, int reset) {
  g_err[0] = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int h[2] = {0, 0};
  e = cudaMemcpyFromSymbol(h, bokt::g_status, sizeof(h));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status)");
  if (code) *code = h[0];
  if (detail) *detail = h[1];
  if (reset) {
    const int z[2] = {0, 0};
    e = cudaMemcpyToSymbol(bokt::g_status, z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status)");
  }
  return BOKT_OK;
}

}  // extern "C"

// =================================================================== allocation-free routing
// bokt_moe_route_noalloc: the routing front end for callers that cannot call
// cudaMalloc (or any allocator) at all.  The per-chunk expert table that
// bokt_moe_route keeps in a caller-provided workspace lives here in a fixed
// device array instead, which every GPU that loads this library holds until
// the process exits.  Host code never dereferences or passes the array's name
// to a kernel: in host code that name is only a host-side stand-in, so the
// device address is looked up with cudaGetSymbolAddress once per device.
namespace {

// chunks * experts int32 words, chunks = ceil(assignments / 4096).
constexpr int64_t kRouteScratchWords = 64 * 1024;  // 256 KiB

static __device__ __align__(256) int32_t g_route_scratch[kRouteScratchWords];

// Resolved device address per device, with the context it was resolved in: a
// different current context (after cudaDeviceReset, or a user-created
// context) loads its own copy of the module, so the address is looked up
// again rather than reusing one from a context that may be gone.
struct ScratchAddr {
  CUcontext ctx;
  int32_t* ptr;
};
ScratchAddr g_route_scratch_addr[kMaxDevices] = {};
std::mutex g_route_scratch_mu;
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
std::once_flag g_ctx_current_once;

// Device address of g_route_scratch in the current device's current context,
// resolved on the first call in that context (that first call must not be
// inside stream capture).
int route_scratch(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(BOKT_ERR_UNSUPPORTED, "device index %d", dev);
  std::call_once(g_ctx_current_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  });
  if (!g_ctx_current) return fail(BOKT_ERR_CUDA, "cuCtxGetCurrent entry point unavailable");
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS) return fail(BOKT_ERR_CUDA, "cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lock(g_route_scratch_mu);
  ScratchAddr& slot = g_route_scratch_addr[dev];
  if (!ctx || !slot.ptr || slot.ctx != ctx) {
    // Also makes the device's primary context current when none is yet.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_route_scratch)");
    if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx)
      return fail(BOKT_ERR_CUDA, "no current CUDA context");
    slot.ctx = ctx;
    slot.ptr = static_cast<int32_t*>(p);
  }
  *out = slot.ptr;
  return BOKT_OK;
}

}  // namespace

extern "C" int64_t bokt_moe_route_noalloc_max_words(void) { return kRouteScratchWords; }

extern "C" int bokt_moe_route_noalloc(const int32_t* expert_ids, int A, int E, int32_t* counts,
                                      int32_t* offsets, int64_t* offsets64, int32_t* perm,
                                      int32_t* inv_perm, void* stream) {
  g_err[0] = 0;
  if (A < 0 || E <= 0) return fail(BOKT_ERR_INVALID, "need A >= 0 and E > 0");
  if (E > bokt::kRouteMaxExperts)
    return fail(BOKT_ERR_UNSUPPORTED, "at most %d experts", bokt::kRouteMaxExperts);
  if (!counts || !offsets || (A > 0 && (!expert_ids || !perm || !inv_perm)))
    return fail(BOKT_ERR_INVALID, "null pointer");
  const int64_t words = bokt_moe_route_workspace_bytes(A, E) / 4;
  if (words > kRouteScratchWords)
    return fail(BOKT_ERR_UNSUPPORTED,
                "bokt_moe_route_noalloc: ceil(A/4096) * E = %lld scratch words exceeds the fixed "
                "%lld-word device array (A=%d, E=%d); use bokt_moe_route with a workspace",
                (long long)words, (long long)kRouteScratchWords, A, E);
  int32_t* scratch = nullptr;
  int rc = route_scratch(&scratch);
  if (rc) return rc;
  // Same kernels as bokt_moe_route.  route_count overwrites every scratch word
  // the later launches read, so no clearing is needed between calls.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return launch_route(expert_ids, A, E, scratch, counts, offsets, offsets64, perm, inv_perm, s,
                      "moe_route_noalloc launch");
}
