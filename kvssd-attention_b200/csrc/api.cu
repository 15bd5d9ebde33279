// C ABI of libkvssd_b200: argument validation, launch planning and kernel dispatch.
//
// Validation mirrors the reference's checks so a caller sees the same refusals:
// PackedBatch.validate (src/kvssd/backends/base.py:29-55), the op bindings
// (csrc/bindings.cpp:26-38) and the kernel launcher (csrc/fused_decode.cu:117-121).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kvssd_b200.h"
#include "common.cuh"
#include "decode.cuh"
#include "records.cuh"

namespace kvb {

using DecodeKernel = void (*)(const DecodeArgs);
DecodeKernel tc_decode_kernel_for(int bits, int d, int group);
DecodeKernel simt_decode_kernel_for(int d);
DecodeKernel async_decode_kernel_for(int bits, int d, int group, int kvh, bool batched);
int async_threads();
int async_warps();
int async_depth();
int async_stage_bytes(int group);
bool tma_decode_supported(int bits, int d, int group, int kvh, int bt);
size_t tma_decode_smem(int kvh, int group, int bits);
int tma_decode_threads(int kvh, int group);
cudaError_t launch_tma_decode(const DecodeArgs& a, int n_splits, cudaStream_t s);
using DequantKernel = void (*)(const uint8_t*, const __half*, long long, int, int, __half*,
                               uint8_t*);
DequantKernel dequant_kernel_for(int bits, int mode);

__global__ void combine_parts_kernel(const float*, const float*, int, int, int, float*, float*,
                                     const unsigned*);
__global__ void merge_chunks_kernel(const float*, const float*, int, int, int, float*, float*);
__global__ void merge_pair_kernel(const float*, const float*, const float*, const float*, int,
                                  int, float*, float*);
constexpr int kCombineThreads = 512;  // 32 * kCombineWarps in combine.cu

namespace {

thread_local std::string g_last_error;
int g_path_override = KVSSD_B200_PATH_AUTO;

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(KVSSD_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Workspace: a 2048-byte header, then the split-KV parts. The caller zeroes the whole
// workspace once after allocating it. Header: the device status word (byte 0) and the fused
// combine's words (byte 128): the epoch of the last call, the test hook (zero in use) and the
// batched combiners' counter (zero between calls). With the fused combine every part value is
// a tagged 64-bit word {f32 value, epoch tag} (combine.cuh), so the parts take 8 bytes a value;
// the separate combine launch reads the same region as plain f32.
constexpr size_t kHeaderBytes = 2048;
constexpr size_t kTicketOffset = 128;
constexpr int kMaxParts = 8192;       // bound on split-KV parts

struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;
};

DeviceInfo device_info(int dev) {
  static std::mutex mu;
  static std::vector<DeviceInfo> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1);
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                           dev);
    if (cache[dev].sms <= 0) cache[dev].sms = 148;
  }
  return cache[dev];
}

int occupancy(DecodeKernel k, int threads) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<void*, int>, int>> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : cache)
    if (e.first.first == reinterpret_cast<void*>(k) && e.first.second == threads) return e.second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, 0) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 1;
  }
  cache.push_back({{reinterpret_cast<void*>(k), threads}, n});
  return n;
}

struct Geometry {
  int n_sel, bt, qh, kvh, d, bits, group;
};

// Geometry checks common to all entry points (bits, packing, GQA divisibility).
int check_geometry(const Geometry& g) {
  if (g.bits != 2 && g.bits != 4) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bits must be 2 or 4");
  if (g.n_sel < 1) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "at least one block is required");
  if (g.bt < 1 || g.qh < 1 || g.kvh < 1 || g.d < 1 || g.group < 1)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "all dimensions must be positive");
  if (g.d % g.group) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "group_size must divide head_dim");
  if ((static_cast<long long>(g.d) * g.bits) % 8)  // wide: head_dim is not yet bounded here
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "packed dimension does not match query head dimension");
  if (g.group % (8 / g.bits))
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "group_size must be positive and pack-aligned");
  if (g.qh % g.kvh) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "query heads must be divisible by KV heads");
  if (g.d > 256) return fail(KVSSD_B200_ERR_UNSUPPORTED, "head_dim > 256 is not supported");
  return KVSSD_B200_OK;
}

struct Plan {
  int path = 0;
  bool streaming = false;  // streaming kernel (fused combine): TMA-fed or cp.async-fed
  bool tma = false;        // streaming kernel fed by TMA copies into a CTA ring
  size_t smem = 0;
  DecodeKernel kernel = nullptr;
  int gqa = 0, n_qsub = 0, n_vheads = 0, heads_per_cta = 0, wph = 0, n_head_groups = 0;
  int threads = 0, n_splits = 0, n_parts = 0, tiles_per_block = 0;
  long long total_tiles = 0;
  size_t ws_bytes = 0;
};

int choose_path(int d, int bits, int group) {
  const bool tc_ok = tc_decode_kernel_for(bits, d, group) != nullptr;
  if (g_path_override == KVSSD_B200_PATH_GENERIC) return KVSSD_B200_PATH_GENERIC;
  if (g_path_override == KVSSD_B200_PATH_TENSOR_CORE ||
      g_path_override == KVSSD_B200_PATH_TENSOR_CORE_REGS ||
      g_path_override == KVSSD_B200_PATH_TENSOR_CORE_CPASYNC)
    return tc_ok ? KVSSD_B200_PATH_TENSOR_CORE : -1;
  return tc_ok ? KVSSD_B200_PATH_TENSOR_CORE : KVSSD_B200_PATH_GENERIC;
}


// Streaming kernel choice and shared memory; false if the geometry does not qualify (INT4,
// head_dim 128, group 32 or 64, KV heads dividing the 16 warps, at most 8 query heads per KV
// head). The TMA-fed kernel is preferred (KV heads 4, 8 or 16, block_tokens a multiple of 16,
// token rows of the pool addressable by 32-bit TMA coordinates: pool_rows < 2^31, 0 when
// unknown); otherwise the per-warp cp.async rings.
bool plan_streaming(const Geometry& g, const DeviceInfo& info, Plan& p, bool allow_tma,
                    long long pool_rows) {
  p.tma = false;
  if (g.d != 128 || p.n_qsub != 1 || async_warps() % g.kvh) return false;
  const size_t merge_bytes = static_cast<size_t>(async_warps() - g.kvh) * 32 * (4 + 4 * (g.d / 16)) * 4;
  const size_t max_smem = static_cast<size_t>(info.max_smem_optin) - 1024;
  if (allow_tma && g_path_override != KVSSD_B200_PATH_TENSOR_CORE_CPASYNC &&
      pool_rows < (1LL << 31) && tma_decode_supported(g.bits, g.d, g.group, g.kvh, g.bt)) {
    const size_t smem = tma_decode_smem(g.kvh, g.group, g.bits);
    if (smem <= max_smem && merge_bytes + 1024 <= smem) {
      p.tma = true;
      p.kernel = nullptr;
      p.smem = smem;
      return true;
    }
  }
  p.kernel = async_decode_kernel_for(g.bits, g.d, g.group, g.kvh, false);
  if (p.kernel == nullptr) return false;
  p.smem = static_cast<size_t>(async_warps()) * async_depth() * async_stage_bytes(g.group);
  return p.smem <= max_smem && merge_bytes <= p.smem;
}

// aligned: packed K/V 16-byte aligned; allow_stream: scales 16-byte aligned as well;
// pool_rows: n_pool_blocks * block_tokens (0 when unknown).
int make_plan(const Geometry& g, bool aligned, bool allow_stream, Plan& p,
              long long pool_rows = 0) {
  int st = check_geometry(g);
  if (st) return st;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const DeviceInfo info = device_info(dev);
  p.path = choose_path(g.d, g.bits, g.group);
  if (p.path < 0)
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "tensor-core path forced for an unsupported shape");
  if (p.path == KVSSD_B200_PATH_TENSOR_CORE && !aligned) {
    if (g_path_override == KVSSD_B200_PATH_TENSOR_CORE)
      return fail(KVSSD_B200_ERR_UNSUPPORTED, "tensor-core path needs 16-byte aligned packed KV");
    p.path = KVSSD_B200_PATH_GENERIC;
  }
  p.gqa = g.qh / g.kvh;
  p.n_qsub = (p.gqa + 7) / 8;
  p.n_vheads = g.kvh * p.n_qsub;
  if (p.path == KVSSD_B200_PATH_TENSOR_CORE && aligned && allow_stream &&
      g_path_override != KVSSD_B200_PATH_TENSOR_CORE_REGS &&
      plan_streaming(g, info, p, true, pool_rows)) {
    p.streaming = true;
    p.heads_per_cta = g.kvh;
    p.wph = async_warps() / g.kvh;
  } else if (p.path == KVSSD_B200_PATH_TENSOR_CORE) {
    p.kernel = tc_decode_kernel_for(g.bits, g.d, g.group);
    p.heads_per_cta = std::min(p.n_vheads, 8);
    p.wph = 8 / p.heads_per_cta;
  } else {
    p.kernel = simt_decode_kernel_for(g.d);
    p.heads_per_cta = 1;
    p.wph = 4;
  }
  p.threads = p.streaming ? (p.tma ? tma_decode_threads(g.kvh, g.group) : async_threads())
                          : 32 * p.heads_per_cta * p.wph;
  p.n_head_groups = (p.n_vheads + p.heads_per_cta - 1) / p.heads_per_cta;
  p.tiles_per_block = (g.bt + 15) / 16;
  p.total_tiles = static_cast<long long>(g.n_sel) * p.tiles_per_block;
  const long long resident =
      p.streaming ? info.sms
            : static_cast<long long>(info.sms) * occupancy(p.kernel, p.threads) / p.n_head_groups;
  const long long by_work = (p.total_tiles + 2 * p.wph - 1) / (2 * p.wph);
  long long splits = std::max(1LL, std::min(resident, by_work));
  if (p.streaming && splits > 32) {
    // The fused combine folds one (query head, 32-dim) slice per combining CTA with all of the
    // CTA's warps (above 32 parts); with fewer CTAs than slices a CTA folds several in turn,
    // ~2.5 us each. So the grid gets at least one CTA per slice where the SMs allow it (CTAs
    // past the work write empty parts).
    const long long n_slices = static_cast<long long>(g.qh) * ((g.d + 31) / 32);
    splits = std::min(resident, std::max(splits, n_slices));
  }
  const int parts_per_split = p.streaming ? 1 : p.wph;  // merged in-CTA by the streaming kernel
  splits = std::min<long long>(splits, kMaxParts / parts_per_split);
  p.n_splits = static_cast<int>(splits);
  p.n_parts = p.n_splits * parts_per_split;
  const size_t part_values = static_cast<size_t>(p.n_parts) * g.qh * (g.d + 2);
  p.ws_bytes = kHeaderBytes + part_values * sizeof(unsigned long long);
  return KVSSD_B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch_combine(const float* part_acc, const float* part_ml, int n_parts, int qh, int d,
                           float* out, float* lse, const unsigned* status, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(qh, (d + 31) / 32, 1);
  cfg.blockDim = dim3(kCombineThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_parts_kernel, part_acc, part_ml, n_parts, qh, d, out,
                            lse, status);
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" {

int kvssd_b200_version(void) { return 1; }

const char* kvssd_b200_status_string(int status) {
  switch (status) {
    case KVSSD_B200_OK: return "ok";
    case KVSSD_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case KVSSD_B200_ERR_UNSUPPORTED: return "unsupported";
    case KVSSD_B200_ERR_WORKSPACE: return "workspace too small";
    case KVSSD_B200_ERR_CUDA: return "CUDA error";
    case KVSSD_B200_ERR_DEVICE_STATUS:
      return "device flagged invalid block-table or valid_tokens entries, or a combine timeout";
    default: return "unknown status";
  }
}

const char* kvssd_b200_last_error(void) { return g_last_error.c_str(); }

int kvssd_b200_decode_workspace_size(int n_sel_blocks, int block_tokens, int query_heads,
                                     int kv_heads, int head_dim, int bits, int group_size,
                                     size_t* bytes) {
  if (!bytes) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  // Large enough for every kernel the geometry may dispatch to (operand alignment decides).
  const Geometry g{n_sel_blocks, block_tokens, query_heads, kv_heads, head_dim, bits, group_size};
  size_t need = 0;
  for (int variant = 0; variant < 3; ++variant) {
    Plan p;
    const int st = make_plan(g, variant < 2, variant == 0, p);
    if (st == KVSSD_B200_ERR_UNSUPPORTED && variant > 0) continue;  // forced path: aligned only
    if (st) return st;
    need = std::max(need, p.ws_bytes);
  }
  *bytes = need;
  return KVSSD_B200_OK;
}

int kvssd_b200_decode_path(int head_dim, int bits, int group_size, int* path) {
  if (!path) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "path must not be NULL");
  const int p = choose_path(head_dim, bits, group_size);
  if (p < 0) return fail(KVSSD_B200_ERR_UNSUPPORTED, "tensor-core path forced for an unsupported shape");
  *path = p;
  return KVSSD_B200_OK;
}

int kvssd_b200_decode_plan(int n_sel_blocks, int block_tokens, int query_heads, int kv_heads,
                           int head_dim, int bits, int group_size, int* kernel, int* n_splits,
                           int* n_parts) {
  if (!kernel || !n_splits || !n_parts) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  const Geometry g{n_sel_blocks, block_tokens, query_heads, kv_heads, head_dim, bits, group_size};
  Plan p;
  const int st = make_plan(g, true, true, p);
  if (st) return st;
  *kernel = p.path == KVSSD_B200_PATH_GENERIC ? KVSSD_B200_PATH_GENERIC
            : p.tma                              ? KVSSD_B200_PATH_TENSOR_CORE
            : p.streaming                        ? KVSSD_B200_PATH_TENSOR_CORE_CPASYNC
                                                 : KVSSD_B200_PATH_TENSOR_CORE_REGS;
  *n_splits = p.n_splits;
  *n_parts = p.n_parts;
  return KVSSD_B200_OK;
}

int kvssd_b200_set_path_override(int path) {
  if (path < KVSSD_B200_PATH_AUTO || path > KVSSD_B200_PATH_TENSOR_CORE_CPASYNC)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "unknown path");
  g_path_override = path;
  return KVSSD_B200_OK;
}

}  // extern "C"

namespace kvb {
namespace {

// Validates a decode call and fills the kernel arguments and launch plan.
int prepare_decode(const void* query, int query_dtype, const uint8_t* packed_k,
                   const uint8_t* packed_v, const uint16_t* scales_k, const uint16_t* scales_v,
                   const int32_t* valid_tokens, const int32_t* block_table, int n_pool_blocks,
                   int n_sel_blocks, int block_tokens, int query_heads, int kv_heads,
                   int head_dim, int bits, int group_size, float sm_scale, void* workspace,
                   size_t workspace_bytes, DecodeArgs& a, Plan& p) {
  if (!query || !packed_k || !packed_v || !scales_k || !scales_v || !valid_tokens)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "tensor pointers must not be NULL");
  if (query_dtype < KVSSD_B200_Q_F32 || query_dtype > KVSSD_B200_Q_F64)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "unknown query dtype");
  if (n_pool_blocks < 1) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "block pool is empty");
  if (!block_table && n_sel_blocks > n_pool_blocks)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "more selected blocks than pool blocks");
  if (!std::isfinite(sm_scale)) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "sm_scale must be finite");
  if ((reinterpret_cast<uintptr_t>(scales_k) | reinterpret_cast<uintptr_t>(scales_v)) & 1u)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "scales must be 2-byte aligned");
  const Geometry g{n_sel_blocks, block_tokens, query_heads, kv_heads, head_dim, bits, group_size};
  int st = make_plan(g, aligned16(packed_k) && aligned16(packed_v),
                     aligned16(scales_k) && aligned16(scales_v), p,
                     static_cast<long long>(n_pool_blocks) * block_tokens);
  if (st) return st;
  if (!workspace || workspace_bytes < p.ws_bytes)
    return fail(KVSSD_B200_ERR_WORKSPACE, "workspace needs " + std::to_string(p.ws_bytes) + " bytes");
  if (reinterpret_cast<uintptr_t>(workspace) & 15u)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  a.q = query;
  a.q_dtype = query_dtype;
  a.kp = packed_k;
  a.vp = packed_v;
  a.ks = reinterpret_cast<const __half*>(scales_k);
  a.vs = reinterpret_cast<const __half*>(scales_v);
  a.valid = valid_tokens;
  a.table = block_table;
  a.n_pool = n_pool_blocks;
  a.n_sel = n_sel_blocks;
  a.bt = block_tokens;
  a.qh = query_heads;
  a.kvh = kv_heads;
  a.d = head_dim;
  a.bits = bits;
  a.group = group_size;
  a.gqa = p.gqa;
  a.n_qsub = p.n_qsub;
  a.n_vheads = p.n_vheads;
  a.heads_per_cta = p.heads_per_cta;
  a.wph = p.wph;
  a.tiles_per_block = p.tiles_per_block;
  a.total_tiles = p.total_tiles;
  a.n_splits = p.n_splits;
  a.score_scale = sm_scale * 1.4426950408889634f;  // log2(e): scores kept in log2 units
  char* ws = static_cast<char*>(workspace);
  a.status = reinterpret_cast<unsigned*>(ws);
  a.part_epoch = reinterpret_cast<unsigned*>(ws + kTicketOffset);
  a.fuse_combine = 0;
  a.out = nullptr;
  a.lse = nullptr;
  a.xworld = 0;
  a.xrank = 0;
  for (int r = 0; r < kMaxExchangeRanks; ++r) a.xpeers[r] = nullptr;
  a.part_ml = reinterpret_cast<float*>(ws + kHeaderBytes);
  a.part_acc = a.part_ml + static_cast<size_t>(p.n_parts) * query_heads * 2;
  a.tpart_acc = reinterpret_cast<unsigned long long*>(ws + kHeaderBytes) +
                static_cast<size_t>(p.n_parts) * query_heads * 2;
  return KVSSD_B200_OK;
}

int launch_split(DecodeArgs& a, const Plan& p, cudaStream_t s);

// The whole decode: the streaming kernel folds its parts itself (fused combine, cooperative
// launch); the other kernels, or a refused cooperative launch, are followed by the combine
// kernel.
int launch_decode(DecodeArgs& a, const Plan& p, float* out, float* lse, cudaStream_t s) {
  if (p.streaming) {
    a.fuse_combine = 1;
    a.out = out;
    a.lse = lse;
    const int st = launch_split(a, p, s);
    if (st == KVSSD_B200_OK || a.fuse_combine) return st;
    // cooperative launch refused (a.fuse_combine cleared): two-launch path below
  }
  int st = launch_split(a, p, s);
  if (st) return st;
  cudaError_t e = launch_combine(a.part_acc, a.part_ml, p.n_parts, a.qh, a.d, out, lse, a.status, s);
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "combine launch");
}

// Raises a kernel's dynamic shared-memory limit (static + dynamic above the 48 KB default
// needs the opt-in) once per (device, kernel, size), not on every launch.
cudaError_t ensure_dynamic_smem(DecodeKernel kernel, size_t bytes) {
  if (bytes <= 16 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, const void*>, size_t>> done;
  std::lock_guard<std::mutex> lock(mu);
  const void* key = reinterpret_cast<const void*>(kernel);
  for (const auto& d : done)
    if (d.first.first == dev && d.first.second == key && d.second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
  if (e == cudaSuccess) done.push_back({{dev, key}, bytes});
  return e;
}

int launch_split(DecodeArgs& a, const Plan& p, cudaStream_t s) {
  if (p.tma) {
    // TMA-fed streaming kernel: programmatic stream serialization, cooperative with the fused
    // combine (as below).
    cudaError_t e = launch_tma_decode(a, p.n_splits, s);
    if (e == cudaErrorCooperativeLaunchTooLarge && a.fuse_combine) {
      cudaGetLastError();
      a.fuse_combine = 0;
      return KVSSD_B200_ERR_UNSUPPORTED;
    }
    return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "TMA decode launch");
  }
  {
    cudaError_t e = ensure_dynamic_smem(p.kernel, p.smem);
    if (e != cudaSuccess) return cuda_fail(e, "shared-memory attribute");
  }
  if (!p.streaming) {
    p.kernel<<<dim3(p.n_splits, p.n_head_groups, 1), dim3(p.threads, 1, 1), p.smem, s>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "decode launch");
  }
  // Streaming kernel: programmatic stream serialization (it waits for the preceding grid
  // itself) and, with the fused combine, a cooperative launch so its CTAs are co-resident.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_splits, p.n_head_groups, 1);
  cfg.blockDim = dim3(p.threads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.fuse_combine ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, p.kernel, a);
  if (e == cudaErrorCooperativeLaunchTooLarge && a.fuse_combine) {
    cudaGetLastError();  // not sticky: fall back to the two-launch decode
    a.fuse_combine = 0;
    return KVSSD_B200_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "decode launch");
}

}  // namespace
}  // namespace kvb

extern "C" {

int kvssd_b200_decode(const void* query, int query_dtype, const uint8_t* packed_k,
                      const uint8_t* packed_v, const uint16_t* scales_k,
                      const uint16_t* scales_v, const int32_t* valid_tokens,
                      const int32_t* block_table, int n_pool_blocks, int n_sel_blocks,
                      int block_tokens, int query_heads, int kv_heads, int head_dim, int bits,
                      int group_size, float sm_scale, float* out, float* lse, void* workspace,
                      size_t workspace_bytes, kvssd_b200_stream_t stream) {
  if (!out || !lse) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "tensor pointers must not be NULL");
  DecodeArgs a;
  Plan p;
  int st = prepare_decode(query, query_dtype, packed_k, packed_v, scales_k, scales_v, valid_tokens,
                          block_table, n_pool_blocks, n_sel_blocks, block_tokens, query_heads,
                          kv_heads, head_dim, bits, group_size, sm_scale, workspace,
                          workspace_bytes, a, p);
  if (st) return st;
  return launch_decode(a, p, out, lse, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace kvb {
namespace {

// Scratch of kvssd_b200_decode_static. A __device__ variable exists once per device context
// that loads this module; no initializer, so nothing is embedded in the binary.
__device__ __align__(256) unsigned char g_static_scratch[KVSSD_B200_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchSlot {
  unsigned long long context = 0;  // driver context id the address belongs to (0: none yet)
  void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];

// Unique id of the calling thread's current driver context (cuCtxGetCurrent + cuCtxGetId,
// resolved once through the runtime, so the library needs no link against libcuda). A device
// reset or a new primary context gives a new id; 0 when it cannot be determined.
unsigned long long current_context_id() {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static const std::pair<GetCurrentFn, GetIdFn> fns = [] {
    void* cur = nullptr;
    void* id = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &cur, 12000, cudaEnableDefault, &q) !=
            cudaSuccess || q != cudaDriverEntryPointSuccess)
      cur = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &id, 12000, cudaEnableDefault, &q) !=
            cudaSuccess || q != cudaDriverEntryPointSuccess)
      id = nullptr;
    return std::make_pair(reinterpret_cast<GetCurrentFn>(cur), reinterpret_cast<GetIdFn>(id));
  }();
  if (!fns.first || !fns.second) return 0;
  CUcontext ctx = nullptr;
  unsigned long long ident = 0;
  if (fns.first(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (fns.second(ctx, &ident) != CUDA_SUCCESS) return 0;
  return ident;
}

// Address of the current device's scratch. The first call per device and context resolves
// the symbol (with the device current) and zeroes the scratch on `s`; a later context
// on the same device (after cudaDeviceReset) is a fresh module instance and is set up again.
int static_scratch(cudaStream_t s, void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "static scratch supports device ordinals below 64");
  // The runtime binds the device's primary context to this thread on its first call above.
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchSlot& slot = g_scratch[dev];
  if (slot.ptr == nullptr || ctx == 0 || slot.context != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "static scratch address");
    if (slot.ptr == nullptr || slot.context != ctx || p != slot.ptr) {
      e = cudaMemsetAsync(p, 0, KVSSD_B200_STATIC_SCRATCH_BYTES, s);  // header and part tags
      if (e != cudaSuccess) return cuda_fail(e, "static scratch clear");
    }
    slot.ptr = p;
    slot.context = ctx;
  }
  *ptr = slot.ptr;
  return KVSSD_B200_OK;
}

}  // namespace
}  // namespace kvb

extern "C" {

int kvssd_b200_decode_static(const void* query, int query_dtype, const uint8_t* packed_k,
                             const uint8_t* packed_v, const uint16_t* scales_k,
                             const uint16_t* scales_v, const int32_t* valid_tokens,
                             const int32_t* block_table, int n_pool_blocks, int n_sel_blocks,
                             int block_tokens, int query_heads, int kv_heads, int head_dim,
                             int bits, int group_size, float sm_scale, float* out, float* lse,
                             void** scratch, kvssd_b200_stream_t stream) {
  if (!out || !lse) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "tensor pointers must not be NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  int st = static_scratch(s, &ws);
  if (st) return st;
  if (scratch) *scratch = ws;
  DecodeArgs a;
  Plan p;
  st = prepare_decode(query, query_dtype, packed_k, packed_v, scales_k, scales_v, valid_tokens,
                      block_table, n_pool_blocks, n_sel_blocks, block_tokens, query_heads,
                      kv_heads, head_dim, bits, group_size, sm_scale, ws,
                      KVSSD_B200_STATIC_SCRATCH_BYTES, a, p);
  if (st == KVSSD_B200_ERR_WORKSPACE)
    return fail(st, "this geometry needs " + std::to_string(p.ws_bytes) +
                        " bytes of scratch; the static scratch holds " +
                        std::to_string(KVSSD_B200_STATIC_SCRATCH_BYTES) +
                        " (use kvssd_b200_decode with a caller workspace)");
  if (st) return st;
  return launch_decode(a, p, out, lse, s);
}

int kvssd_b200_decode_split(const void* query, int query_dtype, const uint8_t* packed_k,
                            const uint8_t* packed_v, const uint16_t* scales_k,
                            const uint16_t* scales_v, const int32_t* valid_tokens,
                            const int32_t* block_table, int n_pool_blocks, int n_sel_blocks,
                            int block_tokens, int query_heads, int kv_heads, int head_dim,
                            int bits, int group_size, float sm_scale, void* workspace,
                            size_t workspace_bytes, int* n_parts, kvssd_b200_stream_t stream) {
  if (!n_parts) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "n_parts must not be NULL");
  DecodeArgs a;
  Plan p;
  int st = prepare_decode(query, query_dtype, packed_k, packed_v, scales_k, scales_v, valid_tokens,
                          block_table, n_pool_blocks, n_sel_blocks, block_tokens, query_heads,
                          kv_heads, head_dim, bits, group_size, sm_scale, workspace,
                          workspace_bytes, a, p);
  if (st) return st;
  *n_parts = p.n_parts;
  return launch_split(a, p, reinterpret_cast<cudaStream_t>(stream));
}

int kvssd_b200_decode_combine(const void* workspace, int n_parts, int query_heads, int head_dim,
                              float* out, float* lse, kvssd_b200_stream_t stream) {
  if (!workspace || !out || !lse) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (n_parts < 1 || n_parts > kMaxParts || query_heads < 1 || head_dim < 1 || head_dim > 256)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bad part geometry");
  const float* ml = reinterpret_cast<const float*>(static_cast<const char*>(workspace) + kHeaderBytes);
  const float* acc = ml + static_cast<size_t>(n_parts) * query_heads * 2;
  cudaError_t e = launch_combine(acc, ml, n_parts, query_heads, head_dim, out, lse,
                                 static_cast<const unsigned*>(workspace),
                                 reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "combine launch");
}

int kvssd_b200_exchange_bytes(int world, int query_heads, int head_dim, size_t* bytes) {
  if (!bytes) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  if (world < 1 || world > kMaxExchangeRanks)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "exchange supports 1 to 8 ranks");
  if (query_heads < 1 || head_dim < 1 || head_dim > 256)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bad exchange geometry");
  *bytes = exchange_bytes(world, query_heads * ((head_dim + 31) / 32));
  return KVSSD_B200_OK;
}

int kvssd_b200_exchange_alloc(size_t bytes, void** buffer) {
  if (!buffer || bytes == 0) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bad exchange buffer request");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "exchange buffer allocation");
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "exchange buffer clear");
  }
  *buffer = p;
  return KVSSD_B200_OK;
}

int kvssd_b200_exchange_clear(void* buffer, size_t bytes) {
  if (!buffer) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  cudaError_t e = cudaMemset(buffer, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "exchange buffer clear");
}

int kvssd_b200_exchange_free(void* buffer) {
  cudaError_t e = cudaFree(buffer);
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "exchange buffer free");
}

int kvssd_b200_ipc_handle(void* buffer, void* handle) {
  if (!buffer || !handle) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, buffer);
  if (e != cudaSuccess) return cuda_fail(e, "IPC handle");
  static_assert(sizeof(h) == KVSSD_B200_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return KVSSD_B200_OK;
}

int kvssd_b200_ipc_open(const void* handle, void** buffer) {
  if (!buffer || !handle) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "IPC open");
}

int kvssd_b200_ipc_close(void* buffer) {
  cudaError_t e = cudaIpcCloseMemHandle(buffer);
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "IPC close");
}

int kvssd_b200_decode_exchange(const void* query, int query_dtype, const uint8_t* packed_k,
                               const uint8_t* packed_v, const uint16_t* scales_k,
                               const uint16_t* scales_v, const int32_t* valid_tokens,
                               const int32_t* block_table, int n_pool_blocks, int n_sel_blocks,
                               int block_tokens, int query_heads, int kv_heads, int head_dim,
                               int bits, int group_size, float sm_scale, int rank, int world,
                               void* const* buffers, float* out, float* lse,
                               void* workspace, size_t workspace_bytes,
                               kvssd_b200_stream_t stream) {
  if (!out || !lse || !buffers)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if (world < 1 || world > kMaxExchangeRanks || rank < 0 || rank >= world)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "rank/world outside 1 to 8 ranks");
  for (int r = 0; r < world; ++r)
    if (!buffers[r] || (reinterpret_cast<uintptr_t>(buffers[r]) & 15u))
      return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "exchange buffers must be 16-byte aligned");
  DecodeArgs a;
  Plan p;
  int st = prepare_decode(query, query_dtype, packed_k, packed_v, scales_k, scales_v, valid_tokens,
                          block_table, n_pool_blocks, n_sel_blocks, block_tokens, query_heads,
                          kv_heads, head_dim, bits, group_size, sm_scale, workspace,
                          workspace_bytes, a, p);
  if (st) return st;
  if (!p.streaming)
    return fail(KVSSD_B200_ERR_UNSUPPORTED,
                "the fused exchange needs a streaming kernel (INT4 or INT2 with 4/8/16 KV heads, "
                "head_dim 128, group 32/64, 16-byte aligned operands)");
  a.xworld = world;
  a.xrank = rank;
  for (int r = 0; r < world; ++r) a.xpeers[r] = static_cast<uint8_t*>(buffers[r]);
  a.fuse_combine = 1;
  a.out = out;
  a.lse = lse;
  st = launch_split(a, p, reinterpret_cast<cudaStream_t>(stream));
  if (st == KVSSD_B200_ERR_UNSUPPORTED)
    return fail(st, "the fused exchange needs a cooperative launch of the whole grid");
  return st;
}

int kvssd_b200_decode_records(const uint8_t* records, size_t record_stride, int n_records,
                              int layer, const int32_t* expected_blocks, int bits,
                              int block_tokens, int kv_heads, int head_dim, int group_size,
                              uint8_t* packed_k, uint8_t* packed_v, uint16_t* scales_k,
                              uint16_t* scales_v, int32_t* valid_tokens, unsigned* record_status,
                              kvssd_b200_stream_t stream) {
  if (n_records < 0) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "n_records must be >= 0");
  if (n_records == 0) return KVSSD_B200_OK;
  if (!records || !packed_k || !packed_v || !scales_k || !scales_v || !valid_tokens ||
      !record_status)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if ((bits != 2 && bits != 4) || block_tokens < 1 || kv_heads < 1 || head_dim < 1 ||
      group_size < 1 || head_dim % group_size || (head_dim * bits) % 8)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bad cache geometry");
  if ((reinterpret_cast<uintptr_t>(records) | record_stride) & 3u)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "records must be 4-byte aligned");
  for (const void* p : {static_cast<const void*>(valid_tokens),
                        static_cast<const void*>(record_status)})
    if (reinterpret_cast<uintptr_t>(p) & 3u)
      return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "valid_tokens/status must be 4-byte aligned");
  const long long rows = static_cast<long long>(block_tokens) * kv_heads;
  const long long scale_bytes = rows * (head_dim / group_size) * 2;
  const long long packed_bytes = rows * (head_dim * bits / 8);
  if (scale_bytes > (1LL << 30) || packed_bytes > (1LL << 30))
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "record sections above 1 GiB");
  const long long payload = 2 * scale_bytes + 2 * packed_bytes;
  if (static_cast<long long>(record_stride) < kRecHeaderBytes + payload)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "record stride smaller than header + payload");
  RecordArgs a{};
  a.records = records;
  a.stride = record_stride;
  a.n = n_records;
  a.layer = layer;
  a.blocks = expected_blocks;
  a.bits = bits;
  a.bt = block_tokens;
  a.kvh = kv_heads;
  a.d = head_dim;
  a.group = group_size;
  a.scale_bytes = static_cast<int>(scale_bytes);
  a.packed_bytes = static_cast<int>(packed_bytes);
  const bool out_aligned = ((reinterpret_cast<uintptr_t>(packed_k) | reinterpret_cast<uintptr_t>(packed_v) |
                             reinterpret_cast<uintptr_t>(scales_k) | reinterpret_cast<uintptr_t>(scales_v)) & 3u) == 0;
  // Word-granular copy and CRC when every section is whole 4-byte words (then the slices are
  // too); slices: the largest power of two <= kRecThreads dividing the payload (in words or
  // bytes). The tree folds need x^(8 * slice_bytes * 2^k) mod P, from x^8 by square-and-multiply.
  a.words = (out_aligned && scale_bytes % 4 == 0 && packed_bytes % 4 == 0) ? 1 : 0;
  const long long unit = a.words ? 4 : 1;
  int slices = kRecThreads;
  while (slices > 1 && payload % (unit * slices)) slices >>= 1;
  a.slices = slices;
  a.slice_bytes = static_cast<int>(payload / slices);
  unsigned x8 = 1u << 31;  // x^0 in the reflected representation
  for (int i = 0; i < 8; ++i) x8 = (x8 & 1u) ? (x8 >> 1) ^ 0xEDB88320u : x8 >> 1;
  unsigned acc = 1u << 31, base = x8;
  for (unsigned e = static_cast<unsigned>(a.slice_bytes); e; e >>= 1) {
    if (e & 1u) acc = crc_mulmod(acc, base);
    base = crc_mulmod(base, base);
  }
  for (int k = 0; k < kRecMaxLevels; ++k) {
    a.shift[k] = acc;
    acc = crc_mulmod(acc, acc);
  }
  a.packed_k = packed_k;
  a.packed_v = packed_v;
  a.scales_k = reinterpret_cast<uint8_t*>(scales_k);
  a.scales_v = reinterpret_cast<uint8_t*>(scales_v);
  a.valid = valid_tokens;
  a.status = record_status;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "record decode device");
  e = launch_record_decode(a, device_info(dev).sms, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "record decode launch");
}

}  // extern "C"

namespace kvb {
namespace {

// Plan of a batched decode: the streaming kernel's geometry checks, CTAs per problem and the
// workspace layout (header, 2 ticket words per problem, then the problems' parts).
struct BatchPlan {
  Plan p;
  int ctas = 0;
  size_t ws_bytes = 0;
};

int plan_batched(int n_problems, int block_tokens, int query_heads, int kv_heads, int head_dim,
                 int bits, int group_size, BatchPlan& bp) {
  if (n_problems < 1) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "n_problems must be >= 1");
  const Geometry g{1, block_tokens, query_heads, kv_heads, head_dim, bits, group_size};
  int st = check_geometry(g);
  if (st) return st;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const DeviceInfo info = device_info(dev);
  if (n_problems > info.sms)
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "a batched decode takes at most one problem per SM");
  Plan& p = bp.p;
  p.gqa = query_heads / kv_heads;
  p.n_qsub = (p.gqa + 7) / 8;
  p.n_vheads = kv_heads * p.n_qsub;
  if (!plan_streaming(g, info, p, false, 0))
    return fail(KVSSD_B200_ERR_UNSUPPORTED,
                "batched decode needs the streaming kernel's shapes (INT4, head_dim 128, group "
                "32 or 64, KV heads dividing 16, at most 8 query heads per KV head)");
  p.kernel = async_decode_kernel_for(bits, head_dim, group_size, kv_heads, true);
  p.streaming = true;
  p.path = KVSSD_B200_PATH_TENSOR_CORE;
  p.heads_per_cta = kv_heads;
  p.wph = async_warps() / kv_heads;
  p.threads = async_threads();
  p.n_head_groups = 1;
  p.tiles_per_block = (block_tokens + 15) / 16;
  bp.ctas = std::max(1, info.sms / n_problems);
  p.n_splits = bp.ctas;
  p.n_parts = bp.ctas * n_problems;
  bp.ws_bytes = kHeaderBytes + static_cast<size_t>(p.n_parts) * query_heads * (head_dim + 2) *
                                  sizeof(unsigned long long);
  return KVSSD_B200_OK;
}

}  // namespace
}  // namespace kvb

extern "C" {

int kvssd_b200_decode_batched_workspace_size(int n_problems, int block_tokens, int query_heads,
                                             int kv_heads, int head_dim, int bits,
                                             int group_size, size_t* bytes) {
  if (!bytes) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  BatchPlan bp;
  const int st = plan_batched(n_problems, block_tokens, query_heads, kv_heads, head_dim, bits,
                              group_size, bp);
  if (st) return st;
  *bytes = bp.ws_bytes;
  return KVSSD_B200_OK;
}

int kvssd_b200_decode_batched(const kvssd_b200_problem* problems, int n_problems,
                              int query_dtype, int block_tokens, int query_heads, int kv_heads,
                              int head_dim, int bits, int group_size, float sm_scale,
                              void* workspace, size_t workspace_bytes,
                              kvssd_b200_stream_t stream) {
  if (!problems) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "problems must not be NULL");
  if (query_dtype < KVSSD_B200_Q_F32 || query_dtype > KVSSD_B200_Q_F64)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "unknown query dtype");
  if (!std::isfinite(sm_scale)) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "sm_scale must be finite");
  BatchPlan bp;
  int st = plan_batched(n_problems, block_tokens, query_heads, kv_heads, head_dim, bits,
                        group_size, bp);
  if (st) return st;
  if (!workspace || workspace_bytes < bp.ws_bytes)
    return fail(KVSSD_B200_ERR_WORKSPACE, "workspace needs " + std::to_string(bp.ws_bytes) + " bytes");
  if (reinterpret_cast<uintptr_t>(workspace) & 15u)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  const Plan& p = bp.p;
  DecodeArgs a{};
  a.q_dtype = query_dtype;
  a.bt = block_tokens;
  a.qh = query_heads;
  a.kvh = kv_heads;
  a.d = head_dim;
  a.bits = bits;
  a.group = group_size;
  a.gqa = p.gqa;
  a.n_qsub = p.n_qsub;
  a.n_vheads = p.n_vheads;
  a.heads_per_cta = p.heads_per_cta;
  a.wph = p.wph;
  a.tiles_per_block = p.tiles_per_block;
  a.n_splits = bp.ctas;
  a.score_scale = sm_scale * 1.4426950408889634f;
  char* ws = static_cast<char*>(workspace);
  a.status = reinterpret_cast<unsigned*>(ws);
  a.part_epoch = reinterpret_cast<unsigned*>(ws + kTicketOffset);
  a.part_ml = reinterpret_cast<float*>(ws + kHeaderBytes);
  a.part_acc = a.part_ml + static_cast<size_t>(p.n_parts) * query_heads * 2;
  a.tpart_acc = reinterpret_cast<unsigned long long*>(ws + kHeaderBytes) +
                static_cast<size_t>(p.n_parts) * query_heads * 2;
  a.problems = problems;
  a.fuse_combine = 1;
  {
    cudaError_t e = ensure_dynamic_smem(p.kernel, p.smem);
    if (e != cudaSuccess) return cuda_fail(e, "shared-memory attribute");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bp.ctas, n_problems, 1);
  cfg.blockDim = dim3(p.threads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, p.kernel, a);
  if (e == cudaErrorCooperativeLaunchTooLarge) {
    cudaGetLastError();
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "the batched grid cannot be co-resident here");
  }
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "batched decode launch");
}

int kvssd_b200_read_status(void* workspace, int clear, unsigned* device_status,
                           kvssd_b200_stream_t stream) {
  if (!workspace || !device_status) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (clear && host) {
    // The status word and the combine's test hook (the stream has drained above, so no kernel
    // of this workspace is running). The epoch stays: parts of earlier calls carry older tags.
    e = cudaMemsetAsync(workspace, 0, sizeof(unsigned), s);
    if (e == cudaSuccess)
      e = cudaMemsetAsync(static_cast<char*>(workspace) + kTicketOffset + 4, 0, 8, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "status clear");
  }
  *device_status = host;
  if (host) return fail(KVSSD_B200_ERR_DEVICE_STATUS, "device status " + std::to_string(host));
  return KVSSD_B200_OK;
}

int kvssd_b200_merge_chunks(const float* outs, const float* lses, int n_chunks, int query_heads,
                            int head_dim, float* out, float* lse, kvssd_b200_stream_t stream) {
  if (!outs || !lses || !out || !lse) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (n_chunks < 1 || query_heads < 1 || head_dim < 1)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "at least one chunk is required");
  if (n_chunks > kMaxParts) return fail(KVSSD_B200_ERR_UNSUPPORTED, "too many chunks");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  merge_chunks_kernel<<<dim3(query_heads, (head_dim + 127) / 128, 1), 128,
                        static_cast<size_t>(n_chunks) * sizeof(float), s>>>(
      outs, lses, n_chunks, query_heads, head_dim, out, lse);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "merge launch");
}

int kvssd_b200_merge_pair(const float* left_out, const float* left_lse, const float* right_out,
                          const float* right_lse, int query_heads, int head_dim, float* out,
                          float* lse, kvssd_b200_stream_t stream) {
  if (!left_out || !left_lse || !right_out || !right_lse || !out || !lse)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (query_heads < 1 || head_dim < 1) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "empty chunk");
  const long long n = static_cast<long long>(query_heads) * head_dim;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  merge_pair_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
      left_out, left_lse, right_out, right_lse, query_heads, head_dim, out, lse);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "merge launch");
}

int kvssd_b200_dequantize(const uint8_t* packed, const uint16_t* scales, long long rows,
                          int head_dim, int bits, int group_size, int mode, uint16_t* values,
                          uint8_t* codes, kvssd_b200_stream_t stream) {
  if (!packed || !scales || !values || !codes) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (bits != 2 && bits != 4) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bits must be 2 or 4");
  if (rows < 1 || head_dim < 1 || group_size < 1 || head_dim % group_size)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "group_size must divide head_dim");
  if ((head_dim * bits) % 32)
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "rows must be whole 32-bit words of codes");
  if (group_size % (16 / bits))
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "group_size must cover whole 16-bit lanes");
  if (mode != 0 && mode != 1) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "mode must be 0 or 1");
  if (mode == 1 && (rows % 2)) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "mode 1 needs an even row count");
  if (reinterpret_cast<uintptr_t>(packed) & 3u) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "packed must be 4-byte aligned");
  const long long items = mode == 0 ? rows * (head_dim * bits / 32) : (rows / 2) * (head_dim * bits / 16);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dequant_kernel_for(bits, mode)<<<static_cast<unsigned>((items + 255) / 256), 256, 0, s>>>(
      packed, reinterpret_cast<const __half*>(scales), rows, head_dim, group_size,
      reinterpret_cast<__half*>(values), codes);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KVSSD_B200_OK : cuda_fail(e, "dequantize launch");
}

}  // extern "C"
