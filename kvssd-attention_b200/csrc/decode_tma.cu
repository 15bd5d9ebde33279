// Streaming split-KV decode fed by TMA (sm_100a): a producer warp copies whole 16-token
// tile-rows of the selection (K, V and both scale rows of ALL KV heads, one tensor copy each)
// into a ring of shared-memory stages; the 16 consumer warps only run the tile math.
//
// Work split as in the cp.async-fed kernel (decode_async.cu): one CTA per SM owns a contiguous
// range of 16-token tile-rows of the selection; consumer warp w serves KV head w % kvh and the
// tile-rows k == w / kvh (mod 16 / kvh), so the 16 / kvh consumer groups interleave tile-rows
// and each group has its own ring of kTmaSlots stages. A stage holds
//   K  [kvh][16 rows][64 B]   one 3-D TMA box (dims: bytes, token rows, heads -- the heads are
//   V  [kvh][16 rows][64 B]   the outer box dimension, so each head's 16 rows are contiguous)
//   KS [16 rows][kvh * G * 2 B], VS [16 rows][kvh * G * 2 B]   one 2-D box each,
// all with the TMA's address-based 16-byte-chunk swizzle (64-byte rows: chunk q of row r at
// q ^ ((r >> 1) & 3), the layout ldmatrix reads without bank conflicts). A tile-row never
// crosses a block (block_tokens is a multiple of 16); the producer resolves the block through
// the block table once per 32 blocks (a warp-wide cache) and copies all 16 rows even when fewer
// are valid (the pool holds whole blocks); the stage's valid row count travels in shared
// memory. A refused block-table entry gets no copy and a zero row count.
//
// Synchronisation: per stage a "full" mbarrier (the producer's arrive with the stage's byte
// count; the TMA completes the bytes) and an "empty" mbarrier (one arrive per consumer warp of
// the group, after its QK MMAs have consumed the tile's last shared-memory loads). Four
// producer warps (16-19, one per SM sub-partition) fill the rings: group g's stages are split
// among producers g, g + WPH, ... by stage index; a producer blocks on the next empty barrier
// of its own stages, so no group waits behind another.
// Every wait is bounded (about a second, and a poll count): on timeout the kernel flags
// kDevStreamTimeout, waits (bounded) for the copies it issued, and finishes with what it has.
#include <cuda.h>

#include <mutex>
#include <vector>

#include "fused_tail.cuh"
#include "stream_math.cuh"
#include "tma.cuh"

namespace kvb {

struct TmaMaps {
  CUtensorMap k, v, ks, vs;
};

constexpr int kTmaSlots = 4;  // ring stages per consumer group
constexpr uint32_t kTmaMaxPolls = 1u << 26;

// Producer warps: four, one per SM sub-partition (warp w runs on sub-partition w % 4). A
// sub-partition that hosts a producer warp runs its consumer warps measurably slower (the CTA
// then waits ~2 us for them at its end), so every sub-partition gets exactly one producer and
// the consumer groups share them: group g's stages are issued by producers g, g + WPH, ...
constexpr int kTmaProducers = 4;

template <int KVH, int G, int BITS>
struct TmaLayout {
  static constexpr int WPH = kStreamWarps / KVH;  // consumer groups (each with its own ring)
  static constexpr int PPG = kTmaProducers / WPH;  // producer warps per group
  static constexpr int THREADS = 32 * (kStreamWarps + kTmaProducers);
  static constexpr int NS = WPH * kTmaSlots;      // ring stages
  static constexpr int PD = 16 * BITS;            // code bytes per (token, head): 64 or 32
  static constexpr int HEAD_TILE = 16 * PD;       // one head's 16 rows in a stage
  static constexpr int SRB = KVH * 2 * G;         // scale bytes per token row
  static constexpr int KV_BYTES = KVH * HEAD_TILE;  // K (or V) bytes per stage
  static constexpr int S_BYTES = 16 * SRB;        // K (or V) scale bytes per stage
  static constexpr int S_SPAN = (S_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_V = KV_BYTES, OFF_KS = 2 * KV_BYTES, OFF_VS = OFF_KS + S_SPAN;
  static constexpr int STAGE = OFF_VS + S_SPAN;   // multiple of 1024: swizzle phase = address
  static constexpr uint32_t TX = 2 * KV_BYTES + 2 * S_BYTES;
  // Scale rows use the TMA swizzle whose span equals the row (16 B rows: none).
  static constexpr uint32_t SWZ = SRB >= 128 ? 7u : SRB == 64 ? 3u : SRB == 32 ? 1u : 0u;
  static constexpr int Q_MAX = 16384;  // query staged in shared memory up to this many bytes
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(NS) * STAGE + Q_MAX;  // + alignment
  __device__ static uint32_t swizzled(uint32_t off) { return off ^ (((off >> 7) & SWZ) << 4); }
};

template <int KVH, int GROUP, int BITS>
__global__ void __launch_bounds__(TmaLayout<KVH, 128 / GROUP, BITS>::THREADS, 1)
    tma_decode_kernel(const DecodeArgs a, const __grid_constant__ TmaMaps maps) {
  constexpr int D = 128, G = D / GROUP;
  using L = TmaLayout<KVH, G, BITS>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[L::NS], empty[L::NS];
  __shared__ int stage_rows[L::NS];
  __shared__ int cta_fault;  // a wait of this CTA gave up: its part is poisoned
  __shared__ __align__(8) uint64_t q_bar;  // the staged query copy has landed
  const uint32_t raw_s = smem_addr(smem_raw);
  const uint32_t ring_s = (raw_s + 1023u) & ~1023u;
  uint8_t* ring = smem_raw + (ring_s - raw_s);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int h = warp % KVH, grp = warp / KVH;
  // Shared-memory and parameter-space setup may overlap the preceding grid's tail.
  if (threadIdx.x == 0) {
    cta_fault = 0;
    for (int s = 0; s < L::NS; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), KVH);
    }
    mbar_init(smem_addr(&q_bar), 1);
    mbar_init_fence();
  }
  // Every warp of every CTA reads the whole (small) query: one bulk copy per CTA into shared
  // memory instead of 16 warps' loads of the same lines from L2.
  const int qsize = a.q_dtype == kQF64 ? 8 : a.q_dtype == kQF32 ? 4 : 2;
  const uint32_t q_bytes = static_cast<uint32_t>(a.qh) * D * qsize;
  const bool q_staged = q_bytes <= L::Q_MAX && (reinterpret_cast<uintptr_t>(a.q) & 15u) == 0;
  uint8_t* q_smem = ring + L::NS * L::STAGE;
  if (warp >= kStreamWarps && lane == 0) {
    prefetch_tensor_map(&maps.k);
    prefetch_tensor_map(&maps.v);
    prefetch_tensor_map(&maps.ks);
    prefetch_tensor_map(&maps.vs);
  }
  // Programmatic stream serialization: wait for the preceding grid before the first global
  // access, and let the next launch start early.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  // Exchange epoch of this call (completed calls + 1), read before this CTA's arrival.
  const unsigned epoch =
      a.xworld ? *reinterpret_cast<const volatile unsigned*>(a.xpeers[a.xrank]) + 1u : 0u;
  // The call's part tags (fused combine): read by producer 0 once it has issued its stages
  // (before this CTA's part is written) into shared memory, out of the streaming loop's
  // registers and off the start-up path.
  __shared__ PartEpoch s_pe;
  auto flag_timeout = [&]() {
    atomicOr(a.status, kDevStreamTimeout);
    cta_fault = 1;
  };
  const unsigned long long deadline = global_ns() + kCombineWaitNs;
  __syncthreads();
  if (q_staged && warp == kStreamWarps && lane == 0) {
    mbar_arrive_expect_tx(smem_addr(&q_bar), q_bytes);
    bulk_load(smem_addr(q_smem), a.q, q_bytes, smem_addr(&q_bar));
  }

  const long long t_begin = a.total_tiles * blockIdx.x / a.n_splits;
  const int n_tiles = static_cast<int>(a.total_tiles * (blockIdx.x + 1) / a.n_splits - t_begin);
  int issued = 0;  // producer: the group's stages up to and including its last own one
  StreamState state;
  const int q0 = h * a.gqa, nq = a.gqa;

  // Producer pi serves consumer group gp = pi % WPH and issues the group's stages i with
  // i % PPG == pp (pp = pi / WPH); `issued` counts the group's stages up to its last own one.
  const int pi = warp - kStreamWarps, gp = pi % L::WPH, pp = pi / L::WPH;
  if (warp >= kStreamWarps) {
    // ---------------- producer pp of group gp
    const uint64_t policy = l2_evict_first();
    BlockInfoCache cache;
    const int n_group = gp < n_tiles ? (n_tiles - gp + L::WPH - 1) / L::WPH : 0;
#pragma unroll 1
    for (int i = pp; i < n_group; i += L::PPG) {
      const int sl = gp * kTmaSlots + i % kTmaSlots;
      const bool free_slot = mbar_wait_until(smem_addr(&empty[sl]),
                                             ((i / kTmaSlots) & 1) ^ 1, deadline,
                                             kTmaMaxPolls);
      if (!__all_sync(0xffffffffu, free_slot)) {  // the warp leaves together
        if (lane == 0) flag_timeout();
        break;
      }
      issued = i + 1;
      const long long t = t_begin + gp + static_cast<long long>(i) * L::WPH;
      const int slot = static_cast<int>(t / a.tiles_per_block);
      const int tib = static_cast<int>(t - static_cast<long long>(slot) * a.tiles_per_block);
      const uint32_t bar = smem_addr(&full[sl]);
      const uint32_t st = ring_s + sl * L::STAGE;
      auto copy = [&](int blk) {
        const int row0 = blk * a.bt + 16 * tib;
        mbar_expect_tx(bar, L::TX);
        tma_load_3d(st, &maps.k, 0, row0, 0, bar, policy);
        tma_load_3d(st + L::OFF_V, &maps.v, 0, row0, 0, bar, policy);
        tma_load_2d(st + L::OFF_KS, &maps.ks, 0, row0, bar, policy);
        tma_load_2d(st + L::OFF_VS, &maps.vs, 0, row0, bar, policy);
      };
      // Without a block table the pool block is the slot itself (slot < n_sel <= n_pool), so
      // the copies go out before the valid count is known; the arrival below then publishes
      // the row count. With a table the entry decides whether to copy at all.
      const bool identity = a.table == nullptr;
      if (identity && lane == 0) copy(slot);
      int blk, valid;
      cache.lookup(a, slot, lane, blk, valid);
      const int rows = blk < 0 ? 0 : min(16, valid - 16 * tib);
      if (lane == 0) {
        if (!identity && rows > 0) copy(blk);
        stage_rows[sl] = rows;
        mbar_arrive(bar);  // completes once the copied bytes (if any) have landed
      }
      __syncwarp();
    }
    if (pi == 0 && lane == 0)
      s_pe = a.fuse_combine ? read_part_epoch(a) : PartEpoch{0u, 0u, false};
  } else {
    // ---------------- consumers
    bool q_ready = true;
    if (q_staged)
      q_ready = __all_sync(0xffffffffu,
                           mbar_wait_until(smem_addr(&q_bar), 0, deadline, kTmaMaxPolls));
    if (!q_ready && lane == 0) flag_timeout();
    const void* qsrc = q_staged && q_ready ? static_cast<const void*>(q_smem) : a.q;
    const uint32_t hs = static_cast<uint32_t>(h * 2 * G);  // head's byte offset in a scale row
    const uint32_t sk_off = L::swizzled(g * L::SRB + hs);
    const uint32_t sv_off = L::swizzled(2 * c * L::SRB + hs);
    const int sv_odd = static_cast<int>(L::swizzled((2 * c + 1) * L::SRB + hs)) -
                       static_cast<int>(sv_off);
    const int n_mine = grp < n_tiles ? (n_tiles - grp + L::WPH - 1) / L::WPH : 0;
    // Waits for stage i of this group; false (the warp leaves together) on timeout.
    auto wait_stage = [&](int i, int sl) {
      const bool landed =
          mbar_wait_until(smem_addr(&full[sl]), (i / kTmaSlots) & 1, deadline, kTmaMaxPolls);
      if (__all_sync(0xffffffffu, landed)) return true;
      if (lane == 0) flag_timeout();
      return false;
    };
    if constexpr (BITS == 4) {
      QueryFrags<GROUP> qfr;
      qfr.load(a, qsrc, q0, nq, g, c);
      const int ld_row = lane & 7, ld_chunk = lane >> 3;
      const uint32_t ld_off =
          static_cast<uint32_t>(ld_row * 64 + ((ld_chunk ^ ((ld_row >> 1) & 3)) << 4));
      // Unrolled by twice the ring depth: stage index, parity and addresses fold to constants
      // (measured, c2 decode: no unroll 40.6 us, 2: 38.8, 4: 37.6, 8: 37.3, 16: 41.5). Group 64
      // keeps 4: its scale handling needs more registers, and 8 spills there.
      constexpr int kUnroll = GROUP == 32 ? 8 : 4;
#pragma unroll kUnroll
      for (int i = 0; i < n_mine; ++i) {
        const int sl = grp * kTmaSlots + i % kTmaSlots;
        if (!wait_stage(i, sl)) break;
        const int rows = stage_rows[sl];
        const uint32_t empty_bar = smem_addr(&empty[sl]);
        if (rows <= 0) {
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar);
          continue;
        }
        const uint32_t st = ring_s + sl * L::STAGE;
        const uint8_t* sp = ring + sl * L::STAGE;
        TileFrags<G> t;
        t.template load<L::SRB>(st + h * L::HEAD_TILE, st + L::OFF_V + h * L::HEAD_TILE, ld_off,
                                sp + L::OFF_KS + sk_off, sp + L::OFF_VS + sv_off, sv_odd);
        float x[4];
        qk_tile<GROUP>(t, qfr, x);
        __syncwarp();  // every lane's loads of the stage have been consumed: release it
        if (lane == 0) mbar_arrive(empty_bar);
        softmax_pv_tile<GROUP, true>(x, rows, g, qfr.unscale, t, state);
      }
      finish_stream<GROUP, true>(state, c);
    } else {
      QueryFrags2<GROUP> qfr;
      qfr.load(a, qsrc, q0, nq, g, c);
      const uint32_t ld_off = ld_off_int2(lane);
#pragma unroll (GROUP == 32 ? 8 : 4)
      for (int i = 0; i < n_mine; ++i) {
        const int sl = grp * kTmaSlots + i % kTmaSlots;
        if (!wait_stage(i, sl)) break;
        const int rows = stage_rows[sl];
        const uint32_t empty_bar = smem_addr(&empty[sl]);
        if (rows <= 0) {
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar);
          continue;
        }
        const uint32_t st = ring_s + sl * L::STAGE;
        const uint8_t* sp = ring + sl * L::STAGE;
        TileFrags2<G> t;
        t.template load<L::SRB>(st + h * L::HEAD_TILE, st + L::OFF_V + h * L::HEAD_TILE, ld_off,
                                sp + L::OFF_KS + sk_off, sp + L::OFF_VS + sv_off, sv_odd);
        float x[4];
        qk_tile2<GROUP>(t, qfr, c, x);
        __syncwarp();  // every lane's loads of the stage have been consumed: release it
        if (lane == 0) mbar_arrive(empty_bar);
        softmax_pv_tile2<GROUP>(x, rows, g, t, state);
      }
    }
  }
  __syncthreads();
  if (warp >= kStreamWarps && lane == 0) {
    // Copies still in flight can only be this producer's stages among the group's last
    // kTmaSlots (after a timeout) and the query copy; wait for them (bounded) before the ring
    // is reused and the CTA exits.
    const unsigned long long drain_deadline = global_ns() + kCombineWaitNs;
    if (pi == 0 && q_staged && !mbar_wait_until(smem_addr(&q_bar), 0, drain_deadline, kTmaMaxPolls))
      flag_timeout();
    for (int idx = max(0, issued - kTmaSlots); idx < issued; ++idx)
      if (idx % L::PPG == pp &&
          !mbar_wait_until(smem_addr(&full[gp * kTmaSlots + idx % kTmaSlots]),
                           (idx / kTmaSlots) & 1, drain_deadline, kTmaMaxPolls))
        flag_timeout();
  }
  __syncthreads();
  const PartEpoch pe = s_pe;
  const unsigned tag = pe.epoch | (pe.poison || cta_fault ? kTagPoison : 0u);
  merge_warps_write_part<KVH, BITS>(a, reinterpret_cast<float*>(ring), warp, lane, q0, nq, state,
                                    tag);
  if (a.fuse_combine) fused_combine_tail<D>(a, epoch, pe, a.n_splits);
}

using TmaKernel = void (*)(const DecodeArgs, const TmaMaps);

template <int GROUP, int BITS>
TmaKernel tma_kernel_for_heads(int kvh) {
  switch (kvh) {
    case 4: return tma_decode_kernel<4, GROUP, BITS>;
    case 8: return tma_decode_kernel<8, GROUP, BITS>;
    case 16: return tma_decode_kernel<16, GROUP, BITS>;
    default: return nullptr;
  }
}

template <int BITS>
TmaKernel tma_kernel_for_group(int group, int kvh) {
  switch (group) {
    case 32: return tma_kernel_for_heads<32, BITS>(kvh);
    case 64: return tma_kernel_for_heads<64, BITS>(kvh);
    default: return nullptr;
  }
}

TmaKernel tma_kernel_for(int bits, int d, int group, int kvh) {
  if (d != 128) return nullptr;
  return bits == 4 ? tma_kernel_for_group<4>(group, kvh)
         : bits == 2 ? tma_kernel_for_group<2>(group, kvh)
                     : nullptr;
}

template <int G, int BITS>
int tma_threads_for_heads(int kvh) {
  switch (kvh) {
    case 4: return TmaLayout<4, G, BITS>::THREADS;
    case 8: return TmaLayout<8, G, BITS>::THREADS;
    case 16: return TmaLayout<16, G, BITS>::THREADS;
    default: return 0;
  }
}

template <int G, int BITS>
size_t tma_smem_for_heads(int kvh) {
  switch (kvh) {
    case 4: return TmaLayout<4, G, BITS>::SMEM;
    case 8: return TmaLayout<8, G, BITS>::SMEM;
    case 16: return TmaLayout<16, G, BITS>::SMEM;
    default: return 0;
  }
}

// ---------------- host side

// Tensor-map encoder from the driver (resolved once through the runtime; no libcuda link).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Encoded maps are cached by (kind, pointer, rows, row bytes): a decode loop over the same
// pools encodes once.
struct MapKey {
  int kind;
  const void* ptr;
  unsigned long long rows;
  int row_bytes;
  int head_bytes;  // K / V: code bytes per (token, head), 64 (INT4) or 32 (INT2)
  bool operator==(const MapKey& o) const {
    return kind == o.kind && ptr == o.ptr && rows == o.rows && row_bytes == o.row_bytes &&
           head_bytes == o.head_bytes;
  }
};

bool encode_cached(const MapKey& key, CUtensorMap* out) {
  static std::mutex mu;
  static std::vector<std::pair<MapKey, CUtensorMap>> cache;
  static size_t next_victim = 0;
  constexpr size_t kCapacity = 256;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : cache)
    if (e.first == key) {
      *out = e.second;
      return true;
    }
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  CUtensorMap m;
  CUresult r;
  if (key.kind < 2) {
    // K or V codes: (pd bytes, token rows, heads) with strides (heads * pd, pd); box
    // {pd, 16, heads} lands as [head][row][pd B] with the swizzle of the row width (64 or 32).
    const int pd = key.head_bytes, heads = key.row_bytes / pd;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(pd), key.rows,
                                static_cast<cuuint64_t>(heads)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(key.row_bytes),
                                   static_cast<cuuint64_t>(pd)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(pd), 16, static_cast<cuuint32_t>(heads)};
    const cuuint32_t elem[3] = {1, 1, 1};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(key.ptr), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
            pd == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // K or V scale rows: (row bytes, token rows); box {row bytes, 16}.
    const int rb = key.row_bytes;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rb), key.rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(rb)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(rb), 16};
    const cuuint32_t elem[2] = {1, 1};
    const CUtensorMapSwizzle swz = rb >= 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : rb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                   : rb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE;
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(key.ptr), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return false;
  if (cache.size() < kCapacity) {
    cache.emplace_back(key, m);
  } else {
    cache[next_victim] = {key, m};
    next_victim = (next_victim + 1) % kCapacity;
  }
  *out = m;
  return true;
}

bool tma_decode_supported(int bits, int d, int group, int kvh, int bt) {
  return tma_kernel_for(bits, d, group, kvh) != nullptr && bt % 16 == 0 &&
         tensor_map_encoder() != nullptr;
}

size_t tma_decode_smem(int kvh, int group, int bits) {
  if (bits == 2) return group == 32 ? tma_smem_for_heads<4, 2>(kvh) : tma_smem_for_heads<2, 2>(kvh);
  return group == 32 ? tma_smem_for_heads<4, 4>(kvh) : tma_smem_for_heads<2, 4>(kvh);
}

int tma_decode_threads(int kvh, int group) {
  // the thread count is the same for every geometry: 16 consumers + 4 producers
  return group == 32 ? tma_threads_for_heads<4, 4>(kvh) : tma_threads_for_heads<2, 4>(kvh);
}

// Launches the TMA-fed decode over grid (n_splits, 1): cooperative when the fused combine is
// on. Returns cudaErrorInvalidValue if the tensor maps cannot be encoded.
cudaError_t launch_tma_decode(const DecodeArgs& a, int n_splits, cudaStream_t s) {
  const TmaKernel kernel = tma_kernel_for(a.bits, a.d, a.group, a.kvh);
  if (!kernel) return cudaErrorInvalidValue;
  const size_t smem = tma_decode_smem(a.kvh, a.group, a.bits);
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::vector<std::pair<int, const void*>> done;
    std::lock_guard<std::mutex> lock(mu);
    const std::pair<int, const void*> key{dev, reinterpret_cast<const void*>(kernel)};
    bool set = false;
    for (const auto& d : done) set = set || d == key;
    if (!set) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      done.push_back(key);
    }
  }
  const unsigned long long rows = static_cast<unsigned long long>(a.n_pool) * a.bt;
  const int srb = a.kvh * 2 * (a.d / a.group);
  const int pd = a.d * a.bits / 8;  // code bytes per (token, head)
  TmaMaps maps;
  if (!encode_cached({0, a.kp, rows, a.kvh * pd, pd}, &maps.k) ||
      !encode_cached({1, a.vp, rows, a.kvh * pd, pd}, &maps.v) ||
      !encode_cached({2, a.ks, rows, srb, 0}, &maps.ks) ||
      !encode_cached({3, a.vs, rows, srb, 0}, &maps.vs))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_splits, 1, 1);
  cfg.blockDim = dim3(tma_decode_threads(a.kvh, a.group), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.fuse_combine ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, a, maps);
}

}  // namespace kvb
