// Streaming split-KV decode for INT4 codes (sm_100a): every warp streams its own KV head's rows
// through a private cp.async ring and runs ldmatrix + mma.sync tile math with the FP16 scales
// factored out of the codes.
//
// Work: one CTA of 16 warps per SM owns a contiguous range of 16-token tiles of the selection
// for ALL KV heads, so the CTA's warps together read contiguous runs of token rows (kvssd's
// record layout interleaves the KV heads of a token, src/kvssd/format.py:165). Warp w serves
// KV head w % kv_heads and takes every wph-th tile of the range (wph = 16 / kv_heads); the
// number of KV heads is a template parameter, so strides and the head mapping are constants.
//
// Feed: each warp copies, for its tiles only, the 16 K rows and 16 V rows of its head (64
// bytes per row, 16-byte cp.async.cg, four lanes per row) and the rows' FP16 scales (8- or
// 4-byte cp.async.ca) into a private ring of `depth` stages: a stage is refilled with the tile
// `depth` ahead as soon as its data has moved to registers.
// Inside a block the copy addresses advance by constant strides and the block table is read
// once per block; tiles with fewer than 16 valid rows are flagged per stage.
// Warps wait only for their own copies (cp.async.wait_group + __syncwarp), never for each
// other, so the 16 warps drift apart and the scheduler interleaves one warp's copies with
// another's tensor-core work. Two stages per warp (74 KB per SM, ~11 MB in flight over the
// GPU, above HBM's bandwidth-latency product) measured fastest: deeper rings (3..6 stages)
// were 1-5 % slower, and the small ring leaves most of the SM's L1 to the 8-byte scale copies,
// whose 32-byte sectors are shared by four KV heads. Rows are stored with chunk q of row r at
// chunk q ^ ((r >> 1) & 3), so the 8 rows an ldmatrix reads fall on 8 distinct bank groups.
//
// Math (per warp, per tile of 16 tokens): with 32 dims per 16-byte chunk and group_size >= 32,
// every k-step of QK and every M-tile of PV lies inside one scale group, so scales are applied
// outside the tensor-core products, which multiply exact centred codes:
//   QK: S[t,n] = sum_group sk[t,group] * (sum_{d in group} (code-mid)[t,d] * q[n,d])
//       -- two m16n8k16 per group into a fresh FP32 accumulator, then one FFMA per element;
//   PV: O^T[d,n] = sum_t (code-mid)[t,d] * (P[t,n] * sv[t,group(d)])
//       -- the V scale is folded into the FP16 P operand of the M-tiles of that group;
//   ldmatrix.trans delivers V with two tokens per 32-bit register, the pairing the PV A
//   fragment needs. The online softmax runs in the log2 domain (q pre-scaled by
//   sm_scale*log2(e)) with a lazily updated running max: the max and the accumulator move only
//   when a score exceeds the running max by 2^8, detected with one warp vote per tile.
// The CTA finally merges the wph warps of each head through shared memory and writes one
// (m, l, acc) part per query head; with the fused combine the last CTAs to finish then fold
// the parts into the output (otherwise the combine kernel does).
#include "fused_tail.cuh"
#include "stream_math.cuh"

namespace kvb {

constexpr int kAsyncWarps = kStreamWarps;
constexpr int kAsyncThreads = 32 * kAsyncWarps;
constexpr int kAsyncDepth = 2;  // ring stages per warp (compile-time: cp.async.wait_group N)


// Copy side of one warp: the addresses of its next tile and the cursor over the selection.
// Consecutive tiles of a warp inside one block are 16 * WPH rows apart, so inside a block the
// lane addresses advance by constant strides; the block table is consulted once per block.
// Lane (r, q) copies 16-byte chunk q of rows r and r + 8 of K and V (chunk q of row r stored at
// chunk q ^ ((r >> 1) & 3)); lanes 0-15 copy K scale row (lane & 15), lanes 16-31 the V one.
template <int KVH, int G>
struct WarpFeed {
  static constexpr int PD = 64, SB = 2 * G, WPH = kAsyncWarps / KVH;
  static constexpr int ROW = KVH * PD, SROW = KVH * SB;  // bytes per token row
  static constexpr int STEP = 16 * WPH;                  // rows between this warp's tiles
  const uint8_t* gk;  // this lane's K / V / scale source for the next tile
  const uint8_t* gv;
  const uint8_t* gs;
  int slot, tib;  // cursor: selection slot and tile-in-block of the next block's first tile
  int off;        // row offset of the next tile in its block (>= block_tokens: block done)
  int valid = 0;  // valid rows of the current block (0 for a refused block-table entry)

  // Moves to the block that holds the next tile: one (cached) block-table lookup.
  __device__ __forceinline__ void enter_block(const DecodeArgs& a, BlockInfoCache& cache,
                                              int lane, int h) {
    const int tpb = a.tiles_per_block;
    while (tib >= tpb) {
      tib -= tpb;
      ++slot;
    }
    int blk;
    cache.lookup(a, slot, lane, blk, valid);
    if (blk < 0) {
      blk = 0;
      valid = 0;
    }
    off = tib * 16;
    tib += (tpb - tib + WPH - 1) / WPH * WPH;  // past this warp's tiles of the block
    const size_t row0 = static_cast<size_t>(blk) * a.bt + off;
    const int cr = lane >> 2, cq = lane & 3, sr = lane & 15;
    gk = a.kp + (row0 + cr) * ROW + h * PD + cq * 16;
    gv = a.vp + (row0 + cr) * ROW + h * PD + cq * 16;
    gs = reinterpret_cast<const uint8_t*>(lane < 16 ? a.ks : a.vs) + (row0 + sr) * SROW + h * SB;
  }

  __device__ __forceinline__ void advance() {
    gk += STEP * ROW;
    gv += STEP * ROW;
    gs += STEP * SROW;
    off += STEP;
  }
};

template <int KVH, int GROUP>
__device__ __forceinline__ void async_decode_body(const DecodeArgs& a) {
  constexpr int D = 128, BITS = 4, G = D / GROUP, DEPTH = kAsyncDepth;
  constexpr int PD = D * BITS / 8;            // 64 bytes of codes per (token, head)
  constexpr int SB = 2 * G;                   // scale bytes per (token, head)
  constexpr int OFF_V = 16 * PD, OFF_KS = 32 * PD, OFF_VS = OFF_KS + 16 * SB;
  constexpr int STAGE = ((OFF_VS + 16 * SB) + 127) / 128 * 128;
  constexpr int WPH = kAsyncWarps / KVH;
  using Feed = WarpFeed<KVH, G>;
  static_assert(G == 4 || G == 2, "scale rows must be whole 4-byte words");
  static_assert(DEPTH <= 32, "partial-tile flags are one bit per stage");
  extern __shared__ __align__(128) uint8_t smem[];
  // Launched with programmatic stream serialization: wait for the preceding grid before the
  // first global access (it may have produced the query or the KV), and let the next decode
  // launch early so its launch latency overlaps this grid's tail.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  // Exchange epoch of this call (completed calls + 1), read before this CTA's arrival.
  const unsigned epoch =
      a.xworld ? *reinterpret_cast<const volatile unsigned*>(a.xpeers[a.xrank]) + 1u : 0u;
  // The call's part tags (fused combine), read before this CTA's part is written.
  const PartEpoch pe = a.fuse_combine ? read_part_epoch(a) : PartEpoch{0u, 0u, false};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int h = warp % KVH, sub = warp / KVH;
  uint8_t* ring = smem + static_cast<size_t>(warp) * DEPTH * STAGE;
  const uint32_t ring_s = smem_addr(ring);
  __shared__ int tile_rows[kAsyncWarps][DEPTH];  // valid rows of stages flagged partial

  const long long t_begin = a.total_tiles * blockIdx.x / a.n_splits;
  const int n_tiles = static_cast<int>(a.total_tiles * (blockIdx.x + 1) / a.n_splits - t_begin);
  const int n_mine = sub < n_tiles ? (n_tiles - sub + WPH - 1) / WPH : 0;

  // ---------------- feed: this warp's copies of its i-th tile into stage i % DEPTH
  const int cr = lane >> 2, sr = lane & 15;
  const uint32_t dst_kv =
      static_cast<uint32_t>(cr * PD + (((lane & 3) ^ ((cr >> 1) & 3)) << 4));
  const uint32_t dst_s = (lane < 16 ? OFF_KS : OFF_VS) + sr * SB;
  const uint64_t policy = l2_evict_first();
  BlockInfoCache cache;
  Feed feed;
  {
    const long long t = t_begin + sub;
    feed.slot = static_cast<int>(t / a.tiles_per_block);
    feed.tib = static_cast<int>(t - static_cast<long long>(feed.slot) * a.tiles_per_block);
  }
  uint32_t partial = 0;  // bit s: stage s holds a tile with fewer than 16 valid rows
  // Copies tile `tile` of this warp into stage `fill_slot` (shared address fill_st).
  auto issue = [&](int tile, int fill_slot, uint32_t fill_st) {
    if (tile < n_mine) {
      if (tile == 0 || feed.off >= a.bt) feed.enter_block(a, cache, lane, h);
      const int rows = feed.valid - feed.off;
      if (rows >= 16) {
        cp_async16(fill_st + dst_kv, feed.gk, policy);
        cp_async16(fill_st + OFF_V + dst_kv, feed.gv, policy);
        cp_async16(fill_st + 8 * PD + dst_kv, feed.gk + 8 * Feed::ROW, policy);
        cp_async16(fill_st + OFF_V + 8 * PD + dst_kv, feed.gv + 8 * Feed::ROW, policy);
        if constexpr (G == 4) cp_async8(fill_st + dst_s, feed.gs, policy);
        else cp_async4(fill_st + dst_s, feed.gs, policy);
        partial &= ~(1u << fill_slot);
      } else {
        // Ragged tail: rows past the valid count are not copied (their scores are masked);
        // their scale rows repeat the last valid row so every scale in the stage is finite.
        const int rc = max(rows, 0);
        if (cr < rc) {
          cp_async16(fill_st + dst_kv, feed.gk, policy);
          cp_async16(fill_st + OFF_V + dst_kv, feed.gv, policy);
        }
        if (cr + 8 < rc) {
          cp_async16(fill_st + 8 * PD + dst_kv, feed.gk + 8 * Feed::ROW, policy);
          cp_async16(fill_st + OFF_V + 8 * PD + dst_kv, feed.gv + 8 * Feed::ROW, policy);
        }
        if (rc > 0) {
          const uint8_t* src = feed.gs + (min(sr, rc - 1) - sr) * Feed::SROW;
          if constexpr (G == 4) cp_async8(fill_st + dst_s, src, policy);
          else cp_async4(fill_st + dst_s, src, policy);
        }
        if (lane == 0) tile_rows[warp][fill_slot] = rc;
        partial |= 1u << fill_slot;
      }
      feed.advance();
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int i = 0; i < DEPTH; ++i) issue(i, i, ring_s + i * STAGE);

  // ---------------- compute state
  const int q0 = h * a.gqa, nq = a.gqa;
  QueryFrags<GROUP> qfr;
  qfr.load(a, a.q, q0, nq, g, c);
  StreamState state;
  // ldmatrix: lane supplies row (lane & 7) of the matrix for 16-byte chunk (lane >> 3), at its
  // swizzled position; rows 8-15 repeat the pattern 8 rows further.
  const int ld_row = lane & 7, ld_chunk = lane >> 3;
  const uint32_t ld_off =
      static_cast<uint32_t>(ld_row * PD + ((ld_chunk ^ ((ld_row >> 1) & 3)) << 4));
  const uint32_t sk_off = OFF_KS + g * SB, sv_off = OFF_VS + 2 * c * SB;

  int slot = 0;
  uint32_t st = ring_s;  // shared address of the stage consumed next
#pragma unroll 1
  for (int i = 0; i < n_mine; ++i) {
    cp_async_wait<DEPTH - 1>();  // this lane's copies of tile i have landed
    __syncwarp();                // ... and every lane's
    int rows = 16;
    if (partial & (1u << slot)) rows = tile_rows[warp][slot];
    const uint8_t* sp = ring + (st - ring_s);
    TileFrags<G> t;
    t.template load<SB>(st, st + OFF_V, ld_off, sp + sk_off, sp + sv_off, SB);
    __syncwarp();                   // the stage's data is in registers: refill it
    issue(i + DEPTH, slot, st);     // with the tile DEPTH ahead
    if (++slot == DEPTH) {
      slot = 0;
      st = ring_s;
    } else {
      st += STAGE;
    }
    if (rows <= 0) continue;
    float x[4];
    qk_tile<GROUP>(t, qfr, x);
    softmax_pv_tile<GROUP, false>(x, rows, g, qfr.unscale, t, state);
  }
  finish_stream<GROUP, false>(state, c);
  cp_async_wait<0>();
  __syncthreads();
  merge_warps_write_part<KVH>(a, reinterpret_cast<float*>(smem), warp, lane, q0, nq, state,
                              pe.epoch | (pe.poison ? kTagPoison : 0u));
  if (a.fuse_combine) fused_combine_tail<D>(a, epoch, pe, a.n_splits);
}

template <int KVH, int GROUP>
__global__ void __launch_bounds__(kAsyncThreads, 1) async_decode_kernel(const DecodeArgs a) {
  async_decode_body<KVH, GROUP>(a);
}

// Batched decode: problem blockIdx.y of a.problems, its splits along x. The problem's fields
// replace the single-problem ones; its parts and tickets are its own slices of the workspace.
template <int KVH, int GROUP>
__global__ void __launch_bounds__(kAsyncThreads, 1) async_decode_batched_kernel(const DecodeArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the descriptors may be fresh
  const kvssd_b200_problem pd = a.problems[blockIdx.y];
  // The host cannot see device-resident descriptors: refuse operands the copies and loads
  // cannot take (every CTA of the problem reaches the same verdict, so none waits for it).
  const int qsize = a.q_dtype == kQF64 ? 8 : a.q_dtype == kQF32 ? 4 : 2;
  const uintptr_t a16 = reinterpret_cast<uintptr_t>(pd.packed_k) | reinterpret_cast<uintptr_t>(pd.packed_v) |
                        reinterpret_cast<uintptr_t>(pd.scales_k) | reinterpret_cast<uintptr_t>(pd.scales_v);
  const uintptr_t a4 = reinterpret_cast<uintptr_t>(pd.valid_tokens) |
                       reinterpret_cast<uintptr_t>(pd.block_table) |
                       reinterpret_cast<uintptr_t>(pd.out) | reinterpret_cast<uintptr_t>(pd.lse);
  if (!pd.packed_k || !pd.packed_v || !pd.scales_k || !pd.scales_v || !pd.valid_tokens ||
      !pd.query || !pd.out || !pd.lse || (a16 & 15u) || (a4 & 3u) ||
      (reinterpret_cast<uintptr_t>(pd.query) % qsize) || pd.n_pool_blocks < 1 ||
      pd.n_sel_blocks < 0) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.status, kDevBadProblem);
    // A combining CTA of the refused problem still counts itself for the epoch store.
    const int n_comb = min(a.n_splits, a.qh * ((a.d + 31) / 32));
    if (threadIdx.x == 0 && static_cast<int>(blockIdx.x) >= a.n_splits - n_comb)
      publish_part_epoch(a, 0u, n_comb);
    return;
  }
  DecodeArgs b = a;
  b.q = pd.query;
  b.kp = pd.packed_k;
  b.vp = pd.packed_v;
  b.ks = reinterpret_cast<const __half*>(pd.scales_k);
  b.vs = reinterpret_cast<const __half*>(pd.scales_v);
  b.valid = pd.valid_tokens;
  b.table = pd.block_table;
  b.n_pool = pd.n_pool_blocks;
  b.n_sel = pd.n_sel_blocks;
  b.total_tiles = static_cast<long long>(pd.n_sel_blocks) * a.tiles_per_block;
  b.out = pd.out;
  b.lse = pd.lse;
  // This problem's slice of the (tagged, 64-bit) part arrays; the epoch is the grid's.
  const size_t parts = static_cast<size_t>(blockIdx.y) * a.n_splits * a.qh;
  b.part_ml = a.part_ml + parts * 4;
  b.tpart_acc = a.tpart_acc + parts * a.d;
  async_decode_body<KVH, GROUP>(b);
}

using DecodeKernel = void (*)(const DecodeArgs);

// INT4, head_dim 128, group_size 32 or 64 (16-byte code chunks inside one scale group; scale
// rows of whole 4-byte words), KV heads dividing the 16 warps of a CTA.
template <int GROUP>
DecodeKernel async_kernel_for_heads(int kvh, bool batched) {
  switch (kvh) {
    case 1: return batched ? async_decode_batched_kernel<1, GROUP> : async_decode_kernel<1, GROUP>;
    case 2: return batched ? async_decode_batched_kernel<2, GROUP> : async_decode_kernel<2, GROUP>;
    case 4: return batched ? async_decode_batched_kernel<4, GROUP> : async_decode_kernel<4, GROUP>;
    case 8: return batched ? async_decode_batched_kernel<8, GROUP> : async_decode_kernel<8, GROUP>;
    case 16:
      return batched ? async_decode_batched_kernel<16, GROUP> : async_decode_kernel<16, GROUP>;
    default: return nullptr;
  }
}

DecodeKernel async_decode_kernel_for(int bits, int d, int group, int kvh, bool batched) {
  if (bits != 4 || d != 128) return nullptr;
  switch (group) {
    case 32: return async_kernel_for_heads<32>(kvh, batched);
    case 64: return async_kernel_for_heads<64>(kvh, batched);
    default: return nullptr;
  }
}

int async_threads() { return kAsyncThreads; }
int async_warps() { return kAsyncWarps; }
int async_depth() { return kAsyncDepth; }
int async_stage_bytes(int group) {
  const int sb = 2 * (128 / group);
  return ((32 * 64 + 32 * sb) + 127) / 128 * 128;
}

}  // namespace kvb
