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
#include "decode_tc.cuh"
#include "fused_tail.cuh"

namespace kvb {

constexpr int kAsyncWarps = 16;
constexpr int kAsyncThreads = 32 * kAsyncWarps;
constexpr int kAsyncDepth = 2;  // ring stages per warp (compile-time: cp.async.wait_group N)


// D = A * B (zero accumulator start).
__device__ __forceinline__ void mma_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

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
  constexpr int D = 128, BITS = 4, G = D / GROUP, MT = D / 16, DEPTH = kAsyncDepth;
  constexpr int PD = D * BITS / 8;            // 64 bytes of codes per (token, head)
  constexpr int SB = 2 * G;                   // scale bytes per (token, head)
  constexpr int OFF_V = 16 * PD, OFF_KS = 32 * PD, OFF_VS = OFF_KS + 16 * SB;
  constexpr int STAGE = ((OFF_VS + 16 * SB) + 127) / 128 * 128;
  constexpr int WPH = kAsyncWarps / KVH;
  constexpr float kLazyMax = 8.f;  // rescale only when a score beats the running max by 2^8
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
  // Q (pre-multiplied by sm_scale*log2(e)) as the B operand: k-step (m, j2) of thread c covers
  // dims 32m + 8c + {2j2, 2j2+4} (b0, even code slots) and 32m + 8c + {2j2+1, 2j2+5} (b1, odd
  // code slots), the order in which the unpacker emits a 32-bit word's codes.
  uint32_t qf[4][2][2];
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int d0 = 32 * m + 8 * c + 2 * j2 + r, d1 = d0 + 4;
        float f0 = 0.f, f1 = 0.f;
        if (g < nq) {
          const long long qb = static_cast<long long>(q0 + g) * D;
          f0 = load_query(a.q, a.q_dtype, qb + d0) * a.score_scale;
          f1 = load_query(a.q, a.q_dtype, qb + d1) * a.score_scale;
        }
        qf[m][j2][r] = h2_as_u32(__floats2half2_rn(f0, f1));
      }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
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
    uint32_t kA[4], kB[4], vA[4], vB[4];
    ScaleRow<G> sk0, sk1, sv[4];
    ldsm_x4(st + ld_off, kA[0], kA[1], kA[2], kA[3]);               // K tokens 0-7
    ldsm_x4(st + ld_off + 8 * PD, kB[0], kB[1], kB[2], kB[3]);      // K tokens 8-15
    ldsm_x4_trans(st + OFF_V + ld_off, vA[0], vA[1], vA[2], vA[3]);
    ldsm_x4_trans(st + OFF_V + ld_off + 8 * PD, vB[0], vB[1], vB[2], vB[3]);
    sk0.load(sp + sk_off);
    sk1.load(sp + sk_off + 8 * SB);
    sv[0].load(sp + sv_off);
    sv[1].load(sp + sv_off + SB);
    sv[2].load(sp + sv_off + 8 * SB);
    sv[3].load(sp + sv_off + 9 * SB);
    __syncwarp();                   // the stage's data is in registers: refill it
    issue(i + DEPTH, slot, st);     // with the tile DEPTH ahead
    if (++slot == DEPTH) {
      slot = 0;
      st = ring_s;
    } else {
      st += STAGE;
    }
    if (rows <= 0) continue;

    // ---- QK per scale group: r4 = sum_group (code - 8) q, then scaled by the K scale
    float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      __half2 p0[4], p1[4];
      LanePairs<BITS>::centred(kA[m], p0);
      LanePairs<BITS>::centred(kB[m], p1);
      float r4[4];
      mma_16816_zero(r4, h2_as_u32(p0[0]), h2_as_u32(p1[0]), h2_as_u32(p0[1]), h2_as_u32(p1[1]),
                     qf[m][0][0], qf[m][0][1]);
      mma_16816(r4, h2_as_u32(p0[2]), h2_as_u32(p1[2]), h2_as_u32(p0[3]), h2_as_u32(p1[3]),
                qf[m][1][0], qf[m][1][1]);
      const int gi = (32 * m) / GROUP;
      const float s0 = __half2float(sk0.s[gi]), s1 = __half2float(sk1.s[gi]);
      x[0] = fmaf(r4[0], s0, x[0]);
      x[1] = fmaf(r4[1], s0, x[1]);
      x[2] = fmaf(r4[2], s1, x[2]);
      x[3] = fmaf(r4[3], s1, x[3]);
    }
    // ---- online softmax in the log2 domain; rows g, g+8 x heads 2c, 2c+1
    if (rows < 16) {  // rows past the valid count hold stale codes: no weight
      if (g >= rows) x[0] = x[1] = -INFINITY;
      if (g + 8 >= rows) x[2] = x[3] = -INFINITY;
    }
    // The running max moves only when some score exceeds it by kLazyMax: p stays <= 2^8.
    const bool up = x[0] > m_run[0] + kLazyMax || x[2] > m_run[0] + kLazyMax ||
                    x[1] > m_run[1] + kLazyMax || x[3] > m_run[1] + kLazyMax;
    if (__any_sync(0xffffffffu, up)) {
      float t0 = fmaxf(x[0], x[2]), t1 = fmaxf(x[1], x[3]);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
      }
      const float n0 = fmaxf(m_run[0], t0), n1 = fmaxf(m_run[1], t1);
      const float al0 = fast_exp2(m_run[0] - n0), al1 = fast_exp2(m_run[1] - n1);
      l_run[0] *= al0;
      l_run[1] *= al1;
#pragma unroll
      for (int k = 0; k < MT; ++k) {
        acc[k][0] *= al0;
        acc[k][1] *= al1;
        acc[k][2] *= al0;
        acc[k][3] *= al1;
      }
      m_run[0] = n0;
      m_run[1] = n1;
    }
    const float e0 = fast_exp2(x[0] - m_run[0]), e1 = fast_exp2(x[1] - m_run[1]);
    const float e2 = fast_exp2(x[2] - m_run[0]), e3 = fast_exp2(x[3] - m_run[1]);
    l_run[0] += e0 + e2;
    l_run[1] += e1 + e3;
    const __half2 pt0 = u32_as_h2(transpose_8x8(h2_as_u32(__floats2half2_rn(e0, e1))));
    const __half2 pt1 = u32_as_h2(transpose_8x8(h2_as_u32(__floats2half2_rn(e2, e3))));
    // ---- PV per 32-dim chunk j (inside one scale group): P' = P * sv[t, group]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gi = (32 * j) / GROUP;
      const __half2 b0 = __hmul2(pt0, __halves2half2(sv[0].s[gi], sv[1].s[gi]));
      const __half2 b1 = __hmul2(pt1, __halves2half2(sv[2].s[gi], sv[3].s[gi]));
      __half2 cA[4], cB[4];
      LanePairs<BITS>::centred(vA[j], cA);
      LanePairs<BITS>::centred(vB[j], cB);
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2)
        mma_16816(acc[2 * j + k2], h2_as_u32(cA[2 * k2]), h2_as_u32(cA[2 * k2 + 1]),
                  h2_as_u32(cB[2 * k2]), h2_as_u32(cB[2 * k2 + 1]), h2_as_u32(b0),
                  h2_as_u32(b1));
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- merge the wph warps of each head through shared memory: [slot][field][lane]
  constexpr int kFields = 4 + 4 * MT;
  float* buf = reinterpret_cast<float*>(smem);
  if (sub > 0) {
    float* dst = buf + static_cast<size_t>((sub - 1) * KVH + h) * kFields * 32 + lane;
    dst[0] = m_run[0];
    dst[32] = m_run[1];
    dst[64] = l_run[0];
    dst[96] = l_run[1];
#pragma unroll
    for (int k = 0; k < MT; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[(4 + 4 * k + e) * 32] = acc[k][e];
  }
  __syncthreads();
  if (sub == 0) {
    for (int o = 1; o < WPH; ++o) {
      const float* src = buf + static_cast<size_t>((o - 1) * KVH + h) * kFields * 32 + lane;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float mo = src[hh * 32], lo = src[(2 + hh) * 32];
        const float mn = fmaxf(m_run[hh], mo);
        const float a0 = mn == -INFINITY ? 0.f : fast_exp2(m_run[hh] - mn);
        const float a1 = mn == -INFINITY ? 0.f : fast_exp2(mo - mn);
        m_run[hh] = mn;
        l_run[hh] = l_run[hh] * a0 + lo * a1;
#pragma unroll
        for (int k = 0; k < MT; ++k) {
          acc[k][hh] = acc[k][hh] * a0 + src[(4 + 4 * k + hh) * 32] * a1;
          acc[k][2 + hh] = acc[k][2 + hh] * a0 + src[(4 + 4 * k + 2 + hh) * 32] * a1;
        }
      }
    }
    // ---- this CTA's part; O^T row g of M-tile (j, k2) is dim 32j + 4g + 2k2, row g+8 the next
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], o);
      l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], o);
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int n = 2 * c + hh;
      if (n >= nq) continue;
      const size_t row = static_cast<size_t>(blockIdx.x) * a.qh + (q0 + n);
      if (g == 0) {
        a.part_ml[row * 2 + 0] = m_run[hh];
        a.part_ml[row * 2 + 1] = l_run[hh];
      }
      float* dst = a.part_acc + row * D + 4 * g;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2)
          *reinterpret_cast<float2*>(dst + 32 * j + 2 * k2) =
              make_float2(acc[2 * j + k2][hh], acc[2 * j + k2][2 + hh]);
    }
  }
  if (a.fuse_combine) fused_combine_tail<D>(a, epoch, a.n_splits);
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
  const size_t parts = static_cast<size_t>(blockIdx.y) * a.n_splits * a.qh;
  b.part_ml = a.part_ml + parts * 2;
  b.part_acc = a.part_acc + parts * a.d;
  b.tickets = a.problem_tickets + 2 * blockIdx.y;
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
