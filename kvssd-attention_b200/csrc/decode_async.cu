// Streaming split-KV decode for INT4 codes (sm_100a): every warp streams its own KV head's rows
// through a private cp.async ring and runs ldmatrix + mma.sync tile math with the FP16 scales
// factored out of the codes.
//
// Work: one CTA of 16 warps per SM owns a contiguous range of 16-token tiles of the selection
// for ALL KV heads, so the CTA's warps together read contiguous runs of token rows (kvssd's
// record layout interleaves the KV heads of a token, src/kvssd/format.py:165). Warp w serves
// KV head w % kv_heads and takes every wph-th tile of the range (wph = 16 / kv_heads).
//
// Feed: each warp copies, for its tiles only, the 16 K rows and 16 V rows of its head (64
// bytes per row, 16-byte cp.async.cg, four lanes per row) and the rows' FP16 scales (8- or
// 4-byte cp.async.ca) into a private ring of `depth` stages, depth-1 tiles ahead of its math.
// Warps wait only for their own copies (cp.async.wait_group + __syncwarp), never for each
// other, so the 16 warps drift apart and the scheduler interleaves one warp's copies and
// shuffles with another's tensor-core work, while ~160 KB per SM stays in flight without
// occupying registers. Rows are stored with chunk q of row r at chunk q ^ ((r >> 1) & 3), so
// the 8 rows an ldmatrix reads fall on 8 distinct bank groups.
//
// Math (per warp, per tile of 16 tokens): with 32 dims per 16-byte chunk and group_size >= 32,
// every k-step of QK and every M-tile of PV lies inside one scale group, so scales are applied
// outside the tensor-core products:
//   QK: S[t,n] = sum_group sk[t,group] * (sum_{d in group} (code-mid)[t,d] * q[n,d]);
//       the codes enter the mma as the raw FP16 values 1024+n / 1024+16n (q pre-divided by 16
//       for the latter); each group's FP32 accumulator starts at -C, C being the constant those
//       encodings add (computed once by the same mma from constant rows), so it ends at the
//       exact centred product; one FFMA per element then applies the K scale;
//   PV: O^T[d,n] = sum_t (code-mid)[t,d] * (P[t,n] * sv[t,group(d)])
//       -- the V scale is folded into the FP16 P operand of the M-tiles of that group;
//   ldmatrix.trans delivers V with two tokens per 32-bit register, the pairing the PV A
//   fragment needs. The online softmax runs in the log2 domain (q pre-scaled by
//   sm_scale*log2(e)) with a lazily updated running max: the max and the accumulator move only
//   when a score exceeds the running max by 2^8, detected with one warp vote per tile.
// The CTA finally merges the wph warps of each head through shared memory and writes one
// (m, l, acc) part per query head for the combine kernel.
#include "decode_tc.cuh"

namespace kvb {

constexpr int kAsyncWarps = 16;
constexpr int kAsyncThreads = 32 * kAsyncWarps;
constexpr int kAsyncDepth = 6;  // ring stages per warp (compile-time: cp.async.wait_group N)

template <int G>
struct ScaleRow {  // the G FP16 scales of one (token, KV head)
  __half s[G];
  __device__ __forceinline__ void load(const uint8_t* p) {
    if constexpr (G == 4) {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      memcpy(s, &w, 8);
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
      memcpy(s, &w, 4);
    }
  }
};

// Raw K codes for the QK mma: (1024 + n) in the even and (1024 + 16n) in the odd code slots of
// each 16-bit lane, two instructions fewer per pair than centring; the constant offsets are
// cancelled exactly through the accumulator start value (see async_decode_kernel).
__device__ __forceinline__ void magic_pairs(uint32_t x, uint32_t (&o)[4]) {
  const uint32_t x8 = x >> 8;
  o[0] = or_magic<0x000F000Fu>(x);
  o[1] = or_magic<0x00F000F0u>(x);
  o[2] = or_magic<0x000F000Fu>(x8);
  o[3] = or_magic<0x00F000F0u>(x8);
}

// D = A * B with a zero accumulator start (no register moves for C).
__device__ __forceinline__ void mma_16816_set(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1, float c0, float c1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1));
}

template <int GROUP>
__global__ void __launch_bounds__(kAsyncThreads, 1) async_decode_kernel(const DecodeArgs a) {
  constexpr int D = 128, BITS = 4, G = D / GROUP, MT = D / 16, DEPTH = kAsyncDepth;
  constexpr int PD = D * BITS / 8;            // 64 bytes of codes per (token, head)
  constexpr int SB = 2 * G;                   // scale bytes per (token, head)
  constexpr int OFF_V = 16 * PD, OFF_KS = 32 * PD, OFF_VS = OFF_KS + 16 * SB;
  constexpr int STAGE = ((OFF_VS + 16 * SB) + 127) / 128 * 128;
  constexpr float kLazyMax = 8.f;  // rescale only when a score beats the running max by 2^8
  static_assert(G == 4 || G == 2, "scale rows must be whole 4-byte words");
  extern __shared__ __align__(128) uint8_t smem[];
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int kvh = a.kvh, wph = a.wph;
  const int h = warp % kvh, sub = warp / kvh;
  uint8_t* ring = smem + static_cast<size_t>(warp) * DEPTH * STAGE;
  const uint32_t ring_s = smem_addr(ring);
  __shared__ int tile_rows[kAsyncWarps][DEPTH];

  const long long t_begin = a.total_tiles * blockIdx.x / a.n_splits;
  const int n_tiles = static_cast<int>(a.total_tiles * (blockIdx.x + 1) / a.n_splits - t_begin);
  const int n_mine = sub < n_tiles ? (n_tiles - sub + wph - 1) / wph : 0;

  // ---------------- feed: this warp's copies of its i-th tile into stage i % DEPTH
  // Lane (r, q) copies 16-byte chunk q of rows r and r+8 of K and V (chunk q of row r is stored
  // at chunk q ^ ((r >> 1) & 3)); lanes 0-15 copy the K scale row, lanes 16-31 the V scale row.
  const int row_bytes = kvh * PD;
  const int srow = kvh * SB;
  const int cr = lane >> 2, cq = lane & 3, sr = lane & 15;
  const uint32_t dst_kv = cr * PD + ((cq ^ ((cr >> 1) & 3)) << 4);
  const uint32_t dst_s = (lane < 16 ? OFF_KS : OFF_VS) + sr * SB;
  const uint8_t* k_lane = a.kp + h * PD + cr * row_bytes + cq * 16;
  const uint8_t* v_lane = a.vp + h * PD + cr * row_bytes + cq * 16;
  const uint8_t* s_lane = reinterpret_cast<const uint8_t*>(lane < 16 ? a.ks : a.vs) + h * SB +
                          sr * srow;
  const uint64_t policy = l2_evict_first();
  BlockInfoCache cache;
  TileCursor cur;
  cur.seek(t_begin + sub, a.tiles_per_block);
  int fill_slot = 0;
  auto issue = [&](int i) {
    if (i < n_mine) {
      const int off = cur.row_offset();
      int blk, valid;
      cache.lookup(a, cur.slot, lane, blk, valid);
      cur.advance(wph, a.tiles_per_block);
      const int rows = blk >= 0 ? max(0, min(valid - off, 16)) : 0;
      if (lane == 0) tile_rows[warp][fill_slot] = rows;
      if (rows > 0) {
        const size_t row0 = static_cast<size_t>(blk) * a.bt + off;
        const size_t kv_off = row0 * row_bytes, s_off = row0 * srow;
        const uint32_t st = ring_s + fill_slot * STAGE;
        if (cr < rows) {
          cp_async16(st + dst_kv, k_lane + kv_off, policy);
          cp_async16(st + OFF_V + dst_kv, v_lane + kv_off, policy);
        }
        if (cr + 8 < rows) {
          cp_async16(st + 8 * PD + dst_kv, k_lane + kv_off + 8 * row_bytes, policy);
          cp_async16(st + OFF_V + 8 * PD + dst_kv, v_lane + kv_off + 8 * row_bytes, policy);
        }
        if (sr < rows) {
          if constexpr (G == 4) cp_async8(st + dst_s, s_lane + s_off, policy);
          else cp_async4(st + dst_s, s_lane + s_off, policy);
        }
      }
      if (++fill_slot == DEPTH) fill_slot = 0;
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int i = 0; i < DEPTH - 1; ++i) issue(i);

  // ---------------- compute state
  const int q0 = h * a.gqa, nq = a.gqa;
  // Q (pre-multiplied by sm_scale*log2(e)) as the B operand: k-step (m, j2) of thread c covers
  // dims 32m + 8c + {2j2, 2j2+4} (b0, even code slots) and 32m + 8c + {2j2+1, 2j2+5} (b1, odd
  // code slots, divided by 16 to match the (1024 + 16n) encoding; exact power-of-two scaling).
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
          const float sc = r ? a.score_scale * 0.0625f : a.score_scale;
          f0 = load_query(a.q, a.q_dtype, qb + d0) * sc;
          f1 = load_query(a.q, a.q_dtype, qb + d1) * sc;
        }
        qf[m][j2][r] = h2_as_u32(__floats2half2_rn(f0, f1));
      }
  // Per group m and head column: the constant the raw encoding adds to the QK product,
  // C = sum_even 1032 q + sum_odd 1152 q/16 -- computed with the same mma from constant A rows,
  // so each group's accumulator starts at -C and ends at sum (code - 8) q exactly.
  float cneg[4][2];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    float c4[4];
    mma_16816_set(c4, 0x64086408u, 0x64086408u, 0x64806480u, 0x64806480u, qf[m][0][0],
                  qf[m][0][1], 0.f, 0.f);
    mma_16816(c4, 0x64086408u, 0x64086408u, 0x64806480u, 0x64806480u, qf[m][1][0], qf[m][1][1]);
    cneg[m][0] = -c4[0];
    cneg[m][1] = -c4[1];
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
#pragma unroll 1
  for (int i = 0; i < n_mine; ++i) {
    cp_async_wait<DEPTH - 2>();  // this lane's copies of tile i have landed
    __syncwarp();                // ... and every lane's
    const int rows = tile_rows[warp][slot];
    const uint32_t st = ring_s + slot * STAGE;
    const uint8_t* sp = ring + slot * STAGE;
    uint32_t kA[4], kB[4], vA[4], vB[4];
    ScaleRow<G> sk0, sk1, sv[4];
    if (rows == 16) {
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
    } else if (rows > 0) {  // partial tile: rows past the valid count re-read the last one
      ldsm_x4(st + ld_off, kA[0], kA[1], kA[2], kA[3]);
      ldsm_x4(st + ld_off + 8 * PD, kB[0], kB[1], kB[2], kB[3]);
      ldsm_x4_trans(st + OFF_V + ld_off, vA[0], vA[1], vA[2], vA[3]);
      ldsm_x4_trans(st + OFF_V + ld_off + 8 * PD, vB[0], vB[1], vB[2], vB[3]);
      const int last = rows - 1;
      sk0.load(sp + OFF_KS + min(g, last) * SB);
      sk1.load(sp + OFF_KS + min(g + 8, last) * SB);
      sv[0].load(sp + OFF_VS + min(2 * c, last) * SB);
      sv[1].load(sp + OFF_VS + min(2 * c + 1, last) * SB);
      sv[2].load(sp + OFF_VS + min(2 * c + 8, last) * SB);
      sv[3].load(sp + OFF_VS + min(2 * c + 9, last) * SB);
    }
    __syncwarp();         // the slot's data is in registers: it may be refilled
    issue(i + DEPTH - 1);  // into the slot consumed one iteration ago
    if (++slot == DEPTH) slot = 0;
    if (rows <= 0) continue;

    // ---- QK per scale group: r4 = sum_group (code - 8) q, then scaled by the K scale
    float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t p0[4], p1[4];
      magic_pairs(kA[m], p0);
      magic_pairs(kB[m], p1);
      float r4[4];
      mma_16816_set(r4, p0[0], p1[0], p0[1], p1[1], qf[m][0][0], qf[m][0][1], cneg[m][0],
                    cneg[m][1]);
      mma_16816(r4, p0[2], p1[2], p0[3], p1[3], qf[m][1][0], qf[m][1][1]);
      const int gi = (32 * m) / GROUP;
      const float s0 = __half2float(sk0.s[gi]), s1 = __half2float(sk1.s[gi]);
      x[0] = fmaf(r4[0], s0, x[0]);
      x[1] = fmaf(r4[1], s0, x[1]);
      x[2] = fmaf(r4[2], s1, x[2]);
      x[3] = fmaf(r4[3], s1, x[3]);
    }
    // ---- online softmax in the log2 domain; rows g, g+8 x heads 2c, 2c+1
    if (rows < 16) {
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
    float* dst = buf + static_cast<size_t>((sub - 1) * kvh + h) * kFields * 32 + lane;
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
  if (sub > 0) return;
  for (int o = 1; o < wph; ++o) {
    const float* src = buf + static_cast<size_t>((o - 1) * kvh + h) * kFields * 32 + lane;
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

using DecodeKernel = void (*)(const DecodeArgs);

// INT4, head_dim 128, group_size 32 or 64 (16-byte code chunks inside one scale group; scale
// rows of whole 4-byte words).
DecodeKernel async_decode_kernel_for(int bits, int d, int group) {
  if (bits != 4 || d != 128) return nullptr;
  switch (group) {
    case 32: return async_decode_kernel<32>;
    case 64: return async_decode_kernel<64>;
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
