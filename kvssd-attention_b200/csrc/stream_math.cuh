// Per-warp tile math of the streaming decode kernels (INT4 codes, head_dim 128, group 32 or
// 64): one warp serves one KV head and up to 8 of its query heads, and consumes 16-token tiles
// whose K and V rows (64 bytes per token) sit in shared memory with 16-byte chunk q of row r
// stored at chunk q ^ ((r >> 1) & 3), plus the tile's FP16 scale rows. The kernels differ only
// in how tiles reach shared memory (decode_async.cu: per-warp cp.async rings; decode_tma.cu:
// TMA copies into a CTA ring).
//
//   QK: S[t,n] = sum_group sk[t,group] * (sum_{d in group} (code-8)[t,d] * q[n,d]). The codes
//       enter the MMAs uncentred (even code slots as FP16 1024 + n, odd slots 1024 + 16n; one
//       LOP3 each), the odd slots' q is divided by 16, and the constant part -- per (scale
//       group, query head) Qg = sum 1032 q_even + 1152 q_odd/16 -- is subtracted by one more
//       MMA per tile whose A operand is the tile's K scale rows (the accumulator starts at
//       -sk x Qg). q is scaled by a per-warp power of two qs so |q| < 4 (Qg stays inside FP16
//       range); scores come out divided by qs and the softmax multiplies by 1/qs (exact).
//   PV: O^T[d,n] = sum_t (code-8)[t,d] * (P[t,n] * sv[t,group(d)]); the V scale is folded into
//       the FP16 P operand (P') of the M-tiles of that group; ldmatrix.trans delivers V with two
//       tokens per 32-bit register, the pairing the PV A fragment needs. Two forms of the V
//       codes (template flag VRAW; each feed is fastest with one of them, measured): centred
//       FP16 values (one LOP3 + one HSUB2/HFMA2 per pair), or -- VRAW -- the codes enter the
//       MMAs uncentred as exact FP16 subnormals (even code slots n * 2^-24, odd slots
//       n * 2^-20; one AND each), so the accumulator holds sum n P' scaled by 2^-24 / 2^-20;
//       the offset 8 * sum_t P' per (query head, scale group) is tracked by one more MMA per
//       tile, S += P^T sv (A = the transposed P the PV step already has, B = the tile's V scale
//       rows), and removed once per warp at the end (finish_stream). S sums the unrounded
//       products P sv rather than the FP16 P', which adds at most 8 x the FP16 rounding of P'
//       -- the same order as the rounding of P' itself.
//   Online softmax in the log2 domain (q pre-scaled by sm_scale * log2 e) with a lazily
//   updated running max: the max and the accumulator move only when a score exceeds the
//   running max by 2^8, detected with one warp vote per tile.
#pragma once

#include "combine.cuh"
#include "decode_tc.cuh"

namespace kvb {

constexpr int kStreamWarps = 16;  // consumer warps of a streaming CTA (warp w: KV head w % kvh)

// D = A * B (zero accumulator start).
__device__ __forceinline__ void mma_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// The B operands of one warp's QK MMAs and the K offset constants.
template <int GROUP>
struct QueryFrags {
  static constexpr int D = 128, G = D / GROUP;
  // k-step (m, j2) of thread c covers dims 32m + 8c + {2j2, 2j2+4} (b0, even code slots) and
  // 32m + 8c + {2j2+1, 2j2+5} (b1, odd code slots), the order in which a word's codes unpack.
  uint32_t qf[4][2][2];
  uint32_t qb[2];  // -Qg split over the four k-slices of the offset MMA (B operand)
  float unscale;   // 1 / qs

  // Query heads q0 .. q0 + nq - 1 (nq <= 8) of this warp from `q` (a.q, or a copy of it in
  // shared memory); thread (g, c) holds head g's q.
  __device__ __forceinline__ void load(const DecodeArgs& a, const void* q, int q0, int nq, int g,
                                       int c) {
    // Thread c needs dims 32m + 8c + 0..7 of chunk m: one 8-element load per chunk.
    float qv[4][8];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[m][e] = 0.f;
      if (g < nq) load_query8(q, a.q_dtype, static_cast<long long>(q0 + g) * D + 32 * m + 8 * c, qv[m]);
    }
    float qmax = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        qv[m][e] *= a.score_scale;
        qmax = fmaxf(qmax, fabsf(qv[m][e]));
      }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, o));
    const int qexp = (__float_as_uint(qmax) >> 23) & 0xff;
    // qmax * qs in [2, 4); qs = 1 for a zero or tiny query (and for non-finite ones).
    const float qs = (qexp >= 2 && qexp <= 253) ? __uint_as_float((255u - qexp) << 23) : 1.f;
    unscale = 1.f / qs;
    float qsum[4];  // this thread's share of chunk m's offset for query head g
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      qsum[m] = 0.f;
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          // dims d0 = 32m + 8c + 2j2 + r and d0 + 4
          const float sc = qs * (r ? 0.0625f : 1.f);
          const __half2 hq = __floats2half2_rn(qv[m][2 * j2 + r] * sc, qv[m][2 * j2 + r + 4] * sc);
          qf[m][j2][r] = h2_as_u32(hq);
          qsum[m] += (r ? 1152.f : 1032.f) * (__low2float(hq) + __high2float(hq));
        }
      qsum[m] += __shfl_xor_sync(0xffffffffu, qsum[m], 1);
      qsum[m] += __shfl_xor_sync(0xffffffffu, qsum[m], 2);
    }
    // Qg per scale group in two FP16 parts: hi = fp16(Qg / 2) from threads c = 0, 1, the
    // remainder Qg - 2 hi from c = 2, nothing from c = 3 (|Qg| < 2^17: no part overflows, and
    // the pair keeps ~22 bits of Qg).
    __half part[4];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      float qg = 0.f;
#pragma unroll
      for (int m = 0; m < 4; ++m)
        if ((32 * m) / GROUP == gi) qg += qsum[m];
      const __half hi = __float2half_rn(0.5f * qg);
      const __half lo = __float2half_rn(qg - 2.f * __half2float(hi));
      part[gi] = __hneg(c < 2 ? hi : c == 2 ? lo : __float2half_rn(0.f));
    }
    qb[0] = h2_as_u32(__halves2half2(part[0], part[1]));
    qb[1] = G == 4 ? h2_as_u32(__halves2half2(part[2], part[3])) : 0u;
  }
};

// One tile's operands in registers: K and V fragments of rows 0-7 (A) and 8-15 (B), the K scale
// rows of tokens g and g + 8 and the V scale rows of tokens 2c, 2c+1, 2c+8, 2c+9.
template <int G>
struct TileFrags {
  uint32_t kA[4], kB[4], vA[4], vB[4];
  ScaleRow<G> sk0, sk1, sv[4];

  // k_tile / v_tile: shared address of row 0 of the head's 16-row K / V tile (64-byte rows,
  // 512-byte aligned so the chunk swizzle is address-based); ld_off: this lane's ldmatrix
  // offset; sk / sv: generic pointers to the K scale row of token g and the V scale row of
  // token 2c; srow: bytes between consecutive scale rows; sv_odd: offset of token 2c + 1's V
  // scale row from token 2c's. The V fragments and scales are loaded before the K ones, so
  // once the QK MMAs have consumed K every shared-memory read of the tile has completed.
  template <int SROW>
  __device__ __forceinline__ void load(uint32_t k_tile, uint32_t v_tile, uint32_t ld_off,
                                       const uint8_t* sk, const uint8_t* sv_row, int sv_odd) {
    ldsm_x4_trans(v_tile + ld_off, vA[0], vA[1], vA[2], vA[3]);
    ldsm_x4_trans(v_tile + ld_off + 8 * 64, vB[0], vB[1], vB[2], vB[3]);
    sv[0].load(sv_row);
    sv[1].load(sv_row + sv_odd);
    sv[2].load(sv_row + 8 * SROW);
    sv[3].load(sv_row + 8 * SROW + sv_odd);
    sk0.load(sk);
    sk1.load(sk + 8 * SROW);
    ldsm_x4(k_tile + ld_off, kA[0], kA[1], kA[2], kA[3]);            // K tokens 0-7
    ldsm_x4(k_tile + ld_off + 8 * 64, kB[0], kB[1], kB[2], kB[3]);   // K tokens 8-15
  }
};

// Scale gi of a scale row as FP32, read straight from its 32-bit word (one conversion).
template <int G>
__device__ __forceinline__ float scale_f32(const ScaleRow<G>& r, int gi) {
  const __half2 w = u32_as_h2(r.word(gi >> 1));
  return (gi & 1) ? __high2float(w) : __low2float(w);
}

// (scale gi of row a, scale gi of row b) as one FP16 pair: one byte permute of the two words.
template <int G>
__device__ __forceinline__ __half2 scale_pair(const ScaleRow<G>& a, const ScaleRow<G>& b, int gi) {
  return u32_as_h2(__byte_perm(a.word(gi >> 1), b.word(gi >> 1), (gi & 1) ? 0x7632u : 0x5410u));
}

// Uncentred INT4 pairs as FP16 subnormals: even code slots n * 2^-24, odd slots 16n * 2^-24
// (one AND each).
__device__ __forceinline__ void subnormal_pairs4(uint32_t x, uint32_t (&o)[4]) {
  const uint32_t x8 = x >> 8;
  o[0] = x & 0x000F000Fu;
  o[1] = x & 0x00F000F0u;
  o[2] = x8 & 0x000F000Fu;
  o[3] = x8 & 0x00F000F0u;
}

struct StreamState {
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc[8][4];  // PV accumulators, uncentred and scaled (see finish_stream)
  float vs[4];      // S = sum_t P[t, head g] sv[t, group 2c + e] in vs[e] (e = 0, 1)
  __device__ __forceinline__ StreamState() {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    vs[0] = vs[1] = vs[2] = vs[3] = 0.f;
  }
};

// Scores of one tile (divided by qs): rows g, g+8 x heads 2c, 2c+1.
template <int GROUP>
__device__ __forceinline__ void qk_tile(const TileFrags<128 / GROUP>& t, const QueryFrags<GROUP>& q,
                                        float (&x)[4]) {
  constexpr int G = 128 / GROUP;
  mma_16816_zero(x, t.sk0.word(0), t.sk1.word(0), t.sk0.word(G == 4 ? 1 : 0),
                 t.sk1.word(G == 4 ? 1 : 0), q.qb[0], q.qb[1]);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint32_t p0[4], p1[4];
    raw_pairs4(t.kA[m], p0);
    raw_pairs4(t.kB[m], p1);
    float r4[4];
    mma_16816_zero(r4, p0[0], p1[0], p0[1], p1[1], q.qf[m][0][0], q.qf[m][0][1]);
    mma_16816(r4, p0[2], p1[2], p0[3], p1[3], q.qf[m][1][0], q.qf[m][1][1]);
    const int gi = (32 * m) / GROUP;
    const float s0 = scale_f32(t.sk0, gi), s1 = scale_f32(t.sk1, gi);
    x[0] = fmaf(r4[0], s0, x[0]);
    x[1] = fmaf(r4[1], s0, x[1]);
    x[2] = fmaf(r4[2], s1, x[2]);
    x[3] = fmaf(r4[3], s1, x[3]);
  }
}

// Online softmax of one tile's scores (rows g, g+8 x heads 2c, 2c+1; multiplied by `unscale`):
// moves the running max lazily, rescales the state, adds the tile's probabilities to l and
// returns them transposed for the PV B operand (pt0: tokens 2c, 2c+1 of head g; pt1: tokens
// 2c+8, 2c+9). rows: valid rows of the tile (rows past it hold stale codes and get no weight).
template <bool VRAW>
__device__ __forceinline__ void softmax_tile(float (&x)[4], int rows, int g, float unscale,
                                             StreamState& s, __half2& pt0, __half2& pt1) {
  constexpr float kLazyMax = 8.f;  // rescale only when a score beats the running max by 2^8
  if (rows < 16) {
    if (g >= rows) x[0] = x[1] = -INFINITY;
    if (g + 8 >= rows) x[2] = x[3] = -INFINITY;
  }
  // Scores relative to the running max: dx = x / qs - m.
  float dx[4] = {fmaf(x[0], unscale, -s.m_run[0]), fmaf(x[1], unscale, -s.m_run[1]),
                 fmaf(x[2], unscale, -s.m_run[0]), fmaf(x[3], unscale, -s.m_run[1])};
  const bool up = dx[0] > kLazyMax || dx[2] > kLazyMax || dx[1] > kLazyMax || dx[3] > kLazyMax;
  if (__any_sync(0xffffffffu, up)) {
    float t0 = fmaxf(x[0], x[2]), t1 = fmaxf(x[1], x[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
      t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
    }
    const float n0 = fmaxf(s.m_run[0], t0 * unscale), n1 = fmaxf(s.m_run[1], t1 * unscale);
    const float al0 = fast_exp2(s.m_run[0] - n0), al1 = fast_exp2(s.m_run[1] - n1);
    s.l_run[0] *= al0;
    s.l_run[1] *= al1;
    // S rows are query heads: head g's factor is al0 / al1 of the lanes with c = g / 2.
    const float a0g = __shfl_sync(0xffffffffu, al0, g >> 1);
    const float a1g = __shfl_sync(0xffffffffu, al1, g >> 1);
    const float alg = (g & 1) ? a1g : a0g;
    if (VRAW) {
      s.vs[0] *= alg;
      s.vs[1] *= alg;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s.acc[k][0] *= al0;
      s.acc[k][1] *= al1;
      s.acc[k][2] *= al0;
      s.acc[k][3] *= al1;
    }
    s.m_run[0] = n0;
    s.m_run[1] = n1;
    dx[0] = fmaf(x[0], unscale, -n0);
    dx[1] = fmaf(x[1], unscale, -n1);
    dx[2] = fmaf(x[2], unscale, -n0);
    dx[3] = fmaf(x[3], unscale, -n1);
  }
  const float e0 = fast_exp2(dx[0]), e1 = fast_exp2(dx[1]);
  const float e2 = fast_exp2(dx[2]), e3 = fast_exp2(dx[3]);
  s.l_run[0] += e0 + e2;
  s.l_run[1] += e1 + e3;
  pt0 = u32_as_h2(transpose_8x8(h2_as_u32(__floats2half2_rn(e0, e1))));
  pt1 = u32_as_h2(transpose_8x8(h2_as_u32(__floats2half2_rn(e2, e3))));
}

// Softmax plus the INT4 PV step. VRAW: subnormal V codes plus the S MMA.
template <int GROUP, bool VRAW>
__device__ __forceinline__ void softmax_pv_tile(float (&x)[4], int rows, int g, float unscale,
                                                const TileFrags<128 / GROUP>& t,
                                                StreamState& s) {
  __half2 pt0, pt1;
  softmax_tile<VRAW>(x, rows, g, unscale, s, pt0, pt1);
  // S += P^T sv: A rows = query heads (pt0 / pt1 hold tokens 2c, 2c+1 / 2c+8, 2c+9 of head g),
  // B columns = scale groups (thread (g, c) supplies group g's scales of those tokens).
  if (VRAW) {
    constexpr int G = 128 / GROUP;
    const int gs = g & (G - 1);
    const uint32_t sel = (gs & 1) ? 0x7632u : 0x5410u;
    const bool hi = G == 4 && (gs & 2);
    const uint32_t b0 = __byte_perm(hi ? t.sv[0].word(1) : t.sv[0].word(0),
                                    hi ? t.sv[1].word(1) : t.sv[1].word(0), sel);
    const uint32_t b1 = __byte_perm(hi ? t.sv[2].word(1) : t.sv[2].word(0),
                                    hi ? t.sv[3].word(1) : t.sv[3].word(0), sel);
    mma_16816(s.vs, h2_as_u32(pt0), 0u, h2_as_u32(pt1), 0u, b0, b1);
  }
  // PV per 32-dim chunk j (inside one scale group): P' = P * sv[t, group]
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gi = (32 * j) / GROUP;
    const __half2 b0 = __hmul2(pt0, scale_pair(t.sv[0], t.sv[1], gi));
    const __half2 b1 = __hmul2(pt1, scale_pair(t.sv[2], t.sv[3], gi));
    uint32_t cA[4], cB[4];
    if (VRAW) {
      subnormal_pairs4(t.vA[j], cA);
      subnormal_pairs4(t.vB[j], cB);
    } else {
      __half2 hA[4], hB[4];
      LanePairs<4>::centred(t.vA[j], hA);
      LanePairs<4>::centred(t.vB[j], hB);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        cA[u] = h2_as_u32(hA[u]);
        cB[u] = h2_as_u32(hB[u]);
      }
    }
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2)
      mma_16816(s.acc[2 * j + k2], cA[2 * k2], cA[2 * k2 + 1], cB[2 * k2], cB[2 * k2 + 1],
                h2_as_u32(b0), h2_as_u32(b1));
  }
}

// VRAW: turns the uncentred accumulators into sum_t (code - 8) P' (once per warp, after the
// stream): rows g of M-tile (j, k2) hold even code slots (scaled by 2^-24), rows g + 8 odd
// slots (2^-20); S for (head n, group gi) lives in lane 4n + gi / 2, element gi & 1.
template <int GROUP, bool VRAW>
__device__ __forceinline__ void finish_stream(StreamState& s, int c) {
  constexpr int G = 128 / GROUP;
  if constexpr (VRAW) {
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      const float v = (gi & 1) ? s.vs[1] : s.vs[0];
      const float s0 = 8.f * __shfl_sync(0xffffffffu, v, 4 * (2 * c) + (gi >> 1));
      const float s1 = 8.f * __shfl_sync(0xffffffffu, v, 4 * (2 * c + 1) + (gi >> 1));
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if ((16 * k) / GROUP != gi) continue;  // M-tile k covers dims 16k .. 16k + 15
        s.acc[k][0] = fmaf(s.acc[k][0], 16777216.f, -s0);
        s.acc[k][1] = fmaf(s.acc[k][1], 16777216.f, -s1);
        s.acc[k][2] = fmaf(s.acc[k][2], 1048576.f, -s0);
        s.acc[k][3] = fmaf(s.acc[k][3], 1048576.f, -s1);
      }
    }
  }
}

// ---------------- INT2 (head_dim 128): 32-byte rows, 64 codes per 16-byte chunk
//
// A 16-byte ldmatrix row of INT2 holds 64 codes -- two scale groups of 32 -- so the INT4 trick of
// factoring the scales out of each MMA does not apply: the tiles are dequantized in registers
// (centred code x FP16 scale, one HMUL2 per pair: exactly kvssd's FP16 dequantized values) and
// the MMAs run on those values. K: ldmatrix.x4 gives thread (g, c) the 16 codes of dims
// 64ch + 16c .. +15 of rows g (matrices 0, 1: chunks ch = 0, 1) and g + 8 (matrices 2, 3); its
// pair k (LanePairs<2>) holds dims (k, k + 8) of those 16, all in one scale group. V:
// ldmatrix.x4.trans gives tokens (2c, 2c+1) (matrices 0, 1) and (2c+8, 2c+9) (2, 3) of dims
// 64ch + 8g .. +7; pair k is dim 64ch + 8g + k of both tokens. PV M-tile (ch, u) takes pairs
// 2u (rows g: dim 64ch + 8g + 2u) and 2u + 1 (rows g + 8: the next dim).

// ldmatrix lane offset in a 16-row tile of 32-byte rows stored with the TMA's 32-byte swizzle
// (16-byte chunk q of row r at q ^ ((r >> 2) & 1)): matrix m = lane / 8 covers rows
// (m / 2) * 8 .. + 7, chunk m % 2.
__device__ __forceinline__ uint32_t ld_off_int2(int lane) {
  const int m = lane >> 3, row = (m >> 1) * 8 + (lane & 7), chunk = m & 1;
  return static_cast<uint32_t>(row * 32 + ((chunk ^ ((row >> 2) & 1)) << 4));
}

// Scale gi of a scale row broadcast to both halves (gi may differ per thread).
template <int G>
__device__ __forceinline__ __half2 scale_bcast(const ScaleRow<G>& r, int gi) {
  return u32_as_h2(__byte_perm(r.word(gi >> 1), 0u, (gi & 1) ? 0x3232u : 0x1010u));
}

template <int GROUP>
struct QueryFrags2 {
  static constexpr int D = 128;
  // MMA t (0..3) of chunk ch: b0 = dims 64ch + 16c + {2t, 2t + 8}, b1 = {2t + 1, 2t + 9}.
  uint32_t qf[2][4][2];
  __device__ __forceinline__ void load(const DecodeArgs& a, const void* q, int q0, int nq, int g,
                                       int c) {
    float lo[2][8], hi[2][8];  // dims 64ch + 16c + 0..7 and + 8..15
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
#pragma unroll
      for (int e = 0; e < 8; ++e) lo[ch][e] = hi[ch][e] = 0.f;
      if (g < nq) {
        const long long base = static_cast<long long>(q0 + g) * D + 64 * ch + 16 * c;
        load_query8(q, a.q_dtype, base, lo[ch]);
        load_query8(q, a.q_dtype, base + 8, hi[ch]);
      }
    }
#pragma unroll
    for (int ch = 0; ch < 2; ++ch)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        qf[ch][t][0] = h2_as_u32(__floats2half2_rn(lo[ch][2 * t] * a.score_scale,
                                                   hi[ch][2 * t] * a.score_scale));
        qf[ch][t][1] = h2_as_u32(__floats2half2_rn(lo[ch][2 * t + 1] * a.score_scale,
                                                   hi[ch][2 * t + 1] * a.score_scale));
      }
  }
};

template <int G>
struct TileFrags2 {
  uint32_t k[4], v[4];
  ScaleRow<G> sk0, sk1, sv[4];
  // As TileFrags::load (V and its scales first, K last), for 32-byte rows.
  template <int SROW>
  __device__ __forceinline__ void load(uint32_t k_tile, uint32_t v_tile, uint32_t ld_off,
                                       const uint8_t* sk, const uint8_t* sv_row, int sv_odd) {
    ldsm_x4_trans(v_tile + ld_off, v[0], v[1], v[2], v[3]);
    sv[0].load(sv_row);
    sv[1].load(sv_row + sv_odd);
    sv[2].load(sv_row + 8 * SROW);
    sv[3].load(sv_row + 8 * SROW + sv_odd);
    sk0.load(sk);
    sk1.load(sk + 8 * SROW);
    ldsm_x4(k_tile + ld_off, k[0], k[1], k[2], k[3]);
  }
};

// Scores of one INT2 tile (rows g, g+8 x heads 2c, 2c+1), in the log2 domain.
template <int GROUP>
__device__ __forceinline__ void qk_tile2(const TileFrags2<128 / GROUP>& t,
                                         const QueryFrags2<GROUP>& q, int c, float (&x)[4]) {
  x[0] = x[1] = x[2] = x[3] = 0.f;
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    const int gk = (64 * ch + 16 * c) / GROUP;
    const __half2 s0 = scale_bcast(t.sk0, gk), s1 = scale_bcast(t.sk1, gk);
    __half2 pa[8], pb[8];
    LanePairs<2>::centred(t.k[ch], pa);
    LanePairs<2>::centred(t.k[2 + ch], pb);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      pa[i] = __hmul2(pa[i], s0);
      pb[i] = __hmul2(pb[i], s1);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      mma_16816(x, h2_as_u32(pa[2 * u]), h2_as_u32(pb[2 * u]), h2_as_u32(pa[2 * u + 1]),
                h2_as_u32(pb[2 * u + 1]), q.qf[ch][u][0], q.qf[ch][u][1]);
  }
}

// Softmax plus the INT2 PV step (acc[4ch + u]: dims 64ch + 8g + 2u (rows g) and + 1).
template <int GROUP>
__device__ __forceinline__ void softmax_pv_tile2(float (&x)[4], int rows, int g,
                                                 const TileFrags2<128 / GROUP>& t,
                                                 StreamState& s) {
  __half2 pt0, pt1;
  softmax_tile<false>(x, rows, g, 1.f, s, pt0, pt1);
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    const int gv = (64 * ch + 8 * g) / GROUP;
    const __half2 sa = scale_pair(t.sv[0], t.sv[1], gv), sb = scale_pair(t.sv[2], t.sv[3], gv);
    __half2 ca[8], cb[8];
    LanePairs<2>::centred(t.v[ch], ca);
    LanePairs<2>::centred(t.v[2 + ch], cb);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ca[i] = __hmul2(ca[i], sa);
      cb[i] = __hmul2(cb[i], sb);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      mma_16816(s.acc[4 * ch + u], h2_as_u32(ca[2 * u]), h2_as_u32(ca[2 * u + 1]),
                h2_as_u32(cb[2 * u]), h2_as_u32(cb[2 * u + 1]), h2_as_u32(pt0), h2_as_u32(pt1));
  }
}

// Shared-memory bytes the in-CTA merge needs (the 16 - kvh non-leading warps' states).
__host__ __device__ constexpr size_t stream_merge_bytes(int kvh) {
  return static_cast<size_t>(kStreamWarps - kvh) * 32 * (4 + 4 * 8) * 4;
}

// Merges the 16 / KVH consumer warps of each KV head through shared memory `buf` and writes
// the CTA's part (m, l, acc) for query heads q0 .. q0 + nq - 1. Every thread of the CTA calls
// it (warps >= 16 only synchronise); `buf` must no longer be written by copies in flight.
template <int KVH, int BITS = 4>
__device__ __forceinline__ void merge_warps_write_part(const DecodeArgs& a, float* buf, int warp,
                                                       int lane, int q0, int nq,
                                                       StreamState& s, unsigned tag) {
  constexpr int kFields = 4 + 4 * 8, WPH = kStreamWarps / KVH, D = 128;
  const int g = lane >> 2, c = lane & 3;
  const bool consumer = warp < kStreamWarps;
  const int h = warp % KVH, sub = warp / KVH;
  if (consumer && sub > 0) {
    float* dst = buf + static_cast<size_t>((sub - 1) * KVH + h) * kFields * 32 + lane;
    dst[0] = s.m_run[0];
    dst[32] = s.m_run[1];
    dst[64] = s.l_run[0];
    dst[96] = s.l_run[1];
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[(4 + 4 * k + e) * 32] = s.acc[k][e];
  }
  __syncthreads();
  if (!consumer || sub != 0) return;
  for (int o = 1; o < WPH; ++o) {
    const float* src = buf + static_cast<size_t>((o - 1) * KVH + h) * kFields * 32 + lane;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float mo = src[hh * 32], lo = src[(2 + hh) * 32];
      const float mn = fmaxf(s.m_run[hh], mo);
      const float a0 = mn == -INFINITY ? 0.f : fast_exp2(s.m_run[hh] - mn);
      const float a1 = mn == -INFINITY ? 0.f : fast_exp2(mo - mn);
      s.m_run[hh] = mn;
      s.l_run[hh] = s.l_run[hh] * a0 + lo * a1;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        s.acc[k][hh] = s.acc[k][hh] * a0 + src[(4 + 4 * k + hh) * 32] * a1;
        s.acc[k][2 + hh] = s.acc[k][2 + hh] * a0 + src[(4 + 4 * k + 2 + hh) * 32] * a1;
      }
    }
  }
  // This CTA's part. INT4: O^T row g of M-tile 2j + k2 is dim 32j + 4g + 2k2; INT2: row g of
  // M-tile 4ch + u is dim 64ch + 8g + 2u; row g+8 is the next dim in both.
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    s.l_run[0] += __shfl_xor_sync(0xffffffffu, s.l_run[0], o);
    s.l_run[1] += __shfl_xor_sync(0xffffffffu, s.l_run[1], o);
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int n = 2 * c + hh;
    if (n >= nq) continue;
    const size_t row = static_cast<size_t>(blockIdx.x) * a.qh + (q0 + n);
    const size_t col = (BITS == 4 ? 4 : 8) * g;
    if (a.fuse_combine) {  // tagged words, polled by the fused combine
      unsigned long long* tml = reinterpret_cast<unsigned long long*>(a.part_ml);
      if (g == 0) st_tagged2(tml + row * 2, tag_word(s.m_run[hh], tag), tag_word(s.l_run[hh], tag));
      unsigned long long* dst = a.tpart_acc + row * D + col;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int off = BITS == 4 ? 32 * (k >> 1) + 2 * (k & 1) : 64 * (k >> 2) + 2 * (k & 3);
        st_tagged2(dst + off, tag_word(s.acc[k][hh], tag), tag_word(s.acc[k][2 + hh], tag));
      }
      continue;
    }
    if (g == 0) {
      a.part_ml[row * 2 + 0] = s.m_run[hh];
      a.part_ml[row * 2 + 1] = s.l_run[hh];
    }
    float* dst = a.part_acc + row * D + col;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int off = BITS == 4 ? 32 * (k >> 1) + 2 * (k & 1) : 64 * (k >> 2) + 2 * (k & 3);
      *reinterpret_cast<float2*>(dst + off) = make_float2(s.acc[k][hh], s.acc[k][2 + hh]);
    }
  }
}

}  // namespace kvb
