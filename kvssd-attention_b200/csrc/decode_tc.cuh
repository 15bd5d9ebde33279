// Tile math shared by the tensor-core decode kernels (register-fed and TMA-fed).
//
// A tile is 16 token rows of one block for one KV head. Thread (g = lane/4, c = lane%4) owns
//   * the K chunk (head_dim/4 codes) of token rows g and g+8 -- the rows and reduction
//     columns of its QK A fragments (m16n8k16: M = 16 tokens, N = 8 query heads);
//   * the V chunk (head_dim/8 codes, dims g*head_dim/8 ...) of token rows 2c, 2c+1, 2c+8,
//     2c+9 -- the rows of its PV A fragments (M = 16 dims, N = 8 heads, K = 16 tokens).
// compute_tile() turns one tile into an online-softmax update of (m, l, acc).
#pragma once

#include <cmath>

#include "common.cuh"
#include "decode.cuh"

namespace kvb {

template <int BITS, int D, int GROUP>
struct TcShape {
  static constexpr int PD = D * BITS / 8;        // packed bytes per (token, KV head)
  static constexpr int CK = PD / 4;              // bytes of one thread's K chunk
  static constexpr int CV = PD / 8;              // bytes of one thread's V chunk
  static constexpr int DK = D / 4;               // dims per K chunk
  static constexpr int DV = D / 8;               // dims per V chunk
  static constexpr int G = D / GROUP;            // scale groups per (token, KV head)
  static constexpr int KW = CK / 4;              // 32-bit words per K chunk
  static constexpr int VHW = CV / 2;             // 16-bit lanes per V chunk
  static constexpr int VW = CV >= 4 ? CV / 4 : 1;
  static constexpr int PPL = 16 / BITS;          // codes per 16-bit lane (pairs per word)
  static constexpr int DPW = 32 / BITS;          // dims per 32-bit word
  static constexpr int KSTEPS = D / 16;
  static constexpr int MT = D / 16;
  static constexpr int KG = DK >= GROUP ? DK / GROUP : 1;
  static constexpr int VG = DV >= GROUP ? DV / GROUP : 1;
  static_assert(CK >= 4 && CV >= 2, "tensor-core path needs head_dim*bits >= 128");
  static_assert(GROUP >= 16 && D % GROUP == 0, "tensor-core path needs group >= 16");
};

template <class S>
struct TileRegs {
  uint32_t k[2][S::KW];   // K chunk of rows g, g+8
  uint32_t v[4][S::VW];   // V chunk of rows 2c, 2c+1, 2c+8, 2c+9
  __half ks[2][S::KG];
  __half vs[4][S::VG];
  int rows;               // valid rows of the tile; 0 = nothing to do
};

template <int BITS, int GROUP, class S>
__device__ __forceinline__ void compute_tile(const TileRegs<S>& T,
                                             const uint32_t (&qf)[S::KSTEPS][2],
                                             float score_scale, int g, float (&m)[2],
                                             float (&l)[2], float (&acc)[S::MT][4]) {
  // ---- S = K Q^T for 16 tokens x 8 heads
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < S::KW; ++w) {
    const int kg = (w * S::DPW) / GROUP;
    __half2 r0[S::PPL], r1[S::PPL];
    dequant_pairs<BITS>(T.k[0][w], __half2half2(T.ks[0][kg]), r0);
    dequant_pairs<BITS>(T.k[1][w], __half2half2(T.ks[1][kg]), r1);
#pragma unroll
    for (int k2 = 0; k2 < S::PPL; k2 += 2) {
      const int j = (w * S::PPL + k2) / 2;
      mma_16816(s, h2_as_u32(r0[k2]), h2_as_u32(r1[k2]), h2_as_u32(r0[k2 + 1]),
                h2_as_u32(r1[k2 + 1]), qf[j][0], qf[j][1]);
    }
  }
  // ---- online softmax; thread holds rows (g, g+8) x heads (2c, 2c+1)
  const bool v0 = g < T.rows, v1 = g + 8 < T.rows;
  const float x0 = v0 ? s[0] * score_scale : -INFINITY;
  const float x1 = v0 ? s[1] * score_scale : -INFINITY;
  const float x2 = v1 ? s[2] * score_scale : -INFINITY;
  const float x3 = v1 ? s[3] * score_scale : -INFINITY;
  float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
    t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
  }
  const float n0 = fmaxf(m[0], t0), n1 = fmaxf(m[1], t1);
  const float u0 = n0 == -INFINITY ? 0.f : n0;  // all rows so far masked: keep p = 0
  const float u1 = n1 == -INFINITY ? 0.f : n1;
  // The accumulator is rescaled only when some head's running max moved in this warp
  // (after the first tiles the max rarely changes, so the 4*MT multiplies are skipped).
  if (__any_sync(0xffffffffu, (n0 > m[0]) || (n1 > m[1]))) {
    const float al0 = fast_exp2(m[0] - u0), al1 = fast_exp2(m[1] - u1);
    l[0] *= al0;
    l[1] *= al1;
#pragma unroll
    for (int i = 0; i < S::MT; ++i) {
      acc[i][0] *= al0;
      acc[i][1] *= al1;
      acc[i][2] *= al0;
      acc[i][3] *= al1;
    }
  }
  m[0] = n0;
  m[1] = n1;
  const float p0 = fast_exp2(x0 - u0), p1 = fast_exp2(x1 - u1);
  const float p2 = fast_exp2(x2 - u0), p3 = fast_exp2(x3 - u1);
  l[0] += p0 + p2;
  l[1] += p1 + p3;
  const uint32_t pt0 = transpose_8x8(h2_as_u32(__floats2half2_rn(p0, p1)));
  const uint32_t pt1 = transpose_8x8(h2_as_u32(__floats2half2_rn(p2, p3)));
  // ---- O^T += V^T P for 16 tokens
#pragma unroll
  for (int hw = 0; hw < S::VHW; ++hw) {
    const int wi = hw >> 1, hs = hw & 1;
    const int vg = (hw * S::PPL) / GROUP;
    const uint32_t x01 = pair_lanes(T.v[0][wi], T.v[1][wi], hs);
    const uint32_t x89 = pair_lanes(T.v[2][wi], T.v[3][wi], hs);
    __half2 r01[S::PPL], r89[S::PPL];
    dequant_pairs<BITS>(x01, __halves2half2(T.vs[0][vg], T.vs[1][vg]), r01);
    dequant_pairs<BITS>(x89, __halves2half2(T.vs[2][vg], T.vs[3][vg]), r89);
#pragma unroll
    for (int k2 = 0; k2 < S::PPL; k2 += 2) {
      const int i = (hw * S::PPL + k2) / 2;
      mma_16816(acc[i], h2_as_u32(r01[k2]), h2_as_u32(r01[k2 + 1]), h2_as_u32(r89[k2]),
                h2_as_u32(r89[k2 + 1]), pt0, pt1);
    }
  }
}

// Position of a tile in the selection (slot in the block table, 16-row offset in the block),
// advanced incrementally so the per-tile loop needs no integer division.
struct TileCursor {
  int slot = 0;
  int tile_in_block = 0;
  __device__ __forceinline__ void seek(long long tile, int tiles_per_block) {
    slot = static_cast<int>(tile / tiles_per_block);
    tile_in_block = static_cast<int>(tile - static_cast<long long>(slot) * tiles_per_block);
  }
  __device__ __forceinline__ void advance(int n, int tiles_per_block) {
    tile_in_block += n;
    while (tile_in_block >= tiles_per_block) {
      tile_in_block -= tiles_per_block;
      ++slot;
    }
  }
  __device__ __forceinline__ int row_offset() const { return tile_in_block * 16; }
};

// Q as the B operand of the QK mma, in the permuted reduction order of the unpacker:
// pair p of thread c covers dims c*DK + (p/PPL)*DPW + p%PPL and that + DPW/2.
template <class S, int D>
__device__ __forceinline__ void load_query_fragments(const DecodeArgs& a, int q0, int nq, int g,
                                                     int c, uint32_t (&qf)[S::KSTEPS][2]) {
#pragma unroll
  for (int j = 0; j < S::KSTEPS; ++j) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int p = 2 * j + r;
      const int d0 = c * S::DK + (p / S::PPL) * S::DPW + (p % S::PPL);
      const int d1 = d0 + S::DPW / 2;
      float f0 = 0.f, f1 = 0.f;
      if (g < nq) {
        const long long base = static_cast<long long>(q0 + g) * D;
        f0 = load_query(a.q, a.q_dtype, base + d0);
        f1 = load_query(a.q, a.q_dtype, base + d1);
      }
      qf[j][r] = h2_as_u32(__floats2half2_rn(f0, f1));
    }
  }
}

// Writes one warp's state as a part: l summed over the 8 row groups (m is uniform).
template <class S, int D>
__device__ __forceinline__ void write_part(const DecodeArgs& a, size_t part, int q0, int nq,
                                           int g, int c, float (&m)[2], float (&l)[2],
                                           float (&acc)[S::MT][4]) {
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], o);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], o);
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int n = 2 * c + hh;
    if (n >= nq) continue;
    const size_t row = part * a.qh + (q0 + n);
    if (g == 0) {
      a.part_ml[row * 2 + 0] = m[hh];
      a.part_ml[row * 2 + 1] = l[hh];
    }
    float* dst = a.part_acc + row * D + g * S::DV;
#pragma unroll
    for (int i = 0; i < S::MT; ++i)
      *reinterpret_cast<float2*>(dst + 2 * i) = make_float2(acc[i][hh], acc[i][2 + hh]);
  }
}

}  // namespace kvb
