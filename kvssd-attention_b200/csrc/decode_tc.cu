// Tensor-core split-KV decode over packed INT2/INT4 blocks (sm_100a).
//
// Replaces the per-query-head SIMT kernel of kvssd (csrc/fused_decode.cu:12-90) with a kernel
// in which one warp serves all query heads of a KV head, so each packed byte is read from
// HBM once however large the GQA ratio:
//
//   QK:  S[t, n]   = sum_d K[t, d] * Q[n, d]       mma m16n8k16, M = 16 tokens, N = 8 heads
//   PV:  O^T[d, n] = sum_t V[t, d] * P[t, n]       mma m16n8k16, M = 16 dims,   N = 8 heads
//
// Operand flow is register-only:
//   * thread (g = lane/4, c = lane%4) loads one contiguous K chunk (head_dim/4 codes, i.e. one
//     16-byte vector for INT4 d=128) of token rows g and g+8, and one V chunk (head_dim/8
//     codes) of token rows 2c, 2c+1, 2c+8, 2c+9 -- exactly the rows its A fragments need;
//   * codes are unpacked and scaled to FP16 in registers (common.cuh), bit-identical to
//     kvssd's dequantize_tensor(..., torch.float16); the reduction axis of QK is permuted to
//     the order the unpacker produces and Q is loaded in the same permuted order;
//   * S comes out of the QK mma in the C layout (rows = tokens); the online softmax runs on
//     it in the log2 domain, P is rounded to FP16 and transposed with movmatrix into the B
//     layout of the PV mma (rows = tokens), so P never touches shared memory.
// Each warp prefetches the next tile's bytes into registers while it computes the current one.
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

template <int GROUP, class S>
__device__ __forceinline__ void load_tile(const DecodeArgs& a, int blk, int rows, int off,
                                          int kvh_idx, int g, int c, TileRegs<S>& T) {
  T.rows = rows;
  if (rows <= 0) return;
  const size_t rs = static_cast<size_t>(a.kvh) * S::PD;
  const size_t srs = static_cast<size_t>(a.kvh) * S::G;
  const size_t row0 = static_cast<size_t>(blk) * a.bt + off;
  const uint8_t* kb = a.kp + row0 * rs + static_cast<size_t>(kvh_idx) * S::PD;
  const uint8_t* vb = a.vp + row0 * rs + static_cast<size_t>(kvh_idx) * S::PD;
  const __half* ksb = a.ks + row0 * srs + static_cast<size_t>(kvh_idx) * S::G;
  const __half* vsb = a.vs + row0 * srs + static_cast<size_t>(kvh_idx) * S::G;
  const int last = rows - 1;  // rows past the valid count re-read the last valid row
  const int kr[2] = {min(g, last), min(g + 8, last)};
  const int kg0 = (c * S::DK) / GROUP;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    VecBytes<S::CK>::load(kb + kr[h] * rs + c * S::CK, T.k[h]);
#pragma unroll
    for (int kg = 0; kg < S::KG; ++kg) T.ks[h][kg] = load_scale(ksb + kr[h] * srs + kg0 + kg);
  }
  const int vr[4] = {min(2 * c, last), min(2 * c + 1, last), min(2 * c + 8, last),
                     min(2 * c + 9, last)};
  const int vg0 = (g * S::DV) / GROUP;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    VecBytes<S::CV>::load(vb + vr[j] * rs + g * S::CV, T.v[j]);
#pragma unroll
    for (int vg = 0; vg < S::VG; ++vg) T.vs[j][vg] = load_scale(vsb + vr[j] * srs + vg0 + vg);
  }
}

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
  const float al0 = fast_exp2(m[0] - u0), al1 = fast_exp2(m[1] - u1);
  m[0] = n0;
  m[1] = n1;
  const float p0 = fast_exp2(x0 - u0), p1 = fast_exp2(x1 - u1);
  const float p2 = fast_exp2(x2 - u0), p3 = fast_exp2(x3 - u1);
  l[0] = fmaf(l[0], al0, p0 + p2);
  l[1] = fmaf(l[1], al1, p1 + p3);
#pragma unroll
  for (int i = 0; i < S::MT; ++i) {
    acc[i][0] *= al0;
    acc[i][1] *= al1;
    acc[i][2] *= al0;
    acc[i][3] *= al1;
  }
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

template <int BITS, int D, int GROUP>
__global__ void __launch_bounds__(256, (D >= 256 ? 1 : 2)) tc_decode_kernel(const DecodeArgs a) {
  using S = TcShape<BITS, D, GROUP>;
  // Let the dependent combine grid launch early; it waits for this grid's completion.
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int hl = warp % a.heads_per_cta, sub = warp / a.heads_per_cta;
  const int vh = blockIdx.y * a.heads_per_cta + hl;
  if (sub >= a.wph || vh >= a.n_vheads) return;
  const int kvh_idx = vh / a.n_qsub, qsub = vh - kvh_idx * a.n_qsub;
  const int q0 = kvh_idx * a.gqa + qsub * 8;
  const int nq = min(8, a.gqa - qsub * 8);

  // Q as the B operand of the QK mma, in the permuted reduction order of the unpacker.
  uint32_t qf[S::KSTEPS][2];
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

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[S::MT][4];
#pragma unroll
  for (int i = 0; i < S::MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  const long long t_end = a.total_tiles * (blockIdx.x + 1) / a.n_splits;
  long long t = a.total_tiles * blockIdx.x / a.n_splits + sub;
  BlockInfoCache cache;
  auto fetch = [&](long long tt, TileRegs<S>& T) {
    T.rows = 0;
    if (tt >= t_end) return;
    const int slot = static_cast<int>(tt / a.tiles_per_block);
    const int off = static_cast<int>(tt - static_cast<long long>(slot) * a.tiles_per_block) * 16;
    int blk, valid;
    cache.lookup(a, slot, lane, blk, valid);
    const int rows = min(valid - off, 16);
    if (blk >= 0 && rows > 0) load_tile<GROUP>(a, blk, rows, off, kvh_idx, g, c, T);
  };

  TileRegs<S> ta, tb;
  fetch(t, ta);
  while (t < t_end) {
    fetch(t + a.wph, tb);
    if (ta.rows > 0) compute_tile<BITS, GROUP>(ta, qf, a.score_scale, g, m, l, acc);
    t += a.wph;
    if (t >= t_end) break;
    fetch(t + a.wph, ta);
    if (tb.rows > 0) compute_tile<BITS, GROUP>(tb, qf, a.score_scale, g, m, l, acc);
    t += a.wph;
  }

  // ---- write this warp's part: l summed over the 8 row groups; m is already uniform.
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], o);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], o);
  }
  const size_t part = static_cast<size_t>(blockIdx.x) * a.wph + sub;
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

// Host-side table of instantiations. Returns nullptr for shapes the tensor-core path does
// not cover (the caller then uses the generic kernel).
using DecodeKernel = void (*)(const DecodeArgs);

template <int BITS, int D>
static DecodeKernel pick_group(int group) {
  switch (group) {
    case 16: return tc_decode_kernel<BITS, D, 16>;
    case 32: return tc_decode_kernel<BITS, D, 32>;
    case 64: return tc_decode_kernel<BITS, D, 64>;
    case 128: return D >= 128 ? tc_decode_kernel<BITS, D, (D >= 128 ? 128 : 64)> : nullptr;
    case 256: return D >= 256 ? tc_decode_kernel<BITS, D, (D >= 256 ? 256 : 64)> : nullptr;
    default: return nullptr;
  }
}

DecodeKernel tc_decode_kernel_for(int bits, int d, int group) {
  if (bits == 4) {
    if (d == 64) return pick_group<4, 64>(group);
    if (d == 128) return pick_group<4, 128>(group);
    if (d == 256) return pick_group<4, 256>(group);
  } else if (bits == 2) {
    if (d == 64) return pick_group<2, 64>(group);
    if (d == 128) return pick_group<2, 128>(group);
    if (d == 256) return pick_group<2, 256>(group);
  }
  return nullptr;
}

}  // namespace kvb
