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
#include "decode_tc.cuh"

namespace kvb {

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

  uint32_t qf[S::KSTEPS][2];
  load_query_fragments<S, D>(a, q0, nq, g, c, qf);

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[S::MT][4];
#pragma unroll
  for (int i = 0; i < S::MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  const long long t_begin = a.total_tiles * blockIdx.x / a.n_splits + sub;
  const int n_mine = t_begin < a.total_tiles * (blockIdx.x + 1) / a.n_splits
                         ? static_cast<int>((a.total_tiles * (blockIdx.x + 1) / a.n_splits -
                                             t_begin + a.wph - 1) / a.wph)
                         : 0;
  BlockInfoCache cache;
  TileCursor cur;
  cur.seek(t_begin, a.tiles_per_block);
  // Loads tile number `i` of this warp (tiles are visited in order, cursor advances by wph).
  auto fetch = [&](int i, TileRegs<S>& T) {
    T.rows = 0;
    if (i >= n_mine) return;
    int blk, valid;
    cache.lookup(a, cur.slot, lane, blk, valid);
    const int off = cur.row_offset();
    cur.advance(a.wph, a.tiles_per_block);
    const int rows = min(valid - off, 16);
    if (blk >= 0 && rows > 0) load_tile<GROUP>(a, blk, rows, off, kvh_idx, g, c, T);
  };

  TileRegs<S> ta, tb;
  fetch(0, ta);
  for (int i = 0; i < n_mine; i += 2) {
    fetch(i + 1, tb);
    if (ta.rows > 0) compute_tile<BITS, GROUP>(ta, qf, a.score_scale, g, m, l, acc);
    if (i + 1 >= n_mine) break;
    fetch(i + 2, ta);
    if (tb.rows > 0) compute_tile<BITS, GROUP>(tb, qf, a.score_scale, g, m, l, acc);
  }

  write_part<S, D>(a, static_cast<size_t>(blockIdx.x) * a.wph + sub, q0, nq, g, c, m, l, acc);
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
