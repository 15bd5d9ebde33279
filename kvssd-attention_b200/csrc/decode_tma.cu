// TMA-fed split-KV decode for INT4 codes (sm_100a): tensor-map bulk loads stream token rows of
// packed KV into a swizzled shared-memory ring; ldmatrix feeds the tensor cores.
//
// Work: one CTA per SM owns a contiguous range of 16-token tiles of the selection for ALL KV
// heads (every tile it loads is a contiguous run of token rows: kvssd's record layout
// interleaves the KV heads of a token, src/kvssd/format.py:165). 16 warps; warp w serves KV head
// w % kv_heads and takes every wph-th tile (wph = 16 / kv_heads).
//
// Loads: the K and V pools are viewed as 2-D tensor maps [token rows][kv_heads*64 bytes]; one
// tile is kv_heads/2 boxes of 16 rows x 128 bytes (two KV heads) for K and as many for V, with
// the 128-byte hardware swizzle (16-byte chunk c of row t lands at chunk c ^ (t & 7)), plus one
// plain bulk copy per scale region. Warp 0 also keeps the ring full: it arms a stage's
// mbarrier with the tile's byte count and issues the copies, checking free stages without
// blocking between its own tiles.
//
// Fragments: ldmatrix (K) and ldmatrix.trans (V) read the swizzled rows without bank
// conflicts; .trans also interleaves two tokens per 32-bit register, which is exactly the
// pairing of the PV A fragment. With 32 dims per 16-byte chunk and group_size >= 32 every
// k-step of QK and every M-tile of PV lies inside one scale group, so the FP16 scales are not
// multiplied into the codes at all:
//   QK: S[t,n] = sum_group sk[t,group] * (sum_{d in group} (code-mid)[t,d] * q[n,d])
//       -- two mma per group into a fresh FP32 accumulator, then one FFMA per element;
//   PV: O^T[d,n] = sum_t (code-mid)[t,d] * (P[t,n] * sv[t,group(d)]) -- the V scale is folded
//       into the FP16 P operand of the M-tiles of that group.
// The centred codes are exact small integers, so the products inside the mma are exact.
// Every mbarrier wait is bounded (%globaltimer); a timeout sets status bit 4 and the kernel
// unwinds after waiting (bounded) for its own copies in flight.
#include "decode_tc.cuh"
#include "tma.cuh"

namespace kvb {

constexpr int kTmaWarps = 16;
constexpr int kTmaThreads = 32 * kTmaWarps;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s
constexpr int kBoxBytes = 16 * 128;                         // one box: 16 rows x 128 bytes

template <int G>
struct ScaleRow {  // the G FP16 scales of one (token, KV head)
  __half s[G];
  __device__ __forceinline__ void load(const __half* p) {
    if constexpr (G == 4) {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      memcpy(s, &w, 8);
    } else if constexpr (G == 2) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
      memcpy(s, &w, 4);
    } else {
      s[0] = *p;
    }
  }
};

template <int GROUP>
__global__ void __launch_bounds__(kTmaThreads, 1)
    tma_decode_kernel(const DecodeArgs a, const __grid_constant__ TmaMaps maps) {
  constexpr int D = 128, BITS = 4, G = D / GROUP, MT = D / 16;
  extern __shared__ uint8_t smem_raw[];
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;

  // 1024-byte aligned ring (the swizzle pattern repeats every 1024 bytes)
  const uint32_t raw_base = smem_addr(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + a.stages;
  int* stage_rows = reinterpret_cast<int*>(empty + a.stages);
  const uint32_t ring = base + a.ring_offset;
  uint8_t* ring_ptr = smem + a.ring_offset;
  const unsigned long long deadline = global_timer_ns() + kWaitLimitNs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(smem_addr(full + s), 1);
      mbar_init(smem_addr(empty + s), a.kvh);
    }
    mbar_init_fence();
    prefetch_tmap(&maps.k);
    prefetch_tmap(&maps.v);
  }
  __syncthreads();

  const long long t_begin = a.total_tiles * blockIdx.x / a.n_splits;
  const int n_tiles = static_cast<int>(a.total_tiles * (blockIdx.x + 1) / a.n_splits - t_begin);
  const int boxes = a.kvh >> 1;
  const uint32_t box_bytes = static_cast<uint32_t>(boxes) * kBoxBytes;
  const long long total_rows = static_cast<long long>(a.n_pool) * a.bt;
  bool ok = true;

  // ---------------- ring filling (warp 0)
  BlockInfoCache cache;
  TileCursor cur;
  int nf = 0, fs = 0;
  uint32_t fparity = 1u;  // a fresh barrier reports the phase before its first as complete
  uint64_t policy = 0;
  if (warp == 0) {
    cur.seek(t_begin, a.tiles_per_block);
    policy = l2_evict_first_policy();
  }
  auto fill_one = [&]() {  // warp 0, warp-uniform; the stage's empty phase has completed
    const int off = cur.row_offset();
    int blk, valid;
    cache.lookup(a, cur.slot, lane, blk, valid);
    cur.advance(1, a.tiles_per_block);
    const int rows = blk >= 0 ? max(0, min(valid - off, 16)) : 0;
    const uint32_t bar = smem_addr(full + fs);
    const long long row0 = static_cast<long long>(blk) * a.bt + off;
    const int scale_rows = rows > 0 ? static_cast<int>(min(16LL, total_rows - row0)) : 0;
    if (lane == 0) {
      stage_rows[fs] = rows;
      mbar_arrive_expect_tx(bar, rows > 0 ? 2u * box_bytes + 2u * scale_rows * a.srb : 0u);
    }
    __syncwarp();
    if (rows > 0) {
      const uint32_t st = ring + static_cast<uint32_t>(fs) * a.stage_bytes;
      if (lane < boxes)
        tma_load_2d(st + lane * kBoxBytes, &maps.k, lane * 128, static_cast<int>(row0), bar, policy);
      else if (lane >= 16 && lane < 16 + boxes)
        tma_load_2d(st + a.off_v + (lane - 16) * kBoxBytes, &maps.v, (lane - 16) * 128,
                    static_cast<int>(row0), bar, policy);
      else if (lane == 14)
        bulk_g2s(st + a.off_ks, reinterpret_cast<const uint8_t*>(a.ks) + row0 * a.srb,
                 scale_rows * a.srb, bar, policy);
      else if (lane == 30)
        bulk_g2s(st + a.off_vs, reinterpret_cast<const uint8_t*>(a.vs) + row0 * a.srb,
                 scale_rows * a.srb, bar, policy);
    }
    ++nf;
    if (++fs == a.stages) {
      fs = 0;
      fparity ^= 1u;
    }
  };
  // Fills while stages are free without waiting; if `need` >= 0, first blocks (bounded) until
  // tile `need` has been issued.
  auto refill = [&](int need) {
    while (ok && nf < n_tiles) {
      const uint32_t bar = smem_addr(empty + fs);
      if (nf <= need) {
        if (!mbar_wait_bounded(bar, fparity, deadline)) {
          ok = false;
          break;
        }
      } else if (!mbar_test_wait(bar, fparity)) {
        break;
      }
      fill_one();
    }
  };
  if (warp == 0) refill(-1);

  // ---------------- consumers (all warps)
  const int h = warp % a.kvh, sub = warp / a.kvh;
  const int q0 = h * a.gqa, nq = a.gqa;
  // Q as the B operand: k-step (m, j2) of thread c covers dims 32m + 8c + {2j2, 2j2+4}
  // (b0) and 32m + 8c + {2j2+1, 2j2+5} (b1), the order the ldmatrix/unpack path produces.
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
          f0 = load_query(a.q, a.q_dtype, qb + d0);
          f1 = load_query(a.q, a.q_dtype, qb + d1);
        }
        qf[m][j2][r] = h2_as_u32(__floats2half2_rn(f0, f1));
      }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  // ldmatrix row addresses (relative to a stage): lane supplies row (lane & 7) of the matrix
  // for 16-byte chunk (lane >> 3) of head h, swizzled by the row index.
  const int ld_row = lane & 7, ld_chunk = ((h & 1) << 2) | (lane >> 3);
  const uint32_t ld_off = static_cast<uint32_t>((h >> 1) * kBoxBytes + ld_row * 128 +
                                                ((ld_chunk ^ ld_row) << 4));
  const int sh = h * G;  // scale-row offset of head h (halves)

  int s = sub % a.stages;
  uint32_t parity = static_cast<uint32_t>((sub / a.stages) & 1);
  for (int k = sub; k < n_tiles; k += a.wph) {
    if (warp == 0) refill(k);
    if (!ok || !mbar_wait_bounded(smem_addr(full + s), parity, deadline)) {
      ok = false;
      break;
    }
    const int rows = stage_rows[s];
    const uint32_t st = ring + static_cast<uint32_t>(s) * a.stage_bytes;
    const uint8_t* stp = ring_ptr + static_cast<size_t>(s) * a.stage_bytes;
    uint32_t kA[4], kB[4], vA[4], vB[4];
    ScaleRow<G> sk0, sk1, sv[4];
    if (rows > 0) {
      ldsm_x4(st + ld_off, kA[0], kA[1], kA[2], kA[3]);               // K tokens 0-7
      ldsm_x4(st + ld_off + 8 * 128, kB[0], kB[1], kB[2], kB[3]);     // K tokens 8-15
      ldsm_x4_trans(st + a.off_v + ld_off, vA[0], vA[1], vA[2], vA[3]);
      ldsm_x4_trans(st + a.off_v + ld_off + 8 * 128, vB[0], vB[1], vB[2], vB[3]);
      const int last = rows - 1;
      const __half* ks = reinterpret_cast<const __half*>(stp + a.off_ks);
      const __half* vs = reinterpret_cast<const __half*>(stp + a.off_vs);
      const int rstride = a.kvh * G;  // halves per token row of scales
      sk0.load(ks + min(g, last) * rstride + sh);
      sk1.load(ks + min(g + 8, last) * rstride + sh);
      sv[0].load(vs + min(2 * c, last) * rstride + sh);
      sv[1].load(vs + min(2 * c + 1, last) * rstride + sh);
      sv[2].load(vs + min(2 * c + 8, last) * rstride + sh);
      sv[3].load(vs + min(2 * c + 9, last) * rstride + sh);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(empty + s));
    if (warp == 0) refill(-1);
    if (rows > 0) {
      // ---- QK per scale group
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        __half2 p0[4], p1[4];
        LanePairs<BITS>::centred(kA[m], p0);
        LanePairs<BITS>::centred(kB[m], p1);
        float r[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j2 = 0; j2 < 2; ++j2)
          mma_16816(r, h2_as_u32(p0[2 * j2]), h2_as_u32(p1[2 * j2]), h2_as_u32(p0[2 * j2 + 1]),
                    h2_as_u32(p1[2 * j2 + 1]), qf[m][j2][0], qf[m][j2][1]);
        const int gi = (32 * m) / GROUP;
        const float s0 = __half2float(sk0.s[gi]), s1 = __half2float(sk1.s[gi]);
        sc[0] = fmaf(r[0], s0, sc[0]);
        sc[1] = fmaf(r[1], s0, sc[1]);
        sc[2] = fmaf(r[2], s1, sc[2]);
        sc[3] = fmaf(r[3], s1, sc[3]);
      }
      // ---- online softmax (log2 domain); rows g, g+8 x heads 2c, 2c+1
      const bool v0 = g < rows, v1 = g + 8 < rows;
      const float x0 = v0 ? sc[0] * a.score_scale : -INFINITY;
      const float x1 = v0 ? sc[1] * a.score_scale : -INFINITY;
      const float x2 = v1 ? sc[2] * a.score_scale : -INFINITY;
      const float x3 = v1 ? sc[3] * a.score_scale : -INFINITY;
      float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
      }
      const float n0 = fmaxf(m_run[0], t0), n1 = fmaxf(m_run[1], t1);
      const float u0 = n0 == -INFINITY ? 0.f : n0, u1 = n1 == -INFINITY ? 0.f : n1;
      if (__any_sync(0xffffffffu, (n0 > m_run[0]) || (n1 > m_run[1]))) {
        const float al0 = fast_exp2(m_run[0] - u0), al1 = fast_exp2(m_run[1] - u1);
        l_run[0] *= al0;
        l_run[1] *= al1;
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          acc[i][0] *= al0;
          acc[i][1] *= al1;
          acc[i][2] *= al0;
          acc[i][3] *= al1;
        }
      }
      m_run[0] = n0;
      m_run[1] = n1;
      const float e0 = fast_exp2(x0 - u0), e1 = fast_exp2(x1 - u1);
      const float e2 = fast_exp2(x2 - u0), e3 = fast_exp2(x3 - u1);
      l_run[0] += e0 + e2;
      l_run[1] += e1 + e3;
      const __half2 pt0 = u32_as_h2(transpose_8x8(h2_as_u32(__floats2half2_rn(e0, e1))));
      const __half2 pt1 = u32_as_h2(transpose_8x8(h2_as_u32(__floats2half2_rn(e2, e3))));
      // ---- PV per 32-dim chunk j (one scale group): P' = P * sv[t, group]
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
    s += a.wph;
    while (s >= a.stages) {
      s -= a.stages;
      parity ^= 1u;
    }
  }
  if (warp == 0) {
    refill(n_tiles);  // issue every remaining tile (other warps still need them)
    // Do not retire while copies this warp issued may still be landing in shared memory.
    int ws = 0;
    uint32_t wp = 0;
    for (int t = 0; t < nf; ++t) {
      if (t + a.stages >= nf &&
          !mbar_wait_bounded(smem_addr(full + ws), wp, deadline + kWaitLimitNs)) {
        ok = false;
        break;
      }
      if (++ws == a.stages) {
        ws = 0;
        wp ^= 1u;
      }
    }
  }
  if (!ok && lane == 0) atomicOr(a.status, kDevPipelineTimeout);

  // ---- merge the wph warps of each head through the drained ring: [slot][field][lane]
  __syncthreads();
  constexpr int kFields = 4 + 4 * MT;
  float* buf = reinterpret_cast<float*>(ring_ptr);
  if (sub > 0) {
    float* dst = buf + static_cast<size_t>((sub - 1) * a.kvh + h) * kFields * 32 + lane;
    dst[0] = m_run[0];
    dst[32] = m_run[1];
    dst[64] = l_run[0];
    dst[96] = l_run[1];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[(4 + 4 * i + e) * 32] = acc[i][e];
  }
  __syncthreads();
  if (sub > 0) return;
  for (int o = 1; o < a.wph; ++o) {
    const float* src = buf + static_cast<size_t>((o - 1) * a.kvh + h) * kFields * 32 + lane;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float mo = src[hh * 32], lo = src[(2 + hh) * 32];
      const float mn = fmaxf(m_run[hh], mo);
      const float a0 = mn == -INFINITY ? 0.f : fast_exp2(m_run[hh] - mn);
      const float a1 = mn == -INFINITY ? 0.f : fast_exp2(mo - mn);
      m_run[hh] = mn;
      l_run[hh] = l_run[hh] * a0 + lo * a1;
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        acc[i][hh] = acc[i][hh] * a0 + src[(4 + 4 * i + hh) * 32] * a1;
        acc[i][2 + hh] = acc[i][2 + hh] * a0 + src[(4 + 4 * i + 2 + hh) * 32] * a1;
      }
    }
  }
  // ---- this CTA's part: l summed over the row groups; O^T row g of M-tile (j, k2) is dim
  // 32j + 4g + 2k2 and row g+8 is the next dim.
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

using TmaKernel = void (*)(const DecodeArgs, const TmaMaps);

// INT4, head_dim 128, group_size >= 32 (each 16-byte chunk of codes inside one scale group).
TmaKernel tma_decode_kernel_for(int bits, int d, int group) {
  if (bits != 4 || d != 128) return nullptr;
  switch (group) {
    case 32: return tma_decode_kernel<32>;
    case 64: return tma_decode_kernel<64>;
    case 128: return tma_decode_kernel<128>;
    default: return nullptr;
  }
}

int tma_threads() { return kTmaThreads; }
int tma_warps() { return kTmaWarps; }

}  // namespace kvb
