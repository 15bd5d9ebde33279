// Generic split-KV decode on CUDA cores: any head_dim <= 256, any pack-aligned group size,
// INT2/INT4, any GQA ratio. It serves the shapes the tensor-core kernel does not cover
// (head_dim 32, group sizes below 16, unaligned views) and is the no-tensor-core variant the
// tensor-core kernel is compared against. Dequantization here is the reference's FP32
// formula (src/kvssd/backends/reference.py:29-33): (code - mid) * float(scale).
//
// One warp per (virtual head, tile stride); lane l owns dims l, l+32, ...; tokens of a tile
// are processed one at a time with warp-shuffle dot products and an online softmax per head.
// The partial state is written in the same part layout as the tensor-core kernel, so both
// share the combine kernel.
#include <cmath>

#include "common.cuh"
#include "decode.cuh"

namespace kvb {

template <int R>  // dims per lane: head_dim <= 32 * R
__global__ void __launch_bounds__(128) simt_decode_kernel(const DecodeArgs a) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, sub = threadIdx.x >> 5;
  const int vh = blockIdx.y;
  if (sub >= a.wph || vh >= a.n_vheads) return;
  const int kvh_idx = vh / a.n_qsub, qsub = vh - kvh_idx * a.n_qsub;
  const int q0 = kvh_idx * a.gqa + qsub * 8;
  const int nq = min(8, a.gqa - qsub * 8);
  const int D = a.d;
  const int per_byte = 8 / a.bits;
  const int code_mask = (1 << a.bits) - 1;
  const float mid = static_cast<float>(1 << (a.bits - 1));
  const int pd = D * a.bits / 8;
  const int G = D / a.group;

  float q[8][R];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int d = lane + 32 * r;
      q[n][r] = (n < nq && d < D) ? load_query(a.q, a.q_dtype, static_cast<long long>(q0 + n) * D + d)
                                  : 0.f;
    }
  float m[8], l[8], acc[8][R];
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    m[n] = -INFINITY;
    l[n] = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) acc[n][r] = 0.f;
  }

  const size_t rs = static_cast<size_t>(a.kvh) * pd;
  const size_t srs = static_cast<size_t>(a.kvh) * G;
  const long long t_end = a.total_tiles * (blockIdx.x + 1) / a.n_splits;
  BlockInfoCache cache;
  for (long long t = a.total_tiles * blockIdx.x / a.n_splits + sub; t < t_end; t += a.wph) {
    const int slot = static_cast<int>(t / a.tiles_per_block);
    const int off = static_cast<int>(t - static_cast<long long>(slot) * a.tiles_per_block) * 16;
    int blk, valid;
    cache.lookup(a, slot, lane, blk, valid);
    const int rows = min(valid - off, 16);
    if (blk < 0 || rows <= 0) continue;
    for (int tok = 0; tok < rows; ++tok) {
      const size_t row = static_cast<size_t>(blk) * a.bt + off + tok;
      const uint8_t* kr = a.kp + row * rs + static_cast<size_t>(kvh_idx) * pd;
      const uint8_t* vr = a.vp + row * rs + static_cast<size_t>(kvh_idx) * pd;
      const __half* ksr = a.ks + row * srs + static_cast<size_t>(kvh_idx) * G;
      const __half* vsr = a.vs + row * srs + static_cast<size_t>(kvh_idx) * G;
      float kv[R], vv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int d = lane + 32 * r;
        kv[r] = vv[r] = 0.f;
        if (d < D) {
          const int byte = d / per_byte, shift = (d % per_byte) * a.bits;
          const float kc = static_cast<float>((kr[byte] >> shift) & code_mask);
          const float vc = static_cast<float>((vr[byte] >> shift) & code_mask);
          kv[r] = (kc - mid) * __half2float(ksr[d / a.group]);
          vv[r] = (vc - mid) * __half2float(vsr[d / a.group]);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n >= nq) break;
        float dot = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r) dot = fmaf(q[n][r], kv[r], dot);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float x = dot * a.score_scale;
        const float nm = fmaxf(m[n], x);
        const float alpha = fast_exp2(m[n] - nm);  // m = -inf on the first token: 0
        const float p = fast_exp2(x - nm);
        m[n] = nm;
        l[n] = fmaf(l[n], alpha, p);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[n][r] = fmaf(acc[n][r], alpha, p * vv[r]);
      }
    }
  }

  const size_t part = static_cast<size_t>(blockIdx.x) * a.wph + sub;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    if (n >= nq) break;
    const size_t row = part * a.qh + (q0 + n);
    if (lane == 0) {
      a.part_ml[row * 2 + 0] = m[n];
      a.part_ml[row * 2 + 1] = l[n];
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int d = lane + 32 * r;
      if (d < D) a.part_acc[row * D + d] = acc[n][r];
    }
  }
}

using DecodeKernel = void (*)(const DecodeArgs);

DecodeKernel simt_decode_kernel_for(int d) {
  if (d <= 32) return simt_decode_kernel<1>;
  if (d <= 64) return simt_decode_kernel<2>;
  if (d <= 128) return simt_decode_kernel<4>;
  if (d <= 256) return simt_decode_kernel<8>;
  return nullptr;
}

}  // namespace kvb
