// Split-KV combine and chunk merges.
//
// combine_parts_kernel: folds the split-KV parts (m in log2 units, l, unnormalised acc)
//   written by the decode kernels into the normalised output and natural-log LSE that
//   kvssd's backends return (src/kvssd/backends/base.py:76-81, docs/v0.2-design.md:51-62).
// merge_chunks_kernel: N-way merge of normalised (out, lse) chunks -- the same algebra as
//   kvssd's merge_attention_chunks (src/kvssd/attention.py:91-102) generalised to N inputs;
//   used to combine per-GPU or per-stage chunks. Empty chunks (lse = -inf) carry no weight.
// merge_pair_kernel: kvssd's two-chunk merge formula evaluated term for term
//   (L = logaddexp(La, Lb); O = Oa*exp(La-L) + Ob*exp(Lb-L)).
#include <cmath>

#include "combine.cuh"
#include "common.cuh"

namespace kvb {

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// grid = (query_heads, ceil(d / 32)), block = 32 * kCombineWarps threads: one slice per CTA.
// status: the decode's device status word; a fatal bit there (a split kernel that gave up
// waiting for its copies) makes the result NaN.
__global__ void __launch_bounds__(32 * kCombineWarps) combine_parts_kernel(
    const float* __restrict__ part_acc, const float* __restrict__ part_ml, int n_parts, int qh,
    int d, float* __restrict__ out, float* __restrict__ lse, const unsigned* status) {
  // Parts are produced by the preceding decode grid (programmatic dependent launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool poison = (ld_acquire_gpu(status) & kDevFatalBits) != 0u;
  combine_slice(part_acc, part_ml, n_parts, qh, d, blockIdx.x, blockIdx.y, out, lse, poison);
}

// grid = (query_heads, ceil(d / blockDim)); outs [n, qh, d], lses [n, qh].
__global__ void __launch_bounds__(128) merge_chunks_kernel(const float* __restrict__ outs,
                                                           const float* __restrict__ lses,
                                                           int n, int qh, int d,
                                                           float* __restrict__ out,
                                                           float* __restrict__ lse) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ float w[];
  __shared__ float red[32];
  const int h = blockIdx.x;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, lses[static_cast<size_t>(i) * qh + h]);
  mx = block_reduce_max(mx, red);
  float ls = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float li = lses[static_cast<size_t>(i) * qh + h];
    const float wi = (li == -INFINITY) ? 0.f : expf(li - mx);
    w[i] = wi;
    ls += wi;
  }
  ls = block_reduce_sum(ls, red);
  const bool empty = (mx == -INFINITY) || !(ls > 0.f);
  const float inv = empty ? 0.f : 1.f / ls;
  const int dd = blockIdx.y * blockDim.x + threadIdx.x;
  if (dd < d) {
    float s = 0.f;
    if (!empty)
      for (int i = 0; i < n; ++i) s = fmaf(outs[(static_cast<size_t>(i) * qh + h) * d + dd], w[i], s);
    out[static_cast<size_t>(h) * d + dd] = s * inv;
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) lse[h] = empty ? -INFINITY : mx + logf(ls);
}

__device__ __forceinline__ float logaddexp_f(float a, float b) {
  if (isinf(a) && a == b) return a;
  const float mx = fmaxf(a, b);
  return mx + log1pf(expf(-fabsf(a - b)));
}

// One thread per output element; lo/ro [qh, d], llse/rlse [qh].
__global__ void merge_pair_kernel(const float* __restrict__ lo, const float* __restrict__ llse,
                                  const float* __restrict__ ro, const float* __restrict__ rlse,
                                  int qh, int d, float* __restrict__ out,
                                  float* __restrict__ lse) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(qh) * d) return;
  const int h = static_cast<int>(i / d);
  const float a = llse[h], b = rlse[h];
  const float L = logaddexp_f(a, b);
  out[i] = lo[i] * expf(a - L) + ro[i] * expf(b - L);
  if (i % d == 0) lse[h] = L;
}

}  // namespace kvb
