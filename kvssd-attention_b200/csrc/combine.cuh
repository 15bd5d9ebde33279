// Split-KV combine of one (query head, 32-dim slice): shared by the standalone combine kernel
// and the tail of the streaming decode kernel. Parts hold (m in log2 units, l, unnormalised
// acc) per query head; the result is the normalised output and the natural-log LSE that
// kvssd's backends return (src/kvssd/backends/base.py:76-81, docs/v0.2-design.md:51-62).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace kvb {

constexpr int kCombineWarps = 16;   // the caller's block is 32 * kCombineWarps threads
constexpr float kLn2 = 0.693147180559945309f;

// Status bits after which a decode's result is not trustworthy: a wait gave up, so parts,
// ring stages or another rank's slices may be missing. A combine that sees any of them in
// the (sticky) status word writes NaN into out and lse instead of a plausible number, so the
// failure reaches the caller through the result itself, without a host synchronisation.
constexpr unsigned kDevFatalBits = kDevCombineTimeout | kDevExchangeTimeout | kDevStreamTimeout;

// Bounds of the fused combine's waits: one second of GPU time, and a poll count as a second
// guard.
constexpr unsigned long long kCombineWaitNs = 1000000000ull;
constexpr unsigned kCombineMaxPolls = 1u << 26;
constexpr unsigned kCombineMaxPollsTagged = 1u << 24;
__device__ __forceinline__ float nan_f32() { return __uint_as_float(0x7fffffffu); }

// Warp w folds the contiguous part range [w*n/W, (w+1)*n/W) for dims [32*chunk, 32*chunk+32),
// 32 parts per batch: all of a batch's loads (lane j: part j's m and l; every lane: its dim of
// the 32 parts' rows) are issued before any of them is used, so a batch costs one round trip
// to L2. Part weights reach the other lanes by shuffle; the W warp states are merged through
// shared memory. Every thread of the block must call it (it synchronises the block; warps past
// the first kCombineWarps only take part in the synchronisation). Parts are
// read with L2-coherent loads (ld.global.cg): they may have been written by other CTAs of the
// same grid.
// Result in warp 0: *o = the normalised output of dim 32 * chunk + lane (0 when the head saw
// no token), *l2 = the slice's LSE in log2 units (-inf when empty). Other warps get nothing.
__device__ __forceinline__ void combine_slice_result(const float* __restrict__ part_acc,
                                                     const float* __restrict__ part_ml,
                                                     int n_parts, int qh, int d, int h,
                                                     int chunk, float* o, float* l2) {
  __shared__ float wm[kCombineWarps], wl[kCombineWarps], wacc[kCombineWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int dd = chunk * 32 + lane;
  const bool has_dim = dd < d;
  const bool active = warp < kCombineWarps;  // larger blocks: the extra warps only synchronise
  const int lo = active ? static_cast<int>(static_cast<long long>(n_parts) * warp / kCombineWarps) : 0;
  const int hi = active ? static_cast<int>(static_cast<long long>(n_parts) * (warp + 1) / kCombineWarps) : 0;
  const size_t stride = static_cast<size_t>(qh) * d;
  float M = -INFINITY, L = 0.f, A = 0.f;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    float mp = -INFINITY, lp = 0.f;
    if (p < hi) {
      const float2 ml =
          __ldcg(reinterpret_cast<const float2*>(part_ml + (static_cast<size_t>(p) * qh + h) * 2));
      mp = ml.x;
      lp = ml.y;
    }
    const float* row = part_acc + (static_cast<size_t>(base) * qh + h) * d + dd;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (base + j < hi && has_dim) ? __ldcg(row + j * stride) : 0.f;
    float cm = mp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const float nm = fmaxf(M, cm);
    if (nm == -INFINITY) continue;  // only empty parts so far
    const float keep = fast_exp2(M - nm);  // 0 while M is -inf
    const float wp = mp == -INFINITY ? 0.f : fast_exp2(mp - nm);
    float ls = wp * lp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    L = fmaf(L, keep, ls);
    A *= keep;
#pragma unroll
    for (int j = 0; j < 32; ++j) A = fmaf(__shfl_sync(0xffffffffu, wp, j), v[j], A);
    M = nm;
  }
  if (active) {
    if (lane == 0) {
      wm[warp] = M;
      wl[warp] = L;
    }
    wacc[warp][lane] = A;
  }
  __syncthreads();
  if (warp == 0) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) mx = fmaxf(mx, wm[w]);
    float ls = 0.f, t = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) {
      const float ww = wm[w] == -INFINITY ? 0.f : fast_exp2(wm[w] - mx);
      ls = fmaf(ww, wl[w], ls);
      t = fmaf(ww, wacc[w][lane], t);
    }
    const bool empty = (mx == -INFINITY) || !(ls > 0.f);
    *o = empty ? 0.f : t / ls;
    *l2 = empty ? -INFINITY : mx + log2f(ls);
  }
  __syncthreads();  // the shared arrays may be reused by the caller's next slice
}

// The slice's normalised output and natural-log LSE written to out [qh, d] / lse [qh].
// poison: write NaN instead (see kDevFatalBits).
__device__ __forceinline__ void combine_slice(const float* __restrict__ part_acc,
                                              const float* __restrict__ part_ml, int n_parts,
                                              int qh, int d, int h, int chunk,
                                              float* __restrict__ out, float* __restrict__ lse,
                                              bool poison) {
  float o = 0.f, l2 = -INFINITY;
  combine_slice_result(part_acc, part_ml, n_parts, qh, d, h, chunk, &o, &l2);
  const int lane = threadIdx.x & 31, dd = chunk * 32 + lane;
  if (threadIdx.x < 32) {
    if (dd < d) out[static_cast<size_t>(h) * d + dd] = poison ? nan_f32() : o;
    if (chunk == 0 && lane == 0) lse[h] = poison ? nan_f32() : l2 * kLn2;
  }
}

// One warp folds all n_parts (<= 32) parts of a slice: lane j loads part j's m and l, every
// lane its dim of each part's row (all loads issued before use), then the weights reach the
// lanes by shuffle. Writes the slice's normalised output and natural-log LSE (NaN: poison).
__device__ __forceinline__ void combine_slice_warp(const float* __restrict__ part_acc,
                                                   const float* __restrict__ part_ml,
                                                   int n_parts, int qh, int d, int h, int chunk,
                                                   float* __restrict__ out,
                                                   float* __restrict__ lse, bool poison) {
  const int lane = threadIdx.x & 31;
  const int dd = chunk * 32 + lane;
  const bool has_dim = dd < d;
  float mp = -INFINITY, lp = 0.f;
  if (lane < n_parts) {
    const float2 ml =
        __ldcg(reinterpret_cast<const float2*>(part_ml + (static_cast<size_t>(lane) * qh + h) * 2));
    mp = ml.x;
    lp = ml.y;
  }
  const float* row = part_acc + static_cast<size_t>(h) * d + dd;
  const size_t stride = static_cast<size_t>(qh) * d;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = (j < n_parts && has_dim) ? __ldcg(row + j * stride) : 0.f;
  float mx = mp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float wp = (mp == -INFINITY || mx == -INFINITY) ? 0.f : fast_exp2(mp - mx);
  float ls = wp * lp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
  float t = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) t = fmaf(__shfl_sync(0xffffffffu, wp, j), v[j], t);
  const bool empty = (mx == -INFINITY) || !(ls > 0.f);
  if (has_dim) out[static_cast<size_t>(h) * d + dd] = poison ? nan_f32() : empty ? 0.f : t / ls;
  if (chunk == 0 && lane == 0)
    lse[h] = poison ? nan_f32() : empty ? -INFINITY : (mx + log2f(ls)) * kLn2;
}

// ---------------------------------------------------------------------------------------------
// Tagged parts (the fused combine). Every value of a part is one 64-bit word: the f32 value in
// the low half and the call's tag in the high half, written with one relaxed store, so a value
// and its readiness arrive together and the combining CTAs poll the data itself: no fence on
// the writer's side, no arrival counter, no second round trip for the data after the wait.
// Tag = epoch (31 bits, never 0) | kTagPoison when the writer's part is not trustworthy. The
// epoch is the call number kept in the workspace header: every CTA reads the previous call's
// at its start, and the combiners store this call's after their fold (they have seen every
// CTA's part, so every CTA of the call has read the header by then).
// What a tag cannot tell apart: a word left by a call 2^31 - 1 calls earlier (the epoch wraps)
// that no call has rewritten since, and plain f32 parts written over the region by the
// separate-combine path, whose high halves are f32 bit patterns (a positive one equal to a
// small epoch is a denormal near 1e-44). Zeroing the workspace at allocation rules out
// leftover garbage.
constexpr unsigned kTagPoison = 0x80000000u;

__device__ __forceinline__ unsigned next_epoch(unsigned prev) {
  const unsigned e = (prev + 1u) & 0x7fffffffu;
  return e == 0u ? 1u : e;
}

__device__ __forceinline__ unsigned long long tag_word(float v, unsigned tag) {
  return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}

__device__ __forceinline__ void st_tagged2(unsigned long long* p, unsigned long long x,
                                           unsigned long long y) {
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(x), "l"(y) : "memory");
}

__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool tag_matches(unsigned long long w, unsigned expect) {
  return (static_cast<unsigned>(w >> 32) & ~kTagPoison) == expect;
}

// Wait state of one combining CTA: its deadline and whether it gave up or saw a poisoned part.
struct TagWait {
  unsigned long long deadline;
  bool timed_out;
  bool poison;
};

// The warp's online-softmax fold (M, L, A for dim `dd` of head h) over the tagged parts
// [lo, hi), in batches of kTagBatch: lane j < kTagBatch polls part j's (m, l) words until every
// pair of the batch carries the expected tag, then every lane loads its dim of the batch's
// rows and re-loads any word that is not yet this call's. `expect0` is the tag expected of
// part 0 (the epoch; a test hook in the workspace header can plant another value there).
// Bounded by the deadline: on timeout the warp stops polling and flags w.timed_out (the
// caller writes NaN).
constexpr int kTagBatch = 16;

__device__ __forceinline__ void fold_tagged_warp(const unsigned long long* __restrict__ tml,
                                                 const unsigned long long* __restrict__ tacc,
                                                 int lo, int hi, int qh, int d, int h, int dd,
                                                 unsigned epoch, unsigned expect0, TagWait& w,
                                                 float& M, float& L, float& A) {
  const int lane = threadIdx.x & 31;
  const bool has_dim = dd < d;
  const size_t stride = static_cast<size_t>(qh) * d;
  for (int base = lo; base < hi; base += kTagBatch) {
    const int p = base + lane, cnt = min(kTagBatch, hi - base);
    const bool mine = lane < cnt;
    const unsigned ex = p == 0 ? expect0 : epoch;
    const unsigned long long* mlp = tml + (static_cast<size_t>(p) * qh + h) * 2;
    unsigned long long wm = 0ull, wl = 0ull;
    bool ready = !mine;
    unsigned polls = 0;
    while (true) {
      if (!ready) {
        wm = ld_tagged(mlp);
        wl = ld_tagged(mlp + 1);
        ready = tag_matches(wm, ex) && tag_matches(wl, ex);
      }
      if (__all_sync(0xffffffffu, ready)) break;
      if (++polls > kCombineMaxPollsTagged || global_ns() > w.deadline) {
        w.timed_out = true;
        return;
      }
      __nanosleep(64);
    }
    bool bad = mine && ((wm | wl) >> 63) != 0ull;
    const unsigned long long* row = tacc + (static_cast<size_t>(base) * qh + h) * d + dd;
    unsigned long long v[kTagBatch];
#pragma unroll
    for (int j = 0; j < kTagBatch; ++j)
      v[j] = (j < cnt && has_dim) ? ld_tagged(row + j * stride) : 0ull;
    // A row word may still be in flight behind the (m, l) pair: re-load until it is this call's.
#pragma unroll 1
    for (unsigned tries = 0;; ++tries) {
      bool all = true;
#pragma unroll
      for (int j = 0; j < kTagBatch; ++j) {
        if (j < cnt && has_dim && !tag_matches(v[j], base + j == 0 ? expect0 : epoch)) {
          all = false;
          v[j] = ld_tagged(row + j * stride);
        }
      }
      if (__all_sync(0xffffffffu, all)) break;
      if (tries > kCombineMaxPollsTagged || global_ns() > w.deadline) {
        w.timed_out = true;
        return;
      }
    }
#pragma unroll
    for (int j = 0; j < kTagBatch; ++j) bad |= (v[j] >> 63) != 0ull;
    if (__any_sync(0xffffffffu, bad)) w.poison = true;
    const float mp = mine ? __uint_as_float(static_cast<unsigned>(wm)) : -INFINITY;
    const float lp = mine ? __uint_as_float(static_cast<unsigned>(wl)) : 0.f;
    float cm = mp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const float nm = fmaxf(M, cm);
    if (nm == -INFINITY) continue;  // only empty parts so far
    const float keep = fast_exp2(M - nm);  // 0 while M is -inf
    const float wp = mp == -INFINITY ? 0.f : fast_exp2(mp - nm);
    float ls = wp * lp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    L = fmaf(L, keep, ls);
    A *= keep;
#pragma unroll
    for (int j = 0; j < kTagBatch; ++j)
      A = fmaf(__shfl_sync(0xffffffffu, wp, j), __uint_as_float(static_cast<unsigned>(v[j])), A);
    M = nm;
  }
}

// combine_slice_result over tagged parts: the block's kCombineWarps warps split the parts,
// their states meet in shared memory; result in warp 0 (see combine_slice_result). Every
// thread of the block must call it. w.timed_out / w.poison are the block's (same in every
// thread on return).
__device__ __forceinline__ void combine_slice_tagged(const unsigned long long* __restrict__ tml,
                                                     const unsigned long long* __restrict__ tacc,
                                                     int n_parts, int qh, int d, int h,
                                                     int chunk, unsigned epoch, unsigned expect0,
                                                     TagWait& w, float* o, float* l2) {
  __shared__ float wm[kCombineWarps], wl[kCombineWarps], wacc[kCombineWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int dd = chunk * 32 + lane;
  const bool active = warp < kCombineWarps;
  float M = -INFINITY, L = 0.f, A = 0.f;
  if (active) {
    const int lo = static_cast<int>(static_cast<long long>(n_parts) * warp / kCombineWarps);
    const int hi = static_cast<int>(static_cast<long long>(n_parts) * (warp + 1) / kCombineWarps);
    fold_tagged_warp(tml, tacc, lo, hi, qh, d, h, dd, epoch, expect0, w, M, L, A);
    if (lane == 0) {
      wm[warp] = M;
      wl[warp] = L;
    }
    wacc[warp][lane] = A;
  }
  w.timed_out = __syncthreads_or(w.timed_out) != 0;
  w.poison = __syncthreads_or(w.poison) != 0;
  if (warp == 0) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kCombineWarps; ++i) mx = fmaxf(mx, wm[i]);
    float ls = 0.f, t = 0.f;
#pragma unroll
    for (int i = 0; i < kCombineWarps; ++i) {
      const float ww = wm[i] == -INFINITY ? 0.f : fast_exp2(wm[i] - mx);
      ls = fmaf(ww, wl[i], ls);
      t = fmaf(ww, wacc[i][lane], t);
    }
    const bool empty = (mx == -INFINITY) || !(ls > 0.f);
    *o = empty ? 0.f : t / ls;
    *l2 = empty ? -INFINITY : mx + log2f(ls);
  }
  __syncthreads();  // the shared arrays may be reused by the caller's next slice
}

}  // namespace kvb
