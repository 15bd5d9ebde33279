// Tail of the streaming decode kernels: the fused split-KV combine (the last CTAs of the grid
// fold all parts) and the cross-GPU exchange of the combined slices. Shared by every kernel
// that is launched with the fused combine.
#pragma once

#include "combine.cuh"
#include "common.cuh"
#include "decode.cuh"

namespace kvb {

// Bounds of a fused-combine wait: one second of GPU time, and a poll count as a second guard.
constexpr unsigned long long kCombineWaitNs = 1000000000ull;
constexpr unsigned kCombineMaxPolls = 1u << 26;

// Cross-GPU exchange of one combined slice, run by warp 0 of the CTA that combined it (token-
// range shards of one context, one rank per GPU). Every value travels as one 64-bit word
// {value, epoch} written with a single store into buffer half (epoch & 1) of every rank's
// exchange buffer (plain peer stores over NVLink; no fence, since an aligned 64-bit store
// arrives whole). Each lane then polls the words of its dim from all ranks in its own buffer
// until their epochs match (bounded: on timeout it flags kDevExchangeTimeout), so a value and
// its readiness arrive together. The ranks' slices are folded in rank order with the exact
// merge O = sum_r 2^(L_r - M) O_r / sum_r 2^(L_r - M): every rank computes the same result.
// Two buffer halves suffice, since a rank can only be one epoch ahead of the slowest reader.
// The epoch is kept on the device (the buffer's header), so a call captured in a CUDA graph
// gets a fresh epoch on every replay.
// poison: this rank's slice is not trustworthy (see kDevFatalBits); it is pushed as NaN, so
// every rank's merged slice becomes NaN. A lane whose wait gives up poisons the whole slice.
template <int D>
__device__ __forceinline__ void exchange_slice(const DecodeArgs& a, unsigned epoch, int slice,
                                               int n_slices, float o, float l2, bool poison) {
  if (poison) o = l2 = nan_f32();
  const int lane = threadIdx.x & 31;
  const int world = a.xworld, par = static_cast<int>(epoch & 1u);
  const unsigned long long tag = static_cast<unsigned long long>(epoch) << 32;
  const size_t mine = ((static_cast<size_t>(par) * world + a.xrank) * n_slices + slice) * 33;
  for (int r = 0; r < world; ++r) {
    unsigned long long* row =
        reinterpret_cast<unsigned long long*>(a.xpeers[r] + kExchangeHeader) + mine;
    st_relaxed_sys_u64(row + lane, tag | __float_as_uint(o));
    if (lane == 0) st_relaxed_sys_u64(row + 32, tag | __float_as_uint(l2));
  }
  const unsigned long long* rows =
      reinterpret_cast<const unsigned long long*>(a.xpeers[a.xrank] + kExchangeHeader);
  float vo[kMaxExchangeRanks], vl[kMaxExchangeRanks];
  const unsigned long long t0 = global_ns();
  bool timed_out = false;
#pragma unroll
  for (int r = 0; r < kMaxExchangeRanks; ++r) {
    vo[r] = 0.f;
    vl[r] = -INFINITY;
    if (r >= world) continue;
    const unsigned long long* row = rows + ((static_cast<size_t>(par) * world + r) * n_slices + slice) * 33;
    unsigned long long wo = ld_relaxed_sys_u64(row + lane);
    unsigned long long wl = lane == 0 ? ld_relaxed_sys_u64(row + 32) : tag;
    unsigned polls = 0;
    while (!timed_out && ((wo >> 32) != epoch || (wl >> 32) != epoch)) {
      if (++polls > kCombineMaxPolls || global_ns() - t0 > kCombineWaitNs) {
        atomicOr(a.status, kDevExchangeTimeout);
        timed_out = true;
        break;
      }
      __nanosleep(32);
      wo = ld_relaxed_sys_u64(row + lane);
      if (lane == 0) wl = ld_relaxed_sys_u64(row + 32);
    }
    vo[r] = __uint_as_float(static_cast<unsigned>(wo));
    if (lane == 0) vl[r] = __uint_as_float(static_cast<unsigned>(wl));
  }
  __syncwarp();
  float M = -INFINITY;
#pragma unroll
  for (int r = 0; r < kMaxExchangeRanks; ++r) {
    vl[r] = __shfl_sync(0xffffffffu, vl[r], 0);
    M = fmaxf(M, vl[r]);
  }
  float num = 0.f, den = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxExchangeRanks; ++r) {
    const float w = vl[r] == -INFINITY ? 0.f : fast_exp2(vl[r] - M);
    num = fmaf(w, vo[r], num);
    den += w;
  }
  constexpr int kChunks = (D + 31) / 32;
  const int h = slice / kChunks, chunk = slice % kChunks, dd = chunk * 32 + lane;
  const bool empty = M == -INFINITY || !(den > 0.f);
  const bool bad = __any_sync(0xffffffffu, timed_out) || poison;
  if (dd < D) a.out[static_cast<size_t>(h) * D + dd] = bad ? nan_f32() : empty ? 0.f : num / den;
  if (chunk == 0 && lane == 0)
    a.lse[h] = bad ? nan_f32() : empty ? -INFINITY : (M + log2f(den)) * kLn2;
}

// Fused split-KV combine at the end of the decode grid (launched cooperatively, so all CTAs
// are co-resident). Every CTA publishes its part and signals its arrival with one release add
// on tickets[0]; the n_comb highest-numbered CTAs (one per (query head, 32-dim) slice, or
// fewer when the grid is smaller) wait until all n_splits parts have arrived and fold one or
// more slices each. Each combiner counts itself on tickets[1] as soon as it has seen every
// arrival -- the atomic's round trip overlaps its fold -- and the last one re-arms both
// counters (zero again for the next call) and publishes the exchange epoch after its fold.
// The wait is bounded: on timeout the CTA flags kDevCombineTimeout and carries on. A combiner
// that timed out, or that finds a fatal bit in the status word once every part has arrived
// (another CTA gave up on its copies, or an earlier call on this workspace failed and nobody
// has cleared the word), writes NaN into its slices of out and lse.
template <int D>
__device__ __forceinline__ void fused_combine_tail(const DecodeArgs& a, unsigned epoch,
                                                   int n_parts) {
  __shared__ int poison_flag;
  __syncthreads();  // every warp's part stores precede the CTA's release below
  constexpr int kChunks = (D + 31) / 32;
  const int n_slices = a.qh * kChunks;
  const int n_comb = min(a.n_splits, n_slices);
  const int k = static_cast<int>(blockIdx.x) - (a.n_splits - n_comb);
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.tickets) : "memory");
    if (k >= 0) {
      const unsigned long long t0 = global_ns();
      unsigned polls = 0;
      bool timed_out = false;
      // Signed: a counter left below zero (a corrupted workspace header) reads as "parts
      // missing" to every combiner, so all of them wait out the bound and fail closed together
      // instead of some folding early.
      while (static_cast<int>(ld_acquire_gpu(a.tickets)) < a.n_splits) {
        if (++polls > kCombineMaxPolls || global_ns() - t0 > kCombineWaitNs) {
          atomicOr(a.status, kDevCombineTimeout);
          timed_out = true;
          break;
        }
        __nanosleep(32);
      }
      poison_flag = timed_out || (ld_acquire_gpu(a.status) & kDevFatalBits) != 0u;
    }
  }
  if (k < 0) return;
  __syncthreads();
  const bool poison = poison_flag != 0;
  // Every combiner has passed its wait when tickets[1] reaches n_comb; the returned count is
  // only needed after the fold.
  unsigned combined_before = 0u;
  if (threadIdx.x == 0) combined_before = atomicAdd(a.tickets + 1, 1u);
  if (a.xworld == 0 && n_parts <= 32) {
    // Few parts (a batched problem's handful of CTAs): one warp folds a whole slice, so the
    // CTA's 16 warps work on 16 of its slices at once.
    const int warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5;
    const int mine = (n_slices - k + n_comb - 1) / n_comb;  // slices k, k + n_comb, ...
    for (int j = warp; j < mine; j += n_warps) {
      const int sl = k + j * n_comb;
      combine_slice_warp(a.part_acc, a.part_ml, n_parts, a.qh, D, sl / kChunks, sl % kChunks,
                         a.out, a.lse, poison);
    }
    __syncthreads();
  } else {
  for (int sl = k; sl < n_slices; sl += n_comb) {
    if (a.xworld == 0) {
      combine_slice(a.part_acc, a.part_ml, n_parts, a.qh, D, sl / kChunks, sl % kChunks,
                    a.out, a.lse, poison);
    } else {
      float o = 0.f, l2 = -INFINITY;
      combine_slice_result(a.part_acc, a.part_ml, n_parts, a.qh, D, sl / kChunks,
                           sl % kChunks, &o, &l2);
      if (threadIdx.x < 32) exchange_slice<D>(a, epoch, sl, n_slices, o, l2, poison);
    }
  }
  }
  if (threadIdx.x == 0 && combined_before == static_cast<unsigned>(n_comb) - 1) {
    atomicExch(a.tickets, 0u);
    atomicExch(a.tickets + 1, 0u);
    // every CTA read the epoch at its start, before its arrival: publish the completed call
    if (a.xworld) *reinterpret_cast<volatile unsigned*>(a.xpeers[a.xrank]) = epoch;
  }
}

}  // namespace kvb
