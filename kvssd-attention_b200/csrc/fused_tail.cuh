// Tail of the streaming decode kernels: the fused split-KV combine (the last CTAs of the grid
// fold all parts) and the cross-GPU exchange of the combined slices. Shared by every kernel
// that is launched with the fused combine.
#pragma once

#include "combine.cuh"
#include "common.cuh"
#include "decode.cuh"

namespace kvb {

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

// The call's part tags, read by every CTA at its start (after the preceding grid): epoch =
// the header's previous epoch + 1; expect0 = the tag the combiners expect of part 0 (the
// epoch, unless the header's test hook word is nonzero: then epoch + hook, which no CTA
// writes, so the combine waits out its bound); poison: the status word already holds a fatal
// bit (an earlier call on this workspace failed and nobody has cleared it).
struct PartEpoch {
  unsigned epoch;
  unsigned expect0;
  bool poison;
};

__device__ __forceinline__ PartEpoch read_part_epoch(const DecodeArgs& a) {
  PartEpoch pe;
  const unsigned prev = *reinterpret_cast<const volatile unsigned*>(a.part_epoch);
  const unsigned hook = *reinterpret_cast<const volatile unsigned*>(a.part_epoch + 1);
  pe.epoch = next_epoch(prev);
  pe.expect0 = hook ? next_epoch(prev + hook) : pe.epoch;
  pe.poison = (*reinterpret_cast<const volatile unsigned*>(a.status) & kDevFatalBits) != 0u;
  return pe;
}

// Stores the call's epoch in the header (and clears the test hook), by thread 0 of a
// combining CTA after its fold. One problem: every combiner stores it (all CTAs of the call
// read the header before writing the parts the combiner waited for). Batched: the problems'
// CTAs share the epoch, and a problem's combiners only wait for their own problem's parts, so
// the last combiner of the whole grid (counted in header word 2, re-armed by that combiner)
// stores it. epoch 0: a CTA of a refused problem that read nothing (the header still holds
// the previous call's epoch when it is the last).
__device__ __forceinline__ void publish_part_epoch(const DecodeArgs& a, unsigned epoch,
                                                   int n_comb) {
  if (a.problems != nullptr) {
    const unsigned total = gridDim.y * static_cast<unsigned>(n_comb);
    if (atomicAdd(a.part_epoch + 2, 1u) != total - 1u) return;
    a.part_epoch[2] = 0u;
    if (epoch == 0u) epoch = next_epoch(*reinterpret_cast<const volatile unsigned*>(a.part_epoch));
  }
  a.part_epoch[0] = epoch;
  a.part_epoch[1] = 0u;
}

// Fused split-KV combine at the end of the decode grid (launched cooperatively, so all CTAs
// are co-resident). Every CTA has written its part as tagged words (merge_warps_write_part);
// the n_comb highest-numbered CTAs (one per (query head, 32-dim) slice, or fewer when the grid
// is smaller) poll the parts of their slices until every word carries this call's epoch and
// fold them (combine_slice_tagged). A combiner that timed out or met a poisoned part writes
// NaN into its slices of out and lse (and flags kDevCombineTimeout on timeout). Each combiner
// then stores the call's epoch in the header and clears the test hook: every CTA of the call
// read them at its start, before writing the part this combiner waited for.
template <int D>
__device__ __forceinline__ void fused_combine_tail(const DecodeArgs& a, unsigned xepoch,
                                                   const PartEpoch& pe, int n_parts) {
  constexpr int kChunks = (D + 31) / 32;
  const int n_slices = a.qh * kChunks;
  const int n_comb = min(a.n_splits, n_slices);
  const int k = static_cast<int>(blockIdx.x) - (a.n_splits - n_comb);
  if (k < 0) return;
  const unsigned long long* tml = reinterpret_cast<const unsigned long long*>(a.part_ml);
  const unsigned long long* tacc = a.tpart_acc;
  TagWait w{global_ns() + kCombineWaitNs, false, false};
  if (a.xworld == 0 && n_parts <= 32) {
    // Few parts (a batched problem's handful of CTAs): one warp folds a whole slice, so the
    // CTA's 16 warps work on 16 of its slices at once.
    const int warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    const int mine = (n_slices - k + n_comb - 1) / n_comb;  // slices k, k + n_comb, ...
    bool gave_up = false;
    for (int j = warp; j < mine; j += n_warps) {
      const int sl = k + j * n_comb, h = sl / kChunks, chunk = sl % kChunks;
      const int dd = chunk * 32 + lane;
      TagWait ww{w.deadline, false, false};
      float M = -INFINITY, L = 0.f, A = 0.f;
      fold_tagged_warp(tml, tacc, 0, n_parts, a.qh, D, h, dd, pe.epoch, pe.expect0, ww, M, L,
                       A);
      gave_up |= ww.timed_out;
      const bool bad = ww.timed_out || ww.poison || pe.poison;
      const bool empty = M == -INFINITY || !(L > 0.f);
      if (dd < D) a.out[static_cast<size_t>(h) * D + dd] = bad ? nan_f32() : empty ? 0.f : A / L;
      if (chunk == 0 && lane == 0)
        a.lse[h] = bad ? nan_f32() : empty ? -INFINITY : (M + log2f(L)) * kLn2;
    }
    if (__syncthreads_or(gave_up) && threadIdx.x == 0) atomicOr(a.status, kDevCombineTimeout);
  } else {
    for (int sl = k; sl < n_slices; sl += n_comb) {
      float o = 0.f, l2 = -INFINITY;
      combine_slice_tagged(tml, tacc, n_parts, a.qh, D, sl / kChunks, sl % kChunks, pe.epoch,
                           pe.expect0, w, &o, &l2);
      const bool poison = w.timed_out || w.poison || pe.poison;
      if (threadIdx.x < 32) {
        const int lane = threadIdx.x, chunk = sl % kChunks, h = sl / kChunks;
        if (a.xworld == 0) {
          const int dd = chunk * 32 + lane;
          if (dd < D) a.out[static_cast<size_t>(h) * D + dd] = poison ? nan_f32() : o;
          if (chunk == 0 && lane == 0) a.lse[h] = poison ? nan_f32() : l2 * kLn2;
        } else {
          exchange_slice<D>(a, xepoch, sl, n_slices, o, l2, poison);
        }
      }
      // after a timeout the later slices stop at their first poll (the deadline has passed)
    }
    if (w.timed_out && threadIdx.x == 0) atomicOr(a.status, kDevCombineTimeout);
  }
  if (threadIdx.x == 0) {
    publish_part_epoch(a, pe.epoch, n_comb);
    // every CTA read the exchange epoch at its start, before its part: publish the call
    if (a.xworld) *reinterpret_cast<volatile unsigned*>(a.xpeers[a.xrank]) = xepoch;
  }
}

}  // namespace kvb
