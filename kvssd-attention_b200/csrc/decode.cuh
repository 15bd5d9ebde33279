// Launch arguments shared by the split-KV decode kernels and the host dispatcher.
//
// Work decomposition (all kernels):
//   * a "virtual head" is one KV head together with up to 8 of its query heads (GQA ratios
//     above 8 use several virtual heads per KV head);
//   * a "tile" is 16 consecutive token rows of one selected block; the selection's tiles are
//     numbered slot-major (slot = position in the block table, tiles_per_block per slot);
//   * grid.x = split: CTA x owns tiles [T*x/n_splits, T*(x+1)/n_splits) for every virtual
//     head of its head group (grid.y), so the CTA's warps read whole token rows (all KV
//     heads of a token are contiguous in kvssd's record layout, src/kvssd/format.py:165);
//   * each warp keeps an online-softmax state (m, l, acc) per query head and writes it as one
//     "part" of the split-KV result; part = split * wph + warp-subindex.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kvssd_b200.h"

namespace kvb {

constexpr int kMaxExchangeRanks = 8;

struct DecodeArgs {
  const void* q;
  int q_dtype;
  const uint8_t* kp;   // [n_pool, bt, kvh, d*bits/8]
  const uint8_t* vp;   // [n_pool, bt, kvh, d*bits/8]
  const __half* ks;    // [n_pool, bt, kvh, d/group]
  const __half* vs;    // [n_pool, bt, kvh, d/group]
  const int32_t* valid;  // [n_pool]
  const int32_t* table;  // [n_sel] pool indices, or nullptr for the identity
  int n_pool, n_sel, bt, qh, kvh, d, bits, group;
  int gqa;            // query heads per KV head
  int n_qsub;         // virtual heads per KV head
  int n_vheads;       // kvh * n_qsub
  int heads_per_cta;  // virtual heads handled by one CTA
  int wph;            // warps per virtual head in a CTA (they interleave tiles)
  int tiles_per_block;
  long long total_tiles;
  int n_splits;
  float score_scale;  // sm_scale * log2(e): scores are kept in the log2 domain
  // Parts: plain f32 [n_parts, qh, 2] (running max in log2 domain, sum of p) at part_ml and
  // [n_parts, qh, d] (unnormalised sum p*v) at part_acc when the combine is a separate launch;
  // with the fused combine the same arrays as tagged 64-bit words (combine.cuh), the (m, l)
  // words at part_ml and the sums at tpart_acc.
  float* part_acc;
  float* part_ml;
  unsigned long long* tpart_acc;
  unsigned* status;   // device status word (DeviceStatusBits)
  // Fused combine (streaming kernel): the last CTAs to finish fold all parts into out/lse.
  int fuse_combine;
  // Header words of the fused combine: [0] epoch of the last call, [1] test hook (0 in use),
  // [2] combiners done (batched calls; 0 between calls). See fused_tail.cuh.
  unsigned* part_epoch;
  float* out;         // [qh, d] normalised output
  float* lse;         // [qh] natural-log LSE
  // Cross-GPU exchange (token-range shards, fused combine only): every combiner pushes its
  // slice to all ranks' exchange buffers and merges all ranks' slices (0 ranks: no exchange).
  int xworld;
  int xrank;
  uint8_t* xpeers[kMaxExchangeRanks];  // every rank's exchange buffer ([xrank] is local)
  // Batched decode: problem blockIdx.y of this device array (nullptr: one problem, the
  // fields above).
  const kvssd_b200_problem* problems;
};

// Exchange buffer layout for `world` ranks and n_slices = qh * ceil(d / 32) slices:
//   header (256 bytes): u32 epoch = number of completed exchange calls on this rank;
//   then words u64 [2][world][n_slices][33]: {f32 value (low half), u32 epoch (high half)} for
//   32 normalised dims and the slice's LSE in log2 units. A call's epoch is the header value
//   + 1; its parity selects the buffer half.
constexpr size_t kExchangeHeader = 256;
__host__ __device__ inline size_t exchange_bytes(int world, int n_slices) {
  return kExchangeHeader + static_cast<size_t>(2) * world * n_slices * 33 * 8;
}

// Resolves slot -> (pool block, clamped valid count) with a per-warp register cache of 32
// consecutive slots, so the dependent block-table/valid loads are paid once per 32 blocks.
struct BlockInfoCache {
  int base = -0x40000000;
  int blk = -1;
  int valid = 0;

  __device__ __forceinline__ void lookup(const DecodeArgs& a, int slot, int lane, int& out_blk,
                                         int& out_valid) {
    if (slot < base || slot - base >= 32) {  // warp-uniform: slot is the same on all lanes
      base = slot;
      const int s = slot + lane;
      blk = -1;
      valid = 0;
      if (s < a.n_sel) {
        int b = a.table ? a.table[s] : s;
        if (b < 0 || b >= a.n_pool) {
          atomicOr(a.status, 1u);
          b = -1;
        } else {
          int v = a.valid[b];
          if (v < 0 || v > a.bt) {
            atomicOr(a.status, 2u);
            v = v < 0 ? 0 : a.bt;
          }
          valid = v;
        }
        blk = b;
      }
    }
    out_blk = __shfl_sync(0xffffffffu, blk, slot - base);
    out_valid = __shfl_sync(0xffffffffu, valid, slot - base);
  }
};

}  // namespace kvb
