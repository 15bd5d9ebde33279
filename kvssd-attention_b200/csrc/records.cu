// On-GPU record decode: raw kvssd records (as read from the store files into device memory)
// to the PackedBatch layout the decode kernels read, with the CRC-32 of every payload checked
// on the device.
//
// Record format (src/kvssd/format.py:16,104-177): a 52-byte little-endian header
//   magic "KVSSD001", version, layer, block, valid, bits, block_tokens, kv_heads, head_dim,
//   group_size, payload_len, crc32 (zlib CRC-32 of the payload)
// followed by the payload -- K scales, V scales (FP16, [bt, kvh, G] each), K codes, V codes
// (u8, [bt, kvh, pd] each) -- and zero padding to a 4 KiB multiple.
//
// One CTA per record. Pass 1 copies the payload's four sections into their PackedBatch tensors
// with coalesced 4-byte words (the payload starts 4-byte aligned; geometries whose sections
// are not whole words are copied byte by byte). Pass 2 checks the CRC: the
// payload is cut into NT equal slices, thread t runs the table-driven reflected CRC-32 over
// slice t (slice-by-4 tables in shared memory; thread 0 starts from the 0xFFFFFFFF preset, the
// others from zero), and the slice CRCs are folded pairwise in log2(NT) levels with
//   crc(A || B) = crc(A) * x^(8 |B|) mod P  xor  crc(B),
// the multiplications by x^(8 |B|) mod P (GF(2) polynomials in the reflected bit order of
// zlib's CRC-32) using constants the host computes once per slice length. The result, inverted,
// is compared with the header's crc32. Bad records are reported per record, never faulted on.
#include "records.cuh"

namespace kvb {

__global__ void __launch_bounds__(kRecThreads) record_decode_kernel(const RecordArgs a) {
  __shared__ unsigned table[4][256];
  __shared__ unsigned crcs[kRecThreads];
  __shared__ unsigned hdr[13];
  const int r = blockIdx.x;
  const int t = threadIdx.x;
  // slice-by-4 tables: T0 is the byte-wise table of the reflected polynomial
  {
    unsigned c = static_cast<unsigned>(t);
    for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0xEDB88320u : c >> 1;
    table[0][t] = c;
  }
  const uint8_t* rec = a.records + static_cast<size_t>(r) * a.stride;
  if (t < 13) hdr[t] = reinterpret_cast<const unsigned*>(rec)[t];
  __syncthreads();
#pragma unroll
  for (int k = 1; k < 4; ++k) {
    const unsigned prev = table[k - 1][t];
    table[k][t] = (prev >> 8) ^ table[0][prev & 0xFFu];
    __syncthreads();
  }
  // header: magic (2 words), version, layer, block, valid, bits, bt, kvh, d, group, len, crc
  unsigned st = 0;
  if (hdr[0] != 0x5353564Bu || hdr[1] != 0x31303044u || hdr[2] != 1u) st |= 1u;  // "KVSSD001"
  if (static_cast<int>(hdr[6]) != a.bits || static_cast<int>(hdr[7]) != a.bt ||
      static_cast<int>(hdr[8]) != a.kvh || static_cast<int>(hdr[9]) != a.d ||
      static_cast<int>(hdr[10]) != a.group)
    st |= 2u;
  const unsigned payload = static_cast<unsigned>(2 * a.scale_bytes + 2 * a.packed_bytes);
  if (hdr[11] != payload || kRecHeaderBytes + static_cast<size_t>(payload) > a.stride) st |= 4u;
  if ((a.layer >= 0 && static_cast<int>(hdr[3]) != a.layer) ||
      (a.blocks && static_cast<int>(hdr[4]) != a.blocks[r]))
    st |= 16u;
  if (hdr[5] > static_cast<unsigned>(a.bt)) st |= 32u;
  if (st & 7u) {  // the payload cannot be trusted to have this layout: leave the slot alone
    if (t == 0) {
      a.status[r] = st;
      a.valid[r] = 0;
    }
    return;
  }
  // ---- pass 1: sections -> PackedBatch slots (coalesced words, or bytes for odd sizes)
  const uint8_t* src8 = rec + kRecHeaderBytes;
  uint8_t* dks = a.scales_k + static_cast<size_t>(r) * a.scale_bytes;
  uint8_t* dvs = a.scales_v + static_cast<size_t>(r) * a.scale_bytes;
  uint8_t* dkp = a.packed_k + static_cast<size_t>(r) * a.packed_bytes;
  uint8_t* dvp = a.packed_v + static_cast<size_t>(r) * a.packed_bytes;
  if (a.words) {
    const unsigned* src = reinterpret_cast<const unsigned*>(src8);
    const int sw = a.scale_bytes / 4, pw = a.packed_bytes / 4;
    for (int i = t; i < sw; i += kRecThreads) reinterpret_cast<unsigned*>(dks)[i] = src[i];
    for (int i = t; i < sw; i += kRecThreads) reinterpret_cast<unsigned*>(dvs)[i] = src[sw + i];
    for (int i = t; i < pw; i += kRecThreads) reinterpret_cast<unsigned*>(dkp)[i] = src[2 * sw + i];
    for (int i = t; i < pw; i += kRecThreads)
      reinterpret_cast<unsigned*>(dvp)[i] = src[2 * sw + pw + i];
  } else {
    const int sb = a.scale_bytes, pb = a.packed_bytes;
    for (int i = t; i < sb; i += kRecThreads) dks[i] = src8[i];
    for (int i = t; i < sb; i += kRecThreads) dvs[i] = src8[sb + i];
    for (int i = t; i < pb; i += kRecThreads) dkp[i] = src8[2 * sb + i];
    for (int i = t; i < pb; i += kRecThreads) dvp[i] = src8[2 * sb + pb + i];
  }
  // ---- pass 2: CRC-32 of the payload, slice t by thread t
  unsigned crc = 0;
  if (t < a.slices) {
    crc = t == 0 ? 0xFFFFFFFFu : 0u;
    if (a.words) {
      const unsigned* w = reinterpret_cast<const unsigned*>(src8) +
                          static_cast<size_t>(t) * (a.slice_bytes / 4);
      const int nw = a.slice_bytes / 4;
      for (int i = 0; i < nw; ++i) {
        crc ^= w[i];
        crc = table[3][crc & 0xFFu] ^ table[2][(crc >> 8) & 0xFFu] ^
              table[1][(crc >> 16) & 0xFFu] ^ table[0][crc >> 24];
      }
    } else {
      const uint8_t* b = src8 + static_cast<size_t>(t) * a.slice_bytes;
      for (int i = 0; i < a.slice_bytes; ++i) crc = table[0][(crc ^ b[i]) & 0xFFu] ^ (crc >> 8);
    }
  }
  crcs[t] = crc;
  __syncthreads();
  int level = 0;
  for (int span = 1; span < a.slices; span <<= 1, ++level) {
    // slices [t, t + span) and [t + span, t + 2 span) fold into t
    if ((t & (2 * span - 1)) == 0 && t + span < a.slices)
      crcs[t] = crc_mulmod(a.shift[level], crcs[t]) ^ crcs[t + span];
    __syncthreads();
  }
  if (t == 0) {
    if (~crcs[0] != hdr[12]) st |= 8u;
    a.status[r] = st;
    a.valid[r] = static_cast<int>(hdr[5] > static_cast<unsigned>(a.bt) ? a.bt : hdr[5]);
  }
}

cudaError_t launch_record_decode(const RecordArgs& a, cudaStream_t s) {
  record_decode_kernel<<<a.n, kRecThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace kvb
