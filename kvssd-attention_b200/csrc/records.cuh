// Raw-record decode on the GPU: launch arguments and the GF(2) helper shared by the kernel
// (records.cu) and the host code that prepares its constants (api.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace kvb {

constexpr int kRecThreads = 256;
constexpr int kRecHeaderBytes = 52;
constexpr int kRecMaxLevels = 8;  // log2(kRecThreads)

struct RecordArgs {
  const uint8_t* records;
  size_t stride;         // bytes between consecutive records (the spec's record_bytes)
  int n;
  int layer;             // expected layer (< 0: not checked)
  const int32_t* blocks; // expected block ids [n] (nullptr: not checked)
  int bits, bt, kvh, d, group;
  int scale_bytes, packed_bytes;  // per section
  int slices;            // NT: the payload is NT slices of slice_bytes
  int slice_bytes;
  int words;             // sections and slices are whole 4-byte words (else bytes are used)
  unsigned shift[kRecMaxLevels];  // x^(8 * slice_bytes * 2^k) mod P (reflected)
  uint8_t* packed_k;
  uint8_t* packed_v;
  uint8_t* scales_k;
  uint8_t* scales_v;
  int32_t* valid;
  unsigned* status;
};

// a * b mod P for reflected CRC-32 polynomials (bit 31 is the coefficient of x^0).
__host__ __device__ inline unsigned crc_mulmod(unsigned a, unsigned b) {
  unsigned p = 0;
  for (unsigned m = 1u << 31; m != 0; m >>= 1) {
    if (a & m) p ^= b;
    b = (b & 1u) ? (b >> 1) ^ 0xEDB88320u : b >> 1;  // b *= x
  }
  return p;
}

cudaError_t launch_record_decode(const RecordArgs& a, cudaStream_t s);

}  // namespace kvb
