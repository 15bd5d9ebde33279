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

// a * x mod P (reflected representation).
__host__ __device__ inline unsigned crc_mulx_host(unsigned a) {
  return (a >> 1) ^ ((a & 1u) ? 0xEDB88320u : 0u);
}

// a * b mod P for reflected CRC-32 polynomials (bit 31 is the coefficient of x^0).
__host__ __device__ inline unsigned crc_mulmod(unsigned a, unsigned b) {
  unsigned p = 0;
  for (unsigned m = 1u << 31; m != 0; m >>= 1) {
    if (a & m) p ^= b;
    b = (b & 1u) ? (b >> 1) ^ 0xEDB88320u : b >> 1;  // b *= x
  }
  return p;
}

// Streaming decode (the fast path): the payload of every record, seen from record offset 48, is
// cut into 16-byte pieces and 512-byte rows of 32 pieces (one per lane of a warp); rows are
// grouped into at most kRecMaxChunks chunks per record. The host fills these constants.
constexpr int kRecStreamThreads = 512;
constexpr int kRecMaxChunks = 128;

struct RecordStreamArgs {
  RecordArgs r;
  int nrows;           // rows per record (pieces 3 .. q_last, the last row zero-extended)
  int rows_per_chunk;
  int nchunks;         // chunks per record
  int q_last;          // last piece that holds payload bytes
  int nj;              // payload size in 16-byte units (the copy's output pieces)
  int sb16, pb16;      // section sizes in 16-byte units
  unsigned init_term;  // 0xFFFFFFFF * x^(8 P) mod P(x): zlib's preset, moved past the payload
  unsigned word_shift[4];    // x^(8 (512 - 4 w)): word w of a piece, then the rest of a row
  unsigned lane_shift[32];   // x^(128 (31 - l)): lane l's stream to the row end
  unsigned chunk_shift[kRecMaxChunks];  // per last chunk of a run (see records.cu)
};

// Fills the streaming plan for `a`; false when the geometry or the alignment of the buffers
// does not allow it (the per-record kernel then runs).
bool record_stream_plan(const RecordArgs& a, RecordStreamArgs* s);

// Decodes the records of `a` with the streaming kernels when record_stream_plan allows it
// (`sms`: the device's SM count), else with the per-record kernel.
cudaError_t launch_record_decode(const RecordArgs& a, int sms, cudaStream_t s);

}  // namespace kvb
