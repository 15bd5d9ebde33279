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
// Two kernels. The streaming one (record_stream_kernel, below) takes every input whose
// buffers are 16-byte aligned and whose sections are whole 16-byte units: one pass over the
// records, copy and CRC together. The per-record kernel (record_decode_kernel) takes the rest:
// one CTA per record. Pass 1 copies the payload's four sections into their PackedBatch tensors
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

#include <algorithm>
#include <mutex>
#include <vector>

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

// ---------------------------------------------------------------------------------------------
// Streaming decode. Every warp walks a run of whole 512-byte rows of the records: lane l loads
// piece 3 + 32 k + l of row k (16 bytes at record offset 48 + 512 k + 16 l, one coalesced 512-byte
// read per warp and row), stores the payload's 16-byte unit that starts 4 bytes into it (the
// payload begins at offset 52, so unit j is words 1..3 of piece 3 + j and word 0 of the next
// piece, taken from the neighbouring lane) into its PackedBatch section, and folds the piece into
// its own CRC register S_l. The lane's stream is "piece, 496 zero bytes, piece, ...", i.e.
//   S_l <- crc(S_l, piece || 0^496) = sum_w word_w(piece ^ S_l) * x^(8 (512 - 4 w)) mod P,
// a linear map of the piece evaluated with 32 nibble tables of 16 entries (one per nibble of the
// piece; a table sits in 16 consecutive banks, so every lookup of a warp is conflict-free). At
// the end of a run the lanes' registers are moved to the row end (S_l * x^(128 (31 - l)), eight
// per-lane nibble tables) and XORed over the warp; that is the CRC (zero preset) of the run's
// rows, times x^(128 * 31). A constant per last chunk moves it to the end of the payload and
// removes the x^(128 * 31) and the zero bytes past the payload (the masked header word before
// the payload, a leading zero, does not change a zero-preset CRC). The runs of one record XOR
// into record_status[r] (the accumulator) and count their rows in valid_tokens[r]; the run that
// completes the count adds zlib's preset and writes the record's final status and valid count.
// Both arrays are zeroed by record_zero_kernel right before (programmatic dependent launch: the
// tables are built while it runs).

__device__ __forceinline__ unsigned crc_mulx(unsigned a) {
  return (a >> 1) ^ ((a & 1u) ? 0xEDB88320u : 0u);
}

// out[n * stride] = (n << 4 j) * c mod P for n < 16 (bit b of a word is the coefficient of
// x^(31 - b)): the table of one nibble of a multiplication by the constant c.
__device__ void nibble_table(unsigned c, int j, unsigned* out, int stride) {
  for (int i = 0; i < 28 - 4 * j; ++i) c = crc_mulx(c);
  const unsigned b3 = c, b2 = crc_mulx(b3), b1 = crc_mulx(b2), b0 = crc_mulx(b1);
  for (int n = 0; n < 16; ++n)
    out[n * stride] = ((n & 1) ? b0 : 0u) ^ ((n & 2) ? b1 : 0u) ^ ((n & 4) ? b2 : 0u) ^
                      ((n & 8) ? b3 : 0u);
}

// Shared-memory word at byte address addr + kOff (immediate offset).
template <int kOff>
__device__ __forceinline__ unsigned lds_at(unsigned addr) {
  unsigned v;
  asm("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(kOff));
  return v;
}

// word_W(piece) * x^(8 (512 - 4 W)) mod P from the tables 8 W .. 8 W + 7 (64 bytes each) of the
// 256-byte aligned table block at shared address `base`. The byte offsets 4 n of a word's
// nibbles are spread over two registers (lo: even nibbles, hi: odd ones, one per byte); one byte
// permute per lookup pastes an offset under the base's upper bytes, the table's own offset
// rides in the load's immediate.
template <int W>
__device__ __forceinline__ unsigned fold_word(unsigned v, unsigned base) {
  const unsigned lo = (v << 2) & 0x3C3C3C3Cu;  // byte k: 4 * nibble 2 k
  const unsigned hi = (v >> 2) & 0x3C3C3C3Cu;  // byte k: 4 * nibble 2 k + 1
  return lds_at<64 * (8 * W + 0)>(__byte_perm(lo, base, 0x7650u)) ^
         lds_at<64 * (8 * W + 1)>(__byte_perm(hi, base, 0x7650u)) ^
         lds_at<64 * (8 * W + 2)>(__byte_perm(lo, base, 0x7651u)) ^
         lds_at<64 * (8 * W + 3)>(__byte_perm(hi, base, 0x7651u)) ^
         lds_at<64 * (8 * W + 4)>(__byte_perm(lo, base, 0x7652u)) ^
         lds_at<64 * (8 * W + 5)>(__byte_perm(hi, base, 0x7652u)) ^
         lds_at<64 * (8 * W + 6)>(__byte_perm(lo, base, 0x7653u)) ^
         lds_at<64 * (8 * W + 7)>(__byte_perm(hi, base, 0x7653u));
}

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void record_zero_kernel(unsigned* status, int32_t* valid, int n) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    status[i] = 0u;
    valid[i] = 0;
  }
}

__global__ void __launch_bounds__(kRecStreamThreads, 2)
    record_stream_kernel(const __grid_constant__ RecordStreamArgs a) {
  __shared__ __align__(256) unsigned s_tab[32 * 16];      // [8 w + j][n]
  __shared__ __align__(16) unsigned s_lane[8 * 16 * 32];  // [j][n][lane]
  const int t = threadIdx.x, lane = t & 31;
  if (t < 256) {
    nibble_table(a.lane_shift[t & 31], t >> 5, s_lane + (t >> 5) * 512 + (t & 31), 32);
  } else if (t < 288) {
    const int u = t - 256;
    nibble_table(a.word_shift[u >> 3], u & 7, s_tab + 16 * u, 1);
  }
  __syncthreads();
  asm volatile("griddepcontrol.wait;" ::: "memory");  // status / valid zeroed, records written
  const unsigned tab = static_cast<unsigned>(__cvta_generic_to_shared(s_tab));
  const RecordArgs& ra = a.r;
  const int nrows = a.nrows, q_last = a.q_last, nj = a.nj;
  // Sections in 16-byte units of the payload: [0, e0) K scales, [e0, e1) V scales,
  // [e1, e2) K codes, [e2, nj) V codes.
  const int e0 = a.sb16, e1 = 2 * a.sb16, e2 = 2 * a.sb16 + a.pb16;
  // Contiguous chunk ranges: per CTA, then per warp.
  const long long total = static_cast<long long>(ra.n) * a.nchunks;
  const long long c0 = total * blockIdx.x / gridDim.x, c1 = total * (blockIdx.x + 1) / gridDim.x;
  const int nw = blockDim.x >> 5, w = t >> 5;
  const long long w0 = c0 + (c1 - c0) * w / nw, w1 = c0 + (c1 - c0) * (w + 1) / nw;
  for (long long c = w0; c < w1;) {
    const int r = static_cast<int>(c / a.nchunks);
    const int cr = static_cast<int>(c - static_cast<long long>(r) * a.nchunks);
    const int cend = static_cast<int>(min(static_cast<long long>(a.nchunks),
                                          w1 - static_cast<long long>(r) * a.nchunks));
    c = static_cast<long long>(r) * a.nchunks + cend;
    const int k0 = cr * a.rows_per_chunk, k1 = min(cend * a.rows_per_chunk, nrows);
    const uint8_t* rec = ra.records + static_cast<size_t>(r) * ra.stride;
    // header: magic (2 words), version, layer, block, valid, bits, bt, kvh, d, group, len, crc
    const unsigned hw = lane < 13 ? reinterpret_cast<const unsigned*>(rec)[lane] : 0u;
    unsigned h[13];
#pragma unroll
    for (int i = 0; i < 13; ++i) h[i] = __shfl_sync(0xffffffffu, hw, i);
    unsigned st = 0;
    if (h[0] != 0x5353564Bu || h[1] != 0x31303044u || h[2] != 1u) st |= 1u;  // "KVSSD001"
    if (static_cast<int>(h[6]) != ra.bits || static_cast<int>(h[7]) != ra.bt ||
        static_cast<int>(h[8]) != ra.kvh || static_cast<int>(h[9]) != ra.d ||
        static_cast<int>(h[10]) != ra.group)
      st |= 2u;
    if (h[11] != static_cast<unsigned>(16 * nj)) st |= 4u;
    if ((ra.layer >= 0 && static_cast<int>(h[3]) != ra.layer) ||
        (ra.blocks && static_cast<int>(h[4]) != ra.blocks[r]))
      st |= 16u;
    const unsigned hvalid = h[5], hcrc = h[12];
    if (hvalid > static_cast<unsigned>(ra.bt)) st |= 32u;
    if (st & 7u) {  // the payload cannot be trusted to have this layout: leave the slots alone
      if (k0 == 0 && lane == 0) {
        ra.status[r] = st;
        ra.valid[r] = 0;
      }
      continue;
    }
    // This lane's output unit j = 32 k + lane goes to dst + j, dst offset so that the unit
    // lands at its place in the current section; bound: the unit where the next one starts.
    const size_t sbytes = static_cast<size_t>(ra.scale_bytes), pbytes = static_cast<size_t>(ra.packed_bytes);
    int j = 32 * k0 + lane, sec = 0, bound = e0;
    uint4* dst = reinterpret_cast<uint4*>(ra.scales_k + r * sbytes);
    auto next_section = [&]() {
      ++sec;
      if (sec == 1) {
        dst = reinterpret_cast<uint4*>(ra.scales_v + r * sbytes) - e0;
        bound = e1;
      } else if (sec == 2) {
        dst = reinterpret_cast<uint4*>(ra.packed_k + r * pbytes) - e1;
        bound = e2;
      } else {
        dst = reinterpret_cast<uint4*>(ra.packed_v + r * pbytes) - e2;
        bound = 0x7fffffff;
      }
    };
    while (j >= bound) next_section();
    // Rows this lane loads: one past the run (the last unit's word 0), none past q_last.
    const int span = q_last - 3 - lane;  // rows [0, span / 32] hold a piece of this lane
    const int klim = span < 0 ? 0 : min(min(k1 + 1, nrows), span / 32 + 1);
    const uint4* src = reinterpret_cast<const uint4*>(rec) + 3 + lane;
    auto load = [&](int k) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (k < klim) v = __ldcs(src + 32 * k);
      return v;
    };
    uint4 cur = load(k0), nxt = load(k0 + 1);
    unsigned S = 0;
    for (int k = k0; k < k1; ++k, j += 32) {
      uint4 p = cur;
      cur = nxt;
      nxt = load(k + 2);
      // copy: unit j is words 1..3 of p and word 0 of the next piece
      const unsigned nx = __shfl_sync(0xffffffffu, lane == 0 ? cur.x : p.x, (lane + 1) & 31);
      if (j < nj) {
        while (j >= bound) next_section();
        dst[j] = make_uint4(p.y, p.z, p.w, nx);
      }
      // CRC: the header word before the payload and the bytes after it count as zeros (the
      // payload is whole 16-byte units and starts at offset 52, so it ends 4 bytes into q_last)
      if (k == 0 || k == nrows - 1) {
        if (k == 0 && lane == 0) p.x = 0u;
        if (3 + j == q_last) p.y = p.z = p.w = 0u;
      }
      p.x ^= S;
      S = fold_word<0>(p.x, tab) ^ fold_word<1>(p.y, tab) ^ fold_word<2>(p.z, tab) ^
          fold_word<3>(p.w, tab);
    }
    // to the row end, then over the warp
    unsigned g = 0;
#pragma unroll
    for (int jn = 0; jn < 8; ++jn) g ^= s_lane[jn * 512 + ((S >> (4 * jn)) & 15u) * 32 + lane];
#pragma unroll
    for (int o = 16; o; o >>= 1) g ^= __shfl_xor_sync(0xffffffffu, g, o);
    if (lane == 0) {
      const unsigned part = crc_mulmod(g, a.chunk_shift[cend - 1]);
      unsigned* acc = ra.status + r;
      atomicXor(acc, part);
      const unsigned rows = static_cast<unsigned>(k1 - k0);
      if (atom_add_acq_rel(reinterpret_cast<unsigned*>(ra.valid + r), rows) + rows ==
          static_cast<unsigned>(nrows)) {
        if (~(ld_relaxed_gpu(acc) ^ a.init_term) != hcrc) st |= 8u;
        *acc = st;
        ra.valid[r] = static_cast<int>(hvalid > static_cast<unsigned>(ra.bt) ? ra.bt : hvalid);
      }
    }
  }
}

namespace {

// x^e mod P in the reflected representation (bit 31 = x^0); e may be negative (x is invertible
// mod P, whose x^0 coefficient is 1: x^-1 * c undoes one multiplication by x).
unsigned crc_xpow(long long e) {
  unsigned base;
  if (e >= 0) {
    base = crc_mulx_host(1u << 31);
  } else {
    const unsigned c = 1u << 31, b = c >> 31, t = c ^ (b ? 0xEDB88320u : 0u);
    base = (t << 1) | b;
    e = -e;
  }
  unsigned acc = 1u << 31;
  for (; e; e >>= 1) {
    if (e & 1) acc = crc_mulmod(acc, base);
    base = crc_mulmod(base, base);
  }
  return acc;
}

}  // namespace

bool record_stream_plan(const RecordArgs& a, RecordStreamArgs* s) {
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a.words || a.stride % 16 || !al16(a.records) || !al16(a.packed_k) || !al16(a.packed_v) ||
      !al16(a.scales_k) || !al16(a.scales_v) || a.scale_bytes % 16 || a.packed_bytes % 16)
    return false;
  const long long payload = 2LL * a.scale_bytes + 2LL * a.packed_bytes;
  const long long end = kRecHeaderBytes + payload;
  const long long q_last = (end - 1) / 16;
  const long long nrows = (q_last - 2 + 31) / 32;  // pieces 3 .. q_last
  if (nrows > (1LL << 24)) return false;
  // The constants depend on the section sizes only; the last few geometries are kept.
  static std::mutex mu;
  static std::vector<RecordStreamArgs> cache;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const RecordStreamArgs& c : cache)
      if (c.r.scale_bytes == a.scale_bytes && c.r.packed_bytes == a.packed_bytes) {
        *s = c;
        s->r = a;
        return true;
      }
  }
  RecordStreamArgs plan{};
  plan.r = a;
  plan.q_last = static_cast<int>(q_last);
  plan.nrows = static_cast<int>(nrows);
  plan.rows_per_chunk = static_cast<int>((nrows + kRecMaxChunks - 1) / kRecMaxChunks);
  plan.nchunks = static_cast<int>((nrows + plan.rows_per_chunk - 1) / plan.rows_per_chunk);
  plan.nj = static_cast<int>(payload / 16);
  plan.sb16 = a.scale_bytes / 16;
  plan.pb16 = a.packed_bytes / 16;
  // The CRC message of a record is bytes [48, 48 + 512 nrows): the payload and tz zero bytes.
  const long long tz = 512 * nrows - 4 - payload;
  plan.init_term = crc_mulmod(0xFFFFFFFFu, crc_xpow(8 * payload));
  for (int w = 0; w < 4; ++w) plan.word_shift[w] = crc_xpow(8LL * (512 - 4 * w));
  for (int l = 0; l < 32; ++l) plan.lane_shift[l] = crc_xpow(128LL * (31 - l));
  for (int c = 0; c < plan.nchunks; ++c) {
    const long long e = std::min<long long>(static_cast<long long>(c + 1) * plan.rows_per_chunk, nrows);
    plan.chunk_shift[c] = crc_xpow(4096 * (nrows - e) - 128LL * 31 - 8 * tz);
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() >= 8) cache.erase(cache.begin());
  cache.push_back(plan);
  *s = plan;
  return true;
}

cudaError_t launch_record_decode(const RecordArgs& a, int sms, cudaStream_t s) {
  RecordStreamArgs plan;
  if (!record_stream_plan(a, &plan)) {
    record_decode_kernel<<<a.n, kRecThreads, 0, s>>>(a);
    return cudaGetLastError();
  }
  record_zero_kernel<<<(a.n + 255) / 256, 256, 0, s>>>(a.status, a.valid, a.n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long total = static_cast<long long>(a.n) * plan.nchunks;
  const int per_cta = kRecStreamThreads / 32;
  const int grid = static_cast<int>(std::min<long long>(2LL * sms, (total + per_cta - 1) / per_cta));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kRecStreamThreads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, record_stream_kernel, plan);
}

}  // namespace kvb
