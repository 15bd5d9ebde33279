/*
 * kvssd_b200.h -- C ABI of the B200 fused dequantize + decode-attention library
 * (libkvssd_b200.so). Plain pointers and sizes only; every pointer argument except the
 * stream is a CUDA device pointer on the current device unless stated otherwise.
 *
 * Data layout (identical to kvssd's PackedBatch, src/kvssd/backends/base.py:19-27, and to the
 * record payload of src/kvssd/format.py:104-131):
 *   packed_k, packed_v : uint8  [n_pool_blocks, block_tokens, kv_heads, head_dim*bits/8]
 *                        codes packed low-bits-first (src/kvssd/quant.py:28-37)
 *   scales_k, scales_v : fp16   [n_pool_blocks, block_tokens, kv_heads, head_dim/group_size]
 *   valid_tokens       : int32  [n_pool_blocks], rows of each block that enter the softmax
 *   block_table        : int32  [n_sel_blocks], pool index of each selected block, in order;
 *                        NULL selects blocks 0..n_sel_blocks-1 (the stacked-PackedBatch case)
 *   query              : [query_heads, head_dim] of type query_dtype (KVSSD_B200_Q_*)
 *   out, lse           : fp32 [query_heads, head_dim] normalised output, fp32 [query_heads]
 *                        natural-log normaliser (kvssd's backend contract, base.py:76-81)
 *
 * Every entry point returns KVSSD_B200_OK (0) or a status below; none aborts or exits.
 * Kernels are enqueued on `stream`; the caller keeps all buffers alive until it completes.
 */
#ifndef KVSSD_B200_H_
#define KVSSD_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KVSSD_B200_API __attribute__((visibility("default")))
#else
#define KVSSD_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kvssd_b200_stream_t; /* == cudaStream_t; NULL = legacy stream */

enum kvssd_b200_status {
  KVSSD_B200_OK = 0,
  KVSSD_B200_ERR_INVALID_ARGUMENT = 1, /* shape/dtype/pointer contract violated */
  KVSSD_B200_ERR_UNSUPPORTED = 2,      /* valid kvssd input outside this library's range */
  KVSSD_B200_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required */
  KVSSD_B200_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed */
  KVSSD_B200_ERR_DEVICE_STATUS = 5     /* kernels flagged bad table/valid entries or a timeout */
};

enum kvssd_b200_query_dtype {
  KVSSD_B200_Q_F32 = 0,
  KVSSD_B200_Q_F16 = 1,
  KVSSD_B200_Q_BF16 = 2,
  KVSSD_B200_Q_F64 = 3
};

/* Decode kernel selection, reported by kvssd_b200_decode_path and settable for A/B runs. */
enum kvssd_b200_path {
  KVSSD_B200_PATH_AUTO = 0,
  KVSSD_B200_PATH_TENSOR_CORE = 1,     /* mma.sync split-KV tile math (head_dim 64/128/256,
                                          group >= 16); streamed where it qualifies: TMA-fed
                                          (INT4/INT2, head_dim 128, 4/8/16 KV heads), else
                                          cp.async-fed */
  KVSSD_B200_PATH_GENERIC = 2,         /* CUDA-core split-KV kernel (any head_dim <= 256) */
  KVSSD_B200_PATH_TENSOR_CORE_REGS = 3, /* override only: tensor-core tile math fed by
                                          per-thread global loads (no shared-memory ring) */
  KVSSD_B200_PATH_TENSOR_CORE_CPASYNC = 4 /* the streaming kernel fed by per-warp cp.async
                                          rings (as an override: never the TMA-fed one) */
};

/* Library ABI version (incremented on any signature change). No reference counterpart. */
KVSSD_B200_API int kvssd_b200_version(void);

/* Static description of a status code. No reference counterpart. */
KVSSD_B200_API const char* kvssd_b200_status_string(int status);

/* Detail of the last error raised on the calling thread (empty if none). No reference
 * counterpart: the reference op raises the message through TORCH_CHECK
 * (csrc/bindings.cpp:26-38). */
KVSSD_B200_API const char* kvssd_b200_last_error(void);

/* Bytes of device workspace kvssd_b200_decode needs for this geometry on the current device.
 * Replaces the per-call torch allocations of the reference op (csrc/fused_decode.cu:125-127). */
KVSSD_B200_API int kvssd_b200_decode_workspace_size(int n_sel_blocks, int block_tokens, int query_heads,
                                     int kv_heads, int head_dim, int bits, int group_size,
                                     size_t* bytes);

/* Fused dequantize + single-token GQA decode attention over the selected packed blocks.
 * Replaces kvssd._C.fused_decode (csrc/bindings.cpp:16-41 -> csrc/fused_decode.cu:92-142),
 * bound from CudaExtensionBackend.run (src/kvssd/backends/cuda.py:31-48). Same preconditions
 * (bindings.cpp:26-38, fused_decode.cu:117-121) plus the block table. Invalid block-table or
 * valid_tokens entries are never dereferenced: they are skipped/clamped and recorded in the
 * workspace status word (see kvssd_b200_read_status). Outputs: out, lse as in the header.
 * The workspace (>= kvssd_b200_decode_workspace_size bytes, 16-byte aligned) starts with a
 * 2048-byte header holding that sticky status word and the call epoch of the fused combine
 * (the streaming kernel folds its split-KV parts itself: every part value is written with the
 * call's epoch beside it and the folding CTAs poll the values), followed by the parts: zero
 * the WHOLE workspace once after allocating it, so that no leftover word carries a future
 * epoch. Calls sharing one workspace must be ordered on the GPU (same stream or explicit
 * events). */
KVSSD_B200_API int kvssd_b200_decode(const void* query, int query_dtype, const uint8_t* packed_k,
                      const uint8_t* packed_v, const uint16_t* scales_k,
                      const uint16_t* scales_v, const int32_t* valid_tokens,
                      const int32_t* block_table, int n_pool_blocks, int n_sel_blocks,
                      int block_tokens, int query_heads, int kv_heads, int head_dim, int bits,
                      int group_size, float sm_scale, float* out, float* lse, void* workspace,
                      size_t workspace_bytes, kvssd_b200_stream_t stream);

/* Bytes of the device scratch behind kvssd_b200_decode_static (one array per device). */
#define KVSSD_B200_STATIC_SCRATCH_BYTES (8u << 20)

/* kvssd_b200_decode without a caller workspace and without allocating anything: the split-KV
 * parts and the status word live in a file-scope __device__ array of
 * KVSSD_B200_STATIC_SCRATCH_BYTES per device. No counterpart in the reference (its op
 * allocates its outputs with torch on every call, csrc/fused_decode.cu:125-127).
 * For callers that cannot allocate device memory on the decode path: hosts that bind the C ABI
 * without a device allocator of their own (a plain C, cgo or JNI host), and serving loops
 * that must not call cudaMalloc/cudaFree there, which synchronise the device.
 * Limits: a geometry whose plan needs more than KVSSD_B200_STATIC_SCRATCH_BYTES (2048 bytes of
 * header plus n_parts * query_heads * (head_dim + 2) * 8; the c2 shape needs 4.9 MB) is
 * rejected with KVSSD_B200_ERR_WORKSPACE before anything is launched. The first call on each
 * device resolves the scratch address and zeroes the scratch on `stream`; make that first call
 * before any stream capture. The address is kept per device and driver context: after
 * cudaDeviceReset the next call (again before any capture) sets the new context's scratch up
 * the same way. After a call that flagged a wait that gave up (status bits 4, 8 or 32), call
 * kvssd_b200_read_status on the scratch with clear = 1: it zeroes the sticky word, and the
 * next call is good again.
 * Every call on a device uses the same scratch, so calls on one device must not overlap in
 * time (one stream, or events between streams): overlapping calls race on the parts.
 * If `scratch` is not NULL it receives the scratch address, which kvssd_b200_read_status
 * accepts as the workspace. Other arguments and outputs as kvssd_b200_decode. */
KVSSD_B200_API int kvssd_b200_decode_static(const void* query, int query_dtype,
                      const uint8_t* packed_k, const uint8_t* packed_v,
                      const uint16_t* scales_k, const uint16_t* scales_v,
                      const int32_t* valid_tokens, const int32_t* block_table,
                      int n_pool_blocks, int n_sel_blocks, int block_tokens, int query_heads,
                      int kv_heads, int head_dim, int bits, int group_size, float sm_scale,
                      float* out, float* lse, void** scratch, kvssd_b200_stream_t stream);

/* The two stages of kvssd_b200_decode, for callers that consume or exchange the split-KV
 * state themselves (e.g. timing the streaming kernel alone). decode_split takes the decode
 * arguments minus out/lse, runs the streaming kernel only and returns in *n_parts the number
 * of (m, l, acc) parts it wrote to the workspace; decode_combine folds them into out/lse.
 * No reference counterpart (the reference op is a single kernel, csrc/fused_decode.cu:92). */
KVSSD_B200_API int kvssd_b200_decode_split(const void* query, int query_dtype, const uint8_t* packed_k,
                            const uint8_t* packed_v, const uint16_t* scales_k,
                            const uint16_t* scales_v, const int32_t* valid_tokens,
                            const int32_t* block_table, int n_pool_blocks, int n_sel_blocks,
                            int block_tokens, int query_heads, int kv_heads, int head_dim,
                            int bits, int group_size, float sm_scale, void* workspace,
                            size_t workspace_bytes, int* n_parts, kvssd_b200_stream_t stream);
KVSSD_B200_API int kvssd_b200_decode_combine(const void* workspace, int n_parts, int query_heads,
                              int head_dim, float* out, float* lse, kvssd_b200_stream_t stream);

/* Which decode kernel kvssd_b200_decode would run for this geometry (KVSSD_B200_PATH_*).
 * No reference counterpart (the reference has one kernel). */
KVSSD_B200_API int kvssd_b200_decode_path(int head_dim, int bits, int group_size, int* path);

/* Launch plan kvssd_b200_decode would use on the current device for 16-byte aligned operands:
 * *kernel = KVSSD_B200_PATH_TENSOR_CORE (TMA-fed streaming kernel), _TENSOR_CORE_CPASYNC
 * (cp.async-fed streaming kernel), _TENSOR_CORE_REGS or _GENERIC; the number of
 * split CTAs and of (m, l, acc) parts. No reference counterpart. */
KVSSD_B200_API int kvssd_b200_decode_plan(int n_sel_blocks, int block_tokens, int query_heads,
                                          int kv_heads, int head_dim, int bits, int group_size,
                                          int* kernel, int* n_splits, int* n_parts);

/* Process-wide override of the decode kernel choice (KVSSD_B200_PATH_*), for A/B
 * measurements and tests; AUTO restores the default. No reference counterpart. */
KVSSD_B200_API int kvssd_b200_set_path_override(int path);

/* Decodes n_records raw kvssd records already in device memory (record i at
 * records + i * record_stride, the store's record_bytes) into PackedBatch tensors: packed_k /
 * packed_v [n, bt, kvh, d*bits/8] u8, scales_k / scales_v [n, bt, kvh, d/group] FP16 bits,
 * valid_tokens [n]. The header of each record (magic, version, geometry, payload length,
 * optionally layer and block) is validated and the payload's zlib CRC-32 recomputed on the
 * device; record_status[i] receives the OR of 1 = bad magic/version, 2 = geometry differs from
 * the arguments, 4 = payload length differs, 8 = CRC mismatch, 16 = layer/block differs from
 * `layer` (if >= 0) / expected_blocks[i] (if not NULL), 32 = valid count above block_tokens
 * (clamped). Records with status bits 1, 2 or 4 are not copied and get valid 0. Asynchronous on
 * `stream`. With 16-byte aligned records, stride and outputs and both section sizes
 * (bt*kvh*(d/group)*2 and bt*kvh*d*bits/8 bytes) multiples of 16, as in the c1-c5 geometries,
 * one streaming kernel does the copy and the CRC in a single pass, after a small kernel that zeroes
 * record_status and valid_tokens (they hold the per-record CRC partials and row counts until
 * the last contribution writes the final values); other inputs take a per-record kernel.
 * Replaces the CPU decode_record of the reference loader (src/kvssd/format.py:134-177,
 * src/kvssd/loader.py:104-128), which checks the CRC on the host. */
KVSSD_B200_API int kvssd_b200_decode_records(const uint8_t* records, size_t record_stride,
                      int n_records, int layer, const int32_t* expected_blocks, int bits,
                      int block_tokens, int kv_heads, int head_dim, int group_size,
                      uint8_t* packed_k, uint8_t* packed_v, uint16_t* scales_k,
                      uint16_t* scales_v, int32_t* valid_tokens, unsigned* record_status,
                      kvssd_b200_stream_t stream);

/* Reads n_records whole records (record_bytes each, at the given byte offsets of the store
 * file `path`) into `destination` (n_records * record_bytes bytes, record i at
 * i * record_bytes) with `threads` reader threads. With `direct` nonzero and 4 KiB-aligned
 * offsets, sizes and destination the file is opened with O_DIRECT (page cache bypassed), else
 * (or where the file system refuses O_DIRECT) with buffered pread; *used_direct (if not NULL)
 * tells which. Host-only: a pinned buffer here feeds kvssd_b200_decode_records after one
 * host-to-device copy. Replaces the reference's storage backends' record reads
 * (src/kvssd/storage/direct.py:64-88, buffered.py:53-76) for whole-record batches. On error
 * kvssd_b200_io_last_error describes it. */
KVSSD_B200_API int kvssd_b200_read_records(const char* path, const long long* offsets,
                                           int n_records, size_t record_bytes, void* destination,
                                           int threads, int direct, int* used_direct);
KVSSD_B200_API const char* kvssd_b200_io_last_error(void);

/* Page-locked store files (the "mapped" storage backend): host_register registers a host
 * range -- a store file mapped read-only with mmap, read_only = 1 -- with the CUDA driver
 * (cudaHostRegister, portable; read-only where asked), and copy_records_h2d then copies
 * n_records records of record_bytes at byte offsets of that range into device_destination +
 * i * record_bytes on `stream`, asynchronously, one cudaMemcpyAsync per run of records that are
 * consecutive in the file: the records travel by DMA from the page cache, with no reader
 * threads and no staging copy (the reference reads them into a host buffer first,
 * src/kvssd/storage/buffered.py:53-76, src/kvssd/pipeline.py:118-165). A record that does not
 * lie wholly inside [0, host_bytes) is refused (KVSSD_B200_ERR_INVALID_ARGUMENT) before anything
 * is copied;
 * a range the driver will not register gives KVSSD_B200_ERR_UNSUPPORTED with the reason in
 * kvssd_b200_host_last_error. */
KVSSD_B200_API int kvssd_b200_host_register(void* ptr, size_t bytes, int read_only);
KVSSD_B200_API int kvssd_b200_host_unregister(void* ptr);
KVSSD_B200_API int kvssd_b200_copy_records_h2d(const void* host_base, size_t host_bytes,
                                               const long long* offsets, int n_records,
                                               size_t record_bytes, void* device_destination,
                                               kvssd_b200_stream_t stream);
KVSSD_B200_API const char* kvssd_b200_host_last_error(void);

/* GPUDirect Storage (cuFile) reads of whole records straight into device memory: kvssd's
 * "gds" storage backend (src/kvssd/storage/gds.py:13-94 over csrc/gds_bindings.cpp:21-98,
 * GDSFile: cuFileDriverOpen, O_DIRECT open, cuFileHandleRegister, cuFileRead). libcufile is
 * loaded at run time; where it, its driver or an O_DIRECT descriptor is unavailable, open
 * returns KVSSD_B200_ERR_UNSUPPORTED and kvssd_b200_gds_last_error gives the reason (the
 * reference's probe() reports the same as unavailable). read_records reads n_records records
 * of record_bytes (a multiple of 4096) at the 4096-aligned file offsets into
 * device_destination + i * record_bytes (4096-byte aligned device memory), with up to
 * `threads` reader threads; synchronous (the data is in device memory on return). Errors:
 * KVSSD_B200_ERR_INVALID_ARGUMENT for misaligned requests, KVSSD_B200_ERR_CUDA for a failed or
 * short cuFileRead (the reference raises OSError / EOFError). */
typedef struct kvssd_b200_gds_file kvssd_b200_gds_file;
KVSSD_B200_API int kvssd_b200_gds_open(const char* path, kvssd_b200_gds_file** file);
KVSSD_B200_API int kvssd_b200_gds_read_records(kvssd_b200_gds_file* file,
                                               const long long* offsets, int n_records,
                                               size_t record_bytes, void* device_destination,
                                               int threads);
KVSSD_B200_API int kvssd_b200_gds_close(kvssd_b200_gds_file* file);
KVSSD_B200_API const char* kvssd_b200_gds_last_error(void);

/* One problem of a batched decode: its query [query_heads, head_dim], block pool
 * (PackedBatch layout), optional block table (NULL = all pool blocks in order) and outputs.
 * Problems of one batch share the geometry; their pools may be shared (a batch of sequences
 * over one paged pool) or separate (several layers). */
typedef struct kvssd_b200_problem {
  const void* query;
  const uint8_t* packed_k;
  const uint8_t* packed_v;
  const uint16_t* scales_k;
  const uint16_t* scales_v;
  const int32_t* valid_tokens;
  const int32_t* block_table;
  float* out;
  float* lse;
  int n_pool_blocks;
  int n_sel_blocks;
} kvssd_b200_problem;

/* Workspace bytes of kvssd_b200_decode_batched for n_problems problems. No reference
 * counterpart. */
KVSSD_B200_API int kvssd_b200_decode_batched_workspace_size(int n_problems, int block_tokens,
                      int query_heads, int kv_heads, int head_dim, int bits, int group_size,
                      size_t* bytes);

/* n_problems independent decodes in ONE launch: `problems` is a DEVICE array of
 * kvssd_b200_problem (so the call can be captured in a CUDA graph and replayed with new
 * descriptor contents). The grid gets floor(SMs / n_problems) CTAs per problem (at least 1);
 * each problem's split-KV parts are folded by its own CTAs in the grid's tail. Needs the
 * streaming kernel's shapes (INT4, head_dim 128, group 32 or 64, 16-byte aligned operands)
 * and n_problems <= the SM count; workspace as kvssd_b200_decode (zero it once). Amortises the per-decode tail and launch over a multi-layer step or a batch of
 * sequences (the reference decodes one layer per call, src/kvssd/pipeline.py:167-187). No
 * reference counterpart. */
KVSSD_B200_API int kvssd_b200_decode_batched(const kvssd_b200_problem* problems, int n_problems,
                      int query_dtype, int block_tokens, int query_heads, int kv_heads,
                      int head_dim, int bits, int group_size, float sm_scale, void* workspace,
                      size_t workspace_bytes, kvssd_b200_stream_t stream);

/* Size of a CUDA IPC memory handle (cudaIpcMemHandle_t). */
#define KVSSD_B200_IPC_HANDLE_BYTES 64

/* Bytes of one rank's exchange buffer for kvssd_b200_decode_exchange with `world` ranks.
 * No reference counterpart (the reference runs on one device). */
KVSSD_B200_API int kvssd_b200_exchange_bytes(int world, int query_heads, int head_dim,
                                             size_t* bytes);

/* Allocates and zeroes an exchange buffer on the current device (cudaMalloc; 256-byte
 * aligned), re-zeroes it (synchronously, e.g. after an exchange timeout) and frees it. Call
 * outside any stream capture. No reference counterpart (the reference runs on one device). */
KVSSD_B200_API int kvssd_b200_exchange_alloc(size_t bytes, void** buffer);
KVSSD_B200_API int kvssd_b200_exchange_clear(void* buffer, size_t bytes);
KVSSD_B200_API int kvssd_b200_exchange_free(void* buffer);

/* CUDA IPC export of an exchange buffer into a KVSSD_B200_IPC_HANDLE_BYTES handle, import of a
 * peer process's handle (peer access enabled lazily) and release of the import. No reference
 * counterpart (the reference runs on one device). */
KVSSD_B200_API int kvssd_b200_ipc_handle(void* buffer, void* handle);
KVSSD_B200_API int kvssd_b200_ipc_open(const void* handle, void** buffer);
KVSSD_B200_API int kvssd_b200_ipc_close(void* buffer);

/* Multi-GPU decode of one context split by token-block ranges, one process per GPU: the
 * decode of this rank's blocks, its split-KV combine and the exact cross-rank merge in ONE
 * kernel. Each combined (query head, 32-dim) slice is pushed with peer stores over NVLink into
 * every rank's exchange buffer (`buffers`: `world` device pointers, this rank's own at index
 * `rank`, peers' from kvssd_b200_ipc_open) and merged from there once all ranks' copies of the
 * slice have arrived; every rank ends with the same out/lse for the whole context. Replaces the
 * per-chunk pairwise merges of the reference pipeline (src/kvssd/pipeline.py:147-153,
 * merge_attention_chunks at src/kvssd/attention.py:91-102) when the chunks live on different
 * GPUs. Every rank makes the same sequence of calls; the calls are numbered on the device (the
 * buffer's header), so they may be captured in a CUDA graph. A rank that does not arrive
 * within about a second makes the others flag status bit 8 (kvssd_b200_read_status) and
 * return; the ranks' call numbers then differ, and the group re-zeroes its buffers (after a
 * barrier) before the next call. Requires a streaming kernel's shapes (INT4 or INT2, head_dim 128,
 * group 32/64, 16-byte aligned operands) and a cooperative launch; other arguments as
 * kvssd_b200_decode. No reference counterpart. */
KVSSD_B200_API int kvssd_b200_decode_exchange(const void* query, int query_dtype,
                      const uint8_t* packed_k, const uint8_t* packed_v,
                      const uint16_t* scales_k, const uint16_t* scales_v,
                      const int32_t* valid_tokens, const int32_t* block_table,
                      int n_pool_blocks, int n_sel_blocks, int block_tokens, int query_heads,
                      int kv_heads, int head_dim, int bits, int group_size, float sm_scale,
                      int rank, int world, void* const* buffers, float* out,
                      float* lse, void* workspace, size_t workspace_bytes,
                      kvssd_b200_stream_t stream);

/* Reads (synchronising `stream`) and optionally clears the device status word of a decode
 * workspace; *device_status receives the OR of flagged conditions (1 = block-table entry out
 * of range, 2 = valid_tokens entry out of [0, block_tokens], 4 = a fused combine gave up after
 * waiting about a second for the other CTAs' parts, 8 = a cross-GPU exchange gave up waiting
 * for another rank, 16 = a batched problem descriptor was refused, 32 = a TMA-fed kernel gave
 * up waiting for its copies). After bits 4, 8 or 32 the kernels write NaN into out and lse of
 * that call and of every later call on the workspace until the word is cleared, so a failure
 * is never returned as a plausible number. clear = 1 with a nonzero word zeroes the word
 * (and the fused combine's test hook), which makes the workspace usable again; the epoch is
 * kept, since the parts of earlier calls carry older ones. Returns KVSSD_B200_ERR_DEVICE_STATUS when the word is nonzero. No
 * reference counterpart (the reference raises through TORCH_CHECK,
 * csrc/fused_decode.cu:141). */
KVSSD_B200_API int kvssd_b200_read_status(void* workspace, int clear, unsigned* device_status,
                           kvssd_b200_stream_t stream);

/* Exact N-way merge of normalised chunks: outs fp32 [n_chunks, query_heads, head_dim],
 * lses fp32 [n_chunks, query_heads] -> out, lse. Generalises merge_attention_chunks
 * (src/kvssd/attention.py:91-102) as used by the streamed pipeline
 * (src/kvssd/pipeline.py:147-153); chunks with lse = -inf contribute nothing. */
KVSSD_B200_API int kvssd_b200_merge_chunks(const float* outs, const float* lses, int n_chunks, int query_heads,
                            int head_dim, float* out, float* lse, kvssd_b200_stream_t stream);

/* merge_attention_chunks (src/kvssd/attention.py:91-102), term for term, for two chunks. */
KVSSD_B200_API int kvssd_b200_merge_pair(const float* left_out, const float* left_lse, const float* right_out,
                          const float* right_lse, int query_heads, int head_dim, float* out,
                          float* lse, kvssd_b200_stream_t stream);

/* Materialises unpacked codes and FP16 dequantized values with the decode kernels' register
 * unpackers, for bit-exact comparison with unpack_codes / dequantize_tensor(q, float16)
 * (src/kvssd/quant.py:40-46, 68-73). packed uint8 [rows, head_dim*bits/8], scales fp16
 * [rows, head_dim/group_size] -> values fp16 [rows, head_dim], codes uint8 [rows, head_dim].
 * mode 0 decodes word-wise (K operand path), mode 1 pairs rows 2r, 2r+1 (V operand path;
 * rows must be even). */
KVSSD_B200_API int kvssd_b200_dequantize(const uint8_t* packed, const uint16_t* scales, long long rows,
                          int head_dim, int bits, int group_size, int mode, uint16_t* values,
                          uint8_t* codes, kvssd_b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KVSSD_B200_H_ */
