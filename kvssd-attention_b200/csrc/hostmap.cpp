// Page-locked record ranges: a store file mapped read-only into the process (mmap) is
// registered with the CUDA driver, so the records of a selection travel to the device by DMA
// straight from the page cache, with no reader threads and no staging copy. Serves the
// "mapped" storage backend of KVCacheStore; the reference reads every record into a host
// buffer first (src/kvssd/storage/buffered.py:53-76, src/kvssd/pipeline.py:118-165). Host
// code: no kernels.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/kvssd_b200.h"

namespace {

thread_local std::string g_map_error;

int map_fail(int code, const std::string& what) {
  g_map_error = what;
  return code;
}

}  // namespace

extern "C" {

const char* kvssd_b200_host_last_error(void) { return g_map_error.c_str(); }

int kvssd_b200_host_register(void* ptr, size_t bytes, int read_only) {
  g_map_error.clear();
  if (!ptr || bytes == 0) return map_fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "empty range");
  unsigned flags = cudaHostRegisterPortable;
  if (read_only) flags |= cudaHostRegisterReadOnly;
  const cudaError_t e = cudaHostRegister(ptr, bytes, flags);
  if (e != cudaSuccess) {
    cudaGetLastError();  // the failure is reported here, not left for the next call
    return map_fail(KVSSD_B200_ERR_UNSUPPORTED,
                    std::string("cudaHostRegister: ") + cudaGetErrorString(e));
  }
  return KVSSD_B200_OK;
}

int kvssd_b200_host_unregister(void* ptr) {
  g_map_error.clear();
  if (!ptr) return KVSSD_B200_OK;
  const cudaError_t e = cudaHostUnregister(ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return map_fail(KVSSD_B200_ERR_CUDA, std::string("cudaHostUnregister: ") + cudaGetErrorString(e));
  }
  return KVSSD_B200_OK;
}

int kvssd_b200_copy_records_h2d(const void* host_base, size_t host_bytes,
                                const long long* offsets, int n_records, size_t record_bytes,
                                void* device_destination, kvssd_b200_stream_t stream) {
  g_map_error.clear();
  if (!host_base || !offsets || !device_destination || n_records < 0 || record_bytes == 0)
    return map_fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bad arguments");
  for (int i = 0; i < n_records; ++i)  // offset + record_bytes <= host_bytes, without overflow
    if (offsets[i] < 0 || record_bytes > host_bytes ||
        static_cast<unsigned long long>(offsets[i]) > host_bytes - record_bytes)
      return map_fail(KVSSD_B200_ERR_INVALID_ARGUMENT,
                      "record " + std::to_string(i) + " lies outside the mapped range");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const auto* src = static_cast<const uint8_t*>(host_base);
  auto* dst = static_cast<uint8_t*>(device_destination);
  // One copy per run of records that are consecutive in the file (and so in the destination).
  for (int i = 0; i < n_records;) {
    int j = i + 1;
    while (j < n_records &&
           offsets[j] == offsets[j - 1] + static_cast<long long>(record_bytes))
      ++j;
    const size_t bytes = static_cast<size_t>(j - i) * record_bytes;
    const cudaError_t e = cudaMemcpyAsync(dst + static_cast<size_t>(i) * record_bytes,
                                          src + offsets[i], bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess)
      return map_fail(KVSSD_B200_ERR_CUDA, std::string("cudaMemcpyAsync: ") + cudaGetErrorString(e));
    i = j;
  }
  return KVSSD_B200_OK;
}

}  // extern "C"
