// GPUDirect Storage record reads: whole kvssd records read by cuFile from the store file
// straight into device memory (kvssd's "gds" storage backend, src/kvssd/storage/gds.py:13-94
// over csrc/gds_bindings.cpp:21-98: O_DIRECT descriptor, cuFileHandleRegister, cuFileRead).
// libcufile is loaded at run time (dlopen), so the library itself has no link dependency on it
// and reports KVSSD_B200_ERR_UNSUPPORTED, with the reason, where cuFile cannot be used. The
// driver is opened once per process on first use and left open. A batch of records is read by
// a pool of threads on the caller's device, one cuFileRead per record (cuFile calls are thread
// safe). Host code: no kernels.
#include <cuda_runtime.h>
#include <cufile.h>
#include <dlfcn.h>
#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/kvssd_b200.h"

struct kvssd_b200_gds_file {
  int fd = -1;
  CUfileHandle_t handle{};
};

namespace {

thread_local std::string g_gds_error;

struct CuFileApi {
  CUfileError_t (*driver_open)() = nullptr;
  CUfileError_t (*handle_register)(CUfileHandle_t*, CUfileDescr_t*) = nullptr;
  void (*handle_deregister)(CUfileHandle_t) = nullptr;
  ssize_t (*read)(CUfileHandle_t, void*, size_t, off_t, off_t) = nullptr;
  std::string error;  // why the API is unusable (empty: usable)
};

std::string describe(CUfileError_t st) {
  return "cuFile error " + std::to_string(static_cast<int>(st.err)) + ", CUDA error " +
         std::to_string(static_cast<int>(st.cu_err));
}

// The resolved entry points and an open driver, or the reason there are none.
const CuFileApi& cufile() {
  static CuFileApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libcufile.so.0", RTLD_NOW | RTLD_LOCAL);
    if (!lib) lib = dlopen("libcufile.so", RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
      api.error = std::string("libcufile could not be loaded: ") + dlerror();
      return;
    }
    api.driver_open = reinterpret_cast<CUfileError_t (*)()>(dlsym(lib, "cuFileDriverOpen"));
    api.handle_register = reinterpret_cast<CUfileError_t (*)(CUfileHandle_t*, CUfileDescr_t*)>(
        dlsym(lib, "cuFileHandleRegister"));
    api.handle_deregister =
        reinterpret_cast<void (*)(CUfileHandle_t)>(dlsym(lib, "cuFileHandleDeregister"));
    api.read = reinterpret_cast<ssize_t (*)(CUfileHandle_t, void*, size_t, off_t, off_t)>(
        dlsym(lib, "cuFileRead"));
    if (!api.driver_open || !api.handle_register || !api.handle_deregister || !api.read) {
      api.error = "libcufile lacks a required entry point";
      return;
    }
    const CUfileError_t st = api.driver_open();
    if (st.err != CU_FILE_SUCCESS) api.error = "cuFileDriverOpen failed: " + describe(st);
  });
  return api;
}

int fail(int code, const std::string& what) {
  g_gds_error = what;
  return code;
}

// One record: exactly `len` bytes at file offset `off` into dst + dst_off (short reads are
// continued; a read that returns 0 before the end is an error).
bool read_record(const CuFileApi& api, kvssd_b200_gds_file* f, void* dst, size_t len,
                 long long off, long long dst_off, std::string* err) {
  size_t done = 0;
  while (done < len) {
    const ssize_t got = api.read(f->handle, dst, len - done, static_cast<off_t>(off + done),
                                 static_cast<off_t>(dst_off + done));
    if (got < 0) {
      *err = "cuFileRead failed (" + std::to_string(got) + ")";
      if (got >= -4096) *err += std::string(": ") + strerror(static_cast<int>(-got));
      return false;
    }
    if (got == 0) {
      *err = "short cuFile read: end of file before the record ends";
      return false;
    }
    done += static_cast<size_t>(got);
  }
  return true;
}

}  // namespace

extern "C" {

const char* kvssd_b200_gds_last_error(void) { return g_gds_error.c_str(); }

int kvssd_b200_gds_open(const char* path, kvssd_b200_gds_file** file) {
  g_gds_error.clear();
  if (!path || !file) return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "NULL pointer");
  *file = nullptr;
  const CuFileApi& api = cufile();
  if (!api.error.empty()) return fail(KVSSD_B200_ERR_UNSUPPORTED, api.error);
  const int fd = ::open(path, O_RDONLY | O_DIRECT);
  if (fd < 0) return fail(KVSSD_B200_ERR_UNSUPPORTED,
                          std::string("O_DIRECT open failed: ") + strerror(errno));
  auto* f = new kvssd_b200_gds_file;
  f->fd = fd;
  CUfileDescr_t descr{};
  descr.handle.fd = fd;
  descr.type = CU_FILE_HANDLE_TYPE_OPAQUE_FD;
  const CUfileError_t st = api.handle_register(&f->handle, &descr);
  if (st.err != CU_FILE_SUCCESS) {
    ::close(fd);
    delete f;
    return fail(KVSSD_B200_ERR_UNSUPPORTED, "cuFileHandleRegister failed: " + describe(st));
  }
  *file = f;
  return KVSSD_B200_OK;
}

int kvssd_b200_gds_read_records(kvssd_b200_gds_file* file, const long long* offsets,
                                int n_records, size_t record_bytes, void* device_destination,
                                int threads) {
  g_gds_error.clear();
  if (!file || !offsets || !device_destination || n_records < 0 || record_bytes == 0)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "bad arguments");
  if (n_records == 0) return KVSSD_B200_OK;
  if (record_bytes % 4096 || reinterpret_cast<uintptr_t>(device_destination) % 4096)
    return fail(KVSSD_B200_ERR_INVALID_ARGUMENT,
                "cuFile record reads need 4096-byte records and a 4096-byte aligned destination");
  for (int i = 0; i < n_records; ++i)
    if (offsets[i] < 0 || offsets[i] % 4096)
      return fail(KVSSD_B200_ERR_INVALID_ARGUMENT, "record offsets must be 4096-byte aligned");
  const CuFileApi& api = cufile();
  if (!api.error.empty()) return fail(KVSSD_B200_ERR_UNSUPPORTED, api.error);
  const int n_threads = std::max(1, std::min(threads, n_records));
  int device = 0;  // the reader threads work on the caller's device
  if (cudaGetDevice(&device) != cudaSuccess)
    return fail(KVSSD_B200_ERR_CUDA, "cudaGetDevice failed");
  std::atomic<int> next{0};
  std::atomic<bool> failed{false};
  std::mutex err_mu;
  std::string first_error;
  auto worker = [&] {
    std::string err;
    cudaSetDevice(device);
    for (int i = next++; i < n_records && !failed.load(); i = next++) {
      if (!read_record(api, file, device_destination, record_bytes, offsets[i],
                       static_cast<long long>(i) * static_cast<long long>(record_bytes), &err)) {
        failed = true;
        std::lock_guard<std::mutex> lock(err_mu);
        if (first_error.empty())
          first_error = "record " + std::to_string(i) + " at offset " +
                        std::to_string(offsets[i]) + ": " + err;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < n_threads; ++t) pool.emplace_back(worker);
  worker();
  for (auto& t : pool) t.join();
  if (failed) return fail(KVSSD_B200_ERR_CUDA, first_error);
  return KVSSD_B200_OK;
}

int kvssd_b200_gds_close(kvssd_b200_gds_file* file) {
  if (!file) return KVSSD_B200_OK;
  const CuFileApi& api = cufile();
  if (api.handle_deregister) api.handle_deregister(file->handle);
  if (file->fd >= 0) ::close(file->fd);
  delete file;
  return KVSSD_B200_OK;
}

}  // extern "C"
