// Native record reader: a batch of kvssd records (4 KiB-aligned offsets and lengths in one store
// file) read into a host buffer by a pool of threads, with O_DIRECT when the file system allows
// it (page-cache bypass, as kvssd's "direct" storage backend, src/kvssd/storage/direct.py:14-21,
// 64-88) and buffered pread otherwise ("buffered", src/kvssd/storage/buffered.py:53-76): where
// the O_DIRECT open fails, or an O_DIRECT read fails with EINVAL, the batch is read buffered.
// Host code only; no CUDA calls.
#include <errno.h>
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <string>
#include <thread>
#include <vector>

#include "../../include/kvssd_b200.h"

namespace {

thread_local std::string g_io_error;

// Reads exactly `len` bytes at `off` (short reads are retried; EOF before `len` is an error).
// On failure *err_no holds the pread errno (0 for a short read).
bool read_full(int fd, uint8_t* dst, size_t len, long long off, std::string* err, int* err_no) {
  size_t done = 0;
  while (done < len) {
    const ssize_t got = pread(fd, dst + done, len - done, static_cast<off_t>(off + done));
    if (got < 0) {
      if (errno == EINTR) continue;
      *err_no = errno;
      *err = std::string("pread: ") + strerror(errno);
      return false;
    }
    if (got == 0) {
      *err_no = 0;
      *err = "short read: end of file before the record ends";
      return false;
    }
    done += static_cast<size_t>(got);
  }
  return true;
}

}  // namespace

extern "C" {

const char* kvssd_b200_io_last_error(void) { return g_io_error.c_str(); }

int kvssd_b200_read_records(const char* path, const long long* offsets, int n_records,
                            size_t record_bytes, void* destination, int threads, int direct,
                            int* used_direct) {
  g_io_error.clear();
  if (!path || !offsets || !destination || n_records < 0 || record_bytes == 0) {
    g_io_error = "bad arguments";
    return KVSSD_B200_ERR_INVALID_ARGUMENT;
  }
  if (used_direct) *used_direct = 0;
  if (n_records == 0) return KVSSD_B200_OK;
  bool use_direct = direct != 0 && record_bytes % 4096 == 0 &&
                    reinterpret_cast<uintptr_t>(destination) % 4096 == 0;
  for (int i = 0; use_direct && i < n_records; ++i)
    if (offsets[i] % 4096) use_direct = false;
  int fd = -1;
#ifdef O_DIRECT
  if (use_direct) fd = open(path, O_RDONLY | O_DIRECT);
#endif
  if (fd < 0) {  // no O_DIRECT here (e.g. tmpfs): buffered reads
    use_direct = false;
    fd = open(path, O_RDONLY);
  }
  if (fd < 0) {
    g_io_error = std::string("open ") + path + ": " + strerror(errno);
    return KVSSD_B200_ERR_INVALID_ARGUMENT;
  }
  const int workers = std::max(1, std::min(threads, n_records));
  std::atomic<bool> failed{false};
  std::atomic<bool> refused{false};  // an O_DIRECT read failed with EINVAL
  std::vector<std::string> errors(workers);
  auto batch = [&] {
    std::atomic<int> next{0};
    auto work = [&](int w) {
      int err_no = 0;
      for (int i = next.fetch_add(1); i < n_records && !failed.load(); i = next.fetch_add(1)) {
        uint8_t* dst = static_cast<uint8_t*>(destination) + static_cast<size_t>(i) * record_bytes;
        if (!read_full(fd, dst, record_bytes, offsets[i], &errors[w], &err_no)) {
          if (err_no == EINVAL) refused.store(true);
          failed.store(true);
        }
      }
    };
    std::vector<std::thread> pool;
    for (int w = 1; w < workers; ++w) pool.emplace_back(work, w);
    work(0);
    for (auto& t : pool) t.join();
  };
  batch();
  if (use_direct && refused.load()) {
    // The file system took the O_DIRECT open but refuses its reads: the batch again, buffered.
    close(fd);
    fd = open(path, O_RDONLY);
    if (fd < 0) {
      g_io_error = std::string("open ") + path + ": " + strerror(errno);
      return KVSSD_B200_ERR_INVALID_ARGUMENT;
    }
    use_direct = false;
    failed.store(false);
    for (auto& e : errors) e.clear();
    batch();
  }
  close(fd);
  if (failed.load()) {
    for (const auto& e : errors)
      if (!e.empty()) g_io_error = e;
    return KVSSD_B200_ERR_INVALID_ARGUMENT;
  }
  if (used_direct) *used_direct = use_direct ? 1 : 0;
  return KVSSD_B200_OK;
}

}  // extern "C"
