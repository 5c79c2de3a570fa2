// Host-side I/O of the weight stores, in native threads:
//   cb_host_copy         multi-threaded memcpy (pageable arena -> pinned
//                        staging slot, weight_store.py:252-261 of the
//                        reference copies with one thread)
//   cb_read_file_ranges  parallel pread of byte ranges of one file straight
//                        into host memory (safetensors tensor data -> the
//                        packed arena, weight_store.py:109-171 of the
//                        reference reads each tensor through torch)
//   cb_host_gather_rows  embedding rows of a host table gathered into a
//                        pinned staging buffer (vocab.py:100-131)
// No CUDA calls: these run on any host thread, including the stager.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <thread>
#include <vector>

#include "cascade_b200.h"
#include "internal.h"

using namespace cb;

namespace {

constexpr int64_t kCopyChunk = int64_t(8) << 20;   // bytes per memcpy task
constexpr int64_t kReadChunk = int64_t(64) << 20;  // bytes per pread task

int clamp_threads(int threads, int64_t tasks) {
  int hw = int(std::thread::hardware_concurrency());
  if (hw < 1) hw = 1;
  if (threads < 1) threads = std::min(hw, 16);
  return int(std::max<int64_t>(1, std::min<int64_t>(threads, tasks)));
}

}  // namespace

namespace cb {

int host_copy_parallel(void* dst, const void* src, int64_t bytes, int threads) {
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fail(kErrInvalid, "cb_host_copy: bad arguments");
  if (bytes == 0) return kOk;
  const int64_t tasks = (bytes + kCopyChunk - 1) / kCopyChunk;
  const int n = clamp_threads(threads, tasks);
  if (n == 1) {
    std::memcpy(dst, src, size_t(bytes));
    return kOk;
  }
  std::atomic<int64_t> next{0};
  auto work = [&] {
    for (int64_t t = next++; t < tasks; t = next++) {
      const int64_t off = t * kCopyChunk;
      std::memcpy(static_cast<char*>(dst) + off, static_cast<const char*>(src) + off,
                  size_t(std::min(kCopyChunk, bytes - off)));
    }
  };
  std::vector<std::thread> pool;
  for (int i = 1; i < n; ++i) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
  return kOk;
}

}  // namespace cb

extern "C" int cb_host_copy(void* dst, const void* src, int64_t bytes, int threads) {
  return host_copy_parallel(dst, src, bytes, threads);
}

// Rows ids[0..n) of a row-major host table (row_bytes each) gathered into
// consecutive rows of dst; ids outside [0, rows) are rejected before any copy.
extern "C" int cb_host_gather_rows(void* dst, const void* table, int64_t rows, int64_t row_bytes,
                                   const int64_t* ids, int64_t n) {
  CB_REQUIRE(n >= 0 && row_bytes > 0 && rows > 0, "cb_host_gather_rows: bad sizes");
  CB_REQUIRE(n == 0 || (dst && table && ids), "cb_host_gather_rows: null pointer");
  for (int64_t i = 0; i < n; ++i)
    CB_REQUIRE(ids[i] >= 0 && ids[i] < rows, "cb_host_gather_rows: id %lld outside [0, %lld)", (long long)ids[i],
               (long long)rows);
  for (int64_t i = 0; i < n; ++i)
    std::memcpy(static_cast<char*>(dst) + i * row_bytes, static_cast<const char*>(table) + ids[i] * row_bytes,
                size_t(row_bytes));
  return kOk;
}

extern "C" int cb_read_file_ranges(const char* path, int n, const int64_t* offsets, void* const* dsts,
                                   const int64_t* sizes, int threads) {
  if (!path || n < 0 || (n > 0 && (!offsets || !dsts || !sizes)))
    return fail(kErrInvalid, "cb_read_file_ranges: bad arguments");
  struct Task {
    int64_t file_off, size;
    char* dst;
  };
  std::vector<Task> tasks;
  for (int i = 0; i < n; ++i) {
    if (offsets[i] < 0 || sizes[i] < 0 || (sizes[i] > 0 && !dsts[i]))
      return fail(kErrInvalid, "cb_read_file_ranges: range %d invalid", i);
    for (int64_t off = 0; off < sizes[i]; off += kReadChunk)
      tasks.push_back({offsets[i] + off, std::min(kReadChunk, sizes[i] - off), static_cast<char*>(dsts[i]) + off});
  }
  if (tasks.empty()) return kOk;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(kErrInvalid, "cb_read_file_ranges: cannot open %s: %s", path, std::strerror(errno));
  std::atomic<int64_t> next{0};
  std::atomic<int> bad{0};
  auto work = [&] {
    for (int64_t t = next++; t < int64_t(tasks.size()) && !bad.load(); t = next++) {
      const Task& k = tasks[size_t(t)];
      int64_t done = 0;
      while (done < k.size) {
        const ssize_t got = pread(fd, k.dst + done, size_t(k.size - done), off_t(k.file_off + done));
        if (got < 0 && errno == EINTR) continue;
        if (got <= 0) {
          bad = 1;
          return;
        }
        done += got;
      }
    }
  };
  const int nt = clamp_threads(threads, int64_t(tasks.size()));
  std::vector<std::thread> pool;
  for (int i = 1; i < nt; ++i) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
  close(fd);
  if (bad.load()) return fail(kErrInvalid, "cb_read_file_ranges: short read from %s", path);
  return kOk;
}
