// Host-side reader for flat token files: fetch many fixed-length chunks, from many files, into one int64 batch.
//
// A training batch is a few thousand positional reads of a few KiB each, scattered over hundreds of files.  Doing them
// one Python call at a time costs more in interpreter and allocation overhead than in I/O, so the batch is read here:
// the caller passes (file, chunk) pairs and a destination matrix (ideally pinned), the reads are split over a few
// threads, every chunk is fetched with one pread and widened from its storage type (1, 2, 4 or 8 bytes, unsigned) to
// int64 in place.  File descriptors are opened once per store and shared by the threads (pread carries its own offset).
// There is no counterpart in the reference, whose dataset reads one chunk per __getitem__ through numpy.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

struct Store {
  std::vector<std::string> paths;
  std::unique_ptr<std::atomic<int>[]> fds;  // -1 until first use
  std::mutex open_mutex;
};

int fd_of(Store* s, int file) {
  int fd = s->fds[file].load(std::memory_order_acquire);
  if (fd >= 0) return fd;
  std::lock_guard<std::mutex> guard(s->open_mutex);
  fd = s->fds[file].load(std::memory_order_relaxed);
  if (fd < 0) {
    fd = ::open(s->paths[file].c_str(), O_RDONLY | O_CLOEXEC);
    s->fds[file].store(fd, std::memory_order_release);
  }
  return fd;
}

// Reads exactly n bytes at `offset`; false on error or a short file.
bool pread_all(int fd, uint8_t* dst, size_t n, int64_t offset) {
  size_t got = 0;
  while (got < n) {
    const ssize_t r = ::pread(fd, dst + got, n - got, offset + static_cast<int64_t>(got));
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    if (r == 0) return false;
    got += static_cast<size_t>(r);
  }
  return true;
}

// The raw chunk sits in the tail of its own int64 row; widening front to back never overwrites unread input.
template <typename T>
void widen_in_place(int64_t* row, int64_t tokens) {
  const T* src = reinterpret_cast<const T*>(reinterpret_cast<uint8_t*>(row) + tokens * (8 - static_cast<int64_t>(sizeof(T))));
  for (int64_t i = 0; i < tokens; ++i) row[i] = static_cast<int64_t>(src[i]);
}

}  // namespace

extern "C" {

// Error codes (negative): -1 bad argument, -2 cannot open a file, -3 read failed or file too short.
void* ob_token_store_open(const char* const* paths, int n_paths) {
  if (paths == nullptr || n_paths <= 0) return nullptr;
  Store* s = new Store();
  s->paths.reserve(n_paths);
  for (int i = 0; i < n_paths; ++i) s->paths.emplace_back(paths[i]);
  s->fds.reset(new std::atomic<int>[n_paths]);
  for (int i = 0; i < n_paths; ++i) s->fds[i].store(-1);
  return s;
}

void ob_token_store_close(void* handle) {
  Store* s = static_cast<Store*>(handle);
  if (s == nullptr) return;
  for (size_t i = 0; i < s->paths.size(); ++i) {
    const int fd = s->fds[i].load();
    if (fd >= 0) ::close(fd);
  }
  delete s;
}

// out[i, :] = tokens [chunk[i] * chunk_tokens, (chunk[i] + 1) * chunk_tokens) of file[i], widened to int64.
// `failed_at` (optional) receives the index of the first request that failed.
int ob_token_store_read(void* handle, const int32_t* file, const int64_t* chunk, int64_t n, int64_t chunk_tokens, int itemsize,
                        int64_t* out, int threads, int64_t* failed_at) {
  Store* s = static_cast<Store*>(handle);
  if (s == nullptr || n < 0 || chunk_tokens <= 0 || (n > 0 && (out == nullptr || file == nullptr || chunk == nullptr))) return -1;
  if (itemsize != 1 && itemsize != 2 && itemsize != 4 && itemsize != 8) return -1;
  for (int64_t i = 0; i < n; ++i)
    if (file[i] < 0 || file[i] >= static_cast<int32_t>(s->paths.size()) || chunk[i] < 0) return -1;
  const size_t chunk_bytes = static_cast<size_t>(chunk_tokens) * static_cast<size_t>(itemsize);
  std::atomic<int> status{0};
  std::atomic<int64_t> first_bad{-1};
  std::atomic<int64_t> next{0};
  auto work = [&]() {
    for (;;) {
      const int64_t i = next.fetch_add(1);
      if (i >= n || status.load() != 0) return;
      const int fd = fd_of(s, file[i]);
      int rc = 0;
      if (fd < 0) {
        rc = -2;
      } else {
        int64_t* row = out + i * chunk_tokens;
        uint8_t* raw = reinterpret_cast<uint8_t*>(row) + static_cast<size_t>(chunk_tokens) * static_cast<size_t>(8 - itemsize);
        if (!pread_all(fd, raw, chunk_bytes, chunk[i] * static_cast<int64_t>(chunk_bytes))) {
          rc = -3;
        } else {
          switch (itemsize) {
            case 1: widen_in_place<uint8_t>(row, chunk_tokens); break;
            case 2: widen_in_place<uint16_t>(row, chunk_tokens); break;
            case 4: widen_in_place<uint32_t>(row, chunk_tokens); break;
            default: break;  // 8-byte tokens are already in place
          }
        }
      }
      if (rc != 0) {
        int expected = 0;
        if (status.compare_exchange_strong(expected, rc)) first_bad.store(i);
        return;
      }
    }
  };
  const int n_threads = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(threads, n)));
  if (n_threads <= 1) {
    work();
  } else {
    std::vector<std::thread> pool;
    pool.reserve(n_threads - 1);
    for (int t = 1; t < n_threads; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
  }
  if (failed_at != nullptr) *failed_at = first_bad.load();
  return status.load();
}

}  // extern "C"
