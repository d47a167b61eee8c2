// Pack-file reads for the FP8 pack loader (pocketlm_b200/fp8_pack.py).
//
// moe_read_tensor_bytes replaces the reference's native_read_tensor_bytes
// (src/pcketlm/native/fp16_loader.cpp:33-67: a Windows ReadFile loop over one
// byte range, codes 1 = null argument, 2 = open failure, 4 = short read) with
// POSIX pread; moe_read_spans reads several ranges of one file (an expert's
// six tensors, or the span that holds them) in one call, split into pieces of
// at least 8 MiB over a few threads so a page-cache-resident pack reads at
// memory bandwidth rather than one core's copy rate.  Host code only.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

constexpr uint64_t kPieceBytes = 8ull << 20;
constexpr uint64_t kMaxPread = 1ull << 30;
constexpr int kMaxThreads = 16;

// codes shared with the reference's reader, plus 3 for a range past the file's end
constexpr int kReadOk = 0, kReadNull = 1, kReadOpen = 2, kReadRange = 3, kReadShort = 4;

int read_range(int fd, uint64_t offset, uint64_t n, uint8_t* out) {
  while (n > 0) {
    const ssize_t got = pread(fd, out, static_cast<size_t>(std::min(n, kMaxPread)), static_cast<off_t>(offset));
    if (got < 0) {
      if (errno == EINTR) continue;
      return kReadShort;
    }
    if (got == 0) return kReadShort;
    out += got;
    offset += static_cast<uint64_t>(got);
    n -= static_cast<uint64_t>(got);
  }
  return kReadOk;
}

struct Piece {
  uint64_t offset, bytes;
  uint8_t* out;
};

}  // namespace

extern "C" {

int moe_read_spans(const char* path, int64_t n, const uint64_t* offsets, const uint64_t* lengths,
                   uint8_t* const* outs, int64_t threads) {
  if (!path || n < 0 || (n > 0 && (!offsets || !lengths || !outs))) return kReadNull;
  for (int64_t i = 0; i < n; ++i)
    if (lengths[i] > 0 && !outs[i]) return kReadNull;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return kReadOpen;
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    return kReadOpen;
  }
  const uint64_t size = static_cast<uint64_t>(st.st_size);
  std::vector<Piece> pieces;
  for (int64_t i = 0; i < n; ++i) {
    if (offsets[i] > size || lengths[i] > size - offsets[i]) {
      close(fd);
      return kReadRange;
    }
    for (uint64_t done = 0; done < lengths[i]; done += kPieceBytes)
      pieces.push_back({offsets[i] + done, std::min(kPieceBytes, lengths[i] - done), outs[i] + done});
  }
  const int64_t want = threads > 0 ? threads : std::min<int64_t>(8, std::max(1u, std::thread::hardware_concurrency()));
  const int workers = static_cast<int>(std::min<int64_t>({want, static_cast<int64_t>(pieces.size()), kMaxThreads}));
  std::atomic<size_t> next{0};
  std::atomic<int> code{kReadOk};
  auto work = [&]() {
    for (size_t i = next++; i < pieces.size() && code.load() == kReadOk; i = next++) {
      const int c = read_range(fd, pieces[i].offset, pieces[i].bytes, pieces[i].out);
      if (c != kReadOk) code.store(c);
    }
  };
  if (workers <= 1) {
    work();
  } else {
    std::vector<std::thread> pool;
    pool.reserve(static_cast<size_t>(workers - 1));
    for (int w = 1; w < workers; ++w) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
  }
  close(fd);
  return code.load();
}

int moe_read_tensor_bytes(const char* path, uint64_t absolute_offset, uint64_t nbytes, uint8_t* out) {
  if (!path || !out) return kReadNull;
  return moe_read_spans(path, 1, &absolute_offset, &nbytes, &out, 0);
}

}  // extern "C"
