// Native token loader: memory-maps a flat token file (uint16 or uint32 ids) and assembles training
// batches of random windows on worker threads into a bounded ring of host buffers, so the next
// batch is ready (and the copy into pinned memory is one memcpy) when the training step asks for it.
//
// Reference behaviour it replaces: crates/brain-data (MmapChunkReader mmap.rs:6-30, prefetch and
// backpressure backpressure.rs:7, PipelineMetrics metrics.rs:9-20, PipelineCheckpoint
// checkpoint.rs:7-20 for resuming at a batch index) and the DistributedSampler's disjoint per-rank
// streams (samplers.rs:37).
//
// Determinism: batch b of rank r draws its B window starts from a SplitMix64 stream (Steele, Lea and
// Flood 2014) seeded with seed * 0x9E3779B97F4A7C15 + (b * world + r); start = draw % (n_tokens - S).
// The result depends only on (seed, b, rank, world), not on the number of workers or their timing, so
// a run resumed at batch b sees the same data. Each window holds S + 1 tokens (inputs and the shifted
// targets), written as int64 or int32 ids.
//
// Every wait is bounded (timeout_ms); a wait that expires returns BRAIN_LOADER_TIMEOUT instead of
// blocking forever.
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define BRAIN_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int BRAIN_LOADER_OK = 0;
constexpr int BRAIN_LOADER_BAD_ARG = -10;
constexpr int BRAIN_LOADER_IO = -11;
constexpr int BRAIN_LOADER_TIMEOUT = -12;
constexpr int BRAIN_LOADER_CLOSED = -13;

inline uint64_t splitmix_next(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

struct Slot {
  std::vector<uint8_t> data;
  int64_t batch = -1;  // batch index held, -1 when free
  bool ready = false;
};

struct Loader {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t map_bytes = 0;
  int token_bytes = 2, out_bytes = 8;
  int64_t n_tokens = 0, B = 0, S = 0;
  uint64_t seed = 0;
  int rank = 0, world = 1;
  int64_t timeout_ms = 60000;
  std::vector<Slot> ring;
  std::mutex mu;
  std::condition_variable cv_ready, cv_free;
  std::atomic<int64_t> next_claim{0};
  int64_t next_consume = 0;
  bool closing = false;
  std::vector<std::thread> workers;
  // statistics
  std::atomic<int64_t> produced{0}, consumed{0}, consumer_wait_ns{0}, producer_wait_ns{0};

  size_t batch_bytes() const { return (size_t)B * (size_t)(S + 1) * (size_t)out_bytes; }

  void fill(int64_t b, uint8_t* dst) const {
    uint64_t st = seed * 0x9E3779B97F4A7C15ull + (uint64_t)(b * world + rank);
    const uint64_t span = (uint64_t)(n_tokens - S);
    for (int64_t i = 0; i < B; ++i) {
      const uint64_t start = splitmix_next(st) % span;
      for (int64_t t = 0; t <= S; ++t) {
        const uint64_t idx = start + (uint64_t)t;
        const uint64_t v = token_bytes == 2 ? (uint64_t)reinterpret_cast<const uint16_t*>(map)[idx]
                                            : (uint64_t)reinterpret_cast<const uint32_t*>(map)[idx];
        const size_t o = (size_t)(i * (S + 1) + t);
        if (out_bytes == 8) {
          reinterpret_cast<int64_t*>(dst)[o] = (int64_t)v;
        } else {
          reinterpret_cast<int32_t*>(dst)[o] = (int32_t)v;
        }
      }
    }
  }

  void worker() {
    const int64_t depth = (int64_t)ring.size();
    for (;;) {
      const int64_t b = next_claim.fetch_add(1);
      Slot& s = ring[(size_t)(b % depth)];
      {
        // the slot is free once the consumer has taken batch b - depth
        auto t0 = std::chrono::steady_clock::now();
        std::unique_lock<std::mutex> lk(mu);
        cv_free.wait(lk, [&] { return closing || (s.batch == -1 && next_consume > b - depth); });
        producer_wait_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
        if (closing) return;
        s.batch = b;
        s.ready = false;
      }
      fill(b, s.data.data());
      {
        std::lock_guard<std::mutex> lk(mu);
        s.ready = true;
      }
      ++produced;
      cv_ready.notify_all();
    }
  }
};

}  // namespace

// Opens the token file and starts `workers` threads filling a ring of `depth` batches, beginning at
// batch `start_batch`. out_bytes selects int64 (8) or int32 (4) ids in the output.
BRAIN_API int brain_loader_open(const char* path, int token_bytes, int out_bytes, int64_t batch, int64_t seq,
                                int64_t seed, int rank, int world, int workers, int depth, int64_t start_batch,
                                int64_t timeout_ms, void** handle_out) {
  if (!path || !handle_out || (token_bytes != 2 && token_bytes != 4) || (out_bytes != 4 && out_bytes != 8) ||
      batch <= 0 || seq <= 0 || workers <= 0 || workers > 64 || depth <= 0 || depth > 1024 || world <= 0 ||
      rank < 0 || rank >= world || start_batch < 0 || timeout_ms <= 0)
    return BRAIN_LOADER_BAD_ARG;
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) return BRAIN_LOADER_IO;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < (off_t)token_bytes) {
    ::close(fd);
    return BRAIN_LOADER_IO;
  }
  const int64_t n_tokens = (int64_t)st.st_size / token_bytes;
  if (n_tokens <= seq) {
    ::close(fd);
    return BRAIN_LOADER_BAD_ARG;
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
  if (m == MAP_FAILED) {
    ::close(fd);
    return BRAIN_LOADER_IO;
  }
  madvise(m, (size_t)st.st_size, MADV_RANDOM);
  auto* L = new Loader();
  L->fd = fd;
  L->map = static_cast<const uint8_t*>(m);
  L->map_bytes = (size_t)st.st_size;
  L->token_bytes = token_bytes;
  L->out_bytes = out_bytes;
  L->n_tokens = n_tokens;
  L->B = batch;
  L->S = seq;
  L->seed = (uint64_t)seed;
  L->rank = rank;
  L->world = world;
  L->timeout_ms = timeout_ms;
  L->ring.resize((size_t)depth);
  for (auto& s : L->ring) s.data.resize(L->batch_bytes());
  L->next_claim = start_batch;
  L->next_consume = start_batch;
  for (int i = 0; i < workers; ++i) L->workers.emplace_back([L] { L->worker(); });
  *handle_out = L;
  return BRAIN_LOADER_OK;
}

// Copies the next batch ([batch, seq + 1] ids) into dst (typically pinned host memory) and writes its
// index to *batch_index. Waits at most timeout_ms for the workers.
BRAIN_API int brain_loader_next(void* handle, void* dst, int64_t* batch_index) {
  auto* L = static_cast<Loader*>(handle);
  if (!L || !dst) return BRAIN_LOADER_BAD_ARG;
  const int64_t depth = (int64_t)L->ring.size();
  std::unique_lock<std::mutex> lk(L->mu);
  const int64_t b = L->next_consume;
  Slot& s = L->ring[(size_t)(b % depth)];
  auto t0 = std::chrono::steady_clock::now();
  const bool ok = L->cv_ready.wait_for(lk, std::chrono::milliseconds(L->timeout_ms),
                                       [&] { return L->closing || (s.batch == b && s.ready); });
  L->consumer_wait_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  if (L->closing) return BRAIN_LOADER_CLOSED;
  if (!ok) return BRAIN_LOADER_TIMEOUT;
  std::memcpy(dst, s.data.data(), L->batch_bytes());
  s.batch = -1;
  s.ready = false;
  L->next_consume = b + 1;
  if (batch_index) *batch_index = b;
  ++L->consumed;
  lk.unlock();
  L->cv_free.notify_all();
  return BRAIN_LOADER_OK;
}

// Fills dst with batch b directly on the calling thread (no ring): the oracle for tests and a way to
// fetch one arbitrary batch.
BRAIN_API int brain_loader_fill(void* handle, int64_t b, void* dst) {
  auto* L = static_cast<Loader*>(handle);
  if (!L || !dst || b < 0) return BRAIN_LOADER_BAD_ARG;
  L->fill(b, static_cast<uint8_t*>(dst));
  return BRAIN_LOADER_OK;
}

// stats[0..4] = batches produced, batches consumed, consumer wait ns, producer wait ns, tokens in file
BRAIN_API int brain_loader_stats(void* handle, int64_t* stats) {
  auto* L = static_cast<Loader*>(handle);
  if (!L || !stats) return BRAIN_LOADER_BAD_ARG;
  stats[0] = L->produced.load();
  stats[1] = L->consumed.load();
  stats[2] = L->consumer_wait_ns.load();
  stats[3] = L->producer_wait_ns.load();
  stats[4] = L->n_tokens;
  return BRAIN_LOADER_OK;
}

BRAIN_API int brain_loader_close(void* handle) {
  auto* L = static_cast<Loader*>(handle);
  if (!L) return BRAIN_LOADER_BAD_ARG;
  {
    std::lock_guard<std::mutex> lk(L->mu);
    L->closing = true;
  }
  L->cv_free.notify_all();
  L->cv_ready.notify_all();
  for (auto& t : L->workers) t.join();
  munmap(const_cast<uint8_t*>(L->map), L->map_bytes);
  ::close(L->fd);
  delete L;
  return BRAIN_LOADER_OK;
}
