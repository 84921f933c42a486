// Host-side data path: bulk document packing, MinHash signatures and a background
// token-shard loader that fills (pinned) batch buffers ahead of the training step.
//
// Packing has the reference's concat-and-chunk contract (EOS after each document,
// per-document segment ids; saint_llm_data/packing.py:23-137).  MinHash uses one 64-bit
// hash per shingle and n_perm universal hash permutations h_i(x) = a_i x + b_i (mod 2^61-1),
// Broder's construction, instead of one SHA1 per (permutation, shingle).
#include <torch/extension.h>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace sv4 {

// ---------------------------------------------------------------- packing
std::vector<torch::Tensor> pack_documents(torch::Tensor tokens, torch::Tensor offsets, int64_t seq_len,
                                          int64_t eos, int64_t pad, bool drop_last) {
  TORCH_CHECK(seq_len > 0, "seq_len must be positive");
  TORCH_CHECK(tokens.dtype() == torch::kInt64 && offsets.dtype() == torch::kInt64, "int64 inputs expected");
  const int64_t* tk = tokens.data_ptr<int64_t>();
  const int64_t* of = offsets.data_ptr<int64_t>();
  const int64_t n_docs = offsets.numel() - 1;
  int64_t total = 0;
  for (int64_t d = 0; d < n_docs; ++d) {
    const int64_t len = of[d + 1] - of[d];
    TORCH_CHECK(len >= 0 && of[d + 1] <= tokens.numel(), "bad document offsets");
    if (len > 0) total += len + 1;
  }
  int64_t rows = total / seq_len;
  const bool tail = !drop_last && total % seq_len != 0;
  if (tail) ++rows;
  auto out_t = torch::empty({rows, seq_len}, torch::kInt64);
  auto out_s = torch::empty({rows, seq_len}, torch::kInt64);
  int64_t* ot = out_t.data_ptr<int64_t>();
  int64_t* os = out_s.data_ptr<int64_t>();
  const int64_t cap = rows * seq_len;
  int64_t w = 0, seg = 0;
  for (int64_t d = 0; d < n_docs && w < cap; ++d) {
    const int64_t len = of[d + 1] - of[d];
    if (len == 0) continue;
    const int64_t n = std::min<int64_t>(len, cap - w);
    std::memcpy(ot + w, tk + of[d], n * sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) os[w + i] = seg;
    w += n;
    if (w < cap) { ot[w] = eos; os[w] = seg; ++w; }
    ++seg;
  }
  const int64_t last_seg = w > 0 ? os[w - 1] : 0;
  for (; w < cap; ++w) { ot[w] = pad; os[w] = last_seg; }
  return {out_t, out_s};
}

// ---------------------------------------------------------------- MinHash
static inline uint64_t mix64(uint64_t x) {  // splitmix64 finaliser
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

static inline uint64_t mod_mersenne61(__uint128_t v) {
  const uint64_t p = (1ULL << 61) - 1;
  uint64_t r = (uint64_t)(v & p) + (uint64_t)(v >> 61);
  r = (r & p) + (r >> 61);
  return r >= p ? r - p : r;
}

// Signatures of UTF-32 code point sequences packed as (flat, offsets); shingles are
// `shingle` consecutive code points.  Returns (n_docs, n_perm) int64.
torch::Tensor minhash_signatures(torch::Tensor codepoints, torch::Tensor offsets, int64_t n_perm, int64_t shingle,
                                 int64_t seed) {
  TORCH_CHECK(codepoints.dtype() == torch::kInt32 && offsets.dtype() == torch::kInt64, "int32 code points, int64 offsets");
  const int32_t* cp = codepoints.data_ptr<int32_t>();
  const int64_t* of = offsets.data_ptr<int64_t>();
  const int64_t n_docs = offsets.numel() - 1;
  const uint64_t p = (1ULL << 61) - 1;
  std::vector<uint64_t> a(n_perm), b(n_perm);
  for (int64_t i = 0; i < n_perm; ++i) {
    a[i] = mix64((uint64_t)seed * 0x100000001b3ULL + 2 * i) % (p - 1) + 1;
    b[i] = mix64((uint64_t)seed * 0x100000001b3ULL + 2 * i + 1) % p;
  }
  auto out = torch::empty({n_docs, n_perm}, torch::kInt64);
  int64_t* o = out.data_ptr<int64_t>();
  at::parallel_for(0, n_docs, 16, [&](int64_t lo, int64_t hi) {
    std::vector<uint64_t> hashes;
    for (int64_t d = lo; d < hi; ++d) {
      const int64_t len = of[d + 1] - of[d];
      const int32_t* s = cp + of[d];
      hashes.clear();
      if (len > 0) {
        const int64_t n_sh = len < shingle ? 1 : len - shingle + 1;
        const int64_t w = len < shingle ? len : shingle;
        for (int64_t i = 0; i < n_sh; ++i) {
          uint64_t h = 0x243f6a8885a308d3ULL;
          for (int64_t j = 0; j < w; ++j) h = mix64(h ^ (uint32_t)s[i + j]);
          hashes.push_back(h % p);
        }
      }
      for (int64_t k = 0; k < n_perm; ++k) {
        uint64_t m = hashes.empty() ? 0 : UINT64_MAX;
        for (uint64_t h : hashes) {
          const uint64_t v = mod_mersenne61((__uint128_t)a[k] * h + b[k]);
          m = v < m ? v : m;
        }
        o[d * n_perm + k] = (int64_t)m;
      }
    }
  });
  return out;
}

// ---------------------------------------------------------------- token shards
// Shard file: 32-byte header {char magic[8] = "SV4TOKS\0"; uint32 version = 1;
// uint32 bytes_per_token (2|4); uint64 n_tokens; uint64 reserved} then the tokens.
struct Shard {
  int fd = -1;
  void* map = nullptr;
  size_t map_len = 0;
  const uint8_t* data = nullptr;
  uint32_t width = 0;
  uint64_t n = 0;
};

class TokenShardLoader {
 public:
  TokenShardLoader(std::vector<std::string> paths, int64_t batch, int64_t seq_len, int64_t seed, int64_t rank,
                   int64_t world, int64_t depth, bool pin)
      : batch_(batch), seq_(seq_len), seed_(seed), rank_(rank), world_(world), depth_(depth) {
    TORCH_CHECK(!paths.empty(), "no token shards given");
    TORCH_CHECK(batch > 0 && seq_len > 0 && depth > 0 && world > 0 && rank >= 0 && rank < world, "bad loader sizes");
    for (auto& p : paths) open_shard(p);
    for (auto& s : shards_) {
      TORCH_CHECK(s.n > (uint64_t)seq_len, "shard shorter than one window");
      cum_.push_back(total_windows_ += s.n - seq_len);
    }
    auto opts = torch::TensorOptions().dtype(torch::kInt64).pinned_memory(pin);
    for (int64_t i = 0; i < depth; ++i) slots_.push_back(torch::empty({batch, seq_len}, opts));
    for (int64_t i = 0; i < depth; ++i) free_.push_back(i);
    worker_ = std::thread([this] { run(); });
  }

  ~TokenShardLoader() { close(); }

  void close() {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (stop_) return;
      stop_ = true;
    }
    cv_.notify_all();
    if (worker_.joinable()) worker_.join();
    for (auto& s : shards_)
      if (s.map) { munmap(s.map, s.map_len); ::close(s.fd); s.map = nullptr; }
  }

  // Blocks until the next batch is ready; returns (slot id, tensor).  The slot stays
  // owned by the caller until release(slot).
  std::tuple<int64_t, torch::Tensor> next() {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [this] { return !ready_.empty() || stop_ || !error_.empty(); });
    if (!error_.empty()) throw std::runtime_error(error_);
    TORCH_CHECK(!stop_, "loader closed");
    const int64_t s = ready_.front();
    ready_.pop_front();
    return {s, slots_[s]};
  }

  void release(int64_t slot) {
    {
      std::lock_guard<std::mutex> g(mu_);
      free_.push_back(slot);
    }
    cv_.notify_all();
  }

  int64_t total_windows() const { return (int64_t)total_windows_; }
  int64_t step() const { return step_.load(); }

  // Deterministic window start (global position) of row `row` at step `step`.
  int64_t window_start(int64_t step, int64_t row) const {
    const uint64_t key = mix64(mix64((uint64_t)seed_ + 0x9e3779b97f4a7c15ULL * (uint64_t)step) ^
                               (uint64_t)(rank_ * batch_ + row));
    return (int64_t)(key % total_windows_);
  }

 private:
  void open_shard(const std::string& path) {
    Shard s;
    s.fd = ::open(path.c_str(), O_RDONLY);
    TORCH_CHECK(s.fd >= 0, "cannot open token shard ", path);
    struct stat st;
    fstat(s.fd, &st);
    TORCH_CHECK(st.st_size >= 32, "token shard too small: ", path);
    s.map_len = (size_t)st.st_size;
    s.map = mmap(nullptr, s.map_len, PROT_READ, MAP_SHARED, s.fd, 0);
    TORCH_CHECK(s.map != MAP_FAILED, "mmap failed for ", path);
    const uint8_t* h = (const uint8_t*)s.map;
    TORCH_CHECK(std::memcmp(h, "SV4TOKS", 7) == 0, "not a token shard: ", path);
    uint32_t ver, width;
    std::memcpy(&ver, h + 8, 4);
    std::memcpy(&width, h + 12, 4);
    std::memcpy(&s.n, h + 16, 8);
    TORCH_CHECK(ver == 1 && (width == 2 || width == 4), "unsupported shard header in ", path);
    TORCH_CHECK(32 + s.n * width <= s.map_len, "truncated token shard ", path);
    madvise(s.map, s.map_len, MADV_RANDOM);
    s.width = width;
    s.data = h + 32;
    shards_.push_back(s);
  }

  void fill(int64_t slot, int64_t step) {
    int64_t* out = slots_[slot].data_ptr<int64_t>();
    for (int64_t r = 0; r < batch_; ++r) {
      uint64_t g = (uint64_t)window_start(step, r);
      size_t k = 0;
      while (g >= cum_[k]) ++k;
      const uint64_t base = k == 0 ? g : g - cum_[k - 1];
      const Shard& s = shards_[k];
      int64_t* o = out + r * seq_;
      if (s.width == 2) {
        const uint16_t* src = (const uint16_t*)s.data + base;
        for (int64_t i = 0; i < seq_; ++i) o[i] = src[i];
      } else {
        const uint32_t* src = (const uint32_t*)s.data + base;
        for (int64_t i = 0; i < seq_; ++i) o[i] = src[i];
      }
    }
  }

  void run() {
    int64_t step = 0;
    for (;;) {
      int64_t slot;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [this] { return !free_.empty() || stop_; });
        if (stop_) return;
        slot = free_.front();
        free_.pop_front();
      }
      try {
        fill(slot, step);
      } catch (const std::exception& e) {
        std::lock_guard<std::mutex> g(mu_);
        error_ = e.what();
        cv_.notify_all();
        return;
      }
      {
        std::lock_guard<std::mutex> g(mu_);
        ready_.push_back(slot);
      }
      step_.store(++step);
      cv_.notify_all();
    }
  }

  int64_t batch_, seq_, seed_, rank_, world_, depth_;
  std::vector<Shard> shards_;
  std::vector<uint64_t> cum_;
  uint64_t total_windows_ = 0;
  std::vector<torch::Tensor> slots_;
  std::deque<int64_t> free_, ready_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::thread worker_;
  bool stop_ = false;
  std::string error_;
  std::atomic<int64_t> step_{0};
};

void bind_data(pybind11::module_& m) {
  m.def("pack_documents", &pack_documents, "concat-and-chunk packing of a flat corpus");
  m.def("minhash_signatures", &minhash_signatures, "MinHash signatures over code-point shingles");
  pybind11::class_<TokenShardLoader>(m, "TokenShardLoader")
      .def(pybind11::init<std::vector<std::string>, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, bool>())
      .def("next", &TokenShardLoader::next, pybind11::call_guard<pybind11::gil_scoped_release>())
      .def("release", &TokenShardLoader::release)
      .def("close", &TokenShardLoader::close, pybind11::call_guard<pybind11::gil_scoped_release>())
      .def("window_start", &TokenShardLoader::window_start)
      .def_property_readonly("total_windows", &TokenShardLoader::total_windows)
      .def_property_readonly("step", &TokenShardLoader::step);
}

}  // namespace sv4
