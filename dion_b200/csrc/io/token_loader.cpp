// Token-file data loader: memory-mapped token shards, deterministic sample
// order, and a background thread that prepares the next batches while the
// GPU trains on the current one.
//
// Role in the reference: torchtitan's HuggingFace text loader (c4_test),
// which tokenizes documents, concatenates them and cuts the stream into
// non-overlapping windows of seq_len + 1 tokens (input = window[:-1],
// label = window[1:]), one split of the dataset per data-parallel rank.
// Here the documents are tokenized ahead of time into token files (see
// dion_b200/data/tokenize.py) and the loader reads windows straight out of
// the page cache:
//
//   * a token file is either this package's format (32-byte header: magic
//     "DB2TOKN1", uint32 version = 1, uint32 bytes per token (2 or 4),
//     uint64 token count, uint64 reserved; then the little-endian tokens) or
//     a raw little-endian uint16 / uint32 array (bytes per token given);
//   * the files are concatenated into one stream; window w covers tokens
//     [w * (S + 1), (w + 1) * (S + 1));
//   * global sample g (counted over the whole job) reads window
//     perm_e(g mod W) of epoch e = g div W, where perm_e is a keyed
//     bijection of [0, W) (a 4-round Feistel network on the next even bit
//     width, cycle-walked into range: Black and Rogaway, "Ciphers with
//     Arbitrary Finite Domains", CT-RSA 2002) or the identity when
//     shuffling is off. No permutation table is stored, so W can be any size;
//   * the batch at position p gives rank r the samples
//     p + r * b + i (i < b); the position then advances by world * b. The
//     position is the loader's whole state: a checkpoint stores it, and a
//     job resumed at another world size continues at the same sample;
//   * every token is checked against the vocabulary size on the host, so an
//     out-of-range id is reported with its file and offset instead of
//     reaching an embedding lookup on the GPU.
#include <torch/extension.h>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

namespace bdion_io {

constexpr char kMagic[8] = {'D', 'B', '2', 'T', 'O', 'K', 'N', '1'};
constexpr size_t kHeaderBytes = 32;
constexpr uint32_t kVersion = 1;

// splitmix64 finaliser (Steele, Lea and Flood, "Fast Splittable
// Pseudorandom Number Generators", OOPSLA 2014): a 64-bit mixing function.
inline uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Keyed bijection of [0, n).
class Permutation {
 public:
  Permutation(uint64_t n, uint64_t key) : n_(n), key_(key) {
    int bits = 2;
    while (bits < 62 && (1ull << bits) < n) bits += 2;
    half_ = bits / 2;
    mask_ = (1ull << half_) - 1;
  }
  uint64_t operator()(uint64_t i) const {
    uint64_t x = i;
    do {
      x = round_trip(x);
    } while (x >= n_);
    return x;
  }

 private:
  uint64_t round_trip(uint64_t x) const {
    uint64_t l = x >> half_, r = x & mask_;
    for (uint64_t k = 0; k < 4; ++k) {
      const uint64_t f = mix64(key_ ^ (k << 58) ^ r) & mask_;
      const uint64_t nl = r;
      r = l ^ f;
      l = nl;
    }
    return (l << half_) | r;
  }
  uint64_t n_, key_, mask_;
  int half_;
};

struct Shard {
  std::string path;
  void* map = nullptr;
  size_t map_len = 0;
  const uint8_t* data = nullptr;
  int64_t n_tokens = 0;
  int bpt = 0;
};

// (token count, bytes per token, header bytes) of one file; raw files need bpt_hint.
static std::tuple<int64_t, int, size_t> probe(const std::string& path, size_t file_len, const uint8_t* head,
                                              int bpt_hint) {
  if (file_len >= kHeaderBytes && std::memcmp(head, kMagic, 8) == 0) {
    uint32_t version, bpt;
    uint64_t n;
    std::memcpy(&version, head + 8, 4);
    std::memcpy(&bpt, head + 12, 4);
    std::memcpy(&n, head + 16, 8);
    if (version != kVersion) throw std::runtime_error(path + ": unsupported token-file version " + std::to_string(version));
    if (bpt != 2 && bpt != 4) throw std::runtime_error(path + ": bytes per token must be 2 or 4, header says " + std::to_string(bpt));
    if (kHeaderBytes + n * bpt > file_len)
      throw std::runtime_error(path + ": header claims " + std::to_string(n) + " tokens but the file is shorter");
    return {(int64_t)n, (int)bpt, kHeaderBytes};
  }
  if (bpt_hint != 2 && bpt_hint != 4)
    throw std::runtime_error(path + ": no token-file header; pass bytes_per_token = 2 or 4 for a raw file");
  if (file_len % bpt_hint != 0)
    throw std::runtime_error(path + ": raw file size is not a multiple of " + std::to_string(bpt_hint));
  return {(int64_t)(file_len / bpt_hint), bpt_hint, 0};
}

class TokenStream {
 public:
  // random: windows are read in a shuffled order (no read-ahead); otherwise in file order
  TokenStream(const std::vector<std::string>& paths, int bpt_hint, bool random) {
    if (paths.empty()) throw std::runtime_error("no token files given");
    int64_t start = 0;
    for (const auto& p : paths) {
      Shard s;
      s.path = p;
      const int fd = ::open(p.c_str(), O_RDONLY);
      if (fd < 0) throw std::runtime_error(p + ": cannot open (" + std::strerror(errno) + ")");
      struct stat st;
      if (::fstat(fd, &st) != 0) {
        ::close(fd);
        throw std::runtime_error(p + ": cannot stat");
      }
      s.map_len = (size_t)st.st_size;
      if (s.map_len == 0) {
        ::close(fd);
        continue;  // an empty shard adds nothing
      }
      s.map = ::mmap(nullptr, s.map_len, PROT_READ, MAP_SHARED, fd, 0);
      ::close(fd);  // the mapping keeps the file referenced
      if (s.map == MAP_FAILED) throw std::runtime_error(p + ": mmap failed");
      ::madvise(s.map, s.map_len, random ? MADV_RANDOM : MADV_SEQUENTIAL);
      const uint8_t* base = static_cast<const uint8_t*>(s.map);
      auto [n, bpt, hdr] = probe(p, s.map_len, base, bpt_hint);
      s.n_tokens = n;
      s.bpt = bpt;
      s.data = base + hdr;
      shards_.push_back(s);
      starts_.push_back(start);
      start += n;
    }
    total_ = start;
  }
  ~TokenStream() {
    for (auto& s : shards_)
      if (s.map) ::munmap(s.map, s.map_len);
  }
  TokenStream(const TokenStream&) = delete;
  TokenStream& operator=(const TokenStream&) = delete;

  int64_t total() const { return total_; }

  // Copy tokens [g0, g0 + n) of the stream into out (as int64); checks ids against vocab when vocab > 0.
  void read(int64_t g0, int64_t n, int64_t* out, int64_t vocab) const {
    size_t s = std::upper_bound(starts_.begin(), starts_.end(), g0) - starts_.begin() - 1;
    while (n > 0) {
      const Shard& sh = shards_[s];
      const int64_t off = g0 - starts_[s];
      const int64_t take = std::min(n, sh.n_tokens - off);
      if (sh.bpt == 2) {
        const uint8_t* p = sh.data + off * 2;
        for (int64_t i = 0; i < take; ++i) {
          uint16_t v;
          std::memcpy(&v, p + 2 * i, 2);
          out[i] = v;
        }
      } else {
        const uint8_t* p = sh.data + off * 4;
        for (int64_t i = 0; i < take; ++i) {
          uint32_t v;
          std::memcpy(&v, p + 4 * i, 4);
          out[i] = v;
        }
      }
      if (vocab > 0) {
        for (int64_t i = 0; i < take; ++i)
          if (out[i] >= vocab)
            throw std::runtime_error(sh.path + ": token " + std::to_string(out[i]) + " at token offset " +
                                     std::to_string(off + i) + " is outside the vocabulary of " +
                                     std::to_string(vocab));
      }
      out += take;
      g0 += take;
      n -= take;
      ++s;
    }
  }

 private:
  std::vector<Shard> shards_;
  std::vector<int64_t> starts_;
  int64_t total_ = 0;
};

class TokenLoader {
 public:
  TokenLoader(std::vector<std::string> paths, int64_t seq_len, int64_t local_batch, int64_t rank, int64_t world,
              uint64_t seed, bool shuffle, int64_t depth, int64_t vocab, int64_t bytes_per_token,
              int64_t position, double timeout_s)
      : stream_(paths, (int)bytes_per_token, shuffle),
        S_(seq_len),
        b_(local_batch),
        rank_(rank),
        world_(world),
        seed_(seed),
        shuffle_(shuffle),
        depth_(std::max<int64_t>(1, depth)),
        vocab_(vocab),
        timeout_s_(timeout_s) {
    if (S_ < 1 || b_ < 1) throw std::invalid_argument("seq_len and local_batch must be positive");
    if (world_ < 1 || rank_ < 0 || rank_ >= world_) throw std::invalid_argument("rank must lie in [0, world)");
    if (position < 0) throw std::invalid_argument("position must be non-negative");
    windows_ = stream_.total() / (S_ + 1);
    if (windows_ < 1)
      throw std::runtime_error("the token files hold " + std::to_string(stream_.total()) +
                               " tokens, fewer than one window of seq_len + 1 = " + std::to_string(S_ + 1));
    start(position);
  }
  ~TokenLoader() { halt(); }

  int64_t total_tokens() const { return stream_.total(); }
  int64_t windows() const { return windows_; }
  int64_t global_batch() const { return world_ * b_; }
  int64_t position() const {
    std::lock_guard<std::mutex> g(mu_);
    return consumed_;
  }

  // Window index read by global sample g.
  int64_t window_of(int64_t g) const {
    if (g < 0) throw std::invalid_argument("sample index must be non-negative");
    const uint64_t e = (uint64_t)(g / windows_), j = (uint64_t)(g % windows_);
    if (!shuffle_) return (int64_t)j;
    return (int64_t)Permutation((uint64_t)windows_, mix64(seed_ ^ mix64(e + 1)))(j);
  }

  // Next batch into tokens / labels ([b, S] int64, contiguous, CPU; pinned or not).
  void next(torch::Tensor tokens, torch::Tensor labels) {
    check_out(tokens, "tokens");
    check_out(labels, "labels");
    int64_t* tk = tokens.data_ptr<int64_t>();
    int64_t* lb = labels.data_ptr<int64_t>();
    Batch batch;
    {
      pybind11::gil_scoped_release nogil;
      std::unique_lock<std::mutex> lk(mu_);
      const auto limit = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s_);
      while (ring_.empty() && error_.empty()) {
        if (ready_cv_.wait_until(lk, limit) == std::cv_status::timeout && ring_.empty() && error_.empty())
          throw std::runtime_error("token loader: no batch within " + std::to_string(timeout_s_) + " s");
      }
      if (ring_.empty()) throw std::runtime_error("token loader: " + error_);
      batch = std::move(ring_.front());
      ring_.pop_front();
      consumed_ = batch.pos + world_ * b_;
      space_cv_.notify_one();
    }
    const int64_t L = S_ + 1;
    for (int64_t i = 0; i < b_; ++i) {
      const int64_t* w = batch.buf.data() + i * L;
      std::memcpy(tk + i * S_, w, S_ * sizeof(int64_t));
      std::memcpy(lb + i * S_, w + 1, S_ * sizeof(int64_t));
    }
  }

  // Restart at global sample `position` (drops the prepared batches).
  void seek(int64_t position) {
    if (position < 0) throw std::invalid_argument("position must be non-negative");
    pybind11::gil_scoped_release nogil;
    halt();
    start(position);
  }

 private:
  struct Batch {
    int64_t pos = 0;
    std::vector<int64_t> buf;
  };

  // Argument errors are raised as std::invalid_argument (ValueError in Python).
  void check_out(const torch::Tensor& t, const std::string& name) const {
    if (!t.device().is_cpu()) throw std::invalid_argument(name + " must be a CPU tensor");
    if (t.scalar_type() != torch::kInt64) throw std::invalid_argument(name + " must be int64");
    if (!t.is_contiguous()) throw std::invalid_argument(name + " must be contiguous");
    if (t.dim() != 2 || t.size(0) != b_ || t.size(1) != S_)
      throw std::invalid_argument(name + " must have shape [" + std::to_string(b_) + ", " + std::to_string(S_) + "]");
  }

  void start(int64_t position) {
    std::lock_guard<std::mutex> g(mu_);
    consumed_ = position;
    next_pos_ = position;
    stop_ = false;
    error_.clear();
    ring_.clear();
    worker_ = std::thread([this] { run(); });
  }

  void halt() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    space_cv_.notify_all();
    if (worker_.joinable()) worker_.join();
  }

  void run() {
    const int64_t L = S_ + 1;
    for (;;) {
      int64_t pos;
      {
        std::unique_lock<std::mutex> lk(mu_);
        space_cv_.wait(lk, [&] { return stop_ || (int64_t)ring_.size() < depth_; });
        if (stop_) return;
        pos = next_pos_;
        next_pos_ += world_ * b_;
      }
      Batch batch;
      batch.pos = pos;
      batch.buf.resize((size_t)(b_ * L));
      try {
        for (int64_t i = 0; i < b_; ++i) {
          const int64_t w = window_of(pos + rank_ * b_ + i);
          stream_.read(w * L, L, batch.buf.data() + i * L, vocab_);
        }
      } catch (const std::exception& e) {
        std::lock_guard<std::mutex> g(mu_);
        error_ = e.what();
        ready_cv_.notify_all();
        return;
      }
      {
        std::lock_guard<std::mutex> g(mu_);
        if (stop_) return;
        ring_.push_back(std::move(batch));
      }
      ready_cv_.notify_one();
    }
  }

  TokenStream stream_;
  const int64_t S_, b_, rank_, world_;
  const uint64_t seed_;
  const bool shuffle_;
  const int64_t depth_, vocab_;
  const double timeout_s_;
  int64_t windows_ = 0;

  mutable std::mutex mu_;
  std::condition_variable ready_cv_, space_cv_;
  std::deque<Batch> ring_;
  std::thread worker_;
  int64_t consumed_ = 0, next_pos_ = 0;
  bool stop_ = false;
  std::string error_;
};

// (token count, bytes per token, header bytes) of a token file.
static std::tuple<int64_t, int64_t, int64_t> file_info(const std::string& path, int64_t bytes_per_token) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error(path + ": cannot open (" + std::strerror(errno) + ")");
  struct stat st;
  uint8_t head[kHeaderBytes] = {0};
  const bool ok = ::fstat(fd, &st) == 0;
  const ssize_t got = ok ? ::pread(fd, head, kHeaderBytes, 0) : -1;
  ::close(fd);
  if (!ok || got < 0) throw std::runtime_error(path + ": cannot read");
  auto [n, bpt, hdr] = probe(path, (size_t)st.st_size, head, (int)bytes_per_token);
  return {n, (int64_t)bpt, (int64_t)hdr};
}

}  // namespace bdion_io

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using bdion_io::TokenLoader;
  m.doc() = "dion_b200 native data loading (memory-mapped token files, background prefetch)";
  pybind11::class_<TokenLoader>(m, "TokenLoader")
      .def(pybind11::init<std::vector<std::string>, int64_t, int64_t, int64_t, int64_t, uint64_t, bool, int64_t,
                          int64_t, int64_t, int64_t, double>(),
           pybind11::arg("paths"), pybind11::arg("seq_len"), pybind11::arg("local_batch"), pybind11::arg("rank"),
           pybind11::arg("world"), pybind11::arg("seed"), pybind11::arg("shuffle"), pybind11::arg("depth"),
           pybind11::arg("vocab"), pybind11::arg("bytes_per_token"), pybind11::arg("position"),
           pybind11::arg("timeout_s"))
      .def("next", &TokenLoader::next, pybind11::arg("tokens"), pybind11::arg("labels"))
      .def("seek", &TokenLoader::seek, pybind11::arg("position"))
      .def("window_of", &TokenLoader::window_of, pybind11::arg("sample"))
      .def_property_readonly("position", &TokenLoader::position)
      .def_property_readonly("windows", &TokenLoader::windows)
      .def_property_readonly("total_tokens", &TokenLoader::total_tokens)
      .def_property_readonly("global_batch", &TokenLoader::global_batch);
  m.def("file_info", &bdion_io::file_info, pybind11::arg("path"), pybind11::arg("bytes_per_token") = 0);
  m.attr("MAGIC") = std::string(bdion_io::kMagic, 8);
  m.attr("HEADER_BYTES") = (int64_t)bdion_io::kHeaderBytes;
  m.attr("VERSION") = (int64_t)bdion_io::kVersion;
}
