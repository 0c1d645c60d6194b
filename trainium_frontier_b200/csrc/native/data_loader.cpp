// Host-side data path: a seeded synthetic document source and the BOS-aligned
// best-fit row packer, in C++ so the per-row O(buffer) search never holds the GIL.
//
// Behaviour mirrored from the reference's trusted loader (prepare.py:456-518):
//   * rows have capacity seq_len + 1 tokens, inputs = row[:-1], targets = row[1:];
//   * a buffer of at least 512 whole documents (each starting with BOS) is kept;
//   * for the remaining capacity of a row, the LONGEST buffered document that still
//     fits is placed whole; if none fits, the SHORTEST one is cropped to fill the row.
// The documents themselves are synthetic (no dataset is available): token ids drawn
// from a seeded Zipf(s) law over [1, vocab) with BOS = 0 prepended, and document
// lengths geometric with a given mean.  Randomness is xoshiro256** (Blackman & Vigna,
// "Scrambled linear pseudorandom number generators", 2018) seeded through SplitMix64,
// so the Python mirror in data/synthetic.py reproduces the stream bit for bit.
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <memory>
#include <vector>

namespace {

inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

struct SplitMix64 {
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
};

struct Xoshiro256ss {
  uint64_t s[4];
  explicit Xoshiro256ss(uint64_t seed) {
    SplitMix64 sm{seed};
    for (auto& v : s) v = sm.next();
  }
  uint64_t next() {
    const uint64_t result = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
  }
  // uniform double in [0, 1) with 53 random bits
  double uniform() { return double(next() >> 11) * (1.0 / 9007199254740992.0); }
};

class ZipfDocSource {
 public:
  ZipfDocSource(int64_t vocab, double s, double mean_doc_len, uint64_t seed, int64_t bos)
      : rng_(seed), bos_(bos), p_geo_(1.0 / std::max(1.0, mean_doc_len)) {
    TORCH_CHECK(vocab > 2, "vocab must be > 2");
    cdf_.resize(vocab - 1);
    double acc = 0.0;
    for (int64_t k = 1; k < vocab; ++k) {
      acc += std::pow(double(k), -s);
      cdf_[k - 1] = acc;
    }
    for (auto& c : cdf_) c /= acc;
    cdf_.back() = 1.0;
    log1mp_ = std::log1p(-p_geo_);
  }

  int64_t sample_token() {
    const double u = rng_.uniform();
    auto it = std::upper_bound(cdf_.begin(), cdf_.end(), u);
    int64_t idx = int64_t(it - cdf_.begin());
    if (idx >= int64_t(cdf_.size())) idx = int64_t(cdf_.size()) - 1;
    return idx + 1;
  }

  // geometric number of content tokens (>= 1), mean 1/p
  int64_t sample_len() {
    double u = rng_.uniform();
    if (u <= 0.0) u = 1e-300;
    const double g = std::floor(std::log(u) / log1mp_);
    return 1 + int64_t(std::min(g, 1e7));
  }

  std::vector<int64_t> next_doc() {
    const int64_t n = sample_len();
    std::vector<int64_t> d;
    d.reserve(n + 1);
    d.push_back(bos_);
    for (int64_t i = 0; i < n; ++i) d.push_back(sample_token());
    return d;
  }

 private:
  Xoshiro256ss rng_;
  int64_t bos_;
  double p_geo_;
  double log1mp_;
  std::vector<double> cdf_;
};

// One row of capacity `cap` from the buffered documents: the longest document that still
// fits the remaining capacity is placed whole; if none fits, the shortest one is cropped
// to fill the row.  `refill` tops the buffer up before every pick (synthetic source) or
// is a no-op (documents pushed by the caller).  Returns false if the buffer ran dry.
template <typename Refill>
bool fill_row(std::vector<std::vector<int64_t>>& buf, int32_t* row, int64_t cap, Refill refill) {
  int64_t pos = 0;
  while (pos < cap) {
    refill();
    if (buf.empty()) return false;
    const int64_t remaining = cap - pos;
    int64_t best = -1, best_len = 0;
    for (int64_t i = 0; i < int64_t(buf.size()); ++i) {
      const int64_t n = int64_t(buf[i].size());
      if (n <= remaining && n > best_len) { best = i; best_len = n; }
    }
    if (best >= 0) {
      const auto& d = buf[best];
      for (int64_t j = 0; j < best_len; ++j) row[pos + j] = int32_t(d[j]);
      pos += best_len;
      buf.erase(buf.begin() + best);
    } else {
      int64_t shortest = 0;
      for (int64_t i = 1; i < int64_t(buf.size()); ++i)
        if (buf[i].size() < buf[shortest].size()) shortest = i;
      const auto& d = buf[shortest];
      for (int64_t j = 0; j < remaining; ++j) row[pos + j] = int32_t(d[j]);
      pos += remaining;
      buf.erase(buf.begin() + shortest);
    }
  }
  return true;
}

class BestFitPacker {
 public:
  BestFitPacker(int64_t vocab, double zipf_s, double mean_doc_len, uint64_t seed, int64_t bos,
                int64_t buffer_min)
      : src_(vocab, zipf_s, mean_doc_len, seed, bos), buffer_min_(buffer_min) {}

  // Fills rows [batch, seq_len + 1] (int32, contiguous) with packed documents.
  void fill(torch::Tensor rows) {
    TORCH_CHECK(rows.dtype() == torch::kInt32 && rows.is_contiguous() && rows.dim() == 2,
                "rows must be a contiguous int32 [B, T+1] tensor");
    TORCH_CHECK(rows.device().is_cpu(), "rows must live in host memory");
    const int64_t B = rows.size(0), cap = rows.size(1);
    int32_t* out = rows.data_ptr<int32_t>();
    pybind11::gil_scoped_release nogil;
    auto refill = [this] {
      while (int64_t(buf_.size()) < buffer_min_) buf_.push_back(src_.next_doc());
    };
    for (int64_t r = 0; r < B; ++r) fill_row(buf_, out + r * cap, cap, refill);
  }

  // Contiguous (unpacked) token stream: documents back to back, used by the
  // eval loader, which chunks a stream into rows without packing.
  void fill_stream(torch::Tensor out_t) {
    TORCH_CHECK(out_t.dtype() == torch::kInt32 && out_t.is_contiguous(), "int32 contiguous");
    int32_t* out = out_t.data_ptr<int32_t>();
    const int64_t n = out_t.numel();
    pybind11::gil_scoped_release nogil;
    int64_t pos = 0;
    while (pos < n) {
      if (stream_.empty() || stream_pos_ >= int64_t(stream_.size())) {
        stream_ = src_.next_doc();
        stream_pos_ = 0;
      }
      const int64_t take = std::min<int64_t>(n - pos, int64_t(stream_.size()) - stream_pos_);
      for (int64_t j = 0; j < take; ++j) out[pos + j] = int32_t(stream_[stream_pos_ + j]);
      pos += take;
      stream_pos_ += take;
    }
  }

  std::vector<int64_t> next_doc() { return src_.next_doc(); }

 private:
  ZipfDocSource src_;
  int64_t buffer_min_;
  std::vector<std::vector<int64_t>> buf_;
  std::vector<int64_t> stream_;
  int64_t stream_pos_ = 0;
};

// The same packing over documents the caller supplies (tokenized text): push() appends
// whole documents (BOS first) to the buffer; fill() packs rows while the buffer holds at
// least `buffer_min` documents at the start of a row (with `drain`, until it is empty, for
// the end of the data) and returns how many rows of [r0, B) it completed.  Unlike the
// synthetic source, which tops the buffer up before every pick, the caller refills
// between fill() calls, so within one row the buffer may dip below buffer_min.
class DocPacker {
 public:
  explicit DocPacker(int64_t buffer_min) : buffer_min_(buffer_min) {}

  void push(torch::Tensor doc) {
    TORCH_CHECK(doc.device().is_cpu() && doc.dim() == 1 && doc.numel() > 0, "a non-empty 1-D host tensor");
    auto d = doc.to(torch::kInt64).contiguous();
    const int64_t* p = d.data_ptr<int64_t>();
    buf_.emplace_back(p, p + d.numel());
  }

  int64_t buffered() const { return int64_t(buf_.size()); }

  int64_t fill(torch::Tensor rows, int64_t r0, bool drain) {
    TORCH_CHECK(rows.dtype() == torch::kInt32 && rows.is_contiguous() && rows.dim() == 2 && rows.device().is_cpu(),
                "rows must be a contiguous int32 [B, T+1] host tensor");
    const int64_t B = rows.size(0), cap = rows.size(1);
    int32_t* out = rows.data_ptr<int32_t>();
    pybind11::gil_scoped_release nogil;
    int64_t r = r0;
    for (; r < B; ++r) {
      if (buf_.empty() || (!drain && int64_t(buf_.size()) < buffer_min_)) break;
      if (!fill_row(buf_, out + r * cap, cap, [] {})) break;
    }
    return r - r0;
  }

 private:
  int64_t buffer_min_;
  std::vector<std::vector<int64_t>> buf_;
};

torch::Tensor token_bytes_table(int64_t vocab, uint64_t seed, int64_t lo, int64_t hi,
                                int64_t n_special) {
  auto t = torch::empty({vocab}, torch::kInt32);
  int32_t* p = t.data_ptr<int32_t>();
  Xoshiro256ss rng(seed);
  const uint64_t span = uint64_t(hi - lo + 1);
  for (int64_t i = 0; i < vocab; ++i) {
    const uint64_t r = rng.next();
    p[i] = (i < n_special) ? 0 : int32_t(lo + int64_t(r % span));
  }
  return t;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "trainium_frontier_b200 native host runtime (data loader)";
  pybind11::class_<BestFitPacker>(m, "BestFitPacker")
      .def(pybind11::init<int64_t, double, double, uint64_t, int64_t, int64_t>(),
           pybind11::arg("vocab"), pybind11::arg("zipf_s"), pybind11::arg("mean_doc_len"),
           pybind11::arg("seed"), pybind11::arg("bos"), pybind11::arg("buffer_min"))
      .def("fill", &BestFitPacker::fill)
      .def("fill_stream", &BestFitPacker::fill_stream)
      .def("next_doc", &BestFitPacker::next_doc);
  pybind11::class_<DocPacker>(m, "DocPacker")
      .def(pybind11::init<int64_t>(), pybind11::arg("buffer_min"))
      .def("push", &DocPacker::push)
      .def("buffered", &DocPacker::buffered)
      .def("fill", &DocPacker::fill, pybind11::arg("rows"), pybind11::arg("r0"), pybind11::arg("drain"));
  m.def("token_bytes_table", &token_bytes_table, "seeded per-token byte lengths");
}
