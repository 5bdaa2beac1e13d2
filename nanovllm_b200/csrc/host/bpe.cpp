// Host-side tokenizer core (no CUDA): byte-level BPE merging of pre-split words.
//
// The reference encodes with Java code (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tokenizer/
// Gpt2ByteBpeCodec.java and BpeMerges.java): bytes are mapped to printable symbols, then the adjacent pair with
// the lowest merge rank is merged, every non-overlapping occurrence left to right, until no pair has a rank.
// Here the symbols are small integers: the Python side interns every symbol string that a merge can produce,
// hands over (left, right) -> (rank, merged) triples and the vocabulary id of every symbol, and this core runs
// the merge rounds on int32 vectors.  A final symbol without a vocabulary id falls back to the ids of its
// characters (a CSR list per symbol), exactly as the Python codec does.
#include <torch/extension.h>

#include <climits>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

struct Merge {
  int32_t rank;
  int32_t merged;
};

class ByteBpeCore {
 public:
  ByteBpeCore(std::vector<int32_t> byte_sym, const std::vector<int32_t>& left, const std::vector<int32_t>& right,
              const std::vector<int32_t>& rank, const std::vector<int32_t>& merged, std::vector<int32_t> sym_vocab,
              std::vector<int32_t> fb_off, std::vector<int32_t> fb_ids)
      : byte_sym_(std::move(byte_sym)), sym_vocab_(std::move(sym_vocab)), fb_off_(std::move(fb_off)),
        fb_ids_(std::move(fb_ids)) {
    TORCH_CHECK(byte_sym_.size() == 256, "byte table needs 256 entries");
    TORCH_CHECK(left.size() == right.size() && left.size() == rank.size() && left.size() == merged.size(),
                "merge arrays differ in length");
    TORCH_CHECK(fb_off_.size() == sym_vocab_.size() + 1, "fallback offsets need one entry per symbol plus one");
    merges_.reserve(left.size() * 2);
    for (size_t i = 0; i < left.size(); ++i) merges_[key(left[i], right[i])] = Merge{rank[i], merged[i]};
  }

  std::vector<int32_t> encode_word(const std::string& bytes) const {
    std::vector<int32_t> out;
    encode_into(bytes, out);
    return out;
  }

  // all words' ids concatenated, with the id count of each word (for the caller's cache)
  std::pair<std::vector<int32_t>, std::vector<int32_t>> encode_words(const std::vector<std::string>& words) const {
    std::vector<int32_t> ids, counts;
    counts.reserve(words.size());
    for (const auto& w : words) {
      size_t before = ids.size();
      encode_into(w, ids);
      counts.push_back(static_cast<int32_t>(ids.size() - before));
    }
    return {ids, counts};
  }

 private:
  static uint64_t key(int32_t a, int32_t b) {
    return (static_cast<uint64_t>(static_cast<uint32_t>(a)) << 32) | static_cast<uint32_t>(b);
  }

  const Merge* find(int32_t a, int32_t b) const {
    auto it = merges_.find(key(a, b));
    return it == merges_.end() ? nullptr : &it->second;
  }

  void encode_into(const std::string& bytes, std::vector<int32_t>& out) const {
    std::vector<int32_t> syms, next;
    syms.reserve(bytes.size());
    for (unsigned char c : bytes) syms.push_back(byte_sym_[c]);
    while (syms.size() > 1) {
      int32_t best = INT32_MAX, best_merged = -1;
      for (size_t i = 0; i + 1 < syms.size(); ++i) {
        const Merge* m = find(syms[i], syms[i + 1]);
        if (m != nullptr && m->rank < best) {
          best = m->rank;
          best_merged = m->merged;
        }
      }
      if (best_merged < 0) break;
      next.clear();
      size_t i = 0;
      while (i < syms.size()) {
        if (i + 1 < syms.size()) {
          const Merge* m = find(syms[i], syms[i + 1]);
          if (m != nullptr && m->rank == best) {
            next.push_back(best_merged);
            i += 2;
            continue;
          }
        }
        next.push_back(syms[i]);
        ++i;
      }
      syms.swap(next);
    }
    for (int32_t s : syms) {
      int32_t v = sym_vocab_[s];
      if (v >= 0) {
        out.push_back(v);
      } else {
        for (int32_t k = fb_off_[s]; k < fb_off_[s + 1]; ++k) out.push_back(fb_ids_[k]);
      }
    }
  }

  std::vector<int32_t> byte_sym_;
  std::unordered_map<uint64_t, Merge> merges_;
  std::vector<int32_t> sym_vocab_;
  std::vector<int32_t> fb_off_;
  std::vector<int32_t> fb_ids_;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "host-side runtime helpers (tokenizer core)";
  pybind11::class_<ByteBpeCore>(m, "ByteBpeCore")
      .def(pybind11::init<std::vector<int32_t>, const std::vector<int32_t>&, const std::vector<int32_t>&,
                          const std::vector<int32_t>&, const std::vector<int32_t>&, std::vector<int32_t>,
                          std::vector<int32_t>, std::vector<int32_t>>())
      .def("encode_word", [](const ByteBpeCore& self, pybind11::bytes b) { return self.encode_word(b); })
      .def("encode_words", &ByteBpeCore::encode_words);
}
