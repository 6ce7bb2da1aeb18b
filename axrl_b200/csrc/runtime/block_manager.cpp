// Paged-KV block manager with a prefix cache (host side of the rollout engine).
//
// Reference counterpart: SGLang's token-to-KV pool + radix cache (reached through
// axrl/worker/sglang_worker.py:80-107; cached_tokens reported at :576).
//
// Pages are fixed-size runs of `page_size` token slots.  Every page has a reference count
// (one per sequence whose block table holds it).  A *full* page can additionally be
// registered in the prefix cache under a chained content hash
//     h_i = mix(h_{i-1}, tokens[i*P .. (i+1)*P))
// so a later request whose prompt starts with the same tokens reuses the page instead of
// recomputing it.  Cached pages whose refcount drops to zero stay resident on an LRU list
// and are evicted only when the free list runs dry.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <list>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace ax_rt {

static inline uint64_t mix64(uint64_t h, uint64_t v) {
  // SplitMix64-style finaliser over (h, v); deterministic across processes.
  uint64_t z = h ^ (v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2));
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

class BlockManager {
 public:
  BlockManager(int64_t num_pages, int64_t page_size)
      : page_size_(page_size), ref_(num_pages, 0), hash_of_(num_pages, 0), cached_(num_pages, false), lru_pos_(num_pages) {
    if (num_pages <= 0 || page_size <= 0) throw std::invalid_argument("num_pages and page_size must be positive");
    free_.reserve(num_pages);
    for (int64_t i = num_pages - 1; i >= 0; --i) free_.push_back((int32_t)i);
  }

  int64_t page_size() const { return page_size_; }
  int64_t num_pages() const { return (int64_t)ref_.size(); }
  // pages obtainable right now (free + evictable cached)
  int64_t num_available() const { return (int64_t)free_.size() + (int64_t)lru_.size(); }
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_cached() const { return (int64_t)index_.size(); }

  std::vector<int32_t> allocate(int64_t n) {
    if (n > num_available()) throw std::runtime_error("KV cache out of pages");
    std::vector<int32_t> out;
    out.reserve(n);
    for (int64_t i = 0; i < n; ++i) {
      if (free_.empty()) evict_one();
      int32_t p = free_.back();
      free_.pop_back();
      ref_[p] = 1;
      out.push_back(p);
    }
    return out;
  }

  void incref(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      check(p);
      if (ref_[p] == 0 && cached_[p]) lru_.erase(lru_pos_[p]);
      ++ref_[p];
    }
  }

  void release(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      check(p);
      if (ref_[p] <= 0) throw std::runtime_error("double free of KV page");
      if (--ref_[p] == 0) {
        if (cached_[p]) {
          lru_.push_back(p);
          lru_pos_[p] = std::prev(lru_.end());
        } else {
          free_.push_back(p);
        }
      }
    }
  }

  // Longest cached prefix of `tokens` in whole pages.  Returns the pages (with refcounts
  // taken) and the number of tokens they cover.
  std::pair<std::vector<int32_t>, int64_t> match_prefix(const std::vector<int64_t>& tokens) {
    std::vector<int32_t> pages;
    uint64_t h = 0;
    int64_t full = (int64_t)tokens.size() / page_size_;
    for (int64_t i = 0; i < full; ++i) {
      h = page_hash(h, tokens, i);
      auto it = index_.find(h);
      if (it == index_.end()) break;
      pages.push_back(it->second);
    }
    incref(pages);
    ++lookups_;
    hit_tokens_ += (int64_t)pages.size() * page_size_;
    return {pages, (int64_t)pages.size() * page_size_};
  }

  // Register the full pages of a sequence (its block table) under their content hashes.
  void insert(const std::vector<int64_t>& tokens, const std::vector<int32_t>& pages) {
    uint64_t h = 0;
    int64_t full = std::min<int64_t>((int64_t)tokens.size() / page_size_, (int64_t)pages.size());
    for (int64_t i = 0; i < full; ++i) {
      h = page_hash(h, tokens, i);
      int32_t p = pages[i];
      check(p);
      if (index_.count(h) || cached_[p]) continue;
      index_[h] = p;
      hash_of_[p] = h;
      cached_[p] = true;
    }
  }

  void clear_cache() {
    for (int32_t p : lru_) {
      cached_[p] = false;
      free_.push_back(p);
    }
    lru_.clear();
    for (auto& kv : index_) cached_[kv.second] = false;
    index_.clear();
  }

  py::dict stats() const {
    py::dict d;
    d["num_pages"] = num_pages();
    d["free"] = num_free();
    d["cached"] = num_cached();
    d["evictable"] = (int64_t)lru_.size();
    d["lookups"] = lookups_;
    d["hit_tokens"] = hit_tokens_;
    return d;
  }

 private:
  uint64_t page_hash(uint64_t h, const std::vector<int64_t>& t, int64_t i) const {
    for (int64_t j = i * page_size_; j < (i + 1) * page_size_; ++j) h = mix64(h, (uint64_t)t[j]);
    return mix64(h, 0xC0FFEEull + (uint64_t)i);
  }
  void check(int32_t p) const {
    if (p < 0 || p >= (int32_t)ref_.size()) throw std::out_of_range("page id out of range");
  }
  void evict_one() {
    if (lru_.empty()) throw std::runtime_error("KV cache out of pages");
    int32_t p = lru_.front();
    lru_.pop_front();
    index_.erase(hash_of_[p]);
    cached_[p] = false;
    free_.push_back(p);
  }

  int64_t page_size_;
  std::vector<int32_t> ref_;
  std::vector<uint64_t> hash_of_;
  std::vector<bool> cached_;
  std::vector<std::list<int32_t>::iterator> lru_pos_;
  std::vector<int32_t> free_;
  std::list<int32_t> lru_;
  std::unordered_map<uint64_t, int32_t> index_;
  int64_t lookups_ = 0, hit_tokens_ = 0;
};

void bind_block_manager(py::module_& m) {
  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int64_t, int64_t>(), py::arg("num_pages"), py::arg("page_size"))
      .def_property_readonly("page_size", &BlockManager::page_size)
      .def_property_readonly("num_pages", &BlockManager::num_pages)
      .def("num_available", &BlockManager::num_available)
      .def("num_free", &BlockManager::num_free)
      .def("num_cached", &BlockManager::num_cached)
      .def("allocate", &BlockManager::allocate)
      .def("incref", &BlockManager::incref)
      .def("release", &BlockManager::release)
      .def("match_prefix", &BlockManager::match_prefix)
      .def("insert", &BlockManager::insert)
      .def("clear_cache", &BlockManager::clear_cache)
      .def("stats", &BlockManager::stats);
}

}  // namespace ax_rt
