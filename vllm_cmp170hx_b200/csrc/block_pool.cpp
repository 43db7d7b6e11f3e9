// Native KV-block allocator with reference counts and a prefix-hash table
// (host side of the paged cache).  Interface mirrors engine/block_pool.py's
// PyBlockPool: allocate / free / cache_block / lookup / touch / ref / num_free.
// Freed blocks go to the tail of the free list, so blocks that still carry a
// cached prefix are reused last (LRU order).
#include <torch/extension.h>

#include <cstdint>
#include <list>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace b200 {

class BlockPool {
 public:
  BlockPool(int64_t num_blocks, int64_t reserved) : ref_(num_blocks, 0), pos_(num_blocks) {
    if (reserved < 0 || reserved > num_blocks) throw std::invalid_argument("bad reserved count");
    for (int64_t b = reserved; b < num_blocks; ++b) pos_[b] = free_.insert(free_.end(), b);
    in_free_.assign(num_blocks, false);
    for (int64_t b = reserved; b < num_blocks; ++b) in_free_[b] = true;
  }

  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_blocks() const { return (int64_t)ref_.size(); }

  std::vector<int64_t> allocate(int64_t n) {
    if (n > (int64_t)free_.size())
      throw std::runtime_error("out of KV blocks: want " + std::to_string(n) + ", have " +
                               std::to_string(free_.size()));
    std::vector<int64_t> out;
    out.reserve(n);
    for (int64_t i = 0; i < n; ++i) {
      const int64_t b = free_.front();
      free_.pop_front();
      in_free_[b] = false;
      auto it = block_hash_.find(b);
      if (it != block_hash_.end()) {
        auto jt = hash_to_block_.find(it->second);
        if (jt != hash_to_block_.end() && jt->second == b) hash_to_block_.erase(jt);
        block_hash_.erase(it);
      }
      ref_[b] = 1;
      out.push_back(b);
    }
    return out;
  }

  void free(const std::vector<int64_t>& blocks) {
    for (int64_t b : blocks) {
      check(b);
      if (ref_[b] <= 0) throw std::runtime_error("double free of block " + std::to_string(b));
      if (--ref_[b] == 0) {
        pos_[b] = free_.insert(free_.end(), b);
        in_free_[b] = true;
      }
    }
  }

  void cache_block(int64_t block, int64_t h) {
    check(block);
    hash_to_block_[h] = block;
    block_hash_[block] = h;
  }

  int64_t lookup(int64_t h) const {
    auto it = hash_to_block_.find(h);
    return it == hash_to_block_.end() ? -1 : it->second;
  }

  void touch(int64_t block) {
    check(block);
    if (ref_[block] == 0 && in_free_[block]) {
      free_.erase(pos_[block]);
      in_free_[block] = false;
    }
    ++ref_[block];
  }

  int64_t ref(int64_t block) const {
    check(block);
    return ref_[block];
  }

 private:
  void check(int64_t b) const {
    if (b < 0 || b >= (int64_t)ref_.size()) throw std::out_of_range("block id " + std::to_string(b));
  }
  std::vector<int64_t> ref_;
  std::list<int64_t> free_;
  std::vector<std::list<int64_t>::iterator> pos_;
  std::vector<bool> in_free_;
  std::unordered_map<int64_t, int64_t> hash_to_block_;
  std::unordered_map<int64_t, int64_t> block_hash_;
};

void register_block_pool(pybind11::module_& m) {
  pybind11::class_<BlockPool>(m, "BlockPool")
      .def(pybind11::init<int64_t, int64_t>(), pybind11::arg("num_blocks"), pybind11::arg("reserved") = 1)
      .def("num_free", &BlockPool::num_free)
      .def("num_blocks", &BlockPool::num_blocks)
      .def("allocate", &BlockPool::allocate)
      .def("free", &BlockPool::free)
      .def("cache_block", &BlockPool::cache_block)
      .def("lookup", &BlockPool::lookup)
      .def("touch", &BlockPool::touch)
      .def("ref", &BlockPool::ref);
}

}  // namespace b200
