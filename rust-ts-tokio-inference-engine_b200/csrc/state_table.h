// Generation-checked state-version table (host side, worker-confined).
//
// Same contract as the reference's StateTable (native/state_table.h:14-38):
// a StateId {owner, slot, generation, position, bytes} is valid only while the
// slot is reserved with exactly that generation and geometry; reserve charges
// bytes against a budget; publish/get/rollback/release/clear. Differences: the
// slot bound is 1..1<<20 (the reference caps at 64 because each MLX version
// copies whole context-capacity buffers; here a version is a page list plus one
// DeltaNet slot), and reserve_at() reserves a specific free slot (used when a
// step consumes its parent in place).
#pragma once
#include <cstdint>
#include <limits>
#include <optional>
#include <stdexcept>
#include <utility>
#include <vector>

#include "../../include/qwen_b200.h"

namespace qwen {

template <class T>
class StateTable {
  struct Entry {
    uint64_t generation = 0, position = 0, bytes = 0;
    bool reserved = false;
    std::optional<T> value;
  };
  uint64_t owner_, cap_, used_ = 0;
  std::vector<Entry> entries_;
  size_t scan_ = 0;

  Entry& checked(StateId id) {
    if (id.owner != owner_ || id.slot >= entries_.size())
      throw std::invalid_argument("foreign state owner/slot");
    auto& e = entries_[id.slot];
    if (!e.reserved || e.generation != id.generation || e.position != id.position ||
        e.bytes != id.bytes)
      throw std::invalid_argument("stale state generation/geometry");
    return e;
  }

 public:
  StateTable(uint64_t owner, size_t slots, uint64_t bytes)
      : owner_(owner), cap_(bytes), entries_(slots) {
    if (!owner || !slots || slots > (size_t(1) << 20) || !bytes)
      throw std::invalid_argument("state table bounds");
  }
  uint64_t owner() const { return owner_; }
  size_t capacity() const { return entries_.size(); }
  StateId reserve_at(size_t slot, uint64_t position, uint64_t bytes) {
    if (slot >= entries_.size()) throw std::invalid_argument("state slot range");
    if (!position || !bytes || bytes > cap_ - used_)
      throw std::runtime_error("resident state byte budget exhausted");
    auto& e = entries_[slot];
    if (e.reserved || e.generation == std::numeric_limits<uint64_t>::max())
      throw std::runtime_error("state slot busy");
    ++e.generation;
    e.position = position;
    e.bytes = bytes;
    e.reserved = true;
    used_ += bytes;
    return {owner_, slot, e.generation, position, bytes};
  }
  StateId reserve(uint64_t position, uint64_t bytes) {
    if (!position || !bytes || bytes > cap_ - used_)
      throw std::runtime_error("resident state byte budget exhausted");
    for (size_t n = 0; n < entries_.size(); ++n) {
      size_t i = (scan_ + n) % entries_.size();
      auto& e = entries_[i];
      if (!e.reserved && e.generation != std::numeric_limits<uint64_t>::max()) {
        scan_ = (i + 1) % entries_.size();
        return reserve_at(i, position, bytes);
      }
    }
    throw std::runtime_error("resident state slots exhausted");
  }
  void publish(StateId id, T value) {
    auto& e = checked(id);
    if (e.value) throw std::invalid_argument("state already published");
    e.value.emplace(std::move(value));
  }
  const T& get(StateId id) {
    auto& e = checked(id);
    if (!e.value) throw std::invalid_argument("unpublished state");
    return *e.value;
  }
  T& get_mut(StateId id) {
    auto& e = checked(id);
    if (!e.value) throw std::invalid_argument("unpublished state");
    return *e.value;
  }
  void rollback(StateId id) {
    auto& e = checked(id);
    e.value.reset();
    e.reserved = false;
    used_ -= e.bytes;
  }
  void release(StateId id) {
    (void)get(id);
    rollback(id);
  }
  uint64_t bytes() const { return used_; }
  size_t residents() const {
    size_t n = 0;
    for (const auto& e : entries_) n += e.reserved;
    return n;
  }
  template <class F>
  void for_each_published(F f) {
    for (size_t i = 0; i < entries_.size(); ++i)
      if (entries_[i].reserved && entries_[i].value) f(i, *entries_[i].value);
  }
  void clear() {
    for (auto& e : entries_) {
      e.value.reset();
      e.reserved = false;
    }
    used_ = 0;
  }
};

}  // namespace qwen
