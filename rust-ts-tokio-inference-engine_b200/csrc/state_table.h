// Version registry for device state (host side, worker-confined).
//
// Interface kept from the reference (native/state_table.h:11-38): a 40-byte
// StateId {owner, slot, generation, position, bytes} names one immutable state
// version; reserve charges its bytes against the session budget, publish makes
// it readable, rollback discards a reserved or published version, release
// discards a published one. The structure here is this backend's own:
//
//  - slots hold a phase (vacant / pending / live) in structure-of-arrays form,
//    with the payloads (page lists, hidden-row counts) kept apart from the
//    handle checks;
//  - vacant slots sit on a LIFO stack with a back-index, so reserve() and
//    reserve_at() are O(1) at any slot count (a cfg4 session holds thousands
//    of versions: 512 sequences plus one candidate per verified token);
//  - reserve_at() claims a named vacant slot, which is how a step that
//    consumes its parent writes the child into the parent's DeltaNet slot;
//  - a slot whose generation counter is exhausted is never handed out again.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../../include/qwen_b200.h"

namespace qwen {

template <class Payload>
class StateTable {
 public:
  StateTable(uint64_t owner, size_t slot_count, uint64_t byte_limit)
      : owner_(owner), limit_(byte_limit) {
    if (owner == 0 || slot_count == 0 || slot_count > kMaxSlots || byte_limit == 0)
      throw std::invalid_argument("state registry: owner, slot count (1..2^20) and byte limit must be non-zero");
    gen_.assign(slot_count, 0);
    pos_.assign(slot_count, 0);
    charge_.assign(slot_count, 0);
    phase_.assign(slot_count, Phase::Vacant);
    payload_.resize(slot_count);
    stack_index_.resize(slot_count);
    vacant_.reserve(slot_count);
    // lowest slot on top of the stack: fresh sessions fill slots 0, 1, 2, ...
    for (size_t i = slot_count; i-- > 0;) push_vacant(i);
  }

  uint64_t owner() const { return owner_; }
  size_t capacity() const { return gen_.size(); }
  uint64_t bytes() const { return charged_; }
  size_t residents() const { return gen_.size() - vacant_.size() - retired_; }

  // Claim any vacant slot for a version at `position` charged `charge` bytes.
  StateId reserve(uint64_t position, uint64_t charge) {
    admit(position, charge);
    if (vacant_.empty()) throw std::runtime_error("state registry: every slot holds a version");
    return claim(vacant_.back(), position, charge);
  }
  // Claim the named slot, which must be vacant.
  StateId reserve_at(size_t slot, uint64_t position, uint64_t charge) {
    if (slot >= gen_.size()) throw std::invalid_argument("state registry: slot index beyond the table");
    admit(position, charge);
    if (phase_[slot] != Phase::Vacant || stack_index_[slot] == kNotVacant)
      throw std::runtime_error("state registry: requested slot is not vacant");
    return claim(slot, position, charge);
  }

  void publish(const StateId& id, Payload value) {
    const size_t s = verify(id);
    if (phase_[s] != Phase::Pending) throw std::invalid_argument("state registry: version was published before");
    payload_[s] = std::move(value);
    phase_[s] = Phase::Live;
  }
  const Payload& get(const StateId& id) const { return payload_[live(id)]; }
  Payload& get_mut(const StateId& id) { return payload_[live(id)]; }

  // Discard a pending or live version and return its bytes to the budget.
  void rollback(const StateId& id) { vacate(verify(id)); }
  // Discard a live version (a pending one is an error: nothing was handed out).
  void release(const StateId& id) { vacate(live(id)); }

  template <class F>
  void for_each_published(F f) {
    for (size_t s = 0; s < gen_.size(); ++s)
      if (phase_[s] == Phase::Live) f(s, payload_[s]);
  }
  // Drop every version (device drain). Generations keep counting, so handles
  // issued before the clear stay invalid.
  void clear() {
    for (size_t s = 0; s < gen_.size(); ++s)
      if (phase_[s] != Phase::Vacant) vacate(s);
  }

 private:
  enum class Phase : uint8_t { Vacant, Pending, Live };
  static constexpr size_t kMaxSlots = size_t(1) << 20;
  static constexpr size_t kNotVacant = ~size_t(0);
  static constexpr uint64_t kLastGeneration = ~uint64_t(0);

  void push_vacant(size_t s) {
    stack_index_[s] = vacant_.size();
    vacant_.push_back(s);
  }
  void pop_vacant(size_t s) {
    const size_t at = stack_index_[s], top = vacant_.back();
    vacant_[at] = top;
    stack_index_[top] = at;
    vacant_.pop_back();
    stack_index_[s] = kNotVacant;
  }
  void admit(uint64_t position, uint64_t charge) const {
    if (position == 0 || charge == 0)
      throw std::invalid_argument("state registry: a version needs a non-zero position and byte charge");
    if (charge > limit_ - charged_) throw std::runtime_error("state registry: byte budget would be exceeded");
  }
  StateId claim(size_t s, uint64_t position, uint64_t charge) {
    pop_vacant(s);
    gen_[s] += 1;
    pos_[s] = position;
    charge_[s] = charge;
    phase_[s] = Phase::Pending;
    charged_ += charge;
    return StateId{owner_, uint64_t(s), gen_[s], position, charge};
  }
  void vacate(size_t s) {
    charged_ -= charge_[s];
    charge_[s] = 0;
    pos_[s] = 0;
    payload_[s] = Payload{};
    phase_[s] = Phase::Vacant;
    if (gen_[s] == kLastGeneration)
      ++retired_;  // counter exhausted: the slot leaves circulation
    else
      push_vacant(s);
  }
  // The slot a handle names, if the handle is current (any non-vacant phase).
  size_t verify(const StateId& id) const {
    if (id.owner != owner_) throw std::invalid_argument("state registry: handle from another session");
    if (id.slot >= gen_.size()) throw std::invalid_argument("state registry: handle slot beyond the table");
    const size_t s = size_t(id.slot);
    if (phase_[s] == Phase::Vacant || gen_[s] != id.generation || pos_[s] != id.position ||
        charge_[s] != id.bytes)
      throw std::invalid_argument("state registry: handle no longer names a current version");
    return s;
  }
  size_t live(const StateId& id) const {
    const size_t s = verify(id);
    if (phase_[s] != Phase::Live) throw std::invalid_argument("state registry: version is reserved but not published");
    return s;
  }

  uint64_t owner_, limit_, charged_ = 0;
  size_t retired_ = 0;
  std::vector<uint64_t> gen_, pos_, charge_;
  std::vector<Phase> phase_;
  std::vector<Payload> payload_;
  std::vector<size_t> vacant_, stack_index_;
};

}  // namespace qwen
