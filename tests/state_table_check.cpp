// Randomised model check of the host version registry (csrc/state_table.h),
// built and run by tests/test_state_table.py with the host C++ compiler.
//
// The registry keeps the reference's handle contract (native/state_table.h:11-38):
// a handle is usable only while its slot holds exactly that generation,
// position and byte charge; reserve charges the byte budget, publish makes the
// payload readable once, rollback frees a reserved or published version,
// release frees a published one. A plain map of live handles is the model.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <random>
#include <stdexcept>
#include <vector>

#include "../rust-ts-tokio-inference-engine_b200/csrc/state_table.h"

using qwen::StateTable;

static long checks = 0;
#define CHECK(cond)                                                   \
  do {                                                                \
    ++checks;                                                         \
    if (!(cond)) {                                                    \
      std::fprintf(stderr, "FAIL line %d: %s\n", __LINE__, #cond);    \
      std::exit(1);                                                   \
    }                                                                 \
  } while (0)

template <class F>
static bool throws(F f) {
  try {
    f();
  } catch (const std::exception&) {
    return true;
  }
  return false;
}

struct Known {
  StateId id;
  bool published;
  int payload;
};

static bool same(const StateId& a, const StateId& b) {
  return a.owner == b.owner && a.slot == b.slot && a.generation == b.generation && a.position == b.position &&
         a.bytes == b.bytes;
}

int main(int argc, char** argv) {
  const unsigned seed = argc > 1 ? unsigned(std::atoi(argv[1])) : 1u;
  // construction bounds
  CHECK(throws([] { StateTable<int>(0, 4, 100); }));
  CHECK(throws([] { StateTable<int>(3, 0, 100); }));
  CHECK(throws([] { StateTable<int>(3, (size_t(1) << 20) + 1, 100); }));
  CHECK(throws([] { StateTable<int>(3, 4, 0); }));

  // directed cases
  {
    StateTable<int> t(7, 2, 100);
    CHECK(throws([&] { t.reserve(0, 10); }));   // position 0 is the empty state, never a version
    CHECK(throws([&] { t.reserve(1, 0); }));    // zero charge
    CHECK(throws([&] { t.reserve(1, 101); }));  // over budget
    StateId a = t.reserve(5, 60);
    CHECK(a.owner == 7 && a.slot == 0 && a.generation == 1 && a.position == 5 && a.bytes == 60);
    CHECK(t.bytes() == 60 && t.residents() == 1);
    CHECK(throws([&] { t.get(a); }));     // reserved, not published
    CHECK(throws([&] { t.release(a); }));  // release needs a published version
    CHECK(throws([&] { t.reserve(1, 41); }));
    t.publish(a, 11);
    CHECK(throws([&] { t.publish(a, 12); }));
    CHECK(t.get(a) == 11);
    StateId b = t.reserve(9, 40);
    CHECK(b.slot == 1);
    CHECK(throws([&] { t.reserve(1, 1); }));  // slots exhausted (and budget)
    StateId forged = a;
    forged.owner = 8;
    CHECK(throws([&] { t.get(forged); }));
    forged = a;
    forged.position = 6;
    CHECK(throws([&] { t.get(forged); }));
    forged = a;
    forged.bytes = 61;
    CHECK(throws([&] { t.get(forged); }));
    forged = a;
    forged.slot = 2;
    CHECK(throws([&] { t.get(forged); }));
    t.release(a);
    CHECK(throws([&] { t.get(a); }));
    CHECK(throws([&] { t.rollback(a); }));
    CHECK(t.bytes() == 40 && t.residents() == 1);
    // the consume-in-place path: release the parent, then claim its slot
    CHECK(throws([&] { t.reserve_at(1, 3, 10); }));  // occupied
    CHECK(throws([&] { t.reserve_at(2, 3, 10); }));  // beyond the table
    StateId c = t.reserve_at(0, 6, 30);
    CHECK(c.slot == 0 && c.generation == 2);
    t.rollback(b);  // a pending version can be rolled back
    CHECK(t.bytes() == 30 && t.residents() == 1);
    t.publish(c, 5);
    int seen = 0;
    t.for_each_published([&](size_t slot, int& v) {
      CHECK(slot == 0 && v == 5);
      ++seen;
    });
    CHECK(seen == 1);
    t.get_mut(c) = 6;
    CHECK(t.get(c) == 6);
    t.clear();
    CHECK(t.bytes() == 0 && t.residents() == 0);
    CHECK(throws([&] { t.get(c); }));
    StateId d = t.reserve(1, 1);
    CHECK(d.generation >= 2);
  }

  // randomised run against the model
  std::mt19937_64 rng(seed);
  for (int round = 0; round < 40; ++round) {
    const size_t slots = 1 + rng() % 24;
    const uint64_t limit = 1 + rng() % 400;
    StateTable<int> t(2 * round + 1, slots, limit);
    std::vector<Known> live;
    std::vector<StateId> dead;
    uint64_t used = 0;
    for (int op = 0; op < 3000; ++op) {
      const int kind = int(rng() % 7);
      if (kind <= 1) {
        const uint64_t pos = 1 + rng() % 50, charge = 1 + rng() % 60;
        const bool fits = charge <= limit - used && live.size() < slots;
        StateId id{};
        const bool threw = throws([&] { id = t.reserve(pos, charge); });
        CHECK(threw == !fits);
        if (!threw) {
          CHECK(id.position == pos && id.bytes == charge && id.slot < slots);
          for (auto& k : live) CHECK(k.id.slot != id.slot);
          used += charge;
          live.push_back({id, false, 0});
        }
      } else if (kind == 2 && !live.empty()) {
        auto& k = live[rng() % live.size()];
        const int v = int(rng() % 1000);
        const bool threw = throws([&] { t.publish(k.id, v); });
        CHECK(threw == k.published);
        if (!threw) {
          k.published = true;
          k.payload = v;
        }
      } else if (kind == 3 && !live.empty()) {
        const size_t i = rng() % live.size();
        const bool threw = throws([&] { t.release(live[i].id); });
        CHECK(threw == !live[i].published);
        if (!threw) {
          used -= live[i].id.bytes;
          dead.push_back(live[i].id);
          live.erase(live.begin() + i);
        }
      } else if (kind == 4 && !live.empty()) {
        const size_t i = rng() % live.size();
        t.rollback(live[i].id);
        used -= live[i].id.bytes;
        dead.push_back(live[i].id);
        live.erase(live.begin() + i);
      } else if (kind == 5 && !dead.empty()) {
        const StateId& id = dead[rng() % dead.size()];
        bool reissued = false;  // a dead handle may never alias a current one
        for (auto& k : live) reissued |= same(k.id, id);
        CHECK(!reissued);
        CHECK(throws([&] { t.get(id); }));
        CHECK(throws([&] { t.rollback(id); }));
      } else if (kind == 6 && !live.empty()) {
        // consume in place: release a published version and claim its slot
        const size_t i = rng() % live.size();
        if (live[i].published) {
          const StateId parent = live[i].id;
          t.release(parent);
          used -= parent.bytes;
          dead.push_back(parent);
          live.erase(live.begin() + i);
          const uint64_t charge = 1 + rng() % 60;
          StateId id{};
          const bool fits = charge <= limit - used;
          const bool threw = throws([&] { id = t.reserve_at(parent.slot, parent.position + 1, charge); });
          CHECK(threw == !fits);
          if (!threw) {
            CHECK(id.slot == parent.slot && id.generation == parent.generation + 1);
            used += charge;
            live.push_back({id, false, 0});
          }
        }
      }
      CHECK(t.bytes() == used);
      CHECK(t.residents() == live.size());
      for (auto& k : live)
        if (k.published) CHECK(t.get(k.id) == k.payload);
    }
  }
  std::printf("PASS state registry checks=%ld\n", checks);
  return 0;
}
