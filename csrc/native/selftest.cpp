// Self-test of the native data plane (ColumnStore, PageAllocator) as a plain program, so it can be built
// with AddressSanitizer + UndefinedBehaviorSanitizer and with ThreadSanitizer
// (tests/test_native_sanitizers_cpu.py). Exits 0 and prints "selftest ok" on success; any failed check
// prints its line and exits 1.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "column_store.h"

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::fprintf(stderr, "selftest: check failed at line %d: %s\n", __LINE__, #c); \
      std::exit(1);                                                \
    }                                                              \
  } while (0)

using Ids = std::vector<int64_t>;

template <class E, class F>
static bool throws(F&& f) {
  try {
    f();
  } catch (const E&) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}

static void single_thread() {
  meshy::ColumnStore cs;
  Ids ids = cs.put_rows("p", {"prompt"}, {{"a", "b", "c", "d"}});
  CHECK((ids == Ids{0, 1, 2, 3}));
  // AND filter: nothing has both columns yet
  CHECK(cs.get_meta("p", {"prompt", "resp"}, 0, 0, "t", 0).empty());
  CHECK(cs.put_columns("p", {1, 3}, {"resp"}, {{"x", "y"}}) == 2);
  CHECK((cs.get_meta("p", {"prompt", "resp"}, 0, 0, "t", 0) == Ids{1, 3}));
  // consumed for task t; a peek still sees them; another task sees them
  CHECK(cs.get_meta("p", {"prompt", "resp"}, 0, 0, "t", 0).empty());
  CHECK((cs.get_meta("p", {"prompt", "resp"}, 0, 1, "t", 0) == Ids{1, 3}));
  CHECK((cs.get_meta("p", {"prompt", "resp"}, 0, 0, "u", 0) == Ids{1, 3}));
  auto d = cs.get_data("p", {3, 1}, {"resp", "prompt"});
  CHECK((d[0] == std::vector<std::string>{"y", "x"}));
  CHECK((d[1] == std::vector<std::string>{"d", "b"}));
  // batch size: exactly n rows or none
  CHECK(cs.get_meta("p", {"prompt"}, 5, 0, "v", 0).empty());
  CHECK((cs.get_meta("p", {"prompt"}, 3, 0, "v", 0) == Ids{0, 1, 2}));
  // re-delivery after a failed step
  cs.reset_consumption("p", "t", {1});
  CHECK((cs.get_meta("p", {"prompt", "resp"}, 0, 0, "t", 0) == Ids{1}));
  // status bitmask over the requested fields
  auto st = cs.status("p", {"prompt", "resp"});
  CHECK(st.size() == 4 && st[0].second == 1u && st[1].second == 3u);
  // clearing removes the rows for every task; writes to cleared rows are skipped
  CHECK(cs.clear("p", {1, 2}) == 2);
  CHECK(cs.num_rows("p") == 2);
  CHECK(cs.put_columns("p", {1, 3}, {"resp"}, {{"z", "w"}}) == 1);
  CHECK((cs.get_data("p", {3}, {"resp"})[0][0] == "w"));
  // errors
  CHECK(throws<std::out_of_range>([&] { cs.get_data("p", {1}, {"prompt"}); }));
  CHECK(throws<std::out_of_range>([&] { cs.get_data("missing", {0}, {"prompt"}); }));
  CHECK(throws<std::invalid_argument>([&] { cs.put_rows("p", {"a", "b"}, {{"1"}, {"1", "2"}}); }));
  CHECK(throws<std::invalid_argument>([&] { cs.put_columns("p", {0, 3}, {"resp"}, {{"only-one"}}); }));
  CHECK((cs.get_data("p", {0}, {"prompt"})[0][0] == "a"));  // the rejected write left row 0 untouched
  cs.clear_partition("p");
  CHECK(cs.partitions().empty());
}

// Producers append rows and later fill a second column; consumers of two tasks wait (bounded) for rows
// with both columns. Every row must reach every task exactly once.
static void threaded() {
  meshy::ColumnStore cs;
  constexpr int kProducers = 4, kRows = 200;
  std::vector<std::thread> th;
  for (int p = 0; p < kProducers; ++p) {
    th.emplace_back([&cs, p] {
      for (int i = 0; i < kRows; ++i) {
        Ids id = cs.put_rows("q", {"prompt"}, {{std::to_string(p * kRows + i)}});
        cs.put_columns("q", id, {"resp"}, {{"r" + std::to_string(p * kRows + i)}});
      }
    });
  }
  std::vector<std::vector<int64_t>> got(4);
  std::atomic<int> total[2] = {{0}, {0}};
  for (int c = 0; c < 4; ++c) {
    th.emplace_back([&, c] {
      const std::string task = c < 2 ? "train" : "critic";
      std::atomic<int>& tot = total[c < 2 ? 0 : 1];
      while (tot.load() < kProducers * kRows) {
        Ids r = cs.get_meta("q", {"prompt", "resp"}, 0, 0, task, 5);
        if (r.empty()) continue;
        auto data = cs.get_data("q", r, {"resp"});
        CHECK(data[0].size() == r.size());
        got[c].insert(got[c].end(), r.begin(), r.end());
        tot.fetch_add((int)r.size());
      }
    });
  }
  for (auto& t : th) t.join();
  for (int task = 0; task < 2; ++task) {
    std::vector<int64_t> all(got[2 * task]);
    all.insert(all.end(), got[2 * task + 1].begin(), got[2 * task + 1].end());
    std::sort(all.begin(), all.end());
    CHECK((int)all.size() == kProducers * kRows);
    for (int i = 0; i < kProducers * kRows; ++i) CHECK(all[i] == i);
  }
}

static void pages() {
  meshy::PageAllocator pa(16, 1);  // page 0 reserved
  CHECK(pa.num_free() == 15);
  auto a = pa.allocate(10);
  CHECK(a.size() == 10 && std::find(a.begin(), a.end(), 0) == a.end());
  CHECK(pa.allocate(6).empty());  // not enough: nothing taken
  CHECK(pa.num_free() == 5);
  std::vector<int32_t> shared(a.begin(), a.begin() + 3);
  pa.retain(shared);  // a shared prefix
  pa.free(a);
  CHECK(pa.num_free() == 12);  // the 3 retained pages stay allocated
  pa.free(shared);
  CHECK(pa.num_free() == 15);
  CHECK(throws<std::logic_error>([&] { pa.free({a[0]}); }));  // double free
  CHECK(throws<std::out_of_range>([&] { pa.free({99}); }));
  CHECK(throws<std::invalid_argument>([] { meshy::PageAllocator bad(4, 4); }));
}

int main() {
  single_thread();
  threaded();
  pages();
  std::printf("selftest ok\n");
  return 0;
}
