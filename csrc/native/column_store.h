// In-memory column store with TransferQueue semantics (C++ core of the data plane).
//
// A partition holds rows addressed by a monotonically increasing global index.
// Each row stores any subset of named columns as opaque byte blobs (the Python
// layer encodes tensors as dtype/shape header + raw bytes).  A consumer
// fetches rows on which *every* requested column has been produced (AND
// filter) and that its task has not consumed yet; ``fetch`` marks them
// consumed for that task, ``force_fetch`` only peeks.  Clearing a row removes
// it for every task.  All operations are thread-safe; ``get_meta`` can block
// (bounded) until enough rows are ready.
#pragma once
#include <condition_variable>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace meshy {

class ColumnStore {
 public:
  // Append rows: values[f][r] is column fields[f] of new row r.  Returns indexes.
  std::vector<int64_t> put_rows(const std::string& part, const std::vector<std::string>& fields,
                                const std::vector<std::vector<std::string>>& values);
  // Write columns onto existing rows (rows that were cleared meanwhile are skipped).
  int64_t put_columns(const std::string& part, const std::vector<int64_t>& idx, const std::vector<std::string>& fields,
                      const std::vector<std::vector<std::string>>& values);
  // mode: 0 fetch (mark consumed for task), 1 force_fetch (peek), 2 insert-order peek of all rows.
  // batch_size <= 0: every ready row; otherwise exactly batch_size rows or none.
  // wait_ms > 0 blocks up to that long for the rows to become ready.
  std::vector<int64_t> get_meta(const std::string& part, const std::vector<std::string>& fields, int64_t batch_size,
                                int mode, const std::string& task, int64_t wait_ms);
  std::vector<std::vector<std::string>> get_data(const std::string& part, const std::vector<int64_t>& idx,
                                                 const std::vector<std::string>& fields);
  int64_t clear(const std::string& part, const std::vector<int64_t>& idx);
  void clear_partition(const std::string& part);
  // Forget that ``task`` consumed these rows (used to re-deliver after a failed step).
  void reset_consumption(const std::string& part, const std::string& task, const std::vector<int64_t>& idx);
  std::vector<std::string> partitions();
  int64_t num_rows(const std::string& part);
  // production status: for each row (ordered), a bitmask over ``fields``
  std::vector<std::pair<int64_t, uint64_t>> status(const std::string& part, const std::vector<std::string>& fields);

 private:
  struct Row {
    std::unordered_map<std::string, std::string> cols;
  };
  struct Partition {
    int64_t next = 0;
    std::map<int64_t, Row> rows;
    std::unordered_map<std::string, std::unordered_set<int64_t>> consumed;
  };
  std::vector<int64_t> ready_locked(Partition& p, const std::vector<std::string>& fields, int mode,
                                    const std::string& task, int64_t limit);
  std::mutex mu_;
  std::condition_variable cv_;
  std::unordered_map<std::string, Partition> parts_;
};

// Fixed-size KV page allocator with reference counts (shared prefixes).
class PageAllocator {
 public:
  PageAllocator(int64_t n_pages, int64_t reserved);
  // Returns n page ids or an empty vector if not enough free pages.
  std::vector<int32_t> allocate(int64_t n);
  void free(const std::vector<int32_t>& pages);
  void retain(const std::vector<int32_t>& pages);
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_pages() const { return n_; }

 private:
  int64_t n_;
  std::vector<int32_t> free_;
  std::vector<int32_t> refs_;
};

}  // namespace meshy
