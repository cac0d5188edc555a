#include "column_store.h"

#include <chrono>
#include <algorithm>
#include <stdexcept>

namespace meshy {

std::vector<int64_t> ColumnStore::put_rows(const std::string& part, const std::vector<std::string>& fields,
                                           const std::vector<std::vector<std::string>>& values) {
  if (values.size() != fields.size()) throw std::invalid_argument("put_rows: one value list per field");
  size_t n = fields.empty() ? 0 : values[0].size();
  for (auto& v : values)
    if (v.size() != n) throw std::invalid_argument("put_rows: ragged column lengths");
  std::vector<int64_t> out;
  out.reserve(n);
  {
    std::lock_guard<std::mutex> g(mu_);
    Partition& p = parts_[part];
    for (size_t r = 0; r < n; ++r) {
      int64_t id = p.next++;
      Row& row = p.rows[id];
      for (size_t f = 0; f < fields.size(); ++f) row.cols[fields[f]] = values[f][r];
      out.push_back(id);
    }
  }
  cv_.notify_all();
  return out;
}

int64_t ColumnStore::put_columns(const std::string& part, const std::vector<int64_t>& idx,
                                 const std::vector<std::string>& fields,
                                 const std::vector<std::vector<std::string>>& values) {
  if (values.size() != fields.size()) throw std::invalid_argument("put_columns: one value list per field");
  for (auto& v : values)  // validate before writing anything
    if (v.size() != idx.size()) throw std::invalid_argument("put_columns: length mismatch");
  int64_t written = 0;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = parts_.find(part);
    if (it == parts_.end()) return 0;
    Partition& p = it->second;
    for (size_t r = 0; r < idx.size(); ++r) {
      auto rit = p.rows.find(idx[r]);
      if (rit == p.rows.end()) continue;
      for (size_t f = 0; f < fields.size(); ++f) rit->second.cols[fields[f]] = values[f][r];
      ++written;
    }
  }
  cv_.notify_all();
  return written;
}

std::vector<int64_t> ColumnStore::ready_locked(Partition& p, const std::vector<std::string>& fields, int mode,
                                               const std::string& task, int64_t limit) {
  std::vector<int64_t> out;
  auto cit = p.consumed.find(task);
  const std::unordered_set<int64_t>* used = (mode == 0 && cit != p.consumed.end()) ? &cit->second : nullptr;
  for (auto& kv : p.rows) {
    if (used && used->count(kv.first)) continue;
    bool ok = true;
    for (auto& f : fields)
      if (!kv.second.cols.count(f)) {
        ok = false;
        break;
      }
    if (!ok) continue;
    out.push_back(kv.first);
    if (limit > 0 && (int64_t)out.size() >= limit) break;
  }
  return out;
}

std::vector<int64_t> ColumnStore::get_meta(const std::string& part, const std::vector<std::string>& fields,
                                           int64_t batch_size, int mode, const std::string& task, int64_t wait_ms) {
  std::unique_lock<std::mutex> lk(mu_);
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(std::max<int64_t>(0, wait_ms));
  while (true) {
    auto it = parts_.find(part);
    if (it != parts_.end()) {
      Partition& p = it->second;
      std::vector<int64_t> r = ready_locked(p, fields, mode, task, batch_size);
      bool enough = batch_size <= 0 ? !r.empty() : (int64_t)r.size() >= batch_size;
      if (enough) {
        if (mode == 0) {
          auto& used = p.consumed[task];
          for (auto i : r) used.insert(i);
        }
        return r;
      }
    }
    if (wait_ms <= 0 || cv_.wait_until(lk, deadline) == std::cv_status::timeout) {
      // one last check after the timeout
      auto it2 = parts_.find(part);
      if (it2 == parts_.end()) return {};
      std::vector<int64_t> r = ready_locked(it2->second, fields, mode, task, batch_size);
      bool enough = batch_size <= 0 ? !r.empty() : (int64_t)r.size() >= batch_size;
      if (!enough) return {};
      if (mode == 0) {
        auto& used = it2->second.consumed[task];
        for (auto i : r) used.insert(i);
      }
      return r;
    }
  }
}

std::vector<std::vector<std::string>> ColumnStore::get_data(const std::string& part, const std::vector<int64_t>& idx,
                                                            const std::vector<std::string>& fields) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<std::vector<std::string>> out(fields.size(), std::vector<std::string>(idx.size()));
  auto it = parts_.find(part);
  if (it == parts_.end()) throw std::out_of_range("partition not found: " + part);
  for (size_t r = 0; r < idx.size(); ++r) {
    auto rit = it->second.rows.find(idx[r]);
    if (rit == it->second.rows.end()) throw std::out_of_range("row " + std::to_string(idx[r]) + " not found");
    for (size_t f = 0; f < fields.size(); ++f) {
      auto c = rit->second.cols.find(fields[f]);
      if (c == rit->second.cols.end()) throw std::out_of_range("column " + fields[f] + " not produced");
      out[f][r] = c->second;
    }
  }
  return out;
}

int64_t ColumnStore::clear(const std::string& part, const std::vector<int64_t>& idx) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = parts_.find(part);
  if (it == parts_.end()) return 0;
  int64_t n = 0;
  for (auto i : idx) {
    n += (int64_t)it->second.rows.erase(i);
    for (auto& kv : it->second.consumed) kv.second.erase(i);
  }
  return n;
}

void ColumnStore::clear_partition(const std::string& part) {
  std::lock_guard<std::mutex> g(mu_);
  parts_.erase(part);
}

void ColumnStore::reset_consumption(const std::string& part, const std::string& task, const std::vector<int64_t>& idx) {
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = parts_.find(part);
    if (it == parts_.end()) return;
    auto c = it->second.consumed.find(task);
    if (c == it->second.consumed.end()) return;
    for (auto i : idx) c->second.erase(i);
  }
  cv_.notify_all();
}

std::vector<std::string> ColumnStore::partitions() {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<std::string> out;
  for (auto& kv : parts_) out.push_back(kv.first);
  return out;
}

int64_t ColumnStore::num_rows(const std::string& part) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = parts_.find(part);
  return it == parts_.end() ? 0 : (int64_t)it->second.rows.size();
}

std::vector<std::pair<int64_t, uint64_t>> ColumnStore::status(const std::string& part,
                                                              const std::vector<std::string>& fields) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<std::pair<int64_t, uint64_t>> out;
  auto it = parts_.find(part);
  if (it == parts_.end()) return out;
  for (auto& kv : it->second.rows) {
    uint64_t m = 0;
    for (size_t f = 0; f < fields.size() && f < 64; ++f)
      if (kv.second.cols.count(fields[f])) m |= (1ull << f);
    out.emplace_back(kv.first, m);
  }
  return out;
}

// ─── pages ────────────────────────────────────────────────────────────────
PageAllocator::PageAllocator(int64_t n_pages, int64_t reserved) : n_(n_pages), refs_(n_pages, 0) {
  if (reserved < 0 || reserved >= n_pages) throw std::invalid_argument("PageAllocator: bad reserved count");
  free_.reserve(n_pages);
  for (int64_t i = n_pages - 1; i >= reserved; --i) free_.push_back((int32_t)i);
  for (int64_t i = 0; i < reserved; ++i) refs_[i] = 1;
}

std::vector<int32_t> PageAllocator::allocate(int64_t n) {
  if (n <= 0) return {};
  if (n > (int64_t)free_.size()) return {};
  std::vector<int32_t> out(free_.end() - n, free_.end());
  free_.resize(free_.size() - n);
  std::reverse(out.begin(), out.end());
  for (auto p : out) refs_[p] = 1;
  return out;
}

void PageAllocator::retain(const std::vector<int32_t>& pages) {
  for (auto p : pages) refs_.at(p) += 1;
}

void PageAllocator::free(const std::vector<int32_t>& pages) {
  for (auto it = pages.rbegin(); it != pages.rend(); ++it) {
    int32_t p = *it;
    if (p < 0 || p >= n_) throw std::out_of_range("PageAllocator::free: bad page id");
    if (refs_[p] <= 0) throw std::logic_error("PageAllocator::free: double free of page " + std::to_string(p));
    if (--refs_[p] == 0) free_.push_back(p);
  }
}

}  // namespace meshy
