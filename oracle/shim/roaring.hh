// Test infrastructure, not product code, and not CRoaring.
//
// The reference's engine layer (planner, metadata columns, segments) includes "roaring.hh" from
// CRoaring v4.2.1 (cmake/Dependencies.cmake:16-26), which is not available here. This header is a
// stand-in with the same set semantics for the subset of roaring::Roaring the engine calls: a
// sorted vector of distinct uint32 values. Filter bitmaps, intersections, differences and
// iteration order are therefore identical to CRoaring's. Only the serialized byte format
// (write/readSafe, used for delete files) is our own; the engine never compares it with CRoaring's.
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <iterator>
#include <stdexcept>
#include <vector>

namespace roaring {

class Roaring {
 public:
  Roaring() = default;

  void add(uint32_t x) {
    auto it = std::lower_bound(v_.begin(), v_.end(), x);
    if (it == v_.end() || *it != x) v_.insert(it, x);
  }
  void addMany(size_t n, const uint32_t* xs) {
    std::vector<uint32_t> add(xs, xs + n);
    std::sort(add.begin(), add.end());
    add.erase(std::unique(add.begin(), add.end()), add.end());
    std::vector<uint32_t> out;
    out.reserve(v_.size() + add.size());
    std::set_union(v_.begin(), v_.end(), add.begin(), add.end(), std::back_inserter(out));
    v_.swap(out);
  }
  // [lo, hi), as CRoaring's C++ addRange.
  void addRange(uint64_t lo, uint64_t hi) {
    std::vector<uint32_t> add;
    for (uint64_t x = lo; x < hi; ++x) add.push_back(static_cast<uint32_t>(x));
    addMany(add.size(), add.data());
  }
  bool contains(uint32_t x) const { return std::binary_search(v_.begin(), v_.end(), x); }
  uint64_t cardinality() const { return v_.size(); }
  bool isEmpty() const { return v_.empty(); }
  uint32_t maximum() const { return v_.empty() ? 0 : v_.back(); }
  uint32_t minimum() const { return v_.empty() ? UINT32_MAX : v_.front(); }
  bool runOptimize() { return false; }
  void shrinkToFit() { v_.shrink_to_fit(); }

  Roaring& operator&=(const Roaring& o) {
    std::vector<uint32_t> out;
    std::set_intersection(v_.begin(), v_.end(), o.v_.begin(), o.v_.end(), std::back_inserter(out));
    v_.swap(out);
    return *this;
  }
  Roaring& operator|=(const Roaring& o) {
    std::vector<uint32_t> out;
    out.reserve(v_.size() + o.v_.size());
    std::set_union(v_.begin(), v_.end(), o.v_.begin(), o.v_.end(), std::back_inserter(out));
    v_.swap(out);
    return *this;
  }
  Roaring& operator-=(const Roaring& o) {
    std::vector<uint32_t> out;
    std::set_difference(v_.begin(), v_.end(), o.v_.begin(), o.v_.end(), std::back_inserter(out));
    v_.swap(out);
    return *this;
  }
  Roaring operator&(const Roaring& o) const { Roaring r = *this; r &= o; return r; }
  Roaring operator|(const Roaring& o) const { Roaring r = *this; r |= o; return r; }
  Roaring operator-(const Roaring& o) const { Roaring r = *this; r -= o; return r; }
  bool operator==(const Roaring& o) const { return v_ == o.v_; }

  // Own portable format: u32 count, then the values (little-endian).
  size_t getSizeInBytes(bool = true) const { return 4 + 4 * v_.size(); }
  size_t write(char* buf, bool = true) const {
    const uint32_t n = static_cast<uint32_t>(v_.size());
    std::memcpy(buf, &n, 4);
    if (n > 0) std::memcpy(buf + 4, v_.data(), 4 * v_.size());
    return getSizeInBytes();
  }
  static Roaring readSafe(const char* buf, size_t maxbytes) {
    Roaring r;
    if (maxbytes < 4) throw std::runtime_error("bad bitmap");
    uint32_t n = 0;
    std::memcpy(&n, buf, 4);
    if (4 + 4 * static_cast<size_t>(n) > maxbytes) throw std::runtime_error("bad bitmap");
    r.v_.resize(n);
    if (n > 0) std::memcpy(r.v_.data(), buf + 4, 4 * static_cast<size_t>(n));
    return r;
  }

  using const_iterator = std::vector<uint32_t>::const_iterator;
  const_iterator begin() const { return v_.begin(); }
  const_iterator end() const { return v_.end(); }

 private:
  std::vector<uint32_t> v_;
};

}  // namespace roaring
