// Test infrastructure, not product code, and not CRoaring.
//
// The reference's engine layer (planner, metadata columns, segments) includes "roaring.hh" from
// CRoaring v4.2.1 (cmake/Dependencies.cmake:16-26), which is not available here. This header is a
// stand-in with the same set semantics for the subset of roaring::Roaring the engine calls: a
// sorted vector of distinct uint32 values. Filter bitmaps, intersections, differences and
// iteration order are therefore identical to CRoaring's. write/readSafe (delete files) use CRoaring's
// portable serialization; the choice between container kinds follows its size rule.
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
  bool runOptimize() {
    run_optimized_ = true;
    for (const Container& c : Containers())
      if (c.kind == kRun) return true;
    return false;
  }
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

  // CRoaring's portable serialization (RoaringFormatSpec): a cookie, the container keys and
  // cardinalities, container offsets, then array (u16 values), bitmap (1024 u64 words) or, after
  // runOptimize(), run containers (u16 count, then start / length-1 pairs) where they are smaller.
  size_t getSizeInBytes(bool = true) const { return Serialize(nullptr); }
  size_t write(char* buf, bool = true) const { return Serialize(buf); }
  static Roaring readSafe(const char* buf, size_t maxbytes) {
    Roaring r;
    size_t at = 0;
    auto need = [&](size_t n) {
      if (maxbytes - at < n || at > maxbytes) throw std::runtime_error("bad bitmap");
    };
    auto u16 = [&]() { need(2); uint16_t x; std::memcpy(&x, buf + at, 2); at += 2; return x; };
    auto u32 = [&]() { need(4); uint32_t x; std::memcpy(&x, buf + at, 4); at += 4; return x; };
    const uint32_t cookie = u32();
    uint32_t size = 0;
    bool runs = false;
    std::vector<uint8_t> runbits;
    if ((cookie & 0xFFFFu) == kCookieRuns) {
      runs = true;
      size = (cookie >> 16) + 1;
      need((size + 7) / 8);
      runbits.assign(buf + at, buf + at + (size + 7) / 8);
      at += (size + 7) / 8;
    } else if (cookie == kCookieNoRuns) {
      size = u32();
    } else {
      throw std::runtime_error("bad bitmap cookie");
    }
    if (size > 65536) throw std::runtime_error("bad bitmap");
    std::vector<uint16_t> keys(size);
    std::vector<uint32_t> cards(size);
    for (uint32_t i = 0; i < size; ++i) {
      keys[i] = u16();
      cards[i] = static_cast<uint32_t>(u16()) + 1;
    }
    if (!runs || size >= kNoOffsetThreshold) {
      need(4 * static_cast<size_t>(size));
      at += 4 * static_cast<size_t>(size);
    }
    for (uint32_t i = 0; i < size; ++i) {
      const uint32_t hi = static_cast<uint32_t>(keys[i]) << 16;
      if (runs && (runbits[i / 8] >> (i % 8) & 1)) {
        const uint16_t nr = u16();
        for (uint16_t k = 0; k < nr; ++k) {
          const uint32_t st = u16(), len = u16();
          for (uint32_t x = st; x <= st + len; ++x) r.v_.push_back(hi | (x & 0xFFFFu));
        }
      } else if (cards[i] > kArrayMax) {
        need(8192);
        for (uint32_t w = 0; w < 1024; ++w) {
          uint64_t word;
          std::memcpy(&word, buf + at + 8 * w, 8);
          for (uint32_t b = 0; b < 64; ++b)
            if (word >> b & 1) r.v_.push_back(hi | (w * 64 + b));
        }
        at += 8192;
      } else {
        for (uint32_t k = 0; k < cards[i]; ++k) r.v_.push_back(hi | u16());
      }
    }
    std::sort(r.v_.begin(), r.v_.end());
    r.v_.erase(std::unique(r.v_.begin(), r.v_.end()), r.v_.end());
    return r;
  }

  using const_iterator = std::vector<uint32_t>::const_iterator;
  const_iterator begin() const { return v_.begin(); }
  const_iterator end() const { return v_.end(); }

 private:
  static constexpr uint32_t kCookieNoRuns = 12346, kCookieRuns = 12347, kNoOffsetThreshold = 4;
  static constexpr uint32_t kArrayMax = 4096;
  enum Kind { kArray, kBitmap, kRun };
  struct Container {
    uint16_t key;
    size_t begin, end;  // range of v_
    uint32_t nruns;
    Kind kind;
  };
  // Container kinds as CRoaring picks them: an array up to 4096 values, else a bitmap; after
  // runOptimize(), a run container where its serialized size is smaller.
  std::vector<Container> Containers() const {
    std::vector<Container> out;
    for (size_t i = 0; i < v_.size();) {
      size_t j = i;
      uint32_t nruns = 0;
      while (j < v_.size() && (v_[j] >> 16) == (v_[i] >> 16)) {
        if (j == i || v_[j] != v_[j - 1] + 1) ++nruns;
        ++j;
      }
      const size_t card = j - i;
      Kind kind = card > kArrayMax ? kBitmap : kArray;
      const size_t as_run = 2 + 4 * static_cast<size_t>(nruns);
      const size_t as_base = kind == kBitmap ? 8192 : 2 + 2 * card;
      if (run_optimized_ && as_run < as_base) kind = kRun;
      out.push_back({static_cast<uint16_t>(v_[i] >> 16), i, j, nruns, kind});
      i = j;
    }
    return out;
  }
  size_t Serialize(char* buf) const {
    const std::vector<Container> cs = Containers();
    const size_t n = cs.size();
    bool runs = false;
    for (const Container& c : cs) runs |= c.kind == kRun;
    size_t at = 0;
    auto put = [&](const void* p, size_t len) {
      if (buf != nullptr) std::memcpy(buf + at, p, len);
      at += len;
    };
    auto put16 = [&](uint32_t x) { const uint16_t y = static_cast<uint16_t>(x); put(&y, 2); };
    auto put32 = [&](uint32_t x) { put(&x, 4); };
    if (runs) {
      put32(kCookieRuns | static_cast<uint32_t>(n - 1) << 16);
      std::vector<uint8_t> bits((n + 7) / 8, 0);
      for (size_t i = 0; i < n; ++i)
        if (cs[i].kind == kRun) bits[i / 8] |= static_cast<uint8_t>(1u << (i % 8));
      put(bits.data(), bits.size());
    } else {
      put32(kCookieNoRuns);
      put32(static_cast<uint32_t>(n));
    }
    for (const Container& c : cs) {
      put16(c.key);
      put16(static_cast<uint32_t>(c.end - c.begin - 1));
    }
    auto body = [&](const Container& c) -> size_t {
      if (c.kind == kRun) return 2 + 4 * static_cast<size_t>(c.nruns);
      if (c.kind == kBitmap) return 8192;
      return 2 * (c.end - c.begin);
    };
    if (!runs || n >= kNoOffsetThreshold) {
      size_t off = at + 4 * n;
      for (const Container& c : cs) {
        put32(static_cast<uint32_t>(off));
        off += body(c);
      }
    }
    for (const Container& c : cs) {
      if (c.kind == kRun) {
        put16(c.nruns);
        for (size_t i = c.begin; i < c.end;) {
          size_t j = i + 1;
          while (j < c.end && v_[j] == v_[j - 1] + 1) ++j;
          put16(v_[i] & 0xFFFFu);
          put16(static_cast<uint32_t>(j - i - 1));
          i = j;
        }
      } else if (c.kind == kBitmap) {
        std::vector<uint64_t> words(1024, 0);
        for (size_t i = c.begin; i < c.end; ++i) words[(v_[i] & 0xFFFFu) / 64] |= 1ull << (v_[i] % 64);
        put(words.data(), 8192);
      } else {
        for (size_t i = c.begin; i < c.end; ++i) put16(v_[i] & 0xFFFFu);
      }
    }
    return at;
  }

  std::vector<uint32_t> v_;
  bool run_optimized_ = false;
};

}  // namespace roaring
