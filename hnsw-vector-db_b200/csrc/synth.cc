// Seeded synthetic workloads for tests and bench.py (harness, not part of the search path).
//
// The reference measures on public ANN datasets that are not available here, so every workload
// is a Gaussian mixture with the shapes, sizes and value distributions of the benchmark configs:
//   flat / HNSW (integer): centres U[0,100]^d, sigma 10, clipped to [0,255], rounded
//   SQ8 cosine:            centres N(0,1)^d, sigma 0.3, then L2-normalised
//   IVF-PQ:                centres U[-1,1]^d, sigma 0.15
//   sharded cosine:        centres U[0,100]^d, sigma 10 (no rounding), then L2-normalised
// Generation is deterministic in (seed, stream) and independent of the thread count: rows are
// produced in fixed chunks, each from its own std::mt19937_64 seeded by SplitMix64(seed, stream,
// chunk). Normalisation restates vdb's NormalizeVector (src/util/dataset.cc:33-40): a double sum
// of squares and a float inverse norm, so rows match what the reference would ingest.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <string>
#include <vector>

namespace {

uint64_t Mix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

constexpr uint64_t kChunk = 16384;

bool Normalize(float* v, size_t dim) {
  double norm = 0;
  for (size_t i = 0; i < dim; ++i) norm += static_cast<double>(v[i]) * v[i];
  if (!(norm > 0) || !std::isfinite(norm)) return false;
  auto inv = static_cast<float>(1.0 / std::sqrt(norm));
  for (size_t i = 0; i < dim; ++i) v[i] *= inv;
  return true;
}

template <class F>
void ParallelChunks(uint64_t nchunks, int threads, F fn) {
  if (threads <= 0) threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  if (threads == 1 || nchunks <= 1) {
    for (uint64_t c = 0; c < nchunks; ++c) fn(c);
    return;
  }
  std::vector<std::thread> ts;
  for (int t = 0; t < threads; ++t)
    ts.emplace_back([&, t] {
      for (uint64_t c = static_cast<uint64_t>(t); c < nchunks; c += static_cast<uint64_t>(threads)) fn(c);
    });
  for (auto& th : ts) th.join();
}

}  // namespace

extern "C" {

// centre_kind: 0 = U[c_lo, c_hi], 1 = N(0, 1). flags: bit 0 = clip to [0,255] and round to the
// nearest integer, bit 1 = L2-normalise. Writes n rows of pd floats (zero padding after dim).
void synth_mixture(uint64_t n, uint32_t dim, uint32_t pd, uint32_t ncentres, int centre_kind,
                   float c_lo, float c_hi, float sigma, int flags, uint64_t seed, uint64_t stream,
                   float* out, int threads) {
  std::vector<float> centres(static_cast<size_t>(ncentres) * dim);
  {
    std::mt19937_64 crng(Mix(seed ^ 0x5EEDC0DEull));
    std::uniform_real_distribution<float> u(c_lo, c_hi);
    std::normal_distribution<float> g(0.f, 1.f);
    for (auto& c : centres) c = centre_kind == 0 ? u(crng) : g(crng);
  }
  const uint64_t nchunks = (n + kChunk - 1) / kChunk;
  ParallelChunks(nchunks, threads, [&](uint64_t chunk) {
    std::mt19937_64 rng(Mix(Mix(seed) ^ Mix(stream + 1) ^ Mix(chunk + 0x1000)));
    std::uniform_int_distribution<uint32_t> pick(0, ncentres - 1);
    std::normal_distribution<float> g(0.f, 1.f);
    const uint64_t b = chunk * kChunk, e = std::min(n, b + kChunk);
    for (uint64_t i = b; i < e; ++i) {
      float* row = out + i * pd;
      const float* c = centres.data() + static_cast<size_t>(pick(rng)) * dim;
      for (uint32_t d = 0; d < dim; ++d) {
        float x = c[d] + sigma * g(rng);
        if (flags & 1) x = std::nearbyint(std::min(255.f, std::max(0.f, x)));
        row[d] = x;
      }
      for (uint32_t d = dim; d < pd; ++d) row[d] = 0.f;
      if (flags & 2) Normalize(row, dim);
    }
  });
}

// Per-row metadata for the sharded filtered workload: year ~ U{year_lo..year_hi}; 1..max_tags
// tags per row, each drawn Zipf(s) over vocab words (word ids 0..vocab-1, rank 1 = id 0).
// tags_out holds max_tags slots per row (unused slots = UINT32_MAX); duplicates are kept as
// drawn (a keyword list may repeat a word; its postings collapse them).
void synth_metadata(uint64_t n, int64_t year_lo, int64_t year_hi, uint32_t max_tags,
                    uint32_t vocab, double zipf_s, uint64_t seed, int64_t* year_out,
                    uint32_t* tags_out, int threads) {
  std::vector<double> cdf(vocab);
  double acc = 0;
  for (uint32_t r = 0; r < vocab; ++r) {
    acc += 1.0 / std::pow(static_cast<double>(r + 1), zipf_s);
    cdf[r] = acc;
  }
  for (auto& c : cdf) c /= acc;
  const uint64_t nchunks = (n + kChunk - 1) / kChunk;
  ParallelChunks(nchunks, threads, [&](uint64_t chunk) {
    std::mt19937_64 rng(Mix(Mix(seed ^ 0xA11CEull) ^ Mix(chunk + 7)));
    std::uniform_int_distribution<int64_t> year(year_lo, year_hi);
    std::uniform_int_distribution<uint32_t> ntags(1, max_tags);
    std::uniform_real_distribution<double> u(0.0, 1.0);
    const uint64_t b = chunk * kChunk, e = std::min(n, b + kChunk);
    for (uint64_t i = b; i < e; ++i) {
      year_out[i] = year(rng);
      uint32_t t = ntags(rng);
      for (uint32_t j = 0; j < max_tags; ++j) {
        uint32_t w = UINT32_MAX;
        if (j < t) {
          double x = u(rng);
          w = static_cast<uint32_t>(std::lower_bound(cdf.begin(), cdf.end(), x) - cdf.begin());
          if (w >= vocab) w = vocab - 1;
        }
        tags_out[i * max_tags + j] = w;
      }
    }
  });
}

// Zipf-drawn query tags (same law as synth_metadata).
void synth_zipf(uint64_t n, uint32_t vocab, double zipf_s, uint64_t seed, uint32_t* out) {
  std::vector<double> cdf(vocab);
  double acc = 0;
  for (uint32_t r = 0; r < vocab; ++r) {
    acc += 1.0 / std::pow(static_cast<double>(r + 1), zipf_s);
    cdf[r] = acc;
  }
  for (auto& c : cdf) c /= acc;
  std::mt19937_64 rng(Mix(seed ^ 0x21FFull));
  std::uniform_real_distribution<double> u(0.0, 1.0);
  for (uint64_t i = 0; i < n; ++i) {
    auto w = static_cast<uint32_t>(std::lower_bound(cdf.begin(), cdf.end(), u(rng)) - cdf.begin());
    out[i] = w >= vocab ? vocab - 1 : w;
  }
}

// The payload of a segment's meta.bin (SegmentWriter, src/storage/segment_writer.cc:103-120) for
// the schema [year int64, tags keyword_list]: u64 rows, u64 offsets[rows + 1], then every row as
// EncodeMetaRow writes it (src/meta/schema.cc:97-124) with the tags as keywords "w<id>" in drawn
// order (unused slots = UINT32_MAX skipped). Returns the payload size; writes only when it fits
// in cap (out may be null to size it).
uint64_t synth_meta_payload(uint64_t n, const int64_t* years, const uint32_t* tags, uint32_t max_tags,
                            uint8_t* out, uint64_t cap) {
  auto row_bytes = [&](uint64_t i) {
    uint64_t b = 2 + (2 + 1 + 8) + (2 + 1 + 4);
    for (uint32_t j = 0; j < max_tags; ++j) {
      const uint32_t w = tags[i * max_tags + j];
      if (w == UINT32_MAX) continue;
      b += 4 + 1 + std::to_string(w).size();
    }
    return b;
  };
  uint64_t total = 8 + (n + 1) * 8;
  for (uint64_t i = 0; i < n; ++i) total += row_bytes(i);
  if (out == nullptr || cap < total) return total;
  auto put = [](uint8_t*& p, const void* v, size_t k) {
    std::memcpy(p, v, k);
    p += k;
  };
  uint8_t* p = out;
  put(p, &n, 8);
  uint8_t* offs = p;
  p += (n + 1) * 8;
  uint8_t* base = p;
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t o = static_cast<uint64_t>(p - base);
    std::memcpy(offs + i * 8, &o, 8);
    const uint16_t count = 2, f0 = 0, f1 = 1;
    const uint8_t t_int = 0, t_list = 3;
    put(p, &count, 2);
    put(p, &f0, 2);
    put(p, &t_int, 1);
    put(p, &years[i], 8);
    put(p, &f1, 2);
    put(p, &t_list, 1);
    uint32_t nt = 0;
    for (uint32_t j = 0; j < max_tags; ++j) nt += tags[i * max_tags + j] != UINT32_MAX ? 1u : 0u;
    put(p, &nt, 4);
    for (uint32_t j = 0; j < max_tags; ++j) {
      const uint32_t w = tags[i * max_tags + j];
      if (w == UINT32_MAX) continue;
      const std::string s = "w" + std::to_string(w);
      const uint32_t len = static_cast<uint32_t>(s.size());
      put(p, &len, 4);
      put(p, s.data(), s.size());
    }
  }
  const uint64_t o = static_cast<uint64_t>(p - base);
  std::memcpy(offs + n * 8, &o, 8);
  return total;
}

}  // extern "C"
