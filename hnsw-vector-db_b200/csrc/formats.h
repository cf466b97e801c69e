// Readers for the reference's on-disk index files (host side). Each reader checks the framing
// and every bound the reference's loader checks, so a corrupt file is rejected before anything
// reaches the GPU.
#pragma once

#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

#include "runtime.h"

namespace vdbgpu {

// CRC32C (Castagnoli, reflected polynomial 0x82F63B78), as src/util/crc32c.h computes it.
uint32_t Crc32c(const void* data, size_t n);
// CRC32C continued over more bytes: Crc32cExtend(Crc32c(a), b) == Crc32c(a followed by b).
uint32_t Crc32cExtend(uint32_t crc, const void* data, size_t n);

// CheckIndexFile (src/index/index.cc:46-56): 8-byte magic, body, CRC32C of everything before
// the 4-byte footer.
Status CheckIndexFile(std::string_view bytes, std::string_view* magic, std::string_view* body);

// Index type for a magic (src/index/*.h kMagic constants), or -1.
int IndexTypeForMagic(std::string_view magic);

// Little-endian reader over a byte range (src/util/coding.h ByteReader).
class Reader {
 public:
  explicit Reader(std::string_view d) : p_(d.data()), end_(d.data() + d.size()) {}
  bool u8(uint8_t* v) { return raw(v, 1); }
  bool u16(uint16_t* v) { return raw(v, 2); }
  bool u32(uint32_t* v) { return raw(v, 4); }
  bool u64(uint64_t* v) { return raw(v, 8); }
  bool i64(int64_t* v) { return raw(v, 8); }
  bool f64(double* v) { return raw(v, 8); }
  bool bytes(size_t n, std::string_view* out) {
    if (static_cast<size_t>(end_ - p_) < n) return false;
    *out = std::string_view(p_, n);
    p_ += n;
    return true;
  }
  size_t remaining() const { return static_cast<size_t>(end_ - p_); }

 private:
  bool raw(void* v, size_t n);
  const char* p_;
  const char* end_;
};

// HnswGraph::serialize (src/index/hnsw/hnsw_graph.h:387-401) / Deserialize (403-449).
struct HnswGraphData {
  uint64_t cap = 0, size = 0;
  uint32_t M = 0, M0 = 0, efc = 0;
  uint64_t seed = 0;
  int32_t max_level = -1;
  uint32_t entry = 0;
  std::vector<uint8_t> level;          // cap
  std::vector<uint32_t> links0;        // cap * (1 + M0)
  std::vector<uint32_t> upper;         // concatenated level*(1+M) blocks
  std::vector<uint64_t> upper_off;     // cap (offset in u32; meaningful when level > 0)
};
Status ParseHnswGraph(Reader& r, uint64_t expected_cap, HnswGraphData* g);

// Sq8Quantizer::serialize (src/index/quant/sq8.cc:42-64).
struct Sq8Data {
  uint32_t dim = 0, pd = 0;
  std::vector<float> vmin, scale;
};
Status ParseSq8(Reader& r, Sq8Data* q);

// ProductQuantizer::serialize (src/index/quant/pq.cc:75-92).
struct PqData {
  uint32_t dim = 0, m = 0, dsub = 0;
  std::vector<float> centroids;  // m * 256 * dsub
};
Status ParsePq(Reader& r, PqData* p);

// IvfPqIndex::save (src/index/quant/ivf_pq.cc:236-249) / load (251-279).
struct IvfPqData {
  uint64_t rows = 0;
  uint32_t pd = 0, nlist = 0;
  std::vector<float> coarse;       // nlist * pd
  PqData pq;
  std::vector<uint64_t> list_off;  // nlist + 1
  std::vector<uint32_t> ids;       // rows
  std::vector<uint8_t> codes;      // rows * m, list-major like ids
};
Status ParseIvfPq(std::string_view body, uint64_t rows, uint32_t pd, uint32_t dim, IvfPqData* out);

}  // namespace vdbgpu
