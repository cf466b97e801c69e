// Readers for the reference's index files and the magic-dispatched loader
// (LoadIndex, src/index/index.cc:58-87).
#include "formats.h"

#include <cstring>

namespace vdbgpu {

namespace {

struct CrcTable {
  uint32_t t[256];
  CrcTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0x82F63B78u : (c >> 1);
      t[i] = c;
    }
  }
};

// The same polynomial with the x86 CRC32 instruction (SSE4.2), 8 bytes at a time.
__attribute__((target("sse4.2"))) uint32_t Crc32cHw(const uint8_t* p, size_t n, uint32_t c) {
  uint64_t c64 = c;
  for (; n >= 8; n -= 8, p += 8) {
    uint64_t w;
    std::memcpy(&w, p, 8);
    c64 = __builtin_ia32_crc32di(c64, w);
  }
  c = static_cast<uint32_t>(c64);
  for (; n > 0; --n, ++p) c = __builtin_ia32_crc32qi(c, *p);
  return c;
}

}  // namespace

uint32_t Crc32cExtend(uint32_t crc, const void* data, size_t n) {
  static const CrcTable table;
  static const bool hw = __builtin_cpu_supports("sse4.2");
  const auto* p = static_cast<const uint8_t*>(data);
  uint32_t c = crc ^ 0xFFFFFFFFu;
  if (hw) return Crc32cHw(p, n, c) ^ 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) c = table.t[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

uint32_t Crc32c(const void* data, size_t n) { return Crc32cExtend(0, data, n); }


bool Reader::raw(void* v, size_t n) {
  if (static_cast<size_t>(end_ - p_) < n) return false;
  std::memcpy(v, p_, n);
  p_ += n;
  return true;
}

Status CheckIndexFile(std::string_view bytes, std::string_view* magic, std::string_view* body) {
  if (bytes.size() < 12) return Status(Status::kCorruption, "index file too short");
  uint32_t stored;
  std::memcpy(&stored, bytes.data() + bytes.size() - 4, 4);
  if (Crc32c(bytes.data(), bytes.size() - 4) != stored)
    return Status(Status::kCorruption, "index file checksum mismatch");
  *magic = bytes.substr(0, 8);
  *body = bytes.substr(8, bytes.size() - 12);
  return Status::OK();
}

int IndexTypeForMagic(std::string_view magic) {
  if (magic == "VDBFLAT1") return kIndexFlat;
  if (magic == "VDBHNSW1") return kIndexHnsw;
  if (magic == "VDBHSQ81") return kIndexHnswSq8;
  if (magic == "VDBPQFL1") return kIndexPqFlat;
  if (magic == "VDBIVFP1") return kIndexIvfPq;
  return -1;
}

Status ParseHnswGraph(Reader& r, uint64_t expected_cap, HnswGraphData* g) {
  uint64_t cap = 0, sz = 0, seed = 0;
  uint32_t m = 0, efc = 0, maxl = 0, ep = 0;
  if (!r.u64(&cap) || !r.u64(&sz) || !r.u32(&m) || !r.u32(&efc) || !r.u64(&seed) ||
      !r.u32(&maxl) || !r.u32(&ep))
    return Status(Status::kCorruption, "truncated hnsw header");
  if (cap != expected_cap || sz > cap || m < 2 || m > 4096)
    return Status(Status::kCorruption, "hnsw header does not match the segment");
  const int max_level = static_cast<int32_t>(maxl);
  if (max_level > 15 || (cap > 0 && ep >= cap)) return Status(Status::kCorruption, "bad hnsw entry point");
  g->cap = cap;
  g->size = sz;
  g->M = m;
  g->M0 = 2 * m;
  g->efc = efc;
  g->seed = seed;
  g->max_level = max_level;
  g->entry = ep;
  std::string_view b;
  if (!r.bytes(cap, &b)) return Status(Status::kCorruption, "truncated hnsw levels");
  g->level.assign(b.begin(), b.end());
  const size_t l0 = cap * (1 + static_cast<size_t>(g->M0));
  if (!r.bytes(l0 * 4, &b)) return Status(Status::kCorruption, "truncated hnsw layer 0");
  g->links0.resize(l0);
  if (l0 > 0) std::memcpy(g->links0.data(), b.data(), l0 * 4);
  g->upper_off.assign(cap, 0);
  g->upper.clear();
  for (uint64_t i = 0; i < cap; ++i) {
    const int lvl = g->level[i];
    if (sz > 0 && lvl > max_level) return Status(Status::kCorruption, "node above the top layer");
    if (lvl == 0) continue;
    const size_t n = static_cast<size_t>(lvl) * (1 + m);
    if (!r.bytes(n * 4, &b)) return Status(Status::kCorruption, "truncated hnsw upper layers");
    g->upper_off[i] = g->upper.size();
    const size_t at = g->upper.size();
    g->upper.resize(at + n);
    std::memcpy(g->upper.data() + at, b.data(), n * 4);
  }
  // The descent starts at the entry point on the top layer, so it must live there.
  if (sz > 0 && cap > 0 && g->level[ep] < max_level)
    return Status(Status::kCorruption, "hnsw entry point is below the top layer");
  // Every link must stay in range (the reference validates the same before searching).
  for (uint64_t i = 0; i < cap; ++i) {
    for (int l = 0; l <= g->level[i]; ++l) {
      const uint32_t* ll = l == 0 ? g->links0.data() + i * (1 + g->M0)
                                  : g->upper.data() + g->upper_off[i] + static_cast<size_t>(l - 1) * (1 + m);
      if (ll[0] > (l == 0 ? g->M0 : m)) return Status(Status::kCorruption, "bad link count");
      for (uint32_t j = 0; j < ll[0]; ++j)
        if (ll[1 + j] >= cap) return Status(Status::kCorruption, "bad link target");
    }
  }
  return Status::OK();
}

Status ParseSq8(Reader& r, Sq8Data* q) {
  uint32_t d = 0, p = 0;
  if (!r.u32(&d) || !r.u32(&p) || d > p || p % 16 != 0)
    return Status(Status::kCorruption, "bad sq8 quantizer");
  std::string_view a, b;
  if (!r.bytes(size_t(p) * 4, &a) || !r.bytes(size_t(p) * 4, &b))
    return Status(Status::kCorruption, "truncated sq8 quantizer");
  q->dim = d;
  q->pd = p;
  q->vmin.resize(p);
  q->scale.resize(p);
  std::memcpy(q->vmin.data(), a.data(), a.size());
  std::memcpy(q->scale.data(), b.data(), b.size());
  return Status::OK();
}

Status ParsePq(Reader& r, PqData* pq) {
  uint32_t d = 0, m = 0;
  if (!r.u32(&d) || !r.u32(&m) || m == 0 || d % m != 0) return Status(Status::kCorruption, "bad pq codebook");
  pq->dim = d;
  pq->m = m;
  pq->dsub = d / m;
  std::string_view b;
  const size_t n = static_cast<size_t>(m) * 256 * pq->dsub;
  if (!r.bytes(n * 4, &b)) return Status(Status::kCorruption, "truncated pq codebook");
  pq->centroids.resize(n);
  std::memcpy(pq->centroids.data(), b.data(), n * 4);
  return Status::OK();
}

Status ParseIvfPq(std::string_view body, uint64_t rows, uint32_t pd, uint32_t dim, IvfPqData* out) {
  Reader r(body);
  uint64_t n = 0;
  uint32_t fpd = 0, nl = 0;
  if (!r.u64(&n) || !r.u32(&fpd) || !r.u32(&nl) || n != rows || fpd != pd)
    return Status(Status::kCorruption, "ivf-pq index does not match the segment");
  out->rows = n;
  out->pd = pd;
  out->nlist = nl;
  std::string_view b;
  if (!r.bytes(size_t(nl) * pd * 4, &b)) return Status(Status::kCorruption, "truncated ivf centroids");
  out->coarse.resize(size_t(nl) * pd);
  if (!b.empty()) std::memcpy(out->coarse.data(), b.data(), b.size());
  // IvfPqIndex::load (ivf_pq.cc:263) reports any codebook fault, truncation included, alike.
  if (!ParsePq(r, &out->pq).ok() || out->pq.dim != dim) return Status(Status::kCorruption, "bad pq codebook");
  const uint32_t m = out->pq.m;
  out->list_off.assign(nl + 1, 0);
  out->ids.clear();
  out->codes.clear();
  out->ids.reserve(n);
  out->codes.reserve(n * m);
  for (uint32_t l = 0; l < nl; ++l) {
    uint64_t sz = 0;
    if (!r.u64(&sz) || sz > n) return Status(Status::kCorruption, "bad ivf list size");
    if (!r.bytes(sz * 4, &b)) return Status(Status::kCorruption, "truncated ivf ids");
    const size_t at = out->ids.size();
    out->ids.resize(at + sz);
    if (sz > 0) std::memcpy(out->ids.data() + at, b.data(), sz * 4);
    for (uint64_t i = 0; i < sz; ++i)
      if (out->ids[at + i] >= n) return Status(Status::kCorruption, "ivf id out of range");
    if (!r.bytes(sz * m, &b)) return Status(Status::kCorruption, "truncated ivf codes");
    out->codes.insert(out->codes.end(), b.begin(), b.end());
    out->list_off[l + 1] = out->ids.size();
  }
  return Status::OK();
}

Status LoadIndexFile(Context& ctx, const void* bytes, size_t nbytes, int metric,
                     const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                     std::unique_ptr<GpuIndex>* out) {
  std::string_view magic, body;
  VDBGPU_RETURN_IF_ERROR(
      CheckIndexFile(std::string_view(static_cast<const char*>(bytes), nbytes), &magic, &body));
  const int type = IndexTypeForMagic(magic);
  switch (type) {
    case kIndexFlat:
      return CreateFlatIndex(ctx, metric, rows, n, dim, pd, out);
    case kIndexHnsw:
    case kIndexHnswSq8:
    case kIndexPqFlat:
    case kIndexIvfPq:
      return LoadGraphOrListIndex(ctx, type, body, metric, rows, n, dim, pd, out);
    default:
      return Status(Status::kCorruption, "unknown index file magic");
  }
}

}  // namespace vdbgpu
