// Index::build for IVF-PQ and PQ-flat on the GPU, producing the same index file as the reference
// (IvfPqIndex::build / PqFlatIndex::build, src/index/quant/ivf_pq.cc:45-58, 106-150, and save,
// :240-252, 92-97).
//
// The reference's k-means (src/index/quant/kmeans.cc:55-174) is deterministic: a seeded
// std::mt19937_64 drives the subsample, the initialisation and the re-seeding of empty clusters;
// assignments take the first nearest centroid; the new centroids are double sums over the
// points in index order. This file replays all of that on the host with the same standard-library
// distributions and moves only the nearest-centroid searches (the O(n k d) part: every Lloyd
// iteration, the assignment of all rows to lists, the PQ encoding) to the GPU, whose kernels sum
// each distance in the reference's order (ivfpq_build.cu). The k-means++ initialisation, used
// when k x points <= 2e7 (PQ codebooks), runs on the host with the same distance arithmetic.
// The result is the reference's index, byte for byte, on the same rows and options.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <random>
#include <thread>
#include <vector>

#include "formats.h"
#include "ivfpq_build.cuh"
#include "runtime.h"

namespace vdbgpu {
namespace {

constexpr size_t kKMeansIters = 25;        // KMeansOptions::iters
constexpr size_t kMaxPqTrainRows = 65536;  // ivf_pq.cc:14
constexpr size_t kCentroids = 256;         // ProductQuantizer::kCentroids

template <typename T>
void Put(std::string* s, T v) {
  s->append(reinterpret_cast<const char*>(&v), sizeof(T));
}

// Host distances of the k-means++ initialisation, with the reference kernels' arithmetic
// (L2SqAny: four partial sums, no FMA; the vector kernels: FMA accumulators and their trees).
float HostL2Any(const float* a, const float* b, size_t d) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  size_t i = 0;
  for (; i + 4 <= d; i += 4) {
    const float t0 = a[i] - b[i], t1 = a[i + 1] - b[i + 1];
    const float t2 = a[i + 2] - b[i + 2], t3 = a[i + 3] - b[i + 3];
    s0 += t0 * t0;
    s1 += t1 * t1;
    s2 += t2 * t2;
    s3 += t3 * t3;
  }
  for (; i < d; ++i) {
    const float t = a[i] - b[i];
    s0 += t * t;
  }
  return (s0 + s1) + (s2 + s3);
}

float HostL2Runtime(const float* a, const float* b, size_t d, int order) {
  if (order == 1) {  // AVX-512
    float acc0[16] = {}, acc1[16] = {}, s[16];
    size_t i = 0;
    for (; i + 32 <= d; i += 32)
      for (int j = 0; j < 16; ++j) {
        const float t0 = a[i + j] - b[i + j], t1 = a[i + 16 + j] - b[i + 16 + j];
        acc0[j] = std::fmaf(t0, t0, acc0[j]);
        acc1[j] = std::fmaf(t1, t1, acc1[j]);
      }
    if (i < d)
      for (int j = 0; j < 16; ++j) {
        const float t0 = a[i + j] - b[i + j];
        acc0[j] = std::fmaf(t0, t0, acc0[j]);
      }
    for (int j = 0; j < 16; ++j) s[j] = acc0[j] + acc1[j];
    for (int j = 0; j < 8; ++j) s[j] = s[8 + j] + s[j];
    for (int j = 0; j < 4; ++j) s[j] = s[4 + j] + s[j];
    return (s[0] + s[2]) + (s[1] + s[3]);
  }
  if (order == 2) {  // AVX2
    float acc0[8] = {}, acc1[8] = {}, v[8];
    for (size_t i = 0; i < d; i += 16)
      for (int j = 0; j < 8; ++j) {
        const float t0 = a[i + j] - b[i + j], t1 = a[i + 8 + j] - b[i + 8 + j];
        acc0[j] = std::fmaf(t0, t0, acc0[j]);
        acc1[j] = std::fmaf(t1, t1, acc1[j]);
      }
    for (int j = 0; j < 8; ++j) v[j] = acc0[j] + acc1[j];
    float s[4];
    for (int j = 0; j < 4; ++j) s[j] = v[j] + v[4 + j];
    return (s[0] + s[1]) + (s[2] + s[3]);
  }
  float s = 0.f;
  for (size_t i = 0; i < d; ++i) {
    const float t = a[i] - b[i];
    s += t * t;
  }
  return s;
}

// PickL2 (kmeans.cc:16-20).
bool RuntimeKernel(size_t d, size_t stride) { return d % 16 == 0 && stride % 16 == 0; }

// Device rows (n x stride floats) plus the nearest-centroid search over them.
class DevicePoints {
 public:
  Status Upload(Context& ctx, const float* x, size_t n, size_t stride) {
    n_ = n;
    stride_ = stride;
    VDBGPU_RETURN_IF_ERROR(buf_.alloc(std::max<size_t>(1, n * stride) * sizeof(float)));
    if (n > 0)
      VDBGPU_CUDA(cudaMemcpyAsync(buf_.get(), x, n * stride * sizeof(float), cudaMemcpyHostToDevice, ctx.stream()));
    return Status::OK();
  }
  // AssignNearest of the rows' first d floats against k x d centroids (host); assign to host.
  Status Assign(Context& ctx, size_t d, const float* centroids, size_t k, DeviceBuffer* cen_dev,
                DeviceBuffer* asg_dev, uint32_t* assign_host) const {
    VDBGPU_RETURN_IF_ERROR(cen_dev->alloc(k * d * sizeof(float)));
    VDBGPU_RETURN_IF_ERROR(asg_dev->alloc(std::max<size_t>(1, n_) * sizeof(uint32_t)));
    VDBGPU_CUDA(cudaMemcpyAsync(cen_dev->get(), centroids, k * d * sizeof(float), cudaMemcpyHostToDevice, ctx.stream()));
    AssignArgs a{};
    a.points = buf_.as<float>();
    a.n = n_;
    a.d = static_cast<int>(d);
    a.stride = static_cast<int>(stride_);
    a.centroids = cen_dev->as<float>();
    a.k = static_cast<int>(k);
    a.kind = RuntimeKernel(d, stride_) ? kAssignRuntime : kAssignAny;
    a.order = ctx.order();
    a.assign = asg_dev->as<uint32_t>();
    VDBGPU_CUDA(LaunchAssignNearest(a, ctx.stream()));
    if (assign_host != nullptr && n_ > 0)
      VDBGPU_CUDA(cudaMemcpyAsync(assign_host, asg_dev->get(), n_ * sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx.stream()));
    return ctx.Sync("nearest-centroid assignment");
  }
  const float* data() const { return buf_.as<float>(); }

 private:
  DeviceBuffer buf_;
  size_t n_ = 0, stride_ = 0;
};

// One k-means run of the reference (KMeans, kmeans.cc:55-174). The subsample and initialisation
// happen in Prepare (host only, so several runs can prepare on host threads at once); Run does
// the Lloyd iterations with the GPU assignments. `rng` carries over between the two, as in the
// reference.
struct KMeansRun {
  const float* data = nullptr;
  size_t n = 0, d = 0, stride = 0, k = 0, mppc = 256;
  uint64_t seed = 42;
  std::mt19937_64 rng;
  std::vector<float> sample;   // the subsample (contiguous) when one was drawn
  const float* x = nullptr;    // the points the iterations use
  size_t m = 0, xs = 0;
  std::vector<float> cen;
  bool done = false;           // n <= k: the centroids are the points themselves

  void Prepare(int order) {
    cen.assign(k * d, 0.f);
    rng.seed(seed);
    if (n <= k) {
      for (size_t c = 0; c < k; ++c) std::memcpy(cen.data() + c * d, data + (c % n) * stride, d * sizeof(float));
      done = true;
      return;
    }
    m = std::min(n, k * std::max<size_t>(1, mppc));
    x = data;
    xs = stride;
    if (m < n) {
      std::vector<size_t> idx(n);
      std::iota(idx.begin(), idx.end(), 0);
      for (size_t i = 0; i < m; ++i) {
        std::uniform_int_distribution<size_t> u(i, n - 1);
        std::swap(idx[i], idx[u(rng)]);
      }
      std::sort(idx.begin(), idx.begin() + static_cast<std::ptrdiff_t>(m));
      sample.resize(m * d);
      for (size_t i = 0; i < m; ++i) std::memcpy(sample.data() + i * d, data + idx[i] * stride, d * sizeof(float));
      x = sample.data();
      xs = d;
    }
    const bool rt = RuntimeKernel(d, xs);
    auto fn = [&](const float* a, const float* b) { return rt ? HostL2Runtime(a, b, d, order) : HostL2Any(a, b, d); };
    float* c0 = cen.data();
    const bool use_pp = static_cast<double>(k) * static_cast<double>(m) <= 2.0e7;
    if (use_pp) {
      std::vector<float> mind(m, std::numeric_limits<float>::infinity());
      std::uniform_int_distribution<size_t> u0(0, m - 1);
      const size_t first = u0(rng);
      std::memcpy(c0, x + first * xs, d * sizeof(float));
      for (size_t c = 1; c < k; ++c) {
        const float* last = c0 + (c - 1) * d;
        double total = 0;
        for (size_t i = 0; i < m; ++i) {
          mind[i] = std::min(mind[i], fn(x + i * xs, last));
          total += mind[i];
        }
        size_t pick = 0;
        if (total > 0) {
          std::uniform_real_distribution<double> ur(0.0, total);
          const double t = ur(rng);
          double acc = 0;
          for (pick = 0; pick + 1 < m; ++pick) {
            acc += mind[pick];
            if (acc >= t) break;
          }
        } else {
          pick = u0(rng);
        }
        std::memcpy(c0 + c * d, x + pick * xs, d * sizeof(float));
      }
    } else {
      std::vector<size_t> idx(m);
      std::iota(idx.begin(), idx.end(), 0);
      for (size_t c = 0; c < k; ++c) {
        std::uniform_int_distribution<size_t> u(c, m - 1);
        std::swap(idx[c], idx[u(rng)]);
        std::memcpy(c0 + c * d, x + idx[c] * xs, d * sizeof(float));
      }
    }
  }

  Status Run(Context& ctx) {
    if (done) return Status::OK();
    DevicePoints pts;
    VDBGPU_RETURN_IF_ERROR(pts.Upload(ctx, x, m, xs));
    DeviceBuffer cen_dev, asg_dev;
    std::vector<uint32_t> assign(m);
    std::vector<double> sums(k * d);
    std::vector<size_t> counts(k);
    constexpr float kEps = 1.0f / 1024.0f;
    for (size_t it = 0; it < kKMeansIters; ++it) {
      VDBGPU_RETURN_IF_ERROR(pts.Assign(ctx, d, cen.data(), k, &cen_dev, &asg_dev, assign.data()));
      std::fill(sums.begin(), sums.end(), 0.0);
      std::fill(counts.begin(), counts.end(), 0);
      for (size_t i = 0; i < m; ++i) {
        const float* p = x + i * xs;
        double* s = sums.data() + static_cast<size_t>(assign[i]) * d;
        for (size_t j = 0; j < d; ++j) s[j] += p[j];
        ++counts[assign[i]];
      }
      for (size_t c = 0; c < k; ++c) {
        if (counts[c] == 0) continue;
        const double inv = 1.0 / static_cast<double>(counts[c]);
        for (size_t j = 0; j < d; ++j) cen[c * d + j] = static_cast<float>(sums[c * d + j] * inv);
      }
      for (size_t c = 0; c < k; ++c) {
        if (counts[c] != 0) continue;
        const size_t big = static_cast<size_t>(std::max_element(counts.begin(), counts.end()) - counts.begin());
        std::uniform_real_distribution<float> noise(-1.f, 1.f);
        for (size_t j = 0; j < d; ++j) {
          const float v = cen[big * d + j];
          const float delta = kEps * (std::fabs(v) + 1e-3f) * noise(rng);
          cen[c * d + j] = v + delta;
          cen[big * d + j] = v - delta;
        }
        counts[c] = counts[big] / 2;
        counts[big] -= counts[c];
      }
    }
    return Status::OK();
  }
};

// ProductQuantizer::train (pq.cc:14-42) over n rows of `stride` floats: m codebooks of 256
// centroids, subspace j from its slice of a strided sample, seed + 7919 j. The k-means++
// initialisations of the subspaces run on host threads.
Status TrainPq(Context& ctx, const float* data, size_t n, size_t stride, size_t dim, size_t m, size_t mppc,
               uint64_t seed, std::vector<float>* codebooks) {
  const size_t dsub = dim / m;
  codebooks->assign(m * kCentroids * dsub, 0.f);
  const size_t cap = std::min(n, kCentroids * std::max<size_t>(1, mppc));
  const size_t step = std::max<size_t>(1, n / std::max<size_t>(1, cap));
  std::vector<std::vector<float>> subs(m);
  std::vector<KMeansRun> runs(m);
  for (size_t j = 0; j < m; ++j) {
    auto& sub = subs[j];
    sub.reserve(cap * dsub);
    for (size_t i = 0, taken = 0; i < n && taken < cap; i += step, ++taken) {
      const float* p = data + i * stride + j * dsub;
      sub.insert(sub.end(), p, p + dsub);
    }
    KMeansRun& r = runs[j];
    r.data = sub.data();
    r.n = sub.size() / dsub;
    r.d = dsub;
    r.stride = dsub;
    r.k = kCentroids;
    r.mppc = mppc;
    r.seed = seed + j * 7919;
  }
  const int order = ctx.order();
  const size_t nt = std::max<size_t>(1, std::min<size_t>(m, std::thread::hardware_concurrency()));
  std::vector<std::thread> th;
  for (size_t t = 0; t < nt; ++t)
    th.emplace_back([&, t] {
      for (size_t j = t; j < m; j += nt) runs[j].Prepare(order);
    });
  for (auto& x : th) x.join();
  for (size_t j = 0; j < m; ++j) {
    VDBGPU_RETURN_IF_ERROR(runs[j].Run(ctx));
    std::memcpy(codebooks->data() + j * kCentroids * dsub, runs[j].cen.data(), kCentroids * dsub * sizeof(float));
  }
  return Status::OK();
}

}  // namespace

Status BuildIvfPqFile(Context& ctx, int type, const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                      uint32_t nlist_opt, uint32_t pq_m, uint32_t mppc, uint64_t seed, std::string* file) {
  if (type != kIndexIvfPq && type != kIndexPqFlat)
    return Status(Status::kInvalidArgument, "the GPU builder makes ivf_pq and pq index files");
  if (pq_m == 0 || dim % pq_m != 0)
    return Status(Status::kInvalidArgument, "pq_m must divide the dimension (dim " + std::to_string(dim) +
                                                ", m " + std::to_string(pq_m) + ")");
  if (pd > static_cast<uint32_t>(kAssignMaxDim))
    return Status(Status::kNotSupported, "the GPU builder supports padded dimensions up to 256");
  if (dim / pq_m > 64)
    return Status(Status::kNotSupported, "the GPU builder supports sub-vectors of up to 64 floats (dim / pq_m)");
  const size_t m = pq_m, dsub = dim / pq_m;
  // Host copy of the rows (the k-means sums, samples and residuals are host work).
  std::vector<float> host;
  const float* hx = rows;
  cudaPointerAttributes attr{};
  if (n > 0 && cudaPointerGetAttributes(&attr, rows) == cudaSuccess && attr.type == cudaMemoryTypeDevice) {
    host.resize(n * pd);
    VDBGPU_CUDA(cudaMemcpy(host.data(), rows, n * pd * sizeof(float), cudaMemcpyDeviceToHost));
    hx = host.data();
  }
  (void)cudaGetLastError();

  std::string out = type == kIndexIvfPq ? "VDBIVFP1" : "VDBPQFL1";
  std::vector<float> pq;
  std::vector<uint8_t> codes(n * m);
  DevicePoints all;
  if (type == kIndexPqFlat) {
    // An empty segment keeps an untrained quantizer: no codebooks in the file.
    if (n > 0) {
      VDBGPU_RETURN_IF_ERROR(TrainPq(ctx, hx, n, pd, dim, m, mppc, seed, &pq));
      VDBGPU_RETURN_IF_ERROR(all.Upload(ctx, hx, n, pd));
    }
  } else {
    const size_t nlist = n == 0 ? 0 : std::clamp<size_t>(nlist_opt, 1, std::max<size_t>(1, n / 39));
    std::vector<float> coarse;
    std::vector<uint32_t> assign(n);
    DeviceBuffer cen_dev, asg_dev;
    if (n > 0) {
      KMeansRun km;
      km.data = hx;
      km.n = n;
      km.d = pd;
      km.stride = pd;
      km.k = nlist;
      km.mppc = mppc;
      km.seed = seed;
      km.Prepare(ctx.order());
      VDBGPU_RETURN_IF_ERROR(km.Run(ctx));
      coarse = std::move(km.cen);
      VDBGPU_RETURN_IF_ERROR(all.Upload(ctx, hx, n, pd));
      VDBGPU_RETURN_IF_ERROR(all.Assign(ctx, pd, coarse.data(), nlist, &cen_dev, &asg_dev, assign.data()));
      // PQ on the residuals of a strided sample (ivf_pq.cc:118-127).
      const size_t step = std::max<size_t>(1, n / kMaxPqTrainRows);
      std::vector<float> res;
      res.reserve(std::min<size_t>(n, kMaxPqTrainRows + 1) * dim);
      for (size_t i = 0; i < n; i += step) {
        const float* xr = hx + i * pd;
        const float* c = coarse.data() + static_cast<size_t>(assign[i]) * pd;
        for (size_t j = 0; j < dim; ++j) res.push_back(xr[j] - c[j]);
      }
      VDBGPU_RETURN_IF_ERROR(TrainPq(ctx, res.data(), res.size() / dim, dim, dim, m, mppc, seed, &pq));
    }
    Put<uint64_t>(&out, n);
    Put<uint32_t>(&out, pd);
    Put<uint32_t>(&out, static_cast<uint32_t>(nlist));
    out.append(reinterpret_cast<const char*>(coarse.data()), coarse.size() * sizeof(float));
    Put<uint32_t>(&out, dim);
    Put<uint32_t>(&out, pq_m);
    out.append(reinterpret_cast<const char*>(pq.data()), pq.size() * sizeof(float));
    if (n > 0) {
      DeviceBuffer pq_dev, codes_dev;
      VDBGPU_RETURN_IF_ERROR(pq_dev.alloc(pq.size() * sizeof(float)));
      VDBGPU_RETURN_IF_ERROR(codes_dev.alloc(n * m));
      VDBGPU_CUDA(cudaMemcpyAsync(pq_dev.get(), pq.data(), pq.size() * sizeof(float), cudaMemcpyHostToDevice, ctx.stream()));
      PqEncodeArgs e{};
      e.rows = all.data();
      e.n = n;
      e.pd = static_cast<int>(pd);
      e.dim = static_cast<int>(dim);
      e.coarse = cen_dev.as<float>();
      e.assign = asg_dev.as<uint32_t>();
      e.pq = pq_dev.as<float>();
      e.m = static_cast<int>(m);
      e.dsub = static_cast<int>(dsub);
      e.codes = codes_dev.as<uint8_t>();
      VDBGPU_CUDA(LaunchPqEncode(e, ctx.stream()));
      VDBGPU_CUDA(cudaMemcpyAsync(codes.data(), codes_dev.get(), n * m, cudaMemcpyDeviceToHost, ctx.stream()));
      VDBGPU_RETURN_IF_ERROR(ctx.Sync("pq encode"));
    }
    // Lists in row order (ivf_pq.cc:141-147).
    std::vector<uint64_t> sizes(nlist, 0);
    for (size_t i = 0; i < n; ++i) ++sizes[assign[i]];
    std::vector<uint64_t> start(nlist + 1, 0);
    for (size_t l = 0; l < nlist; ++l) start[l + 1] = start[l] + sizes[l];
    std::vector<uint32_t> ids(n);
    std::vector<uint64_t> pos(start.begin(), start.end() - (nlist > 0 ? 1 : 0));
    for (size_t i = 0; i < n; ++i) ids[pos[assign[i]]++] = static_cast<uint32_t>(i);
    for (size_t l = 0; l < nlist; ++l) {
      Put<uint64_t>(&out, sizes[l]);
      out.append(reinterpret_cast<const char*>(ids.data() + start[l]), sizes[l] * sizeof(uint32_t));
      for (uint64_t t = start[l]; t < start[l + 1]; ++t)
        out.append(reinterpret_cast<const char*>(codes.data() + static_cast<size_t>(ids[t]) * m), m);
    }
    Put<uint32_t>(&out, Crc32c(out.data(), out.size()));
    *file = std::move(out);
    return Status::OK();
  }
  // PQ-flat: u64 rows, the codebooks, the codes in row order (PqFlatIndex::save).
  if (n > 0) {
    DeviceBuffer pq_dev, codes_dev;
    VDBGPU_RETURN_IF_ERROR(pq_dev.alloc(pq.size() * sizeof(float)));
    VDBGPU_RETURN_IF_ERROR(codes_dev.alloc(n * m));
    VDBGPU_CUDA(cudaMemcpyAsync(pq_dev.get(), pq.data(), pq.size() * sizeof(float), cudaMemcpyHostToDevice, ctx.stream()));
    PqEncodeArgs e{};
    e.rows = all.data();
    e.n = n;
    e.pd = static_cast<int>(pd);
    e.dim = static_cast<int>(dim);
    e.pq = pq_dev.as<float>();
    e.m = static_cast<int>(m);
    e.dsub = static_cast<int>(dsub);
    e.codes = codes_dev.as<uint8_t>();
    VDBGPU_CUDA(LaunchPqEncode(e, ctx.stream()));
    VDBGPU_CUDA(cudaMemcpyAsync(codes.data(), codes_dev.get(), n * m, cudaMemcpyDeviceToHost, ctx.stream()));
    VDBGPU_RETURN_IF_ERROR(ctx.Sync("pq encode"));
  }
  Put<uint64_t>(&out, n);
  Put<uint32_t>(&out, dim);
  Put<uint32_t>(&out, pq_m);
  out.append(reinterpret_cast<const char*>(pq.data()), pq.size() * sizeof(float));
  out.append(reinterpret_cast<const char*>(codes.data()), codes.size());
  Put<uint32_t>(&out, Crc32c(out.data(), out.size()));
  *file = std::move(out);
  return Status::OK();
}

}  // namespace vdbgpu
