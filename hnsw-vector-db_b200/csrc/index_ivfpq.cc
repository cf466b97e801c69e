// IVF-PQ and PQ-flat on the GPU (src/index/quant/ivf_pq.h).
#include "formats.h"
#include "runtime.h"

namespace vdbgpu {

Status LoadIvfPqIndex(Context&, int type, std::string_view, int, const float*, uint64_t, uint32_t,
                      uint32_t, std::unique_ptr<GpuIndex>*) {
  return Status(Status::kNotSupported,
                "index type " + std::to_string(type) + " is not available on the GPU yet");
}

}  // namespace vdbgpu
