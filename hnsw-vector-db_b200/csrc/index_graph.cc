// Loaders for the graph (HNSW, HNSW-SQ8) and list (PQ-flat, IVF-PQ) index types.
#include "formats.h"
#include "runtime.h"

namespace vdbgpu {

Status LoadGraphOrListIndex(Context&, int type, std::string_view, int, const float*, uint64_t,
                            uint32_t, uint32_t, std::unique_ptr<GpuIndex>*) {
  return Status(Status::kNotSupported,
                "index type " + std::to_string(type) + " is not available on the GPU yet");
}

}  // namespace vdbgpu
