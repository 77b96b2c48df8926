// Per-call resources of the RaggedRoute v0.2 C++ API (compatible with the
// reference's include/raggedroute/runtime.h).
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>

#include "raggedroute/types.h"

namespace raggedroute {

struct RuntimeContext {
  cudaStream_t stream = nullptr;
  void* workspace = nullptr;
  std::size_t workspace_bytes = 0;
  DeviceArchitecture architecture = DeviceArchitecture::kAuto;
};

}  // namespace raggedroute
