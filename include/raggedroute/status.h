// Allocation-free status of the RaggedRoute v0.2 C++ API (compatible with the
// reference's include/raggedroute/status.h). Appended code: kCommError, used by
// the expert-parallel runtime only.
#pragma once

#include <cuda_runtime_api.h>

namespace raggedroute {

enum class StatusCode {
  kSuccess = 0,
  kInvalidArgument,
  kUnsupportedArchitecture,
  kUnsupportedDataType,
  kUnsupportedLayout,
  kUnsupportedKernelVariant,
  kInsufficientWorkspace,
  kCudaError,
  kCommError,
};

// message always points to a string literal; a Status never owns memory.
struct Status {
  StatusCode code = StatusCode::kSuccess;
  cudaError_t cuda_error = cudaSuccess;
  const char* message = "success";

  constexpr bool ok() const noexcept { return code == StatusCode::kSuccess; }
  constexpr explicit operator bool() const noexcept { return ok(); }
};

constexpr Status success_status() noexcept { return {}; }

}  // namespace raggedroute
