// Dispatch API of the RaggedRoute v0.2 C++ API (compatible with the reference's
// include/raggedroute/dispatch.h). This library executes on kSm100 only.
#pragma once

#include <optional>

#include "raggedroute/status.h"
#include "raggedroute/types.h"

namespace raggedroute {

// Floating operand roles; std::nullopt = role not part of the operator.
struct OperatorSignature {
  std::optional<TensorSpec> input;
  std::optional<TensorSpec> weight;
  std::optional<ScalarType> accumulator;
  std::optional<TensorSpec> output;
};

struct DispatchRequest {
  OperatorKind operator_kind = OperatorKind::kDenseGemm;
  DeviceArchitecture architecture = DeviceArchitecture::kAuto;
  KernelSelection requested_kernel;
  OperatorSignature signature;
};

struct DispatchDecision {
  OperatorKind operator_kind = OperatorKind::kDenseGemm;
  DeviceArchitecture architecture = DeviceArchitecture::kOther;
  KernelSelection kernel;
};

DeviceArchitecture classify_compute_capability(int major, int minor) noexcept;
Status query_current_device_architecture(DeviceArchitecture* architecture) noexcept;
Status resolve_device_architecture(DeviceArchitecture requested,
                                   DeviceArchitecture* resolved) noexcept;
Status select_kernel(const DispatchRequest& request, DispatchDecision* decision) noexcept;

}  // namespace raggedroute
