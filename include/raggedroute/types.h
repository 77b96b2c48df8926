// Public vocabulary of the RaggedRoute v0.2 C++ API, kept declaration-for-
// declaration compatible with include/raggedroute/types.h of the reference so
// that its callers (benchmark adapters, tests, find_package consumers) build
// unchanged against libraggedroute_b200. Appended values: DeviceArchitecture::kSm100.
#pragma once

#include <array>
#include <cstdint>

namespace raggedroute {

enum class OperatorKind {
  kDenseGemm = 0,
  kTopKGate,
  kHistogram,
  kExclusiveScan,
  kTokenPermute,
  kGroupedGemm,
  kUnpermute,
  kHistogramExclusiveScan,
};

// An architecture is executable only where this library ships kernels for it:
// kSm100 (compute capability 10.0, B200). The other values stay for ABI
// compatibility and resolve to kUnsupportedArchitecture.
enum class DeviceArchitecture {
  kAuto = 0,
  kSm86,
  kSm90,
  kOther,
  kSm100,
};

enum class KernelFamily {
  kAuto = 0,
  kCudaNaive,
  kCudaOptimized,
};

struct KernelSelection {
  KernelFamily family = KernelFamily::kAuto;
  // 0 selects the family default; non-zero ids are operator-local.
  std::uint32_t implementation_id = 0;
};

enum class ScalarType {
  kFp32 = 0,
  kFp16,
  kBf16,
  kFp8E4M3,
  kFp8E5M2,
  kFp6E2M3,
  kFp6E3M2,
  kFp4E2M1,
};

enum class TensorLayout {
  kRowMajorContiguous = 0,
  kColumnMajorContiguous,
  kStrided,
};

// Strides in elements, logical dimension order; all zero = contiguous.
struct TensorSpec {
  ScalarType dtype = ScalarType::kFp32;
  TensorLayout layout = TensorLayout::kRowMajorContiguous;
  std::array<std::int64_t, 3> strides = {0, 0, 0};
};

struct ConstTensorView {
  const void* data = nullptr;
  TensorSpec spec{};
};

struct MutableTensorView {
  void* data = nullptr;
  TensorSpec spec{};
};

enum class TopKNormalization {
  kSelectedSoftmax = 0,
};

enum class TopKTieBreak {
  kLowerExpertId = 0,
};

// NaN orders as -inf; an all-NaN row yields ids {0,1} and weights {0.5,0.5}.
enum class TopKNaNPolicy {
  kNegativeInfinityAllNaNFallback01 = 0,
};

}  // namespace raggedroute
