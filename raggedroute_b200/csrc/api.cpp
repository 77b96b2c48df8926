// Operator runtime of libraggedroute_b200: the raggedroute:: C++ API, the
// raggedroute::ops:: low-level launchers and the rr_* C ABI.
//
// Each wrapper validates in the same order and with the same status codes as
// the reference wrapper it replaces (cited per function), then enqueues the
// B200 kernels on the caller's stream. Differences from the reference, all
// deliberate: the executable architecture is kSm100 (the reference accepts
// SM86 only, src/runtime/dispatch.cpp:239-242); the expert cap is 1024
// instead of 64; every kernel family and research id the reference accepts
// runs the same B200 kernel; token_permute produces the stable slot order
// with the reference's experts*4 bytes of workspace for every input size.
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstring>
#include <limits>

#include "../../include/raggedroute/baseline_ops.h"
#include "../../include/raggedroute/chain.h"
#include "../../include/raggedroute/dispatch.h"
#include "../../include/raggedroute/operators.h"
#include "../../include/raggedroute_b200.h"
#include "common.cuh"

namespace rrb {
unsigned long long launch_count();
cudaError_t consume_device_error(cudaStream_t stream, unsigned* out);
}  // namespace rrb

// Helpers shared by the wrappers below. They are not part of the reference's
// exported API, so they stay out of the library's dynamic symbol table (a
// caller that compiles the reference's own inline helpers of the same names
// keeps its copies).
#define RR_INTERNAL __attribute__((visibility("hidden")))

namespace raggedroute {
namespace detail {

inline Status make_status(StatusCode code, const char* message,
                          cudaError_t cuda_error = cudaSuccess) noexcept {
  return {code, cuda_error, message};
}

inline Status cuda_status(cudaError_t error, const char* message) noexcept {
  return error == cudaSuccess ? success_status()
                              : make_status(StatusCode::kCudaError, message, error);
}

inline Status invalid_argument(const char* message) noexcept {
  return make_status(StatusCode::kInvalidArgument, message);
}

inline bool is_aligned(const void* pointer, std::size_t alignment) noexcept {
  return pointer == nullptr || reinterpret_cast<std::uintptr_t>(pointer) % alignment == 0;
}

inline OperatorSignature compute_signature(const ConstTensorView& input,
                                           const ConstTensorView& weight, ScalarType accumulator,
                                           const MutableTensorView& output) {
  return {input.spec, weight.spec, accumulator, output.spec};
}

RR_INTERNAL Status dispatch_operator(OperatorKind kind, const OperatorSignature& signature,
                         KernelSelection requested, DeviceArchitecture architecture,
                         DispatchDecision* decision) noexcept {
  DeviceArchitecture resolved = DeviceArchitecture::kOther;
  Status status = resolve_device_architecture(architecture, &resolved);
  if (!status.ok()) return status;
  DispatchRequest request;
  request.operator_kind = kind;
  request.architecture = resolved;
  request.requested_kernel = requested;
  request.signature = signature;
  return select_kernel(request, decision);
}

// Grouped GEMM and unpermute expose only the default family publicly
// (src/runtime/operator_internal.h:42-49).
inline Status require_default_family(const DispatchDecision& decision) noexcept {
  if (decision.kernel.family != KernelFamily::kCudaNaive ||
      decision.kernel.implementation_id != 0) {
    return make_status(StatusCode::kUnsupportedKernelVariant,
                       "operator wrapper does not implement the selected kernel");
  }
  return success_status();
}

RR_INTERNAL bool ranges_overlap(const void* a, std::size_t a_bytes, const void* b,
                    std::size_t b_bytes) noexcept {
  if (a_bytes == 0 || b_bytes == 0) return false;
  const auto a0 = reinterpret_cast<std::uintptr_t>(a);
  const auto b0 = reinterpret_cast<std::uintptr_t>(b);
  return a0 < b0 + b_bytes && b0 < a0 + a_bytes;
}

}  // namespace detail

namespace {

constexpr int kMaxExperts = rrb::kMaxExperts;

bool has_zero_strides(const TensorSpec& spec) noexcept {
  return spec.strides[0] == 0 && spec.strides[1] == 0 && spec.strides[2] == 0;
}

bool contiguous_layout(const std::optional<TensorSpec>& spec) noexcept {
  return !spec || (spec->layout == TensorLayout::kRowMajorContiguous && has_zero_strides(*spec));
}

bool storage_type(ScalarType type) noexcept {
  return type == ScalarType::kFp32 || type == ScalarType::kFp16 || type == ScalarType::kBf16;
}

bool has_roles(const OperatorSignature& s, bool input, bool weight, bool accumulator,
               bool output) noexcept {
  return s.input.has_value() == input && s.weight.has_value() == weight &&
         s.accumulator.has_value() == accumulator && s.output.has_value() == output;
}

// Role/dtype rules of src/runtime/dispatch.cpp:105-137.
bool valid_dtype_signature(OperatorKind kind, const OperatorSignature& s) noexcept {
  switch (kind) {
    case OperatorKind::kDenseGemm:
    case OperatorKind::kGroupedGemm: {
      if (!has_roles(s, true, true, true, true)) return false;
      const ScalarType in = s.input->dtype;
      return storage_type(in) && s.weight->dtype == in && *s.accumulator == ScalarType::kFp32 &&
             (s.output->dtype == in || s.output->dtype == ScalarType::kFp32);
    }
    case OperatorKind::kTopKGate:
      return has_roles(s, true, false, true, true) && s.input->dtype == ScalarType::kFp32 &&
             *s.accumulator == ScalarType::kFp32 && s.output->dtype == ScalarType::kFp32;
    case OperatorKind::kHistogram:
    case OperatorKind::kExclusiveScan:
    case OperatorKind::kHistogramExclusiveScan:
      return has_roles(s, false, false, false, false);
    case OperatorKind::kTokenPermute:
      return has_roles(s, true, false, false, true) && storage_type(s.input->dtype) &&
             s.output->dtype == s.input->dtype;
    case OperatorKind::kUnpermute: {
      if (!has_roles(s, true, true, true, true)) return false;
      const ScalarType in = s.input->dtype;
      return storage_type(in) && s.weight->dtype == ScalarType::kFp32 &&
             *s.accumulator == ScalarType::kFp32 &&
             (s.output->dtype == in || s.output->dtype == ScalarType::kFp32);
    }
  }
  return false;
}

bool all_fp32(const OperatorSignature& s) noexcept {
  return (!s.input || s.input->dtype == ScalarType::kFp32) &&
         (!s.weight || s.weight->dtype == ScalarType::kFp32) &&
         (!s.accumulator || *s.accumulator == ScalarType::kFp32) &&
         (!s.output || s.output->dtype == ScalarType::kFp32);
}

// Research ids the reference's public dispatch accepts for kCudaOptimized
// (src/*/cuda_candidate/*internal.h); all run the B200 kernel here.
bool accepted_optimized_id(OperatorKind kind, std::uint32_t id) noexcept {
  switch (kind) {
    case OperatorKind::kDenseGemm: return id >= 1 && id <= 7;
    case OperatorKind::kTopKGate: return id >= 1 && id <= 4;
    case OperatorKind::kHistogram: return id == 101;
    case OperatorKind::kHistogramExclusiveScan: return id == 2;
    case OperatorKind::kTokenPermute: return id >= 1 && id <= 10;
    default: return false;
  }
}

}  // namespace

// ---- dispatch (src/runtime/dispatch.cpp:148-291) ----------------------------

DeviceArchitecture classify_compute_capability(int major, int minor) noexcept {
  if (major == 10 && minor == 0) return DeviceArchitecture::kSm100;
  if (major == 8 && minor == 6) return DeviceArchitecture::kSm86;
  if (major == 9 && minor == 0) return DeviceArchitecture::kSm90;
  return DeviceArchitecture::kOther;
}

Status query_current_device_architecture(DeviceArchitecture* architecture) noexcept {
  if (architecture == nullptr) {
    return detail::invalid_argument("architecture output must not be null");
  }
  int device = 0;
  cudaError_t error = cudaGetDevice(&device);
  if (error != cudaSuccess) {
    return detail::cuda_status(error, "cudaGetDevice failed while resolving architecture");
  }
  int major = 0, minor = 0;
  error = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (error == cudaSuccess) {
    error = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  }
  if (error != cudaSuccess) {
    return detail::cuda_status(error, "cudaDeviceGetAttribute failed while resolving architecture");
  }
  *architecture = classify_compute_capability(major, minor);
  return success_status();
}

Status resolve_device_architecture(DeviceArchitecture requested,
                                   DeviceArchitecture* resolved) noexcept {
  if (resolved == nullptr) {
    return detail::invalid_argument("resolved architecture output must not be null");
  }
  if (requested == DeviceArchitecture::kAuto) return query_current_device_architecture(resolved);
  *resolved = requested;
  return success_status();
}

Status select_kernel(const DispatchRequest& request, DispatchDecision* decision) noexcept {
  if (decision == nullptr) {
    return detail::invalid_argument("dispatch decision output must not be null");
  }
  bool roles_valid = false;
  const OperatorSignature& s = request.signature;
  switch (request.operator_kind) {
    case OperatorKind::kDenseGemm:
    case OperatorKind::kGroupedGemm:
    case OperatorKind::kUnpermute:
      roles_valid = has_roles(s, true, true, true, true);
      break;
    case OperatorKind::kTopKGate:
      roles_valid = has_roles(s, true, false, true, true);
      break;
    case OperatorKind::kTokenPermute:
      roles_valid = has_roles(s, true, false, false, true);
      break;
    case OperatorKind::kHistogram:
    case OperatorKind::kExclusiveScan:
    case OperatorKind::kHistogramExclusiveScan:
      roles_valid = has_roles(s, false, false, false, false);
      break;
    default:
      return detail::invalid_argument("unknown operator kind");
  }
  if (!roles_valid) {
    return detail::invalid_argument("dispatch signature roles do not match the operator");
  }
  if (!contiguous_layout(s.input) || !contiguous_layout(s.weight) || !contiguous_layout(s.output)) {
    return detail::make_status(StatusCode::kUnsupportedLayout,
                               "dispatch requires zero-stride contiguous row-major tensors");
  }
  if (!valid_dtype_signature(request.operator_kind, s) || !all_fp32(s)) {
    return detail::make_status(StatusCode::kUnsupportedDataType,
                               "the requested dtype signature has no kernel");
  }
  if (request.architecture == DeviceArchitecture::kAuto) {
    return detail::invalid_argument("select_kernel requires a resolved architecture");
  }
  if (request.architecture != DeviceArchitecture::kSm100) {
    return detail::make_status(StatusCode::kUnsupportedArchitecture,
                               "libraggedroute_b200 ships sm_100a kernels only");
  }
  const KernelSelection requested = request.requested_kernel;
  if (requested.family == KernelFamily::kAuto && requested.implementation_id != 0) {
    return detail::make_status(StatusCode::kUnsupportedKernelVariant,
                               "automatic kernel selection requires implementation_id=0");
  }
  if (requested.family == KernelFamily::kCudaNaive && requested.implementation_id != 0) {
    return detail::make_status(StatusCode::kUnsupportedKernelVariant,
                               "the naive family has no non-default implementation");
  }
  decision->operator_kind = request.operator_kind;
  decision->architecture = DeviceArchitecture::kSm100;
  if (requested.family == KernelFamily::kCudaOptimized) {
    if (!accepted_optimized_id(request.operator_kind, requested.implementation_id)) {
      return detail::make_status(StatusCode::kUnsupportedKernelVariant,
                                 "requested optimized kernel is not implemented");
    }
    decision->kernel = requested;
    return success_status();
  }
  if (requested.family != KernelFamily::kAuto && requested.family != KernelFamily::kCudaNaive) {
    return detail::make_status(StatusCode::kUnsupportedKernelVariant,
                               "requested kernel family is not implemented");
  }
  if (requested.family == KernelFamily::kAuto && request.operator_kind == OperatorKind::kHistogram) {
    decision->kernel = {KernelFamily::kCudaOptimized, 101};
  } else if (requested.family == KernelFamily::kAuto &&
             request.operator_kind == OperatorKind::kHistogramExclusiveScan) {
    decision->kernel = {KernelFamily::kCudaOptimized, 2};
  } else {
    decision->kernel = {KernelFamily::kCudaNaive, 0};
  }
  return success_status();
}

// ---- workspace queries --------------------------------------------------------

std::size_t get_dense_gemm_workspace_size(const DenseGemmArgs&) noexcept { return 0; }
std::size_t get_topk_gate_workspace_size(const TopKGateArgs&) noexcept { return 0; }
std::size_t get_histogram_workspace_size(const HistogramArgs&) noexcept { return 0; }
std::size_t get_exclusive_scan_workspace_size(const ExclusiveScanArgs&) noexcept { return 0; }
std::size_t get_histogram_exclusive_scan_workspace_size(
    const HistogramExclusiveScanArgs&) noexcept {
  return 0;
}
std::size_t get_grouped_gemm_workspace_size(const GroupedGemmArgs&) noexcept { return 0; }
std::size_t get_unpermute_workspace_size(const UnpermuteArgs&) noexcept { return 0; }

// experts*4 bytes of cursors (src/permute/operator.cpp:17-19), for every
// input size.
std::size_t get_token_permute_workspace_size(const TokenPermuteArgs& args) noexcept {
  return rrb::permute_workspace_bytes(args.tokens, args.experts, args.top_k);
}

// ---- operators -------------------------------------------------------------------

// src/dense_gemm/operator.cpp:18-58.
Status dense_gemm(const DenseGemmArgs& args, const RuntimeContext& context) noexcept {
  if (args.m < 0 || args.n < 0 || args.k < 0) {
    return detail::invalid_argument("dense_gemm dimensions must be non-negative");
  }
  if (args.alpha != 1.0F || args.beta != 0.0F) {
    return detail::invalid_argument("dense_gemm supports alpha=1 and beta=0 only");
  }
  DispatchDecision decision;
  Status status = detail::dispatch_operator(
      OperatorKind::kDenseGemm,
      detail::compute_signature(args.a, args.b, args.accumulator_dtype, args.c), args.kernel,
      context.architecture, &decision);
  if (!status.ok()) return status;
  if (args.m == 0 || args.n == 0) return success_status();
  if (args.c.data == nullptr ||
      (args.k != 0 && (args.a.data == nullptr || args.b.data == nullptr))) {
    return detail::invalid_argument("dense_gemm received a null device pointer");
  }
  if (!detail::is_aligned(args.a.data, alignof(float)) ||
      !detail::is_aligned(args.b.data, alignof(float)) ||
      !detail::is_aligned(args.c.data, alignof(float))) {
    return detail::invalid_argument("dense_gemm FP32 buffers must be 4-byte aligned");
  }
  return detail::cuda_status(
      rrb::launch_grouped_gemm(static_cast<const float*>(args.a.data),
                               static_cast<const float*>(args.b.data), nullptr,
                               static_cast<float*>(args.c.data), 1, args.m, args.k, args.n,
                               context.stream),
      "dense_gemm kernel launch failed");
}

namespace detail {
RR_INTERNAL Status topk_gate_impl(const TopKGateArgs& args, const float* bias,
                      const RuntimeContext& context) noexcept;
}  // namespace detail

// src/topk_gate/operator.cpp:18-60.
Status topk_gate(const TopKGateArgs& args, const RuntimeContext& context) noexcept {
  return detail::topk_gate_impl(args, nullptr, context);
}

Status detail::topk_gate_impl(const TopKGateArgs& args, const float* bias,
                              const RuntimeContext& context) noexcept {
  if (args.tokens < 0 || args.experts < 2 || args.experts > kMaxExperts || args.top_k != 2) {
    return detail::invalid_argument("topk_gate requires tokens>=0, 2<=E<=1024, and top_k=2");
  }
  if (args.normalization != TopKNormalization::kSelectedSoftmax ||
      args.tie_break != TopKTieBreak::kLowerExpertId ||
      args.nan_policy != TopKNaNPolicy::kNegativeInfinityAllNaNFallback01) {
    return detail::invalid_argument("topk_gate received unsupported semantic policy");
  }
  OperatorSignature signature;
  signature.input = args.logits.spec;
  signature.accumulator = args.accumulator_dtype;
  signature.output = args.weights.spec;
  DispatchDecision decision;
  Status status = detail::dispatch_operator(OperatorKind::kTopKGate, signature, args.kernel,
                                            context.architecture, &decision);
  if (!status.ok()) return status;
  if (args.tokens == 0) return success_status();
  if (args.logits.data == nullptr || args.expert_ids == nullptr || args.weights.data == nullptr) {
    return detail::invalid_argument("topk_gate received a null device pointer");
  }
  if (!detail::is_aligned(args.logits.data, alignof(float)) ||
      !detail::is_aligned(args.weights.data, alignof(float))) {
    return detail::invalid_argument("topk_gate FP32 buffers must be 4-byte aligned");
  }
  return detail::cuda_status(
      rrb::launch_topk_gate(static_cast<const float*>(args.logits.data), bias, args.expert_ids,
                            static_cast<float*>(args.weights.data), args.tokens, args.experts,
                            context.stream),
      "topk_gate kernel launch failed");
}

// src/histogram/operator.cpp:20-57. The counts reset is part of the call.
Status histogram(const HistogramArgs& args, const RuntimeContext& context) noexcept {
  if (args.route_pairs < 0 || args.experts <= 0 || args.experts > kMaxExperts) {
    return detail::invalid_argument("histogram requires route_pairs>=0 and 1<=E<=1024");
  }
  DispatchDecision decision;
  Status status = detail::dispatch_operator(OperatorKind::kHistogram, {}, args.kernel,
                                            context.architecture, &decision);
  if (!status.ok()) return status;
  if (args.counts == nullptr || (args.route_pairs != 0 && args.expert_ids == nullptr)) {
    return detail::invalid_argument("histogram received a null device pointer");
  }
  return detail::cuda_status(rrb::launch_histogram(args.expert_ids, args.counts, args.route_pairs,
                                                   args.experts, context.stream),
                             "histogram kernel launch failed");
}

// src/scan/operator.cpp:51-74.
Status exclusive_scan(const ExclusiveScanArgs& args, const RuntimeContext& context) noexcept {
  if (args.experts <= 0 || args.experts > kMaxExperts) {
    return detail::invalid_argument("exclusive_scan requires 1<=E<=1024");
  }
  DispatchDecision decision;
  Status status = detail::dispatch_operator(OperatorKind::kExclusiveScan, {}, args.kernel,
                                            context.architecture, &decision);
  if (!status.ok()) return status;
  if (args.counts == nullptr || args.offsets == nullptr) {
    return detail::invalid_argument("exclusive_scan received a null device pointer");
  }
  if (!detail::is_aligned(args.counts, alignof(std::int32_t)) ||
      !detail::is_aligned(args.offsets, alignof(std::int32_t))) {
    return detail::invalid_argument("exclusive_scan buffers must be 4-byte aligned");
  }
  return detail::cuda_status(
      rrb::launch_exclusive_scan(args.counts, args.offsets, args.experts, context.stream),
      "exclusive_scan kernel launch failed");
}

// src/scan/operator.cpp:84-134. Always the fused kernel; no workspace.
Status histogram_exclusive_scan(const HistogramExclusiveScanArgs& args,
                                const RuntimeContext& context) noexcept {
  if (args.route_pairs < 0 || args.experts <= 0 || args.experts > kMaxExperts) {
    return detail::invalid_argument(
        "histogram_exclusive_scan requires route_pairs>=0 and 1<=E<=1024");
  }
  if (args.counts == nullptr || args.offsets == nullptr ||
      (args.route_pairs != 0 && args.expert_ids == nullptr)) {
    return detail::invalid_argument("histogram_exclusive_scan received a null device pointer");
  }
  if (!detail::is_aligned(args.expert_ids, alignof(std::int32_t)) ||
      !detail::is_aligned(args.counts, alignof(std::int32_t)) ||
      !detail::is_aligned(args.offsets, alignof(std::int32_t))) {
    return detail::invalid_argument("histogram_exclusive_scan buffers must be 4-byte aligned");
  }
  const std::size_t ids_bytes = static_cast<std::size_t>(args.route_pairs) * sizeof(std::int32_t);
  const std::size_t counts_bytes = static_cast<std::size_t>(args.experts) * sizeof(std::int32_t);
  const std::size_t offsets_bytes =
      static_cast<std::size_t>(args.experts + 1) * sizeof(std::int32_t);
  if (detail::ranges_overlap(args.expert_ids, ids_bytes, args.counts, counts_bytes) ||
      detail::ranges_overlap(args.expert_ids, ids_bytes, args.offsets, offsets_bytes) ||
      detail::ranges_overlap(args.counts, counts_bytes, args.offsets, offsets_bytes)) {
    return detail::invalid_argument(
        "histogram_exclusive_scan input and outputs must be pairwise non-overlapping");
  }
  DispatchDecision decision;
  Status status = detail::dispatch_operator(OperatorKind::kHistogramExclusiveScan, {},
                                            args.kernel, context.architecture, &decision);
  if (!status.ok()) return status;
  return detail::cuda_status(
      rrb::launch_histogram_exclusive_scan(args.expert_ids, args.counts, args.offsets,
                                           args.route_pairs, args.experts, context.stream),
      "histogram_exclusive_scan kernel launch failed");
}

// src/permute/operator.cpp:22-83.
Status token_permute(const TokenPermuteArgs& args, const RuntimeContext& context) noexcept {
  if (args.tokens < 0 || args.experts <= 0 || args.experts > kMaxExperts || args.top_k <= 0 ||
      args.top_k > args.experts || args.hidden < 0) {
    return detail::invalid_argument(
        "token_permute requires T>=0, 1<=top_k<=E<=1024, and hidden>=0");
  }
  if (args.tokens > 0 && args.tokens > (std::numeric_limits<int>::max() / args.top_k)) {
    return detail::invalid_argument("token_permute route count exceeds int32 indexing");
  }
  OperatorSignature signature;
  signature.input = args.x.spec;
  signature.output = args.x_permuted.spec;
  DispatchDecision decision;
  Status status = detail::dispatch_operator(OperatorKind::kTokenPermute, signature, args.kernel,
                                            context.architecture, &decision);
  if (!status.ok()) return status;
  if (args.tokens == 0) return success_status();
  if (args.expert_ids == nullptr || args.offsets == nullptr || args.route_pos == nullptr ||
      (args.hidden != 0 && (args.x.data == nullptr || args.x_permuted.data == nullptr))) {
    return detail::invalid_argument("token_permute received a null device pointer");
  }
  if (!detail::is_aligned(args.x.data, alignof(float)) ||
      !detail::is_aligned(args.x_permuted.data, alignof(float))) {
    return detail::invalid_argument("token_permute FP32 buffers must be 4-byte aligned");
  }
  const std::size_t workspace_bytes = get_token_permute_workspace_size(args);
  if (context.workspace == nullptr || context.workspace_bytes < workspace_bytes) {
    return detail::make_status(StatusCode::kInsufficientWorkspace,
                               "token_permute requires the queried int32 cursor workspace");
  }
  if (reinterpret_cast<std::uintptr_t>(context.workspace) % alignof(std::int32_t) != 0) {
    return detail::invalid_argument("token_permute workspace is not int32 aligned");
  }
  return detail::cuda_status(
      rrb::launch_token_permute(static_cast<const float*>(args.x.data), args.expert_ids,
                                args.offsets, static_cast<float*>(args.x_permuted.data),
                                args.route_pos, args.sorted_route, args.tokens, args.experts,
                                args.top_k, args.hidden, context.workspace, context.stream),
      "token_permute kernel launch failed");
}

// src/grouped_gemm/operator.cpp:17-49.
Status grouped_gemm(const GroupedGemmArgs& args, const RuntimeContext& context) noexcept {
  if (args.experts <= 0 || args.experts > kMaxExperts || args.hidden < 0 || args.output < 0 ||
      args.max_expert_tokens < 0) {
    return detail::invalid_argument(
        "grouped_gemm requires 1<=E<=1024 and non-negative dimensions");
  }
  DispatchDecision decision;
  Status status = detail::dispatch_operator(
      OperatorKind::kGroupedGemm,
      detail::compute_signature(args.x_permuted, args.expert_weights, args.accumulator_dtype,
                                args.y_permuted),
      args.kernel, context.architecture, &decision);
  if (!status.ok()) return status;
  status = detail::require_default_family(decision);
  if (!status.ok()) return status;
  if (args.max_expert_tokens == 0 || args.output == 0) return success_status();
  if (args.offsets == nullptr || args.y_permuted.data == nullptr ||
      (args.hidden != 0 &&
       (args.x_permuted.data == nullptr || args.expert_weights.data == nullptr))) {
    return detail::invalid_argument("grouped_gemm received a null device pointer");
  }
  if (!detail::is_aligned(args.x_permuted.data, alignof(float)) ||
      !detail::is_aligned(args.expert_weights.data, alignof(float)) ||
      !detail::is_aligned(args.y_permuted.data, alignof(float))) {
    return detail::invalid_argument("grouped_gemm FP32 buffers must be 4-byte aligned");
  }
  return detail::cuda_status(
      rrb::launch_grouped_gemm(static_cast<const float*>(args.x_permuted.data),
                               static_cast<const float*>(args.expert_weights.data), args.offsets,
                               static_cast<float*>(args.y_permuted.data), args.experts, 0,
                               args.hidden, args.output, context.stream),
      "grouped_gemm kernel launch failed");
}

// src/unpermute/operator.cpp:19-57.
Status unpermute(const UnpermuteArgs& args, const RuntimeContext& context) noexcept {
  if (args.tokens < 0 || args.top_k <= 0 || args.top_k > 64 || args.output < 0) {
    return detail::invalid_argument("unpermute requires tokens>=0, 1<=top_k<=64, and output>=0");
  }
  if (args.tokens > 0 && args.tokens > std::numeric_limits<int>::max() / args.top_k) {
    return detail::invalid_argument("unpermute route count exceeds int32 indexing");
  }
  if (args.tokens > 0 && args.output > 0 &&
      args.tokens > std::numeric_limits<int>::max() / args.output) {
    return detail::invalid_argument("unpermute output count exceeds int32 indexing");
  }
  DispatchDecision decision;
  Status status =
      detail::dispatch_operator(OperatorKind::kUnpermute,
                                detail::compute_signature(args.y_permuted, args.route_weights,
                                                          args.accumulator_dtype, args.y),
                                args.kernel, context.architecture, &decision);
  if (!status.ok()) return status;
  status = detail::require_default_family(decision);
  if (!status.ok()) return status;
  if (args.tokens == 0 || args.output == 0) return success_status();
  if (args.y_permuted.data == nullptr || args.route_pos == nullptr ||
      args.route_weights.data == nullptr || args.y.data == nullptr) {
    return detail::invalid_argument("unpermute received a null device pointer");
  }
  if (!detail::is_aligned(args.y_permuted.data, alignof(float)) ||
      !detail::is_aligned(args.route_weights.data, alignof(float)) ||
      !detail::is_aligned(args.y.data, alignof(float))) {
    return detail::invalid_argument("unpermute FP32 buffers must be 4-byte aligned");
  }
  return detail::cuda_status(
      rrb::launch_unpermute(static_cast<const float*>(args.y_permuted.data), args.route_pos,
                            static_cast<const float*>(args.route_weights.data),
                            static_cast<float*>(args.y.data), args.tokens, args.top_k,
                            args.output, context.stream),
      "unpermute kernel launch failed");
}

// ---- L3 chains (benchmarks/adapters/chain_adapter.cpp:263-467) --------------

// Permute workspace, then (256-byte aligned) room for sorted_route [2T],
// which the row-gathering chains keep there.
std::size_t chain_sorted_route_offset(int tokens, int experts) noexcept {
  const std::size_t p = rrb::permute_workspace_bytes(tokens, experts, 2);
  return (p + 255) & ~static_cast<std::size_t>(255);
}

std::size_t get_chain_workspace_size(int tokens, int, int experts, int) noexcept {
  if (tokens <= 0 || experts <= 0) return 0;
  return chain_sorted_route_offset(tokens, experts) + static_cast<std::size_t>(tokens) * 2 * 4;
}

namespace {

// One NVTX push/pop range per chain stage ("raggedroute_<stage>") around its
// launch, so a profiler can select a stage, e.g. ncu --nvtx --nvtx-include
// "raggedroute_grouped_gemm/" (a '/' in a range name would read as nesting).
// Without a tool attached a range is a null check (NVTX v3, header-only).
class StageRange {
 public:
  explicit StageRange(const char* name) noexcept { nvtxRangePushA(name); }
  ~StageRange() { nvtxRangePop(); }
  StageRange(const StageRange&) = delete;
  StageRange& operator=(const StageRange&) = delete;
};

Status validate_chain_shape(int tokens, int hidden, int experts, int output) noexcept {
  if (tokens < 0 || hidden < 0 || output < 0 || experts < 2 || experts > kMaxExperts) {
    return detail::invalid_argument("chain requires T,K,N>=0 and 2<=E<=1024");
  }
  if (tokens > std::numeric_limits<int>::max() / 2) {
    return detail::invalid_argument("chain route count exceeds int32 indexing");
  }
  const long long routes = 2LL * tokens;
  if (routes * std::max(hidden, output) > std::numeric_limits<int>::max() * 4LL) {
    return detail::invalid_argument("chain tensor exceeds the supported size");
  }
  return success_status();
}

Status chain_after_logits(const float* logits, const float* logit_bias, const float* x,
                          const float* expert_w, const ChainBuffers& b, int tokens, int hidden,
                          int experts, int output, const RuntimeContext& context,
                          bool gather_rows, bool prepared_weights, bool fused_combine) noexcept {
  cudaStream_t stream = context.stream;
  Status s = success_status();
  {
    StageRange r("raggedroute_topk_gate");
    s = detail::cuda_status(rrb::launch_topk_gate(logits, logit_bias, b.expert_ids,
                                                  b.route_weights, tokens, experts, stream),
                            "chain topk_gate launch failed");
  }
  if (!s.ok()) return s;
  const int routes = 2 * tokens;
  {
    StageRange r("raggedroute_histogram_exclusive_scan");
    s = detail::cuda_status(rrb::launch_histogram_exclusive_scan(b.expert_ids, b.counts,
                                                                 b.offsets, routes, experts,
                                                                 stream),
                            "chain histogram_exclusive_scan launch failed");
  }
  if (!s.ok()) return s;
  if (fused_combine) {
    // The permute also records each permuted row's route (in the
    // workspace); the grouped GEMM adds every weighted output row into its
    // token's row of y, so neither y_permuted nor the unpermute launch exist.
    int32_t* sorted_route = reinterpret_cast<int32_t*>(
        static_cast<char*>(context.workspace) + chain_sorted_route_offset(tokens, experts));
    {
      StageRange r("raggedroute_token_permute");
      s = detail::cuda_status(
          rrb::launch_token_permute(x, b.expert_ids, b.offsets, gather_rows ? nullptr : b.x_permuted,
                                    b.route_pos, sorted_route, tokens, experts, 2,
                                    gather_rows ? 0 : hidden, context.workspace, stream),
          "chain token_permute launch failed");
    }
    if (!s.ok()) return s;
    const rrb::RowGather gather{x, sorted_route, 2};
    const float* lo =
        prepared_weights
            ? reinterpret_cast<const float*>(
                  reinterpret_cast<const char*>(expert_w) +
                  rrb::prepared_weights_half_bytes(experts, hidden, output))
            : nullptr;
    StageRange r("raggedroute_grouped_gemm");
    return detail::cuda_status(
        rrb::launch_grouped_gemm_combine(gather_rows ? x : b.x_permuted, expert_w, lo, b.offsets,
                                         sorted_route, b.route_weights, b.y, experts, routes,
                                         tokens, 2, hidden, output, stream,
                                         gather_rows ? &gather : nullptr),
        "chain grouped_gemm (fused combine) launch failed");
  }
  if (gather_rows) {
    // Ranks only (no row copy); the grouped GEMM gathers its rows from x
    // through sorted_route, kept in the workspace.
    int32_t* sorted_route = reinterpret_cast<int32_t*>(
        static_cast<char*>(context.workspace) + chain_sorted_route_offset(tokens, experts));
    {
      StageRange r("raggedroute_token_permute");
      s = detail::cuda_status(
          rrb::launch_token_permute(x, b.expert_ids, b.offsets, nullptr, b.route_pos,
                                    sorted_route, tokens, experts, 2, 0, context.workspace,
                                    stream),
          "chain token_permute launch failed");
    }
    if (!s.ok()) return s;
    const rrb::RowGather gather{x, sorted_route, 2};
    StageRange r("raggedroute_grouped_gemm");
    s = detail::cuda_status(rrb::launch_grouped_gemm(x, expert_w, b.offsets, b.y_permuted,
                                                     experts, routes, hidden, output, stream, 0,
                                                     nullptr, &gather),
                            "chain grouped_gemm launch failed");
  } else {
    {
      StageRange r("raggedroute_token_permute");
      s = detail::cuda_status(
          rrb::launch_token_permute(x, b.expert_ids, b.offsets, b.x_permuted, b.route_pos,
                                    nullptr, tokens, experts, 2, hidden, context.workspace,
                                    stream),
          "chain token_permute launch failed");
    }
    if (!s.ok()) return s;
    StageRange r("raggedroute_grouped_gemm");
    if (prepared_weights) {
      const float* hi = expert_w;
      const float* lo = reinterpret_cast<const float*>(
          reinterpret_cast<const char*>(expert_w) +
          rrb::prepared_weights_half_bytes(experts, hidden, output));
      s = detail::cuda_status(rrb::launch_grouped_gemm_prepared(b.x_permuted, hi, lo, b.offsets,
                                                                b.y_permuted, experts, routes,
                                                                hidden, output, stream),
                              "chain grouped_gemm (prepared weights) launch failed");
    } else {
      s = detail::cuda_status(rrb::launch_grouped_gemm(b.x_permuted, expert_w, b.offsets,
                                                       b.y_permuted, experts, routes, hidden,
                                                       output, stream),
                              "chain grouped_gemm launch failed");
    }
  }
  if (!s.ok()) return s;
  StageRange r("raggedroute_unpermute");
  return detail::cuda_status(rrb::launch_unpermute(b.y_permuted, b.route_pos, b.route_weights,
                                                   b.y, tokens, 2, output, stream),
                             "chain unpermute launch failed");
}

Status validate_chain_buffers(const ChainBuffers& b, bool need_logits, int hidden,
                              int output, bool gather_rows, bool fused_combine) noexcept {
  if ((need_logits && b.logits == nullptr) || b.expert_ids == nullptr ||
      b.route_weights == nullptr || b.counts == nullptr || b.offsets == nullptr ||
      b.route_pos == nullptr ||
      (output > 0 && (b.y == nullptr || (!fused_combine && b.y_permuted == nullptr))) ||
      (hidden > 0 && !gather_rows && b.x_permuted == nullptr)) {
    return detail::invalid_argument("chain received a null device buffer");
  }
  return success_status();
}

// Prepared expert weights: the tcgen05 engine only (no FP32 fallback reads
// that layout), so the shapes and buffers TMA needs are required up front.
Status validate_prepared(bool prepared, bool gather_rows, bool fused_combine,
                         const void* weights, const ChainBuffers& b, int hidden,
                         int output) noexcept {
  if (!prepared) return success_status();
  if (gather_rows) {
    return detail::make_status(StatusCode::kUnsupportedKernelVariant,
                               "prepared expert weights do not combine with row gathering");
  }
  // The prepared engine stores into y_permuted, or adds into y when the
  // combine is fused.
  const float* out = fused_combine ? b.y : b.y_permuted;
  if (hidden % 4 != 0 || output % 4 != 0 || !rrb::aligned_to(weights, 256) ||
      !rrb::aligned_to(b.x_permuted, 16) || !rrb::aligned_to(out, 16)) {
    return detail::invalid_argument(
        "prepared expert weights need K and N multiples of 4, a 256-byte aligned prepared "
        "buffer and 16-byte aligned x_permuted / y_permuted (y with a fused combine)");
  }
  return success_status();
}

Status resolve_chain_architecture(const RuntimeContext& context) noexcept {
  DeviceArchitecture arch = DeviceArchitecture::kOther;
  Status s = resolve_device_architecture(context.architecture, &arch);
  if (!s.ok()) return s;
  if (arch != DeviceArchitecture::kSm100) {
    return detail::make_status(StatusCode::kUnsupportedArchitecture,
                               "libraggedroute_b200 ships sm_100a kernels only");
  }
  return success_status();
}

}  // namespace

// Architecture check shared by the library's own (non-reference) entry
// points: B200 (CC 10.0) only.
RR_INTERNAL Status detail_resolve_sm100(const RuntimeContext& context) noexcept {
  return resolve_chain_architecture(context);
}

Status chain_from_tokens(const ChainFromTokensArgs& args, const RuntimeContext& context) noexcept {
  Status s = validate_chain_shape(args.tokens, args.hidden, args.experts, args.output);
  if (!s.ok()) return s;
  s = resolve_chain_architecture(context);
  if (!s.ok()) return s;
  if (args.tokens == 0) return success_status();
  if (args.x == nullptr && args.hidden > 0) return detail::invalid_argument("chain x is null");
  if (args.router_weights == nullptr && args.hidden > 0) {
    return detail::invalid_argument("chain router weights are null");
  }
  if (args.expert_weights == nullptr && args.hidden > 0 && args.output > 0) {
    return detail::invalid_argument("chain expert weights are null");
  }
  s = validate_chain_buffers(args.buffers, true, args.hidden, args.output, args.gather_rows,
                             args.fused_combine);
  if (!s.ok()) return s;
  s = validate_prepared(args.prepared_weights, args.gather_rows, args.fused_combine,
                        args.expert_weights, args.buffers, args.hidden, args.output);
  if (!s.ok()) return s;
  const std::size_t need = get_chain_workspace_size(args.tokens, args.hidden, args.experts,
                                                    args.output);
  if (context.workspace == nullptr || context.workspace_bytes < need) {
    return detail::make_status(StatusCode::kInsufficientWorkspace,
                               "chain requires the queried workspace");
  }
  {
    StageRange r("raggedroute_dense_gemm");
    s = detail::cuda_status(
        rrb::launch_grouped_gemm(args.x, args.router_weights, nullptr, args.buffers.logits, 1,
                                 args.tokens, args.hidden, args.experts, context.stream),
        "chain dense_gemm launch failed");
  }
  if (!s.ok()) return s;
  return chain_after_logits(args.buffers.logits, args.logit_bias, args.x, args.expert_weights,
                            args.buffers, args.tokens, args.hidden, args.experts, args.output,
                            context, args.gather_rows, args.prepared_weights,
                            args.fused_combine);
}

Status chain_from_logits(const ChainFromLogitsArgs& args, const RuntimeContext& context) noexcept {
  Status s = validate_chain_shape(args.tokens, args.hidden, args.experts, args.output);
  if (!s.ok()) return s;
  s = resolve_chain_architecture(context);
  if (!s.ok()) return s;
  if (args.tokens == 0) return success_status();
  if (args.logits == nullptr) return detail::invalid_argument("chain logits are null");
  if (args.x == nullptr && args.hidden > 0) return detail::invalid_argument("chain x is null");
  if (args.expert_weights == nullptr && args.hidden > 0 && args.output > 0) {
    return detail::invalid_argument("chain expert weights are null");
  }
  s = validate_chain_buffers(args.buffers, false, args.hidden, args.output, args.gather_rows,
                             args.fused_combine);
  if (!s.ok()) return s;
  s = validate_prepared(args.prepared_weights, args.gather_rows, args.fused_combine,
                        args.expert_weights, args.buffers, args.hidden, args.output);
  if (!s.ok()) return s;
  const std::size_t need = get_chain_workspace_size(args.tokens, args.hidden, args.experts,
                                                    args.output);
  if (context.workspace == nullptr || context.workspace_bytes < need) {
    return detail::make_status(StatusCode::kInsufficientWorkspace,
                               "chain requires the queried workspace");
  }
  return chain_after_logits(args.logits, nullptr, args.x, args.expert_weights, args.buffers,
                            args.tokens, args.hidden, args.experts, args.output, context,
                            args.gather_rows, args.prepared_weights, args.fused_combine);
}

std::size_t get_route_chain_workspace_size(int tokens, int top_k, int experts) noexcept {
  if (tokens <= 0 || top_k <= 0 || experts <= 0) return 0;
  return rrb::permute_workspace_bytes(tokens, experts, top_k);
}

// Post-route chain: benchmarks/adapters/postroute_chain_adapter.cpp:240-354
// (histogram + scan, token_permute with sorted_route, grouped GEMM,
// unpermute) with the B200 kernels. top_k in [1, 8] (the reference's suite
// runs 2, 4 and 8); route ids outside [0, E) are outside the contract and
// are skipped by every stage.
Status chain_from_route_ids(const ChainFromRouteIdsArgs& args,
                            const RuntimeContext& context) noexcept {
  if (args.top_k < 1 || args.top_k > 8 || args.top_k > args.experts) {
    return detail::invalid_argument("chain_from_route_ids requires 1<=top_k<=min(8,E)");
  }
  if (args.fused_combine && args.top_k > 2) {
    return detail::make_status(StatusCode::kUnsupportedKernelVariant,
                               "a fused combine needs top_k <= 2");
  }
  if (args.tokens < 0 || args.hidden < 0 || args.output < 0 || args.experts < 2 ||
      args.experts > kMaxExperts) {
    return detail::invalid_argument("chain requires T,K,N>=0 and 2<=E<=1024");
  }
  const long long routes = static_cast<long long>(args.tokens) * args.top_k;
  if (routes > std::numeric_limits<int>::max() ||
      routes * std::max(args.hidden, args.output) > std::numeric_limits<int>::max() * 4LL) {
    return detail::invalid_argument("chain tensor exceeds the supported size");
  }
  Status s = resolve_chain_architecture(context);
  if (!s.ok()) return s;
  const RouteChainBuffers& b = args.buffers;
  if (b.counts == nullptr || b.offsets == nullptr) {
    return detail::invalid_argument("chain received a null device buffer");
  }
  if (args.tokens > 0) {
    if (args.expert_ids == nullptr || args.route_weights == nullptr ||
        b.route_pos == nullptr ||
        (args.hidden > 0 &&
         (args.x == nullptr || (!args.gather_rows && b.x_permuted == nullptr) ||
          (args.gather_rows && b.sorted_route == nullptr))) ||
        (args.output > 0 &&
         (b.y == nullptr || (!args.fused_combine && b.y_permuted == nullptr) ||
          (args.fused_combine && b.sorted_route == nullptr))) ||
        (args.hidden > 0 && args.output > 0 && args.expert_weights == nullptr)) {
      return detail::invalid_argument("chain received a null device buffer");
    }
  }
  const std::size_t need = get_route_chain_workspace_size(args.tokens, args.top_k, args.experts);
  if (need > 0 && (context.workspace == nullptr || context.workspace_bytes < need)) {
    return detail::make_status(StatusCode::kInsufficientWorkspace,
                               "chain requires the queried workspace");
  }
  cudaStream_t stream = context.stream;
  const int r = static_cast<int>(routes);
  s = detail::cuda_status(rrb::launch_histogram_exclusive_scan(args.expert_ids, b.counts,
                                                               b.offsets, r, args.experts, stream),
                          "chain histogram_exclusive_scan launch failed");
  if (!s.ok() || args.tokens == 0) return s;
  const bool gather = args.gather_rows && args.hidden > 0;
  s = detail::cuda_status(
      rrb::launch_token_permute(args.x, args.expert_ids, b.offsets, gather ? nullptr : b.x_permuted,
                                b.route_pos, b.sorted_route, args.tokens, args.experts,
                                args.top_k, gather ? 0 : args.hidden, context.workspace, stream),
      "chain token_permute launch failed");
  if (!s.ok() || args.output == 0) return s;
  if (args.fused_combine) {
    const rrb::RowGather g{args.x, b.sorted_route, args.top_k};
    return detail::cuda_status(
        rrb::launch_grouped_gemm_combine(gather ? args.x : b.x_permuted, args.expert_weights,
                                         nullptr, b.offsets, b.sorted_route, args.route_weights,
                                         b.y, args.experts, r, args.tokens, args.top_k,
                                         args.hidden, args.output, stream,
                                         gather ? &g : nullptr),
        "chain grouped_gemm (fused combine) launch failed");
  }
  if (gather) {
    const rrb::RowGather g{args.x, b.sorted_route, args.top_k};
    s = detail::cuda_status(rrb::launch_grouped_gemm(args.x, args.expert_weights, b.offsets,
                                                     b.y_permuted, args.experts, r, args.hidden,
                                                     args.output, stream, 0, nullptr, &g),
                            "chain grouped_gemm launch failed");
  } else {
    s = detail::cuda_status(rrb::launch_grouped_gemm(b.x_permuted, args.expert_weights,
                                                     b.offsets, b.y_permuted, args.experts, r,
                                                     args.hidden, args.output, stream),
                            "chain grouped_gemm launch failed");
  }
  if (!s.ok()) return s;
  return detail::cuda_status(rrb::launch_unpermute(b.y_permuted, b.route_pos, args.route_weights,
                                                   b.y, args.tokens, args.top_k, args.output,
                                                   stream),
                             "chain unpermute launch failed");
}

// ---- low-level launchers (include/raggedroute/baseline_ops.h:14-42) ----------

namespace ops {

// src/dense_gemm/cuda_naive/baseline.cu:42-58.
cudaError_t launch_dense_gemm_naive(const float* a, const float* b, float* c, int m, int n, int k,
                                    cudaStream_t caller_stream) {
  if (m < 0 || n < 0 || k < 0) return cudaErrorInvalidValue;
  if (m == 0 || n == 0) return cudaSuccess;
  if (c == nullptr || (k != 0 && (a == nullptr || b == nullptr))) return cudaErrorInvalidValue;
  return rrb::launch_grouped_gemm(a, b, nullptr, c, 1, m, k, n, caller_stream);
}

// src/topk_gate/cuda_naive/baseline.cu:90-105.
cudaError_t launch_topk_gate_naive(const float* logits, std::int32_t* expert_ids, float* weights,
                                   int tokens, int experts, cudaStream_t caller_stream) {
  if (tokens < 0 || experts < 2 || experts > kMaxExperts) return cudaErrorInvalidValue;
  if (tokens == 0) return cudaSuccess;
  if (logits == nullptr || expert_ids == nullptr || weights == nullptr) {
    return cudaErrorInvalidValue;
  }
  return rrb::launch_topk_gate(logits, nullptr, expert_ids, weights, tokens, experts,
                               caller_stream);
}

// src/histogram/cuda_naive/baseline.cu:37-52. Accumulates into counts.
cudaError_t launch_histogram_naive(const std::int32_t* expert_ids, std::int32_t* counts,
                                   int route_pairs, int experts, cudaStream_t caller_stream) {
  if (route_pairs < 0 || experts <= 0 || experts > kMaxExperts) return cudaErrorInvalidValue;
  if (route_pairs == 0) return cudaSuccess;
  if (expert_ids == nullptr || counts == nullptr) return cudaErrorInvalidValue;
  return rrb::launch_histogram_accumulate(expert_ids, counts, route_pairs, experts,
                                          caller_stream);
}

// src/scan/cuda_naive/baseline.cu:30-38.
cudaError_t launch_exclusive_scan_naive(const std::int32_t* counts, std::int32_t* offsets,
                                        int experts, cudaStream_t caller_stream) {
  if (experts <= 0 || experts > kMaxExperts || offsets == nullptr || counts == nullptr) {
    return cudaErrorInvalidValue;
  }
  return rrb::launch_exclusive_scan(counts, offsets, experts, caller_stream);
}

// src/permute/cuda_naive/baseline.cu:38-55. Cursors accumulate the per-expert
// counts; the slot order is the stable one.
cudaError_t launch_token_permute_naive(const float* x, const std::int32_t* expert_ids,
                                       const std::int32_t* offsets, std::int32_t* cursors,
                                       float* x_permuted, std::int32_t* route_pos,
                                       std::int32_t* sorted_route, int tokens, int top_k,
                                       int hidden, cudaStream_t caller_stream) {
  if (tokens < 0 || top_k <= 0 || hidden < 0) return cudaErrorInvalidValue;
  if (tokens == 0) return cudaSuccess;
  if (tokens > std::numeric_limits<int>::max() / top_k) return cudaErrorInvalidValue;
  if (expert_ids == nullptr || offsets == nullptr || cursors == nullptr || route_pos == nullptr ||
      (hidden != 0 && (x == nullptr || x_permuted == nullptr))) {
    return cudaErrorInvalidValue;
  }
  return rrb::launch_token_permute_cursor(x, expert_ids, offsets, cursors, x_permuted, route_pos,
                                          sorted_route, tokens, top_k, hidden, caller_stream);
}

// src/grouped_gemm/cuda_naive/baseline.cu:35-57.
cudaError_t launch_grouped_gemm_naive(const float* x_permuted, const float* expert_weights,
                                      const std::int32_t* offsets, float* y_permuted, int experts,
                                      int hidden, int output, int max_expert_tokens,
                                      cudaStream_t caller_stream) {
  if (experts <= 0 || experts > kMaxExperts || hidden < 0 || output < 0 ||
      max_expert_tokens < 0) {
    return cudaErrorInvalidValue;
  }
  if (max_expert_tokens == 0 || output == 0) return cudaSuccess;
  if (offsets == nullptr || y_permuted == nullptr ||
      (hidden != 0 && (x_permuted == nullptr || expert_weights == nullptr))) {
    return cudaErrorInvalidValue;
  }
  return rrb::launch_grouped_gemm(x_permuted, expert_weights, offsets, y_permuted, experts, 0,
                                  hidden, output, caller_stream);
}

// Research entry point of the reference's post-route gather chain
// (src/grouped_gemm/cuda_candidate/grouped_optimized_internal.h:105-109):
// row r of segment e is x[sorted_route[r] / top_k] . W[e]. The workspace is
// not needed here (accepted and ignored).
cudaError_t launch_grouped_gemm_sm86_fp32_gather_v1(
    const float* x, const std::int32_t* sorted_route, int top_k, const float* expert_weights,
    const std::int32_t* offsets, float* y_permuted, int experts, int hidden, int output,
    int max_expert_tokens, void*, std::size_t, cudaStream_t caller_stream) {
  if (experts <= 0 || experts > kMaxExperts || hidden < 0 || output < 0 ||
      max_expert_tokens < 0 || top_k < 1) {
    return cudaErrorInvalidValue;
  }
  if (output == 0 || max_expert_tokens == 0) return cudaSuccess;
  if (offsets == nullptr || y_permuted == nullptr ||
      (hidden > 0 && (x == nullptr || sorted_route == nullptr || expert_weights == nullptr))) {
    return cudaErrorInvalidValue;
  }
  const rrb::RowGather gather{x, sorted_route, top_k};
  return rrb::launch_grouped_gemm(x, expert_weights, offsets, y_permuted, experts, 0, hidden,
                                  output, caller_stream, 0, nullptr, hidden > 0 ? &gather : nullptr);
}

// src/unpermute/cuda_naive/baseline.cu:33-50.
cudaError_t launch_unpermute_naive(const float* y_permuted, const std::int32_t* route_pos,
                                   const float* route_weights, float* y, int tokens, int top_k,
                                   int output, cudaStream_t caller_stream) {
  if (tokens < 0 || top_k <= 0 || output < 0) return cudaErrorInvalidValue;
  if (tokens == 0 || output == 0) return cudaSuccess;
  if (tokens > std::numeric_limits<int>::max() / top_k) return cudaErrorInvalidValue;
  if (tokens > std::numeric_limits<int>::max() / output) return cudaErrorInvalidValue;
  if (y_permuted == nullptr || route_pos == nullptr || route_weights == nullptr || y == nullptr) {
    return cudaErrorInvalidValue;
  }
  return rrb::launch_unpermute(y_permuted, route_pos, route_weights, y, tokens, top_k, output,
                               caller_stream);
}

// src/benchmark/cache_scrub.cu:38-50.
cudaError_t launch_cache_scrub(std::uint32_t* buffer, std::size_t elements,
                               cudaStream_t caller_stream) {
  if (elements == 0) return cudaSuccess;
  if (buffer == nullptr) return cudaErrorInvalidValue;
  return rrb::launch_cache_scrub(buffer, elements, caller_stream);
}

}  // namespace ops
}  // namespace raggedroute

// ---- C ABI ----------------------------------------------------------------------

namespace {

using raggedroute::Status;

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

rr_status to_c(const Status& s) {
  rr_status out;
  out.code = static_cast<int32_t>(s.code);
  out.cuda_error = static_cast<int32_t>(s.cuda_error);
  out.message = s.message;
  return out;
}

rr_status null_context() {
  return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
               "rr_context must not be null"});
}

raggedroute::RuntimeContext to_runtime(const rr_context* ctx) {
  raggedroute::RuntimeContext r;
  r.stream = static_cast<cudaStream_t>(ctx->stream);
  r.workspace = ctx->workspace;
  r.workspace_bytes = ctx->workspace_bytes;
  r.architecture = static_cast<raggedroute::DeviceArchitecture>(ctx->architecture);
  return r;
}

raggedroute::KernelSelection to_kernel(const rr_context* ctx) {
  raggedroute::KernelSelection k;
  k.family = static_cast<raggedroute::KernelFamily>(ctx->kernel_family);
  k.implementation_id = ctx->implementation_id;
  return k;
}

}  // namespace

extern "C" {

rr_status rr_dense_gemm(const float* a, const float* b, float* c, int m, int n, int k,
                        const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::DenseGemmArgs args;
  args.a.data = a;
  args.b.data = b;
  args.c.data = c;
  args.m = m;
  args.n = n;
  args.k = k;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::dense_gemm(args, to_runtime(ctx)));
}
size_t rr_dense_gemm_workspace_size(int, int, int) { return 0; }

rr_status rr_topk_gate(const float* logits, int32_t* expert_ids, float* weights, int tokens,
                       int experts, int top_k, const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::TopKGateArgs args;
  args.logits.data = logits;
  args.expert_ids = expert_ids;
  args.weights.data = weights;
  args.tokens = tokens;
  args.experts = experts;
  args.top_k = top_k;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::topk_gate(args, to_runtime(ctx)));
}
size_t rr_topk_gate_workspace_size(int, int) { return 0; }

rr_status rr_topk_gate_biased(const float* logits, const float* logit_bias, int32_t* expert_ids,
                              float* weights, int tokens, int experts, int top_k,
                              const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  if (logit_bias != nullptr && reinterpret_cast<std::uintptr_t>(logit_bias) % 4 != 0) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "topk_gate bias must be 4-byte aligned"});
  }
  raggedroute::TopKGateArgs args;
  args.logits.data = logits;
  args.expert_ids = expert_ids;
  args.weights.data = weights;
  args.tokens = tokens;
  args.experts = experts;
  args.top_k = top_k;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::detail::topk_gate_impl(args, logit_bias, to_runtime(ctx)));
}

rr_status rr_histogram(const int32_t* expert_ids, int32_t* counts, int route_pairs, int experts,
                       const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::HistogramArgs args;
  args.expert_ids = expert_ids;
  args.counts = counts;
  args.route_pairs = route_pairs;
  args.experts = experts;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::histogram(args, to_runtime(ctx)));
}
size_t rr_histogram_workspace_size(int, int) { return 0; }

rr_status rr_exclusive_scan(const int32_t* counts, int32_t* offsets, int experts,
                            const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::ExclusiveScanArgs args;
  args.counts = counts;
  args.offsets = offsets;
  args.experts = experts;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::exclusive_scan(args, to_runtime(ctx)));
}
size_t rr_exclusive_scan_workspace_size(int) { return 0; }

rr_status rr_histogram_exclusive_scan(const int32_t* expert_ids, int32_t* counts,
                                      int32_t* offsets, int route_pairs, int experts,
                                      const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::HistogramExclusiveScanArgs args;
  args.expert_ids = expert_ids;
  args.counts = counts;
  args.offsets = offsets;
  args.route_pairs = route_pairs;
  args.experts = experts;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::histogram_exclusive_scan(args, to_runtime(ctx)));
}
size_t rr_histogram_exclusive_scan_workspace_size(int, int) { return 0; }

rr_status rr_token_permute(const float* x, const int32_t* expert_ids, const int32_t* offsets,
                           float* x_permuted, int32_t* route_pos, int32_t* sorted_route,
                           int tokens, int experts, int top_k, int hidden,
                           const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::TokenPermuteArgs args;
  args.x.data = x;
  args.expert_ids = expert_ids;
  args.offsets = offsets;
  args.x_permuted.data = x_permuted;
  args.route_pos = route_pos;
  args.sorted_route = sorted_route;
  args.tokens = tokens;
  args.experts = experts;
  args.top_k = top_k;
  args.hidden = hidden;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::token_permute(args, to_runtime(ctx)));
}
size_t rr_token_permute_workspace_size(int tokens, int experts, int top_k, int hidden) {
  raggedroute::TokenPermuteArgs args;
  args.tokens = tokens;
  args.experts = experts;
  args.top_k = top_k;
  args.hidden = hidden;
  return raggedroute::get_token_permute_workspace_size(args);
}

rr_status rr_grouped_gemm(const float* x_permuted, const float* expert_weights,
                          const int32_t* offsets, float* y_permuted, int experts, int hidden,
                          int output, int max_expert_tokens, const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::GroupedGemmArgs args;
  args.x_permuted.data = x_permuted;
  args.expert_weights.data = expert_weights;
  args.offsets = offsets;
  args.y_permuted.data = y_permuted;
  args.experts = experts;
  args.hidden = hidden;
  args.output = output;
  args.max_expert_tokens = max_expert_tokens;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::grouped_gemm(args, to_runtime(ctx)));
}
size_t rr_grouped_gemm_workspace_size(int, int, int) { return 0; }

rr_status rr_grouped_gemm_gather(const float* x, const int32_t* sorted_route, int top_k,
                                 const float* expert_weights, const int32_t* offsets,
                                 float* y_permuted, int route_pairs, int hidden, int experts,
                                 int output, const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  const raggedroute::Status a = raggedroute::detail_resolve_sm100(to_runtime(ctx));
  if (!a.ok()) return to_c(a);
  const cudaError_t e = raggedroute::ops::launch_grouped_gemm_sm86_fp32_gather_v1(
      x, sorted_route, top_k, expert_weights, offsets, y_permuted, experts, hidden, output,
      route_pairs, nullptr, 0, as_stream(ctx->stream));
  if (e == cudaErrorInvalidValue) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, e,
                 "grouped_gemm_gather requires 1<=E<=1024, top_k>=1 and device buffers"});
  }
  if (e != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, e, "grouped_gemm_gather launch failed"});
  }
  return to_c(raggedroute::success_status());
}

rr_status rr_grouped_gemm_combine(const float* x_permuted, const float* expert_weights,
                                  const int32_t* offsets, const int32_t* sorted_route,
                                  const float* route_weights, float* y, int experts, int hidden,
                                  int output, int route_pairs, int tokens, int top_k,
                                  const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  if (experts <= 0 || experts > rrb::kMaxExperts || hidden < 0 || output < 0 ||
      route_pairs < 0 || tokens < 0 || top_k < 1 ||
      static_cast<long long>(tokens) * top_k < route_pairs) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "grouped_gemm_combine requires 1<=E<=1024, K, N, R, T >= 0 and R <= T*top_k"});
  }
  if (top_k > 2) {
    return to_c({raggedroute::StatusCode::kUnsupportedKernelVariant, cudaSuccess,
                 "a fused combine needs top_k <= 2"});
  }
  if (tokens == 0 || output == 0) return to_c(raggedroute::success_status());
  if (y == nullptr || (route_pairs > 0 && (offsets == nullptr || sorted_route == nullptr ||
                                           route_weights == nullptr ||
                                           (hidden > 0 && (x_permuted == nullptr ||
                                                           expert_weights == nullptr))))) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "grouped_gemm_combine received a null device buffer"});
  }
  const raggedroute::Status a = raggedroute::detail_resolve_sm100(to_runtime(ctx));
  if (!a.ok()) return to_c(a);
  const cudaError_t e = rrb::launch_grouped_gemm_combine(
      x_permuted, expert_weights, nullptr, offsets, sorted_route, route_weights, y, experts,
      route_pairs, tokens, top_k, hidden, output, as_stream(ctx->stream));
  if (e != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, e, "grouped_gemm_combine launch failed"});
  }
  return to_c(raggedroute::success_status());
}

rr_status rr_grouped_gemm_scatter(const float* x_permuted, const float* expert_weights,
                                  const int32_t* offsets, const int64_t* row_address,
                                  float* const* bases, int nbases, int64_t row_limit,
                                  int experts, int hidden, int output, int route_pairs,
                                  const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  if (experts <= 0 || experts > rrb::kMaxExperts || hidden < 0 || output < 0 ||
      route_pairs < 0 || nbases < 0 || row_limit < 0) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "grouped_gemm_scatter requires 1<=E<=1024 and K, N, R, nbases, row_limit >= 0"});
  }
  if (route_pairs == 0 || output == 0) return to_c(raggedroute::success_status());
  if (offsets == nullptr || row_address == nullptr || (nbases > 0 && bases == nullptr) ||
      (hidden > 0 && (x_permuted == nullptr || expert_weights == nullptr))) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "grouped_gemm_scatter received a null device buffer"});
  }
  const raggedroute::Status a = raggedroute::detail_resolve_sm100(to_runtime(ctx));
  if (!a.ok()) return to_c(a);
  rrb::RowScatter sc;
  sc.dst = row_address;
  sc.base = bases;
  sc.nranks = nbases;
  sc.row_limit = row_limit;
  // y is only the engine's alignment witness here: every stored row goes to
  // a resolved address.
  const cudaError_t e = rrb::launch_grouped_gemm(x_permuted, expert_weights, offsets, nullptr,
                                                 experts, route_pairs, hidden, output,
                                                 as_stream(ctx->stream), 0, &sc);
  if (e != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, e, "grouped_gemm_scatter launch failed"});
  }
  return to_c(raggedroute::success_status());
}

rr_status rr_unpermute(const float* y_permuted, const int32_t* route_pos,
                       const float* route_weights, float* y, int tokens, int top_k, int output,
                       const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::UnpermuteArgs args;
  args.y_permuted.data = y_permuted;
  args.route_pos = route_pos;
  args.route_weights.data = route_weights;
  args.y.data = y;
  args.tokens = tokens;
  args.top_k = top_k;
  args.output = output;
  args.kernel = to_kernel(ctx);
  return to_c(raggedroute::unpermute(args, to_runtime(ctx)));
}
size_t rr_unpermute_workspace_size(int, int, int) { return 0; }

// Chains read ctx->implementation_id as bits: RR_CHAIN_IMPL_GATHER_ROWS
// gathers the grouped GEMM's rows from x, RR_CHAIN_IMPL_PREPARED_WEIGHTS
// (token and logit chains, where `prepared` is given) takes expert_weights
// as a buffer from rr_prepare_expert_weights, RR_CHAIN_IMPL_FUSED_COMBINE
// fuses the unpermute into the grouped GEMM. Unknown bits are rejected here;
// gather with prepared weights by the chain's own validation.
rr_status chain_impl(const rr_context* ctx, bool* gather_rows, bool* fused_combine,
                     bool* prepared = nullptr) {
  const uint32_t id = ctx->implementation_id;
  const uint32_t known = RR_CHAIN_IMPL_GATHER_ROWS | RR_CHAIN_IMPL_FUSED_COMBINE |
                         (prepared != nullptr ? RR_CHAIN_IMPL_PREPARED_WEIGHTS : 0u);
  if ((id & ~known) != 0) {
    return to_c({raggedroute::StatusCode::kUnsupportedKernelVariant, cudaSuccess,
                 "unknown chain implementation id"});
  }
  *gather_rows = (id & RR_CHAIN_IMPL_GATHER_ROWS) != 0;
  *fused_combine = (id & RR_CHAIN_IMPL_FUSED_COMBINE) != 0;
  if (prepared != nullptr) *prepared = (id & RR_CHAIN_IMPL_PREPARED_WEIGHTS) != 0;
  return to_c(raggedroute::success_status());
}

size_t rr_prepared_expert_weights_size(int experts, int hidden, int output) {
  if (experts <= 0 || hidden <= 0 || output <= 0) return 0;
  return 2 * rrb::prepared_weights_half_bytes(experts, hidden, output);
}

rr_status rr_prepare_expert_weights(const float* expert_weights, int experts, int hidden,
                                    int output, void* prepared, size_t prepared_bytes,
                                    const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  if (experts <= 0 || experts > rrb::kMaxExperts || hidden <= 0 || output <= 0 ||
      hidden % 4 != 0 || output % 4 != 0) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "prepare_expert_weights requires 1<=E<=1024 and K, N positive multiples of 4"});
  }
  if (expert_weights == nullptr || prepared == nullptr || !rrb::aligned_to(prepared, 256)) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "prepare_expert_weights needs the weights and a 256-byte aligned buffer"});
  }
  if (prepared_bytes < rr_prepared_expert_weights_size(experts, hidden, output)) {
    return to_c({raggedroute::StatusCode::kInsufficientWorkspace, cudaSuccess,
                 "prepared buffer is smaller than rr_prepared_expert_weights_size"});
  }
  const raggedroute::Status a = raggedroute::detail_resolve_sm100(to_runtime(ctx));
  if (!a.ok()) return to_c(a);
  float* hi = static_cast<float*>(prepared);
  float* lo = reinterpret_cast<float*>(static_cast<char*>(prepared) +
                                       rrb::prepared_weights_half_bytes(experts, hidden, output));
  const cudaError_t e = rrb::launch_prepare_weights(expert_weights, hi, lo, experts, hidden,
                                                    output, as_stream(ctx->stream));
  if (e != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, e, "prepare_expert_weights launch failed"});
  }
  return to_c(raggedroute::success_status());
}

rr_status rr_grouped_gemm_prepared(const float* x_permuted, const void* prepared,
                                   const int32_t* offsets, float* y_permuted, int experts,
                                   int hidden, int output, int route_pairs,
                                   const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  if (experts <= 0 || experts > rrb::kMaxExperts || hidden <= 0 || output <= 0 ||
      hidden % 4 != 0 || output % 4 != 0 || route_pairs < 0) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "grouped_gemm_prepared requires 1<=E<=1024, K, N positive multiples of 4"});
  }
  if (route_pairs == 0) return to_c(raggedroute::success_status());
  if (x_permuted == nullptr || prepared == nullptr || offsets == nullptr ||
      y_permuted == nullptr || !rrb::aligned_to(prepared, 256)) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "grouped_gemm_prepared received a null or misaligned buffer"});
  }
  const raggedroute::Status a = raggedroute::detail_resolve_sm100(to_runtime(ctx));
  if (!a.ok()) return to_c(a);
  const float* hi = static_cast<const float*>(prepared);
  const float* lo = reinterpret_cast<const float*>(
      static_cast<const char*>(prepared) +
      rrb::prepared_weights_half_bytes(experts, hidden, output));
  const cudaError_t e = rrb::launch_grouped_gemm_prepared(
      x_permuted, hi, lo, offsets, y_permuted, experts, route_pairs, hidden, output,
      as_stream(ctx->stream));
  if (e == cudaErrorInvalidValue) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, e,
                 "grouped_gemm_prepared needs 16-byte aligned x_permuted / y_permuted"});
  }
  if (e != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, e, "grouped_gemm_prepared launch failed"});
  }
  return to_c(raggedroute::success_status());
}

rr_status rr_chain_from_tokens(const float* x, const float* router_weights,
                               const float* logit_bias, const float* expert_weights,
                               float* logits, int32_t* expert_ids, float* route_weights,
                               int32_t* counts, int32_t* offsets, float* x_permuted,
                               int32_t* route_pos, float* y_permuted, float* y, int tokens,
                               int hidden, int experts, int output, const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::ChainFromTokensArgs args;
  args.x = x;
  args.router_weights = router_weights;
  args.logit_bias = logit_bias;
  args.expert_weights = expert_weights;
  args.buffers = {logits, expert_ids, route_weights, counts, offsets, x_permuted,
                  route_pos, y_permuted, y};
  args.tokens = tokens;
  args.hidden = hidden;
  args.experts = experts;
  args.output = output;
  const rr_status impl =
      chain_impl(ctx, &args.gather_rows, &args.fused_combine, &args.prepared_weights);
  if (impl.code != RR_SUCCESS) return impl;
  return to_c(raggedroute::chain_from_tokens(args, to_runtime(ctx)));
}

rr_status rr_chain_from_route_ids(const float* x, const int32_t* expert_ids,
                                  const float* route_weights, const float* expert_weights,
                                  int32_t* counts, int32_t* offsets, float* x_permuted,
                                  int32_t* route_pos, int32_t* sorted_route, float* y_permuted,
                                  float* y, int tokens, int top_k, int hidden, int experts,
                                  int output, const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::ChainFromRouteIdsArgs args;
  args.x = x;
  args.expert_ids = expert_ids;
  args.route_weights = route_weights;
  args.expert_weights = expert_weights;
  args.buffers = {counts, offsets, x_permuted, route_pos, sorted_route, y_permuted, y};
  args.tokens = tokens;
  args.top_k = top_k;
  args.hidden = hidden;
  args.experts = experts;
  args.output = output;
  const rr_status impl = chain_impl(ctx, &args.gather_rows, &args.fused_combine);
  if (impl.code != RR_SUCCESS) return impl;
  return to_c(raggedroute::chain_from_route_ids(args, to_runtime(ctx)));
}

size_t rr_route_chain_workspace_size(int tokens, int top_k, int experts) {
  return raggedroute::get_route_chain_workspace_size(tokens, top_k, experts);
}

rr_status rr_chain_from_logits(const float* logits, const float* x, const float* expert_weights,
                               int32_t* expert_ids, float* route_weights, int32_t* counts,
                               int32_t* offsets, float* x_permuted, int32_t* route_pos,
                               float* y_permuted, float* y, int tokens, int hidden, int experts,
                               int output, const rr_context* ctx) {
  if (ctx == nullptr) return null_context();
  raggedroute::ChainFromLogitsArgs args;
  args.logits = logits;
  args.x = x;
  args.expert_weights = expert_weights;
  args.buffers = {nullptr, expert_ids, route_weights, counts, offsets, x_permuted,
                  route_pos, y_permuted, y};
  args.tokens = tokens;
  args.hidden = hidden;
  args.experts = experts;
  args.output = output;
  const rr_status impl =
      chain_impl(ctx, &args.gather_rows, &args.fused_combine, &args.prepared_weights);
  if (impl.code != RR_SUCCESS) return impl;
  return to_c(raggedroute::chain_from_logits(args, to_runtime(ctx)));
}

size_t rr_chain_workspace_size(int tokens, int hidden, int experts, int output) {
  return raggedroute::get_chain_workspace_size(tokens, hidden, experts, output);
}

int rr_launch_dense_gemm_naive(const float* a, const float* b, float* c, int m, int n, int k,
                               void* stream) {
  return raggedroute::ops::launch_dense_gemm_naive(a, b, c, m, n, k, as_stream(stream));
}
int rr_launch_topk_gate_naive(const float* logits, int32_t* expert_ids, float* weights,
                              int tokens, int experts, void* stream) {
  return raggedroute::ops::launch_topk_gate_naive(logits, expert_ids, weights, tokens, experts,
                                                  as_stream(stream));
}
int rr_launch_histogram_naive(const int32_t* expert_ids, int32_t* counts, int route_pairs,
                              int experts, void* stream) {
  return raggedroute::ops::launch_histogram_naive(expert_ids, counts, route_pairs, experts,
                                                  as_stream(stream));
}
int rr_launch_exclusive_scan_naive(const int32_t* counts, int32_t* offsets, int experts,
                                   void* stream) {
  return raggedroute::ops::launch_exclusive_scan_naive(counts, offsets, experts,
                                                       as_stream(stream));
}
int rr_launch_token_permute_naive(const float* x, const int32_t* expert_ids,
                                  const int32_t* offsets, int32_t* cursors, float* x_permuted,
                                  int32_t* route_pos, int32_t* sorted_route, int tokens,
                                  int top_k, int hidden, void* stream) {
  return raggedroute::ops::launch_token_permute_naive(x, expert_ids, offsets, cursors, x_permuted,
                                                      route_pos, sorted_route, tokens, top_k,
                                                      hidden, as_stream(stream));
}
int rr_launch_grouped_gemm_naive(const float* x_permuted, const float* expert_weights,
                                 const int32_t* offsets, float* y_permuted, int experts,
                                 int hidden, int output, int max_expert_tokens, void* stream) {
  return raggedroute::ops::launch_grouped_gemm_naive(x_permuted, expert_weights, offsets,
                                                     y_permuted, experts, hidden, output,
                                                     max_expert_tokens, as_stream(stream));
}
int rr_launch_unpermute_naive(const float* y_permuted, const int32_t* route_pos,
                              const float* route_weights, float* y, int tokens, int top_k,
                              int output, void* stream) {
  return raggedroute::ops::launch_unpermute_naive(y_permuted, route_pos, route_weights, y, tokens,
                                                  top_k, output, as_stream(stream));
}
int rr_launch_cache_scrub(uint32_t* buffer, size_t elements, void* stream) {
  return raggedroute::ops::launch_cache_scrub(buffer, elements, as_stream(stream));
}

int32_t rr_classify_compute_capability(int major, int minor) {
  return static_cast<int32_t>(raggedroute::classify_compute_capability(major, minor));
}

rr_status rr_query_current_device_architecture(int32_t* architecture) {
  raggedroute::DeviceArchitecture a = raggedroute::DeviceArchitecture::kOther;
  Status s = raggedroute::query_current_device_architecture(&a);
  if (s.ok() && architecture != nullptr) *architecture = static_cast<int32_t>(a);
  if (architecture == nullptr) {
    s = {raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
         "architecture output must not be null"};
  }
  return to_c(s);
}

uint64_t rr_kernel_launch_count(void) { return rrb::launch_count(); }

rr_status rr_consume_device_error(void* stream, uint32_t* error_word) {
  unsigned v = 0;
  const cudaError_t err = rrb::consume_device_error(as_stream(stream), &v);
  if (error_word != nullptr) *error_word = v;
  if (err != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, err, "reading the device error word failed"});
  }
  return to_c(raggedroute::success_status());
}

int rr_grouped_gemm_engine(const float* x_permuted, const float* expert_weights,
                           float* y_permuted, int hidden, int output) {
  if (!rrb::tc_gemm_supported(x_permuted, expert_weights, y_permuted, hidden, output)) return 2;
  return (rrb::gemm_pairs_enabled() && rrb::grouped_gemm_pair_units() > 0 &&
          rrb::gemm_mixed_split(hidden))
             ? 3
             : 1;
}

rr_status rr_bounded_wait_selftest(uint64_t limit_ns, unsigned long long* elapsed_ns,
                                   void* stream) {
  if (elapsed_ns == nullptr || limit_ns == 0 || limit_ns > 10000000000ull) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "rr_bounded_wait_selftest requires a device result and 0 < limit <= 10 s"});
  }
  const cudaError_t err = rrb::launch_bounded_wait_selftest(limit_ns, elapsed_ns,
                                                            as_stream(stream));
  if (err != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, err, "bounded wait self-test failed"});
  }
  return to_c(raggedroute::success_status());
}

rr_status rr_tf32_rounding_selfcheck(const uint32_t* bits, int64_t n,
                                     unsigned long long* mismatches, void* stream) {
  if (n < 0 || (n > 0 && (bits == nullptr || mismatches == nullptr))) {
    return to_c({raggedroute::StatusCode::kInvalidArgument, cudaSuccess,
                 "rr_tf32_rounding_selfcheck requires device buffers"});
  }
  const cudaError_t err = rrb::launch_tf32_round_check(bits, n, mismatches, as_stream(stream));
  if (err != cudaSuccess) {
    return to_c({raggedroute::StatusCode::kCudaError, err, "TF32 rounding self-check failed"});
  }
  return to_c(raggedroute::success_status());
}

const char* rr_version(void) { return "raggedroute_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
