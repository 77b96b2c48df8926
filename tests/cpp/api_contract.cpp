// Host-only contract checks of the reference-compatible C++ API, compiled
// against include/raggedroute/*.h and linked with libraggedroute_b200.so.
// Needs no GPU: every call here either is pure dispatch or fails validation
// before any CUDA call. Mirrors the pure-dispatch and argument cases of the
// reference's tests/operator_api_tests.cpp:63-316, adapted to a B200 library
// (kSm100 is the executable architecture).
#include <cstdio>
#include <cstdlib>

#include "raggedroute/baseline_ops.h"
#include "raggedroute/chain.h"
#include "raggedroute/dispatch.h"
#include "raggedroute/operators.h"

namespace {
int failures = 0;
void require(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAIL: %s\n", what);
    ++failures;
  }
}
}  // namespace

int main() {
  using namespace raggedroute;
  require(classify_compute_capability(10, 0) == DeviceArchitecture::kSm100, "classify 10.0");
  require(classify_compute_capability(8, 6) == DeviceArchitecture::kSm86, "classify 8.6");
  require(classify_compute_capability(12, 0) == DeviceArchitecture::kOther, "classify 12.0");

  DispatchRequest req;
  DispatchDecision dec;
  req.operator_kind = OperatorKind::kHistogram;
  req.architecture = DeviceArchitecture::kSm100;
  require(select_kernel(req, &dec).ok(), "histogram dispatch on sm100");
  require(dec.kernel.family == KernelFamily::kCudaOptimized && dec.kernel.implementation_id == 101,
          "histogram auto decision");
  req.architecture = DeviceArchitecture::kSm86;
  require(select_kernel(req, &dec).code == StatusCode::kUnsupportedArchitecture, "sm86 rejected");
  req.architecture = DeviceArchitecture::kAuto;
  require(select_kernel(req, &dec).code == StatusCode::kInvalidArgument, "auto unresolved");
  req.architecture = DeviceArchitecture::kSm100;
  req.requested_kernel = {KernelFamily::kAuto, 3};
  require(select_kernel(req, &dec).code == StatusCode::kUnsupportedKernelVariant, "auto id");
  req.requested_kernel = {KernelFamily::kCudaOptimized, 102};
  require(select_kernel(req, &dec).code == StatusCode::kUnsupportedKernelVariant, "hist id 102");
  require(select_kernel(req, nullptr).code == StatusCode::kInvalidArgument, "null decision");

  DispatchRequest gemm;
  gemm.operator_kind = OperatorKind::kGroupedGemm;
  gemm.architecture = DeviceArchitecture::kSm100;
  require(select_kernel(gemm, &dec).code == StatusCode::kInvalidArgument, "gemm roles");
  gemm.signature.input = TensorSpec{};
  gemm.signature.weight = TensorSpec{};
  gemm.signature.accumulator = ScalarType::kFp32;
  gemm.signature.output = TensorSpec{};
  require(select_kernel(gemm, &dec).ok(), "gemm fp32 signature");
  gemm.signature.input->strides = {1, 0, 0};
  require(select_kernel(gemm, &dec).code == StatusCode::kUnsupportedLayout, "gemm strides");
  gemm.signature.input = TensorSpec{};
  gemm.signature.input->dtype = ScalarType::kFp16;
  gemm.signature.weight->dtype = ScalarType::kFp16;
  require(select_kernel(gemm, &dec).code == StatusCode::kUnsupportedDataType, "gemm fp16");

  RuntimeContext ctx;
  ctx.architecture = DeviceArchitecture::kSm100;
  DenseGemmArgs dense;
  dense.m = -1;
  require(dense_gemm(dense, ctx).code == StatusCode::kInvalidArgument, "dense negative");
  dense = {};
  dense.alpha = 2.0F;
  require(dense_gemm(dense, ctx).code == StatusCode::kInvalidArgument, "dense alpha");
  dense = {};
  dense.a.spec.dtype = ScalarType::kFp16;
  dense.b.spec.dtype = ScalarType::kFp16;
  dense.c.spec.dtype = ScalarType::kFp16;
  require(dense_gemm(dense, ctx).code == StatusCode::kUnsupportedDataType, "dense fp16");
  dense = {};
  dense.a.spec.strides[0] = 1;
  require(dense_gemm(dense, ctx).code == StatusCode::kUnsupportedLayout, "dense stride");
  dense = {};
  dense.m = 1;
  dense.n = 1;
  alignas(float) unsigned char misaligned[sizeof(float) + 1]{};
  dense.c.data = misaligned + 1;
  require(dense_gemm(dense, ctx).code == StatusCode::kInvalidArgument, "dense misaligned");
  dense = {};
  require(dense_gemm(dense, ctx).ok(), "empty dense is a no-op");

  TopKGateArgs topk;
  topk.tokens = 4;
  topk.experts = 1;
  require(topk_gate(topk, ctx).code == StatusCode::kInvalidArgument, "topk E=1");
  topk.experts = 1025;
  require(topk_gate(topk, ctx).code == StatusCode::kInvalidArgument, "topk E=1025");
  topk.experts = 8;
  topk.top_k = 3;
  require(topk_gate(topk, ctx).code == StatusCode::kInvalidArgument, "topk k=3");
  topk.top_k = 2;
  topk.tokens = 0;
  require(topk_gate(topk, ctx).ok(), "topk T=0 is a no-op");

  TokenPermuteArgs mism;
  mism.experts = 2;
  mism.top_k = 1;
  mism.x.spec.dtype = ScalarType::kFp16;
  mism.x_permuted.spec.dtype = ScalarType::kBf16;
  require(token_permute(mism, ctx).code == StatusCode::kUnsupportedDataType, "permute dtypes");
  TokenPermuteArgs permute;
  permute.tokens = 1;
  permute.experts = 2;
  permute.top_k = 1;
  std::int32_t placeholder = 0;
  permute.expert_ids = &placeholder;
  permute.offsets = &placeholder;
  permute.route_pos = &placeholder;
  require(get_token_permute_workspace_size(permute) == 2 * sizeof(std::int32_t), "permute ws");
  require(token_permute(permute, ctx).code == StatusCode::kInsufficientWorkspace,
          "permute missing workspace");
  permute.tokens = 1 << 20;
  require(get_token_permute_workspace_size(permute) == 2 * sizeof(std::int32_t),
          "the permute workspace is the E cursors at every size");

  ExclusiveScanArgs scan;
  scan.experts = 0;
  require(exclusive_scan(scan, ctx).code == StatusCode::kInvalidArgument, "scan E=0");
  require(get_exclusive_scan_workspace_size(scan) == 0, "scan workspace-free");
  HistogramExclusiveScanArgs fused;
  require(get_histogram_exclusive_scan_workspace_size(fused) == 0, "fused workspace-free");
  std::int32_t buf[16] = {};
  fused.expert_ids = buf;
  fused.counts = buf + 2;
  fused.offsets = buf + 8;
  fused.route_pairs = 4;
  fused.experts = 4;
  require(histogram_exclusive_scan(fused, ctx).code == StatusCode::kInvalidArgument,
          "fused overlap");

  GroupedGemmArgs grouped;
  grouped.experts = 0;
  require(grouped_gemm(grouped, ctx).code == StatusCode::kInvalidArgument, "grouped E=0");
  grouped.experts = 4;
  grouped.kernel = {KernelFamily::kCudaOptimized, 5};
  require(grouped_gemm(grouped, ctx).code == StatusCode::kUnsupportedKernelVariant,
          "grouped optimized id");
  grouped.kernel = {};
  require(grouped_gemm(grouped, ctx).ok(), "grouped max_expert_tokens=0 no-op");

  UnpermuteArgs un;
  un.top_k = 65;
  require(unpermute(un, ctx).code == StatusCode::kInvalidArgument, "unpermute top_k 65");

  require(ops::launch_topk_gate_naive(nullptr, nullptr, nullptr, 0, 8, nullptr) == cudaSuccess,
          "empty topk launcher");
  require(ops::launch_topk_gate_naive(nullptr, nullptr, nullptr, 1, 1, nullptr) ==
              cudaErrorInvalidValue,
          "topk launcher E=1");
  require(ops::launch_token_permute_naive(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                          nullptr, 0, 2, 7, nullptr) == cudaSuccess,
          "empty permute launcher");
  require(ops::launch_grouped_gemm_naive(nullptr, nullptr, nullptr, nullptr, 4, 7, 5, 0,
                                         nullptr) == cudaSuccess,
          "empty grouped launcher");
  require(ops::launch_unpermute_naive(nullptr, nullptr, nullptr, nullptr, 0, 2, 7, nullptr) ==
              cudaSuccess,
          "empty unpermute launcher");
  require(ops::launch_dense_gemm_naive(nullptr, nullptr, nullptr, 0, 5, 3, nullptr) ==
              cudaSuccess,
          "empty dense launcher");

  ChainFromTokensArgs chain;
  chain.experts = 1;
  require(chain_from_tokens(chain, ctx).code == StatusCode::kInvalidArgument, "chain E=1");
  require(get_chain_workspace_size(65536, 4096, 128, 1408) > 128 * 4, "chain workspace");

  if (failures == 0) std::printf("api_contract: all checks passed\n");
  return failures == 0 ? 0 : 1;
}
