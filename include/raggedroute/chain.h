// L3 chain entry points of libraggedroute_b200 (C++ side). The reference
// composes these in its benchmark adapter (benchmarks/adapters/
// chain_adapter.cpp:263-467: dense_gemm -> topk_gate -> histogram(+scan) ->
// token_permute -> grouped_gemm -> unpermute on one stream); here they are
// library calls with the same stage order and caller-owned buffers.
#pragma once

#include <cstddef>
#include <cstdint>

#include "raggedroute/operators.h"

namespace raggedroute {

struct ChainBuffers {
  float* logits = nullptr;          // [T, E]  (chain_from_tokens writes it)
  std::int32_t* expert_ids = nullptr;  // [T, 2]
  float* route_weights = nullptr;   // [T, 2]
  std::int32_t* counts = nullptr;   // [E]
  std::int32_t* offsets = nullptr;  // [E + 1]
  float* x_permuted = nullptr;      // [2T, K]
  std::int32_t* route_pos = nullptr;  // [2T]
  float* y_permuted = nullptr;      // [2T, N]
  float* y = nullptr;               // [T, N]  (the output)
};

struct ChainFromTokensArgs {
  const float* x = nullptr;               // [T, K]
  const float* router_weights = nullptr;  // [K, E]
  const float* logit_bias = nullptr;      // optional [E], added before the gate
  const float* expert_weights = nullptr;  // [E, K, N]
  ChainBuffers buffers;
  int tokens = 0;
  int hidden = 0;
  int experts = 0;
  int output = 0;
  // The grouped GEMM gathers its rows from x through sorted_route (kept in
  // the workspace); buffers.x_permuted is not written and may be null.
  bool gather_rows = false;
  // expert_weights is a buffer filled by rr_prepare_expert_weights (new: no
  // reference counterpart), not W itself; K and N multiples of 4.
  bool prepared_weights = false;
  // The unpermute runs inside the grouped GEMM's epilogue (new: no reference
  // counterpart): each output row is weighted and added into its token's row
  // of y, so buffers.y_permuted is not written and may be null. y is the
  // same bit for bit (both paths round each product, then add with subnormal
  // operands and results flushed to zero, and a sum of two terms does not
  // depend on their order).
  bool fused_combine = false;
};

struct ChainFromLogitsArgs {
  const float* logits = nullptr;          // [T, E]
  const float* x = nullptr;               // [T, K]
  const float* expert_weights = nullptr;  // [E, K, N]
  ChainBuffers buffers;                   // buffers.logits unused
  int tokens = 0;
  int hidden = 0;
  int experts = 0;
  int output = 0;
  bool gather_rows = false;       // as in ChainFromTokensArgs
  bool prepared_weights = false;  // as in ChainFromTokensArgs
  bool fused_combine = false;     // as in ChainFromTokensArgs
};

// Buffers of the post-route chain (top_k routes per token, R = T * top_k).
struct RouteChainBuffers {
  std::int32_t* counts = nullptr;        // [E]
  std::int32_t* offsets = nullptr;       // [E + 1]
  float* x_permuted = nullptr;           // [R, K]
  std::int32_t* route_pos = nullptr;     // [R]
  std::int32_t* sorted_route = nullptr;  // optional [R]: route held by each permuted row
  float* y_permuted = nullptr;           // [R, N]
  float* y = nullptr;                    // [T, N]  (the output)
};

// chain_from_route_ids (benchmarks/adapters/postroute_chain_adapter.cpp:
// 240-354 of the reference): routing decided elsewhere; histogram + scan ->
// stable token_permute -> grouped_gemm -> unpermute for top_k in [1, 8].
struct ChainFromRouteIdsArgs {
  const float* x = nullptr;                 // [T, K]
  const std::int32_t* expert_ids = nullptr;  // [T, top_k], ids in [0, E)
  const float* route_weights = nullptr;     // [T, top_k]
  const float* expert_weights = nullptr;    // [E, K, N]
  RouteChainBuffers buffers;
  int tokens = 0;
  int top_k = 0;
  int hidden = 0;
  int experts = 0;
  int output = 0;
  // The grouped GEMM gathers its rows from x through buffers.sorted_route
  // (then required); buffers.x_permuted is not written and may be null.
  bool gather_rows = false;
  // As in ChainFromTokensArgs, for top_k 1 or 2 (a larger top_k is
  // kUnsupportedKernelVariant: the sum of three or more terms would depend on
  // their order); buffers.sorted_route is then required.
  bool fused_combine = false;
};

// Workspace (bytes) for either chain: the token_permute workspace at 2T
// routes plus room for sorted_route [2T] (used when gather_rows is set).
std::size_t get_chain_workspace_size(int tokens, int hidden, int experts, int output) noexcept;

Status chain_from_tokens(const ChainFromTokensArgs& args, const RuntimeContext& context) noexcept;
Status chain_from_logits(const ChainFromLogitsArgs& args, const RuntimeContext& context) noexcept;

// Workspace (bytes) for chain_from_route_ids: the token_permute workspace at
// T * top_k routes.
std::size_t get_route_chain_workspace_size(int tokens, int top_k, int experts) noexcept;
Status chain_from_route_ids(const ChainFromRouteIdsArgs& args,
                            const RuntimeContext& context) noexcept;

}  // namespace raggedroute
