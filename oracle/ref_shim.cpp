// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A thin extern "C" layer over RaggedRoute's own CPU reference functions, so
// the Python tests and bench.py's reference arm can call them through ctypes.
// oracle/build_oracle.py compiles this file together with the reference's
// sources where they lie (src/*/cpu_reference/reference.cpp,
// src/correctness/{framework.cu,reference_validation.cpp,report.cpp} and the
// header-only include/raggedroute/benchmark/adapter_utils.h) into
// oracle/_ref/librr_ref.so. No reference source is copied into this repository.
//
// The reference has no CPU producer for token_permute (only the set-contract
// validator src/permute/cpu_reference/reference.cpp:22-81), so the chain below
// uses a stable counting sort written here, then checks it with the
// reference's validate_permute.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

#include "raggedroute/benchmark/adapter_utils.h"
#include "raggedroute/correctness/framework.h"

namespace rc = raggedroute::correctness;

namespace {

std::vector<double> to_double(const float* p, std::size_t n) {
  return std::vector<double>(p, p + n);
}

template <typename F>
void parallel_for(int items, int threads, F&& body) {
  threads = std::max(1, std::min(threads, items));
  std::vector<std::thread> pool;
  std::vector<std::exception_ptr> errors(static_cast<std::size_t>(threads));
  for (int w = 0; w < threads; ++w) {
    pool.emplace_back([&, w] {
      try {
        for (int i = w; i < items; i += threads) body(i);
      } catch (...) {
        errors[static_cast<std::size_t>(w)] = std::current_exception();
      }
    });
  }
  for (auto& t : pool) t.join();
  for (auto& e : errors) {
    if (e) std::rethrow_exception(e);
  }
}

}  // namespace

extern "C" {

// src/topk_gate/cpu_reference/reference.cpp:12-72 (double).
int rr_ref_top2_f64(const double* logits, int tokens, int experts, int32_t* ids, double* weights) {
  try {
    std::vector<double> l(logits, logits + static_cast<std::size_t>(tokens) * experts);
    const auto r = rc::top2_selected_softmax_reference(l, tokens, experts);
    std::copy(r.ids.begin(), r.ids.end(), ids);
    std::copy(r.weights.begin(), r.weights.end(), weights);
    return 0;
  } catch (...) {
    return -1;
  }
}

// include/raggedroute/benchmark/adapter_utils.h:363-418 (float).
int rr_ref_top2_f32(const float* logits, int tokens, int experts, int32_t* ids, float* weights) {
  try {
    std::vector<float> l(logits, logits + static_cast<std::size_t>(tokens) * experts);
    std::vector<std::int32_t> i;
    std::vector<float> w;
    raggedroute::benchmark::top2_selected_softmax_reference(l, tokens, experts, i, w);
    std::copy(i.begin(), i.end(), ids);
    std::copy(w.begin(), w.end(), weights);
    return 0;
  } catch (...) {
    return -1;
  }
}

// src/histogram/cpu_reference/reference.cpp:11-22.
int rr_ref_histogram(const int32_t* ids, int64_t routes, int experts, int32_t* counts) {
  try {
    std::vector<std::int32_t> v(ids, ids + routes);
    const auto c = rc::histogram_reference(v, experts);
    std::copy(c.begin(), c.end(), counts);
    return 0;
  } catch (...) {
    return -1;
  }
}

// src/scan/cpu_reference/reference.cpp:9-20.
int rr_ref_exclusive_scan(const int32_t* counts, int experts, int32_t* offsets) {
  try {
    std::vector<std::int32_t> v(counts, counts + experts);
    const auto o = rc::exclusive_scan_reference(v);
    std::copy(o.begin(), o.end(), offsets);
    return 0;
  } catch (...) {
    return -1;
  }
}

// src/permute/cpu_reference/reference.cpp:22-81: returns 1 when the permute
// output satisfies the reference's segment/bijection/inverse/row-copy checks.
int rr_ref_validate_permute(const float* x, const int32_t* ids, const int32_t* offsets,
                            int experts, const float* xp, const int32_t* route_pos,
                            const int32_t* sorted_route, int tokens, int top_k, int hidden) {
  try {
    const std::size_t routes = static_cast<std::size_t>(tokens) * top_k;
    rc::CaseDescriptor d;
    d.case_id = "oracle_pin";
    d.operator_name = "token_permute";
    std::vector<std::int32_t> sr;
    if (sorted_route != nullptr) sr.assign(sorted_route, sorted_route + routes);
    const auto report = rc::validate_permute(
        d, to_double(x, static_cast<std::size_t>(tokens) * hidden),
        std::vector<std::int32_t>(ids, ids + routes),
        std::vector<std::int32_t>(offsets, offsets + experts + 1),
        to_double(xp, routes * static_cast<std::size_t>(hidden)),
        std::vector<std::int32_t>(route_pos, route_pos + routes),
        sorted_route != nullptr ? &sr : nullptr, tokens, top_k, hidden);
    return report.ok() ? 1 : 0;
  } catch (...) {
    return -1;
  }
}

// src/dense_gemm/cpu_reference/reference.cpp:10-35.
int rr_ref_dense_gemm(const float* a, const float* b, double* c, int m, int n, int k) {
  try {
    const auto out = rc::dense_gemm_reference(to_double(a, static_cast<std::size_t>(m) * k),
                                              to_double(b, static_cast<std::size_t>(k) * n), {}, m,
                                              n, k, 1.0, 0.0);
    std::copy(out.begin(), out.end(), c);
    return 0;
  } catch (...) {
    return -1;
  }
}

// src/grouped_gemm/cpu_reference/reference.cpp:10-44.
int rr_ref_grouped_gemm(const float* x, const float* w, const int32_t* offsets, int experts,
                        int hidden, int output, double* y) {
  try {
    const std::size_t routes = static_cast<std::size_t>(offsets[experts]);
    const auto out = rc::grouped_gemm_reference(
        to_double(x, routes * hidden),
        to_double(w, static_cast<std::size_t>(experts) * hidden * output),
        std::vector<std::int32_t>(offsets, offsets + experts + 1), experts, hidden, output);
    std::copy(out.begin(), out.end(), y);
    return 0;
  } catch (...) {
    return -1;
  }
}

// src/unpermute/cpu_reference/reference.cpp:10-37.
int rr_ref_unpermute(const float* yp, const int32_t* route_pos, const float* route_weights,
                     int tokens, int top_k, int output, double* y) {
  try {
    const std::size_t routes = static_cast<std::size_t>(tokens) * top_k;
    const auto out = rc::unpermute_reference(
        to_double(yp, routes * output), std::vector<std::int32_t>(route_pos, route_pos + routes),
        to_double(route_weights, routes), tokens, top_k, output);
    std::copy(out.begin(), out.end(), y);
    return 0;
  } catch (...) {
    return -1;
  }
}

// The reference's CPU path for chain_from_tokens, spread over host threads:
// dense_gemm_reference (token shards) -> optional logit bias ->
// top2_selected_softmax_reference -> histogram_reference ->
// exclusive_scan_reference -> stable counting-sort permute ->
// grouped_gemm_reference (expert shards) -> unpermute_reference (token shards).
// Every contraction and reduction is the reference's own double-precision
// function; only the permute producer and the sharding are written here.
// Returns 0 on success; y receives the float-rounded output [T, N].
int rr_ref_chain_from_tokens(const float* x, const float* router_w, const float* logit_bias,
                             const float* expert_w, int tokens, int hidden, int experts,
                             int output, int threads, float* y) {
  try {
    const int shards = std::max(1, threads);
    // Router GEMM on token shards.
    std::vector<double> logits(static_cast<std::size_t>(tokens) * experts);
    const auto wr = to_double(router_w, static_cast<std::size_t>(hidden) * experts);
    const int token_block = std::max(1, (tokens + shards - 1) / shards);
    const int token_blocks = (tokens + token_block - 1) / token_block;
    parallel_for(token_blocks, shards, [&](int blk) {
      const int t0 = blk * token_block;
      const int t1 = std::min(tokens, t0 + token_block);
      const auto part = rc::dense_gemm_reference(
          to_double(x + static_cast<std::size_t>(t0) * hidden,
                    static_cast<std::size_t>(t1 - t0) * hidden),
          wr, {}, t1 - t0, experts, hidden, 1.0, 0.0);
      std::copy(part.begin(), part.end(), logits.begin() + static_cast<std::ptrdiff_t>(t0) * experts);
    });
    if (logit_bias != nullptr) {
      for (int t = 0; t < tokens; ++t)
        for (int e = 0; e < experts; ++e)
          logits[static_cast<std::size_t>(t) * experts + e] += static_cast<double>(logit_bias[e]);
    }
    const auto gate = rc::top2_selected_softmax_reference(logits, tokens, experts);
    const auto counts = rc::histogram_reference(gate.ids, experts);
    const auto offsets = rc::exclusive_scan_reference(counts);
    const std::size_t routes = static_cast<std::size_t>(tokens) * 2;
    // Stable permute (counting sort; route-ascending within each expert).
    std::vector<std::int32_t> route_pos(routes);
    std::vector<std::int32_t> cursor(static_cast<std::size_t>(experts), 0);
    for (std::size_t r = 0; r < routes; ++r) {
      const int e = gate.ids[r];
      route_pos[r] = offsets[static_cast<std::size_t>(e)] + cursor[static_cast<std::size_t>(e)]++;
    }
    // Grouped GEMM per expert on that expert's gathered rows.
    std::vector<std::vector<std::size_t>> members(static_cast<std::size_t>(experts));
    for (std::size_t r = 0; r < routes; ++r) members[static_cast<std::size_t>(gate.ids[r])].push_back(r);
    std::vector<double> yp(routes * static_cast<std::size_t>(output), 0.0);
    parallel_for(experts, shards, [&](int e) {
      const auto& rows = members[static_cast<std::size_t>(e)];
      if (rows.empty()) return;
      std::vector<double> xe;
      xe.reserve(rows.size() * static_cast<std::size_t>(hidden));
      for (std::size_t r : rows) {
        const float* src = x + (r / 2) * static_cast<std::size_t>(hidden);
        xe.insert(xe.end(), src, src + hidden);
      }
      const auto we = to_double(expert_w + static_cast<std::size_t>(e) * hidden * output,
                                static_cast<std::size_t>(hidden) * output);
      const auto ye = rc::grouped_gemm_reference(
          xe, we, {0, static_cast<std::int32_t>(rows.size())}, 1, hidden, output);
      for (std::size_t i = 0; i < rows.size(); ++i) {
        std::copy(ye.begin() + static_cast<std::ptrdiff_t>(i * output),
                  ye.begin() + static_cast<std::ptrdiff_t>((i + 1) * output),
                  yp.begin() + static_cast<std::ptrdiff_t>(route_pos[rows[i]]) * output);
      }
    });
    // Unpermute on token shards.
    parallel_for(token_blocks, shards, [&](int blk) {
      const int t0 = blk * token_block;
      const int t1 = std::min(tokens, t0 + token_block);
      const int nt = t1 - t0;
      // Rebase this shard's rows so route_pos indexes a compact Yp slice.
      std::vector<std::int32_t> pos(static_cast<std::size_t>(nt) * 2);
      std::vector<double> ysub(static_cast<std::size_t>(nt) * 2 * output);
      std::vector<double> wsub(static_cast<std::size_t>(nt) * 2);
      for (int i = 0; i < nt * 2; ++i) {
        const std::size_t r = static_cast<std::size_t>(t0) * 2 + i;
        pos[static_cast<std::size_t>(i)] = i;
        wsub[static_cast<std::size_t>(i)] = gate.weights[r];
        std::copy(yp.begin() + static_cast<std::ptrdiff_t>(route_pos[r]) * output,
                  yp.begin() + static_cast<std::ptrdiff_t>(route_pos[r] + 1) * output,
                  ysub.begin() + static_cast<std::ptrdiff_t>(i) * output);
      }
      const auto out = rc::unpermute_reference(ysub, pos, wsub, nt, 2, output);
      for (std::size_t i = 0; i < out.size(); ++i)
        y[static_cast<std::size_t>(t0) * output + i] = static_cast<float>(out[i]);
    });
    return 0;
  } catch (...) {
    return -1;
  }
}

}  // extern "C"
