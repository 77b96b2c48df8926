/*
 * rr_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of RaggedRoute's CPU reference for the seven-stage MoE
 * top-2 routing path. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load this library, and only as the
 * checker (or the timed CPU baseline). The product path never calls it.
 *
 * Each function cites the reference file:line it restates (paths are relative
 * to the RaggedRoute project root). Parity of this restatement is pinned in
 * tests/test_oracle.py against the reference's own known-answer tests and
 * against the reference's CPU sources compiled into oracle/_ref.
 *
 * Build: see oracle/build_oracle.py (gcc -O2 -ffp-contract=off -fPIC -shared).
 * -ffp-contract=off matters: the reference's float chain oracle is ISO C++
 * without FMA contraction (benchmarks/adapters/chain_adapter.cpp:197-206).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define RR_ORACLE_OK 0
#define RR_ORACLE_BAD_SHAPE -1
#define RR_ORACLE_ID_RANGE -2
#define RR_ORACLE_OVERFLOW -3
#define RR_ORACLE_NEGATIVE -4
#define RR_ORACLE_NO_MEMORY -5

/* ------------------------------------------------------------------------ */
/* Top-2 selected softmax.                                                   */
/* ------------------------------------------------------------------------ */

/* Candidate ordering: NaN is read as -inf, larger value first, equal values
 * resolve to the lower expert id, and any candidate beats an empty slot.
 * Follows src/topk_gate/cpu_reference/reference.cpp:22-24. */
static int precedes_d(double value, int id, double incumbent, int incumbent_id) {
  return incumbent_id < 0 || value > incumbent || (value == incumbent && id < incumbent_id);
}

static int precedes_f(float value, int id, float incumbent, int incumbent_id) {
  return incumbent_id < 0 || value > incumbent || (value == incumbent && id < incumbent_id);
}

/* Double-precision top-2 reference.
 * src/topk_gate/cpu_reference/reference.cpp:12-72. */
int rr_oracle_top2_f64(const double* logits, int tokens, int experts, int32_t* ids,
                       double* weights) {
  if (tokens < 0 || experts < 2) return RR_ORACLE_BAD_SHAPE;
  for (int t = 0; t < tokens; ++t) {
    double first = -INFINITY, second = -INFINITY;
    int first_id = -1, second_id = -1;
    int saw_non_nan = 0;
    for (int e = 0; e < experts; ++e) {
      const double raw = logits[(size_t)t * experts + e];
      const int is_nan = isnan(raw);
      const double v = is_nan ? -INFINITY : raw;
      saw_non_nan = saw_non_nan || !is_nan;
      if (precedes_d(v, e, first, first_id)) {
        second = first;
        second_id = first_id;
        first = v;
        first_id = e;
      } else if (precedes_d(v, e, second, second_id)) {
        second = v;
        second_id = e;
      }
    }
    double w0 = 0.5, w1 = 0.5;
    if (!saw_non_nan) {
      first_id = 0;
      second_id = 1;
    } else if (first != second) {
      if (first == INFINITY || second == -INFINITY) {
        w0 = 1.0;
        w1 = 0.0;
      } else {
        const double rel = exp(second - first);
        w0 = 1.0 / (1.0 + rel);
        w1 = rel * w0;
      }
    }
    ids[2 * (size_t)t] = first_id;
    ids[2 * (size_t)t + 1] = second_id;
    weights[2 * (size_t)t] = w0;
    weights[2 * (size_t)t + 1] = w1;
  }
  return RR_ORACLE_OK;
}

/* Single-precision top-2 reference used by the L3 chain validation.
 * include/raggedroute/benchmark/adapter_utils.h:363-418 (std::exp on float
 * resolves to expf). An optional per-expert bias (NULL for none) is added to
 * each logit before selection; the reference chain has no bias, the
 * expert-parallel config uses it to skew expert load. */
int rr_oracle_top2_f32(const float* logits, const float* bias, int tokens, int experts,
                       int32_t* ids, float* weights) {
  if (tokens < 0 || experts < 2) return RR_ORACLE_BAD_SHAPE;
  for (int t = 0; t < tokens; ++t) {
    float first = -INFINITY, second = -INFINITY;
    int first_id = -1, second_id = -1;
    int saw_non_nan = 0;
    for (int e = 0; e < experts; ++e) {
      float raw = logits[(size_t)t * experts + e];
      if (bias != NULL) raw = raw + bias[e];
      const int is_nan = isnan(raw);
      const float v = is_nan ? -INFINITY : raw;
      saw_non_nan = saw_non_nan || !is_nan;
      if (precedes_f(v, e, first, first_id)) {
        second = first;
        second_id = first_id;
        first = v;
        first_id = e;
      } else if (precedes_f(v, e, second, second_id)) {
        second = v;
        second_id = e;
      }
    }
    float w0 = 0.5f, w1 = 0.5f;
    if (!saw_non_nan) {
      first_id = 0;
      second_id = 1;
    } else if (first != second) {
      if (first == INFINITY || second == -INFINITY) {
        w0 = 1.0f;
        w1 = 0.0f;
      } else {
        const float rel = expf(second - first);
        w0 = 1.0f / (1.0f + rel);
        w1 = rel * w0;
      }
    }
    ids[2 * (size_t)t] = first_id;
    ids[2 * (size_t)t + 1] = second_id;
    weights[2 * (size_t)t] = w0;
    weights[2 * (size_t)t + 1] = w1;
  }
  return RR_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* Routing metadata.                                                         */
/* ------------------------------------------------------------------------ */

/* counts[e] = #{r : ids[r] == e}; ids outside [0, E) are an error.
 * src/histogram/cpu_reference/reference.cpp:11-22. */
int rr_oracle_histogram(const int32_t* ids, int64_t routes, int experts, int32_t* counts) {
  if (experts < 1 || routes < 0) return RR_ORACLE_BAD_SHAPE;
  memset(counts, 0, sizeof(int32_t) * (size_t)experts);
  for (int64_t r = 0; r < routes; ++r) {
    const int32_t id = ids[r];
    if (id < 0 || id >= experts) return RR_ORACLE_ID_RANGE;
    if (counts[id] == INT32_MAX) return RR_ORACLE_OVERFLOW;
    ++counts[id];
  }
  return RR_ORACLE_OK;
}

/* offsets[0] = 0, offsets[e+1] = offsets[e] + counts[e]; int32 overflow and
 * negative counts are errors. src/scan/cpu_reference/reference.cpp:9-20. */
int rr_oracle_exclusive_scan(const int32_t* counts, int experts, int32_t* offsets) {
  if (experts < 0) return RR_ORACLE_BAD_SHAPE;
  int64_t total = 0;
  for (int e = 0; e < experts; ++e) {
    if (counts[e] < 0) return RR_ORACLE_NEGATIVE;
    offsets[e] = (int32_t)total;
    total += counts[e];
    if (total > INT32_MAX) return RR_ORACLE_OVERFLOW;
  }
  offsets[experts] = (int32_t)total;
  return RR_ORACLE_OK;
}

/* Stable token permute: the route r = t*top_k + k of expert e lands at
 *   route_pos[r] = offsets[e] + #{r' < r : ids[r'] == e},
 * i.e. a sequential counting sort. The reference assigns the in-segment slot
 * with an atomic cursor (src/permute/cuda_naive/baseline.cu:23) and checks
 * only the set contract (src/permute/cpu_reference/reference.cpp:43-80); this
 * build fixes the order to ascending route index, which satisfies every one of
 * those checks. Rows are copied bit-for-bit: x_permuted[route_pos[r], :] =
 * x[r / top_k, :]. sorted_route (optional) is the inverse map and cursors
 * (optional, E entries) end equal to the per-expert counts, the reference
 * wrapper's post-state (tests/operator_api_tests.cpp:776-778). */
int rr_oracle_stable_permute(const float* x, const int32_t* ids, const int32_t* offsets,
                             int tokens, int top_k, int hidden, int experts, float* x_permuted,
                             int32_t* route_pos, int32_t* sorted_route, int32_t* cursors) {
  if (tokens < 0 || top_k < 1 || hidden < 0 || experts < 1) return RR_ORACLE_BAD_SHAPE;
  int32_t* cursor = (int32_t*)calloc((size_t)experts, sizeof(int32_t));
  if (cursor == NULL) return RR_ORACLE_NO_MEMORY;
  const int64_t routes = (int64_t)tokens * top_k;
  for (int64_t r = 0; r < routes; ++r) {
    const int32_t e = ids[r];
    if (e < 0 || e >= experts) {
      free(cursor);
      return RR_ORACLE_ID_RANGE;
    }
    const int32_t dest = offsets[e] + cursor[e]++;
    route_pos[r] = dest;
    if (sorted_route != NULL) sorted_route[dest] = (int32_t)r;
    if (x_permuted != NULL && hidden > 0) {
      memcpy(x_permuted + (size_t)dest * hidden, x + (size_t)(r / top_k) * hidden,
             sizeof(float) * (size_t)hidden);
    }
  }
  if (cursors != NULL) memcpy(cursors, cursor, sizeof(int32_t) * (size_t)experts);
  free(cursor);
  return RR_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* Contractions (double accumulation, inputs promoted from float).           */
/* ------------------------------------------------------------------------ */

/* C[M,N] = A[M,K] . B[K,N], row-major, double accumulation in k order.
 * src/dense_gemm/cpu_reference/reference.cpp:10-35 (alpha=1, beta=0). */
int rr_oracle_dense_gemm_f64(const float* a, const float* b, double* c, int m, int n, int k) {
  if (m < 0 || n < 0 || k < 0) return RR_ORACLE_BAD_SHAPE;
  for (int i = 0; i < m; ++i) {
    for (int j = 0; j < n; ++j) {
      double sum = 0.0;
      for (int p = 0; p < k; ++p) sum += (double)a[(size_t)i * k + p] * (double)b[(size_t)p * n + j];
      c[(size_t)i * n + j] = sum;
    }
  }
  return RR_ORACLE_OK;
}

/* Y[r, :] = X[r, :] . W[e] for each row r in expert e's segment
 * [offsets[e], offsets[e+1]). src/grouped_gemm/cpu_reference/reference.cpp:10-44.
 * Rows outside every segment are left untouched. */
int rr_oracle_grouped_gemm_f64(const float* x, const float* w, const int32_t* offsets,
                               int experts, int hidden, int output, double* y) {
  if (experts < 1 || hidden < 0 || output < 0) return RR_ORACLE_BAD_SHAPE;
  for (int e = 0; e < experts; ++e) {
    if (offsets[e] < 0 || offsets[e] > offsets[e + 1]) return RR_ORACLE_BAD_SHAPE;
  }
  double* acc = (double*)malloc(sizeof(double) * (size_t)(output > 0 ? output : 1));
  if (acc == NULL) return RR_ORACLE_NO_MEMORY;
  for (int e = 0; e < experts; ++e) {
    const float* we = w + (size_t)e * hidden * output;
    for (int r = offsets[e]; r < offsets[e + 1]; ++r) {
      for (int j = 0; j < output; ++j) acc[j] = 0.0;
      const float* xr = x + (size_t)r * hidden;
      for (int p = 0; p < hidden; ++p) {
        const double xv = (double)xr[p];
        const float* wrow = we + (size_t)p * output;
        for (int j = 0; j < output; ++j) acc[j] += xv * (double)wrow[j];
      }
      for (int j = 0; j < output; ++j) y[(size_t)r * output + j] = acc[j];
    }
  }
  free(acc);
  return RR_ORACLE_OK;
}

/* Y[t, c] = sum_{k=0..top_k-1} w[t*top_k+k] * Yp[route_pos[t*top_k+k], c],
 * accumulated in rank order in double.
 * src/unpermute/cpu_reference/reference.cpp:10-37. */
int rr_oracle_unpermute_f64(const float* y_permuted, const int32_t* route_pos,
                            const float* route_weights, int tokens, int top_k, int output,
                            double* y) {
  if (tokens < 0 || top_k < 1 || output < 0) return RR_ORACLE_BAD_SHAPE;
  const int64_t routes = (int64_t)tokens * top_k;
  for (int t = 0; t < tokens; ++t) {
    for (int c = 0; c < output; ++c) {
      double sum = 0.0;
      for (int k = 0; k < top_k; ++k) {
        const int64_t r = (int64_t)t * top_k + k;
        const int32_t src = route_pos[r];
        if (src < 0 || src >= routes) return RR_ORACLE_ID_RANGE;
        sum += (double)route_weights[r] * (double)y_permuted[(size_t)src * output + c];
      }
      y[(size_t)t * output + c] = sum;
    }
  }
  return RR_ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* The L3 chain oracle in float (benchmark-side validation).                 */
/* ------------------------------------------------------------------------ */

/* logits[t, e] = sequential float sum over k of x[t,k] * w[k,e], no FMA.
 * benchmarks/adapters/chain_adapter.cpp:197-206. */
int rr_oracle_chain_logits_f32(const float* x, const float* router_w, int tokens, int hidden,
                               int experts, float* logits) {
  if (tokens < 0 || hidden < 0 || experts < 1) return RR_ORACLE_BAD_SHAPE;
  for (int t = 0; t < tokens; ++t) {
    for (int e = 0; e < experts; ++e) {
      float sum = 0.0f;
      for (int p = 0; p < hidden; ++p) {
        const float prod = x[(size_t)t * hidden + p] * router_w[(size_t)p * experts + e];
        sum = sum + prod;
      }
      logits[(size_t)t * experts + e] = sum;
    }
  }
  return RR_ORACLE_OK;
}

/* Final chain output in float: for each token and column, the sum over the two
 * ranks of weight * (sequential float projection of x through the expert).
 * benchmarks/adapters/chain_adapter.cpp:858-879. */
/* Output of the post-route chain for top_k routes per token
 * (benchmarks/adapters/postroute_chain_adapter.cpp:654-675): per token and
 * column, combined += w[route] * projection in rank order, projection the
 * float sum over hidden in order. With top_k = 2 this is also the L3 chain
 * oracle's output half (chain_adapter.cpp:858-879). */
int rr_oracle_route_chain_output_f32(const float* x, const float* expert_w, const int32_t* ids,
                                     const float* weights, int tokens, int top_k, int hidden,
                                     int output, int experts, float* y) {
  if (tokens < 0 || top_k < 1 || hidden < 0 || output < 0 || experts < 1) {
    return RR_ORACLE_BAD_SHAPE;
  }
  for (int t = 0; t < tokens; ++t) {
    for (int c = 0; c < output; ++c) {
      float combined = 0.0f;
      for (int k = 0; k < top_k; ++k) {
        const size_t r = (size_t)t * top_k + k;
        const int e = ids[r];
        if (e < 0 || e >= experts) return RR_ORACLE_ID_RANGE;
        float projection = 0.0f;
        for (int p = 0; p < hidden; ++p) {
          const float prod =
              x[(size_t)t * hidden + p] * expert_w[((size_t)e * hidden + p) * output + c];
          projection = projection + prod;
        }
        const float term = weights[r] * projection;
        combined = combined + term;
      }
      y[(size_t)t * output + c] = combined;
    }
  }
  return RR_ORACLE_OK;
}

int rr_oracle_chain_output_f32(const float* x, const float* expert_w, const int32_t* ids,
                               const float* weights, int tokens, int hidden, int output,
                               int experts, float* y) {
  return rr_oracle_route_chain_output_f32(x, expert_w, ids, weights, tokens, 2, hidden, output,
                                          experts, y);
}
