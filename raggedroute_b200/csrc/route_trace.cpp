// Route-trace input ("raggedroute.route_trace.v1" text files, .rrtrace).
//
// Format and validation follow the reference's loader
// (include/raggedroute/benchmark/adapter_utils.h:250-322): line 1 the schema
// name, line 2 a portable trace id ([A-Za-z0-9._-]+), line 3 the source kind
// (production | captured | synthetic_fixture), then "tokens experts top_k
// frame_count", then per frame a portable, unique frame id followed by
// tokens*top_k expert ids, each in [0, experts) and distinct within a token;
// nothing may follow the last frame. The reference caps experts at 64 (its
// kernels' limit); this library's limit is 1024. Host-only code; the chain
// consumes a frame through rr_route_trace_logits + rr_chain_from_logits
// (benchmarks/adapters/chain_adapter.cpp:207-228) or directly as route ids
// through rr_chain_from_route_ids.
#include <algorithm>
#include <cctype>
#include <cstring>
#include <fstream>
#include <set>
#include <string>
#include <vector>

#include "../../include/raggedroute_b200.h"

namespace {

rr_status st(int32_t code, const char* msg) {
  rr_status s;
  s.code = code;
  s.cuda_error = 0;
  s.message = msg;
  return s;
}

bool portable(const std::string& v) {
  if (v.empty()) return false;
  return std::all_of(v.begin(), v.end(), [](char c) {
    return std::isalnum(static_cast<unsigned char>(c)) != 0 || c == '.' || c == '_' || c == '-';
  });
}

void copy_name(char* dst, std::size_t cap, const std::string& src) {
  if (dst == nullptr || cap == 0) return;
  const std::size_t n = std::min(cap - 1, src.size());
  std::memcpy(dst, src.data(), n);
  dst[n] = '\0';
}

}  // namespace

extern "C" {

rr_status rr_route_trace_read(const char* path, int frame, rr_route_trace_info* info,
                              int32_t* expert_ids, int64_t ids_capacity) {
  if (path == nullptr || info == nullptr || frame < 0) {
    return st(RR_INVALID_ARGUMENT, "route trace path, info and frame are invalid");
  }
  std::memset(info, 0, sizeof(*info));
  std::ifstream in(path);
  if (!in) return st(RR_INVALID_ARGUMENT, "cannot open route trace");
  std::string schema, trace_id, source;
  int tokens = 0, experts = 0, top_k = 0, frames = 0;
  if (!std::getline(in, schema) || schema != "raggedroute.route_trace.v1" ||
      !std::getline(in, trace_id) || !std::getline(in, source) ||
      !(in >> tokens >> experts >> top_k >> frames)) {
    return st(RR_INVALID_ARGUMENT, "invalid route trace header");
  }
  if (!portable(trace_id) ||
      (source != "production" && source != "captured" && source != "synthetic_fixture") ||
      tokens < 1 || experts < 1 || experts > RR_MAX_EXPERTS || top_k < 1 || top_k > experts ||
      frames < 1 || frame >= frames ||
      static_cast<int64_t>(tokens) * top_k > (int64_t{1} << 31) - 1) {
    return st(RR_INVALID_ARGUMENT, "invalid route trace metadata");
  }
  const std::size_t routes = static_cast<std::size_t>(tokens) * static_cast<std::size_t>(top_k);
  if (expert_ids != nullptr && ids_capacity < static_cast<int64_t>(routes)) {
    return st(RR_INVALID_ARGUMENT, "route trace ids buffer is smaller than tokens*top_k");
  }
  std::set<std::string> seen;
  std::vector<int32_t> ids(routes);
  std::vector<int32_t> row(static_cast<std::size_t>(top_k));
  for (int f = 0; f < frames; ++f) {
    std::string frame_id;
    if (!(in >> frame_id) || !portable(frame_id) || !seen.insert(frame_id).second) {
      return st(RR_INVALID_ARGUMENT, "route trace frame id is invalid or duplicated");
    }
    for (std::size_t r = 0; r < routes; ++r) {
      long long v = -1;
      if (!(in >> v) || v < 0 || v >= experts) {
        return st(RR_INVALID_ARGUMENT, "route trace contains an invalid expert id");
      }
      ids[r] = static_cast<int32_t>(v);
    }
    for (int t = 0; t < tokens; ++t) {
      std::copy(ids.begin() + static_cast<std::ptrdiff_t>(t) * top_k,
                ids.begin() + static_cast<std::ptrdiff_t>(t + 1) * top_k, row.begin());
      std::sort(row.begin(), row.end());
      if (std::adjacent_find(row.begin(), row.end()) != row.end()) {
        return st(RR_INVALID_ARGUMENT, "route trace repeats an expert within one token");
      }
    }
    if (f == frame) {
      copy_name(info->frame_id, sizeof(info->frame_id), frame_id);
      if (expert_ids != nullptr) std::copy(ids.begin(), ids.end(), expert_ids);
    }
  }
  std::string trailing;
  if (in >> trailing) return st(RR_INVALID_ARGUMENT, "route trace has trailing data");
  info->tokens = tokens;
  info->experts = experts;
  info->top_k = top_k;
  info->frame_count = frames;
  copy_name(info->trace_id, sizeof(info->trace_id), trace_id);
  copy_name(info->source_kind, sizeof(info->source_kind), source);
  return st(RR_SUCCESS, "success");
}

// Logits that make the top-2 gate select a trace frame's routes
// (chain_adapter.cpp:222-228): -8 everywhere, 2 for the first id of each
// token and 1 for the second. Host buffers, logits [tokens, experts].
rr_status rr_route_trace_logits(const int32_t* expert_ids, int tokens, int experts,
                                float* logits) {
  if (expert_ids == nullptr || logits == nullptr || tokens < 0 || experts < 2) {
    return st(RR_INVALID_ARGUMENT, "route trace logits need ids, logits and E >= 2");
  }
  std::fill(logits, logits + static_cast<std::size_t>(tokens) * experts, -8.0f);
  for (int t = 0; t < tokens; ++t) {
    const int32_t a = expert_ids[static_cast<std::size_t>(t) * 2];
    const int32_t b = expert_ids[static_cast<std::size_t>(t) * 2 + 1];
    if (a < 0 || a >= experts || b < 0 || b >= experts || a == b) {
      return st(RR_INVALID_ARGUMENT, "route trace ids out of range or repeated");
    }
    logits[static_cast<std::size_t>(t) * experts + a] = 2.0f;
    logits[static_cast<std::size_t>(t) * experts + b] = 1.0f;
  }
  return st(RR_SUCCESS, "success");
}

}  // extern "C"
