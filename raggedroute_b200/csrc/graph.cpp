// CUDA-graph capture of operator sequences (no reference counterpart; the
// reference's chain benchmark captures its own adapter calls,
// benchmarks/adapters/chain_adapter.cpp:730-826).
//
// Every rr_* operator and chain enqueues on ctx->stream without host
// synchronisation, allocation or host reads of device data, and the grouped
// GEMM derives its tile schedule from offsets on the device, so a captured
// chain stays valid for any routing of the same shapes: replaying the graph
// after writing new tokens into the captured input buffer runs the whole
// chain with one launch call. Capture uses the relaxed mode, so the one-time
// kernel attribute setup inside the launchers is allowed while capturing.
#include <cuda_runtime.h>

#include <new>

#include "../../include/raggedroute_b200.h"

struct rr_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int nodes = 0;
};

namespace {

rr_status st(int32_t code, const char* msg, int32_t cuda_err = 0) {
  rr_status s;
  s.code = code;
  s.cuda_error = cuda_err;
  s.message = msg;
  return s;
}

}  // namespace

extern "C" {

rr_status rr_graph_capture_begin(void* stream) {
  if (stream == nullptr) {
    return st(RR_INVALID_ARGUMENT, "capture needs a created stream (not the legacy default)");
  }
  const cudaError_t e =
      cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "cudaStreamBeginCapture failed", e);
  return st(RR_SUCCESS, "success");
}

rr_status rr_graph_capture_end(void* stream, rr_graph** out) {
  if (stream == nullptr || out == nullptr) {
    return st(RR_INVALID_ARGUMENT, "stream and out are required");
  }
  *out = nullptr;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &graph);
  if (e != cudaSuccess) {
    if (graph != nullptr) cudaGraphDestroy(graph);
    return st(RR_CUDA_ERROR, "cudaStreamEndCapture failed (an operation inside the capture "
                             "failed or was not capturable)", e);
  }
  rr_graph* g = new (std::nothrow) rr_graph();
  if (g == nullptr) {
    cudaGraphDestroy(graph);
    return st(RR_INVALID_ARGUMENT, "out of host memory");
  }
  g->graph = graph;
  size_t n = 0;
  if (cudaGraphGetNodes(graph, nullptr, &n) == cudaSuccess) g->nodes = static_cast<int>(n);
  e = cudaGraphInstantiate(&g->exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    delete g;
    return st(RR_CUDA_ERROR, "cudaGraphInstantiate failed", e);
  }
  *out = g;
  return st(RR_SUCCESS, "success");
}

rr_status rr_graph_launch(rr_graph* g, void* stream) {
  if (g == nullptr) return st(RR_INVALID_ARGUMENT, "graph must not be null");
  const cudaError_t e = cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "cudaGraphLaunch failed", e);
  return st(RR_SUCCESS, "success");
}

int rr_graph_node_count(const rr_graph* g) { return g != nullptr ? g->nodes : 0; }

rr_status rr_graph_destroy(rr_graph* g) {
  if (g != nullptr) {
    if (g->exec != nullptr) cudaGraphExecDestroy(g->exec);
    if (g->graph != nullptr) cudaGraphDestroy(g->graph);
    delete g;
  }
  return st(RR_SUCCESS, "success");
}

}  // extern "C"
