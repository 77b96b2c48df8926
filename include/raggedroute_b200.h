/*
 * raggedroute_b200.h -- C ABI of the B200-native RaggedRoute routing path.
 *
 * libraggedroute_b200.so exports these entry points for any FFI (ctypes, cgo,
 * JNI, N-API). Every buffer is a CUDA device pointer unless a comment says
 * otherwise; every call enqueues on ctx->stream and never synchronizes, never
 * allocates on the hot path and validates all arguments before any launch.
 * Storage is FP32 (int32 for ids/counts/offsets/positions), contiguous,
 * row-major. Each entry point cites the RaggedRoute interface it replaces
 * (path:line relative to the RaggedRoute project root).
 *
 * Library-wide limits: 1 <= experts <= RR_MAX_EXPERTS (the reference caps
 * at 64), route counts and element offsets fit int32 indexing as in the
 * reference.
 */
#ifndef RAGGEDROUTE_B200_H_
#define RAGGEDROUTE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RR_MAX_EXPERTS 1024

/* Status codes; values 0..7 equal raggedroute::StatusCode
 * (include/raggedroute/status.h:7-16). RR_COMM_ERROR is new (expert
 * parallelism only). */
enum {
  RR_SUCCESS = 0,
  RR_INVALID_ARGUMENT = 1,
  RR_UNSUPPORTED_ARCHITECTURE = 2,
  RR_UNSUPPORTED_DATA_TYPE = 3,
  RR_UNSUPPORTED_LAYOUT = 4,
  RR_UNSUPPORTED_KERNEL_VARIANT = 5,
  RR_INSUFFICIENT_WORKSPACE = 6,
  RR_CUDA_ERROR = 7,
  RR_COMM_ERROR = 8
};

/* Architecture values equal raggedroute::DeviceArchitecture
 * (include/raggedroute/types.h:20-25) plus RR_ARCH_SM100. */
enum { RR_ARCH_AUTO = 0, RR_ARCH_SM86 = 1, RR_ARCH_SM90 = 2, RR_ARCH_OTHER = 3, RR_ARCH_SM100 = 4 };

/* Kernel families equal raggedroute::KernelFamily (types.h:29-33). */
enum { RR_FAMILY_AUTO = 0, RR_FAMILY_CUDA_NAIVE = 1, RR_FAMILY_CUDA_OPTIMIZED = 2 };

/* Replaces raggedroute::Status (include/raggedroute/status.h:18-27). message
 * points to static storage and is never freed. */
typedef struct rr_status {
  int32_t code;
  int32_t cuda_error; /* cudaError_t value */
  const char* message;
} rr_status;

/* Replaces raggedroute::RuntimeContext (include/raggedroute/runtime.h:13-18)
 * plus the KernelSelection carried by every reference argument struct
 * (include/raggedroute/types.h:35-40). */
typedef struct rr_context {
  void* stream; /* cudaStream_t; NULL = legacy default stream */
  void* workspace;
  size_t workspace_bytes;
  int32_t architecture;       /* RR_ARCH_* */
  int32_t kernel_family;      /* RR_FAMILY_* */
  uint32_t implementation_id; /* operator-local research id, 0 = default */
} rr_context;

/* ---- operators (include/raggedroute/operators.h:114-135) ---------------- */

/* raggedroute::dense_gemm, src/dense_gemm/operator.cpp:18-58.
 * C[m,n] = A[m,k] . B[k,n]; alpha = 1, beta = 0 only. */
rr_status rr_dense_gemm(const float* a, const float* b, float* c, int m, int n, int k,
                        const rr_context* ctx);
size_t rr_dense_gemm_workspace_size(int m, int n, int k);

/* raggedroute::topk_gate, src/topk_gate/operator.cpp:18-60. Deterministic top-2
 * selected softmax; ties go to the lower expert id, NaN reads as -inf, an
 * all-NaN row yields ids {0,1} and weights {0.5,0.5}. top_k must be 2. */
rr_status rr_topk_gate(const float* logits, int32_t* expert_ids, float* weights, int tokens,
                       int experts, int top_k, const rr_context* ctx);
size_t rr_topk_gate_workspace_size(int tokens, int experts);

/* rr_topk_gate with an optional per-expert bias[experts] added to every logit
 * row before selection (NULL = rr_topk_gate). No reference counterpart: the
 * expert-parallel configuration skews expert load through this bias, and
 * the chain entry points use it as their gate stage. */
rr_status rr_topk_gate_biased(const float* logits, const float* logit_bias, int32_t* expert_ids,
                              float* weights, int tokens, int experts, int top_k,
                              const rr_context* ctx);

/* raggedroute::histogram, src/histogram/operator.cpp:20-57. counts is reset
 * inside the call; ids outside [0, experts) are skipped. */
rr_status rr_histogram(const int32_t* expert_ids, int32_t* counts, int route_pairs, int experts,
                       const rr_context* ctx);
size_t rr_histogram_workspace_size(int route_pairs, int experts);

/* raggedroute::exclusive_scan, src/scan/operator.cpp:51-74. offsets[E+1];
 * counts and offsets may alias (in-place scan). */
rr_status rr_exclusive_scan(const int32_t* counts, int32_t* offsets, int experts,
                            const rr_context* ctx);
size_t rr_exclusive_scan_workspace_size(int experts);

/* raggedroute::histogram_exclusive_scan, src/scan/operator.cpp:84-134.
 * The input and both outputs must be pairwise non-overlapping. */
rr_status rr_histogram_exclusive_scan(const int32_t* expert_ids, int32_t* counts,
                                      int32_t* offsets, int route_pairs, int experts,
                                      const rr_context* ctx);
size_t rr_histogram_exclusive_scan_workspace_size(int route_pairs, int experts);

/* raggedroute::token_permute, src/permute/operator.cpp:22-83.
 * route_pos[r] = offsets[ids[r]] + #{r' < r : ids[r'] == ids[r]} (stable,
 * route-ascending within each expert segment); x_permuted[route_pos[r], :] =
 * x[r / top_k, :]; sorted_route (optional, may be NULL) is the inverse map.
 * ctx->workspace must hold rr_token_permute_workspace_size(...) bytes (the
 * reference's experts * 4, whatever the number of tokens); its
 * first experts int32 entries end equal to the per-expert route counts (the
 * reference's cursor post-state). */
rr_status rr_token_permute(const float* x, const int32_t* expert_ids, const int32_t* offsets,
                           float* x_permuted, int32_t* route_pos, int32_t* sorted_route,
                           int tokens, int experts, int top_k, int hidden,
                           const rr_context* ctx);
size_t rr_token_permute_workspace_size(int tokens, int experts, int top_k, int hidden);

/* rr_token_permute for callers that cannot allocate device memory: same
 * arguments, results and checks, but ctx->workspace is ignored and the
 * scratch lives in a fixed 4 KB array inside the library (1024 int32, held
 * by every GPU that loads it until exit). It has no counterpart in the
 * reference; it exists for callers whose device memory is owned by a planner
 * or pool with nothing spare, or that reach this library through a binding
 * without access to a CUDA allocator. A call whose
 * rr_token_permute_workspace_size exceeds the array fails with
 * RR_INVALID_ARGUMENT (checked right after the shape checks; every other
 * check is rr_token_permute's, dispatch checks first).
 * It never allocates or frees. All calls share the array, so calls that
 * overlap on the GPU race and must be serialised by the caller. The array's
 * address is looked up on the first call in each CUDA context (the first
 * call on a device, and the first after that device's context was reset or
 * replaced) and cached under the context's id; that first call should come
 * before any stream capture. */
rr_status rr_token_permute_no_alloc(const float* x, const int32_t* expert_ids,
                                    const int32_t* offsets, float* x_permuted, int32_t* route_pos,
                                    int32_t* sorted_route, int tokens, int experts, int top_k,
                                    int hidden, const rr_context* ctx);

/* raggedroute::grouped_gemm, src/grouped_gemm/operator.cpp:17-49.
 * y_permuted[r, :] = x_permuted[r, :] . W[e] for r in [offsets[e],
 * offsets[e+1]); W is [experts, hidden, output]. max_expert_tokens is the
 * caller's launch bound (0 = no-op); the tile schedule itself is read from
 * offsets on the device, so it may be any positive value. */
rr_status rr_grouped_gemm(const float* x_permuted, const float* expert_weights,
                          const int32_t* offsets, float* y_permuted, int experts, int hidden,
                          int output, int max_expert_tokens, const rr_context* ctx);
size_t rr_grouped_gemm_workspace_size(int experts, int hidden, int output);

/* raggedroute::unpermute, src/unpermute/operator.cpp:19-57.
 * y[t, c] = sum_k w[t*top_k+k] * y_permuted[route_pos[t*top_k+k], c], summed
 * in rank order. */
rr_status rr_unpermute(const float* y_permuted, const int32_t* route_pos,
                       const float* route_weights, float* y, int tokens, int top_k, int output,
                       const rr_context* ctx);
size_t rr_unpermute_workspace_size(int tokens, int top_k, int output);

/* ---- L3 chains (benchmarks/adapters/chain_adapter.cpp:263-467) ----------- */

/* Chains read ctx->implementation_id as a set of bits; 0 (default) runs
 * every stage as its own operator and leaves each intermediate buffer
 * holding its stage's result.
 * RR_CHAIN_IMPL_GATHER_ROWS has the grouped GEMM gather its rows from x
 * through sorted_route (the permute only ranks), so x_permuted is not
 * written (may be NULL) and the permute's row copy and the GEMM's re-read
 * of it disappear; outputs are bit-identical. RR_CHAIN_IMPL_PREPARED_WEIGHTS
 * (token and logit chains) takes expert_weights as a buffer filled by
 * rr_prepare_expert_weights (below). RR_CHAIN_IMPL_FUSED_COMBINE runs the
 * unpermute inside the grouped GEMM's epilogue (every output row weighted
 * and added into its token's row of y with a global float reduction; y is
 * zeroed first), so y_permuted is not written (may be NULL) and the
 * unpermute launch disappears; y is bit-identical (top_k <= 2 only: the
 * route-id chain returns RR_UNSUPPORTED_KERNEL_VARIANT above 2 and then
 * needs sorted_route). FUSED_COMBINE combines with either of the other two;
 * GATHER_ROWS with PREPARED_WEIGHTS, and any other bit, is
 * RR_UNSUPPORTED_KERNEL_VARIANT. None has a reference counterpart. */
#define RR_CHAIN_IMPL_GATHER_ROWS 1u
#define RR_CHAIN_IMPL_PREPARED_WEIGHTS 2u
#define RR_CHAIN_IMPL_FUSED_COMBINE 4u

/* ---- prepared expert weights (new: no reference counterpart) -------------
 * For expert weights that stay fixed across calls (inference), the B side
 * of the 3xTF32 split is done once: W [E][K][N] is written as two K-major
 * arrays [E][N][K], hi = W and lo = W - (W with its low 13 mantissa bits
 * cleared), into a caller buffer of rr_prepared_expert_weights_size bytes
 * (256-byte aligned; 2x the weights). The grouped GEMM then loads both B
 * operands ready for its MMAs and splits only the token rows. K and N must
 * be multiples of 4. Results differ from the raw-weight path in the last
 * bits (B hi is truncated instead of rounded); both hold the FP32 contract. */
size_t rr_prepared_expert_weights_size(int experts, int hidden, int output);
rr_status rr_prepare_expert_weights(const float* expert_weights, int experts, int hidden,
                                    int output, void* prepared, size_t prepared_bytes,
                                    const rr_context* ctx);
/* grouped_gemm on prepared weights: y_permuted[r] = x_permuted[r] . W[e]
 * for r in [offsets[e], offsets[e+1]). */
rr_status rr_grouped_gemm_prepared(const float* x_permuted, const void* prepared,
                                   const int32_t* offsets, float* y_permuted, int experts,
                                   int hidden, int output, int route_pairs,
                                   const rr_context* ctx);

/* chain_from_tokens: dense_gemm -> topk_gate -> histogram_exclusive_scan ->
 * token_permute -> grouped_gemm -> unpermute on ctx->stream, no host sync.
 * Intermediate buffers are caller-owned and are left holding each stage's
 * result: logits[T,E], expert_ids[T,2], route_weights[T,2], counts[E],
 * offsets[E+1], x_permuted[2T,K], route_pos[2T], y_permuted[2T,N]; y[T,N] is
 * the output. logit_bias (optional, [E]) is added to every logit row before
 * the gate (NULL in the reference chain). ctx->workspace must hold
 * rr_chain_workspace_size(...) bytes. */
rr_status rr_chain_from_tokens(const float* x, const float* router_weights,
                               const float* logit_bias, const float* expert_weights,
                               float* logits, int32_t* expert_ids, float* route_weights,
                               int32_t* counts, int32_t* offsets, float* x_permuted,
                               int32_t* route_pos, float* y_permuted, float* y, int tokens,
                               int hidden, int experts, int output, const rr_context* ctx);

/* chain_from_logits: the same chain starting from caller-provided logits. */
/* Grouped GEMM with row gather (the reference's research entry point
 * launch_grouped_gemm_sm86_fp32_gather_v1, src/grouped_gemm/cuda_candidate/
 * grouped_optimized_internal.h:105-109): row r of segment e is
 * x[sorted_route[r] / top_k] . W[e]; y_permuted [R, N]. */
rr_status rr_grouped_gemm_gather(const float* x, const int32_t* sorted_route, int top_k,
                                 const float* expert_weights, const int32_t* offsets,
                                 float* y_permuted, int route_pairs, int hidden, int experts,
                                 int output, const rr_context* ctx);

/* Grouped GEMM with the unpermute fused into its epilogue (new: no
 * reference counterpart; the fused form of raggedroute::grouped_gemm followed
 * by raggedroute::unpermute, src/grouped_gemm/operator.cpp and
 * src/unpermute/operator.cpp). y [tokens, N] is zeroed, then row r of segment
 * e (route q = sorted_route[r]) adds route_weights[q] * (x_permuted[r] .
 * W[e]) into y[q / top_k]. sorted_route is the stable permute's [R] route
 * order, route_weights the gate's [R] weights; R = route_pairs <= tokens *
 * top_k. top_k 1 or 2: y then equals rr_grouped_gemm followed by
 * rr_unpermute bit for bit (both round each product, then add with
 * subnormal operands and results flushed to zero; two terms in either order
 * give the same sum). */
rr_status rr_grouped_gemm_combine(const float* x_permuted, const float* expert_weights,
                                  const int32_t* offsets, const int32_t* sorted_route,
                                  const float* route_weights, float* y, int experts, int hidden,
                                  int output, int route_pairs, int tokens, int top_k,
                                  const rr_context* ctx);

/* Grouped GEMM with a row-address epilogue (new: the expert-parallel combine
 * step). Output row r of segment e is stored at bases[b] + row * N where
 * row_address[r] = (b << 40) | row; rows whose address is negative, whose b
 * is not below nbases or whose row is not below row_limit are not stored.
 * bases is a DEVICE array of nbases row-buffer pointers (this process's
 * mappings of other GPUs' buffers included). The kernel ends with a
 * system-scope fence so a following barrier publishes the rows. */
rr_status rr_grouped_gemm_scatter(const float* x_permuted, const float* expert_weights,
                                  const int32_t* offsets, const int64_t* row_address,
                                  float* const* bases, int nbases, int64_t row_limit,
                                  int experts, int hidden, int output, int route_pairs,
                                  const rr_context* ctx);

rr_status rr_chain_from_logits(const float* logits, const float* x, const float* expert_weights,
                               int32_t* expert_ids, float* route_weights, int32_t* counts,
                               int32_t* offsets, float* x_permuted, int32_t* route_pos,
                               float* y_permuted, float* y, int tokens, int hidden, int experts,
                               int output, const rr_context* ctx);
size_t rr_chain_workspace_size(int tokens, int hidden, int experts, int output);

/* chain_from_route_ids (benchmarks/adapters/postroute_chain_adapter.cpp:
 * 240-354): routing already decided, R = T*top_k routes with 1 <= top_k <=
 * min(8, E). histogram + scan -> stable token_permute (route_pos, and
 * sorted_route when non-NULL) -> grouped_gemm -> unpermute. expert_ids and
 * route_weights are [T, top_k]; x_permuted [R, K], y_permuted [R, N], y
 * [T, N]; ctx->workspace holds rr_route_chain_workspace_size(T, top_k, E)
 * bytes. */
rr_status rr_chain_from_route_ids(const float* x, const int32_t* expert_ids,
                                  const float* route_weights, const float* expert_weights,
                                  int32_t* counts, int32_t* offsets, float* x_permuted,
                                  int32_t* route_pos, int32_t* sorted_route, float* y_permuted,
                                  float* y, int tokens, int top_k, int hidden, int experts,
                                  int output, const rr_context* ctx);
size_t rr_route_chain_workspace_size(int tokens, int top_k, int experts);

/* ---- route traces (include/raggedroute/benchmark/adapter_utils.h:250-322) --
 * Reads frame `frame` of a "raggedroute.route_trace.v1" text file (.rrtrace)
 * with the reference loader's validation (header, portable ids, source kind,
 * ids in [0, E) and distinct within a token, no trailing data; E <= 1024
 * here). expert_ids (host, may be NULL to read the header only) receives
 * tokens*top_k ids. */
typedef struct rr_route_trace_info {
  int32_t tokens;
  int32_t experts;
  int32_t top_k;
  int32_t frame_count;
  char trace_id[128];
  char source_kind[32];
  char frame_id[128];
} rr_route_trace_info;
rr_status rr_route_trace_read(const char* path, int frame, rr_route_trace_info* info,
                              int32_t* expert_ids, int64_t ids_capacity);
/* Host logits [tokens, experts] that make the top-2 gate pick a top-2
 * frame's ids in order (benchmarks/adapters/chain_adapter.cpp:222-228). */
rr_status rr_route_trace_logits(const int32_t* expert_ids, int tokens, int experts,
                                float* logits);

/* ---- CUDA-graph capture (new: no reference counterpart) -------------------
 * Every rr_* operator and chain above enqueues without host synchronisation,
 * allocation or host reads of device data, and the grouped GEMM reads its
 * tile schedule from offsets on the device, so a sequence of calls can be
 * captured once and replayed with one launch: write new inputs into the
 * captured buffers (any routing, same shapes) and call rr_graph_launch.
 * Capture runs on a created stream in relaxed mode. The expert-parallel and
 * host-memory chains are not capturable (they synchronise with the host). */
typedef struct rr_graph rr_graph;
rr_status rr_graph_capture_begin(void* stream /* cudaStream_t, not NULL */);
rr_status rr_graph_capture_end(void* stream, rr_graph** out);
rr_status rr_graph_launch(rr_graph* graph, void* stream);
int rr_graph_node_count(const rr_graph* graph);
rr_status rr_graph_destroy(rr_graph* graph);

/* ---- chain over host memory (new: no reference counterpart) --------------
 * chain_from_tokens for tokens that live in host memory. The batch is cut
 * into chunks of chunk_tokens; each chunk's X is copied in on one copy
 * stream, runs the seven-stage chain on ctx->stream and its Y is copied out
 * on another, with two device slots, so the copies of neighbouring chunks
 * overlap the chain. Y is bit-identical to rr_chain_from_tokens over the
 * whole batch. Plan-time allocation only (two slots of chain buffers). */
typedef struct rr_host_chain rr_host_chain;
rr_status rr_host_chain_create(int chunk_tokens, int hidden, int experts, int output,
                               rr_host_chain** out);
rr_status rr_host_chain_destroy(rr_host_chain* plan);
/* Plan flags (rr_host_chain_set_flags; 0 by default).
 * RR_HOST_CHAIN_INPUT_READY: x_host is complete when the call is made (the
 * caller does not produce it with work enqueued earlier on ctx->stream), so
 * the host-to-device copies need not wait for that work. Back-to-back calls
 * then overlap: the first copies of a call run while the previous call's
 * last chunks compute and copy out. The chain itself and the completion of
 * the call stay ordered on ctx->stream either way. */
#define RR_HOST_CHAIN_INPUT_READY 1u
rr_status rr_host_chain_set_flags(rr_host_chain* plan, uint32_t flags);
/* x_host [tokens, K] and y_host [tokens, N] should be pinned (pageable
 * memory works but serialises the copies). router_weights, logit_bias
 * (optional) and expert_weights are device buffers as for
 * rr_chain_from_tokens. expert_ids_host / route_weights_host ([tokens, 2],
 * optional) receive the routing decisions. Enqueue only; completion is
 * ordered on ctx->stream (ctx->workspace is not used). One call at a time
 * per plan. */
rr_status rr_chain_from_tokens_host(rr_host_chain* plan, const float* x_host,
                                    const float* router_weights, const float* logit_bias,
                                    const float* expert_weights, float* y_host,
                                    int32_t* expert_ids_host, float* route_weights_host,
                                    int tokens, const rr_context* ctx);

/* ---- expert parallelism (new: the reference is single-GPU) ----------------
 * One process per GPU. The router scores R real experts; the gate maps each
 * selected id through a per-rank remap table to one of V virtual experts
 * (a real expert's weights on one rank; hot experts get several), and rank
 * g owns virtual experts [g*V/G, (g+1)*V/G). Two transports move the rows:
 *
 * RR_EP_TRANSPORT_PEER (one node, GPUs that map each other's memory): every
 *   rank's receive buffers are mapped into every other rank at create time.
 *   A step runs the local routing stages, all-gathers the per-virtual-expert
 *   counts, and then the permute kernel writes each route's row straight into
 *   its owner's receive buffer (dispatch fused into the permute), the owner's
 *   grouped GEMM writes each output row straight back into the source rank's
 *   buffer (combine fused into the GEMM epilogue), and the source
 *   unpermutes. Two one-word NCCL all-reduces order the phases across ranks.
 *   No host synchronisation inside a step; x_permuted and y_permuted are not
 *   used (may be NULL).
 * RR_EP_TRANSPORT_NCCL: x_permuted rows move with NCCL send/recv in pairwise
 *   rounds overlapped with the grouped GEMM of arrived blocks and come back
 *   the same way into y_permuted; one pinned host read of the counts per step
 *   sizes the rounds.
 * RR_EP_TRANSPORT_AUTO picks PEER when every rank can map every other rank's
 * memory, else NCCL. All work is ordered on ctx->stream. Every host wait has
 * a deadline; on expiry the communicator is aborted and RR_COMM_ERROR
 * returned. */
#define RR_EP_UNIQUE_ID_BYTES 128
#define RR_EP_TRANSPORT_AUTO 0
#define RR_EP_TRANSPORT_NCCL 1
#define RR_EP_TRANSPORT_PEER 2
typedef struct rr_ep rr_ep;

/* Rank 0 creates the id; the caller distributes it to the other ranks. */
rr_status rr_ep_get_unique_id(void* unique_id /* RR_EP_UNIQUE_ID_BYTES, host */);
/* Plan-time: NCCL communicator (non-blocking), worst-case receive buffers
 * (nranks * 2 * max_tokens rows, below 2^31) and, for the peer transport,
 * the cross-rank mappings. experts must be a multiple of nranks. Collective:
 * every rank calls it with the same sizes and transport. */
rr_status rr_ep_create(const void* unique_id, int nranks, int rank, int router_experts,
                       int experts, int max_tokens, int hidden, int output,
                       double timeout_seconds, int transport, rr_ep** out);
/* Collective when nranks > 1 (a barrier precedes the unmapping). */
rr_status rr_ep_destroy(rr_ep* ep);
/* The transport the plan uses (RR_EP_TRANSPORT_NCCL or _PEER). */
rr_status rr_ep_transport(const rr_ep* ep, int* transport);
/* chain_from_tokens across ranks: x [tokens, K]; router weights [K, R] and
 * bias [R] (optional) replicated on every rank; expert_remap [R] (device;
 * NULL only when R == V) maps this rank's routes to virtual experts;
 * local_expert_weights [V/G, K, N] are this rank's virtual experts. logits is
 * [tokens, R]; expert_ids receive virtual ids; counts/offsets are over V;
 * ctx->workspace holds rr_chain_workspace_size(tokens, K, V, N) bytes. */
rr_status rr_ep_chain_from_tokens(rr_ep* ep, const float* x, const float* router_weights,
                                  const float* logit_bias, const int32_t* expert_remap,
                                  const float* local_expert_weights,
                                  float* logits, int32_t* expert_ids, float* route_weights,
                                  int32_t* counts, int32_t* offsets, float* x_permuted,
                                  int32_t* route_pos, float* y_permuted, float* y, int tokens,
                                  const rr_context* ctx);
/* Rows this rank sent / received in its last step (load-balance reporting);
 * waits, with the plan's deadline, for that step to finish on the device. */
rr_status rr_ep_last_step_rows(const rr_ep* ep, int64_t* rows_sent, int64_t* rows_received);
/* The exchange plan of one rank from the [nranks][experts] counts (pure host
 * arithmetic): rows sent to / received from each peer and block offsets. */
rr_status rr_ep_plan(const int32_t* count_all, int nranks, int rank, int experts,
                     int64_t* send_rows, int64_t* send_offsets, int64_t* recv_rows,
                     int64_t* recv_offsets);

/* ---- low-level launchers (include/raggedroute/baseline_ops.h:14-42) ------
 * Return a cudaError_t value: cudaErrorInvalidValue (1) on bad arguments,
 * cudaSuccess for empty work. Preconditions as in the reference: histogram
 * counts and permute cursors are zeroed by the caller (the launchers
 * accumulate into them). */
int rr_launch_dense_gemm_naive(const float* a, const float* b, float* c, int m, int n, int k,
                               void* stream);
int rr_launch_topk_gate_naive(const float* logits, int32_t* expert_ids, float* weights,
                              int tokens, int experts, void* stream);
int rr_launch_histogram_naive(const int32_t* expert_ids, int32_t* counts, int route_pairs,
                              int experts, void* stream);
int rr_launch_exclusive_scan_naive(const int32_t* counts, int32_t* offsets, int experts,
                                   void* stream);
int rr_launch_token_permute_naive(const float* x, const int32_t* expert_ids,
                                  const int32_t* offsets, int32_t* cursors, float* x_permuted,
                                  int32_t* route_pos, int32_t* sorted_route, int tokens,
                                  int top_k, int hidden, void* stream);
int rr_launch_grouped_gemm_naive(const float* x_permuted, const float* expert_weights,
                                 const int32_t* offsets, float* y_permuted, int experts,
                                 int hidden, int output, int max_expert_tokens, void* stream);
int rr_launch_unpermute_naive(const float* y_permuted, const int32_t* route_pos,
                              const float* route_weights, float* y, int tokens, int top_k,
                              int output, void* stream);
/* src/benchmark/cache_scrub.cu:17-50: rewrites a scrub buffer to evict L2. */
int rr_launch_cache_scrub(uint32_t* buffer, size_t elements, void* stream);

/* ---- dispatch (include/raggedroute/dispatch.h:32-46) --------------------- */
/* Maps a compute capability to RR_ARCH_*; only 10.0 is RR_ARCH_SM100. */
int32_t rr_classify_compute_capability(int major, int minor);
/* Resolves the current CUDA device's architecture. */
rr_status rr_query_current_device_architecture(int32_t* architecture);

/* ---- library introspection (new) ---------------------------------------- */
/* Number of CUDA kernels this library has launched in this process. */
uint64_t rr_kernel_launch_count(void);
/* Reads and clears the device-side error word set by bounded waits in the
 * library's kernels (0 = no error). Synchronizes the given stream. */
rr_status rr_consume_device_error(void* stream, uint32_t* error_word);
/* Which grouped-GEMM engine a shape takes (plain grouped GEMM, no row
 * gathering or prepared weights): 1 = tcgen05 with the 3xTF32 split, 2 = FP32
 * SIMT, 3 = tcgen05 CTA pairs with the mixed split (TF32 hi.hi plus bfloat16
 * corrections; K >= 128 unless RAGGEDROUTE_B200_GEMM_MIXED=0). */
int rr_grouped_gemm_engine(const float* x_permuted, const float* expert_weights,
                           float* y_permuted, int hidden, int output);
const char* rr_version(void);
/* Failure-detection self-test (no reference counterpart): launches a kernel
 * that waits, through the same bounded mbarrier wait the GEMM uses, on a
 * barrier nothing arrives on. After limit_ns the wait gives up, the kernel
 * sets bit 0 (timeout) of the device error word and returns; elapsed_ns
 * (device) receives the time waited. Read the word with
 * rr_consume_device_error. */
rr_status rr_bounded_wait_selftest(uint64_t limit_ns, unsigned long long* elapsed_ns,
                                   void* stream);
/* Device self-check of the GEMM's TF32 split (no reference counterpart):
 * adds to *mismatches (device, caller-zeroed) the number of the n bit
 * patterns (device) whose integer round-to-nearest-away TF32 rounding
 * differs from the cvt.rna.tf32.f32 instruction; NaN patterns are skipped. */
rr_status rr_tf32_rounding_selfcheck(const uint32_t* bits, int64_t n,
                                     unsigned long long* mismatches, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* RAGGEDROUTE_B200_H_ */
