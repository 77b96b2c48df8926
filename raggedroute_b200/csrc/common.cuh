// Shared device helpers and the internal launcher interface of
// libraggedroute_b200. Every launcher here enqueues on the given stream,
// performs no allocation and no host synchronization, and returns the launch
// status from cudaGetLastError().
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace rrb {

constexpr int kMaxExperts = 1024;
constexpr int kNumSms = 148;  // B200; the launchers query the real count once.

// Bits of the device error word (set by bounded waits, read by
// rr_consume_device_error).
constexpr unsigned kErrMbarTimeout = 1u << 0;
constexpr unsigned kErrTmemAlloc = 1u << 1;
constexpr unsigned kErrScheduler = 1u << 2;
constexpr unsigned kErrEpCapacity = 1u << 3;

// Expert-parallel peer transport. A packed row address names a row of a
// buffer that one rank owns: (rank << kPeerRankShift) | row.
constexpr int kPeerRankShift = 40;
constexpr long long kPeerRowMask = (1LL << kPeerRankShift) - 1;

// Output-row redirection for a GEMM: output row r is written to
// base[dst[r] >> 40] + (dst[r] & kPeerRowMask) * output. base is a device
// array of one pointer per rank (this process's mapping of every rank's
// buffer, its own included). An address whose rank is not below nranks or
// whose row is not below row_limit is not stored.
//
// Combine mode (combine != nullptr, dst == nullptr): the unpermute fused
// into the epilogue. Output row r belongs to route q = route[r] (the stable
// permute's sorted_route); it is multiplied by weight[q] (rounded product)
// and added with one global float reduction into row q / top_k of combine,
// which must hold zeros before the launch. The reduction adds with
// round-to-nearest and flushes subnormal operands and results to zero
// (measured on sm_100); for top_k <= 2 the result,
// ftz(ftz(0 + a) + b) = ftz(a + b), does not depend on which of a token's
// two rows lands first, and equals launch_unpermute's rank-order sum.
struct RowScatter {
  const int64_t* dst = nullptr;
  float* const* base = nullptr;
  int nranks = 0;
  long long row_limit = 0;
  // Abort fence (optional, host memory mapped into the device): read once at
  // kernel start; when non-zero no row is stored.
  const volatile int* abort = nullptr;
  float* combine = nullptr;
  const int32_t* route = nullptr;
  const float* weight = nullptr;
  int top_k = 1;
  // > 0: the persistent GEMM uses at most this many SMs (CTAs), leaving the
  // rest to a kernel that runs beside it (the expert-parallel dispatch).
  int max_ctas = 0;
};

// Resolves a packed row address, or nullptr when it is out of range.
__device__ __forceinline__ float* scatter_row(const RowScatter& sc, long long row, int output) {
  const long long d = __ldg(sc.dst + row);
  const long long rank = d >> kPeerRankShift;
  const long long r = d & kPeerRowMask;
  if (d < 0 || rank >= sc.nranks || r >= sc.row_limit) return nullptr;
  return sc.base[rank] + r * output;
}

// Combine mode: the token row that output row `row` adds into, and its
// route weight.
__device__ __forceinline__ float* combine_row(const RowScatter& sc, long long row, int output,
                                              float& weight) {
  const int q = __ldg(sc.route + row);
  weight = __ldg(sc.weight + q);
  return sc.combine + static_cast<long long>(q / sc.top_k) * output;
}

// Global float reductions (no return value): round to nearest, subnormal
// operands and results flushed to zero.
__device__ __forceinline__ void red_add_f32(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}
__device__ __forceinline__ void red_add_v4_f32(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// acc + v rounded to nearest with subnormal operands and result flushed to
// zero: the arithmetic of red_add_f32, for sums that must equal it.
__device__ __forceinline__ float add_ftz(float acc, float v) {
  float r;
  asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(acc), "f"(v));
  return r;
}

// Row gather for a GEMM's A operand: row r of the problem is row
// route[r] / div of x (the token matrix), so no permuted copy of x is
// materialised (route = sorted_route of the stable permute, div = top_k).
struct RowGather {
  const float* x = nullptr;
  const int32_t* route = nullptr;
  int div = 1;
};

// Dispatch side of the peer transport, used by the token permute: a route to
// virtual expert e (owner rank e / local) is copied to
// x_base[owner] + (dest_off[e] + rank of the route inside e) * hidden, and
// its return address (me << 40 | local permuted slot) goes to
// ret_base[owner][same row]. Rows at or beyond `capacity` are dropped and
// flagged (kErrEpCapacity).
struct PeerDispatch {
  float* const* x_base = nullptr;
  int64_t* const* ret_base = nullptr;
  const int32_t* dest_off = nullptr;
  int local = 1;
  int me = 0;
  long long capacity = 0;
  unsigned* err = nullptr;
  // Abort fence, as in RowScatter: when set at kernel start, nothing is
  // written to any rank's buffers.
  const volatile int* abort = nullptr;
  // Only routes whose local expert index (expert % local) is in
  // [le_lo, le_hi) are sent (a dispatch split by expert range).
  int le_lo = 0;
  int le_hi = 1 << 30;
};

// Counts every kernel this library launches (for the bench's launch claim).
void note_launch(int n = 1);
int sm_count();
unsigned* device_error_word();

__device__ __forceinline__ void raise_device_error(unsigned* word, unsigned bits) {
  if (word != nullptr) atomicOr(word, bits);
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

inline bool aligned_to(const void* p, std::size_t a) {
  return (reinterpret_cast<std::uintptr_t>(p) % a) == 0;
}

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// ---- launchers (implemented in the .cu files) -------------------------------

// topk_gate.cu. remap (optional, [experts]) replaces each selected id by
// remap[id] on output (the expert-parallel runtime's virtual expert ids).
cudaError_t launch_topk_gate(const float* logits, const float* bias, int32_t* ids, float* weights,
                             int tokens, int experts, cudaStream_t stream,
                             const int32_t* remap = nullptr);

// routing.cu
cudaError_t launch_histogram_accumulate(const int32_t* ids, int32_t* counts, int routes,
                                        int experts, cudaStream_t stream);
// Histogram that overwrites counts (the reset is part of the call).
cudaError_t launch_histogram(const int32_t* ids, int32_t* counts, int routes, int experts,
                             cudaStream_t stream);
cudaError_t launch_exclusive_scan(const int32_t* counts, int32_t* offsets, int experts,
                                  cudaStream_t stream);
// Fused histogram + exclusive scan; overwrites counts and offsets (reset is
// part of the call).
cudaError_t launch_histogram_exclusive_scan(const int32_t* ids, int32_t* counts,
                                            int32_t* offsets, int routes, int experts,
                                            cudaStream_t stream);

// Expert-parallel receive offsets (nranks * local <= 1024 groups).
cudaError_t launch_ep_recv_offsets(const int32_t* count_all, int32_t* recv_offsets, int nranks,
                                   int experts, int rank, int local, cudaStream_t stream);
// Peer-transport layout from count_all [nranks][experts]: every rank's
// receive buffer is expert-major (local expert, then source rank). Writes
// dest_off[experts] (where this rank's rows of each expert start on its
// owner) and recv_offsets[local + 1] (this rank's grouped-GEMM offsets,
// clipped to capacity; an overflow sets kErrEpCapacity in err).
cudaError_t launch_ep_peer_layout(const int32_t* count_all, int32_t* dest_off,
                                  int32_t* recv_offsets, int nranks, int experts, int rank,
                                  int local, long long capacity, unsigned* err,
                                  cudaStream_t stream);

// permute.cu
std::size_t permute_workspace_bytes(int tokens, int experts, int top_k);
// Stable permute; workspace holds >= permute_workspace_bytes(...) bytes and
// its first `experts` ints end as the per-expert counts.
cudaError_t launch_token_permute(const float* x, const int32_t* ids, const int32_t* offsets,
                                 float* x_permuted, int32_t* route_pos, int32_t* sorted_route,
                                 int tokens, int experts, int top_k, int hidden, void* workspace,
                                 cudaStream_t stream);
// The same permute (identical route_pos) whose copy goes to other ranks'
// receive buffers through the peer mapping instead of to x_permuted (only
// the routes in peer's local-expert range).
cudaError_t launch_token_permute_peer(const float* x, const int32_t* ids, const int32_t* offsets,
                                      int32_t* route_pos, int tokens, int experts, int top_k,
                                      int hidden, void* workspace, const PeerDispatch& peer,
                                      cudaStream_t stream);
// The rest of a split dispatch, after launch_token_permute_peer wrote
// route_pos: the routes in peer's local-expert range are sent from `sms`
// SMs (an even number; clusters of two CTAs, one CTA per SM) so that it can
// run beside a grouped GEMM limited to the other SMs.
cudaError_t launch_ep_dispatch_rest(const float* x, const int32_t* ids, const int32_t* offsets,
                                    const int32_t* route_pos, int tokens, int experts, int top_k,
                                    int hidden, const PeerDispatch& peer, int sms,
                                    cudaStream_t stream);
// Workspace-free stable permute for the low-level launcher: the expert count
// is unknown, cursors accumulate (caller zeroes them).
cudaError_t launch_token_permute_cursor(const float* x, const int32_t* ids,
                                        const int32_t* offsets, int32_t* cursors,
                                        float* x_permuted, int32_t* route_pos,
                                        int32_t* sorted_route, int tokens, int top_k, int hidden,
                                        cudaStream_t stream);

// unpermute.cu
cudaError_t launch_unpermute(const float* y_permuted, const int32_t* route_pos,
                             const float* route_weights, float* y, int tokens, int top_k,
                             int output, cudaStream_t stream);

// gemm_simt.cu / gemm_tc.cu
// Grouped GEMM with rows split by offsets[experts+1] (`experts` row groups);
// offsets == nullptr means one group covering `rows` rows (dense GEMM). Group
// g multiplies by weight set (g % weight_sets) of w[weight_sets, hidden,
// output]; weight_sets = 0 means one weight set per group. The
// expert-parallel runtime uses weight_sets < experts for its
// (source rank, local expert) groups. scatter (optional) redirects every
// stored output row (peer transport combine) or, in combine mode, adds it
// weighted into its token's row; y is then only an alignment witness for the
// engine choice. gather (optional, gather->x == x) reads A
// row r from x[route[r] / div] instead of x[r].
cudaError_t launch_grouped_gemm(const float* x, const float* w, const int32_t* offsets,
                                float* y, int experts, int rows, int hidden, int output,
                                cudaStream_t stream, int weight_sets = 0,
                                const RowScatter* scatter = nullptr,
                                const RowGather* gather = nullptr);
cudaError_t launch_grouped_gemm_simt(const float* x, const float* w, const int32_t* offsets,
                                     float* y, int experts, int rows, int hidden, int output,
                                     cudaStream_t stream, int weight_sets = 0,
                                     const RowScatter* scatter = nullptr,
                                     const RowGather* gather = nullptr);
bool tc_gemm_supported(const float* x, const float* w, const float* y, int hidden, int output);
// Dense GEMM with N <= 128 computed transposed (gemm_narrow.cu): y[rows,
// output] = x . w, x [rows, hidden], w [hidden, output]; hidden and output
// multiples of 4, 16-byte aligned buffers. cudaErrorNotSupported when the
// kernel cannot be configured. RAGGEDROUTE_B200_NARROW_DENSE=0 turns it off.
bool dense_narrow_enabled();
cudaError_t launch_dense_narrow(const float* x, const float* w, float* y, int rows, int hidden,
                                int output, cudaStream_t stream);
// CTA-pair engine (gemm_pair.cu) for the plain grouped/dense GEMM: 256 x 256
// tiles on two SMs. cudaErrorNotSupported when no pair can be scheduled.
bool gemm_pairs_enabled();
// Whether the pair engine runs the mixed split (TF32 hi.hi plus bfloat16
// corrections) for this K; RAGGEDROUTE_B200_GEMM_MIXED=0 keeps 3xTF32.
bool gemm_mixed_split(int hidden);
int grouped_gemm_pair_units();
cudaError_t launch_grouped_gemm_pair(const float* x, const float* w, const int32_t* offsets,
                                     float* y, int experts, int rows, int hidden, int output,
                                     cudaStream_t stream, int weight_sets,
                                     const RowScatter* scatter);
cudaError_t launch_grouped_gemm_tc(const float* x, const float* w, const int32_t* offsets,
                                   float* y, int experts, int rows, int hidden, int output,
                                   cudaStream_t stream, int weight_sets = 0,
                                   const RowScatter* scatter = nullptr,
                                   const RowGather* gather = nullptr);
// Grouped GEMM on prepared expert weights (w_hi, w_lo: K-major [E][N][K],
// hi = W, lo = W - trunc_tf32(W); prepare.cu). K and N multiples of 4, all
// buffers 16-byte aligned, else cudaErrorInvalidValue; no SIMT fallback.
// scatter as for launch_grouped_gemm.
cudaError_t launch_grouped_gemm_prepared(const float* x, const float* w_hi, const float* w_lo,
                                         const int32_t* offsets, float* y, int experts, int rows,
                                         int hidden, int output, cudaStream_t stream,
                                         const RowScatter* scatter = nullptr);

// The unpermute fused into the grouped GEMM (combine mode of RowScatter):
// zeroes y[tokens, output], then runs the grouped GEMM of x (or of the rows
// gather names) against w with every output row weighted and added into its
// token's row of y. top_k is 1 or 2 (where the sum does not depend on the
// order in which a token's rows land); sorted_route and route_weights are
// the stable permute's [R] route order and the gate's [R] weights.
// prepared_lo != nullptr: w is the hi half of prepared weights.
cudaError_t launch_grouped_gemm_combine(const float* x, const float* w, const float* prepared_lo,
                                        const int32_t* offsets, const int32_t* sorted_route,
                                        const float* route_weights, float* y, int experts,
                                        int rows, int tokens, int top_k, int hidden, int output,
                                        cudaStream_t stream, const RowGather* gather = nullptr);

// prepare.cu: bytes of one half (hi or lo) of a prepared weight buffer,
// 256-byte aligned; the buffer is hi | lo.
std::size_t prepared_weights_half_bytes(int experts, int hidden, int output);
cudaError_t launch_prepare_weights(const float* w, float* hi, float* lo, int experts, int hidden,
                                   int output, cudaStream_t stream);

// misc.cu
cudaError_t launch_cache_scrub(uint32_t* buffer, std::size_t elements, cudaStream_t stream);
// Bounded-wait self-test: a kernel waits on an mbarrier nothing arrives on;
// after limit_ns it sets kErrMbarTimeout and returns (*elapsed_ns, device).
cudaError_t launch_bounded_wait_selftest(unsigned long long limit_ns,
                                         unsigned long long* elapsed_ns, cudaStream_t stream);
// Adds to *mismatches (device) the number of non-NaN inputs whose integer
// TF32 rounding differs from the conversion instruction.
cudaError_t launch_tf32_round_check(const uint32_t* bits, long long n,
                                    unsigned long long* mismatches, cudaStream_t stream);

}  // namespace rrb
