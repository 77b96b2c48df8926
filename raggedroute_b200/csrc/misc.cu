// Library-wide utilities: launch accounting, device properties, the device
// error word, and the L2 cache scrub used between benchmark samples
// (src/benchmark/cache_scrub.cu:17-50 of the reference).
#include <atomic>
#include <mutex>

#include "sm100.cuh"

namespace rrb {
namespace {

std::atomic<unsigned long long> g_launches{0};

__device__ unsigned g_device_error_word = 0;

__global__ void cache_scrub_kernel(uint32_t* buffer, std::size_t elements) {
  const std::size_t stride = static_cast<std::size_t>(blockDim.x) * gridDim.x;
  for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < elements; i += stride) {
    buffer[i] = buffer[i] * 1664525u + 1013904223u + static_cast<uint32_t>(i);
  }
}

// Counts inputs whose integer TF32 rounding differs from cvt.rna.tf32.f32
// (NaN inputs are skipped: the two may pick different NaN/inf patterns).
__global__ void tf32_round_check_kernel(const uint32_t* __restrict__ bits, long long n,
                                        unsigned long long* __restrict__ mismatches) {
  unsigned long long local = 0;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float x = __uint_as_float(bits[i]);
    if (x != x) continue;
    if (__float_as_uint(sm100::tf32_rna(x)) != __float_as_uint(sm100::tf32_rna_cvt(x))) ++local;
  }
  if (local != 0) atomicAdd(mismatches, local);
}

// Failure-path self-test of the bounded waits: one CTA waits, with the
// library's mbar_wait, on an mbarrier that nothing arrives on. After
// limit_ns the wait gives up, sets kErrMbarTimeout in the device error word
// and the kernel returns normally; *elapsed_ns records how long it waited.
__global__ void bounded_wait_selftest_kernel(unsigned long long limit_ns, unsigned* err,
                                             unsigned long long* elapsed_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int failed;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    failed = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = sm100::global_timer_ns();
    volatile int* f = &failed;
    const bool ok = sm100::mbar_wait(&bar, 0, err, f, limit_ns);
    *elapsed_ns = ok ? 0ull : static_cast<unsigned long long>(sm100::global_timer_ns() - t0);
  }
}

}  // namespace

cudaError_t launch_bounded_wait_selftest(unsigned long long limit_ns,
                                         unsigned long long* elapsed_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, device_error_word(), elapsed_ns);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_tf32_round_check(const uint32_t* bits, long long n,
                                    unsigned long long* mismatches, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  tf32_round_check_kernel<<<2 * sm_count(), 256, 0, stream>>>(bits, n, mismatches);
  note_launch();
  return cudaGetLastError();
}

void note_launch(int n) { g_launches.fetch_add(static_cast<unsigned long long>(n)); }

unsigned long long launch_count() { return g_launches.load(); }

int sm_count() {
  static std::once_flag once;
  static int count = kNumSms;
  std::call_once(once, [] {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
      int v = 0;
      if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
        count = v;
    }
  });
  return count;
}

unsigned* device_error_word() {
  // One word per process; resolved lazily for the current device.
  unsigned* ptr = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_device_error_word) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return ptr;
}

cudaError_t consume_device_error(cudaStream_t stream, unsigned* out) {
  unsigned v = 0;
  cudaError_t err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess) return err;
  err = cudaMemcpyFromSymbol(&v, g_device_error_word, sizeof(v));
  if (err != cudaSuccess) return err;
  const unsigned zero = 0;
  err = cudaMemcpyToSymbol(g_device_error_word, &zero, sizeof(zero));
  if (out != nullptr) *out = v;
  return err;
}

cudaError_t launch_cache_scrub(uint32_t* buffer, std::size_t elements, cudaStream_t stream) {
  if (elements == 0) return cudaSuccess;
  const std::size_t want = (elements + 255) / 256;
  const int blocks = static_cast<int>(want < static_cast<std::size_t>(8 * sm_count())
                                          ? want
                                          : static_cast<std::size_t>(8 * sm_count()));
  cache_scrub_kernel<<<blocks, 256, 0, stream>>>(buffer, elements);
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
