// Library-wide utilities: launch accounting, device properties, the device
// error word, and the L2 cache scrub used between benchmark samples
// (src/benchmark/cache_scrub.cu:17-50 of the reference).
#include <atomic>
#include <mutex>

#include "common.cuh"

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

}  // namespace

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
