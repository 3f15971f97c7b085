// Process-wide launch counter and the per-device error record used by bounded waits.
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace b200 {

std::atomic<long long>& launch_counter() {
  static std::atomic<long long> counter{0};
  return counter;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ZB_PDL");
    return v == nullptr || std::string(v) != "0";
  }();
  return on;
}

DeviceErrors* device_errors_ptr() {
  static std::mutex mu;
  static std::vector<DeviceErrors*> per_device;
  int dev = 0;
  B200_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if ((int)per_device.size() <= dev) per_device.resize(dev + 1, nullptr);
  if (per_device[dev] == nullptr) {
    DeviceErrors* p = nullptr;
    B200_CUDA_CHECK(cudaMalloc(&p, sizeof(DeviceErrors)));
    B200_CUDA_CHECK(cudaMemset(p, 0, sizeof(DeviceErrors)));
    per_device[dev] = p;
  }
  return per_device[dev];
}

namespace {
// Records `code` in the error record when a == b does not hold (two device scalars; one thread).
__global__ void record_if_different_kernel(const float* a, const float* b, int code, DeviceErrors* errs) {
  if (threadIdx.x == 0 && blockIdx.x == 0 && *a != *b) report_error(errs, code, 0);
}
}  // namespace

void record_if_different(const float* a, const float* b, int code, cudaStream_t s) {
  record_if_different_kernel<<<1, 32, 0, s>>>(a, b, code, device_errors_ptr());
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace b200
