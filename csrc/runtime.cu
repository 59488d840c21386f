// Device-side error word written by bounded waits (mbarrier / peer flags) that time
// out. Kernels never trap: they record the failure here and exit; the host reads it.
#include "common.h"

namespace ns {

static int* g_err[64] = {nullptr};
static std::mutex g_err_mu;

int* device_error_flag() {
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  NS_CHECK(dev >= 0 && dev < 64, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_err_mu);
  if (!g_err[dev]) {
    NS_CUDA(cudaMalloc(&g_err[dev], sizeof(int)));
    NS_CUDA(cudaMemset(g_err[dev], 0, sizeof(int)));
  }
  return g_err[dev];
}

// The error word as a one-element int32 CUDA tensor (a view, not a copy), so the
// host can snapshot it with an asynchronous copy on any stream without waiting.
at::Tensor device_error_tensor() {
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  return at::from_blob(device_error_flag(), {1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
}

void gemm_reset_counters();

// After a bounded wait timed out: wait for the device, clear the split-K arrival
// counters that an abandoned CTA may have left non-zero, and clear the error word.
void reset_device_error_state() {
  gemm_reset_counters();
  NS_CUDA(cudaMemset(device_error_flag(), 0, sizeof(int)));
  NS_CUDA(cudaDeviceSynchronize());
}

int64_t device_error() {
  int h = 0;
  NS_CUDA(cudaMemcpy(&h, device_error_flag(), sizeof(int), cudaMemcpyDeviceToHost));
  return h;
}

void clear_device_error() { NS_CUDA(cudaMemset(device_error_flag(), 0, sizeof(int))); }

void check_device_error() {
  NS_CHECK(device_error() == 0, "a kernel's bounded wait timed out (device error flag set)");
}

}  // namespace ns
