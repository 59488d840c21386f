// Device-side error word written by bounded waits (mbarrier / peer flags) that time
// out. Kernels never trap: they record the failure here and exit; the host reads it.
#include "common.h"

namespace ns {

static int* g_err[16] = {nullptr};

int* device_error_flag() {
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  if (!g_err[dev]) {
    NS_CUDA(cudaMalloc(&g_err[dev], sizeof(int)));
    NS_CUDA(cudaMemset(g_err[dev], 0, sizeof(int)));
  }
  return g_err[dev];
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
