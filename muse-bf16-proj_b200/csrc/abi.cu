// Library-level entry points: version, device check, the device status word (one per translation unit) and the
// limit of the kernels' bounded waits.
#include <atomic>

#include "common.cuh"

namespace mbp {
namespace {
std::atomic<unsigned long long> g_wait_ns{kDefaultWaitLimitNs};
}
uint64_t wait_limit_ns() { return g_wait_ns.load(std::memory_order_relaxed); }
}  // namespace mbp

int mbp_status_pack(int* v, int clear);
int mbp_status_gemv(int* v, int clear);
int mbp_status_gemm(int* v, int clear);
int mbp_status_tp(int* v, int clear);

extern "C" {

int mbp_version(void) { return 1; }

int mbp_device_check(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    cudaGetLastError();
    return MBP_ERR_DEVICE;
  }
  return prop.major == 10 && prop.minor == 0 ? MBP_OK : MBP_ERR_DEVICE;
}

unsigned long long mbp_set_wait_limit(unsigned long long ns) {
  return mbp::g_wait_ns.exchange(ns ? ns : mbp::kDefaultWaitLimitNs);
}

int mbp_status(int* status, int clear) {
  if (!status) return MBP_ERR_ARG;
  *status = 0;
  int rc = mbp_status_pack(status, clear);
  if (rc == MBP_OK) rc = mbp_status_gemv(status, clear);
  if (rc == MBP_OK) rc = mbp_status_gemm(status, clear);
  if (rc == MBP_OK) rc = mbp_status_tp(status, clear);
  return rc;
}

}  // extern "C"
