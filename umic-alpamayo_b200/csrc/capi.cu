// Library-wide state of the C ABI: error messages, the device error word and
// per-device attribute caches.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace umic {

namespace {
thread_local char g_msg[512] = {0};

// Bits set by kernels that detect a condition they cannot report through a
// return value (device-side KV overflow, a bounded wait that ran out).
__device__ uint32_t g_device_error_word;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t* g_err_ptr[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};

std::atomic<int> g_stall_kernel{0};
std::atomic<long long> g_stall_limit{0};

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_msg[0] = 0; }

uint32_t* device_error_word() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[d]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    g_err_ptr[d] = static_cast<uint32_t*>(p);
  }
  return g_err_ptr[d];
}

int sm_count() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[d]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    g_sms[d] = n;
  }
  return g_sms[d];
}

bool take_stall(int kernel, long long* limit) {
  int expected = kernel;
  if (!g_stall_kernel.compare_exchange_strong(expected, 0)) return false;
  *limit = g_stall_limit.load();
  return true;
}

}  // namespace umic

extern "C" {

int umic_debug_stall(int kernel, int64_t wait_limit_cycles) {
  if (kernel < umic::kStallGemm || kernel > umic::kGemvGeneralMerge || wait_limit_cycles <= 0)
    return umic::fail(UMIC_ERR_INVALID_ARG, "umic_debug_stall: kernel %d, limit %lld", kernel,
                      (long long)wait_limit_cycles);
  umic::g_stall_limit.store(wait_limit_cycles);
  umic::g_stall_kernel.store(kernel);
  return UMIC_OK;
}

int umic_abi_version(void) { return 2; }

const char* umic_last_error_message(void) { return umic::g_msg; }

int umic_set_device(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess)
    return umic::fail(UMIC_ERR_DEVICE, "umic_set_device(%d): %s", device, cudaGetErrorString(e));
  return UMIC_OK;
}

int umic_device_errors(uint32_t* flags, int clear) {
  if (!flags) return umic::fail(UMIC_ERR_INVALID_ARG, "umic_device_errors: flags is NULL");
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, umic::g_device_error_word, sizeof(v));
  if (e != cudaSuccess)
    return umic::fail(UMIC_ERR_LAUNCH, "umic_device_errors: %s", cudaGetErrorString(e));
  *flags = v;
  if (clear) {
    uint32_t z = 0;
    e = cudaMemcpyToSymbol(umic::g_device_error_word, &z, sizeof(z));
    if (e != cudaSuccess)
      return umic::fail(UMIC_ERR_LAUNCH, "umic_device_errors: %s", cudaGetErrorString(e));
  }
  return UMIC_OK;
}

}  // extern "C"
