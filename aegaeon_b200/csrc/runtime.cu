// Library-wide host utilities: thread-local error text, version, SM count cache and the
// sticky device error word reader.
#include "aeg_common.cuh"

#include <mutex>
#include <vector>

namespace aeg {

namespace {
thread_local std::string t_last_error;
}

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error.assign(buf);
  return code;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace aeg

extern "C" {

int aeg_version(void) { return 100; }

const char* aeg_last_error(void) { return aeg::t_last_error.c_str(); }

int aeg_read_device_errors(void* stream, uint32_t* flags) {
  AEG_CHECK_ARG(flags != nullptr, "aeg_read_device_errors: flags is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e[5] = {cudaSuccess, cudaSuccess, cudaSuccess, cudaSuccess, cudaSuccess};
  uint32_t f = aeg::deverr_read_and_clear_copy(s, &e[0]);
  f |= aeg::deverr_read_and_clear_cache(s, &e[1]);
  f |= aeg::deverr_read_and_clear_attn(s, &e[2]);
  f |= aeg::deverr_read_and_clear_step(s, &e[3]);
  f |= aeg::deverr_read_and_clear_prefill(s, &e[4]);
  for (cudaError_t x : e)
    if (x != cudaSuccess)
      return aeg::set_error(AEG_ERR_CUDA, "aeg_read_device_errors: %s", cudaGetErrorString(x));
  *flags = f;
  return AEG_OK;
}

}  // extern "C"
