// Library-wide plumbing of the rf_moe C ABI: per-thread error message,
// version, device error words, sizing helpers.
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace rf {

static thread_local std::string t_last_error;

void set_error(const std::string &msg) { t_last_error = msg; }

int fail(int status, const std::string &msg) {
  set_error(msg);
  return status;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(RF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return RF_OK;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

size_t dtype_size(int dtype) { return dtype == RF_F32 ? 4 : 2; }
bool valid_dtype(int dtype) { return dtype == RF_F32 || dtype == RF_F16 || dtype == RF_BF16; }

static std::vector<ErrorWordReader> &readers() {
  static std::vector<ErrorWordReader> r;
  return r;
}

ErrorWordRegistrar::ErrorWordRegistrar(ErrorWordReader fn) { readers().push_back(fn); }

int read_clear_all_error_words(int *code) {
  int first = RF_DEV_OK;
  for (ErrorWordReader fn : readers()) {
    int v = fn();
    if (v < 0) return fail(RF_ERR_CUDA, "reading the device error word failed");
    if (v != RF_DEV_OK && first == RF_DEV_OK) first = v;
  }
  *code = first;
  return RF_OK;
}

}  // namespace rf

extern "C" {

const char *rf_moe_last_error(void) { return rf::t_last_error.c_str(); }

int rf_moe_version(void) { return 100; }

int rf_moe_device_status(int *code) {
  if (!code) return rf::fail(RF_ERR_ARG, "rf_moe_device_status: code is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess)
    return rf::fail(RF_ERR_CUDA, std::string("rf_moe_device_status: ") + cudaGetErrorString(e));
  return rf::read_clear_all_error_words(code);
}

int64_t rf_moe_rows_capacity(int64_t n_pairs, int64_t num_experts, int64_t align) {
  if (n_pairs < 0 || num_experts <= 0 || align <= 0) return -1;
  return n_pairs + num_experts * (align - 1);
}

}  // extern "C"
