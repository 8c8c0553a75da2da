// Status strings, the thread-local error message and the device-side error word.
#include <mutex>
#include <string>

#include "common.cuh"

namespace dsm {

__device__ int g_device_error = 0;

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int status, const std::string& msg) {
  set_error(msg);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DSM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return DSM_OK;
}

thread_local int t_grid_ctas = 0;

int persistent_ctas() { return t_grid_ctas > 0 ? t_grid_ctas : num_sms(); }

GridLimit::GridLimit(int ctas) : prev_(t_grid_ctas) { t_grid_ctas = ctas; }
GridLimit::~GridLimit() { t_grid_ctas = prev_; }

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

}  // namespace dsm

extern "C" {

int dsm_abi_version(void) { return DSM_ABI_VERSION; }

const char* dsm_status_string(int status) {
  switch (status) {
    case DSM_OK: return "ok";
    case DSM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DSM_ERR_UNSUPPORTED: return "unsupported configuration";
    case DSM_ERR_WORKSPACE: return "workspace too small";
    case DSM_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* dsm_last_error_message(void) { return dsm::t_last_error.c_str(); }

int dsm_device_error(int* code, int clear, void* stream) {
  if (!code) return dsm::fail(DSM_ERR_INVALID_ARGUMENT, "dsm_device_error: code is NULL");
  cudaStream_t s = dsm::as_stream(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, dsm::g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(dsm::g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  if (e != cudaSuccess) return dsm::fail(DSM_ERR_CUDA, std::string("dsm_device_error: ") + cudaGetErrorString(e));
  *code = v;
  return DSM_OK;
}

}  // extern "C"
