// Library-level entry points: version, error reporting, device queries,
// launch mode.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "common.cuh"
#include "../../include/kavor_b200.h"

namespace kvb {

static thread_local char t_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return status;
}

static std::atomic<int> g_pdl{0};

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return kOk;
  set_error((int)e, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
  return (int)e;
}

// Error-word readers defined by each kernel translation unit.
int read_device_error_elementwise(unsigned*, int);
int read_device_error_decode(unsigned*, int);
int read_device_error_prefill(unsigned*, int);
int read_device_error_sampler(unsigned*, int);
int read_device_error_gemm(unsigned*, int);
int read_device_error_allreduce(unsigned*, int);
int read_device_error_gemm_pair(unsigned*, int);
int read_device_error_gemm_sk(unsigned*, int);
int set_pdl_trigger_elementwise(int);
int set_pdl_trigger_decode(int);
int set_pdl_trigger_prefill(int);
int set_pdl_trigger_sampler(int);
int set_pdl_trigger_gemm(int);
int set_pdl_trigger_allreduce(int);
int set_pdl_trigger_gemm_pair(int);
int set_pdl_trigger_gemm_sk(int);

}  // namespace kvb

extern "C" int kvb_version(void) { return 100; }

extern "C" const char* kvb_last_error(void) { return kvb::t_last_error; }

extern "C" int kvb_device_error(unsigned* bits, int clear) {
  if (!bits) return kvb::set_error(kvb::kInvalid, "kvb_device_error: bits is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return kvb::cuda_status(e, "kvb_device_error: synchronize");
  unsigned acc = 0, w = 0;
  int (*readers[])(unsigned*, int) = {kvb::read_device_error_elementwise, kvb::read_device_error_decode,
                                      kvb::read_device_error_prefill, kvb::read_device_error_sampler,
                                      kvb::read_device_error_gemm, kvb::read_device_error_allreduce,
                                      kvb::read_device_error_gemm_pair, kvb::read_device_error_gemm_sk};
  for (auto fn : readers) {
    int rc = fn(&w, clear);
    if (rc) return rc;
    acc |= w;
  }
  *bits = acc;
  return kvb::kOk;
}

extern "C" int kvb_set_pdl(int enable) {
  if (enable != 0 && enable != 1) return kvb::set_error(kvb::kInvalid, "kvb_set_pdl: enable must be 0 or 1");
  int (*setters[])(int) = {kvb::set_pdl_trigger_elementwise, kvb::set_pdl_trigger_decode,
                           kvb::set_pdl_trigger_prefill, kvb::set_pdl_trigger_sampler, kvb::set_pdl_trigger_gemm,
                           kvb::set_pdl_trigger_allreduce, kvb::set_pdl_trigger_gemm_pair,
                           kvb::set_pdl_trigger_gemm_sk};
  for (auto fn : setters) {
    int rc = fn(enable);
    if (rc) return rc;
  }
  kvb::g_pdl.store(enable, std::memory_order_relaxed);
  return kvb::kOk;
}

extern "C" int kvb_sm_count(int* out) {
  if (!out) return kvb::set_error(kvb::kInvalid, "kvb_sm_count: out is NULL");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return kvb::cuda_status(e, "kvb_sm_count: cudaGetDevice");
  e = cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev);
  return kvb::cuda_status(e, "kvb_sm_count: attribute");
}
