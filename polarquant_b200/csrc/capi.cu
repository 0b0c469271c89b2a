// Error reporting and small C-ABI helpers.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace pqb {


static thread_local char t_err[512] = "";
long long g_launches = 0;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace pqb

extern "C" {

int pq_version(void) { return 1 * 10000 + 0 * 100 + 0; }

const char* pq_last_error(void) { return pqb::t_err; }

int pq_device_status(int* code) {
  if (!code) return pqb::fail(PQ_ERR_INVALID, "null code pointer");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess)
    return pqb::fail(PQ_ERR_CUDA, "cudaDeviceSynchronize failed: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, pqb::g_device_error, sizeof(int));
  if (e != cudaSuccess)
    return pqb::fail(PQ_ERR_CUDA, "reading the device error word failed: %s",
                     cudaGetErrorString(e));
  *code = v;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(pqb::g_device_error, &zero, sizeof(int));
  }
  return PQ_OK;
}

int64_t pq_launch_count(void) { return __atomic_load_n(&pqb::g_launches, __ATOMIC_RELAXED); }

int64_t pq_row_bytes(int d, int bits) {
  if (d < 0 || !pqb::supported_bits(bits)) return -1;
  return pqb::row_bytes(d, bits);
}

}  // extern "C"
