// Shared helpers for the polarquant_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/polarquant_b200.h"

namespace pqb {

// ---------------------------------------------------------------------------
// Host-side error state (thread-local message, returned by pq_last_error()).
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

#define PQ_CHECK_ARG(cond, ...)                                   \
  do {                                                            \
    if (!(cond)) return ::pqb::fail(PQ_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define PQ_CUDA_TRY(expr)                                                        \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess)                                                       \
      return ::pqb::fail(PQ_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

// Every kernel launch of the library is followed by PQ_LAUNCH_CHECK, which
// also counts it (pq_launch_count()).
extern long long g_launches;

#define PQ_LAUNCH_CHECK(what)                                                       \
  do {                                                                              \
    __atomic_fetch_add(&::pqb::g_launches, 1, __ATOMIC_RELAXED);                    \
    cudaError_t _e = cudaGetLastError();                                            \
    if (_e != cudaSuccess)                                                          \
      return ::pqb::fail(PQ_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(_e)); \
  } while (0)

// Device-side error word: kernels that wait on a barrier with an iteration
// limit record the first failure here instead of hanging or trapping.
__device__ int g_device_error = 0;  // the library is built as one translation unit

__device__ __forceinline__ void device_fail(int code) { atomicCAS(&g_device_error, 0, code); }

inline bool supported_bits(int b) { return b == 1 || b == 2 || b == 3 || b == 4 || b == 8; }

// Bytes of one packed row of d codes at b bits (remex/packing.py:130-150 with n=1).
inline int64_t row_bytes(int64_t d, int bits) {
  switch (bits) {
    case 8: return d;
    case 4: return (d + 1) / 2;
    case 2: return (d + 3) / 4;
    case 1: return (d + 7) / 8;
    case 3: return ((d + 7) / 8) * 3;
  }
  return -1;
}

inline int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Workspace carving: consecutive 256-byte aligned slices of one buffer.
struct Carve {
  char* base;
  size_t cap, off;
  Carve(void* b, size_t c) : base((char*)b), cap(c), off(0) {}
  template <class T>
  T* take(size_t count) {
    off = align_up(off, 256);
    T* p = (T*)(base + off);
    off += count * sizeof(T);
    return p;
  }
  bool ok() const { return off <= cap; }
};

// Total order used by every top-k in the library: higher score first, and
// among equal scores the lower row id first.  Deterministic and independent
// of launch shape.
__device__ __forceinline__ bool better(float sa, long long ia, float sb, long long ib) {
  return sa > sb || (sa == sb && (unsigned long long)ia < (unsigned long long)ib);
}

}  // namespace pqb
