// ADC scan + top-k with no allocation at all, for callers that cannot
// allocate device memory: hosts that hand the whole GPU memory to their own
// pool up front (serving engines that reserve HBM for their caches and forbid
// other allocations), and callers on latency-critical paths that cannot pay
// for cudaMalloc/cudaFree, which may synchronise the device.  Such callers
// provide only the corpus, the queries and the output buffers.
//
// The scan's scratch (the per-block candidate lists, and the byte-table
// scan's tables and partial sums when they also fit) lives in a file-scope
// __device__ array of kNoAllocScratchBytes.  Every GPU that loads this
// library holds that array until the process exits.  All calls on a device
// share it and it keeps the last call's contents; nothing in it needs to start
// at zero, because every slot a call reads was written earlier by that same
// call.  Calls whose work overlaps on the GPU (different streams, or host
// threads racing) therefore race on the array and must be serialised by the
// caller.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace pqb {

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;  // 16 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// In host code `g_noalloc_scratch` names a host-side shadow, not device memory;
// the device address is looked up (cudaGetSymbolAddress) with the device
// current, once per device and context: the cached address is dropped when
// the device's current context is no longer the one it was taken in (after a
// cudaDeviceReset the primary context is re-created and the array may live at
// another address).  The context id comes from the driver (cuCtxGetCurrent,
// cuCtxGetId), reached through cudaGetDriverEntryPoint.
static void* g_noalloc_addr[256];
static unsigned long long g_noalloc_ctx[256];
static std::mutex g_noalloc_mu;

typedef CUresult (*PfnCtxGetCurrent)(CUcontext*);
typedef CUresult (*PfnCtxGetId)(CUcontext, unsigned long long*);

// Id of the calling thread's current context, 0 when there is none (or the
// driver cannot say).
static unsigned long long current_ctx_id() {
  static PfnCtxGetCurrent get_current = nullptr;
  static PfnCtxGetId get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PfnCtxGetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PfnCtxGetId>(p);
    looked_up = true;
  }
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

static int noalloc_scratch(void** out) {
  int dev = 0;
  PQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) return fail(PQ_ERR_CUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  const unsigned long long ctx = current_ctx_id();
  if (!g_noalloc_addr[dev] || ctx == 0 || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(PQ_ERR_CUDA, "cudaGetSymbolAddress of the scan scratch failed: %s",
                  cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = current_ctx_id();  // the lookup above made the context current
  }
  *out = g_noalloc_addr[dev];
  return PQ_OK;
}

}  // namespace pqb

extern "C" size_t pq_adc_scan_noalloc_scratch_bytes(void) { return pqb::kNoAllocScratchBytes; }

extern "C" int pq_adc_scan_noalloc(const uint8_t* packed, int64_t ldb, const float* norms,
                                   int64_t n, int d, int bits, int precision, const float* qrot,
                                   int nq, const float* cent, int k, int64_t row_offset,
                                   float* out_scores, int64_t* out_ids, void* stream) {
  using namespace pqb;
  PQ_CHECK_ARG(k >= 1 && k <= PQ_TOPK_MAX,
               "k must be in [1, %d] for the allocation-free scan (got %d)", PQ_TOPK_MAX, k);
  if (nq > 0 && n > 0) {
    // pq_adc_scan takes any workspace that holds its candidate lists and runs
    // the byte-table scan only when the rest also holds that scan's tables
    // and partial sums (else a scan that needs nothing more), so the lists
    // alone bound a call.
    const size_t need = scan_ws_base(n, nq, k);
    if (need > kNoAllocScratchBytes)
      return fail(PQ_ERR_WORKSPACE,
                  "this scan needs %zu bytes of scratch but the allocation-free entry point has "
                  "%zu; pass fewer queries or a smaller k per call",
                  need, kNoAllocScratchBytes);
  }
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return pq_adc_scan(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, k, row_offset,
                     out_scores, out_ids, scratch, kNoAllocScratchBytes, stream);
}
