// Query rotation q_rot = R @ q for query batches (remex/core.py:615, :682,
// :759; remex/ivf.py:331): Y = X @ R^T with X (nq x d) and R (d x d), f32 in
// and out.  Products of the f32 inputs are exact in f64 and are accumulated
// in f64, so Y is the correctly rounded f32 of the exact product (the
// reference's sgemv result differs from it only by sgemv's own rounding).
//
// Work per call is nq * d^2 multiply-adds -- at most ~2.4e10 for a 10,000
// query batch at d = 1536 -- which is small next to the scans it feeds, so a
// register-tiled SIMT kernel is used rather than the tensor-core encode GEMM.
#include "common.cuh"

namespace pqb {

constexpr int kRotTile = 64;   // queries x outputs per block
constexpr int kRotK = 16;      // K slice staged in shared memory
constexpr int kRotThreads = 256;  // 16 x 16 threads, 4 x 4 outputs each

__global__ void __launch_bounds__(kRotThreads)
rotate_kernel(const float* __restrict__ X, int64_t nq, int d, const float* __restrict__ R,
              float* __restrict__ Y, const float* __restrict__ row_scale) {
  __shared__ float xs[kRotK][kRotTile + 1];
  __shared__ float rs[kRotK][kRotTile + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t q0 = (int64_t)blockIdx.y * kRotTile;
  const int o0 = blockIdx.x * kRotTile;
  double acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.0;
  for (int k0 = 0; k0 < d; k0 += kRotK) {
    for (int i = threadIdx.x; i < kRotK * kRotTile; i += kRotThreads) {
      const int row = i / kRotK, kk = i % kRotK;
      const int64_t qi = q0 + row;
      const int oi = o0 + row, k = k0 + kk;
      xs[kk][row] = (qi < nq && k < d) ? X[qi * d + k] : 0.f;
      rs[kk][row] = (oi < d && k < d) ? R[(int64_t)oi * d + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kRotK; ++kk) {
      double xv[4], rv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) xv[a] = (double)xs[kk][ty + 16 * a];
#pragma unroll
      for (int b = 0; b < 4; ++b) rv[b] = (double)rs[kk][tx + 16 * b];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fma(xv[a], rv[b], acc[a][b]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t qi = q0 + ty + 16 * a;
    if (qi >= nq) continue;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int oi = o0 + tx + 16 * b;
      if (oi < d) {
        const float y = (float)acc[a][b];
        Y[qi * d + oi] = row_scale ? y * row_scale[qi] : y;
      }
    }
  }
}

}  // namespace pqb

extern "C" int pq_rotate(const float* X, int64_t nq, int d, const float* R, float* Y,
                         void* stream) {
  using namespace pqb;
  PQ_CHECK_ARG(d > 0, "d must be positive (got %d)", d);
  PQ_CHECK_ARG(nq >= 0, "nq must be >= 0");
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(X && R && Y, "null pointer argument");
  const int64_t gy = (nq + kRotTile - 1) / kRotTile;
  PQ_CHECK_ARG(gy < 65536, "too many queries in one call (%lld)", (long long)nq);
  dim3 grid((d + kRotTile - 1) / kRotTile, (unsigned)gy);
  rotate_kernel<<<grid, kRotThreads, 0, (cudaStream_t)stream>>>(X, nq, d, R, Y, nullptr);
  PQ_LAUNCH_CHECK("rotate_kernel");
  return PQ_OK;
}

// ---------------------------------------------------------------------------
// Decode (remex/core.py:513-532): X_hat = (cent[codes >> shift] @ R) * norms.
// The dequantised rows are staged in the workspace in chunks, rotated by R
// (passed transposed, so the same kernel computes X_hat_rot @ R), rounded to
// f32 and then scaled by the norm in f32, as the reference orders it.
// ---------------------------------------------------------------------------

namespace pqb {

__global__ void dequantize_kernel(const uint8_t* __restrict__ packed, int64_t ldb, int64_t m,
                                  int d, int B, int shift, const float* __restrict__ cent,
                                  float* __restrict__ out) {
  const int64_t total = m * (int64_t)d;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / d;
    const int j = (int)(t - r * d);
    const uint8_t* row = packed + r * ldb;
    const int p = j * B;
    const uint32_t v = ((uint32_t)row[p >> 3] << 8) | (uint32_t)row[(p >> 3) + 1];
    const uint32_t c = ((v >> (16 - B - (p & 7))) & ((1u << B) - 1u)) >> shift;
    out[t] = cent[c];
  }
}

constexpr int64_t kDecodeChunk = 65536;

}  // namespace pqb

extern "C" size_t pq_decode_workspace_bytes(int64_t n, int d) {
  const int64_t ch = n < pqb::kDecodeChunk ? (n < 1 ? 1 : n) : pqb::kDecodeChunk;
  return (size_t)ch * (size_t)(d > 0 ? d : 1) * sizeof(float) + 256;
}

extern "C" int pq_decode(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                         int bits, int precision, const float* cent, const float* RT, float* out,
                         void* ws, size_t ws_bytes, void* stream) {
  using namespace pqb;
  PQ_CHECK_ARG(supported_bits(bits), "bits must be one of 1,2,3,4,8 (got %d)", bits);
  PQ_CHECK_ARG(precision >= 1 && precision <= bits, "precision must be 1-%d, got %d", bits,
               precision);
  PQ_CHECK_ARG(d > 0 && n >= 0, "bad shape");
  PQ_CHECK_ARG(ldb >= row_bytes(d, bits), "ldb too small");
  if (n == 0) return PQ_OK;
  PQ_CHECK_ARG(packed && norms && cent && RT && out && ws, "null pointer argument");
  if (ws_bytes < pq_decode_workspace_bytes(n, d))
    return fail(PQ_ERR_WORKSPACE, "pq_decode needs %zu workspace bytes",
                pq_decode_workspace_bytes(n, d));
  cudaStream_t st = (cudaStream_t)stream;
  float* xr = (float*)ws;
  for (int64_t r0 = 0; r0 < n; r0 += kDecodeChunk) {
    const int64_t m = (n - r0 < kDecodeChunk) ? n - r0 : kDecodeChunk;
    int64_t g = (m * d + 255) / 256;
    if (g > (int64_t)num_sms() * 32) g = (int64_t)num_sms() * 32;
    dequantize_kernel<<<(int)g, 256, 0, st>>>(packed + r0 * ldb, ldb, m, d, bits, bits - precision,
                                              cent, xr);
    PQ_LAUNCH_CHECK("dequantize_kernel");
    dim3 grid((d + kRotTile - 1) / kRotTile, (unsigned)((m + kRotTile - 1) / kRotTile));
    rotate_kernel<<<grid, kRotThreads, 0, st>>>(xr, m, d, RT, out + r0 * d, norms + r0);
    PQ_LAUNCH_CHECK("rotate_kernel");
  }
  return PQ_OK;
}
