// Row softmax over a [rows, cols] fp32 batch (sm_100a), with the arithmetic of
// the reference's ncb_softmax_rows_kernel (Neuraval.Cuda.Native/src/navcuda.cu:
// 616-671) so that every output bit is the same:
//   max  = the row maximum (fmaxf from -FLT_MAX; NaN never wins);
//   e_j  = expf(x_j - max);
//   p_t  = sequential fp32 sum of e_j over j = t, t+256, t+512, ... (t < 256),
//          then the tree s[t] += s[t + stride] for stride = 128, 64, ..., 1;
//   y_j  = e_j / p_0 (IEEE division).
// The maximum is exact whatever the order (and the sign of a zero maximum
// never changes x - max), so it is reduced with 128-bit loads in any order.
// The 256 partial sums keep their element order and their tree; the sums pass
// keeps 16 loads per thread in flight instead of storing e_j, and the output
// pass recomputes e_j (the same bits) and writes e_j / p_0 once. Rows are
// launched in groups whose data fits half of L2, so of the three reads of a
// row only the first comes from HBM: one read and one write of the batch.
//
// This translation unit is compiled with nvcc's default floating-point
// contraction, as the reference is, so that expf is the same function.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "navsampler.h"

int ncb_record_status(int st);

namespace nvs {

constexpr int SMX_CHAINS = 256;   // the reference's NCB_REDUCE_THREADS
constexpr int SMX_PREFETCH = 16;  // loads in flight per chain in the sums pass
// Rows of one launch: their data (read three times) stays within this part of
// the 126 MB L2, so the second and third passes are L2 hits.
constexpr size_t SMX_L2_BYTES = 72ull << 20;
constexpr int SMX_TILE = 8192;    // columns per shared-memory tile of the sums pass

// One CTA per row. NT threads read in the order-free passes (maximum, outputs);
// the first SMX_CHAINS of them run the partial sums.
template <int NT>
__global__ void __launch_bounds__(NT) softmax_rows_kernel(const float* in, float* out, int cols) {
  static_assert(NT >= SMX_CHAINS && NT % SMX_CHAINS == 0, "the partial sums need 256 threads");
  __shared__ float sh[NT];
  const int t = threadIdx.x;
  const float* x = in + (size_t)blockIdx.x * cols;
  float* y = out + (size_t)blockIdx.x * cols;
  // 16-byte aligned body [a0, a0 + 4 n4) as float4, scalar head and tail
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)x & 15u)) & 15u) >> 2);
  const int a0 = head < cols ? head : cols;
  const int n4 = (cols - a0) >> 2;
  const int a1 = a0 + 4 * n4;
  const bool aligned_out = ((uintptr_t)y & 15u) == ((uintptr_t)x & 15u);

  // ---- maximum (any order) ----------------------------------------------------
  float m = -FLT_MAX;
  {
    const float4* body = reinterpret_cast<const float4*>(x + a0);
    for (int j = t; j < a0; j += NT) m = fmaxf(m, x[j]);
    for (int j = a1 + t; j < cols; j += NT) m = fmaxf(m, x[j]);
#pragma unroll 4
    for (int q = t; q < n4; q += NT) {
      const float4 v = __ldcg(body + q);
      m = fmaxf(fmaxf(m, v.x), fmaxf(fmaxf(v.y, v.z), v.w));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((t & 31) == 0) sh[t >> 5] = m;
  __syncthreads();
  if (t < 32) {
    float w = t < NT / 32 ? sh[t] : -FLT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (t == 0) sh[NT - 1] = w;
  }
  __syncthreads();
  const float rmax = sh[NT - 1];
  __syncthreads();

  // ---- the 256 partial sums, each in element order, and their tree -------------
  if constexpr (NT == SMX_CHAINS) {
    float s = 0.0f;
    int j = t;
    for (; j + (SMX_PREFETCH - 1) * SMX_CHAINS < cols; j += SMX_PREFETCH * SMX_CHAINS) {
      float v[SMX_PREFETCH];
#pragma unroll
      for (int u = 0; u < SMX_PREFETCH; ++u) v[u] = __ldcg(x + j + u * SMX_CHAINS);
#pragma unroll
      for (int u = 0; u < SMX_PREFETCH; ++u) s += expf(v[u] - rmax);
    }
    for (; j < cols; j += SMX_CHAINS) s += expf(__ldcg(x + j) - rmax);
    sh[t] = s;
  } else {
    // Tiles of SMX_TILE columns: every thread exponentiates NT-strided columns
    // of the tile into shared memory (the next tile's loads already in flight),
    // then chain t adds columns t, t+256, ... of the tile in order. Columns past
    // the row add +0, which leaves a sum unchanged.
    constexpr int PER = SMX_TILE / NT;
    __shared__ float tile[SMX_TILE];
    float s = 0.0f;
    float v[PER], w[PER];  // this tile's and the next tile's columns, loads in flight
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int j = t + u * NT;
      v[u] = j < cols ? __ldcg(x + j) : 0.0f;
      w[u] = j + SMX_TILE < cols ? __ldcg(x + j + SMX_TILE) : 0.0f;
    }
    for (int base = 0; base < cols; base += SMX_TILE) {
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int j = base + t + u * NT;
        tile[t + u * NT] = j < cols ? expf(v[u] - rmax) : 0.0f;
        v[u] = w[u];
      }
      __syncthreads();
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int j = base + 2 * SMX_TILE + t + u * NT;
        w[u] = j < cols ? __ldcg(x + j) : 0.0f;
      }
      if (t < SMX_CHAINS) {
#pragma unroll 8
        for (int k = 0; k < SMX_TILE / SMX_CHAINS; ++k) s += tile[k * SMX_CHAINS + t];
      }
      __syncthreads();
    }
    if (t < SMX_CHAINS) sh[t] = s;
  }
  __syncthreads();
  for (int stride = SMX_CHAINS / 2; stride > 0; stride >>= 1) {
    if (t < stride) sh[t] += sh[t + stride];
    __syncthreads();
  }
  const float rsum = sh[0];

  // ---- outputs (any order): e_j / sum ---------------------------------------------
  if (aligned_out) {
    const float4* body = reinterpret_cast<const float4*>(x + a0);
    float4* ob = reinterpret_cast<float4*>(y + a0);
    for (int j = t; j < a0; j += NT) y[j] = expf(x[j] - rmax) / rsum;
    for (int j = a1 + t; j < cols; j += NT) y[j] = expf(x[j] - rmax) / rsum;
#pragma unroll 4
    for (int q = t; q < n4; q += NT) {
      const float4 v = __ldcg(body + q);
      ob[q] = make_float4(expf(v.x - rmax) / rsum, expf(v.y - rmax) / rsum,
                          expf(v.z - rmax) / rsum, expf(v.w - rmax) / rsum);
    }
  } else {
#pragma unroll 4
    for (int j = t; j < cols; j += NT) y[j] = expf(__ldcg(x + j) - rmax) / rsum;
  }
}

}  // namespace nvs

extern "C" NCB_API int ncb_softmax_rows_device(const float* d_in, float* d_out, int rows, int cols,
                                               void* stream) {
  if (rows <= 0 || cols <= 0 || !d_in || !d_out)
    return ncb_record_status(NCB_ERROR_INVALID_ARGUMENT);
  if ((reinterpret_cast<uintptr_t>(d_in) & 3u) != 0u || (reinterpret_cast<uintptr_t>(d_out) & 3u) != 0u)
    return ncb_record_status(NCB_ERROR_INVALID_ARGUMENT);
  // rows go in launches whose data fits the L2 budget (passes 2 and 3 re-read it)
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t row_bytes = (size_t)cols * 4;
  int fit = (int)(nvs::SMX_L2_BYTES / row_bytes);
  if (fit < 1) fit = 1;
  const int groups = (rows + fit - 1) / fit;
  const int chunk = (rows + groups - 1) / groups;  // equal groups keep every launch full
  for (int r0 = 0; r0 < rows; r0 += chunk) {
    const int n = rows - r0 < chunk ? rows - r0 : chunk;
    const float* i0 = d_in + (size_t)r0 * cols;
    float* o0 = d_out + (size_t)r0 * cols;
    if (cols >= 4096)
      nvs::softmax_rows_kernel<1024><<<n, 1024, 0, st>>>(i0, o0, cols);
    else
      nvs::softmax_rows_kernel<nvs::SMX_CHAINS><<<n, nvs::SMX_CHAINS, 0, st>>>(i0, o0, cols);
  }
  return ncb_record_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}
