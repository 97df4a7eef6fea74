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
// Wide rows take softmax_rows_cluster_kernel instead: a cluster of SMX_CL
// CTAs per row, CTA k owning the 32 chains 32k .. 32k+31. Chain t reads
// columns t, t+256, ..., so CTA k reads one 128-byte piece of every 1 KiB of
// the row (coalesced), keeps it in shared memory, and each chain stays whole
// inside one CTA, added in element order by one thread. The CTAs exchange their
// maxima through distributed shared memory, CTA 0 gathers the 256 chain sums
// and runs the reference's tree, and every CTA writes e_j / p_0 for its own
// columns: one read and one write of the batch from HBM, one expf per element.
//
// This translation unit is compiled with nvcc's default floating-point
// contraction, as the reference is, so that expf is the same function.
#include <cooperative_groups.h>
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

// Cluster of SMX_CL CTAs per row (see the header comment). pieces = ceil(cols /
// 256); e[] holds this CTA's 32 columns of every piece: e[32 i + l] is column
// 256 i + 32 k + l.
constexpr int SMX_CL = 8;
constexpr int SMX_CL_THREADS = 512;
constexpr int SMX_CL_MAX_PIECES = 1536;  // 192 KiB of shared memory: cols <= 393216
__global__ void __cluster_dims__(SMX_CL, 1, 1) __launch_bounds__(SMX_CL_THREADS)
    softmax_rows_cluster_kernel(const float* in, float* out, int cols, int pieces) {
  namespace cg = cooperative_groups;
  extern __shared__ float e[];
  __shared__ float s_red[SMX_CL_THREADS / 32];
  __shared__ float s_max[SMX_CL];
  __shared__ float s_sums[SMX_CHAINS];
  __shared__ float s_rsum;
  cg::cluster_group cl = cg::this_cluster();
  const int k = (int)cl.block_rank();
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  constexpr int NW = SMX_CL_THREADS / 32;
  const size_t row = blockIdx.x / SMX_CL;
  const float* x = in + row * (size_t)cols;
  float* y = out + row * (size_t)cols;
  const int c0 = 32 * k + lane;  // this lane's column in piece 0
  // ---- load this CTA's columns (warp w: pieces w, w + NW, ...) and its maximum,
  // SMX_CL_INFLIGHT loads per lane in flight before any is stored --------------
  constexpr int SMX_CL_INFLIGHT = 16;
  float m = -FLT_MAX;
  for (int i0 = warp; i0 < pieces; i0 += NW * SMX_CL_INFLIGHT) {
    float v[SMX_CL_INFLIGHT];
#pragma unroll
    for (int u = 0; u < SMX_CL_INFLIGHT; ++u) {
      const int i = i0 + u * NW, j = 256 * i + c0;
      v[u] = (i < pieces && j < cols) ? __ldcs(x + j) : -FLT_MAX;
    }
#pragma unroll
    for (int u = 0; u < SMX_CL_INFLIGHT; ++u) {
      const int i = i0 + u * NW;
      if (i < pieces) e[32 * i + lane] = v[u];
      m = fmaxf(m, v[u]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    float w = lane < NW ? s_red[lane] : -FLT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane < SMX_CL) *cl.map_shared_rank(&s_max[k], lane) = w;  // every CTA's slot k
  }
  cl.sync();
  float rmax = -FLT_MAX;
#pragma unroll
  for (int r = 0; r < SMX_CL; ++r) rmax = fmaxf(rmax, s_max[r]);
  // ---- e_j = expf(x_j - max), in place ---------------------------------------------
  for (int i = warp; i < pieces; i += NW) {
    const int j = 256 * i + c0;
    if (j < cols) e[32 * i + lane] = expf(e[32 * i + lane] - rmax);
  }
  __syncthreads();
  // ---- warp 0: chain 32 k + lane over its columns in order, to CTA 0 ---------------
  if (warp == 0) {
    float sum = 0.0f;
    int i = 0;
    for (; i + 8 <= pieces && 256 * (i + 7) + c0 < cols; i += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = e[32 * (i + u) + lane];
#pragma unroll
      for (int u = 0; u < 8; ++u) sum += v[u];
    }
    for (; i < pieces && 256 * i + c0 < cols; ++i) sum += e[32 * i + lane];
    *cl.map_shared_rank(&s_sums[32 * k + lane], 0) = sum;
  }
  cl.sync();
  // ---- CTA 0: the reference's tree over the 256 chain sums, total to every CTA -----
  if (k == 0) {
    for (int stride = SMX_CHAINS / 2; stride > 0; stride >>= 1) {
      if (t < stride) s_sums[t] += s_sums[t + stride];
      __syncthreads();
    }
    if (t < SMX_CL) *cl.map_shared_rank(&s_rsum, t) = s_sums[0];
  }
  cl.sync();
  const float rsum = s_rsum;
  // ---- outputs: e_j / sum for this CTA's columns ----------------------------------
  for (int i = warp; i < pieces; i += NW) {
    const int j = 256 * i + c0;
    if (j < cols) __stcs(y + j, e[32 * i + lane] / rsum);
  }
}

}  // namespace nvs

extern "C" NCB_API int ncb_softmax_rows_device(const float* d_in, float* d_out, int rows, int cols,
                                               void* stream) {
  if (rows <= 0 || cols <= 0 || !d_in || !d_out)
    return ncb_record_status(NCB_ERROR_INVALID_ARGUMENT);
  if ((reinterpret_cast<uintptr_t>(d_in) & 3u) != 0u || (reinterpret_cast<uintptr_t>(d_out) & 3u) != 0u)
    return ncb_record_status(NCB_ERROR_INVALID_ARGUMENT);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // wide rows: one cluster per row, one HBM read and one write
  const int pieces = (cols + nvs::SMX_CHAINS - 1) / nvs::SMX_CHAINS;
  if (cols >= 8192 && pieces <= nvs::SMX_CL_MAX_PIECES &&
      (long long)rows * nvs::SMX_CL <= 0x7FFFFFFFLL) {
    const size_t smem = (size_t)pieces * 32 * sizeof(float);
    static bool attr_set = false;  // the attribute is per function; setting it twice is harmless
    if (!attr_set) {
      if (cudaFuncSetAttribute(nvs::softmax_rows_cluster_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)(nvs::SMX_CL_MAX_PIECES * 32 * sizeof(float))) != cudaSuccess)
        return ncb_record_status(NCB_ERROR_LAUNCH_FAILED);
      attr_set = true;
    }
    nvs::softmax_rows_cluster_kernel<<<rows * nvs::SMX_CL, nvs::SMX_CL_THREADS, smem, st>>>(
        d_in, d_out, cols, pieces);
    return ncb_record_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
  }
  // rows go in launches whose data fits the L2 budget (passes 2 and 3 re-read it)
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
