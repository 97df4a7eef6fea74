// LogitsProcessor, batched over [rows, V] on sm_100a (in place).
// Reference: Neuraval/Generation/LogitsProcessor.cs:8-114.
#pragma once

#include "sampler_device.cuh"

namespace nvs {

constexpr int LP_THREADS = 512;

// ApplyRepetitionPenalty (LogitsProcessor.cs:8-36): each distinct in-range id
// of the row's history is penalised once (v>0 ? v/p : v*p). The first thread to
// set an id's bit in the shared bitmap applies it.
__global__ void __launch_bounds__(LP_THREADS) repetition_penalty_kernel(
    float* logits, int V, const int32_t* hist, const int32_t* hoff, float penalty) {
  extern __shared__ uint32_t seen[];
  const int row = blockIdx.x;
  const int words = (V + 31) >> 5;
  for (int i = threadIdx.x; i < words; i += blockDim.x) seen[i] = 0u;
  __syncthreads();
  float* lrow = logits + (size_t)row * V;
  for (int h = hoff[row] + threadIdx.x; h < hoff[row + 1]; h += blockDim.x) {
    const int id = hist[h];
    if (id < 0 || id >= V) continue;
    const uint32_t bit = 1u << (id & 31);
    if (atomicOr(&seen[id >> 5], bit) & bit) continue;
    const float v = lrow[id];
    lrow[id] = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
  }
}

// New (no reference counterpart): v - count*frequency - [count>0]*presence.
// The row's in-range history is sorted in shared memory; the first id of each
// run of equal ids applies the run length as its count.
__global__ void __launch_bounds__(LP_THREADS) frequency_presence_kernel(
    float* logits, int V, const int32_t* hist, const int32_t* hoff, float freq, float pres,
    int h_cap, uint32_t* rowflags) {
  extern __shared__ int32_t ids[];
  __shared__ int s_n;
  const int row = blockIdx.x;
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  for (int h = hoff[row] + threadIdx.x; h < hoff[row + 1]; h += blockDim.x) {
    const int id = hist[h];
    if (id < 0 || id >= V) continue;
    const int slot = atomicAdd(&s_n, 1);
    if (slot < h_cap) ids[slot] = id;
  }
  __syncthreads();
  const int n = s_n;
  if (n > h_cap) {
    if (threadIdx.x == 0 && rowflags) rowflags[row] = FLAG_BAD_HISTORY;
    return;
  }
  const int np = next_pow2(n > 0 ? n : 1);
  for (int i = n + threadIdx.x; i < np; i += blockDim.x) ids[i] = 0x7FFFFFFF;
  __syncthreads();
  cta_bitonic_sort_asc(ids, np);
  float* lrow = logits + (size_t)row * V;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (i > 0 && ids[i - 1] == ids[i]) continue;
    int e = i + 1;
    while (e < n && ids[e] == ids[i]) ++e;
    float v = lrow[ids[i]];
    v = __fsub_rn(v, __fmul_rn((float)(e - i), freq));
    v = __fsub_rn(v, pres);
    lrow[ids[i]] = v;
  }
  if (threadIdx.x == 0 && rowflags) rowflags[row] = 0u;
}

// ApplyTemperature (LogitsProcessor.cs:38-51): IEEE division by T.
__global__ void temperature_kernel(float* x, size_t n, float t) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t n4 = n / 4;
  float4* x4 = reinterpret_cast<float4*>(x);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = x4[i];
    v.x = __fdiv_rn(v.x, t);
    v.y = __fdiv_rn(v.y, t);
    v.z = __fdiv_rn(v.z, t);
    v.w = __fdiv_rn(v.w, t);
    x4[i] = v;
  }
  for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    x[i] = __fdiv_rn(x[i], t);
}
__global__ void temperature_kernel_unaligned(float* x, size_t n, float t) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    x[i] = __fdiv_rn(x[i], t);
}

// FilterTopK (LogitsProcessor.cs:53-73): threshold = the K-th largest value
// counting multiplicity (sorted[V-K] of an ascending sort); values strictly
// below it become -inf. NaNs are never counted (C#'s Array.Sort puts them
// first, below every number) and are left untouched.
__global__ void __launch_bounds__(1024) filter_top_k_kernel(float* logits, int V, int K) {
  __shared__ uint32_t hist[256];
  __shared__ int sh[2];
  float* lrow = logits + (size_t)blockIdx.x * V;
  const uint32_t key = cta_kth_largest(
      [&](int i) {
        const float v = lrow[i];
        return v != v ? 0u : fkey(canon(v));
      },
      V, K, hist, sh);
  if (key == 0u) return;
  const float thr = kval(key);
  for (int i = threadIdx.x; i < V; i += blockDim.x)
    if (lrow[i] < thr) lrow[i] = -INFINITY;
}

}  // namespace nvs
