// Exact K-th value of a small candidate union by direct ranks (sm_100a).
//
// Used where a few hundred candidates from several lists meet: the last CTA
// of a row split over CTAs, and the merge of vocabulary-shard records. Every
// value's rank is the number of larger keys (value desc, id asc; ids are
// unique) in the union, counted against all of it; the key of rank K-1 is
// the K-th value (TokenSampler.cs:73-84 counts with multiplicity, and so do
// ranks over value-then-id keys). Every value >= it is a candidate
// (:88-93), and its rank is its place in the descending sort (:95), so the
// candidates land sorted with their weights exp(v - max) (:96-103) computed
// in parallel.
#pragma once

#include "sampler_device.cuh"

namespace nvs {

constexpr int RS_MAX = 1024;  // union size served (two keys per thread at 512 threads)

struct RankSel {
  bool ok;        // false: more than 64 candidates, or no finite maximum
  int c;          // candidates, sorted in sk[0..c), weights in sw[0..c)
  uint64_t x;     // key of the K-th value (the smallest key when fewer than K)
  bool slow;      // a weight needed the double-double exp
};

// uv/uid[0..U) in shared memory (U <= RS_MAX, U <= 2 * blockDim.x); keys: U
// keys of shared scratch; sk/sw: 64 each. All threads call; every thread gets
// the same result; ends with __syncthreads().
__device__ RankSel cta_rank_select(const float* uv, const int* uid, int U, int K, uint64_t* keys,
                                   uint64_t* sk, float* sw) {
  __shared__ uint64_t s_x, s_mx;
  __shared__ int s_c, s_f;
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int i = tid; i < U; i += nt) keys[i] = cand_key(uv[i], uid[i]);
  if (tid == 0) {
    s_x = 0ull;
    s_mx = 0ull;
    s_c = 0;
    s_f = 0;
  }
  __syncthreads();
  uint64_t k[2];
  int r[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int i = tid + t * nt;
    k[t] = i < U ? keys[i] : 0ull;
    r[t] = 0;
  }
#pragma unroll 4
  for (int j = 0; j < U; ++j) {
    const uint64_t y = keys[j];
    r[0] += y > k[0];
    r[1] += y > k[1];
  }
  const int kk = min(K, U);  // fewer than K values: every one is a candidate
#pragma unroll
  for (int t = 0; t < 2; ++t)
    if (k[t] != 0ull) {
      if (r[t] == kk - 1) s_x = k[t];
      if (r[t] == 0) s_mx = k[t];
    }
  __syncthreads();
  const uint32_t xv = (uint32_t)(s_x >> 32);
  const float vmax = cand_val(s_mx);
  const bool finite = s_x != 0ull && vmax > -INFINITY;
  if (finite) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
      if (k[t] != 0ull && (uint32_t)(k[t] >> 32) >= xv) {
        if (r[t] < 64) {
          bool slow = false;
          sk[r[t]] = k[t];
          sw[r[t]] = exp_cr(__fsub_rn(cand_val(k[t]), vmax), slow);
          if (slow) atomicOr(&s_f, 2);
        } else {
          atomicOr(&s_f, 1);
        }
        atomicAdd(&s_c, 1);
      }
  }
  __syncthreads();
  RankSel rs;
  rs.ok = finite && (s_f & 1) == 0;
  rs.c = s_c;
  rs.x = s_x;
  rs.slow = (s_f & 2) != 0;
  return rs;
}

}  // namespace nvs
