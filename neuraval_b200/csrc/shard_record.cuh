// Per-row candidate records of a vocabulary shard (sm_100a).
//
// When the vocabulary of a [rows, V] batch is split in contiguous column
// ranges over several GPUs, each GPU reduces its range of every row to one
// fixed-size record; the records of all shards are exchanged (all-gather) and
// a merge kernel finishes every row exactly as the single-GPU kernels do
// (TokenSampler.cs:54-135 for top-k rows, :38-51 for greedy rows).
//
// Top-k record: every value of the shard >= the shard's K-th largest value
// (ties included), as (value, global id). The global K-th largest value is the
// K-th largest of the union of these sets, and every global candidate is in
// the union, unless a shard had more ties at its own K-th value than the
// record holds and that value is the global K-th value: the merge flags such a
// row (token -1, NCB_FLAG_TIES_OVERFLOW).
// Greedy record: the shard's first strict maximum and whether global id 0 is
// in the shard with a NaN value.
#pragma once

#include "sampler_device.cuh"

namespace nvs {

constexpr int VS_CAP = 128;                       // candidates per record
constexpr int VS_HDR = 4;                         // header words
constexpr int VS_REC_WORDS = VS_HDR + 2 * VS_CAP; // 260 words = 1040 bytes
// record state bits (beside FLAG_NONFINITE and FLAG_BAD_HISTORY)
constexpr uint32_t VS_OVF_AT_KTH = 0x1000u;   // ties at the shard's K-th value were cut
constexpr uint32_t VS_OVF_UNKNOWN = 0x2000u;  // buffers overflowed before the exact select
constexpr uint32_t VS_NAN0 = 0x4000u;         // greedy: global id 0 is NaN

// header: [0] stored candidates n, [1] state, [2] the shard's K-th value
// (float bits), [3] candidates >= that value before any cut.
__device__ __forceinline__ float* vs_values(uint32_t* rec) {
  return reinterpret_cast<float*>(rec + VS_HDR);
}
__device__ __forceinline__ int32_t* vs_ids(uint32_t* rec) {
  return reinterpret_cast<int32_t*>(rec + VS_HDR + VS_CAP);
}

// Writes a top-k record from the m candidates (cv, cid) >= kth, all held in
// shared memory. `state` carries the kernel's row state bits. All threads of
// the CTA call; ends with __syncthreads().
__device__ void write_topk_record(uint32_t* rec, const float* cv, const int* cid, int m,
                                  uint32_t state, float kth) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t st = state & (FLAG_NONFINITE | FLAG_BAD_HISTORY);
  if (state & (RSTATE_OVERFLOW | RSTATE_TIMEOUT)) st |= VS_OVF_UNKNOWN;
  if (st != 0u) m = 0;
  float* rv = vs_values(rec);
  int32_t* ri = vs_ids(rec);
  if (m <= VS_CAP) {
    for (int i = tid; i < m; i += blockDim.x) {
      rv[i] = cv[i];
      ri[i] = cid[i];
    }
    if (tid == 0) {
      rec[0] = (uint32_t)m;
      rec[1] = st;
      rec[2] = __float_as_uint(kth);
      rec[3] = (uint32_t)m;
    }
  } else if (tid < 32) {
    // every value above kth (fewer than K <= 64 of them), then ties up to VS_CAP
    int n = 0;
    for (int pass = 0; pass < 2; ++pass) {
      for (int i0 = 0; i0 < m; i0 += 32) {
        const int i = i0 + lane;
        const bool ok = i < m && (pass == 0 ? cv[i] > kth : cv[i] == kth);
        const unsigned b = __ballot_sync(0xffffffffu, ok);
        const int pos = n + __popc(b & ((1u << lane) - 1u));
        if (ok && pos < VS_CAP) {
          rv[pos] = cv[i];
          ri[pos] = cid[i];
        }
        n += __popc(b);
      }
    }
    if (lane == 0) {
      rec[0] = (uint32_t)min(n, VS_CAP);
      rec[1] = st | (n > VS_CAP ? VS_OVF_AT_KTH : 0u);
      rec[2] = __float_as_uint(kth);
      rec[3] = (uint32_t)m;
    }
  }
  __syncthreads();
}

// Greedy record: best (value, id) of the shard, id -1 when it has none.
__device__ __forceinline__ void write_greedy_record(uint32_t* rec, float v, int id, bool bad_hist,
                                                    bool nan0) {
  rec[0] = id >= 0 ? 1u : 0u;
  rec[1] = (bad_hist ? FLAG_BAD_HISTORY : 0u) | (nan0 ? VS_NAN0 : 0u);
  rec[2] = 0u;
  rec[3] = 0u;
  vs_values(rec)[0] = v;
  vs_ids(rec)[0] = id;
}

}  // namespace nvs
