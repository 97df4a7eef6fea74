// Warp-level candidate buffers and the one-warp finishing stage shared by
// the streaming top-k kernels (sm_100a).
//
// A warp keeps the values >= its threshold in a private shared-memory buffer
// (appends by ballot + popc, no atomics). A full buffer is sorted in registers
// (bitonic network on 64-bit value/id keys) and cut to its top K plus every
// value equal to the K-th, which raises the warp's threshold; that cut is a
// lower bound of the segment's K-th largest value, so no candidate of the
// final threshold is ever dropped. Ties that fill the buffer mark the row for
// the full-vocabulary fix-up kernel.
#pragma once

#include "sampler_device.cuh"
#include "topk_kernels.cuh"

namespace nvs {

constexpr int TW_WCAP = 128;   // candidate entries per warp buffer

// Warp bitonic sort, descending, of 128 keys held 4 per lane at index r*32+lane.
__device__ __forceinline__ void warp_sort128_desc(uint64_t (&k)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 128; size <<= 1) {
#pragma unroll
    for (int j = size >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = r * 32 + lane;
        const bool down = (i & size) == 0;  // this block sorts descending
        if (j >= 32) {
          const int rr = r ^ (j >> 5);
          if (rr > r) {
            const uint64_t x = k[r], y = k[rr];
            const bool sw = down ? (x < y) : (x > y);
            if (sw) { k[r] = y; k[rr] = x; }
          }
        } else {
          const uint64_t o = __shfl_xor_sync(0xffffffffu, k[r], j);
          const bool lower = (lane & j) == 0;
          // lower index keeps the larger key in a descending block
          const uint64_t mx = k[r] > o ? k[r] : o, mn = k[r] > o ? o : k[r];
          k[r] = (lower == down) ? mx : mn;
        }
      }
    }
  }
}

// Sorts the warp's buffer, keeps the top K values plus every value equal to the
// K-th (a sorted prefix), and returns the new count; theta_w becomes the K-th
// value. When the kept prefix would leave no room for another ballot of 32,
// *tie_overflow is set.
__device__ __noinline__ int warp_compact(float* wv, int* wi, int count, int K, float& theta_w,
                                         bool& tie_overflow) {
  const int lane = threadIdx.x & 31;
  // entries were appended by other lanes: make their shared-memory writes
  // visible (ballot/shuffle synchronise execution, not memory)
  __syncwarp();
  uint64_t k[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = r * 32 + lane;
    k[r] = i < count ? cand_key(wv[i], wi[i]) : 0ull;
  }
  warp_sort128_desc(k);
  // key of the K-th entry (index K-1 = r*32+lane)
  const int rK = (K - 1) >> 5, lK = (K - 1) & 31;
  uint64_t kk = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r)
    if (r == rK) kk = __shfl_sync(0xffffffffu, k[r], lK);
  const uint32_t tkey = (uint32_t)(kk >> 32);
  int keep = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = r * 32 + lane;
    const bool kp = i < count && (uint32_t)(k[r] >> 32) >= tkey;
    keep += __popc(__ballot_sync(0xffffffffu, kp));
  }
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = r * 32 + lane;
    if (i < keep) {
      wv[i] = cand_val(k[r]);
      wi[i] = cand_id(k[r]);
    }
  }
  __syncwarp();
  theta_w = kval(tkey);
  if (keep > TW_WCAP - 32) tie_overflow = true;
  return keep;
}

struct Compacted {
  int count;    // entries kept (the top K plus ties, a sorted prefix)
  float theta;  // the warp's new threshold: the K-th value
  int overflow; // ties leave no room for another ballot of 32
};

// Out of line: the compaction runs a few times per warp and row, and keeping
// its sorting network out of the stream loop keeps that loop small.
__device__ __noinline__ Compacted warp_compact_nl(float* wv, int* wi, int count, int K) {
  float th = 0.0f;
  bool ovf = false;
  const int n = warp_compact(wv, wi, count, K, th, ovf);
  return {n, th, ovf ? 1 : 0};
}

// Appends the lanes' candidate (value c_v at column c_id when `c`) to the warp
// buffer; count/theta/overflow are warp-uniform registers of the caller.
__device__ __forceinline__ void warp_append_reg(bool c, float c_v, int c_id, float* wv, int* wi,
                                               int K, int& count, float& theta, bool& ovf) {
  unsigned b = __ballot_sync(0xffffffffu, c);
  if (b == 0u) return;
  if (count + __popc(b) > TW_WCAP) {
    if (!ovf) {
      const Compacted r = warp_compact_nl(wv, wi, count, K);
      count = r.count;
      theta = r.theta;
      ovf = r.overflow != 0;
      c = c && c_v >= theta;
      b = __ballot_sync(0xffffffffu, c);
      if (count + __popc(b) > TW_WCAP) ovf = true;
    }
    if (ovf) return;  // the row is redone by the fix-up kernel
  }
  if (c) {
    const int slot = count + __popc(b & ((1u << (threadIdx.x & 31)) - 1u));
    wv[slot] = c_v;
    wi[slot] = c_id;
  }
  count += __popc(b);
}

// Sorts 4 keys of one thread descending (5 compare-exchanges).
__device__ __forceinline__ void sort4_desc(uint64_t (&k)[4]) {
  auto cx = [](uint64_t& a, uint64_t& b) {
    if (a < b) {
      const uint64_t t = a;
      a = b;
      b = t;
    }
  };
  cx(k[0], k[1]);
  cx(k[2], k[3]);
  cx(k[0], k[2]);
  cx(k[1], k[3]);
  cx(k[1], k[2]);
}

// Warp bitonic sort, descending, of 64 keys held 2 per lane at index r*32+lane.
__device__ __forceinline__ void warp_sort64_desc(uint64_t& k0, uint64_t& k1) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int j = size >> 1; j > 0; j >>= 1) {
      if (j == 32) {
        // size 64: one descending block, k0 holds the lower indices
        if (k0 < k1) {
          const uint64_t t = k0;
          k0 = k1;
          k1 = t;
        }
      } else {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          uint64_t& k = r == 0 ? k0 : k1;
          const int i = r * 32 + lane;
          const bool down = (i & size) == 0;
          const uint64_t o = __shfl_xor_sync(0xffffffffu, k, j);
          const bool lower = (lane & j) == 0;
          const uint64_t mx = k > o ? k : o, mn = k > o ? o : k;
          k = (lower == down) ? mx : mn;
        }
      }
    }
  }
}

__device__ void finish_keys_warp(const SampleArgs& a, int row, uint64_t k0, uint64_t k1, int m,
                                 float* wsm, float u);
__device__ void finish_weights_warp(const SampleArgs& a, int row, uint64_t k0, uint64_t k1, int m,
                                    const float* __restrict__ w, float* __restrict__ S,
                                    bool any_slow, float u);

// Finishing stage by one warp for m <= 64 candidates (TokenSampler.cs:95-132).
// `wsm` holds 128 floats of shared memory. Only warp 0 calls.
__device__ __noinline__ void finish_row_warp(const SampleArgs& a, int row, const float* cv,
                                            const int* cid, int m, float* wsm,
                                            bool presorted = false, float u = -1.0f) {
  const int lane = threadIdx.x & 31;
  uint64_t k0 = lane < m ? cand_key(cv[lane], cid[lane]) : 0ull;
  uint64_t k1 = lane + 32 < m ? cand_key(cv[lane + 32], cid[lane + 32]) : 0ull;
  if (!presorted) warp_sort64_desc(k0, k1);
  finish_keys_warp(a, row, k0, k1, m, wsm, u >= 0.0f ? u : a.uniforms[row]);
}

// The same from keys already sorted descending (index r*32+lane in k0/k1; the
// first m are the candidates) and the row's uniform u.
__device__ __noinline__ void finish_keys_warp(const SampleArgs& a, int row, uint64_t k0,
                                             uint64_t k1, int m, float* wsm, float u) {
  const int lane = threadIdx.x & 31;
  uint64_t k[2] = {k0, k1};
  const float vmax = cand_val(__shfl_sync(0xffffffffu, k[0], 0));
  float* w = wsm;        // [64]
  float* S = wsm + 64;   // [64]
  if (!(vmax > -INFINITY)) {
    if (lane == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_NONFINITE;
    }
    return;
  }
  bool slow = false;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = r * 32 + lane;
    if (i < m) w[i] = exp_cr(__fsub_rn(cand_val(k[r]), vmax), slow);
  }
  const bool any_slow = __any_sync(0xffffffffu, slow);
  __syncwarp();
  finish_weights_warp(a, row, k0, k1, m, w, S, any_slow, u);
}

// The rest of the finish once the weights w[i] = exp(v_i - max) of the m
// sorted candidates are in shared memory (`S`: 64 floats of shared scratch).
// Lane 0 runs the sequential fp32 sums (TokenSampler.cs:96-103) into S; every
// lane keeps S[lane] and S[lane + 32], so the cutoff (:105-119) and draw
// (:125-132) searches are ballots on registers; the boundary tests run on
// four lanes at once.
__device__ __noinline__ void finish_weights_warp(const SampleArgs& a, int row, uint64_t k0,
                                                uint64_t k1, int m, const float* __restrict__ w,
                                                float* __restrict__ S, bool any_slow, float u) {
  const int lane = threadIdx.x & 31;
  uint64_t k[2] = {k0, k1};
  const float w_lo = lane < m ? w[lane] : 0.0f;
  const float w_hi = lane + 32 < m ? w[lane + 32] : 0.0f;
  // lane 0 runs the sequential sums from shared memory (the loads run ahead
  // of the chain of adds), every lane then reads its S_i
  if (lane == 0) {
    float t = 0.0f;
#pragma unroll 8
    for (int i = 0; i < m; ++i) {
      t = __fadd_rn(t, w[i]);
      S[i] = t;
    }
  }
  __syncwarp();
  const float s_lo = lane < m ? S[lane] : 0.0f;
  const float s_hi = lane + 32 < m ? S[lane + 32] : 0.0f;
  const float total = m > 0 ? S[m - 1] : 0.0f;
  __syncwarp();
  // S[i] for a per-lane index i (every lane calls)
  auto S_at = [&](int i) -> float {
    const float lo = __shfl_sync(0xffffffffu, s_lo, i & 31);
    const float hi = __shfl_sync(0xffffffffu, s_hi, i & 31);
    return i < 32 ? lo : hi;
  };
  int cutoff = m;
  float target = 0.0f;
  if (a.p.top_p < 1.0f) {
    target = __fmul_rn(total, a.p.top_p);  // total = S[m - 1]
    const unsigned b0 = __ballot_sync(0xffffffffu, lane < m && s_lo >= target);
    const unsigned b1 = __ballot_sync(0xffffffffu, lane + 32 < m && s_hi >= target);
    cutoff = b0 ? __ffs(b0) : (b1 ? 32 + __ffs(b1) : m);
  }
  const float retained = S_at(cutoff - 1);
  const float sample = __fmul_rn(u, retained);
  int sel;
  {
    const unsigned b0 = __ballot_sync(0xffffffffu, lane < cutoff && sample <= s_lo);
    const unsigned b1 = __ballot_sync(0xffffffffu, lane + 32 < cutoff && sample <= s_hi);
    sel = b0 ? __ffs(b0) - 1 : (b1 ? 32 + __ffs(b1) - 1 : cutoff - 1);
  }
  // boundary tests: lanes 0/1 the draw against S[sel] and S[sel - 1], lanes
  // 2/3 the cutoff against S[cutoff - 1] and S[cutoff - 2]
  const int ti = lane == 0 ? sel : lane == 1 ? sel - 1 : lane == 2 ? cutoff - 1 : cutoff - 2;
  const float sv = S_at(ti > 0 ? ti : 0);
  bool hit = false;
  if (lane < 2) {
    const double tol = 1e-6 * (double)retained;
    hit = ti >= 0 && fabs((double)sample - (double)sv) <= tol;
  } else if (lane < 4 && a.p.top_p < 1.0f) {
    const double tt = 1e-6 * (double)target;
    hit = ti >= 0 && fabs((double)sv - (double)target) <= tt;
  }
  const unsigned fb = __ballot_sync(0xffffffffu, hit);
  // token and the tie flag from the sorted keys
  const int rs = sel >> 5, ls = sel & 31;
  uint64_t ksel = 0, kprev = 0, knext = 0;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint64_t t0 = __shfl_sync(0xffffffffu, k[r], ls);
    if (r == rs) ksel = t0;
    const int ip = sel - 1, in = sel + 1;
    const uint64_t tp = __shfl_sync(0xffffffffu, k[r], ip & 31);
    const uint64_t tn = __shfl_sync(0xffffffffu, k[r], in & 31);
    if (ip >= 0 && r == (ip >> 5)) kprev = tp;
    if (r == (in >> 5)) knext = tn;
  }
  if (lane == 0) {
    const uint32_t ks = (uint32_t)(ksel >> 32);
    const bool tie = (sel > 0 && (uint32_t)(kprev >> 32) == ks) ||
                     (sel + 1 < m && (uint32_t)(knext >> 32) == ks);
    a.tokens[row] = cand_id(ksel);
    if (a.flags) {
      uint32_t f = any_slow ? FLAG_EXP_SLOW : 0u;
      if (fb & 3u) f |= FLAG_DRAW_BOUNDARY;
      if (fb & 12u) f |= FLAG_CUTOFF_BOUNDARY;
      if (tie) f |= FLAG_TIE_AT_DRAW;
      a.flags[row] = f;
    }
  }
  if (a.probs) {
    float* prow = a.probs + (size_t)row * a.V;
    if (lane < cutoff) prow[cand_id(k[0])] = __fdiv_rn(w_lo, retained);
    if (lane + 32 < cutoff) prow[cand_id(k[1])] = __fdiv_rn(w_hi, retained);
  }
}


}  // namespace nvs
