// Warp-streaming top-k sampling kernel for k <= 64 (sm_100a).
//
// Same semantics as topk_kernel (TokenSampler.cs:54-135); different schedule:
// every warp of the CTA owns a private two-stage ring of TMA bulk copies and a
// private candidate buffer, so streaming a row segment needs no CTA-wide
// barrier. Warps take the segment's 2 KiB chunks round-robin.
//
//  1. each warp waits for its first chunk, applies penalties and the
//     temperature scale in place; one CTA-wide radix select over all first
//     chunks gives theta0, the K-th largest of that sample -- a lower bound of
//     the segment's K-th largest value, so nothing >= the final threshold is
//     ever dropped;
//  2. each warp streams its chunks, appending values >= its threshold to its
//     buffer (ballot + popc, no atomics); a full buffer is sorted in registers
//     (warp bitonic network on 64-bit value/id keys) and cut to its top K plus
//     ties, which raises the warp's threshold;
//  3. one CTA select over the warp buffers gives the segment's K-th largest;
//     the row is finished by one warp (<= 64 candidates) or by the CTA.
// Rows whose ties at the K-th value overflow the buffers are marked for the
// full-vocabulary fix-up kernel.
#pragma once

#include "sampler_device.cuh"
#include "topk_kernels.cuh"

namespace nvs {

constexpr int TW_THREADS = 512;
constexpr int TW_WARPS = TW_THREADS / 32;
constexpr int TW_CH = 512;     // floats per warp chunk (2 KiB)
constexpr int TW_CH4 = TW_CH / 4;
constexpr int TW_NST = 2;      // ring stages per warp
constexpr int TW_WCAP = 128;   // candidate entries per warp
constexpr int TW_KMAX = 64;
constexpr int TW_RING_FLOATS = TW_WARPS * TW_NST * TW_CH;  // 64 KiB

inline size_t tw_smem_bytes(int bm_words, int h_cap) {
  return (size_t)TW_RING_FLOATS * 4 + (size_t)TW_WARPS * TW_WCAP * 8 + 256 * 4 +
         (size_t)TW_WARPS * TW_NST * 8 + (size_t)bm_words * 4 + (size_t)h_cap * 4;
}

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

// Finishing stage by one warp for m <= 64 candidates (TokenSampler.cs:95-132).
// `wsm` holds 128 floats of shared memory. Only warp 0 calls.
__device__ __noinline__ void finish_row_warp(const SampleArgs& a, int row, const float* cv,
                                            const int* cid, int m, float* wsm) {
  const int lane = threadIdx.x & 31;
  uint64_t k[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = r * 32 + lane;
    k[r] = i < m ? cand_key(cv[i], cid[i]) : 0ull;
  }
  // bitonic sort of 64 keys, descending
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int j = size >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int i = r * 32 + lane;
        const bool down = (i & size) == 0;
        if (j >= 32) {
          if (r == 0) {
            const uint64_t x = k[0], y = k[1];
            const bool sw = down ? (x < y) : (x > y);
            if (sw) { k[0] = y; k[1] = x; }
          }
        } else {
          const uint64_t o = __shfl_xor_sync(0xffffffffu, k[r], j);
          const bool lower = (lane & j) == 0;
          const uint64_t mx = k[r] > o ? k[r] : o, mn = k[r] > o ? o : k[r];
          k[r] = (lower == down) ? mx : mn;
        }
      }
    }
  }
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
  int cutoff = m, sel = 0;
  float retained = 0.0f;
  if (lane == 0) {
    float total = 0.0f;
    for (int i = 0; i < m; ++i) {
      total = __fadd_rn(total, w[i]);
      S[i] = total;
    }
    float target = 0.0f;
    if (a.p.top_p < 1.0f) {
      target = __fmul_rn(total, a.p.top_p);
      for (int i = 0; i < m; ++i)
        if (S[i] >= target) { cutoff = i + 1; break; }
    }
    retained = S[cutoff - 1];
    const float sample = __fmul_rn(a.uniforms[row], retained);
    sel = cutoff - 1;
    for (int i = 0; i < cutoff; ++i)
      if (sample <= S[i]) { sel = i; break; }
    uint32_t f = any_slow ? FLAG_EXP_SLOW : 0u;
    const double tol = 1e-6 * (double)retained;
    if (fabs((double)sample - (double)S[sel]) <= tol ||
        (sel >= 1 && fabs((double)sample - (double)S[sel - 1]) <= tol))
      f |= FLAG_DRAW_BOUNDARY;
    if (a.p.top_p < 1.0f) {
      const double tt = 1e-6 * (double)target;
      if (fabs((double)S[cutoff - 1] - (double)target) <= tt ||
          (cutoff >= 2 && fabs((double)S[cutoff - 2] - (double)target) <= tt))
        f |= FLAG_CUTOFF_BOUNDARY;
    }
    if (a.flags) a.flags[row] = f;
  }
  cutoff = __shfl_sync(0xffffffffu, cutoff, 0);
  sel = __shfl_sync(0xffffffffu, sel, 0);
  retained = __shfl_sync(0xffffffffu, retained, 0);
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
    if (tie && a.flags) a.flags[row] |= FLAG_TIE_AT_DRAW;
  }
  if (a.probs) {
    float* prow = a.probs + (size_t)row * a.V;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = r * 32 + lane;
      if (i < cutoff) prow[cand_id(k[r])] = __fdiv_rn(w[i], retained);
    }
  }
}

template <bool kCounts>
__global__ void __launch_bounds__(TW_THREADS, 2) topk_warp_kernel(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* ring = reinterpret_cast<float*>(smem);                          // [W][NST][CH]
  float* wvall = ring + TW_RING_FLOATS;                                  // [W][WCAP]
  int* wiall = reinterpret_cast<int*>(wvall + TW_WARPS * TW_WCAP);       // [W][WCAP]
  uint32_t* hist = reinterpret_cast<uint32_t*>(wiall + TW_WARPS * TW_WCAP);
  uint64_t* bars = reinterpret_cast<uint64_t*>(hist + 256);               // [W][NST]
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(bars + TW_WARPS * TW_NST);
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);
  // after streaming, the ring is reused for the compact candidate list + finish
  float* cv = ring;                                                       // [CAPB]
  int* cid = reinterpret_cast<int*>(ring + TK_CAPB);                      // [CAPB]
  unsigned char* work = reinterpret_cast<unsigned char*>(ring + 2 * TK_CAPB);

  __shared__ int s_hn, s_nonfinite, s_timeout, s_overflow, s_count, s_last, s_ovf;
  __shared__ int s_wn[TW_WARPS];
  __shared__ int s_sh[2];
  __shared__ float s_theta0;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const int V = a.V;
  const int K = min(a.p.top_k, V);
  const int c0 = split * a.seg_len;
  const int c1 = min(V, c0 + a.seg_len);
  const float* lrow = a.logits + (size_t)row * V;
  const float scale = __fdiv_rn(1.0f, a.p.temperature);  // TokenSampler.cs:68

  Penalty P;
  const bool hist_ok = setup_penalty<kCounts>(P, a, row, c0, c1, bitmap, hsorted, &s_hn);

  const int head = (int)(((16u - ((uint32_t)(uintptr_t)(lrow + c0) & 15u)) & 15u) >> 2);
  const int a0 = min(c0 + head, c1);
  const int a1 = a0 + ((c1 - a0) & ~3);
  const int nch = (a1 - a0 + TW_CH - 1) / TW_CH;                 // chunks in the segment
  const int my_n = nch > warp ? (nch - warp + TW_WARPS - 1) / TW_WARPS : 0;  // my chunks

  float* myring = ring + warp * TW_NST * TW_CH;
  uint64_t* mybars = bars + warp * TW_NST;
  float* wv = wvall + warp * TW_WCAP;
  int* wi = wiall + warp * TW_WCAP;

  if (tid == 0) {
    s_nonfinite = 0;
    s_timeout = 0;
    s_overflow = 0;
  }
  if (lane == 0) {
    for (int i = 0; i < TW_NST; ++i) mbar_init(&mybars[i], 1);
    fence_mbar_init();
  }
  if (a.probs) {
    float* prow = a.probs + (size_t)row * V;
    for (int c = c0 + tid; c < c1; c += TW_THREADS) prow[c] = 0.0f;
  }
  __syncwarp();
  auto chunk_len = [&](int j) {  // floats in my j-th chunk
    const int c = warp + j * TW_WARPS;
    return min(TW_CH, a1 - (a0 + c * TW_CH));
  };
  auto issue = [&](int j) {
    const int c = warp + j * TW_WARPS;
    const int len = chunk_len(j);
    uint64_t* bar = &mybars[j % TW_NST];
    mbar_arrive_expect_tx(bar, (uint32_t)len * 4u);
    bulk_g2s(myring + (j % TW_NST) * TW_CH, lrow + a0 + c * TW_CH, (uint32_t)len * 4u, bar);
  };
  int issued = 0;
  if (hist_ok && lane == 0) {
    for (int j = 0; j < min(TW_NST, my_n); ++j) issue(j);
  }
  issued = hist_ok ? min(TW_NST, my_n) : 0;

  // values exactly as the reference computes them; NaN/+inf flag the row
  auto val = [&](float l, int col) -> float {
    return __fmul_rn(adjust(P, l, col), scale);
  };
  // Penalties active on this row, and whether they can only lower a value
  // (repetition >= 1 divides positives and multiplies non-positives by >= 1;
  // non-negative frequency/presence subtract): then raw*scale >= theta is a
  // superset test and exact values are needed only for candidates.
  const bool pen_active = P.rep || P.cnt;
  const bool pen_lowers = !(P.rep && P.pen < 1.0f) && !(P.cnt && (P.freq < 0.0f || P.pres < 0.0f));

  // ---- 1. first chunk of every warp -> theta0 ------------------------------
  int consumed = 0;
  int first_len = 0;
  if (hist_ok && my_n > 0) {
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&mybars[0], 0u));
    if (!ok) {
      if (lane == 0) s_timeout = 1;
    } else {
      first_len = chunk_len(0);
      float4* q4 = reinterpret_cast<float4*>(myring);
      const int base = a0 + warp * TW_CH;
      for (int q = lane; q < first_len / 4; q += 32) {
        float4 x = q4[q];
        const int col = base + 4 * q;
        x.x = val(x.x, col);
        x.y = val(x.y, col + 1);
        x.z = val(x.z, col + 2);
        x.w = val(x.w, col + 3);
        if (!(x.x < INFINITY) || !(x.y < INFINITY) || !(x.z < INFINITY) || !(x.w < INFINITY))
          s_nonfinite = 1;
        q4[q] = x;
      }
      // these generic-proxy writes must be ordered before the TMA copy that
      // later refills this stage: every writing thread fences
      fence_proxy_async();
    }
  }
  if (lane == 0) s_wn[warp] = first_len;
  __syncthreads();
  {
    const uint32_t key = cta_kth_largest(
        [&](int i) -> uint32_t {
          const int w = i / TW_CH, r = i % TW_CH;
          if (r >= s_wn[w]) return 0u;
          const float v = ring[w * TW_NST * TW_CH + r];
          return (v < INFINITY) ? fkey(canon(v)) : 0u;
        },
        TW_WARPS * TW_CH, K, hist, s_sh, 2);
    // two radix passes: the sample's K-th largest key with its low 16 bits
    // cleared, still a lower bound of the segment's K-th largest value
    // keys at or below the key of -inf decode to NaN patterns: accept all
    if (tid == 0) s_theta0 = key <= fkey(-INFINITY) ? -INFINITY : kval(key);
  }
  __syncthreads();
  float theta_w = s_theta0;
  int count = 0;
  bool tie_ovf = false;

  // head/tail scalars (<= 6) go to warp 0's buffer
  if (warp == 0 && hist_ok) {
    const int nh = a0 - c0, nt = c1 - a1;
    const bool act = lane < nh + nt;
    float v = -INFINITY;
    int col = 0;
    if (act) {
      col = lane < nh ? c0 + lane : a1 + (lane - nh);
      v = val(lrow[col], col);
      if (!(v < INFINITY)) {
        s_nonfinite = 1;
        v = -INFINITY;
      }
    }
    warp_append_reg(act && v >= theta_w, canon(v), col, wv, wi, K, count, theta_w, tie_ovf);
  }

  // ---- 2. stream ------------------------------------------------------------
  if (hist_ok && !s_timeout) {
    for (int j = 0; j < my_n; ++j) {
      const int st = j % TW_NST;
      const int len = chunk_len(j);
      const int base = a0 + (warp + j * TW_WARPS) * TW_CH;
      const float4* q4 = reinterpret_cast<const float4*>(myring + st * TW_CH);
      if (j > 0) {
        const bool ok =
            __all_sync(0xffffffffu, mbar_wait_bounded(&mybars[st], (uint32_t)((j / TW_NST) & 1)));
        if (!ok) {
          if (lane == 0) s_timeout = 1;
          break;
        }
      }
#pragma unroll 1
      for (int m4 = 0; m4 < TW_CH4 / 32; ++m4) {
        const int q = lane + 32 * m4;
        const bool valid = q < (len >> 2);
        const int col = base + 4 * q;
        float vv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        bool any = false;
        // `exact`: vv already holds the penalised values
        bool exact = (j == 0) || !pen_active;
        if (valid) {
          x = q4[q];
          if (j == 0) {  // already penalised and scaled in place
            vv[0] = x.x; vv[1] = x.y; vv[2] = x.z; vv[3] = x.w;
          } else {
            vv[0] = __fmul_rn(x.x, scale);
            vv[1] = __fmul_rn(x.y, scale);
            vv[2] = __fmul_rn(x.z, scale);
            vv[3] = __fmul_rn(x.w, scale);
            if (!(vv[0] < INFINITY) || !(vv[1] < INFINITY) || !(vv[2] < INFINITY) ||
                !(vv[3] < INFINITY))
              s_nonfinite = 1;
            if (pen_active && !pen_lowers && penalty_bits4(P, col) != 0u) {
              // a penalty that can raise a value: exact values up front
              vv[0] = val(x.x, col);
              vv[1] = val(x.y, col + 1);
              vv[2] = val(x.z, col + 2);
              vv[3] = val(x.w, col + 3);
              if (!(vv[0] < INFINITY) || !(vv[1] < INFINITY) || !(vv[2] < INFINITY) ||
                  !(vv[3] < INFINITY))
                s_nonfinite = 1;
              exact = true;
            }
          }
          // penalties that only lower values: raw*scale >= theta is a superset test
          any = vv[0] >= theta_w || vv[1] >= theta_w || vv[2] >= theta_w || vv[3] >= theta_w;
        }
        if (__any_sync(0xffffffffu, any)) {
          if (!exact && any) {
            // exact penalised values for this lane's four (only near the threshold)
            vv[0] = val(x.x, col);
            vv[1] = val(x.y, col + 1);
            vv[2] = val(x.z, col + 2);
            vv[3] = val(x.w, col + 3);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e)
            warp_append_reg(valid && vv[e] >= theta_w && vv[e] < INFINITY, canon(vv[e]), col + e,
                            wv, wi, K, count, theta_w, tie_ovf);
        }
      }
      __syncwarp();
      consumed = j + 1;
      if (lane == 0 && j + TW_NST < my_n) {
        fence_proxy_async();
        issue(j + TW_NST);
      }
      if (j + TW_NST < my_n) issued = j + TW_NST + 1;
    }
  }
  // copies still in flight after an early exit (bounded waits)
  if (lane == 0) {
    for (int j = consumed; j < issued; ++j)
      (void)mbar_wait_bounded(&mybars[j % TW_NST], (uint32_t)((j / TW_NST) & 1));
  }
  // (no final per-warp cut: the segment select below reads the buffers whole)
  if (tie_ovf && lane == 0) s_overflow = 1;
  if (lane == 0) s_wn[warp] = count;
  __syncthreads();

  // ---- 3. segment threshold over the warp buffers ---------------------------
  uint32_t state = 0u;
  if (!hist_ok) state |= FLAG_BAD_HISTORY;
  if (s_nonfinite) state |= FLAG_NONFINITE;
  if (s_overflow) state |= RSTATE_OVERFLOW;
  if (s_timeout) state |= RSTATE_TIMEOUT;
  int m = 0;
  if (state == 0u) {
    const uint32_t key = cta_kth_largest(
        [&](int i) -> uint32_t {
          const int w = i / TW_WCAP, r = i % TW_WCAP;
          return r < s_wn[w] ? fkey(wvall[i]) : 0u;
        },
        TW_WARPS * TW_WCAP, K, hist, s_sh);
    if (tid == 0) {
      s_count = 0;
      s_ovf = 0;
    }
    __syncthreads();
    for (int i0 = 0; i0 < TW_WARPS * TW_WCAP; i0 += TW_THREADS) {
      const int i = i0 + tid;
      const int w = i / TW_WCAP, r = i % TW_WCAP;
      const bool ok = r < s_wn[w] && fkey(wvall[i]) >= key;
      warp_append(ok, ok ? wvall[i] : 0.f, ok ? wiall[i] : 0, cv, cid, &s_count, &s_ovf);
    }
    __syncthreads();
    m = min(s_count, TK_CAPB);
    if (s_ovf) state |= RSTATE_OVERFLOW;
  }
  if (s_timeout && tid == 0) atomicOr(a.s.error_word, 1u);

  if (S == 1) {
    if (state == 0u && m > 0 && m <= 64) {
      if (warp == 0) finish_row_warp(a, row, cv, cid, m, reinterpret_cast<float*>(work));
    } else {
      finish_row(a, row, cv, cid, m, state, work);
    }
    return;
  }

  // ---- multi-CTA rows: publish, the last CTA merges --------------------------
  const int cta = row * S + split;
  for (int i = tid; i < m; i += TW_THREADS) {
    a.s.cand_v[(size_t)cta * TK_CAPB + i] = cv[i];
    a.s.cand_id[(size_t)cta * TK_CAPB + i] = cid[i];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    a.s.cand_n[cta] = m;
    if (state) atomicOr(&a.s.rowstate[row], state);
    __threadfence();
    const uint32_t t = atomicAdd(&a.s.tickets[row], 1u);
    s_last = (t == (uint32_t)(S - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // union of the segment lists in the ring area after cv/cid
  float* uv = reinterpret_cast<float*>(work);
  int* uid = reinterpret_cast<int*>(uv + TK_CAPB);
  const int ucap = TK_CAPB;  // ring: cv|cid|uv|uid|finish work (<= 32 KiB) = 64 KiB
  __shared__ uint32_t s_state;
  __shared__ int s_tot;
  if (tid == 0) {
    s_state = __ldcg(&a.s.rowstate[row]);
    int tot = 0;
    for (int sp = 0; sp < S; ++sp) tot += __ldcg(&a.s.cand_n[row * S + sp]);
    s_tot = tot;
  }
  __syncthreads();
  uint32_t mstate = s_state;
  const int total = s_tot;
  if (total > ucap) mstate |= RSTATE_OVERFLOW;
  int mm = 0;
  if (mstate == 0u) {
    int off = 0;
    for (int sp = 0; sp < S; ++sp) {
      const int n = __ldcg(&a.s.cand_n[row * S + sp]);
      const size_t g = (size_t)(row * S + sp) * TK_CAPB;
      for (int i = tid; i < n; i += TW_THREADS) {
        uv[off + i] = __ldcg(&a.s.cand_v[g + i]);
        uid[off + i] = __ldcg(&a.s.cand_id[g + i]);
      }
      off += n;
    }
    __syncthreads();
    const uint32_t key = cta_kth_largest([&](int i) { return fkey(uv[i]); }, total, K, hist, s_sh);
    if (tid == 0) {
      s_count = 0;
      s_ovf = 0;
    }
    __syncthreads();
    for (int i0 = 0; i0 < total; i0 += TW_THREADS) {
      const int i = i0 + tid;
      const bool ok = i < total && fkey(uv[i]) >= key;
      warp_append(ok, ok ? uv[i] : 0.f, ok ? uid[i] : 0, cv, cid, &s_count, &s_ovf);
    }
    __syncthreads();
    if (s_ovf) mstate |= RSTATE_OVERFLOW;
    mm = min(s_count, TK_CAPB);
  }
  __syncthreads();
  // the finish work area follows the union area
  unsigned char* work2 = reinterpret_cast<unsigned char*>(uid + ucap);
  if (mstate == 0u && mm > 0 && mm <= 64) {
    if (warp == 0) finish_row_warp(a, row, cv, cid, mm, reinterpret_cast<float*>(work2));
  } else {
    finish_row(a, row, cv, cid, mm, mstate, work2);
  }
  __syncthreads();
  if (tid == 0) {
    a.s.rowstate[row] = 0u;
    a.s.tickets[row] = 0u;
  }
}

}  // namespace nvs
