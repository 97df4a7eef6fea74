// Streaming top-k sampling kernel for k <= 64 (sm_100a), 128-bit loads.
//
// Same semantics as topk_kernel (TokenSampler.cs:54-135); the schedule is
// built for HBM throughput:
//  - every thread streams its float4s with four independent 128-bit loads in
//    flight (evict-first), so the row is read once with no shared-memory
//    staging and no barrier in the loop. Per value the loop does one multiply,
//    one NaN/+inf test and one threshold test; one vote per step of 16 values
//    decides whether the out-of-line candidate path runs at all;
//  - the first step is also the sample: exact (penalised) values, each
//    thread's maximum, and the K-th largest of those 512 maxima -- distinct
//    elements of the segment, so a lower bound of its K-th largest value;
//  - candidates go to per-warp buffers (ballot + popc); a full buffer is
//    sorted in registers and cut to its top K plus ties, raising that warp's
//    threshold;
//  - one CTA select over the warp buffers gives the segment's K-th largest;
//    one warp (or the CTA, above 64 candidates) runs the exact finish.
// Penalties that can only lower a value (repetition >= 1, frequency and
// presence >= 0) are applied to candidates only: raw*scale >= theta is a
// superset test. Other penalties take the exact path for every float4 that
// holds a penalised id.
#pragma once

#include "sampler_device.cuh"
#include "topk_kernels.cuh"
#include "warp_select.cuh"

namespace nvs {

constexpr int TL_THREADS = 512;
constexpr int TL_WARPS = TL_THREADS / 32;
constexpr int TL_UNROLL = 4;                       // float4 loads in flight per thread
constexpr int TL_STEP = TL_THREADS * TL_UNROLL;    // float4 per CTA step
constexpr int TL_KMAX = 64;
constexpr int TL_WORK = 32768;                     // finish / merge / histogram work area

inline size_t tl_smem_bytes(int bm_words, int h_cap) {
  return (size_t)TL_WARPS * TW_WCAP * 8      // warp buffers
         + (size_t)TK_CAPB * 8               // compact candidate list
         + (size_t)TL_WORK                   // finish / merge work, per-warp histograms
         + 256 * 4                           // radix histogram
         + (size_t)bm_words * 4 + (size_t)h_cap * 4;
}

// k-th largest key (low bits cleared when passes < 4) among the N keys each
// thread holds (key 0 = not an element). Histograms are private per warp
// (`whist`, 256 words per warp) and summed per pass, so equal keys only
// contend within a warp. Returns 0 when fewer than k elements exist. All
// threads call; ends with __syncthreads().
template <int N>
__device__ uint32_t cta_kth_largest_warphist(const uint32_t (&keys)[N], int k, int passes,
                                             uint32_t* whist, uint32_t* hist, int* sh) {
  uint32_t prefix = 0u, mask = 0u;
  int krem = k;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
#pragma unroll 1
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < nw * 256; i += blockDim.x) whist[i] = 0u;
    __syncthreads();
    uint32_t* mine = whist + warp * 256;
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (keys[j] != 0u && (keys[j] & mask) == prefix) atomicAdd(&mine[(keys[j] >> shift) & 255u], 1u);
    __syncthreads();
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
      uint32_t s = 0u;
      for (int w = 0; w < nw; ++w) s += whist[w * 256 + b];
      hist[b] = s;
    }
    __syncthreads();
    if (warp == 0) {
      int c[8];
      int sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = (int)hist[255 - 8 * lane - j];
        sum += c[j];
      }
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      if (lane == 0 && total < krem) {
        sh[0] = -1;
        sh[1] = 0;
      }
      const int excl = incl - sum;
      if (total >= krem && excl < krem && krem <= incl) {
        int run = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (run + c[j] >= krem) {
            sh[0] = 255 - 8 * lane - j;
            sh[1] = run;
            break;
          }
          run += c[j];
        }
      }
    }
    __syncthreads();
    const int digit = sh[0];
    if (digit < 0) {
      __syncthreads();
      return 0u;
    }
    krem -= sh[1];
    prefix |= (uint32_t)digit << shift;
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  return prefix;
}

// Warp state carried through the stream loop (warp-uniform).
struct TlWarp {
  int count;
  float theta;
  int overflow;
  int nonfinite;  // an exact value of this lane was NaN or +inf
};

// Rare path of the stream loop, out of line: the lanes' candidates among one
// step's 16 values (4 float4, columns col0 + 4*u*TL_THREADS ... ) are made
// exact (penalties) and appended to the warp buffer. `x` holds raw logits.
// With `all_exact` (a penalty that can raise a value) every value is made
// exact; otherwise only those at or above the threshold, or not finite.
__device__ __noinline__ TlWarp tl_candidates(TlWarp st, const Penalty* P, float scale, float4 x0,
                                             float4 x1, float4 x2, float4 x3, int col0,
                                             int nvalid, float* wv, int* wi, int K,
                                             bool all_exact) {
  const float4 xs[4] = {x0, x1, x2, x3};
  float ev[16];
  uint32_t mine = 0u;  // bit (u*4+j): candidate
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float r[4] = {xs[u].x, xs[u].y, xs[u].z, xs[u].w};
    const int col = col0 + 4 * u * TL_THREADS;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v = -INFINITY;
      if (u < nvalid) {
        v = __fmul_rn(r[j], scale);
        // exact value near the threshold, and wherever raw*scale is not finite
        if ((all_exact || v >= st.theta || !(v < INFINITY)) && (P->rep || P->cnt))
          v = __fmul_rn(adjust(*P, r[j], col + j), scale);
        if (!(v < INFINITY)) {
          st.nonfinite = 1;
          v = -INFINITY;
        }
      }
      ev[u * 4 + j] = v;
      if (v >= st.theta) mine |= 1u << (u * 4 + j);
    }
  }
  uint32_t any = __reduce_or_sync(0xffffffffu, mine);
  while (any != 0u) {
    const int bit = __ffs(any) - 1;
    any &= any - 1u;
    float v = -INFINITY;
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (t == bit) v = ev[t];
    const int col = col0 + 4 * (bit >> 2) * TL_THREADS + (bit & 3);
    bool ovf = st.overflow != 0;
    warp_append_reg(((mine >> bit) & 1u) && v >= st.theta, canon(v), col, wv, wi, K, st.count,
                    st.theta, ovf);
    st.overflow = ovf ? 1 : 0;
  }
  return st;
}

template <bool kCounts>
__global__ void __launch_bounds__(TL_THREADS, 2)
    topk_ldg_kernel(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* wvall = reinterpret_cast<float*>(smem);                           // [W][WCAP]
  int* wiall = reinterpret_cast<int*>(wvall + TL_WARPS * TW_WCAP);         // [W][WCAP]
  float* cv = reinterpret_cast<float*>(wiall + TL_WARPS * TW_WCAP);        // [CAPB]
  int* cid = reinterpret_cast<int*>(cv + TK_CAPB);                         // [CAPB]
  unsigned char* work = reinterpret_cast<unsigned char*>(cid + TK_CAPB);   // TL_WORK
  uint32_t* whist = reinterpret_cast<uint32_t*>(work);                     // [W][256] in work
  uint32_t* hist = reinterpret_cast<uint32_t*>(work + TL_WORK);            // [256]
  uint32_t* bitmap = hist + 256;
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);

  __shared__ int s_hn, s_nonfinite, s_overflow, s_count, s_last, s_ovf, s_tot;
  __shared__ int s_wn[TL_WARPS];
  __shared__ int s_sh[2];
  __shared__ float s_theta0;
  __shared__ uint32_t s_state;
  __shared__ Penalty s_pen;

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
  if (tid == 0) {
    s_pen = P;
    s_nonfinite = 0;
    s_overflow = 0;
  }
  const bool pen_active = P.rep || P.cnt;
  const bool pen_lowers = !(P.rep && P.pen < 1.0f) && !(P.cnt && (P.freq < 0.0f || P.pres < 0.0f));
  auto val = [&](float l, int col) -> float { return __fmul_rn(adjust(P, l, col), scale); };
  if (a.probs) {
    float* prow = a.probs + (size_t)row * V;
    for (int c = c0 + tid; c < c1; c += TL_THREADS) prow[c] = 0.0f;
  }
  __syncthreads();

  // 16-byte aligned body [a0,a1) as float4; <=3 head and <=3 tail scalars
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)(lrow + c0) & 15u)) & 15u) >> 2);
  const int a0 = min(c0 + head, c1);
  const int a1 = a0 + ((c1 - a0) & ~3);
  const int n4 = (a1 - a0) >> 2;
  const float4* body = reinterpret_cast<const float4*>(lrow + a0);

  float* wv = wvall + warp * TW_WCAP;
  int* wi = wiall + warp * TW_WCAP;
  TlWarp st{0, -INFINITY, 0, 0};
  bool nonfinite = false;

  // ---- first step: exact values, per-thread maxima -> theta0 ----------------
  float4 x[TL_UNROLL];
#pragma unroll
  for (int u = 0; u < TL_UNROLL; ++u) {
    const int q = tid + u * TL_THREADS;
    x[u] = (hist_ok && q < n4) ? __ldcs(body + q) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  {
    float tmax = -INFINITY;
    bool have = false;
#pragma unroll
    for (int u = 0; u < TL_UNROLL; ++u) {
      const int q = tid + u * TL_THREADS;
      if (hist_ok && q < n4) {
        const int col = a0 + 4 * q;
        const float e[4] = {val(x[u].x, col), val(x[u].y, col + 1), val(x[u].z, col + 2),
                            val(x[u].w, col + 3)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (e[j] < INFINITY) {
            tmax = have ? fmaxf(tmax, e[j]) : e[j];
            have = true;
          } else if (e[j] == e[j] || e[j] == INFINITY) {
            nonfinite = true;  // +inf
          } else {
            nonfinite = true;  // NaN
          }
        }
      }
    }
    uint32_t k1[1] = {have ? fkey(canon(tmax)) : 0u};
    const uint32_t key = cta_kth_largest_warphist(k1, K, 4, whist, hist, s_sh);
    // keys at or below the key of -inf decode to NaN patterns: accept all
    if (tid == 0) s_theta0 = key <= fkey(-INFINITY) ? -INFINITY : kval(key);
  }
  __syncthreads();
  st.theta = s_theta0;

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
        nonfinite = true;
        v = -INFINITY;
      }
    }
    bool ovf = false;
    warp_append_reg(act && v >= st.theta, canon(v), col, wv, wi, K, st.count, st.theta, ovf);
    st.overflow = ovf ? 1 : 0;
  }

  // ---- stream: the first step's values are still in registers ---------------
  if (hist_ok) {
#pragma unroll 1
    for (int base = tid; base - tid < n4; base += TL_STEP) {
      if (base != tid) {
#pragma unroll
        for (int u = 0; u < TL_UNROLL; ++u) {
          const int q = base + u * TL_THREADS;
          x[u] = q < n4 ? __ldcs(body + q)
                        : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
      }
      const int nvalid = min(TL_UNROLL, max(0, (n4 - base + TL_THREADS - 1) / TL_THREADS));
      bool cand = false;
      bool bad = false;
#pragma unroll
      for (int u = 0; u < TL_UNROLL; ++u) {
        const float v0 = __fmul_rn(x[u].x, scale), v1 = __fmul_rn(x[u].y, scale);
        const float v2 = __fmul_rn(x[u].z, scale), v3 = __fmul_rn(x[u].w, scale);
        // NaN or +inf: !(v < inf)
        bad = bad || !(v0 < INFINITY) || !(v1 < INFINITY) || !(v2 < INFINITY) || !(v3 < INFINITY);
        cand = cand || v0 >= st.theta || v1 >= st.theta || v2 >= st.theta || v3 >= st.theta;
      }
      // NaN/+inf take the exact path, which decides (a penalty can bring an
      // overflowed raw*scale back to a finite value)
      bool force = bad;
      if (pen_active && !pen_lowers) {
        // a penalty that can raise a value: penalised ids always take the exact path
#pragma unroll
        for (int u = 0; u < TL_UNROLL; ++u)
          if (u < nvalid && penalty_bits4(P, a0 + 4 * (base + u * TL_THREADS)) != 0u) force = true;
      }
      if (__any_sync(0xffffffffu, (cand || force) && nvalid > 0)) {
        st = tl_candidates(st, &s_pen, scale, x[0], x[1], x[2], x[3], a0 + 4 * base, nvalid, wv,
                           wi, K, pen_active && !pen_lowers);
      }
    }
  }
  if (nonfinite || st.nonfinite) s_nonfinite = 1;
  if (st.overflow && lane == 0) s_overflow = 1;
  if (lane == 0) s_wn[warp] = st.count;
  __syncwarp();
  __syncthreads();

  // ---- segment threshold over the warp buffers ------------------------------
  uint32_t state = 0u;
  if (!hist_ok) state |= FLAG_BAD_HISTORY;
  if (s_nonfinite) state |= FLAG_NONFINITE;
  if (s_overflow) state |= RSTATE_OVERFLOW;
  int m = 0;
  if (state == 0u) {
    uint32_t wk[TW_WCAP / 32];
#pragma unroll
    for (int r = 0; r < TW_WCAP / 32; ++r) {
      const int i = tid + r * TL_THREADS;  // flattened [W][WCAP]
      const int w = i / TW_WCAP, e = i % TW_WCAP;
      wk[r] = e < s_wn[w] ? fkey(wvall[i]) : 0u;
    }
    const uint32_t key = cta_kth_largest_warphist(wk, K, 4, whist, hist, s_sh);
    if (tid == 0) {
      s_count = 0;
      s_ovf = 0;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < TW_WCAP / 32; ++r) {
      const int i = tid + r * TL_THREADS;
      const bool ok = wk[r] != 0u && wk[r] >= key;
      warp_append(ok, ok ? wvall[i] : 0.f, ok ? wiall[i] : 0, cv, cid, &s_count, &s_ovf);
    }
    __syncthreads();
    m = min(s_count, TK_CAPB);
    if (s_ovf) state |= RSTATE_OVERFLOW;
  }

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
  for (int i = tid; i < m; i += TL_THREADS) {
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
  float* uv = reinterpret_cast<float*>(work);            // union: [0, 8 KiB)
  int* uid = reinterpret_cast<int*>(uv + TK_CAPB);        //        [8, 16 KiB)
  if (tid == 0) {
    s_state = __ldcg(&a.s.rowstate[row]);
    int tot = 0;
    for (int sp = 0; sp < S; ++sp) tot += __ldcg(&a.s.cand_n[row * S + sp]);
    s_tot = tot;
  }
  __syncthreads();
  uint32_t mstate = s_state;
  const int total = s_tot;
  if (total > TK_CAPB) mstate |= RSTATE_OVERFLOW;
  int mm = 0;
  if (mstate == 0u) {
    int off = 0;
    for (int sp = 0; sp < S; ++sp) {
      const int n = __ldcg(&a.s.cand_n[row * S + sp]);
      const size_t g = (size_t)(row * S + sp) * TK_CAPB;
      for (int i = tid; i < n; i += TL_THREADS) {
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
    for (int i0 = 0; i0 < total; i0 += TL_THREADS) {
      const int i = i0 + tid;
      const bool ok = i < total && fkey(uv[i]) >= key;
      warp_append(ok, ok ? uv[i] : 0.f, ok ? uid[i] : 0, cv, cid, &s_count, &s_ovf);
    }
    __syncthreads();
    if (s_ovf) mstate |= RSTATE_OVERFLOW;
    mm = min(s_count, TK_CAPB);
  }
  __syncthreads();
  // the union is dead now: the finish reuses the work area
  if (mstate == 0u && mm > 0 && mm <= 64) {
    if (warp == 0) finish_row_warp(a, row, cv, cid, mm, reinterpret_cast<float*>(work));
  } else {
    finish_row(a, row, cv, cid, mm, mstate, work);
  }
  __syncthreads();
  if (tid == 0) {
    a.s.rowstate[row] = 0u;
    a.s.tickets[row] = 0u;
  }
}

}  // namespace nvs
