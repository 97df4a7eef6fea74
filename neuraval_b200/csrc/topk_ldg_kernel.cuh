// Streaming top-k sampling kernel for k <= 64 (sm_100a), 128-bit loads.
//
// Same semantics as topk_kernel (TokenSampler.cs:54-135); the schedule is
// built for HBM throughput:
//  - every thread streams its float4s with four independent 128-bit loads in
//    flight (evict-first), so the row is read once with no shared-memory
//    staging and no barrier in the loop. Per value the loop does one multiply,
//    one NaN/+inf test and one threshold test; one ballot per float4 queues
//    the float4s that may hold a candidate (values and indices, in shared
//    memory) for a drain outside the loop;
//  - the first step is also the sample: exact (penalised) values, each
//    thread's maximum, and a lower bound of the K-th largest of those 512
//    maxima -- distinct elements of the segment, so a lower bound of its K-th
//    largest value;
//  - candidates go to per-warp buffers (ballot + popc); a full buffer is
//    sorted in registers and cut to its top K plus ties, raising that warp's
//    threshold;
//  - after the stream every warp publishes its 16 largest keys; ranks by
//    binary search across those lists give the K-th value and the sorted
//    candidates directly, weights are computed in parallel and one warp runs
//    the sequential sums and the draw (a split row's segments publish their
//    sorted candidates and the last CTA ranks their union). Full lists and
//    ties beyond 64 candidates fall back to histogram selects over all
//    buffered values.
// Penalties that can only lower a value (repetition >= 1, frequency and
// presence >= 0) are applied to candidates only: raw*scale >= theta is a
// superset test. Other penalties take the exact path for every float4 that
// holds a penalised id.
#pragma once

#include "sampler_device.cuh"
#include "topk_kernels.cuh"
#include "warp_select.cuh"
#include "rank_select.cuh"

namespace nvs {

constexpr int TL_THREADS = 512;
constexpr int TL_WARPS = TL_THREADS / 32;
constexpr int TL_UNROLL = 4;                       // float4 loads in flight per thread
constexpr int TL_STEP = TL_THREADS * TL_UNROLL;    // float4 per CTA step
constexpr int TL_KMAX = 64;
constexpr int TL_WORK = 32768;                     // select / finish / merge area
// Queued float4s per warp during the stream (value and index), in the
// candidate-list and work areas (contiguous, 48 KiB, unused while streaming).
constexpr int TL_QV = 152;
static_assert(TL_WARPS * TL_QV * 20 <= TK_CAPB * 8 + TL_WORK, "stream queues do not fit");

inline size_t tl_smem_bytes(int bm_words, int h_cap) {
  return (size_t)TL_WARPS * TW_WCAP * 8      // warp buffers
         + (size_t)TK_CAPB * 8               // compact candidate list
         + (size_t)TL_WORK                   // select, finish and merge work
                                             // (with the candidate list: stream queues)
         + 256 * 4                           // radix histogram
         + (size_t)bm_words * 4 + (size_t)h_cap * 4;
}

constexpr int TL_NB = 1024;   // linear bins of the selection histograms (2 per thread)
constexpr int TL_GCAP = 1024;  // candidates gathered by the final select (lower half of cv/cid)
constexpr int TL_BINCAP = 256; // values of the K-th value's bin
constexpr int TL_TOPW = 16;    // keys per warp in the final lists (16 x 16 = 256)
constexpr int TL_LISTV = 512;  // float offset in cv of the lists' value keys (after 256 keys)

// k-th largest of the values held N per thread (valid[j] marks real values;
// -inf, NaN and +inf must not be marked), via one histogram of TL_NB linear
// bins over [lo, hi] (bin 0 holds the largest values).
//  exact == false: returns a lower bound of the k-th largest (the smallest
//                  value in its bin).
//  exact == true : returns the k-th largest exactly; values of its bin are
//                  ranked in shared memory (`work`, TL_WORK bytes: the bins,
//                  then the bin's values) and, when that bin is crowded, by a
//                  radix select (`hist256`, `sh`).
// Returns -inf when fewer than k values are marked. All threads call.
template <int N>
__device__ float cta_select_linear(const float (&v)[N], const bool (&valid)[N], int k, bool exact,
                                   unsigned char* work, uint32_t* hist256, int* sh) {
  __shared__ float s_red[2][TL_WARPS];
  __shared__ int s_cnt[TL_WARPS];
  __shared__ float s_hi, s_lo, s_res;
  __shared__ int s_bstar, s_above, s_nbin, s_total;
  __shared__ uint32_t s_minkey;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* bins = reinterpret_cast<uint32_t*>(work);              // [TL_NB]
  float* binv = reinterpret_cast<float*>(work + TL_NB * 4);        // values of bin b*
  const int binv_cap = (TL_WORK - TL_NB * 4) / 4;
  // 1. max, min, count
  float hi = -INFINITY, lo = INFINITY;
  int c = 0;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (valid[j]) {
      hi = fmaxf(hi, v[j]);
      lo = fminf(lo, v[j]);
      ++c;
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  if (lane == 0) {
    s_red[0][warp] = hi;
    s_red[1][warp] = lo;
    s_cnt[warp] = c;
  }
  for (int i = tid; i < TL_NB; i += blockDim.x) bins[i] = 0u;
  __syncthreads();
  if (tid == 0) {
    float h = -INFINITY, l = INFINITY;
    int t = 0;
    for (int w = 0; w < TL_WARPS; ++w) {
      h = fmaxf(h, s_red[0][w]);
      l = fminf(l, s_red[1][w]);
      t += s_cnt[w];
    }
    s_hi = h;
    s_lo = l;
    s_total = t;
    s_nbin = 0;
  }
  __syncthreads();
  hi = s_hi;
  lo = s_lo;
  const int total = s_total;
  if (total < k) return -INFINITY;
  if (!(hi > lo)) return hi;  // all marked values equal
  const float sc = __fdiv_rn((float)TL_NB, __fsub_rn(hi, lo));
  auto bin_of = [&](float x) {
    const float f = __fmul_rn(__fsub_rn(hi, x), sc);  // monotone: larger x -> smaller bin
    const int b = (int)f;
    return b < TL_NB - 1 ? b : TL_NB - 1;
  };
  // 2. histogram
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (valid[j]) atomicAdd(&bins[bin_of(v[j])], 1u);
  __syncthreads();
  // 3. first bin where the count from the top reaches k: CTA-wide scan over
  //    the bins, TL_NB / blockDim per thread
  {
    constexpr int PER = TL_NB / TL_THREADS;
    int cb[PER];
    int sum = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      cb[j] = (int)bins[tid * PER + j];
      sum += cb[j];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) s_cnt[warp] = incl;
    __syncthreads();
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += s_cnt[w];
    const int excl = wbase + incl - sum;
    if (excl < k && k <= excl + sum) {
      int run = excl;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        if (run + cb[j] >= k) {
          s_bstar = tid * PER + j;
          s_above = run;
          break;
        }
        run += cb[j];
      }
    }
  }
  if (tid == 0) {
    s_res = INFINITY;
    s_minkey = 0xFFFFFFFFu;
  }
  __syncthreads();
  const int bstar = s_bstar;
  const int above = s_above;
  // 4. the values of bin b*
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (valid[j] && bin_of(v[j]) == bstar) {
      const int slot = atomicAdd(&s_nbin, 1);
      if (slot < binv_cap) binv[slot] = v[j];
      if (!exact) atomicMin(&s_minkey, fkey(v[j]));
    }
  __syncthreads();
  if (!exact) return kval(s_minkey);
  const int nb = s_nbin;
  const int r = k - above;  // rank of the answer inside bin b* (1-based)
  if (nb <= 32) {
    if (warp == 0) {
      const float x = lane < nb ? binv[lane] : -INFINITY;
      int gt = 0, ge = 0;
      for (int i = 0; i < nb; ++i) {
        const float y = binv[i];
        gt += y > x;
        ge += y >= x;
      }
      if (lane < nb && gt < r && r <= ge) s_res = x;
    }
    __syncthreads();
    return s_res;
  }
  // crowded bin: exact radix select among its values
  const int n = min(nb, binv_cap);
  const uint32_t key = cta_kth_largest([&](int i) { return fkey(binv[i]); }, n, r, hist256, sh);
  return kval(key);
}

template <bool kCounts, bool kShard>
__device__ __forceinline__ void topk_ldg_body(const SampleArgs& a, int* owner);

template <bool kCounts, bool kShard = false>
__global__ void __launch_bounds__(TL_THREADS, 2)
    topk_ldg_kernel(const __grid_constant__ SampleArgs a) {
  __shared__ int s_owner;
  // launched as a programmatic dependent of whatever precedes it on the stream
  // (the producer of the logits, the previous call's fix-up): its launch
  // overlaps that kernel's end, and nothing is read before that kernel's
  // writes are visible (a no-op for an ordinary launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // fix-up mode: rows the chunked finish kernel could not prove, nothing else
  // (every segment of a row reads the same mark; the CTA that completes the
  // row clears it, after every segment of the row has started)
  if (a.fixup_only && __ldcg(a.s.fixup + blockIdx.y) == 0u) return;
  topk_ldg_body<kCounts, kShard>(a, &s_owner);
  if constexpr (kShard) {
    if (a.px.shards > 0) {
      __syncthreads();
      shard_px_epilogue(a.px, a.shard_out + (size_t)blockIdx.y * VS_REC_WORDS, blockIdx.y,
                        s_owner != 0);
    }
  }
  if (a.fixup_only) {
    __syncthreads();
    if (s_owner != 0 && threadIdx.x == 0) a.s.fixup[blockIdx.y] = 0u;
  }
}

template <bool kCounts, bool kShard>
__device__ __forceinline__ void topk_ldg_body(const SampleArgs& a, int* owner) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* wvall = reinterpret_cast<float*>(smem);                           // [W][WCAP]
  int* wiall = reinterpret_cast<int*>(wvall + TL_WARPS * TW_WCAP);         // [W][WCAP]
  float* cv = reinterpret_cast<float*>(wiall + TL_WARPS * TW_WCAP);        // [CAPB]
  int* cid = reinterpret_cast<int*>(cv + TK_CAPB);                         // [CAPB]
  unsigned char* work = reinterpret_cast<unsigned char*>(cid + TK_CAPB);   // TL_WORK
  uint32_t* hist = reinterpret_cast<uint32_t*>(work + TL_WORK);            // [256]
  uint32_t* bitmap = hist + 256;
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);

  __shared__ int s_hn, s_nonfinite, s_overflow, s_count, s_last, s_ovf, s_tot;
  __shared__ int s_wn[TL_WARPS];
  __shared__ float s_wtheta[TL_WARPS], s_wmax[TL_WARPS];
  __shared__ int s_bstar, s_above, s_nbin, s_mode;
  __shared__ float s_kth;
  __shared__ uint64_t s_xkey, s_maxkey;
  __shared__ int s_flags2, s_c;
  __shared__ int s_sh[2];
  __shared__ float s_theta0, s_u;
  __shared__ uint32_t s_state;
  __shared__ Penalty s_pen;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const int V = a.V;
  const int K = min(a.p.top_k, V);
  const int lo = kShard ? a.col_lo : 0, hi = kShard ? a.col_hi : V;
  const int c0 = lo + split * a.seg_len;
  const int c1 = min(hi, c0 + a.seg_len);
  // shard rows are addressed by global column: lrow[c] for c in [lo, hi)
  const float* lrow = kShard ? a.logits + (size_t)row * a.ld - lo : a.logits + (size_t)row * V;
  if (tid == 0) *owner = S == 1;  // the CTA that writes the row's result
  const float scale = __fdiv_rn(1.0f, a.p.temperature);  // TokenSampler.cs:68

  // 16-byte aligned body [a0,a1) as float4; <=3 head and <=3 tail scalars
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)(lrow + c0) & 15u)) & 15u) >> 2);
  const int a0 = min(c0 + head, c1);
  const int a1 = a0 + ((c1 - a0) & ~3);
  const int n4 = (a1 - a0) >> 2;
  const float4* body = reinterpret_cast<const float4*>(lrow + a0);

  // the history offsets, then the sample's loads; the penalty tables are built
  // while the sample is in flight
  const int hb = a.hoff[row], he = a.hoff[row + 1];
  float4 x0[TL_UNROLL];
#pragma unroll
  for (int u = 0; u < TL_UNROLL; ++u) {
    const int q = tid + u * TL_THREADS;
    x0[u] = q < n4 ? __ldcs(body + q) : make_float4(0.f, 0.f, 0.f, 0.f);
  }

  if (!kShard && tid == 0) s_u = a.uniforms[row];  // read by the finish

  Penalty P;
  const bool hist_ok =
      setup_penalty_range<kCounts>(P, a, hb, he, c0, c1, bitmap, hsorted, &s_hn);
  if (tid == 0) {
    s_pen = P;
    s_nonfinite = 0;
    s_overflow = 0;
  }
  const bool pen_active = P.rep || P.cnt;
  const bool pen_lowers = !(P.rep && P.pen < 1.0f) && !(P.cnt && (P.freq < 0.0f || P.pres < 0.0f));
  auto val = [&](float l, int col) -> float { return __fmul_rn(adjust(P, l, col), scale); };
  if (!kShard && a.probs) {
    float* prow = a.probs + (size_t)row * V;
    for (int c = c0 + tid; c < c1; c += TL_THREADS) prow[c] = 0.0f;
  }
  __syncthreads();

  float* wv = wvall + warp * TW_WCAP;
  int* wi = wiall + warp * TW_WCAP;
  int count = 0;
  float theta = -INFINITY;
  bool tie_ovf = false;
  bool nonfinite = false;

  // ---- sample: exact values of the first step, per-thread maxima -> theta0 --
  {
    float tmax = -INFINITY;
    bool have = false;
#pragma unroll
    for (int u = 0; u < TL_UNROLL; ++u) {
      const int q = tid + u * TL_THREADS;
      if (hist_ok && q < n4) {
        const int col = a0 + 4 * q;
        const float e[4] = {val(x0[u].x, col), val(x0[u].y, col + 1), val(x0[u].z, col + 2),
                            val(x0[u].w, col + 3)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (e[j] < INFINITY && e[j] > -INFINITY) {
            tmax = have ? fmaxf(tmax, e[j]) : e[j];
            have = true;
          }
        }
      }
    }
    // while the select below runs (no loads of this CTA in flight), each warp
    // has L2 fetch its own part of the next two steps (bulk prefetch, no
    // registers; the stream's loads of them then hit L2)
    if (lane == 0 && hist_ok) {
#pragma unroll
      for (int st = 1; st <= 2; ++st)
#pragma unroll
        for (int u = 0; u < TL_UNROLL; ++u) {
          const int q = st * TL_STEP + u * TL_THREADS + warp * 32;
          const int e = min(n4, q + 32);
          if (q < e)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(body + q),
                         "r"((unsigned)(e - q) * 16u)
                         : "memory");
        }
    }
    // the smallest maximum in the bin of the K-th largest maximum: distinct
    // elements of the segment, so a lower bound of its K-th largest value
    const float sv[1] = {tmax};
    const bool sok[1] = {have};
    const float lb = cta_select_linear(sv, sok, K, false, work, hist, s_sh);
    if (tid == 0) s_theta0 = lb;
  }
  __syncthreads();
  theta = s_theta0;
  // a shard's record holds finite values only: -inf can be a global candidate
  // only in a row with fewer than K finite values, where it never decides the
  // token (its weight is exp(-inf) = 0)
  if constexpr (kShard) theta = fmaxf(theta, -3.40282347e+38f);

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
    warp_append_reg(act && v >= theta, canon(v), col, wv, wi, K, count, theta, tie_ovf);
  }

  // ---- stream -----------------------------------------------------------------
  // The loop only queues every float4 that may hold a candidate (raw*scale >=
  // theta, a superset when penalties only lower values), a NaN or +inf, or --
  // for penalties that can raise a value -- a penalised id: its value and
  // index, so the drain outside the loop reads nothing from global memory
  // again (exact values, then warp appends).
  float4* qval = reinterpret_cast<float4*>(cv) + warp * TL_QV;
  int* qidx = reinterpret_cast<int*>(reinterpret_cast<float4*>(cv) + TL_WARPS * TL_QV) +
              warp * TL_QV;
  const bool force_pen = pen_active && !pen_lowers;
  int qn = 0;
  int base = tid;
  bool more = hist_ok;
  while (more) {
    more = false;
#pragma unroll 1
    for (; base - tid < n4; base += TL_STEP) {
      float4 x[TL_UNROLL];
#pragma unroll
      for (int u = 0; u < TL_UNROLL; ++u) {
        const int q = base + u * TL_THREADS;
        x[u] = q < n4 ? __ldcs(body + q) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
#pragma unroll
      for (int u = 0; u < TL_UNROLL; ++u) {
        const int q = base + u * TL_THREADS;
        const float v0 = __fmul_rn(x[u].x, scale), v1 = __fmul_rn(x[u].y, scale);
        const float v2 = __fmul_rn(x[u].z, scale), v3 = __fmul_rn(x[u].w, scale);
        bool flag = v0 >= theta || v1 >= theta || v2 >= theta || v3 >= theta ||
                    !(v0 < INFINITY) || !(v1 < INFINITY) || !(v2 < INFINITY) || !(v3 < INFINITY);
        if (force_pen && q < n4 && penalty_bits4(P, a0 + 4 * q) != 0u) flag = true;
        flag = flag && q < n4;
        const unsigned b = __ballot_sync(0xffffffffu, flag);
        if (b != 0u) {
          if (flag) {
            const int at = qn + __popc(b & ((1u << lane) - 1u));
            qval[at] = x[u];
            qidx[at] = q;
          }
          qn += __popc(b);
        }
      }
      if (qn > TL_QV - 32 * TL_UNROLL) {
        base += TL_STEP;
        more = true;
        break;
      }
    }
    // drain: exact values of the queued float4s, appended to the warp buffer
    __syncwarp();
    for (int i0 = 0; i0 < qn; i0 += 32) {
      const int i = i0 + lane;
      const bool valid = i < qn;
      const int q = valid ? qidx[i] : 0;
      const float4 x = valid ? qval[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      const int col = a0 + 4 * q;
      float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = valid ? val(e[j], col + j) : -INFINITY;
        if (!(v < INFINITY)) {
          nonfinite = nonfinite || valid;
          v = -INFINITY;
        }
        e[j] = v;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        warp_append_reg(valid && e[j] >= theta, canon(e[j]), col + j, wv, wi, K, count, theta,
                        tie_ovf);
    }
    __syncwarp();
    qn = 0;
  }
  // every warp's queue is drained before the lists below reuse that area
  __syncthreads();
  // the stream is done: the kernel that follows (the fix-up) may be scheduled
  // once every CTA is here; it waits for this grid's completion before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (nonfinite) s_nonfinite = 1;
  if (tie_ovf && lane == 0) s_overflow = 1;
  // the final select's histogram range: [largest warp threshold, largest
  // buffered value]; its bins (upper half of cv) are free during the stream
  uint32_t* bins = reinterpret_cast<uint32_t*>(cv + TL_GCAP);  // [TL_NB]
  {
    float wmx = -INFINITY;
#pragma unroll
    for (int r = 0; r < TW_WCAP / 32; ++r)
      if (r * 32 + lane < count) wmx = fmaxf(wmx, wv[r * 32 + lane]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wmx = fmaxf(wmx, __shfl_xor_sync(0xffffffffu, wmx, o));
    if (lane == 0) {
      s_wn[warp] = count;
      s_wtheta[warp] = theta;  // a lower bound of the segment's K-th value
      s_wmax[warp] = wmx;
    }
    // the warp's TL_TOPW largest keys, descending, to the list area (cv[0..)):
    // each lane sorts its 4 entries, then rounds of warp max (redux) pop heads
    uint64_t k[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = r * 32 + lane;
      k[r] = i < count ? cand_key(wv[i], wi[i]) : 0ull;
    }
    sort4_desc(k);
    uint64_t mine = 0ull;
#pragma unroll
    for (int t = 0; t < TL_TOPW; ++t) {
      const uint32_t hv = __reduce_max_sync(0xffffffffu, (uint32_t)(k[0] >> 32));
      const bool eq = (uint32_t)(k[0] >> 32) == hv;
      const uint32_t lv = __reduce_max_sync(0xffffffffu, eq ? (uint32_t)k[0] : 0u);
      if (lane == t) mine = ((uint64_t)hv << 32) | lv;
      if (eq && (uint32_t)k[0] == lv && k[0] != 0ull) {
        k[0] = k[1];
        k[1] = k[2];
        k[2] = k[3];
        k[3] = 0ull;
      }
    }
    if (lane < TL_TOPW) {
      reinterpret_cast<uint64_t*>(cv)[warp * TL_TOPW + lane] = mine;
      reinterpret_cast<uint32_t*>(cv + TL_LISTV)[warp * TL_TOPW + lane] = (uint32_t)(mine >> 32);
    }
    if (tid == 0) {
      s_xkey = 0ull;
      s_maxkey = 0ull;
      s_flags2 = 0;
      s_c = 0;
    }
#pragma unroll
    for (int j = lane; j < TL_NB / TL_WARPS; j += 32) bins[warp * (TL_NB / TL_WARPS) + j] = 0u;
  }
  __syncwarp();
  __syncthreads();

  // ---- segment threshold over the warp buffers ------------------------------
  uint32_t state = 0u;
  if (!hist_ok) state |= FLAG_BAD_HISTORY;
  if (s_nonfinite) state |= FLAG_NONFINITE;
  if (s_overflow) state |= RSTATE_OVERFLOW;
  int m = 0;
  float kth = -INFINITY;  // the segment's K-th largest value

  // ---- exact K-th value over the warp buffers ---------------------------------
  // One linear histogram of the buffered values >= lo (the largest warp
  // threshold, a lower bound of the K-th value) over [lo, hi]; warp 0 finds
  // the bin b* holding the K-th value; one pass appends every value of the
  // bins above b* (all candidates) and collects bin b*; warp 0 ranks bin b*
  // and appends its values >= the K-th. Unusual inputs (no finite lower bound,
  // a crowded bin b*, too many candidates) take the general select below.
  bool done = false;
  // One-CTA rows: every warp published its 16 largest keys (sorted). Each key
  // gets its rank among all 256 by binary searches in the other lists; the
  // key of rank K-1 is x. No warp holds more than its list above x unless its
  // 16th key is >= x, so then every candidate (value >= x) is a list key and
  // its rank is its place in the sorted order: the candidates are scattered
  // to their places with their weights, and warp 0 finishes. Otherwise (a
  // full list, too many ties, too few keys) the selects below run.
  bool published = false;  // a split row's segment candidates already in scratch
  if (state == 0u) {
    const uint64_t* lists = reinterpret_cast<const uint64_t*>(cv);  // [TL_WARPS][TL_TOPW]
    const uint32_t* lval = reinterpret_cast<const uint32_t*>(cv + TL_LISTV);  // value keys
    uint64_t* sk = reinterpret_cast<uint64_t*>(cid);                // [64] keys by rank
    float* sw = reinterpret_cast<float*>(cid + 128);                // [64] weights by rank
    // lb: every warp holds >= kq+1 keys >= its (kq+1)-th key and
    // TL_WARPS*(kq+1) >= K, so the smallest of those is a lower bound of the
    // K-th value; keys below it need no rank
    const int kq = (K + TL_WARPS - 1) / TL_WARPS - 1;
    uint32_t lb = lval[(lane & (TL_WARPS - 1)) * TL_TOPW + kq];
#pragma unroll
    for (int o = TL_WARPS / 2; o > 0; o >>= 1) lb = min(lb, __shfl_xor_sync(0xffffffffu, lb, o));
    const int j = lane & (TL_TOPW - 1), half = lane >> 4;
    const uint64_t key = lists[warp * TL_TOPW + j];
    const uint32_t vk = (uint32_t)(key >> 32);
    int cnt = 0;
    if (key != 0ull && vk >= lb) {
      // values of each list greater than vk (a sorted prefix): the eight
      // searches are independent chains the scheduler interleaves; equal
      // values, which rank by id, are rare and counted afterwards
      constexpr int NL = TL_WARPS / 2;
      int pos[NL];
#pragma unroll
      for (int t = 0; t < NL; ++t) {
        const uint32_t* L = lval + (half * NL + t) * TL_TOPW;
        int p = 0;
#pragma unroll
        for (int step = TL_TOPW / 2; step > 0; step >>= 1)
          if (L[p + step - 1] > vk) p += step;
        p += L[p] > vk ? 1 : 0;
        pos[t] = p;
      }
      unsigned eq = 0u;
#pragma unroll
      for (int t = 0; t < NL; ++t) {
        const int l = half * NL + t;
        if (l == warp) continue;  // within its own list a key's rank is its place j
        cnt += pos[t];
        if (pos[t] < TL_TOPW && lval[l * TL_TOPW + pos[t]] == vk) eq |= 1u << t;
      }
      if (eq != 0u) {
#pragma unroll
        for (int t = 0; t < NL; ++t) {
          if (!(eq & (1u << t))) continue;
          const int l = half * NL + t;
          // equal values rank by id: count those with a larger full key
          for (int q = pos[t]; q < TL_TOPW && lval[l * TL_TOPW + q] == vk; ++q)
            cnt += lists[l * TL_TOPW + q] > key;
        }
      }
    }
    cnt += __shfl_xor_sync(0xffffffffu, cnt, 16);
    const int rank = j + cnt;
    if (half == 0 && key != 0ull && vk >= lb) {
      if (rank == K - 1) s_xkey = key;
      if (rank == 0) s_maxkey = key;
    }
    __syncthreads();
    const uint64_t x = s_xkey;
    const float vmax = cand_val(s_maxkey);
    if (x != 0ull && vmax > -INFINITY) {
      const uint32_t xv = (uint32_t)(x >> 32);
      if (lane == 0) {
        const uint64_t last = lists[warp * TL_TOPW + TL_TOPW - 1];
        if (last != 0ull && (uint32_t)(last >> 32) >= xv) atomicOr(&s_flags2, 1);  // full list
      }
      if (half == 0 && key != 0ull && vk >= lb && vk >= xv) {
        if (rank < 64) {
          bool slow = false;
          sk[rank] = key;
          sw[rank] = exp_cr(__fsub_rn(cand_val(key), vmax), slow);
          if (slow) atomicOr(&s_flags2, 4);
        } else {
          atomicOr(&s_flags2, 2);  // more than 64 candidates
        }
        atomicAdd(&s_c, 1);
      }
    }
    __syncthreads();
    if (x != 0ull && vmax > -INFINITY && (s_flags2 & 3) == 0 && S > 1) {
      // a split row: this segment's candidates (sorted) go to the row's scratch
      const int c = s_c;
      const int cta = row * S + split;
      for (int i = tid; i < c; i += TL_THREADS) {
        a.s.cand_v[(size_t)cta * TK_CAPB + i] = cand_val(sk[i]);
        a.s.cand_id[(size_t)cta * TK_CAPB + i] = cand_id(sk[i]);
      }
      m = c;
      kth = cand_val(x);
      done = true;
      published = true;
    } else if (x != 0ull && vmax > -INFINITY && (s_flags2 & 3) == 0) {
      if (warp == 0) {
        const int c = s_c;
        const uint64_t k0 = lane < c ? sk[lane] : 0ull;
        const uint64_t k1 = lane + 32 < c ? sk[lane + 32] : 0ull;
        if constexpr (kShard) {
          uint32_t* rec = a.shard_out + (size_t)row * VS_REC_WORDS;
          float* rv = vs_values(rec);
          int32_t* ri = vs_ids(rec);
          if (lane < c) {
            rv[lane] = cand_val(k0);
            ri[lane] = cand_id(k0);
          }
          if (lane + 32 < c) {
            rv[lane + 32] = cand_val(k1);
            ri[lane + 32] = cand_id(k1);
          }
          if (lane == 0) {
            rec[0] = (uint32_t)c;
            rec[1] = 0u;
            rec[2] = __float_as_uint(cand_val(x));
            rec[3] = (uint32_t)c;
          }
        } else {
          finish_weights_warp(a, row, k0, k1, c, sw, reinterpret_cast<float*>(work),
                              (s_flags2 & 4) != 0, s_u);
        }
      }
      return;
    }
  }
  if (state == 0u && !done) {
    float lo = s_wtheta[lane & (TL_WARPS - 1)], hi = s_wmax[lane & (TL_WARPS - 1)];
#pragma unroll
    for (int o = TL_WARPS / 2; o > 0; o >>= 1) {
      lo = fmaxf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lo > -INFINITY && hi > lo) {
      const float sc = __fdiv_rn((float)TL_NB, __fsub_rn(hi, lo));
      auto bin_of = [&](float x) {
        const int b = (int)__fmul_rn(__fsub_rn(hi, x), sc);  // larger x -> smaller bin
        return b < TL_NB - 1 ? b : TL_NB - 1;
      };
      float fv[TW_WCAP / 32];
      bool fok[TW_WCAP / 32];
#pragma unroll
      for (int r = 0; r < TW_WCAP / 32; ++r) {
        const int i = tid + r * TL_THREADS;  // flattened [W][WCAP]
        const int w = i / TW_WCAP, e = i % TW_WCAP;
        fv[r] = e < s_wn[w] ? wvall[i] : -INFINITY;
        fok[r] = fv[r] >= lo;
        if (fok[r]) atomicAdd(&bins[bin_of(fv[r])], 1u);
      }
      if (tid == 0) {
        s_count = 0;
        s_ovf = 0;
        s_nbin = 0;
        s_bstar = -1;
        s_mode = 0;
      }
      __syncthreads();
      if (warp == 0) {
        // lane l owns bins [32l, 32l+32): totals, scan, then the crossing lane
        constexpr int PER = TL_NB / 32;
        int c = 0;
#pragma unroll 8
        for (int j = 0; j < PER; ++j) c += (int)bins[lane * PER + j];
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const int excl = incl - c;
        if (excl < K && K <= incl) {
          int run = excl, j = 0;
          for (; j < PER; ++j) {
            const int cb = (int)bins[lane * PER + j];
            if (run + cb >= K) break;
            run += cb;
          }
          s_bstar = lane * PER + j;
          s_above = run;
        }
      }
      __syncthreads();
      const int bstar = s_bstar;
      if (bstar >= 0) {
        float* binv = reinterpret_cast<float*>(cid + TL_GCAP);  // [TL_BINCAP]
        int* bini = cid + TL_GCAP + TL_BINCAP;                   // [TL_BINCAP]
#pragma unroll
        for (int r = 0; r < TW_WCAP / 32; ++r) {
          const int i = tid + r * TL_THREADS;
          const int b = fok[r] ? bin_of(fv[r]) : TL_NB;
          const bool above = b < bstar;
          warp_append(above, fv[r], above ? wiall[i] : 0, cv, cid, &s_count, &s_ovf, TL_GCAP);
          if (b == bstar) {
            const int slot = atomicAdd(&s_nbin, 1);
            if (slot < TL_BINCAP) {
              binv[slot] = fv[r];
              bini[slot] = wiall[i];
            }
          }
        }
        __syncthreads();
        if (warp == 0) {
          const int nb = s_nbin;
          const int rk = K - s_above;  // rank of the K-th value inside bin b* (1-based)
          if (nb <= TL_BINCAP && !s_ovf) {
            // the K-th value: the bin entry x with #(> x) < rk <= #(>= x)
            float T = -INFINITY;
            for (int j0 = 0; j0 < nb; j0 += 32) {
              const int j = j0 + lane;
              const float x = j < nb ? binv[j] : -INFINITY;
              int gt = 0, ge = 0;
              for (int t = 0; t < nb; ++t) {
                const float y = binv[t];
                gt += y > x;
                ge += y >= x;
              }
              const bool hit = j < nb && gt < rk && rk <= ge;
              const unsigned hb = __ballot_sync(0xffffffffu, hit);
              if (hb) T = __shfl_sync(0xffffffffu, x, __ffs(hb) - 1);
            }
            // bin b* values >= T join the candidates
            for (int j0 = 0; j0 < nb; j0 += 32) {
              const int j = j0 + lane;
              const bool ok = j < nb && binv[j] >= T;
              warp_append(ok, ok ? binv[j] : 0.f, ok ? bini[j] : 0, cv, cid, &s_count, &s_ovf,
                          TL_GCAP);
            }
            __syncwarp();
            const int mm = s_count;
            if (!s_ovf) {
              if (!kShard && S == 1 && mm <= 64) {
                finish_row_warp(a, row, cv, cid, mm, reinterpret_cast<float*>(work), false, s_u);
                if (lane == 0) s_mode = 2;  // finished
              } else if (lane == 0) {
                s_mode = 1;  // candidates ready
                s_kth = T;
              }
            }
          }
        }
        __syncthreads();
        if (s_mode == 2) return;
        if (s_mode == 1) {
          done = true;
          kth = s_kth;
          m = s_count;
        }
      }
    }
  }

  if (state == 0u && !done) {
    // exact K-th largest over the warp buffers (finite values; -inf entries
    // are below any finite K-th value and are all kept when it is -inf)
    float fv[TW_WCAP / 32];
    bool fok[TW_WCAP / 32];
    bool inb[TW_WCAP / 32];
#pragma unroll
    for (int r = 0; r < TW_WCAP / 32; ++r) {
      const int i = tid + r * TL_THREADS;  // flattened [W][WCAP]
      const int w = i / TW_WCAP, e = i % TW_WCAP;
      inb[r] = e < s_wn[w];
      fv[r] = inb[r] ? wvall[i] : -INFINITY;
      fok[r] = inb[r] && fv[r] > -INFINITY;
    }
    const float T = cta_select_linear(fv, fok, K, true, work, hist, s_sh);
    kth = T;
    if (tid == 0) {
      s_count = 0;
      s_ovf = 0;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < TW_WCAP / 32; ++r) {
      const int i = tid + r * TL_THREADS;
      const bool ok = inb[r] && fv[r] >= T;
      warp_append(ok, ok ? fv[r] : 0.f, ok ? wiall[i] : 0, cv, cid, &s_count, &s_ovf);
    }
    __syncthreads();
    m = min(s_count, TK_CAPB);
    if (s_ovf) state |= RSTATE_OVERFLOW;
  }

  if (S == 1) {
    if constexpr (kShard) {
      write_topk_record(a.shard_out + (size_t)row * VS_REC_WORDS, cv, cid, m, state, kth);
      return;
    }
    if (state == 0u && m > 0 && m <= 64) {
      if (warp == 0) finish_row_warp(a, row, cv, cid, m, reinterpret_cast<float*>(work));
    } else {
      finish_row(a, row, cv, cid, m, state, work);
    }
    return;
  }

  // ---- multi-CTA rows: publish, the last CTA merges --------------------------
  const int cta = row * S + split;
  if (!published)
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
    *owner = s_last;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* uv = reinterpret_cast<float*>(work);            // union: [0, 8 KiB)
  int* uid = reinterpret_cast<int*>(uv + TK_CAPB);        //        [8, 16 KiB)
  // the segments' candidate counts, one thread per segment, then offsets
  constexpr int MAX_SEG = 64;
  __shared__ int s_segoff[MAX_SEG + 1];
  const bool flat = S <= MAX_SEG;
  if (flat && tid < S) s_segoff[tid + 1] = __ldcg(&a.s.cand_n[row * S + tid]);
  if (tid == 0) s_state = __ldcg(&a.s.rowstate[row]);
  __syncthreads();
  if (tid == 0) {
    int tot = 0;
    if (flat) {
      s_segoff[0] = 0;
      for (int sp = 0; sp < S; ++sp) s_segoff[sp + 1] = (tot += s_segoff[sp + 1]);
    } else {
      for (int sp = 0; sp < S; ++sp) tot += __ldcg(&a.s.cand_n[row * S + sp]);
    }
    s_tot = tot;
  }
  __syncthreads();
  uint32_t mstate = s_state;
  const int total = s_tot;
  if (total > TK_CAPB) mstate |= RSTATE_OVERFLOW;
  int mm = 0;
  float mkth = -INFINITY;
  if (mstate == 0u) {
    if (flat) {
      // every segment's candidates in one flat pass (loads in flight together)
      for (int j = tid; j < total; j += TL_THREADS) {
        int lo = 0, hi = S - 1;  // the segment sp with s_segoff[sp] <= j < s_segoff[sp + 1]
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_segoff[mid] <= j) lo = mid;
          else hi = mid - 1;
        }
        const size_t g = (size_t)(row * S + lo) * TK_CAPB + (j - s_segoff[lo]);
        uv[j] = __ldcg(&a.s.cand_v[g]);
        uid[j] = __ldcg(&a.s.cand_id[g]);
      }
    } else {
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
    }
    __syncthreads();
    if (total <= RS_MAX) {
      // direct ranks over the union: sorted candidates and their weights
      uint64_t* sk = reinterpret_cast<uint64_t*>(work + 16384);  // [64]
      float* sw = reinterpret_cast<float*>(work + 16384 + 512);  // [64]
      float* s64 = sw + 64;                                      // [64]
      const RankSel rs = cta_rank_select(uv, uid, total, K, reinterpret_cast<uint64_t*>(cv), sk, sw);
      if (rs.ok) {
        if (warp == 0) {
          const uint64_t k0 = lane < rs.c ? sk[lane] : 0ull;
          const uint64_t k1 = lane + 32 < rs.c ? sk[lane + 32] : 0ull;
          if constexpr (kShard) {
            uint32_t* rec = a.shard_out + (size_t)row * VS_REC_WORDS;
            if (lane < rs.c) {
              vs_values(rec)[lane] = cand_val(k0);
              vs_ids(rec)[lane] = cand_id(k0);
            }
            if (lane + 32 < rs.c) {
              vs_values(rec)[lane + 32] = cand_val(k1);
              vs_ids(rec)[lane + 32] = cand_id(k1);
            }
            if (lane == 0) {
              rec[0] = (uint32_t)rs.c;
              rec[1] = 0u;
              rec[2] = __float_as_uint(total < K ? -INFINITY : cand_val(rs.x));
              rec[3] = (uint32_t)rs.c;
            }
          } else {
            finish_weights_warp(a, row, k0, k1, rs.c, sw, s64, rs.slow, a.uniforms[row]);
          }
        }
        __syncthreads();
        if (tid == 0) {
          a.s.rowstate[row] = 0u;
          a.s.tickets[row] = 0u;
        }
        return;
      }
    }
    const uint32_t key = cta_kth_largest([&](int i) { return fkey(uv[i]); }, total, K, hist, s_sh);
    mkth = key <= fkey(-INFINITY) ? -INFINITY : kval(key);
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
  if constexpr (kShard) {
    write_topk_record(a.shard_out + (size_t)row * VS_REC_WORDS, cv, cid, mm, mstate, mkth);
  } else if (mstate == 0u && mm > 0 && mm <= 64) {
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
