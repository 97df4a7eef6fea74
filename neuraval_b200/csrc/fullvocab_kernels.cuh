// Full-vocabulary sampling path (sm_100a): top_k >= V (the reference's "no
// top-k", GenerationOptions.cs:79) and top-k values above the top-k kernel's
// limit.
//
// The reference (TokenSampler.cs:67-132) keeps every value >= the K-th largest,
// sorts all candidates descending, and sums exp(v_i - max) sequentially in
// fp32 -- for K >= V that is a 150k-long dependent chain whose rounding the
// token depends on. This path reproduces those sums bit for bit:
//
//  1. pass 1 over the row: penalised/scaled values, their maximum;
//  2. pass 2: histogram of x = v - max over NB linear bins on [-17, 0]; values
//     below -17 have exp(x) < 2^-24 and, since the running sum is >= 1 after
//     the first (maximum) element, can never change it nor be drawn;
//  3. pass 3: scatter (value, id) keys into bin order in global scratch;
//  4. walk the bins in order in groups of <= FV_GCAP keys: sort each group in
//     shared memory, compute the weights, and run an exact parallel scan of
//     the sequential fp32 sum: while the running sum S stays in one binade
//     [2^e, 2^(e+1)) every fl(S + w) equals S + round(w / 2^(e-23)) on the
//     2^(e-23) grid, i.e. an integer addition, except that a weight exactly
//     halfway between grid points rounds to even and so depends on the parity
//     of S. Each element is a 2-state transducer (parity in -> increment,
//     parity out); transducers compose associatively, so a block scan gives
//     every prefix sum. The first element whose sum leaves the binade is added
//     with a plain __fadd_rn and the scan restarts in the next binade;
//  5. binary searches over the stored sums give the top-p cutoff and the draw.
#pragma once

#include "sampler_device.cuh"
#include "topk_kernels.cuh"

namespace nvs {

constexpr int FV_THREADS = 1024;
constexpr int FV_NB = 4096;          // value bins over x in [-17, 0]
constexpr int FV_GCAP = 4096;        // keys per group sorted in shared memory
constexpr float FV_XMIN = -17.0f;    // exp(-17) < 2^-24
constexpr int FV_FIXUP_MAX_LIST = 1024;

struct FvLayout {
  size_t comp_bytes, sum_bytes, total_bytes;
  int max_rows, max_vocab;
};
struct FvScratch {
  uint64_t* comp;  // [max_rows * max_vocab]: ~key(v) << 32 | id, bin order then sorted
  float* ssum;     // [max_rows * max_vocab]: sequential sums at sorted positions
  int max_vocab;
};

inline FvLayout fv_layout(int max_rows, int max_vocab) {
  FvLayout l;
  l.max_rows = max_rows;
  l.max_vocab = max_vocab;
  l.comp_bytes = (size_t)max_rows * max_vocab * sizeof(uint64_t);
  l.sum_bytes = (size_t)max_rows * max_vocab * sizeof(float);
  l.total_bytes = l.comp_bytes + 256 + l.sum_bytes;
  return l;
}
inline FvScratch fv_carve(char* base, const FvLayout& l) {
  FvScratch f;
  f.comp = reinterpret_cast<uint64_t*>(base);
  f.ssum = reinterpret_cast<float*>(base + (l.comp_bytes + 255) / 256 * 256);
  f.max_vocab = l.max_vocab;
  return f;
}

// ascending composite: larger value first, then smaller id
__device__ __forceinline__ uint64_t fv_comp(float v, int id) {
  return ((uint64_t)(~fkey(v)) << 32) | (uint32_t)id;
}
__device__ __forceinline__ float fv_val(uint64_t c) { return kval(~(uint32_t)(c >> 32)); }
__device__ __forceinline__ int fv_id(uint64_t c) { return (int)(uint32_t)(c & 0xFFFFFFFFu); }

__device__ __forceinline__ int fv_bin(float x) {
  int b = (int)__fmul_rn(-x, (float)FV_NB / 17.0f);
  return b < FV_NB - 1 ? b : FV_NB - 1;
}

// Sort a[0..n) ascending (any n): bitonic network written so every compare-
// exchange puts the smaller key at the lower index; positions >= n act as +inf
// and are never touched. Works on shared or (CTA-private) global memory.
__device__ void cta_sort_any_n(uint64_t* a, int n) {
  if (n <= 1) return;
  const int np = next_pow2(n);
  for (int k = 2; k <= np; k <<= 1) {
    // flip stage
    for (int i = threadIdx.x; i < np / 2; i += blockDim.x) {
      const int blk = i / (k / 2), off = i % (k / 2);
      const int lo = blk * k + off;
      const int hi = blk * k + k - 1 - off;
      if (hi < n) {
        uint64_t x = a[lo], y = a[hi];
        if (x > y) { a[lo] = y; a[hi] = x; }
      }
    }
    __syncthreads();
    for (int j = k >> 2; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < np / 2; i += blockDim.x) {
        const int blk = i / j, off = i % j;
        const int lo = blk * 2 * j + off;
        const int hi = lo + j;
        if (hi < n) {
          uint64_t x = a[lo], y = a[hi];
          if (x > y) { a[lo] = y; a[hi] = x; }
        }
      }
      __syncthreads();
    }
  }
}

// Parity transducer of one fp32 addition on a fixed grid: for the parity p of
// S (in grid units) the addition adds inc[p] grid units and leaves parity par[p].
struct Tdu {
  int inc0, inc1;
  int par;  // bit0: parity out for p=0, bit1: parity out for p=1
};
__device__ __forceinline__ Tdu tdu_identity() { return {0, 0, 0b10}; }
__device__ __forceinline__ int sat25(int x) { return x < (1 << 25) ? x : (1 << 25); }
// first A, then B
__device__ __forceinline__ Tdu tdu_compose(Tdu A, Tdu B) {
  const int pa0 = A.par & 1, pa1 = (A.par >> 1) & 1;
  Tdu r;
  r.inc0 = sat25(A.inc0 + (pa0 ? B.inc1 : B.inc0));
  r.inc1 = sat25(A.inc1 + (pa1 ? B.inc1 : B.inc0));
  const int pb0 = B.par & 1, pb1 = (B.par >> 1) & 1;
  r.par = (pa0 ? pb1 : pb0) | ((pa1 ? pb1 : pb0) << 1);
  return r;
}
__device__ __forceinline__ Tdu tdu_shfl_up(Tdu t, int d) {
  Tdu r;
  r.inc0 = __shfl_up_sync(0xffffffffu, t.inc0, d);
  r.inc1 = __shfl_up_sync(0xffffffffu, t.inc1, d);
  r.par = __shfl_up_sync(0xffffffffu, t.par, d);
  return r;
}

// Weight w on the grid 2^g (g = exponent(S) - 23): transducer of fl(S + w).
__device__ __forceinline__ Tdu tdu_of(float w, float inv_grid) {
  const float x = __fmul_rn(w, inv_grid);  // exact (power-of-two scale, x < 2^24)
  const float m = floorf(x);
  const float frac = __fsub_rn(x, m);    // exact
  const int mi = (int)m;
  Tdu t;
  if (frac == 0.5f) {
    // round half to even: result S+m or S+m+1, whichever is even
    const int odd0 = mi & 1;           // parity of S+m when S is even
    t.inc0 = odd0 ? mi + 1 : mi;
    t.inc1 = odd0 ? mi : mi + 1;
    t.par = 0;
  } else {
    const int q = mi + (frac > 0.5f ? 1 : 0);
    t.inc0 = q;
    t.inc1 = q;
    t.par = (q & 1) ? 0b01 : 0b10;
  }
  return t;
}

// Exact sequential fp32 sum over w[0..n) (shared memory) starting from S_in
// (0 or an exact earlier sum, a normal float), writing every prefix to sout[0..n).
// All FV_THREADS threads call. Returns the final sum.
__device__ float exact_prefix_sums(const float* w, int n, float S_in, float* sout, Tdu* s_warp,
                                   int* s_cross) {
  __shared__ float s_S;
  __shared__ int s_pos;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    s_S = S_in;
    s_pos = 0;
    if (S_in == 0.0f && n > 0) {
      sout[0] = w[0];  // fl(0 + w) = w
      s_S = w[0];
      s_pos = 1;
    }
  }
  __syncthreads();
  for (;;) {
    const int pos = s_pos;
    const float S = s_S;
    if (pos >= n) break;
    const uint32_t sb = __float_as_uint(S);
    const int e = (int)((sb >> 23) & 0xFF) - 127;  // S is a normal float
    const int g = e - 23;
    const float inv_grid = __int_as_float((127 - g) << 23);
    const float grid = __int_as_float((127 + g) << 23);
    const int M = (int)((sb & 0x7FFFFFu) | 0x800000u);  // S / grid
    constexpr int PER = FV_GCAP / FV_THREADS;
    const int first = pos + tid * PER;
    Tdu t = tdu_identity();
    Tdu el[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = first + j;
      el[j] = i < n ? tdu_of(w[i], inv_grid) : tdu_identity();
      t = tdu_compose(t, el[j]);
    }
    // block exclusive scan of t
    Tdu inc = t;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      Tdu o = tdu_shfl_up(inc, d);
      if (lane >= d) inc = tdu_compose(o, inc);
    }
    Tdu ex = tdu_shfl_up(inc, 1);
    if (lane == 0) ex = tdu_identity();
    if (lane == 31) s_warp[warp] = inc;
    if (tid == 0) *s_cross = 0x7FFFFFFF;
    __syncthreads();
    if (warp == 0) {
      Tdu wv = lane < (FV_THREADS / 32) ? s_warp[lane] : tdu_identity();
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        Tdu o = tdu_shfl_up(wv, d);
        if (lane >= d) wv = tdu_compose(o, wv);
      }
      Tdu wex = tdu_shfl_up(wv, 1);
      if (lane == 0) wex = tdu_identity();
      __syncwarp();
      s_warp[lane] = wex;
    }
    __syncthreads();
    const Tdu pre = tdu_compose(s_warp[warp], ex);
    const int p0 = M & 1;
    int D = p0 ? pre.inc1 : pre.inc0;
    int p = p0 ? ((pre.par >> 1) & 1) : (pre.par & 1);
    int mycross = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = first + j;
      if (i < n && mycross == 0x7FFFFFFF) {
        D = sat25(D + (p ? el[j].inc1 : el[j].inc0));
        p = p ? ((el[j].par >> 1) & 1) : (el[j].par & 1);
        const int cum = M + D;
        if (cum >= (1 << 24)) mycross = i;
        else sout[i] = __fmul_rn((float)cum, grid);
      }
    }
    if (mycross != 0x7FFFFFFF) atomicMin(s_cross, mycross);
    __syncthreads();
    const int c = *s_cross;
    if (tid == 0) {
      if (c != 0x7FFFFFFF) {
        const float prev = (c == pos) ? S : sout[c - 1];
        const float sc = __fadd_rn(prev, w[c]);
        sout[c] = sc;
        s_S = sc;
        s_pos = c + 1;
      } else {
        const int last = min(n, pos + FV_GCAP) - 1;
        s_S = sout[last];
        s_pos = last + 1;
      }
    }
    __syncthreads();
  }
  return s_S;
}

template <bool kCounts>
__device__ void fullvocab_row(const SampleArgs& a, const FvScratch& f, int K, int row,
                              unsigned char* smem) {
  uint64_t* gkeys = reinterpret_cast<uint64_t*>(smem);                  // [GCAP]
  float* gw = reinterpret_cast<float*>(gkeys + FV_GCAP);                // [GCAP]
  float* gs = gw + FV_GCAP;                                             // [GCAP]
  int* binoff = reinterpret_cast<int*>(gs + FV_GCAP);                   // [NB+1]
  int* cursor = binoff + FV_NB + 1;                                     // [NB]
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(cursor + FV_NB);
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);

  __shared__ float s_red[FV_THREADS / 32];
  __shared__ int s_ired[FV_THREADS / 32];
  __shared__ Tdu s_warp[32];
  __shared__ int s_cross, s_hn, s_nonfinite, s_ncand, s_stop;
  __shared__ float s_vmax, s_S;
  __shared__ uint32_t s_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.V;
  const float* lrow = a.logits + (size_t)row * V;
  uint64_t* comp = f.comp + (size_t)row * f.max_vocab;
  float* ssum = f.ssum + (size_t)row * f.max_vocab;
  const float scale = __fdiv_rn(1.0f, a.p.temperature);

  Penalty P;
  const bool hist_ok = setup_penalty<kCounts>(P, a, row, 0, V, bitmap, hsorted, &s_hn);
  if (tid == 0) {
    s_nonfinite = 0;
    s_flag = 0u;
  }
  if (a.probs) {
    float* prow = a.probs + (size_t)row * V;
    for (int c = tid; c < V; c += FV_THREADS) prow[c] = 0.0f;
  }
  __syncthreads();
  if (!hist_ok) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_BAD_HISTORY;
    }
    return;
  }

  auto value = [&](int c) -> float { return canon(__fmul_rn(adjust(P, __ldcs(lrow + c), c), scale)); };

  // 1. maximum
  float vmax = -INFINITY;
  bool nf = false;
  for (int c = tid; c < V; c += FV_THREADS) {
    const float v = value(c);
    if (v != v || v == INFINITY) nf = true;
    else vmax = fmaxf(vmax, v);
  }
  if (nf) s_nonfinite = 1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
  if (lane == 0) s_red[warp] = vmax;
  for (int i = tid; i < FV_NB; i += FV_THREADS) cursor[i] = 0;
  __syncthreads();
  if (warp == 0) {
    float m = lane < FV_THREADS / 32 ? s_red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_vmax = m;
  }
  __syncthreads();
  vmax = s_vmax;
  if (s_nonfinite || !(vmax > -INFINITY)) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_NONFINITE;
    }
    return;
  }

  // 2. histogram of relevant values (x >= -17)
  for (int c = tid; c < V; c += FV_THREADS) {
    const float x = __fsub_rn(value(c), vmax);
    if (x >= FV_XMIN) atomicAdd(&cursor[fv_bin(x)], 1);
  }
  __syncthreads();
  // exclusive scan of the NB counts -> binoff (4 per thread)
  {
    constexpr int PER = FV_NB / FV_THREADS;
    int loc[PER];
    int sum = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      loc[j] = cursor[tid * PER + j];
      sum += loc[j];
    }
    int inc = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      int o = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += o;
    }
    if (lane == 31) s_ired[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      int wv = lane < FV_THREADS / 32 ? s_ired[lane] : 0;
      int wi = wv;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        int o = __shfl_up_sync(0xffffffffu, wi, d);
        if (lane >= d) wi += o;
      }
      __syncwarp();
      if (lane < FV_THREADS / 32) s_ired[lane] = wi - wv;
    }
    __syncthreads();
    int run = s_ired[warp] + inc - sum;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      binoff[tid * PER + j] = run;
      cursor[tid * PER + j] = run;
      run += loc[j];
    }
    if (tid == FV_THREADS - 1) binoff[FV_NB] = run;
  }
  __syncthreads();
  const int nrel = binoff[FV_NB];

  // 3. scatter keys into bin order
  for (int c = tid; c < V; c += FV_THREADS) {
    const float v = value(c);
    const float x = __fsub_rn(v, vmax);
    if (x >= FV_XMIN) {
      const int pos = atomicAdd(&cursor[fv_bin(x)], 1);
      comp[pos] = fv_comp(v, c);
    }
  }
  __syncthreads();

  // 4. walk groups of bins in order
  // candidates: every value >= the K-th largest; with K <= nrel the candidate
  // count is K plus the ties of the K-th value (found in its group).
  if (tid == 0) {
    s_ncand = (K < nrel) ? -1 : nrel;  // -1: not known yet
    s_S = 0.0f;
    s_stop = 0;
  }
  __syncthreads();
  int b = 0;
  int pos0 = 0;  // sorted position of the group's first key
  bool slow_any = false;
  while (b < FV_NB && pos0 < nrel) {
    // group = bins [b, b2) with <= GCAP keys, or one oversized bin
    int b2 = b;
    while (b2 < FV_NB && binoff[b2 + 1] - pos0 <= FV_GCAP) ++b2;
    const bool big = (b2 == b);
    int gn;
    if (big) {
      // one bin larger than a group: sort it in place in global scratch
      const int bn = binoff[b + 1] - binoff[b];
      cta_sort_any_n(comp + pos0, bn);
      __threadfence_block();
      __syncthreads();
      gn = bn;
    } else {
      gn = binoff[b2] - pos0;
    }
    // process [pos0, pos0+gn) in slices of GCAP
    for (int s0 = 0; s0 < gn; s0 += FV_GCAP) {
      const int sn = min(FV_GCAP, gn - s0);
      for (int i = tid; i < sn; i += FV_THREADS) gkeys[i] = comp[pos0 + s0 + i];
      __syncthreads();
      if (!big) cta_sort_any_n(gkeys, sn);
      // candidate limit
      if (tid == 0 && s_ncand < 0) {
        const int kpos = K - 1 - (pos0 + s0);
        if (kpos >= 0 && kpos < sn) {
          // equal values share a bin; an oversized bin is already sorted in
          // place in `comp`, so its ties may continue past this slice
          const uint32_t kk = (uint32_t)(gkeys[kpos] >> 32);
          int e = pos0 + s0 + kpos;
          const int gend = pos0 + gn;
          if (big) {
            while (e + 1 < gend && (uint32_t)(comp[e + 1] >> 32) == kk) ++e;
          } else {
            while (e + 1 < gend && (uint32_t)(gkeys[e + 1 - pos0] >> 32) == kk) ++e;
          }
          s_ncand = e + 1;
        }
      }
      __syncthreads();
      const int lim = s_ncand < 0 ? sn : min(sn, s_ncand - (pos0 + s0));
      bool slow = false;
      for (int i = tid; i < lim; i += FV_THREADS)
        gw[i] = exp_cr(__fsub_rn(fv_val(gkeys[i]), vmax), slow);
      slow_any |= slow;
      __syncthreads();
      const float Sn = exact_prefix_sums(gw, lim, s_S, gs, s_warp, &s_cross);
      for (int i = tid; i < lim; i += FV_THREADS) {
        comp[pos0 + s0 + i] = gkeys[i];
        ssum[pos0 + s0 + i] = gs[i];
      }
      __syncthreads();
      if (tid == 0) {
        s_S = Sn;
        if (lim < sn || (s_ncand >= 0 && pos0 + s0 + lim >= s_ncand)) s_stop = 1;
      }
      __syncthreads();
      if (s_stop) break;
    }
    if (s_stop) break;
    pos0 += gn;
    b = big ? b + 1 : b2;
  }
  if (slow_any) atomicOr(&s_flag, FLAG_EXP_SLOW);
  __syncthreads();
  const int n = s_ncand < 0 ? nrel : min(s_ncand, nrel);

  // 5. cutoff and draw (TokenSampler.cs:105-132) by binary search on the sums
  __shared__ int s_cut;
  __shared__ float s_ret;
  if (tid == 0) {
    const float total = ssum[n - 1];
    int cutoff = n;
    float target = 0.0f;
    auto first_ge = [&](float t, int hi) {
      int lo = 0;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (ssum[mid] >= t) hi = mid; else lo = mid + 1;
      }
      return lo;
    };
    if (a.p.top_p < 1.0f) {
      target = __fmul_rn(total, a.p.top_p);
      cutoff = first_ge(target, n) + 1;
      if (cutoff > n) cutoff = n;
    }
    const float retained = ssum[cutoff - 1];
    const float sample = __fmul_rn(a.uniforms[row], retained);
    int sel = first_ge(sample, cutoff - 1);
    uint32_t fl = s_flag;
    const double tol = 1e-6 * (double)retained;
    if (fabs((double)sample - (double)ssum[sel]) <= tol ||
        (sel >= 1 && fabs((double)sample - (double)ssum[sel - 1]) <= tol))
      fl |= FLAG_DRAW_BOUNDARY;
    if (a.p.top_p < 1.0f) {
      const double tt = 1e-6 * (double)target;
      if (fabs((double)ssum[cutoff - 1] - (double)target) <= tt ||
          (cutoff >= 2 && fabs((double)ssum[cutoff - 2] - (double)target) <= tt))
        fl |= FLAG_CUTOFF_BOUNDARY;
    }
    const uint32_t ks = (uint32_t)(comp[sel] >> 32);
    if ((sel > 0 && (uint32_t)(comp[sel - 1] >> 32) == ks) ||
        (sel + 1 < n && (uint32_t)(comp[sel + 1] >> 32) == ks))
      fl |= FLAG_TIE_AT_DRAW;
    a.tokens[row] = fv_id(comp[sel]);
    if (a.flags) a.flags[row] = fl;
    s_cut = cutoff;
    s_ret = retained;
  }
  __syncthreads();
  if (a.probs) {
    float* prow = a.probs + (size_t)row * V;
    const int cut = s_cut;
    const float ret = s_ret;
    for (int i = tid; i < cut; i += FV_THREADS) {
      const uint64_t c = comp[i];
      bool slow = false;
      const float w = exp_cr(__fsub_rn(fv_val(c), vmax), slow);
      prow[fv_id(c)] = __fdiv_rn(w, ret);
    }
    // With top_p == 1 every candidate is retained, including those whose
    // weight is too small to change the sum (x < -17): they still get w/retained.
    if (!(a.p.top_p < 1.0f) && K > nrel) {
      __shared__ uint32_t s_hist[256];
      __shared__ int s_sh[2];
      uint32_t thr = 0u;
      if (K < V) {
        thr = cta_kth_largest(
            [&](int c) {
              const float v = value(c);
              return __fsub_rn(v, vmax) < FV_XMIN ? fkey(v) : 0u;
            },
            V, K - nrel, s_hist, s_sh);
      }
      for (int c = tid; c < V; c += FV_THREADS) {
        const float v = value(c);
        const float x = __fsub_rn(v, vmax);
        if (x < FV_XMIN && fkey(v) >= thr) {
          bool slow = false;
          prow[c] = __fdiv_rn(exp_cr(x, slow), ret);
        }
      }
    }
  }
  __syncthreads();
}

// One CTA per row.
template <bool kCounts>
__global__ void __launch_bounds__(FV_THREADS, 1) fullvocab_kernel(const __grid_constant__ SampleArgs a, FvScratch f, int K) {
  extern __shared__ __align__(128) unsigned char smem[];
  fullvocab_row<kCounts>(a, f, K, blockIdx.x, smem);
}

// Fix-up after the top-k kernel: CTAs stride over the rows and redo, on this
// path, every row the top-k kernel marked (ties at the k-th value overflowing
// its candidate buffers). Unmarked rows cost one load.
template <bool kCounts>
__global__ void __launch_bounds__(FV_THREADS, 1) fullvocab_fixup_kernel(const __grid_constant__ SampleArgs a, FvScratch f,
                                                                        int K, int rows) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_list[FV_FIXUP_MAX_LIST];
  __shared__ int s_n;
  // the next launch on the stream may be scheduled now; it waits for this
  // grid's completion before it reads anything
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // launched as a programmatic dependent of the top-k kernel: it may start
  // while that kernel drains, and waits here until its writes are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // one parallel pass collects the marked rows (no dependent loads per row)
  for (int base = 0; base < rows; base += FV_FIXUP_MAX_LIST) {
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    for (int r = base + threadIdx.x; r < min(rows, base + FV_FIXUP_MAX_LIST); r += blockDim.x)
      if (a.s.fixup[r] != 0u && (r % gridDim.x) == blockIdx.x) s_list[atomicAdd(&s_n, 1)] = r;
    __syncthreads();
    const int n = s_n;
    for (int i = 0; i < n; ++i) {
      const int row = s_list[i];
      fullvocab_row<kCounts>(a, f, K, row, smem);
      if (threadIdx.x == 0) {
        a.s.fixup[row] = 0u;
        if (a.s.stats) atomicAdd(a.s.stats, 1u);
      }
      __syncthreads();
    }
  }
}

// Exclusive scan of FV_NB counts in cnt[] -> off[0..NB] and cursor copy
// (FV_THREADS threads, 4 bins each).
__device__ void fv_scan_bins(int* cnt, int* off, int* s_ired) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int PER = FV_NB / FV_THREADS;
  int loc[PER];
  int sum = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    loc[j] = cnt[tid * PER + j];
    sum += loc[j];
  }
  int inc = sum;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    int o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += o;
  }
  if (lane == 31) s_ired[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int wv = lane < FV_THREADS / 32 ? s_ired[lane] : 0;
    int wi = wv;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      int o = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= d) wi += o;
    }
    __syncwarp();
    if (lane < FV_THREADS / 32) s_ired[lane] = wi - wv;
  }
  __syncthreads();
  int run = s_ired[warp] + inc - sum;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    off[tid * PER + j] = run;
    cnt[tid * PER + j] = run;
    run += loc[j];
  }
  if (tid == FV_THREADS - 1) off[FV_NB] = run;
  __syncthreads();
}

// FilterTopP on probabilities (LogitsProcessor.cs:75-114), one CTA per row:
// descending order (equal probabilities by ascending id), cutoff = first
// position whose sequential fp32 sum is >= top_p, kept entries divided by the
// retained sum, the rest set to 0. Probabilities below 2^(e0-24), e0 the
// exponent of the largest one, cannot change the running sum and are only
// renormalised (when the cutoff is never reached). Rows whose largest
// probability is below 2^-100 (or not finite) are left unchanged and flagged.
__global__ void __launch_bounds__(FV_THREADS, 1)
    filter_top_p_kernel(float* probs, int V, float top_p, uint32_t* flags, FvScratch f) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* gkeys = reinterpret_cast<uint64_t*>(smem);
  float* gw = reinterpret_cast<float*>(gkeys + FV_GCAP);
  float* gs = gw + FV_GCAP;
  int* binoff = reinterpret_cast<int*>(gs + FV_GCAP);
  int* cursor = binoff + FV_NB + 1;
  __shared__ float s_red[FV_THREADS / 32];
  __shared__ int s_ired[FV_THREADS / 32];
  __shared__ Tdu s_warp[32];
  __shared__ int s_cross, s_cut, s_done, s_bad;
  __shared__ float s_S, s_pmax;
  __shared__ uint64_t s_cutkey;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  float* prow = probs + (size_t)row * V;
  uint64_t* comp = f.comp + (size_t)row * f.max_vocab;
  float* ssum = f.ssum + (size_t)row * f.max_vocab;

  float pm = 0.0f;
  bool bad = false;
  for (int c = tid; c < V; c += FV_THREADS) {
    const float p = prow[c];
    if (p != p || p == INFINITY) bad = true;
    else pm = fmaxf(pm, p);
  }
  if (tid == 0) s_bad = 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
  if (lane == 0) s_red[warp] = pm;
  for (int i = tid; i < FV_NB; i += FV_THREADS) cursor[i] = 0;
  __syncthreads();
  if (bad) s_bad = 1;
  if (warp == 0) {
    float m = lane < FV_THREADS / 32 ? s_red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_pmax = m;
  }
  __syncthreads();
  const float pmax = s_pmax;
  if (s_bad || !(pmax >= 0x1p-100f)) {
    if (tid == 0 && flags) flags[row] = FLAG_NONFINITE;
    return;
  }
  const uint32_t kmax = __float_as_uint(pmax);
  const int e0 = (int)((kmax >> 23) & 0xFF) - 127;
  const float pmin = __int_as_float((127 + e0 - 24) << 23);  // 2^(e0-24)
  auto bin_of = [&](float p) { return (int)((kmax - __float_as_uint(p)) >> 16); };

  for (int c = tid; c < V; c += FV_THREADS) {
    const float p = canon(prow[c]);
    if (p >= pmin) atomicAdd(&cursor[bin_of(p)], 1);
  }
  __syncthreads();
  fv_scan_bins(cursor, binoff, s_ired);
  const int nrel = binoff[FV_NB];
  for (int c = tid; c < V; c += FV_THREADS) {
    const float p = canon(prow[c]);
    if (p >= pmin) {
      const int pos = atomicAdd(&cursor[bin_of(p)], 1);
      comp[pos] = fv_comp(p, c);
    }
  }
  if (tid == 0) {
    s_S = 0.0f;
    s_done = 0;
    s_cut = -1;
  }
  __syncthreads();

  int b = 0, pos0 = 0;
  while (b < FV_NB && pos0 < nrel) {
    int b2 = b;
    while (b2 < FV_NB && binoff[b2 + 1] - pos0 <= FV_GCAP) ++b2;
    const bool big = (b2 == b);
    int gn;
    if (big) {
      gn = binoff[b + 1] - binoff[b];
      cta_sort_any_n(comp + pos0, gn);
      __syncthreads();
    } else {
      gn = binoff[b2] - pos0;
    }
    for (int s0 = 0; s0 < gn; s0 += FV_GCAP) {
      const int sn = min(FV_GCAP, gn - s0);
      for (int i = tid; i < sn; i += FV_THREADS) gkeys[i] = comp[pos0 + s0 + i];
      __syncthreads();
      if (!big) cta_sort_any_n(gkeys, sn);
      for (int i = tid; i < sn; i += FV_THREADS) gw[i] = fv_val(gkeys[i]);
      __syncthreads();
      const float Sn = exact_prefix_sums(gw, sn, s_S, gs, s_warp, &s_cross);
      for (int i = tid; i < sn; i += FV_THREADS) {
        comp[pos0 + s0 + i] = gkeys[i];
        ssum[pos0 + s0 + i] = gs[i];
      }
      if (tid == 0) {
        s_S = Sn;
        if (Sn >= top_p) {
          int lo = 0, hi = sn;
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (gs[mid] >= top_p) hi = mid; else lo = mid + 1;
          }
          s_cut = pos0 + s0 + lo + 1;
          s_done = 1;
        }
      }
      __syncthreads();
      if (s_done) break;
    }
    if (s_done) break;
    pos0 += gn;
    b = big ? b + 1 : b2;
  }
  __syncthreads();
  // cutoff (-1: never reached -> every entry is kept) and the retained sum
  if (tid == 0) {
    const int cut = s_cut;
    if (cut > 0) {
      s_S = ssum[cut - 1];
      s_cutkey = comp[cut - 1];
      uint32_t fl = 0u;
      if (cut < nrel && (uint32_t)(comp[cut] >> 32) == (uint32_t)(comp[cut - 1] >> 32))
        fl |= FLAG_TIE_AT_DRAW;
      // the element after the cutoff may be an irrelevant one equal in value
      // only if it is relevant too, so checking within [0,nrel) suffices
      if (flags) flags[row] = fl;
    } else {
      s_cutkey = ~0ull;
      if (flags) flags[row] = 0u;
    }
  }
  __syncthreads();
  const float retained = s_S;
  const uint64_t ck = s_cutkey;
  for (int c = tid; c < V; c += FV_THREADS) {
    const float p = prow[c];
    const bool keep = fv_comp(canon(p), c) <= ck;
    prow[c] = keep ? (retained > 0.0f ? __fdiv_rn(p, retained) : 0.0f) : 0.0f;
  }
}

inline size_t fv_smem_bytes(int bm_words, int h_cap) {
  return (size_t)FV_GCAP * 8 + (size_t)FV_GCAP * 4 * 2 + (size_t)(FV_NB + 1) * 4 +
         (size_t)FV_NB * 4 + (size_t)bm_words * 4 + (size_t)h_cap * 4;
}

inline int launch_fullvocab(const FvScratch& f, SampleArgs a, int rows, int K, int max_smem,
                            cudaStream_t stream, bool fixup, int fixup_ctas) {
  if (a.V > f.max_vocab) return 8;  // NCB_ERROR_CAPACITY
  a.seg_len = a.V;
  a.bm_words = (a.V + 31) / 32 + 1;
  const bool counts = (a.p.frequency_penalty != 0.0f || a.p.presence_penalty != 0.0f);
  const size_t smem = fv_smem_bytes(a.bm_words, counts ? a.h_cap : 0);
  if ((int)smem > max_smem) return 8;
  if (fixup) {
    const int g = rows < fixup_ctas ? rows : fixup_ctas;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(g);
    cfg.blockDim = dim3(FV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = counts ? cudaLaunchKernelEx(&cfg, fullvocab_fixup_kernel<true>, a, f, K, rows)
                           : cudaLaunchKernelEx(&cfg, fullvocab_fixup_kernel<false>, a, f, K, rows);
    return e == cudaSuccess ? 0 : 5;
  } else if (counts) {
    fullvocab_kernel<true><<<rows, FV_THREADS, smem, stream>>>(a, f, K);
  } else {
    fullvocab_kernel<false><<<rows, FV_THREADS, smem, stream>>>(a, f, K);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 5;
}

}  // namespace nvs
