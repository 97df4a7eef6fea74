// Full-vocabulary nucleus sampling by value buckets (sm_100a): the path of
// TokenSampler.SampleFiltered (TokenSampler.cs:54-135) when TopK >= V ("no
// top-k", GenerationOptions.cs:79) or TopK is above the top-k kernels' limit,
// with the same result bits as the sorted sequential sums it restates.
//
// The reference sorts every candidate descending and adds the weights
// w_i = exp(v_i - max) one after another in fp32. While the running sum S
// stays in one binade [2^e, 2^(e+1)), fl(S + w) = S + round(w / g) g with the
// grid g = 2^(e-23): an integer addition whose order does not matter, except
// for a weight exactly halfway between two grid points (its rounding follows
// the parity of S). So one CTA per row (its shape below):
//   1. pass over the row: maximum and minimum of the penalised, scaled values;
//   2. pass: histogram of x = v - max over NC_NB buckets spanning
//      [max(min - max, -17), 0] (a weight below e^-17 < 2^-24 never changes a
//      sum that is >= 1 after the first, largest, element);
//   3. from the counts and each bucket's weight bounds, an estimate of S at
//      every bucket: buckets whose S range may hold a binade change are
//      "special", every other bucket gets the binade of its estimate;
//   4. pass: weights of normal buckets are rounded onto their grid (an __expf
//      estimate decides unless it lies within its error bound of a half grid
//      point, then the correctly rounded exp does) and added per bucket as
//      integers; elements of special buckets are gathered; a bucket holding an
//      exact half is made special and gathered by one more pass;
//   5. special buckets are sorted (value descending, id ascending) and one warp
//      walks the row: whole regions of normal buckets by their integer sums,
//      special buckets element by element (carry-save scan of the additions,
//      a plain fp32 addition where the binade changes);
//   6. every normal bucket is checked against the binade its region really
//      had and that no prefix left it; the sums at bucket ends are exact;
//   7. the buckets that hold the top-p cutoff and the drawn position are
//      gathered by one more pass, sorted and summed element by element from
//      their exact start.
// A row that fails a check (an estimate off by more than its margin, a special
// bucket larger than NC_SORT_BIG) is marked for the exact full-sort kernel,
// launched after this one.
#pragma once

#include "fullvocab_kernels.cuh"

namespace nvs {

// A CTA's shape: threads, value buckets, CTAs per SM. A batch that fits one
// wave of SMs takes NcOne (1024 threads, 4096 buckets, one CTA per SM: the
// row's latency decides); a larger one NcTwo (512 threads, 2560 buckets, two
// CTAs per SM, so that one row's latency-bound phases - estimate, sorts, walk -
// overlap the other's passes) when two of its CTAs fit an SM's shared memory.
template <int kThreads, int kBuckets, int kCtasPerSm>
struct NcShape {
  static constexpr int T = kThreads, NB = kBuckets, PER = kBuckets / kThreads;
  static constexpr int W = kThreads / 32, M = kCtasPerSm;
  static_assert(kBuckets % kThreads == 0 && kBuckets % 32 == 0, "buckets: whole per thread");
};
using NcOne = NcShape<1024, 4096, 1>;
using NcTwo = NcShape<512, 2560, 2>;
// NcTwo's dynamic shared memory limit for two CTAs per SM (228 KB per SM, less
// each CTA's static shared memory and reserve)
constexpr size_t NC_TWO_SMEM_MAX = (size_t)110 << 10;
// the shape's figures under the names the code below uses
#define NC_SHAPE_NAMES                                                          \
  constexpr int NC_THREADS = C::T, NC_NB = C::NB, NC_PER = C::PER, NC_WARPS = C::W; \
  (void)NC_THREADS; (void)NC_NB; (void)NC_PER; (void)NC_WARPS
constexpr int NC_SORT_WARP = 256;       // buckets up to this size are sorted by one warp
constexpr int NC_SORT_BIG = 8192;       // a special bucket above this hands the row over
// bk[]: the low byte holds a normal bucket's binade e (grid 2^(e-23)); flags:
constexpr uint32_t NC_SPECIAL = 0x8000u;  // elements gathered, sorted and walked one by one
constexpr uint32_t NC_EXCL = 0x4000u;     // after the top-k cut
constexpr uint32_t NC_UNIFORM = 0x2000u;  // every weight rounds to the same grid units
constexpr uint32_t NC_GATHER = 0x1000u;   // may hold the cutoff or the draw: gathered too
constexpr uint32_t NC_STRADDLE = 0x0800u; // one half grid point inside: units by two x thresholds
constexpr uint32_t NC_TIEF = 0x0400u;     // straddling bucket with weights exactly at the half point
constexpr uint32_t NC_MULTI = 0x0200u;    // several half points inside: gathered, units per element
constexpr int NC_TIES = 64;               // such weights per row
constexpr uint32_t NC_EMASK = 0x00FFu;
constexpr uint32_t NC_QMAX = 1u << 23;  // a normal bucket's grid units stay below this
constexpr int NC_GATHER_CAP = 4096;     // elements of predicted cutoff / draw buckets

// Bound on |__expf(x) - expf_correctly_rounded(x)| for x in [-17, 0], in ulps of
// __expf(x): the documented 2 + floor(|1.173 x|) = 21 ulps of the exact value,
// plus half an ulp of the rounded one, doubled for a binade change between the
// two. The ambiguity test below uses 64.
constexpr int NC_FAST_EXP_ULPS = 21;

struct NcSmem {
  uint32_t* pos;    // [NB+1] first sorted position of each bucket
  uint32_t* cur;    // [NB+1] counts, then gather cursors (entry NB counts the values
                    // below e^-17 relative to the maximum, which never matter)
  uint32_t* qs;     // [NB] grid units of a normal bucket, then their exclusive prefix
  uint32_t* kq;     // [NB] straddling bucket: units of a weight below its half point;
                    // multi bucket: offset of its elements in the per-element pass;
                    // special bucket, after that: offset of its elements in the walk's stage
  float* send;      // [NB+1] exact running sum after each bucket (before: pass 3's lower
                    // threshold of each bucket)
  float* regS;      // [NB+1] running sum at the start of each region (before: pass 3's
                    // upper threshold of each bucket)
  uint16_t* splist; // [NB] special non-empty buckets, ascending
  uint16_t* bk;     // [NB+1] binade of a normal bucket | NC_* flags (entry NB: 0)
  uint32_t* tie;    // [NB/32] buckets holding an exact half (made special)
  uint32_t* gat;    // [NB/32] buckets to gather in the current pass
  uint32_t* bitmap;
  int32_t* hsorted;
};

template <class C>
inline size_t nc_smem_bytes(int bm_words, int h_cap) {
  NC_SHAPE_NAMES;
  return (size_t)(NC_NB + 1) * 4 + (size_t)(NC_NB + 4) * 4 + (size_t)NC_NB * 4 * 2 +
         (size_t)(NC_NB + 1) * 4 * 2 + 8 +
         (size_t)NC_NB * 2 * 2 + (size_t)NC_NB / 32 * 4 * 2 + 64 +
         (size_t)bm_words * 4 + (size_t)h_cap * 4;
}

template <class C>
__device__ __forceinline__ NcSmem nc_carve(unsigned char* smem, int bm_words) {
  NC_SHAPE_NAMES;
  NcSmem s;
  unsigned char* p = smem;
  s.pos = reinterpret_cast<uint32_t*>(p); p += (NC_NB + 1) * 4;
  s.cur = reinterpret_cast<uint32_t*>(p); p += (NC_NB + 4) * 4;
  s.qs = reinterpret_cast<uint32_t*>(p); p += NC_NB * 4;
  s.kq = reinterpret_cast<uint32_t*>(p); p += NC_NB * 4;
  s.send = reinterpret_cast<float*>(p); p += (NC_NB + 1) * 4;
  s.regS = reinterpret_cast<float*>(p); p += (NC_NB + 1) * 4;
  s.tie = reinterpret_cast<uint32_t*>(p); p += NC_NB / 32 * 4;
  s.gat = reinterpret_cast<uint32_t*>(p); p += NC_NB / 32 * 4;
  s.bitmap = reinterpret_cast<uint32_t*>(p); p += (size_t)bm_words * 4;
  s.splist = reinterpret_cast<uint16_t*>(p); p += NC_NB * 2;
  s.bk = reinterpret_cast<uint16_t*>(p); p += NC_NB * 2 + 8;
  p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
  s.hsorted = reinterpret_cast<int32_t*>(p);
  return s;
}

// The member branch of AdjustLogit (TokenSampler.cs:137-143) plus the
// frequency/presence term, for an id known to be in the history.
__device__ __forceinline__ float nc_adjust_member(const Penalty& P, float l, int id) {
  float v = l;
  if (P.rep) v = (v > 0.0f) ? __fdiv_rn(v, P.pen) : __fmul_rn(v, P.pen);
  if (P.cnt) {
    const int c = count_in_sorted(P.hsorted, P.hn, id);
    v = __fsub_rn(v, __fmul_rn((float)c, P.freq));
    v = __fsub_rn(v, P.pres);
  }
  return v;
}

// Calls f(v, c) for every column c of the row with v the penalised, scaled,
// canonical value; 16-byte loads for the aligned body, NC_INFLIGHT of them
// issued before any is used.
constexpr int NC_INFLIGHT = 4;
template <class C, typename F>
__device__ __forceinline__ void nc_stream(const float* lrow, int V, const Penalty& P, float scale,
                                          F&& f) {
  NC_SHAPE_NAMES;
  const bool pen = P.rep || P.cnt;
  auto val = [&](float l, bool member, int c) {
    return canon(__fmul_rn(member ? nc_adjust_member(P, l, c) : l, scale));
  };
  auto bit = [&](int c) { return pen && ((P.bitmap[c >> 5] >> (c & 31)) & 1u); };
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)lrow & 15u)) & 15u) >> 2);
  const int a0 = head < V ? head : V;
  const int n4 = (V - a0) >> 2;
  const int a1 = a0 + 4 * n4;
  for (int c = threadIdx.x; c < a0; c += NC_THREADS) f(val(lrow[c], bit(c), c), c);
  for (int c = a1 + threadIdx.x; c < V; c += NC_THREADS) f(val(lrow[c], bit(c), c), c);
  const float4* body = reinterpret_cast<const float4*>(lrow + a0);
  for (int q0 = threadIdx.x; q0 < n4; q0 += NC_THREADS * NC_INFLIGHT) {
    float4 buf[NC_INFLIGHT];
#pragma unroll
    for (int u = 0; u < NC_INFLIGHT; ++u) {
      const int q = q0 + u * NC_THREADS;
      if (q < n4) buf[u] = __ldg(body + q);
    }
#pragma unroll
    for (int u = 0; u < NC_INFLIGHT; ++u) {
      const int q = q0 + u * NC_THREADS;
      if (q < n4) {
        const int c = a0 + 4 * q;
        uint32_t bits = 0u;
        if (pen) {
          const int w = c >> 5, sh = c & 31;
          const uint64_t win = (uint64_t)P.bitmap[w] | ((uint64_t)P.bitmap[w + 1] << 32);
          bits = (uint32_t)(win >> sh) & 0xFu;
        }
        f(val(buf[u].x, bits & 1u, c), c);
        f(val(buf[u].y, bits & 2u, c + 1), c + 1);
        f(val(buf[u].z, bits & 4u, c + 2), c + 2);
        f(val(buf[u].w, bits & 8u, c + 3), c + 3);
      }
    }
  }
}

// nc_stream with the aligned body handed over four values at a time:
// f4(v0, v1, v2, v3, c) for columns c..c+3, f(v, c) for the unaligned ends.
template <class C, typename F, typename F4>
__device__ __forceinline__ void nc_stream4(const float* lrow, int V, const Penalty& P, float scale,
                                           F&& f, F4&& f4) {
  NC_SHAPE_NAMES;
  const bool pen = P.rep || P.cnt;
  auto val = [&](float l, bool member, int c) {
    return canon(__fmul_rn(member ? nc_adjust_member(P, l, c) : l, scale));
  };
  auto bit = [&](int c) { return pen && ((P.bitmap[c >> 5] >> (c & 31)) & 1u); };
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)lrow & 15u)) & 15u) >> 2);
  const int a0 = head < V ? head : V;
  const int n4 = (V - a0) >> 2;
  const int a1 = a0 + 4 * n4;
  for (int c = threadIdx.x; c < a0; c += NC_THREADS) f(val(lrow[c], bit(c), c), c);
  for (int c = a1 + threadIdx.x; c < V; c += NC_THREADS) f(val(lrow[c], bit(c), c), c);
  const float4* body = reinterpret_cast<const float4*>(lrow + a0);
  for (int q0 = threadIdx.x; q0 < n4; q0 += NC_THREADS * NC_INFLIGHT) {
    float4 buf[NC_INFLIGHT];
#pragma unroll
    for (int u = 0; u < NC_INFLIGHT; ++u) {
      const int q = q0 + u * NC_THREADS;
      if (q < n4) buf[u] = __ldg(body + q);
    }
#pragma unroll
    for (int u = 0; u < NC_INFLIGHT; ++u) {
      const int q = q0 + u * NC_THREADS;
      if (q < n4) {
        const int c = a0 + 4 * q;
        uint32_t bits = 0u;
        if (pen) {
          const int w = c >> 5, sh = c & 31;
          const uint64_t win = (uint64_t)P.bitmap[w] | ((uint64_t)P.bitmap[w + 1] << 32);
          bits = (uint32_t)(win >> sh) & 0xFu;
        }
        f4(val(buf[u].x, bits & 1u, c), val(buf[u].y, bits & 2u, c + 1),
           val(buf[u].z, bits & 4u, c + 2), val(buf[u].w, bits & 8u, c + 3), c);
      }
    }
  }
}

// Grid units of one weight by the correctly rounded exp (the fast estimate was
// too close to a half grid point): returns false for an exact half.
__device__ __noinline__ bool nc_units_exact(float x, float sc, uint32_t* q, int* slow_flag) {
  bool slow = false;
  const float te = __fmul_rn(exp_cr(x, slow), sc);
  if (slow) *slow_flag = 1;
  const float fe = floorf(te);
  const float fre = __fsub_rn(te, fe);
  *q = (uint32_t)fe + (fre > 0.5f ? 1u : 0u);
  return fre != 0.5f;
}

// Exclusive block scan of one value per thread (NC_THREADS threads); returns
// the thread's base and writes the total to *total. Ends synchronised.
template <class C, typename T>
__device__ __forceinline__ T nc_block_scan(T v, T* s_tmp, T* total) {
  NC_SHAPE_NAMES;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const T o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += o;
  }
  if (lane == 31) s_tmp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const T wv = lane < NC_WARPS ? s_tmp[lane] : T(0);
    T wi = wv;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const T o = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= d) wi += o;
    }
    if (lane < NC_WARPS) s_tmp[lane] = wi - wv;
    if (lane == 31) s_tmp[32] = wi;
  }
  __syncthreads();
  const T base = s_tmp[warp] + inc - v;
  *total = s_tmp[32];
  __syncthreads();
  return base;
}

// Sorts a[0..n) ascending with one warp, R keys per lane (n <= 32 R).
template <int R>
__device__ __forceinline__ void nc_warp_sort(uint64_t* a, int n) {
  const int lane = threadIdx.x & 31;
  uint64_t k[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane * R + r;
    k[r] = i < n ? a[i] : ~0ull;
  }
#pragma unroll
  for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= R) {
        const int lm = stride / R;
        const bool lower = (lane & lm) == 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const bool up = (((lane * R + r) & size) == 0);
          const uint64_t o = __shfl_xor_sync(0xffffffffu, k[r], lm);
          const uint64_t mn = k[r] < o ? k[r] : o, mx = k[r] < o ? o : k[r];
          k[r] = (lower == up) ? mn : mx;
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int p = r ^ stride;
          if (p > r) {
            const bool up = (((lane * R + r) & size) == 0);
            const uint64_t x = k[r], y = k[p];
            if ((x > y) == up) {
              k[r] = y;
              k[p] = x;
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane * R + r;
    if (i < n) a[i] = k[r];
  }
}

__device__ __forceinline__ void nc_warp_sort_any(uint64_t* a, int n) {
  if (n <= 1) return;
  if (n <= 32) nc_warp_sort<1>(a, n);
  else if (n <= 64) nc_warp_sort<2>(a, n);
  else if (n <= 128) nc_warp_sort<4>(a, n);
  else nc_warp_sort<8>(a, n);
}

// One warp: the sequential fp32 sums of ws[0..n) (weights, in the order they
// are added) starting from S, written over the weights; returns the last sum.
// Within a binade a carry-save scan of the grid increments (parity transducers,
// exact also at halves); an addition that leaves the binade is done as a plain
// fp32 addition and the scan restarts after it.
__device__ float nc_warp_exact_run(float* ws, int n, float S) {
  const int lane = threadIdx.x & 31;
  int i = 0;
  while (i < n) {
    const bool valid = i + lane < n;
    const float w = valid ? ws[i + lane] : 0.0f;
    if (S == 0.0f) {  // the row's first element: fl(0 + w) = w
      const float w0 = __shfl_sync(0xffffffffu, w, 0);
      if (lane == 0) ws[i] = w0;
      __syncwarp();
      S = w0;
      i += 1;
      continue;
    }
    const uint32_t sb = __float_as_uint(S);
    const int e = (int)((sb >> 23) & 0xFFu) - 127;
    const float inv_grid = __int_as_float((127 - (e - 23)) << 23);
    const float grid = __int_as_float((127 + (e - 23)) << 23);
    const int M = (int)((sb & 0x7FFFFFu) | 0x800000u);
    Tdu inc = valid ? tdu_of(w, inv_grid) : tdu_identity();
    int cum;
    if (__ballot_sync(0xffffffffu, inc.inc0 != inc.inc1) == 0u) {
      // no exact half in the window: every addition adds its units whatever
      // the parity, an integer prefix sum
      int v = inc.inc0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v = min(v + o, 1 << 25);
      }
      cum = M + v;
    } else {
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const Tdu o = tdu_shfl_up(inc, d);
        if (lane >= d) inc = tdu_compose(o, inc);
      }
      cum = M + ((M & 1) ? inc.inc1 : inc.inc0);
    }
    const uint32_t cross = __ballot_sync(0xffffffffu, valid && cum >= (1 << 24));
    const int c = cross ? __ffs(cross) - 1 : 32;
    if (valid && lane < c) ws[i + lane] = __fmul_rn((float)cum, grid);
    if (c < 32) {
      const int cum_prev = __shfl_sync(0xffffffffu, cum, (c + 31) & 31);
      const float wc = __shfl_sync(0xffffffffu, w, c);
      const float prev = c == 0 ? S : __fmul_rn((float)cum_prev, grid);
      const float Sc = __fadd_rn(prev, wc);
      if (lane == c) ws[i + c] = Sc;
      S = Sc;
      i += c + 1;
    } else {
      const int nv = n - i < 32 ? n - i : 32;
      const int cl = __shfl_sync(0xffffffffu, cum, nv - 1);
      S = __fmul_rn((float)cl, grid);
      i += nv;
    }
    __syncwarp();
  }
  return S;
}

// Smallest float x < 0 whose correctly rounded exp is >= w (gt = false) or > w
// (gt = true), by steps of one float from x0 (close to log w); false when the
// steps run out. exp_cr is monotone, so every x below the result rounds below.
__device__ __noinline__ bool nc_exp_threshold(float w, bool gt, float x0, float* out, int* slow_flag) {
  auto ok = [&](float x) {
    bool sl = false;
    const float e = exp_cr(x, sl);
    if (sl) *slow_flag = 1;
    return gt ? e > w : e >= w;
  };
  // for x < 0 the next float up (toward 0) has the bit pattern minus one
  float x = x0;
  if (!(x < -0x1p-100f)) return false;
  if (ok(x)) {
    for (int i = 0; i < 64; ++i) {
      const float y = __uint_as_float(__float_as_uint(x) + 1u);
      if (!ok(y)) {
        *out = x;
        return true;
      }
      x = y;
    }
  } else {
    for (int i = 0; i < 64 && x < -0x1p-100f; ++i) {
      x = __uint_as_float(__float_as_uint(x) - 1u);
      if (ok(x)) {
        *out = x;
        return true;
      }
    }
  }
  return false;
}

// The same from the logarithm: exp(x) of a float x != 0 is irrational, never a
// midpoint between two floats, so exp_cr(x) >= w exactly when x > L = ln(the
// midpoint of w and the float below it), and exp_cr(x) > w when x > ln(the
// midpoint of w and the float above it). The smallest float above L is the
// double logarithm rounded up when that lies clear of both neighbouring float
// boundaries by more than its error (1 ulp documented; 4 allowed); otherwise the
// stepping search decides. w is a positive normal float below 1.
__device__ __forceinline__ bool nc_exp_threshold_log(float w, bool gt, float* out, int* slow_flag) {
  const uint32_t wb = __float_as_uint(w);
  const float nb = __uint_as_float(gt ? wb + 1u : wb - 1u);
  const double L = log(0.5 * ((double)w + (double)nb));  // the midpoint is exact in double
  float f = __double2float_ru(L);                          // smallest float >= L (L < 0)
  if ((double)f == L) f = __uint_as_float(__float_as_uint(f) - 1u);
  const float fp = __uint_as_float(__float_as_uint(f) + 1u);  // the float below f
  const double err = fabs(L) * 0x1p-50;
  if ((double)f - L > err && L - (double)fp > err) {
    *out = f;
    return true;
  }
  return nc_exp_threshold(w, gt, f, out, slow_flag);
}

// First index in [lo, hi) with a[i] >= t (hi when none).
__device__ __forceinline__ int nc_first_ge(const float* a, int lo, int hi, float t) {
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] >= t) hi = mid; else lo = mid + 1;
  }
  return lo;
}

template <bool kCounts, class C>
__global__ void __launch_bounds__(C::T, C::M)
    nucleus_kernel(const __grid_constant__ SampleArgs a, FvScratch f, int K) {
  NC_SHAPE_NAMES;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float s_fred[2][NC_WARPS];
  __shared__ uint32_t s_u32[33];
  __shared__ double s_dbl[33];
  __shared__ int s_hn, s_nf, s_fail, s_slow, s_last, s_bK, s_cutn, s_nsp, s_again, s_done;
  __shared__ uint32_t s_qend;
  __shared__ int s_ntie;
  __shared__ uint16_t s_tlist[NC_TIES];
  __shared__ uint32_t s_tna[NC_TIES];  // weights above the half point in that bucket
  __shared__ float s_vmax, s_vmin, s_total;
  // target state (thread 0): cutoff bucket / index, retained, sample, drawn bucket / index
  __shared__ int s_bc, s_ic, s_bs, s_is;
  __shared__ float s_ret, s_sample, s_target;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int V = a.V;
  NcSmem s = nc_carve<C>(smem, a.bm_words);
  const float* lrow = a.logits + (size_t)row * V;
  uint64_t* comp = f.comp + (size_t)row * f.max_vocab;
  float* ssum = f.ssum + (size_t)row * f.max_vocab;
  const float scale = __fdiv_rn(1.0f, a.p.temperature);

  Penalty P;
  const bool hist_ok = setup_penalty<kCounts>(P, a, row, 0, V, s.bitmap, s.hsorted, &s_hn);
  if (tid == 0) {
    s_nf = 0;
    s_fail = 0;
    s_slow = 0;
    s_last = 0;
    s_bK = -1;
  }
  for (int i = tid; i <= NC_NB; i += NC_THREADS) s.cur[i] = 0u;
  if (tid < NC_NB / 32) s.tie[tid] = 0u;
  if (tid == 0) s.bk[NC_NB] = 0;
  __syncthreads();
  if (!hist_ok) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_BAD_HISTORY;
    }
    return;
  }

  // ---- 1. maximum and minimum ------------------------------------------------
  {
    float mx = -INFINITY, mn = INFINITY;
    bool nf = false;
    nc_stream<C>(lrow, V, P, scale, [&](float v, int) {
      if (v != v || v == INFINITY) nf = true;
      mx = fmaxf(mx, v);
      mn = fminf(mn, v);
    });
    if (__any_sync(0xffffffffu, nf) && lane == 0) s_nf = 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    }
    if (lane == 0) {
      s_fred[0][warp] = mx;
      s_fred[1][warp] = mn;
    }
    __syncthreads();
    if (warp == 0) {
      mx = lane < NC_WARPS ? s_fred[0][lane] : -INFINITY;
      mn = lane < NC_WARPS ? s_fred[1][lane] : INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      }
      if (lane == 0) {
        s_vmax = mx;
        s_vmin = mn;
      }
    }
    __syncthreads();
  }
  const float vmax = s_vmax;
  if (s_nf || !(vmax > -INFINITY)) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_NONFINITE;
    }
    return;
  }
  // buckets: b = floor(x * bscale), x in [xlo, 0], larger values first
  float xlo = fmaxf(__fsub_rn(s_vmin, vmax), FV_XMIN);
  if (xlo > -0x1p-20f) xlo = -0x1p-20f;
  const float bscale = __fdiv_rn((float)NC_NB, xlo);  // < 0
  auto bin = [&](float x) {
    const int b = (int)__fmul_rn(x, bscale);
    return b < NC_NB - 1 ? b : NC_NB - 1;
  };

  // ---- 2. histogram -------------------------------------------------------------
  auto bin_rel = [&](float v) {  // bucket of a value, NC_NB when it never matters
    const float x = __fsub_rn(v, vmax);
    return x >= FV_XMIN ? bin(x) : NC_NB;
  };
  nc_stream4<C>(
      lrow, V, P, scale, [&](float v, int) { atomicAdd(&s.cur[bin_rel(v)], 1u); },
      [&](float v0, float v1, float v2, float v3, int) {
        const int b0 = bin_rel(v0), b1 = bin_rel(v1), b2 = bin_rel(v2), b3 = bin_rel(v3);
        atomicAdd(&s.cur[b0], 1u);
        atomicAdd(&s.cur[b1], 1u);
        atomicAdd(&s.cur[b2], 1u);
        atomicAdd(&s.cur[b3], 1u);
      });
  __syncthreads();
  uint32_t cnt[NC_PER];
  int nrel;
  {
    uint32_t sum = 0u;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      cnt[j] = s.cur[tid * NC_PER + j];
      sum += cnt[j];
      if (cnt[j]) atomicMax(&s_last, tid * NC_PER + j);
    }
    uint32_t total;
    uint32_t run = nc_block_scan<C, uint32_t>(sum, s_u32, &total);
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      s.pos[tid * NC_PER + j] = run;
      run += cnt[j];
    }
    if (tid == 0) s.pos[NC_NB] = total;
    nrel = (int)total;
  }
  __syncthreads();
  // top-k cut (K < candidates): the bucket holding sorted position K-1
  if (K < nrel) {
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      if ((int)s.pos[b] <= K - 1 && K - 1 < (int)s.pos[b + 1]) s_bK = b;
    }
  }
  __syncthreads();
  const int bK = s_bK;
  const int last = bK >= 0 ? bK : s_last;

  // ---- 3. estimated binade of the running sum at every bucket -----------------
  {
    double wlo[NC_PER], whi[NC_PER];
    double clo = 0.0, chi = 0.0;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      // x in bucket b: b <= fl(x bscale) < b + 1
      const double xb_hi = (double)b / (double)bscale;
      double xb_lo = (double)(b + 1) / (double)bscale;
      if (xb_lo < (double)xlo) xb_lo = (double)xlo;
      whi[j] = exp(xb_hi + 1e-6 * (1.0 - xb_hi));
      wlo[j] = exp(xb_lo - 1e-6 * (1.0 - xb_lo));
      if (b <= last) {
        // the cut bucket holds at least K - pos candidates
        clo += (double)(b == bK ? (uint32_t)K - s.pos[b] : cnt[j]) * wlo[j];
        chi += (double)cnt[j] * whi[j];
      }
    }
    double tl, th;
    double lo = nc_block_scan<C, double>(clo, s_dbl, &tl);
    double hi = nc_block_scan<C, double>(chi, s_dbl, &th);
    double bl[NC_PER], bh[NC_PER];  // running sum bounds at each bucket's start / end
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      const double hi_end = hi + (double)cnt[j] * whi[j];
      // margin for the fp32 sums' rounding against the exact ones
      const double m = 0x1p-12 + 0x1p-21 * sqrt((double)s.pos[b + 1] + 1.0);
      bl[j] = lo * (1.0 - m);
      bh[j] = hi_end * (1.0 + m);
      uint32_t code, q = 0u;
      if (b > last) {
        code = NC_EXCL;
      } else if (b == bK || bl[j] < 1.0) {
        code = NC_SPECIAL;
      } else {
        const int el = ilogb(bl[j]), eh = ilogb(bh[j]);
        if (el != eh || el > 30) {
          code = NC_SPECIAL;
        } else {
          code = (uint32_t)el;
          // a bucket whose weights, correctly rounded, all lie strictly inside
          // one half-open grid interval adds the same units per element
          const double sc = ldexp(1.0, 23 - el);
          const double tlo = wlo[j] * (1.0 - 0x1p-20) * sc, thi = whi[j] * (1.0 + 0x1p-20) * sc;
          const double hq = floor(tlo + 0.5);
          float xl, xh;
          if (tlo > hq - 0.5 && thi < hq + 0.5 && (double)cnt[j] * hq < (double)NC_QMAX) {
            code |= NC_UNIFORM;
            q = cnt[j] * (uint32_t)hq;
          } else if (tlo > hq - 0.5 && thi < hq + 1.5 &&
                     (double)cnt[j] * (hq + 1.0) < (double)NC_QMAX) {
            // one half point w_h = (hq + 1/2) grid: a weight rounds to hq units
            // below it, hq + 1 above, and depends on the parity exactly at it;
            // x thresholds of the correctly rounded exp decide which
            const float wh = (float)((hq + 0.5) / sc);  // (2 hq + 1) 2^(e-24): exact
            if (nc_exp_threshold_log(wh, false, &xl, &s_slow) &&
                nc_exp_threshold_log(wh, true, &xh, &s_slow)) {
              code |= NC_STRADDLE;
              q = cnt[j] * (uint32_t)hq;
              s.kq[b] = (uint32_t)hq;
              s.send[b] = xl;  // weights at the half point from here
              s.regS[b] = xh;  // weights above it from here
            } else {
              code = NC_SPECIAL;
            }
          } else {
            code |= NC_MULTI;
          }
        }
      }
      s.bk[b] = (uint16_t)code;
      s.qs[b] = q;
      s.cur[b] = s.pos[b];
      lo += (double)cnt[j] * wlo[j];
      hi = hi_end;
    }
    // The buckets that may hold the top-p cutoff and the draw, from the same
    // bounds, are gathered by the next pass too (they are checked later).
    const double mt = 0x1p-12 + 0x1p-21 * sqrt((double)nrel + 1.0);
    const double tot_lo = tl * (1.0 - mt), tot_hi = th * (1.0 + mt);
    const bool has_p = a.p.top_p < 1.0f;
    const double t_lo = (double)a.p.top_p * tot_lo * (1.0 - 0x1p-20);
    const double t_hi = (double)a.p.top_p * tot_hi * (1.0 + 0x1p-20);
    bool cand[NC_PER];
    double rmax = 0.0;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      cand[j] = has_p && b <= last && bh[j] >= t_lo && bl[j] <= t_hi;
      if (cand[j]) rmax = fmax(rmax, bh[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) rmax = fmax(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
    if (lane == 0) s_dbl[warp] = rmax;
    __syncthreads();
    if (warp == 0) {
      double r = lane < NC_WARPS ? s_dbl[lane] : 0.0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) r = fmax(r, __shfl_xor_sync(0xffffffffu, r, o));
      if (lane == 0) s_dbl[32] = r;
    }
    __syncthreads();
    const double u = (double)a.uniforms[row];
    const double r_lo = has_p ? t_lo : tot_lo, r_hi = has_p ? s_dbl[32] : tot_hi;
    const double d_lo = u * r_lo * (1.0 - 0x1p-20), d_hi = u * r_hi * (1.0 + 0x1p-20);
    uint32_t ncand = 0u;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      cand[j] = cand[j] || (b <= last && bh[j] >= d_lo && bl[j] <= d_hi);
      if (cand[j]) ncand += cnt[j];
    }
    uint32_t ncand_tot;
    (void)nc_block_scan<C, uint32_t>(ncand, s_u32, &ncand_tot);
    if (ncand_tot <= (uint32_t)NC_GATHER_CAP) {
#pragma unroll
      for (int j = 0; j < NC_PER; ++j) {
        const int b = tid * NC_PER + j;
        if (cand[j] && !(s.bk[b] & (NC_SPECIAL | NC_EXCL))) s.bk[b] = (uint16_t)(s.bk[b] | NC_GATHER);
      }
    }
    // pass 3's thresholds: a value x >= regS[b] adds one grid unit to the
    // bucket, one in [send[b], regS[b]) goes the slow way (gathered, or a
    // weight exactly at a straddling bucket's half point). A gathered bucket
    // takes the slow way whole; a straddling one gathered too gets its units
    // per element from its keys, like a multi bucket.
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      uint32_t code = s.bk[b];
      if (code & (NC_SPECIAL | NC_GATHER | NC_MULTI)) {
        if (code & NC_STRADDLE) {
          code = (code & ~NC_STRADDLE) | NC_MULTI;
          s.bk[b] = (uint16_t)code;
          s.qs[b] = 0u;
        }
        s.regS[b] = INFINITY;
        s.send[b] = -INFINITY;
      } else if (!(code & NC_STRADDLE)) {
        s.regS[b] = INFINITY;
        s.send[b] = INFINITY;
      }
    }
    if (tid == 0) {  // values that never matter
      s.regS[NC_NB] = INFINITY;
      s.send[NC_NB] = INFINITY;
    }
  }
  __syncthreads();

  // ---- 4. pass: keys of special and predicted buckets; straddling buckets count ----
  // the weights above their half point and note the ones exactly at it
  if (tid == 0) s_ntie = 0;
  __syncthreads();
  // the slow way: a gathered bucket's key, or a weight at a half point
  auto p3_slow = [&](float v, int c, int b) {
    if (s.bk[b] & (NC_SPECIAL | NC_GATHER | NC_MULTI)) {
      comp[atomicAdd(&s.cur[b], 1u)] = fv_comp(v, c);
    } else {
      const int i = atomicAdd(&s_ntie, 1);
      if (i < NC_TIES) s_tlist[i] = (uint16_t)b;
    }
  };
  nc_stream4<C>(
      lrow, V, P, scale,
      [&](float v, int c) {
        const int b = bin_rel(v);
        const float x = __fsub_rn(v, vmax);
        if (x >= s.regS[b]) atomicAdd(&s.qs[b], 1u);
        else if (x >= s.send[b]) p3_slow(v, c, b);
      },
      [&](float v0, float v1, float v2, float v3, int c) {
        const int b0 = bin_rel(v0), b1 = bin_rel(v1), b2 = bin_rel(v2), b3 = bin_rel(v3);
        const float x0 = __fsub_rn(v0, vmax), x1 = __fsub_rn(v1, vmax);
        const float x2 = __fsub_rn(v2, vmax), x3 = __fsub_rn(v3, vmax);
        const float h0 = s.regS[b0], h1 = s.regS[b1], h2 = s.regS[b2], h3 = s.regS[b3];
        const float l0 = s.send[b0], l1 = s.send[b1], l2 = s.send[b2], l3 = s.send[b3];
        if (x0 >= h0) atomicAdd(&s.qs[b0], 1u);
        if (x1 >= h1) atomicAdd(&s.qs[b1], 1u);
        if (x2 >= h2) atomicAdd(&s.qs[b2], 1u);
        if (x3 >= h3) atomicAdd(&s.qs[b3], 1u);
        const bool w0 = x0 < h0 && x0 >= l0, w1 = x1 < h1 && x1 >= l1;
        const bool w2 = x2 < h2 && x2 >= l2, w3 = x3 < h3 && x3 >= l3;
        if (w0 | w1 | w2 | w3) {
          if (w0) p3_slow(v0, c, b0);
          if (w1) p3_slow(v1, c + 1, b1);
          if (w2) p3_slow(v2, c + 2, b2);
          if (w3) p3_slow(v3, c + 3, b3);
        }
      });
  __syncthreads();
  if (s_ntie > NC_TIES) {
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }
  // straddling buckets with weights at the half point are resolved in the walk
  // from the parity of the sum before them: keep their count above it
  if (tid < s_ntie) {
    const int b = s_tlist[tid];
    atomicOr(&s.tie[b >> 5], 1u << (b & 31));
    s_tna[tid] = s.qs[b] - (s.pos[b + 1] - s.pos[b]) * s.kq[b];
  }
  __syncthreads();
  for (int b = tid; b < NC_NB; b += NC_THREADS)
    if ((s.tie[b >> 5] >> (b & 31)) & 1u) s.bk[b] = (uint16_t)(s.bk[b] | NC_TIEF);
  __syncthreads();

  // ---- 4b. grid units of multi buckets, one element per thread (gathered keys) ------
  {
    uint32_t nm[NC_PER], sum = 0u;
    uint32_t ism = 0u;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      const bool m = (s.bk[b] & NC_MULTI) && s.pos[b + 1] > s.pos[b];
      nm[j] = m ? s.pos[b + 1] - s.pos[b] : 0u;
      ism += m ? 1u : 0u;
      sum += nm[j];
    }
    uint32_t tot, ntot;
    uint32_t off = nc_block_scan<C, uint32_t>(sum, s_u32, &tot);
    uint32_t li = nc_block_scan<C, uint32_t>(ism, s_u32, &ntot);
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      if (nm[j]) {
        s.kq[b] = off;  // first flat index of the bucket
        s.splist[li++] = (uint16_t)b;
        off += nm[j];
      }
    }
    if (tid < NC_NB / 32) s.gat[tid] = 0u;
    __syncthreads();
    for (uint32_t i = tid; i < tot; i += NC_THREADS) {
      // the multi bucket holding flat index i: the last with kq <= i
      int lo = 0, hi = (int)ntot - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s.kq[s.splist[mid]] <= i) lo = mid; else hi = mid - 1;
      }
      const int b = s.splist[lo];
      const float x = __fsub_rn(fv_val(comp[s.pos[b] + (i - s.kq[b])]), vmax);
      const float sc = __int_as_float((127 + 23 - (int)(s.bk[b] & NC_EMASK)) << 23);  // 1 / grid
      const float wa = __expf(x);
      const float t = __fmul_rn(wa, sc);
      const float fl = floorf(t);
      const float fr = __fsub_rn(t, fl);
      // 64 ulps of wa, in grid units, bound the distance to the correctly rounded weight
      const float r =
          __fmul_rn(__uint_as_float((__float_as_uint(wa) & 0x7F800000u) - (17u << 23)), sc);
      uint32_t q;
      bool ok = true;
      if (fabsf(__fsub_rn(fr, 0.5f)) > r) q = (uint32_t)fl + (fr > 0.5f ? 1u : 0u);
      else ok = nc_units_exact(x, sc, &q, &s_slow);
      if (!ok) atomicOr(&s.gat[b >> 5], 1u << (b & 31));
      else if (q != 0u && atomicAdd(&s.qs[b], q) + q >= NC_QMAX) s_fail = 1;
    }
    __syncthreads();
    // a multi bucket holding an exact half is walked element by element (its keys
    // are gathered already)
    for (int b = tid; b < NC_NB; b += NC_THREADS)
      if ((s.gat[b >> 5] >> (b & 31)) & 1u) s.bk[b] = (uint16_t)NC_SPECIAL;
    __syncthreads();
  }


  // ---- 5. sort special buckets, their weights; prefix of the grid units ----------
  {
    uint32_t isp[NC_PER];
    uint32_t nsp_local = 0u, qsum = 0u;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      const bool sp = ((s.bk[b] & NC_SPECIAL) && s.pos[b + 1] > s.pos[b]) || (s.bk[b] & NC_TIEF);
      isp[j] = sp ? 1u : 0u;
      nsp_local += isp[j];
      if (s.bk[b] & (NC_SPECIAL | NC_EXCL | NC_TIEF)) s.qs[b] = 0u;
      qsum += s.qs[b];
    }
    uint32_t nsp, qtot;
    uint32_t o = nc_block_scan<C, uint32_t>(nsp_local, s_u32, &nsp);
    uint32_t qrun = nc_block_scan<C, uint32_t>(qsum, s_u32, &qtot);
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      if (isp[j]) s.splist[o++] = (uint16_t)b;
      const uint32_t q = s.qs[b];
      s.qs[b] = qrun;  // exclusive prefix (mod 2^32; exact where it is used)
      qrun += q;
    }
    if (tid == 0) {
      s_nsp = (int)nsp;
      s_qend = qtot;
    }
    __syncthreads();
  }
  const int nsp = s_nsp;
  // exclusive prefix of the grid units at bucket b (b <= NB)
  auto qpre = [&](int b) { return b < NC_NB ? s.qs[b] : s_qend; };
  // sort: one warp per bucket up to NC_SORT_WARP keys; larger ones by the block
  for (int k = warp; k < nsp; k += NC_WARPS) {
    const int b = s.splist[k];
    const int n = (int)(s.pos[b + 1] - s.pos[b]);
    if (n <= NC_SORT_WARP && !(s.bk[b] & NC_TIEF)) nc_warp_sort_any(comp + s.pos[b], n);
  }
  __syncthreads();
  for (int k = 0; k < nsp; ++k) {
    const int b = s.splist[k];
    const int n = (int)(s.pos[b + 1] - s.pos[b]);
    if (n > NC_SORT_WARP && !(s.bk[b] & NC_TIEF)) {
      if (n > NC_SORT_BIG) {
        if (tid == 0) s_fail = 1;
        break;
      }
      cta_sort_any_n(comp + s.pos[b], n);
      __syncthreads();
    }
  }
  __syncthreads();
  if (s_fail) {
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }
  // top-k cut inside bK: position K-1 and the ties of its value
  if (tid == 0) {
    s_cutn = 0;
    if (bK >= 0) {
      const int p0 = (int)s.pos[bK], p1 = (int)s.pos[bK + 1];
      int e = K - 1;
      const uint32_t kk = (uint32_t)(comp[e] >> 32);
      while (e + 1 < p1 && (uint32_t)(comp[e + 1] >> 32) == kk) ++e;
      s_cutn = e + 1 - p0;
    }
  }
  __syncthreads();
  const int cutn = s_cutn;
  auto n_eff = [&](int b) { return b == bK ? cutn : (int)(s.pos[b + 1] - s.pos[b]); };
  // elements the walk takes one by one (none for a straddling bucket)
  auto n_walk = [&](int b) { return (s.bk[b] & NC_TIEF) ? 0 : n_eff(b); };
  // the walk reads the special elements' weights from shared memory (the
  // cursor array, free until the cutoff search) when they fit, in splist order
  float* stage = reinterpret_cast<float*>(s.cur);
  bool staged;
  {
    uint32_t ne[NC_PER], sum = 0u;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int k = tid * NC_PER + j;
      ne[j] = k < nsp ? (uint32_t)n_walk(s.splist[k]) : 0u;
      sum += ne[j];
    }
    uint32_t total;
    uint32_t run = nc_block_scan<C, uint32_t>(sum, s_u32, &total);
    staged = total <= (uint32_t)NC_NB;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int k = tid * NC_PER + j;
      if (k < nsp && staged && !(s.bk[s.splist[k]] & NC_TIEF)) s.kq[s.splist[k]] = run;
      run += ne[j];
    }
    __syncthreads();
  }
  // weights of the special elements (correctly rounded exp), in place of the sums
  {
    bool slow = false;
    for (int k = warp; k < nsp; k += NC_WARPS) {
      const int b = s.splist[k];
      const int p0 = (int)s.pos[b], n = n_walk(b);
      float* w = staged ? stage + (n ? s.kq[b] : 0u) : ssum + p0;
      for (int i = lane; i < n; i += 32) w[i] = exp_cr(__fsub_rn(fv_val(comp[p0 + i]), vmax), slow);
    }
    if (slow) s_slow = 1;
  }
  __syncthreads();

  // ---- 5b. the walk (one warp): regions by their grid units, specials one by one --
  if (warp == 0) {
    float S = 0.0f;
    int prev = 0;  // first bucket of the current region
    int k = 0;
    bool fail = false;
    auto region = [&](int b_end) {  // normal buckets [prev, b_end)
      const uint32_t D = qpre(b_end) - qpre(prev);
      if (D != 0u) {
        const uint32_t sb = __float_as_uint(S);
        const uint32_t M = (sb & 0x7FFFFFu) | 0x800000u;
        if (S == 0.0f || D >= NC_QMAX || M + D >= (1u << 24)) {
          fail = true;
        } else {
          S = __uint_as_float((sb & 0xFF800000u) | ((M + D) & 0x7FFFFFu));
        }
      }
    };
    while (k < nsp && !fail) {
      const int b0 = s.splist[k];
      if (lane == 0) s.regS[k] = S;
      region(b0);
      if (fail) break;
      if (s.bk[b0] & NC_TIEF) {
        // in sorted order: na weights above the half point (kq + 1 units
        // each), the nt at it (kq units plus one when that makes the sum's
        // last mantissa bit even), the rest below (kq units)
        const uint32_t sb = __float_as_uint(S);
        const int e = (int)((sb >> 23) & 0xFFu) - 127;
        if (S == 0.0f || e != (int)(s.bk[b0] & NC_EMASK)) {
          fail = true;
          break;
        }
        const uint64_t kq = s.kq[b0], cntb = s.pos[b0 + 1] - s.pos[b0];
        uint64_t nt = 0, na = 0;
        for (int i = 0; i < s_ntie; ++i)
          if (s_tlist[i] == b0) {
            ++nt;
            na = s_tna[i];
          }
        uint64_t M = ((sb & 0x7FFFFFu) | 0x800000u) + na * (kq + 1u);
        for (uint64_t t = 0; t < nt && M < (1u << 24); ++t) M += kq + ((M + kq) & 1u);
        M += (cntb - na - nt) * kq;
        if (na + nt > cntb || M >= (1u << 24)) {
          fail = true;
          break;
        }
        S = __uint_as_float((sb & 0xFF800000u) | ((uint32_t)M & 0x7FFFFFu));
        if (lane == 0) s.send[b0] = S;
        prev = b0 + 1;
        k = k + 1;
        continue;
      }
      int k2 = k;
      while (k2 + 1 < nsp && s.splist[k2 + 1] == s.splist[k2] + 1 &&
             !(s.bk[s.splist[k2 + 1]] & NC_TIEF))
        ++k2;
      const int bl = s.splist[k2];
      const int p0 = (int)s.pos[b0];
      const int len = (int)s.pos[bl] + n_eff(bl) - p0;
      float* run = staged ? stage + s.kq[b0] : ssum + p0;
      S = nc_warp_exact_run(run, len, S);
      for (int kk = k + lane; kk <= k2; kk += 32) {
        const int b = s.splist[kk];
        const int ne = n_eff(b);
        s.send[b] = run[(int)s.pos[b] - p0 + ne - 1];
      }
      prev = bl + 1;
      k = k2 + 1;
    }
    if (!fail) {
      if (lane == 0) s.regS[nsp] = S;
      region(last + 1);
    }
    if (lane == 0) {
      s_total = S;
      if (fail) s_fail = 1;
    }
  }
  __syncthreads();
  if (staged) {  // the element sums of special buckets, for the cutoff search
    for (int k = warp; k < nsp; k += NC_WARPS) {
      const int b = s.splist[k];
      const int p0 = (int)s.pos[b], n = n_walk(b);
      for (int i = lane; i < n; i += 32) ssum[p0 + i] = stage[s.kq[b] + i];
    }
    __syncthreads();
  }
  if (s_fail) {
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }

  // ---- 6. sums at the ends of normal buckets, each checked -------------------------
  for (int b = tid; b <= last; b += NC_THREADS) {
    if (s.bk[b] & NC_TIEF) continue;  // set by the walk
    if (s.bk[b] & NC_SPECIAL) {
      if (s.pos[b + 1] == s.pos[b]) s.send[b] = 0.0f;  // empty special: filled below
      continue;
    }
    // region k: the first special bucket after b ends it
    int lo = 0, hi = nsp;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((int)s.splist[mid] < b) lo = mid + 1; else hi = mid;
    }
    const int r0 = lo == 0 ? 0 : (int)s.splist[lo - 1] + 1;
    const float S0 = s.regS[lo];
    const uint32_t D = qpre(b + 1) - qpre(r0);
    const uint32_t sb = __float_as_uint(S0);
    const uint32_t M = (sb & 0x7FFFFFu) | 0x800000u;
    const bool nonempty = s.pos[b + 1] > s.pos[b];
    if (S0 == 0.0f) {
      if (D != 0u || nonempty) s_fail = 1;
      s.send[b] = 0.0f;
      continue;
    }
    const int e = (int)((sb >> 23) & 0xFFu) - 127;
    if ((nonempty && (int)(s.bk[b] & NC_EMASK) != e) || D >= NC_QMAX || M + D >= (1u << 24)) {
      s_fail = 1;
      continue;
    }
    s.send[b] = __uint_as_float((sb & 0xFF800000u) | ((M + D) & 0x7FFFFFu));
  }
  __syncthreads();
  // empty special buckets carry the sum of the nearest bucket before them that
  // has one (a running maximum of defining bucket indices)
  {
    int src[NC_PER];
    int run = -1;
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      const bool empty_sp = (s.bk[b] & NC_SPECIAL) && s.pos[b + 1] == s.pos[b];
      if (b <= last && !empty_sp) run = b;
      src[j] = run;
    }
    // exclusive max-scan of the threads' last defining index
    const int lane_ = tid & 31;
    int inc = run;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane_ >= d) inc = max(inc, o);
    }
    __shared__ int s_wmax[NC_WARPS];
    if (lane_ == 31) s_wmax[warp] = inc;
    __syncthreads();
    int before = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane_ == 0) before = -1;
    for (int w = 0; w < warp; ++w) before = max(before, s_wmax[w]);
    float vals[NC_PER];
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      const int sidx = max(src[j], before);
      vals[j] = (b <= last && src[j] != b) ? (sidx >= 0 ? s.send[sidx] : 0.0f) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NC_PER; ++j) {
      const int b = tid * NC_PER + j;
      if (b <= last && src[j] != b) s.send[b] = vals[j];
    }
  }
  __syncthreads();
  if (s_fail) {
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }

  // ---- 7. cutoff and draw (TokenSampler.cs:105-132) --------------------------------
  // thread 0 decides which buckets it needs summed element by element; their
  // elements are in place already (special, or gathered as predicted) or are
  // gathered by one more pass
  auto sstart = [&](int b) { return b == 0 ? 0.0f : s.send[b - 1]; };
  auto gathered = [&](int b) { return (s.bk[b] & NC_SPECIAL) != 0; };  // element sums ready
  auto marked = [&](int b) { return ((s.gat[b >> 5] >> (b & 31)) & 1u) != 0; };
  __shared__ int s_pass;
  auto request = [&](int b) {
    s.gat[b >> 5] |= 1u << (b & 31);
    s_again = 1;
    if (!(s.bk[b] & (NC_GATHER | NC_MULTI))) s_pass = 1;
  };
  if (tid < NC_NB / 32) s.gat[tid] = 0u;
  if (tid == 0) {
    const float total = s_total;
    s_done = 0;
    s_bc = -1;
    s_bs = -1;
    if (a.p.top_p < 1.0f) {
      s_target = __fmul_rn(total, a.p.top_p);
    } else {
      s_ret = total;
      s_sample = __fmul_rn(a.uniforms[row], total);
    }
  }
  __syncthreads();
  for (int round = 0; round < 4; ++round) {
    if (tid == 0) {
      s_again = 0;
      s_pass = 0;
      // the cutoff's bucket: the first whose end sum reaches the target
      if (a.p.top_p < 1.0f && s_bc < 0) {
        const int bc = nc_first_ge(s.send, 0, last + 1, s_target);
        if (gathered(bc)) {
          const int p0 = (int)s.pos[bc];
          const int ic = nc_first_ge(ssum, p0, p0 + n_eff(bc), s_target) - p0;
          s_bc = bc;
          s_ic = ic;
          s_ret = ssum[p0 + ic];
          s_sample = __fmul_rn(a.uniforms[row], s_ret);
        } else {
          request(bc);
          // the draw lies between u * (sum before bc) and u * (sum after bc)
          const float u = a.uniforms[row];
          const int lo = nc_first_ge(s.send, 0, last + 1, __fmul_rn(u, sstart(bc)));
          const int hi = nc_first_ge(s.send, 0, last + 1, __fmul_rn(u, s.send[bc]));
          if (hi - lo < 8)
            for (int b = lo; b <= hi && b <= last; ++b)
              if (!gathered(b) && !marked(b)) request(b);
        }
      }
      if ((a.p.top_p >= 1.0f || s_bc >= 0) && s_bs < 0) {
        const int bs = nc_first_ge(s.send, 0, last + 1, s_sample);
        if (gathered(bs)) {
          const int p0 = (int)s.pos[bs];
          s_bs = bs;
          s_is = nc_first_ge(ssum, p0, p0 + n_eff(bs), s_sample) - p0;
          s_done = 1;
        } else {
          request(bs);
        }
      }
    }
    __syncthreads();
    if (s_done || !s_again) break;
    // gather the marked buckets not in place yet, sort every marked one, and
    // sum them from their exact start
    if (s_pass) {
      for (int b = tid; b <= last; b += NC_THREADS)
        if (marked(b) && !(s.bk[b] & (NC_GATHER | NC_MULTI))) s.cur[b] = s.pos[b];
      __syncthreads();
      nc_stream<C>(lrow, V, P, scale, [&](float v, int c) {
        const float x = __fsub_rn(v, vmax);
        if (!(x >= FV_XMIN)) return;
        const int b = bin(x);
        if (b <= last && marked(b) && !(s.bk[b] & (NC_GATHER | NC_MULTI)))
          comp[atomicAdd(&s.cur[b], 1u)] = fv_comp(v, c);
      });
      __syncthreads();
    }
    // one warp per marked bucket (a marked normal bucket is below NC_QMAX grid
    // units but may hold many keys: large ones are sorted by the block)
    if (tid == 0) s_nsp = 0;
    __syncthreads();
    for (int b = tid; b <= last; b += NC_THREADS)
      if (marked(b) && !(s.bk[b] & NC_SPECIAL))
        s.splist[NC_NB - 1 - atomicAdd(&s_nsp, 1)] = (uint16_t)b;  // from the top end
    __syncthreads();
    const int ng = s_nsp;
    for (int k = warp; k < ng; k += NC_WARPS) {
      const int b = s.splist[NC_NB - 1 - k];
      const int n = (int)(s.pos[b + 1] - s.pos[b]);
      if (n <= NC_SORT_WARP) nc_warp_sort_any(comp + s.pos[b], n);
    }
    __syncthreads();
    for (int k = 0; k < ng; ++k) {
      const int b = s.splist[NC_NB - 1 - k];
      const int n = (int)(s.pos[b + 1] - s.pos[b]);
      if (n > NC_SORT_WARP) {
        if (n > NC_SORT_BIG) {
          if (tid == 0) s_fail = 1;
          break;
        }
        cta_sort_any_n(comp + s.pos[b], n);
        __syncthreads();
      }
    }
    __syncthreads();
    if (s_fail) {
      if (tid == 0) a.s.fixup[row] = 1u;
      return;
    }
    {
      bool slow = false;
      for (int k = warp; k < ng; k += NC_WARPS) {
        const int b = s.splist[NC_NB - 1 - k];
        const int p0 = (int)s.pos[b], n = n_eff(b);
        for (int i = lane; i < n; i += 32)
          ssum[p0 + i] = exp_cr(__fsub_rn(fv_val(comp[p0 + i]), vmax), slow);
        __syncwarp();
        // the element sums must end where the bucket's grid units said
        if (nc_warp_exact_run(ssum + p0, n, sstart(b)) != s.send[b] && lane == 0) s_fail = 1;
      }
      if (slow) s_slow = 1;
    }
    __syncthreads();
    // the gathered buckets now count as special for the decisions above
    for (int b = tid; b <= last; b += NC_THREADS)
      if (marked(b)) s.bk[b] = (uint16_t)(s.bk[b] | NC_SPECIAL);
    __syncthreads();
    if (tid < NC_NB / 32) s.gat[tid] = 0u;
    __syncthreads();
  }
  if (!s_done) {  // not settled within the rounds (should not happen)
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }

  if (tid == 0) {
    const int bs = s_bs, is = s_is;
    const int ps = (int)s.pos[bs];
    const float retained = s_ret, sample = s_sample;
    uint32_t fl = s_slow ? FLAG_EXP_SLOW : 0u;
    // the sum before a position: the previous element's, or the previous bucket's end
    auto before = [&](int b, int i) { return i > 0 ? ssum[s.pos[b] + i - 1] : sstart(b); };
    const bool first_pos = (bs == 0 && is == 0);
    const double tol = 1e-6 * (double)retained;
    if (fabs((double)sample - (double)ssum[ps + is]) <= tol ||
        (!first_pos && fabs((double)sample - (double)before(bs, is)) <= tol))
      fl |= FLAG_DRAW_BOUNDARY;
    if (a.p.top_p < 1.0f) {
      const float target = s_target;
      const double tt = 1e-6 * (double)target;
      const bool cfirst = (s_bc == 0 && s_ic == 0);
      if (fabs((double)retained - (double)target) <= tt ||
          (!cfirst && fabs((double)before(s_bc, s_ic) - (double)target) <= tt))
        fl |= FLAG_CUTOFF_BOUNDARY;
    }
    const uint32_t ks = (uint32_t)(comp[ps + is] >> 32);
    if ((is > 0 && (uint32_t)(comp[ps + is - 1] >> 32) == ks) ||
        (is + 1 < n_eff(bs) && (uint32_t)(comp[ps + is + 1] >> 32) == ks))
      fl |= FLAG_TIE_AT_DRAW;
    a.tokens[row] = fv_id(comp[ps + is]);
    if (a.flags) a.flags[row] = fl;
  }
}

// Largest distance in float steps between __expf(x) and the correctly rounded
// exp over the bit patterns [k0, k1] of non-positive floats x.
__global__ void fast_exp_steps_kernel(uint32_t k0, uint32_t k1, uint32_t* out) {
  uint32_t worst = 0u;
  for (uint64_t k = (uint64_t)k0 + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k <= k1;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const float x = __uint_as_float((uint32_t)k);
    bool slow = false;
    const uint32_t a = __float_as_uint(__expf(x)), b = __float_as_uint(exp_cr(x, slow));
    const uint32_t d = a > b ? a - b : b - a;  // positive floats: bit distance = steps
    worst = d > worst ? d : worst;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t t = __shfl_xor_sync(0xffffffffu, worst, o);
    worst = t > worst ? t : worst;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(out, worst);
}

template <class C>
inline int launch_nucleus_shape(const FvScratch& f, const SampleArgs& a, int rows, int K,
                                size_t smem, cudaStream_t stream) {
  const bool counts = (a.p.frequency_penalty != 0.0f || a.p.presence_penalty != 0.0f);
  if (counts) nucleus_kernel<true, C><<<rows, C::T, smem, stream>>>(a, f, K);
  else nucleus_kernel<false, C><<<rows, C::T, smem, stream>>>(a, f, K);
  return cudaGetLastError() == cudaSuccess ? 0 : 5;
}

// Rows that fit one wave of SMs run one 1024-thread CTA per SM; more rows run
// two 512-thread CTAs per SM where two fit (else the one-CTA shape again).
inline int launch_nucleus(const FvScratch& f, SampleArgs a, int rows, int K, int max_smem,
                          int num_sms, cudaStream_t stream) {
  if (a.V > f.max_vocab) return 8;  // NCB_ERROR_CAPACITY
  a.seg_len = a.V;
  a.bm_words = (a.V + 31) / 32 + 1;
  const bool counts = (a.p.frequency_penalty != 0.0f || a.p.presence_penalty != 0.0f);
  const int h_cap = counts ? a.h_cap : 0;
  const size_t smem_two = nc_smem_bytes<NcTwo>(a.bm_words, h_cap);
  int st;
  if (rows > num_sms && smem_two <= NC_TWO_SMEM_MAX) {
    st = launch_nucleus_shape<NcTwo>(f, a, rows, K, smem_two, stream);
  } else {
    const size_t smem = nc_smem_bytes<NcOne>(a.bm_words, h_cap);
    if ((int)smem > max_smem) return 8;  // NCB_ERROR_CAPACITY
    st = launch_nucleus_shape<NcOne>(f, a, rows, K, smem, stream);
  }
  if (st != 0) return st;
  // rows a check handed over
  return launch_fullvocab(f, a, rows, K, max_smem, stream, true, 8);
}

}  // namespace nvs
