// Device building blocks of the sm_100a sampling kernels.
//
// Everything that decides a token is written with explicit IEEE round-to-
// nearest intrinsics (__fmul_rn/__fdiv_rn/__fsub_rn/__fadd_rn) so the results
// match the fp32 arithmetic of Neuraval/Generation/TokenSampler.cs bit for bit;
// the library is also compiled with -fmad=false.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nvs {

constexpr uint32_t FLAG_DRAW_BOUNDARY = 0x1u;
constexpr uint32_t FLAG_CUTOFF_BOUNDARY = 0x2u;
constexpr uint32_t FLAG_TIE_AT_DRAW = 0x4u;
constexpr uint32_t FLAG_NONFINITE = 0x8u;
constexpr uint32_t FLAG_EXP_SLOW = 0x10u;
constexpr uint32_t FLAG_BAD_HISTORY = 0x20u;
constexpr uint32_t FLAG_TIES_OVERFLOW = 0x40u;
// internal row states carried in scratch between kernels (never returned)
constexpr uint32_t RSTATE_OVERFLOW = 0x100u;  // candidates (ties) exceed the top-k buffers
constexpr uint32_t RSTATE_TIMEOUT = 0x200u;   // a bounded wait gave up

struct Params {
  int32_t greedy;
  float temperature;
  float top_p;
  int32_t top_k;
  float repetition_penalty;
  float frequency_penalty;
  float presence_penalty;
};

// ---------------------------------------------------------------------------
// Order-preserving keys. Values are canonicalised first (-0 -> +0, as C#'s
// float.CompareTo treats them as equal), so equal values have equal keys.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float canon(float v) { return __fadd_rn(v, 0.0f); }

__device__ __forceinline__ uint32_t fkey(float v) {
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
// fkey packed into a float's bits / back, so atomicMin on the bits orders by value
__device__ __forceinline__ float fkey_as_float(float v) { return __uint_as_float(fkey(v)); }
__device__ __forceinline__ float kval(uint32_t k);
__device__ __forceinline__ float kval_from_float(float k) { return kval(__float_as_uint(k)); }
__device__ __forceinline__ float kval(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}
// descending (value, then ascending id) as one descending 64-bit key
__device__ __forceinline__ uint64_t cand_key(float v, int32_t id) {
  return ((uint64_t)fkey(v) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)id);
}
__device__ __forceinline__ int32_t cand_id(uint64_t k) {
  return (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu));
}
__device__ __forceinline__ float cand_val(uint64_t k) { return kval((uint32_t)(k >> 32)); }

// ---------------------------------------------------------------------------
// Correctly rounded expf.
// CUDA's double exp() (max error 1 ulp) rounded to float is correct unless the
// double result lies within 2^-51 relative of a float rounding midpoint; those
// rare arguments take a double-double evaluation (relative error < 2^-90).
// ---------------------------------------------------------------------------
struct dd {
  double hi, lo;
};
__device__ __forceinline__ dd dd_two_sum(double a, double b) {
  double s = __dadd_rn(a, b);
  double bb = __dsub_rn(s, a);
  double e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
  return {s, e};
}
__device__ __forceinline__ dd dd_fast_two_sum(double a, double b) {
  double s = __dadd_rn(a, b);
  return {s, __dsub_rn(b, __dsub_rn(s, a))};
}
__device__ __forceinline__ dd dd_add(dd a, dd b) {
  dd s = dd_two_sum(a.hi, b.hi);
  dd t = dd_two_sum(a.lo, b.lo);
  s.lo = __dadd_rn(s.lo, t.hi);
  s = dd_fast_two_sum(s.hi, s.lo);
  s.lo = __dadd_rn(s.lo, t.lo);
  return dd_fast_two_sum(s.hi, s.lo);
}
__device__ __forceinline__ dd dd_mul(dd a, dd b) {
  double p = __dmul_rn(a.hi, b.hi);
  double e = __fma_rn(a.hi, b.hi, -p);
  e = __dadd_rn(e, __dadd_rn(__dmul_rn(a.hi, b.lo), __dmul_rn(a.lo, b.hi)));
  return dd_fast_two_sum(p, e);
}

// exp(x) = 2^k * (Taylor(r/256))^256 with x = k*ln2 + r; ln2 is split into two
// 40-bit heads and a tail so that k*head is exact for |k| < 2^13.
__device__ __noinline__ dd dd_exp(double x) {
  const double LN2_A = 0x1.62e42fefa4000p-1;
  const double LN2_B = -0x1.8432a1b0e2000p-43;
  const double LN2_C = -0x1.8cff81a12a17ep-85;
  const double INV_LN2 = 0x1.71547652b82fep+0;
  double k = rint(__dmul_rn(x, INV_LN2));
  dd r = dd_two_sum(__fma_rn(-k, LN2_A, x), __dmul_rn(-k, LN2_B));
  r = dd_add(r, dd{__dmul_rn(-k, LN2_C), 0.0});
  dd s{scalbn(r.hi, -8), scalbn(r.lo, -8)};
  dd acc{1.0, 0.0};
  for (int n = 11; n >= 1; --n) {
    acc = dd_mul(acc, s);
    double q = __ddiv_rn(acc.hi, (double)n);
    double rem = __dadd_rn(__fma_rn(-q, (double)n, acc.hi), acc.lo);
    dd t = dd_fast_two_sum(q, __ddiv_rn(rem, (double)n));
    acc = dd_add(t, dd{1.0, 0.0});
  }
  for (int i = 0; i < 8; ++i) acc = dd_mul(acc, acc);
  int ki = (int)k;
  return {scalbn(acc.hi, ki), scalbn(acc.lo, ki)};
}

__device__ __forceinline__ float next_float_toward(float f, bool up) {
  uint32_t u = __float_as_uint(f);  // f >= 0
  if (up) u += 1u;
  else if (u > 0u) u -= 1u;
  return __uint_as_float(u);
}

__device__ __noinline__ float dd_to_float(dd v) {
  float f = __double2float_rn(v.hi);
  double fd = (double)f;
  double res = __dadd_rn(__dsub_rn(v.hi, fd), v.lo);
  if (res == 0.0) return f;
  float nb = next_float_toward(f, res > 0.0);
  double mid = __dmul_rn(__dadd_rn(fd, (double)nb), 0.5);
  double side = __dadd_rn(__dsub_rn(v.hi, mid), v.lo);
  if ((res > 0.0 && side > 0.0) || (res < 0.0 && side < 0.0)) return nb;
  return f;
}

// x <= 0 or any finite x; returns the correctly rounded float of e^x.
__device__ __forceinline__ float exp_cr(float x, bool& slow) {
  if (x != x) return x;
  double y = exp((double)x);
  float f = __double2float_rn(y);
  if (y == 0.0 || isinf(f)) return f;
  double fd = (double)f;
  double d = __dsub_rn(y, fd);
  if (d == 0.0) return f;
  float nb = next_float_toward(f, d > 0.0);
  double mid = __dmul_rn(__dadd_rn(fd, (double)nb), 0.5);
  if (fabs(__dsub_rn(y, mid)) > __dmul_rn(0x1p-51, y)) return f;
  slow = true;
  return dd_to_float(dd_exp((double)x));
}

// ---------------------------------------------------------------------------
// Penalties: TokenSampler.AdjustLogit (TokenSampler.cs:137-143) plus the new
// frequency/presence term. Membership comes from a bitmap over the CTA's column
// range; occurrence counts from the range's history ids, sorted in smem.
// ---------------------------------------------------------------------------
struct Penalty {
  const uint32_t* bitmap;   // bit (id - c0)
  const int32_t* hsorted;   // ascending ids in [c0,c1) (counts only)
  int hn;
  int c0;
  bool rep;
  bool cnt;
  float pen, freq, pres;
};

__device__ __forceinline__ int count_in_sorted(const int32_t* a, int n, int32_t id) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (a[mid] < id) lo = mid + 1; else hi = mid;
  }
  int first = lo;
  hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (a[mid] <= id) lo = mid + 1; else hi = mid;
  }
  return lo - first;
}

// Penalty bits of ids col..col+3 (the bitmap has one spare word at the end).
__device__ __forceinline__ uint32_t penalty_bits4(const Penalty& P, int col) {
  const int rel = col - P.c0;
  const int w = rel >> 5, sh = rel & 31;
  const uint64_t win = (uint64_t)P.bitmap[w] | ((uint64_t)P.bitmap[w + 1] << 32);
  return (uint32_t)(win >> sh) & 0xFu;
}

// Value before the temperature scale.
__device__ __forceinline__ float adjust(const Penalty& P, float l, int id) {
  float v = l;
  if (P.rep || P.cnt) {
    int rel = id - P.c0;
    if ((P.bitmap[rel >> 5] >> (rel & 31)) & 1u) {
      if (P.rep) v = (v > 0.0f) ? __fdiv_rn(v, P.pen) : __fmul_rn(v, P.pen);
      if (P.cnt) {
        int c = count_in_sorted(P.hsorted, P.hn, id);
        v = __fsub_rn(v, __fmul_rn((float)c, P.freq));
        v = __fsub_rn(v, P.pres);
      }
    }
  }
  return v;
}

// ---------------------------------------------------------------------------
// CTA-wide helpers (blockDim.x threads, all participate)
// ---------------------------------------------------------------------------
template <typename T>
__device__ void cta_bitonic_sort_asc(T* a, int n_pow2) {
  for (int k = 2; k <= n_pow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
        int ixj = i ^ j;
        if (ixj > i) {
          T x = a[i], y = a[ixj];
          bool up = (i & k) == 0;
          if ((x > y) == up) { a[i] = y; a[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
}
template <typename T>
__device__ void cta_bitonic_sort_desc(T* a, int n_pow2) {
  for (int k = 2; k <= n_pow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
        int ixj = i ^ j;
        if (ixj > i) {
          T x = a[i], y = a[ixj];
          bool down = (i & k) == 0;
          if ((x < y) == down) { a[i] = y; a[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int next_pow2(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// Radix select over keys: the k-th largest key (counting multiplicity) among
// getKey(0..n) with key 0 meaning "not an element" (only the all-ones NaN maps
// to 0 under fkey, and callers replace NaNs). Returns 0 (keep everything) when
// fewer than k elements exist. 8 bits per pass; `hist` = 256 words of smem,
// `sh` = 2 ints of smem. Ends with a __syncthreads().
// With passes < 4 the result is the k-th largest key with its low bits
// cleared: a lower bound of it (what a threshold filter needs).
template <typename GetKey>
__device__ uint32_t cta_kth_largest(GetKey getKey, int n, int k, uint32_t* hist, int* sh,
                                    int passes = 4) {
  if (k <= 0) return 0u;
  uint32_t prefix = 0u, mask = 0u;
  int krem = k;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll 1
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = getKey(i);
      if (key != 0u && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
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
        int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      if (lane == 0 && total < krem) {
        sh[0] = -1;  // fewer than k elements (only possible on the first pass)
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

// k-th largest value's key over the union of two float arrays.
template <typename GetA, typename GetB>
__device__ uint32_t cta_kth_largest_key(GetA getA, int na, GetB getB, int nb, int k,
                                        uint32_t* hist, int* sh) {
  return cta_kth_largest([&](int i) { return fkey(i < na ? getA(i) : getB(i - na)); }, na + nb,
                         k, hist, sh);
}

// ---------------------------------------------------------------------------
// Bulk-async (TMA engine) copies global -> shared with mbarrier completion.
// Every copy lands in the issuing CTA's own shared memory, from this GPU's memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// try_wait suspends the calling thread until the phase completes or the
// suspend-time hint (ns) runs out, so a waiting warp sleeps instead of
// spinning and leaves issue slots to the warps that have data.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0u;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait (about 2 s of wall time); false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > 2000000000ull) return false;
  }
}

}  // namespace nvs
