// Chunked top-k sampling for k <= 64 over wide rows (sm_100a): two kernels.
//
// TokenSampler.SampleFiltered (TokenSampler.cs:54-135) needs, per row, the
// K-th largest adjusted value, every value >= it (ties included) in
// descending order, and the sequential fp32 sums over their weights. The
// one-CTA-per-row kernel (topk_ldg_kernel) pays a per-row head (history,
// sample threshold) and tail before and after its stream, and with whole rows
// per CTA the SMs that hold two rows stream twice the bytes of the others.
// Here the stream and the selection are separate launches:
//
//  1. topk_chunk_kernel: the rows are cut into chunks of at most 2048 float4
//     (32 KiB), one short CTA of 256 threads per chunk, every thread with its
//     eight 128-bit loads in flight at once. The hardware block scheduler
//     hands chunks to SMs as slots free up, so every SM streams about the same
//     bytes, and no CTA waits for anything before its loads. Each warp (1024
//     values) keeps every raw value >= the 8th largest of its 32 lane maxima
//     (at least its 8 largest values; the 4th largest lane maximum when that
//     would keep more than 16). Whatever it drops is below its smallest kept
//     value. No history, no temperature: penalties that can only lower a
//     value (repetition >= 1, frequency and presence >= 0) and the positive
//     temperature scale keep the order of the raw values as an upper bound.
//  2. topk_chunk_finish_kernel: one CTA per row gathers the row's kept
//     values, applies the exact penalties and temperature (AdjustLogit,
//     TokenSampler.cs:137-143, then *1/T, :68-71), takes the K-th largest T
//     of those, and proves it is the row's K-th largest: every value a warp
//     dropped is at most (prev(smallest kept) * scale) after any lowering
//     penalty, and that bound must lie below T. A row that fails the proof
//     (a warp holding more than 8 of the row's top K, too many ties, rows
//     with fewer than K finite values) is marked for the exact
//     full-vocabulary fix-up kernel that runs after it. The candidates >= T
//     are ranked (value desc, id asc), weighted exp(v - max) with the
//     correctly rounded exp, and one warp runs the sequential sums, top-p
//     cutoff and draw (finish_weights_warp).
//
// Both kernels are programmatic dependent launches: each waits
// (griddepcontrol.wait) for its predecessor before reading anything.
#pragma once

#include "sampler_device.cuh"
#include "topk_kernels.cuh"
#include "warp_select.cuh"

namespace nvs {

constexpr int CK_THREADS = 256;
constexpr int CK_WARPS = CK_THREADS / 32;
constexpr int CK_LOADS = 8;                        // float4 loads in flight per thread
constexpr int CK_F4 = CK_THREADS * CK_LOADS;       // float4 per chunk at most
constexpr int CK_KEYS = 16;                        // kept values per warp (group) at most
constexpr int CK_RANK = 8;                         // cutoff: this largest lane maximum
constexpr int CK_MAX_CHUNKS = 32;                  // chunks per row (vocab <= 262144)
constexpr int CK_GROUPS_MAX = CK_MAX_CHUNKS * CK_WARPS;
constexpr int FK_THREADS = 512;
constexpr int FK_CAND = 256;                       // candidates ranked by the finish
// group words: kept count in the low 16 bits, and
constexpr uint32_t CK_W_NONFINITE = 0x40000000u;   // a NaN or +inf among the raw values
constexpr uint32_t CK_W_ALLKEPT = 0x20000000u;     // every finite value kept (nothing dropped)
constexpr uint32_t CK_W_OVERFLOW = 0x10000000u;    // more than CK_KEYS values to keep

// Chunks per row for `width` columns (the float4 body is split evenly).
__host__ __device__ inline int ck_chunks(int width) {
  const int n4 = width / 4;
  return n4 <= CK_F4 ? 1 : (n4 + CK_F4 - 1) / CK_F4;
}

// max with NaN propagation (max.NaN.f32): a NaN anywhere reaches the lane maximum
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

template <bool kShard = false>
__global__ void __launch_bounds__(CK_THREADS, 4) topk_chunk_kernel(const __grid_constant__ SampleArgs a) {
  // the logits may be written by the kernel before this one on the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the finish kernel may be scheduled now; it waits for this grid to complete
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = blockIdx.x, J = gridDim.x, row = blockIdx.y;
  const int lo = kShard ? a.col_lo : 0, hi = kShard ? a.col_hi : a.V;
  // shard rows are addressed by global column: lrow[c] for c in [lo, hi)
  const float* lrow = kShard ? a.logits + (size_t)row * a.ld - lo : a.logits + (size_t)row * a.V;
  // 16-byte aligned body [a0, a1) as float4, split evenly over the J chunks
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)(lrow + lo) & 15u)) & 15u) >> 2);
  const int a0 = min(lo + head, hi);
  const int n4 = (hi - a0) >> 2;
  const int a1 = a0 + 4 * n4;
  const int q0 = (int)((long long)j * n4 / J), q1 = (int)((long long)(j + 1) * n4 / J);
  const float4* body = reinterpret_cast<const float4*>(lrow + a0);
  float4 x[CK_LOADS];
#pragma unroll
  for (int u = 0; u < CK_LOADS; ++u) {
    const int q = q0 + warp * 32 + lane + u * CK_THREADS;
    x[u] = q < q1 ? __ldcs(body + q) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
  // the <= 3 head and <= 3 tail scalars: one extra value on lanes of chunk 0's warp 0
  float xs = -INFINITY;
  int cs = 0;
  if (j == 0 && warp == 0) {
    const int nh = a0 - lo, nt = hi - a1;
    if (lane < nh + nt) {
      cs = lane < nh ? lo + lane : a1 + (lane - nh);
      xs = lrow[cs];
    }
  }
  float m = xs;
#pragma unroll
  for (int u = 0; u < CK_LOADS; ++u)
    m = fmax_nan(fmax_nan(fmax_nan(m, x[u].x), fmax_nan(x[u].y, x[u].z)), x[u].w);
  const size_t g = ((size_t)row * J + j) * CK_WARPS + warp;
  uint2* keys = a.s.ck_keys + g * CK_KEYS;
  uint32_t word;
  if (__any_sync(0xffffffffu, !(m < INFINITY))) {
    word = CK_W_NONFINITE;
  } else {
    // t0: the CK_RANK-th largest lane maximum (bitonic sort across lanes, descending)
    float s = m;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
      for (int jj = k >> 1; jj > 0; jj >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, s, jj);
        const bool desc = (lane & k) == 0, lower = (lane & jj) == 0;
        s = (desc == lower) ? fmaxf(s, o) : fminf(s, o);
      }
    // kept: finite values >= t (t == -inf: fewer than CK_RANK lanes hold a
    // finite value, and every finite value is kept)
    auto count_kept = [&](float t, int& excl) {
      auto keep = [&](float v) { return v >= t && v > -INFINITY; };
      int c = keep(xs) ? 1 : 0;
#pragma unroll
      for (int u = 0; u < CK_LOADS; ++u)
        c += (keep(x[u].x) ? 1 : 0) + (keep(x[u].y) ? 1 : 0) + (keep(x[u].z) ? 1 : 0) +
             (keep(x[u].w) ? 1 : 0);
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t2 = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t2;
      }
      excl = incl - c;
      return __shfl_sync(0xffffffffu, incl, 31);
    };
    float t0 = __shfl_sync(0xffffffffu, s, CK_RANK - 1);
    int excl;
    int total = count_kept(t0, excl);
    if (total > CK_KEYS) {
      // rare: more than CK_KEYS values reach the 8th lane maximum; the 4th
      // keeps fewer (the finish still proves or redoes the row)
      t0 = __shfl_sync(0xffffffffu, s, CK_RANK / 2 - 1);
      total = count_kept(t0, excl);
    }
    if (total > CK_KEYS) {
      word = CK_W_OVERFLOW | (uint32_t)min(total, 0xFFFF);
    } else {
      auto keep = [&](float v) { return v >= t0 && v > -INFINITY; };
      int pos = excl;
      if (keep(xs)) keys[pos++] = make_uint2(__float_as_uint(xs), (uint32_t)cs);
#pragma unroll
      for (int u = 0; u < CK_LOADS; ++u) {
        const int col = a0 + 4 * (q0 + warp * 32 + lane + u * CK_THREADS);
        if (keep(x[u].x)) keys[pos++] = make_uint2(__float_as_uint(x[u].x), (uint32_t)col);
        if (keep(x[u].y)) keys[pos++] = make_uint2(__float_as_uint(x[u].y), (uint32_t)(col + 1));
        if (keep(x[u].z)) keys[pos++] = make_uint2(__float_as_uint(x[u].z), (uint32_t)(col + 2));
        if (keep(x[u].w)) keys[pos++] = make_uint2(__float_as_uint(x[u].w), (uint32_t)(col + 3));
      }
      word = (uint32_t)total | (t0 == -INFINITY ? CK_W_ALLKEPT : 0u);
    }
  }
  if (lane == 0) a.s.ck_cnt[g] = word;
}

// float just below x (x finite): the largest float < x
__device__ __forceinline__ float prev_float(float x) {
  if (x == 0.0f) return -1.40129846e-45f;
  const uint32_t b = __float_as_uint(x);
  return __uint_as_float(x > 0.0f ? b - 1u : b + 1u);
}

inline size_t fk_smem_bytes(int bm_words, int h_cap) {
  return (size_t)FK_THREADS * 4          // the groups' largest exact values
         + (size_t)FK_CAND * 8 * 2       // candidate keys, then in rank order
         + 128 * 4                       // weights and scratch of the finish
         + (size_t)bm_words * 4 + (size_t)h_cap * 4;
}

// FK_SLOTS key slots per thread: J * CK_WARPS * CK_KEYS <= FK_SLOTS * FK_THREADS.
template <bool kCounts, int FK_SLOTS>
__global__ void __launch_bounds__(FK_THREADS, 2) topk_chunk_finish_kernel(const __grid_constant__ SampleArgs a, int J) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* gtop = reinterpret_cast<float*>(smem);                        // [FK_THREADS]
  uint64_t* cand = reinterpret_cast<uint64_t*>(gtop + FK_THREADS);     // [FK_CAND]
  uint64_t* sorted = cand + FK_CAND;                                   // [FK_CAND]
  float* w = reinterpret_cast<float*>(sorted + FK_CAND);               // [64] weights
  float* wS = w + 64;                                                  // [64]
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(wS + 64);
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);
  __shared__ int s_hn, s_nc, s_flags, s_c;
  __shared__ uint32_t s_bkey, s_any;
  __shared__ float s_L, s_u;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int V = a.V;
  const int K = min(a.p.top_k, V);
  const int G = J * CK_WARPS;
  // each group contributes its M largest exact values to the lower bound of
  // the K-th value (G * M >= K distinct elements)
  const int M = (K + G - 1) / G;
  const float scale = __fdiv_rn(1.0f, a.p.temperature);  // TokenSampler.cs:68
  const size_t gbase = (size_t)row * G;

  // the row's kept values (every slot of every group; counts mask them below)
  uint2 kv[FK_SLOTS];
  uint32_t gw[FK_SLOTS];
#pragma unroll
  for (int k = 0; k < FK_SLOTS; ++k) {
    const int s = tid + k * FK_THREADS, gi = s / CK_KEYS;
    if (gi < G) {
      kv[k] = __ldcg(a.s.ck_keys + (gbase + gi) * CK_KEYS + (s % CK_KEYS));
      gw[k] = __ldcg(a.s.ck_cnt + gbase + gi);
    } else {
      kv[k] = make_uint2(0u, 0u);
      gw[k] = 0u;
    }
  }
  if (tid == 0) {
    s_nc = 0;
    s_flags = 0;
    s_c = 0;
    s_bkey = 0u;
    s_any = 0u;
    s_u = a.uniforms[row];
  }
  Penalty P;
  const bool hist_ok =
      setup_penalty_range<kCounts>(P, a, a.hoff[row], a.hoff[row + 1], 0, V, bitmap, hsorted, &s_hn);

  // exact values of the kept slots; per group (16 consecutive threads) the
  // largest exact value and the bound of what the group dropped
  uint32_t any = 0u;  // bit 0 nonfinite group, bit 1 overflow, bit 2 exact +inf
  float v[FK_SLOTS];
#pragma unroll
  for (int k = 0; k < FK_SLOTS; ++k) {
    const int s = tid + k * FK_THREADS, gi = s / CK_KEYS, e = s % CK_KEYS;
    const uint32_t word = gw[k];
    const bool valid = gi < G && !(word & (CK_W_NONFINITE | CK_W_OVERFLOW)) &&
                       e < (int)(word & 0xFFFFu);
    if (gi < G && e == 0) {
      if (word & CK_W_NONFINITE) any |= 1u;
      if (word & CK_W_OVERFLOW) any |= 2u;
    }
    float ev = -INFINITY, raw = INFINITY;
    if (valid) {
      raw = __uint_as_float(kv[k].x);
      ev = canon(__fmul_rn(adjust(P, raw, (int)kv[k].y), scale));
      if (!(ev < INFINITY)) any |= 4u;  // scaled past the float range, as the reference's value
    }
    v[k] = ev;
    float gm = ev, tmin = raw;
    int em = e;  // the slot of the group's largest value (lowest slot among equals)
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      const float og = __shfl_xor_sync(0xffffffffu, gm, o);
      const int oe = __shfl_xor_sync(0xffffffffu, em, o);
      if (og > gm || (og == gm && oe < em)) {
        gm = og;
        em = oe;
      }
      tmin = fminf(tmin, __shfl_xor_sync(0xffffffffu, tmin, o));
    }
    float g2 = e == em ? -INFINITY : ev;  // the second largest (M == 2)
    if (M > 1) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) g2 = fmaxf(g2, __shfl_xor_sync(0xffffffffu, g2, o));
    }
    if (gi < G && e == 0) {
      if (M <= 2 && gi * M < FK_THREADS) {
        gtop[gi * M] = gm;
        if (M == 2) gtop[gi * M + 1] = g2;
      }
      // a group that dropped values: they are < its smallest kept raw value
      if (!(word & (CK_W_NONFINITE | CK_W_OVERFLOW | CK_W_ALLKEPT)) && tmin < INFINITY) {
        const float b = canon(__fmul_rn(prev_float(tmin), scale));
        atomicMax(&s_bkey, fkey(b));
      }
    }
  }
  any = __reduce_or_sync(0xffffffffu, any);
  if (lane == 0 && any) atomicOr(&s_any, any);
  __syncthreads();
  const uint32_t anyall = s_any;
  uint32_t state = 0u;
  if (!hist_ok) state = FLAG_BAD_HISTORY;
  else if (anyall & 5u) state = FLAG_NONFINITE;
  if (state) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = state;
    }
    return;
  }
  const int NT = G * M;
  bool fallback = (anyall & 2u) != 0u || M > 2 || NT > FK_THREADS;
  // L: the K-th largest of the groups' M largest values (distinct elements,
  // so a lower bound of the row's K-th largest value)
  if (!fallback) {
    if (tid < NT) {
      const float x = gtop[tid];
      int r = 0;
      for (int h = 0; h < NT; ++h) {
        const float y = gtop[h];
        r += (y > x) || (y == x && h < tid);
      }
      if (r == K - 1) s_L = x;
    }
    __syncthreads();
    const float L = s_L;
    if (!(L > -INFINITY)) {
      fallback = true;  // fewer than K finite values: the exact path decides
    } else {
      // candidates: kept values >= L, as descending (value, id asc) keys
#pragma unroll
      for (int k = 0; k < FK_SLOTS; ++k) {
        const bool ok = v[k] >= L;
        const unsigned b = __ballot_sync(0xffffffffu, ok);
        if (b) {
          const int leader = __ffs(b) - 1;
          int base = 0;
          if (lane == leader) base = atomicAdd(&s_nc, __popc(b));
          base = __shfl_sync(0xffffffffu, base, leader);
          const int slot = base + __popc(b & ((1u << lane) - 1u));
          if (ok && slot < FK_CAND) cand[slot] = cand_key(v[k], (int)kv[k].y);
        }
      }
      __syncthreads();
      const int nc = s_nc;
      if (nc > FK_CAND || nc < K) {
        fallback = true;
      } else {
        // rank sort: the keys are distinct (ids are)
        if (tid < nc) {
          const uint64_t key = cand[tid];
          int r = 0;
          for (int h = 0; h < nc; ++h) r += cand[h] > key;
          sorted[r] = key;
        }
        __syncthreads();
        const uint64_t kth = sorted[K - 1];
        const uint32_t tk = (uint32_t)(kth >> 32);
        // every dropped value lies below the K-th value: it is the row's
        if (s_bkey >= tk) {
          fallback = true;
        } else {
          // the candidates: everything >= the K-th value (ties included)
          if (tid >= K - 1 && tid < nc) {
            const bool in = (uint32_t)(sorted[tid] >> 32) == tk;
            const bool next_out = tid + 1 >= nc || (uint32_t)(sorted[tid + 1] >> 32) != tk;
            if (in && next_out) s_c = tid + 1;
          }
          __syncthreads();
          const int c = s_c;
          if (c > 64) {
            fallback = true;
          } else {
            const float vmax = cand_val(sorted[0]);
            bool slow = false;
            if (tid < c) w[tid] = exp_cr(__fsub_rn(cand_val(sorted[tid]), vmax), slow);
            if (__any_sync(0xffffffffu, slow) && lane == 0) atomicOr(&s_flags, 1);
            __syncthreads();
            if (warp == 0) {
              const uint64_t k0 = lane < c ? sorted[lane] : 0ull;
              const uint64_t k1 = lane + 32 < c ? sorted[lane + 32] : 0ull;
              finish_weights_warp(a, row, k0, k1, c, w, wS, s_flags != 0, s_u);
            }
            return;
          }
        }
      }
    }
  }
  // the exact full-vocabulary kernel launched after this one redoes the row
  if (fallback && tid == 0) a.s.fixup[row] = 1u;
}

}  // namespace nvs
