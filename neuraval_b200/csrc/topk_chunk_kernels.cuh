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
// the three-input form (sm_100)
__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// all ones when a >= b, else zero (set.ge.u32.f32; false when either is NaN)
__device__ __forceinline__ uint32_t fge_mask(float a, float b) {
  uint32_t d;
  asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(d) : "f"(a), "f"(b));
  return d;
}

// One warp group of 1024 values: lane l holds x[u] = the float4 at index
// l + 32 u of the group (missing ones are -inf), also staged at sp (as
// floats), whose first column is col0; plus one optional scalar xs at column
// cs. Keeps every finite value >= the CK_RANK-th largest lane maximum (the
// CK_RANK/2-th when that would keep more than CK_KEYS), writes them to keys[]
// and the cutoff to *cut, and returns the group
// word. All 32 lanes call; sp must stay valid until the call returns.
__device__ __forceinline__ uint32_t ck_group(const float4 (&x)[CK_LOADS], const float* sp,
                                             float xs, int cs, int col0, uint2* keys,
                                             float* cut) {
  static_assert(CK_LOADS == 8, "the maximum tree below reads eight float4");
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  // lane maximum of the 32 values and xs: a tree of three-input maxima
  float t[11];
#pragma unroll
  for (int u = 0; u < 8; ++u) t[u] = fmax3_nan(x[u].x, x[u].y, x[u].z);
  t[8] = fmax3_nan(x[0].w, x[1].w, x[2].w);
  t[9] = fmax3_nan(x[3].w, x[4].w, x[5].w);
  t[10] = fmax3_nan(x[6].w, x[7].w, xs);
  const float m = fmax3_nan(fmax3_nan(t[0], t[1], t[2]), fmax3_nan(t[3], t[4], t[5]),
                            fmax3_nan(fmax3_nan(t[6], t[7], t[8]), t[9], t[10]));
  if (__any_sync(0xffffffffu, !(m < INFINITY))) return CK_W_NONFINITE;
  // the CK_RANK-th and CK_RANK/2-th largest lane maxima, counted with
  // multiplicity (order-preserving keys): each round takes the largest
  // remaining maximum and every lane holding it, until CK_RANK are counted
  uint32_t key = fkey(m);
  uint32_t k4 = 0u, k8 = 0u;
  int taken = 0;
#pragma unroll
  for (int r = 0; r < CK_RANK; ++r) {
    if (taken < CK_RANK) {
      const uint32_t mx = __reduce_max_sync(0xffffffffu, key);
      const bool mine = key == mx;
      const int now = taken + __popc(__ballot_sync(0xffffffffu, mine));
      if (mine) key = 0u;
      if (taken < CK_RANK / 2 && now >= CK_RANK / 2) k4 = mx;
      if (now >= CK_RANK) k8 = mx;
      taken = now;
    }
  }
  for (int pass = 0; pass < 2; ++pass) {
    const float t0 = kval(pass == 0 ? k8 : k4);
    // kept: finite values >= t0 (t0 == -inf: fewer lanes than the rank hold a
    // finite value, and every finite value is kept); no value here is NaN or
    // +inf, so "finite and >= t0" is ">= max(t0, lowest float)"
    const float tf = fmaxf(t0, -3.40282347e+38f);
    uint32_t mask = 0u;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      mask |= fge_mask(x[u].x, tf) & (1u << (4 * u));
      mask |= fge_mask(x[u].y, tf) & (1u << (4 * u + 1));
      mask |= fge_mask(x[u].z, tf) & (1u << (4 * u + 2));
      mask |= fge_mask(x[u].w, tf) & (1u << (4 * u + 3));
    }
    const bool ks = xs >= tf;
    const int c = __popc(mask) + (ks ? 1 : 0);  // <= 33
    const int total = __reduce_add_sync(0xffffffffu, (unsigned)c);
    if (total > CK_KEYS) continue;
    // exclusive prefix of c (<= CK_KEYS here) over the lanes, from its bits
    int pos = 0;
#pragma unroll
    for (int b = 0; b < 5; ++b) pos += __popc(__ballot_sync(0xffffffffu, (c >> b) & 1) & lt) << b;
    if (ks) keys[pos++] = make_uint2(__float_as_uint(xs), (uint32_t)cs);
    while (mask) {
      const int k = __ffs(mask) - 1;
      mask &= mask - 1u;
      const int f = 4 * (lane + 32 * (k >> 2)) + (k & 3);  // float index within the group
      keys[pos++] = make_uint2(__float_as_uint(sp[f]), (uint32_t)(col0 + f));
    }
    *cut = t0;
    return (uint32_t)total | (t0 == -INFINITY ? CK_W_ALLKEPT : 0u);
  }
  return CK_W_OVERFLOW | 0xFFFFu;
}

// Geometry of one row's columns [lo, hi) at base lrow (lrow[c] is column c):
// the 16-byte aligned float4 body [a0, a0 + 4 n4) and the <= 3 + 3 scalars
// around it.
struct CkRow {
  int a0, n4;
};
__device__ __forceinline__ CkRow ck_row(const float* lrow, int lo, int hi) {
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)(lrow + lo) & 15u)) & 15u) >> 2);
  CkRow r;
  r.a0 = min(lo + head, hi);
  r.n4 = (hi - r.a0) >> 2;
  return r;
}

// The stream: one CTA per SM, each over a contiguous share of the batch's
// chunks (chunk t = row t / J, part t % J of the row's float4 body). A
// producer warp keeps CR_STAGES 32 KiB bulk copies (cp.async.bulk, this GPU's
// memory into this CTA's shared memory, mbarrier completion) in flight; three
// teams of 8 consumer warps take the stages in turn (team t the stages i with
// i % 3 == t), one 1024-value group per warp. Every wait is
// bounded (about 2 s); a wait that gives up marks the chunk's groups so the
// finish returns -1 for the row, and sets the error word.
// mbarrier wait without a suspend-time hint, bounded by %globaltimer (about
// 2 s); false when it gave up
__device__ __forceinline__ bool cr_wait(uint64_t* bar, uint32_t parity) {
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 63) == 0) {
      const uint64_t t = global_ns();
      if (it == 0) t0 = t;
      else if (t - t0 > 2000000000ull) return false;
    }
  }
}
// global -> own shared memory bulk copy with an L2 evict-first policy: the
// streamed logits must not push the kept values out of L2
__device__ __forceinline__ void cr_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                        uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

constexpr int CR_STAGES = 6;
constexpr int CR_TEAMS = 3;
constexpr int CR_CONSUMERS = 8 * CR_TEAMS;
constexpr int CR_THREADS = (CR_CONSUMERS + 1) * 32;
constexpr uint32_t CK_W_TIMEOUT = 0x08000000u;  // a stage never arrived (group word)
inline size_t cr_smem_bytes() { return (size_t)CR_STAGES * CK_F4 * 16 + 2 * CR_STAGES * 8; }

template <bool kShard = false>
__global__ void __launch_bounds__(CR_THREADS, 1) topk_chunk_kernel(const __grid_constant__ SampleArgs a, int J,
                                                                   int nchunks) {
  extern __shared__ __align__(128) unsigned char smem[];
  float4* stage = reinterpret_cast<float4*>(smem);                           // [STAGES][CK_F4]
  uint64_t* full = reinterpret_cast<uint64_t*>(stage + CR_STAGES * CK_F4);   // [STAGES]
  uint64_t* empty = full + CR_STAGES;                                        // [STAGES]
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0c = (int)((long long)blockIdx.x * nchunks / gridDim.x);
  const int t1c = (int)((long long)(blockIdx.x + 1) * nchunks / gridDim.x);
  const int n = t1c - t0c;
  const int lo = kShard ? a.col_lo : 0, hi = kShard ? a.col_hi : a.V;
  if (tid == 0) {
    for (int i = 0; i < CR_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CK_WARPS);  // the 8 warps of the team that read it
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  // the logits may be written by the kernel before this one on the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the finish kernel may be scheduled now; it waits for this grid to complete
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // chunk (row, j): part j of the row's float4 body, [q0, q1). Callers walk
  // the chunks with a fixed stride and carry (row, j) along (no division by J
  // per chunk); j * n4 stays below 2^32 (J <= CK_MAX_CHUNKS, n4 < 2^26).
  auto chunk = [&](int row, int j, const float*& lrow, int& q0, int& q1, CkRow& g) {
    lrow = kShard ? a.logits + (size_t)row * a.ld - lo : a.logits + (size_t)row * a.V;
    g = ck_row(lrow, lo, hi);
    q0 = (int)(((uint32_t)j * (uint32_t)g.n4) / (uint32_t)J);
    q1 = (int)(((uint32_t)(j + 1) * (uint32_t)g.n4) / (uint32_t)J);
  };
  // (row, j) of chunk t0c + first, advanced by `stride` chunks
  auto first_chunk = [&](int first, int& row, int& j) {
    row = (t0c + first) / J;
    j = t0c + first - row * J;
  };
  auto advance = [&](int stride, int& row, int& j) {
    j += stride;
    while (j >= J) {
      j -= J;
      ++row;
    }
  };
  if (warp == CR_CONSUMERS) {
    // producer: one elected lane issues the copies
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      int row, j;
      first_chunk(0, row, j);
      for (int i = 0; i < n; ++i, advance(1, row, j)) {
        const int st = i % CR_STAGES;
        if (i >= CR_STAGES && !cr_wait(&empty[st], (uint32_t)(((i / CR_STAGES) - 1) & 1))) {
          atomicOr(&s_abort, 1);
          break;
        }
        if (*(volatile int*)&s_abort) break;
        const float* lrow;
        int q0, q1;
        CkRow g;
        chunk(row, j, lrow, q0, q1, g);
        const uint32_t bytes = (uint32_t)(q1 - q0) * 16u;
        mbar_arrive_expect_tx(&full[st], bytes);
        if (bytes)
          cr_copy(stage + (size_t)st * CK_F4, reinterpret_cast<const float4*>(lrow + g.a0) + q0,
                  bytes, &full[st], policy);
      }
    }
  } else {
    const int team = warp / CK_WARPS, sub = warp % CK_WARPS;
    int row, j;
    first_chunk(team, row, j);
    for (int i = team; i < n; i += CR_TEAMS, advance(CR_TEAMS, row, j)) {
      const int st = i % CR_STAGES;
      const float* lrow;
      int q0, q1;
      CkRow g;
      chunk(row, j, lrow, q0, q1, g);
      const size_t gidx = ((size_t)row * J + j) * CK_WARPS + sub;
      const bool ok = cr_wait(&full[st], (uint32_t)((i / CR_STAGES) & 1));
      if (!ok) {
        if (lane == 0) {
          a.s.ck_cnt[gidx] = CK_W_TIMEOUT;
          atomicOr(&s_abort, 1);
          atomicOr(a.s.error_word, 1u);
        }
        break;
      }
      const int nq = q1 - q0;
      const float4* sp = stage + (size_t)st * CK_F4 + sub * 256;
      float4 x[CK_LOADS];
#pragma unroll
      for (int u = 0; u < CK_LOADS; ++u) {
        const int q = sub * 256 + lane + 32 * u;
        x[u] = q < nq ? sp[lane + 32 * u] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
      // the <= 3 head and <= 3 tail scalars of the row: group 0 of part 0
      float xs = -INFINITY;
      int cs = 0;
      if (j == 0 && sub == 0) {
        const int a1 = g.a0 + 4 * g.n4;
        const int nh = g.a0 - lo, nt = hi - a1;
        if (lane < nh + nt) {
          cs = lane < nh ? lo + lane : a1 + (lane - nh);
          xs = lrow[cs];
        }
      }
      float cut = -INFINITY;
      const uint32_t word = ck_group(x, reinterpret_cast<const float*>(sp), xs, cs,
                                     g.a0 + 4 * (q0 + sub * 256), a.s.ck_keys + gidx * CK_KEYS,
                                     &cut);
      if (lane == 0) {
        a.s.ck_cnt[gidx] = word;
        a.s.ck_cut[gidx] = cut;
      }
      __syncwarp();
      // the stage is read: release it to the producer
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[st])) : "memory");
    }
  }
  // no bulk copy may still be landing in this CTA's shared memory when it exits
  __syncthreads();
  if (tid == 0 && s_abort) {
    for (int st = 0; st < CR_STAGES && st < n; ++st) {
      const int fills = (n - st + CR_STAGES - 1) / CR_STAGES;  // issued at most
      cr_wait(&full[st], (uint32_t)((fills - 1) & 1));
    }
  }
}

// AdjustLogit for a value whose id is in the history (rare among the kept
// values): one out-of-line copy instead of one per unrolled slot.
__device__ __noinline__ float ck_adjust(const Penalty P, float raw, int col) {
  return adjust(P, raw, col);
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

// One CTA per row. Slot s = tid + k * FK_THREADS of the row's G * CK_KEYS
// kept-value slots is thread tid's k-th: group s / CK_KEYS, place s % CK_KEYS,
// so the 16 slots of a group are 16 consecutive lanes (loads coalesce, group
// reductions are half-warp shuffles). FK_SLOTS * FK_THREADS >= G * CK_KEYS.
// The shard record of a finished row: every candidate >= the K-th (sorted
// holds the n candidates in descending order, all of the shard's values >= the
// K-th among them), stored into the peers' areas when a.px has peers. Every
// thread of the CTA calls; cv / cid are scratch for n entries.
__device__ __forceinline__ void ck_shard_record(const SampleArgs& a, int row, int K, int n,
                                                const uint64_t* sorted, float* cv, int* cid) {
  const int tid = threadIdx.x;
  const uint32_t tk = (uint32_t)(sorted[K - 1] >> 32);
  int c = 0;
  for (int i = tid; i < n; i += FK_THREADS) {
    cv[i] = cand_val(sorted[i]);
    cid[i] = cand_id(sorted[i]);
    if ((uint32_t)(sorted[i] >> 32) >= tk) ++c;
  }
  c = __syncthreads_count(c > 0 ? c : 0);  // n <= FK_THREADS: one entry per thread
  write_topk_record(a.shard_out + (size_t)row * VS_REC_WORDS, cv, cid, c, 0u, kval(tk));
  if (a.px.shards > 0) shard_px_epilogue(a.px, a.shard_out + (size_t)row * VS_REC_WORDS, row, true);
}

// kShard: the row is one GPU's columns [a.col_lo, a.col_hi) of a vocabulary
// split; instead of sampling, the CTA writes the row's shard record (every
// value >= the shard's K-th largest, ties included; shard_record.cuh) and
// stores it into the peers' areas when a.px has peers.
template <bool kCounts, int FK_SLOTS, bool kShard = false>
__global__ void __launch_bounds__(FK_THREADS, 2) topk_chunk_finish_kernel(const __grid_constant__ SampleArgs a, int J) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* gtop = reinterpret_cast<float*>(smem);                        // [FK_THREADS]
  uint64_t* cand = reinterpret_cast<uint64_t*>(gtop + FK_THREADS);     // [FK_CAND]
  uint64_t* sorted = cand + FK_CAND;                                   // [FK_CAND]
  float* w = reinterpret_cast<float*>(sorted + FK_CAND);               // [64] weights
  float* wS = w + 64;                                                  // [64]
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(wS + 64);
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);
  __shared__ int s_hn, s_nc, s_rescan;
  __shared__ uint32_t s_bkey, s_any, s_lkey, s_vmax, s_slow[2];
  __shared__ float s_u;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x;
  const int V = a.V;
  const int K = min(a.p.top_k, V);
  const int G = J * CK_WARPS;
  // each group contributes its M largest exact values to the lower bound of
  // the K-th value (G * M >= K distinct elements); with fewer than 2K groups,
  // two per group keep the bound tight (one per group would make it the
  // smallest group maximum, and let most kept values through as candidates)
  const int M = max((K + G - 1) / G, 2 * K > G ? 2 : 1);
  const int NT = G * M;
  const float scale = __fdiv_rn(1.0f, a.p.temperature);  // TokenSampler.cs:68
  const size_t gbase = (size_t)row * G;
  const int lo = kShard ? a.col_lo : 0, hi = kShard ? a.col_hi : V;

  // Prologue on the call's inputs only (history, uniform): they were written
  // before the chunk kernel started, which itself waited for them, so this
  // part may overlap the chunk kernel's last CTAs. The chunk kernel's outputs
  // are read after the wait below.
  if (tid == 0) {
    s_nc = 0;
    s_rescan = 0;
    s_bkey = 0u;
    s_any = 0u;
    s_lkey = 0xFFFFFFFFu;
    s_vmax = 0u;
    s_slow[0] = 0u;
    s_slow[1] = 0u;
    s_u = kShard ? 0.0f : a.uniforms[row];
  }
  Penalty P;
  const bool hist_ok =
      setup_penalty_range<kCounts>(P, a, a.hoff[row], a.hoff[row + 1], lo, hi, bitmap, hsorted, &s_hn);
  const bool pen = P.rep || P.cnt;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  uint2 kv[FK_SLOTS];
  uint32_t gw[FK_SLOTS];
  float cut[FK_SLOTS];
#pragma unroll
  for (int k = 0; k < FK_SLOTS; ++k) {
    const int s = tid + k * FK_THREADS, gi = s / CK_KEYS;
    if (gi < G) {
      kv[k] = __ldcg(a.s.ck_keys + (gbase + gi) * CK_KEYS + (s % CK_KEYS));
      gw[k] = __ldcg(a.s.ck_cnt + gbase + gi);
      cut[k] = (s % CK_KEYS) == 0 ? __ldcg(a.s.ck_cut + gbase + gi) : 0.0f;
    } else {
      kv[k] = make_uint2(0u, 0u);
      gw[k] = 0u;
      cut[k] = 0.0f;
    }
  }

  // exact values of the kept slots; per group (16 consecutive lanes) its
  // largest exact values and the bound of what the group dropped
  uint32_t any = 0u;  // bit 0: nonfinite group or exact +inf, bit 1: overflow
  uint32_t bk = 0u, vk = 0u;
  float v[FK_SLOTS];
#pragma unroll
  for (int k = 0; k < FK_SLOTS; ++k) {
    const int s = tid + k * FK_THREADS, gi = s / CK_KEYS, e = s % CK_KEYS;
    const uint32_t word = gw[k];
    const bool valid = gi < G && !(word & (CK_W_NONFINITE | CK_W_OVERFLOW | CK_W_TIMEOUT)) &&
                       e < (int)(word & 0xFFFFu);
    if (gi < G && e == 0) {
      if (word & (CK_W_NONFINITE | CK_W_TIMEOUT)) any |= 1u;
      if (word & CK_W_OVERFLOW) any |= 2u;
    }
    float ev = -INFINITY;
    if (valid) {
      const float raw = __uint_as_float(kv[k].x);
      const int col = (int)kv[k].y;
      float av = raw;
      const int rc = col - lo;  // the bitmap covers [lo, hi)
      if (pen && ((bitmap[rc >> 5] >> (rc & 31)) & 1u)) av = ck_adjust(P, raw, col);
      ev = canon(__fmul_rn(av, scale));
      if (!(ev < INFINITY)) any |= 1u;  // scaled past the float range, as the reference's value
    }
    v[k] = ev;
    if (valid) vk = max(vk, fkey(ev));
    // the group's values for the lower bound: its largest exact value, and
    // when M == 2 also its second largest
    float gm = ev, g2 = -INFINITY;
    if (M == 1) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    } else {
      gm = ev;
      int em = e;  // the slot of the group's largest value (lowest slot among equals)
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float og = __shfl_xor_sync(0xffffffffu, gm, o);
        const int oe = __shfl_xor_sync(0xffffffffu, em, o);
        if (og > gm || (og == gm && oe < em)) {
          gm = og;
          em = oe;
        }
      }
      g2 = e == em ? -INFINITY : ev;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) g2 = fmaxf(g2, __shfl_xor_sync(0xffffffffu, g2, o));
    }
    if (gi < G && e == 0) {
      if (M <= 2 && gi * M + M <= FK_THREADS) {
        gtop[gi * M] = gm;
        if (M == 2) gtop[gi * M + 1] = g2;
      }
      // a group that dropped values: they are below its cutoff
      if (!(word & (CK_W_NONFINITE | CK_W_OVERFLOW | CK_W_ALLKEPT | CK_W_TIMEOUT)) &&
          (word & 0xFFFFu) > 0u)
        bk = max(bk, fkey(canon(__fmul_rn(prev_float(cut[k]), scale))));
    }
  }
  any = __reduce_or_sync(0xffffffffu, any);
  bk = __reduce_max_sync(0xffffffffu, bk);
  vk = __reduce_max_sync(0xffffffffu, vk);
  if (lane == 0) {
    if (any) atomicOr(&s_any, any);
    if (bk) atomicMax(&s_bkey, bk);
    if (vk) atomicMax(&s_vmax, vk);
  }
  __syncthreads();
  const uint32_t anyall = s_any;
  uint32_t state = 0u;
  if (!hist_ok) state = FLAG_BAD_HISTORY;
  else if (anyall & 1u) state = FLAG_NONFINITE;
  if (state) {
    if constexpr (kShard) {  // a record carrying the state: the merge returns -1
      write_topk_record(a.shard_out + (size_t)row * VS_REC_WORDS, gtop,
                        reinterpret_cast<const int*>(cand), 0, state, -INFINITY);
      if (a.px.shards > 0) shard_px_epilogue(a.px, a.shard_out + (size_t)row * VS_REC_WORDS, row, true);
    } else if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = state;
    }
    return;
  }
  if ((anyall & 2u) || M > 2 || NT > FK_THREADS || s_vmax == 0u) {
    // the exact full-vocabulary kernel launched after this one redoes the row
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }
  // L, a lower bound of the row's K-th largest value: warp w holds up to 32
  // of the NT group values (distinct elements) and pops its q_w largest
  // (q_w = ceil(K n_w / NT), so the q_w sum to >= K); L is the smallest of
  // the warps' q_w-th largest values, so >= K elements are >= L.
  if (warp < (NT + 31) / 32) {
    const int nw = min(32, NT - 32 * warp);
    const int q = (K * nw + NT - 1) / NT;
    uint32_t key = lane < nw ? fkey(gtop[32 * warp + lane]) : 0u;
    uint32_t qth = 0u;
    for (int r = 0; r < q; ++r) {
      qth = __reduce_max_sync(0xffffffffu, key);
      const unsigned hit = __ballot_sync(0xffffffffu, key == qth);
      if (lane == __ffs(hit) - 1) key = 0u;
    }
    if (lane == 0) atomicMin(&s_lkey, qth);
  }
  __syncthreads();
  if (s_lkey <= fkey(-INFINITY)) {  // fewer than K finite values: the exact path decides
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }
  const float L = kval(s_lkey);
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
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }
  // rank sort (the keys are distinct: ids are) and the weights of the first
  // 64 places, exp(v - max) with the row's largest value
  const float vmax = kval(s_vmax);
  if (tid < nc) {
    const uint64_t key = cand[tid];
    int r = 0;
    int h = 0;
    for (; h + 8 <= nc; h += 8) {
#pragma unroll
      for (int d = 0; d < 8; ++d) r += cand[h + d] > key;
    }
    for (; h < nc; ++h) r += cand[h] > key;
    sorted[r] = key;
    if (!kShard && r < 64) {
      bool slow = false;
      w[r] = exp_cr(__fsub_rn(cand_val(key), vmax), slow);
      if (slow) atomicOr(&s_slow[r >> 5], 1u << (r & 31));
    }
  }
  __syncthreads();
  if constexpr (kShard) {
    // the K-th value T, proven as below; the record holds every candidate >= T
    // (all of the shard's values >= T are candidates: they are above every
    // dropped value, and L <= T)
    if (s_bkey < (uint32_t)(sorted[K - 1] >> 32)) {
      ck_shard_record(a, row, K, nc, sorted, gtop, reinterpret_cast<int*>(cand));
      return;
    }
    // unproven: the rescan below
  }
  // warp 0: the K-th value, the proof, the candidates (ties included) and the finish
  if (warp == 0) {
    const uint32_t tk = (uint32_t)(sorted[K - 1] >> 32);
    const uint64_t k0 = lane < nc ? sorted[lane] : 0ull;
    const uint64_t k1 = lane + 32 < nc ? sorted[lane + 32] : 0ull;
    const bool over = nc > 64 && (uint32_t)(sorted[64] >> 32) == tk;  // > 64 candidates
    // every dropped value lies below the K-th value: it is the row's
    if (over) {
      if (lane == 0) a.s.fixup[row] = 1u;
    } else if (s_bkey >= tk) {
      if (lane == 0) s_rescan = 1;  // unproven: the rescan below
    } else {
      const unsigned b0 = __ballot_sync(0xffffffffu, k0 != 0ull && (uint32_t)(k0 >> 32) >= tk);
      const unsigned b1 = __ballot_sync(0xffffffffu, k1 != 0ull && (uint32_t)(k1 >> 32) >= tk);
      const int c = __popc(b0) + __popc(b1);
      const bool any_slow = (s_slow[0] & b0) != 0u || (s_slow[1] & b1) != 0u;
      finish_weights_warp(a, row, lane < c ? k0 : 0ull, lane + 32 < c ? k1 : 0ull, c, w, wS,
                          any_slow, s_u);
    }
  }
  if constexpr (!kShard) {
    __syncthreads();
    if (!s_rescan) return;
  }
  // A group held more of the row's top K than it kept, so a dropped value may
  // lie above the K-th value. The CTA reads the whole row again (one column
  // per lane and step: a rare path, placed after the common one) and takes
  // every value >= L (at least K of them exist, whatever was dropped): the
  // candidates are then complete without a proof; more than FK_CAND of them
  // hand the row to the fix-up kernel.
  __syncthreads();
  if (tid == 0) {
    s_nc = 0;
    s_vmax = 0u;
    s_slow[0] = 0u;
    s_slow[1] = 0u;
  }
  __syncthreads();
  {
    const float* lrow = kShard ? a.logits + (size_t)row * a.ld - lo : a.logits + (size_t)row * V;
    uint32_t vk2 = 0u;
    for (int c0 = lo + warp * 32; c0 < hi; c0 += FK_THREADS) {
      const int c = c0 + lane;
      float ev = -INFINITY;
      if (c < hi) {
        const float raw = __ldcs(lrow + c);
        const int rc = c - lo;
        const float av = (pen && ((bitmap[rc >> 5] >> (rc & 31)) & 1u)) ? ck_adjust(P, raw, c) : raw;
        ev = canon(__fmul_rn(av, scale));
      }
      const bool ok = ev >= L;
      const unsigned b = __ballot_sync(0xffffffffu, ok);
      if (b) {
        const int leader = __ffs(b) - 1;
        int base = 0;
        if (lane == leader) base = atomicAdd(&s_nc, __popc(b));
        base = __shfl_sync(0xffffffffu, base, leader);
        const int slot = base + __popc(b & ((1u << lane) - 1u));
        if (ok && slot < FK_CAND) cand[slot] = cand_key(ev, c);
        if (ok) vk2 = max(vk2, fkey(ev));
      }
    }
    vk2 = __reduce_max_sync(0xffffffffu, vk2);
    if (lane == 0 && vk2) atomicMax(&s_vmax, vk2);
  }
  __syncthreads();
  const int n2 = s_nc;
  if (n2 > FK_CAND || n2 < K) {
    if (tid == 0) a.s.fixup[row] = 1u;
    return;
  }
  {
    const float vmax2 = kval(s_vmax);
    if (tid < n2) {
      const uint64_t key = cand[tid];
      int r = 0;
      for (int h = 0; h < n2; ++h) r += cand[h] > key;
      sorted[r] = key;
      if (!kShard && r < 64) {
        bool slow = false;
        w[r] = exp_cr(__fsub_rn(cand_val(key), vmax2), slow);
        if (slow) atomicOr(&s_slow[r >> 5], 1u << (r & 31));
      }
    }
  }
  __syncthreads();
  if constexpr (kShard) {
    ck_shard_record(a, row, K, n2, sorted, gtop, reinterpret_cast<int*>(cand));
  } else if (warp == 0) {
    const uint32_t tk = (uint32_t)(sorted[K - 1] >> 32);
    const uint64_t k0 = lane < n2 ? sorted[lane] : 0ull;
    const uint64_t k1 = lane + 32 < n2 ? sorted[lane + 32] : 0ull;
    if (n2 > 64 && (uint32_t)(sorted[64] >> 32) == tk) {  // > 64 candidates
      if (lane == 0) a.s.fixup[row] = 1u;
    } else {
      const unsigned b0 = __ballot_sync(0xffffffffu, k0 != 0ull && (uint32_t)(k0 >> 32) >= tk);
      const unsigned b1 = __ballot_sync(0xffffffffu, k1 != 0ull && (uint32_t)(k1 >> 32) >= tk);
      const int c = __popc(b0) + __popc(b1);
      const bool any_slow = (s_slow[0] & b0) != 0u || (s_slow[1] & b1) != 0u;
      finish_weights_warp(a, row, lane < c ? k0 : 0ull, lane + 32 < c ? k1 : 0ull, c, w, wS,
                          any_slow, s_u);
    }
  }
}

}  // namespace nvs
