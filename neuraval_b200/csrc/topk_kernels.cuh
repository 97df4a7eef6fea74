// Greedy and top-k sampling kernels (sm_100a).
//
// Reference semantics: Neuraval/Generation/TokenSampler.cs
//   SampleGreedy   :32-52   first strict maximum of AdjustLogit(l_i)
//   SampleFiltered :54-135  K-th largest threshold (with multiplicity), every
//                           value >= threshold is a candidate, candidates sorted
//                           descending, w_i = exp(v_i - max), sequential fp32
//                           sums, top-p cutoff, inverse-CDF draw on u.
//
// Layout: grid (splits, rows). Each CTA streams one contiguous column segment
// of one row through a ring of TMA bulk copies into shared memory, applies the
// penalties and the temperature scale in place, and keeps every value >= a
// running threshold (a lower bound of the segment's K-th largest value) in a
// shared-memory candidate buffer. When the buffer would overflow, an exact
// radix select over buffer + staged chunk raises the threshold. The CTA that
// finishes a row last (atomic ticket, no waiting) merges the segments'
// candidates and runs the exact finishing stage.
#pragma once

#include "sampler_device.cuh"
#include "shard_record.cuh"
#include "peer_exchange.cuh"

namespace nvs {

constexpr int TK_THREADS = 512;
constexpr int TK_CHUNK = 4096;   // floats per staged chunk (16 KiB)
constexpr int TK_NSTAGE = 3;     // ring depth
constexpr int TK_CAPB = 2048;    // candidate buffer entries per CTA (and per segment in scratch)
constexpr int TK_KMAX = 1024;    // largest top-k served by this kernel
constexpr int GR_THREADS = 512;

struct Scratch {
  float* cand_v;        // [max_ctas * TK_CAPB]
  int32_t* cand_id;     // [max_ctas * TK_CAPB]
  int32_t* cand_n;      // [max_ctas]
  uint32_t* tickets;    // [max_rows]  zero between launches
  uint32_t* rowstate;   // [max_rows]  zero between launches
  float* gv;            // [max_ctas]  greedy partial maxima
  int32_t* gi;          // [max_ctas]
  uint32_t* error_word; // [1] sticky error bits (timeouts)
  uint32_t* fixup;      // [max_rows]  1: row must be redone on the full-vocabulary path
  uint32_t* px_ticket;  // [4] peer exchange: [2] merge CTAs (zero between launches),
                        // [3] epoch of the last merged call; [0], [1] unused
  uint32_t* stats;      // [1] rows redone by the full-sort kernel (null: not counted)
  uint2* ck_keys;       // chunked top-k: kept (raw value bits, column) per warp group,
                        // [rows][chunks][8 warps][16]
  uint32_t* ck_cnt;     // chunked top-k: count and state word per warp group
  float* ck_cut;        // chunked top-k: per warp group, the cutoff (kept values are >= it,
                        // dropped ones below it)
};

struct SampleArgs {
  const float* logits;
  int V;
  int seg_len;          // columns per split (multiple of 4)
  const int32_t* hist;
  const int32_t* hoff;
  const float* uniforms;
  Params p;
  int32_t* tokens;
  uint32_t* flags;
  float* probs;
  int bm_words;         // bitmap words per CTA (columns/32 rounded up, plus one spare)
  int h_cap;            // history ids per CTA in smem (counts only), power of 2
  Scratch s;
  // vocabulary shards only (kShard kernels): `logits` holds columns
  // [col_lo, col_hi) of each row with row stride `ld`; `V` stays the full
  // vocabulary; every row's record goes to shard_out + row * VS_REC_WORDS
  int ld;
  int col_lo;
  int col_hi;
  uint32_t* shard_out;
  PxArgs px;            // peers of a shard kernel (px.shards == 0: none)
  int fixup_only;       // topk_ldg_kernel: only rows with s.fixup[row] set, which it clears
};

constexpr int HIST_PRE = 4;  // history ids per thread loaded before any is used

// Shared penalty state for the CTA's column range [c0,c1), from the row's
// history ids [hb, he). Returns false when the row's in-range history does
// not fit h_cap (BAD_HISTORY).
template <bool kCounts>
__device__ bool setup_penalty_range(Penalty& P, const SampleArgs& a, int hb, int he, int c0,
                                    int c1, uint32_t* bitmap, int32_t* hsorted, int* s_hn) {
  const int H = he - hb;
  P.bitmap = bitmap;
  P.hsorted = hsorted;
  P.hn = 0;
  P.c0 = c0;
  P.pen = a.p.repetition_penalty;
  P.freq = a.p.frequency_penalty;
  P.pres = a.p.presence_penalty;
  // TokenSampler.cs:61-63: the repeated set exists only for penalty != 1 and a
  // non-empty history (ids outside [0,V) are in the set but never match).
  P.rep = (P.pen != 1.0f) && H > 0;
  P.cnt = kCounts && (P.freq != 0.0f || P.pres != 0.0f) && H > 0;
  if (!P.rep && !P.cnt) return true;
  // occurrence counts matter only through cnt * frequency: with a zero
  // frequency (either sign) cnt * f is that zero for every count, so the ids
  // are neither collected nor sorted (P.hn stays 0, every count reads 0)
  const bool counting = kCounts && P.cnt && P.freq != 0.0f;
  // the thread's first ids are all in flight before any is used (one round
  // trip, hidden behind the bitmap clear)
  int pre[HIST_PRE];
#pragma unroll
  for (int k = 0; k < HIST_PRE; ++k) {
    const int h = hb + (int)threadIdx.x + k * (int)blockDim.x;
    pre[k] = h < he ? a.hist[h] : 0;
  }
  const int words = ((c1 - c0 + 31) >> 5) + 1;  // one spare word for 4-id windows
  for (int i = threadIdx.x; i < words; i += blockDim.x) bitmap[i] = 0u;
  if (threadIdx.x == 0) *s_hn = 0;
  __syncthreads();
  auto put = [&](int id) {
    if (id >= c0 && id < c1) {
      const int rel = id - c0;
      atomicOr(&bitmap[rel >> 5], 1u << (rel & 31));
      if (counting) {
        const int slot = atomicAdd(s_hn, 1);
        if (slot < a.h_cap) hsorted[slot] = id;
      }
    }
  };
#pragma unroll
  for (int k = 0; k < HIST_PRE; ++k)
    if (hb + (int)threadIdx.x + k * (int)blockDim.x < he) put(pre[k]);
  for (int h = hb + (int)threadIdx.x + HIST_PRE * (int)blockDim.x; h < he; h += blockDim.x)
    put(a.hist[h]);
  __syncthreads();
  bool ok = true;
  if (counting) {
    const int n = *s_hn;
    if (n > a.h_cap) {
      ok = false;
    } else {
      const int np = next_pow2(n > 0 ? n : 1);
      for (int i = n + threadIdx.x; i < np; i += blockDim.x) hsorted[i] = 0x7FFFFFFF;
      __syncthreads();
      cta_bitonic_sort_asc(hsorted, np);
      P.hn = n;
    }
  }
  return ok;
}

template <bool kCounts>
__device__ bool setup_penalty(Penalty& P, const SampleArgs& a, int row, int c0, int c1,
                              uint32_t* bitmap, int32_t* hsorted, int* s_hn) {
  return setup_penalty_range<kCounts>(P, a, a.hoff[row], a.hoff[row + 1], c0, c1, bitmap,
                                      hsorted, s_hn);
}

// ---------------------------------------------------------------------------
// Greedy: first strict maximum (TokenSampler.cs:38-51). A NaN at index 0 is
// kept (nothing compares greater); a NaN anywhere else never wins.
// ---------------------------------------------------------------------------
struct Best {
  float v;
  int i;  // -1: none
};
__device__ __forceinline__ Best better(Best a, Best b) {
  if (b.i < 0) return a;
  if (a.i < 0) return b;
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best t{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
    b = better(b, t);
  }
  return b;
}

template <bool kCounts, bool kShard>
__device__ __forceinline__ void greedy_body(const SampleArgs& a, int* owner);

template <bool kCounts, bool kShard = false>
__global__ void __launch_bounds__(GR_THREADS) greedy_kernel(const __grid_constant__ SampleArgs a) {
  __shared__ int s_owner;
  greedy_body<kCounts, kShard>(a, &s_owner);
  if constexpr (kShard) {
    if (a.px.shards > 0) {
      __syncthreads();
      shard_px_epilogue(a.px, a.shard_out + (size_t)blockIdx.y * VS_REC_WORDS, blockIdx.y,
                        s_owner != 0);
    }
  }
}

template <bool kCounts, bool kShard>
__device__ __forceinline__ void greedy_body(const SampleArgs& a, int* owner) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem);
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);
  __shared__ int s_hn;
  __shared__ Best s_w[GR_THREADS / 32];
  __shared__ int s_last;
  __shared__ int s_nan0;

  const int row = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const int V = a.V;
  const int lo = kShard ? a.col_lo : 0, hi = kShard ? a.col_hi : V;
  const int c0 = lo + split * a.seg_len;
  const int c1 = min(hi, c0 + a.seg_len);
  const float* lrow = kShard ? a.logits + (size_t)row * a.ld - lo : a.logits + (size_t)row * V;
  if (threadIdx.x == 0) *owner = S == 1;  // the CTA that writes the row's result

  Penalty P;
  const bool ok = setup_penalty<kCounts>(P, a, row, c0, c1, bitmap, hsorted, &s_hn);
  if (threadIdx.x == 0) s_nan0 = 0;
  __syncthreads();

  Best b{0.0f, -1};
  if (ok) {
    for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
      float v = canon(adjust(P, __ldcs(lrow + c), c));
      if (v != v) {
        if (c == 0) s_nan0 = 1;
        continue;
      }
      b = better(b, Best{v, c});
    }
  }
  b = warp_best(b);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x < 32) {
    Best t = threadIdx.x < (int)(blockDim.x >> 5) ? s_w[threadIdx.x] : Best{0.0f, -1};
    t = warp_best(t);
    if (threadIdx.x == 0) s_w[0] = t;
  }
  __syncthreads();

  if (S == 1) {
    if (threadIdx.x == 0) {
      Best r = s_w[0];
      if constexpr (kShard) {
        write_greedy_record(a.shard_out + (size_t)row * VS_REC_WORDS, r.v, r.i, !ok, s_nan0 != 0);
        return;
      }
      int tok = (s_nan0 || r.i < 0) ? 0 : r.i;
      a.tokens[row] = ok ? tok : -1;
      if (a.flags) a.flags[row] = ok ? 0u : FLAG_BAD_HISTORY;
    }
    return;
  }
  const int cta = row * S + split;
  if (threadIdx.x == 0) {
    a.s.gv[cta] = s_w[0].v;
    a.s.gi[cta] = s_w[0].i;
    uint32_t st = (ok ? 0u : FLAG_BAD_HISTORY) | (s_nan0 ? 0x40000000u : 0u);
    if (st) atomicOr(&a.s.rowstate[row], st);
    __threadfence();
    const uint32_t t = atomicAdd(&a.s.tickets[row], 1u);
    s_last = (t == (uint32_t)(S - 1));
    *owner = s_last;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    Best r{0.0f, -1};
    for (int sp = threadIdx.x; sp < S; sp += 32) {
      Best t{__ldcg(&a.s.gv[row * S + sp]), __ldcg(&a.s.gi[row * S + sp])};
      r = better(r, t);
    }
    r = warp_best(r);
    if (threadIdx.x == 0) {
      const uint32_t st = __ldcg(&a.s.rowstate[row]);
      const bool bad = (st & FLAG_BAD_HISTORY) != 0u;
      const bool nan0 = (st & 0x40000000u) != 0u;
      if constexpr (kShard) {
        write_greedy_record(a.shard_out + (size_t)row * VS_REC_WORDS, r.v, r.i, bad, nan0);
      } else {
        int tok = (nan0 || r.i < 0) ? 0 : r.i;
        a.tokens[row] = bad ? -1 : tok;
        if (a.flags) a.flags[row] = bad ? FLAG_BAD_HISTORY : 0u;
      }
      a.s.rowstate[row] = 0u;
      a.s.tickets[row] = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
// Top-k sampling
// ---------------------------------------------------------------------------

// Warp-aggregated append of one optional candidate per lane. All 32 lanes call.
__device__ __forceinline__ void warp_append(bool pred, float v, int id, float* cv, int* cid,
                                            int* s_count, int* s_overflow, int cap = TK_CAPB) {
  const unsigned b = __ballot_sync(0xffffffffu, pred);
  if (b == 0u) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(b) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(s_count, __popc(b));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (pred) {
    const int slot = base + __popc(b & ((1u << lane) - 1u));
    if (slot < cap) {
      cv[slot] = v;
      cid[slot] = id;
    } else {
      *s_overflow = 1;
    }
  }
}

// Exact finishing stage for one row (TokenSampler.cs:95-132). Candidates are
// cv/cid[0..m) (unsorted). `work` holds >= next_pow2(m)*8 + 2*m*4 bytes.
// All threads call; thread 0 runs the sequential fp32 sums in sorted order.
__device__ void finish_row(const SampleArgs& a, int row, const float* cv, const int* cid, int m,
                           uint32_t state, unsigned char* work) {
  __shared__ int s_cut;
  __shared__ float s_ret;
  __shared__ uint32_t s_flag;
  const int V = a.V;
  if ((state & RSTATE_OVERFLOW) && !(state & (FLAG_NONFINITE | FLAG_BAD_HISTORY | RSTATE_TIMEOUT))) {
    // ties at the K-th value exceed the buffers: the full-vocabulary kernel
    // launched after this one redoes the row
    if (threadIdx.x == 0) a.s.fixup[row] = 1u;
    return;
  }
  if (state & (FLAG_NONFINITE | FLAG_BAD_HISTORY | RSTATE_TIMEOUT) || m <= 0) {
    if (threadIdx.x == 0) {
      a.tokens[row] = -1;
      uint32_t f = state & (FLAG_NONFINITE | FLAG_BAD_HISTORY);
      if (state & RSTATE_TIMEOUT) f |= FLAG_NONFINITE;
      if (a.flags) a.flags[row] = f;
    }
    return;
  }
  const int np = next_pow2(m);
  uint64_t* keys = reinterpret_cast<uint64_t*>(work);
  float* w = reinterpret_cast<float*>(keys + np);
  float* S = w + m;
  for (int i = threadIdx.x; i < np; i += blockDim.x)
    keys[i] = i < m ? cand_key(cv[i], cid[i]) : 0ull;
  __syncthreads();
  cta_bitonic_sort_desc(keys, np);
  const float vmax = cand_val(keys[0]);
  if (threadIdx.x == 0) s_flag = 0u;
  __syncthreads();
  if (!(vmax > -INFINITY)) {
    if (threadIdx.x == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_NONFINITE;
    }
    return;
  }
  bool slow = false;
  for (int i = threadIdx.x; i < m; i += blockDim.x)
    w[i] = exp_cr(__fsub_rn(cand_val(keys[i]), vmax), slow);
  if (slow) atomicOr(&s_flag, FLAG_EXP_SLOW);
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int i = 0; i < m; ++i) {
      total = __fadd_rn(total, w[i]);
      S[i] = total;
    }
    int cutoff = m;
    float target = 0.0f;
    if (a.p.top_p < 1.0f) {
      target = __fmul_rn(total, a.p.top_p);
      for (int i = 0; i < m; ++i)
        if (S[i] >= target) { cutoff = i + 1; break; }
    }
    const float retained = S[cutoff - 1];
    const float sample = __fmul_rn(a.uniforms[row], retained);
    int sel = cutoff - 1;
    for (int i = 0; i < cutoff; ++i)
      if (sample <= S[i]) { sel = i; break; }
    uint32_t f = s_flag;
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
    const uint32_t ks = (uint32_t)(keys[sel] >> 32);
    if ((sel > 0 && (uint32_t)(keys[sel - 1] >> 32) == ks) ||
        (sel + 1 < m && (uint32_t)(keys[sel + 1] >> 32) == ks))
      f |= FLAG_TIE_AT_DRAW;
    a.tokens[row] = cand_id(keys[sel]);
    if (a.flags) a.flags[row] = f;
    s_cut = cutoff;
    s_ret = retained;
  }
  __syncthreads();
  if (a.probs) {
    float* prow = a.probs + (size_t)row * V;
    for (int i = threadIdx.x; i < s_cut; i += blockDim.x)
      prow[cand_id(keys[i])] = __fdiv_rn(w[i], s_ret);
  }
}

template <bool kCounts>
__global__ void __launch_bounds__(TK_THREADS, 2) topk_kernel(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* stage = reinterpret_cast<float*>(smem);                 // [NSTAGE][CHUNK]
  float* cv = stage + TK_NSTAGE * TK_CHUNK;                       // [CAPB]
  int* cid = reinterpret_cast<int*>(cv + TK_CAPB);                // [CAPB]
  uint32_t* hist = reinterpret_cast<uint32_t*>(cid + TK_CAPB);    // [256]
  uint64_t* bars = reinterpret_cast<uint64_t*>(hist + 256);       // [NSTAGE]
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(bars + TK_NSTAGE);
  int32_t* hsorted = reinterpret_cast<int32_t*>(bitmap + a.bm_words);

  __shared__ int s_count, s_cnt_before, s_overflow, s_row_overflow, s_nonfinite, s_hn, s_last;
  __shared__ int s_timeout, s_issued;
  __shared__ uint32_t s_theta;
  __shared__ int s_sh[2];

  const int tid = threadIdx.x;
  const int row = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const int V = a.V;
  const int K = min(a.p.top_k, V);
  const int c0 = split * a.seg_len;
  const int c1 = min(V, c0 + a.seg_len);
  const float* lrow = a.logits + (size_t)row * V;
  const float scale = __fdiv_rn(1.0f, a.p.temperature);  // TokenSampler.cs:68

  Penalty P;
  const bool hist_ok = setup_penalty<kCounts>(P, a, row, c0, c1, bitmap, hsorted, &s_hn);

  // 16-byte aligned body [a0,a1) goes through the TMA ring; <=3 head and <=3
  // tail elements are loaded directly.
  const int head = (int)(((16u - ((uint32_t)(uintptr_t)(lrow + c0) & 15u)) & 15u) >> 2);
  const int a0 = min(c0 + head, c1);
  const int a1 = a0 + ((c1 - a0) & ~3);
  const int nch = (a1 - a0 + TK_CHUNK - 1) / TK_CHUNK;

  if (tid == 0) {
    s_count = 0;
    s_cnt_before = 0;
    s_overflow = 0;
    s_row_overflow = 0;
    s_nonfinite = 0;
    s_timeout = 0;
    s_theta = 0u;  // accept everything (the key of -inf is > 0)
    for (int i = 0; i < TK_NSTAGE; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  if (a.probs) {
    float* prow = a.probs + (size_t)row * V;
    for (int c = c0 + tid; c < c1; c += TK_THREADS) prow[c] = 0.0f;
  }
  __syncthreads();

  if (tid == 0) s_issued = 0;
  if (tid == 0 && hist_ok) {
    s_issued = min(TK_NSTAGE, nch);
    for (int t = 0; t < min(TK_NSTAGE, nch); ++t) {
      const int len = min(TK_CHUNK, a1 - (a0 + t * TK_CHUNK));
      mbar_arrive_expect_tx(&bars[t], (uint32_t)len * 4u);
      bulk_g2s(stage + t * TK_CHUNK, lrow + a0 + t * TK_CHUNK, (uint32_t)len * 4u, &bars[t]);
    }
  }
  // head and tail elements
  {
    const int nh = a0 - c0, nt = c1 - a1;
    const bool act = hist_ok && tid < nh + nt;
    float v = -INFINITY;
    int col = 0;
    if (act) {
      col = tid < nh ? c0 + tid : a1 + (tid - nh);
      v = canon(__fmul_rn(adjust(P, lrow[col], col), scale));
      if (v != v || v == INFINITY) {
        s_nonfinite = 1;
        v = -INFINITY;
      }
    }
    if (tid < 32) warp_append(act, v, col, cv, cid, &s_count, &s_overflow);
  }
  __syncthreads();

  if (hist_ok) {
    int consumed = 0;  // chunks whose stage has been fully read
    for (int t = 0; t < nch; ++t) {
      const int st = t % TK_NSTAGE;
      const uint32_t parity = (uint32_t)((t / TK_NSTAGE) & 1);
      if (!mbar_wait_bounded(&bars[st], parity)) s_timeout = 1;
      __syncthreads();
      if (s_timeout) break;
      const int len = min(TK_CHUNK, a1 - (a0 + t * TK_CHUNK));
      const int nq = len >> 2;
      const int base = a0 + t * TK_CHUNK;
      float4* sq = reinterpret_cast<float4*>(stage + st * TK_CHUNK);
      const uint32_t tkey = s_theta;
      const float theta = tkey == 0u ? -INFINITY : kval(tkey);  // key 0: accept everything
#pragma unroll
      for (int k = 0; k < TK_CHUNK / 4 / TK_THREADS; ++k) {
        const int q = tid + k * TK_THREADS;
        const bool valid = q < nq;
        const int col = base + 4 * q;
        float vv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        bool any = false;
        if (valid) {
          const float4 x = sq[q];
          vv[0] = __fmul_rn(x.x, scale);
          vv[1] = __fmul_rn(x.y, scale);
          vv[2] = __fmul_rn(x.z, scale);
          vv[3] = __fmul_rn(x.w, scale);
          if ((P.rep || P.cnt) && penalty_bits4(P, col) != 0u) {
            // a penalised id among the four: exact per-element path
            vv[0] = __fmul_rn(adjust(P, x.x, col), scale);
            vv[1] = __fmul_rn(adjust(P, x.y, col + 1), scale);
            vv[2] = __fmul_rn(adjust(P, x.z, col + 2), scale);
            vv[3] = __fmul_rn(adjust(P, x.w, col + 3), scale);
          }
          // NaN or +inf: !(v < inf); -inf is a legal value
          if (!(vv[0] < INFINITY) || !(vv[1] < INFINITY) || !(vv[2] < INFINITY) ||
              !(vv[3] < INFINITY))
            s_nonfinite = 1;
          any = vv[0] >= theta || vv[1] >= theta || vv[2] >= theta || vv[3] >= theta;
        }
        if (__any_sync(0xffffffffu, any)) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const bool c = any && vv[j] >= theta;
            warp_append(c, canon(vv[j]), col + j, cv, cid, &s_count, &s_overflow);
          }
        }
      }
      __syncthreads();
      if (s_overflow) {
        // exact K-th largest of (earlier candidates) + (this chunk)
        const int nb = s_cnt_before;
        const float* sraw = stage + st * TK_CHUNK;
        // staged values are raw logits: recompute exactly as the fast path does
        auto sval = [&](int i) -> float {
          const float v = canon(__fmul_rn(adjust(P, sraw[i], base + i), scale));
          return (v < INFINITY) ? v : -INFINITY;
        };
        const uint32_t key = cta_kth_largest_key([&](int i) { return cv[i]; }, nb, sval, len, K,
                                                 hist, s_sh);
        constexpr int PER = TK_CAPB / TK_THREADS;
        float rv[PER];
        int rid[PER];
        bool keep[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) {
          const int i = tid + k * TK_THREADS;
          keep[k] = i < nb && fkey(cv[i]) >= key;
          rv[k] = keep[k] ? cv[i] : 0.f;
          rid[k] = keep[k] ? cid[i] : 0;
        }
        __syncthreads();
        if (tid == 0) {
          s_count = 0;
          s_overflow = 0;
          s_theta = key;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < PER; ++k) warp_append(keep[k], rv[k], rid[k], cv, cid, &s_count, &s_overflow);
        for (int i0 = 0; i0 < len; i0 += TK_THREADS) {
          const int i = i0 + tid;
          const float v = i < len ? sval(i) : -INFINITY;
          const bool ok = i < len && fkey(v) >= key;
          warp_append(ok, v, base + i, cv, cid, &s_count, &s_overflow);
        }
        __syncthreads();
        if (tid == 0 && s_overflow) {
          s_row_overflow = 1;  // ties at the threshold exceed the buffer
          s_overflow = 0;
        }
      }
      if (tid == 0) {
        s_cnt_before = min(s_count, TK_CAPB);
        if (t + TK_NSTAGE < nch) {
          const int tn = t + TK_NSTAGE;
          const int lenn = min(TK_CHUNK, a1 - (a0 + tn * TK_CHUNK));
          fence_proxy_async();
          mbar_arrive_expect_tx(&bars[st], (uint32_t)lenn * 4u);
          bulk_g2s(stage + st * TK_CHUNK, lrow + a0 + tn * TK_CHUNK, (uint32_t)lenn * 4u, &bars[st]);
          s_issued = tn + 1;
        }
      }
      __syncthreads();
      consumed = t + 1;
      if (s_row_overflow) break;
    }
    // Copies still in flight after an early exit: wait for them (bounded)
    // before the CTA's shared memory is reused or released.
    if (tid == 0) {
      for (int c = consumed; c < s_issued; ++c)
        (void)mbar_wait_bounded(&bars[c % TK_NSTAGE], (uint32_t)((c / TK_NSTAGE) & 1));
    }
    __syncthreads();
  }

  // Final exact K-th largest of the segment; keep every value >= it.
  uint32_t state = 0u;
  if (!hist_ok) state |= FLAG_BAD_HISTORY;
  if (s_nonfinite) state |= FLAG_NONFINITE;
  if (s_row_overflow) state |= RSTATE_OVERFLOW;
  if (s_timeout) state |= RSTATE_TIMEOUT;
  int m = min(s_count, TK_CAPB);
  if (state == 0u) {
    const uint32_t key = cta_kth_largest_key([&](int i) { return cv[i]; }, m,
                                             [&](int) { return 0.0f; }, 0, K, hist, s_sh);
    constexpr int PER = TK_CAPB / TK_THREADS;
    float rv[PER];
    int rid[PER];
    bool keep[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = tid + k * TK_THREADS;
      keep[k] = i < m && fkey(cv[i]) >= key;
      rv[k] = keep[k] ? cv[i] : 0.f;
      rid[k] = keep[k] ? cid[i] : 0;
    }
    __syncthreads();
    if (tid == 0) s_count = 0;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < PER; ++k) warp_append(keep[k], rv[k], rid[k], cv, cid, &s_count, &s_overflow);
    __syncthreads();
    m = s_count;
  }
  if (s_timeout && tid == 0) atomicOr(a.s.error_word, 1u);

  if (S == 1) {
    finish_row(a, row, cv, cid, m, state, reinterpret_cast<unsigned char*>(stage));
    return;
  }

  // Publish this segment's candidates; the last CTA of the row merges.
  const int cta = row * S + split;
  for (int i = tid; i < m; i += TK_THREADS) {
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

  // Merge: gather the union into the (now idle) stage ring.
  float* uv = stage;
  int* uid = reinterpret_cast<int*>(stage + (TK_NSTAGE * TK_CHUNK) / 2);
  const int ucap = (TK_NSTAGE * TK_CHUNK) / 2;
  __shared__ int s_off[1];
  __shared__ uint32_t s_state;
  if (tid == 0) {
    s_state = __ldcg(&a.s.rowstate[row]);
    int tot = 0;
    for (int sp = 0; sp < S; ++sp) tot += __ldcg(&a.s.cand_n[row * S + sp]);
    s_off[0] = tot;
  }
  __syncthreads();
  uint32_t mstate = s_state;
  const int total = s_off[0];
  if (total > ucap) mstate |= RSTATE_OVERFLOW;
  int mm = 0;
  if (mstate == 0u) {
    // segment lists are copied one after another
    int off = 0;
    for (int sp = 0; sp < S; ++sp) {
      const int n = __ldcg(&a.s.cand_n[row * S + sp]);
      const size_t g = (size_t)(row * S + sp) * TK_CAPB;
      for (int i = tid; i < n; i += TK_THREADS) {
        uv[off + i] = __ldcg(&a.s.cand_v[g + i]);
        uid[off + i] = __ldcg(&a.s.cand_id[g + i]);
      }
      off += n;
    }
    __syncthreads();
    const uint32_t key = cta_kth_largest_key([&](int i) { return uv[i]; }, total,
                                             [&](int) { return 0.0f; }, 0, K, hist, s_sh);
    if (tid == 0) {
      s_count = 0;
      s_overflow = 0;
    }
    __syncthreads();
    for (int i0 = 0; i0 < total; i0 += TK_THREADS) {
      const int i = i0 + tid;
      const bool ok = i < total && fkey(uv[i]) >= key;
      warp_append(ok, ok ? uv[i] : 0.f, ok ? uid[i] : 0, cv, cid, &s_count, &s_overflow);
    }
    __syncthreads();
    if (s_overflow) mstate |= RSTATE_OVERFLOW;
    mm = min(s_count, TK_CAPB);
  }
  __syncthreads();
  finish_row(a, row, cv, cid, mm, mstate, reinterpret_cast<unsigned char*>(stage));
  if (tid == 0) {
    a.s.rowstate[row] = 0u;
    a.s.tickets[row] = 0u;
  }
}

}  // namespace nvs
