// Merge of vocabulary-shard records (sm_100a): one CTA per row reads the
// records of all shards ([shards][rows][VS_REC_WORDS], shard order = column
// order) and finishes the row as the single-GPU kernels do.
//  - top-k rows: the global K-th largest value over the union of the shards'
//    candidates (TokenSampler.cs:73-84), every candidate >= it (:88-93), then
//    the shared finish (sort, exp, sequential sums, top-p, draw; :95-132);
//  - greedy rows: the first strict maximum over the shards' maxima, id 0 when
//    global id 0 is NaN (:38-51).
#pragma once

#include "shard_record.cuh"
#include "topk_kernels.cuh"
#include "warp_select.cuh"
#include "rank_select.cuh"
#include "peer_exchange.cuh"

namespace nvs {

constexpr int VM_THREADS = 512;
constexpr int VM_MAX_SHARDS = TK_CAPB / VS_CAP;  // 16: the union fits the candidate list
constexpr int VM_WORK = 32768;

inline size_t vm_smem_bytes() { return (size_t)TK_CAPB * 8 + VM_WORK + 256 * 4; }

struct MergeArgs {
  const uint32_t* recs;  // [shards][rows][VS_REC_WORDS]
  int shards;
  int rows;
  SampleArgs a;          // V = full vocabulary, p, uniforms, tokens, flags (probs unused)
  // peer-memory exchange only (null otherwise): this GPU's tagged words
  // ([2][shards][max_rows][VS_REC_WORDS]), unpacked into recs (then writable)
  // once every word of the row carries this call's epoch; the last CTA
  // advances the epoch
  const uint64_t* tagged;
  uint32_t* unpack;      // = recs, writable
  int max_rows;
  uint32_t* epoch;       // local: the last merged call's epoch
  uint32_t* ticket;      // local, zero between launches
};

__device__ void merge_row(const MergeArgs& g);

__global__ void __launch_bounds__(VM_THREADS) vocab_merge_kernel(const __grid_constant__ MergeArgs g) {
  __shared__ int s_last;
  const int tid = threadIdx.x, row = blockIdx.x;
  if (g.tagged) {
    const uint32_t e = __ldcg(g.epoch) + 1u;
    // every word of this row's records, each waited for (one deadline per
    // thread, about 2 s), unpacked into the plain layout merge_row reads
    const uint64_t* src = g.tagged + (size_t)(e & 1u) * g.shards * g.max_rows * VS_REC_WORDS;
    uint64_t t0 = 0;
    bool ok = true;
    for (int idx = tid; idx < g.shards * VS_REC_WORDS; idx += VM_THREADS) {
      const int s = idx / VS_REC_WORDS, i = idx - s * VS_REC_WORDS;
      const uint64_t* w = src + ((size_t)s * g.max_rows + row) * VS_REC_WORDS + i;
      uint64_t v = ld_u64_sys(w);
      for (int it = 0; ok && (uint32_t)(v >> 32) != e; ++it) {
        if ((it & 15) == 0) {
          const uint64_t t = global_ns();
          if (t0 == 0) t0 = t;
          else if (t - t0 > 2000000000ull) ok = false;
        }
        __nanosleep(100);
        v = ld_u64_sys(w);
      }
      g.unpack[((size_t)s * g.rows + row) * VS_REC_WORDS + i] = (uint32_t)v;
    }
    // launched as a programmatic dependent of the shard kernels (the words
    // above need no ordering: their tags prove them); everything else this
    // kernel reads was written before those kernels
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (__syncthreads_and(ok ? 1 : 0)) {
      merge_row(g);
    } else if (tid == 0) {
      g.a.tokens[row] = -1;
      if (g.a.flags) g.a.flags[row] = FLAG_PEER_TIMEOUT;
    }
    // the last CTA advances the epoch (every CTA has read the words by then)
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(g.ticket, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (s_last && tid == 0) {
      *g.epoch = e;
      *g.ticket = 0u;
    }
  } else {
    merge_row(g);
  }
}

__device__ void merge_row(const MergeArgs& g) {
  extern __shared__ __align__(128) unsigned char smem[];
  float* cv = reinterpret_cast<float*>(smem);                            // [CAPB]
  int* cid = reinterpret_cast<int*>(cv + TK_CAPB);                       // [CAPB]
  unsigned char* work = reinterpret_cast<unsigned char*>(cid + TK_CAPB);  // VM_WORK
  uint32_t* hist = reinterpret_cast<uint32_t*>(work + VM_WORK);          // [256]
  __shared__ int s_n[VM_MAX_SHARDS], s_off[VM_MAX_SHARDS + 1], s_cnt[VM_MAX_SHARDS];
  __shared__ uint32_t s_state, s_kth[VM_MAX_SHARDS], s_rst[VM_MAX_SHARDS];
  __shared__ int s_sh[2], s_count, s_ovf, s_nu;
  __shared__ float s_lb;

  const SampleArgs& a = g.a;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = g.shards;
  const size_t stride = (size_t)g.rows * VS_REC_WORDS;
  const uint32_t* rec0 = g.recs + (size_t)row * VS_REC_WORDS;

  // every shard's header at once (one thread per shard), then the offsets
  if (tid < G) {
    const uint32_t* r = rec0 + tid * stride;
    const uint32_t h0 = r[0], h1 = r[1], h2 = r[2], h3 = r[3];
    s_n[tid] = min((int)h0, VS_CAP);
    s_rst[tid] = h1;
    s_kth[tid] = h2;
    s_cnt[tid] = (int)h3;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t st = 0u;
    int off = 0;
    for (int s = 0; s < G; ++s) {
      s_off[s] = off;
      off += s_n[s];
      st |= s_rst[s];
    }
    s_off[G] = off;
    s_state = st;
  }
  __syncthreads();
  // the shard holding union entry j (entries in shard order)
  auto shard_of = [&](int j) {
    int s = 0;
    while (s + 1 < G && s_off[s + 1] <= j) ++s;
    return s;
  };
  const uint32_t st = s_state;
  const int total = s_off[G];

  if (a.p.greedy) {
    if (warp == 0) {
      Best b{0.0f, -1};
      for (int s = lane; s < G; s += 32) {
        const uint32_t* r = rec0 + s * stride;
        if (s_n[s] > 0) b = better(b, Best{__uint_as_float(r[VS_HDR]), (int)r[VS_HDR + VS_CAP]});
      }
      b = warp_best(b);
      if (lane == 0) {
        const bool bad = (st & FLAG_BAD_HISTORY) != 0u;
        const int tok = ((st & VS_NAN0) || b.i < 0) ? 0 : b.i;
        a.tokens[row] = bad ? -1 : tok;
        if (a.flags) a.flags[row] = bad ? FLAG_BAD_HISTORY : 0u;
      }
    }
    return;
  }

  if (st & (FLAG_NONFINITE | FLAG_BAD_HISTORY)) {
    finish_row(a, row, cv, cid, 0, st & (FLAG_NONFINITE | FLAG_BAD_HISTORY), work);
    return;
  }
  if (st & VS_OVF_UNKNOWN) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_TIES_OVERFLOW;
    }
    return;
  }
  if (total == 0) {  // no finite value in any shard
    finish_row(a, row, cv, cid, 0, FLAG_NONFINITE, work);
    return;
  }

  // union of the shards' candidates
  float* uv = reinterpret_cast<float*>(work);            // [CAPB]
  int* uid = reinterpret_cast<int*>(uv + TK_CAPB);        // [CAPB]
  const int K = min(a.p.top_k, a.V);
  {
    // Direct ranks over the candidates >= lb, the largest K-th value of a
    // shard that holds K values (a lower bound of the global K-th value).
    if (tid == 0) {
      float lb = -INFINITY;
      for (int s = 0; s < G; ++s)
        if (s_cnt[s] >= K) lb = fmaxf(lb, __uint_as_float(s_kth[s]));
      s_lb = lb;
      s_nu = 0;
    }
    __syncthreads();
    const float lb = s_lb;
    // all shards' entries in one flat pass: every thread's loads are in flight
    // together instead of one shard after another
    for (int j = tid; j < total; j += VM_THREADS) {
      const int s = shard_of(j);
      const uint32_t* r = rec0 + s * stride;
      const int i = j - s_off[s];
      const float v = __uint_as_float(r[VS_HDR + i]);
      const int id = (int)r[VS_HDR + VS_CAP + i];
      if (v >= lb) {
        const int slot = atomicAdd(&s_nu, 1);
        if (slot < RS_MAX) {
          uv[slot] = v;
          uid[slot] = id;
        }
      }
    }
    __syncthreads();
    const int U = s_nu;
    if (U <= RS_MAX) {
      uint64_t* sk = reinterpret_cast<uint64_t*>(work + 16384);  // [64]
      float* sw = reinterpret_cast<float*>(work + 16384 + 512);  // [64]
      float* s64 = sw + 64;                                      // [64]
      const RankSel rs = cta_rank_select(uv, uid, U, K, reinterpret_cast<uint64_t*>(cv), sk, sw);
      if (rs.ok) {
        if (tid == 0) {
          bool cut = false;
          if (st & VS_OVF_AT_KTH)
            for (int s = 0; s < G; ++s)
              if ((s_rst[s] & VS_OVF_AT_KTH) && __uint_as_float(s_kth[s]) == cand_val(rs.x))
                cut = true;
          s_ovf = cut ? 1 : 0;
        }
        __syncthreads();
        if (s_ovf) {
          if (tid == 0) {
            a.tokens[row] = -1;
            if (a.flags) a.flags[row] = FLAG_TIES_OVERFLOW;
          }
          return;
        }
        if (warp == 0) {
          const uint64_t k0 = lane < rs.c ? sk[lane] : 0ull;
          const uint64_t k1 = lane + 32 < rs.c ? sk[lane + 32] : 0ull;
          finish_weights_warp(a, row, k0, k1, rs.c, sw, s64, rs.slow, a.uniforms[row]);
        }
        return;
      }
    }
    __syncthreads();
  }
  for (int j = tid; j < total; j += VM_THREADS) {
    const int s = shard_of(j);
    const uint32_t* r = rec0 + s * stride;
    const int i = j - s_off[s];
    uv[j] = __uint_as_float(r[VS_HDR + i]);
    uid[j] = (int)r[VS_HDR + VS_CAP + i];
  }
  __syncthreads();
  // fewer than K finite values in the whole row: every finite value is a
  // candidate (key 0 below), the row's -inf values would only add zero weights
  const uint32_t key = cta_kth_largest([&](int i) { return fkey(uv[i]); }, total, K, hist, s_sh);
  const float theta = key <= fkey(-INFINITY) ? -INFINITY : kval(key);
  if (tid == 0) {
    // a shard that cut ties at its K-th value matters only when that value is
    // the global K-th value
    bool cut = false;
    if (st & VS_OVF_AT_KTH)
      for (int s = 0; s < G; ++s)
        if ((s_rst[s] & VS_OVF_AT_KTH) && __uint_as_float(s_kth[s]) == theta) cut = true;
    s_ovf = cut ? 1 : 0;
    s_count = 0;
  }
  __syncthreads();
  if (s_ovf) {
    if (tid == 0) {
      a.tokens[row] = -1;
      if (a.flags) a.flags[row] = FLAG_TIES_OVERFLOW;
    }
    return;
  }
  for (int i0 = 0; i0 < total; i0 += VM_THREADS) {
    const int i = i0 + tid;
    const bool ok = i < total && fkey(uv[i]) >= key;
    warp_append(ok, ok ? uv[i] : 0.f, ok ? uid[i] : 0, cv, cid, &s_count, &s_ovf);
  }
  __syncthreads();
  const int m = min(s_count, TK_CAPB);
  // the union is dead now: the finish reuses the work area
  if (m > 0 && m <= 64) {
    if (warp == 0) finish_row_warp(a, row, cv, cid, m, reinterpret_cast<float*>(work));
  } else {
    finish_row(a, row, cv, cid, m, 0u, work);
  }
}

}  // namespace nvs
