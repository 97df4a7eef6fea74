// Vocabulary-shard records exchanged through peer memory (sm_100a).
//
// Each GPU of a vocabulary split owns one exchange area (one cudaMalloc,
// shared with the other GPUs by CUDA IPC):
//   records [shards][rows][VS_REC_WORDS]  slot s written by shard s
//   flags   [16]   flags[s] = epoch: shard s's records of that call are here
//   acks    [16]   acks[s]  = epoch: shard s has merged that call, so its
//                  slot for this GPU may be overwritten
// Per call (epoch e, counted on the device) on GPU r: the shard kernel writes
// slot r of its own area, and each CTA that completes a row's record waits
// until every peer acked e-1 and stores that record into every peer's area
// over NVLink (plain stores, no multicast); the kernel's last CTA releases
// flags[r] = e on every GPU; the merge kernel waits until all flags
// reach e, merges, and its last CTA releases acks[r] = e on every peer. Every
// wait is bounded (about 2 s of %globaltimer); a merge that gives up returns
// -1 with NCB_FLAG_PEER_TIMEOUT for its rows, and a push that gives up stores
// and signals nothing, so its peers time out too.
#pragma once

#include "shard_record.cuh"

namespace nvs {

constexpr int PX_MAX = 16;           // shards (VM_MAX_SHARDS)
constexpr int PX_THREADS = 256;
constexpr int PX_CTAS_PER_PEER = 4;
constexpr uint32_t FLAG_PEER_TIMEOUT = 0x80u;

struct PeerLayout {
  size_t flags_off;  // bytes from the area base
  size_t acks_off;
  size_t bytes;
};
inline PeerLayout peer_layout(int shards, int max_rows) {
  PeerLayout l;
  const size_t rec = (size_t)shards * max_rows * VS_REC_WORDS * 4;
  l.flags_off = (rec + 255) / 256 * 256;
  l.acks_off = l.flags_off + 256;
  l.bytes = l.acks_off + 256;
  return l;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Waits until every word w[i] (i < n) reaches `target` (epochs increase);
// false when about 2 s passed first.
__device__ __forceinline__ bool wait_words_bounded(const uint32_t* w, int n, uint32_t target) {
  uint64_t t0 = 0;
  for (int i = 0; i < n; ++i) {
    while ((int32_t)(ld_acquire_sys(w + i) - target) < 0) {
      const uint64_t now = global_ns();
      if (t0 == 0) t0 = now;
      if (now - t0 > 2000000000ull) return false;
      __nanosleep(200);
    }
  }
  return true;
}

// Exchange arguments of a shard kernel that stores its records into the
// peers' areas itself (shards == 0: no peers, records stay local).
struct PxArgs {
  uint32_t* dst[PX_MAX];     // this shard's slot in every area (dst[me] unused)
  uint32_t* flag[PX_MAX];    // flags[me] in every area (own included)
  const uint32_t* acks;      // this GPU's acks[0..shards)
  uint32_t* ticket;          // local [2]: CTA count, failed waits; zero between launches
  uint32_t* epoch;           // local: the last call's epoch
  int shards, me;
};

// Epilogue of a shard kernel, every CTA once: the CTA that completed row
// `row`'s record (owner) stores it into every peer's area; the grid's last CTA
// releases this call's flag on every GPU. `rec` is the owner's finished record
// (written by this CTA before the call). All threads call.
__device__ __forceinline__ void shard_px_epilogue(const PxArgs& px, const uint32_t* rec, int row,
                                                  bool owner) {
  __shared__ int s_go, s_last;
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = __ldcg(px.epoch) + 1u;
    bool ok = true;
    if (owner)  // every peer has merged the previous call: its slot for us is free
      for (int s = 0; s < px.shards && ok; ++s)
        if (s != px.me) ok = wait_words_bounded(px.acks + s, 1, s_epoch - 1u);
    s_go = ok ? 1 : 0;
    if (!ok) atomicOr(px.ticket + 1, 1u);
  }
  __syncthreads();
  if (owner && s_go && px.shards > 1) {
    const size_t off = (size_t)row * VS_REC_WORDS;
    for (int i = tid; i < VS_REC_WORDS; i += blockDim.x) {
      const uint32_t v = __ldcg(rec + i);
      for (int s = 0; s < px.shards; ++s)
        if (s != px.me) px.dst[s][off + i] = v;
    }
  }
  __syncthreads();
  if (tid == 0) {
    // the barrier orders the CTA's peer stores before this one system fence
    if (owner && s_go && px.shards > 1) __threadfence_system();
    s_last = atomicAdd(px.ticket, 1u) == gridDim.x * gridDim.y - 1u;
  }
  __syncthreads();
  if (s_last && tid == 0) {
    __threadfence_system();
    // a call whose stores could not all go signals nothing: the merges time out
    if (atomicOr(px.ticket + 1, 0u) == 0u)
      for (int s = 0; s < px.shards; ++s) st_release_sys(px.flag[s], s_epoch);
    *px.epoch = s_epoch;
    px.ticket[1] = 0u;
    px.ticket[0] = 0u;
  }
}

}  // namespace nvs
