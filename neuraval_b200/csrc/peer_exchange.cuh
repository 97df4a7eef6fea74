// Vocabulary-shard records exchanged through peer memory (sm_100a).
//
// Each GPU of a vocabulary split owns one exchange area (one cudaMalloc,
// shared with the other GPUs by CUDA IPC), laid out for `shards` GPUs and
// `max_rows` rows (connect checks that every GPU's area has the same layout):
//   tagged [2][shards][max_rows][VS_REC_WORDS]  64-bit words (record word,
//                  epoch); slot s written by shard s, a call of epoch e uses
//                  copy e & 1
//   plain  [shards][rows][VS_REC_WORDS]  the merge's unpacked records (local)
//   own    [max_rows][VS_REC_WORDS]      the shard kernel's own records (local)
// Per call (epoch e, counted on the device) on GPU r: the shard kernel writes
// its records into `own`, and the CTA that completes a row's record stores it,
// each word tagged with e, into slot r of copy e & 1 of every GPU's area over
// NVLink (plain stores, no multicast). The merge kernel (one CTA per row)
// polls its own area until every word of its row carries e, unpacks the
// records, merges, and its last CTA advances the epoch. A word is one
// single-copy-atomic 8-byte access on both sides, so its tag proves its value:
// no fences, flags or acks. A peer's copy e & 1 is free again when this GPU
// stores call e + 2: this GPU's merge of e + 1 needed every peer's e + 1
// words, which each peer stores after its own merge of e has completed. Every
// wait is bounded (about 2 s of %globaltimer); a row whose words do not all
// arrive returns -1 with NCB_FLAG_PEER_TIMEOUT.
#pragma once

#include "shard_record.cuh"

namespace nvs {

constexpr int PX_MAX = 16;           // shards (VM_MAX_SHARDS)
constexpr int PX_THREADS = 256;
constexpr int PX_CTAS_PER_PEER = 4;
constexpr uint32_t FLAG_PEER_TIMEOUT = 0x80u;

struct PeerLayout {
  size_t plain_off;  // bytes from the area base
  size_t own_off;
  size_t bytes;
};
inline PeerLayout peer_layout(int shards, int max_rows) {
  PeerLayout l;
  const size_t rec = (size_t)shards * max_rows * VS_REC_WORDS;  // words of one copy
  l.plain_off = (2 * rec * 8 + 255) / 256 * 256;
  l.own_off = l.plain_off + (rec * 4 + 255) / 256 * 256;
  l.bytes = l.own_off + ((size_t)max_rows * VS_REC_WORDS * 4 + 255) / 256 * 256;
  return l;
}

__device__ __forceinline__ void st_u64_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_u64_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Exchange arguments of a shard kernel that stores its records into the
// peers' areas itself (shards == 0: no peers, records stay local).
struct PxArgs {
  uint64_t* tagged[PX_MAX];  // every GPU's tagged words as mapped here (own included)
  const uint32_t* epoch;     // local: the last merged call's epoch
  int shards, me, max_rows;
};

// Epilogue of a shard kernel, every CTA once: the CTA that completed row
// `row`'s record (owner) stores it, each word tagged with this call's epoch,
// into slot me of every GPU's area. `rec` is the owner's finished record
// (written by this CTA before the call). All threads call.
__device__ __forceinline__ void shard_px_epilogue(const PxArgs& px, const uint32_t* rec, int row,
                                                  bool owner) {
  if (!owner) return;
  const uint32_t e = __ldcg(px.epoch) + 1u;
  const uint64_t tag = (uint64_t)e << 32;
  const size_t off =
      (((size_t)(e & 1u) * px.shards + px.me) * px.max_rows + row) * (size_t)VS_REC_WORDS;
  for (int i = threadIdx.x; i < VS_REC_WORDS; i += blockDim.x) {
    const uint64_t w = tag | __ldcg(rec + i);
    for (int s = 0; s < px.shards; ++s) st_u64_sys(px.tagged[s] + off + i, w);
  }
}

}  // namespace nvs
