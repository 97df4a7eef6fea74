// Row-split batches: every GPU's tokens and flags gathered to every GPU
// through peer memory (sm_100a).
//
// TokenSampler.SampleNext (TokenSampler.cs:10-30) treats every row on its
// own, so a batch split by rows over G GPUs needs no exchange to sample; each
// GPU only needs every other GPU's tokens afterwards. Each GPU owns one gather
// area (one cudaMalloc, shared with the others by CUDA IPC):
//   copy[2][rows_total][2]  64-bit words: (token, epoch) and (flags, epoch) of
//                           every row; a call of epoch e uses copy e & 1
//   staging[2][rows_total]  this GPU's own rows, written by the sampling kernels
//                           (sized by rows_total, which every GPU shares, so
//                           the copies sit at the same offset in every area)
//   epoch                   the last call's epoch (this GPU's own counter)
// row_gather_kernel, after the sampling kernels of call e: stores each of its
// rows as two 64-bit words tagged with e into copy e & 1 of every GPU's area
// over NVLink, then polls its own copy until every word carries e (bounded,
// about 2 s) and copies the rows out. A word is one single-copy-atomic 8-byte
// access on both sides, so its tag proves its value is this call's: no fence,
// no separate flag. A peer's copy e & 1 is free again when this GPU writes
// call e + 2: this GPU finished call e + 1 only after every peer had stored
// its e + 1 words, which each peer does after its own call e (copy-out
// included) has completed. A word still stale after the wait makes its row
// -1 with NCB_FLAG_PEER_TIMEOUT.
#pragma once

#include "peer_exchange.cuh"

namespace nvs {

constexpr int RG_THREADS = 256;

struct RgLayout {
  size_t staging_off;  // bytes from the area base
  size_t epoch_off;
  size_t bytes;
};
inline RgLayout rg_layout(int rows_total) {
  RgLayout l;
  const size_t copies = (size_t)2 * rows_total * 16;
  l.staging_off = (copies + 255) / 256 * 256;
  l.epoch_off = l.staging_off + ((size_t)2 * rows_total * 4 + 255) / 256 * 256;
  l.bytes = l.epoch_off + 256;
  return l;
}

struct RgArgs {
  char* area[PX_MAX];   // every GPU's area as mapped here (own included)
  RgLayout l;
  int ranks, me, rows_total, row_begin, rows;
  int32_t* out_tok;     // [rows_total]
  uint32_t* out_flg;    // [rows_total], may be null
};

__global__ void __launch_bounds__(RG_THREADS) row_gather_kernel(const __grid_constant__ RgArgs g) {
  __shared__ uint32_t s_epoch;
  // the sampling kernels (and their fix-up) come first on the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  char* own = g.area[g.me];
  uint32_t* epoch = reinterpret_cast<uint32_t*>(own + g.l.epoch_off);
  if (tid == 0) s_epoch = *epoch + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const size_t cbase = (size_t)(e & 1u) * g.rows_total * 2;  // in words
  const int32_t* st_tok = reinterpret_cast<const int32_t*>(own + g.l.staging_off);
  const uint32_t* st_flg = reinterpret_cast<const uint32_t*>(st_tok + g.rows_total);
  const uint64_t tag = (uint64_t)e << 32;
  for (int i = tid; i < g.rows; i += RG_THREADS) {
    const uint64_t wt = tag | (uint32_t)st_tok[i];
    const uint64_t wf = tag | st_flg[i];
    const size_t w = cbase + (size_t)(g.row_begin + i) * 2;
    for (int p = 0; p < g.ranks; ++p) {
      uint64_t* c = reinterpret_cast<uint64_t*>(g.area[p]) + w;
      st_u64_sys(c, wt);
      st_u64_sys(c + 1, wf);
    }
  }
  // every row of the batch from the own copy, each word waited for (one
  // deadline per thread, about 2 s)
  const uint64_t* cp = reinterpret_cast<const uint64_t*>(own) + cbase;
  uint64_t t0 = 0;
  bool late = false;
  for (int i = tid; i < g.rows_total; i += RG_THREADS) {
    uint64_t wt = ld_u64_sys(cp + 2 * i), wf = ld_u64_sys(cp + 2 * i + 1);
    for (int it = 0; !late && ((uint32_t)(wt >> 32) != e || (uint32_t)(wf >> 32) != e); ++it) {
      if ((it & 15) == 0) {
        const uint64_t t = global_ns();
        if (t0 == 0) t0 = t;
        else if (t - t0 > 2000000000ull) late = true;
      }
      __nanosleep(100);
      wt = ld_u64_sys(cp + 2 * i);
      wf = ld_u64_sys(cp + 2 * i + 1);
    }
    const bool ok = (uint32_t)(wt >> 32) == e && (uint32_t)(wf >> 32) == e;
    g.out_tok[i] = ok ? (int32_t)(uint32_t)wt : -1;
    if (g.out_flg) g.out_flg[i] = ok ? (uint32_t)wf : FLAG_PEER_TIMEOUT;
  }
  __syncthreads();
  if (tid == 0) *epoch = e;
}

}  // namespace nvs
