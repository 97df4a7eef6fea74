// Row-split batches: every GPU's tokens and flags gathered to every GPU
// through peer memory (sm_100a).
//
// TokenSampler.SampleNext (TokenSampler.cs:10-30) treats every row on its
// own, so a batch split by rows over G GPUs needs no exchange to sample; each
// GPU only needs every other GPU's tokens afterwards. Each GPU owns one gather
// area (one cudaMalloc, shared with the others by CUDA IPC):
//   copy[2][rows_total]     (token, flags) pairs of all rows, 8 bytes a row; a
//                           call of epoch e uses copy e & 1
//   staging[2][rows_total]  this GPU's own rows, written by the sampling kernels
//                           (sized by rows_total, which every GPU shares, so the
//                           flags sit at the same offset in every GPU's area)
//   flags[16]               flags[g] = e: GPU g's rows of call e are here
//   epoch                   the last call's epoch (this GPU's own counter)
// row_gather_kernel, after the sampling kernels of call e: stores the staged
// rows into copy e & 1 of every area over NVLink (one 8-byte store per row
// and GPU), a CTA barrier, then one thread fences at system scope, releases
// flags[me] = e on every GPU, waits (bounded, about 2 s) until its own
// flags[] all reach e, and the CTA copies that copy to the caller's outputs.
// A peer's copy e & 1 is free again when this GPU writes call e + 2: that
// peer released flags = e + 1, which it does only after its own copy-out of
// call e. A wait that gives up returns every row as -1 with
// NCB_FLAG_PEER_TIMEOUT.
#pragma once

#include "peer_exchange.cuh"

namespace nvs {

constexpr int RG_THREADS = 256;

struct RgLayout {
  size_t staging_off;  // bytes from the area base
  size_t flags_off;
  size_t epoch_off;
  size_t bytes;
};
inline RgLayout rg_layout(int rows_total) {
  RgLayout l;
  const size_t copies = (size_t)2 * rows_total * 8;
  l.staging_off = (copies + 255) / 256 * 256;
  l.flags_off = l.staging_off + ((size_t)2 * rows_total * 4 + 255) / 256 * 256;
  l.epoch_off = l.flags_off + 128;
  l.bytes = l.flags_off + 256;
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
  __shared__ int s_ok;
  // the sampling kernels (and their fix-up) come first on the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  char* own = g.area[g.me];
  uint32_t* epoch = reinterpret_cast<uint32_t*>(own + g.l.epoch_off);
  if (tid == 0) s_epoch = *epoch + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int c = (int)(e & 1u);
  const int32_t* st_tok = reinterpret_cast<const int32_t*>(own + g.l.staging_off);
  const uint32_t* st_flg = reinterpret_cast<const uint32_t*>(st_tok + g.rows_total);
  for (int i = tid; i < g.rows; i += RG_THREADS) {
    const uint2 v = make_uint2((uint32_t)st_tok[i], st_flg[i]);
    for (int p = 0; p < g.ranks; ++p)
      reinterpret_cast<uint2*>(g.area[p])[(size_t)c * g.rows_total + g.row_begin + i] = v;
  }
  // The barrier orders every thread's stores before thread 0's system fence
  // and its releases (the barrier-then-one-fence pattern of a grid barrier).
  __syncthreads();
  if (tid == 0) {
    // one fence, then relaxed flag stores: a release pattern for every flag
    __threadfence_system();
    for (int p = 0; p < g.ranks; ++p)
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;"
                   ::"l"(reinterpret_cast<uint32_t*>(g.area[p] + g.l.flags_off) + g.me), "r"(e)
                   : "memory");
    s_ok = wait_words_bounded(reinterpret_cast<const uint32_t*>(own + g.l.flags_off), g.ranks, e)
               ? 1 : 0;
  }
  __syncthreads();
  const uint2* cp = reinterpret_cast<const uint2*>(own) + (size_t)c * g.rows_total;
  for (int i = tid; i < g.rows_total; i += RG_THREADS) {
    uint2 v = make_uint2(0xffffffffu, FLAG_PEER_TIMEOUT);
    if (s_ok) v = __ldcv(cp + i);
    g.out_tok[i] = (int32_t)v.x;
    if (g.out_flg) g.out_flg[i] = v.y;
  }
  if (tid == 0) *epoch = e;
}

}  // namespace nvs
