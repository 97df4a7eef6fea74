// navsampler: C ABI of the sm_100a sampling library (include/navsampler.h).
//
// Host-side conventions follow Neuraval.Cuda.Native/src/navcuda.cu: extern "C"
// exports with default visibility (:9-13), NcbStatus codes (:19-29) and a
// process-wide last status (:31-39, read through ncb_sampler_last_status as
// CudaDevice.ThrowIfError does with ncb_cuda_last_status). Unlike navcuda's
// global recursive mutex, a sampler handle carries its own lock, and the
// host-array entry point reuses handle-owned device buffers instead of
// allocating per call.
#include "navsampler.h"

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <array>
#include <mutex>
#include <vector>

#include "fullvocab_kernels.cuh"
#include "logits_ops.cuh"
#include "nucleus_kernel.cuh"
#include "sampler_device.cuh"
#include "topk_kernels.cuh"
#include "topk_ldg_kernel.cuh"
#include "topk_chunk_kernels.cuh"
#include "vocab_merge.cuh"
#include "row_gather.cuh"

namespace {

std::atomic<int> g_last_status{NCB_OK};

int set_status(int st) {
  g_last_status.store(st);
  return st;
}

struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev == dev) {
      prev = -1;  // nothing to restore
      ok = true;
    } else {
      ok = cudaSetDevice(dev) == cudaSuccess;
    }
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int round_up(int x, int m) { return (x + m - 1) / m * m; }
int pow2_at_least(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace

// The last status of every entry point, also for those compiled in other
// translation units of the library (hidden symbol).
int ncb_record_status(int st) { return set_status(st); }

struct NcbSampler {
  int device = 0;
  int max_rows = 0, max_vocab = 0, max_history = 0;
  int num_sms = 0;
  int max_ctas = 0;
  int max_smem_optin = 0;
  int max_dyn_smem = 0;  // dynamic shared memory a launch may request (opt-in minus static)
  int forced_splits = 0;  // NAVSAMPLER_SPLITS at creation (tuning only)
  bool chunked = true;    // NAVSAMPLER_CHUNKED=0 at creation: top-k <= 64 on the one-CTA-per-row kernel
  int ck_jmax = 0;        // chunks per row the chunked top-k scratch holds
  std::recursive_mutex mu;  // host-array entry points call the device ones under it
  void* scratch = nullptr;
  nvs::Scratch s{};
  nvs::FvScratch fv{};
  // host-array staging (allocated on first ncb_sample_rows call)
  float* h_logits_dev = nullptr;
  int32_t* h_hist_dev = nullptr;
  int32_t* h_hoff_dev = nullptr;
  float* h_u_dev = nullptr;
  int32_t* h_tok_dev = nullptr;
  uint32_t* h_flags_dev = nullptr;
  float* h_probs_dev = nullptr;
  size_t h_hist_cap = 0;
  cudaStream_t host_stream = nullptr;  // sampling and the copies out
  int32_t* h_out_pinned = nullptr;     // [2][max_rows] tokens and flags on their way out
  cudaStream_t copy_stream = nullptr;  // the copies in, slice by slice
  cudaEvent_t slice_ev[8] = {};        // slice i of the logits is on the device
  // vocabulary shards exchanged through peer memory
  char* px_area = nullptr;  // this GPU's exchange area (tagged, unpacked and own records)
  int px_shards = 0, px_me = -1;
  bool px_connected = false;
  nvs::PeerLayout px_layout{};
  char* px_base[nvs::PX_MAX] = {};  // every shard's area as mapped here
  bool px_imported[nvs::PX_MAX] = {};
  bool px_pushed = false;
  // rows split over GPUs: tokens and flags gathered through peer memory
  char* rg_area = nullptr;
  int rg_ranks = 0, rg_me = -1, rg_rows_total = 0;
  bool rg_connected = false;
  nvs::RgLayout rg_layout{};
  char* rg_base[nvs::PX_MAX] = {};
  bool rg_imported[nvs::PX_MAX] = {};
};

namespace {
// Exchange areas exported by this process: a handle of our own resolves to
// the pointer directly (CUDA IPC does not open a process's own handles).
std::mutex g_px_mu;
std::vector<std::pair<std::array<char, sizeof(cudaIpcMemHandle_t)>, char*>> g_px_local;
}  // namespace

static bool params_ok(const NcbSamplerParams* p) {
  if (!p) return false;
  // GenerationOptions.Create (GenerationOptions.cs:56-72)
  if (!(p->temperature > 0.0f)) return false;
  if (!(p->top_p > 0.0f) || p->top_p > 1.0f) return false;
  if (p->top_k <= 0) return false;
  if (!(p->repetition_penalty > 0.0f)) return false;
  if (p->frequency_penalty != p->frequency_penalty) return false;
  if (p->presence_penalty != p->presence_penalty) return false;
  return true;
}

static nvs::Params to_params(const NcbSamplerParams* p) {
  nvs::Params q;
  q.greedy = p->greedy;
  q.temperature = p->temperature;
  q.top_p = p->top_p;
  q.top_k = p->top_k;
  q.repetition_penalty = p->repetition_penalty;
  q.frequency_penalty = p->frequency_penalty;
  q.presence_penalty = p->presence_penalty;
  return q;
}

// Column splits per row: enough CTAs to fill the GPU twice over when rows are
// few, never a segment shorter than 8192 columns. NAVSAMPLER_SPLITS overrides
// (tuning only).
static int choose_splits(int rows, int V, int num_sms, int forced) {
  if (forced >= 1) return forced;
  int S = (2 * num_sms) / (rows > 0 ? rows : 1);
  if (S < 1) S = 1;
  int maxS = V / 8192;
  if (maxS < 1) maxS = 1;
  if (S > maxS) S = maxS;
  return S;
}

// Column segments per row for the k <= 64 top-k kernel: every extra segment
// of a row costs its own head and tail plus the merge of the row's segments
// (about 12 us on a B200), against a stream of 4*V/S bytes at one CTA's rate
// (about 26 GB/s). S minimises 12*[S > 1] + 4V / (S * 26e3) us over powers of
// two up to 8 that keep the grid in one wave (rows * S <= 2 * SMs) and
// segments of at least 8192 columns. NAVSAMPLER_SPLITS overrides.
static int choose_splits_topk(int rows, int V, int num_sms, int forced) {
  if (forced >= 1) return forced;
  int best = 1;
  double tbest = 4.0 * V / 26000.0;
  for (int S = 2; S <= 8; S *= 2) {
    if ((long long)rows * S > 2LL * num_sms || V / S < 8192) break;
    const double t = 12.0 + 4.0 * V / (S * 26000.0);
    if (t < tbest) {
      tbest = t;
      best = S;
    }
  }
  return best;
}

// The dynamic shared memory limit of every kernel is raised once per handle
// (a per-function attribute), not on every call.
static bool raise_smem_limits(int limit) {
  bool ok = true;
  auto set = [&](const void* fn) {
    // static + dynamic shared memory may not exceed the opt-in limit
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess) {
      ok = false;
      return;
    }
    const int dyn = limit - (int)fa.sharedSizeBytes;
    ok = ok && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) ==
                   cudaSuccess;
  };
  set((const void*)nvs::topk_kernel<true>);
  set((const void*)nvs::topk_kernel<false>);
  set((const void*)nvs::topk_ldg_kernel<true>);
  set((const void*)nvs::topk_ldg_kernel<false>);
  set((const void*)nvs::greedy_kernel<true>);
  set((const void*)nvs::greedy_kernel<false>);
  set((const void*)nvs::topk_ldg_kernel<true, true>);
  set((const void*)nvs::topk_ldg_kernel<false, true>);
  set((const void*)nvs::greedy_kernel<true, true>);
  set((const void*)nvs::greedy_kernel<false, true>);
  set((const void*)nvs::vocab_merge_kernel);
  set((const void*)nvs::nucleus_kernel<true, nvs::NcOne>);
  set((const void*)nvs::nucleus_kernel<false, nvs::NcOne>);
  set((const void*)nvs::nucleus_kernel<true, nvs::NcTwo>);
  set((const void*)nvs::nucleus_kernel<false, nvs::NcTwo>);
  set((const void*)nvs::fullvocab_kernel<true>);
  set((const void*)nvs::fullvocab_kernel<false>);
  set((const void*)nvs::topk_chunk_kernel<false>);
  set((const void*)nvs::topk_chunk_finish_kernel<true, 4>);
  set((const void*)nvs::topk_chunk_finish_kernel<false, 4>);
  set((const void*)nvs::topk_chunk_finish_kernel<true, 8>);
  set((const void*)nvs::topk_chunk_finish_kernel<false, 8>);
  set((const void*)nvs::topk_chunk_kernel<true>);
  set((const void*)nvs::topk_chunk_finish_kernel<true, 4, true>);
  set((const void*)nvs::topk_chunk_finish_kernel<false, 4, true>);
  set((const void*)nvs::topk_chunk_finish_kernel<true, 8, true>);
  set((const void*)nvs::topk_chunk_finish_kernel<false, 8, true>);
  set((const void*)nvs::fullvocab_fixup_kernel<true>);
  set((const void*)nvs::fullvocab_fixup_kernel<false>);
  set((const void*)nvs::filter_top_p_kernel);
  set((const void*)nvs::repetition_penalty_kernel);
  set((const void*)nvs::frequency_presence_kernel);
  return ok;
}

extern "C" {

NCB_API int ncb_sampler_params_validate(const NcbSamplerParams* params) {
  return set_status(params_ok(params) ? NCB_OK : NCB_ERROR_INVALID_ARGUMENT);
}

NCB_API int ncb_sampler_last_status(void) { return g_last_status.load(); }

NCB_API int ncb_sampler_full_sort_rows(NcbSampler* h, uint64_t* out_rows) {
  if (!h || !out_rows) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  uint32_t n = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&n, h->s.stats, sizeof(n), cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_status(NCB_ERROR_COPY_FAILED);
  *out_rows = n;
  return set_status(NCB_OK);
}

NCB_API int ncb_fast_exp_max_steps(float x_lo, float x_hi, uint32_t* out_steps) {
  if (!out_steps || !(x_lo <= x_hi) || !(x_hi <= 0.0f)) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  uint32_t* d = nullptr;
  if (cudaMalloc(&d, sizeof(uint32_t)) != cudaSuccess) return set_status(NCB_ERROR_ALLOC_FAILED);
  int st = NCB_OK;
  if (cudaMemset(d, 0, sizeof(uint32_t)) != cudaSuccess) st = NCB_ERROR_LAUNCH_FAILED;
  // every float in [x_lo, x_hi]: for x <= 0 the bit pattern grows as x falls,
  // from 0x80000000 (-0)
  const uint32_t k0 = x_hi == 0.0f ? 0x80000000u : __builtin_bit_cast(uint32_t, x_hi);
  const uint32_t k1 = __builtin_bit_cast(uint32_t, x_lo);
  if (st == NCB_OK) {
    nvs::fast_exp_steps_kernel<<<148 * 8, 256>>>(k0, k1, d);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
      st = NCB_ERROR_LAUNCH_FAILED;
  }
  if (st == NCB_OK && cudaMemcpy(out_steps, d, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
    st = NCB_ERROR_COPY_FAILED;
  cudaFree(d);
  return set_status(st);
}

NCB_API const char* ncb_sampler_status_message(int status) {
  switch (status) {
    case NCB_OK: return "OK";
    case NCB_ERROR_NO_DEVICE: return "no CUDA device";
    case NCB_ERROR_INIT_FAILED: return "could not initialise the CUDA device";
    case NCB_ERROR_ALLOC_FAILED: return "device allocation failed";
    case NCB_ERROR_COPY_FAILED: return "host/device copy failed";
    case NCB_ERROR_LAUNCH_FAILED: return "kernel launch failed";
    case NCB_ERROR_NOT_INITIALIZED: return "sampler handle not initialised";
    case NCB_ERROR_INVALID_ARGUMENT: return "invalid argument";
    case NCB_ERROR_CAPACITY: return "size exceeds the sampler handle's capacity";
    default: return "unknown status";
  }
}

NCB_API int ncb_sampler_create(int device, int max_rows, int max_vocab, int max_history,
                               NcbSampler** out) {
  if (!out) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  *out = nullptr;
  if (max_rows <= 0 || max_vocab <= 0 || max_history < 0 || device < 0)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0)
    return set_status(NCB_ERROR_NO_DEVICE);
  if (device >= count) return set_status(NCB_ERROR_NO_DEVICE);
  DeviceGuard g(device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);

  NcbSampler* h = new NcbSampler();
  h->device = device;
  h->max_rows = max_rows;
  h->max_vocab = max_vocab;
  h->max_history = max_history;
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&h->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  h->max_dyn_smem = h->max_smem_optin - 4096;  // every kernel uses < 4 KiB of static smem
  if (const char* e = std::getenv("NAVSAMPLER_SPLITS")) h->forced_splits = std::atoi(e);
  if (const char* e = std::getenv("NAVSAMPLER_CHUNKED")) h->chunked = std::atoi(e) != 0;
  h->ck_jmax = nvs::ck_chunks(max_vocab);
  if (h->ck_jmax > nvs::CK_MAX_CHUNKS) h->ck_jmax = nvs::CK_MAX_CHUNKS;
  h->max_ctas = max_rows > 2 * h->num_sms ? max_rows : 2 * h->num_sms;
  if (h->forced_splits > 0 && (size_t)max_rows * h->forced_splits > (size_t)h->max_ctas)
    h->max_ctas = max_rows * h->forced_splits;
  // a single-row call may split into V/8192 segments
  const int vsplits = max_vocab / 8192 + 1;
  if (h->max_ctas < vsplits) h->max_ctas = vsplits;

  // One scratch allocation, carved into aligned pieces.
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t mc = (size_t)h->max_ctas;
  const size_t o_cv = carve(mc * nvs::TK_CAPB * sizeof(float));
  const size_t o_ci = carve(mc * nvs::TK_CAPB * sizeof(int32_t));
  const size_t o_cn = carve(mc * sizeof(int32_t));
  const size_t o_tk = carve((size_t)max_rows * sizeof(uint32_t));
  const size_t o_rs = carve((size_t)max_rows * sizeof(uint32_t));
  const size_t o_gv = carve(mc * sizeof(float));
  const size_t o_gi = carve(mc * sizeof(int32_t));
  const size_t o_er = carve(sizeof(uint32_t));
  const size_t o_fx = carve((size_t)max_rows * sizeof(uint32_t));
  const size_t o_px = carve(4 * sizeof(uint32_t));
  const size_t o_st = carve(4 * sizeof(uint32_t));
  const size_t ck_groups = (size_t)max_rows * h->ck_jmax * nvs::CK_WARPS;
  const size_t o_ck = carve(ck_groups * nvs::CK_KEYS * sizeof(uint2));
  const size_t o_cc = carve(ck_groups * sizeof(uint32_t));
  const size_t o_ct = carve(ck_groups * sizeof(float));
  const nvs::FvLayout fl = nvs::fv_layout(max_rows, max_vocab);
  const size_t o_fv = carve(fl.total_bytes);
  if (cudaMalloc(&h->scratch, off) != cudaSuccess) {
    delete h;
    return set_status(NCB_ERROR_ALLOC_FAILED);
  }
  char* b = static_cast<char*>(h->scratch);
  h->s.cand_v = reinterpret_cast<float*>(b + o_cv);
  h->s.cand_id = reinterpret_cast<int32_t*>(b + o_ci);
  h->s.cand_n = reinterpret_cast<int32_t*>(b + o_cn);
  h->s.tickets = reinterpret_cast<uint32_t*>(b + o_tk);
  h->s.rowstate = reinterpret_cast<uint32_t*>(b + o_rs);
  h->s.gv = reinterpret_cast<float*>(b + o_gv);
  h->s.gi = reinterpret_cast<int32_t*>(b + o_gi);
  h->s.error_word = reinterpret_cast<uint32_t*>(b + o_er);
  h->s.fixup = reinterpret_cast<uint32_t*>(b + o_fx);
  h->s.px_ticket = reinterpret_cast<uint32_t*>(b + o_px);
  h->s.stats = reinterpret_cast<uint32_t*>(b + o_st);
  h->s.ck_keys = reinterpret_cast<uint2*>(b + o_ck);
  h->s.ck_cnt = reinterpret_cast<uint32_t*>(b + o_cc);
  h->s.ck_cut = reinterpret_cast<float*>(b + o_ct);
  h->fv = nvs::fv_carve(b + o_fv, fl);
  // tickets/rowstate/error word must start at zero; the kernels restore zero
  if (!raise_smem_limits(h->max_smem_optin) || cudaMemset(h->scratch, 0, off) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(h->scratch);
    delete h;
    return set_status(NCB_ERROR_INIT_FAILED);
  }
  *out = h;
  return set_status(NCB_OK);
}

NCB_API int ncb_sampler_destroy(NcbSampler* h) {
  if (!h) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  {
    DeviceGuard g(h->device);
    cudaDeviceSynchronize();
    if (h->px_area) {
      for (int s = 0; s < nvs::PX_MAX; ++s)
        if (h->px_imported[s]) cudaIpcCloseMemHandle(h->px_base[s]);
      std::lock_guard<std::mutex> lk(g_px_mu);
      for (size_t i = 0; i < g_px_local.size(); ++i)
        if (g_px_local[i].second == h->px_area) {
          g_px_local.erase(g_px_local.begin() + i);
          break;
        }
      cudaFree(h->px_area);
    }
    if (h->rg_area) {
      for (int s = 0; s < nvs::PX_MAX; ++s)
        if (h->rg_imported[s]) cudaIpcCloseMemHandle(h->rg_base[s]);
      std::lock_guard<std::mutex> lk(g_px_mu);
      for (size_t i = 0; i < g_px_local.size(); ++i)
        if (g_px_local[i].second == h->rg_area) {
          g_px_local.erase(g_px_local.begin() + i);
          break;
        }
      cudaFree(h->rg_area);
    }
    cudaFree(h->scratch);
    cudaFree(h->h_logits_dev);
    cudaFree(h->h_hist_dev);
    cudaFree(h->h_hoff_dev);
    cudaFree(h->h_u_dev);
    cudaFree(h->h_tok_dev);
    cudaFree(h->h_flags_dev);
    cudaFree(h->h_probs_dev);
    if (h->host_stream) cudaStreamDestroy(h->host_stream);
    if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
    if (h->h_out_pinned) cudaFreeHost(h->h_out_pinned);
    for (cudaEvent_t e : h->slice_ev)
      if (e) cudaEventDestroy(e);
  }
  delete h;
  return set_status(NCB_OK);
}

// Launches the sampling kernels for one batch; caller holds h->mu and the
// device guard.
static int launch_sample(NcbSampler* h, const float* d_logits, int rows, int V,
                         const int32_t* d_hist, const int32_t* d_hoff, const float* d_u,
                         const NcbSamplerParams* prm, int32_t* d_tok, uint32_t* d_flags,
                         float* d_probs, cudaStream_t stream) {
  if (rows == 0) return NCB_OK;
  nvs::SampleArgs a{};
  a.logits = d_logits;
  a.V = V;
  a.hist = d_hist;
  a.hoff = d_hoff;
  a.uniforms = d_u;
  a.p = to_params(prm);
  a.tokens = d_tok;
  a.flags = d_flags;
  a.probs = d_probs;
  a.s = h->s;
  const bool counts = (prm->frequency_penalty != 0.0f || prm->presence_penalty != 0.0f);
  a.h_cap = counts ? pow2_at_least(h->max_history > 0 ? h->max_history : 1) : 0;

  if (prm->greedy) {
    int S = choose_splits(rows, V, h->num_sms, h->forced_splits);
    a.seg_len = round_up((V + S - 1) / S, 4);
    S = (V + a.seg_len - 1) / a.seg_len;
    a.bm_words = (a.seg_len + 31) / 32 + 1;
    const size_t smem = (size_t)a.bm_words * 4 + (size_t)a.h_cap * 4;
    if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    dim3 grid(S, rows);
    if (counts) {
      nvs::greedy_kernel<true><<<grid, nvs::GR_THREADS, smem, stream>>>(a);
    } else {
      nvs::greedy_kernel<false><<<grid, nvs::GR_THREADS, smem, stream>>>(a);
    }
    return cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED;
  }

  const int K = prm->top_k < V ? prm->top_k : V;
  // The chunked kernels: wide rows whose penalties can only lower a value,
  // no probability output, and at most ~1.5 of the row's top K expected in
  // one warp's 1024 values (a warp keeps >= 8 of them; a warp holding more
  // sends the row to the exact fix-up).
  const bool lowering = !(prm->repetition_penalty < 1.0f) && !(prm->frequency_penalty < 0.0f) &&
                        !(prm->presence_penalty < 0.0f);
  const int J = nvs::ck_chunks(V);
  if (h->chunked && h->forced_splits == 0 && K < V && K <= nvs::TL_KMAX && !d_probs && lowering &&
      V >= 8192 && J <= h->ck_jmax && 683LL * K <= (long long)V) {
    a.bm_words = (V + 31) / 32 + 1;
    const size_t smem = nvs::fk_smem_bytes(a.bm_words, a.h_cap);
    if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const int nchunks = rows * J;
    const size_t ring = nvs::cr_smem_bytes();
    if ((int)ring > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    cudaLaunchConfig_t c1{};
    c1.gridDim = dim3(nchunks < h->num_sms ? nchunks : h->num_sms);
    c1.blockDim = dim3(nvs::CR_THREADS);
    c1.dynamicSmemBytes = ring;
    c1.stream = stream;
    c1.attrs = attr;
    c1.numAttrs = 1;
    if (cudaLaunchKernelEx(&c1, nvs::topk_chunk_kernel<false>, a, J, nchunks) != cudaSuccess)
      return NCB_ERROR_LAUNCH_FAILED;
    cudaLaunchConfig_t c2{};
    c2.gridDim = dim3(rows);
    c2.blockDim = dim3(nvs::FK_THREADS);
    c2.dynamicSmemBytes = smem;
    c2.stream = stream;
    c2.attrs = attr;
    c2.numAttrs = 1;
    const bool wide = J * nvs::CK_WARPS * nvs::CK_KEYS > 4 * nvs::FK_THREADS;
    cudaError_t e;
    if (counts)
      e = wide ? cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<true, 8>, a, J)
               : cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<true, 4>, a, J);
    else
      e = wide ? cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<false, 8>, a, J)
               : cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<false, 4>, a, J);
    if (e != cudaSuccess) return NCB_ERROR_LAUNCH_FAILED;
    // rows the finish could not prove (normally none)
    return nvs::launch_fullvocab(h->fv, a, rows, K, h->max_dyn_smem, stream, true, 8);
  }
  if (K < V && K <= nvs::TL_KMAX) {
    int S = choose_splits_topk(rows, V, h->num_sms, h->forced_splits);
    a.seg_len = round_up((V + S - 1) / S, 4);
    S = (V + a.seg_len - 1) / a.seg_len;
    if ((size_t)rows * S > (size_t)h->max_ctas) return NCB_ERROR_CAPACITY;
    a.bm_words = (a.seg_len + 31) / 32 + 1;
    const size_t smem = nvs::tl_smem_bytes(a.bm_words, a.h_cap);
    if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    // a programmatic dependent launch: scheduled while the previous kernel on
    // the stream finishes; the kernel waits for it before its first read
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(S, rows);
    cfg.blockDim = dim3(nvs::TL_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = counts ? cudaLaunchKernelEx(&cfg, nvs::topk_ldg_kernel<true, false>, a)
                                 : cudaLaunchKernelEx(&cfg, nvs::topk_ldg_kernel<false, false>, a);
    if (e != cudaSuccess) return NCB_ERROR_LAUNCH_FAILED;
    // rows whose ties overflowed the candidate buffers (normally none)
    return nvs::launch_fullvocab(h->fv, a, rows, K, h->max_dyn_smem, stream, true, 8);
  }
  if (K < V && K <= nvs::TK_KMAX) {
    int S = choose_splits(rows, V, h->num_sms, h->forced_splits);
    a.seg_len = round_up((V + S - 1) / S, 4);
    S = (V + a.seg_len - 1) / a.seg_len;
    if ((size_t)rows * S > (size_t)h->max_ctas) return NCB_ERROR_CAPACITY;
    a.bm_words = (a.seg_len + 31) / 32 + 1;
    const size_t smem = (size_t)nvs::TK_NSTAGE * nvs::TK_CHUNK * 4 + (size_t)nvs::TK_CAPB * 8 +
                        256 * 4 + nvs::TK_NSTAGE * 8 + (size_t)a.bm_words * 4 +
                        (size_t)a.h_cap * 4;
    if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    dim3 grid(S, rows);
    if (counts) {
      nvs::topk_kernel<true><<<grid, nvs::TK_THREADS, smem, stream>>>(a);
    } else {
      nvs::topk_kernel<false><<<grid, nvs::TK_THREADS, smem, stream>>>(a);
    }
    if (cudaGetLastError() != cudaSuccess) return NCB_ERROR_LAUNCH_FAILED;
    // rows whose ties overflowed the top-k buffers (normally none)
    const int fst = nvs::launch_fullvocab(h->fv, a, rows, K, h->max_dyn_smem, stream, true, 8);
    return fst;
  }

  // Full-vocabulary nucleus (no effective top-k) and very large top-k: the
  // bucketed kernel, with the full-sort kernel for the rows it hands over and
  // for calls that want the probabilities written.
  if (!d_probs) return nvs::launch_nucleus(h->fv, a, rows, K, h->max_dyn_smem, h->num_sms, stream);
  return nvs::launch_fullvocab(h->fv, a, rows, K, h->max_dyn_smem, stream, false, 0);
}

// Lazily sized staging buffers owned by the handle, for the host-array entry
// points; caller holds h->mu and the device.
static bool ensure_staging(NcbSampler* h, size_t nh, bool probs) {
  if (!h->h_logits_dev) {
    const size_t nl = (size_t)h->max_rows * h->max_vocab;
    if (cudaMalloc(&h->h_logits_dev, nl * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->h_hoff_dev, ((size_t)h->max_rows + 1) * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&h->h_u_dev, (size_t)h->max_rows * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->h_tok_dev, (size_t)h->max_rows * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&h->h_flags_dev, (size_t)h->max_rows * sizeof(uint32_t)) != cudaSuccess ||
        cudaStreamCreateWithFlags(&h->host_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMallocHost(&h->h_out_pinned, (size_t)h->max_rows * 2 * sizeof(int32_t)) != cudaSuccess)
      return false;
    for (cudaEvent_t& e : h->slice_ev)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return false;
  }
  if (nh > h->h_hist_cap) {
    cudaFree(h->h_hist_dev);
    h->h_hist_dev = nullptr;
    const size_t cap = nh < 1024 ? 1024 : nh;
    if (cudaMalloc(&h->h_hist_dev, cap * sizeof(int32_t)) != cudaSuccess) return false;
    h->h_hist_cap = cap;
  }
  if (probs && !h->h_probs_dev &&
      cudaMalloc(&h->h_probs_dev, (size_t)h->max_rows * h->max_vocab * sizeof(float)) != cudaSuccess)
    return false;
  return true;
}

// CSR offsets of `rows` host histories: start at 0, non-decreasing.
static bool host_offsets_ok(const int32_t* hist, const int32_t* off, int rows) {
  if (!off || off[0] != 0) return false;
  for (int r = 0; r < rows; ++r)
    if (off[r + 1] < off[r]) return false;
  return off[rows] == 0 || hist != nullptr;
}

static int validate_sample_args(NcbSampler* h, const void* logits, int rows, int vocab,
                                const void* hist, const void* hoff, const void* u,
                                const NcbSamplerParams* prm, const void* tok) {
  if (!h) return NCB_ERROR_NOT_INITIALIZED;
  if (!prm || !params_ok(prm)) return NCB_ERROR_INVALID_ARGUMENT;
  if (rows < 0 || vocab <= 0) return NCB_ERROR_INVALID_ARGUMENT;
  if (rows == 0) return NCB_OK;  // an empty batch needs no buffers
  if (!logits || !hoff || !tok) return NCB_ERROR_INVALID_ARGUMENT;
  if (!prm->greedy && !u) return NCB_ERROR_INVALID_ARGUMENT;
  if (rows > h->max_rows || vocab > h->max_vocab) return NCB_ERROR_CAPACITY;
  if ((reinterpret_cast<uintptr_t>(logits) & 3u) != 0u) return NCB_ERROR_INVALID_ARGUMENT;
  (void)hist;
  return NCB_OK;
}

NCB_API int ncb_sample_rows_device(NcbSampler* h, const float* d_logits, int rows, int vocab,
                                   const int32_t* d_hist, const int32_t* d_hist_offsets,
                                   const float* d_uniforms, const NcbSamplerParams* params,
                                   int32_t* d_tokens, uint32_t* d_flags, float* d_probs,
                                   void* stream) {
  int st = validate_sample_args(h, d_logits, rows, vocab, d_hist, d_hist_offsets, d_uniforms,
                                params, d_tokens);
  if (st != NCB_OK) return set_status(st);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  st = launch_sample(h, d_logits, rows, vocab, d_hist, d_hist_offsets, d_uniforms, params,
                     d_tokens, d_flags, d_probs, static_cast<cudaStream_t>(stream));
  return set_status(st);
}

NCB_API int ncb_sample_rows(NcbSampler* h, const float* h_logits, int rows, int vocab,
                            const int32_t* h_hist, const int32_t* h_hist_offsets,
                            const float* h_uniforms, const NcbSamplerParams* params,
                            int32_t* h_tokens, uint32_t* h_flags, float* h_probs) {
  int st = validate_sample_args(h, h_logits, rows, vocab, h_hist, h_hist_offsets, h_uniforms,
                                params, h_tokens);
  if (st != NCB_OK) return set_status(st);
  if (rows == 0) return set_status(NCB_OK);
  const int64_t nh = h_hist_offsets[rows];
  if (h_hist_offsets[0] != 0 || nh < 0 || (nh > 0 && !h_hist)) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  for (int r = 0; r < rows; ++r)
    if (h_hist_offsets[r + 1] < h_hist_offsets[r]) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  if (!ensure_staging(h, (size_t)nh, h_probs != nullptr)) return set_status(NCB_ERROR_ALLOC_FAILED);
  // The logits go in slices on the copy stream; slice i's sampling (on the
  // sampling stream) waits for its own copy only, so sampling slice i overlaps
  // copying slice i + 1 and the call ends one slice's sampling after the last
  // copy. Rows are independent (TokenSampler.cs:10-30), so the slices' tokens
  // equal the whole batch's.
  cudaStream_t s = h->host_stream, cs = h->copy_stream;
  const size_t row_bytes = (size_t)vocab * sizeof(float);
  int slices = 1;
  if ((size_t)rows * row_bytes >= ((size_t)16 << 20) && rows >= 32)
    slices = rows / 16 < 8 ? rows / 16 : 8;
  bool ok = cudaMemcpyAsync(h->h_hoff_dev, h_hist_offsets, ((size_t)rows + 1) * sizeof(int32_t),
                            cudaMemcpyHostToDevice, cs) == cudaSuccess;
  if (nh > 0)
    ok = ok && cudaMemcpyAsync(h->h_hist_dev, h_hist, (size_t)nh * sizeof(int32_t),
                               cudaMemcpyHostToDevice, cs) == cudaSuccess;
  if (!params->greedy)
    ok = ok && cudaMemcpyAsync(h->h_u_dev, h_uniforms, (size_t)rows * sizeof(float),
                               cudaMemcpyHostToDevice, cs) == cudaSuccess;
  for (int i = 0; i < slices && ok; ++i) {
    const int r0 = (int)((int64_t)rows * i / slices), r1 = (int)((int64_t)rows * (i + 1) / slices);
    ok = cudaMemcpyAsync(h->h_logits_dev + (size_t)r0 * vocab, h_logits + (size_t)r0 * vocab,
                         (size_t)(r1 - r0) * row_bytes, cudaMemcpyHostToDevice, cs) == cudaSuccess &&
         cudaEventRecord(h->slice_ev[i], cs) == cudaSuccess;
  }
  if (!ok) {
    cudaStreamSynchronize(cs);
    return set_status(NCB_ERROR_COPY_FAILED);
  }
  for (int i = 0; i < slices; ++i) {
    const int r0 = (int)((int64_t)rows * i / slices), r1 = (int)((int64_t)rows * (i + 1) / slices);
    if (cudaStreamWaitEvent(s, h->slice_ev[i], 0) != cudaSuccess) st = NCB_ERROR_LAUNCH_FAILED;
    if (st == NCB_OK)
      st = launch_sample(h, h->h_logits_dev + (size_t)r0 * vocab, r1 - r0, vocab, h->h_hist_dev,
                         h->h_hoff_dev + r0, h->h_u_dev + r0, params, h->h_tok_dev + r0,
                         h->h_flags_dev + r0,
                         h_probs ? h->h_probs_dev + (size_t)r0 * vocab : nullptr, s);
    if (st != NCB_OK) {
      cudaStreamSynchronize(cs);
      cudaStreamSynchronize(s);
      return set_status(st);
    }
  }
  // tokens and flags through the handle's pinned buffer (a copy into the
  // caller's pageable memory would be staged by the driver), copied on the
  // host after the synchronisation
  int32_t* pt = h->h_out_pinned;
  uint32_t* pf = reinterpret_cast<uint32_t*>(h->h_out_pinned + h->max_rows);
  ok = cudaMemcpyAsync(pt, h->h_tok_dev, (size_t)rows * sizeof(int32_t), cudaMemcpyDeviceToHost,
                       s) == cudaSuccess;
  if (h_flags)
    ok = ok && cudaMemcpyAsync(pf, h->h_flags_dev, (size_t)rows * sizeof(uint32_t),
                               cudaMemcpyDeviceToHost, s) == cudaSuccess;
  if (h_probs)
    ok = ok && cudaMemcpyAsync(h_probs, h->h_probs_dev, (size_t)rows * vocab * sizeof(float),
                               cudaMemcpyDeviceToHost, s) == cudaSuccess;
  if (!ok) return set_status(NCB_ERROR_COPY_FAILED);
  if (cudaStreamSynchronize(s) != cudaSuccess) return set_status(NCB_ERROR_LAUNCH_FAILED);
  std::memcpy(h_tokens, pt, (size_t)rows * sizeof(int32_t));
  if (h_flags) std::memcpy(h_flags, pf, (size_t)rows * sizeof(uint32_t));
  return set_status(NCB_OK);
}

// ---- LogitsProcessor --------------------------------------------------------

static int check_rows(NcbSampler* h, const void* x, int rows, int vocab) {
  if (!h) return NCB_ERROR_NOT_INITIALIZED;
  if (!x || rows < 0 || vocab <= 0) return NCB_ERROR_INVALID_ARGUMENT;
  if (rows > h->max_rows || vocab > h->max_vocab) return NCB_ERROR_CAPACITY;
  return NCB_OK;
}

NCB_API int ncb_logits_repetition_penalty_device(NcbSampler* h, float* d_logits, int rows,
                                                 int vocab, const int32_t* d_hist,
                                                 const int32_t* d_hist_offsets, float penalty,
                                                 void* stream) {
  int st = check_rows(h, d_logits, rows, vocab);
  if (st != NCB_OK) return set_status(st);
  if (!d_hist_offsets || !(penalty > 0.0f)) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if (penalty == 1.0f || rows == 0) return set_status(NCB_OK);  // LogitsProcessor.cs:17-18
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  const size_t smem = (size_t)((vocab + 31) / 32) * 4;
  if ((int)smem > h->max_dyn_smem) return set_status(NCB_ERROR_CAPACITY);
  nvs::repetition_penalty_kernel<<<rows, nvs::LP_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
      d_logits, vocab, d_hist, d_hist_offsets, penalty);
  return set_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}

NCB_API int ncb_logits_frequency_presence_penalty_device(NcbSampler* h, float* d_logits,
                                                         int rows, int vocab,
                                                         const int32_t* d_hist,
                                                         const int32_t* d_hist_offsets,
                                                         float frequency, float presence,
                                                         void* stream) {
  int st = check_rows(h, d_logits, rows, vocab);
  if (st != NCB_OK) return set_status(st);
  if (!d_hist_offsets || frequency != frequency || presence != presence)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if ((frequency == 0.0f && presence == 0.0f) || rows == 0) return set_status(NCB_OK);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  const int h_cap = pow2_at_least(h->max_history > 0 ? h->max_history : 1);
  const size_t smem = (size_t)h_cap * 4;
  if ((int)smem > h->max_dyn_smem) return set_status(NCB_ERROR_CAPACITY);
  nvs::frequency_presence_kernel<<<rows, nvs::LP_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
      d_logits, vocab, d_hist, d_hist_offsets, frequency, presence, h_cap, nullptr);
  return set_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}

NCB_API int ncb_logits_temperature_device(NcbSampler* h, float* d_logits, int rows, int vocab,
                                          float temperature, void* stream) {
  int st = check_rows(h, d_logits, rows, vocab);
  if (st != NCB_OK) return set_status(st);
  if (!(temperature > 0.0f)) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if (temperature == 1.0f || rows == 0) return set_status(NCB_OK);  // LogitsProcessor.cs:44-45
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  const size_t n = (size_t)rows * vocab;
  const int grid = 4 * h->num_sms;
  if ((reinterpret_cast<uintptr_t>(d_logits) & 15u) == 0u)
    nvs::temperature_kernel<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(d_logits, n, temperature);
  else
    nvs::temperature_kernel_unaligned<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(d_logits, n,
                                                                                         temperature);
  return set_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}

NCB_API int ncb_logits_filter_top_k_device(NcbSampler* h, float* d_logits, int rows, int vocab,
                                           int top_k, void* stream) {
  int st = check_rows(h, d_logits, rows, vocab);
  if (st != NCB_OK) return set_status(st);
  if (top_k <= 0) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if (top_k >= vocab || rows == 0) return set_status(NCB_OK);  // LogitsProcessor.cs:62-63
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  nvs::filter_top_k_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(d_logits, vocab, top_k);
  return set_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}

NCB_API int ncb_logits_filter_top_p_device(NcbSampler* h, float* d_probs, int rows, int vocab,
                                           float top_p, uint32_t* d_flags, void* stream) {
  int st = check_rows(h, d_probs, rows, vocab);
  if (st != NCB_OK) return set_status(st);
  if (!(top_p > 0.0f) || top_p > 1.0f) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (top_p >= 1.0f || rows == 0) {  // LogitsProcessor.cs:84-85
    if (d_flags && rows > 0 && cudaMemsetAsync(d_flags, 0, (size_t)rows * 4, s) != cudaSuccess)
      return set_status(NCB_ERROR_LAUNCH_FAILED);
    return set_status(NCB_OK);
  }
  const size_t smem = (size_t)nvs::FV_GCAP * 16 + (size_t)(2 * nvs::FV_NB + 1) * 4;
  nvs::filter_top_p_kernel<<<rows, nvs::FV_THREADS, smem, s>>>(d_probs, vocab, top_p, d_flags, h->fv);
  return set_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}

}  // extern "C"

// ---- allocation-free sampling -----------------------------------------------
//
// Scratch for ncb_sample_rows_noalloc_device lives in one file-scope device
// array instead of a handle's cudaMalloc'd buffer. Host code cannot use its
// name as a device address: the address is looked up per device with
// cudaGetSymbolAddress and passed to the kernels.

namespace {

constexpr int NA_MAX_ROWS = 1024;
constexpr int NA_MAX_SEGMENTS = 512;   // rows x column segments per call
constexpr int NA_MAX_HISTORY = 4096;   // per-row ids counted for frequency/presence
constexpr int NA_MAX_DEVICES = 64;

constexpr size_t na_align(size_t x) { return (x + 255) / 256 * 256; }
constexpr size_t NA_OFF_CV = 0;
constexpr size_t NA_OFF_CI = NA_OFF_CV + na_align((size_t)NA_MAX_SEGMENTS * nvs::TK_CAPB * 4);
constexpr size_t NA_OFF_CN = NA_OFF_CI + na_align((size_t)NA_MAX_SEGMENTS * nvs::TK_CAPB * 4);
constexpr size_t NA_OFF_GV = NA_OFF_CN + na_align((size_t)NA_MAX_SEGMENTS * 4);
constexpr size_t NA_OFF_GI = NA_OFF_GV + na_align((size_t)NA_MAX_SEGMENTS * 4);
// everything from here on must be zero when a call starts
constexpr size_t NA_OFF_ZERO = NA_OFF_GI + na_align((size_t)NA_MAX_SEGMENTS * 4);
constexpr size_t NA_OFF_TK = NA_OFF_ZERO;
constexpr size_t NA_OFF_RS = NA_OFF_TK + na_align((size_t)NA_MAX_ROWS * 4);
constexpr size_t NA_OFF_FX = NA_OFF_RS + na_align((size_t)NA_MAX_ROWS * 4);
constexpr size_t NA_OFF_ER = NA_OFF_FX + na_align((size_t)NA_MAX_ROWS * 4);
constexpr size_t NA_BYTES = NA_OFF_ER + 256;  // 8 MiB + 16 KiB

struct NaDevice {
  char* base = nullptr;  // device address of g_noalloc_scratch on this device
  int num_sms = 0;
  int max_dyn_smem = 0;
};
NaDevice g_na_dev[NA_MAX_DEVICES];
std::mutex g_na_mu;

}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

namespace nvs {
// Rows the top-k kernel marked for the full-vocabulary fix-up: without that
// path's scratch they are reported as -1 / NCB_FLAG_TIES_OVERFLOW.
__global__ void noalloc_finalize_kernel(int rows, uint32_t* fixup, int32_t* tokens,
                                        uint32_t* flags) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    if (fixup[r] != 0u) {
      tokens[r] = -1;
      if (flags) flags[r] = NCB_FLAG_TIES_OVERFLOW;
      fixup[r] = 0u;
    }
  }
}
}  // namespace nvs

extern "C" NCB_API int ncb_sample_rows_noalloc_device(const float* d_logits, int rows, int vocab,
                                                      const int32_t* d_hist,
                                                      const int32_t* d_hist_offsets,
                                                      const float* d_uniforms,
                                                      const NcbSamplerParams* prm,
                                                      int32_t* d_tokens, uint32_t* d_flags,
                                                      float* d_probs, void* stream_) {
  if (!prm || !params_ok(prm) || rows < 0 || vocab <= 0)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if (rows == 0) return set_status(NCB_OK);
  if (!d_logits || !d_hist_offsets || !d_tokens || (!prm->greedy && !d_uniforms))
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if ((reinterpret_cast<uintptr_t>(d_logits) & 3u) != 0u)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  const int K = prm->top_k < vocab ? prm->top_k : vocab;
  if (rows > NA_MAX_ROWS || vocab > (1 << 24)) return set_status(NCB_ERROR_CAPACITY);
  if (!prm->greedy && !(K < vocab && K <= nvs::TL_KMAX)) return set_status(NCB_ERROR_CAPACITY);

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES)
    return set_status(NCB_ERROR_NO_DEVICE);
  NaDevice nd;
  {
    // first call on this device: look up the scratch array's device address
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_dev[dev].base) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr)
        return set_status(NCB_ERROR_INIT_FAILED);
      int sms = 0, optin = 0;
      if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
              cudaSuccess ||
          !raise_smem_limits(optin))
        return set_status(NCB_ERROR_INIT_FAILED);
      g_na_dev[dev].num_sms = sms;
      g_na_dev[dev].max_dyn_smem = optin - 4096;
      g_na_dev[dev].base = static_cast<char*>(ptr);
    }
    nd = g_na_dev[dev];
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);

  nvs::SampleArgs a{};
  a.logits = d_logits;
  a.V = vocab;
  a.hist = d_hist;
  a.hoff = d_hist_offsets;
  a.uniforms = d_uniforms;
  a.p = to_params(prm);
  a.tokens = d_tokens;
  a.flags = d_flags;
  a.probs = d_probs;
  a.s.cand_v = reinterpret_cast<float*>(nd.base + NA_OFF_CV);
  a.s.cand_id = reinterpret_cast<int32_t*>(nd.base + NA_OFF_CI);
  a.s.cand_n = reinterpret_cast<int32_t*>(nd.base + NA_OFF_CN);
  a.s.gv = reinterpret_cast<float*>(nd.base + NA_OFF_GV);
  a.s.gi = reinterpret_cast<int32_t*>(nd.base + NA_OFF_GI);
  a.s.tickets = reinterpret_cast<uint32_t*>(nd.base + NA_OFF_TK);
  a.s.rowstate = reinterpret_cast<uint32_t*>(nd.base + NA_OFF_RS);
  a.s.fixup = reinterpret_cast<uint32_t*>(nd.base + NA_OFF_FX);
  a.s.error_word = reinterpret_cast<uint32_t*>(nd.base + NA_OFF_ER);
  const bool counts = (prm->frequency_penalty != 0.0f || prm->presence_penalty != 0.0f);
  a.h_cap = counts ? NA_MAX_HISTORY : 0;

  // what a previous call may have left behind must start at zero
  if (cudaMemsetAsync(nd.base + NA_OFF_ZERO, 0, NA_BYTES - NA_OFF_ZERO, stream) != cudaSuccess)
    return set_status(NCB_ERROR_LAUNCH_FAILED);

  // top-k rows split like the handle path's (at most 8 segments, so a split
  // row's merge holds K x S <= 512 candidates, within its 2048-entry buffer)
  int S = prm->greedy ? choose_splits(rows, vocab, nd.num_sms, 0)
                      : choose_splits_topk(rows, vocab, nd.num_sms, 0);
  if (rows * S > NA_MAX_SEGMENTS) S = NA_MAX_SEGMENTS / rows > 0 ? NA_MAX_SEGMENTS / rows : 1;
  a.seg_len = round_up((vocab + S - 1) / S, 4);
  S = (vocab + a.seg_len - 1) / a.seg_len;
  a.bm_words = (a.seg_len + 31) / 32 + 1;
  dim3 grid(S, rows);
  if (prm->greedy) {
    const size_t smem = (size_t)a.bm_words * 4 + (size_t)a.h_cap * 4;
    if ((int)smem > nd.max_dyn_smem) return set_status(NCB_ERROR_CAPACITY);
    if (counts) nvs::greedy_kernel<true><<<grid, nvs::GR_THREADS, smem, stream>>>(a);
    else nvs::greedy_kernel<false><<<grid, nvs::GR_THREADS, smem, stream>>>(a);
  } else {
    const size_t smem = nvs::tl_smem_bytes(a.bm_words, a.h_cap);
    if ((int)smem > nd.max_dyn_smem) return set_status(NCB_ERROR_CAPACITY);
    if (counts) nvs::topk_ldg_kernel<true><<<grid, nvs::TL_THREADS, smem, stream>>>(a);
    else nvs::topk_ldg_kernel<false><<<grid, nvs::TL_THREADS, smem, stream>>>(a);
    if (cudaGetLastError() != cudaSuccess) return set_status(NCB_ERROR_LAUNCH_FAILED);
    nvs::noalloc_finalize_kernel<<<(rows + 255) / 256, 256, 0, stream>>>(rows, a.s.fixup,
                                                                        d_tokens, d_flags);
  }
  return set_status(cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED);
}

// ---- vocabulary shards ------------------------------------------------------

static int check_shard_args(NcbSampler* h, const float* d_logits, int rows, int vocab,
                            int col_begin, int col_end, int ld, const int32_t* d_hoff,
                            const NcbSamplerParams* prm) {
  if (!h) return NCB_ERROR_NOT_INITIALIZED;
  if (!prm || !params_ok(prm) || rows < 0 || vocab <= 0 || col_begin < 0 ||
      col_end <= col_begin || col_end > vocab || ld < col_end - col_begin)
    return NCB_ERROR_INVALID_ARGUMENT;
  if (rows == 0) return NCB_OK;
  if (!d_logits || !d_hoff || (reinterpret_cast<uintptr_t>(d_logits) & 3u) != 0u)
    return NCB_ERROR_INVALID_ARGUMENT;
  if (rows > h->max_rows || col_end - col_begin > h->max_vocab) return NCB_ERROR_CAPACITY;
  const int K = prm->top_k < vocab ? prm->top_k : vocab;
  if (!prm->greedy && K > nvs::TL_KMAX) return NCB_ERROR_CAPACITY;
  return NCB_OK;
}

// The shard kernel for one column range; caller holds h->mu and the device.
static int launch_shard_candidates(NcbSampler* h, const float* d_logits, int rows, int vocab,
                                   int col_begin, int col_end, int ld, const int32_t* d_hist,
                                   const int32_t* d_hoff, const NcbSamplerParams* prm,
                                   uint32_t* records, cudaStream_t stream,
                                   const nvs::PxArgs* px = nullptr) {
  const int width = col_end - col_begin;
  nvs::SampleArgs a{};
  if (px) a.px = *px;
  a.logits = d_logits;
  a.V = vocab;
  a.hist = d_hist;
  a.hoff = d_hoff;
  a.p = to_params(prm);
  a.s = h->s;
  a.ld = ld;
  a.col_lo = col_begin;
  a.col_hi = col_end;
  a.shard_out = records;
  const bool counts = (prm->frequency_penalty != 0.0f || prm->presence_penalty != 0.0f);
  a.h_cap = counts ? pow2_at_least(h->max_history > 0 ? h->max_history : 1) : 0;
  // Wide shards with k <= 64 and lowering penalties: the chunked stream and
  // finish kernels (the finish writes the records), then the shard kernel below
  // in fix-up mode for the rows the finish could not prove.
  const int K = prm->top_k < vocab ? prm->top_k : vocab;
  const bool lowering = prm->repetition_penalty >= 1.0f && prm->frequency_penalty >= 0.0f &&
                        prm->presence_penalty >= 0.0f;
  const int J = nvs::ck_chunks(width);
  const bool chunked = !prm->greedy && h->chunked && h->forced_splits == 0 && K < width &&
                       K <= nvs::TL_KMAX && lowering && width >= 8192 && J <= h->ck_jmax &&
                       683LL * K <= (long long)width;
  if (chunked) {
    a.bm_words = (width + 31) / 32 + 1;
    const size_t fsmem = nvs::fk_smem_bytes(a.bm_words, a.h_cap);
    const size_t ring = nvs::cr_smem_bytes();
    if ((int)fsmem > h->max_dyn_smem || (int)ring > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const int nchunks = rows * J;
    cudaLaunchConfig_t c1{};
    c1.gridDim = dim3(nchunks < h->num_sms ? nchunks : h->num_sms);
    c1.blockDim = dim3(nvs::CR_THREADS);
    c1.dynamicSmemBytes = ring;
    c1.stream = stream;
    c1.attrs = attr;
    c1.numAttrs = 1;
    if (cudaLaunchKernelEx(&c1, nvs::topk_chunk_kernel<true>, a, J, nchunks) != cudaSuccess)
      return NCB_ERROR_LAUNCH_FAILED;
    cudaLaunchConfig_t c2 = c1;
    c2.gridDim = dim3(rows);
    c2.blockDim = dim3(nvs::FK_THREADS);
    c2.dynamicSmemBytes = fsmem;
    const bool wide = J * nvs::CK_WARPS * nvs::CK_KEYS > 4 * nvs::FK_THREADS;
    cudaError_t e;
    if (counts)
      e = wide ? cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<true, 8, true>, a, J)
               : cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<true, 4, true>, a, J);
    else
      e = wide ? cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<false, 8, true>, a, J)
               : cudaLaunchKernelEx(&c2, nvs::topk_chunk_finish_kernel<false, 4, true>, a, J);
    if (e != cudaSuccess) return NCB_ERROR_LAUNCH_FAILED;
    a.fixup_only = 1;
  }
  int S = prm->greedy ? choose_splits(rows, width, h->num_sms, h->forced_splits)
                      : choose_splits_topk(rows, width, h->num_sms, h->forced_splits);
  a.seg_len = round_up((width + S - 1) / S, 4);
  S = (width + a.seg_len - 1) / a.seg_len;
  if ((size_t)rows * S > (size_t)h->max_ctas) return NCB_ERROR_CAPACITY;
  a.bm_words = (a.seg_len + 31) / 32 + 1;
  dim3 grid(S, rows);
  if (prm->greedy) {
    const size_t smem = (size_t)a.bm_words * 4 + (size_t)a.h_cap * 4;
    if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    if (counts) nvs::greedy_kernel<true, true><<<grid, nvs::GR_THREADS, smem, stream>>>(a);
    else nvs::greedy_kernel<false, true><<<grid, nvs::GR_THREADS, smem, stream>>>(a);
  } else {
    const size_t smem = nvs::tl_smem_bytes(a.bm_words, a.h_cap);
    if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
    cudaLaunchConfig_t c{};
    c.gridDim = grid;
    c.blockDim = dim3(nvs::TL_THREADS);
    c.dynamicSmemBytes = smem;
    c.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = attr;
    c.numAttrs = a.fixup_only ? 1 : 0;  // the fix-up follows the finish kernel closely
    const cudaError_t e = counts ? cudaLaunchKernelEx(&c, nvs::topk_ldg_kernel<true, true>, a)
                                 : cudaLaunchKernelEx(&c, nvs::topk_ldg_kernel<false, true>, a);
    if (e != cudaSuccess) return NCB_ERROR_LAUNCH_FAILED;
  }
  return cudaGetLastError() == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED;
}

// The merge kernel; with `tagged` (peer-memory exchange) it first waits for
// this call's tagged record words and unpacks them into `unpack`.
static int launch_merge(NcbSampler* h, const uint32_t* recs, int shards, int rows, int vocab,
                        const float* d_u, const NcbSamplerParams* prm, int32_t* d_tok,
                        uint32_t* d_flags, const uint64_t* tagged, uint32_t* unpack,
                        cudaStream_t stream) {
  nvs::MergeArgs m{};
  m.recs = tagged ? unpack : recs;
  m.shards = shards;
  m.rows = rows;
  m.a.V = vocab;
  m.a.uniforms = d_u;
  m.a.p = to_params(prm);
  m.a.tokens = d_tok;
  m.a.flags = d_flags;
  m.a.s = h->s;
  if (tagged) {
    m.tagged = tagged;
    m.unpack = unpack;
    m.max_rows = h->max_rows;
    m.epoch = h->s.px_ticket + 3;
    m.ticket = h->s.px_ticket + 2;
  }
  const size_t smem = nvs::vm_smem_bytes();
  if ((int)smem > h->max_dyn_smem) return NCB_ERROR_CAPACITY;
  // with tagged words the merge may start polling while the shard kernels
  // drain (a programmatic dependent launch); gathered records need stream order
  cudaLaunchConfig_t c{};
  c.gridDim = dim3(rows);
  c.blockDim = dim3(nvs::VM_THREADS);
  c.dynamicSmemBytes = smem;
  c.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = tagged ? 1 : 0;
  return cudaLaunchKernelEx(&c, nvs::vocab_merge_kernel, m) == cudaSuccess ? NCB_OK
                                                                           : NCB_ERROR_LAUNCH_FAILED;
}

//
// A batch whose vocabulary is split in contiguous column ranges over several
// GPUs: each GPU reduces its range of every row to a fixed-size record
// (ncb_vocab_shard_candidates_device), the caller all-gathers the records of
// all shards in column order, and every GPU merges them
// (ncb_vocab_shard_merge_device) into the same tokens the single-GPU entry
// point gives for the whole rows.

extern "C" {

NCB_API int ncb_vocab_shard_record_bytes(void) { return nvs::VS_REC_WORDS * 4; }

NCB_API int ncb_vocab_shard_candidates_device(NcbSampler* h, const float* d_logits, int rows,
                                              int vocab, int col_begin, int col_end, int ld,
                                              const int32_t* d_hist,
                                              const int32_t* d_hist_offsets,
                                              const NcbSamplerParams* prm, void* d_records,
                                              void* stream_) {
  int st = check_shard_args(h, d_logits, rows, vocab, col_begin, col_end, ld, d_hist_offsets, prm);
  if (st != NCB_OK || rows == 0) return set_status(st);
  if (!d_records || (reinterpret_cast<uintptr_t>(d_records) & 3u) != 0u)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  return set_status(launch_shard_candidates(h, d_logits, rows, vocab, col_begin, col_end, ld, d_hist,
                                            d_hist_offsets, prm, static_cast<uint32_t*>(d_records),
                                            static_cast<cudaStream_t>(stream_)));
}

NCB_API int ncb_vocab_shard_merge_device(NcbSampler* h, const void* d_records, int shards,
                                         int rows, int vocab, const float* d_uniforms,
                                         const NcbSamplerParams* prm, int32_t* d_tokens,
                                         uint32_t* d_flags, void* stream_) {
  if (!h) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (!prm || !params_ok(prm) || rows < 0 || vocab <= 0 || shards <= 0)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if (rows == 0) return set_status(NCB_OK);
  if (!d_records || !d_tokens || (!prm->greedy && !d_uniforms) ||
      (reinterpret_cast<uintptr_t>(d_records) & 3u) != 0u)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  const int K = prm->top_k < vocab ? prm->top_k : vocab;
  if (shards > nvs::VM_MAX_SHARDS || (!prm->greedy && K > nvs::TL_KMAX))
    return set_status(NCB_ERROR_CAPACITY);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  return set_status(launch_merge(h, static_cast<const uint32_t*>(d_records), shards, rows, vocab,
                                 d_uniforms, prm, d_tokens, d_flags, nullptr, nullptr,
                                 static_cast<cudaStream_t>(stream_)));
}

}  // extern "C"

// ---- vocabulary shards through peer memory ------------------------------------
//
// The exchange of ncb_vocab_shard_* done by the library itself: the shard
// kernels store every finished record straight into every GPU's exchange area
// over NVLink (CUDA IPC mappings), each word tagged with the call's epoch; the
// merge waits for its row's words. No collective, no extra kernel.

extern "C" {

}  // extern "C"

// What each GPU publishes for a peer-memory exchange: its area's CUDA IPC
// handle and what the area was laid out for. Every GPU's area must have the
// same layout (a peer writes at offsets computed from its own), so connect
// refuses blobs that disagree instead of corrupting a peer's memory.
struct PeerBlob {
  cudaIpcMemHandle_t ipc;
  uint32_t magic;  // kPeerMagic
  uint32_t kind;   // kPeerVocab or kPeerRows
  uint32_t size;   // vocabulary shards: rows per call; row gather: rows of the whole batch
  uint32_t ranks;
};
constexpr uint32_t kPeerMagic = 0x5850564Eu;  // "NVPX"
constexpr uint32_t kPeerVocab = 1u, kPeerRows = 2u;

static void write_blob(void* out, const cudaIpcMemHandle_t& hd, uint32_t kind, int size, int ranks) {
  PeerBlob b{};
  b.ipc = hd;
  b.magic = kPeerMagic;
  b.kind = kind;
  b.size = (uint32_t)size;
  b.ranks = (uint32_t)ranks;
  std::memcpy(out, &b, sizeof(b));
}

// Blob s of `handles` if it agrees with (kind, size, ranks), else false.
static bool read_blob(const void* handles, int s, uint32_t kind, int size, int ranks, PeerBlob* b) {
  std::memcpy(b, static_cast<const char*>(handles) + (size_t)s * sizeof(PeerBlob), sizeof(*b));
  return b->magic == kPeerMagic && b->kind == kind && b->size == (uint32_t)size &&
         b->ranks == (uint32_t)ranks;
}

extern "C" {

NCB_API int ncb_peer_handle_bytes(void) { return (int)sizeof(PeerBlob); }

NCB_API int ncb_vocab_shard_peer_setup(NcbSampler* h, int shards, int me, void* handle_out) {
  if (!h) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (shards < 1 || shards > nvs::PX_MAX || me < 0 || me >= shards || !handle_out || h->px_area)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  const nvs::PeerLayout l = nvs::peer_layout(shards, h->max_rows);
  void* area = nullptr;
  if (cudaMalloc(&area, l.bytes) != cudaSuccess) return set_status(NCB_ERROR_ALLOC_FAILED);
  cudaIpcMemHandle_t hd;
  if (cudaMemset(area, 0, l.bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&hd, area) != cudaSuccess) {
    cudaFree(area);
    return set_status(NCB_ERROR_INIT_FAILED);
  }
  write_blob(handle_out, hd, kPeerVocab, h->max_rows, shards);
  {
    std::lock_guard<std::mutex> lk2(g_px_mu);
    std::array<char, sizeof(cudaIpcMemHandle_t)> key;
    std::memcpy(key.data(), &hd, sizeof(hd));
    g_px_local.emplace_back(key, static_cast<char*>(area));
  }
  h->px_area = static_cast<char*>(area);
  h->px_shards = shards;
  h->px_me = me;
  h->px_layout = l;
  h->px_base[me] = h->px_area;
  return set_status(NCB_OK);
}

NCB_API int ncb_vocab_shard_peer_connect(NcbSampler* h, const void* handles) {
  if (!h) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (!h->px_area || h->px_connected || !handles) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  for (int s = 0; s < h->px_shards; ++s) {
    PeerBlob b;
    if (!read_blob(handles, s, kPeerVocab, h->max_rows, h->px_shards, &b))
      return set_status(NCB_ERROR_INVALID_ARGUMENT);
  }
  for (int s = 0; s < h->px_shards; ++s) {
    if (s == h->px_me) continue;
    PeerBlob b;
    read_blob(handles, s, kPeerVocab, h->max_rows, h->px_shards, &b);
    std::array<char, sizeof(cudaIpcMemHandle_t)> key;
    std::memcpy(key.data(), &b.ipc, key.size());
    char* local = nullptr;
    {
      std::lock_guard<std::mutex> lk2(g_px_mu);
      for (const auto& e : g_px_local)
        if (e.first == key) local = e.second;
    }
    if (local) {
      h->px_base[s] = local;
      continue;
    }
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, key.data(), sizeof(hd));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return set_status(NCB_ERROR_INIT_FAILED);
    h->px_base[s] = static_cast<char*>(p);
    h->px_imported[s] = true;
  }
  h->px_connected = true;
  return set_status(NCB_OK);
}

NCB_API int ncb_vocab_shard_push_peer_device(NcbSampler* h, const float* d_logits, int rows,
                                             int vocab, int col_begin, int col_end, int ld,
                                             const int32_t* d_hist,
                                             const int32_t* d_hist_offsets,
                                             const NcbSamplerParams* prm, void* stream_) {
  int st = check_shard_args(h, d_logits, rows, vocab, col_begin, col_end, ld, d_hist_offsets, prm);
  if (st != NCB_OK || rows == 0) return set_status(st);
  if (!h->px_connected) return set_status(NCB_ERROR_NOT_INITIALIZED);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  h->px_pushed = true;
  uint32_t* own = reinterpret_cast<uint32_t*>(h->px_area + h->px_layout.own_off);
  nvs::PxArgs px{};
  for (int s = 0; s < h->px_shards; ++s) px.tagged[s] = reinterpret_cast<uint64_t*>(h->px_base[s]);
  px.epoch = h->s.px_ticket + 3;
  px.shards = h->px_shards;
  px.me = h->px_me;
  px.max_rows = h->max_rows;
  // the shard kernel stores each finished record into every peer's area itself
  st = launch_shard_candidates(h, d_logits, rows, vocab, col_begin, col_end, ld, d_hist,
                               d_hist_offsets, prm, own, stream, &px);
  return set_status(st);
}

NCB_API int ncb_vocab_shard_merge_peer_device(NcbSampler* h, int rows, int vocab,
                                              const float* d_uniforms,
                                              const NcbSamplerParams* prm, int32_t* d_tokens,
                                              uint32_t* d_flags, void* stream_) {
  if (!h) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (!prm || !params_ok(prm) || rows < 0 || vocab <= 0) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  if (!h->px_connected || !h->px_pushed) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (rows == 0) return set_status(NCB_OK);
  if (rows > h->max_rows || !d_tokens || (!prm->greedy && !d_uniforms))
    return set_status(rows > h->max_rows ? NCB_ERROR_CAPACITY : NCB_ERROR_INVALID_ARGUMENT);
  const int K = prm->top_k < vocab ? prm->top_k : vocab;
  if (!prm->greedy && K > nvs::TL_KMAX) return set_status(NCB_ERROR_CAPACITY);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  return set_status(launch_merge(
      h, nullptr, h->px_shards, rows, vocab, d_uniforms, prm, d_tokens, d_flags,
      reinterpret_cast<const uint64_t*>(h->px_area),
      reinterpret_cast<uint32_t*>(h->px_area + h->px_layout.plain_off),
      static_cast<cudaStream_t>(stream_)));
}

}  // extern "C"

// ---- LogitsProcessor on host arrays ---------------------------------------------
//
// LogitsProcessor.* (LogitsProcessor.cs:8-114) operate in place on a float[]:
// these copy the rows in through the handle's staging buffers, run the device
// entry point, and copy them back.

namespace {
template <typename F>
int host_logits_call(NcbSampler* h, float* h_x, int rows, int vocab, const int32_t* h_hist,
                     const int32_t* h_off, bool need_hist, uint32_t* h_flags, F&& device_call) {
  if (!h) return NCB_ERROR_NOT_INITIALIZED;
  if (!h_x || rows < 0 || vocab <= 0) return NCB_ERROR_INVALID_ARGUMENT;
  if (rows > h->max_rows || vocab > h->max_vocab) return NCB_ERROR_CAPACITY;
  if (rows == 0) return NCB_OK;
  if (need_hist && !host_offsets_ok(h_hist, h_off, rows)) return NCB_ERROR_INVALID_ARGUMENT;
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return NCB_ERROR_INIT_FAILED;
  const size_t nh = need_hist ? (size_t)h_off[rows] : 0;
  if (!ensure_staging(h, nh, false)) return NCB_ERROR_ALLOC_FAILED;
  cudaStream_t s = h->host_stream;
  const size_t bytes = (size_t)rows * vocab * sizeof(float);
  bool ok = cudaMemcpyAsync(h->h_logits_dev, h_x, bytes, cudaMemcpyHostToDevice, s) == cudaSuccess;
  if (need_hist) {
    ok = ok && cudaMemcpyAsync(h->h_hoff_dev, h_off, ((size_t)rows + 1) * sizeof(int32_t),
                               cudaMemcpyHostToDevice, s) == cudaSuccess;
    if (nh > 0)
      ok = ok && cudaMemcpyAsync(h->h_hist_dev, h_hist, nh * sizeof(int32_t),
                                 cudaMemcpyHostToDevice, s) == cudaSuccess;
  }
  if (!ok) return NCB_ERROR_COPY_FAILED;
  const int st = device_call(h->h_logits_dev, s);
  if (st != NCB_OK) return st;
  ok = cudaMemcpyAsync(h_x, h->h_logits_dev, bytes, cudaMemcpyDeviceToHost, s) == cudaSuccess;
  if (h_flags)
    ok = ok && cudaMemcpyAsync(h_flags, h->h_flags_dev, (size_t)rows * sizeof(uint32_t),
                               cudaMemcpyDeviceToHost, s) == cudaSuccess;
  if (!ok) return NCB_ERROR_COPY_FAILED;
  return cudaStreamSynchronize(s) == cudaSuccess ? NCB_OK : NCB_ERROR_LAUNCH_FAILED;
}
}  // namespace

extern "C" {

NCB_API int ncb_logits_repetition_penalty(NcbSampler* h, float* h_logits, int rows, int vocab,
                                          const int32_t* h_hist, const int32_t* h_hist_offsets,
                                          float penalty) {
  return set_status(host_logits_call(h, h_logits, rows, vocab, h_hist, h_hist_offsets, true,
                                     nullptr, [&](float* d, cudaStream_t s) {
    return ncb_logits_repetition_penalty_device(h, d, rows, vocab, h->h_hist_dev, h->h_hoff_dev,
                                                penalty, s);
  }));
}

NCB_API int ncb_logits_frequency_presence_penalty(NcbSampler* h, float* h_logits, int rows,
                                                  int vocab, const int32_t* h_hist,
                                                  const int32_t* h_hist_offsets, float frequency,
                                                  float presence) {
  return set_status(host_logits_call(h, h_logits, rows, vocab, h_hist, h_hist_offsets, true,
                                     nullptr, [&](float* d, cudaStream_t s) {
    return ncb_logits_frequency_presence_penalty_device(h, d, rows, vocab, h->h_hist_dev,
                                                        h->h_hoff_dev, frequency, presence, s);
  }));
}

NCB_API int ncb_logits_temperature(NcbSampler* h, float* h_logits, int rows, int vocab,
                                   float temperature) {
  if (!(temperature > 0.0f)) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  return set_status(host_logits_call(h, h_logits, rows, vocab, nullptr, nullptr, false, nullptr,
                                     [&](float* d, cudaStream_t s) {
    return ncb_logits_temperature_device(h, d, rows, vocab, temperature, s);
  }));
}

NCB_API int ncb_logits_filter_top_k(NcbSampler* h, float* h_logits, int rows, int vocab,
                                    int top_k) {
  if (top_k <= 0) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  return set_status(host_logits_call(h, h_logits, rows, vocab, nullptr, nullptr, false, nullptr,
                                     [&](float* d, cudaStream_t s) {
    return ncb_logits_filter_top_k_device(h, d, rows, vocab, top_k, s);
  }));
}

NCB_API int ncb_logits_filter_top_p(NcbSampler* h, float* h_probs, int rows, int vocab,
                                    float top_p, uint32_t* h_flags) {
  if (!(top_p > 0.0f) || top_p > 1.0f) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  return set_status(host_logits_call(h, h_probs, rows, vocab, nullptr, nullptr, false, h_flags,
                                     [&](float* d, cudaStream_t s) {
    return ncb_logits_filter_top_p_device(h, d, rows, vocab, top_p, h->h_flags_dev, s);
  }));
}


// ---- rows split over GPUs, gathered through peer memory --------------------

NCB_API int ncb_row_gather_setup(NcbSampler* h, int ranks, int me, int rows_total,
                                 void* handle_out) {
  if (!h) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (ranks < 1 || ranks > nvs::PX_MAX || me < 0 || me >= ranks || rows_total <= 0 ||
      !handle_out || h->rg_area)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  const nvs::RgLayout l = nvs::rg_layout(rows_total);
  void* area = nullptr;
  if (cudaMalloc(&area, l.bytes) != cudaSuccess) return set_status(NCB_ERROR_ALLOC_FAILED);
  cudaIpcMemHandle_t hd;
  if (cudaMemset(area, 0, l.bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&hd, area) != cudaSuccess) {
    cudaFree(area);
    return set_status(NCB_ERROR_INIT_FAILED);
  }
  write_blob(handle_out, hd, kPeerRows, rows_total, ranks);
  {
    std::lock_guard<std::mutex> lk2(g_px_mu);
    std::array<char, sizeof(cudaIpcMemHandle_t)> key;
    std::memcpy(key.data(), &hd, sizeof(hd));
    g_px_local.emplace_back(key, static_cast<char*>(area));
  }
  h->rg_area = static_cast<char*>(area);
  h->rg_ranks = ranks;
  h->rg_me = me;
  h->rg_rows_total = rows_total;
  h->rg_layout = l;
  h->rg_base[me] = h->rg_area;
  return set_status(NCB_OK);
}

NCB_API int ncb_row_gather_connect(NcbSampler* h, const void* handles) {
  if (!h) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (!h->rg_area || h->rg_connected || !handles) return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  for (int s = 0; s < h->rg_ranks; ++s) {
    PeerBlob b;
    if (!read_blob(handles, s, kPeerRows, h->rg_rows_total, h->rg_ranks, &b))
      return set_status(NCB_ERROR_INVALID_ARGUMENT);
  }
  for (int s = 0; s < h->rg_ranks; ++s) {
    if (s == h->rg_me) continue;
    PeerBlob b;
    read_blob(handles, s, kPeerRows, h->rg_rows_total, h->rg_ranks, &b);
    std::array<char, sizeof(cudaIpcMemHandle_t)> key;
    std::memcpy(key.data(), &b.ipc, key.size());
    char* local = nullptr;
    {
      std::lock_guard<std::mutex> lk2(g_px_mu);
      for (const auto& e : g_px_local)
        if (e.first == key) local = e.second;
    }
    if (local) {
      h->rg_base[s] = local;
      continue;
    }
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, key.data(), sizeof(hd));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return set_status(NCB_ERROR_INIT_FAILED);
    h->rg_base[s] = static_cast<char*>(p);
    h->rg_imported[s] = true;
  }
  h->rg_connected = true;
  return set_status(NCB_OK);
}

NCB_API int ncb_sample_rows_gather_device(NcbSampler* h, const float* d_logits, int rows,
                                          int vocab, int row_begin, const int32_t* d_hist,
                                          const int32_t* d_hist_offsets,
                                          const float* d_uniforms,
                                          const NcbSamplerParams* params,
                                          int32_t* d_tokens_all, uint32_t* d_flags_all,
                                          void* stream_) {
  int st = validate_sample_args(h, d_logits, rows, vocab, d_hist, d_hist_offsets, d_uniforms,
                                params, d_tokens_all);
  if (st != NCB_OK) return set_status(st);
  if (!h->rg_connected) return set_status(NCB_ERROR_NOT_INITIALIZED);
  if (!d_tokens_all || row_begin < 0 || row_begin + rows > h->rg_rows_total)
    return set_status(NCB_ERROR_INVALID_ARGUMENT);
  std::lock_guard<std::recursive_mutex> lk(h->mu);
  DeviceGuard g(h->device);
  if (!g.ok) return set_status(NCB_ERROR_INIT_FAILED);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int32_t* st_tok = reinterpret_cast<int32_t*>(h->rg_area + h->rg_layout.staging_off);
  uint32_t* st_flg = reinterpret_cast<uint32_t*>(st_tok + h->rg_rows_total);
  if (rows > 0) {
    st = launch_sample(h, d_logits, rows, vocab, d_hist, d_hist_offsets, d_uniforms, params, st_tok,
                       st_flg, nullptr, stream);
    if (st != NCB_OK) return set_status(st);
  }
  nvs::RgArgs ga{};
  for (int s = 0; s < h->rg_ranks; ++s) ga.area[s] = h->rg_base[s];
  ga.l = h->rg_layout;
  ga.ranks = h->rg_ranks;
  ga.me = h->rg_me;
  ga.rows_total = h->rg_rows_total;
  ga.row_begin = row_begin;
  ga.rows = rows;
  ga.out_tok = d_tokens_all;
  ga.out_flg = d_flags_all;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(nvs::RG_THREADS);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, nvs::row_gather_kernel, ga) != cudaSuccess)
    return set_status(NCB_ERROR_LAUNCH_FAILED);
  return set_status(NCB_OK);
}

}  // extern "C"
