// C++ mirror of the reference's generation interface for the sampling path
// (Neuraval.Core.Generation: GenerationOptions, TokenSampler, LogitsProcessor;
// Neuraval/Generation/*.cs) over libnavsampler's C ABI (navsampler.h). Same
// names, argument meaning and argument checks, in the same order, with the
// exception types of the C# code:
//   ArgumentException           -> neuraval::ArgumentException
//   ArgumentNullException       -> neuraval::ArgumentNullException
//   ArgumentOutOfRangeException -> neuraval::ArgumentOutOfRangeException
//   CudaException               -> neuraval::CudaException (a non-OK status)
// C# references become pointers where the reference checks them for null
// (the pointer overloads), with reference overloads for ordinary use.
// The C# classes are static; here a Device owns the sampler handle (device
// scratch), and TokenSampler / LogitsProcessor borrow it.
#pragma once

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <optional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "navsampler.h"

namespace neuraval {

struct ArgumentException : std::invalid_argument {
  explicit ArgumentException(const std::string& param) : std::invalid_argument(param) {}
};
struct ArgumentNullException : std::invalid_argument {
  explicit ArgumentNullException(const std::string& param) : std::invalid_argument(param) {}
};
struct ArgumentOutOfRangeException : std::out_of_range {
  explicit ArgumentOutOfRangeException(const std::string& param) : std::out_of_range(param) {}
};
struct CudaException : std::runtime_error {
  int status;
  CudaException(int st, const std::string& where)
      : std::runtime_error(where + ": " + ncb_sampler_status_message(st)), status(st) {}
};

inline void check(int st, const char* where) {
  if (st != NCB_OK) throw CudaException(st, where);
}

// GenerationOptions (GenerationOptions.cs:5-98) plus the new frequency and
// presence penalties (0 = off).
class GenerationOptions {
 public:
  bool Greedy() const { return greedy_; }
  float Temperature() const { return temperature_; }
  float TopP() const { return top_p_; }
  int TopK() const { return top_k_; }
  float RepetitionPenalty() const { return repetition_penalty_; }
  int MaxNewTokens() const { return max_new_tokens_; }
  const std::vector<int>& StopTokenIds() const { return stop_token_ids_; }
  std::optional<int> Seed() const { return seed_; }
  float FrequencyPenalty() const { return frequency_penalty_; }
  float PresencePenalty() const { return presence_penalty_; }

  // GenerationOptions.Create (:44-75): the same checks in the same order.
  static GenerationOptions Create(bool greedy, float temperature, float topP, int topK,
                                  float repetitionPenalty, int maxNewTokens,
                                  const std::vector<int>* stopTokenIds,
                                  std::optional<int> seed = std::nullopt) {
    if (temperature <= 0.0f) throw ArgumentOutOfRangeException("temperature");
    if (topP <= 0.0f || topP > 1.0f) throw ArgumentOutOfRangeException("topP");
    if (topK <= 0) throw ArgumentOutOfRangeException("topK");
    if (repetitionPenalty <= 0.0f) throw ArgumentOutOfRangeException("repetitionPenalty");
    if (maxNewTokens <= 0) throw ArgumentOutOfRangeException("maxNewTokens");
    if (!stopTokenIds) throw ArgumentNullException("stopTokenIds");
    GenerationOptions o;
    o.greedy_ = greedy;
    o.temperature_ = temperature;
    o.top_p_ = topP;
    o.top_k_ = topK;
    o.repetition_penalty_ = repetitionPenalty;
    o.max_new_tokens_ = maxNewTokens;
    o.stop_token_ids_ = *stopTokenIds;
    o.seed_ = seed;
    return o;
  }
  static GenerationOptions Create(bool greedy, float temperature, float topP, int topK,
                                  float repetitionPenalty, int maxNewTokens,
                                  const std::vector<int>& stopTokenIds,
                                  std::optional<int> seed = std::nullopt) {
    return Create(greedy, temperature, topP, topK, repetitionPenalty, maxNewTokens,
                  &stopTokenIds, seed);
  }
  // GenerationOptions.CreateGreedy (:77-80) and Default (:82-85).
  static GenerationOptions CreateGreedy(int maxNewTokens, const std::vector<int>& stopTokenIds,
                                        std::optional<int> seed = std::nullopt) {
    return Create(true, 1.0f, 1.0f, INT_MAX, 1.0f, maxNewTokens, stopTokenIds, seed);
  }
  static GenerationOptions Default(const std::vector<int>& stopTokenIds,
                                   std::optional<int> seed = std::nullopt) {
    return Create(false, 0.7f, 0.9f, 40, 1.1f, 256, stopTokenIds, seed);
  }
  // New: a copy with frequency and presence penalties (applied after the
  // repetition penalty, before the temperature).
  GenerationOptions WithPenalties(float frequency, float presence) const {
    GenerationOptions o = *this;
    o.frequency_penalty_ = frequency;
    o.presence_penalty_ = presence;
    return o;
  }

  NcbSamplerParams ToParams() const {
    NcbSamplerParams p{};
    p.greedy = greedy_ ? 1 : 0;
    p.temperature = temperature_;
    p.top_p = top_p_;
    p.top_k = top_k_;
    p.repetition_penalty = repetition_penalty_;
    p.frequency_penalty = frequency_penalty_;
    p.presence_penalty = presence_penalty_;
    return p;
  }

 private:
  GenerationOptions() = default;
  bool greedy_ = false;
  float temperature_ = 1.0f, top_p_ = 1.0f;
  int top_k_ = INT_MAX;
  float repetition_penalty_ = 1.0f;
  int max_new_tokens_ = 1;
  std::vector<int> stop_token_ids_;
  std::optional<int> seed_;
  float frequency_penalty_ = 0.0f, presence_penalty_ = 0.0f;
};

// The uniform source of the draw: TokenSampler.cs:125 uses
// (float)random.NextDouble(). Any generator with NextDouble() in [0, 1) fits.
struct Random {
  virtual ~Random() = default;
  virtual double NextDouble() = 0;
};
class DefaultRandom final : public Random {
 public:
  explicit DefaultRandom(uint64_t seed = 0) : gen_(seed) {}
  double NextDouble() override { return std::uniform_real_distribution<double>(0.0, 1.0)(gen_); }

 private:
  std::mt19937_64 gen_;
};

// One GPU's sampler handle (ncb_sampler_create): scratch for up to maxRows rows
// of up to maxVocab columns and maxHistory generated ids per row.
class Device {
 public:
  explicit Device(int device = 0, int maxRows = 1, int maxVocab = 262144, int maxHistory = 4096) {
    check(ncb_sampler_create(device, maxRows, maxVocab, maxHistory, &h_), "ncb_sampler_create");
  }
  ~Device() {
    if (h_) ncb_sampler_destroy(h_);
  }
  Device(const Device&) = delete;
  Device& operator=(const Device&) = delete;
  NcbSampler* handle() const { return h_; }

 private:
  NcbSampler* h_ = nullptr;
};

// TokenSampler (TokenSampler.cs:10-143) on the GPU.
class TokenSampler {
 public:
  explicit TokenSampler(Device& device) : d_(device) {}

  // TokenSampler.SampleNext (:10-30): argument checks in the reference's order,
  // then one row through ncb_sample_rows. A non-finite row (NaN/+inf, no finite
  // maximum) or a history beyond the handle's capacity throws CudaException.
  int SampleNext(const std::vector<float>* logits, const GenerationOptions* options,
                 const std::vector<int>* generatedTokenIds, Random* random) const {
    if (!logits) throw ArgumentNullException("logits");
    if (!options) throw ArgumentNullException("options");
    if (!generatedTokenIds) throw ArgumentNullException("generatedTokenIds");
    if (!random) throw ArgumentNullException("random");
    const NcbSamplerParams p = options->ToParams();
    // the reference draws only on the filtered path (:125)
    const float u = options->Greedy() ? 0.0f : static_cast<float>(random->NextDouble());
    const int32_t offsets[2] = {0, static_cast<int32_t>(generatedTokenIds->size())};
    int32_t token = -1;
    uint32_t flags = 0;
    check(ncb_sample_rows(d_.handle(), logits->data(), 1, static_cast<int>(logits->size()),
                          generatedTokenIds->empty() ? nullptr : generatedTokenIds->data(),
                          offsets, &u, &p, &token, &flags, nullptr),
          "ncb_sample_rows");
    if (token < 0) throw CudaException(NCB_ERROR_INVALID_ARGUMENT, "SampleNext: row not sampled");
    return token;
  }
  int SampleNext(const std::vector<float>& logits, const GenerationOptions& options,
                 const std::vector<int>& generatedTokenIds, Random& random) const {
    return SampleNext(&logits, &options, &generatedTokenIds, &random);
  }

  // Batched form: rows x vocab logits (row-major), one history per row. Each
  // row consumes one NextDouble() unless greedy, in row order.
  std::vector<int> SampleNextBatch(const std::vector<float>& logits, int rows,
                                   const GenerationOptions& options,
                                   const std::vector<std::vector<int>>& generatedTokenIds,
                                   Random& random, std::vector<uint32_t>* flagsOut = nullptr) const {
    if (rows < 0 || (rows > 0 && logits.size() % rows != 0) ||
        generatedTokenIds.size() != static_cast<size_t>(rows))
      throw ArgumentOutOfRangeException("rows");
    std::vector<int32_t> offsets(rows + 1, 0), hist;
    for (int r = 0; r < rows; ++r) {
      hist.insert(hist.end(), generatedTokenIds[r].begin(), generatedTokenIds[r].end());
      offsets[r + 1] = static_cast<int32_t>(hist.size());
    }
    std::vector<float> u(rows, 0.0f);
    if (!options.Greedy())
      for (float& x : u) x = static_cast<float>(random.NextDouble());
    std::vector<int32_t> tokens(rows, -1);
    std::vector<uint32_t> flags(rows, 0);
    const NcbSamplerParams p = options.ToParams();
    const int vocab = rows > 0 ? static_cast<int>(logits.size() / rows) : 1;
    check(ncb_sample_rows(d_.handle(), logits.data(), rows, vocab, hist.empty() ? nullptr : hist.data(),
                          offsets.data(), u.data(), &p, tokens.data(), flags.data(), nullptr),
          "ncb_sample_rows");
    if (flagsOut) *flagsOut = flags;
    return std::vector<int>(tokens.begin(), tokens.end());
  }

 private:
  Device& d_;
};

// LogitsProcessor (LogitsProcessor.cs:8-114) on the GPU, in place.
class LogitsProcessor {
 public:
  explicit LogitsProcessor(Device& device) : d_(device) {}

  // ApplyRepetitionPenalty (:8-36)
  void ApplyRepetitionPenalty(std::vector<float>* logits, const std::vector<int>* generatedTokenIds,
                              float penalty) const {
    if (!logits) throw ArgumentNullException("logits");
    if (!generatedTokenIds) throw ArgumentNullException("generatedTokenIds");
    if (penalty <= 0.0f) throw ArgumentOutOfRangeException("penalty");
    if (penalty == 1.0f || generatedTokenIds->empty() || logits->empty()) return;
    const int32_t offsets[2] = {0, static_cast<int32_t>(generatedTokenIds->size())};
    check(ncb_logits_repetition_penalty(d_.handle(), logits->data(), 1,
                                        static_cast<int>(logits->size()), generatedTokenIds->data(),
                                        offsets, penalty),
          "ncb_logits_repetition_penalty");
  }
  // ApplyTemperature (:38-51)
  void ApplyTemperature(std::vector<float>* logits, float temperature) const {
    if (!logits) throw ArgumentNullException("logits");
    if (temperature <= 0.0f) throw ArgumentOutOfRangeException("temperature");
    if (temperature == 1.0f || logits->empty()) return;
    check(ncb_logits_temperature(d_.handle(), logits->data(), 1, static_cast<int>(logits->size()),
                                 temperature),
          "ncb_logits_temperature");
  }
  // FilterTopK (:53-73)
  void FilterTopK(std::vector<float>* logits, int topK) const {
    if (!logits) throw ArgumentNullException("logits");
    if (topK <= 0) throw ArgumentOutOfRangeException("topK");
    if (topK >= static_cast<int>(logits->size())) return;
    check(ncb_logits_filter_top_k(d_.handle(), logits->data(), 1, static_cast<int>(logits->size()),
                                  topK),
          "ncb_logits_filter_top_k");
  }
  // FilterTopP (:75-114)
  void FilterTopP(std::vector<float>* probabilities, float topP) const {
    if (!probabilities) throw ArgumentNullException("probabilities");
    if (topP <= 0.0f || topP > 1.0f) throw ArgumentOutOfRangeException("topP");
    if (topP >= 1.0f || probabilities->empty()) return;
    check(ncb_logits_filter_top_p(d_.handle(), probabilities->data(), 1,
                                  static_cast<int>(probabilities->size()), topP, nullptr),
          "ncb_logits_filter_top_p");
  }

 private:
  Device& d_;
};

// GenerationFinishReason (GenerationFinishReason.cs) and GenerationResult
// (GenerationResult.cs:7-27).
enum class GenerationFinishReason { MaxNewTokens, StopToken };
struct GenerationResult {
  std::vector<int> GeneratedTokenIds;
  GenerationFinishReason FinishReason = GenerationFinishReason::MaxNewTokens;
};

// TextGenerator.Generate (TextGenerator.cs:19-51): the decode loop around
// TokenSampler.SampleNext. The model is a callable from the context window's
// token ids to the last position's logits (_model.Forward followed by
// ExtractLastPositionLogits, :34-35); the context is the sequence trimmed to
// the model's last maxPositionEmbeddings ids (TrimToContextWindow,
// :128-139). The history passed to the sampler is the generated ids only
// (:37), and the random source is drawn once per non-greedy step and never
// on a greedy step (TokenSampler.cs:125). Without a random source the loop
// seeds its own from options.Seed(), as :26 does (a std::mt19937_64, not
// .NET's Random: the draws differ from the reference's for the same seed).
class TextGenerator {
 public:
  using Model = std::function<std::vector<float>(const std::vector<int>& context)>;
  // The device-resident handoff: the model leaves the last position's logits
  // in device memory it owns (`vocab` floats, complete in stream order on
  // `stream`) and returns their address; the sampler reads them in place
  // (the D2H copy of ModernDecoderModel.cs:169-170 is gone).
  using DeviceModel = std::function<const float*(const std::vector<int>& context,
                                                 cudaStream_t stream)>;

  TextGenerator(Device& device, int maxPositionEmbeddings)
      : device_(device), sampler_(device), max_positions_(maxPositionEmbeddings) {
    if (maxPositionEmbeddings < 1) throw ArgumentOutOfRangeException("maxPositionEmbeddings");
  }

  GenerationResult Generate(const Model& model, const std::vector<int>& promptTokenIds,
                            const GenerationOptions& options, Random* random = nullptr) const {
    if (!model) throw ArgumentNullException("model");
    if (promptTokenIds.empty()) throw ArgumentException("promptTokenIds");
    std::optional<DefaultRandom> own;
    if (!random) random = &own.emplace(SeedOf(options));
    std::vector<int> sequence(promptTokenIds), generated;
    GenerationResult result;
    for (int step = 0; step < options.MaxNewTokens(); ++step) {
      const std::vector<float> logits = model(Trim(sequence));
      const int next = sampler_.SampleNext(logits, options, generated, *random);
      generated.push_back(next);
      sequence.push_back(next);
      if (IsStop(options, next)) {
        result.FinishReason = GenerationFinishReason::StopToken;
        break;
      }
    }
    result.GeneratedTokenIds = std::move(generated);
    return result;
  }

  // Generate with the logits left on the device. Per step: the model's
  // launches, one 12-byte copy to the device (the history length and the
  // uniform, from pinned memory), ncb_sample_rows_device writing the token
  // straight into the device history (its next slot), and one 4-byte copy
  // back for the stop test and the next context.
  GenerationResult GenerateDevice(const DeviceModel& model, int vocab,
                                  const std::vector<int>& promptTokenIds,
                                  const GenerationOptions& options, cudaStream_t stream,
                                  Random* random = nullptr) const {
    if (!model) throw ArgumentNullException("model");
    if (promptTokenIds.empty()) throw ArgumentException("promptTokenIds");
    if (vocab <= 0) throw ArgumentOutOfRangeException("vocab");
    std::optional<DefaultRandom> own;
    if (!random) random = &own.emplace(SeedOf(options));
    const int cap = std::max(1, options.MaxNewTokens());
    auto dev_free = [](void* p) { cudaFree(p); };
    auto host_free = [](void* p) { cudaFreeHost(p); };
    void* p = nullptr;
    cuda(cudaMalloc(&p, sizeof(int32_t) * (size_t)(cap + 4)), "cudaMalloc");
    std::unique_ptr<void, decltype(dev_free)> dmem(p, dev_free);
    p = nullptr;
    cuda(cudaMallocHost(&p, sizeof(int32_t) * 4), "cudaMallocHost");
    std::unique_ptr<void, decltype(host_free)> hmem(p, host_free);
    int32_t* d_hist = static_cast<int32_t*>(dmem.get());  // [cap] generated ids
    int32_t* d_step = d_hist + cap;                       // {0, n, bits of u}
    int32_t* h_step = static_cast<int32_t*>(hmem.get());  // pinned {0, n, u, token}
    const NcbSamplerParams prm = options.ToParams();
    std::vector<int> sequence(promptTokenIds), generated;
    GenerationResult result;
    for (int step = 0; step < options.MaxNewTokens(); ++step) {
      const float* d_logits = model(Trim(sequence), stream);
      if (!d_logits) throw ArgumentNullException("logits");
      const float u = options.Greedy() ? 0.0f : static_cast<float>(random->NextDouble());
      h_step[0] = 0;
      h_step[1] = step;
      std::memcpy(&h_step[2], &u, sizeof(float));
      cuda(cudaMemcpyAsync(d_step, h_step, 3 * sizeof(int32_t), cudaMemcpyHostToDevice, stream),
           "cudaMemcpyAsync");
      check(ncb_sample_rows_device(device_.handle(), d_logits, 1, vocab, d_hist, d_step,
                                   reinterpret_cast<const float*>(d_step + 2), &prm,
                                   d_hist + step, nullptr, nullptr, stream),
            "ncb_sample_rows_device");
      cuda(cudaMemcpyAsync(&h_step[3], d_hist + step, sizeof(int32_t), cudaMemcpyDeviceToHost,
                           stream),
           "cudaMemcpyAsync");
      cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
      const int next = h_step[3];
      if (next < 0) throw CudaException(NCB_ERROR_INVALID_ARGUMENT, "GenerateDevice: row not sampled");
      generated.push_back(next);
      sequence.push_back(next);
      if (IsStop(options, next)) {
        result.FinishReason = GenerationFinishReason::StopToken;
        break;
      }
    }
    result.GeneratedTokenIds = std::move(generated);
    return result;
  }

 private:
  static uint64_t SeedOf(const GenerationOptions& o) {
    return o.Seed() ? static_cast<uint64_t>(*o.Seed()) : std::random_device{}();
  }
  static bool IsStop(const GenerationOptions& o, int token) {
    const std::vector<int>& s = o.StopTokenIds();
    return std::find(s.begin(), s.end(), token) != s.end();
  }
  static void cuda(cudaError_t e, const char* where) {
    if (e != cudaSuccess) throw CudaException(NCB_ERROR_LAUNCH_FAILED, where);
  }
  std::vector<int> Trim(const std::vector<int>& sequence) const {
    if ((int)sequence.size() <= max_positions_) return sequence;
    return std::vector<int>(sequence.end() - max_positions_, sequence.end());
  }

  Device& device_;
  TokenSampler sampler_;
  int max_positions_;
};

}  // namespace neuraval
