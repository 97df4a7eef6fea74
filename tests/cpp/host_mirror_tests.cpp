// The reference's own tests for the sampling path (TokenSamplerTests.cs,
// LogitsProcessorTests.cs, GenerationOptionsTests.cs), run against the C++
// mirror (neuraval_generation.hpp) over libnavsampler. Cases come from the
// golden fixture (kats.inc is generated from it). `--options-only` runs the
// GenerationOptions checks, which need no GPU.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "neuraval_generation.hpp"

using namespace neuraval;

struct SamplerKat {
  const char* src;
  std::vector<float> logits;
  std::vector<int> history;
  bool greedy;
  float temperature, top_p;
  int top_k;
  float repetition_penalty;
  std::vector<float> uniforms;
  int expect;
};
enum ExpectKind { kValues, kInvalid, kNucleus2 };
struct ProcessorKat {
  const char* src;
  const char* op;
  std::vector<float> logits;
  std::vector<int> history;
  float arg;
  ExpectKind kind;
  std::vector<float> expect;
};
struct OptionsBase {
  bool greedy;
  float temperature, top_p;
  int top_k;
  float repetition_penalty;
};
struct OptionsKat {
  const char* src;
  const char* field;
  float value;
};

#include "kats.inc"

static int g_fail = 0, g_run = 0;
#define EXPECT(cond, what)                                                        \
  do {                                                                            \
    ++g_run;                                                                      \
    if (!(cond)) {                                                                \
      ++g_fail;                                                                   \
      std::fprintf(stderr, "FAIL %s: %s\n", std::string(what).c_str(), #cond);    \
    }                                                                             \
  } while (0)

template <typename E, typename F>
static bool throws(F&& f) {
  try {
    f();
  } catch (const E&) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}

// A fixed sequence of NextDouble() values (the reference's Random draws).
struct Scripted final : Random {
  std::vector<double> v;
  size_t i = 0;
  explicit Scripted(std::vector<double> x) : v(std::move(x)) {}
  double NextDouble() override { return v[i++ % v.size()]; }
};

static void options_tests() {
  const std::vector<int> none;
  // GenerationOptionsTests.cs:11-25: valid values are kept
  const auto o = GenerationOptions::Create(false, 0.7f, 0.9f, 40, 1.1f, 128, none, 7);
  EXPECT(!o.Greedy() && o.Temperature() == 0.7f && o.TopP() == 0.9f && o.TopK() == 40 &&
             o.RepetitionPenalty() == 1.1f && o.MaxNewTokens() == 128 && o.Seed() == 7,
         "Create_ValidValues_SetsAllProperties");
  for (const auto& c : kOptionsKats) {
    OptionsBase b = kOptionsBase;
    const std::string f = c.field;
    if (f == "temperature") b.temperature = c.value;
    if (f == "top_p") b.top_p = c.value;
    if (f == "top_k") b.top_k = static_cast<int>(c.value);
    if (f == "repetition_penalty") b.repetition_penalty = c.value;
    EXPECT(throws<ArgumentOutOfRangeException>([&] {
             GenerationOptions::Create(b.greedy, b.temperature, b.top_p, b.top_k,
                                       b.repetition_penalty, 10, none);
           }),
           c.src);
  }
  EXPECT(throws<ArgumentOutOfRangeException>(
             [&] { GenerationOptions::Create(false, 1.0f, 1.0f, 1, 1.0f, 0, none); }),
         "maxNewTokens <= 0 (GenerationOptions.cs:68)");
  EXPECT(throws<ArgumentNullException>(
             [&] { GenerationOptions::Create(false, 1.0f, 1.0f, 1, 1.0f, 1, nullptr); }),
         "stopTokenIds null (GenerationOptions.cs:71)");
  const auto g = GenerationOptions::CreateGreedy(10, none);
  EXPECT(g.Greedy() && g.TopK() == INT_MAX && g.Temperature() == 1.0f, "CreateGreedy");
}

static void sampler_tests(Device& dev) {
  TokenSampler ts(dev);
  const std::vector<int> none;
  for (const auto& c : kSamplerKats) {
    const auto o = GenerationOptions::Create(c.greedy, c.temperature, c.top_p, c.top_k,
                                             c.repetition_penalty, 10, none);
    for (float u : c.uniforms) {
      Scripted r({u});
      EXPECT(ts.SampleNext(c.logits, o, c.history, r) == c.expect, c.src);
    }
  }
  // TokenSamplerTests.cs:71-110: null arguments throw ArgumentNullException
  const auto o = GenerationOptions::CreateGreedy(10, none);
  const std::vector<float> lg = {1.0f, 2.0f};
  const std::vector<int> gen;
  DefaultRandom r(1);
  EXPECT(throws<ArgumentNullException>([&] { ts.SampleNext(nullptr, &o, &gen, &r); }),
         "SampleNext_NullLogits_Throws");
  EXPECT(throws<ArgumentNullException>([&] { ts.SampleNext(&lg, nullptr, &gen, &r); }),
         "SampleNext_NullOptions_Throws");
  EXPECT(throws<ArgumentNullException>([&] { ts.SampleNext(&lg, &o, nullptr, &r); }),
         "SampleNext_NullGenerated_Throws");
  EXPECT(throws<ArgumentNullException>([&] { ts.SampleNext(&lg, &o, &gen, nullptr); }),
         "SampleNext_NullRandom_Throws");
  // batched rows consume one draw each, in order
  const std::vector<float> two = {1.0f, 2.0f, 9.0f, 3.0f, 1.0f, 2.0f, 9.0f, 3.0f};
  const auto k1 = GenerationOptions::Create(false, 0.7f, 1.0f, 1, 1.0f, 10, none);
  Scripted rr({0.1, 0.9});
  const auto toks = ts.SampleNextBatch(two, 2, k1, {{}, {}}, rr);
  EXPECT(toks.size() == 2 && toks[0] == 2 && toks[1] == 2, "SampleNextBatch top-k 1");
}

static void processor_tests(Device& dev) {
  LogitsProcessor lp(dev);
  for (const auto& c : kProcessorKats) {
    std::vector<float> x = c.logits;
    const std::string op = c.op;
    auto run = [&] {
      if (op == "repetition_penalty") lp.ApplyRepetitionPenalty(&x, &c.history, c.arg);
      if (op == "temperature") lp.ApplyTemperature(&x, c.arg);
      if (op == "filter_top_k") lp.FilterTopK(&x, static_cast<int>(c.arg));
      if (op == "filter_top_p") lp.FilterTopP(&x, c.arg);
    };
    if (c.kind == kInvalid) {
      EXPECT(throws<ArgumentOutOfRangeException>(run), c.src);
      continue;
    }
    run();
    if (c.kind == kNucleus2) {
      // LogitsProcessorTests.cs:132-139: the two largest kept and renormalised
      double sum = 0;
      for (float v : x) sum += v;
      EXPECT(x[2] == 0.0f && x[3] == 0.0f && x[0] > 0.0f && x[1] > 0.0f &&
                 std::fabs(sum - 1.0) < 5e-6,
             c.src);
      continue;
    }
    bool same = x.size() == c.expect.size();
    for (size_t i = 0; same && i < x.size(); ++i) same = x[i] == c.expect[i];
    EXPECT(same, c.src);
  }
  std::vector<float> x = {1.0f};
  EXPECT(throws<ArgumentNullException>([&] { lp.ApplyTemperature(nullptr, 2.0f); }),
         "ApplyTemperature null");
  EXPECT(throws<ArgumentNullException>([&] { lp.ApplyRepetitionPenalty(&x, nullptr, 2.0f); }),
         "ApplyRepetitionPenalty null history");
}

// TextGenerator.Generate (TextGenerator.cs:19-51) over a toy model: the logits
// are a fixed function of the context window, so every step can be replayed.
static std::vector<float> toy_logits(const std::vector<int>& ctx, int V) {
  uint64_t h = 1469598103934665603ull;
  for (int t : ctx) h = (h ^ (uint64_t)(uint32_t)t) * 1099511628211ull;
  std::vector<float> x(V);
  for (int i = 0; i < V; ++i) {
    uint64_t z = h + 0x9E3779B97F4A7C15ull * (uint64_t)(i + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    x[i] = (float)((double)(z >> 11) * 0x1p-53 * 12.0 - 6.0);  // uniform in [-6, 6)
  }
  return x;
}

// Counts the draws and remembers them.
struct Counting final : Random {
  DefaultRandom r;
  std::vector<double> seen;
  explicit Counting(uint64_t seed) : r(seed) {}
  double NextDouble() override {
    seen.push_back(r.NextDouble());
    return seen.back();
  }
};

static void generator_tests(Device& dev) {
  const int V = 4096, window = 16;
  int forwards = 0;
  size_t longest = 0;
  TextGenerator gen(dev, window);
  const TextGenerator::Model model = [&](const std::vector<int>& ctx) {
    ++forwards;
    longest = std::max(longest, ctx.size());
    return toy_logits(ctx, V);
  };
  const std::vector<int> prompt = {5, 17, 42};
  const std::vector<int> none;
  EXPECT(throws<ArgumentException>([&] { gen.Generate(model, {}, GenerationOptions::Default(none)); }),
         "Generate empty prompt");

  // greedy steps never draw (TokenSampler.cs:25-26 takes the greedy path first)
  const auto greedy = GenerationOptions::Create(true, 1.0f, 1.0f, INT_MAX, 1.1f, 24, none);
  Counting rg(7);
  GenerationResult res = gen.Generate(model, prompt, greedy, &rg);
  EXPECT(rg.seen.empty(), "greedy steps draw nothing");
  EXPECT(res.GeneratedTokenIds.size() == 24 && res.FinishReason == GenerationFinishReason::MaxNewTokens,
         "greedy runs to MaxNewTokens");
  EXPECT(longest <= (size_t)window, "context trimmed to the window");

  // filtered steps draw exactly once each, in step order; replaying the steps
  // through SampleNext with the same draws gives the same tokens
  const auto filt = GenerationOptions::Create(false, 0.8f, 0.9f, 40, 1.1f, 24, none);
  Counting rf(11);
  forwards = 0;
  res = gen.Generate(model, prompt, filt, &rf);
  EXPECT(rf.seen.size() == 24 && forwards == 24, "one draw and one forward per filtered step");
  {
    TokenSampler ts(dev);
    std::vector<int> seq(prompt), hist;
    bool same = true;
    for (size_t i = 0; i < res.GeneratedTokenIds.size(); ++i) {
      std::vector<int> ctx(seq.size() > (size_t)window ? seq.end() - window : seq.begin(), seq.end());
      Scripted one({rf.seen[i]});
      const int t = ts.SampleNext(toy_logits(ctx, V), filt, hist, one);
      same = same && t == res.GeneratedTokenIds[i];
      hist.push_back(t);
      seq.push_back(t);
    }
    EXPECT(same, "each step is SampleNext on the window's logits, the generated ids and its draw");
  }

  // a stop id ends the loop at its first occurrence, the stop id included (:40-47)
  const int stop = res.GeneratedTokenIds[9];
  size_t first = 0;
  while (res.GeneratedTokenIds[first] != stop) ++first;
  const auto filt_stop = GenerationOptions::Create(false, 0.8f, 0.9f, 40, 1.1f, 24, {stop});
  Counting rs(11);
  GenerationResult rstop = gen.Generate(model, prompt, filt_stop, &rs);
  EXPECT(rstop.FinishReason == GenerationFinishReason::StopToken &&
             rstop.GeneratedTokenIds.size() == first + 1 && rstop.GeneratedTokenIds.back() == stop &&
             rs.seen.size() == first + 1,
         "stop token ends generation");

  // device-resident logits: the same tokens and draws as the host loop
  float* d_logits = nullptr;
  if (cudaMalloc(reinterpret_cast<void**>(&d_logits), sizeof(float) * V) != cudaSuccess) {
    EXPECT(false, "cudaMalloc for the device model");
    return;
  }
  const TextGenerator::DeviceModel dmodel = [&](const std::vector<int>& ctx, cudaStream_t st) {
    const std::vector<float> x = toy_logits(ctx, V);
    cudaMemcpyAsync(d_logits, x.data(), sizeof(float) * V, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);  // x is a temporary
    return static_cast<const float*>(d_logits);
  };
  cudaStream_t st = nullptr;
  cudaStreamCreate(&st);
  for (const GenerationOptions* o : {&greedy, &filt, &filt_stop}) {
    Counting a(23), b(23);
    const GenerationResult h = gen.Generate(model, prompt, *o, &a);
    const GenerationResult d = gen.GenerateDevice(dmodel, V, prompt, *o, st, &b);
    EXPECT(h.GeneratedTokenIds == d.GeneratedTokenIds && h.FinishReason == d.FinishReason &&
               a.seen == b.seen,
           "device-resident loop equals the host loop");
  }
  cudaStreamDestroy(st);
  cudaFree(d_logits);
}

int main(int argc, char** argv) {
  const bool options_only = argc > 1 && std::strcmp(argv[1], "--options-only") == 0;
  options_tests();
  if (!options_only) {
    Device dev(0, 4, 4096, 64);
    sampler_tests(dev);
    processor_tests(dev);
    generator_tests(dev);
  }
  std::printf("%d checks, %d failed\n", g_run, g_fail);
  return g_fail == 0 ? 0 : 1;
}
