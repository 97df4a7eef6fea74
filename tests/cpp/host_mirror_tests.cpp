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

int main(int argc, char** argv) {
  const bool options_only = argc > 1 && std::strcmp(argv[1], "--options-only") == 0;
  options_tests();
  if (!options_only) {
    Device dev(0, 4, 4096, 64);
    sampler_tests(dev);
    processor_tests(dev);
  }
  std::printf("%d checks, %d failed\n", g_run, g_fail);
  return g_fail == 0 ? 0 : 1;
}
