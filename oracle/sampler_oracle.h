/*
 * CPU oracle for Neuraval's decode-time logits processing and token sampling.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads or
 * calls this code. Only the pytest suite, `__graft_entry__.smoke()` and the
 * CPU-baseline leg of `bench.py` use it, and only as the oracle to compare with or as the
 * timed CPU stand-in for the reference's C# implementation.
 *
 * It restates, in strict IEEE fp32 C, the C# reference:
 *   Neuraval/Generation/TokenSampler.cs:10-143    (SampleNext, SampleGreedy,
 *                                                  SampleFiltered, AdjustLogit)
 *   Neuraval/Generation/LogitsProcessor.cs:8-114  (ApplyRepetitionPenalty,
 *                                                  ApplyTemperature, FilterTopK,
 *                                                  FilterTopP)
 * plus the frequency/presence penalty, which the reference does not have and
 * which this library defines as  v - cnt*f - [cnt>0]*p  applied after the
 * repetition penalty and before the temperature scale.
 */
#ifndef NEURAVAL_SAMPLER_ORACLE_H
#define NEURAVAL_SAMPLER_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as NcbSamplerParams in include/navsampler.h. */
typedef struct OracleParams {
    int32_t greedy;
    float temperature;
    float top_p;
    int32_t top_k;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
} OracleParams;

/* Row flags; same bit values as NCB_FLAG_* in include/navsampler.h. */
#define ORACLE_FLAG_DRAW_BOUNDARY   0x1u  /* |u*retained - S_j| or |.. - S_{j-1}| <= 1e-6*retained */
#define ORACLE_FLAG_CUTOFF_BOUNDARY 0x2u  /* top-p test S_i >= target within 1e-6 relative */
#define ORACLE_FLAG_TIE_AT_DRAW     0x4u  /* drawn position sits in a group of equal values */
#define ORACLE_FLAG_NONFINITE       0x8u  /* NaN / +inf value or no finite maximum: token -1 */
#define ORACLE_FLAG_EXP_SLOW        0x10u /* a weight needed the double-double exp path */

/* Exponential used for the candidate weights. */
#define ORACLE_EXP_GLIBC 0  /* libm expf: what MathF.Exp resolves to on Linux */
#define ORACLE_EXP_CR    1  /* correctly rounded expf (what the CUDA kernels compute) */

/* Status codes (NcbStatus in Neuraval.Cuda.Native/src/navcuda.cu:19-29). */
#define ORACLE_OK 0
#define ORACLE_ERROR_INVALID_ARGUMENT 7

/* Correctly rounded expf (double exp, with a double-double fallback when the
 * double result is within 2^-51 relative of a float rounding midpoint).
 * *slow is set to 1 when the fallback ran (may be NULL). */
float oracle_expf_cr(float x, int* slow);

/* The double-double path of oracle_expf_cr, always taken (for testing it). */
float oracle_expf_dd(float x);

/* One row: TokenSampler.SampleNext. `hist` holds H generated token ids (any
 * value; ids outside [0,V) never match). `u` stands for
 * (float)random.NextDouble() and is only read on the non-greedy path.
 * `probs_out` (optional, V floats) receives w_i/retained for the retained
 * candidates and 0 elsewhere. Returns the token id, or -1 with
 * ORACLE_FLAG_NONFINITE set, or -2 for invalid arguments. */
int32_t oracle_sample_row(const float* logits, int32_t V, const int32_t* hist,
                          int32_t H, const OracleParams* p, float u,
                          int exp_mode, uint32_t* flags, float* probs_out);

/* Batched front end over a [B,V] row-major matrix and CSR histories
 * (hist_offsets has B+1 entries). Rows are spread over `threads` POSIX
 * threads (<=1 runs them in order on the caller's thread). */
int oracle_sample_rows(const float* logits, int32_t B, int32_t V,
                       const int32_t* hist, const int64_t* hist_offsets,
                       const float* uniforms, const OracleParams* p,
                       int exp_mode, int threads, int32_t* tokens,
                       uint32_t* flags, float* probs_out);

/* LogitsProcessor, one row each. Return ORACLE_OK or
 * ORACLE_ERROR_INVALID_ARGUMENT (the C# ArgumentOutOfRange/Null cases). */
int oracle_apply_repetition_penalty(float* logits, int32_t V, const int32_t* hist,
                                    int32_t H, float penalty);
int oracle_apply_frequency_presence_penalty(float* logits, int32_t V,
                                            const int32_t* hist, int32_t H,
                                            float frequency, float presence);
int oracle_apply_temperature(float* logits, int32_t V, float temperature);
int oracle_filter_top_k(float* logits, int32_t V, int32_t top_k);
/* `tie_flag` (optional) is set to 1 when the cutoff falls inside a group of
 * equal probabilities, where the C# unstable sort decides which ids survive. */
int oracle_filter_top_p(float* probs, int32_t V, float top_p, uint32_t* tie_flag);

#ifdef __cplusplus
}
#endif

#endif
