/*
 * CPU oracle for Neuraval's decode-time logits processing and token sampling.
 *
 * TEST INFRASTRUCTURE ONLY (see sampler_oracle.h). Build with
 * -O2 -ffp-contract=off and without -ffast-math: every float expression here
 * must round exactly as the C# code's fp32 arithmetic does (RyuJIT neither
 * contracts a*b+c into an FMA nor keeps float temporaries in wider registers).
 *
 * Parity notes
 *  - Candidate order: the reference sorts with List<T>.Sort, an unstable
 *    introsort (TokenSampler.cs:95). Equal values keep ascending id order here,
 *    and a row whose draw lands on such a tie is flagged
 *    (ORACLE_FLAG_TIE_AT_DRAW) because the C# order among them is unknowable
 *    without running .NET.
 *  - -0.0f and +0.0f compare equal in C#'s float.CompareTo, so they tie here too.
 *  - MathF.Exp resolves to the platform expf; ORACLE_EXP_GLIBC calls libm's expf.
 *    ORACLE_EXP_CR uses a correctly rounded expf, the function the CUDA kernels
 *    implement, so the two modes differ only where libm misrounds (< 0.502 ulp).
 *  - NaN or +inf values, or a row without a finite maximum, make the C# code
 *    depend on heap layout and element position; this oracle and the CUDA
 *    kernels both return -1 with ORACLE_FLAG_NONFINITE for such rows.
 */
#include "sampler_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* Correctly rounded expf                                                      */
/* ------------------------------------------------------------------------- */

/* ln 2 split into two 40-bit heads and a tail (derived from a 80-digit value
 * of ln 2), so that k*LN2_A and k*LN2_B are exact for |k| < 2^13. */
static const double LN2_A = 0x1.62e42fefa4000p-1;
static const double LN2_B = -0x1.8432a1b0e2000p-43;
static const double LN2_C = -0x1.8cff81a12a17ep-85;
static const double INV_LN2 = 0x1.71547652b82fep+0;

typedef struct { double hi, lo; } dd_t;

static dd_t dd_two_sum(double a, double b) {
    double s = a + b;
    double bb = s - a;
    double e = (a - (s - bb)) + (b - bb);
    dd_t r = {s, e};
    return r;
}
static dd_t dd_fast_two_sum(double a, double b) {
    double s = a + b;
    dd_t r = {s, b - (s - a)};
    return r;
}
static dd_t dd_add(dd_t a, dd_t b) {
    dd_t s = dd_two_sum(a.hi, b.hi);
    dd_t t = dd_two_sum(a.lo, b.lo);
    s.lo += t.hi;
    s = dd_fast_two_sum(s.hi, s.lo);
    s.lo += t.lo;
    return dd_fast_two_sum(s.hi, s.lo);
}
static dd_t dd_mul(dd_t a, dd_t b) {
    double p = a.hi * b.hi;
    double e = fma(a.hi, b.hi, -p);
    e += a.hi * b.lo + a.lo * b.hi;
    return dd_fast_two_sum(p, e);
}
static dd_t dd_mul_d(dd_t a, double b) {
    double p = a.hi * b;
    double e = fma(a.hi, b, -p);
    e += a.lo * b;
    return dd_fast_two_sum(p, e);
}

/* exp(x) as a double-double, relative error far below 2^-90 for x in
 * [-104, 89]: x = k ln2 + r, exp(r) = (Taylor(r/256))^(2^8), times 2^k. */
static dd_t dd_exp(double x) {
    double k = nearbyint(x * INV_LN2);
    dd_t r = dd_two_sum(x - k * LN2_A, -k * LN2_B);
    r = dd_add(r, (dd_t){-k * LN2_C, 0.0});
    dd_t s = {ldexp(r.hi, -8), ldexp(r.lo, -8)};
    /* Horner for sum_{n=0..11} s^n/n! */
    dd_t acc = {1.0, 0.0};
    for (int n = 11; n >= 1; --n) {
        acc = dd_mul(acc, s);
        /* acc = acc / n + ... : compute acc*(1/n) exactly enough via division */
        double q = acc.hi / n;
        double rem = fma(-q, (double)n, acc.hi) + acc.lo;
        dd_t t = dd_fast_two_sum(q, rem / n);
        acc = dd_add(t, (dd_t){1.0, 0.0});
    }
    for (int i = 0; i < 8; ++i) acc = dd_mul(acc, acc);
    int ki = (int)k;
    acc.hi = ldexp(acc.hi, ki);
    acc.lo = ldexp(acc.lo, ki);
    return acc;
}

static float next_toward(float f, int up) {
    /* f >= 0 here */
    union { float f; uint32_t u; } c = {f};
    if (up) c.u += 1u; else if (c.u > 0) c.u -= 1u;
    return c.f;
}

/* Round the double-double value (hi, lo) >= 0 to the nearest float. */
static float dd_to_float(dd_t v) {
    float f = (float)v.hi;
    double fd = (double)f;
    double res = (v.hi - fd) + v.lo;
    if (res == 0.0) return f;
    float nb = next_toward(f, res > 0.0);
    double mid = (fd + (double)nb) * 0.5;
    double side = (v.hi - mid) + v.lo;
    if ((res > 0.0 && side > 0.0) || (res < 0.0 && side < 0.0)) return nb;
    return f;
}

float oracle_expf_cr(float x, int* slow) {
    if (slow) *slow = 0;
    if (x != x) return x;
    if (x == -INFINITY) return 0.0f;
    double y = exp((double)x);
    float f = (float)y;
    if (y == 0.0 || isinf(f)) return f;
    double fd = (double)f;
    double d = y - fd;
    if (d == 0.0) return f;  /* only x == 0 */
    float nb = next_toward(f, d > 0.0);
    double mid = (fd + (double)nb) * 0.5;
    if (fabs(y - mid) > 0x1p-51 * y) return f;
    if (slow) *slow = 1;
    return dd_to_float(dd_exp((double)x));
}

float oracle_expf_dd(float x) {
    if (x != x) return x;
    if (x == -INFINITY) return 0.0f;
    return dd_to_float(dd_exp((double)x));
}

static inline float weight_exp(float x, int mode, uint32_t* flags) {
    if (mode == ORACLE_EXP_GLIBC) return expf(x);
    int slow = 0;
    float r = oracle_expf_cr(x, &slow);
    if (slow && flags) *flags |= ORACLE_FLAG_EXP_SLOW;
    return r;
}

/* ------------------------------------------------------------------------- */
/* Penalties (TokenSampler.AdjustLogit, TokenSampler.cs:137-143)               */
/* ------------------------------------------------------------------------- */

typedef struct {
    uint8_t* member;   /* V bytes: id present in history (HashSet semantics) */
    int32_t* count;    /* V ints: occurrences in history, or NULL */
    int use_rep;       /* repetition penalty active (penalty != 1 and H > 0) */
} PenaltyState;

static int penalty_init(PenaltyState* ps, int32_t V, const int32_t* hist, int32_t H,
                        const OracleParams* p) {
    memset(ps, 0, sizeof(*ps));
    /* TokenSampler.cs:34-36, 61-63: the set exists only when the penalty is not 1
     * and the history is not empty; ids outside [0,V) never match a token id. */
    ps->use_rep = (p->repetition_penalty != 1.0f && H > 0);
    int need_count = (p->frequency_penalty != 0.0f || p->presence_penalty != 0.0f) && H > 0;
    if (ps->use_rep || need_count) {
        ps->member = (uint8_t*)calloc((size_t)V, 1);
        if (!ps->member) return -1;
    }
    if (need_count) {
        ps->count = (int32_t*)calloc((size_t)V, sizeof(int32_t));
        if (!ps->count) return -1;
    }
    for (int32_t i = 0; i < H; ++i) {
        int32_t t = hist[i];
        if (t < 0 || t >= V) continue;
        if (ps->member) ps->member[t] = 1;
        if (ps->count) ps->count[t] += 1;
    }
    return 0;
}

static void penalty_free(PenaltyState* ps) {
    free(ps->member);
    free(ps->count);
}

/* Value before the temperature scale: AdjustLogit, then the frequency/presence
 * penalty (new; v - cnt*f - [cnt>0]*p). */
static inline float adjusted(const PenaltyState* ps, const OracleParams* p,
                             float l, int32_t i) {
    float v = l;
    if (ps->use_rep && ps->member[i])
        v = (v > 0.0f) ? v / p->repetition_penalty : v * p->repetition_penalty;
    if (ps->count && ps->count[i] > 0) {
        float c = (float)ps->count[i];
        v = v - c * p->frequency_penalty;
        v = v - p->presence_penalty;
    }
    return v;
}

/* ------------------------------------------------------------------------- */
/* SampleGreedy (TokenSampler.cs:32-52)                                        */
/* ------------------------------------------------------------------------- */

static int32_t sample_greedy(const float* logits, int32_t V, const PenaltyState* ps,
                             const OracleParams* p) {
    int32_t best = 0;
    float bestv = adjusted(ps, p, logits[0], 0);
    for (int32_t i = 1; i < V; ++i) {
        float v = adjusted(ps, p, logits[i], i);
        if (v > bestv) { bestv = v; best = i; }
    }
    return best;
}

/* ------------------------------------------------------------------------- */
/* SampleFiltered (TokenSampler.cs:54-135)                                     */
/* ------------------------------------------------------------------------- */

typedef struct { int32_t id; float v; } Cand;

/* Binary min-heap of floats: PriorityQueue<Candidate,float> keeps the
 * candidateLimit largest values; only its minimum is ever read. */
static void heap_sift_down(float* h, int32_t n, int32_t i) {
    for (;;) {
        int32_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && h[l] < h[m]) m = l;
        if (r < n && h[r] < h[m]) m = r;
        if (m == i) return;
        float t = h[i]; h[i] = h[m]; h[m] = t;
        i = m;
    }
}
static void heap_push(float* h, int32_t* n, float v) {
    int32_t i = (*n)++;
    h[i] = v;
    while (i > 0) {
        int32_t par = (i - 1) / 2;
        if (!(h[i] < h[par])) break;
        float t = h[i]; h[i] = h[par]; h[par] = t;
        i = par;
    }
}

/* descending value, ascending id among equal values (-0 == +0) */
static int cand_cmp(const void* a, const void* b) {
    const Cand* x = (const Cand*)a;
    const Cand* y = (const Cand*)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

static int32_t sample_filtered(const float* logits, int32_t V, const PenaltyState* ps,
                               const OracleParams* p, float u, int exp_mode,
                               uint32_t* flags, float* probs_out) {
    int32_t limit = p->top_k < V ? p->top_k : V;
    float scale = 1.0f / p->temperature;

    float* heap = (float*)malloc(sizeof(float) * (size_t)limit);
    if (!heap) return -2;
    int32_t hn = 0;
    int nonfinite = 0;
    for (int32_t i = 0; i < V; ++i) {
        float v = adjusted(ps, p, logits[i], i) * scale;
        if (v != v || v == INFINITY) { nonfinite = 1; break; }
        if (hn < limit) heap_push(heap, &hn, v);
        else if (v > heap[0]) { heap[0] = v; heap_sift_down(heap, hn, 0); }
    }
    if (nonfinite) { free(heap); *flags |= ORACLE_FLAG_NONFINITE; return -1; }
    float threshold = heap[0];
    free(heap);

    /* TokenSampler.cs:88-93: every value >= threshold, in ascending id order */
    int32_t cap = limit + 16, n = 0;
    Cand* c = (Cand*)malloc(sizeof(Cand) * (size_t)cap);
    if (!c) return -2;
    for (int32_t i = 0; i < V; ++i) {
        float v = adjusted(ps, p, logits[i], i) * scale;
        if (v >= threshold) {
            if (n == cap) {
                cap *= 2;
                Cand* nc = (Cand*)realloc(c, sizeof(Cand) * (size_t)cap);
                if (!nc) { free(c); return -2; }
                c = nc;
            }
            c[n].id = i;
            c[n].v = v + 0.0f; /* -0 -> +0: they compare equal in C# */
            ++n;
        }
    }
    qsort(c, (size_t)n, sizeof(Cand), cand_cmp);

    float maxv = c[0].v;
    if (!(maxv > -INFINITY)) { free(c); *flags |= ORACLE_FLAG_NONFINITE; return -1; }

    float* w = (float*)malloc(sizeof(float) * (size_t)n);
    float* S = (float*)malloc(sizeof(float) * (size_t)n);
    if (!w || !S) { free(c); free(w); free(S); return -2; }
    float total = 0.0f;
    for (int32_t i = 0; i < n; ++i) {
        w[i] = weight_exp(c[i].v - maxv, exp_mode, flags);
        total += w[i];
        S[i] = total;
    }

    int32_t cutoff = n;
    float target = 0.0f;
    if (p->top_p < 1.0f) {
        target = total * p->top_p;
        float cum = 0.0f;
        for (int32_t i = 0; i < n; ++i) {
            cum += w[i];
            if (cum >= target) { cutoff = i + 1; break; }
        }
    }
    float retained = 0.0f;
    for (int32_t i = 0; i < cutoff; ++i) retained += w[i];

    float sample = u * retained;
    float cum = 0.0f;
    int32_t sel = cutoff - 1;  /* cutoff >= 1: the maximum is always a candidate */
    for (int32_t i = 0; i < cutoff; ++i) {
        cum += w[i];
        if (sample <= cum || i == cutoff - 1) { sel = i; break; }
    }

    /* flags (the CUDA kernels derive the same bits from the same sums) */
    double tol = 1e-6 * (double)retained;
    if (fabs((double)sample - (double)S[sel]) <= tol ||
        (sel >= 1 && fabs((double)sample - (double)S[sel - 1]) <= tol))
        *flags |= ORACLE_FLAG_DRAW_BOUNDARY;
    if (p->top_p < 1.0f) {
        double tt = 1e-6 * (double)target;
        if (fabs((double)S[cutoff - 1] - (double)target) <= tt ||
            (cutoff >= 2 && fabs((double)S[cutoff - 2] - (double)target) <= tt))
            *flags |= ORACLE_FLAG_CUTOFF_BOUNDARY;
    }
    if ((sel > 0 && c[sel - 1].v == c[sel].v) || (sel + 1 < n && c[sel + 1].v == c[sel].v))
        *flags |= ORACLE_FLAG_TIE_AT_DRAW;

    if (probs_out) {
        for (int32_t i = 0; i < cutoff; ++i) probs_out[c[i].id] = w[i] / retained;
    }
    int32_t token = c[sel].id;
    free(c); free(w); free(S);
    return token;
}

static int params_valid(const OracleParams* p) {
    /* GenerationOptions.Create (GenerationOptions.cs:56-72) */
    if (!(p->temperature > 0.0f)) return 0;
    if (!(p->top_p > 0.0f) || p->top_p > 1.0f) return 0;
    if (p->top_k <= 0) return 0;
    if (!(p->repetition_penalty > 0.0f)) return 0;
    if (!(p->frequency_penalty == p->frequency_penalty)) return 0;
    if (!(p->presence_penalty == p->presence_penalty)) return 0;
    return 1;
}

int32_t oracle_sample_row(const float* logits, int32_t V, const int32_t* hist,
                          int32_t H, const OracleParams* p, float u,
                          int exp_mode, uint32_t* flags, float* probs_out) {
    uint32_t fl = 0;
    if (!logits || !p || V <= 0 || H < 0 || (H > 0 && !hist)) return -2;
    if (!params_valid(p)) return -2;
    if (probs_out) memset(probs_out, 0, sizeof(float) * (size_t)V);
    PenaltyState ps;
    if (penalty_init(&ps, V, hist, H, p) != 0) { penalty_free(&ps); return -2; }
    int32_t tok;
    if (p->greedy) tok = sample_greedy(logits, V, &ps, p);
    else tok = sample_filtered(logits, V, &ps, p, u, exp_mode, &fl, probs_out);
    penalty_free(&ps);
    if (flags) *flags = fl;
    return tok;
}

/* ------------------------------------------------------------------------- */
/* Batched front end                                                           */
/* ------------------------------------------------------------------------- */

typedef struct {
    const float* logits; int32_t B, V;
    const int32_t* hist; const int64_t* off;
    const float* uniforms; const OracleParams* p;
    int exp_mode; int32_t* tokens; uint32_t* flags; float* probs;
    int32_t first, step;
    int status;
} RowJob;

static void* row_worker(void* arg) {
    RowJob* j = (RowJob*)arg;
    for (int32_t r = j->first; r < j->B; r += j->step) {
        int64_t a = j->off[r], b = j->off[r + 1];
        uint32_t f = 0;
        int32_t t = oracle_sample_row(j->logits + (size_t)r * j->V, j->V,
                                      j->hist ? j->hist + a : NULL, (int32_t)(b - a),
                                      j->p, j->uniforms ? j->uniforms[r] : 0.0f,
                                      j->exp_mode, &f,
                                      j->probs ? j->probs + (size_t)r * j->V : NULL);
        if (t == -2) j->status = ORACLE_ERROR_INVALID_ARGUMENT;
        j->tokens[r] = t;
        if (j->flags) j->flags[r] = f;
    }
    return NULL;
}

int oracle_sample_rows(const float* logits, int32_t B, int32_t V,
                       const int32_t* hist, const int64_t* hist_offsets,
                       const float* uniforms, const OracleParams* p,
                       int exp_mode, int threads, int32_t* tokens,
                       uint32_t* flags, float* probs_out) {
    if (!logits || !hist_offsets || !p || !tokens || B < 0 || V <= 0)
        return ORACLE_ERROR_INVALID_ARGUMENT;
    if (!params_valid(p)) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (threads < 1) threads = 1;
    if (threads > B) threads = B > 0 ? B : 1;
    RowJob* jobs = (RowJob*)calloc((size_t)threads, sizeof(RowJob));
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    if (!jobs || !tids) { free(jobs); free(tids); return ORACLE_ERROR_INVALID_ARGUMENT; }
    for (int t = 0; t < threads; ++t) {
        RowJob j = {logits, B, V, hist, hist_offsets, uniforms, p, exp_mode,
                    tokens, flags, probs_out, t, threads, ORACLE_OK};
        jobs[t] = j;
    }
    if (threads == 1) {
        row_worker(&jobs[0]);
    } else {
        for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, row_worker, &jobs[t]);
        for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
    }
    int st = ORACLE_OK;
    for (int t = 0; t < threads; ++t) if (jobs[t].status != ORACLE_OK) st = jobs[t].status;
    free(jobs); free(tids);
    return st;
}

/* ------------------------------------------------------------------------- */
/* LogitsProcessor (LogitsProcessor.cs:8-114)                                  */
/* ------------------------------------------------------------------------- */

int oracle_apply_repetition_penalty(float* logits, int32_t V, const int32_t* hist,
                                    int32_t H, float penalty) {
    if (!logits || (H > 0 && !hist) || V < 0 || H < 0) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (!(penalty > 0.0f)) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (penalty == 1.0f || H == 0) return ORACLE_OK;
    uint8_t* seen = (uint8_t*)calloc((size_t)V + 1, 1);
    if (!seen) return ORACLE_ERROR_INVALID_ARGUMENT;
    for (int32_t i = 0; i < H; ++i) {
        int32_t t = hist[i];
        if (t < 0 || t >= V) continue;
        if (seen[t]) continue;
        seen[t] = 1;
        logits[t] = logits[t] > 0.0f ? logits[t] / penalty : logits[t] * penalty;
    }
    free(seen);
    return ORACLE_OK;
}

int oracle_apply_frequency_presence_penalty(float* logits, int32_t V,
                                            const int32_t* hist, int32_t H,
                                            float frequency, float presence) {
    if (!logits || (H > 0 && !hist) || V < 0 || H < 0) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (frequency != frequency || presence != presence) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (H == 0 || (frequency == 0.0f && presence == 0.0f)) return ORACLE_OK;
    int32_t* cnt = (int32_t*)calloc((size_t)V + 1, sizeof(int32_t));
    if (!cnt) return ORACLE_ERROR_INVALID_ARGUMENT;
    for (int32_t i = 0; i < H; ++i) {
        int32_t t = hist[i];
        if (t >= 0 && t < V) cnt[t] += 1;
    }
    for (int32_t i = 0; i < V; ++i) {
        if (cnt[i] > 0) {
            float v = logits[i];
            v = v - (float)cnt[i] * frequency;
            v = v - presence;
            logits[i] = v;
        }
    }
    free(cnt);
    return ORACLE_OK;
}

int oracle_apply_temperature(float* logits, int32_t V, float temperature) {
    if (!logits || V < 0) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (!(temperature > 0.0f)) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (temperature == 1.0f) return ORACLE_OK;
    for (int32_t i = 0; i < V; ++i) logits[i] /= temperature;
    return ORACLE_OK;
}

static int float_asc(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

int oracle_filter_top_k(float* logits, int32_t V, int32_t top_k) {
    if (!logits || V < 0) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (top_k <= 0) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (top_k >= V) return ORACLE_OK;
    float* sorted = (float*)malloc(sizeof(float) * (size_t)V);
    if (!sorted) return ORACLE_ERROR_INVALID_ARGUMENT;
    memcpy(sorted, logits, sizeof(float) * (size_t)V);
    qsort(sorted, (size_t)V, sizeof(float), float_asc);
    float threshold = sorted[V - top_k];
    free(sorted);
    for (int32_t i = 0; i < V; ++i)
        if (logits[i] < threshold) logits[i] = -INFINITY;
    return ORACLE_OK;
}

typedef struct { int32_t id; float p; } ProbIdx;
static int prob_desc(const void* a, const void* b) {
    const ProbIdx* x = (const ProbIdx*)a;
    const ProbIdx* y = (const ProbIdx*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

int oracle_filter_top_p(float* probs, int32_t V, float top_p, uint32_t* tie_flag) {
    if (tie_flag) *tie_flag = 0;
    if (!probs || V < 0) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (!(top_p > 0.0f) || top_p > 1.0f) return ORACLE_ERROR_INVALID_ARGUMENT;
    if (top_p >= 1.0f) return ORACLE_OK;
    ProbIdx* o = (ProbIdx*)malloc(sizeof(ProbIdx) * (size_t)(V > 0 ? V : 1));
    if (!o) return ORACLE_ERROR_INVALID_ARGUMENT;
    for (int32_t i = 0; i < V; ++i) { o[i].id = i; o[i].p = probs[i] + 0.0f; }
    qsort(o, (size_t)V, sizeof(ProbIdx), prob_desc);
    int32_t cutoff = V;
    float cum = 0.0f;
    for (int32_t i = 0; i < V; ++i) {
        cum += probs[o[i].id];
        if (cum >= top_p) { cutoff = i + 1; break; }
    }
    float retained = 0.0f;
    for (int32_t i = 0; i < cutoff; ++i) retained += probs[o[i].id];
    if (tie_flag && cutoff < V && cutoff > 0 && o[cutoff - 1].p == o[cutoff].p) *tie_flag = 1;
    float* filtered = (float*)calloc((size_t)(V > 0 ? V : 1), sizeof(float));
    if (!filtered) { free(o); return ORACLE_ERROR_INVALID_ARGUMENT; }
    for (int32_t i = 0; i < cutoff; ++i)
        filtered[o[i].id] = retained > 0.0f ? probs[o[i].id] / retained : 0.0f;
    memcpy(probs, filtered, sizeof(float) * (size_t)V);
    free(filtered);
    free(o);
    return ORACLE_OK;
}
