/*
 * CPU oracle for the masked-selection path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference implementation of
 * karthikeyansura/bitmask-speculation for the masked-selection hot path.  It is
 * the checker the CUDA kernels are compared against and the CPU baseline that
 * the benchmark times; nothing in the shipped library links or calls it.
 *
 *   orc_mask_count       grammar/density.py:23-48 (packed_mask_count):
 *                        popcount of signed int32 words, bits at or beyond the
 *                        vocabulary ignored.
 *   orc_reduce_rows      benchmarks/reductions.py:9-17 (torch_reduce) with the
 *                        native status/token convention of csrc/argmax.cu:77-98:
 *                        status 2 when any logit of the row is NaN (masked or
 *                        not), 1 when no token is valid, else 0; the token is the
 *                        lowest valid index whose logit equals the masked maximum
 *                        (grammar/selection.py:12-32), -1 on error.
 *   orc_sample_row       kernels/reference.py:10-52 (masked_sample_reference):
 *                        fp64 weights exp((x - max) / T), cutoff = u * fsum(w),
 *                        first token with cutoff < running sum, last positive
 *                        weight as the rounding fallback.  Status codes follow
 *                        csrc/sample.cu:24-25,65-67 (2 NaN, 5 +inf valid,
 *                        1 empty, 4 no finite mass, 3 bad uniform).
 *   orc_fsum             CPython math.fsum: Shewchuk's exact partial sums
 *                        ("Adaptive precision floating-point arithmetic", 1997)
 *                        with round-half-even correction of the final sum.
 *   orc_budget           decoding/scheduling.py:40-46 (DensityPolicy.budget)
 *                        and the linear density schedule (kind 1).
 *   orc_verify           decoding/verification.py:18-48 (verify_prefix) applied
 *                        to per-row targets, as models/transformers.py:181-201
 *                        consumes them: rows after the first mismatch are never
 *                        looked at, so their status cannot fail a sequence.
 *
 * dtype codes: 0 float32, 1 bfloat16, 2 float16 (exact widening to float).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float f32_from_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, sizeof f);
    return f;
}

static inline float bf16_to_f32(uint16_t h) { return f32_from_bits((uint32_t)h << 16); }

static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while (!(man & 0x400u));
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    return f32_from_bits(bits);
}

static inline float load_logit(const void *row, int dtype, int64_t i) {
    if (dtype == 0) return ((const float *)row)[i];
    if (dtype == 1) return bf16_to_f32(((const uint16_t *)row)[i]);
    return f16_to_f32(((const uint16_t *)row)[i]);
}

static inline size_t dtype_size(int dtype) { return dtype == 0 ? 4 : 2; }

static inline int bit_at(const int32_t *mask, int64_t t) {
    return (int)(((uint32_t)mask[t >> 5] >> (t & 31)) & 1u);
}

/* Widen one row to float32 (exact for all three dtypes). */
void orc_widen(const void *row, int dtype, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = load_logit(row, dtype, i);
}

int64_t orc_mask_count(const int32_t *mask, int64_t vocab) {
    int64_t words = (vocab + 31) / 32, count = 0;
    for (int64_t w = 0; w + 1 < words; ++w) count += __builtin_popcount((uint32_t)mask[w]);
    int tail = (int)(vocab % 32);
    uint32_t last = (uint32_t)mask[words - 1];
    if (tail) last &= (1u << tail) - 1u;
    return count + __builtin_popcount(last);
}

static void reduce_one(const void *row, int dtype, const int32_t *mask, int64_t vocab,
                       int64_t *token, int64_t *count, int32_t *status) {
    int nan = 0, have = 0;
    float best = 0.0f;
    int64_t best_index = -1, valid = 0;
    for (int64_t t = 0; t < vocab; ++t) {
        float v = load_logit(row, dtype, t);
        int allowed = bit_at(mask, t);
        valid += allowed;
        if (isnan(v)) {
            nan = 1;
            continue;
        }
        if (!allowed) continue;
        /* Strict '>' keeps the first (lowest) index among equal maxima;
           -0.0 and +0.0 compare equal, as torch's `logits == maximum` does. */
        if (!have || v > best) {
            best = v;
            best_index = t;
            have = 1;
        }
    }
    int code = nan ? 2 : (valid == 0 ? 1 : 0);
    *status = code;
    *token = code == 0 ? best_index : -1;
    if (count) *count = valid;
}

void orc_reduce_rows(const void *logits, int dtype, const int32_t *masks, int64_t rows,
                     int64_t vocab, int64_t *tokens, int64_t *counts, int32_t *status,
                     int threads) {
    int64_t words = (vocab + 31) / 32;
    size_t es = dtype_size(dtype);
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
    for (int64_t r = 0; r < rows; ++r) {
        reduce_one((const char *)logits + (size_t)r * (size_t)vocab * es, dtype,
                   masks + r * words, vocab, tokens + r, counts ? counts + r : NULL,
                   status + r);
    }
}

/* ---- exact summation (CPython math.fsum) ------------------------------- */
typedef struct {
    double *p;
    int n, cap;
} partials_t;

static void partials_add(partials_t *ps, double x) {
    int i = 0;
    for (int j = 0; j < ps->n; ++j) {
        double y = ps->p[j];
        if (fabs(x) < fabs(y)) {
            double t = x;
            x = y;
            y = t;
        }
        double hi = x + y;
        double lo = y - (hi - x);
        if (lo != 0.0) ps->p[i++] = lo;
        x = hi;
    }
    if (i >= ps->cap) {
        ps->cap = ps->cap ? ps->cap * 2 : 32;
        ps->p = (double *)realloc(ps->p, sizeof(double) * (size_t)ps->cap);
    }
    ps->p[i] = x;
    ps->n = i + 1;
}

static double partials_round(const partials_t *ps) {
    int n = ps->n;
    if (n == 0) return 0.0;
    double hi = ps->p[--n], lo = 0.0;
    while (n > 0) {
        double x = hi, y = ps->p[--n];
        hi = x + y;
        double yr = hi - x;
        lo = y - yr;
        if (lo != 0.0) break;
    }
    if (n > 0 && ((lo < 0.0 && ps->p[n - 1] < 0.0) || (lo > 0.0 && ps->p[n - 1] > 0.0))) {
        double y = lo * 2.0;
        double x = hi + y;
        double yr = x - hi;
        if (y == yr) hi = x;
    }
    return hi;
}

double orc_fsum(const double *values, int64_t n) {
    partials_t ps = {0, 0, 0};
    for (int64_t i = 0; i < n; ++i) partials_add(&ps, values[i]);
    double s = partials_round(&ps);
    free(ps.p);
    return s;
}

/* ---- sampler ------------------------------------------------------------ */
static void sample_one(const void *row, int dtype, const int32_t *mask, int64_t vocab,
                       double temperature, double uniform, int64_t *token, int32_t *status,
                       double *weights /* scratch of vocab doubles */) {
    if (temperature == 0.0) { /* csrc/sample.cu:120: zero temperature is argmax */
        reduce_one(row, dtype, mask, vocab, token, NULL, status);
        return;
    }
    int nan = 0, found = 0, posinf = 0;
    double maximum = -INFINITY;
    for (int64_t t = 0; t < vocab; ++t) {
        float v = load_logit(row, dtype, t);
        if (isnan(v)) {
            nan = 1;
            continue;
        }
        if (!bit_at(mask, t)) continue;
        found = 1;
        if (isinf(v) && v > 0) posinf = 1;
        if ((double)v > maximum) maximum = v;
    }
    int code = nan ? 2 : posinf ? 5 : !found ? 1 : !isfinite(maximum) ? 4 : 0;
    if (!code && !(uniform >= 0.0 && uniform < 1.0)) code = 3;
    *status = code;
    *token = -1;
    if (code) return;
    int64_t k = 0;
    for (int64_t t = 0; t < vocab; ++t) {
        if (!bit_at(mask, t)) continue;
        double v = load_logit(row, dtype, t);
        weights[k++] = exp((v - maximum) / temperature);
    }
    double cutoff = uniform * orc_fsum(weights, k);
    double cumulative = 0.0;
    int64_t last_positive = -1;
    k = 0;
    for (int64_t t = 0; t < vocab; ++t) {
        if (!bit_at(mask, t)) continue;
        double w = weights[k++];
        if (w == 0.0) continue;
        last_positive = t;
        cumulative += w;
        if (cutoff < cumulative) {
            *token = t;
            return;
        }
    }
    *token = last_positive;
}

void orc_sample_rows(const void *logits, int dtype, const int32_t *masks, int64_t rows,
                     int64_t vocab, double temperature, const double *uniforms,
                     int64_t *tokens, int32_t *status, int threads) {
    int64_t words = (vocab + 31) / 32;
    size_t es = dtype_size(dtype);
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        double *weights = (double *)malloc(sizeof(double) * (size_t)vocab);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            sample_one((const char *)logits + (size_t)r * (size_t)vocab * es, dtype,
                       masks + r * words, vocab, temperature, uniforms[r], tokens + r,
                       status + r, weights);
        }
        free(weights);
    }
}

/* ---- draft budget policy ------------------------------------------------ */
/* kind 0: DensityPolicy three bands; kind 1: linear between low and high. */
int32_t orc_budget(int32_t kind, double low, double high, int32_t min_budget,
                   int32_t max_budget, double density) {
    if (kind == 0) {
        if (density < low) return max_budget;
        if (density < high) return (min_budget + max_budget) / 2;
        return min_budget;
    }
    if (density < low) return max_budget;
    if (density > high) return min_budget;
    double span = (double)(max_budget - min_budget);
    double frac = (density - low) / (high - low);
    return max_budget - (int32_t)floor(span * frac);
}

void orc_budget_rows(int32_t kind, double low, double high, int32_t min_budget,
                     int32_t max_budget, const int64_t *counts, int64_t rows, int64_t vocab,
                     double *density, int32_t *budget) {
    for (int64_t r = 0; r < rows; ++r) {
        double d = (double)counts[r] / (double)vocab;
        if (density) density[r] = d;
        budget[r] = orc_budget(kind, low, high, min_budget, max_budget, d);
    }
}

/* ---- verification ------------------------------------------------------- */
/* kind: 0 correction, 1 bonus, 2 fallback; seq_status is the status of the
   first consumed row that failed (then token = -1), else 0. */
void orc_verify(const int64_t *row_tokens, const int32_t *row_status, int64_t seqs,
                int64_t rows_per_seq, const int64_t *proposals, const int32_t *lengths,
                int32_t *accept_len, int64_t *token, int32_t *kind, int32_t *seq_status) {
    int64_t k_max = rows_per_seq - 1;
    for (int64_t s = 0; s < seqs; ++s) {
        const int64_t *tok = row_tokens + s * rows_per_seq;
        const int32_t *st = row_status + s * rows_per_seq;
        const int64_t *prop = proposals + s * k_max;
        int32_t len = lengths[s];
        int32_t i = 0;
        accept_len[s] = 0;
        token[s] = -1;
        kind[s] = 0;
        seq_status[s] = 0;
        if (len < 0 || len > k_max) {
            seq_status[s] = 6;
            continue;
        }
        for (;; ++i) {
            if (st[i] != 0) {
                accept_len[s] = i;
                seq_status[s] = st[i];
                break;
            }
            if (i == len) {
                accept_len[s] = len;
                token[s] = tok[i];
                kind[s] = len > 0 ? 1 : 2;
                break;
            }
            if (tok[i] != prop[i]) {
                accept_len[s] = i;
                token[s] = tok[i];
                kind[s] = 0;
                break;
            }
        }
    }
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
