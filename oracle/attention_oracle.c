/*
 * CPU oracle for the FP32 attention path. TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load it. The CUDA library does not link it and has
 * no CPU fallback.
 *
 * It restates, in plain C, the reference's CPU attention `ReferenceAttention`
 * (ROCmKernels.Tests/AttentionTests.cpp:28-125): forward and backward in double precision with
 * FP32 storage, the same loop order, the same guards and the same float accumulation of the
 * gradients, so that a build with the same compiler produces bit-identical results. The
 * restatement is pinned bit-for-bit against the reference's own function, compiled from the
 * reference tree (oracle/Makefile, target `ref`), and against the committed golden vectors in
 * tests/golden/.
 *
 * It also restates the reference's CPU rotary embedding `ReferenceRotary`
 * (ROCmKernels.Tests/PositionalTests.cpp:18-50), pinned bit-for-bit the same way.
 *
 * It also restates the reference's input generator (ROCmKernels.Tests/TestSupport.hpp:11-21:
 * std::mt19937 + std::uniform_real_distribution<float>) and the libstdc++ normal distribution
 * used for the synthetic benchmark inputs, so Python code can reproduce the reference's inputs.
 *
 * Build flags: -O2 -ffp-contract=off, generic x86-64 (no FMA), matching how the reference's
 * test is compiled by g++ so that no product is contracted.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------ */
/* MT19937 (Matsumoto & Nishimura 1998), the engine behind std::mt19937.                       */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    uint32_t state[624];
    int index;
} oracle_mt19937;

static void mt_seed(oracle_mt19937 *engine, uint32_t seed) {
    engine->state[0] = seed;
    for (int i = 1; i < 624; ++i) {
        const uint32_t previous = engine->state[i - 1];
        engine->state[i] = 1812433253u * (previous ^ (previous >> 30)) + (uint32_t)i;
    }
    engine->index = 624;
}

static void mt_twist(oracle_mt19937 *engine) {
    for (int i = 0; i < 624; ++i) {
        const uint32_t y = (engine->state[i] & 0x80000000u) | (engine->state[(i + 1) % 624] & 0x7fffffffu);
        uint32_t next = engine->state[(i + 397) % 624] ^ (y >> 1);
        if (y & 1u) next ^= 0x9908b0dfu;
        engine->state[i] = next;
    }
    engine->index = 0;
}

static uint32_t mt_next(oracle_mt19937 *engine) {
    if (engine->index >= 624) mt_twist(engine);
    uint32_t y = engine->state[engine->index++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* libstdc++ generate_canonical<float, 24> over a 32-bit engine: one draw, converted to float
 * (round to nearest), scaled by 2^-32, clamped below 1. */
static float canonical_float(oracle_mt19937 *engine) {
    const float sum = (float)mt_next(engine);
    float value = sum / 4294967296.0f;
    if (value >= 1.0f) value = nextafterf(1.0f, 0.0f);
    return value;
}

/* std::uniform_real_distribution<float>(low, high) as libstdc++ evaluates it. */
void oracle_uniform_fill(float *out, size_t count, uint32_t seed, float low, float high) {
    oracle_mt19937 engine;
    mt_seed(&engine, seed);
    for (size_t i = 0; i < count; ++i) out[i] = canonical_float(&engine) * (high - low) + low;
}

/* std::normal_distribution<float>(mean, stddev) as libstdc++ evaluates it (Marsaglia polar
 * method; the second variate of each pair is cached and returned on the next call). */
void oracle_normal_fill(float *out, size_t count, uint32_t seed, float mean, float stddev) {
    oracle_mt19937 engine;
    mt_seed(&engine, seed);
    int saved_available = 0;
    float saved = 0.0f;
    for (size_t i = 0; i < count; ++i) {
        float value;
        if (saved_available) {
            saved_available = 0;
            value = saved;
        } else {
            float x, y, r2;
            do {
                x = (float)((double)(2.0f * canonical_float(&engine)) - 1.0);
                y = (float)((double)(2.0f * canonical_float(&engine)) - 1.0);
                r2 = x * x + y * y;
            } while (r2 > 1.0 || r2 == 0.0);
            const float mult = sqrtf(-2 * logf(r2) / r2);
            saved = x * mult;
            saved_available = 1;
            value = y * mult;
        }
        out[i] = value * stddev + mean;
    }
}

/* Raw engine output, for pinning against std::mt19937's published 10000th value. */
void oracle_mt19937_raw(uint32_t *out, size_t count, uint32_t seed) {
    oracle_mt19937 engine;
    mt_seed(&engine, seed);
    for (size_t i = 0; i < count; ++i) out[i] = mt_next(&engine);
}

/* Valid key lengths for the padded benchmark configurations: low + (draw mod span), one draw
 * per sequence from MT19937(seed). This is this build's own convention (the reference has no
 * length generator). */
void oracle_lengths(int32_t *out, int count, uint32_t seed, int32_t low, int32_t high) {
    oracle_mt19937 engine;
    mt_seed(&engine, seed);
    const uint32_t span = (uint32_t)(high - low + 1);
    for (int i = 0; i < count; ++i) out[i] = low + (int32_t)(mt_next(&engine) % span);
}

/* ------------------------------------------------------------------------------------------ */
/* Reference attention (ROCmKernels.Tests/AttentionTests.cpp:28-125).                          */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    const float *q, *k, *v, *upstream;
    const uint8_t *mask;
    int head_width, batch, heads, queries, keys, radius;
    int forward_only;
    int double_gradients;
    float *output, *lse, *grad_q, *grad_k, *grad_v;
    int slice_begin, slice_end; /* (batch, head) slices [begin, end) */
    int next_slice;             /* work counter shared by the threads */
    pthread_mutex_t lock;
} oracle_job;

/* One (batch, head) slice. The loop body follows AttentionTests.cpp:47-119 statement by
 * statement; only the slice loop around it is reorganised so that slices can run on threads
 * (slices never write the same element, so the result is identical to the serial loop). */
static void oracle_slice(const oracle_job *job, int slice, double *scores, double *probabilities,
                         double *gq, double *gk, double *gv) {
    const int D = job->head_width, H = job->heads, Q = job->queries, K = job->keys;
    const int batch = slice / H, head = slice % H;
    const double scale = 1.0 / sqrt((double)D); /* :33 */
    const size_t kSlice = ((size_t)batch * H + head) * (size_t)K * D;
    if (job->double_gradients) {
        memset(gk, 0, sizeof(double) * (size_t)K * D);
        memset(gv, 0, sizeof(double) * (size_t)K * D);
    }

    for (int query = 0; query < Q; ++query) {
        const size_t qBase = ((size_t)batch * H + head) * (size_t)Q * D + (size_t)query * D; /* :48-49 */

        double maximum = -INFINITY; /* :51-69 */
        for (int key = 0; key < K; ++key) {
            scores[key] = -INFINITY;
            if (!job->mask[(size_t)batch * K + key]) continue;
            if (job->radius >= 0 && abs(query - key) > job->radius) continue;
            const size_t kBase = kSlice + (size_t)key * D;
            double dot = 0;
            for (int column = 0; column < D; ++column) dot += (double)job->q[qBase + column] * job->k[kBase + column];
            scores[key] = dot * scale;
            maximum = (maximum < scores[key]) ? scores[key] : maximum; /* std::max(maximum, s) */
        }

        double total = 0; /* :71-75 */
        for (int key = 0; key < K; ++key) {
            probabilities[key] = maximum == -INFINITY ? 0.0 : exp(scores[key] - maximum);
            total += probabilities[key];
        }

        const size_t row = ((size_t)batch * H + head) * Q + query; /* :77-79 */
        job->lse[row * 2] = maximum == -INFINITY ? -INFINITY : (float)maximum;
        job->lse[row * 2 + 1] = (float)total;

        for (int column = 0; column < D; ++column) { /* :81-92 */
            double value = 0;
            for (int key = 0; key < K; ++key) {
                if (probabilities[key] == 0.0) continue;
                const size_t vBase = kSlice + (size_t)key * D;
                value += probabilities[key] * job->v[vBase + column];
            }
            job->output[qBase + column] = (float)(total > 0 ? value / total : 0.0);
        }
        if (job->forward_only) continue;

        double delta = 0; /* :94-97 */
        for (int column = 0; column < D; ++column) delta += (double)job->upstream[qBase + column] * job->output[qBase + column];

        if (job->double_gradients) memset(gq, 0, sizeof(double) * (size_t)D);
        for (int key = 0; key < K; ++key) { /* :99-119 */
            if (probabilities[key] == 0.0) continue;
            const size_t kBase = kSlice + (size_t)key * D;
            const double probability = probabilities[key] / total;
            double valueScore = 0;
            for (int column = 0; column < D; ++column) valueScore += (double)job->upstream[qBase + column] * job->v[kBase + column];
            const double derivative = probability * (valueScore - delta);
            if (job->double_gradients) {
                /* Diagnostic variant: the same sums accumulated in double, to bound the
                 * oracle's own float-accumulation noise. */
                for (int column = 0; column < D; ++column) {
                    gq[column] += derivative * job->k[kBase + column] * scale;
                    gk[(size_t)key * D + column] += derivative * job->q[qBase + column] * scale;
                    gv[(size_t)key * D + column] += probability * job->upstream[qBase + column];
                }
            } else {
                for (int column = 0; column < D; ++column) {
                    job->grad_q[qBase + column] += (float)(derivative * job->k[kBase + column] * scale);
                    job->grad_k[kBase + column] += (float)(derivative * job->q[qBase + column] * scale);
                    job->grad_v[kBase + column] += (float)(probability * job->upstream[qBase + column]);
                }
            }
        }
        if (job->double_gradients)
            for (int column = 0; column < D; ++column) job->grad_q[qBase + column] = (float)gq[column];
    }
    if (job->double_gradients && !job->forward_only) {
        for (size_t i = 0; i < (size_t)K * D; ++i) {
            job->grad_k[kSlice + i] = (float)gk[i];
            job->grad_v[kSlice + i] = (float)gv[i];
        }
    }
}

static void *oracle_worker(void *argument) {
    oracle_job *job = (oracle_job *)argument;
    const size_t K = (size_t)job->keys, D = (size_t)job->head_width;
    double *scores = (double *)malloc(sizeof(double) * K);
    double *probabilities = (double *)malloc(sizeof(double) * K);
    double *gq = NULL, *gk = NULL, *gv = NULL;
    if (job->double_gradients) {
        gq = (double *)malloc(sizeof(double) * D);
        gk = (double *)malloc(sizeof(double) * K * D);
        gv = (double *)malloc(sizeof(double) * K * D);
    }
    for (;;) {
        pthread_mutex_lock(&job->lock);
        const int slice = job->next_slice++;
        pthread_mutex_unlock(&job->lock);
        if (slice >= job->slice_end) break;
        oracle_slice(job, slice, scores, probabilities, gq, gk, gv);
    }
    free(scores);
    free(probabilities);
    free(gq);
    free(gk);
    free(gv);
    return NULL;
}

/*
 * Runs the reference attention over the (batch, head) slices [slice_begin, slice_end) of a
 * contiguous [batch][heads][tokens][head_width] problem. Output, lse and gradient elements of
 * the processed slices are zeroed first, as the reference's `assign(..., 0.0f)` does (:36-40);
 * elements of other slices are left untouched. `threads` <= 1 runs serially.
 * Returns 0, or -1 for invalid arguments.
 */
int oracle_attention_slices(const float *q, const float *k, const float *v, const uint8_t *mask, const float *upstream,
                            int head_width, int batch, int heads, int queries, int keys, int radius, float *output,
                            float *lse, float *grad_q, float *grad_k, float *grad_v, int slice_begin, int slice_end,
                            int threads, int forward_only, int double_gradients) {
    if (!q || !k || !v || !mask || !output || !lse || head_width <= 0 || batch <= 0 || heads <= 0 || queries <= 0 ||
        keys <= 0)
        return -1;
    if (!forward_only && (!upstream || !grad_q || !grad_k || !grad_v)) return -1;
    if (slice_begin < 0 || slice_end > batch * heads || slice_begin > slice_end) return -1;
    const size_t qSlice = (size_t)queries * head_width, kSlice = (size_t)keys * head_width;
    for (int s = slice_begin; s < slice_end; ++s) {
        memset(output + (size_t)s * qSlice, 0, sizeof(float) * qSlice);
        memset(lse + (size_t)s * queries * 2, 0, sizeof(float) * (size_t)queries * 2);
        if (!forward_only) {
            memset(grad_q + (size_t)s * qSlice, 0, sizeof(float) * qSlice);
            memset(grad_k + (size_t)s * kSlice, 0, sizeof(float) * kSlice);
            memset(grad_v + (size_t)s * kSlice, 0, sizeof(float) * kSlice);
        }
    }
    oracle_job job = {q, k, v, upstream, mask, head_width, batch, heads, queries, keys, radius,
                      forward_only, double_gradients, output, lse, grad_q, grad_k, grad_v,
                      slice_begin, slice_end, slice_begin, PTHREAD_MUTEX_INITIALIZER};
    if (threads <= 1) {
        oracle_worker(&job);
    } else {
        pthread_t *pool = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
        for (int t = 0; t < threads; ++t) pthread_create(&pool[t], NULL, oracle_worker, &job);
        for (int t = 0; t < threads; ++t) pthread_join(pool[t], NULL);
        free(pool);
    }
    pthread_mutex_destroy(&job.lock);
    return 0;
}

/* The whole problem, as ReferenceAttention(q, k, v, mask, upstream, D, B, H, Q, K, radius). */
int oracle_attention(const float *q, const float *k, const float *v, const uint8_t *mask, const float *upstream,
                     int head_width, int batch, int heads, int queries, int keys, int radius, float *output, float *lse,
                     float *grad_q, float *grad_k, float *grad_v, int threads) {
    return oracle_attention_slices(q, k, v, mask, upstream, head_width, batch, heads, queries, keys, radius, output, lse,
                                   grad_q, grad_k, grad_v, 0, batch * heads, threads, 0, 0);
}

/* ------------------------------------------------------------------------------------------ */
/* Reference rotary embedding (ROCmKernels.Tests/PositionalTests.cpp:18-50), 32-wide heads.     */
/* ------------------------------------------------------------------------------------------ */

/*
 * input/output: token-major [batch][length][heads][32]; cosine/sine: [batch][length][32].
 * Each head's low half (columns 0-15) and high half (16-31) rotate as pairs (column c with
 * c + 16): forward lo' = lo*cos_lo - hi*sin_lo, hi' = hi*cos_hi + lo*sin_hi (:42-44); backward
 * (the transposed rotation) lo' = lo*cos_lo + hi*sin_hi, hi' = hi*cos_hi - lo*sin_lo (:39-41).
 */
void oracle_rotary(const float *input, const float *cosine, const float *sine, float *output, int batch, int heads,
                   int length, int backward) {
    enum { kHeadWidth = 32 };
    for (int b = 0; b < batch; ++b) {
        for (int token = 0; token < length; ++token) {
            const size_t bufferBase = ((size_t)b * length + token) * kHeadWidth; /* :24 */
            for (int head = 0; head < heads; ++head) {
                const size_t base = ((size_t)b * length + token) * heads * kHeadWidth + (size_t)head * kHeadWidth;
                for (int column = 0; column < kHeadWidth / 2; ++column) { /* :31-46 */
                    const float low = input[base + column];
                    const float high = input[base + column + 16];
                    const float cosineLow = cosine[bufferBase + column];
                    const float cosineHigh = cosine[bufferBase + column + 16];
                    const float sineLow = sine[bufferBase + column];
                    const float sineHigh = sine[bufferBase + column + 16];
                    if (backward) {
                        output[base + column] = low * cosineLow + high * sineHigh;
                        output[base + column + 16] = high * cosineHigh - low * sineLow;
                    } else {
                        output[base + column] = low * cosineLow - high * sineLow;
                        output[base + column + 16] = high * cosineHigh + low * sineHigh;
                    }
                }
            }
        }
    }
}
