/*
 * Seeded synthetic inputs for the benchmark and tests (host code, no GPU).
 *
 * Generator: PCG32 (O'Neill 2014, "PCG: A Family of Simple Fast
 * Space-Efficient Statistically Good Algorithms for Random Number
 * Generation", XSH-RR 64/32 output, LCG multiplier 6364136223846793005),
 * seeded like pcg32_srandom(seed, stream).  Bounded integers use Lemire's
 * nearly-divisionless method (Lemire 2019); normals use fp64 Box-Muller.
 *
 * Determinism under threading: the output is cut into fixed chunks of
 * 2^20 elements; chunk c draws from the (seed, stream) sequence advanced by
 * c * 2^40 steps (Brown 1994 LCG jump-ahead), so the result does not depend on
 * the number of threads.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef struct { uint64_t state, inc; } pcg32_t;

#define PCG_MULT 6364136223846793005ULL
#define CHUNK (1ull << 20)
#define CHUNK_STRIDE_LOG2 40

static inline uint32_t pcg32_next(pcg32_t* r) {
    const uint64_t old = r->state;
    r->state = old * PCG_MULT + r->inc;
    const uint32_t xs = (uint32_t)(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = (uint32_t)(old >> 59u);
    return (xs >> rot) | (xs << ((-rot) & 31u));
}

static void pcg32_seed(pcg32_t* r, uint64_t seed, uint64_t stream) {
    r->state = 0;
    r->inc = (stream << 1u) | 1u;
    pcg32_next(r);
    r->state += seed;
    pcg32_next(r);
}

/* Advance the LCG by delta steps in O(log delta). */
static void pcg32_advance(pcg32_t* r, uint64_t delta) {
    uint64_t cur_mult = PCG_MULT, cur_plus = r->inc, acc_mult = 1, acc_plus = 0;
    while (delta) {
        if (delta & 1) {
            acc_mult *= cur_mult;
            acc_plus = acc_plus * cur_mult + cur_plus;
        }
        cur_plus = (cur_mult + 1) * cur_plus;
        cur_mult *= cur_mult;
        delta >>= 1;
    }
    r->state = acc_mult * r->state + acc_plus;
}

/* Lemire's bounded draw in [0, bound), bound >= 1. */
static inline uint32_t pcg32_bounded(pcg32_t* r, uint32_t bound) {
    uint64_t m = (uint64_t)pcg32_next(r) * bound;
    uint32_t l = (uint32_t)m;
    if (l < bound) {
        const uint32_t t = (uint32_t)(-bound) % bound;
        while (l < t) {
            m = (uint64_t)pcg32_next(r) * bound;
            l = (uint32_t)m;
        }
    }
    return (uint32_t)(m >> 32);
}

static inline double pcg32_unit53(pcg32_t* r) { /* uniform in (0,1) */
    const uint64_t a = pcg32_next(r) >> 5, b = pcg32_next(r) >> 6;
    return ((double)(a * 67108864.0 + b) + 0.5) / 9007199254740992.0;
}

typedef enum {
    GEN_U32 = 0,        /* raw 32-bit                               */
    GEN_I32_RANGE = 1,  /* lo + bounded(hi - lo + 1), int32           */
    GEN_U32_BOUND = 2,  /* bounded(bound), uint32                     */
    GEN_F32_NORMAL = 3, /* N(0,1) in fp64, rounded to f32             */
    GEN_F32_UNIT = 4,   /* U[0,1) with 24-bit resolution              */
    GEN_U64 = 5,        /* raw 64-bit (hi draw << 32 | lo draw)       */
    GEN_U32_MASK = 6    /* raw 32-bit & mask                          */
} gen_kind;

typedef struct {
    int kind;
    void* out;
    uint64_t n;
    uint64_t seed, stream;
    int64_t a, b; /* kind parameters */
    uint64_t next_chunk;
    pthread_mutex_t mu;
} gen_job;

static void gen_chunk(gen_job* j, uint64_t c) {
    pcg32_t r;
    pcg32_seed(&r, j->seed, j->stream);
    pcg32_advance(&r, c << CHUNK_STRIDE_LOG2);
    const uint64_t b = c * CHUNK;
    const uint64_t e = b + CHUNK < j->n ? b + CHUNK : j->n;
    switch (j->kind) {
        case GEN_U32: {
            uint32_t* o = (uint32_t*)j->out;
            for (uint64_t i = b; i < e; ++i) o[i] = pcg32_next(&r);
        } break;
        case GEN_U32_MASK: {
            uint32_t* o = (uint32_t*)j->out;
            const uint32_t m = (uint32_t)j->a;
            for (uint64_t i = b; i < e; ++i) o[i] = pcg32_next(&r) & m;
        } break;
        case GEN_I32_RANGE: {
            int32_t* o = (int32_t*)j->out;
            const uint32_t span = (uint32_t)(j->b - j->a + 1);
            for (uint64_t i = b; i < e; ++i) o[i] = (int32_t)(j->a + (int64_t)pcg32_bounded(&r, span));
        } break;
        case GEN_U32_BOUND: {
            uint32_t* o = (uint32_t*)j->out;
            for (uint64_t i = b; i < e; ++i) o[i] = pcg32_bounded(&r, (uint32_t)j->a);
        } break;
        case GEN_F32_NORMAL: {
            float* o = (float*)j->out;
            for (uint64_t i = b; i < e; i += 2) {
                const double u1 = pcg32_unit53(&r), u2 = pcg32_unit53(&r);
                const double rad = sqrt(-2.0 * log(u1));
                o[i] = (float)(rad * cos(6.283185307179586 * u2));
                if (i + 1 < e) o[i + 1] = (float)(rad * sin(6.283185307179586 * u2));
            }
        } break;
        case GEN_F32_UNIT: {
            float* o = (float*)j->out;
            for (uint64_t i = b; i < e; ++i) o[i] = (float)(pcg32_next(&r) >> 8) * (1.0f / 16777216.0f);
        } break;
        case GEN_U64: {
            uint64_t* o = (uint64_t*)j->out;
            for (uint64_t i = b; i < e; ++i) {
                const uint64_t hi = pcg32_next(&r);
                o[i] = (hi << 32) | pcg32_next(&r);
            }
        } break;
    }
}

static void* gen_worker(void* p) {
    gen_job* j = (gen_job*)p;
    const uint64_t chunks = (j->n + CHUNK - 1) / CHUNK;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        const uint64_t c = j->next_chunk++;
        pthread_mutex_unlock(&j->mu);
        if (c >= chunks) break;
        gen_chunk(j, c);
    }
    return NULL;
}

/* Fill out[0..n) with distribution `kind` (see gen_kind); a, b are the
 * kind's parameters (range lo/hi, bound, mask).  threads <= 0: all cores. */
int pcg_fill(int kind, void* out, uint64_t n, uint64_t seed, uint64_t stream, int64_t a, int64_t b,
             int threads) {
    if (kind < 0 || kind > 6 || (!out && n)) return -1;
    gen_job j;
    memset(&j, 0, sizeof(j));
    j.kind = kind; j.out = out; j.n = n; j.seed = seed; j.stream = stream; j.a = a; j.b = b;
    pthread_mutex_init(&j.mu, NULL);
    if (threads <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        threads = c > 0 ? (int)c : 1;
    }
    if (threads > 256) threads = 256;
    const uint64_t chunks = (n + CHUNK - 1) / CHUNK;
    if ((uint64_t)threads > chunks) threads = (int)(chunks ? chunks : 1);
    pthread_t tid[256];
    for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, gen_worker, &j);
    gen_worker(&j);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
    pthread_mutex_destroy(&j.mu);
    return 0;
}

/* out[i] = start + i */
void fill_iota_u32(uint32_t* out, uint64_t n, uint32_t start) {
    for (uint64_t i = 0; i < n; ++i) out[i] = start + (uint32_t)i;
}

/* CSR offsets[S+1] for S segments covering exactly N items: raw lengths
 * round(exp(mu + sigma*z)), z ~ N(0,1), forced to 0 with probability
 * p_empty, then scaled so that they sum to N (floor of the scaled length;
 * leftover items go to the last non-empty segments).  Sequential. */
int pcg_segments_lognormal(uint32_t* offsets, uint64_t S, uint64_t N, double mu, double sigma,
                           double p_empty, uint64_t seed, uint64_t stream) {
    if (!offsets || S == 0) return -1;
    double* raw = (double*)malloc(S * sizeof(double));
    if (!raw) return -1;
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    double total = 0.0;
    for (uint64_t s = 0; s < S; ++s) {
        const double u1 = pcg32_unit53(&r), u2 = pcg32_unit53(&r);
        const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        const int empty = pcg32_unit53(&r) < p_empty;
        raw[s] = empty ? 0.0 : floor(exp(mu + sigma * z) + 0.5);
        total += raw[s];
    }
    const double scale = total > 0 ? (double)N / total : 0.0;
    uint64_t acc = 0;
    for (uint64_t s = 0; s < S; ++s) {
        raw[s] = raw[s] > 0 ? floor(raw[s] * scale) + 0.25 : 0.0; /* +0.25 marks non-empty */
        acc += (uint64_t)raw[s];
    }
    /* hand the remainder out one item at a time from the last segment back */
    uint64_t left = N > acc ? N - acc : 0;
    int any = total > 0;
    for (int64_t s = (int64_t)S - 1; left; s = s == 0 ? (int64_t)S - 1 : s - 1) {
        if (raw[s] > 0 || !any) { raw[s] += 1.0; left--; }
    }
    acc = 0;
    offsets[0] = 0;
    for (uint64_t s = 0; s < S; ++s) {
        acc += (uint64_t)raw[s];
        offsets[s + 1] = (uint32_t)acc;
    }
    free(raw);
    return 0;
}
