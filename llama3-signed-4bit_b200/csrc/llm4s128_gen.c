/*
 * Seeded writer for the LLM4S128 block-128 4-bit weight file.
 *
 * The reference ships no quantiser or converter (its weight file is downloaded), so this file
 * provides the producer side of the format read by LlamaEngineState::load
 * (src/llama_engine.cpp:865-906) and SignedBlock128Matrix::map_from_buffer
 * (src/llama_engine.cpp:164-180):
 *
 *   "LLM4S128" | u32 layers, dim, ffn, vocab, heads, kv_heads, block(=128)
 *   f32 final_norm[dim]
 *   per layer: f32 in_norm[dim], f32 post_norm[dim], then Wq, Wk, Wv, Wo, Wgate, Wup, Wdown
 *   lm_head (tied with the token embedding)
 *   matrix = u32 out_dim, in_dim, num_blocks | u8 nibbles[num_blocks*64]
 *            | u16 step[num_blocks] | u16 min[num_blocks]      (step/min are bf16 bit patterns)
 *
 * A block is 128 consecutive weights of one row; row n owns blocks n*K/128 .. n*K/128+K/128-1.
 * Byte j of a block holds weight 2j in its low nibble and weight 2j+1 in its high nibble
 * (src/llama_engine.cpp:213-216).  A weight decodes as  min + q*step  with q in 0..15.
 *
 * Quantiser (affine, per block): min = block minimum, step = (max-min)/15, both rounded to
 * bf16 (round-to-nearest-even); q = clamp(rint((w - min_bf16)/step_bf16), 0, 15).
 *
 * Randomness is counter-based: every (seed, tensor, row) pair seeds its own xoshiro256**
 * stream through splitmix64, so the output does not depend on the thread count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef struct { uint64_t s[4]; } rng_t;

static uint64_t splitmix64(uint64_t* x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static void rng_seed(rng_t* r, uint64_t seed, uint64_t tensor, uint64_t row) {
    uint64_t x = seed * 0x100000001B3ull ^ (tensor << 40) ^ row ^ 0x5851F42D4C957F2Dull;
    for (int i = 0; i < 4; ++i) r->s[i] = splitmix64(&x);
}

static inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

static inline uint64_t rng_next(rng_t* r) {
    uint64_t* s = r->s;
    uint64_t result = rotl(s[1] * 5, 7) * 9;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0]; s[3] ^= s[1]; s[1] ^= s[2]; s[0] ^= s[3];
    s[2] ^= t; s[3] = rotl(s[3], 45);
    return result;
}

/* uniform double in [0,1) with 53 random bits */
static inline double rng_uniform(rng_t* r) { return (double)(rng_next(r) >> 11) * 0x1.0p-53; }

/* standard normal, Box-Muller in double precision; returns one value, caches the pair */
typedef struct { rng_t r; int have; double spare; } nrng_t;
static inline double rng_normal(nrng_t* g) {
    if (g->have) { g->have = 0; return g->spare; }
    double u1 = rng_uniform(&g->r), u2 = rng_uniform(&g->r);
    if (u1 < 1e-300) u1 = 1e-300;
    double rad = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
    g->spare = rad * sin(th); g->have = 1;
    return rad * cos(th);
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16); /* inf/nan pass through */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f;
}

/* Quantise one row of K fp32 weights (K % 128 == 0) into nibbles/step/min. */
static void quantise_row(const float* w, int K, uint8_t* nib, uint16_t* step, uint16_t* mn) {
    for (int b = 0; b < K / 128; ++b) {
        const float* wb = w + (size_t)b * 128;
        float lo = wb[0], hi = wb[0];
        for (int i = 1; i < 128; ++i) { if (wb[i] < lo) lo = wb[i]; if (wb[i] > hi) hi = wb[i]; }
        uint16_t sb = f32_to_bf16_rne((hi - lo) / 15.0f);
        uint16_t mb = f32_to_bf16_rne(lo);
        float s = bf16_to_f32(sb), m = bf16_to_f32(mb);
        for (int j = 0; j < 64; ++j) {
            int q[2];
            for (int h = 0; h < 2; ++h) {
                int v = 0;
                if (s > 0.0f) {
                    v = (int)rintf((wb[2 * j + h] - m) / s);
                    if (v < 0) v = 0;
                    if (v > 15) v = 15;
                }
                q[h] = v;
            }
            nib[(size_t)b * 64 + j] = (uint8_t)(q[0] | (q[1] << 4));
        }
        step[b] = sb;
        mn[b] = mb;
    }
}

/* Weight distributions */
enum { DIST_NORMAL = 0, DIST_UNIFORM_CODES = 1, DIST_SOURCE = 2 };

typedef struct {
    int dist;          /* DIST_NORMAL: w ~ N(0, sigma) then quantised; DIST_UNIFORM_CODES: see below;
                          DIST_SOURCE: rows of src quantised */
    const float* src;  /* DIST_SOURCE: N x K row-major weights */
    double sigma;
    uint64_t seed, tensor;
    int N, K;
    uint8_t* nib;      /* N*K/2 */
    uint16_t* step;    /* N*K/128 */
    uint16_t* mn;      /* N*K/128 */
    int row_begin, row_end;
} mat_job_t;

/* DIST_UNIFORM_CODES: nibbles uniform 0..15, step ~ U(1e-3, 2e-2), min = -8*step*U(0.8, 1.2). */
static void* mat_worker(void* arg) {
    mat_job_t* j = (mat_job_t*)arg;
    int nb = j->K / 128;
    float* w = (float*)malloc(sizeof(float) * (size_t)j->K);
    for (int n = j->row_begin; n < j->row_end; ++n) {
        nrng_t g; rng_seed(&g.r, j->seed, j->tensor, (uint64_t)n); g.have = 0;
        uint8_t* nib = j->nib + (size_t)n * (j->K / 2);
        uint16_t* st = j->step + (size_t)n * nb;
        uint16_t* mn = j->mn + (size_t)n * nb;
        if (j->dist == DIST_SOURCE) {
            quantise_row(j->src + (size_t)n * j->K, j->K, nib, st, mn);
        } else if (j->dist == DIST_NORMAL) {
            for (int k = 0; k < j->K; ++k) w[k] = (float)(rng_normal(&g) * j->sigma);
            quantise_row(w, j->K, nib, st, mn);
        } else {
            for (int b = 0; b < nb; ++b) {
                for (int i = 0; i < 64; i += 8) {
                    uint64_t r = rng_next(&g.r);
                    memcpy(nib + (size_t)b * 64 + i, &r, 8);
                }
                float s = (float)(1e-3 + (2e-2 - 1e-3) * rng_uniform(&g.r));
                uint16_t sb = f32_to_bf16_rne(s);
                float m = -8.0f * bf16_to_f32(sb) * (float)(0.8 + 0.4 * rng_uniform(&g.r));
                st[b] = sb;
                mn[b] = f32_to_bf16_rne(m);
            }
        }
    }
    free(w);
    return NULL;
}

static int n_threads_default(void) {
    const char* e = getenv("LLM4S128_GEN_THREADS");
    if (e && atoi(e) > 0) return atoi(e);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    return (int)n;
}

static void gen_matrix_src(int dist, const float* src, double sigma, uint64_t seed, uint64_t tensor, int N,
                           int K, uint8_t* nib, uint16_t* step, uint16_t* mn, int threads) {
    if (threads <= 0) threads = n_threads_default();
    if (threads > N) threads = N > 0 ? N : 1;
    pthread_t tid[64];
    mat_job_t jobs[64];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (mat_job_t){dist, src, sigma, seed, tensor, N, K, nib, step, mn,
                              (int)((int64_t)N * t / threads), (int)((int64_t)N * (t + 1) / threads)};
        pthread_create(&tid[t], NULL, mat_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
}

static void gen_matrix(int dist, double sigma, uint64_t seed, uint64_t tensor, int N, int K,
                       uint8_t* nib, uint16_t* step, uint16_t* mn, int threads) {
    gen_matrix_src(dist, NULL, sigma, seed, tensor, N, K, nib, step, mn, threads);
}

/* ---------------------------------------------------------------------------------------- */
/* Public C interface                                                                        */
/* ---------------------------------------------------------------------------------------- */

/* One quantised matrix with the block-128 layout; dist = 0 (normal, sigma) or 1 (uniform codes). */
int llm4s128_gen_matrix(int dist, double sigma, uint64_t seed, uint64_t tensor, int N, int K,
                        uint8_t* nib, uint16_t* step, uint16_t* mn) {
    if (N <= 0 || K <= 0 || K % 128 != 0 || !nib || !step || !mn) return -1;
    gen_matrix(dist, sigma, seed, tensor, N, K, nib, step, mn, 0);
    return 0;
}

/* Quantises an N x K row-major fp32 matrix (K % 128 == 0) with the affine block rule above,
 * rows spread over threads (the output does not depend on the thread count). */
int llm4s128_quantize(const float* w, int N, int K, uint8_t* nib, uint16_t* step, uint16_t* mn) {
    if (!w || N <= 0 || K <= 0 || K % 128 != 0 || !nib || !step || !mn) return -1;
    gen_matrix_src(DIST_SOURCE, w, 0.0, 0, 0, N, K, nib, step, mn, 0);
    return 0;
}

static int write_all(FILE* f, const void* p, size_t n) { return fwrite(p, 1, n, f) == n ? 0 : -1; }

/*
 * Writes a whole model file.  norm_mode 0: all norm weights 1.0; 1: norm weights U(0.8, 1.2)
 * (used by tests so that a kernel ignoring the norm weights cannot pass).
 * Returns 0 on success.
 */
int llm4s128_write_model(const char* path, uint32_t layers, uint32_t dim, uint32_t ffn,
                         uint32_t vocab, uint32_t heads, uint32_t kv_heads, uint64_t seed,
                         double sigma, int norm_mode) {
    if (!path || dim % 128 || ffn % 128 || heads == 0 || kv_heads == 0 || dim % heads) return -1;
    FILE* f = fopen(path, "wb");
    if (!f) return -2;
    int rc = 0;
    uint32_t hdr[7] = {layers, dim, ffn, vocab, heads, kv_heads, 128};
    rc |= write_all(f, "LLM4S128", 8);
    rc |= write_all(f, hdr, sizeof(hdr));

    uint32_t head_dim = dim / heads, kv_dim = kv_heads * head_dim;
    float* norm = (float*)malloc(sizeof(float) * dim);
    uint64_t tensor = 0;
    /* norms: tensor ids 1..; matrices: tensor ids 1000.. */
    #define WRITE_NORM() do { \
        nrng_t g; rng_seed(&g.r, seed, ++tensor, 0); g.have = 0; \
        for (uint32_t i = 0; i < dim; ++i) norm[i] = norm_mode ? (float)(0.8 + 0.4 * rng_uniform(&g.r)) : 1.0f; \
        rc |= write_all(f, norm, sizeof(float) * dim); } while (0)

    uint64_t mat_id = 1000;
    size_t cap = 0;
    uint8_t* nib = NULL; uint16_t* st = NULL; uint16_t* mn = NULL;
    #define WRITE_MAT(NN, KK) do { \
        uint32_t n_ = (NN), k_ = (KK), nb_ = n_ * (k_ / 128); \
        size_t need = (size_t)nb_; \
        if (need > cap) { free(nib); free(st); free(mn); cap = need; \
            nib = (uint8_t*)malloc(cap * 64); st = (uint16_t*)malloc(cap * 2); mn = (uint16_t*)malloc(cap * 2); } \
        gen_matrix(DIST_NORMAL, sigma, seed, mat_id++, (int)n_, (int)k_, nib, st, mn, 0); \
        uint32_t mh[3] = {n_, k_, nb_}; \
        rc |= write_all(f, mh, sizeof(mh)); \
        rc |= write_all(f, nib, (size_t)nb_ * 64); \
        rc |= write_all(f, st, (size_t)nb_ * 2); \
        rc |= write_all(f, mn, (size_t)nb_ * 2); } while (0)

    WRITE_NORM(); /* final_norm */
    for (uint32_t l = 0; l < layers; ++l) {
        WRITE_NORM(); /* in_norm */
        WRITE_NORM(); /* post_norm */
        WRITE_MAT(dim, dim);     /* Wq */
        WRITE_MAT(kv_dim, dim);  /* Wk */
        WRITE_MAT(kv_dim, dim);  /* Wv */
        WRITE_MAT(dim, dim);     /* Wo */
        WRITE_MAT(ffn, dim);     /* Wgate */
        WRITE_MAT(ffn, dim);     /* Wup */
        WRITE_MAT(dim, ffn);     /* Wdown */
    }
    WRITE_MAT(vocab, dim);       /* shared lm_head / embedding */
    #undef WRITE_MAT
    #undef WRITE_NORM
    free(nib); free(st); free(mn); free(norm);
    if (fclose(f) != 0) rc = -3;
    return rc ? -3 : 0;
}
