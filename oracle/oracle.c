/*
 * ORACLE — test infrastructure only.  Never linked into, loaded by, or called from the product
 * library; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and only
 * as the reference results the GPU path is compared with.
 *
 * A plain-C, single-threaded restatement of the reference engine's token loop, following the
 * scalar (non-NEON) code path that the reference compiles to on Linux/x86
 * (src/llama_engine.cpp, HAS_ARM_NEON undefined, parallel_for serial at :79-80).  Every float
 * expression keeps the reference's evaluation order, so with the same compiler flags
 * (-O3, no -march, no fast-math) the outputs are bit-identical to the reference build; the test
 * suite checks this against the reference compiled from its own source (oracle/Makefile).
 *
 * Citations are file:line in the reference project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define ORC_MAX_SEQ_LEN 8192 /* src/llama_engine.cpp:26 */

/* src/llama_engine.cpp:28-33 */
static inline float orc_bf16_to_f32(uint16_t v) {
    uint32_t bits = (uint32_t)v << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

typedef struct {
    uint32_t out_dim, in_dim, num_blocks;
    const uint8_t* nibbles;
    const uint16_t* step;
    const uint16_t* min;
} orc_matrix;

/* src/llama_engine.cpp:87-115 (scalar branch :110-113) */
void orc_rms_norm(const float* x, const float* w, float* out, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += x[i] * x[i];
    float inv = 1.0f / sqrtf((sum / (float)n) + 1e-5f);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * w[i] * inv;
}

/* src/llama_engine.cpp:120-151 (scalar branch :141-148) */
void orc_apply_rope(float* vec, size_t n_heads, size_t head_dim, size_t pos,
                    const float* cos_tab, const float* sin_tab) {
    const float* c = &cos_tab[pos * (head_dim / 2)];
    const float* s = &sin_tab[pos * (head_dim / 2)];
    for (size_t h = 0; h < n_heads; ++h) {
        float* hp = &vec[h * head_dim];
        for (size_t i = 0; i < head_dim / 2; ++i) {
            float r0 = hp[i], r1 = hp[i + head_dim / 2];
            hp[i] = r0 * c[i] - r1 * s[i];
            hp[i + head_dim / 2] = r0 * s[i] + r1 * c[i];
        }
    }
}

/* src/llama_engine.cpp:164-180 */
static size_t orc_map_matrix(orc_matrix* m, const uint8_t* p) {
    size_t off = 0;
    memcpy(&m->out_dim, p + off, 4); off += 4;
    memcpy(&m->in_dim, p + off, 4); off += 4;
    memcpy(&m->num_blocks, p + off, 4); off += 4;
    m->nibbles = p + off; off += (size_t)m->num_blocks * 64;
    m->step = (const uint16_t*)(p + off); off += (size_t)m->num_blocks * 2;
    m->min = (const uint16_t*)(p + off); off += (size_t)m->num_blocks * 2;
    return off;
}

/* src/llama_engine.cpp:182-220 (scalar branch :212-217) */
void orc_dequant_row(const uint8_t* nibbles, const uint16_t* step, const uint16_t* mn,
                     uint32_t in_dim, size_t row, float* out) {
    size_t bpr = in_dim / 128, b0 = row * bpr;
    for (size_t b = 0; b < bpr; ++b) {
        size_t blk = b0 + b;
        float st = orc_bf16_to_f32(step[blk]);
        float mv = orc_bf16_to_f32(mn[blk]);
        const uint8_t* np = &nibbles[blk * 64];
        for (int j = 0; j < 64; ++j) {
            uint8_t byte = np[j];
            out[b * 128 + j * 2 + 0] = mv + (float)(byte & 0x0F) * st;
            out[b * 128 + j * 2 + 1] = mv + (float)(byte >> 4) * st;
        }
    }
}

/* src/llama_engine.cpp:496-521 (scalar branch :515-519) */
void orc_block_sums(const float* x, size_t K, float* sums) {
    for (size_t b = 0; b < K / 128; ++b) {
        float s = 0.0f;
        for (size_t i = 0; i < 128; ++i) s += x[b * 128 + i];
        sums[b] = s;
    }
}

/*
 * Factored block-128 GEMV, y[n] = sum_b (min*xs_b + step*sum_j(q_lo*x_2j + q_hi*x_2j+1)).
 * src/llama_engine.cpp:233-357 (scalar branch :322-355).  The reference walks rows in groups
 * of four; rows are independent, so a row-at-a-time loop yields the same bits.
 */
void orc_gemv(const uint8_t* nibbles, const uint16_t* step, const uint16_t* mn, uint32_t N,
              uint32_t K, const float* x, const float* xs, float* y) {
    size_t bpr = K / 128;
    for (size_t n = 0; n < N; ++n) {
        float total = 0.0f;
        for (size_t b = 0; b < bpr; ++b) {
            size_t blk = n * bpr + b;
            float st = orc_bf16_to_f32(step[blk]), mv = orc_bf16_to_f32(mn[blk]);
            const uint8_t* np = &nibbles[blk * 64];
            const float* px = &x[b * 128];
            float qd = 0.0f;
            for (int j = 0; j < 64; ++j) {
                float x0 = px[j * 2 + 0], x1 = px[j * 2 + 1];
                qd += (float)(np[j] & 0xF) * x0 + (float)(np[j] >> 4) * x1;
            }
            total += mv * xs[b] + st * qd;
        }
        y[n] = total;
    }
}

/* silu(v) = v / (1 + exp(-v)); src/llama_engine.cpp:373 */
static inline float orc_silu(float v) { return v / (1.0f + expf(-v)); }

/* src/llama_engine.cpp:362-491 (scalar branch :460-489) */
void orc_swiglu(const uint8_t* g_nib, const uint16_t* g_step, const uint16_t* g_min,
                const uint8_t* u_nib, const uint16_t* u_step, const uint16_t* u_min, uint32_t N,
                uint32_t K, const float* x, const float* xs, float* act) {
    size_t bpr = K / 128;
    for (size_t n = 0; n < N; ++n) {
        float gt = 0.0f, ut = 0.0f;
        for (size_t b = 0; b < bpr; ++b) {
            size_t blk = n * bpr + b;
            float gs = orc_bf16_to_f32(g_step[blk]), gm = orc_bf16_to_f32(g_min[blk]);
            float us = orc_bf16_to_f32(u_step[blk]), um = orc_bf16_to_f32(u_min[blk]);
            const uint8_t* gp = &g_nib[blk * 64];
            const uint8_t* up = &u_nib[blk * 64];
            const float* px = &x[b * 128];
            float gq = 0.0f, uq = 0.0f;
            for (int j = 0; j < 64; ++j) {
                float x0 = px[j * 2 + 0], x1 = px[j * 2 + 1];
                gq += (float)(gp[j] & 0xF) * x0 + (float)(gp[j] >> 4) * x1;
                uq += (float)(up[j] & 0xF) * x0 + (float)(up[j] >> 4) * x1;
            }
            float s = xs[b];
            gt += gm * s + gs * gq;
            ut += um * s + us * uq;
        }
        act[n] = orc_silu(gt) * ut;
    }
}

/*
 * Greedy / temperature + top-p sampler; src/llama_engine.cpp:784-839.  Overwrites logits with
 * probabilities when temperature > 0.01, and draws with libc rand() exactly as the reference.
 */
int32_t orc_sample(float* logits, size_t vocab, float temperature, float top_p) {
    if (temperature <= 0.01f) {
        int32_t best = 0;
        float bv = -1e30f;
        for (size_t i = 0; i < vocab; ++i)
            if (logits[i] > bv) { bv = logits[i]; best = (int32_t)i; }
        return best;
    }
    float inv_t = 1.0f / temperature;
    for (size_t i = 0; i < vocab; ++i) logits[i] *= inv_t;
    float mx = -1e30f;
    for (size_t i = 0; i < vocab; ++i) if (logits[i] > mx) mx = logits[i];
    float se = 0.0f;
    for (size_t i = 0; i < vocab; ++i) { logits[i] = expf(logits[i] - mx); se += logits[i]; }
    float inv_s = 1.0f / se;
    for (size_t i = 0; i < vocab; ++i) logits[i] *= inv_s;

    size_t k = vocab < 64 ? vocab : 64;
    int32_t ids[64];
    float vals[64];
    for (size_t i = 0; i < k; ++i) { ids[i] = (int32_t)i; vals[i] = logits[i]; }
    for (size_t i = k; i < vocab; ++i) {
        float v = logits[i];
        if (v > vals[k - 1]) {
            size_t p = k - 1;
            while (p > 0 && v > vals[p - 1]) { vals[p] = vals[p - 1]; ids[p] = ids[p - 1]; --p; }
            vals[p] = v; ids[p] = (int32_t)i;
        }
    }
    float cum = 0.0f;
    size_t last = 0;
    for (size_t i = 0; i < k; ++i) { cum += vals[i]; last = i; if (cum >= top_p) break; }
    float r = ((float)rand() / (float)RAND_MAX) * cum;
    float run = 0.0f;
    for (size_t i = 0; i <= last; ++i) { run += vals[i]; if (run >= r) return ids[i]; }
    return ids[0];
}

/* ------------------------------------------------------------------------------------------ */
/* Engine state: src/llama_engine.cpp:844-1043                                                 */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    const float* in_norm;
    const float* post_norm;
    orc_matrix wq, wk, wv, wo, wg, wu, wd;
} orc_layer;

typedef struct {
    int fd;
    size_t size;
    const uint8_t* data;
    uint32_t num_layers, dim, ffn_dim, vocab, n_heads, n_kv_heads, block;
    size_t head_dim, kv_dim;
    const float* final_norm;
    orc_layer* layers;
    orc_matrix lm_head;
    float *rope_cos, *rope_sin;
    float **kc, **vc;
    /* scratch: src/llama_engine.cpp:749-777 */
    float *x, *norm_buf, *bs_dim, *bs_ffn, *q, *k, *v, *attn, *proj_o, *act, *mlp_out, *logits;
    float* scores;
} orc_engine;

void orc_free(orc_engine* e);

/* src/llama_engine.cpp:865-928 (no size validation, like the reference) */
orc_engine* orc_create(const char* path) {
    if (!path) return NULL;
    orc_engine* e = (orc_engine*)calloc(1, sizeof(orc_engine));
    e->fd = open(path, O_RDONLY);
    if (e->fd < 0) { free(e); return NULL; }
    struct stat sb;
    fstat(e->fd, &sb);
    e->size = (size_t)sb.st_size;
    void* p = mmap(NULL, e->size, PROT_READ, MAP_SHARED, e->fd, 0);
    if (p == MAP_FAILED) { close(e->fd); free(e); return NULL; }
    e->data = (const uint8_t*)p;
    if (e->size < 36 || memcmp(e->data, "LLM4S128", 8) != 0) { orc_free(e); return NULL; }
    size_t off = 8;
    uint32_t h[7];
    memcpy(h, e->data + off, 28); off += 28;
    e->num_layers = h[0]; e->dim = h[1]; e->ffn_dim = h[2]; e->vocab = h[3];
    e->n_heads = h[4]; e->n_kv_heads = h[5]; e->block = h[6];
    e->head_dim = e->dim / e->n_heads;
    e->kv_dim = e->n_kv_heads * e->head_dim;
    e->final_norm = (const float*)(e->data + off); off += (size_t)e->dim * 4;
    e->layers = (orc_layer*)calloc(e->num_layers, sizeof(orc_layer));
    for (uint32_t l = 0; l < e->num_layers; ++l) {
        orc_layer* L = &e->layers[l];
        L->in_norm = (const float*)(e->data + off); off += (size_t)e->dim * 4;
        L->post_norm = (const float*)(e->data + off); off += (size_t)e->dim * 4;
        off += orc_map_matrix(&L->wq, e->data + off);
        off += orc_map_matrix(&L->wk, e->data + off);
        off += orc_map_matrix(&L->wv, e->data + off);
        off += orc_map_matrix(&L->wo, e->data + off);
        off += orc_map_matrix(&L->wg, e->data + off);
        off += orc_map_matrix(&L->wu, e->data + off);
        off += orc_map_matrix(&L->wd, e->data + off);
    }
    off += orc_map_matrix(&e->lm_head, e->data + off);

    /* RoPE table, src/llama_engine.cpp:908-917 (theta 500000, no llama3 scaling) */
    size_t hd2 = e->head_dim / 2;
    e->rope_cos = (float*)calloc(ORC_MAX_SEQ_LEN * hd2, 4);
    e->rope_sin = (float*)calloc(ORC_MAX_SEQ_LEN * hd2, 4);
    for (size_t pos = 0; pos < ORC_MAX_SEQ_LEN; ++pos) {
        for (size_t i = 0; i < hd2; ++i) {
            float theta = powf(500000.0f, -2.0f * (float)i / (float)e->head_dim);
            e->rope_cos[pos * hd2 + i] = cosf((float)pos * theta);
            e->rope_sin[pos * hd2 + i] = sinf((float)pos * theta);
        }
    }
    /* KV caches, src/llama_engine.cpp:919-924 */
    e->kc = (float**)calloc(e->num_layers, sizeof(float*));
    e->vc = (float**)calloc(e->num_layers, sizeof(float*));
    for (uint32_t l = 0; l < e->num_layers; ++l) {
        e->kc[l] = (float*)calloc(ORC_MAX_SEQ_LEN * e->kv_dim, 4);
        e->vc[l] = (float*)calloc(ORC_MAX_SEQ_LEN * e->kv_dim, 4);
    }
    size_t D = e->dim, F = e->ffn_dim;
    e->x = (float*)calloc(D, 4);
    e->norm_buf = (float*)calloc(D > F ? D : F, 4);
    e->bs_dim = (float*)calloc(D / 128, 4);
    e->bs_ffn = (float*)calloc(F / 128, 4);
    e->q = (float*)calloc(D, 4);
    e->k = (float*)calloc(e->kv_dim, 4);
    e->v = (float*)calloc(e->kv_dim, 4);
    e->attn = (float*)calloc(D, 4);
    e->proj_o = (float*)calloc(D, 4);
    e->act = (float*)calloc(F, 4);
    e->mlp_out = (float*)calloc(D, 4);
    e->logits = (float*)calloc(e->vocab, 4);
    e->scores = (float*)calloc(ORC_MAX_SEQ_LEN, 4);
    return e;
}

void orc_free(orc_engine* e) {
    if (!e) return;
    if (e->kc) for (uint32_t l = 0; l < e->num_layers; ++l) { free(e->kc[l]); free(e->vc[l]); }
    free(e->kc); free(e->vc); free(e->layers);
    free(e->rope_cos); free(e->rope_sin);
    free(e->x); free(e->norm_buf); free(e->bs_dim); free(e->bs_ffn); free(e->q); free(e->k);
    free(e->v); free(e->attn); free(e->proj_o); free(e->act); free(e->mlp_out); free(e->logits);
    free(e->scores);
    if (e->data) munmap((void*)e->data, e->size);
    if (e->fd >= 0) close(e->fd);
    free(e);
}

static void orc_mat_gemv(const orc_matrix* W, const float* x, const float* xs, float* y) {
    orc_gemv(W->nibbles, W->step, W->min, W->out_dim, W->in_dim, x, xs, y);
}

/* src/llama_engine.cpp:935-1042 */
void orc_forward_token(orc_engine* e, int32_t token, size_t pos, int compute_logits) {
    if (pos >= ORC_MAX_SEQ_LEN) return;
    if (token < 0 || token >= (int32_t)e->vocab) token = 0;
    size_t D = e->dim, hd = e->head_dim, kvd = e->kv_dim;
    orc_dequant_row(e->lm_head.nibbles, e->lm_head.step, e->lm_head.min, e->lm_head.in_dim,
                    (size_t)token, e->x);
    for (uint32_t l = 0; l < e->num_layers; ++l) {
        const orc_layer* L = &e->layers[l];
        float* kc = e->kc[l];
        float* vc = e->vc[l];
        orc_rms_norm(e->x, L->in_norm, e->norm_buf, D);
        orc_block_sums(e->norm_buf, D, e->bs_dim);
        orc_mat_gemv(&L->wq, e->norm_buf, e->bs_dim, e->q);
        orc_mat_gemv(&L->wk, e->norm_buf, e->bs_dim, e->k);
        orc_mat_gemv(&L->wv, e->norm_buf, e->bs_dim, e->v);
        orc_apply_rope(e->q, e->n_heads, hd, pos, e->rope_cos, e->rope_sin);
        orc_apply_rope(e->k, e->n_kv_heads, hd, pos, e->rope_cos, e->rope_sin);
        memcpy(&kc[pos * kvd], e->k, kvd * 4);
        memcpy(&vc[pos * kvd], e->v, kvd * 4);
        /* attention, src/llama_engine.cpp:958-1021: 32 heads as 4 groups of 8, kv_h = h/4 */
        for (size_t h = 0; h < 32; ++h) {
            size_t kvh = h / 4;
            const float* qp = &e->q[h * hd];
            float mx = -1e30f;
            for (size_t t = 0; t <= pos; ++t) {
                const float* kp = &kc[t * kvd + kvh * hd];
                float dot = 0.0f;
                for (size_t d = 0; d < hd; ++d) dot += qp[d] * kp[d];
                float s = dot * 0.125f;
                e->scores[t] = s;
                if (s > mx) mx = s;
            }
            float se = 0.0f;
            for (size_t t = 0; t <= pos; ++t) {
                float ex = expf(e->scores[t] - mx);
                e->scores[t] = ex;
                se += ex;
            }
            float inv = 1.0f / se;
            for (size_t t = 0; t <= pos; ++t) e->scores[t] *= inv;
            float* op = &e->attn[h * hd];
            memset(op, 0, hd * 4);
            for (size_t t = 0; t <= pos; ++t) {
                const float* vp = &vc[t * kvd + kvh * hd];
                float w = e->scores[t];
                for (size_t d = 0; d < 64; ++d) op[d] += w * vp[d];
            }
        }
        orc_block_sums(e->attn, D, e->bs_dim);
        orc_mat_gemv(&L->wo, e->attn, e->bs_dim, e->proj_o);
        for (size_t i = 0; i < D; ++i) e->x[i] += e->proj_o[i];
        orc_rms_norm(e->x, L->post_norm, e->norm_buf, D);
        orc_block_sums(e->norm_buf, D, e->bs_dim);
        orc_swiglu(L->wg.nibbles, L->wg.step, L->wg.min, L->wu.nibbles, L->wu.step, L->wu.min,
                   L->wg.out_dim, L->wg.in_dim, e->norm_buf, e->bs_dim, e->act);
        orc_block_sums(e->act, e->ffn_dim, e->bs_ffn);
        orc_mat_gemv(&L->wd, e->act, e->bs_ffn, e->mlp_out);
        for (size_t i = 0; i < D; ++i) e->x[i] += e->mlp_out[i];
    }
    if (compute_logits) {
        orc_rms_norm(e->x, e->final_norm, e->norm_buf, D);
        orc_block_sums(e->norm_buf, D, e->bs_dim);
        orc_mat_gemv(&e->lm_head, e->norm_buf, e->bs_dim, e->logits);
    }
}

/* src/llama_engine.cpp:1118-1127 */
int orc_prefill(orc_engine* e, const int32_t* ids, size_t count, size_t start, int last_logits) {
    if (!e || !ids) return -1;
    for (size_t i = 0; i < count; ++i) {
        int comp = (i + 1 == count) && last_logits;
        orc_forward_token(e, ids[i], start + i, comp);
    }
    return 0;
}

int32_t orc_sample_engine(orc_engine* e, float temperature, float top_p) {
    return orc_sample(e->logits, e->vocab, temperature, top_p);
}

const float* orc_get_logits(orc_engine* e) { return e->logits; }

/* Read access to the state used by the tests (KV cache rows, residual stream, RoPE table). */
const float* orc_get_kv(orc_engine* e, int layer, int which) {
    return which == 0 ? e->kc[layer] : e->vc[layer];
}
const float* orc_get_x(orc_engine* e) { return e->x; }
const float* orc_get_rope(orc_engine* e, int which) { return which == 0 ? e->rope_cos : e->rope_sin; }
uint32_t orc_get_vocab(orc_engine* e) { return e->vocab; }

/* Full-model greedy loop used by fixtures and the CPU baseline: prefill n_prompt-1 tokens,
 * then n_gen x (forward(prev) + greedy).  Writes n_gen tokens and the top-2 margin per step. */
int orc_greedy_run(orc_engine* e, const int32_t* prompt, size_t n_prompt, size_t n_gen,
                   int32_t* out_tokens, float* out_margin) {
    if (!e || !prompt || n_prompt == 0) return -1;
    orc_prefill(e, prompt, n_prompt - 1, 0, 0);
    int32_t tok = prompt[n_prompt - 1];
    size_t pos = n_prompt - 1;
    for (size_t s = 0; s < n_gen; ++s) {
        orc_forward_token(e, tok, pos, 1);
        int32_t nx = orc_sample(e->logits, e->vocab, 0.0f, 0.9f);
        if (out_margin) {
            float b1 = -1e30f, b2 = -1e30f;
            for (size_t i = 0; i < e->vocab; ++i) {
                float v = e->logits[i];
                if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
            }
            out_margin[s] = b1 - b2;
        }
        out_tokens[s] = nx;
        tok = nx;
        ++pos;
    }
    return 0;
}
