/*
 * TEST INFRASTRUCTURE ONLY — see kk_oracle.h. Plain C11, compiled without
 * floating-point contraction (-ffp-contract=off) so each FP32 operation is
 * rounded exactly as written, in the reference's order of operations.
 */
#include "kk_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------- FP16 codec (IEEE binary16, round to nearest even) -------- */

uint16_t kko_f2h(float value)
{
    uint32_t x;
    memcpy(&x, &value, 4);
    uint32_t const sign = (x >> 16) & 0x8000u;
    x &= 0x7fffffffu;
    if (x >= 0x7f800000u) {
        return (uint16_t)(sign | (x == 0x7f800000u ? 0x7c00u : 0x7e00u));
    }
    int const e = (int)(x >> 23) - 112;
    uint32_t m = x & 0x7fffffu;
    if (e >= 31) {
        return (uint16_t)(sign | 0x7c00u);
    }
    if (e <= 0) {
        uint32_t const shift = (uint32_t)(126 - (int)(x >> 23));
        if (shift > 24) {
            return (uint16_t)sign;
        }
        m |= 0x800000u;
        uint32_t q = m >> shift;
        uint32_t const rest = m & ((1u << shift) - 1u);
        uint32_t const half = 1u << (shift - 1u);
        if (rest > half || (rest == half && (q & 1u))) {
            ++q;
        }
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (m >> 13);
    uint32_t const rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (q & 1u))) {
        ++q;
    }
    return (uint16_t)(sign | q);
}

float kko_h2f(uint16_t h)
{
    uint32_t const sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t const e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0x1f) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m != 0) {
        int ex = 113;
        while (!(m & 0x400u)) {
            m <<= 1;
            --ex;
        }
        bits = sign | ((uint32_t)ex << 23) | ((m & 0x3ffu) << 13);
    } else {
        bits = sign;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float round16(float v) { return kko_h2f(kko_f2h(v)); }

/* ---------------- attention ------------------------------------------------ */

/* offset in [layer][K/V][token][head][dim] with a token capacity */
static size_t kv_offset(uint32_t heads, uint32_t dim, uint32_t layer, uint32_t comp, uint32_t token,
    uint32_t head, uint32_t d, uint32_t capacity)
{
    return ((((size_t)layer * 2 + comp) * capacity + token) * heads + head) * dim + d;
}

int kko_reference_attention(uint32_t layers, uint32_t heads, uint32_t dim, const uint16_t* kv,
    uint32_t tokens, const float* query, float* output)
{
    if (tokens == 0) {
        return 0;
    }
    float* scores = (float*)malloc(sizeof(float) * tokens);
    if (!scores) {
        return 0;
    }
    float const scale = 1.0f / sqrtf((float)dim);
    int ok = 1;
    for (uint32_t l = 0; l < layers && ok; ++l) {
        for (uint32_t h = 0; h < heads && ok; ++h) {
            size_t const qb = ((size_t)l * heads + h) * dim;
            float maximum = -INFINITY;
            for (uint32_t t = 0; t < tokens; ++t) {
                float dot = 0.0f;
                for (uint32_t d = 0; d < dim; ++d) {
                    dot += query[qb + d] * kko_h2f(kv[kv_offset(heads, dim, l, 0, t, h, d, tokens)]);
                }
                scores[t] = dot * scale;
                maximum = scores[t] > maximum ? scores[t] : maximum;
            }
            float denom = 0.0f;
            for (uint32_t t = 0; t < tokens; ++t) {
                scores[t] = expf(scores[t] - maximum);
                denom += scores[t];
            }
            if (!(denom > 0.0f) || !isfinite(denom)) {
                ok = 0;
                break;
            }
            for (uint32_t d = 0; d < dim; ++d) {
                float acc = 0.0f;
                for (uint32_t t = 0; t < tokens; ++t) {
                    acc += scores[t] * kko_h2f(kv[kv_offset(heads, dim, l, 1, t, h, d, tokens)]);
                }
                output[qb + d] = acc / denom;
            }
        }
    }
    free(scores);
    return ok;
}

int kko_paged_attention(const uint16_t* micro, const uint16_t* extent, uint32_t layers,
    uint32_t kv_heads, uint32_t dim, uint32_t layer, uint32_t q_heads, const uint32_t* slot,
    const uint32_t* valid, const uint8_t* kind, uint32_t entries, const uint16_t* q, uint16_t* out)
{
    uint32_t tokens = 0;
    for (uint32_t e = 0; e < entries; ++e) {
        tokens += valid[e];
    }
    if (tokens == 0 || kv_heads == 0 || q_heads % kv_heads != 0) {
        return 0;
    }
    /* Gather this layer, one KV head at a time, into a contiguous
     * [1 layer][K/V][token][1 head][dim] buffer. */
    uint16_t* kv = (uint16_t*)malloc(sizeof(uint16_t) * 2 * (size_t)tokens * dim);
    float* qf = (float*)malloc(sizeof(float) * dim);
    float* of = (float*)malloc(sizeof(float) * dim);
    if (!kv || !qf || !of) {
        free(kv);
        free(qf);
        free(of);
        return 0;
    }
    uint32_t const group = q_heads / kv_heads;
    int ok = 1;
    for (uint32_t h = 0; h < kv_heads && ok; ++h) {
        uint32_t t = 0;
        for (uint32_t e = 0; e < entries; ++e) {
            uint32_t const cap = kind[e] == 0 ? 8u : 64u;
            size_t const page = (size_t)layers * 2 * cap * kv_heads * dim;
            const uint16_t* base = (kind[e] == 0 ? micro : extent) + (size_t)slot[e] * page;
            for (uint32_t i = 0; i < valid[e]; ++i, ++t) {
                for (uint32_t c = 0; c < 2; ++c) {
                    memcpy(kv + ((size_t)c * tokens + t) * dim,
                        base + kv_offset(kv_heads, dim, layer, c, i, h, 0, cap), dim * sizeof(uint16_t));
                }
            }
        }
        for (uint32_t g = 0; g < group && ok; ++g) {
            uint32_t const qh = h * group + g;
            for (uint32_t d = 0; d < dim; ++d) {
                qf[d] = kko_h2f(q[(size_t)qh * dim + d]);
            }
            ok = kko_reference_attention(1, 1, dim, kv, tokens, qf, of);
            for (uint32_t d = 0; d < dim && ok; ++d) {
                out[(size_t)qh * dim + d] = kko_f2h(of[d]);
            }
        }
    }
    free(kv);
    free(qf);
    free(of);
    return ok;
}

uint32_t kko_argmax(const float* v, uint32_t n)
{
    uint32_t best = 0;
    for (uint32_t i = 1; i < n; ++i) {
        if (v[i] > v[best]) {
            best = i;
        }
    }
    return best;
}

/* ---------------- decoder ----------------------------------------------------- */

typedef struct {
    float *in_norm, *post_norm, *q, *k, *v, *o, *gate, *up, *down;
} layer_w;

typedef struct {
    uint64_t id;
    uint32_t length, capacity;
    float** keys;    /* [layers] -> [capacity][kv] */
    float** values;
    int live;
} sequence;

typedef struct {
    kko_config c;
    uint32_t threads;
    /* 1: the summation-order twin (kko_model_set_wide_sums) */
    int wide;
    float *embed, *lm_head, *final_norm;
    layer_w* layer;
    sequence* seqs;
    uint32_t nseq, capseq;
} model;

static float* widen(const uint16_t* src, size_t n)
{
    float* out = (float*)malloc(sizeof(float) * (n ? n : 1));
    if (out) {
        for (size_t i = 0; i < n; ++i) {
            out[i] = kko_h2f(src[i]);
        }
    }
    return out;
}

void* kko_model_create(const kko_config* c, const uint16_t* const* w, uint32_t threads)
{
    model* m = (model*)calloc(1, sizeof(model));
    if (!m) {
        return NULL;
    }
    m->c = *c;
    m->threads = threads ? threads : 1;
    size_t const H = c->hidden, I = c->intermediate, V = c->vocab;
    size_t const KV = (size_t)c->kv_heads * c->head_dim;
    m->embed = widen(w[0], V * H);
    m->lm_head = widen(w[1], V * H);
    m->final_norm = widen(w[2], H);
    m->layer = (layer_w*)calloc(c->layers, sizeof(layer_w));
    for (uint32_t l = 0; l < c->layers; ++l) {
        const uint16_t* const* lw = w + 3 + 9 * (size_t)l;
        layer_w* L = &m->layer[l];
        L->in_norm = widen(lw[0], H);
        L->post_norm = widen(lw[1], H);
        L->q = widen(lw[2], H * H);
        L->k = widen(lw[3], KV * H);
        L->v = widen(lw[4], KV * H);
        L->o = widen(lw[5], H * H);
        L->gate = widen(lw[6], I * H);
        L->up = widen(lw[7], I * H);
        L->down = widen(lw[8], H * I);
    }
    return m;
}

static void free_seq(model* m, sequence* s)
{
    if (s->keys) {
        for (uint32_t l = 0; l < m->c.layers; ++l) {
            free(s->keys[l]);
            free(s->values[l]);
        }
    }
    free(s->keys);
    free(s->values);
    memset(s, 0, sizeof(*s));
}

void kko_model_destroy(void* mp)
{
    model* m = (model*)mp;
    if (!m) {
        return;
    }
    for (uint32_t i = 0; i < m->nseq; ++i) {
        free_seq(m, &m->seqs[i]);
    }
    free(m->seqs);
    for (uint32_t l = 0; l < m->c.layers; ++l) {
        layer_w* L = &m->layer[l];
        free(L->in_norm); free(L->post_norm); free(L->q); free(L->k); free(L->v);
        free(L->o); free(L->gate); free(L->up); free(L->down);
    }
    free(m->layer);
    free(m->embed);
    free(m->lm_head);
    free(m->final_norm);
    free(m);
}

static sequence* find_seq(model* m, uint64_t id)
{
    for (uint32_t i = 0; i < m->nseq; ++i) {
        if (m->seqs[i].live && m->seqs[i].id == id) {
            return &m->seqs[i];
        }
    }
    return NULL;
}

static sequence* new_seq(model* m, uint64_t id)
{
    if (find_seq(m, id)) {
        return NULL;
    }
    for (uint32_t i = 0; i < m->nseq; ++i) {
        if (!m->seqs[i].live) {
            m->seqs[i].live = 1;
            m->seqs[i].id = id;
            return &m->seqs[i];
        }
    }
    if (m->nseq == m->capseq) {
        uint32_t const cap = m->capseq ? m->capseq * 2 : 16;
        sequence* grown = (sequence*)realloc(m->seqs, cap * sizeof(sequence));
        if (!grown) {
            return NULL;
        }
        memset(grown + m->capseq, 0, (cap - m->capseq) * sizeof(sequence));
        m->seqs = grown;
        m->capseq = cap;
    }
    sequence* s = &m->seqs[m->nseq++];
    s->live = 1;
    s->id = id;
    return s;
}

static int reserve_seq(model* m, sequence* s, uint32_t n)
{
    size_t const KV = (size_t)m->c.kv_heads * m->c.head_dim;
    if (!s->keys) {
        s->keys = (float**)calloc(m->c.layers, sizeof(float*));
        s->values = (float**)calloc(m->c.layers, sizeof(float*));
        if (!s->keys || !s->values) {
            return 0;
        }
    }
    if (n <= s->capacity) {
        return 1;
    }
    uint32_t cap = s->capacity ? s->capacity : 64;
    while (cap < n) {
        cap *= 2;
    }
    for (uint32_t l = 0; l < m->c.layers; ++l) {
        float* k = (float*)realloc(s->keys[l], sizeof(float) * KV * cap);
        float* v = (float*)realloc(s->values[l], sizeof(float) * KV * cap);
        if (!k || !v) {
            return 0;
        }
        s->keys[l] = k;
        s->values[l] = v;
    }
    s->capacity = cap;
    return 1;
}

int kko_seq_create(void* mp, uint64_t id) { return new_seq((model*)mp, id) != NULL; }

int kko_seq_release(void* mp, uint64_t id)
{
    model* m = (model*)mp;
    sequence* s = find_seq(m, id);
    if (!s) {
        return 0;
    }
    free_seq(m, s);
    return 1;
}

uint32_t kko_seq_length(void* mp, uint64_t id)
{
    sequence* s = find_seq((model*)mp, id);
    return s ? s->length : 0;
}

int kko_seq_fork(void* mp, uint64_t source, uint64_t child)
{
    model* m = (model*)mp;
    sequence* src = find_seq(m, source);
    if (!src) {
        return 0;
    }
    uint64_t const sid = src->id;
    sequence* dst = new_seq(m, child);
    src = find_seq(m, sid); /* new_seq may have moved the array */
    if (!dst || !src || !reserve_seq(m, dst, src->length ? src->length : 1)) {
        return 0;
    }
    size_t const KV = (size_t)m->c.kv_heads * m->c.head_dim;
    for (uint32_t l = 0; src->length != 0 && l < m->c.layers; ++l) {
        memcpy(dst->keys[l], src->keys[l], sizeof(float) * KV * src->length);
        memcpy(dst->values[l], src->values[l], sizeof(float) * KV * src->length);
    }
    dst->length = src->length;
    return 1;
}

int kko_seq_append_kv(void* mp, uint64_t id, uint32_t n, const uint16_t* k, const uint16_t* v)
{
    model* m = (model*)mp;
    sequence* s = find_seq(m, id);
    if (!s || !reserve_seq(m, s, s->length + n)) {
        return 0;
    }
    size_t const KV = (size_t)m->c.kv_heads * m->c.head_dim;
    for (uint32_t t = 0; t < n; ++t) {
        for (uint32_t l = 0; l < m->c.layers; ++l) {
            const uint16_t* ks = k + ((size_t)t * m->c.layers + l) * KV;
            const uint16_t* vs = v + ((size_t)t * m->c.layers + l) * KV;
            for (size_t i = 0; i < KV; ++i) {
                s->keys[l][(s->length + t) * KV + i] = kko_h2f(ks[i]);
                s->values[l][(s->length + t) * KV + i] = kko_h2f(vs[i]);
            }
        }
    }
    s->length += n;
    return 1;
}

/* ---- threaded helpers ---- */

typedef void (*task_fn)(void* ctx, uint32_t index);
typedef struct {
    task_fn fn;
    void* ctx;
    uint32_t n, stride, first;
} task_range;

static void* run_range(void* arg)
{
    task_range* r = (task_range*)arg;
    for (uint32_t i = r->first; i < r->n; i += r->stride) {
        r->fn(r->ctx, i);
    }
    return NULL;
}

static void parallel_for(uint32_t threads, uint32_t n, task_fn fn, void* ctx)
{
    if (threads <= 1 || n < 2) {
        for (uint32_t i = 0; i < n; ++i) {
            fn(ctx, i);
        }
        return;
    }
    if (threads > n) {
        threads = n;
    }
    pthread_t tid[256];
    task_range r[256];
    if (threads > 256) {
        threads = 256;
    }
    for (uint32_t t = 0; t < threads; ++t) {
        r[t] = (task_range){fn, ctx, n, threads, t};
        if (t > 0 && pthread_create(&tid[t], NULL, run_range, &r[t]) != 0) {
            run_range(&r[t]);
            tid[t] = 0;
        }
    }
    run_range(&r[0]);
    for (uint32_t t = 1; t < threads; ++t) {
        if (tid[t]) {
            pthread_join(tid[t], NULL);
        }
    }
}

/* y[b][row] = sum_c W[row][c] x[b][c] (sequential over c), rounded unless raw. */
typedef struct {
    const float* w;
    const float* x;
    float* y;
    uint32_t rows, cols, batch, round, wide;
} matvec_ctx;

static void matvec_row(void* p, uint32_t row)
{
    matvec_ctx* c = (matvec_ctx*)p;
    const float* w = c->w + (size_t)row * c->cols;
    for (uint32_t b = 0; b < c->batch; ++b) {
        const float* x = c->x + (size_t)b * c->cols;
        float sum = 0.0f;
        if (c->wide) {
            double d = 0.0;
            for (uint32_t i = 0; i < c->cols; ++i) {
                d += (double)w[i] * (double)x[i];
            }
            sum = (float)d;
        } else {
            for (uint32_t i = 0; i < c->cols; ++i) {
                sum += w[i] * x[i];
            }
        }
        c->y[(size_t)b * c->rows + row] = c->round ? round16(sum) : sum;
    }
}

static void matvec(model* m, const float* w, const float* x, float* y, uint32_t rows, uint32_t cols,
    uint32_t batch, int round)
{
    matvec_ctx c = {w, x, y, rows, cols, batch, (uint32_t)round, (uint32_t)m->wide};
    parallel_for(m->threads, rows, matvec_row, &c);
}

/* The summation-order twin: the same arithmetic and FP16 rounding points,
 * with the projection dot products summed in double precision and rounded
 * to float once. Comparing the two measures how far a different (equally
 * valid) summation order alone moves the outputs of this model: the noise
 * floor any other implementation of the reference arithmetic meets. */
void kko_model_set_wide_sums(void* mp, int wide)
{
    ((model*)mp)->wide = wide != 0;
}

static void rms_norm(const float* x, const float* w, float* y, uint32_t n, float eps)
{
    float sq = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        sq += x[i] * x[i];
    }
    float const scale = 1.0f / sqrtf(sq / (float)n + eps);
    for (uint32_t i = 0; i < n; ++i) {
        y[i] = round16(x[i] * scale * w[i]);
    }
}

static void rope(float* v, uint32_t heads, uint32_t dim, uint32_t position, float theta)
{
    uint32_t const half = dim / 2;
    for (uint32_t h = 0; h < heads; ++h) {
        for (uint32_t d = 0; d < half; ++d) {
            size_t const a = (size_t)h * dim + d;
            size_t const b = a + half;
            float const angle = (float)position * powf(theta, -2.0f * (float)d / (float)dim);
            float const l = v[a], r = v[b];
            v[a] = round16(l * cosf(angle) - r * sinf(angle));
            v[b] = round16(r * cosf(angle) + l * sinf(angle));
        }
    }
}

typedef struct {
    model* m;
    sequence** seqs;
    uint32_t layer;
    const float* q; /* [batch][H] */
    float* out;     /* [batch][H] */
} attn_ctx;

static void attend_one(void* p, uint32_t task)
{
    attn_ctx* a = (attn_ctx*)p;
    kko_config const* c = &a->m->c;
    uint32_t const b = task / c->q_heads;
    uint32_t const qh = task % c->q_heads;
    sequence* s = a->seqs[b];
    uint32_t const group = c->q_heads / c->kv_heads;
    uint32_t const kvh = qh / group;
    uint32_t const D = c->head_dim;
    size_t const KV = (size_t)c->kv_heads * D;
    const float* q = a->q + (size_t)b * c->hidden + (size_t)qh * D;
    const float* keys = s->keys[a->layer];
    const float* vals = s->values[a->layer];
    float* scores = (float*)malloc(sizeof(float) * s->length);
    float const scale = 1.0f / sqrtf((float)D);
    float maximum = -INFINITY;
    for (uint32_t t = 0; t < s->length; ++t) {
        float dot = 0.0f;
        for (uint32_t d = 0; d < D; ++d) {
            dot += q[d] * keys[t * KV + kvh * D + d];
        }
        scores[t] = dot * scale;
        maximum = scores[t] > maximum ? scores[t] : maximum;
    }
    float denom = 0.0f;
    for (uint32_t t = 0; t < s->length; ++t) {
        denom += expf(scores[t] - maximum);
    }
    for (uint32_t d = 0; d < D; ++d) {
        float o = 0.0f;
        for (uint32_t t = 0; t < s->length; ++t) {
            o += expf(scores[t] - maximum) / denom * vals[t * KV + kvh * D + d];
        }
        a->out[(size_t)b * c->hidden + (size_t)qh * D + d] = round16(o);
    }
    free(scores);
}

int kko_forward_batch(void* mp, uint32_t n, const uint64_t* ids, const uint32_t* tokens,
    const uint32_t* positions, float* logits_out, uint16_t* hidden_out, uint32_t* greedy)
{
    model* m = (model*)mp;
    kko_config const* c = &m->c;
    uint32_t const H = c->hidden, I = c->intermediate, V = c->vocab, D = c->head_dim;
    uint32_t const KV = c->kv_heads * D;
    sequence** seqs = (sequence**)malloc(sizeof(sequence*) * n);
    for (uint32_t b = 0; b < n; ++b) {
        seqs[b] = find_seq(m, ids[b]);
        if (!seqs[b] || seqs[b]->length != positions[b] || tokens[b] >= V
            || !reserve_seq(m, seqs[b], seqs[b]->length + 1)) {
            free(seqs);
            return 0;
        }
    }
    float* hidden = (float*)malloc(sizeof(float) * n * H);
    float* normed = (float*)malloc(sizeof(float) * n * H);
    float* q = (float*)malloc(sizeof(float) * n * H);
    float* k = (float*)malloc(sizeof(float) * n * KV);
    float* v = (float*)malloc(sizeof(float) * n * KV);
    float* attn = (float*)malloc(sizeof(float) * n * H);
    float* proj = (float*)malloc(sizeof(float) * n * H);
    float* gate = (float*)malloc(sizeof(float) * n * I);
    float* up = (float*)malloc(sizeof(float) * n * I);
    float* logits = (float*)malloc(sizeof(float) * n * V);
    for (uint32_t b = 0; b < n; ++b) {
        memcpy(hidden + (size_t)b * H, m->embed + (size_t)tokens[b] * H, sizeof(float) * H);
    }
    for (uint32_t l = 0; l < c->layers; ++l) {
        layer_w const* L = &m->layer[l];
        for (uint32_t b = 0; b < n; ++b) {
            rms_norm(hidden + (size_t)b * H, L->in_norm, normed + (size_t)b * H, H, c->eps);
        }
        matvec(m, L->q, normed, q, H, H, n, 1);
        matvec(m, L->k, normed, k, KV, H, n, 1);
        matvec(m, L->v, normed, v, KV, H, n, 1);
        for (uint32_t b = 0; b < n; ++b) {
            rope(q + (size_t)b * H, c->q_heads, D, positions[b], c->theta);
            rope(k + (size_t)b * KV, c->kv_heads, D, positions[b], c->theta);
            sequence* s = seqs[b];
            memcpy(s->keys[l] + (size_t)s->length * KV, k + (size_t)b * KV, sizeof(float) * KV);
            memcpy(s->values[l] + (size_t)s->length * KV, v + (size_t)b * KV, sizeof(float) * KV);
        }
        for (uint32_t b = 0; b < n; ++b) {
            ++seqs[b]->length; /* attend over the current token too */
        }
        attn_ctx actx = {m, seqs, l, q, attn};
        parallel_for(m->threads, n * c->q_heads, attend_one, &actx);
        for (uint32_t b = 0; b < n; ++b) {
            --seqs[b]->length;
        }
        matvec(m, L->o, attn, proj, H, H, n, 1);
        for (size_t i = 0; i < (size_t)n * H; ++i) {
            hidden[i] = round16(hidden[i] + proj[i]);
        }
        for (uint32_t b = 0; b < n; ++b) {
            rms_norm(hidden + (size_t)b * H, L->post_norm, normed + (size_t)b * H, H, c->eps);
        }
        matvec(m, L->gate, normed, gate, I, H, n, 1);
        matvec(m, L->up, normed, up, I, H, n, 1);
        for (size_t i = 0; i < (size_t)n * I; ++i) {
            gate[i] = round16(gate[i] / (1.0f + expf(-gate[i])) * up[i]);
        }
        matvec(m, L->down, gate, proj, H, I, n, 1);
        for (size_t i = 0; i < (size_t)n * H; ++i) {
            hidden[i] = round16(hidden[i] + proj[i]);
        }
    }
    for (uint32_t b = 0; b < n; ++b) {
        ++seqs[b]->length;
        rms_norm(hidden + (size_t)b * H, m->final_norm, normed + (size_t)b * H, H, c->eps);
        if (hidden_out) {
            for (uint32_t i = 0; i < H; ++i) {
                hidden_out[(size_t)b * H + i] = kko_f2h(normed[(size_t)b * H + i]);
            }
        }
    }
    matvec(m, m->lm_head, normed, logits, V, H, n, 0);
    for (uint32_t b = 0; b < n; ++b) {
        greedy[b] = kko_argmax(logits + (size_t)b * V, V);
    }
    if (logits_out) {
        memcpy(logits_out, logits, sizeof(float) * n * V);
    }
    free(seqs); free(hidden); free(normed); free(q); free(k); free(v); free(attn);
    free(proj); free(gate); free(up); free(logits);
    return 1;
}
