/*
 * Test infrastructure only: the ORACLE. A plain-C restatement of the Qwen3-0.6B forward pass
 * of asriva32/Qwen3.cpp (src/inference.cpp), used by tests/, the smoke check and the
 * CPU-baseline leg of bench.py to check the CUDA path. Nothing in the product links it.
 *
 * Every function cites the reference lines it restates. Arithmetic follows the reference
 * operation by operation: fp32 activations, bf16 weights widened exactly to fp32, and the
 * reference's FastDotProduct lane structure (two 8-lane FMA accumulators over 16-element
 * chunks, src/inference.cpp:285-303) and horizontal reduction (:267-276). Pinned against the
 * reference itself (oracle/_ref, built from the reference sources by oracle/Makefile) and the
 * reference's own known-answer tests (tst/test_block.cpp) by tests/test_oracle.py.
 *
 * Status codes: 0 ok, 2 invalid_argument, 3 out_of_range (the exception types the reference
 * throws at src/inference.cpp:594-599, :774-790).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define Q3O_OK 0
#define Q3O_INVALID_ARGUMENT 2
#define Q3O_OUT_OF_RANGE 3

static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* float -> bf16, round to nearest even (static_cast<std::bfloat16_t>, src/inference.cpp:813). */
static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* Reduce (src/inference.cpp:267-276): low+high 128-bit halves, then two horizontal adds. */
static inline float reduce8(const float s[8]) {
    float t0 = s[0] + s[4], t1 = s[1] + s[5], t2 = s[2] + s[6], t3 = s[3] + s[7];
    return (t0 + t1) + (t2 + t3);
}

/* FastDotProduct (src/inference.cpp:285-303). */
static float dot_bf16(const uint16_t* w, const float* x, int m) {
    float lo[8] = {0}, hi[8] = {0}, s[8];
    int j = 0;
    for (; j + 16 <= m; j += 16) {
        for (int l = 0; l < 8; ++l) {
            lo[l] = fmaf(bf2f(w[j + l]), x[j + l], lo[l]);
            hi[l] = fmaf(bf2f(w[j + 8 + l]), x[j + 8 + l], hi[l]);
        }
    }
    for (int l = 0; l < 8; ++l) s[l] = lo[l] + hi[l];
    float sum = reduce8(s);
    for (; j < m; ++j) sum += bf2f(w[j]) * x[j];
    return sum;
}

/* RmsNorm (src/inference.cpp:887-923). */
void q3o_rmsnorm(float* out, const float* x, const uint16_t* w, float eps, int n) {
    float acc[8] = {0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(x[i + l], x[i + l], acc[l]);
    float rms = reduce8(acc);
    for (; i < n; ++i) rms += x[i] * x[i];
    rms = sqrtf(rms / (float)n + eps);
    const float inv = 1.0f / rms;
    for (int j = 0; j < n; ++j) out[j] = (x[j] * inv) * bf2f(w[j]);
}

/* Softmax (src/inference.cpp:925-946). */
void q3o_softmax(float* out, const float* x, int n) {
    float mx = -3.40282347e+38f;
    for (int i = 0; i < n; ++i) mx = x[i] > mx ? x[i] : mx;
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        out[i] = expf(x[i] - mx);
        sum += out[i];
    }
    for (int i = 0; i < n; ++i) out[i] /= sum;
}

/* Silu (src/inference.cpp:948-950). */
float q3o_silu(float x) { return x / (1.0f + expf(-x)); }

/* MatMul (src/inference.cpp:952-966): out[n] = W[n,m] . x[m], W bf16 row-major. */
void q3o_matmul(float* out, const float* x, const uint16_t* w, int n, int m) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) out[i] = dot_bf16(w + (size_t)i * m, x, m);
}

/* ApplyRotaryEmb (src/inference.cpp:968-991): NeoX rotate-half on pairs (i, i + rotary/2). */
void q3o_rope(float* out, int d, int head_dim, int pos, float theta, int rotary_dim) {
    const int half = rotary_dim / 2;
    for (int h0 = 0; h0 < d; h0 += head_dim) {
        for (int i = 0; i < half; ++i) {
            const float freq = 1.0f / powf(theta, 2.0f * (float)i / (float)rotary_dim);
            const float angle = (float)pos * freq;
            const float c = cosf(angle), s = sinf(angle);
            const float a = out[h0 + i], b = out[h0 + i + half];
            out[h0 + i] = a * c - b * s;
            out[h0 + i + half] = b * c + a * s;
        }
    }
}

/* FeedForwardNetwork (src/inference.cpp:993-1015). */
void q3o_ffn(float* out, float* lin1, float* lin2, const float* x, const uint16_t* w1,
             const uint16_t* w2, const uint16_t* w3, int hidden_dim, int dim) {
    q3o_matmul(lin1, x, w1, hidden_dim, dim);
    q3o_matmul(lin2, x, w3, hidden_dim, dim);
    for (int i = 0; i < hidden_dim; ++i) lin1[i] = q3o_silu(lin1[i]) * lin2[i];
    q3o_matmul(out, lin1, w2, dim, hidden_dim);
}

/* FastAttn (src/inference.cpp:1017-1058) for one query head; k/v point at the head's first
 * element in a [kv_len, n_kv_heads*head_dim] bf16 cache. */
void q3o_attn(float* out, float* atth, const float* q, const uint16_t* k, const uint16_t* v,
              int head_dim, int n_kv_heads, int kv_len) {
    const int stride = n_kv_heads * head_dim;
    const float sq = sqrtf((float)head_dim);
    for (int i = 0; i < kv_len; ++i) atth[i] = dot_bf16(k + (size_t)i * stride, q, head_dim) / sq;
    q3o_softmax(atth, atth, kv_len);
    for (int i = 0; i < head_dim; ++i) out[i] = 0.0f;
    for (int t = 0; t < kv_len; ++t) {
        const float p = atth[t];
        const uint16_t* vr = v + (size_t)t * stride;
        for (int i = 0; i < head_dim; ++i) out[i] = bf2f(vr[i]) * p + out[i];
    }
}

/* Sampler::Greedy (src/inference.cpp:703-709): first index of the maximum. */
int q3o_greedy(const float* logits, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (logits[best] < logits[i]) best = i;
    return best;
}

/* ------------------------------------------------------------------ block */

typedef struct {
    int dim, hidden_dim, head_dim, n_heads, n_kv_heads, max_seq_len, rotary_dim;
    float rope_theta, norm_eps;
} q3o_cfg;

/* Weight order: attn_norm q_norm k_norm wq wk wv wo mlp_norm w1 w2 w3 (BlockWeights,
 * include/inference.h:163-176). Pointers are borrowed, not copied. */
typedef struct {
    q3o_cfg c;
    const uint16_t* w[11];
    uint16_t* k_cache; /* [max_seq_len, n_kv_heads*head_dim] */
    uint16_t* v_cache;
    float *norm, *q, *k, *v, *att, *proj, *scores, *lin1, *lin2;
} q3o_block;

q3o_block* q3o_block_create(const q3o_cfg* c, const uint16_t* const* w) {
    q3o_block* b = (q3o_block*)calloc(1, sizeof(q3o_block));
    b->c = *c;
    memcpy(b->w, w, sizeof(b->w));
    const size_t qd = (size_t)c->n_heads * c->head_dim, kvd = (size_t)c->n_kv_heads * c->head_dim;
    b->k_cache = (uint16_t*)calloc((size_t)c->max_seq_len * kvd, 2);
    b->v_cache = (uint16_t*)calloc((size_t)c->max_seq_len * kvd, 2);
    b->norm = (float*)calloc(c->dim, 4);
    b->q = (float*)calloc(qd, 4);
    b->k = (float*)calloc(kvd, 4);
    b->v = (float*)calloc(kvd, 4);
    b->att = (float*)calloc(qd, 4);
    b->proj = (float*)calloc(c->dim, 4);
    b->scores = (float*)calloc((size_t)c->n_heads * c->max_seq_len, 4);
    b->lin1 = (float*)calloc(c->hidden_dim, 4);
    b->lin2 = (float*)calloc(c->hidden_dim, 4);
    return b;
}

void q3o_block_free(q3o_block* b) {
    if (!b) return;
    free(b->k_cache); free(b->v_cache); free(b->norm); free(b->q); free(b->k); free(b->v);
    free(b->att); free(b->proj); free(b->scores); free(b->lin1); free(b->lin2);
    free(b);
}

/* Block::ResetCache (src/inference.cpp:732-735). */
void q3o_block_reset(q3o_block* b) {
    const size_t n = (size_t)b->c.max_seq_len * b->c.n_kv_heads * b->c.head_dim;
    memset(b->k_cache, 0, n * 2);
    memset(b->v_cache, 0, n * 2);
}

uint16_t* q3o_block_k_cache(q3o_block* b) { return b->k_cache; }
uint16_t* q3o_block_v_cache(q3o_block* b) { return b->v_cache; }

/* Block::forward (src/inference.cpp:766-866). */
int q3o_block_forward(q3o_block* b, float* x, int pos, int num_sink, int kv_pos, int kv_len) {
    const q3o_cfg* c = &b->c;
    if (!x) return Q3O_INVALID_ARGUMENT;
    if (pos < 0 || kv_len <= 0 || kv_len > c->max_seq_len || kv_pos < 0 || kv_pos >= kv_len ||
        num_sink < 0 || num_sink > kv_len || num_sink >= c->max_seq_len || kv_pos < num_sink)
        return Q3O_OUT_OF_RANGE;
    const int hd = c->head_dim, qd = c->n_heads * hd, kvd = c->n_kv_heads * hd;
    const uint16_t *attn_norm = b->w[0], *q_norm = b->w[1], *k_norm = b->w[2], *wq = b->w[3],
                   *wk = b->w[4], *wv = b->w[5], *wo = b->w[6], *mlp_norm = b->w[7],
                   *w1 = b->w[8], *w2 = b->w[9], *w3 = b->w[10];

    q3o_rmsnorm(b->norm, x, attn_norm, c->norm_eps, c->dim);
    q3o_matmul(b->q, b->norm, wq, qd, c->dim);
    q3o_matmul(b->k, b->norm, wk, kvd, c->dim);
    q3o_matmul(b->v, b->norm, wv, kvd, c->dim);
    for (int h = 0; h < c->n_heads; ++h)
        q3o_rmsnorm(b->q + h * hd, b->q + h * hd, q_norm, c->norm_eps, hd);
    for (int h = 0; h < c->n_kv_heads; ++h)
        q3o_rmsnorm(b->k + h * hd, b->k + h * hd, k_norm, c->norm_eps, hd);
    q3o_rope(b->q, qd, hd, pos, c->rope_theta, c->rotary_dim);
    q3o_rope(b->k, kvd, hd, pos, c->rope_theta, c->rotary_dim);

    for (int i = 0; i < kvd; ++i) {
        b->k_cache[(size_t)kv_pos * kvd + i] = f2bf(b->k[i]);
        b->v_cache[(size_t)kv_pos * kvd + i] = f2bf(b->v[i]);
    }
    /* Sink re-rotation once the ring buffer has wrapped (src/inference.cpp:817-827). */
    for (int s = 0; s < num_sink; ++s) {
        for (int i = 0; i < kvd; ++i) b->k[i] = bf2f(b->k_cache[(size_t)s * kvd + i]);
        q3o_rope(b->k, kvd, hd, 1, c->rope_theta, c->rotary_dim);
        for (int i = 0; i < kvd; ++i) b->k_cache[(size_t)s * kvd + i] = f2bf(b->k[i]);
    }

    const int per_kv = c->n_heads / c->n_kv_heads;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < c->n_heads; ++h) {
        const int g = h / per_kv;
        q3o_attn(b->att + h * hd, b->scores + (size_t)h * c->max_seq_len, b->q + h * hd,
                 b->k_cache + g * hd, b->v_cache + g * hd, hd, c->n_kv_heads, kv_len);
    }

    q3o_matmul(b->proj, b->att, wo, c->dim, qd);
    for (int i = 0; i < c->dim; ++i) x[i] += b->proj[i];

    q3o_rmsnorm(b->norm, x, mlp_norm, c->norm_eps, c->dim);
    q3o_ffn(b->proj, b->lin1, b->lin2, b->norm, w1, w2, w3, c->hidden_dim, c->dim);
    for (int i = 0; i < c->dim; ++i) x[i] += b->proj[i];
    return Q3O_OK;
}

/* ------------------------------------------------------------------ model */

typedef struct {
    q3o_cfg c;
    int n_layers, vocab_size;
    const uint16_t* embed;      /* [vocab, dim], also the tied classifier */
    const uint16_t* final_norm; /* [dim] */
    q3o_block** blocks;
    float *hidden, *normed, *logits;
} q3o_model;

/* layer_w: n_layers * 11 pointers in BlockWeights order; c->max_seq_len is the runtime
 * context (Qwen3::InitializeInference overwrites it, src/inference.cpp:534). */
q3o_model* q3o_model_create(const q3o_cfg* c, int n_layers, int vocab_size,
                            const uint16_t* embed, const uint16_t* final_norm,
                            const uint16_t* const* layer_w) {
    q3o_model* m = (q3o_model*)calloc(1, sizeof(q3o_model));
    m->c = *c;
    m->n_layers = n_layers;
    m->vocab_size = vocab_size;
    m->embed = embed;
    m->final_norm = final_norm;
    m->blocks = (q3o_block**)calloc(n_layers, sizeof(q3o_block*));
    for (int l = 0; l < n_layers; ++l) m->blocks[l] = q3o_block_create(c, layer_w + 11 * l);
    m->hidden = (float*)calloc(c->dim, 4);
    m->normed = (float*)calloc(c->dim, 4);
    m->logits = (float*)calloc(vocab_size, 4);
    return m;
}

void q3o_model_free(q3o_model* m) {
    if (!m) return;
    for (int l = 0; l < m->n_layers; ++l) q3o_block_free(m->blocks[l]);
    free(m->blocks); free(m->hidden); free(m->normed); free(m->logits);
    free(m);
}

/* Qwen3::ResetInference (src/inference.cpp:583-590). */
void q3o_model_reset(q3o_model* m) {
    for (int l = 0; l < m->n_layers; ++l) q3o_block_reset(m->blocks[l]);
    memset(m->hidden, 0, m->c.dim * 4);
    memset(m->normed, 0, m->c.dim * 4);
    memset(m->logits, 0, (size_t)m->vocab_size * 4);
}

/* Attention-sink / ring-buffer position math (src/inference.cpp:605-613). */
void q3o_positions(int pos, int ctx, int* num_sink, int* kv_pos, int* kv_len) {
    const int sinks = 4;
    *num_sink = pos >= ctx ? (sinks < ctx - 1 ? sinks : ctx - 1) : 0;
    *kv_pos = pos < ctx ? pos : *num_sink + (pos - *num_sink) % (ctx - *num_sink);
    *kv_len = pos + 1 < ctx ? pos + 1 : ctx;
}

/* Qwen3::ForwardToken (src/inference.cpp:592-637). hidden_layers (nullable) receives the
 * embedding row and the hidden state after every layer: [(n_layers+1), dim]. */
int q3o_model_forward(q3o_model* m, int token, int pos, float* hidden_layers, float* logits) {
    const q3o_cfg* c = &m->c;
    if (token < 0 || token >= m->vocab_size) return Q3O_OUT_OF_RANGE;
    if (pos < 0) return Q3O_OUT_OF_RANGE;
    const uint16_t* row = m->embed + (size_t)token * c->dim;
    for (int i = 0; i < c->dim; ++i) m->hidden[i] = bf2f(row[i]);
    int num_sink, kv_pos, kv_len;
    q3o_positions(pos, c->max_seq_len, &num_sink, &kv_pos, &kv_len);
    if (hidden_layers) memcpy(hidden_layers, m->hidden, (size_t)c->dim * 4);
    for (int l = 0; l < m->n_layers; ++l) {
        int st = q3o_block_forward(m->blocks[l], m->hidden, pos, num_sink, kv_pos, kv_len);
        if (st) return st;
        if (hidden_layers) memcpy(hidden_layers + (size_t)(l + 1) * c->dim, m->hidden, (size_t)c->dim * 4);
    }
    q3o_rmsnorm(m->normed, m->hidden, m->final_norm, c->norm_eps, c->dim);
    q3o_matmul(m->logits, m->normed, m->embed, m->vocab_size, c->dim);
    if (logits) memcpy(logits, m->logits, (size_t)m->vocab_size * 4);
    return Q3O_OK;
}

int q3o_model_kv_row(q3o_model* m, int layer, int kv_pos, uint16_t* k, uint16_t* v) {
    if (layer < 0 || layer >= m->n_layers || kv_pos < 0 || kv_pos >= m->c.max_seq_len)
        return Q3O_OUT_OF_RANGE;
    const size_t kvd = (size_t)m->c.n_kv_heads * m->c.head_dim;
    memcpy(k, m->blocks[layer]->k_cache + (size_t)kv_pos * kvd, kvd * 2);
    memcpy(v, m->blocks[layer]->v_cache + (size_t)kv_pos * kvd, kvd * 2);
    return Q3O_OK;
}
