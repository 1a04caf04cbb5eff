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
#include <immintrin.h>
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

/* ------------------------------------------------------------------ many tokens at once
 *
 * The oracle for long prompts: ForwardToken over tokens[0..n) at positions pos0.. run layer by
 * layer over all the tokens instead of token by token. Every value is computed by the same
 * functions in the same order as q3o_model_forward computes it for that token (each dot product
 * is dot_bf16 over the same operands; token t attends to cache rows 0..pos0+t, which hold the same
 * bf16 values either way), so the results are bit-identical to n calls of q3o_model_forward;
 * only the loop order differs, which lets the weights be reused from cache across tokens. The
 * ring buffer must not wrap (pos0 + n <= context). */

/* dot_bf16 of one weight row with four activation vectors at once, written with AVX2 lanes:
 * lane l of the low / high accumulator is the scalar code's lo[l] / hi[l] (the same fmaf chain
 * in the same order), followed by the same reduction, so each result equals dot_bf16's bit for
 * bit. m % 16 == 0. */
static inline __m256 bf16x8_to_f32(const uint16_t* p) {
    const __m128i h = _mm_loadu_si128((const __m128i*)p);
    return _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(h), 16));
}
static inline float reduce_lanes(__m256 lo, __m256 hi) {
    float s[8];
    _mm256_storeu_ps(s, _mm256_add_ps(lo, hi));
    return reduce8(s);
}
static void dot4_bf16(const uint16_t* w, const float* x0, const float* x1, const float* x2,
                      const float* x3, int m, float* o) {
    __m256 l0 = _mm256_setzero_ps(), h0 = l0, l1 = l0, h1 = l0, l2 = l0, h2 = l0, l3 = l0, h3 = l0;
    for (int j = 0; j < m; j += 16) {
        const __m256 wl = bf16x8_to_f32(w + j), wh = bf16x8_to_f32(w + j + 8);
        l0 = _mm256_fmadd_ps(wl, _mm256_loadu_ps(x0 + j), l0);
        h0 = _mm256_fmadd_ps(wh, _mm256_loadu_ps(x0 + j + 8), h0);
        l1 = _mm256_fmadd_ps(wl, _mm256_loadu_ps(x1 + j), l1);
        h1 = _mm256_fmadd_ps(wh, _mm256_loadu_ps(x1 + j + 8), h1);
        l2 = _mm256_fmadd_ps(wl, _mm256_loadu_ps(x2 + j), l2);
        h2 = _mm256_fmadd_ps(wh, _mm256_loadu_ps(x2 + j + 8), h2);
        l3 = _mm256_fmadd_ps(wl, _mm256_loadu_ps(x3 + j), l3);
        h3 = _mm256_fmadd_ps(wh, _mm256_loadu_ps(x3 + j + 8), h3);
    }
    o[0] = reduce_lanes(l0, h0);
    o[1] = reduce_lanes(l1, h1);
    o[2] = reduce_lanes(l2, h2);
    o[3] = reduce_lanes(l3, h3);
}

/* out[t * ldo + i] = dot_bf16(W row i, x + t * ldx) for t < n, i < rows. */
static void matmul_many(float* out, int ldo, const float* x, int ldx, const uint16_t* w, int rows,
                        int m, int n) {
    const int RB = 32, TB = 64;
    const int nrb = (rows + RB - 1) / RB, ntb = (n + TB - 1) / TB;
#pragma omp parallel for schedule(dynamic) collapse(2)
    for (int tb = 0; tb < ntb; ++tb) {
        for (int rb = 0; rb < nrb; ++rb) {
            const int t1 = (tb + 1) * TB < n ? (tb + 1) * TB : n;
            const int r1 = (rb + 1) * RB < rows ? (rb + 1) * RB : rows;
            int t = tb * TB;
            if (m % 16 == 0) {
                for (; t + 4 <= t1; t += 4) {
                    const float* xt = x + (size_t)t * ldx;
                    for (int i = rb * RB; i < r1; ++i) {
                        float o[4];
                        dot4_bf16(w + (size_t)i * m, xt, xt + ldx, xt + 2 * (size_t)ldx,
                                  xt + 3 * (size_t)ldx, m, o);
                        for (int k = 0; k < 4; ++k) out[(size_t)(t + k) * ldo + i] = o[k];
                    }
                }
            }
            for (; t < t1; ++t)
                for (int i = rb * RB; i < r1; ++i)
                    out[(size_t)t * ldo + i] = dot_bf16(w + (size_t)i * m, x + (size_t)t * ldx, m);
        }
    }
}

/* hidden_last (nullable): [(n_layers + 1), dim] of the last token (as q3o_model_forward's
 * hidden_layers). want (nullable, n flags): tokens whose logits are computed; logits_out
 * receives them in token order ([count of flagged tokens, vocab]) and argmax_out[t] their greedy
 * token (-1 for tokens not flagged). */
int q3o_model_prefill(q3o_model* m, const int* tokens, int n, int pos0, const unsigned char* want,
                      float* logits_out, int* argmax_out, float* hidden_last) {
    const q3o_cfg* c = &m->c;
    if (n <= 0 || pos0 < 0 || pos0 + n > c->max_seq_len) return Q3O_OUT_OF_RANGE;
    for (int t = 0; t < n; ++t)
        if (tokens[t] < 0 || tokens[t] >= m->vocab_size) return Q3O_OUT_OF_RANGE;
    const int D = c->dim, hd = c->head_dim, qd = c->n_heads * hd, kvd = c->n_kv_heads * hd;
    const int Hd = c->hidden_dim, per_kv = c->n_heads / c->n_kv_heads;
    float* X = (float*)malloc((size_t)n * D * 4);
    float* N = (float*)malloc((size_t)n * D * 4);
    float* Q = (float*)malloc((size_t)n * qd * 4);
    float* K = (float*)malloc((size_t)n * kvd * 4);
    float* V = (float*)malloc((size_t)n * kvd * 4);
    float* A = (float*)malloc((size_t)n * qd * 4);
    float* P = (float*)malloc((size_t)n * D * 4);
    float* L1 = (float*)malloc((size_t)n * Hd * 4);
    float* L2 = (float*)malloc((size_t)n * Hd * 4);
    if (!X || !N || !Q || !K || !V || !A || !P || !L1 || !L2) {
        free(X); free(N); free(Q); free(K); free(V); free(A); free(P); free(L1); free(L2);
        return Q3O_INVALID_ARGUMENT;
    }
    for (int t = 0; t < n; ++t) {
        const uint16_t* row = m->embed + (size_t)tokens[t] * D;
        for (int i = 0; i < D; ++i) X[(size_t)t * D + i] = bf2f(row[i]);
    }
    if (hidden_last) memcpy(hidden_last, X + (size_t)(n - 1) * D, (size_t)D * 4);
    for (int l = 0; l < m->n_layers; ++l) {
        q3o_block* b = m->blocks[l];
        const uint16_t *attn_norm = b->w[0], *q_norm = b->w[1], *k_norm = b->w[2], *wq = b->w[3],
                       *wk = b->w[4], *wv = b->w[5], *wo = b->w[6], *mlp_norm = b->w[7],
                       *w1 = b->w[8], *w2 = b->w[9], *w3 = b->w[10];
#pragma omp parallel for schedule(static)
        for (int t = 0; t < n; ++t)
            q3o_rmsnorm(N + (size_t)t * D, X + (size_t)t * D, attn_norm, c->norm_eps, D);
        matmul_many(Q, qd, N, D, wq, qd, D, n);
        matmul_many(K, kvd, N, D, wk, kvd, D, n);
        matmul_many(V, kvd, N, D, wv, kvd, D, n);
#pragma omp parallel for schedule(static)
        for (int t = 0; t < n; ++t) {
            float* q = Q + (size_t)t * qd;
            float* k = K + (size_t)t * kvd;
            const float* v = V + (size_t)t * kvd;
            for (int h = 0; h < c->n_heads; ++h) q3o_rmsnorm(q + h * hd, q + h * hd, q_norm, c->norm_eps, hd);
            for (int h = 0; h < c->n_kv_heads; ++h) q3o_rmsnorm(k + h * hd, k + h * hd, k_norm, c->norm_eps, hd);
            q3o_rope(q, qd, hd, pos0 + t, c->rope_theta, c->rotary_dim);
            q3o_rope(k, kvd, hd, pos0 + t, c->rope_theta, c->rotary_dim);
            const size_t kv_pos = (size_t)(pos0 + t);
            for (int i = 0; i < kvd; ++i) {
                b->k_cache[kv_pos * kvd + i] = f2bf(k[i]);
                b->v_cache[kv_pos * kvd + i] = f2bf(v[i]);
            }
        }
#pragma omp parallel
        {
            float* sc = (float*)malloc((size_t)(pos0 + n) * 4);
#pragma omp for schedule(dynamic) collapse(2)
            for (int t = 0; t < n; ++t) {
                for (int h = 0; h < c->n_heads; ++h) {
                    const int g = h / per_kv;
                    q3o_attn(A + (size_t)t * qd + h * hd, sc, Q + (size_t)t * qd + h * hd,
                             b->k_cache + g * hd, b->v_cache + g * hd, hd, c->n_kv_heads, pos0 + t + 1);
                }
            }
            free(sc);
        }
        matmul_many(P, D, A, qd, wo, D, qd, n);
#pragma omp parallel for schedule(static)
        for (int t = 0; t < n; ++t) {
            float* x = X + (size_t)t * D;
            const float* p = P + (size_t)t * D;
            for (int i = 0; i < D; ++i) x[i] += p[i];
            q3o_rmsnorm(N + (size_t)t * D, x, mlp_norm, c->norm_eps, D);
        }
        matmul_many(L1, Hd, N, D, w1, Hd, D, n);
        matmul_many(L2, Hd, N, D, w3, Hd, D, n);
#pragma omp parallel for schedule(static)
        for (int t = 0; t < n; ++t)
            for (int i = 0; i < Hd; ++i)
                L1[(size_t)t * Hd + i] = q3o_silu(L1[(size_t)t * Hd + i]) * L2[(size_t)t * Hd + i];
        matmul_many(P, D, L1, Hd, w2, D, Hd, n);
#pragma omp parallel for schedule(static)
        for (int t = 0; t < n; ++t) {
            float* x = X + (size_t)t * D;
            const float* p = P + (size_t)t * D;
            for (int i = 0; i < D; ++i) x[i] += p[i];
        }
        if (hidden_last) memcpy(hidden_last + (size_t)(l + 1) * D, X + (size_t)(n - 1) * D, (size_t)D * 4);
    }
    /* Final RmsNorm and the tied lm_head of the flagged tokens, in chunks of 64 tokens. */
    const int CH = 64;
    float* lg = (float*)malloc((size_t)CH * m->vocab_size * 4);
    int* idx = (int*)malloc((size_t)CH * sizeof(int));
    size_t emitted = 0;
    for (int t0 = 0; t0 < n && lg && idx; t0 += CH) {
        int cnt = 0;
        for (int t = t0; t < n && t < t0 + CH; ++t) {
            if (argmax_out) argmax_out[t] = -1;
            if (!want || want[t]) {
                q3o_rmsnorm(N + (size_t)cnt * D, X + (size_t)t * D, m->final_norm, c->norm_eps, D);
                idx[cnt++] = t;
            }
        }
        if (!cnt) continue;
        matmul_many(lg, m->vocab_size, N, D, m->embed, m->vocab_size, D, cnt);
        for (int j = 0; j < cnt; ++j) {
            const float* row = lg + (size_t)j * m->vocab_size;
            if (argmax_out) argmax_out[idx[j]] = q3o_greedy(row, m->vocab_size);
            if (logits_out) memcpy(logits_out + emitted * m->vocab_size, row, (size_t)m->vocab_size * 4);
            ++emitted;
        }
    }
    const int ok = lg && idx;
    free(lg); free(idx);
    free(X); free(N); free(Q); free(K); free(V); free(A); free(P); free(L1); free(L2);
    return ok ? Q3O_OK : Q3O_INVALID_ARGUMENT;
}

int q3o_model_kv_row(q3o_model* m, int layer, int kv_pos, uint16_t* k, uint16_t* v) {
    if (layer < 0 || layer >= m->n_layers || kv_pos < 0 || kv_pos >= m->c.max_seq_len)
        return Q3O_OUT_OF_RANGE;
    const size_t kvd = (size_t)m->c.n_kv_heads * m->c.head_dim;
    memcpy(k, m->blocks[layer]->k_cache + (size_t)kv_pos * kvd, kvd * 2);
    memcpy(v, m->blocks[layer]->v_cache + (size_t)kv_pos * kvd, kvd * 2);
    return Q3O_OK;
}
