/* CPU restatement of the GGUF llama / qwen2 forward -- TEST INFRASTRUCTURE ONLY.
 *
 * The reference's GGUF path runs llama.cpp b4514 (commit ec7f3ac9, not vendored and
 * not available offline) with only the matmuls offloaded to the bridge.  This file
 * restates that graph for the two architectures from llama.cpp's public behaviour:
 *   - inp = dequant(token_embd[token])
 *   - per layer: cur = rms_norm(inp, eps) * attn_norm; q/k/v = W*cur (+bias for qwen2);
 *     RoPE on q and k with theta_i = pos * base^(-2i/head_dim) / freq_factor[i]
 *     (interleaved pairs (2i, 2i+1) for llama, split-half pairs (i, i+d/2) for qwen2);
 *     causal soft-max(q.k / sqrt(head_dim)) over positions 0..pos, weighted V,
 *     grouped queries (head h uses KV head h / (heads/kv_heads));
 *     inp += Wo*attn; cur = rms_norm(inp) * ffn_norm; inp += Wd*(silu(Wg*cur) * (Wu*cur))
 *   - logits = token_embd * (rms_norm(inp) * output_norm)  (tied embeddings)
 * in fp32 with weights dequantised exactly (gguf_oracle.c).  llama.cpp's own CPU
 * path quantises activations to Q8_K for its dot products; this restatement keeps
 * fp32 activations, like the bridge does.  Parity with llama.cpp itself is unpinned.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gguf_oracle.h"

typedef struct {
    int type;  /* 0 = F32, else ggml quant id */
    int rows, cols;
    const void *data;
} go_tensor;

typedef struct {
    int layers, dim, heads, kv_heads, head_dim, ffn, vocab, context, neox;
    float eps, rope_base;
    go_tensor embd, out_norm, rope_freqs; /* rope_freqs.data may be NULL */
    const go_tensor *attn_norm, *wq, *wk, *wv, *bq, *bk, *bv, *wo, *ffn_norm, *wg, *wu, *wd; /* [layers] */
} go_model;

typedef struct {
    go_model m;
    float *kc, *vc; /* [layer][kv_head][pos][head_dim] */
    float *x, *xn, *q, *k, *v, *att, *g, *u, *row, *score;
} go_state;

static void rms_norm(const float *x, const float *g, int n, float eps, float *y)
{
    float sum = 0;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    const float s = 1.0f / sqrtf(sum / n + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * s * g[i];
}

/* y[r] (+)= dequant(W[r]) . x, rows in parallel */
static void matvec(const go_tensor *w, const float *x, float *y, int add)
{
    const unsigned rb = gguf_o_row_bytes(w->type, w->cols);
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)w->cols);
#pragma omp for schedule(static)
        for (int r = 0; r < w->rows; r++) {
            gguf_o_dequant_row(w->type, (const uint8_t *)w->data + (size_t)r * rb, w->cols, row);
            float sum = 0;
            for (int c = 0; c < w->cols; c++) sum += row[c] * x[c];
            y[r] = add ? y[r] + sum : sum;
        }
        free(row);
    }
}

go_state *go_create(const go_model *m)
{
    go_state *s = (go_state *)calloc(1, sizeof *s);
    if (!s) return NULL;
    s->m = *m;
    const size_t kv = (size_t)m->layers * m->kv_heads * m->context * m->head_dim;
    s->kc = (float *)calloc(kv, sizeof(float));
    s->vc = (float *)calloc(kv, sizeof(float));
    const int kvd = m->kv_heads * m->head_dim;
    s->x = (float *)calloc(m->dim, sizeof(float));
    s->xn = (float *)calloc(m->dim, sizeof(float));
    s->q = (float *)calloc(m->dim, sizeof(float));
    s->k = (float *)calloc(kvd, sizeof(float));
    s->v = (float *)calloc(kvd, sizeof(float));
    s->att = (float *)calloc(m->dim, sizeof(float));
    s->g = (float *)calloc(m->ffn, sizeof(float));
    s->u = (float *)calloc(m->ffn, sizeof(float));
    s->row = (float *)calloc(m->dim > m->ffn ? m->dim : m->ffn, sizeof(float));
    s->score = (float *)calloc(m->context, sizeof(float));
    return s;
}

void go_destroy(go_state *s)
{
    if (!s) return;
    float *p[] = {s->kc, s->vc, s->x, s->xn, s->q, s->k, s->v, s->att, s->g, s->u, s->row, s->score};
    for (unsigned i = 0; i < sizeof p / sizeof p[0]; i++) free(p[i]);
    free(s);
}

static void rope(float *vec, int heads, int head_dim, int neox, int pos, float base, const float *ff)
{
    const int half = head_dim / 2;
    for (int h = 0; h < heads; h++)
        for (int i = 0; i < half; i++) {
            const float theta = pos * powf(base, -2.0f * i / head_dim) / (ff ? ff[i] : 1.0f);
            const float cs = cosf(theta), sn = sinf(theta);
            const int a = h * head_dim + (neox ? i : 2 * i), b = neox ? a + half : a + 1;
            const float x0 = vec[a], x1 = vec[b];
            vec[a] = x0 * cs - x1 * sn;
            vec[b] = x0 * sn + x1 * cs;
        }
}

/* one step; logits (vocab floats) filled when non-NULL */
void go_forward(go_state *s, int token, int pos, float *logits)
{
    const go_model *m = &s->m;
    const int dim = m->dim, hd = m->head_dim, kvd = m->kv_heads * hd, group = m->heads / m->kv_heads;
    const float *ff = (const float *)m->rope_freqs.data;
    gguf_o_dequant_row(m->embd.type,
                       (const uint8_t *)m->embd.data + (size_t)token * gguf_o_row_bytes(m->embd.type, dim), dim, s->x);
    for (int l = 0; l < m->layers; l++) {
        rms_norm(s->x, (const float *)m->attn_norm[l].data, dim, m->eps, s->xn);
        matvec(&m->wq[l], s->xn, s->q, 0);
        matvec(&m->wk[l], s->xn, s->k, 0);
        matvec(&m->wv[l], s->xn, s->v, 0);
        if (m->bq && m->bq[l].data) {
            const float *bq = (const float *)m->bq[l].data, *bk = (const float *)m->bk[l].data,
                        *bv = (const float *)m->bv[l].data;
            for (int i = 0; i < dim; i++) s->q[i] += bq[i];
            for (int i = 0; i < kvd; i++) {
                s->k[i] += bk[i];
                s->v[i] += bv[i];
            }
        }
        rope(s->q, m->heads, hd, m->neox, pos, m->rope_base, ff);
        rope(s->k, m->kv_heads, hd, m->neox, pos, m->rope_base, ff);
        for (int kh = 0; kh < m->kv_heads; kh++) {
            const size_t o = (((size_t)l * m->kv_heads + kh) * m->context + pos) * hd;
            memcpy(s->kc + o, s->k + kh * hd, sizeof(float) * hd);
            memcpy(s->vc + o, s->v + kh * hd, sizeof(float) * hd);
        }
        const float scale = 1.0f / sqrtf((float)hd);
        for (int h = 0; h < m->heads; h++) {
            const int kh = h / group;
            const float *kb = s->kc + ((size_t)l * m->kv_heads + kh) * m->context * hd;
            const float *vb = s->vc + ((size_t)l * m->kv_heads + kh) * m->context * hd;
            float mx = -INFINITY;
            for (int p = 0; p <= pos; p++) {
                float z = 0;
                for (int d = 0; d < hd; d++) z += s->q[h * hd + d] * kb[(size_t)p * hd + d];
                s->score[p] = z * scale;
                if (s->score[p] > mx) mx = s->score[p];
            }
            float total = 0;
            for (int p = 0; p <= pos; p++) {
                s->score[p] = expf(s->score[p] - mx);
                total += s->score[p];
            }
            for (int d = 0; d < hd; d++) {
                float z = 0;
                for (int p = 0; p <= pos; p++) z += s->score[p] * vb[(size_t)p * hd + d];
                s->att[h * hd + d] = z / total;
            }
        }
        matvec(&m->wo[l], s->att, s->x, 1);
        rms_norm(s->x, (const float *)m->ffn_norm[l].data, dim, m->eps, s->xn);
        matvec(&m->wg[l], s->xn, s->g, 0);
        matvec(&m->wu[l], s->xn, s->u, 0);
        for (int i = 0; i < m->ffn; i++) s->g[i] = (s->g[i] / (1.0f + expf(-s->g[i]))) * s->u[i];
        matvec(&m->wd[l], s->g, s->x, 1);
    }
    if (logits) {
        rms_norm(s->x, (const float *)m->out_norm.data, dim, m->eps, s->xn);
        matvec(&m->embd, s->xn, logits, 0);
    }
}
