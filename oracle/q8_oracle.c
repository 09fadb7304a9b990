/* CPU restatement of the reference grouped-Q8 engine -- TEST INFRASTRUCTURE ONLY.
 *
 * Follows src/minimind.cpp (the reference's own CPU path) operation by operation so
 * that, built with -ffp-contract=off like the reference (tools/build-minimind.sh:9),
 * every float result is bit-identical to the reference's cpu().  The summation
 * orders, the float/int promotions and the libm calls (powf, cosf, sinf, expf,
 * sqrtf) are therefore the reference's; the code structure is this project's.
 * Only tests/, the smoke check and bench.py's CPU-baseline leg use this file.
 */
#include "q8_oracle.h"

#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define RMS_EPS 1e-6f

struct q8o_model {
    const uint8_t *base;
    size_t bytes;
    const q8o_tensor *t;
    float *keys;   /* [layer][pos][128], post-RoPE keys (src/minimind.cpp:53,65-66) */
    float *values; /* [layer][pos][128] (src/minimind.cpp:68) */
};

static const int8_t *q8_data(const q8o_model *m, q8o_tensor t) { return (const int8_t *)(m->base + t.data); }
static const float *f32_data(const q8o_model *m, uint32_t off) { return (const float *)(m->base + off); }

q8o_model *q8o_create(const void *file, size_t bytes)
{
    /* header checks of src/minimind.cpp:89-93 */
    const uint32_t *h = (const uint32_t *)file;
    if (bytes < Q8O_HEADER_BYTES || h[0] != 0x384D4D4Du || h[1] != 1 || h[2] != (uint32_t)bytes ||
        h[3] != Q8O_DIM || h[4] != Q8O_HIDDEN || h[5] != Q8O_LAYERS || h[6] != Q8O_VOCAB || h[7] != 64)
        return NULL;
    const q8o_tensor *t = (const q8o_tensor *)(h + 8);
    for (int i = 0; i < Q8O_TENSORS; i++) {
        uint64_t size = (uint64_t)t[i].rows * (t[i].scales ? t[i].cols : 4);
        if (t[i].data < Q8O_HEADER_BYTES || t[i].data + size > bytes) return NULL;
        if (t[i].scales && (t[i].cols % 64 || t[i].scales + size / 64 * 4 > bytes)) return NULL;
    }
    q8o_model *m = (q8o_model *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->base = (const uint8_t *)file;
    m->bytes = bytes;
    m->t = t;
    size_t kv = (size_t)Q8O_LAYERS * Q8O_CONTEXT * Q8O_KV;
    m->keys = (float *)calloc(kv, sizeof(float));
    m->values = (float *)calloc(kv, sizeof(float));
    if (!m->keys || !m->values) { q8o_destroy(m); return NULL; }
    return m;
}

void q8o_destroy(q8o_model *m)
{
    if (!m) return;
    free(m->keys);
    free(m->values);
    free(m);
}

void q8o_reset(q8o_model *m)
{
    size_t kv = (size_t)Q8O_LAYERS * Q8O_CONTEXT * Q8O_KV;
    memset(m->keys, 0, kv * sizeof(float));
    memset(m->values, 0, kv * sizeof(float));
}

const q8o_tensor *q8o_tensors(const q8o_model *m) { return m->t; }
const uint8_t *q8o_base(const q8o_model *m) { return m->base; }

/* src/minimind.cpp:24-46, scalar branch (:40): a sequential 64-term float dot per
 * group, then sum += dot * scale, groups in order.  Rows are independent, so the
 * OpenMP split does not change any result. */
void q8o_matvec(const int8_t *w, const float *s, unsigned rows, unsigned cols,
                const float *x, float *y, int add, unsigned first)
{
    const unsigned groups = cols / 64;
#pragma omp parallel for schedule(static) if (rows - first > 256)
    for (long r = (long)first; r < (long)rows; r++) {
        float sum = 0;
        for (unsigned g = 0; g < groups; g++) {
            const size_t off = (size_t)r * cols + (size_t)g * 64;
            float dot = 0;
            for (int j = 0; j < 64; j++) dot += (float)w[off + j] * x[g * 64 + j];
            sum += dot * s[off / 64];
        }
        if (add) y[r] += sum;
        else y[r] = sum;
    }
}

/* src/minimind.cpp:47-50: sequential sum of squares, s = 1/sqrt(sum/n + eps),
 * y = (x*s)*g. */
void q8o_rmsnorm(const float *x, const float *gain, int n, float eps, float *y)
{
    float sum = 0;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    float s = 1 / sqrtf(sum / n + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * s * gain[i];
}

static void mat(const q8o_model *m, q8o_tensor t, const float *x, float *y, int add)
{
    q8o_matvec(q8_data(m, t), f32_data(m, t.scales), t.rows, t.cols, x, y, add, 0);
}

/* src/minimind.cpp:51-82 */
void q8o_forward(q8o_model *m, int token, int pos, int project, int hidden_only, float *out)
{
    enum { DIM = Q8O_DIM, HID = Q8O_HIDDEN, KV = Q8O_KV, CTX = Q8O_CONTEXT };
    static float x[DIM], n[DIM], q[DIM], k[KV], v[KV], a[CTX], gate[HID], up[HID];
    const q8o_tensor *t = m->t;

    /* embedding row dequant, src/minimind.cpp:23,55 */
    {
        const int8_t *e = q8_data(m, t[0]);
        const float *es = f32_data(m, t[0].scales);
        for (int i = 0; i < DIM; i++) {
            int idx = token * DIM + i;
            x[i] = e[idx] * es[idx / 64];
        }
    }
    for (int l = 0; l < Q8O_LAYERS; l++) {
        const int b = 1 + l * Q8O_STRIDE;
        const size_t layer_kv = (size_t)l * CTX * KV;
        q8o_rmsnorm(x, f32_data(m, t[b].data), DIM, RMS_EPS, n);
        mat(m, t[b + 1], n, q, 0);
        mat(m, t[b + 2], n, k, 0);
        mat(m, t[b + 3], n, v, 0);
        /* QKV bias, src/minimind.cpp:59-60 */
        const float *bq = f32_data(m, t[b + 9].data), *bk = f32_data(m, t[b + 10].data),
                    *bv = f32_data(m, t[b + 11].data);
        for (int i = 0; i < DIM; i++) q[i] += bq[i];
        for (int i = 0; i < KV; i++) { k[i] += bk[i]; v[i] += bv[i]; }
        /* split-half RoPE, src/minimind.cpp:62-67: pairs (i, i+32) per head,
         * angle = pos * 1e6^(-2i/64); keys of the two KV heads go to the cache. */
        for (int h = 0; h < DIM / 64; h++) {
            for (int i = 0; i < 32; i++) {
                float angle = pos * powf(1000000.f, -2.f * i / 64);
                float cs = cosf(angle), sn = sinf(angle);
                int j = h * 64 + i;
                float lo = q[j], hi = q[j + 32];
                q[j] = lo * cs - hi * sn;
                q[j + 32] = hi * cs + lo * sn;
                if (h < 2) {
                    lo = k[j];
                    hi = k[j + 32];
                    size_t o = layer_kv + (size_t)pos * KV + j;
                    m->keys[o] = lo * cs - hi * sn;
                    m->keys[o + 32] = hi * cs + lo * sn;
                }
            }
        }
        for (int i = 0; i < KV; i++) m->values[layer_kv + (size_t)pos * KV + i] = v[i];
        /* GQA attention with a two-pass softmax, src/minimind.cpp:69-75 */
        for (int h = 0; h < DIM / 64; h++) {
            const size_t kv_off = (size_t)(h / (DIM / KV)) * 64;
            float largest = -1e30f, total = 0;
            for (int s = 0; s <= pos; s++) {
                const float *key = m->keys + layer_kv + (size_t)s * KV + kv_off;
                float z = 0;
                for (int i = 0; i < 64; i++) z += q[h * 64 + i] * key[i];
                a[s] = z * .125f;
                if (largest < a[s]) largest = a[s];
            }
            for (int s = 0; s <= pos; s++) {
                a[s] = expf(a[s] - largest);
                total += a[s];
            }
            for (int i = 0; i < 64; i++) {
                float z = 0;
                for (int s = 0; s <= pos; s++)
                    z += (a[s] / total) * m->values[layer_kv + (size_t)s * KV + kv_off + i];
                n[h * 64 + i] = z;
            }
        }
        mat(m, t[b + 4], n, x, 1);
        q8o_rmsnorm(x, f32_data(m, t[b + 8].data), DIM, RMS_EPS, n);
        mat(m, t[b + 5], n, gate, 0);
        mat(m, t[b + 6], n, up, 0);
        /* SwiGLU, src/minimind.cpp:77 */
        for (int i = 0; i < HID; i++) gate[i] = (gate[i] / (1 + expf(-gate[i]))) * up[i];
        mat(m, t[b + 7], gate, x, 1);
    }
    if (project) {
        q8o_rmsnorm(x, f32_data(m, t[Q8O_TENSORS - 1].data), DIM, RMS_EPS, n);
        if (hidden_only) memcpy(out, n, sizeof n);
        else mat(m, t[0], n, out, 0);
    }
}

/* ---- sampling -------------------------------------------------------------- */

static const float *g_rank_logits;
/* ordering of src/minimind.cpp:173: larger value first, ties to the lower id */
static int rank_cmp(const void *pa, const void *pb)
{
    int a = *(const int *)pa, b = *(const int *)pb;
    float va = g_rank_logits[a], vb = g_rank_logits[b];
    if (va > vb) return -1;
    if (vb > va) return 1;
    return (a > b) - (a < b);
}

static void penalise(float *logits, float penalty)
{
    *logits = *logits < 0 ? *logits * penalty : *logits / penalty;
}

int q8o_sample(float *logits, int vocab, const int *history, int history_len, float penalty,
               float temp, int top_k, float top_p, uint32_t *seed, int skip_penalty)
{
    /* penalty on distinct ids of the last 64 history entries, src/minimind.cpp:160-164 */
    if (!skip_penalty) {
        unsigned char *seen = (unsigned char *)calloc((size_t)vocab, 1);
        for (int j = history_len > 64 ? history_len - 64 : 0; j < history_len; j++) {
            int id = history[j];
            if (!seen[id]) { penalise(&logits[id], penalty); seen[id] = 1; }
        }
        free(seen);
    }
    /* control-token mask, src/minimind.cpp:167 */
    for (int id = Q8O_CONTROL_FIRST; id < vocab; id++)
        if (id != Q8O_EOS) logits[id] = -1e30f;
    if (temp == 0) { /* first maximum, src/minimind.cpp:171 */
        int best = 0;
        for (int i = 1; i < vocab; i++)
            if (logits[best] < logits[i]) best = i;
        return best;
    }
    /* top-k, softmax with temperature, top-p cutoff, xorshift32 draw (:172-179) */
    int *order = (int *)malloc(sizeof(int) * (size_t)vocab);
    for (int i = 0; i < vocab; i++) order[i] = i;
    g_rank_logits = logits;
    qsort(order, (size_t)vocab, sizeof(int), rank_cmp);
    float largest = logits[order[0]], sum = 0;
    for (int j = 0; j < top_k; j++) {
        int i = order[j];
        logits[i] = expf((logits[i] - largest) / temp);
        sum += logits[i];
    }
    float cutoff = 0;
    int kept = 0;
    while (kept < top_k && cutoff < sum * top_p) cutoff += logits[order[kept++]];
    uint32_t s = *seed;
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    *seed = s;
    float r = (float)((s / 4294967296.0) * cutoff);
    int token = order[kept - 1];
    for (int j = 0; j < kept; j++) {
        int i = order[j];
        r -= logits[i];
        if (r <= 0) { token = i; break; }
    }
    free(order);
    return token;
}

/* src/minimind.cu:135-162 (64 partitions of ids b*128 + t + j*8192, t<128, j<19;
 * penalty on the first history match, control mask, k rounds of
 * (value desc, id asc) selection) and the host scatter of :193-194. */
int q8o_collect(const float *logits, float *out, const int *recent, int count, float penalty,
                int k, int rows)
{
    if (k < 1 || k > 64 || count < 0 || count > 64) return 1;
    enum { PARTS = 64, THREADS = 128, PER = 19, SLOTS = THREADS * PER };
    for (int i = 0; i < rows; i++) out[i] = -FLT_MAX;
    float *val = (float *)malloc(sizeof(float) * SLOTS);
    int *ids = (int *)malloc(sizeof(int) * SLOTS);
    for (int b = 0; b < PARTS; b++) {
        for (int t = 0; t < THREADS; t++) {
            for (int j = 0; j < PER; j++) {
                int id = b * THREADS + t + j * PARTS * THREADS;
                float v = id < rows ? logits[id] : -FLT_MAX;
                if (id < rows) {
                    for (int h = 0; h < count; h++)
                        if (recent[h] == id) { penalise(&v, penalty); break; }
                    if (id >= Q8O_CONTROL_FIRST && id != Q8O_EOS) v = -1e30f;
                }
                val[t * PER + j] = v;
                ids[t * PER + j] = id;
            }
        }
        for (int rank = 0; rank < k; rank++) {
            int best = -1;
            for (int i = 0; i < SLOTS; i++) {
                if (best < 0 || val[i] > val[best] || (val[i] == val[best] && ids[i] < ids[best])) best = i;
            }
            int id = ids[best];
            if (id >= 0 && id < rows) out[id] = val[best];
            val[best] = -FLT_MAX;
        }
    }
    free(val);
    free(ids);
    return 0;
}
