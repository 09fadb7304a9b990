/* CPU restatement of the reference GGUF bridge -- TEST INFRASTRUCTURE ONLY.
 *
 * Block formats are ggml's (MIT): Q8_0 = fp16 d + 32 int8 (34 B per 32 weights);
 * Q4_K = fp16 d, fp16 dmin, 12 B of packed 6-bit sub-block scales/mins, 128 B of
 * nibbles (144 B per 256); Q6_K = 128 B low nibbles, 64 B high 2-bit pairs,
 * 16 int8 scales, fp16 d (210 B per 256).  The value formulas follow the
 * reference's scalar `weight()` (src/gguf-cuda.cu:28-44), evaluated without
 * fused multiply-add as the reference builds with --fmad=false
 * (tools/build-gguf-cuda.sh:9): Q4_K (d*sc)*q - dmin*m, Q6_K (d*sc)*q, Q8_0 d*q. */
#include "gguf_oracle.h"

#include <stdlib.h>
#include <string.h>

/* exact binary16 -> binary32 including subnormals and inf/nan (src/gguf-cuda.cu:23-27) */
float gguf_o_half(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 0) {
        float f = (float)m * 5.9604644775390625e-8f; /* m * 2^-24 */
        return sign ? -f : f;
    }
    uint32_t bits = sign | ((e == 31 ? 255u : e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

unsigned gguf_o_row_bytes(int type, int cols)
{
    if (cols <= 0) return 0;
    switch (type) {
    case GGUF_O_Q8_0: return cols % 32 ? 0 : (unsigned)(cols / 32) * 34u;
    case GGUF_O_Q4_K: return cols % 256 ? 0 : (unsigned)(cols / 256) * 144u;
    case GGUF_O_Q6_K: return cols % 256 ? 0 : (unsigned)(cols / 256) * 210u;
    default: return 0;
    }
}

/* 6-bit scale and min of sub-block j (0..7) from the 12 packed bytes */
static void q4k_scale_min(const uint8_t *s, int j, unsigned *sc, unsigned *mn)
{
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (s[j + 4] & 15u) | ((unsigned)(s[j - 4] >> 6) << 4);
        *mn = (unsigned)(s[j + 4] >> 4) | ((unsigned)(s[j] >> 6) << 4);
    }
}

static void dequant_q4k_block(const uint8_t *p, float *y)
{
    const float d = gguf_o_half(rd16(p)), dmin = gguf_o_half(rd16(p + 2));
    for (int i = 0; i < 256; i++) {
        int j = i / 32;
        unsigned sc, mn;
        q4k_scale_min(p + 4, j, &sc, &mn);
        unsigned q = p[16 + (i / 64) * 32 + (i & 31)];
        q = (j & 1) ? q >> 4 : q & 15u;
        float a = d * (float)sc;
        float b = dmin * (float)mn;
        y[i] = a * (float)q - b;
    }
}

static void dequant_q6k_block(const uint8_t *p, float *y)
{
    const float d = gguf_o_half(rd16(p + 208));
    for (int i = 0; i < 256; i++) {
        int half = i / 128, quarter = (i & 127) / 32, l = i & 31;
        unsigned lo = p[half * 64 + (quarter & 1) * 32 + l];
        lo = quarter < 2 ? lo & 15u : lo >> 4;
        unsigned hi = (p[128 + half * 32 + l] >> (2 * quarter)) & 3u;
        int q = (int)(lo | (hi << 4)) - 32;
        int sc = (int8_t)p[192 + i / 16];
        float a = d * (float)sc;
        y[i] = a * (float)q;
    }
}

static void dequant_q80_block(const uint8_t *p, float *y)
{
    const float d = gguf_o_half(rd16(p));
    for (int i = 0; i < 32; i++) y[i] = d * (float)(int8_t)p[2 + i];
}

void gguf_o_dequant_row(int type, const uint8_t *row, int cols, float *out)
{
    if (type == GGUF_O_Q8_0) {
        for (int b = 0; b < cols / 32; b++) dequant_q80_block(row + b * 34, out + b * 32);
    } else if (type == GGUF_O_Q4_K) {
        for (int b = 0; b < cols / 256; b++) dequant_q4k_block(row + b * 144, out + b * 256);
    } else if (type == GGUF_O_Q6_K) {
        for (int b = 0; b < cols / 256; b++) dequant_q6k_block(row + b * 210, out + b * 256);
    }
}

/* argument contract of src/gguf-cuda.cu:111 */
int gguf_o_matmul(int type, const void *w, int cols, int rows, const float *x, int vectors,
                  unsigned x_stride, float *y, unsigned y_stride)
{
    if ((type != 8 && type != 12 && type != 14) || cols <= 0 || rows <= 0 || vectors < 1 || vectors > 32 ||
        cols % 256)
        return 1;
    unsigned rb = gguf_o_row_bytes(type, cols);
    float *deq = (float *)malloc(sizeof(float) * (size_t)cols);
    if (!deq) return 1;
    for (int r = 0; r < rows; r++) {
        gguf_o_dequant_row(type, (const uint8_t *)w + (size_t)r * rb, cols, deq);
        for (int v = 0; v < vectors; v++) {
            const float *xv = (const float *)((const uint8_t *)x + (size_t)v * x_stride);
            float sum = 0;
            for (int c = 0; c < cols; c++) sum += deq[c] * xv[c];
            ((float *)((uint8_t *)y + (size_t)v * y_stride))[r] = sum;
        }
    }
    free(deq);
    return 0;
}
