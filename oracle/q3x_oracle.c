/*
 * q3x_oracle.c -- CPU restatement of qwen3x's packed-weight matrix path.
 *
 * TEST INFRASTRUCTURE ONLY (see q3x_oracle.h).  Compiled with
 * -ffp-contract=off so that, like the reference's ISO C++17 build, no
 * multiply-add is fused: every FP32 operation below happens in the same order
 * as in the cited reference routine.
 */
#include "q3x_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define Q8_BLOCK 32
#define Q8_BYTES 34
#define Q4_BLOCK 32
#define Q4_BYTES 18
#define MAX_TOP_K 8 /* model_config.h:14 */

static uint16_t load_u16(const uint8_t* p) {
    uint16_t v;
    memcpy(&v, p, sizeof v);
    return v;
}

/* arch/cpu.cpp:31-52 */
float q3xo_f16(uint16_t value) {
    const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
    uint32_t exponent = (value >> 10) & 0x1fu;
    uint32_t mantissa = value & 0x03ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            exponent = 113;
            while (!(mantissa & 0x0400u)) { mantissa <<= 1; --exponent; }
            bits = sign | (exponent << 23) | ((mantissa & 0x03ffu) << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112) << 23) | (mantissa << 13);
    }
    float result;
    memcpy(&result, &bits, sizeof result);
    return result;
}

/* IEEE 754 binary32 -> binary16, round to nearest, ties to even. */
uint16_t q3xo_f32_to_f16(float value) {
    uint32_t x;
    memcpy(&x, &value, sizeof x);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x0200u : 0u));
    const int e = (int)(a >> 23);
    if (e >= 113) { /* normal binary16 range (may round up to inf) */
        uint32_t h = (a >> 13) - (112u << 10);
        const uint32_t rest = a & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
        if (h >= 0x7c00u) h = 0x7c00u;
        return (uint16_t)(sign | h);
    }
    if (e < 102) return sign; /* below half the smallest subnormal */
    const uint32_t m = (a & 0x7fffffu) | 0x800000u;
    const int s = 126 - e; /* 14..24 */
    uint32_t q = m >> s;
    const uint32_t rem = m & ((1u << s) - 1u), half = 1u << (s - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

/* engine.cpp:181-186 */
float q3xo_bf16(uint16_t value) {
    const uint32_t bits = (uint32_t)value << 16;
    float result;
    memcpy(&result, &bits, sizeof result);
    return result;
}

/* arch/cpu.cpp:161-179 */
int q3xo_quantized_bytes(uint32_t type, int rows, int cols, size_t* bytes) {
    int block_size;
    size_t block_bytes;
    if (type == Q3XO_Q8_0) { block_size = Q8_BLOCK; block_bytes = Q8_BYTES; }
    else if (type == Q3XO_Q4_0) { block_size = Q4_BLOCK; block_bytes = Q4_BYTES; }
    else return 0;
    if (rows <= 0 || cols <= 0 || cols % block_size != 0) return 0;
    const size_t blocks = (size_t)cols / (size_t)block_size;
    const size_t maximum = SIZE_MAX;
    if (blocks > maximum / block_bytes) return 0;
    const size_t row_bytes = blocks * block_bytes;
    if ((size_t)rows > maximum / row_bytes) return 0;
    *bytes = (size_t)rows * row_bytes;
    return 1;
}

/* arch/cpu.cpp:64-73 */
float q3xo_dot_q8_0(const void* blocks, const float* x, int n) {
    const uint8_t* b = (const uint8_t*)blocks;
    float sum = 0.0f;
    for (int block = 0; block < n / Q8_BLOCK; ++block) {
        const uint8_t* blk = b + (size_t)block * Q8_BYTES;
        const int8_t* q = (const int8_t*)(blk + 2);
        float inner = 0.0f;
        for (int i = 0; i < Q8_BLOCK; ++i)
            inner += (float)q[i] * x[block * Q8_BLOCK + i];
        sum += q3xo_f16(load_u16(blk)) * inner;
    }
    return sum;
}

/* q4.h:31-36 -- element i < 16 is the low nibble of byte i, i >= 16 the high
 * nibble of byte i - 16; value = nibble - 8. */
static int q4_value(const uint8_t* blk, int index) {
    const uint8_t packed = blk[2 + index % (Q4_BLOCK / 2)];
    const int quant = index < Q4_BLOCK / 2 ? (packed & 0x0f) : (packed >> 4);
    return quant - 8;
}

/* arch/cpu.cpp:91-101 */
float q3xo_dot_q4_0(const void* blocks, const float* x, int n) {
    const uint8_t* b = (const uint8_t*)blocks;
    float sum = 0.0f;
    for (int block = 0; block < n / Q4_BLOCK; ++block) {
        const uint8_t* blk = b + (size_t)block * Q4_BYTES;
        float inner = 0.0f;
        for (int i = 0; i < Q4_BLOCK; ++i)
            inner += (float)q4_value(blk, i) * x[block * Q4_BLOCK + i];
        sum += q3xo_f16(load_u16(blk)) * inner;
    }
    return sum;
}

/* engine.cpp:201-205 */
float q3xo_dot_bf16(const uint16_t* a, const float* b, int n) {
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum += q3xo_bf16(a[i]) * b[i];
    return sum;
}

/* arch/cpu.cpp:55-63 and :81-90 */
int q3xo_embed(const void* w, uint32_t type, int cols, int token, float* out) {
    if (type == Q3XO_Q8_0) {
        const int blocks = cols / Q8_BLOCK;
        const uint8_t* row = (const uint8_t*)w + (size_t)token * blocks * Q8_BYTES;
        for (int block = 0; block < blocks; ++block) {
            const uint8_t* blk = row + (size_t)block * Q8_BYTES;
            const float scale = q3xo_f16(load_u16(blk));
            const int8_t* q = (const int8_t*)(blk + 2);
            for (int i = 0; i < Q8_BLOCK; ++i) out[block * Q8_BLOCK + i] = scale * (float)q[i];
        }
        return 0;
    }
    if (type == Q3XO_Q4_0) {
        const int blocks = cols / Q4_BLOCK;
        const uint8_t* row = (const uint8_t*)w + (size_t)token * blocks * Q4_BYTES;
        for (int block = 0; block < blocks; ++block) {
            const uint8_t* blk = row + (size_t)block * Q4_BYTES;
            const float scale = q3xo_f16(load_u16(blk));
            for (int i = 0; i < Q4_BLOCK; ++i)
                out[block * Q4_BLOCK + i] = scale * (float)q4_value(blk, i);
        }
        return 0;
    }
    if (type == Q3XO_BF16) {
        const uint16_t* row = (const uint16_t*)w + (size_t)token * cols;
        for (int i = 0; i < cols; ++i) out[i] = q3xo_bf16(row[i]);
        return 0;
    }
    return -1;
}

static size_t row_bytes(uint32_t type, int cols) {
    if (type == Q3XO_Q8_0) return (size_t)(cols / Q8_BLOCK) * Q8_BYTES;
    if (type == Q3XO_Q4_0) return (size_t)(cols / Q4_BLOCK) * Q4_BYTES;
    return (size_t)cols * 2;
}

static float dot_row(const void* w, uint32_t type, int row, int cols, const float* x) {
    const uint8_t* r = (const uint8_t*)w + (size_t)row * row_bytes(type, cols);
    if (type == Q3XO_Q8_0) return q3xo_dot_q8_0(r, x, cols);
    if (type == Q3XO_Q4_0) return q3xo_dot_q4_0(r, x, cols);
    return q3xo_dot_bf16((const uint16_t*)r, x, cols);
}

typedef struct {
    const void* w;
    uint32_t type;
    int cols, row0, row1;
    const float* x;
    float* y;
} mv_slice;

static void* mv_worker(void* arg) {
    const mv_slice* s = (const mv_slice*)arg;
    for (int row = s->row0; row < s->row1; ++row)
        s->y[row] = dot_row(s->w, s->type, row, s->cols, s->x);
    return NULL;
}

/* arch/cpu.cpp:192-226 (Q8_0/Q4_0) and engine.cpp:207-212 (BF16 baseline). */
int q3xo_mv(const void* w, uint32_t type, int rows, int cols,
            const float* x, float* y, int threads) {
    if (type > Q3XO_Q4_0 || rows <= 0 || cols <= 0) return -1;
    if (type != Q3XO_BF16 && cols % 32) return -1;
    if (threads < 1) threads = 1;
    if (threads > rows) threads = rows;
    if (threads > 256) threads = 256;
    if (threads == 1) {
        for (int row = 0; row < rows; ++row) y[row] = dot_row(w, type, row, cols, x);
        return 0;
    }
    pthread_t tid[256];
    mv_slice slice[256];
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        slice[t].w = w; slice[t].type = type; slice[t].cols = cols;
        slice[t].row0 = (int)((long long)rows * t / threads);
        slice[t].row1 = (int)((long long)rows * (t + 1) / threads);
        slice[t].x = x; slice[t].y = y;
        if (t == 0) continue;
        if (pthread_create(&tid[t], NULL, mv_worker, &slice[t]) != 0) {
            mv_worker(&slice[t]); /* run inline: same rows, same result */
            tid[t] = 0;
        } else {
            ++started;
        }
    }
    mv_worker(&slice[0]);
    for (int t = 1; t < threads; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
    (void)started;
    return 0;
}

/* engine.cpp:580-583: per-token mv. */
int q3xo_gemm(const void* w, uint32_t type, int rows, int cols,
              const float* X, int T, float* Y, int threads) {
    for (int t = 0; t < T; ++t) {
        const int rc = q3xo_mv(w, type, rows, cols, X + (size_t)t * cols,
                               Y + (size_t)t * rows, threads);
        if (rc) return rc;
    }
    return 0;
}

/* engine.cpp:214-224 */
int q3xo_expert_mv(const void* w, uint32_t type, int experts, int rows,
                   int cols, int expert, const float* x, float* y) {
    if (expert < 0 || expert >= experts) return -1;
    size_t bytes = (size_t)rows * cols * 2;
    if (type != Q3XO_BF16 && !q3xo_quantized_bytes(type, rows, cols, &bytes)) return -1;
    return q3xo_mv((const uint8_t*)w + (size_t)expert * bytes, type, rows, cols, x, y, 1);
}

/* engine.cpp:187-191 */
static float sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}
static float silu(float x) { return x * sigmoid(x); }

/* engine.cpp:377-405 */
int q3xo_router_top_k(const float* logits, int experts, int top_k,
                      int* ids, float* probabilities) {
    if (!(experts > 0 && top_k > 0 && top_k <= experts)) return -1;
    float maximum = -INFINITY;
    for (int e = 0; e < experts; ++e) maximum = maximum < logits[e] ? logits[e] : maximum; /* std::max */
    float total = 0.0f;
    for (int e = 0; e < experts; ++e) total += probabilities[e] = expf(logits[e] - maximum);
    for (int e = 0; e < experts; ++e) probabilities[e] /= total;
    float selected_total = 0.0f;
    for (int slot = 0; slot < top_k; ++slot) {
        int selected = -1;
        for (int e = 0; e < experts; ++e) {
            int used = 0;
            for (int p = 0; p < slot; ++p) used = used || ids[p] == e;
            if (!used && (selected < 0 || probabilities[e] > probabilities[selected])) selected = e;
        }
        if (selected < 0) return -1;
        ids[slot] = selected;
        selected_total += probabilities[selected];
    }
    for (int slot = 0; slot < top_k; ++slot) probabilities[ids[slot]] /= selected_total;
    return 0;
}

/* engine.cpp:406-430 */
int q3xo_moe(const uint16_t* router, const void* gate_up, const void* down,
             const void* shared_gate, const void* shared_up,
             const void* shared_down, const uint16_t* shared_scale,
             uint32_t type, int experts, int top_k, int H, int I,
             int shared_I, const float* input, float* out,
             int* ids_out, float* weights_out) {
    if (top_k > MAX_TOP_K || experts <= 0) return -1;
    const int width = I > shared_I ? I : shared_I;
    float* router_logits = (float*)malloc(sizeof(float) * (size_t)experts);
    float* probs = (float*)malloc(sizeof(float) * (size_t)experts);
    float* gate_up_buf = (float*)malloc(sizeof(float) * 2 * (size_t)width);
    float* branch = (float*)malloc(sizeof(float) * (size_t)H);
    int ids[MAX_TOP_K];
    int rc = -1;
    if (!router_logits || !probs || !gate_up_buf || !branch) goto done;
    q3xo_mv(router, Q3XO_BF16, experts, H, input, router_logits, 1);
    if (q3xo_router_top_k(router_logits, experts, top_k, ids, probs)) goto done;
    for (int i = 0; i < H; ++i) out[i] = 0.0f;
    for (int slot = 0; slot < top_k; ++slot) {
        const int expert = ids[slot];
        float* gate = gate_up_buf;
        float* up = gate_up_buf + I;
        if (q3xo_expert_mv(gate_up, type, experts, 2 * I, H, expert, input, gate_up_buf)) goto done;
        for (int i = 0; i < I; ++i) gate[i] = silu(gate[i]) * up[i];
        if (q3xo_expert_mv(down, type, experts, H, I, expert, gate, branch)) goto done;
        const float weight = probs[expert];
        for (int i = 0; i < H; ++i) out[i] += weight * branch[i];
        if (ids_out) ids_out[slot] = expert;
        if (weights_out) weights_out[slot] = weight;
    }
    {
        /* engine.cpp:422-429: ffn_gate / ffn_up alias the 2I work buffer. */
        float* gate = gate_up_buf;
        float* up = gate_up_buf + I;
        q3xo_mv(shared_gate, type, shared_I, H, input, gate, 1);
        q3xo_mv(shared_up, type, shared_I, H, input, up, 1);
        for (int i = 0; i < shared_I; ++i) gate[i] = silu(gate[i]) * up[i];
        q3xo_mv(shared_down, type, H, shared_I, gate, branch, 1);
        q3xo_mv(shared_scale, Q3XO_BF16, 1, H, input, router_logits, 1);
        const float scale = sigmoid(router_logits[0]);
        for (int i = 0; i < H; ++i) out[i] += scale * branch[i];
    }
    rc = 0;
done:
    free(router_logits); free(probs); free(gate_up_buf); free(branch);
    return rc;
}

/* engine.cpp:601-605 */
int q3xo_argmax(const float* logits, int n) {
    if (n <= 0) return -1;
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (logits[best] < logits[i]) best = i;
    return best;
}

static int finite_block(const float* v, int n) {
    for (int i = 0; i < n; ++i)
        if (!isfinite(v[i])) return 0;
    return 1;
}

/* scripts/pack_weights.py:299-318 */
int q3xo_quantize_q8_0(const uint16_t* bf16, size_t count, void* blocks) {
    if (count % Q8_BLOCK) return -1;
    uint8_t* out = (uint8_t*)blocks;
    for (size_t b = 0; b < count / Q8_BLOCK; ++b) {
        float v[Q8_BLOCK];
        for (int i = 0; i < Q8_BLOCK; ++i) v[i] = q3xo_bf16(bf16[b * Q8_BLOCK + i]);
        if (!finite_block(v, Q8_BLOCK)) return -1;
        float maximum = 0.0f;
        for (int i = 0; i < Q8_BLOCK; ++i) maximum = fabsf(v[i]) > maximum ? fabsf(v[i]) : maximum;
        const float scale = maximum / 127.0f;
        const float inverse = scale != 0.0f ? 1.0f / scale : 0.0f;
        uint8_t* blk = out + b * Q8_BYTES;
        const uint16_t h = q3xo_f32_to_f16(scale);
        memcpy(blk, &h, 2);
        for (int i = 0; i < Q8_BLOCK; ++i) {
            const float n = v[i] * inverse;
            float r = copysignf(floorf(fabsf(n) + 0.5f), n);
            if (r > 127.0f) r = 127.0f;
            if (r < -127.0f) r = -127.0f;
            ((int8_t*)(blk + 2))[i] = (int8_t)r;
        }
    }
    return 0;
}

/* scripts/pack_weights.py:321-343 (ggml Q4_0) */
int q3xo_quantize_q4_0(const uint16_t* bf16, size_t count, void* blocks) {
    if (count % Q4_BLOCK) return -1;
    uint8_t* out = (uint8_t*)blocks;
    for (size_t b = 0; b < count / Q4_BLOCK; ++b) {
        float v[Q4_BLOCK];
        for (int i = 0; i < Q4_BLOCK; ++i) v[i] = q3xo_bf16(bf16[b * Q4_BLOCK + i]);
        if (!finite_block(v, Q4_BLOCK)) return -1;
        int largest = 0;
        for (int i = 1; i < Q4_BLOCK; ++i)
            if (fabsf(v[i]) > fabsf(v[largest])) largest = i;
        const float scale = v[largest] / -8.0f;
        const float inverse = scale != 0.0f ? 1.0f / scale : 0.0f;
        uint8_t q[Q4_BLOCK];
        for (int i = 0; i < Q4_BLOCK; ++i) {
            float t = truncf(v[i] * inverse + 8.5f);
            if (t > 15.0f) t = 15.0f;
            q[i] = (uint8_t)t;
        }
        uint8_t* blk = out + b * Q4_BYTES;
        const uint16_t h = q3xo_f32_to_f16(scale);
        memcpy(blk, &h, 2);
        for (int i = 0; i < 16; ++i) blk[2 + i] = (uint8_t)(q[i] | (q[16 + i] << 4));
    }
    return 0;
}
