/* fyodor_oracle.c - CPU restatement of the Fyodor engine's decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the B200
 * provider; it is never linked into the provider and never measured as the
 * product. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it.
 *
 * Each function restates the reference algorithm it cites (paths relative to
 * the Fyodor repository). Accumulation order and rounding follow the
 * reference exactly, so for F32 KV the results are bit-identical to the
 * engine's scalar path (checked against the compiled reference engine by
 * tests/test_oracle_pin.py and tests/golden/).
 *
 * The one intentional extension is the fp16 KV cache: with kv_f16 set the
 * rotated key and the value are rounded to binary16 (round-to-nearest-even)
 * before they are stored, which is the semantics of the reference's own F16
 * KV experiment (backend/benchmarks/stage5-rejected/f16-experiment.patch,
 * decode hunk at :444-446) and of nya_llm_round_f16 (llm_quant.c:46-67).
 *
 * Build: gcc -std=c17 -O2 (ISO mode disables FMA contraction, as the
 * reference's C17 build does), see oracle/Makefile.
 */
#include "fyodor_b200_abi.h"

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* llm_quant.c:5-39 - IEEE binary16 to float by integer field assembly. */
float orc_half_to_float(uint16_t half)
{
    uint32_t sign = (uint32_t)(half & 0x8000U) << 16;
    int32_t exponent = (int32_t)((half >> 10) & 0x1FU);
    uint32_t fraction = half & 0x03FFU, bits;
    float value;
    if (exponent == 0) {
        if (fraction == 0) bits = sign;
        else {
            exponent = 1;
            while ((fraction & 0x0400U) == 0) { fraction <<= 1; exponent -= 1; }
            fraction &= 0x03FFU;
            bits = sign | ((uint32_t)(exponent + 112) << 23) | (fraction << 13);
        }
    } else if (exponent == 31) bits = sign | 0x7F800000U | (fraction << 13);
    else bits = sign | ((uint32_t)(exponent + 112) << 23) | (fraction << 13);
    memcpy(&value, &bits, sizeof(value));
    return value;
}

static float orc_half_at(const unsigned char *p)
{
    return orc_half_to_float((uint16_t)((uint16_t)p[0] | ((uint16_t)p[1] << 8)));
}

/* llm_quant.c:46-67 - round to binary16 with ties-to-even, by integer ops. */
uint16_t orc_float_to_half_bits(float value)
{
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    uint32_t sign = (bits >> 16) & 0x8000U, magnitude = bits & 0x7fffffffU, result;
    if (magnitude >= 0x7f800000U) result = magnitude == 0x7f800000U ? 0x7c00U : 0x7e00U;
    else if (magnitude >= 0x477ff000U) result = 0x7c00U;
    else if (magnitude < 0x33000000U) result = 0;
    else {
        uint32_t exponent = magnitude >> 23;
        uint32_t shift = exponent < 113U ? 126U - exponent : 13U;
        uint32_t mantissa = (magnitude & 0x7fffffU) | (exponent < 113U ? 0x800000U : 0U);
        uint32_t rounded = mantissa >> shift;
        uint32_t remainder = mantissa & ((1U << shift) - 1U), midpoint = 1U << (shift - 1U);
        if (remainder > midpoint || (remainder == midpoint && (rounded & 1U))) ++rounded;
        result = exponent < 113U ? rounded : ((exponent - 112U) << 10) + rounded;
    }
    return (uint16_t)(sign | result);
}

float orc_round_f16(float value) { return orc_half_to_float(orc_float_to_half_bits(value)); }

/* llm_quant.c:70-89 - one K-quant scalar. Q4_K: d*sc*q - dmin*m with the
   6-bit packed scale/min table; Q6_K: d*sc16*(q6-32). */
static float orc_k_quant_value(uint32_t type, const unsigned char *block, size_t index)
{
    if (type == NYA_LLM_TENSOR_Q4_K) {
        size_t group = index / 32;
        const unsigned char *s = block + 4;
        unsigned sc = group < 4 ? s[group] & 63U : (s[group + 4] & 15U) | ((unsigned)(s[group - 4] >> 6) << 4);
        unsigned mn = group < 4 ? s[group + 4] & 63U : (s[group + 4] >> 4) | ((unsigned)(s[group] >> 6) << 4);
        unsigned q = (block[16 + group / 2 * 32 + index % 32] >> (group % 2 * 4)) & 15U;
        return orc_half_at(block) * (float)sc * (float)q - orc_half_at(block + 2) * (float)mn;
    } else {
        size_t half = index / 128, quarter = index % 128 / 32, lane = index % 32;
        unsigned lo = block[half * 64 + quarter % 2 * 32 + lane];
        unsigned hi = block[128 + half * 32 + lane];
        int q = (int)(((lo >> (quarter / 2 * 4)) & 15U) | (((hi >> (quarter * 2)) & 3U) << 4)) - 32;
        int8_t scale;
        memcpy(&scale, block + 192 + half * 8 + quarter * 2 + lane / 16, 1);
        return orc_half_at(block + 208) * (float)scale * (float)q;
    }
}

/* llm_quant.c:91-142 - value at flat index of a supported storage type. */
float orc_tensor_value(const nya_llm_tensor *t, size_t index)
{
    if (t->type == NYA_LLM_TENSOR_Q4_K || t->type == NYA_LLM_TENSOR_Q6_K) {
        size_t bytes = t->type == NYA_LLM_TENSOR_Q4_K ? 144 : 210;
        return orc_k_quant_value(t->type, t->data + index / 256 * bytes, index % 256);
    }
    if (t->type == NYA_LLM_TENSOR_F32) { float v; memcpy(&v, t->data + index * 4, 4); return v; }
    if (t->type == NYA_LLM_TENSOR_F16) return orc_half_at(t->data + index * 2);
    if (t->type == NYA_LLM_TENSOR_BF16) {
        const unsigned char *p = t->data + index * 2;
        uint32_t bits = ((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << 16;
        float v; memcpy(&v, &bits, 4); return v;
    }
    if (t->type == NYA_LLM_TENSOR_Q8_0) {
        const unsigned char *d = t->data + index / 32 * 34;
        int8_t q; memcpy(&q, d + 2 + index % 32, 1);
        return orc_half_at(d) * q;
    }
    if (t->type == NYA_LLM_TENSOR_Q4_0) {
        const unsigned char *d = t->data + index / 32 * 18;
        size_t o = index % 32;
        unsigned char packed = d[2 + o % 16];
        int q = o < 16 ? (packed & 0x0F) : (packed >> 4);
        return orc_half_at(d) * (float)(q - 8);
    }
    return 0.0f;
}

/* Bulk form of orc_tensor_value for the dequantization parity tests. */
void orc_dequantize(const unsigned char *data, uint32_t type, size_t count, float *out)
{
    nya_llm_tensor t;
    memset(&t, 0, sizeof(t));
    t.data = data; t.type = type;
    for (size_t i = 0; i < count; ++i) out[i] = orc_tensor_value(&t, i);
}

/* K-quant rows [row0, row1) four at a time: the four running sums are
   independent chains, each updated in exactly the order of the scalar loop
   below (block, group, value), so every row's result is bit-identical to
   llm_quant.c:145-312; only the instruction-level interleaving differs. */
static void orc_kquant_rows4(float *output, const unsigned char *data, uint32_t type, const float *input,
    size_t columns, size_t row0)
{
    size_t block_bytes = type == NYA_LLM_TENSOR_Q4_K ? 144 : 210, blocks = columns / 256;
    float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (size_t b = 0; b < blocks; ++b) {
        const unsigned char *blk[4];
        for (int r = 0; r < 4; ++r) blk[r] = data + (row0 + (size_t)r) * blocks * block_bytes + b * block_bytes;
        const float *x = input + b * 256;
        if (type == NYA_LLM_TENSOR_Q4_K) {
            float d[4], minimum[4];
            for (int r = 0; r < 4; ++r) { d[r] = orc_half_at(blk[r]); minimum[r] = orc_half_at(blk[r] + 2); }
            for (size_t g = 0; g < 8; ++g) {
                float factor[4], bias[4];
                const unsigned char *packed[4];
                for (int r = 0; r < 4; ++r) {
                    const unsigned char *s = blk[r] + 4;
                    unsigned sc = g < 4 ? s[g] & 63U : (s[g + 4] & 15U) | ((unsigned)(s[g - 4] >> 6) << 4);
                    unsigned mn = g < 4 ? s[g + 4] & 63U : (s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
                    factor[r] = d[r] * (float)sc;
                    bias[r] = minimum[r] * (float)mn;
                    packed[r] = blk[r] + 16 + g / 2 * 32;
                }
                unsigned shift = (unsigned)(g % 2 * 4);
                for (size_t j = 0; j < 32; ++j) {
                    float xv = x[g * 32 + j];
                    for (int r = 0; r < 4; ++r)
                        sum[r] += (factor[r] * (float)((packed[r][j] >> shift) & 15U) - bias[r]) * xv;
                }
            }
        } else {
            float d[4];
            for (int r = 0; r < 4; ++r) d[r] = orc_half_at(blk[r] + 208);
            for (size_t g = 0; g < 16; ++g) {
                size_t half = g / 8, quarter = g % 8 / 2, lane_base = g % 2 * 16;
                float factor[4];
                for (int r = 0; r < 4; ++r) {
                    int8_t sc; memcpy(&sc, blk[r] + 192 + g, 1);
                    factor[r] = d[r] * (float)sc;
                }
                for (size_t j = 0; j < 16; ++j) {
                    size_t lane = lane_base + j;
                    float xv = x[g * 16 + j];
                    for (int r = 0; r < 4; ++r) {
                        unsigned lo = blk[r][half * 64 + quarter % 2 * 32 + lane];
                        unsigned hi = blk[r][128 + half * 32 + lane];
                        int q = (int)(((lo >> (quarter / 2 * 4)) & 15U) | (((hi >> (quarter * 2)) & 3U) << 4)) - 32;
                        sum[r] += factor[r] * (float)q * xv;
                    }
                }
            }
        }
    }
    for (int r = 0; r < 4; ++r) output[row0 + (size_t)r] = sum[r];
}

/* llm_quant.c:145-312 - scalar reference matvec over rows [row0, row1);
   identical summation order. */
static void orc_matvec_range(float *output, const unsigned char *data, uint32_t type,
    const float *input, size_t columns, size_t row0, size_t rows)
{
    if (type == NYA_LLM_TENSOR_F32) {
        for (size_t row = row0; row < rows; ++row) {
            const unsigned char *w = data + row * columns * 4;
            double sum = 0.0f;
            for (size_t c = 0; c < columns; ++c) { float v; memcpy(&v, w + c * 4, 4); sum += (double)v * input[c]; }
            output[row] = (float)sum;
        }
        return;
    }
    if (type == NYA_LLM_TENSOR_F16 || type == NYA_LLM_TENSOR_BF16) {
        for (size_t row = row0; row < rows; ++row) {
            const unsigned char *w = data + row * columns * 2;
            float sum = 0.0f;
            for (size_t c = 0; c < columns; ++c) {
                if (type == NYA_LLM_TENSOR_BF16) {
                    const unsigned char *p = w + c * 2;
                    uint32_t bits = ((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << 16;
                    float v; memcpy(&v, &bits, 4);
                    sum += v * input[c];
                } else sum += orc_half_at(w + c * 2) * input[c];
            }
            output[row] = sum;
        }
        return;
    }
    if (type == NYA_LLM_TENSOR_Q8_0) {
        size_t row_bytes = columns / 32 * 34;
        for (size_t row = row0; row < rows; ++row) {
            const unsigned char *w = data + row * row_bytes;
            float sum = 0.0f;
            for (size_t b = 0; b < columns / 32; ++b) {
                const unsigned char *bd = w + b * 34;
                float scale = orc_half_at(bd);
                for (size_t i = 0; i < 32; ++i) {
                    int8_t q; memcpy(&q, bd + 2 + i, 1);
                    sum += scale * (float)q * input[b * 32 + i];
                }
            }
            output[row] = sum;
        }
        return;
    }
    if (type == NYA_LLM_TENSOR_Q4_K || type == NYA_LLM_TENSOR_Q6_K) {
        size_t block_bytes = type == NYA_LLM_TENSOR_Q4_K ? 144 : 210, blocks = columns / 256;
        for (; row0 + 4 <= rows; row0 += 4) orc_kquant_rows4(output, data, type, input, columns, row0);
        for (size_t row = row0; row < rows; ++row) {
            const unsigned char *row_data = data + row * blocks * block_bytes;
            float sum = 0.0f;
            for (size_t b = 0; b < blocks; ++b) {
                const unsigned char *block = row_data + b * block_bytes;
                const float *x = input + b * 256;
                if (type == NYA_LLM_TENSOR_Q4_K) {
                    float d = orc_half_at(block), minimum = orc_half_at(block + 2);
                    const unsigned char *s = block + 4;
                    for (size_t g = 0; g < 8; ++g) {
                        unsigned sc = g < 4 ? s[g] & 63U : (s[g + 4] & 15U) | ((unsigned)(s[g - 4] >> 6) << 4);
                        unsigned mn = g < 4 ? s[g + 4] & 63U : (s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
                        float factor = d * (float)sc, bias = minimum * (float)mn;
                        const unsigned char *packed = block + 16 + g / 2 * 32;
                        unsigned shift = (unsigned)(g % 2 * 4);
                        for (size_t j = 0; j < 32; ++j)
                            sum += (factor * (float)((packed[j] >> shift) & 15U) - bias) * x[g * 32 + j];
                    }
                } else {
                    float d = orc_half_at(block + 208);
                    for (size_t g = 0; g < 16; ++g) {
                        size_t half = g / 8, quarter = g % 8 / 2, lane_base = g % 2 * 16;
                        int8_t sc; memcpy(&sc, block + 192 + g, 1);
                        float factor = d * (float)sc;
                        for (size_t j = 0; j < 16; ++j) {
                            size_t lane = lane_base + j;
                            unsigned lo = block[half * 64 + quarter % 2 * 32 + lane];
                            unsigned hi = block[128 + half * 32 + lane];
                            int q = (int)(((lo >> (quarter / 2 * 4)) & 15U) | (((hi >> (quarter * 2)) & 3U) << 4)) - 32;
                            sum += factor * (float)q * x[g * 16 + j];
                        }
                    }
                }
            }
            output[row] = sum;
        }
        return;
    }
    {   /* Q4_0: llm_quant.c:278-311 */
        size_t row_bytes = columns / 32 * 18;
        for (size_t row = row0; row < rows; ++row) {
            const unsigned char *w = data + row * row_bytes;
            float sum = 0.0f;
            for (size_t b = 0; b < columns / 32; ++b) {
                const unsigned char *bd = w + b * 18;
                float scale = orc_half_at(bd);
                for (size_t i = 0; i < 16; ++i) {
                    unsigned char packed = bd[2 + i];
                    float low = (float)((int)(packed & 0x0F) - 8), high = (float)((int)(packed >> 4) - 8);
                    sum += scale * low * input[b * 32 + i];
                    sum += scale * high * input[b * 32 + i + 16];
                }
            }
            output[row] = sum;
        }
    }
}

/* Worker of the threaded matvec: rows [row0, row1) of one call. */
typedef struct {
    float *output;
    const unsigned char *data;
    const float *input;
    size_t columns, row0, row1;
    uint32_t type;
} orc_matvec_job;

static void *orc_matvec_worker(void *arg)
{
    orc_matvec_job *j = (orc_matvec_job *)arg;
    orc_matvec_range(j->output, j->data, j->type, j->input, j->columns, j->row0, j->row1);
    return NULL;
}

static int orc_threads = 1;

/* Threads used by the session's matrix products (rows split evenly; each
   row is still summed in the reference order, so results do not depend on
   the count). */
void orc_set_threads(int threads) { orc_threads = threads < 1 ? 1 : threads > 256 ? 256 : threads; }

/* llm_quant.c:145-312, the engine's scalar matvec: one thread per call. */
void orc_matvec(float *output, const unsigned char *data, uint32_t type,
    const float *input, size_t columns, size_t rows)
{
    orc_matvec_range(output, data, type, input, columns, 0, rows);
}

/* The same products with rows spread over orc_threads threads. */
void orc_matvec_threaded(float *output, const unsigned char *data, uint32_t type,
    const float *input, size_t columns, size_t rows)
{
    int n = orc_threads;
    if (n <= 1 || rows < 64) { orc_matvec_range(output, data, type, input, columns, 0, rows); return; }
    if ((size_t)n > rows / 16) n = (int)(rows / 16);
    pthread_t tid[256];
    int started[256];
    orc_matvec_job job[256];
    for (int t = 0; t < n; ++t) {
        /* boundaries on multiples of four rows keep the four-row groups whole */
        size_t a = rows * (size_t)t / (size_t)n / 4 * 4;
        size_t b = t + 1 == n ? rows : rows * (size_t)(t + 1) / (size_t)n / 4 * 4;
        job[t] = (orc_matvec_job){output, data, input, columns, a, b, type};
        started[t] = t + 1 < n && pthread_create(&tid[t], NULL, orc_matvec_worker, &job[t]) == 0;
        if (!started[t]) orc_matvec_worker(&job[t]);  /* the last share, or one whose thread did not start */
    }
    for (int t = 0; t < n; ++t) if (started[t]) pthread_join(tid[t], NULL);
}

/* llm_cpu.c:83-103 - RMSNorm; the sum of squares is accumulated in double. */
static void orc_rms_norm(float *out, const float *in, const nya_llm_tensor *w, size_t n, float eps)
{
    double sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += (double)in[i] * in[i];
    float scale = (float)(1.0 / sqrt(sum / (double)n + eps));
    for (size_t i = 0; i < n; ++i) out[i] = in[i] * scale * (w == NULL ? 1.0f : orc_tensor_value(w, i));
}

/* llm_cpu.c:106-125 - stable softmax in float. */
static int orc_softmax(float *v, size_t n)
{
    if (n == 0) return -1;
    float maximum = v[0], sum = 0.0f;
    for (size_t i = 1; i < n; ++i) if (v[i] > maximum) maximum = v[i];
    for (size_t i = 0; i < n; ++i) { v[i] = expf(v[i] - maximum); sum += v[i]; }
    if (!(sum > 0.0f) || !isfinite(sum)) return -1;
    for (size_t i = 0; i < n; ++i) v[i] /= sum;
    return 0;
}

/* llm_cpu.c:298-327 - interleaved-pair LLaMA RoPE. */
static void orc_rope(float *v, size_t heads, size_t hd, const float *co, const float *si)
{
    for (size_t h = 0; h < heads; ++h) {
        float *p = v + h * hd;
        for (size_t c = 0; c < hd; c += 2) {
            float cs = co[c / 2], sn = si[c / 2], a = p[c], b = p[c + 1];
            p[c] = a * cs - b * sn;
            p[c + 1] = a * sn + b * cs;
        }
    }
}

/* Decode attention for one query token over [first, end] of one layer's cache
   (llm_cpu.c:510-535): scores q.k * scale, float softmax, then the
   probability-weighted value sum. Cache layout: [capacity][kv_heads][hd]. */
int orc_attention(const float *query, const float *keys, const float *values, float *out,
    size_t heads, size_t kv_heads, size_t hd, size_t first, size_t end, float scale, float *scratch)
{
    size_t kvdim = kv_heads * hd, length = end - first + 1;
    for (size_t head = 0; head < heads; ++head) {
        const float *q = query + head * hd;
        size_t kvh = head / (heads / kv_heads);
        float *o = out + head * hd;
        for (size_t t = first; t <= end; ++t) {
            const float *k = keys + t * kvdim + kvh * hd;
            float score = 0.0f;
            for (size_t j = 0; j < hd; ++j) score += q[j] * k[j];
            scratch[t - first] = score * scale;
        }
        if (orc_softmax(scratch, length) != 0) return -1;
        memset(o, 0, hd * sizeof(float));
        for (size_t t = first; t <= end; ++t) {
            const float *v = values + t * kvdim + kvh * hd;
            float p = scratch[t - first];
            for (size_t j = 0; j < hd; ++j) o[j] += p * v[j];
        }
    }
    return 0;
}

/* A dense LLaMA session (llm_cpu.c:128-265 state, :424-578 forward). */
typedef struct orc_session {
    const nya_llm_context *c;
    size_t capacity;
    int kv_f16;
    float *x, *norm, *residual, *gate, *up, *query, *scores, *logits;
    float *keys, *values, *freq, *co, *si;
} orc_session;

void orc_session_free(orc_session *s)
{
    if (!s) return;
    free(s->x); free(s->norm); free(s->residual); free(s->gate); free(s->up); free(s->query);
    free(s->scores); free(s->logits); free(s->keys); free(s->values); free(s->freq); free(s->co); free(s->si);
    free(s);
}

orc_session *orc_session_create(const nya_llm_context *c, size_t capacity, int kv_f16)
{
    if (!c || capacity == 0 || capacity > c->context_length || c->is_gemma || c->is_assistant) return NULL;
    orc_session *s = calloc(1, sizeof(*s));
    if (!s) return NULL;
    size_t d = c->embedding_length, h = c->maximum_hidden_length, q = c->maximum_query_length;
    size_t pairs = 0;
    for (size_t i = 0; i < c->block_count; ++i)
        if (c->layers[i].head_dimension / 2 > pairs) pairs = c->layers[i].head_dimension / 2;
    s->c = c; s->capacity = capacity; s->kv_f16 = kv_f16;
    s->x = malloc(d * 4); s->norm = malloc((d > q ? d : q) * 4); s->residual = malloc(d * 4);
    s->gate = malloc(h * 4); s->up = malloc(h * 4); s->query = malloc(q * 4);
    s->scores = malloc(capacity * 4); s->logits = malloc((size_t)c->tokenizer.vocabulary_size * 4);
    s->keys = malloc(c->cache_width * capacity * 4); s->values = malloc(c->cache_width * capacity * 4);
    s->freq = calloc(pairs ? pairs : 1, 4); s->co = malloc((pairs ? pairs : 1) * 4); s->si = malloc((pairs ? pairs : 1) * 4);
    if (!s->x || !s->norm || !s->residual || !s->gate || !s->up || !s->query || !s->scores || !s->logits ||
        !s->keys || !s->values || !s->freq || !s->co || !s->si) { orc_session_free(s); return NULL; }
    /* llm_cpu.c:216-229: frequencies powf(base, -j/pairs), computed once. */
    size_t hd_pairs = c->layers[0].head_dimension / 2;
    for (size_t j = 0; j < hd_pairs; ++j)
        s->freq[j] = powf(c->rope_frequency_base, -(float)j / (float)hd_pairs) / 1.0f;
    return s;
}

/* One causal token step (llm_cpu.c:424-578, dense LLaMA branch). */
int orc_session_forward(orc_session *s, uint32_t token, size_t position, int compute_logits)
{
    const nya_llm_context *c = s->c;
    size_t d = c->embedding_length;
    if (token >= c->tokenizer.vocabulary_size || position >= s->capacity) return -1;
    size_t pairs = c->layers[0].head_dimension / 2;
    for (size_t j = 0; j < pairs; ++j) {
        float angle = (float)position * s->freq[j];
        s->co[j] = cosf(angle); s->si[j] = sinf(angle);
    }
    for (size_t i = 0; i < d; ++i) s->x[i] = orc_tensor_value(c->token_embedding, (size_t)token * d + i);
    for (size_t layer = 0; layer < c->block_count; ++layer) {
        const nya_llm_layer *w = &c->layers[layer];
        size_t hd = w->head_dimension, heads = w->head_count, kvh = w->kv_head_count;
        size_t qdim = heads * hd, kvdim = kvh * hd, hid = w->hidden_length;
        size_t offset = w->cache_offset * s->capacity;
        float *key = s->keys + offset + position * kvdim, *value = s->values + offset + position * kvdim;
        orc_rms_norm(s->norm, s->x, w->attention_norm, d, c->norm_epsilon);
        orc_matvec_threaded(s->query, w->query->data, w->query->type, s->norm, d, qdim);
        orc_matvec_threaded(key, w->key->data, w->key->type, s->norm, d, kvdim);
        orc_matvec_threaded(value, w->value->data, w->value->type, s->norm, d, kvdim);
        orc_rope(key, kvh, hd, s->co, s->si);
        if (s->kv_f16) for (size_t j = 0; j < kvdim; ++j) { key[j] = orc_round_f16(key[j]); value[j] = orc_round_f16(value[j]); }
        orc_rope(s->query, heads, hd, s->co, s->si);
        if (orc_attention(s->query, s->keys + offset, s->values + offset, s->norm, heads, kvh, hd,
                0, position, 1.0f / sqrtf((float)hd), s->scores) != 0) return -1;
        orc_matvec_threaded(s->residual, w->attention_output->data, w->attention_output->type, s->norm, qdim, d);
        for (size_t j = 0; j < d; ++j) s->x[j] += s->residual[j];
        orc_rms_norm(s->norm, s->x, w->feed_forward_norm, d, c->norm_epsilon);
        orc_matvec_threaded(s->gate, w->feed_forward_gate->data, w->feed_forward_gate->type, s->norm, d, hid);
        orc_matvec_threaded(s->up, w->feed_forward_up->data, w->feed_forward_up->type, s->norm, d, hid);
        for (size_t j = 0; j < hid; ++j) { float g = s->gate[j]; s->gate[j] = g / (1.0f + expf(-g)) * s->up[j]; }
        orc_matvec_threaded(s->residual, w->feed_forward_down->data, w->feed_forward_down->type, s->gate, hid, d);
        for (size_t j = 0; j < d; ++j) s->x[j] += s->residual[j];
    }
    if (!compute_logits) return 0;
    orc_rms_norm(s->norm, s->x, c->output_norm, d, c->norm_epsilon);
    orc_matvec_threaded(s->logits, c->output->data, c->output->type, s->norm, d, c->tokenizer.vocabulary_size);
    for (size_t j = 0; j < c->tokenizer.vocabulary_size; ++j) if (!isfinite(s->logits[j])) return -1;
    for (size_t j = 0; j < c->tokenizer.suppressed_count; ++j) s->logits[c->tokenizer.suppressed_tokens[j]] = -INFINITY;
    return 0;
}

const float *orc_session_logits(const orc_session *s) { return s->logits; }
const float *orc_session_hidden(const orc_session *s) { return s->x; }

/* Snapshot of one layer's cache rows [position, position+count), F32. */
int orc_session_read_kv(const orc_session *s, size_t layer, size_t position, size_t count, float *k, float *v)
{
    const nya_llm_layer *w = &s->c->layers[layer];
    size_t width = w->head_dimension * w->kv_head_count, offset = w->cache_offset * s->capacity + position * width;
    memcpy(k, s->keys + offset, count * width * 4);
    memcpy(v, s->values + offset, count * width * 4);
    return 0;
}

/* llm_cpu.c:896-905 - greedy: first index of the maximum; NaN/+inf reject. */
int orc_argmax(const float *logits, size_t n, uint32_t *token)
{
    size_t best = 0;
    if (n == 0) return -1;
    for (size_t j = 0; j < n; ++j) {
        if (isnan(logits[j]) || logits[j] == INFINITY) return -1;
        if (logits[j] > logits[best]) best = j;
    }
    if (!isfinite(logits[best])) return -1;
    *token = (uint32_t)best;
    return 0;
}
