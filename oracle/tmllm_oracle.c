/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the per-layer KV-cache decode path.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this.
 * See tmllm_oracle.h for the parity status.  Every function cites the reference file and
 * lines (Lee-Dongwook/RustLLM) whose arithmetic it restates.
 *
 * Built with -ffp-contract=off so that `a*b + c` rounds twice, exactly as written.
 */
#include "tmllm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------ */
/* binary16                                                                              */
/* ------------------------------------------------------------------------------------ */

uint16_t orc_f32_to_f16(float x) {
    uint32_t f;
    memcpy(&f, &x, 4);
    uint32_t sign = (f >> 16) & 0x8000u;
    uint32_t exp = (f >> 23) & 0xffu;
    uint32_t mant = f & 0x7fffffu;
    if (exp == 0xffu) {
        if (mant) return (uint16_t)(sign | 0x7e00u | (mant >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t hm = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

static float f16_to_f32_slow(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t mant = (uint32_t)h & 0x3ffu;
    uint32_t f;
    if (exp == 0) {
        if (mant == 0) {
            f = sign;
        } else {
            int e = -1;
            do {
                e++;
                mant <<= 1;
            } while (!(mant & 0x400u));
            mant &= 0x3ffu;
            f = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        f = sign | 0x7f800000u | (mant << 13);
    } else {
        f = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &f, 4);
    return out;
}

static float g_f16_table[65536];
static pthread_once_t g_f16_once = PTHREAD_ONCE_INIT;
static void init_f16_table(void) {
    for (uint32_t i = 0; i < 65536u; ++i) g_f16_table[i] = f16_to_f32_slow((uint16_t)i);
}
static inline const float* f16_table(void) {
    pthread_once(&g_f16_once, init_f16_table);
    return g_f16_table;
}

float orc_f16_to_f32(uint16_t h) { return f16_table()[h]; }

void orc_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(in[i]);
}

void orc_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
    const float* t = f16_table();
    for (size_t i = 0; i < n; ++i) out[i] = t[in[i]];
}

/* ------------------------------------------------------------------------------------ */
/* copies                                                                                */
/* ------------------------------------------------------------------------------------ */

/* kernels/kv_cache_write.metal:13-18: one work item per source element id:
 *   dim = id % head_dim; row = id / head_dim; seq = row % source_seq; head = row / source_seq;
 *   cache[(head*max_seq + start + seq)*head_dim + dim] = source[id]. */
void orc_kv_cache_write(int elem_bytes, void* cache, const void* source, uint32_t start,
                        uint32_t source_seq, uint32_t max_seq, uint32_t head_dim,
                        uint32_t numel) {
    for (uint32_t id = 0; id < numel; ++id) {
        uint32_t dim = id % head_dim;
        uint32_t row = id / head_dim;
        uint32_t seq = row % source_seq;
        uint32_t head = row / source_seq;
        size_t dst = ((size_t)head * max_seq + start + seq) * head_dim + dim;
        memcpy((char*)cache + dst * (size_t)elem_bytes,
               (const char*)source + (size_t)id * (size_t)elem_bytes, (size_t)elem_bytes);
    }
}

/* kernels/concat_sequence.metal:30-88: out[b,h,s,d] = s < L ? left[b,h,s,d]
 * : right[b,h,s-L,d]. */
void orc_concat_sequence(int elem_bytes, const void* left, const void* right, void* output,
                         uint32_t batch, uint32_t num_heads, uint32_t left_seq,
                         uint32_t right_seq, uint32_t head_dim) {
    uint32_t out_seq = left_seq + right_seq;
    size_t total = (size_t)batch * num_heads * out_seq * head_dim;
    for (size_t index = 0; index < total; ++index) {
        size_t per_batch = (size_t)num_heads * out_seq * head_dim;
        size_t b = index / per_batch;
        size_t off = index % per_batch;
        size_t h = off / ((size_t)out_seq * head_dim);
        size_t hoff = off % ((size_t)out_seq * head_dim);
        size_t s = hoff / head_dim;
        size_t d = hoff % head_dim;
        const char* src;
        if (s < left_seq) {
            src = (const char*)left +
                  (((b * num_heads + h) * left_seq + s) * head_dim + d) * (size_t)elem_bytes;
        } else {
            src = (const char*)right +
                  (((b * num_heads + h) * right_seq + (s - left_seq)) * head_dim + d) *
                      (size_t)elem_bytes;
        }
        memcpy((char*)output + index * (size_t)elem_bytes, src, (size_t)elem_bytes);
    }
}

/* kernels/repeat_kv.metal:16-30: out[b,qh,s,d] = in[b, qh/r, s, d]. */
void orc_repeat_kv(int elem_bytes, const void* input, void* output, uint32_t batch,
                   uint32_t kv_heads, uint32_t seq_len, uint32_t head_dim, uint32_t repeats) {
    uint32_t q_heads = kv_heads * repeats;
    size_t total = (size_t)batch * q_heads * seq_len * head_dim;
    for (size_t index = 0; index < total; ++index) {
        size_t d = index % head_dim;
        size_t t = index / head_dim;
        size_t s = t % seq_len;
        t /= seq_len;
        size_t qh = t % q_heads;
        size_t b = t / q_heads;
        size_t kvh = qh / repeats;
        size_t src = ((b * kv_heads + kvh) * seq_len + s) * head_dim + d;
        memcpy((char*)output + index * (size_t)elem_bytes,
               (const char*)input + src * (size_t)elem_bytes, (size_t)elem_bytes);
    }
}

/* ------------------------------------------------------------------------------------ */
/* attention ops                                                                         */
/* ------------------------------------------------------------------------------------ */

/* kernels/gqa_matmul.metal:25-160: S[b,qh,i,j] = sum_d Q[b,qh,i,d] * K[b,qh/G,j,d], the
 * sum running over d in increasing order in one F32 accumulator; K base
 * (b*Hkv + kvh)*kv_capacity*D (:59-65). */
void orc_gqa_qk_f32(const float* q, const float* k, float* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity) {
    uint32_t groups = q_heads / kv_heads;
    for (uint32_t b = 0; b < batch; ++b)
        for (uint32_t qh = 0; qh < q_heads; ++qh) {
            uint32_t kvh = qh / groups;
            const float* qb = q + ((size_t)b * q_heads + qh) * q_len * head_dim;
            const float* kb = k + ((size_t)b * kv_heads + kvh) * kv_capacity * head_dim;
            float* ob = out + ((size_t)b * q_heads + qh) * q_len * kv_len;
            for (uint32_t i = 0; i < q_len; ++i)
                for (uint32_t j = 0; j < kv_len; ++j) {
                    float sum = 0.0f;
                    for (uint32_t d = 0; d < head_dim; ++d)
                        sum += qb[(size_t)i * head_dim + d] * kb[(size_t)j * head_dim + d];
                    ob[(size_t)i * kv_len + j] = sum;
                }
        }
}

/* kernels/gqa_matmul.metal:163-321: same walk, float(half)*float(half) summed in F32,
 * stored as half(sum) (:319). */
void orc_gqa_qk_f16(const uint16_t* q, const uint16_t* k, uint16_t* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity) {
    const float* t = f16_table();
    uint32_t groups = q_heads / kv_heads;
    for (uint32_t b = 0; b < batch; ++b)
        for (uint32_t qh = 0; qh < q_heads; ++qh) {
            uint32_t kvh = qh / groups;
            const uint16_t* qb = q + ((size_t)b * q_heads + qh) * q_len * head_dim;
            const uint16_t* kb = k + ((size_t)b * kv_heads + kvh) * kv_capacity * head_dim;
            uint16_t* ob = out + ((size_t)b * q_heads + qh) * q_len * kv_len;
            for (uint32_t i = 0; i < q_len; ++i)
                for (uint32_t j = 0; j < kv_len; ++j) {
                    float sum = 0.0f;
                    for (uint32_t d = 0; d < head_dim; ++d)
                        sum += t[qb[(size_t)i * head_dim + d]] * t[kb[(size_t)j * head_dim + d]];
                    ob[(size_t)i * kv_len + j] = orc_f32_to_f16(sum);
                }
        }
}

/* kernels/gqa_matmul.metal:341-472: O[b,qh,i,d] = sum_j P[b,qh,i,j] * V[b,qh/G,j,d], j
 * increasing, one F32 accumulator. */
void orc_gqa_pv_f32(const float* probs, const float* v, float* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity) {
    uint32_t groups = q_heads / kv_heads;
    for (uint32_t b = 0; b < batch; ++b)
        for (uint32_t qh = 0; qh < q_heads; ++qh) {
            uint32_t kvh = qh / groups;
            const float* pb = probs + ((size_t)b * q_heads + qh) * q_len * kv_len;
            const float* vb = v + ((size_t)b * kv_heads + kvh) * kv_capacity * head_dim;
            float* ob = out + ((size_t)b * q_heads + qh) * q_len * head_dim;
            for (uint32_t i = 0; i < q_len; ++i)
                for (uint32_t d = 0; d < head_dim; ++d) {
                    float sum = 0.0f;
                    for (uint32_t j = 0; j < kv_len; ++j)
                        sum += pb[(size_t)i * kv_len + j] * vb[(size_t)j * head_dim + d];
                    ob[(size_t)i * head_dim + d] = sum;
                }
        }
}

/* kernels/gqa_matmul.metal:493-628: F16 variant, half store at :627. */
void orc_gqa_pv_f16(const uint16_t* probs, const uint16_t* v, uint16_t* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity) {
    const float* t = f16_table();
    uint32_t groups = q_heads / kv_heads;
    for (uint32_t b = 0; b < batch; ++b)
        for (uint32_t qh = 0; qh < q_heads; ++qh) {
            uint32_t kvh = qh / groups;
            const uint16_t* pb = probs + ((size_t)b * q_heads + qh) * q_len * kv_len;
            const uint16_t* vb = v + ((size_t)b * kv_heads + kvh) * kv_capacity * head_dim;
            uint16_t* ob = out + ((size_t)b * q_heads + qh) * q_len * head_dim;
            for (uint32_t i = 0; i < q_len; ++i)
                for (uint32_t d = 0; d < head_dim; ++d) {
                    float sum = 0.0f;
                    for (uint32_t j = 0; j < kv_len; ++j)
                        sum += t[pb[(size_t)i * kv_len + j]] * t[vb[(size_t)j * head_dim + d]];
                    ob[(size_t)i * head_dim + d] = orc_f32_to_f16(sum);
                }
        }
}

/* kernels/attention_scale_mask.metal:21-41: key > start + (row % query_len) ? -inf
 * : x*scale. */
void orc_scale_mask_f32(const float* in, float* out, float scale, uint32_t query_len,
                        uint32_t key_len, uint32_t query_start_pos, uint32_t numel) {
    for (uint32_t id = 0; id < numel; ++id) {
        uint32_t key_index = id % key_len;
        uint32_t query_index = (id / key_len) % query_len;
        uint32_t abs_q = query_start_pos + query_index;
        out[id] = key_index > abs_q ? -INFINITY : in[id] * scale;
    }
}

/* kernels/attention_scale_mask.metal:62-70: F32 multiply, half store. */
void orc_scale_mask_f16(const uint16_t* in, uint16_t* out, float scale, uint32_t query_len,
                        uint32_t key_len, uint32_t query_start_pos, uint32_t numel) {
    const float* t = f16_table();
    for (uint32_t id = 0; id < numel; ++id) {
        uint32_t key_index = id % key_len;
        uint32_t query_index = (id / key_len) % query_len;
        uint32_t abs_q = query_start_pos + query_index;
        out[id] = key_index > abs_q ? (uint16_t)0xfc00u : orc_f32_to_f16(t[in[id]] * scale);
    }
}

#define ORC_TG 256

/* Reduction order of kernels/softmax.metal:28-131: work item t (of 256) folds elements
 * t, t+256, ... in order, then a halving tree (stride 128 .. 1) combines the 256
 * partials. */
static float tree_max(float* s) {
    for (uint32_t stride = ORC_TG / 2; stride > 0; stride /= 2)
        for (uint32_t t = 0; t < stride; ++t) s[t] = fmaxf(s[t], s[t + stride]);
    return s[0];
}
static float tree_sum(float* s) {
    for (uint32_t stride = ORC_TG / 2; stride > 0; stride /= 2)
        for (uint32_t t = 0; t < stride; ++t) s[t] = s[t] + s[t + stride];
    return s[0];
}

static void softmax_row_f32(const float* x, float* y, uint32_t width) {
    float s[ORC_TG];
    for (uint32_t t = 0; t < ORC_TG; ++t) {
        float m = -INFINITY;
        for (uint32_t i = t; i < width; i += ORC_TG) m = fmaxf(m, x[i]);
        s[t] = m;
    }
    float row_max = tree_max(s);
    for (uint32_t t = 0; t < ORC_TG; ++t) {
        float acc = 0.0f;
        for (uint32_t i = t; i < width; i += ORC_TG) acc += expf(x[i] - row_max);
        s[t] = acc;
    }
    float denom = tree_sum(s);
    for (uint32_t i = 0; i < width; ++i) y[i] = expf(x[i] - row_max) / denom;
}

/* kernels/softmax.metal:7-132 (F32, no all-masked guard). */
void orc_softmax_f32(const float* in, float* out, uint32_t rows, uint32_t width) {
    for (uint32_t r = 0; r < rows; ++r)
        softmax_row_f32(in + (size_t)r * width, out + (size_t)r * width, width);
}

static void softmax_row_f16(const uint16_t* x, uint16_t* y, uint32_t width) {
    const float* t = f16_table();
    float s[ORC_TG];
    for (uint32_t w = 0; w < ORC_TG; ++w) {
        float m = -INFINITY;
        for (uint32_t i = w; i < width; i += ORC_TG) m = fmaxf(m, t[x[i]]);
        s[w] = m;
    }
    float row_max = tree_max(s);
    if (isinf(row_max) && row_max < 0.0f) { /* softmax.metal:166-173 */
        for (uint32_t i = 0; i < width; ++i) y[i] = 0;
        return;
    }
    for (uint32_t w = 0; w < ORC_TG; ++w) {
        float acc = 0.0f;
        for (uint32_t i = w; i < width; i += ORC_TG) acc += expf(t[x[i]] - row_max);
        s[w] = acc;
    }
    float denom = tree_sum(s);
    for (uint32_t i = 0; i < width; ++i) y[i] = orc_f32_to_f16(expf(t[x[i]] - row_max) / denom);
}

/* kernels/softmax.metal:136-195 (F16 storage, F32 math, zero-row guard). */
void orc_softmax_f16(const uint16_t* in, uint16_t* out, uint32_t rows, uint32_t width) {
    for (uint32_t r = 0; r < rows; ++r)
        softmax_row_f16(in + (size_t)r * width, out + (size_t)r * width, width);
}

/* kernels/batched_matmul.metal:20-132: out[b,r,c] = sum_i a[b,r,i]*b[b,i,c], i increasing. */
void orc_batched_matmul_f32(const float* a, const float* b, float* out, uint32_t batch,
                            uint32_t m, uint32_t k, uint32_t n) {
    for (uint32_t z = 0; z < batch; ++z)
        for (uint32_t r = 0; r < m; ++r)
            for (uint32_t c = 0; c < n; ++c) {
                float sum = 0.0f;
                for (uint32_t i = 0; i < k; ++i)
                    sum += a[(size_t)z * m * k + (size_t)r * k + i] *
                           b[(size_t)z * k * n + (size_t)i * n + c];
                out[(size_t)z * m * n + (size_t)r * n + c] = sum;
            }
}

/* kernels/batched_matmul.metal:151-196: F32 accumulation, half store. */
void orc_batched_matmul_f16(const uint16_t* a, const uint16_t* b, uint16_t* out,
                            uint32_t batch, uint32_t m, uint32_t k, uint32_t n) {
    const float* t = f16_table();
    for (uint32_t z = 0; z < batch; ++z)
        for (uint32_t r = 0; r < m; ++r)
            for (uint32_t c = 0; c < n; ++c) {
                float sum = 0.0f;
                for (uint32_t i = 0; i < k; ++i)
                    sum += t[a[(size_t)z * m * k + (size_t)r * k + i]] *
                           t[b[(size_t)z * k * n + (size_t)i * n + c]];
                out[(size_t)z * m * n + (size_t)r * n + c] = orc_f32_to_f16(sum);
            }
}

/* src/nn/rope.rs:44-62: exponent = (2i) as f32 / D as f32; inv = 1/theta^exponent;
 * angle = pos as f32 * inv; tables hold cos/sin(angle) in F32, [max_seq, D/2]. */
void orc_rope_tables(float* cos_table, float* sin_table, uint32_t head_dim,
                     uint32_t max_seq_len, float theta) {
    uint32_t half_dim = head_dim / 2;
    for (uint32_t pos = 0; pos < max_seq_len; ++pos)
        for (uint32_t i = 0; i < half_dim; ++i) {
            float exponent = (float)(2 * i) / (float)head_dim;
            float inv = 1.0f / powf(theta, exponent);
            float angle = (float)pos * inv;
            cos_table[(size_t)pos * half_dim + i] = cosf(angle);
            sin_table[(size_t)pos * half_dim + i] = sinf(angle);
        }
}

/* kernels/rope.metal:23-63: pair (i, i + D/2) of each row, position = row % seq_len,
 * table index (start + position)*D/2 + i; x1' = x1*c - x2*s, x2' = x2*c + x1*s. */
void orc_rope_f32(const float* in, const float* cos_table, const float* sin_table,
                  float* out, uint32_t seq_len, uint32_t head_dim, uint32_t start_pos,
                  uint32_t total_pairs) {
    uint32_t half_dim = head_dim / 2;
    for (uint32_t id = 0; id < total_pairs; ++id) {
        uint32_t pair = id % half_dim;
        uint32_t row = id / half_dim;
        uint32_t position = row % seq_len;
        size_t base = (size_t)row * head_dim;
        size_t first = base + pair, second = base + half_dim + pair;
        size_t ti = (size_t)(start_pos + position) * half_dim + pair;
        float c = cos_table[ti], s = sin_table[ti];
        float x1 = in[first], x2 = in[second];
        out[first] = x1 * c - x2 * s;
        out[second] = x2 * c + x1 * s;
    }
}

/* kernels/rope.metal:82-96: F32 math, half stores. */
void orc_rope_f16(const uint16_t* in, const float* cos_table, const float* sin_table,
                  uint16_t* out, uint32_t seq_len, uint32_t head_dim, uint32_t start_pos,
                  uint32_t total_pairs) {
    const float* t = f16_table();
    uint32_t half_dim = head_dim / 2;
    for (uint32_t id = 0; id < total_pairs; ++id) {
        uint32_t pair = id % half_dim;
        uint32_t row = id / half_dim;
        uint32_t position = row % seq_len;
        size_t base = (size_t)row * head_dim;
        size_t first = base + pair, second = base + half_dim + pair;
        size_t ti = (size_t)(start_pos + position) * half_dim + pair;
        float c = cos_table[ti], s = sin_table[ti];
        float x1 = t[in[first]], x2 = t[in[second]];
        out[first] = orc_f32_to_f16(x1 * c - x2 * s);
        out[second] = orc_f32_to_f16(x2 * c + x1 * s);
    }
}

/* ------------------------------------------------------------------------------------ */
/* chained attention core                                                                */
/* ------------------------------------------------------------------------------------ */

typedef struct {
    int dtype;
    const void *q, *k, *v;
    void* out;
    double *wout, *wlse;
    const float *wq, *wk, *wv;
    uint32_t batch, q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity, start_pos;
    float scale;
    double wscale;
    uint32_t row_begin, row_end; /* rows are (b, qh) pairs */
} core_job;

/* One (b, qh) pair through src/nn/attention.rs:216-247 in the reference's op order:
 * gqa_qk (or batched_matmul with K^T; same sum order) -> attention_scale_mask(1/sqrt(D),
 * start_pos) -> softmax_last_dim -> gqa_pv (or batched_matmul). */
static void core_rows_faithful(const core_job* j) {
    const float* t = f16_table();
    uint32_t groups = j->q_heads / j->kv_heads;
    uint32_t L = j->kv_len, D = j->head_dim;
    float* sc = (float*)malloc(sizeof(float) * L);
    float* pr = (float*)malloc(sizeof(float) * L);
    uint16_t* sh = (uint16_t*)malloc(sizeof(uint16_t) * L);
    uint16_t* ph = (uint16_t*)malloc(sizeof(uint16_t) * L);
    for (uint32_t row = j->row_begin; row < j->row_end; ++row) {
        uint32_t b = row / j->q_heads, qh = row % j->q_heads, kvh = qh / groups;
        size_t kbase = ((size_t)b * j->kv_heads + kvh) * j->kv_capacity * D;
        for (uint32_t i = 0; i < j->q_len; ++i) {
            size_t qoff = (((size_t)b * j->q_heads + qh) * j->q_len + i) * D;
            uint32_t abs_q = j->start_pos + i;
            if (j->dtype == 0) {
                const float* q = (const float*)j->q + qoff;
                const float* k = (const float*)j->k + kbase;
                const float* v = (const float*)j->v + kbase;
                for (uint32_t c = 0; c < L; ++c) {
                    float sum = 0.0f;
                    for (uint32_t d = 0; d < D; ++d) sum += q[d] * k[(size_t)c * D + d];
                    sc[c] = c > abs_q ? -INFINITY : sum * j->scale;
                }
                softmax_row_f32(sc, pr, L);
                float* o = (float*)j->out + qoff;
                for (uint32_t d = 0; d < D; ++d) {
                    float sum = 0.0f;
                    for (uint32_t c = 0; c < L; ++c) sum += pr[c] * v[(size_t)c * D + d];
                    o[d] = sum;
                }
            } else {
                const uint16_t* q = (const uint16_t*)j->q + qoff;
                const uint16_t* k = (const uint16_t*)j->k + kbase;
                const uint16_t* v = (const uint16_t*)j->v + kbase;
                for (uint32_t c = 0; c < L; ++c) {
                    float sum = 0.0f;
                    for (uint32_t d = 0; d < D; ++d) sum += t[q[d]] * t[k[(size_t)c * D + d]];
                    uint16_t s16 = orc_f32_to_f16(sum);                      /* :319 */
                    sh[c] = c > abs_q ? (uint16_t)0xfc00u
                                      : orc_f32_to_f16(t[s16] * j->scale);   /* :69 */
                }
                softmax_row_f16(sh, ph, L);                                   /* :193 */
                uint16_t* o = (uint16_t*)j->out + qoff;
                for (uint32_t d = 0; d < D; ++d) {
                    float sum = 0.0f;
                    for (uint32_t c = 0; c < L; ++c) sum += t[ph[c]] * t[v[(size_t)c * D + d]];
                    o[d] = orc_f32_to_f16(sum);                               /* :627 */
                }
            }
        }
    }
    free(sc);
    free(pr);
    free(sh);
    free(ph);
}

static void core_rows_wide(const core_job* j) {
    uint32_t groups = j->q_heads / j->kv_heads;
    uint32_t L = j->kv_len, D = j->head_dim;
    double* sc = (double*)malloc(sizeof(double) * L);
    double* acc = (double*)malloc(sizeof(double) * D);
    for (uint32_t row = j->row_begin; row < j->row_end; ++row) {
        uint32_t b = row / j->q_heads, qh = row % j->q_heads, kvh = qh / groups;
        size_t kbase = ((size_t)b * j->kv_heads + kvh) * j->kv_capacity * D;
        const float* k = j->wk + kbase;
        const float* v = j->wv + kbase;
        for (uint32_t i = 0; i < j->q_len; ++i) {
            size_t qoff = (((size_t)b * j->q_heads + qh) * j->q_len + i) * D;
            const float* q = j->wq + qoff;
            uint32_t abs_q = j->start_pos + i;
            uint32_t n = abs_q + 1 < L ? abs_q + 1 : L; /* unmasked keys */
            double m = -INFINITY;
            for (uint32_t c = 0; c < n; ++c) {
                double s = 0.0;
                for (uint32_t d = 0; d < D; ++d) s += (double)q[d] * (double)k[(size_t)c * D + d];
                sc[c] = s * j->wscale;
                if (sc[c] > m) m = sc[c];
            }
            double l = 0.0;
            for (uint32_t d = 0; d < D; ++d) acc[d] = 0.0;
            for (uint32_t c = 0; c < n; ++c) {
                double p = exp(sc[c] - m);
                l += p;
                for (uint32_t d = 0; d < D; ++d) acc[d] += p * (double)v[(size_t)c * D + d];
            }
            for (uint32_t d = 0; d < D; ++d) j->wout[qoff + d] = n ? acc[d] / l : 0.0;
            if (j->wlse) j->wlse[qoff / D] = n ? m + log(l) : -INFINITY;
        }
    }
    free(sc);
    free(acc);
}

static void* core_thread_faithful(void* arg) {
    core_rows_faithful((const core_job*)arg);
    return NULL;
}
static void* core_thread_wide(void* arg) {
    core_rows_wide((const core_job*)arg);
    return NULL;
}

static void run_rows(core_job* base, int threads, int wide) {
    uint32_t rows = base->batch * base->q_heads;
    if (threads <= 1 || rows <= 1) {
        base->row_begin = 0;
        base->row_end = rows;
        if (wide) core_rows_wide(base); else core_rows_faithful(base);
        return;
    }
    if ((uint32_t)threads > rows) threads = (int)rows;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    core_job* jobs = (core_job*)malloc(sizeof(core_job) * (size_t)threads);
    for (int w = 0; w < threads; ++w) {
        jobs[w] = *base;
        jobs[w].row_begin = (uint32_t)((uint64_t)rows * (uint64_t)w / (uint64_t)threads);
        jobs[w].row_end = (uint32_t)((uint64_t)rows * (uint64_t)(w + 1) / (uint64_t)threads);
        pthread_create(&tid[w], NULL, wide ? core_thread_wide : core_thread_faithful, &jobs[w]);
    }
    for (int w = 0; w < threads; ++w) pthread_join(tid[w], NULL);
    free(tid);
    free(jobs);
}

static int core_args_ok(uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                        uint32_t head_dim, uint32_t kv_capacity, uint32_t start_pos) {
    if (q_heads == 0 || kv_heads == 0 || q_heads % kv_heads) return 0;
    if (q_len == 0 || kv_len == 0 || head_dim == 0 || kv_capacity < kv_len) return 0;
    if ((uint64_t)start_pos + q_len > kv_len) return 0; /* attention_scale_mask.rs validate */
    return 1;
}

int orc_attention_core(int dtype, const void* q, const void* k, const void* v, void* out,
                       uint32_t batch, uint32_t q_heads, uint32_t kv_heads, uint32_t q_len,
                       uint32_t kv_len, uint32_t head_dim, uint32_t kv_capacity,
                       uint32_t start_pos, float scale, int threads) {
    if (!core_args_ok(q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity, start_pos))
        return -1;
    if (dtype != 0 && dtype != 1) return -1;
    core_job j;
    memset(&j, 0, sizeof(j));
    j.dtype = dtype;
    j.q = q; j.k = k; j.v = v; j.out = out;
    j.batch = batch; j.q_heads = q_heads; j.kv_heads = kv_heads; j.q_len = q_len;
    j.kv_len = kv_len; j.head_dim = head_dim; j.kv_capacity = kv_capacity;
    j.start_pos = start_pos; j.scale = scale;
    (void)f16_table();
    run_rows(&j, threads, 0);
    return 0;
}

int orc_attention_core_wide(const float* q, const float* k, const float* v, double* out,
                            double* out_lse, uint32_t batch, uint32_t q_heads,
                            uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                            uint32_t head_dim, uint32_t kv_capacity, uint32_t start_pos,
                            double scale, int threads) {
    if (!core_args_ok(q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity, start_pos))
        return -1;
    core_job j;
    memset(&j, 0, sizeof(j));
    j.wq = q; j.wk = k; j.wv = v; j.wout = out; j.wlse = out_lse;
    j.batch = batch; j.q_heads = q_heads; j.kv_heads = kv_heads; j.q_len = q_len;
    j.kv_len = kv_len; j.head_dim = head_dim; j.kv_capacity = kv_capacity;
    j.start_pos = start_pos; j.wscale = scale;
    run_rows(&j, threads, 1);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* paged layout helpers and the log-sum-exp merge                                        */
/* ------------------------------------------------------------------------------------ */

static inline size_t paged_offset(const int32_t* table, uint32_t max_blocks, uint32_t seq,
                                  uint32_t pos, uint32_t block_size, uint32_t num_kv_heads,
                                  uint32_t h, uint32_t head_dim) {
    size_t blk = (size_t)table[(size_t)seq * max_blocks + pos / block_size];
    return ((blk * num_kv_heads + h) * block_size + pos % block_size) * head_dim;
}

void orc_paged_gather(int elem_bytes, const void* arena, const int32_t* table,
                      uint32_t max_blocks, uint32_t seq, uint32_t len, uint32_t block_size,
                      uint32_t num_kv_heads, uint32_t head_dim, void* out) {
    size_t row = (size_t)head_dim * (size_t)elem_bytes;
    for (uint32_t h = 0; h < num_kv_heads; ++h)
        for (uint32_t p = 0; p < len; ++p) {
            size_t src = paged_offset(table, max_blocks, seq, p, block_size, num_kv_heads, h,
                                      head_dim);
            memcpy((char*)out + ((size_t)h * len + p) * row,
                   (const char*)arena + src * (size_t)elem_bytes, row);
        }
}

void orc_paged_scatter(int elem_bytes, void* arena, const int32_t* table, uint32_t max_blocks,
                       uint32_t seq, uint32_t start, uint32_t n, uint32_t block_size,
                       uint32_t num_kv_heads, uint32_t head_dim, const void* in) {
    size_t row = (size_t)head_dim * (size_t)elem_bytes;
    for (uint32_t h = 0; h < num_kv_heads; ++h)
        for (uint32_t s = 0; s < n; ++s) {
            size_t dst = paged_offset(table, max_blocks, seq, start + s, block_size,
                                      num_kv_heads, h, head_dim);
            memcpy((char*)arena + dst * (size_t)elem_bytes,
                   (const char*)in + ((size_t)h * n + s) * row, row);
        }
}

void orc_merge_lse(const float* parts_o, const float* parts_lse, uint32_t n, uint32_t rows,
                   uint32_t head_dim, float* out, float* out_lse) {
    for (uint32_t r = 0; r < rows; ++r) {
        double m = -INFINITY;
        for (uint32_t p = 0; p < n; ++p) {
            double l = parts_lse[(size_t)p * rows + r];
            if (l > m) m = l;
        }
        double denom = 0.0;
        for (uint32_t d = 0; d < head_dim; ++d) out[(size_t)r * head_dim + d] = 0.0f;
        if (isinf(m) && m < 0) {
            if (out_lse) out_lse[r] = -INFINITY;
            continue;
        }
        double* acc = (double*)calloc(head_dim, sizeof(double));
        for (uint32_t p = 0; p < n; ++p) {
            double w = exp((double)parts_lse[(size_t)p * rows + r] - m);
            denom += w;
            for (uint32_t d = 0; d < head_dim; ++d)
                acc[d] += w * (double)parts_o[((size_t)p * rows + r) * head_dim + d];
        }
        for (uint32_t d = 0; d < head_dim; ++d)
            out[(size_t)r * head_dim + d] = (float)(acc[d] / denom);
        if (out_lse) out_lse[r] = (float)(m + log(denom));
        free(acc);
    }
}
