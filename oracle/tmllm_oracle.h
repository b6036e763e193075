/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the per-layer KV-cache decode path.
 *
 * This is a scalar C restatement of the reference's Metal kernels (Lee-Dongwook/RustLLM,
 * `kernels/` Metal files) and of the order in which `src/nn/attention.rs` and
 * `src/model/kv_cache.rs` chain them.  It exists to check the CUDA path: only `tests/`,
 * `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py` may load it.  The
 * product library (`rustllm_b200/libtmllm_b200.so`) never links or calls it.
 *
 * Parity status: the reference is Rust + Apple Metal and cannot be built or run on Linux,
 * so the oracle is pinned by the reference's own known-answer tests (exact cache layout,
 * repeat_kv values, scale/mask values, masked-probability zeros), transcribed with their
 * file:line into tests/golden/reference_kats.json.  Attention values beyond those tests
 * are pinned to this restatement only.
 *
 * F16 storage is IEEE binary16; f32->f16 rounds to nearest-even (the behaviour of Metal's
 * `half(x)` and of `half` 2.x `f16::from_f32`).  "Faithful" functions round to half at the
 * exact store points of the Metal kernels; `*_wide` functions compute in double.
 */
#ifndef TMLLM_ORACLE_H
#define TMLLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- binary16 conversion ---- */
uint16_t orc_f32_to_f16(float x);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_array(const float* in, uint16_t* out, size_t n);
void orc_f16_to_f32_array(const uint16_t* in, float* out, size_t n);

/* ---- copies (bit-exact) ---- */
/* kernels/kv_cache_write.metal:4-36 ; cache [H, max_seq, D], source [H, source_seq, D] */
void orc_kv_cache_write(int elem_bytes, void* cache, const void* source, uint32_t start,
                        uint32_t source_seq, uint32_t max_seq, uint32_t head_dim,
                        uint32_t numel);
/* kernels/concat_sequence.metal:5-89 ; left [B,H,Sl,D] ++ right [B,H,Sr,D] along S */
void orc_concat_sequence(int elem_bytes, const void* left, const void* right, void* output,
                         uint32_t batch, uint32_t num_heads, uint32_t left_seq,
                         uint32_t right_seq, uint32_t head_dim);
/* kernels/repeat_kv.metal:5-72 ; [B,Hkv,S,D] -> [B,Hkv*r,S,D] */
void orc_repeat_kv(int elem_bytes, const void* input, void* output, uint32_t batch,
                   uint32_t kv_heads, uint32_t seq_len, uint32_t head_dim, uint32_t repeats);

/* ---- attention ops (faithful) ---- */
/* kernels/gqa_matmul.metal:7-161 (f32), 163-321 (f16: F32 sum, half store at :319) */
void orc_gqa_qk_f32(const float* q, const float* k, float* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity);
void orc_gqa_qk_f16(const uint16_t* q, const uint16_t* k, uint16_t* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity);
/* kernels/gqa_matmul.metal:323-473 (f32), 475-629 (f16: half store at :627) */
void orc_gqa_pv_f32(const float* probs, const float* v, float* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity);
void orc_gqa_pv_f16(const uint16_t* probs, const uint16_t* v, uint16_t* out, uint32_t batch,
                    uint32_t q_heads, uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                    uint32_t head_dim, uint32_t kv_capacity);
/* kernels/attention_scale_mask.metal:5-42 (f32), 46-71 (f16) */
void orc_scale_mask_f32(const float* in, float* out, float scale, uint32_t query_len,
                        uint32_t key_len, uint32_t query_start_pos, uint32_t numel);
void orc_scale_mask_f16(const uint16_t* in, uint16_t* out, float scale, uint32_t query_len,
                        uint32_t key_len, uint32_t query_start_pos, uint32_t numel);
/* kernels/softmax.metal:7-132 (f32), 136-195 (f16, zero-row guard at :166-173) */
void orc_softmax_f32(const float* in, float* out, uint32_t rows, uint32_t width);
void orc_softmax_f16(const uint16_t* in, uint16_t* out, uint32_t rows, uint32_t width);
/* kernels/batched_matmul.metal:7-133 (f32), 138-197 (f16) ; [batch,m,k] x [batch,k,n] */
void orc_batched_matmul_f32(const float* a, const float* b, float* out, uint32_t batch,
                            uint32_t m, uint32_t k, uint32_t n);
void orc_batched_matmul_f16(const uint16_t* a, const uint16_t* b, uint16_t* out,
                            uint32_t batch, uint32_t m, uint32_t k, uint32_t n);
/* src/nn/rope.rs:44-62 ; tables [max_seq, head_dim/2] */
void orc_rope_tables(float* cos_table, float* sin_table, uint32_t head_dim,
                     uint32_t max_seq_len, float theta);
/* kernels/rope.metal:5-64 (f32), 66-97 (f16) ; input [rows, seq_len, head_dim] */
void orc_rope_f32(const float* in, const float* cos_table, const float* sin_table,
                  float* out, uint32_t seq_len, uint32_t head_dim, uint32_t start_pos,
                  uint32_t total_pairs);
void orc_rope_f16(const uint16_t* in, const float* cos_table, const float* sin_table,
                  uint16_t* out, uint32_t seq_len, uint32_t head_dim, uint32_t start_pos,
                  uint32_t total_pairs);

/* ---- the chained attention core ----
 * src/nn/attention.rs:216-247: scores = QK (gqa_qk, or batched_matmul with K^T when
 * Hq==Hkv), scale_mask(1/sqrt(D), start_pos), softmax, PV.  q [B,Hq,S,D]; k,v read through
 * kv_capacity: element (b,h,j,d) at ((b*Hkv+h)*kv_capacity + j)*D + d; out [B,Hq,S,D].
 * dtype 0 = F32, 1 = F16 (faithful half rounding).  threads <= 1 runs single-threaded;
 * otherwise (b, q-head) rows are spread over that many POSIX threads.  Returns 0 on
 * success, -1 on bad arguments. */
int orc_attention_core(int dtype, const void* q, const void* k, const void* v, void* out,
                       uint32_t batch, uint32_t q_heads, uint32_t kv_heads, uint32_t q_len,
                       uint32_t kv_len, uint32_t head_dim, uint32_t kv_capacity,
                       uint32_t start_pos, float scale, int threads);
/* Same chain in double precision from float inputs (already rounded to the storage
 * dtype by the caller); out_lse (may be NULL) receives log-sum-exp of the scaled,
 * masked scores per (b, qh, i). */
int orc_attention_core_wide(const float* q, const float* k, const float* v, double* out,
                            double* out_lse, uint32_t batch, uint32_t q_heads,
                            uint32_t kv_heads, uint32_t q_len, uint32_t kv_len,
                            uint32_t head_dim, uint32_t kv_capacity, uint32_t start_pos,
                            double scale, int threads);

/* ---- paged-cache helpers (the layout the CUDA path stores) ----
 * Element (h, pos, d) of sequence s lives at
 *   ((table[s*max_blocks + pos/block_size]*num_kv_heads + h)*block_size + pos%block_size)*D + d.
 * gather copies positions [0, len) of sequence s into a dense [Hkv, len, D] tensor. */
void orc_paged_gather(int elem_bytes, const void* arena, const int32_t* table,
                      uint32_t max_blocks, uint32_t seq, uint32_t len, uint32_t block_size,
                      uint32_t num_kv_heads, uint32_t head_dim, void* out);
/* scatter writes [Hkv, n, D] into positions [start, start+n) of sequence s. */
void orc_paged_scatter(int elem_bytes, void* arena, const int32_t* table, uint32_t max_blocks,
                       uint32_t seq, uint32_t start, uint32_t n, uint32_t block_size,
                       uint32_t num_kv_heads, uint32_t head_dim, const void* in);

/* Merge split partials with log-sum-exp (the combine of flash-decoding and of the
 * cross-GPU sequence split): parts_o [n, rows, D] normalised outputs, parts_lse [n, rows];
 * out [rows, D], out_lse [rows]. */
void orc_merge_lse(const float* parts_o, const float* parts_lse, uint32_t n, uint32_t rows,
                   uint32_t head_dim, float* out, float* out_lse);

#ifdef __cplusplus
}
#endif
#endif
