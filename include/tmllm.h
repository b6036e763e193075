/*
 * tmllm.h — C ABI of the B200 (sm_100a) KV-cache decode path.
 *
 * This is the drop-in boundary for Lee-Dongwook/RustLLM's per-layer KV-cache decode
 * path: the KV-cache append, concat_sequence, repeat_kv and the GQA attention chain
 * (QK^T -> scale/mask -> softmax -> PV).  A Rust `build.rs` links `libtmllm_b200.so`
 * and binds these functions with `extern "C"` (plain pointers, sizes and C structs; no
 * C++ or CUDA types cross the boundary).
 *
 * Conventions
 *  - Every function returns an `int` status (tmllm_status).  0 is success.  Non-zero
 *    codes map one-to-one onto the reference's `TinyError` variants (src/error.rs:3-43)
 *    plus three codes the new runtime needs.  tmllm_last_error() returns a
 *    human-readable message for the calling thread's last failure, and
 *    tmllm_last_error_fields() the fields of the structured variants.
 *  - Arguments are validated on the host BEFORE anything is enqueued or mutated; a
 *    rejected call leaves every buffer and every cache length unchanged (the reference's
 *    rule, src/model/kv_cache.rs:18-53 and its test at :295-306).
 *  - Tensor arguments are device pointers to dense row-major data in the given dtype.
 *  - Work is enqueued on `stream` (NULL = the legacy default stream) and is asynchronous.
 *    Nothing here synchronises the device except tmllm_sync and the setup-time bulk
 *    copies documented on tmllm_cache_reserve.
 *  - A cache handle is not thread-safe (the reference's MetalContext is !Sync,
 *    src/metal/context.rs:14-17).
 *  - There is no CPU fallback: on a machine without a usable sm_100 device every call
 *    that needs the GPU returns TMLLM_DEVICE_ERROR.
 */
#ifndef TMLLM_H
#define TMLLM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* tmllm_stream;

typedef enum tmllm_status {
    TMLLM_OK = 0,
    TMLLM_INVALID_ARGUMENT = 1,      /* TinyError::InvalidArgument      src/error.rs:4 */
    TMLLM_INVALID_SHAPE = 2,         /* TinyError::InvalidShape         src/error.rs:5 */
    TMLLM_SHAPE_MISMATCH = 3,        /* TinyError::ShapeMismatch        src/error.rs:6-9 */
    TMLLM_INVALID_DIMENSION = 4,     /* TinyError::InvalidDimension     src/error.rs:10 */
    TMLLM_UNSUPPORTED_DTYPE = 5,     /* TinyError::UnsupportedDType     src/error.rs:17 */
    TMLLM_NON_CONTIGUOUS = 6,        /* TinyError::NonContiguousTensor  src/error.rs:18 */
    TMLLM_POSITION_OUT_OF_RANGE = 7, /* TinyError::PositionOutOfRange   src/error.rs:19-23 */
    TMLLM_MODEL_FORMAT = 8,          /* TinyError::ModelFormat          src/error.rs:31 */
    TMLLM_DEVICE_ERROR = 9,          /* TinyError::Metal -> a CUDA runtime error */
    TMLLM_OUT_OF_BLOCKS = 10,        /* new: the paged block pool is exhausted */
    TMLLM_TIMEOUT = 11,              /* new: a bounded device-side wait expired */
    TMLLM_NOT_RESERVED = 12          /* new: a write targets a position with no block */
} tmllm_status;

/* src/tensor (DType::{F32, F16}) */
typedef enum tmllm_dtype { TMLLM_F32 = 0, TMLLM_F16 = 1 } tmllm_dtype;

/* ---------------------------------------------------------------------------------- */
/* Library                                                                             */
/* ---------------------------------------------------------------------------------- */

/* ABI version (major*10000 + minor*100 + patch). */
int tmllm_version(void);
/* Static name of a status code ("TMLLM_INVALID_SHAPE", ...). */
const char* tmllm_status_name(int status);
/* Message of the calling thread's most recent failure ("" if none). */
const char* tmllm_last_error(void);

/* Fields of the calling thread's most recent failure, for the reference's two structured
 * error variants (src/error.rs:6-9, 19-23), so a binding rebuilds them exactly:
 *   TMLLM_POSITION_OUT_OF_RANGE -> TinyError::PositionOutOfRange { start_pos, seq_len,
 *     max_seq_len } (raised as in src/model/kv_cache.rs:46-50, src/ops/kv_cache_write.rs:106,
 *     src/nn/rope.rs:122 for the RoPE table);
 *   TMLLM_SHAPE_MISMATCH -> TinyError::ShapeMismatch { left, right } (the first left_rank /
 *     right_rank entries of left / right).
 * `status` is that failure's status (TMLLM_OK after a successful call: every entry point
 * clears the record on entry); the other fields are zero unless the status uses them. */
#define TMLLM_MAX_RANK 8
typedef struct tmllm_error_fields {
    int32_t status;
    int32_t left_rank;
    int32_t right_rank;
    int32_t reserved;
    int64_t start_pos;
    int64_t seq_len;
    int64_t max_seq_len;
    int64_t left[TMLLM_MAX_RANK];
    int64_t right[TMLLM_MAX_RANK];
} tmllm_error_fields;
int tmllm_last_error_fields(tmllm_error_fields* out);
/* Blocks until all work on `stream` is done (MetalExecution::finish's wait,
 * src/metal/execution.rs:30-36). */
int tmllm_sync(tmllm_stream stream);

/* ---------------------------------------------------------------------------------- */
/* Op-level entry points (stateless; contiguous device tensors)                        */
/* ---------------------------------------------------------------------------------- */

/* Replaces kv_cache_write_f32/_f16[_encode] (src/ops/kv_cache_write.rs:9-141):
 * cache [num_heads, max_seq, head_dim] (a LayerKvCache buffer, batch 1),
 * source [num_heads, source_seq, head_dim]; writes positions [start, start+source_seq).
 * Errors: POSITION_OUT_OF_RANGE when start+source_seq > max_seq (:577-586). */
int tmllm_kv_cache_write(tmllm_dtype dtype, void* cache, const void* source, size_t num_heads,
                         size_t max_seq, size_t head_dim, size_t start, size_t source_seq,
                         tmllm_stream stream);

/* Replaces concat_sequence_f32 (src/ops/concat_sequence.rs:13-115), extended to F16:
 * out [B,H,Sl+Sr,D] = left [B,H,Sl,D] ++ right [B,H,Sr,D] along the sequence axis. */
int tmllm_concat_sequence(tmllm_dtype dtype, const void* left, const void* right, void* out,
                          size_t batch, size_t num_heads, size_t left_seq, size_t right_seq,
                          size_t head_dim, tmllm_stream stream);

/* Replaces Tensor::repeat_kv / repeat_kv (src/tensor/repeat_kv.rs:13-81,
 * src/tensor/tensor.rs:686-688): out [B,Hkv*r,S,D][b,qh] = in [B,Hkv,S,D][b,qh/r].
 * repeats == 1 copies the input (the reference returns the same tensor, :27-29). */
int tmllm_repeat_kv(tmllm_dtype dtype, const void* in, void* out, size_t batch,
                    size_t kv_heads, size_t seq_len, size_t head_dim, size_t repeats,
                    tmllm_stream stream);

/* Replaces gqa_qk_matmul[_encode] (src/tensor/gqa_matmul.rs:16-62): scores
 * [B,Hq,Sq,L] = Q [B,Hq,Sq,D] . K^T where K is read as [B,Hkv,kv_capacity,D] for its
 * first kv_len rows (the `narrow` view of a cache, gqa_matmul.rs:59).  F16 stores
 * half(sum) of an F32 sum over d in increasing order (gqa_matmul.metal:319). */
int tmllm_gqa_qk(tmllm_dtype dtype, const void* q, const void* k, void* out, size_t batch,
                 size_t q_heads, size_t kv_heads, size_t q_len, size_t kv_len,
                 size_t head_dim, size_t kv_capacity, tmllm_stream stream);

/* Replaces gqa_pv_matmul[_encode] (src/tensor/gqa_matmul.rs:65-105): out [B,Hq,Sq,D] =
 * P [B,Hq,Sq,L] . V with V read as [B,Hkv,kv_capacity,D]. */
int tmllm_gqa_pv(tmllm_dtype dtype, const void* probs, const void* v, void* out,
                 size_t batch, size_t q_heads, size_t kv_heads, size_t q_len, size_t kv_len,
                 size_t head_dim, size_t kv_capacity, tmllm_stream stream);

/* Replaces Tensor::attention_scale_mask (src/tensor/tensor.rs:604-668,
 * src/ops/attention_scale_mask.rs:10-216): scores [..., query_len, key_len];
 * key > start + q ? -inf : x*scale.  Errors mirror attention_scale_mask.rs:120-160. */
int tmllm_attention_scale_mask(tmllm_dtype dtype, const void* in, void* out, size_t numel,
                               size_t query_len, size_t key_len, size_t query_start_pos,
                               float scale, tmllm_stream stream);

/* Replaces Tensor::softmax_last_dim (src/tensor/tensor.rs:458-495, src/ops/softmax.rs):
 * stable row softmax over `width`; F16 rows that are entirely -inf become zeros. */
int tmllm_softmax_last_dim(tmllm_dtype dtype, const void* in, void* out, size_t rows,
                           size_t width, tmllm_stream stream);

/* Replaces Tensor::batched_matmul (src/tensor/tensor.rs:497-602,
 * src/ops/batched_matmul.rs): out [batch,m,n] = a [batch,m,k] . b [batch,k,n]. */
int tmllm_batched_matmul(tmllm_dtype dtype, const void* a, const void* b, void* out,
                         size_t batch, size_t m, size_t k, size_t n, tmllm_stream stream);

/* Replaces RotaryEmbedding::new's table build (src/nn/rope.rs:44-62).  Fills HOST
 * arrays cos/sin [max_seq_len, head_dim/2] in F32, as the reference does on the CPU. */
int tmllm_rope_tables(float* cos_table, float* sin_table, size_t head_dim,
                      size_t max_seq_len, float theta);

/* Replaces rope / rope_encode (src/ops/rope.rs:277-370): in/out [rows, seq_len, head_dim]
 * (rows = batch*heads), device tables [table_len, head_dim/2] F32; half-split pairs
 * (i, i+D/2) at positions start_pos + s. */
int tmllm_rope(tmllm_dtype dtype, const void* in, void* out, const float* cos_table,
               const float* sin_table, size_t table_len, size_t rows, size_t seq_len,
               size_t head_dim, size_t start_pos, tmllm_stream stream);

/* ---------------------------------------------------------------------------------- */
/* Decoder layers around the attention path                                            */
/* ---------------------------------------------------------------------------------- */

/* Replaces Embedding::forward_encode (src/ops/embedding.rs, kernels/embedding.metal:39-53):
 * out [n, hidden] = table [vocab, hidden][ids].  A device id outside [0, vocab) yields a
 * zero row and sets *bad_id_flag (device int, may be NULL); the reference rejects such
 * ids on the host (TinyError::InvalidTokenId). */
int tmllm_embedding(tmllm_dtype dtype, const void* table, const int32_t* ids, void* out,
                    size_t n, size_t hidden, size_t vocab, int32_t* bad_id_flag,
                    tmllm_stream stream);

/* Replaces the residual add (Tensor::add_encode, kernels/vector_add.metal:15-21) and
 * RmsNorm::forward_encode (src/nn/rmsnorm.rs, kernels/rmsnorm.metal:71-126) that follow
 * each other in TransformerBlock (src/nn/transformer_block.rs:137-158):
 * s = x + residual (storage-rounded; residual may be NULL: s = x), written to sum_out
 * (may be NULL), and out = s * rsqrt(mean(s^2) + eps) * weight, per row of `hidden`. */
int tmllm_add_rmsnorm(tmllm_dtype dtype, const void* x, const void* residual, const void* weight,
                      void* out, void* sum_out, size_t rows, size_t hidden, float eps,
                      tmllm_stream stream);

/* Replaces SwiGlu (kernels/silu.metal:38-46) on a fused projection: gate_up [rows,
 * 2*inter] holds gate then up; out [rows, inter] = silu(gate) * up. */
int tmllm_swiglu(tmllm_dtype dtype, const void* gate_up, void* out, size_t rows, size_t inter,
                 tmllm_stream stream);

/* Replaces, for the few rows of a decode step, Linear::forward_encode (src/nn/linear.rs:105-170,
 * out = x · W with W [in, out] row-major, F16 in and out, F32 accumulation) together with
 * the element-wise kernels around it in TransformerBlock::forward_with_cache_encode
 * (src/nn/transformer_block.rs:128-158), in one launch:
 *   norm_weight != NULL: x is first RMS-normalised per row as kernels/rmsnorm.metal:71-126
 *     does (half(x * rsqrt(mean(x^2) + eps) * norm_weight)), the mean over all k columns;
 *     stats_in (may be NULL) holds the row statistics of x that the call which produced x
 *     wrote to its stats_out, else the rows are read once more to compute them;
 *   swiglu = 1: w is [k, 2n] holding the gate columns then the up columns, and
 *     out = half(silu(half(x·Wg)) * half(x·Wu)) (kernels/silu.metal:38-46);
 *   residual != NULL (swiglu = 0 only): out = half(residual + half(x · W))
 *     (kernels/vector_add.metal:15-21); residual may alias out;
 *   stats_out != NULL: receives the row statistics of out (tmllm_linear_stats_bytes(n)
 *     bytes of 16-byte aligned device memory: one partial sum of squares per 16 columns
 *     and row), for a
 *     later call that RMS-normalises out (its k = this n, the same rows).
 * rows <= 64; k and n multiples of 8; ldx / ldw / ldo / ldr are row strides in elements,
 * multiples of 8, and x, w, out, residual and norm_weight are 16-byte aligned.
 * flags: TMLLM_LINEAR_OVERLAP lets the launch overlap the tail of the work queued before it
 * on `stream` (programmatic dependent launch): w is read before that work has finished, so
 * the caller promises that it does not write w; x, residual, stats_in and norm_weight are
 * read only after it has finished.  The summation order depends on k and n only, so the
 * result does not depend on `rows` beyond the row itself: a row computed alone equals the
 * same row in any batch, bit for bit. */
#define TMLLM_LINEAR_OVERLAP 1u
size_t tmllm_linear_stats_bytes(int32_t n);
/* Reads and clears the status word of tmllm_linear's kernels: TMLLM_TIMEOUT when a bounded
 * device-side wait (the receipt of another CTA's partial sums) expired since the last read
 * (the outputs of that call are undefined), else TMLLM_OK.  Synchronises with the device. */
int tmllm_linear_status(int32_t* status);
int tmllm_linear(const void* x, int64_t ldx, const void* norm_weight, const float* stats_in,
                 float eps, const void* w, int64_t ldw, void* out, int64_t ldo,
                 const void* residual, int64_t ldr, float* stats_out, int32_t rows, int32_t k,
                 int32_t n, int32_t swiglu, uint32_t flags, tmllm_stream stream);

/* Replaces greedy sampling (src/generation/sampler.rs:79-88, on the CPU in the reference):
 * ids[r] = index of the largest finite logit of logits [rows, vocab] row r under
 * f32::total_cmp (-0 < +0; NaN and infinities are skipped), the last of equal maxima;
 * -1 when row r has no finite logit (the reference returns TinyError::Sampling). */
int tmllm_argmax(tmllm_dtype dtype, const void* logits, int32_t* ids, size_t rows, size_t vocab,
                 tmllm_stream stream);

/* Replaces the tail of a decode step in one launch: the final RmsNorm and the lm_head Linear
 * of Transformer::forward_with_cache_encode (src/model/transformer/cache.rs:72-77, i.e.
 * kernels/rmsnorm.metal:71-126 then Linear::forward_encode, src/nn/linear.rs:141-149) and,
 * optionally, the greedy pick of src/generation/sampler.rs:79-88 on the result.
 *   logits [rows, n] = half(xn · W), W [k, n] row-major F16, F32 accumulation, where
 *     x' = half(x + residual) when residual != NULL (kernels/vector_add.metal), else x, and
 *     xn = half(x' * rsqrt(mean(x'^2) + eps) * norm_weight) row by row (bit-identical to
 *     tmllm_add_rmsnorm), or xn = x' when norm_weight is NULL;
 *   ids != NULL: ids[r] = the pick of tmllm_argmax over the stored F16 logits of row r
 *     (the last of equal finite maxima under total order, -1 without a finite logit).
 * The argmax needs `workspace`: tmllm_lm_head_workspace_bytes() bytes of 8-byte aligned
 * device memory, zeroed once before its first use; every call leaves it zeroed again, so
 * one workspace serves any number of calls that do not run concurrently on the GPU.
 * rows <= 64 (with rows x k small enough for the rows to sit in shared memory: k <= 1344
 * at 64 rows); k and n multiples of 8; ldx / ldr / ldw / ld_logits multiples of 8 and x,
 * residual, w, logits and norm_weight 16-byte aligned.  flags: TMLLM_LINEAR_OVERLAP as for
 * tmllm_linear (w may be read before the work queued ahead on `stream` has finished).  Its
 * device-side waits are bounded: an expired one is reported by tmllm_linear_status (the
 * outputs of that call are then undefined; the workspace is still left zeroed). */
size_t tmllm_lm_head_workspace_bytes(void);
int tmllm_lm_head(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                  const void* norm_weight, float eps, const void* w, int64_t ldw, void* logits,
                  int64_t ld_logits, int32_t* ids, void* workspace, int32_t rows, int32_t k,
                  int32_t n, uint32_t flags, tmllm_stream stream);

/* ---------------------------------------------------------------------------------- */
/* Fused paged decode attention (the hot path)                                         */
/* ---------------------------------------------------------------------------------- */

/* A block-paged KV store for one layer.  Each arena is
 *   [num_blocks, num_kv_heads, block_size, head_dim]  (dtype),
 * so element (h, pos, d) of sequence s is at
 *   ((block_table[s*max_blocks_per_seq + pos/block_size]*num_kv_heads + h)*block_size
 *     + pos%block_size)*head_dim + d.
 * With block_size == capacity and one block per sequence this is exactly the
 * reference's LayerKvCache buffer [1, Hkv, max_seq, D] (src/model/kv_cache.rs:66). */
typedef struct tmllm_paged_kv {
    void* k_cache;
    void* v_cache;
    const int32_t* block_table; /* device, [num_seqs, max_blocks_per_seq] */
    const int32_t* seq_lens;    /* device, [num_seqs]: tokens cached before this call */
    int64_t num_blocks;
    int32_t num_seqs;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t block_size;
    int32_t max_blocks_per_seq;
    int32_t dtype;              /* tmllm_dtype */
} tmllm_paged_kv;

/* Optional inputs of tmllm_gqa_decode. */
typedef struct tmllm_decode_opts {
    float scale;            /* logit scale; <= 0 means 1/sqrt(head_dim) (attention.rs:236) */
    int32_t num_splits;     /* sequence splits per (seq, kv head); 0 = automatic */
    int32_t out_f32;        /* 0: `out` has the cache dtype; 1: `out` is F32 (partials) */
    const float* rope_cos;  /* optional device RoPE tables [rope_len, head_dim/2]; when   */
    const float* rope_sin;  /* given, q and k_new are rotated at position               */
    int32_t rope_len;       /* seq_lens[s] + rope_pos_offset (attention.rs:202-207)     */
    int32_t rope_pos_offset;
    int64_t max_len_hint;   /* longest sequence this call sees, for the split choice;  */
                            /* 0 = the capacity.  Affects speed only, never results.   */
    int32_t variant;        /* 0 = automatic; 1 = CUDA-core FMA kernel; 2 = tensor-core */
                            /* (mma.sync) kernel, F16 with head_dim 64 or 128 only     */
    int32_t flags;          /* TMLLM_DECODE_OVERLAP or 0                                */
    int64_t q_seq_stride;   /* elements between sequences in q (0 = q_heads*head_dim),  */
    int64_t kv_seq_stride;  /* and in k_new/v_new (0 = num_kv_heads*head_dim): lets the */
                            /* outputs of one fused QKV projection be read in place.    */
} tmllm_decode_opts;

/* tmllm_decode_opts.flags: the tensor-core decode launch may overlap the tail of the work
 * queued before it on the stream (programmatic dependent launch).  The lengths, block table
 * and cached K/V are read before that work has finished, so the caller promises it does not
 * write them; q, k_new and v_new are read, and anything is written, only after it has
 * finished.  With the cross-GPU exchange (tmllm_gqa_decode_exchange) the same holds on
 * every rank: a step's prologue may run while the previous step exchanges.  Ignored by the
 * CUDA-core kernels (always launched plainly) and by tmllm_cache_decode on a call that
 * assigns a new block (the table update it queues must finish first). */
#define TMLLM_DECODE_OVERLAP 1

/* Bytes of scratch tmllm_gqa_decode needs for `num_splits` splits (0 = enough for any
 * automatic choice for this shape on this device).  Zero it once (tmllm_decode_workspace_init)
 * before its first use; every successful call leaves it ready for the next. */
size_t tmllm_decode_workspace_bytes(int32_t num_seqs, int32_t q_heads, int32_t kv_heads,
                                    int32_t head_dim, int32_t num_splits);
int tmllm_decode_workspace_init(void* workspace, size_t bytes, tmllm_stream stream);
/* The split count tmllm_gqa_decode chooses when opts->num_splits == 0. */
int32_t tmllm_decode_auto_splits(int32_t num_seqs, int32_t kv_heads, int64_t max_len);

/* Fused KV-append + GQA decode attention for one query token per sequence.
 * Replaces, for q_len == 1, the chain SelfAttention::forward_with_cache_encode runs
 * (src/nn/attention.rs:303-313): LayerKvCache::append_encode (kv_cache.rs:112-142,
 * kv_cache_write.metal) followed by attention_core_encode (attention.rs:216-247:
 * gqa_qk / batched_matmul, attention_scale_mask, softmax, gqa_pv / batched_matmul).
 *   q      [num_seqs, q_heads, head_dim]        (kv dtype)
 *   k_new  [num_seqs, num_kv_heads, head_dim]   appended at position seq_lens[s];
 *   v_new  [num_seqs, num_kv_heads, head_dim]   both NULL = attend the cache only
 *   out    [num_seqs, q_heads, head_dim]        (cache dtype, or F32 if opts->out_f32)
 *   lse    [num_seqs, q_heads] F32, natural-log log-sum-exp of the scaled logits (NULL ok)
 * Each sequence attends keys [0, seq_lens[s] + (k_new != NULL)).  The block for the new
 * position must already be in the block table.  seq_lens is NOT advanced.
 * q_heads must be a multiple of num_kv_heads (gqa_matmul.rs:163-170). */
int tmllm_gqa_decode(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                     const void* v_new, void* out, float* lse, int32_t q_heads,
                     const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                     tmllm_stream stream);

/* Size of the split scratch built into the library for tmllm_gqa_decode_noalloc. */
#define TMLLM_NOALLOC_SCRATCH_BYTES (2 * 1024 * 1024)

/* No counterpart in the reference (its Metal path allocates a buffer per op).
 * tmllm_gqa_decode without a workspace argument, for callers that cannot allocate device
 * memory at decode time: code inside a stream capture that must not add allocations,
 * embedders whose memory comes from a pool they do not own, real-time loops that may not
 * take allocator locks.  It calls no cudaMalloc/cudaFree and no allocating library
 * routine; its split scratch is a TMLLM_NOALLOC_SCRATCH_BYTES (2 MiB) array compiled into
 * the library, held on every GPU that loads the library until the process exits.
 *  - The first call on a device (that device current) looks up the array's device address;
 *    make it before any stream capture.
 *  - All calls share the array and it keeps the last call's contents; the counters that
 *    must start at zero are cleared on `stream` before each launch.  Calls that overlap on
 *    the GPU race on it: serialise them.
 *  - A call whose split partials exceed the array is rejected with TMLLM_INVALID_SHAPE
 *    before anything is enqueued (config 4, 32 query heads x 128 dims x 37 splits, needs
 *    about 0.6 MiB).
 * Arguments and results are those of tmllm_gqa_decode. */
int tmllm_gqa_decode_noalloc(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                             const void* v_new, void* out, float* lse, int32_t q_heads,
                             const tmllm_decode_opts* opts, tmllm_stream stream);

/* Fused KV-append + causal attention for a chunk of new tokens per sequence (prefill).
 * Replaces, for q_len > 1, the chain SelfAttention::forward_with_cache_encode runs
 * (src/nn/attention.rs:303-315): LayerKvCache::append_encode (kv_cache.rs:112-142) of the
 * RoPE'd keys and the values, then attention_core_encode (attention.rs:216-247) with
 * start = the cached length, i.e. query row i of a sequence attends keys
 * [0, seq_lens[s] + i] (attention_scale_mask.metal:21-41).
 *   q      [total_rows, q_heads, head_dim]       (cache dtype; row stride opts->q_seq_stride)
 *   k_new  [total_rows, num_kv_heads, head_dim]  appended at seq_lens[s] + i
 *   v_new  [total_rows, num_kv_heads, head_dim]  (row stride opts->kv_seq_stride); both
 *          NULL = attend only: those positions already hold the rows
 *   out    [total_rows, q_heads, head_dim]       (cache dtype, or F32 if opts->out_f32)
 * Rows are grouped by sequence.  q_start (device, int32 [num_seqs + 1]) gives each
 * sequence's first row; with q_start == NULL every sequence has rows_per_seq rows and
 * max_rows / total_rows are ignored.  Otherwise max_rows is the largest row count and
 * total_rows = q_start[num_seqs].  RoPE (opts->rope_*) rotates q and k at position
 * seq_lens[s] + i + opts->rope_pos_offset.  Blocks for the new positions must already be in
 * the block table; seq_lens is NOT advanced.  opts->num_splits, max_len_hint and lse are not
 * used.  F16 with head_dim 64/128 and power-of-two pages of >= 16 positions runs on the
 * tensor cores (opts->variant 0 or 2); everything else on the CUDA cores (variant 1 forces
 * that path). */
int tmllm_gqa_prefill(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                      const void* v_new, const int32_t* q_start, int32_t rows_per_seq,
                      int32_t max_rows, int32_t total_rows, void* out, int32_t q_heads,
                      const tmllm_decode_opts* opts, tmllm_stream stream);
/* New (the reference's kernels cannot stall).  Reads and clears the status word of the
 * prefill kernel's bounded waits on the current device: TMLLM_OK, or TMLLM_TIMEOUT when a
 * wait inside the kernel expired (that launch's output rows are unspecified).
 * Synchronises with the device. */
int tmllm_prefill_status(int32_t* status);

/* Log-sum-exp merge of partial attention results (the combine step of a sequence split
 * across GPUs).  Part p's normalised output rows are at parts_o + p*o_stride ([rows,
 * head_dim] F32) and its log-sum-exp values at parts_lse + p*lse_stride ([rows] F32);
 * strides are in floats, 0 = packed (rows*head_dim and rows).  Writes out [rows,
 * head_dim] (out_dtype) and out_lse [rows] (NULL ok). */
int tmllm_merge_lse(const float* parts_o, const float* parts_lse, int32_t num_parts,
                    int32_t rows, int32_t head_dim, int64_t o_stride, int64_t lse_stride,
                    void* out, int32_t out_dtype, float* out_lse, tmllm_stream stream);

/* ---------------------------------------------------------------------------------- */
/* Sequence split across GPUs, exchanged inside the decode kernel                      */
/* ---------------------------------------------------------------------------------- */

/* New (the reference is single-device).  One sequence split along its positions across
 * `world` GPUs (BASELINE config 4's multi-GPU form): each rank holds a contiguous share of
 * the positions in its own paged cache.  Instead of a separate collective, the decode
 * kernel's final CTA of each (sequence, KV head) stores its normalised rows and their
 * log-sum-exp into every other rank's receive buffer over NVLink as {value, step} 8-byte
 * cells, reads the other ranks' rows from its own buffer as their cells reach this step
 * (waiting at most 2 s by default), and merges them into `out`: every rank ends with the
 * full result.  Ranks must issue the same sequence of
 * tmllm_gqa_decode_exchange calls.  An expired wait writes zeros and sets the status that
 * tmllm_exchange_status returns (TMLLM_TIMEOUT). */
#define TMLLM_IPC_HANDLE_BYTES 64
typedef struct tmllm_exchange tmllm_exchange;

/* Allocates this rank's buffer on the current device for `rows` = num_seqs * q_heads
 * output rows in `groups` = num_seqs * num_kv_heads groups, and writes its CUDA IPC handle
 * (TMLLM_IPC_HANDLE_BYTES bytes) to ipc_handle_out (may be NULL). */
int tmllm_exchange_create(int32_t world, int32_t rank, int32_t rows, int32_t groups,
                          int32_t head_dim, tmllm_exchange** out, void* ipc_handle_out);
/* Maps every other rank's buffer from the gathered handles ([world][64] bytes, rank order;
 * this rank's own entry is ignored).  One process per GPU. */
int tmllm_exchange_connect(tmllm_exchange* ex, const void* handles);
/* The same for exchanges created in this process (one process driving several GPUs, or
 * ranks emulated on one GPU): ranks[p] is rank p's exchange. */
int tmllm_exchange_connect_local(tmllm_exchange* ex, tmllm_exchange* const* ranks);
/* Bound of the in-kernel wait for the other ranks, in nanoseconds of %globaltimer. */
int tmllm_exchange_set_timeout(tmllm_exchange* ex, uint64_t timeout_ns);
/* Reads (synchronously) and clears this rank's status: 0, or TMLLM_TIMEOUT if a wait expired. */
int tmllm_exchange_status(tmllm_exchange* ex, int32_t* status);
int tmllm_exchange_destroy(tmllm_exchange* ex);
/* tmllm_gqa_decode over this rank's share, finished by the exchange and merge: `out` and
 * `lse` receive the result over all ranks' positions.  F16 caches with head_dim 64 or 128.
 * k_new/v_new: the new token on the rank that holds the sequence's tail, NULL elsewhere;
 * RoPE positions come from opts->rope_pos_offset (global position minus local length). */
int tmllm_gqa_decode_exchange(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                              const void* v_new, void* out, float* lse, int32_t q_heads,
                              const tmllm_decode_opts* opts, void* workspace,
                              size_t workspace_bytes, tmllm_exchange* ex, tmllm_stream stream);

/* ---------------------------------------------------------------------------------- */
/* Paged KV cache runtime                                                              */
/* ---------------------------------------------------------------------------------- */

typedef struct tmllm_cache tmllm_cache;

typedef struct tmllm_cache_config {
    int32_t device;         /* CUDA device ordinal */
    int32_t num_layers;     /* one K and one V arena per layer, one block table for all */
    int32_t num_seqs;
    int32_t max_seq_len;    /* per-sequence capacity (LayerKvCache max, kv_cache.rs:57) */
    int32_t block_size;     /* tokens per block; == max_seq_len gives the reference layout */
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t dtype;          /* tmllm_dtype */
    int64_t num_blocks;     /* pool size; 0 = num_seqs * ceil(max_seq_len / block_size) */
    uint64_t shuffle_seed;  /* 0 = blocks handed out in pool order; else a seeded shuffle */
} tmllm_cache_config;

/* Replaces LayerKvCache::new (src/model/kv_cache.rs:54-75) and KvCache::new (:150-164).
 * Errors: INVALID_SHAPE for zero dimensions (:61-65). */
int tmllm_cache_create(const tmllm_cache_config* config, tmllm_cache** out);
int tmllm_cache_destroy(tmllm_cache* cache);
/* LayerKvCache::len (kv_cache.rs:76-78), per sequence. */
int tmllm_cache_len(const tmllm_cache* cache, int32_t seq, int64_t* out);
/* LayerKvCache::capacity (kv_cache.rs:83-85). */
int tmllm_cache_capacity(const tmllm_cache* cache, int64_t* out);
/* LayerKvCache::storage_bytes / KvCache::storage_bytes (kv_cache.rs:87-89,176-178):
 * bytes of all K and V arenas. */
int tmllm_cache_storage_bytes(const tmllm_cache* cache, int64_t* out);
/* LayerKvCache::reset / KvCache::reset (kv_cache.rs:92-94,179-183): length 0, blocks
 * back to the pool; device memory is not cleared.  seq < 0 resets every sequence. */
int tmllm_cache_reset(tmllm_cache* cache, int32_t seq, tmllm_stream stream);
/* New: give sequence `seq` blocks for positions [len, len+n).  Validates first
 * (POSITION_OUT_OF_RANGE past capacity, OUT_OF_BLOCKS when the pool is empty) and
 * changes nothing on failure.  Table updates of up to 32 entries are enqueued on
 * `stream`; larger ones (prefill-sized) are copied synchronously. */
int tmllm_cache_reserve(tmllm_cache* cache, int32_t seq, int64_t n, tmllm_stream stream);
/* Replaces LayerKvCache::append_encode's write half (kv_cache.rs:112-138): k, v
 * [num_kv_heads, n, head_dim] (dtype) written at positions [len, len+n) of `seq` in
 * `layer`, reserving blocks as needed.  The length is NOT advanced (every layer of a
 * step writes the same positions); see tmllm_cache_advance. */
int tmllm_cache_append(tmllm_cache* cache, int32_t layer, int32_t seq, const void* k,
                       const void* v, int64_t n, int32_t dtype, tmllm_stream stream);
/* The `self.len = new_len` of append_encode (kv_cache.rs:140): len += n for `seq`
 * (every sequence when seq < 0), on the host and on the device copy of the lengths. */
int tmllm_cache_advance(tmllm_cache* cache, int32_t seq, int64_t n, tmllm_stream stream);
/* Device pointers of one layer's store, for tmllm_gqa_decode. */
int tmllm_cache_view(const tmllm_cache* cache, int32_t layer, tmllm_paged_kv* out);
/* Host copy of a sequence's block table (the first ceil(len/block_size) entries and any
 * reserved beyond); *n receives the number of valid entries. */
int tmllm_cache_block_table(const tmllm_cache* cache, int32_t seq, int32_t* out,
                            int64_t capacity, int64_t* n);
/* Replaces LayerKvCache::key()/value() (kv_cache.rs:98-103) followed by contiguous():
 * dense copies [num_kv_heads, len, head_dim] of positions [0, len) (either may be NULL). */
int tmllm_cache_gather(const tmllm_cache* cache, int32_t layer, int32_t seq, void* k_out,
                       void* v_out, tmllm_stream stream);
/* Fused append + decode attention over every sequence of the cache for `layer` (see
 * tmllm_gqa_decode), with a workspace the cache owns.  Blocks for the new positions are
 * reserved first.  The first call for a given (q_heads, splits) shape allocates that
 * workspace; make it before any stream capture.  Lengths are not advanced. */
int tmllm_cache_decode(tmllm_cache* cache, int32_t layer, const void* q, const void* k_new,
                       const void* v_new, void* out, float* lse, int32_t q_heads,
                       const tmllm_decode_opts* opts, tmllm_stream stream);
/* Fused append + causal prefill attention over every sequence of the cache for `layer`
 * (see tmllm_gqa_prefill): sequence s owns rows [s * n, (s + 1) * n) of q / k_new / v_new /
 * out.  Blocks for the n new positions of every sequence are reserved first.  Lengths are
 * not advanced (tmllm_cache_advance by n after the last layer). */
int tmllm_cache_prefill(tmllm_cache* cache, int32_t layer, const void* q, const void* k_new,
                        const void* v_new, int64_t n, void* out, int32_t q_heads,
                        const tmllm_decode_opts* opts, tmllm_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* TMLLM_H */
