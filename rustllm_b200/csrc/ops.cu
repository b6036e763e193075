// Op-level kernels: the reference's stand-alone operators, one CUDA kernel each.
//
// These are not the hot path (the fused decode kernel in decode.cu is); they give the
// reference's op-by-op API surface with the reference's arithmetic: every sum runs in the
// same order as the Metal kernel's single accumulator, products and sums are rounded
// separately (__fmul_rn/__fadd_rn, no contraction) and F16 results are rounded at the
// same store points.  Results are therefore bit-identical to the CPU restatement except
// where exp() is involved (softmax), which differs by at most a couple of ulp.
#include <cmath>
#include <vector>

#include "common.cuh"

namespace tmllm {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t total) {
    int64_t blocks = (total + kThreads - 1) / kThreads;
    int64_t cap = static_cast<int64_t>(device_sm_count()) * 32;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return static_cast<int>(blocks);
}

// ---- row gathers: kv_cache_write, concat_sequence, repeat_kv --------------------------

// kernels/kv_cache_write.metal:13-18 lifted from elements to rows: source row
// r = head*source_seq + s goes to cache row head*max_seq + start + s.
struct KvWriteMap {
    int64_t source_seq, max_seq, start;
    __device__ int64_t dst_row(int64_t r) const {
        return (r / source_seq) * max_seq + start + r % source_seq;
    }
    __device__ int64_t src_row(int64_t r, int* which) const {
        *which = 0;
        return r;
    }
};

// kernels/concat_sequence.metal:66-88 by rows: out row (bh, s) reads left row
// (bh, s) when s < left_seq, else right row (bh, s - left_seq).
struct ConcatMap {
    int64_t left_seq, right_seq;
    __device__ int64_t dst_row(int64_t r) const { return r; }
    __device__ int64_t src_row(int64_t r, int* which) const {
        int64_t out_seq = left_seq + right_seq;
        int64_t bh = r / out_seq, s = r % out_seq;
        if (s < left_seq) {
            *which = 0;
            return bh * left_seq + s;
        }
        *which = 1;
        return bh * right_seq + (s - left_seq);
    }
};

// kernels/repeat_kv.metal:16-30 by rows: out row (b, qh, s) reads (b, qh/r, s).
struct RepeatMap {
    int64_t kv_heads, seq_len, repeats;
    __device__ int64_t dst_row(int64_t r) const { return r; }
    __device__ int64_t src_row(int64_t r, int* which) const {
        *which = 0;
        int64_t s = r % seq_len, t = r / seq_len;
        int64_t qh = t % (kv_heads * repeats), b = t / (kv_heads * repeats);
        return (b * kv_heads + qh / repeats) * seq_len + s;
    }
};

template <typename V, typename Map>
__global__ void gather_rows_kernel(V* __restrict__ dst, const V* __restrict__ src0,
                                   const V* __restrict__ src1, int64_t nrows, int64_t row_vecs,
                                   Map map) {
    const int64_t total = nrows * row_vecs;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t row = i / row_vecs, c = i - row * row_vecs;
        int which;
        int64_t sr = map.src_row(row, &which);
        const V* s = which ? src1 : src0;
        dst[map.dst_row(row) * row_vecs + c] = s[sr * row_vecs + c];
    }
}

template <typename Map>
int launch_gather(void* dst, const void* s0, const void* s1, int64_t nrows, int64_t row_bytes,
                  size_t esize, Map map, cudaStream_t stream) {
    if (nrows == 0 || row_bytes == 0) return TMLLM_OK;
    const bool vec = (row_bytes % 16 == 0) && aligned16(dst) && aligned16(s0) &&
                     (s1 == nullptr || aligned16(s1));
    if (vec) {
        int64_t rv = row_bytes / 16;
        gather_rows_kernel<uint4, Map><<<grid_for(nrows * rv), kThreads, 0, stream>>>(
            static_cast<uint4*>(dst), static_cast<const uint4*>(s0),
            static_cast<const uint4*>(s1), nrows, rv, map);
    } else if (esize == 2) {
        int64_t rv = row_bytes / 2;
        gather_rows_kernel<uint16_t, Map><<<grid_for(nrows * rv), kThreads, 0, stream>>>(
            static_cast<uint16_t*>(dst), static_cast<const uint16_t*>(s0),
            static_cast<const uint16_t*>(s1), nrows, rv, map);
    } else {
        int64_t rv = row_bytes / 4;
        gather_rows_kernel<uint32_t, Map><<<grid_for(nrows * rv), kThreads, 0, stream>>>(
            static_cast<uint32_t*>(dst), static_cast<const uint32_t*>(s0),
            static_cast<const uint32_t*>(s1), nrows, rv, map);
    }
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

// ---- attention ops ------------------------------------------------------------------

// kernels/gqa_matmul.metal:25-160 / 163-321: one output per thread, d increasing.
template <typename T>
__global__ void gqa_qk_kernel(const T* __restrict__ q, const T* __restrict__ k,
                              T* __restrict__ out, int64_t q_heads, int64_t kv_heads,
                              int64_t q_len, int64_t kv_len, int64_t head_dim, int64_t cap,
                              int64_t total) {
    const int64_t groups = q_heads / kv_heads;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t j = idx % kv_len, t = idx / kv_len;
        int64_t i = t % q_len;
        t /= q_len;
        int64_t qh = t % q_heads, b = t / q_heads;
        const T* qr = q + ((b * q_heads + qh) * q_len + i) * head_dim;
        const T* kr = k + ((b * kv_heads + qh / groups) * cap + j) * head_dim;
        float sum = 0.0f;
        for (int64_t d = 0; d < head_dim; ++d)
            sum = __fadd_rn(sum, __fmul_rn(to_f32<T>(qr[d]), to_f32<T>(kr[d])));
        out[idx] = from_f32<T>(sum);
    }
}

// kernels/gqa_matmul.metal:341-472 / 493-628: one output per thread, key j increasing.
template <typename T>
__global__ void gqa_pv_kernel(const T* __restrict__ p, const T* __restrict__ v,
                              T* __restrict__ out, int64_t q_heads, int64_t kv_heads,
                              int64_t q_len, int64_t kv_len, int64_t head_dim, int64_t cap,
                              int64_t total) {
    const int64_t groups = q_heads / kv_heads;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t d = idx % head_dim, t = idx / head_dim;
        int64_t i = t % q_len;
        t /= q_len;
        int64_t qh = t % q_heads, b = t / q_heads;
        const T* pr = p + ((b * q_heads + qh) * q_len + i) * kv_len;
        const T* vr = v + (b * kv_heads + qh / groups) * cap * head_dim + d;
        float sum = 0.0f;
        for (int64_t j = 0; j < kv_len; ++j)
            sum = __fadd_rn(sum, __fmul_rn(to_f32<T>(pr[j]), to_f32<T>(vr[j * head_dim])));
        out[idx] = from_f32<T>(sum);
    }
}

// kernels/attention_scale_mask.metal:21-41 / 62-70.
template <typename T>
__global__ void scale_mask_kernel(const T* __restrict__ in, T* __restrict__ out, float scale,
                                  int64_t query_len, int64_t key_len, int64_t start,
                                  int64_t total) {
    for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < total;
         id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t key = id % key_len;
        int64_t qi = (id / key_len) % query_len;
        out[id] = key > start + qi ? from_f32<T>(-INFINITY)
                                   : from_f32<T>(__fmul_rn(to_f32<T>(in[id]), scale));
    }
}

// The same with one 16-byte chunk per thread (key_len a multiple of the chunk's elements,
// 16-byte aligned tensors): the row of a chunk is found once, not per element.
template <typename T>
__global__ void scale_mask_vec_kernel(const T* __restrict__ in, T* __restrict__ out,
                                      float scale, int64_t query_len, int64_t key_len,
                                      int64_t start, int64_t chunks) {
    constexpr int EPC = 16 / sizeof(T);
    const int64_t cpr = key_len / EPC;  // chunks per row
    for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < chunks;
         id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = id / cpr;
        const int64_t key0 = (id - row * cpr) * EPC;
        const int64_t lim = start + row % query_len;  // keys > lim are masked
        uint4 raw = __ldg(reinterpret_cast<const uint4*>(in) + id);
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int k = 0; k < EPC; ++k)
            e[k] = key0 + k > lim ? from_f32<T>(-INFINITY)
                                  : from_f32<T>(__fmul_rn(to_f32<T>(e[k]), scale));
        reinterpret_cast<uint4*>(out)[id] = raw;
    }
}

// kernels/softmax.metal: one 256-thread block per row; element t, t+256, ... folded by
// thread t, then a halving tree over the 256 partials (the reference's order).
template <typename T, bool kZeroMaskedRow>
__global__ void __launch_bounds__(256) softmax_kernel(const T* __restrict__ in,
                                                      T* __restrict__ out, int64_t width) {
    __shared__ float sh[256];
    const int t = threadIdx.x;
    const T* x = in + blockIdx.x * width;
    T* y = out + blockIdx.x * width;
    float m = -INFINITY;
    for (int64_t i = t; i < width; i += 256) m = fmaxf(m, to_f32<T>(x[i]));
    sh[t] = m;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (t < s) sh[t] = fmaxf(sh[t], sh[t + s]);
        __syncthreads();
    }
    const float row_max = sh[0];
    __syncthreads();
    if (kZeroMaskedRow && isinf(row_max) && row_max < 0.0f) {  // softmax.metal:166-173
        for (int64_t i = t; i < width; i += 256) y[i] = from_f32<T>(0.0f);
        return;
    }
    float acc = 0.0f;
    for (int64_t i = t; i < width; i += 256)
        acc = __fadd_rn(acc, expf(__fsub_rn(to_f32<T>(x[i]), row_max)));
    sh[t] = acc;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (t < s) sh[t] = __fadd_rn(sh[t], sh[t + s]);
        __syncthreads();
    }
    const float denom = sh[0];
    for (int64_t i = t; i < width; i += 256)
        y[i] = from_f32<T>(__fdiv_rn(expf(__fsub_rn(to_f32<T>(x[i]), row_max)), denom));
}

// kernels/batched_matmul.metal:20-132 / 151-196.
template <typename T>
__global__ void bmm_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out,
                           int64_t m, int64_t k, int64_t n, int64_t total) {
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t c = idx % n, t = idx / n;
        int64_t r = t % m, z = t / m;
        const T* ar = a + (z * m + r) * k;
        const T* bc = b + z * k * n + c;
        float sum = 0.0f;
        for (int64_t i = 0; i < k; ++i)
            sum = __fadd_rn(sum, __fmul_rn(to_f32<T>(ar[i]), to_f32<T>(bc[i * n])));
        out[idx] = from_f32<T>(sum);
    }
}

// kernels/rope.metal:23-63 / 82-96: half-split pairs.
template <typename T>
__global__ void rope_kernel(const T* __restrict__ in, T* __restrict__ out,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            int64_t seq_len, int64_t head_dim, int64_t start, int64_t total) {
    const int64_t half = head_dim / 2;
    for (int64_t id = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; id < total;
         id += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t pair = id % half, row = id / half;
        int64_t pos = row % seq_len;
        int64_t f = row * head_dim + pair, s = f + half;
        int64_t ti = (start + pos) * half + pair;
        float c = cos_t[ti], sn = sin_t[ti];
        float x1 = to_f32<T>(in[f]), x2 = to_f32<T>(in[s]);
        out[f] = from_f32<T>(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
        out[s] = from_f32<T>(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn)));
    }
}

int check_dtype(int dtype) {
    if (!valid_dtype(dtype)) return fail(TMLLM_UNSUPPORTED_DTYPE, "unknown dtype %d", dtype);
    return TMLLM_OK;
}

}  // namespace
}  // namespace tmllm

using namespace tmllm;

extern "C" {

int tmllm_kv_cache_write(tmllm_dtype dtype, void* cache, const void* source, size_t num_heads,
                         size_t max_seq, size_t head_dim, size_t start, size_t source_seq,
                         tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (num_heads == 0 || max_seq == 0 || head_dim == 0)
        return fail(TMLLM_INVALID_SHAPE, "invalid KV cache write shape");
    if (start > max_seq || source_seq > max_seq - start)
        return fail_position(static_cast<int64_t>(start), static_cast<int64_t>(source_seq),
                             static_cast<int64_t>(max_seq));
    int64_t numel;
    if (!checked_numel({num_heads, max_seq, head_dim, dtype_size(dtype)}, &numel) ||
        numel / static_cast<int64_t>(dtype_size(dtype)) > UINT32_MAX)
        return fail(TMLLM_INVALID_SHAPE, "KV cache dimension exceeds u32");
    if (source_seq == 0) return TMLLM_OK;
    if (!cache || !source) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    KvWriteMap map{static_cast<int64_t>(source_seq), static_cast<int64_t>(max_seq),
                   static_cast<int64_t>(start)};
    return launch_gather(cache, source, nullptr, static_cast<int64_t>(num_heads * source_seq),
                         static_cast<int64_t>(head_dim * dtype_size(dtype)), dtype_size(dtype),
                         map, reinterpret_cast<cudaStream_t>(stream));
}

int tmllm_concat_sequence(tmllm_dtype dtype, const void* left, const void* right, void* out,
                          size_t batch, size_t num_heads, size_t left_seq, size_t right_seq,
                          size_t head_dim, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    int64_t numel;
    if (left_seq > SIZE_MAX - right_seq ||
        !checked_numel({batch, num_heads, left_seq + right_seq, head_dim, dtype_size(dtype)},
                       &numel))
        return fail(TMLLM_INVALID_SHAPE, "concatenated tensor size overflow");
    if (numel == 0) return TMLLM_OK;
    if (!out || (left_seq && !left) || (right_seq && !right))
        return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    ConcatMap map{static_cast<int64_t>(left_seq), static_cast<int64_t>(right_seq)};
    return launch_gather(out, left ? left : right, right ? right : left,
                         static_cast<int64_t>(batch * num_heads * (left_seq + right_seq)),
                         static_cast<int64_t>(head_dim * dtype_size(dtype)), dtype_size(dtype),
                         map, reinterpret_cast<cudaStream_t>(stream));
}

int tmllm_repeat_kv(tmllm_dtype dtype, const void* in, void* out, size_t batch,
                    size_t kv_heads, size_t seq_len, size_t head_dim, size_t repeats,
                    tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (repeats == 0)
        return fail(TMLLM_MODEL_FORMAT, "repeat_kv repeats must be greater than zero");
    int64_t numel;
    if (!checked_numel({batch, kv_heads, repeats, seq_len, head_dim, dtype_size(dtype)}, &numel))
        return fail(TMLLM_MODEL_FORMAT, "repeat_kv head count overflow");
    if (numel == 0) return TMLLM_OK;
    if (!in || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    RepeatMap map{static_cast<int64_t>(kv_heads), static_cast<int64_t>(seq_len),
                  static_cast<int64_t>(repeats)};
    return launch_gather(out, in, nullptr,
                         static_cast<int64_t>(batch * kv_heads * repeats * seq_len),
                         static_cast<int64_t>(head_dim * dtype_size(dtype)), dtype_size(dtype),
                         map, reinterpret_cast<cudaStream_t>(stream));
}

static int validate_gqa(size_t q_heads, size_t kv_heads, size_t kv_len, size_t kv_capacity) {
    if (kv_heads == 0 || q_heads % kv_heads != 0)
        return fail(TMLLM_MODEL_FORMAT, "Q heads %zu must be divisible by non-zero KV heads %zu",
                    q_heads, kv_heads);
    if (kv_capacity < kv_len)
        return fail(TMLLM_INVALID_SHAPE, "KV capacity %zu is smaller than KV length %zu",
                    kv_capacity, kv_len);
    return TMLLM_OK;
}

int tmllm_gqa_qk(tmllm_dtype dtype, const void* q, const void* k, void* out, size_t batch,
                 size_t q_heads, size_t kv_heads, size_t q_len, size_t kv_len,
                 size_t head_dim, size_t kv_capacity, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (int st = validate_gqa(q_heads, kv_heads, kv_len, kv_capacity)) return st;
    int64_t total, kbytes;
    if (!checked_numel({batch, q_heads, q_len, kv_len}, &total) ||
        !checked_numel({batch, kv_heads, kv_capacity, head_dim}, &kbytes) ||
        total > static_cast<int64_t>(UINT32_MAX) * 16)
        return fail(TMLLM_INVALID_SHAPE, "GQA dimension exceeds u32");
    if (total == 0) return TMLLM_OK;
    if (!q || !k || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        gqa_qk_kernel<__half><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const __half*>(q), static_cast<const __half*>(k),
            static_cast<__half*>(out), q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity,
            total);
    else
        gqa_qk_kernel<float><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const float*>(q), static_cast<const float*>(k), static_cast<float*>(out),
            q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity, total);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_gqa_pv(tmllm_dtype dtype, const void* probs, const void* v, void* out,
                 size_t batch, size_t q_heads, size_t kv_heads, size_t q_len, size_t kv_len,
                 size_t head_dim, size_t kv_capacity, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (int st = validate_gqa(q_heads, kv_heads, kv_len, kv_capacity)) return st;
    int64_t total, pbytes;
    if (!checked_numel({batch, q_heads, q_len, head_dim}, &total) ||
        !checked_numel({batch, q_heads, q_len, kv_len}, &pbytes))
        return fail(TMLLM_INVALID_SHAPE, "GQA dimension exceeds u32");
    if (total == 0) return TMLLM_OK;
    if (!probs || !v || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        gqa_pv_kernel<__half><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const __half*>(probs), static_cast<const __half*>(v),
            static_cast<__half*>(out), q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity,
            total);
    else
        gqa_pv_kernel<float><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const float*>(probs), static_cast<const float*>(v),
            static_cast<float*>(out), q_heads, kv_heads, q_len, kv_len, head_dim, kv_capacity,
            total);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_attention_scale_mask(tmllm_dtype dtype, const void* in, void* out, size_t numel,
                               size_t query_len, size_t key_len, size_t query_start_pos,
                               float scale, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    // src/ops/attention_scale_mask.rs:120-160
    if (query_len == 0 || key_len == 0)
        return fail(TMLLM_INVALID_SHAPE, "attention query/key length cannot be zero");
    if (!std::isfinite(scale) || scale <= 0.0f)
        return fail(TMLLM_INVALID_SHAPE, "attention scale must be positive and finite, got %g",
                    static_cast<double>(scale));
    if (query_start_pos > SIZE_MAX - query_len || query_start_pos + query_len > key_len)
        return fail(TMLLM_INVALID_SHAPE,
                    "attention query range [%zu, %zu) exceeds key length %zu", query_start_pos,
                    query_start_pos + query_len, key_len);
    int64_t qk;
    if (!checked_numel({query_len, key_len}, &qk) || numel % static_cast<size_t>(qk) != 0)
        return fail(TMLLM_INVALID_SHAPE,
                    "attention score buffer has %zu elements, incompatible with query_len=%zu, "
                    "key_len=%zu",
                    numel, query_len, key_len);
    if (numel == 0) return TMLLM_OK;
    if (!in || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    int64_t total = static_cast<int64_t>(numel);
    const int64_t epc = dtype == TMLLM_F16 ? 8 : 4;
    if (static_cast<int64_t>(key_len) % epc == 0 && aligned16(in) && aligned16(out)) {
        const int64_t chunks = total / epc;
        if (dtype == TMLLM_F16)
            scale_mask_vec_kernel<__half><<<grid_for(chunks), kThreads, 0, s>>>(
                static_cast<const __half*>(in), static_cast<__half*>(out), scale, query_len,
                key_len, query_start_pos, chunks);
        else
            scale_mask_vec_kernel<float><<<grid_for(chunks), kThreads, 0, s>>>(
                static_cast<const float*>(in), static_cast<float*>(out), scale, query_len,
                key_len, query_start_pos, chunks);
        TMLLM_LAUNCH_TRY();
        return TMLLM_OK;
    }
    if (dtype == TMLLM_F16)
        scale_mask_kernel<__half><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const __half*>(in), static_cast<__half*>(out), scale, query_len, key_len,
            query_start_pos, total);
    else
        scale_mask_kernel<float><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const float*>(in), static_cast<float*>(out), scale, query_len, key_len,
            query_start_pos, total);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_softmax_last_dim(tmllm_dtype dtype, const void* in, void* out, size_t rows,
                           size_t width, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (rows == 0 || width == 0)  // src/ops/softmax.rs:91-96
        return fail(TMLLM_INVALID_SHAPE, "Softmax rows and width must be greater than zero");
    if (width > UINT32_MAX) return fail(TMLLM_INVALID_SHAPE, "Softmax width exceeds u32");
    if (rows > 0x7fffffffull) return fail(TMLLM_INVALID_SHAPE, "Softmax row count too large");
    if (!in || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        softmax_kernel<__half, true><<<static_cast<unsigned>(rows), 256, 0, s>>>(
            static_cast<const __half*>(in), static_cast<__half*>(out), width);
    else
        softmax_kernel<float, false><<<static_cast<unsigned>(rows), 256, 0, s>>>(
            static_cast<const float*>(in), static_cast<float*>(out), width);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_batched_matmul(tmllm_dtype dtype, const void* a, const void* b, void* out,
                         size_t batch, size_t m, size_t k, size_t n, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    int64_t total, ta, tb;
    if (!checked_numel({batch, m, n}, &total) || !checked_numel({batch, m, k}, &ta) ||
        !checked_numel({batch, k, n}, &tb))
        return fail(TMLLM_INVALID_SHAPE, "batched matmul size overflow");
    if (total == 0) return TMLLM_OK;
    if (!a || !b || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        bmm_kernel<__half><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const __half*>(a), static_cast<const __half*>(b),
            static_cast<__half*>(out), m, k, n, total);
    else
        bmm_kernel<float><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(out),
            m, k, n, total);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_rope_tables(float* cos_table, float* sin_table, size_t head_dim,
                      size_t max_seq_len, float theta) {
    clear_error();
    // src/nn/rope.rs:26-42
    if (head_dim == 0 || head_dim % 2 != 0)
        return fail(TMLLM_INVALID_SHAPE, "RoPE head dimension must be positive and even, got %zu",
                    head_dim);
    if (max_seq_len == 0)
        return fail(TMLLM_INVALID_SHAPE, "RoPE max sequence length cannot be zero");
    if (!(theta > 0.0f)) return fail(TMLLM_INVALID_SHAPE, "RoPE theta must be positive");
    if (!cos_table || !sin_table) return fail(TMLLM_INVALID_ARGUMENT, "null table pointer");
    const size_t half = head_dim / 2;
    for (size_t pos = 0; pos < max_seq_len; ++pos)
        for (size_t i = 0; i < half; ++i) {
            float exponent = static_cast<float>(2 * i) / static_cast<float>(head_dim);
            float inv = 1.0f / powf(theta, exponent);
            float angle = static_cast<float>(pos) * inv;
            cos_table[pos * half + i] = cosf(angle);
            sin_table[pos * half + i] = sinf(angle);
        }
    return TMLLM_OK;
}

int tmllm_rope(tmllm_dtype dtype, const void* in, void* out, const float* cos_table,
               const float* sin_table, size_t table_len, size_t rows, size_t seq_len,
               size_t head_dim, size_t start_pos, tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (head_dim == 0 || head_dim % 2 != 0)
        return fail(TMLLM_INVALID_SHAPE, "RoPE head dimension must be positive and even, got %zu",
                    head_dim);
    if (start_pos > SIZE_MAX - seq_len || start_pos + seq_len > table_len)
        return fail(TMLLM_INVALID_SHAPE, "RoPE cos/sin table shape or position range is invalid");
    int64_t total;
    if (!checked_numel({rows, seq_len, head_dim / 2}, &total))
        return fail(TMLLM_INVALID_SHAPE, "RoPE size overflow");
    if (total == 0) return TMLLM_OK;
    if (!in || !out || !cos_table || !sin_table)
        return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        rope_kernel<__half><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const __half*>(in), static_cast<__half*>(out), cos_table, sin_table,
            seq_len, head_dim, start_pos, total);
    else
        rope_kernel<float><<<grid_for(total), kThreads, 0, s>>>(
            static_cast<const float*>(in), static_cast<float*>(out), cos_table, sin_table,
            seq_len, head_dim, start_pos, total);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

}  // extern "C"
