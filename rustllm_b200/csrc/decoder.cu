// The decoder layers around the attention path, as the decode step needs them on the GPU:
// token embedding gather, residual add fused with RMSNorm, SwiGLU, and greedy argmax.
// Each follows the reference kernel it replaces (kernels/embedding.metal,
// kernels/vector_add.metal + kernels/rmsnorm.metal, kernels/silu.metal, and the CPU sampler
// src/generation/sampler.rs) in its storage roundings; the plain GEMMs between them are
// library calls.
#include <cmath>

#include "common.cuh"

namespace tmllm {
namespace {

int grid_rows(int64_t total, int per_block) {
    int64_t b = (total + per_block - 1) / per_block;
    int64_t cap = static_cast<int64_t>(device_sm_count()) * 32;
    return static_cast<int>(b < 1 ? 1 : (b > cap ? cap : b));
}

// kernels/embedding.metal:39-53: out[t, :] = table[ids[t], :].  Ids outside the table
// produce a zero row and set *bad (the host validates ids it provides).
template <typename V>
__global__ void embedding_kernel(V* __restrict__ out, const V* __restrict__ table,
                                 const int32_t* __restrict__ ids, int64_t n, int64_t row_vecs,
                                 int64_t vocab, int* bad) {
    const int64_t total = n * row_vecs;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / row_vecs, c = i - t * row_vecs;
        const int64_t id = ids[t];
        if (id < 0 || id >= vocab) {
            out[i] = V{};
            if (bad && c == 0) atomicExch(bad, 1);
            continue;
        }
        out[i] = table[id * row_vecs + c];
    }
}

// kernels/vector_add.metal:15-21 (half(float(a)+float(b))) followed by
// kernels/rmsnorm.metal:71-126 on the stored sum: y = half(x * rsqrt(mean(x^2) + eps) * w).
// One 256-thread block per row.
template <typename T>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(
    const T* x, const T* __restrict__ residual, const T* __restrict__ w, T* __restrict__ y,
    T* sum_out, int64_t hidden, float eps) {
    __shared__ float part[256];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * hidden;
    const T* rr = residual ? residual + row * hidden : nullptr;
    T* so = sum_out ? sum_out + row * hidden : nullptr;
    float acc = 0.f;
    for (int64_t i = threadIdx.x; i < hidden; i += 256) {
        float v = to_f32<T>(xr[i]);
        if (rr) v = round_store<T>(__fadd_rn(v, to_f32<T>(rr[i])));
        if (so) so[i] = from_f32<T>(v);
        acc = fmaf(v, v, acc);
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) part[threadIdx.x] += part[threadIdx.x + s];
        __syncthreads();
    }
    const float inv = rsqrtf(part[0] / static_cast<float>(hidden) + eps);
    for (int64_t i = threadIdx.x; i < hidden; i += 256) {
        // the stored sum when there is one (sum_out may alias x), else recompute it
        float v;
        if (so) {
            v = to_f32<T>(so[i]);
        } else {
            v = to_f32<T>(xr[i]);
            if (rr) v = round_store<T>(__fadd_rn(v, to_f32<T>(rr[i])));
        }
        y[row * hidden + i] = from_f32<T>(v * inv * to_f32<T>(w[i]));
    }
}

// kernels/silu.metal:38-46 on a fused [gate | up] projection: out = half(silu(g) * u),
// silu(g) = g / (1 + exp(-g)).
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows,
                              int64_t inter) {
    const int64_t total = rows * inter;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / inter, c = i - r * inter;
        const float g = to_f32<T>(gu[r * 2 * inter + c]);
        const float u = to_f32<T>(gu[r * 2 * inter + inter + c]);
        out[i] = from_f32<T>((g / (1.0f + expf(-g))) * u);
    }
}

// Greedy next token (src/generation/sampler.rs:79-88): the index of the largest logit;
// among equal maxima the last one wins (Iterator::max_by keeps the last maximum).
template <typename T>
__global__ void __launch_bounds__(256) argmax_kernel(const T* __restrict__ logits,
                                                     int32_t* __restrict__ ids, int64_t vocab) {
    __shared__ float bv[256];
    __shared__ int64_t bi[256];
    const T* row = logits + static_cast<int64_t>(blockIdx.x) * vocab;
    float best = -INFINITY;
    int64_t idx = -1;
    for (int64_t i = threadIdx.x; i < vocab; i += 256) {
        const float v = to_f32<T>(row[i]);
        if (idx < 0 || v >= best) {  // later index wins ties within a thread
            best = v;
            idx = i;
        }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = bv[threadIdx.x + s];
            const int64_t oi = bi[threadIdx.x + s];
            const bool take = oi >= 0 && (bi[threadIdx.x] < 0 || ov > bv[threadIdx.x] ||
                                          (ov == bv[threadIdx.x] && oi > bi[threadIdx.x]));
            if (take) {
                bv[threadIdx.x] = ov;
                bi[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) ids[blockIdx.x] = static_cast<int32_t>(bi[0] < 0 ? 0 : bi[0]);
}

int check_dtype(int dtype) {
    if (!valid_dtype(dtype)) return fail(TMLLM_UNSUPPORTED_DTYPE, "unknown dtype %d", dtype);
    return TMLLM_OK;
}

}  // namespace
}  // namespace tmllm

using namespace tmllm;

extern "C" {

int tmllm_embedding(tmllm_dtype dtype, const void* table, const int32_t* ids, void* out,
                    size_t n, size_t hidden, size_t vocab, int32_t* bad_id_flag,
                    tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (hidden == 0 || vocab == 0) return fail(TMLLM_INVALID_SHAPE, "embedding dimensions must be positive");
    if (n == 0) return TMLLM_OK;
    if (!table || !ids || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    const size_t row_bytes = hidden * dtype_size(dtype);
    int* bad = reinterpret_cast<int*>(bad_id_flag);
    if (row_bytes % 16 == 0 && aligned16(table) && aligned16(out)) {
        const int64_t rv = row_bytes / 16;
        embedding_kernel<uint4><<<grid_rows(n * rv, 256), 256, 0, s>>>(
            static_cast<uint4*>(out), static_cast<const uint4*>(table), ids, n, rv, vocab, bad);
    } else if (dtype == TMLLM_F16) {
        embedding_kernel<uint16_t><<<grid_rows(n * hidden, 256), 256, 0, s>>>(
            static_cast<uint16_t*>(out), static_cast<const uint16_t*>(table), ids, n, hidden,
            vocab, bad);
    } else {
        embedding_kernel<uint32_t><<<grid_rows(n * hidden, 256), 256, 0, s>>>(
            static_cast<uint32_t*>(out), static_cast<const uint32_t*>(table), ids, n, hidden,
            vocab, bad);
    }
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_add_rmsnorm(tmllm_dtype dtype, const void* x, const void* residual, const void* weight,
                      void* out, void* sum_out, size_t rows, size_t hidden, float eps,
                      tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (hidden == 0) return fail(TMLLM_INVALID_SHAPE, "RMSNorm hidden size cannot be zero");
    if (!std::isfinite(eps) || eps <= 0.0f)  // src/nn/rmsnorm.rs:29-33
        return fail(TMLLM_INVALID_SHAPE, "RMSNorm epsilon must be positive, got %g",
                    static_cast<double>(eps));
    if (rows == 0) return TMLLM_OK;
    if (rows > 0x7fffffffull) return fail(TMLLM_INVALID_SHAPE, "too many rows");
    if (!x || !weight || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        add_rmsnorm_kernel<__half><<<static_cast<unsigned>(rows), 256, 0, s>>>(
            static_cast<const __half*>(x), static_cast<const __half*>(residual),
            static_cast<const __half*>(weight), static_cast<__half*>(out),
            static_cast<__half*>(sum_out), hidden, eps);
    else
        add_rmsnorm_kernel<float><<<static_cast<unsigned>(rows), 256, 0, s>>>(
            static_cast<const float*>(x), static_cast<const float*>(residual),
            static_cast<const float*>(weight), static_cast<float*>(out),
            static_cast<float*>(sum_out), hidden, eps);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_swiglu(tmllm_dtype dtype, const void* gate_up, void* out, size_t rows, size_t inter,
                 tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (rows == 0 || inter == 0) return TMLLM_OK;
    if (!gate_up || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t total = static_cast<int64_t>(rows * inter);
    if (dtype == TMLLM_F16)
        swiglu_kernel<__half><<<grid_rows(total, 256), 256, 0, s>>>(
            static_cast<const __half*>(gate_up), static_cast<__half*>(out), rows, inter);
    else
        swiglu_kernel<float><<<grid_rows(total, 256), 256, 0, s>>>(
            static_cast<const float*>(gate_up), static_cast<float*>(out), rows, inter);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_argmax(tmllm_dtype dtype, const void* logits, int32_t* ids, size_t rows, size_t vocab,
                 tmllm_stream stream) {
    clear_error();
    if (int st = check_dtype(dtype)) return st;
    if (vocab == 0) return fail(TMLLM_INVALID_SHAPE, "vocabulary size cannot be zero");
    if (vocab > INT32_MAX) return fail(TMLLM_INVALID_SHAPE, "vocabulary exceeds i32");
    if (rows == 0) return TMLLM_OK;
    if (rows > 0x7fffffffull) return fail(TMLLM_INVALID_SHAPE, "too many rows");
    if (!logits || !ids) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == TMLLM_F16)
        argmax_kernel<__half><<<static_cast<unsigned>(rows), 256, 0, s>>>(
            static_cast<const __half*>(logits), ids, vocab);
    else
        argmax_kernel<float><<<static_cast<unsigned>(rows), 256, 0, s>>>(
            static_cast<const float*>(logits), ids, vocab);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

}  // extern "C"
