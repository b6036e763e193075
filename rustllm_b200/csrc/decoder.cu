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

// The same operation with one warp per row (8 rows per 256-thread block), the row held in
// registers as 16-byte chunks of 8 halves: one read of x and residual, one write of the sum
// and of y, a shuffle reduction.  For F16 rows of hidden % 8 == 0 and hidden <= 2048.
constexpr int kNormChunks = 8;  // chunks per lane: hidden <= 32 * 8 * 8
__global__ void __launch_bounds__(256) add_rmsnorm_warp_kernel(
    const __half* x, const __half* __restrict__ residual, const __half* __restrict__ w,
    __half* __restrict__ y, __half* sum_out, int64_t rows, int64_t hidden, float eps) {
    const int64_t row = blockIdx.x * 8LL + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int nc = static_cast<int>(hidden / 8);
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * hidden);
    const uint4* rr = residual ? reinterpret_cast<const uint4*>(residual + row * hidden) : nullptr;
    float v[kNormChunks][8];
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kNormChunks; ++k) {
        const int c = lane + 32 * k;
        if (c >= nc) break;
        Chunk<__half>::unpack(xr[c], v[k]);
        if (rr) {
            float r8[8];
            Chunk<__half>::unpack(rr[c], r8);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[k][e] = round_store<__half>(__fadd_rn(v[k][e], r8[e]));
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(v[k][e], v[k][e], acc);
    }
    acc = warp_sum(acc);
    const float inv = rsqrtf(acc / static_cast<float>(hidden) + eps);
    uint4* so = sum_out ? reinterpret_cast<uint4*>(sum_out + row * hidden) : nullptr;
    uint4* yr = reinterpret_cast<uint4*>(y + row * hidden);
    const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
    for (int k = 0; k < kNormChunks; ++k) {
        const int c = lane + 32 * k;
        if (c >= nc) break;
        float w8[8];
        Chunk<__half>::unpack(wr[c], w8);
        uint4 ys, ss;
        __half2* yh = reinterpret_cast<__half2*>(&ys);
        __half2* sh = reinterpret_cast<__half2*>(&ss);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            yh[e] = __floats2half2_rn(v[k][2 * e] * inv * w8[2 * e],
                                      v[k][2 * e + 1] * inv * w8[2 * e + 1]);
            sh[e] = __floats2half2_rn(v[k][2 * e], v[k][2 * e + 1]);
        }
        if (so) so[c] = ss;
        yr[c] = ys;
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

// swiglu_kernel on 8 F16 outputs per thread (16-byte loads of gate and up, one store).
__global__ void swiglu_vec_kernel(const __half* __restrict__ gu, __half* __restrict__ out,
                                  int64_t rows, int64_t inter) {
    const int64_t per_row = inter / 8;
    const int64_t total = rows * per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_row, c = i - r * per_row;
        const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter) + c);
        const uint4 u4 = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter) + c);
        float g[8], u[8];
        Chunk<__half>::unpack(g4, g);
        Chunk<__half>::unpack(u4, u);
        uint4 o;
        __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            oh[e] = __floats2half2_rn((g[2 * e] / (1.0f + expf(-g[2 * e]))) * u[2 * e],
                                      (g[2 * e + 1] / (1.0f + expf(-g[2 * e + 1]))) * u[2 * e + 1]);
        reinterpret_cast<uint4*>(out + r * inter)[c] = o;
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
    if (dtype == TMLLM_F16 && hidden % 8 == 0 && hidden <= 32 * kNormChunks * 8 &&
        aligned16(x) && aligned16(weight) && aligned16(out) &&
        (!residual || aligned16(residual)) && (!sum_out || aligned16(sum_out))) {
        add_rmsnorm_warp_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(
            static_cast<const __half*>(x), static_cast<const __half*>(residual),
            static_cast<const __half*>(weight), static_cast<__half*>(out),
            static_cast<__half*>(sum_out), static_cast<int64_t>(rows),
            static_cast<int64_t>(hidden), eps);
    } else if (dtype == TMLLM_F16)
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
    if (dtype == TMLLM_F16 && inter % 8 == 0 && aligned16(gate_up) && aligned16(out))
        swiglu_vec_kernel<<<grid_rows(total / 8, 256), 256, 0, s>>>(
            static_cast<const __half*>(gate_up), static_cast<__half*>(out), rows, inter);
    else if (dtype == TMLLM_F16)
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
