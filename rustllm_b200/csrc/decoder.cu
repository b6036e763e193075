// The decoder layers around the attention path, as the decode step needs them on the GPU:
// token embedding gather, residual add fused with RMSNorm, SwiGLU, and greedy argmax.
// Each follows the reference kernel it replaces (kernels/embedding.metal,
// kernels/vector_add.metal + kernels/rmsnorm.metal, kernels/silu.metal, and the CPU sampler
// src/generation/sampler.rs) in its storage roundings.  The projections of a decode step
// (at most 64 rows) run in tmllm_linear, with the norm, SwiGLU and residual add fused into
// it; the projections of a prompt (many rows) are library GEMMs.
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "tc.cuh"


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

// Greedy next token (src/generation/sampler.rs:79-88, greedy_from_slice): the index of the
// largest FINITE logit under f32::total_cmp (so -0 < +0), the last one among equal maxima
// (Iterator::max_by keeps the last maximum); -1 when a row holds no finite logit (the
// reference's TinyError::Sampling).  A candidate is the 64-bit key (total-order bits of the
// value) << 32 | index, so one unsigned max picks the value and, among equal values, the
// largest index.  One 1024-thread CTA per row; with 16-byte aligned rows every thread
// issues its 16-byte loads (up to eight at a time) before it compares.
__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t i) {
    if (!isfinite(v)) return 0ull;
    const uint32_t u = __float_as_uint(v);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // total_cmp order
    return (static_cast<unsigned long long>(ord) << 32) | static_cast<uint32_t>(i);
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ logits,
                                                      int32_t* __restrict__ ids, int64_t vocab,
                                                      bool vec) {
    __shared__ unsigned long long best_w[32];
    const T* row = logits + static_cast<int64_t>(blockIdx.x) * vocab;
    const int tid = threadIdx.x;
    unsigned long long best = 0ull;  // below every finite key
    if (vec) {
        constexpr int E = 16 / sizeof(T);  // elements per 16-byte chunk
        const int64_t nch = vocab / E;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        for (int64_t c0 = tid; c0 < nch; c0 += 8 * 1024) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t c = c0 + static_cast<int64_t>(u) * 1024;
                v[u] = c < nch ? __ldg(rv + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t c = c0 + static_cast<int64_t>(u) * 1024;
                if (c >= nch) break;
                float f[E];
                Chunk<T>::unpack(v[u], f);
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const unsigned long long k = argmax_key(f[e], c * E + e);
                    best = k > best ? k : best;
                }
            }
        }
        for (int64_t i = nch * E + tid; i < vocab; i += 1024) {  // tail (vocab % E)
            const unsigned long long k = argmax_key(to_f32<T>(row[i]), i);
            best = k > best ? k : best;
        }
    } else {
        for (int64_t i = tid; i < vocab; i += 1024) {
            const unsigned long long k = argmax_key(to_f32<T>(row[i]), i);
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((tid & 31) == 0) best_w[tid >> 5] = best;
    __syncthreads();
    if (tid < 32) {
        best = best_w[tid];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
            best = k > best ? k : best;
        }
        if (tid == 0)
            ids[blockIdx.x] = best ? static_cast<int32_t>(best & 0xffffffffull) : -1;
    }
}

// ---- Linear layers of a decode step (src/nn/linear.rs: y = x · W with W [in, out]) --------
// With the few rows of a decode step (M <= 64) a projection streams its weight matrix once
// and does little arithmetic, so it is written as a weight-streaming kernel with the
// decoder's neighbouring element-wise work folded in:
//  * RMSNorm of the input rows (kernels/rmsnorm.metal:71-126) as the A operand is staged:
//    1/rms per row comes from row statistics the producing projection wrote (stats_in) or
//    from a pass over the rows, and each staged tile is rewritten in shared memory as
//    half(x * inv * w), the reference's rounding of the normed rows;
//  * SwiGLU (kernels/silu.metal:38-46) on a fused [gate | up] weight: the CTA owns the same
//    columns of both halves and writes half(silu(half(g)) * half(u));
//  * a residual add (kernels/vector_add.metal:15-21): out = half(resid + half(x · W)),
//    optionally with the per-row sums of squares of the stored output (stats_out) that the
//    next norm-fused projection reads instead of re-reading the rows.
// CTA tile: every row (<= 64) × 64 output columns over one K chunk.  The K chunks of a
// column tile are the CTAs of one thread-block cluster (grid y = cluster y <= 8): CTA r
// finishes the row band [r*rbr, (r+1)*rbr); every CTA pushes each band of its F32 partial
// tile into the band owner's shared memory with one bulk copy (cp.async.bulk
// shared::cta -> shared::cluster, completing on the owner's mbarrier), and the owner sums
// the received slots in split order, so the split-K reduction never touches global memory
// and needs no cluster barrier after the K loop.  Weight and x tiles move through a cp.async
// ring; products run on the warp-level tensor cores (mma.sync m16n8k16, F16 in, F32
// accumulate; weight tiles through ldmatrix.trans): with 1-64 rows the layer is bound by
// the weight bytes and by latency, not by the MMA rate.
// Launched with programmatic stream serialisation (opt-in, TMLLM_LINEAR_OVERLAP), a CTA
// starts its weight prefetch while the previous kernel on the stream drains and waits for
// that kernel's results (griddepcontrol.wait) only before it reads x, residual or stats.
constexpr int kLinRows = 64;
constexpr int kLinCols = 64;
constexpr int kLinK = 64;
constexpr int kLinThreads = 128;
constexpr int kLinMaxSplits = 8;                 // portable cluster size
constexpr int kLinSlab = kLinK * kLinCols * 2;  // one 64 x 64 F16 tile (weight or x)
// row statistics hold one partial sum of squares per 16 output columns and row:
// [ceil(N / 16)][64] floats
constexpr int kStatCols = 16;

constexpr unsigned long long kLinWaitNs = 1000000000ull;  // bounded waits: 1 s

__device__ int g_linear_status;

template <int NW> struct LinCfg {
    static constexpr int STAGES = NW == 1 ? 4 : 3;  // 66 / 74 KB: three CTAs per SM
    static constexpr int STAGE = (NW + 1) * kLinSlab + 128;
    static constexpr int PSTRIDE = kLinCols * NW + 4;  // floats per partial row
    static constexpr int RING = STAGES * STAGE;
    static constexpr int OFF_INV = RING;               // [64] floats
    static constexpr int OFF_RECV = RING + 256;        // receive barrier of the partial rows
    static constexpr int OFF_RB = RING + 384;          // [splits][rows a CTA finishes][PSTRIDE]
    // the receive buffer holds at most rows + splits - 1 partial rows
    static constexpr size_t SMEM_MAX =
        OFF_RB + static_cast<size_t>(kLinRows + kLinMaxSplits - 1) * PSTRIDE * 4;
    static_assert(RING >= kLinRows * PSTRIDE * 4, "the partial tile reuses the ring");
};

struct LinearArgs {
    const __half* x;         // [M, K], row stride ldx
    const __half* norm_w;    // [K] RMSNorm weight, or null
    const float* stats_in;   // [ceil(K/64)][64] row sums of squares of x, or null
    const __half* w;         // [K, N] (or [K, 2N] with swiglu), row stride ldw
    __half* out;             // [M, N], row stride ldo
    const __half* resid;     // [M, N] added in the epilogue, or null (may alias out)
    float* stats_out;        // [ceil(N/64)][64] row sums of squares of out, or null
    int64_t ldx, ldw, ldo, ldr;
    int M, K, N, kchunk;
    float eps;
};

__device__ __forceinline__ uint32_t lin_smem(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool lin_mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase: false after kLinWaitNs, recording TMLLM_TIMEOUT (a
// correct run waits microseconds).
__device__ __forceinline__ bool lin_wait(uint32_t bar, uint32_t parity) {
    unsigned long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (lin_mbar_test(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > kLinWaitNs) {
                atomicExch(&g_linear_status, TMLLM_TIMEOUT);
                return false;
            }
        }
    }
}

// 1/rms of rows [0, M) from the row statistics of x ([ceil(K/16)][64] partial sums of
// squares, as the producing projection wrote them): rows in groups of four (one 16-byte
// load per column group), P lanes of one warp per group, each summing a fixed subset with
// eight loads in flight, then a fixed shuffle tree, so the sum has one order.  Every
// thread of the block calls it.
template <int THREADS>
__device__ __forceinline__ void rows_inv_from_stats(const float* __restrict__ stats, int M,
                                                    int K, float eps, float* inv_s) {
    const int tid = threadIdx.x;
    const int groups = (M + 3) / 4;
    int gp = 1;
    while (gp < groups) gp <<= 1;
    const int P = min(32, THREADS / gp);
    const int grp = tid / P, part = tid % P;
    const int kt = (K + kStatCols - 1) / kStatCols;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    if (grp < groups) {
        for (int t0 = part; t0 < kt; t0 += 8 * P) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int t = t0 + u * P;
                v[u] = t < kt ? __ldcg(reinterpret_cast<const float4*>(stats + t * kLinRows + grp * 4))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                s[0] += v[u].x;
                s[1] += v[u].y;
                s[2] += v[u].z;
                s[3] += v[u].w;
            }
        }
    }
    for (int o = P / 2; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
    if (part == 0 && grp < groups)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (grp * 4 + j < M) inv_s[grp * 4 + j] = rsqrtf(s[j] / static_cast<float>(K) + eps);
}

template <int NW>
__global__ void __launch_bounds__(kLinThreads) linear_kernel(const LinearArgs a) {
    using Cfg = LinCfg<NW>;
    constexpr int S = Cfg::STAGES, STAGE = Cfg::STAGE;
    extern __shared__ __align__(128) unsigned char smem[];
    float* inv_s = reinterpret_cast<float*>(smem + Cfg::OFF_INV);  // [64]
    const uint32_t recv = lin_smem(smem + Cfg::OFF_RECV);
    float* rb = reinterpret_cast<float*>(smem + Cfg::OFF_RB);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
    const int n0 = tile * kLinCols;
    const int k0 = split * a.kchunk;
    const int k1 = min(a.K, k0 + a.kchunk);
    const int nkt = k1 > k0 ? (k1 - k0 + kLinK - 1) / kLinK : 0;
    const int MT = (a.M + 15) / 16;
    const bool norm = a.norm_w != nullptr;
    launch_dependents();  // the next projection may start prefetching its weights
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(recv) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // published to the cluster here, awaited only before the partial rows are pushed
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");

    // stage layout: NW weight slabs, the x tile, 64 norm weights; 16-byte chunks swizzled
    // by row (chunk c of row r at r*128 + ((c ^ (r & 7)) << 4)); out-of-range chunks are
    // zero-filled, so K tails add nothing and padding rows / columns are never stored
    auto load_w = [&](int t, int slot) {
        unsigned char* st = smem + slot * STAGE;
        const int kb = k0 + t * kLinK, c = tid & 7;
#pragma unroll
        for (int sl = 0; sl < NW; ++sl) {
            const int colb = sl * a.N + n0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = (tid >> 3) + 16 * i;
                const int k = kb + r, col = n0 + c * 8;
                const bool ok = k < k1 && col < a.N;
                const __half* src = ok ? a.w + static_cast<int64_t>(k) * a.ldw + colb + c * 8 : a.w;
                cp_async16(st + sl * kLinSlab + r * 128 + ((c ^ (r & 7)) << 4), src, ok ? 16 : 0);
            }
        }
    };
    auto load_x = [&](int t, int slot) {
        unsigned char* st = smem + slot * STAGE;
        const int kb = k0 + t * kLinK, c = tid & 7;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = (tid >> 3) + 16 * i;
            if (r >= MT * 16) break;
            const int k = kb + c * 8;
            const bool ok = r < a.M && k < k1;
            const __half* src = ok ? a.x + static_cast<int64_t>(r) * a.ldx + k : a.x;
            cp_async16(st + NW * kLinSlab + r * 128 + ((c ^ (r & 7)) << 4), src, ok ? 16 : 0);
        }
        if (norm && tid < 8) {
            const int k = kb + tid * 8;
            const bool ok = k < k1;
            cp_async16(st + (NW + 1) * kLinSlab + tid * 16, ok ? a.norm_w + k : a.norm_w,
                       ok ? 16 : 0);
        }
    };
    // weights first (constant through a decode step), then wait for the previous kernel;
    // a K chunk that fits the ring is loaded whole here, so none of its weight loads waits
    // for the previous kernel
    const int pro = nkt <= S ? nkt : S - 1;
    for (int t = 0; t < pro; ++t) load_w(t, t);
    grid_dependency_wait();
    for (int t = 0; t < pro; ++t) load_x(t, t);
    cp_async_commit();
    // 1/rms of every row over the whole K while the prologue lands
    if (norm) {
        if (a.stats_in) {
            rows_inv_from_stats<kLinThreads>(a.stats_in, a.M, a.K, a.eps, inv_s);
        } else {
            // four rows per warp at a time, four 16-byte loads per row in flight
            const int nch = a.K / 8;
            for (int m0 = warp * 4; m0 < a.M; m0 += 16) {
                float ss[4] = {0.f, 0.f, 0.f, 0.f};
                for (int c = lane; c < nch; c += 128) {
                    uint4 v[4][4];
#pragma unroll
                    for (int r = 0; r < 4; ++r)
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int cc = c + 32 * u, m = m0 + r;
                            v[r][u] = (m < a.M && cc < nch)
                                          ? __ldg(reinterpret_cast<const uint4*>(
                                                      a.x + static_cast<int64_t>(m) * a.ldx) + cc)
                                          : make_uint4(0, 0, 0, 0);
                        }
#pragma unroll
                    for (int r = 0; r < 4; ++r)
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            float f[8];
                            Chunk<__half>::unpack(v[r][u], f);
#pragma unroll
                            for (int e = 0; e < 8; ++e) ss[r] = fmaf(f[e], f[e], ss[r]);
                        }
                }
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float t = warp_sum(ss[r]);
                    if (lane == 0 && m0 + r < a.M)
                        inv_s[m0 + r] = rsqrtf(t / static_cast<float>(a.K) + a.eps);
                }
            }
        }
    }
    cp_async_wait<0>();

    float acc[4][2 * NW][4];
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int j = 0; j < 2 * NW; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;

    const int mi = lane >> 3;
    for (int t = 0; t < nkt; ++t) {
        // stage t landed (the prologue completely, later stages S-2 groups back); every
        // thread is done with stage t-1, whose slot receives stage t + S - 1
        cp_async_wait<S - 2>();
        __syncthreads();
        {
            const int tn = t + S - 1;
            if (tn >= pro && tn < nkt) {
                load_w(tn, tn % S);
                load_x(tn, tn % S);
            }
            cp_async_commit();
        }
        unsigned char* st = smem + (t % S) * STAGE;
        unsigned char* xs = st + NW * kLinSlab;
        if (norm) {  // rewrite this thread's x chunks as half(x * inv * w)
            const int c = tid & 7;
            float g[8];
            Chunk<__half>::unpack(*reinterpret_cast<const uint4*>(st + (NW + 1) * kLinSlab + c * 16),
                                  g);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = (tid >> 3) + 16 * i;
                if (r >= a.M) break;
                uint4* p = reinterpret_cast<uint4*>(xs + r * 128 + ((c ^ (r & 7)) << 4));
                float v[8];
                Chunk<__half>::unpack(*p, v);
                const float inv = inv_s[r];
                uint4 u;
                __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    h[e] = __floats2half2_rn(v[2 * e] * inv * g[2 * e],
                                             v[2 * e + 1] * inv * g[2 * e + 1]);
                *p = u;
            }
            __syncthreads();
        }
#pragma unroll
        for (int kk = 0; kk < kLinK / 16; ++kk) {
            uint32_t b[NW][4];
#pragma unroll
            for (int sl = 0; sl < NW; ++sl) {
                const int r = kk * 16 + (mi & 1) * 8 + (lane & 7);
                const int c = warp * 2 + (mi >> 1);
                ldsm_x4_t(static_cast<uint32_t>(__cvta_generic_to_shared(
                              st + sl * kLinSlab + r * 128 + ((c ^ (r & 7)) << 4))),
                          b[sl][0], b[sl][1], b[sl][2], b[sl][3]);
            }
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                if (mt >= MT) break;
                const int r = mt * 16 + (mi & 1) * 8 + (lane & 7);
                const int c = kk * 2 + (mi >> 1);
                uint32_t a0, a1, a2, a3;
                ldsm_x4(static_cast<uint32_t>(__cvta_generic_to_shared(
                            xs + r * 128 + ((c ^ (r & 7)) << 4))),
                        a0, a1, a2, a3);
#pragma unroll
                for (int sl = 0; sl < NW; ++sl) {
                    mma16816(acc[mt][2 * sl], a0, a1, a2, a3, b[sl][0], b[sl][1]);
                    mma16816(acc[mt][2 * sl + 1], a0, a1, a2, a3, b[sl][2], b[sl][3]);
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // the ring is free: it holds this CTA's partial tile from here on

    // partial tile ps[m][cl] (cl < 64: gate / plain columns, cl >= 64: up columns); fragment
    // (mt, j, e) is row mt*16 + g4 (+8 for e >= 2), column (j/2)*64 + warp*16 + (j%2)*8 +
    // t4*2 + (e & 1)
    float* ps = reinterpret_cast<float*>(smem);
    const int g4 = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        if (mt >= MT) break;
#pragma unroll
        for (int j = 0; j < 2 * NW; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = mt * 16 + g4 + 8 * h;
                const int cl = (j >> 1) * kLinCols + warp * 16 + (j & 1) * 8 + t4 * 2;
                *reinterpret_cast<float2*>(ps + m * Cfg::PSTRIDE + cl) =
                    make_float2(acc[mt][j][2 * h], acc[mt][j][2 * h + 1]);
            }
    }
    // rows are finished in bands: CTA `split` owns rows [split*rbr, split*rbr + rbr).  Each
    // CTA pushes the band of its partial tile to the band's owner with one bulk copy into
    // the owner's receive buffer (slot = the sender's split); the owner sums the slots in
    // split order.  A single K chunk finishes straight from its own partial tile.
    const int rbr = (a.M + splits - 1) / splits;
    const int m0 = split * rbr;
    const int mine = max(0, min(a.M, m0 + rbr) - m0);
    const float* src = ps;
    // this thread's first output chunk: its residual is loaded now, so the load overlaps
    // the exchange of the partial rows (the residual may alias out: this CTA alone writes
    // these rows and columns, later)
    uint4 resid0 = make_uint4(0, 0, 0, 0);
    if (a.resid && (tid >> 3) < mine && n0 + (tid & 7) * 8 < a.N)
        resid0 = *reinterpret_cast<const uint4*>(
            a.resid + static_cast<int64_t>(m0 + (tid >> 3)) * a.ldr + n0 + (tid & 7) * 8);
    if (splits > 1) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // ps, for the copy engine
        __syncthreads();
        asm volatile("barrier.cluster.wait;" ::: "memory");  // every receive barrier is initialised
        if (tid < splits) {  // thread r pushes band r to its owner, the copies issued in parallel
            const int r = tid;
            const int b0 = r * rbr, b1 = min(a.M, b0 + rbr);
            if (b1 > b0) {
                uint32_t dst, bar;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                             : "=r"(dst)
                             : "r"(lin_smem(rb + split * rbr * Cfg::PSTRIDE)), "r"(r));
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(recv), "r"(r));
                asm volatile(
                    "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes"
                    " [%0], [%1], %2, [%3];" ::"r"(dst),
                    "r"(lin_smem(ps + b0 * Cfg::PSTRIDE)),
                    "r"(static_cast<uint32_t>((b1 - b0) * Cfg::PSTRIDE * 4)), "r"(bar)
                    : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        bool ok = true;
        if (mine > 0) {
            if (tid == 0)
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(recv),
                             "r"(static_cast<uint32_t>(splits * mine * Cfg::PSTRIDE * 4))
                             : "memory");
            ok = lin_wait(recv, 0);
        }
        src = ok ? rb : nullptr;
    } else {
        asm volatile("barrier.cluster.wait;" ::: "memory");
        __syncthreads();
    }

    // 16-byte stores of 8 outputs per thread and item, the residual added on the way; the
    // 8 chunks of a row sit in 8 neighbouring lanes, which sum the row's squares
    const int slot = splits > 1 ? rbr * Cfg::PSTRIDE : 0;  // floats between receive slots
    const int items = ((mine * 8 + kLinThreads - 1) / kLinThreads) * kLinThreads;
    for (int q = tid; q < items; q += kLinThreads) {
        const int m = m0 + (q >> 3), c = q & 7;
        const int col = n0 + c * 8;
        const bool live = src != nullptr && (q >> 3) < mine && col < a.N;
        float sq = 0.f;
        if (live) {
            // every split's partial loaded together, then summed in split order
            const float* base = src + (splits > 1 ? (m - m0) : m) * Cfg::PSTRIDE + c * 8;
            float4 pg[kLinMaxSplits][2], pu[kLinMaxSplits][2];
#pragma unroll
            for (int r = 0; r < kLinMaxSplits; ++r) {
                if (r < splits) {
                    const float4* pr = reinterpret_cast<const float4*>(base + r * slot);
                    pg[r][0] = pr[0];
                    pg[r][1] = pr[1];
                    if (NW == 2) {
                        pu[r][0] = pr[kLinCols / 4];
                        pu[r][1] = pr[kLinCols / 4 + 1];
                    }
                }
            }
            float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            float u[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < kLinMaxSplits; ++r) {
                if (r < splits) {
                    g[0] += pg[r][0].x; g[1] += pg[r][0].y; g[2] += pg[r][0].z; g[3] += pg[r][0].w;
                    g[4] += pg[r][1].x; g[5] += pg[r][1].y; g[6] += pg[r][1].z; g[7] += pg[r][1].w;
                    if (NW == 2) {
                        u[0] += pu[r][0].x; u[1] += pu[r][0].y; u[2] += pu[r][0].z; u[3] += pu[r][0].w;
                        u[4] += pu[r][1].x; u[5] += pu[r][1].y; u[6] += pu[r][1].z; u[7] += pu[r][1].w;
                    }
                }
            }
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float gh = __half2float(__float2half_rn(g[e]));
                if (NW == 1) {
                    y[e] = gh;
                } else {
                    const float uh = __half2float(__float2half_rn(u[e]));
                    y[e] = (gh / (1.0f + expf(-gh))) * uh;
                }
            }
            if (a.resid) {
                float r[8];
                Chunk<__half>::unpack(
                    q == tid ? resid0
                             : *reinterpret_cast<const uint4*>(a.resid + static_cast<int64_t>(m) * a.ldr + col),
                    r);
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(y[e], r[e]);
            }
            uint4 o;
            __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                oh[e] = __floats2half2_rn(y[2 * e], y[2 * e + 1]);
                const float2 f = __half22float2(oh[e]);
                sq = fmaf(f.x, f.x, sq);
                sq = fmaf(f.y, f.y, sq);
            }
            *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(m) * a.ldo + col) = o;
        }
        if (a.stats_out) {  // one partial per 16 columns: chunks 2j and 2j+1 of the row
            sq += __shfl_xor_sync(0xffffffffu, sq, 1);
            if (src != nullptr && (c & 1) == 0 && (q >> 3) < mine && col < a.N)
                a.stats_out[(tile * (kLinCols / kStatCols) + (c >> 1)) * kLinRows + m] = sq;
        }
    }
    if (splits > 1 && tid < splits)  // the pushed rows have left this CTA's shared memory
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

struct LinearPlan {
    int tiles, splits, kchunk;
};
// Dynamic shared memory of a launch: the ring, and with a split K the receive buffer of
// the rows a CTA finishes (every split's partial band).
template <int NW>
size_t linear_smem_bytes(int splits, int rows) {
    const int rbr = (rows + splits - 1) / splits;
    return LinCfg<NW>::OFF_RB +
           (splits > 1 ? static_cast<size_t>(splits) * rbr * LinCfg<NW>::PSTRIDE * 4 : 0);
}

// K splits so that the grid fills the SMs once (three CTAs an SM, less an eighth for the
// packing of clusters), in chunks of whole 64-deep tiles, at most one cluster (8) per
// column tile, and never more CTAs than one wave holds at the largest batch (64 rows: the
// receive buffer, and so the CTAs an SM holds, depends on the rows; B200 has 228 KB of
// shared memory an SM, 1 KB of it reserved per CTA).  The plan depends on the shape only,
// so a row's result is the same in every batch.
template <int NW>
LinearPlan plan_linear(int64_t k, int64_t n) {
    constexpr int64_t kSmemPerSm = 233472, kSmemReserved = 1024;
    LinearPlan p{};
    p.tiles = static_cast<int>((n + kLinCols - 1) / kLinCols);
    const int64_t sms = device_sm_count();
    const int64_t target = sms * 3 * 7 / 8;
    int64_t sp = target / p.tiles;
    const int64_t kt = (k + kLinK - 1) / kLinK;
    if (sp > kt) sp = kt;
    if (sp > kLinMaxSplits) sp = kLinMaxSplits;
    if (sp < 1) sp = 1;
    for (;; --sp) {
        int64_t chunk = (k + sp - 1) / sp;
        chunk = ((chunk + kLinK - 1) / kLinK) * kLinK;
        p.kchunk = static_cast<int>(chunk);
        p.splits = static_cast<int>((k + chunk - 1) / chunk);
        const int64_t per_sm =
            kSmemPerSm / (static_cast<int64_t>(linear_smem_bytes<NW>(p.splits, kLinRows)) +
                          kSmemReserved);
        if (sp == 1 || static_cast<int64_t>(p.tiles) * p.splits <= sms * per_sm) break;
    }
    return p;
}

template <int NW>
int launch_linear(const LinearArgs& a, const LinearPlan& p, bool overlap, cudaStream_t s) {
    // the shared-memory opt-in once per device (bit d of the mask)
    static std::atomic<uint64_t> opted{0};
    int dev = 0;
    TMLLM_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (!bit || !(opted.load(std::memory_order_relaxed) & bit)) {
        TMLLM_CUDA_TRY(cudaFuncSetAttribute(linear_kernel<NW>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(LinCfg<NW>::SMEM_MAX)));
        opted.fetch_or(bit, std::memory_order_relaxed);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(p.tiles), static_cast<unsigned>(p.splits));
    cfg.blockDim = dim3(kLinThreads);
    cfg.dynamicSmemBytes = linear_smem_bytes<NW>(p.splits, a.M);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(p.splits);
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 2 : 1;
    TMLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, linear_kernel<NW>, a));
    return TMLLM_OK;
}

// ---- Vocabulary head of a decode step: final RMSNorm, x · W_head, greedy argmax ----------
// The last three stages of the reference's cached forward (transformer/cache.rs:72-77: the
// final RmsNorm, the lm_head Linear; then greedy_from_slice, generation/sampler.rs:79-88) as
// one kernel.  The head weight is the largest tensor a decode step reads (K x vocab halves,
// 57-94 MB for the BASELINE models) and every other operand is tiny, so the kernel is a
// weight stream.  Column tiles of 4 x WN columns (64 with up to 32 rows, 128 above) are dealt
// to persistent CTAs in equal numbers (the grid is the tile count over the tiles a CTA must
// take, so no CTA runs a lone extra round at a fraction of the bandwidth).  Each CTA moves
// its tiles through a ring of 16 KB stages (128 or 64 weight rows) that runs ahead across
// tile boundaries, as deep as shared memory allows (two CTAs an SM with 4-12 stages each
// where the rows leave room, else one with 3-12): a producer warp fills a stage with one or
// two TMA tensor loads (64-column boxes in the 128-byte swizzle, so the eight rows of an
// ldmatrix.trans tile fall into different banks; boxes reaching past K or N are zero-filled
// by the copy engine) completing on the stage's full barrier, as soon as the four MMA warps
// have released the slot on its empty barrier.  The rows (<= 64) sit in shared memory for
// the whole
// kernel, RMS-normalised in place once (the arithmetic of add_rmsnorm_warp_kernel, so the
// normed rows equal tmllm_add_rmsnorm's bit for bit).  Warp w multiplies the rows by columns
// [w*WN, (w+1)*WN) of a tile on the warp-level tensor cores (mma.sync m16n8k16, F16 in, F32
// accumulate), one 16-row tile of rows per m-tile.  The epilogue stores the F16 logits and
// keeps, per row, the best (value, index) key of the stored values (argmax_key: finite
// values under total order, the last maximum wins); each CTA folds its keys into a per-row
// 64-bit maximum in the caller's workspace, and the CTA that takes the last ticket turns
// those maxima into token ids (-1 for a row without a finite logit) and resets the
// workspace to zero for the next call.  Stage waits are bounded (TMLLM_TIMEOUT in the
// status word tmllm_linear_status reads).
constexpr int kHeadConsumers = 4;                     // MMA warps
constexpr int kHeadThreads = 32 * (kHeadConsumers + 1);  // + one TMA producer warp
constexpr int kHeadMaxRows = 64;
constexpr int kHeadMinStages = 3, kHeadMaxStages = 12;
constexpr int kHeadOffBest = 0;                                    // [4 warps][64] keys
constexpr int kHeadOffBar = kHeadOffBest + 4 * kHeadMaxRows * 8;   // full and empty barriers
constexpr int kHeadOffFlag = kHeadOffBar + 2 * kHeadMaxStages * 8;  // last-CTA / abort flags
constexpr int kHeadOffX = kHeadOffFlag + 64;                       // the rows, then the ring
constexpr int kHeadStage = 16384;                                  // bytes of one stage
constexpr int kHeadSmemMax = 227 * 1024;
constexpr int kHeadSmemPair = 113 * 1024;  // two CTAs an SM

struct HeadArgs {
    const __half* x;
    const __half* norm_w;  // null: the rows are used as they are
    const __half* resid;   // null: no residual add before the norm
    const __half* w;
    __half* logits;
    int32_t* ids;                // null: no argmax
    unsigned long long* best;    // [64] per-row keys (zero between calls)
    unsigned int* ticket;        // CTAs finished (zero between calls)
    int64_t ldx, ldr, ldw, ldo;
    int M, K, N, stages;
    float eps;
};

// columns a warp owns: 16 with up to two 16-row tiles of rows, else 32 (more products per
// weight fragment, fewer reloads of the row fragments)
__host__ __device__ constexpr int head_wn(int mt) { return mt <= 2 ? 16 : 32; }
// weight rows of one stage (16 KB of weight: one or two 128-byte-wide panels)
__host__ __device__ constexpr int head_krows(int mt) { return kHeadStage / (8 * head_wn(mt)); }
// bytes of one staged input row: K rounded up to a whole stage, plus 16 so that the eight
// rows of an ldmatrix tile fall into different banks
__host__ __device__ inline int head_xstride(int mt, int K) {
    const int kr = head_krows(mt);
    return ((K + kr - 1) / kr) * kr * 2 + 16;
}
// the rows, the norm weight (K rounded up to a stage), then the ring on a 1024-byte
// boundary (the swizzle pattern's period): up to 1008 bytes of padding
size_t head_smem_bytes(int M, int K, int stages) {
    const int mt = (M + 15) / 16;
    const int kr = head_krows(mt);
    return static_cast<size_t>(kHeadOffX) + static_cast<size_t>(mt) * 16 * head_xstride(mt, K) +
           static_cast<size_t>((K + kr - 1) / kr) * kr * 2 + 1024 +
           static_cast<size_t>(stages) * kHeadStage;
}
// ring depth: as deep as fits with two CTAs an SM (each in half of the shared memory) when
// that leaves at least four stages, else with one CTA an SM (measured: two CTAs with a few
// stages each stream the weight faster than one CTA with twice the stages in flight);
// 0 when not even the shallowest ring fits
int head_stages(int M, int K) {
    for (int per_sm : {2, 1}) {
        const size_t budget = per_sm == 2 ? kHeadSmemPair : kHeadSmemMax;
        int st = kHeadMaxStages;
        while (st >= kHeadMinStages && head_smem_bytes(M, K, st) > budget) --st;
        if (st >= (per_sm == 2 ? 4 : kHeadMinStages)) return st;
    }
    return 0;
}

template <int MT>
__global__ void __launch_bounds__(kHeadThreads)
    head_kernel(const __grid_constant__ CUtensorMap wmap, const HeadArgs a) {
    constexpr int WN = head_wn(MT), TC = 4 * WN;  // columns a warp / a tile owns
    constexpr int KR = head_krows(MT);            // weight rows per stage
    constexpr int PANEL = KR * 128;               // bytes of one 64-column panel of a stage
    constexpr int NB = WN / 16;                   // ldmatrix.x4.trans per k16 step and warp
    constexpr int CT = kHeadConsumers * 32;       // threads of the consumer warps
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned long long* best_s = reinterpret_cast<unsigned long long*>(smem + kHeadOffBest);
    volatile int* flags_s = reinterpret_cast<volatile int*>(smem + kHeadOffFlag);  // last, abort
    unsigned char* xs = smem + kHeadOffX;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.K, M = a.M, N = a.N, S = a.stages;
    const int ks = (K + KR - 1) / KR;  // ring stages per tile
    const int kp = ks * KR;
    const int xstride = head_xstride(MT, K);
    unsigned char* nws = xs + MT * 16 * xstride;  // [kp] norm weight
    const uint32_t ring_u = (lin_smem(nws + kp * 2) + 1023u) & ~1023u;
    const uint32_t full0 = lin_smem(smem + kHeadOffBar);  // [S] stage landed (TMA bytes)
    const uint32_t empty0 = full0 + 8 * kHeadMaxStages;   // [S] stage read by every consumer
    const int ntiles = (N + TC - 1) / TC;
    const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    const int nmine = cta < ntiles ? (ntiles - 1 - cta) / G + 1 : 0;
    const int total = nmine * ks;  // ring stages of this CTA
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * i), "r"(1)
                         : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty0 + 8 * i),
                         "r"(kHeadConsumers)
                         : "memory");
        }
        flags_s[0] = 0;
        flags_s[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    launch_dependents();

    if (warp == kHeadConsumers) {
        // ===== producer (one lane): stage q = weight rows [kk*KR, +KR) of tile q / ks, one
        // 64-column box per panel (the bytes of every box count, zero-filled ones included),
        // into slot q % S once the consumers have released that slot's previous stage.  The
        // weight is constant, so none of this waits for the kernel ahead.
        if (lane == 0) {
            int q = 0;
            for (; q < total; ++q) {
                const int kk = q % ks, slot = q % S;
                if (q >= S && !lin_wait(empty0 + 8 * slot, static_cast<uint32_t>(((q / S) - 1) & 1))) {
                    flags_s[1] = 1;
                    break;
                }
                if (flags_s[1]) break;
                const int n0 = (cta + (q / ks) * G) * TC;
                const uint32_t bar = full0 + 8 * slot;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                             "r"(static_cast<uint32_t>(kHeadStage))
                             : "memory");
#pragma unroll
                for (int p = 0; p < TC / 64; ++p)
                    tma_load_2d(ring_u + slot * kHeadStage + p * PANEL, &wmap, n0 + 64 * p,
                                kk * KR, bar);
            }
            // on an abort, wait (bounded) for the stages in flight, so no copy lands after
            // the CTA has exited
            for (int r = q - S; r < q; ++r)
                if (r >= 0) lin_wait(full0 + 8 * (r % S), static_cast<uint32_t>((r / S) & 1));
        }
    } else {
        // ===== consumers (warps 0-3)
        if (a.norm_w)  // constant: staged before the dependency wait
            for (int c = tid; c < kp / 8; c += CT)
                cp_async16(nws + c * 16, c * 8 < K ? a.norm_w + c * 8 : a.norm_w, c * 8 < K ? 16 : 0);
        cp_async_commit();
        grid_dependency_wait();  // the rows are current from here on
        // the rows, zero-filled to whole 16-row tiles and whole stages
        const int cpx = kp / 8;  // 16-byte chunks per staged row
        for (int i = tid; i < MT * 16 * cpx; i += CT) {
            const int m = i / cpx, c = i - m * cpx;
            const bool ok = m < M && c * 8 < K;
            cp_async16(xs + m * xstride + c * 16,
                       ok ? a.x + static_cast<int64_t>(m) * a.ldx + c * 8 : a.x, ok ? 16 : 0);
        }
        cp_async_commit();
        cp_async_wait<0>();
        asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
        if (a.norm_w || a.resid) {
            // row m on warp m % 4, as add_rmsnorm_warp_kernel does one row: the residual
            // added with the sum rounded to F16 (kernels/vector_add.metal), lane sums chunks
            // lane, lane + 32, ... in order, then the shuffle tree; the row is rewritten as
            // half(x * inv * w).  A warp's rows advance together, chunk by chunk, so their
            // loads and sums overlap.
            constexpr int RPW = MT * 16 / kHeadConsumers;  // rows per warp at most
            const int nr = (M - warp + kHeadConsumers - 1) / kHeadConsumers;  // this warp's
            float ss[RPW];
#pragma unroll
            for (int j = 0; j < RPW; ++j) ss[j] = 0.f;
            for (int c = lane; c < K / 8; c += 32) {
                uint4 rv[RPW];
                if (a.resid) {
#pragma unroll
                    for (int j = 0; j < RPW; ++j)
                        if (j < nr)
                            rv[j] = __ldg(reinterpret_cast<const uint4*>(
                                              a.resid + static_cast<int64_t>(warp + kHeadConsumers * j) * a.ldr) +
                                          c);
                }
#pragma unroll
                for (int j = 0; j < RPW; ++j) {
                    if (j >= nr) break;
                    unsigned char* row = xs + (warp + kHeadConsumers * j) * xstride;
                    float f[8];
                    Chunk<__half>::unpack(*reinterpret_cast<const uint4*>(row + c * 16), f);
                    if (a.resid) {
                        float r8[8];
                        Chunk<__half>::unpack(rv[j], r8);
                        uint4 sv;
                        __half2* sh = reinterpret_cast<__half2*>(&sv);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = round_store<__half>(__fadd_rn(f[e], r8[e]));
#pragma unroll
                        for (int e = 0; e < 4; ++e) sh[e] = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
                        *reinterpret_cast<uint4*>(row + c * 16) = sv;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) ss[j] = fmaf(f[e], f[e], ss[j]);
                }
            }
            if (a.norm_w) {
                float inv[RPW];
#pragma unroll
                for (int j = 0; j < RPW; ++j)
                    inv[j] = j < nr ? rsqrtf(warp_sum(ss[j]) / static_cast<float>(K) + a.eps) : 0.f;
                for (int c = lane; c < K / 8; c += 32) {
                    float w8[8];
                    Chunk<__half>::unpack(*reinterpret_cast<const uint4*>(nws + c * 16), w8);
#pragma unroll
                    for (int j = 0; j < RPW; ++j) {
                        if (j >= nr) break;
                        unsigned char* row = xs + (warp + kHeadConsumers * j) * xstride;
                        float f[8];
                        Chunk<__half>::unpack(*reinterpret_cast<const uint4*>(row + c * 16), f);
                        uint4 y;
                        __half2* yh = reinterpret_cast<__half2*>(&y);
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            yh[e] = __floats2half2_rn(f[2 * e] * inv[j] * w8[2 * e],
                                                      f[2 * e + 1] * inv[j] * w8[2 * e + 1]);
                        *reinterpret_cast<uint4*>(row + c * 16) = y;
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
        }

        const int g = lane >> 2, t = lane & 3;
        float acc[MT][2 * NB][4];
        unsigned long long bk[MT][2];  // best key of rows g and g + 8 of each m-tile
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) bk[mt][0] = bk[mt][1] = 0ull;
        const uint32_t xs_u = lin_smem(xs);
        // ldmatrix addresses of this lane: A (rows) matrix lane/8 = (row half, k half);
        // B (weight, transposed) matrix lane/8 = (k half, column half): column chunk
        // bch + 2p of a stage lives in panel chunk/8 at chunk (chunk % 8) ^ (row % 8)
        const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
        const int bch = warp * (WN / 8) + (lane >> 4);
        for (int q = 0; q < total; ++q) {
            const int kk = q % ks, slot = q % S;
            const bool ok = lin_wait(full0 + 8 * slot, static_cast<uint32_t>((q / S) & 1));
            // one decision for the whole warp (the MMAs below are warp-collective): give up
            // when any lane's wait expired or another warp has given up
            if (!__all_sync(0xffffffffu, ok) || __any_sync(0xffffffffu, flags_s[1] != 0)) {
                flags_s[1] = 1;
                break;
            }
            if (kk == 0) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 2 * NB; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
            }
            const uint32_t st = ring_u + slot * kHeadStage;
            const int nk = (min(KR, K - kk * KR) + 15) / 16;  // k16 steps holding rows < K
#pragma unroll 4
            for (int s16 = 0; s16 < nk; ++s16) {
                uint32_t af[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    ldsm_x4(xs_u + (mt * 16 + arow) * xstride + (kk * KR + s16 * 16 + acol) * 2,
                            af[mt][0], af[mt][1], af[mt][2], af[mt][3]);
                const int r = s16 * 16 + arow;
#pragma unroll
                for (int p = 0; p < NB; ++p) {
                    const int ch = bch + 2 * p;
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(st + (ch >> 3) * PANEL + r * 128 + (((ch & 7) ^ (r & 7)) << 4), b0,
                              b1, b2, b3);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        mma16816(acc[mt][2 * p], af[mt][0], af[mt][1], af[mt][2], af[mt][3], b0, b1);
                        mma16816(acc[mt][2 * p + 1], af[mt][0], af[mt][1], af[mt][2], af[mt][3], b2,
                                 b3);
                    }
                }
            }
            // this warp is done with the slot (its shared-memory reads are complete once
            // the fragments are in registers)
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty0 + 8 * slot)
                             : "memory");
            if (kk == ks - 1) {
                // the tile is complete: F16 logits out, the best key of the stored values kept
                const int n0 = (cta + (q / ks) * G) * TC + warp * WN;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int m = mt * 16 + g + 8 * hh;
#pragma unroll
                        for (int nt = 0; nt < 2 * NB; ++nt) {
                            const int col = n0 + nt * 8 + 2 * t;
                            const __half2 hv =
                                __floats2half2_rn(acc[mt][nt][2 * hh], acc[mt][nt][2 * hh + 1]);
                            if (m < M && col < N) {
                                *reinterpret_cast<__half2*>(a.logits + static_cast<int64_t>(m) * a.ldo +
                                                            col) = hv;
                                const float2 f = __half22float2(hv);
                                const unsigned long long k0 = argmax_key(f.x, col);
                                const unsigned long long k1 = argmax_key(f.y, col + 1);
                                const unsigned long long kb = k1 > k0 ? k1 : k0;
                                bk[mt][hh] = kb > bk[mt][hh] ? kb : bk[mt][hh];
                            }
                        }
                    }
            }
        }
        if (a.ids) {
            // per row: the four lanes of a row group, then the four warps, then every CTA
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    unsigned long long k = bk[mt][hh];
#pragma unroll
                    for (int o = 1; o <= 2; o <<= 1) {
                        const unsigned long long v = __shfl_xor_sync(0xffffffffu, k, o);
                        k = v > k ? v : k;
                    }
                    if (t == 0) best_s[warp * kHeadMaxRows + mt * 16 + g + 8 * hh] = k;
                }
        }
    }
    if (!a.ids) return;
    __syncthreads();
    if (tid < M) {
        unsigned long long k = best_s[tid];
#pragma unroll
        for (int w = 1; w < kHeadConsumers; ++w) {
            const unsigned long long v = best_s[w * kHeadMaxRows + tid];
            k = v > k ? v : k;
        }
        if (k) atomicMax(a.best + tid, k);
    }
    // the ticket is taken with release and acquire semantics at device scope: the barrier
    // orders this CTA's maxima before thread 0's release, and the last CTA's acquire before
    // its reads of every CTA's maxima.  A CTA that gave up on a wait (recorded in the
    // status word) still takes its ticket, so later calls start from a zeroed workspace.
    __syncthreads();
    if (tid == 0) {
        unsigned int t;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(a.ticket)
                     : "memory");
        flags_s[0] = t == gridDim.x - 1;
    }
    __syncthreads();
    if (!flags_s[0]) return;
    if (tid < M) {  // every CTA's maxima are in: read and clear them
        const unsigned long long k = atomicExch(a.best + tid, 0ull);
        a.ids[tid] = k ? static_cast<int32_t>(k & 0xffffffffull) : -1;
    }
    if (tid == 0) atomicExch(a.ticket, 0u);
}

template <int MT>
int launch_head(const HeadArgs& a, bool overlap, cudaStream_t s) {
    const size_t smem = head_smem_bytes(a.M, a.K, a.stages);
    // the weight as K rows of N halves, boxes of 64 columns x one stage's rows; the map of
    // the last call is kept per thread (a decode loop calls with one head weight)
    struct MapKey {
        const void* w;
        int64_t n, k, ldw;
        int kr;
    };
    thread_local MapKey key{nullptr, 0, 0, 0, 0};
    thread_local CUtensorMap wmap;
    const MapKey want{a.w, a.N, a.K, a.ldw, head_krows(MT)};
    if (key.w != want.w || key.n != want.n || key.k != want.k || key.ldw != want.ldw ||
        key.kr != want.kr) {
        if (int st = make_map(&wmap, a.w, a.N, a.K, a.ldw * 2, head_krows(MT))) return st;
        key = want;
    }
    static std::atomic<uint64_t> opted{0};
    int dev = 0;
    TMLLM_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (!bit || !(opted.load(std::memory_order_relaxed) & bit)) {
        TMLLM_CUDA_TRY(cudaFuncSetAttribute(head_kernel<MT>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kHeadSmemMax));
        opted.fetch_or(bit, std::memory_order_relaxed);
    }
    int per_sm = 0;
    TMLLM_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, head_kernel<MT>,
                                                                 kHeadThreads, smem));
    if (per_sm < 1) per_sm = 1;
    // equal shares: every CTA takes `rounds` tiles (the last few one fewer)
    const int64_t ntiles = (a.N + 4 * head_wn(MT) - 1) / (4 * head_wn(MT));
    const int64_t slots = static_cast<int64_t>(device_sm_count()) * per_sm;
    const int64_t rounds = (ntiles + slots - 1) / slots;
    const int64_t grid = (ntiles + rounds - 1) / rounds;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kHeadThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    TMLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, head_kernel<MT>, wmap, a));
    return TMLLM_OK;
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

int tmllm_linear_status(int32_t* status) {
    clear_error();
    if (!status) return fail(TMLLM_INVALID_ARGUMENT, "null status pointer");
    int v = 0, zero = 0;
    TMLLM_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_linear_status, sizeof(int)));
    TMLLM_CUDA_TRY(cudaMemcpyToSymbol(g_linear_status, &zero, sizeof(int)));
    *status = v;
    return TMLLM_OK;
}

size_t tmllm_linear_stats_bytes(int32_t n) {
    if (n <= 0) return 0;
    return static_cast<size_t>((n + kStatCols - 1) / kStatCols) * kLinRows * sizeof(float);
}

int tmllm_linear(const void* x, int64_t ldx, const void* norm_weight, const float* stats_in,
                 float eps, const void* w, int64_t ldw, void* out, int64_t ldo,
                 const void* residual, int64_t ldr, float* stats_out, int32_t rows, int32_t k,
                 int32_t n, int32_t swiglu, uint32_t flags, tmllm_stream stream) {
    clear_error();
    if (rows <= 0 || k <= 0 || n <= 0)
        return fail(TMLLM_INVALID_SHAPE, "linear dimensions must be positive");
    if (rows > kLinRows)
        return fail(TMLLM_INVALID_SHAPE, "tmllm_linear takes at most %d rows, got %d", kLinRows,
                    rows);
    if (swiglu != 0 && swiglu != 1) return fail(TMLLM_INVALID_ARGUMENT, "swiglu must be 0 or 1");
    if (flags & ~static_cast<uint32_t>(TMLLM_LINEAR_OVERLAP))
        return fail(TMLLM_INVALID_ARGUMENT, "unknown linear flags 0x%x", flags);
    if (swiglu && residual)
        return fail(TMLLM_INVALID_ARGUMENT, "a residual add and SwiGLU cannot be combined");
    if (stats_in && !norm_weight)
        return fail(TMLLM_INVALID_ARGUMENT, "row statistics are an input of the RMSNorm only");
    if (!x || !w || !out) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    if (k % 8 || n % 8)
        return fail(TMLLM_INVALID_SHAPE, "linear K and N must be multiples of 8 (got %d, %d)", k, n);
    const int64_t wcols = static_cast<int64_t>(n) * (swiglu ? 2 : 1);
    if (ldx < k || ldw < wcols || ldo < n || (residual && ldr < n))
        return fail(TMLLM_INVALID_SHAPE, "row strides must cover a row");
    if (!aligned16(x) || !aligned16(w) || !aligned16(out) || (residual && !aligned16(residual)) ||
        (norm_weight && !aligned16(norm_weight)) || ldx % 8 || ldw % 8 || ldo % 8 ||
        (residual && ldr % 8))
        return fail(TMLLM_INVALID_ARGUMENT,
                    "x, w, out, the residual and the norm weight need 16-byte aligned rows");
    if ((stats_in && !aligned16(stats_in)) || (stats_out && !aligned16(stats_out)))
        return fail(TMLLM_INVALID_ARGUMENT, "row statistics need 16-byte aligned buffers");
    if (norm_weight && (!std::isfinite(eps) || eps <= 0.0f))
        return fail(TMLLM_INVALID_SHAPE, "RMSNorm epsilon must be positive, got %g",
                    static_cast<double>(eps));
    LinearArgs a{};
    a.x = static_cast<const __half*>(x);
    a.norm_w = static_cast<const __half*>(norm_weight);
    a.stats_in = stats_in;
    a.w = static_cast<const __half*>(w);
    a.out = static_cast<__half*>(out);
    a.resid = static_cast<const __half*>(residual);
    a.stats_out = stats_out;
    a.ldx = ldx;
    a.ldw = ldw;
    a.ldo = ldo;
    a.ldr = ldr;
    a.M = rows;
    a.K = k;
    a.N = n;
    a.eps = eps;
    auto s = reinterpret_cast<cudaStream_t>(stream);
    const bool overlap = (flags & TMLLM_LINEAR_OVERLAP) != 0;
    int rc;
    {
        const LinearPlan p = swiglu ? plan_linear<2>(k, n) : plan_linear<1>(k, n);
        a.kchunk = p.kchunk;
        rc = swiglu ? launch_linear<2>(a, p, overlap, s) : launch_linear<1>(a, p, overlap, s);
    }
    if (rc != TMLLM_OK) return rc;
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
    const size_t row_bytes = vocab * (dtype == TMLLM_F16 ? 2 : 4);
    const bool vec = aligned16(logits) && row_bytes % 16 == 0;  // every row 16-byte aligned
    if (dtype == TMLLM_F16)
        argmax_kernel<__half><<<static_cast<unsigned>(rows), 1024, 0, s>>>(
            static_cast<const __half*>(logits), ids, static_cast<int64_t>(vocab), vec);
    else
        argmax_kernel<float><<<static_cast<unsigned>(rows), 1024, 0, s>>>(
            static_cast<const float*>(logits), ids, static_cast<int64_t>(vocab), vec);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

size_t tmllm_lm_head_workspace_bytes(void) { return 1024; }

int tmllm_lm_head(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                  const void* norm_weight, float eps, const void* w, int64_t ldw, void* logits,
                  int64_t ld_logits, int32_t* ids, void* workspace, int32_t rows, int32_t k,
                  int32_t n, uint32_t flags, tmllm_stream stream) {
    clear_error();
    if (rows <= 0 || k <= 0 || n <= 0)
        return fail(TMLLM_INVALID_SHAPE, "lm_head dimensions must be positive");
    if (rows > kHeadMaxRows)
        return fail(TMLLM_INVALID_SHAPE, "tmllm_lm_head takes at most %d rows, got %d",
                    kHeadMaxRows, rows);
    if (flags & ~static_cast<uint32_t>(TMLLM_LINEAR_OVERLAP))
        return fail(TMLLM_INVALID_ARGUMENT, "unknown lm_head flags 0x%x", flags);
    if (!x || !w || !logits) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    if (ids && !workspace)
        return fail(TMLLM_INVALID_ARGUMENT, "the argmax needs the lm_head workspace");
    if (k % 8 || n % 8)
        return fail(TMLLM_INVALID_SHAPE, "lm_head K and N must be multiples of 8 (got %d, %d)",
                    k, n);
    if (ldx < k || ldw < n || ld_logits < n || (residual && ldr < k))
        return fail(TMLLM_INVALID_SHAPE, "row strides must cover a row");
    if (!aligned16(x) || !aligned16(w) || !aligned16(logits) ||
        (norm_weight && !aligned16(norm_weight)) || (residual && !aligned16(residual)) ||
        ldx % 8 || ldw % 8 || ld_logits % 8 || (residual && ldr % 8))
        return fail(TMLLM_INVALID_ARGUMENT,
                    "x, the residual, w, logits and the norm weight need 16-byte aligned rows");
    if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 7u))
        return fail(TMLLM_INVALID_ARGUMENT, "the lm_head workspace needs 8-byte alignment");
    if (norm_weight && (!std::isfinite(eps) || eps <= 0.0f))
        return fail(TMLLM_INVALID_SHAPE, "RMSNorm epsilon must be positive, got %g",
                    static_cast<double>(eps));
    const int stages = head_stages(rows, k);
    if (stages == 0)
        return fail(TMLLM_INVALID_SHAPE,
                    "lm_head rows x K too large for shared memory (%d x %d)", rows, k);
    HeadArgs a{};
    a.x = static_cast<const __half*>(x);
    a.norm_w = static_cast<const __half*>(norm_weight);
    a.resid = static_cast<const __half*>(residual);
    a.ldr = ldr;
    a.w = static_cast<const __half*>(w);
    a.logits = static_cast<__half*>(logits);
    a.ids = ids;
    a.best = static_cast<unsigned long long*>(workspace);
    a.ticket = workspace ? reinterpret_cast<unsigned int*>(static_cast<unsigned char*>(workspace) +
                                                           kHeadMaxRows * 8)
                         : nullptr;
    a.ldx = ldx;
    a.ldw = ldw;
    a.ldo = ld_logits;
    a.M = rows;
    a.K = k;
    a.N = n;
    a.stages = stages;
    a.eps = eps;
    auto s = reinterpret_cast<cudaStream_t>(stream);
    const bool overlap = (flags & TMLLM_LINEAR_OVERLAP) != 0;
    int rc;
    switch ((rows + 15) / 16) {
        case 1: rc = launch_head<1>(a, overlap, s); break;
        case 2: rc = launch_head<2>(a, overlap, s); break;
        case 3: rc = launch_head<3>(a, overlap, s); break;
        default: rc = launch_head<4>(a, overlap, s); break;
    }
    if (rc != TMLLM_OK) return rc;
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

}  // extern "C"
