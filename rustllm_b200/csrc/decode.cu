// Fused KV-append + GQA decode attention over a block-paged cache (sm_100a).
//
// One query token per sequence.  The reference runs this as six dispatches with the score
// tensor [Hq, L] travelling through memory four times and every KV head read once per
// query head (src/nn/attention.rs:216-247, kernels/gqa_matmul.metal, softmax.metal,
// attention_scale_mask.metal, kv_cache_write.metal).  Here it is one kernel:
//
//   grid (splits, kv_heads, seqs), 128 threads.  A CTA owns one KV head of one sequence
//   and a contiguous chunk of its positions, and serves all G = Hq/Hkv query heads of that
//   KV head, so every K/V byte is read from HBM exactly once.
//   K/V tiles of TT positions stream through a STAGES-deep cp.async ring in shared
//   memory (16-byte copies, rows XOR-swizzled so the per-token reads below hit 8 distinct
//   bank groups).  QK^T: one thread per (token, slice of D), q held in shared memory as
//   F32 [D][GP] and read by broadcast.  Online softmax in the log2 domain with
//   warp-shuffle max/sum.  PV: each warp owns TT/4 tokens, each lane D/32 dims, F32
//   accumulators in registers; all warps share the CTA's running max, so their partial
//   outputs simply add at the end.
//   The CTA whose chunk holds the new position rotates (optional RoPE) and writes k_new /
//   v_new into their paged slot and uses them from shared memory (no read-after-write
//   through memory).  With several splits, each CTA writes (O, m, l) partials and the
//   last CTA of a (seq, kv head) -- found with an atomic ticket -- merges them.
#include <atomic>
#include <cmath>

#include "common.cuh"

namespace tmllm {
namespace {

constexpr int kDecodeThreads = 128;
// Ring depth (16-position sub-tiles per warp) of the head_dim-64 tensor-core kernel and the
// CTAs per SM its shared memory and registers allow.
#ifndef TMLLM_D64_STAGES
#define TMLLM_D64_STAGES 3
#endif
constexpr int kD64Stages = TMLLM_D64_STAGES;
constexpr int kD64MinBlocks = kD64Stages <= 3 ? 4 : (kD64Stages == 4 ? 3 : 2);
// The positions-major kernel (head_dim 64, up to 8 query heads per KV head) consumes 32
// positions (two 16-position sub-tiles) per softmax update; its ring holds this many such
// items per warp.
#ifndef TMLLM_D64_PT_STAGES
#define TMLLM_D64_PT_STAGES 2
#endif
constexpr int kD64PtStages = TMLLM_D64_PT_STAGES;
constexpr int kD64PtMinBlocks = kD64PtStages <= 2 ? 3 : 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct DecodeArgs {
    const void* q;
    const void* k_new;
    const void* v_new;
    void* k_cache;
    void* v_cache;
    const int32_t* block_table;
    const int32_t* seq_lens;
    void* out;
    float* lse;
    int32_t* counters;  // [B * Hkv]
    float* part_ml;     // [B, Hkv, max_splits, G, 2]
    float* part_o;      // [B, Hkv, max_splits, G, D]
    const float* rope_cos;
    const float* rope_sin;
    int64_t num_blocks;
    int32_t q_heads, kv_heads, group, block_size, bs_shift, max_blocks, chunk;
    int32_t rope_len, rope_off, out_f32;
    float scale_log2;
    const ExchangeArgs* ex;  // cross-GPU split exchange, or null
    uint32_t epoch;          // exchange step number (1, 2, ...)
    int64_t q_stride;        // elements between sequences in q
    int64_t kv_stride;       // elements between sequences in k_new / v_new
    int32_t overlap;         // launched with programmatic stream serialisation
    int32_t clear_tickets;   // host side: zero the split tickets on the stream before launch
};

// Physical slot of 16-byte chunk `c` of tile row `r` (XOR swizzle inside groups of 8).
template <int C>
__device__ __forceinline__ int swz(int r, int c) {
    constexpr int M = (C >= 8 ? 8 : C) - 1;
    return c ^ (r & M);
}

// Arena block of position `pos` of sequence b, or -1 when the position is outside the
// table (negative, or past max_blocks entries) or its entry names no block.
__device__ __forceinline__ int64_t block_of(const DecodeArgs& a, int b, int64_t pos) {
    if (pos < 0) return -1;
    const int64_t idx = a.bs_shift >= 0 ? (pos >> a.bs_shift) : (pos / a.block_size);
    if (idx >= a.max_blocks) return -1;
    int64_t blk = __ldg(&a.block_table[static_cast<int64_t>(b) * a.max_blocks + idx]);
    return (blk >= 0 && blk < a.num_blocks) ? blk : -1;
}

__device__ __forceinline__ int offset_in_block(const DecodeArgs& a, int pos) {
    return a.bs_shift >= 0 ? (pos & (a.block_size - 1)) : (pos % a.block_size);
}

// Rotates the pair (x1, x2) = (x[i], x[i + D/2]) at `pos`; identity when no table is given
// or `pos` is outside it.  Same arithmetic as kernels/rope.metal:57-63 without contraction.
__device__ __forceinline__ void rope_pair(const DecodeArgs& a, int pos, int i, int half,
                                          float& x1, float& x2) {
    if (a.rope_cos == nullptr || pos < 0 || pos >= a.rope_len) return;
    float c = __ldg(&a.rope_cos[static_cast<int64_t>(pos) * half + i]);
    float s = __ldg(&a.rope_sin[static_cast<int64_t>(pos) * half + i]);
    float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    x1 = y1;
    x2 = y2;
}

template <typename T, int D, int GP, int TT, int STAGES>
struct DecodeCfg {
    static constexpr int EPC = 16 / sizeof(T);  // elements per 16-byte chunk
    static constexpr int C = D / EPC;           // chunks per row
    static constexpr int NH = kDecodeThreads / TT;  // D slices in QK
    static constexpr int CPT = C / NH;          // chunks per thread in QK
    static constexpr int DPL = D / 32;          // dims per lane in PV
    static constexpr int TPW = TT / 4;          // tokens per warp in PV
    static constexpr int ROW = D * static_cast<int>(sizeof(T));
    static constexpr int TILE = TT * ROW;
    static constexpr int LOADS = TT * C / kDecodeThreads;
    static constexpr int RSTEP = kDecodeThreads / C;  // rows between a thread's loads
    static_assert(C % NH == 0, "D slices must split the row into whole chunks");
    static_assert((TT * C) % kDecodeThreads == 0 && kDecodeThreads % C == 0, "load mapping");
    static_assert(D % 32 == 0 && TT % 32 == 0 && TT <= 128, "shape");
    static_assert((DPL * sizeof(T)) == 4 || (DPL * sizeof(T)) == 8 || (DPL * sizeof(T)) == 16,
                  "PV lane width");
    // shared-memory carve-up (bytes)
    static constexpr int OFF_Q = STAGES * 2 * TILE;
    static constexpr int OFF_SPART = OFF_Q + D * GP * 4;
    static constexpr int OFF_P = OFF_SPART + NH * TT * GP * 4;
    static constexpr int OFF_ST = OFF_P + TT * GP * 4;  // alpha, m, l [GP] each + flag
    static constexpr int OFF_NEW = OFF_ST + 4 * GP * 4 + 16;
    static constexpr int BYTES = OFF_NEW + 2 * ROW;
    static_assert(STAGES * 2 * TILE >= 4 * GP * D * 4, "reduction scratch fits in the ring");
};

template <int N> struct VecBytes;
template <> struct VecBytes<4> { using type = uint32_t; };
template <> struct VecBytes<8> { using type = uint2; };
template <> struct VecBytes<16> { using type = uint4; };

template <typename T, int N>
__device__ __forceinline__ void unpack_n(const void* p, float* f) {
    using V = typename VecBytes<N * sizeof(T)>::type;
    V raw = *reinterpret_cast<const V*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = to_f32<T>(e[i]);
}

template <typename T, int D, int GP, int TT, int STAGES>
__global__ void __launch_bounds__(kDecodeThreads, 2) decode_split_kernel(const DecodeArgs a) {
    using Cfg = DecodeCfg<T, D, GP, TT, STAGES>;
    constexpr int C = Cfg::C, EPC = Cfg::EPC, NH = Cfg::NH, CPT = Cfg::CPT, DPL = Cfg::DPL;
    constexpr int TPW = Cfg::TPW, ROW = Cfg::ROW, TILE = Cfg::TILE;
    extern __shared__ __align__(128) unsigned char smem[];
    float* q_s = reinterpret_cast<float*>(smem + Cfg::OFF_Q);        // [D][GP]
    float* s_part = reinterpret_cast<float*>(smem + Cfg::OFF_SPART);  // [NH][TT][GP]
    float* p_s = reinterpret_cast<float*>(smem + Cfg::OFF_P);         // [TT][GP]
    float* alpha_s = reinterpret_cast<float*>(smem + Cfg::OFF_ST);    // [GP]
    float* m_s = alpha_s + GP;
    float* l_s = m_s + GP;
    int* flag_s = reinterpret_cast<int*>(l_s + GP);
    T* knew_s = reinterpret_cast<T*>(smem + Cfg::OFF_NEW);            // [D]
    T* vnew_s = knew_s + D;                                           // [D]

    const int split = blockIdx.z, kvh = blockIdx.x, b = blockIdx.y;  // splits slowest
    const int nsplit = gridDim.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.group;
    const int cached = a.seq_lens[b] < 0 ? 0 : a.seq_lens[b];
    const bool has_new = a.k_new != nullptr;
    const int L = cached + (has_new ? 1 : 0);
    int splits_b = (L + a.chunk - 1) / a.chunk;
    if (splits_b < 1) splits_b = 1;
    if (splits_b > nsplit) splits_b = nsplit;
    if (split >= splits_b) return;
    const int t0 = split * a.chunk;
    const int t1 = (split == splits_b - 1) ? L : min(L, t0 + a.chunk);
    const int ntiles = t1 > t0 ? (t1 - t0 + TT - 1) / TT : 0;
    const bool owns_new = has_new && cached >= t0 && cached < t1;
    const int half = D / 2;
    const int qpos = cached + a.rope_off;

    // ---- q (rotated, storage-rounded) into q_s; padded heads are zero
    for (int idx = tid; idx < GP * half; idx += kDecodeThreads) {
        int g = idx / half, i = idx - g * half;
        float x1 = 0.f, x2 = 0.f;
        if (g < G) {
            const T* qr = static_cast<const T*>(a.q) + static_cast<int64_t>(b) * a.q_stride +
                          static_cast<int64_t>(kvh * G + g) * D;
            x1 = to_f32<T>(qr[i]);
            x2 = to_f32<T>(qr[i + half]);
            rope_pair(a, qpos, i, half, x1, x2);
            x1 = round_store<T>(x1);
            x2 = round_store<T>(x2);
        }
        q_s[i * GP + g] = x1;
        q_s[(i + half) * GP + g] = x2;
    }
    for (int idx = tid; idx < TT * GP; idx += kDecodeThreads) p_s[idx] = 0.f;
    if (tid < GP) {
        alpha_s[tid] = 1.f;
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    // ---- the new token: rotate k, keep both rows in shared memory, write them to the cache
    if (owns_new) {
        const int64_t nrow = static_cast<int64_t>(b) * a.kv_stride + static_cast<int64_t>(kvh) * D;
        const T* kn = static_cast<const T*>(a.k_new) + nrow;
        const T* vn = static_cast<const T*>(a.v_new) + nrow;
        for (int i = tid; i < half; i += kDecodeThreads) {
            float x1 = to_f32<T>(kn[i]), x2 = to_f32<T>(kn[i + half]);
            rope_pair(a, qpos, i, half, x1, x2);
            knew_s[i] = from_f32<T>(x1);
            knew_s[i + half] = from_f32<T>(x2);
            vnew_s[i] = vn[i];
            vnew_s[i + half] = vn[i + half];
        }
    }
    __syncthreads();
    if (owns_new) {
        const int64_t blk = block_of(a, b, cached);
        if (blk >= 0) {
            const int64_t off =
                ((blk * a.kv_heads + kvh) * a.block_size + offset_in_block(a, cached)) * D;
            T* kd = static_cast<T*>(a.k_cache) + off;
            T* vd = static_cast<T*>(a.v_cache) + off;
            for (int i = tid; i < D; i += kDecodeThreads) {
                kd[i] = knew_s[i];
                vd[i] = vnew_s[i];
            }
        }
    }

    // ---- cp.async producer: thread `tid` copies chunk (tid % C) of rows tid/C + k*RSTEP
    const int lc = tid % C;
    const int lr0 = tid / C;
    const unsigned char* kbase = static_cast<const unsigned char*>(a.k_cache);
    const unsigned char* vbase = static_cast<const unsigned char*>(a.v_cache);
    auto load_tile = [&](int tile, int stage) {
        unsigned char* ks = smem + stage * 2 * TILE;
        unsigned char* vs = ks + TILE;
        const int base = t0 + tile * TT;
#pragma unroll
        for (int k = 0; k < Cfg::LOADS; ++k) {
            const int r = lr0 + k * Cfg::RSTEP;
            const int pos = base + r;
            const unsigned char* ksrc = kbase;
            const unsigned char* vsrc = vbase;
            int bytes = 0;
            if (pos < cached && pos < t1) {
                const int64_t blk = block_of(a, b, pos);
                if (blk >= 0) {
                    const int64_t off =
                        ((blk * a.kv_heads + kvh) * a.block_size + offset_in_block(a, pos)) *
                            ROW +
                        lc * 16;
                    ksrc += off;
                    vsrc += off;
                    bytes = 16;
                }
            }
            const int dst = r * ROW + swz<C>(r, lc) * 16;
            cp_async16(ks + dst, ksrc, bytes);
            cp_async16(vs + dst, vsrc, bytes);
        }
    };

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < ntiles) load_tile(s, s);
        cp_async_commit();
    }

    // consumer roles
    const int tq = (warp % (TT / 32)) * 32 + lane;  // QK: token of this thread
    const int hq = warp / (TT / 32);                 // QK: D slice of this thread
    float acc_o[GP][DPL];
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc_o[g][e] = 0.f;

    for (int it = 0; it < ntiles; ++it) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            const int nt = it + STAGES - 1;
            if (nt < ntiles) load_tile(nt, nt % STAGES);
            cp_async_commit();
        }
        unsigned char* ks = smem + (it % STAGES) * 2 * TILE;
        unsigned char* vs = ks + TILE;
        const int base = t0 + it * TT;
        if (owns_new && cached >= base && cached < base + TT) {
            const int r = cached - base;
            if (tid < C) {
                *reinterpret_cast<uint4*>(ks + r * ROW + swz<C>(r, tid) * 16) =
                    *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(knew_s) + tid * 16);
            } else if (tid < 2 * C) {
                const int c = tid - C;
                *reinterpret_cast<uint4*>(vs + r * ROW + swz<C>(r, c) * 16) =
                    *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(vnew_s) + c * 16);
            }
            __syncthreads();
        }

        // ---- QK^T partial over this thread's D slice
        {
            float acc[GP];
#pragma unroll
            for (int g = 0; g < GP; ++g) acc[g] = 0.f;
            const unsigned char* krow = ks + tq * ROW;
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int c = hq * CPT + j;
                uint4 raw = *reinterpret_cast<const uint4*>(krow + swz<C>(tq, c) * 16);
                float kf[EPC];
                Chunk<T>::unpack(raw, kf);
#pragma unroll
                for (int e = 0; e < EPC; ++e) {
                    const float* qd = q_s + (c * EPC + e) * GP;
#pragma unroll
                    for (int g4 = 0; g4 < GP; g4 += 4) {
                        float4 qv = *reinterpret_cast<const float4*>(qd + g4);
                        acc[g4 + 0] = fmaf(qv.x, kf[e], acc[g4 + 0]);
                        acc[g4 + 1] = fmaf(qv.y, kf[e], acc[g4 + 1]);
                        acc[g4 + 2] = fmaf(qv.z, kf[e], acc[g4 + 2]);
                        acc[g4 + 3] = fmaf(qv.w, kf[e], acc[g4 + 3]);
                    }
                }
            }
            float* sp = s_part + (hq * TT + tq) * GP;
#pragma unroll
            for (int g4 = 0; g4 < GP; g4 += 4)
                *reinterpret_cast<float4*>(sp + g4) =
                    make_float4(acc[g4], acc[g4 + 1], acc[g4 + 2], acc[g4 + 3]);
        }
        __syncthreads();

        // ---- online softmax, one warp per query head
        for (int g = warp; g < G; g += 4) {
            float sv[TT / 32];
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < TT / 32; ++k) {
                const int t = lane + 32 * k;
                float v = 0.f;
#pragma unroll
                for (int h = 0; h < NH; ++h) v += s_part[(h * TT + t) * GP + g];
                v = (base + t < t1) ? v * a.scale_log2 : -INFINITY;
                sv[k] = v;
                mx = fmaxf(mx, v);
            }
            mx = warp_max(mx);
            const float m_old = m_s[g];
            const float m_new = fmaxf(m_old, mx);
            float alpha, sum = 0.f;
            if (m_new == -INFINITY) {
                alpha = 1.f;
#pragma unroll
                for (int k = 0; k < TT / 32; ++k) p_s[(lane + 32 * k) * GP + g] = 0.f;
            } else {
                alpha = exp2f(m_old - m_new);
#pragma unroll
                for (int k = 0; k < TT / 32; ++k) {
                    float p = exp2f(sv[k] - m_new);
                    p_s[(lane + 32 * k) * GP + g] = p;
                    sum += p;
                }
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                alpha_s[g] = alpha;
                m_s[g] = m_new;
                l_s[g] = l_s[g] * alpha + sum;
            }
        }
        __syncthreads();

        // ---- PV: warp owns tokens [warp*TPW, +TPW), lane owns dims [lane*DPL, +DPL)
        {
#pragma unroll
            for (int g = 0; g < GP; ++g) {
                const float al = alpha_s[g];
#pragma unroll
                for (int e = 0; e < DPL; ++e) acc_o[g][e] *= al;
            }
            constexpr int LB = DPL * static_cast<int>(sizeof(T));  // bytes per lane
            const int lbyte = lane * LB;
            const int lch = lbyte / 16, lin = lbyte % 16;
#pragma unroll 4
            for (int i = 0; i < TPW; ++i) {
                const int t = warp * TPW + i;
                float vf[DPL];
                unpack_n<T, DPL>(vs + t * ROW + swz<C>(t, lch) * 16 + lin, vf);
                const float* pr = p_s + t * GP;
#pragma unroll
                for (int g4 = 0; g4 < GP; g4 += 4) {
                    float4 pv = *reinterpret_cast<const float4*>(pr + g4);
#pragma unroll
                    for (int e = 0; e < DPL; ++e) {
                        acc_o[g4 + 0][e] = fmaf(pv.x, vf[e], acc_o[g4 + 0][e]);
                        acc_o[g4 + 1][e] = fmaf(pv.y, vf[e], acc_o[g4 + 1][e]);
                        acc_o[g4 + 2][e] = fmaf(pv.z, vf[e], acc_o[g4 + 2][e]);
                        acc_o[g4 + 3][e] = fmaf(pv.w, vf[e], acc_o[g4 + 3][e]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---- sum the four warps' partial outputs (the ring is free now)
    float* red = reinterpret_cast<float*>(smem);  // [4][GP][D]
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int e = 0; e < DPL; ++e) red[(warp * GP + g) * D + lane * DPL + e] = acc_o[g][e];
    __syncthreads();

    const int64_t qh0 = static_cast<int64_t>(b) * a.q_heads + static_cast<int64_t>(kvh) * G;
    if (splits_b == 1) {
        for (int idx = tid; idx < G * D; idx += kDecodeThreads) {
            const int g = idx / D, d = idx - g * D;
            float o = red[g * D + d] + red[(GP + g) * D + d] + red[(2 * GP + g) * D + d] +
                      red[(3 * GP + g) * D + d];
            const float l = l_s[g];
            o = l > 0.f ? o / l : 0.f;
            if (a.out_f32)
                static_cast<float*>(a.out)[(qh0 + g) * D + d] = o;
            else
                static_cast<T*>(a.out)[(qh0 + g) * D + d] = from_f32<T>(o);
            if (d == 0 && a.lse)
                a.lse[qh0 + g] = l > 0.f ? (m_s[g] + log2f(l)) * kLn2 : -INFINITY;
        }
        return;
    }

    // ---- several splits: publish (O, m, l), last CTA of this (seq, kv head) merges
    const int64_t pbase =
        ((static_cast<int64_t>(b) * a.kv_heads + kvh) * nsplit) * G;  // part row of split 0
    for (int idx = tid; idx < G * D; idx += kDecodeThreads) {
        const int g = idx / D, d = idx - g * D;
        float o = red[g * D + d] + red[(GP + g) * D + d] + red[(2 * GP + g) * D + d] +
                  red[(3 * GP + g) * D + d];
        a.part_o[(pbase + static_cast<int64_t>(split) * G + g) * D + d] = o;
    }
    if (tid < G) {
        a.part_ml[(pbase + static_cast<int64_t>(split) * G + tid) * 2 + 0] = m_s[tid];
        a.part_ml[(pbase + static_cast<int64_t>(split) * G + tid) * 2 + 1] = l_s[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int ticket = atomicAdd(&a.counters[static_cast<int64_t>(b) * a.kv_heads + kvh], 1);
        *flag_s = (ticket == splits_b - 1);
    }
    __syncthreads();
    if (!*flag_s) return;
    __threadfence();

    // merge weights w[s][g] = 2^(m_s - M_g), kept in the free ring
    float* wts = reinterpret_cast<float*>(smem);  // [splits_b][GP]
    float* lsp = wts + static_cast<int64_t>(nsplit) * GP;  // [splits_b][GP]
    float* Ms = lsp + static_cast<int64_t>(nsplit) * GP;
    float* den = Ms + GP;
    for (int i = tid; i < splits_b * G; i += kDecodeThreads) {
        const int s = i / G, g = i - s * G;
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + pbase + i);
        wts[s * GP + g] = ml.x;
        lsp[s * GP + g] = ml.y;
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s = 0; s < splits_b; ++s) M = fmaxf(M, wts[s * GP + tid]);
        float dsum = 0.f;
        for (int s = 0; s < splits_b; ++s) {
            const float w = (M == -INFINITY) ? 0.f : exp2f(wts[s * GP + tid] - M);
            wts[s * GP + tid] = w;
            dsum += w * lsp[s * GP + tid];
        }
        Ms[tid] = M;
        den[tid] = dsum;
    }
    __syncthreads();
    for (int idx = tid; idx < G * D; idx += kDecodeThreads) {
        const int g = idx / D, d = idx - g * D;
        float num = 0.f;
#pragma unroll 8
        for (int s = 0; s < splits_b; ++s)
            num += wts[s * GP + g] *
                   __ldcg(&a.part_o[(pbase + static_cast<int64_t>(s) * G + g) * D + d]);
        const float dn = den[g];
        const float o = dn > 0.f ? num / dn : 0.f;
        if (a.out_f32)
            static_cast<float*>(a.out)[(qh0 + g) * D + d] = o;
        else
            static_cast<T*>(a.out)[(qh0 + g) * D + d] = from_f32<T>(o);
        if (d == 0 && a.lse) a.lse[qh0 + g] = dn > 0.f ? (Ms[g] + log2f(dn)) * kLn2 : -INFINITY;
    }
    if (tid == 0) a.counters[static_cast<int64_t>(b) * a.kv_heads + kvh] = 0;
}

// ---- F16 tensor-core variant ----------------------------------------------------------
//
// Same contract as decode_split_kernel, for F16 caches with D in {64, 128} and G <= 16.
// The two skinny contractions run on the warp-level tensor cores (mma.sync m16n8k16, F16
// inputs, F32 accumulation): S[16 x 16] = Q[16 x D] K^T per 16-position sub-tile with the
// query heads (padded to 16 rows) as M, and O[16 x D] += P[16 x 16] V with P taken straight
// from S's accumulator registers (the C layout of S is the A layout of P).  Each of the 4
// warps runs its own cp.async ring of 16-position sub-tiles (sub-tiles w, w+4, ... of the
// CTA's chunk) and its own online softmax, so warps never wait on each other inside the
// loop; the four (m, l, O) states are combined once at the end.

// 2^x with the MUFU unit (PTX ex2.approx.ftz.f32: relative error about 2^-22; 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_cell(uint2* p, float v, unsigned step) {
    asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)),
                 "r"(step)
                 : "memory");
}
__device__ __forceinline__ uint2 ld_cell(const uint2* p) {
    uint2 v;
    asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p)
                 : "memory");
    return v;
}

// Reads cell `p` once it carries `step`; gives up (and returns false) once `deadline`
// of %globaltimer has passed.
__device__ __forceinline__ bool wait_cell(const uint2* p, unsigned step,
                                          unsigned long long deadline, float* out) {
    for (int spin = 0;; ++spin) {
        const uint2 c = ld_cell(p);
        if (c.y == step) {
            *out = __uint_as_float(c.x);
            return true;
        }
        if ((spin & 15) == 15) {
            if (global_ns() > deadline) return false;
            __nanosleep(32);
        }
    }
}

// Final step of a sequence split across GPUs, run by the CTA that holds the final
// (O, lse) of one (sequence, KV head) group on this rank (G rows from `row0`, staged in
// shared memory `fin`/`flse`): store the rows into every other rank's receive buffer over
// NVLink as {value, step} cells, then read the other ranks' rows of this group from this
// rank's buffer as their cells turn to this step (waiting at most ex->timeout_ns), and
// merge everything by log-sum-exp into `out`/`lse`.  Slots alternate by step parity, so a
// rank one step ahead never overwrites cells another rank is still reading.
// The reads are batched so their round trips overlap: first every other rank's lse of the
// group's rows, one cell per thread, then each thread's output cells of all ranks as one
// burst of independent loads (only cells not yet at this step are polled again).
// `scratch` is >= (kMaxRanks + 2) * 16 floats of free shared memory.
template <typename T>
__device__ void exchange_tail(const DecodeArgs& a, const float* fin, const float* flse, int G,
                              int D, int64_t row0, int* flag_s, float* scratch) {
    const ExchangeArgs* ex = a.ex;
    const int tid = threadIdx.x, world = ex->world, rank = ex->rank;
    const int64_t rows = ex->rows;
    const unsigned step = a.epoch;
    const int64_t par = static_cast<int64_t>(step & 1u) * world;
    const int64_t mine = (par + rank) * rows + row0;
    for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        uint2* dst = ex->recv_o[p] + mine * D;
        for (int i = tid; i < G * D; i += kDecodeThreads) st_cell(dst + i, fin[i], step);
        if (tid < G) st_cell(ex->recv_lse[p] + mine + tid, flse[tid], step);
    }
    float* wgt = scratch;                    // [kMaxRanks][16] merge weights e^(lse_p - M_g)
    float* den = scratch + kMaxRanks * 16;   // [16] their sums
    float* mx = den + 16;                    // [16] M_g
    if (tid == 0) *flag_s = 0;
    __syncthreads();
    const unsigned long long deadline = global_ns() + ex->timeout_ns;
    bool ok = true;
    // (1) every rank's lse of the group's rows, one cell per thread
    for (int c = tid; c < world * G; c += kDecodeThreads) {
        const int p = c / G, g = c - p * G;
        float v = flse[g];
        if (p != rank) {
            const uint2* cp = ex->recv_lse[rank] + (par + p) * rows + row0 + g;
            const uint2 cell = ld_cell(cp);
            if (cell.y == step) v = __uint_as_float(cell.x);
            else if (!wait_cell(cp, step, deadline, &v)) ok = false;
        }
        wgt[p * 16 + g] = v;
    }
    if (!ok) *flag_s = 1;
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int p = 0; p < world; ++p) M = fmaxf(M, wgt[p * 16 + tid]);
        float dsum = 0.f;
        for (int p = 0; p < world; ++p) {
            const float w = (M == -INFINITY) ? 0.f : __expf(wgt[p * 16 + tid] - M);
            wgt[p * 16 + tid] = w;
            dsum += w;
        }
        den[tid] = dsum;
        mx[tid] = M;
    }
    __syncthreads();
    ok = !*flag_s;
    // (2) the output cells: KB outputs of this thread x every other rank, loaded at once
    constexpr int KB = 4;
    for (int base = tid; base < G * D; base += KB * kDecodeThreads) {
        uint2 cell[KB][kMaxRanks];
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const int idx = base + k * kDecodeThreads;
#pragma unroll
            for (int p = 0; p < kMaxRanks; ++p) {
                cell[k][p] = make_uint2(0u, step);
                if (ok && idx < G * D && p < world && p != rank)
                    cell[k][p] = ld_cell(ex->recv_o[rank] + ((par + p) * rows + row0) * D + idx);
            }
        }
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const int idx = base + k * kDecodeThreads;
            if (idx >= G * D) break;
            const int g = idx / D, d = idx - g * D;
            float num = 0.f;
#pragma unroll
            for (int p = 0; p < kMaxRanks; ++p) {
                if (p >= world) break;
                float o = fin[idx];
                if (p != rank) {
                    if (cell[k][p].y == step) {
                        o = __uint_as_float(cell[k][p].x);
                    } else if (ok) {
                        ok = wait_cell(ex->recv_o[rank] + ((par + p) * rows + row0) * D + idx,
                                       step, deadline, &o);
                    }
                }
                num += wgt[p * 16 + g] * o;
            }
            const float dn = den[g];
            const float ov = (!ok || !(dn > 0.f)) ? 0.f : num / dn;
            const int64_t row = row0 + g;
            if (a.out_f32)
                static_cast<float*>(a.out)[row * D + d] = ov;
            else
                static_cast<T*>(a.out)[row * D + d] = from_f32<T>(ov);
            if (d == 0 && a.lse)
                a.lse[row] = (!ok || !(dn > 0.f)) ? -INFINITY : mx[g] + logf(dn);
        }
    }
    if (!ok) {
        atomicExch(ex->status, TMLLM_TIMEOUT);
        *flag_s = 1;
    }
}

template <int D, int STAGES, int PS = 1>
struct MmaCfg {
    static constexpr int C = D / 8;         // 16-byte chunks per row
    static constexpr int ROW = D * 2;       // bytes per row
    static constexpr int SUB = 16;          // positions per warp sub-tile
    static constexpr int SUBB = SUB * ROW;  // bytes of one K (or V) sub-tile
    // a ring stage holds one item of PS sub-tiles: K sub-tiles, then V sub-tiles
    static constexpr int WARP_RING = STAGES * 2 * SUBB * PS;
    static constexpr int QROW = D + 8;      // padded q row (halves)
    static constexpr int OFF_Q = 4 * WARP_RING;
    static constexpr int OFF_ST = OFF_Q + 16 * QROW * 2;  // m, l per warp x row + flag
    static constexpr int OFF_NEW = OFF_ST + (2 * 4 * 16 + 16) * 4;
    static constexpr int BYTES = OFF_NEW + 2 * ROW;
    // exchange staging (final rows of a group) at the end of the rings: [16][D] + [16] F32
    static constexpr int OFF_FIN = 4 * WARP_RING - (16 * D + 16) * 4;
    static constexpr int LOADS = SUB * C / 32;  // 16-byte copies per lane per K sub-tile
    static constexpr int RSTEP = 32 / C;
    static_assert(C == 8 || C == 16, "D must be 64 or 128");
    static_assert(OFF_FIN >= 4 * 16 * D * 4, "warp-merge scratch and staging fit in the rings");
};

// PT (positions-major, D = 64 and G <= 8): S^T[16 positions x 8 heads] = K Q^T with K as
// the A operand and the query heads as N, O^T[D x 8] += V^T P^T with V (ldmatrix.trans) as
// A and P^T as B, moved from S^T's accumulator layout by movmatrix.trans.  Half the MMAs
// and rescales and 6 instead of 10 exponentials a thread per sub-tile compared with the
// head-major form (whose M = 16 rows carry only G real query heads): at short contexts the
// loop is bound by a warp's per-sub-tile chain, not by memory bandwidth.
template <int D, int STAGES, bool PT>
__global__ void __launch_bounds__(kDecodeThreads, D == 64 ? (PT ? kD64PtMinBlocks : kD64MinBlocks) : 2)
    decode_mma_kernel(const DecodeArgs a) {
    constexpr int PS = PT ? 2 : 1;  // 16-position sub-tiles per item (one softmax update)
    using Cfg = MmaCfg<D, STAGES, PS>;
    static_assert(!PT || D == 64, "the positions-major form is instantiated for D = 64");
    constexpr int C = Cfg::C, ROW = Cfg::ROW, SUBB = Cfg::SUBB, QROW = Cfg::QROW;
    constexpr int KS = D / 16;  // k-steps of QK
    constexpr int NT = D / 8;   // n-tiles of PV
    extern __shared__ __align__(128) unsigned char smem[];
    __half* q_s = reinterpret_cast<__half*>(smem + Cfg::OFF_Q);  // [16][QROW]
    float* wm = reinterpret_cast<float*>(smem + Cfg::OFF_ST);    // [4][16]
    float* wl = wm + 64;                                          // [4][16]
    int* flag_s = reinterpret_cast<int*>(wl + 64);
    __half* knew_s = reinterpret_cast<__half*>(smem + Cfg::OFF_NEW);
    __half* vnew_s = knew_s + D;
    float* fin = reinterpret_cast<float*>(smem + Cfg::OFF_FIN);  // [16][D] exchange staging
    float* flse = fin + 16 * D;                                  // [16]

    const int split = blockIdx.z, kvh = blockIdx.x, b = blockIdx.y;  // splits slowest
    const int nsplit = gridDim.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.group;
    launch_dependents();
    // With an overlapped launch (TMLLM_DECODE_OVERLAP) everything up to the K/V ring's
    // prologue reads only the cache (lengths, block table, cached K/V), which the kernel
    // ahead of this one does not write; q, k_new and v_new are read after its completion.
    const bool whole_blocks = (a.block_size % 16) == 0;
    const int t0 = split * a.chunk;
    // A warp takes items warp, warp + 4, ... of the chunk; item j holds PS sub-tiles, so
    // sub-tile s of this warp (item s / PS, part s % PS) starts at position
    // t0 + ((warp + 4 (s / PS)) PS + s % PS) 16.
    // Block-table entry of this warp's sub-tile s (with whole blocks a sub-tile lies in one
    // block; out-of-table positions give -1).  At D = 64 (short sub-tiles, where a table
    // read per sub-tile left the ring waiting at short contexts) the entries sit 32 at a
    // time in the lanes: lane l holds the entry of sub-tile jb + l (`cur`) and of
    // jb + 32 + l (`nxt`, read a batch ahead), so issuing a sub-tile's copies never waits
    // on a table read; the first two batches depend on the chunk only and are read
    // together with the length.  At D = 128 the entry is read at issue (measured 1.5 %
    // faster there: fewer registers on the critical loop).
    auto sub_pos = [&](int sidx) -> int64_t {  // may run past the chunk: 64-bit position
        return static_cast<int64_t>(t0) + ((warp + 4 * (sidx / PS)) * PS + sidx % PS) * 16;
    };
    auto entry = [&](int sidx) -> int64_t {
        return whole_blocks ? block_of(a, b, sub_pos(sidx)) : -1;
    };
    constexpr bool kLaneTable = D == 64;
    int64_t cur = -1, nxt = -1;
    if (kLaneTable) {
        cur = entry(lane);
        nxt = entry(32 + lane);
    }
    const int cached = a.seq_lens[b] < 0 ? 0 : a.seq_lens[b];
    const bool has_new = a.k_new != nullptr;
    const int L = cached + (has_new ? 1 : 0);
    int splits_b = (L + a.chunk - 1) / a.chunk;
    if (splits_b < 1) splits_b = 1;
    if (splits_b > nsplit) splits_b = nsplit;
    if (split >= splits_b) return;
    const int t1 = (split == splits_b - 1) ? L : min(L, t0 + a.chunk);
    const int nitem = t1 > t0 ? (t1 - t0 + 16 * PS - 1) / (16 * PS) : 0;
    const bool owns_new = has_new && cached >= t0 && cached < t1;
    const int half = D / 2;
    const int qpos = cached + a.rope_off;

    // ---- this warp's cp.async ring: items warp, warp+4, ... of the chunk
    unsigned char* ring = smem + warp * Cfg::WARP_RING;
    const int nmine = nitem > warp ? (nitem - warp + 3) / 4 : 0;
    const unsigned char* kbase = static_cast<const unsigned char*>(a.k_cache);
    const unsigned char* vbase = static_cast<const unsigned char*>(a.v_cache);
    const int lc = lane % C, lr0 = lane / C;
    int dst_off[Cfg::LOADS];
#pragma unroll
    for (int k = 0; k < Cfg::LOADS; ++k) {
        const int r = lr0 + k * Cfg::RSTEP;
        dst_off[k] = r * ROW + swz<C>(r, lc) * 16;
    }
    // called with warp-uniform sub-tile indices 0, 1, 2, ... (items < nmine)
    int jb = 0;
    auto sub_block = [&](int sidx) -> int64_t {
        if (!kLaneTable)
            return whole_blocks && sidx / PS < nmine ? block_of(a, b, sub_pos(sidx)) : -1;
        if (sidx >= jb + 32) {
            jb += 32;
            cur = nxt;
            nxt = entry(jb + 32 + lane);
        }
        return __shfl_sync(0xffffffffu, cur, sidx - jb);
    };
    // one 16-position sub-tile starting at `base` into ks / vs
    auto load_sub = [&](int base, unsigned char* ks, unsigned char* vs, int64_t blk) {
        int64_t row0 = -1;  // arena row of position `base` when the sub-tile is one block
        if (whole_blocks) {
            if (blk >= 0)
                row0 = (blk * a.kv_heads + kvh) * a.block_size + offset_in_block(a, base);
        }
        if (row0 >= 0 && base + 16 <= cached && base + 16 <= t1) {
            // the common case: 16 cached positions inside one block
            const int64_t off0 = row0 * ROW + lr0 * ROW + lc * 16;
#pragma unroll
            for (int k = 0; k < Cfg::LOADS; ++k) {
                const int64_t off = off0 + static_cast<int64_t>(k * Cfg::RSTEP) * ROW;
                cp_async16(ks + dst_off[k], kbase + off, 16);
                cp_async16(vs + dst_off[k], vbase + off, 16);
            }
            return;
        }
#pragma unroll
        for (int k = 0; k < Cfg::LOADS; ++k) {
            const int r = lr0 + k * Cfg::RSTEP;
            const int pos = base + r;
            const unsigned char* ksrc = kbase;
            const unsigned char* vsrc = vbase;
            int bytes = 0;
            if (pos < cached && pos < t1) {
                int64_t arow = -1;
                if (whole_blocks) {
                    if (row0 >= 0) arow = row0 + r;
                } else {
                    const int64_t blk = block_of(a, b, pos);
                    if (blk >= 0)
                        arow = (blk * a.kv_heads + kvh) * a.block_size + offset_in_block(a, pos);
                }
                if (arow >= 0) {
                    const int64_t off = arow * ROW + lc * 16;
                    ksrc += off;
                    vsrc += off;
                    bytes = 16;
                }
            }
            cp_async16(ks + dst_off[k], ksrc, bytes);
            cp_async16(vs + dst_off[k], vsrc, bytes);
        }
    };
    // item j (its PS sub-tiles) into ring stage `stage`
    auto load_item = [&](int j, int stage) {
        unsigned char* kst = ring + stage * 2 * PS * SUBB;
#pragma unroll
        for (int k = 0; k < PS; ++k)
            load_sub(t0 + ((warp + 4 * j) * PS + k) * 16, kst + k * SUBB,
                     kst + (PS + k) * SUBB, sub_block(j * PS + k));
    };
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nmine) load_item(s, s);
        cp_async_commit();
    }
    if (a.overlap) grid_dependency_wait();  // q, k_new, v_new come from the kernel ahead

    // ---- (while the first K/V tiles are in flight) q rows, rotated and rounded to F16,
    // into q_s; rows >= G are zero
    for (int idx = tid; idx < 16 * half; idx += kDecodeThreads) {
        const int g = idx / half, i = idx - g * half;
        float x1 = 0.f, x2 = 0.f;
        if (g < G) {
            const __half* qr = static_cast<const __half*>(a.q) +
                               static_cast<int64_t>(b) * a.q_stride +
                               static_cast<int64_t>(kvh * G + g) * D;
            x1 = __half2float(qr[i]);
            x2 = __half2float(qr[i + half]);
            rope_pair(a, qpos, i, half, x1, x2);
        }
        q_s[g * QROW + i] = __float2half_rn(x1);
        q_s[g * QROW + i + half] = __float2half_rn(x2);
    }
    if (owns_new) {
        const int64_t nrow = static_cast<int64_t>(b) * a.kv_stride + static_cast<int64_t>(kvh) * D;
        const __half* kn = static_cast<const __half*>(a.k_new) + nrow;
        const __half* vn = static_cast<const __half*>(a.v_new) + nrow;
        for (int i = tid; i < half; i += kDecodeThreads) {
            float x1 = __half2float(kn[i]), x2 = __half2float(kn[i + half]);
            rope_pair(a, qpos, i, half, x1, x2);
            knew_s[i] = __float2half_rn(x1);
            knew_s[i + half] = __float2half_rn(x2);
            vnew_s[i] = vn[i];
            vnew_s[i + half] = vn[i + half];
        }
    }
    __syncthreads();
    if (owns_new) {
        const int64_t blk = block_of(a, b, cached);
        if (blk >= 0) {
            const int64_t off =
                ((blk * a.kv_heads + kvh) * a.block_size + offset_in_block(a, cached)) * D;
            __half* kd = static_cast<__half*>(a.k_cache) + off;
            __half* vd = static_cast<__half*>(a.v_cache) + off;
            for (int i = tid; i < D; i += kDecodeThreads) {
                kd[i] = knew_s[i];
                vd[i] = vnew_s[i];
            }
        }
    }

    const int g4 = lane >> 2, t4 = lane & 3;
    // ---- Q fragments into registers: head-major, A operand (16 rows x D); positions-major,
    // B operand (Q^T: k = dims, n = the 8 heads): thread holds q[g4][16ks + 2t4 (+8) ..+1]
    constexpr int QA = PT ? 2 : 4;
    uint32_t qa[KS][QA];
    if constexpr (PT) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            qa[ks][0] = *reinterpret_cast<const uint32_t*>(q_s + g4 * QROW + ks * 16 + 2 * t4);
            qa[ks][1] = *reinterpret_cast<const uint32_t*>(q_s + g4 * QROW + ks * 16 + 8 + 2 * t4);
        }
    } else {
        const int mi = lane >> 3, r = (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int col = ks * 16 + (mi >> 1) * 8;
            ldsm_x4(smem_u32(q_s + r * QROW + col), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
        }
    }

    // head-major: o[j] = O[rows g4, g4+8][dims 8j + 2t4 ..]; m_r / l_r of rows g4, g4 + 8.
    // positions-major: o[mt] = O^T[dims 16mt + g4 (+8)][heads 2t4, 2t4+1]; m_r / l_r of
    // heads 2t4, 2t4 + 1.
    constexpr int NO = PT ? D / 16 : NT;
    float o[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

    for (int it = 0; it < nmine; ++it) {
        cp_async_wait<STAGES - 2>();
        __syncwarp();
        {
            const int nt = it + STAGES - 1;
            if (nt < nmine) load_item(nt, nt % STAGES);
            cp_async_commit();
        }
        unsigned char* kst = ring + (it % STAGES) * 2 * PS * SUBB;  // K sub-tiles of the item
        unsigned char* vst = kst + PS * SUBB;                        // then its V sub-tiles
        const int base = t0 + (warp + 4 * it) * 16 * PS;
        if (owns_new && cached >= base && cached < base + 16 * PS) {
            const int rr = cached - base, kk = rr >> 4, r = rr & 15;
            if (lane < C) {
                *reinterpret_cast<uint4*>(kst + kk * SUBB + r * ROW + swz<C>(r, lane) * 16) =
                    reinterpret_cast<const uint4*>(knew_s)[lane];
                *reinterpret_cast<uint4*>(vst + kk * SUBB + r * ROW + swz<C>(r, lane) * 16) =
                    reinterpret_cast<const uint4*>(vnew_s)[lane];
            }
            __syncwarp();
        }
        if constexpr (PT) {
            // S^T = K Q^T per sub-tile: A = K rows (positions) by ldmatrix, B = Q^T from
            // registers; even and odd k-steps in separate accumulators, the PS sub-tiles'
            // chains independent.  st[k][e]: sub-tile k, positions g4 (e < 2) and g4 + 8,
            // heads 2t4 + (e & 1).
            float st[PS][4], sx[PS][4];
#pragma unroll
            for (int k = 0; k < PS; ++k)
#pragma unroll
                for (int e = 0; e < 4; ++e) st[k][e] = sx[k][e] = 0.f;
            {
                const int mi = lane >> 3, r = (mi & 1) * 8 + (lane & 7);
#pragma unroll
                for (int kstep = 0; kstep < KS; ++kstep) {
#pragma unroll
                    for (int k = 0; k < PS; ++k) {
                        const uint32_t rbase = smem_u32(kst + k * SUBB + r * ROW);
                        const int c = kstep * 2 + (mi >> 1);
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4(rbase + swz<C>(r, c) * 16, a0, a1, a2, a3);
                        mma16816((kstep & 1) ? sx[k] : st[k], a0, a1, a2, a3, qa[kstep][0],
                                 qa[kstep][1]);
                    }
                }
            }
            const bool full = base + 16 * PS <= t1;
#pragma unroll
            for (int k = 0; k < PS; ++k)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = (st[k][e] + sx[k][e]) * a.scale_log2;
                    if (!full && base + 16 * k + g4 + (e >= 2 ? 8 : 0) >= t1) v = -INFINITY;
                    st[k][e] = v;
                }
            // one online-softmax update per head over the item's 16 PS positions (8 lanes of
            // equal t4 x 2 rows x PS sub-tiles)
            float alpha[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float mx = fmaxf(st[0][h], st[0][2 + h]);
#pragma unroll
                for (int k = 1; k < PS; ++k) mx = fmaxf(mx, fmaxf(st[k][h], st[k][2 + h]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float m_new = fmaxf(m_r[h], mx);
                const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
                alpha[h] = fast_exp2(m_r[h] - m_use);
                float sum = 0.f;
#pragma unroll
                for (int k = 0; k < PS; ++k) {
                    const float p0 = fast_exp2(st[k][h] - m_use);
                    const float p1 = fast_exp2(st[k][2 + h] - m_use);
                    st[k][h] = p0;
                    st[k][2 + h] = p1;
                    sum += p0 + p1;
                }
                l_r[h] = l_r[h] * alpha[h] + sum;
                m_r[h] = m_new;
            }
            if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
                for (int mt = 0; mt < NO; ++mt) {
                    o[mt][0] *= alpha[0];
                    o[mt][1] *= alpha[1];
                    o[mt][2] *= alpha[0];
                    o[mt][3] *= alpha[1];
                }
            }
            // P^T of each sub-tile as a B operand: the 8 x 8 blocks (positions 0-7 | 8-15) x
            // heads of the accumulator layout, transposed across the warp
            uint32_t pb[PS][2];
#pragma unroll
            for (int k = 0; k < PS; ++k) {
                const uint32_t pk0 = pack_half2(st[k][0], st[k][1]);
                const uint32_t pk1 = pack_half2(st[k][2], st[k][3]);
                asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(pb[k][0]) : "r"(pk0));
                asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(pb[k][1]) : "r"(pk1));
            }
            // O^T += V^T P^T over the item's sub-tiles: A = V^T (dims x positions) by
            // ldmatrix.trans of the V rows
            {
                const int mi = lane >> 3, r = (mi >> 1) * 8 + (lane & 7);
#pragma unroll
                for (int mt = 0; mt < NO; ++mt) {
#pragma unroll
                    for (int k = 0; k < PS; ++k) {
                        const uint32_t rbase = smem_u32(vst + k * SUBB + r * ROW);
                        const int c = mt * 2 + (mi & 1);
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(rbase + swz<C>(r, c) * 16, a0, a1, a2, a3);
                        mma16816(o[mt], a0, a1, a2, a3, pb[k][0], pb[k][1]);
                    }
                }
            }
        } else {
            unsigned char* ks = kst;  // PS = 1: the item is one sub-tile
            unsigned char* vs = vst;
            // S = Q K^T: two n-tiles of 8 positions, even/odd k-steps in separate accumulators
            float sc[2][4], sx[2][4];
    #pragma unroll
            for (int n = 0; n < 2; ++n)
    #pragma unroll
                for (int e = 0; e < 4; ++e) sc[n][e] = sx[n][e] = 0.f;
            {
                const int mi = lane >> 3, r = (mi >> 1) * 8 + (lane & 7);
                const uint32_t rbase = smem_u32(ks + r * ROW);
    #pragma unroll
                for (int kstep = 0; kstep < KS; ++kstep) {
                    const int c = kstep * 2 + (mi & 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(rbase + swz<C>(r, c) * 16, b0, b1, b2, b3);
                    float* c0 = (kstep & 1) ? sx[0] : sc[0];
                    float* c1 = (kstep & 1) ? sx[1] : sc[1];
                    mma16816(c0, qa[kstep][0], qa[kstep][1], qa[kstep][2], qa[kstep][3], b0, b1);
                    mma16816(c1, qa[kstep][0], qa[kstep][1], qa[kstep][2], qa[kstep][3], b2, b3);
                }
            }
            const bool full = base + 16 <= t1;
    #pragma unroll
            for (int n = 0; n < 2; ++n)
    #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = (sc[n][e] + sx[n][e]) * a.scale_log2;
                    if (!full && base + n * 8 + t4 * 2 + (e & 1) >= t1) v = -INFINITY;
                    sc[n][e] = v;
                }
            // online softmax over the 16 positions, rows g4 and g4 + 8
            float alpha[2];
    #pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                float mx = fmaxf(fmaxf(sc[0][rr * 2], sc[0][rr * 2 + 1]),
                                 fmaxf(sc[1][rr * 2], sc[1][rr * 2 + 1]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float m_new = fmaxf(m_r[rr], mx);
                // rows that have seen no position yet keep m = -inf: use 0 as the reference
                const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
                alpha[rr] = fast_exp2(m_r[rr] - m_use);
                float sum = 0.f;
    #pragma unroll
                for (int n = 0; n < 2; ++n)
    #pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float p = fast_exp2(sc[n][rr * 2 + e] - m_use);
                        sc[n][rr * 2 + e] = p;
                        sum += p;
                    }
                l_r[rr] = l_r[rr] * alpha[rr] + sum;
                m_r[rr] = m_new;
            }
            if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
    #pragma unroll
                for (int j = 0; j < NT; ++j) {
                    o[j][0] *= alpha[0];
                    o[j][1] *= alpha[0];
                    o[j][2] *= alpha[1];
                    o[j][3] *= alpha[1];
                }
            }
            // O += P V: P's A fragment is S's accumulator layout
            const uint32_t pa0 = pack_half2(sc[0][0], sc[0][1]);
            const uint32_t pa1 = pack_half2(sc[0][2], sc[0][3]);
            const uint32_t pa2 = pack_half2(sc[1][0], sc[1][1]);
            const uint32_t pa3 = pack_half2(sc[1][2], sc[1][3]);
            {
                const int mi = lane >> 3, r = (mi & 1) * 8 + (lane & 7);
                const uint32_t rbase = smem_u32(vs + r * ROW);
    #pragma unroll
                for (int jj = 0; jj < NT / 2; ++jj) {
                    const int c = jj * 2 + (mi >> 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(rbase + swz<C>(r, c) * 16, b0, b1, b2, b3);
                    mma16816(o[2 * jj], pa0, pa1, pa2, pa3, b0, b1);
                    mma16816(o[2 * jj + 1], pa0, pa1, pa2, pa3, b2, b3);
                }
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        if constexpr (PT) {  // a head's positions sit in the 8 lanes of equal t4
            l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 4);
            l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 8);
            l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 16);
        } else {
            l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
            l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
        }
    }
    __syncthreads();

    // ---- combine the four warps: red[w][16][D] (rings are free now)
    float* red = reinterpret_cast<float*>(smem);
    if constexpr (PT) {  // rows = heads 2t4, 2t4 + 1 (< 8), dims 16mt + g4 (+8)
#pragma unroll
        for (int mt = 0; mt < NO; ++mt) {
            const int d = mt * 16 + g4;
            red[(warp * 16 + 2 * t4) * D + d] = o[mt][0];
            red[(warp * 16 + 2 * t4 + 1) * D + d] = o[mt][1];
            red[(warp * 16 + 2 * t4) * D + d + 8] = o[mt][2];
            red[(warp * 16 + 2 * t4 + 1) * D + d + 8] = o[mt][3];
        }
        if (g4 == 0) {
            wm[warp * 16 + 2 * t4] = m_r[0];
            wm[warp * 16 + 2 * t4 + 1] = m_r[1];
            wl[warp * 16 + 2 * t4] = l_r[0];
            wl[warp * 16 + 2 * t4 + 1] = l_r[1];
        }
    } else {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int d = j * 8 + t4 * 2;
            red[(warp * 16 + g4) * D + d] = o[j][0];
            red[(warp * 16 + g4) * D + d + 1] = o[j][1];
            red[(warp * 16 + g4 + 8) * D + d] = o[j][2];
            red[(warp * 16 + g4 + 8) * D + d + 1] = o[j][3];
        }
        if (t4 == 0) {
            wm[warp * 16 + g4] = m_r[0];
            wm[warp * 16 + g4 + 8] = m_r[1];
            wl[warp * 16 + g4] = l_r[0];
            wl[warp * 16 + g4 + 8] = l_r[1];
        }
    }
    __syncthreads();
    // per row g: M = max_w m_w, weights 2^(m_w - M)
    const int64_t qh0 = static_cast<int64_t>(b) * a.q_heads + static_cast<int64_t>(kvh) * G;
    const int64_t pbase = ((static_cast<int64_t>(b) * a.kv_heads + kvh) * nsplit) * G;
    for (int idx = tid; idx < G * D; idx += kDecodeThreads) {
        const int g = idx / D, d = idx - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w * 16 + g]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float wt = (M == -INFINITY) ? 0.f : exp2f(wm[w * 16 + g] - M);
            num += wt * red[(w * 16 + g) * D + d];
            den += wt * wl[w * 16 + g];
        }
        if (splits_b == 1) {
            const float ov = den > 0.f ? num / den : 0.f;
            const float lv = den > 0.f ? (M + log2f(den)) * kLn2 : -INFINITY;
            if (a.ex) {
                fin[g * D + d] = ov;
                if (d == 0) flse[g] = lv;
            } else {
                if (a.out_f32)
                    static_cast<float*>(a.out)[(qh0 + g) * D + d] = ov;
                else
                    static_cast<__half*>(a.out)[(qh0 + g) * D + d] = __float2half_rn(ov);
                if (d == 0 && a.lse) a.lse[qh0 + g] = lv;
            }
        } else {
            a.part_o[(pbase + static_cast<int64_t>(split) * G + g) * D + d] = num;
            if (d == 0) {
                a.part_ml[(pbase + static_cast<int64_t>(split) * G + g) * 2 + 0] = M;
                a.part_ml[(pbase + static_cast<int64_t>(split) * G + g) * 2 + 1] = den;
            }
        }
    }
    if (splits_b == 1) {
        if constexpr (!PT) {  // the positions-major form never runs with the exchange
            if (a.ex) {
                __syncthreads();
                exchange_tail<__half>(a, fin, flse, G, D, qh0, flag_s,
                                      reinterpret_cast<float*>(smem));
            }
        }
        return;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int ticket = atomicAdd(&a.counters[static_cast<int64_t>(b) * a.kv_heads + kvh], 1);
        *flag_s = (ticket == splits_b - 1);
    }
    __syncthreads();
    if (!*flag_s) return;
    __threadfence();
    float* wts = reinterpret_cast<float*>(smem);  // [splits_b][16] (red is consumed)
    float* lsp = wts + static_cast<int64_t>(nsplit) * 16;  // [splits_b][16]
    float* Ms = lsp + static_cast<int64_t>(nsplit) * 16;
    float* dens = Ms + 16;
    // Each thread merges 4 consecutive dims of one head.  When all partial outputs fit in
    // the free rings they are staged there with one burst of cp.async, issued before the
    // (m, l) pairs are read, so both travel in one L2 round trip and the merge weights are
    // computed while the outputs are in flight; otherwise they are read with one 16-byte
    // L2 load per split.
    const int64_t stride4 = static_cast<int64_t>(G) * D / 4;
    const float4* src0 = reinterpret_cast<const float4*>(a.part_o + pbase * D);
    const size_t stage_bytes = static_cast<size_t>(splits_b) * stride4 * 16;
    const size_t stage_off = static_cast<size_t>(2 * nsplit * 16 + 32) * 4;
    const bool staged = stage_off + stage_bytes <= static_cast<size_t>(Cfg::OFF_FIN);
    float4* stage = reinterpret_cast<float4*>(smem + ((stage_off + 15) & ~static_cast<size_t>(15)));
    if (staged) {
        for (int64_t i = tid; i < splits_b * stride4; i += kDecodeThreads)
            cp_async16(stage + i, src0 + i, 16);
        cp_async_commit();
    }
    // all (m, l) pairs of this (sequence, KV head)
    for (int i = tid; i < splits_b * G; i += kDecodeThreads) {
        const int s2 = i / G, g = i - s2 * G;
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + pbase + i);
        wts[s2 * 16 + g] = ml.x;
        lsp[s2 * 16 + g] = ml.y;
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < splits_b; ++s2) M = fmaxf(M, wts[s2 * 16 + tid]);
        float dsum = 0.f;
        for (int s2 = 0; s2 < splits_b; ++s2) {
            const float w = (M == -INFINITY) ? 0.f : exp2f(wts[s2 * 16 + tid] - M);
            wts[s2 * 16 + tid] = w;
            dsum += w * lsp[s2 * 16 + tid];
        }
        Ms[tid] = M;
        dens[tid] = dsum;
    }
    if (staged) cp_async_wait<0>();
    __syncthreads();
    for (int idx = tid; idx < stride4; idx += kDecodeThreads) {
        const int g = idx / (D / 4), d = (idx - g * (D / 4)) * 4;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int s2 = 0; s2 < splits_b; ++s2) {
            const float w = wts[s2 * 16 + g];
            const float4 v = staged ? stage[s2 * stride4 + idx] : __ldcg(src0 + s2 * stride4 + idx);
            num.x += w * v.x;
            num.y += w * v.y;
            num.z += w * v.z;
            num.w += w * v.w;
        }
        const float dn = dens[g];
        const float inv = dn > 0.f ? 1.f / dn : 0.f;
        const float ov[4] = {num.x * inv, num.y * inv, num.z * inv, num.w * inv};
        const float lv = dn > 0.f ? (Ms[g] + log2f(dn)) * kLn2 : -INFINITY;
        if (a.ex) {
            for (int e = 0; e < 4; ++e) fin[g * D + d + e] = ov[e];
            if (d == 0) flse[g] = lv;
            continue;
        }
        for (int e = 0; e < 4; ++e) {
            if (a.out_f32)
                static_cast<float*>(a.out)[(qh0 + g) * D + d + e] = ov[e];
            else
                static_cast<__half*>(a.out)[(qh0 + g) * D + d + e] = __float2half_rn(ov[e]);
        }
        if (d == 0 && a.lse) a.lse[qh0 + g] = lv;
    }
    if (tid == 0) a.counters[static_cast<int64_t>(b) * a.kv_heads + kvh] = 0;
    if constexpr (!PT) {
        if (a.ex) {  // the rings are free: their start is the exchange's scratch
            __syncthreads();
            exchange_tail<__half>(a, fin, flse, G, D, qh0, flag_s,
                                  reinterpret_cast<float*>(smem));
        }
    }
}

// Any even head_dim: one CTA per (seq, query head), tiles of 128 positions, one thread per
// position for QK^T and one thread per dimension for PV.  Used for head sizes the tiled
// kernel does not instantiate (the reference's unit tests use D = 2 and 4).
template <typename T>
__global__ void __launch_bounds__(128) decode_generic_kernel(const DecodeArgs a, int D) {
    extern __shared__ __align__(128) unsigned char smem[];
    float* q_s = reinterpret_cast<float*>(smem);  // [D]
    float* kn_s = q_s + D;                        // [D] rotated k_new
    float* vn_s = kn_s + D;                       // [D]
    float* p_s = vn_s + D;                        // [128]
    float* red = p_s + 128;                       // [4]
    const int qh = blockIdx.x, b = blockIdx.y;
    const int kvh = qh / a.group, g = qh % a.group;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cached = a.seq_lens[b] < 0 ? 0 : a.seq_lens[b];
    const bool has_new = a.k_new != nullptr;
    const int L = cached + (has_new ? 1 : 0);
    const int half = D / 2;
    const int qpos = cached + a.rope_off;
    const T* qr = static_cast<const T*>(a.q) + static_cast<int64_t>(b) * a.q_stride +
                  static_cast<int64_t>(qh) * D;
    for (int i = tid; i < half; i += 128) {
        float x1 = to_f32<T>(qr[i]), x2 = to_f32<T>(qr[i + half]);
        rope_pair(a, qpos, i, half, x1, x2);
        q_s[i] = round_store<T>(x1);
        q_s[i + half] = round_store<T>(x2);
    }
    if (has_new) {
        const int64_t nrow = static_cast<int64_t>(b) * a.kv_stride + static_cast<int64_t>(kvh) * D;
        const T* kn = static_cast<const T*>(a.k_new) + nrow;
        const T* vn = static_cast<const T*>(a.v_new) + nrow;
        for (int i = tid; i < half; i += 128) {
            float x1 = to_f32<T>(kn[i]), x2 = to_f32<T>(kn[i + half]);
            rope_pair(a, qpos, i, half, x1, x2);
            kn_s[i] = round_store<T>(x1);
            kn_s[i + half] = round_store<T>(x2);
            vn_s[i] = to_f32<T>(vn[i]);
            vn_s[i + half] = to_f32<T>(vn[i + half]);
        }
    }
    __syncthreads();
    if (has_new && g == 0) {
        const int64_t blk = block_of(a, b, cached);
        if (blk >= 0) {
            const int64_t off =
                ((blk * a.kv_heads + kvh) * a.block_size + offset_in_block(a, cached)) * D;
            for (int i = tid; i < D; i += 128) {
                static_cast<T*>(a.k_cache)[off + i] = from_f32<T>(kn_s[i]);
                static_cast<T*>(a.v_cache)[off + i] = from_f32<T>(vn_s[i]);
            }
        }
    }
    float m = -INFINITY, l = 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // dims tid, tid+128, ... (D <= 512)
    const T* kc = static_cast<const T*>(a.k_cache);
    const T* vc = static_cast<const T*>(a.v_cache);
    for (int base = 0; base < L; base += 128) {
        const int pos = base + tid;
        float s = -INFINITY;
        if (pos < L) {
            float dot = 0.f;
            if (pos == cached && has_new) {
                for (int d = 0; d < D; ++d) dot = fmaf(q_s[d], kn_s[d], dot);
                s = dot * a.scale_log2;
            } else {
                const int64_t blk = block_of(a, b, pos);
                if (blk >= 0) {
                    const T* kr = kc + ((blk * a.kv_heads + kvh) * a.block_size +
                                        offset_in_block(a, pos)) * static_cast<int64_t>(D);
                    for (int d = 0; d < D; ++d) dot = fmaf(q_s[d], to_f32<T>(kr[d]), dot);
                    s = dot * a.scale_log2;
                }
            }
        }
        float mx = warp_max(s);
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        __syncthreads();
        const float m_new = fmaxf(m, mx);
        const float p = (m_new == -INFINITY || s == -INFINITY) ? 0.f : exp2f(s - m_new);
        const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m - m_new);
        p_s[tid] = p;
        float ps = warp_sum(p);
        if (lane == 0) red[warp] = ps;
        __syncthreads();
        ps = red[0] + red[1] + red[2] + red[3];
        l = l * alpha + ps;
        m = m_new;
        const int n = min(128, L - base);
        for (int k = 0; k < 4; ++k) {
            const int d = tid + 128 * k;
            if (d >= D) break;
            float o = acc[k] * alpha;
            for (int t = 0; t < n; ++t) {
                const int ps_pos = base + t;
                float vv;
                if (ps_pos == cached && has_new) {
                    vv = vn_s[d];
                } else {
                    const int64_t blk = block_of(a, b, ps_pos);
                    vv = blk < 0 ? 0.f
                                 : to_f32<T>(vc[((blk * a.kv_heads + kvh) * a.block_size +
                                                 offset_in_block(a, ps_pos)) *
                                                    static_cast<int64_t>(D) + d]);
                }
                o = fmaf(p_s[t], vv, o);
            }
            acc[k] = o;
        }
        __syncthreads();
    }
    const int64_t orow = (static_cast<int64_t>(b) * a.q_heads + qh) * D;
    for (int k = 0; k < 4; ++k) {
        const int d = tid + 128 * k;
        if (d >= D) break;
        const float o = l > 0.f ? acc[k] / l : 0.f;
        if (a.out_f32)
            static_cast<float*>(a.out)[orow + d] = o;
        else
            static_cast<T*>(a.out)[orow + d] = from_f32<T>(o);
    }
    if (tid == 0 && a.lse)
        a.lse[static_cast<int64_t>(b) * a.q_heads + qh] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
}

// Log-sum-exp merge of normalised partials: one block per row, threads over D.
template <typename OutT>
__global__ void merge_lse_kernel(const float* __restrict__ po, const float* __restrict__ pl,
                                 int n, int rows, int D, int64_t os, int64_t ls,
                                 OutT* __restrict__ out, float* __restrict__ out_lse) {
    const int r = blockIdx.x;
    float M = -INFINITY;
    for (int p = 0; p < n; ++p) M = fmaxf(M, pl[p * ls + r]);
    float den = 0.f;
    for (int p = 0; p < n; ++p) den += (M == -INFINITY) ? 0.f : expf(pl[p * ls + r] - M);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float num = 0.f;
        for (int p = 0; p < n; ++p) {
            const float w = (M == -INFINITY) ? 0.f : expf(pl[p * ls + r] - M);
            num += w * po[p * os + static_cast<int64_t>(r) * D + d];
        }
        out[static_cast<int64_t>(r) * D + d] = from_f32<OutT>(den > 0.f ? num / den : 0.f);
    }
    if (threadIdx.x == 0 && out_lse) out_lse[r] = den > 0.f ? M + logf(den) : -INFINITY;
}

// The same merge with one warp per row and 16-byte loads (parts 16-byte aligned, D and the
// part stride multiples of 4 floats, at most 32 parts): lane p holds part p's lse, the
// weights travel by shuffle, and each lane accumulates 4 consecutive dims of every part.
template <typename OutT>
__global__ void __launch_bounds__(128) merge_lse_vec_kernel(
    const float* __restrict__ po, const float* __restrict__ pl, int n, int rows, int D,
    int64_t os, int64_t ls, OutT* __restrict__ out, float* __restrict__ out_lse) {
    const int r = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;  // warp-uniform
    const float lp = lane < n ? pl[lane * ls + r] : -INFINITY;
    const float M = warp_max(lp);
    const float w = (M == -INFINITY || lane >= n) ? 0.f : expf(lp - M);
    const float den = warp_sum(w);
    for (int d4 = lane; d4 < D / 4; d4 += 32) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int p = 0; p < n; ++p) {
            const float wp = __shfl_sync(0xffffffffu, w, p);
            const float4 v = __ldg(reinterpret_cast<const float4*>(
                po + p * os + static_cast<int64_t>(r) * D + 4 * d4));
            acc.x += wp * v.x;
            acc.y += wp * v.y;
            acc.z += wp * v.z;
            acc.w += wp * v.w;
        }
        OutT* o = out + static_cast<int64_t>(r) * D + 4 * d4;
        o[0] = from_f32<OutT>(den > 0.f ? acc.x / den : 0.f);
        o[1] = from_f32<OutT>(den > 0.f ? acc.y / den : 0.f);
        o[2] = from_f32<OutT>(den > 0.f ? acc.z / den : 0.f);
        o[3] = from_f32<OutT>(den > 0.f ? acc.w / den : 0.f);
    }
    if (lane == 0 && out_lse) out_lse[r] = den > 0.f ? M + logf(den) : -INFINITY;
}

// ---- launch plumbing -------------------------------------------------------------------

// Opts `fn` into `bytes` of dynamic shared memory on the current device, once per device
// (bit d of `mask`, one mask per kernel instantiation): the attribute call costs more host
// time than the launch itself on short decode steps.
template <typename F>
int opt_in_smem(F* fn, size_t bytes, std::atomic<uint64_t>& mask) {
    int dev = 0;
    TMLLM_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (bit && (mask.load(std::memory_order_relaxed) & bit)) return TMLLM_OK;
    TMLLM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(bytes)));
    mask.fetch_or(bit, std::memory_order_relaxed);
    return TMLLM_OK;
}

// When asked (the allocation-free entry point, whose scratch keeps the previous call's
// contents), zero the split tickets on the stream right before the launch -- after every
// argument check, so a refused call enqueues nothing.  Tickets exist only with splits.
int clear_split_tickets(const DecodeArgs& a, dim3 grid, cudaStream_t s) {
    if (a.clear_tickets && grid.z > 1 && a.counters)
        TMLLM_CUDA_TRY(cudaMemsetAsync(a.counters, 0,
                                       static_cast<size_t>(grid.x) * grid.y * sizeof(int32_t), s));
    return TMLLM_OK;
}

struct WorkspaceLayout {
    size_t counters, part_ml, part_o, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

WorkspaceLayout workspace_layout(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t S) {
    WorkspaceLayout w;
    w.counters = 0;
    size_t c = align256(static_cast<size_t>(B * Hkv) * sizeof(int32_t));
    w.part_ml = c;
    size_t ml = align256(static_cast<size_t>(B * Hq * S * 2) * sizeof(float));
    w.part_o = c + ml;
    w.total = c + ml + align256(static_cast<size_t>(B * Hq * S * D) * sizeof(float));
    return w;
}

template <typename T, int D, int GP, int TT, int STAGES>
int launch_tiled(const DecodeArgs& a, dim3 grid, cudaStream_t s) {
    using Cfg = DecodeCfg<T, D, GP, TT, STAGES>;
    auto* fn = decode_split_kernel<T, D, GP, TT, STAGES>;
    const size_t bytes = static_cast<size_t>(Cfg::BYTES);
    const size_t need_merge = (2 * static_cast<size_t>(grid.z) + 2) * GP * 4;
    if (need_merge > static_cast<size_t>(STAGES * 2 * Cfg::TILE))
        return fail(TMLLM_INVALID_ARGUMENT, "too many splits (%u) for the merge scratch", grid.z);
    static std::atomic<uint64_t> opted{0};
    if (int st = opt_in_smem(fn, bytes, opted)) return st;
    if (int st = clear_split_tickets(a, grid, s)) return st;
    // Always a plain launch: this kernel reads q / k_new / v_new without a grid-dependency
    // wait, so it must not start before the kernel ahead of it has finished.
    fn<<<grid, kDecodeThreads, bytes, s>>>(a);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

template <int D, int STAGES, bool PT = false>
int launch_mma(const DecodeArgs& a, dim3 grid, cudaStream_t s) {
    using Cfg = MmaCfg<D, STAGES, PT ? 2 : 1>;
    auto* fn = decode_mma_kernel<D, STAGES, PT>;
    const size_t bytes = static_cast<size_t>(Cfg::BYTES);
    if ((2 * static_cast<size_t>(grid.z) + 2) * 16 * 4 > static_cast<size_t>(Cfg::OFF_FIN))
        return fail(TMLLM_INVALID_ARGUMENT, "too many splits (%u) for the merge scratch", grid.z);
    static std::atomic<uint64_t> opted{0};
    if (int st = opt_in_smem(fn, bytes, opted)) return st;
    if (int st = clear_split_tickets(a, grid, s)) return st;
    if (a.overlap) {
        // programmatic stream serialisation: the kernel may start while the one ahead of it
        // is still running; it reads q / k_new / v_new only after griddepcontrol.wait
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kDecodeThreads);
        cfg.dynamicSmemBytes = bytes;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        TMLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, a));
    } else {
        fn<<<grid, kDecodeThreads, bytes, s>>>(a);
    }
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

template <typename T, int D, int TT, int STAGES>
int launch_gp(const DecodeArgs& a, dim3 grid, cudaStream_t s) {
    if (a.group <= 4) return launch_tiled<T, D, 4, TT, STAGES>(a, grid, s);
    return launch_tiled<T, D, 8, TT, STAGES>(a, grid, s);
}

// Tiled configurations: (tile positions, ring depth) per (dtype, head_dim), each stage
// 32 KB (K+V) so three stages fit two CTAs per SM.
int launch_decode(int dtype, int D, int variant, const DecodeArgs& a, dim3 grid, cudaStream_t s,
                  bool* done) {
    *done = true;
    if (dtype == TMLLM_F16 && a.group <= 16 && variant != 1) {
        if (D == 64 && a.group <= 8 && a.ex == nullptr)
            return launch_mma<64, kD64PtStages, true>(a, grid, s);
        if (D == 64) return launch_mma<64, kD64Stages>(a, grid, s);
        if (D == 128) return launch_mma<128, 3>(a, grid, s);
    }
    if (dtype == TMLLM_F16 && a.group <= 8) {
        if (D == 64) return launch_gp<__half, 64, 128, 3>(a, grid, s);
        if (D == 128) return launch_gp<__half, 128, 64, 3>(a, grid, s);
        if (D == 256) return launch_gp<__half, 256, 32, 3>(a, grid, s);
    } else if (dtype == TMLLM_F32 && a.group <= 8) {
        if (D == 64) return launch_gp<float, 64, 64, 3>(a, grid, s);
        if (D == 128) return launch_gp<float, 128, 32, 3>(a, grid, s);
    }
    *done = false;
    return TMLLM_OK;
}

// Splits per (sequence, KV head): enough CTAs to fill every SM twice (two CTAs are
// resident per SM), at least two for long sequences of a big batch so lengths balance,
// and never chunks shorter than 256 positions.
int32_t auto_splits(int64_t B, int64_t Hkv, int64_t max_len) {
    const int64_t slots = static_cast<int64_t>(device_sm_count()) * 2;
    int64_t bh = B * Hkv;
    if (bh < 1) bh = 1;
    // as many splits as fit one wave of resident CTAs (a partial second wave would double
    // the time), at least two for long sequences of a big batch so lengths balance
    int64_t s = slots / bh;
    if (s < 2 && max_len > 1024) s = 2;
    const int64_t by_len = (max_len + 255) / 256;  // and never chunks under 256 positions
    if (s > by_len) s = by_len;
    if (s < 1) s = 1;
    if (s > 1024) s = 1024;
    return static_cast<int32_t>(s);
}

int32_t auto_splits_bound(int64_t B, int64_t Hkv) {
    const int64_t slots = static_cast<int64_t>(device_sm_count()) * 2;
    int64_t bh = B * Hkv;
    if (bh < 1) bh = 1;
    int64_t s = (slots + bh - 1) / bh;
    if (s < 2) s = 2;
    if (s > 1024) s = 1024;
    return static_cast<int32_t>(s);
}

}  // namespace

int decode_impl_ex(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                   const void* v_new, void* out, float* lse, int32_t q_heads,
                   const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                   int64_t max_len_hint, const ExchangeArgs* ex, uint32_t epoch,
                   bool clear_tickets, cudaStream_t stream, int64_t chunk_override = 0);

int decode_impl(const tmllm_paged_kv* kv, const void* q, const void* k_new, const void* v_new,
                void* out, float* lse, int32_t q_heads, const tmllm_decode_opts* opts,
                void* workspace, size_t workspace_bytes, int64_t max_len_hint,
                cudaStream_t stream) {
    return decode_impl_ex(kv, q, k_new, v_new, out, lse, q_heads, opts, workspace,
                          workspace_bytes, max_len_hint, nullptr, 0, false, stream);
}

// `ex` (device-resident) makes the launch finish a sequence split across GPUs: the final
// rows are exchanged with every rank and merged (tensor-core kernel only).  With
// `clear_tickets` the split tickets in the workspace are zeroed on `stream` right before
// the launch (only when the call passed every check and uses splits).  `chunk_override`
// > 0 sets the positions per split directly (rounded up to 128; the split count follows
// from the longest length), instead of deriving them from opts->num_splits.
int decode_impl_ex(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                   const void* v_new, void* out, float* lse, int32_t q_heads,
                   const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                   int64_t max_len_hint, const ExchangeArgs* ex, uint32_t epoch,
                   bool clear_tickets, cudaStream_t stream, int64_t chunk_override) {
    if (!kv) return fail(TMLLM_INVALID_ARGUMENT, "null paged KV descriptor");
    if (!valid_dtype(kv->dtype)) return fail(TMLLM_UNSUPPORTED_DTYPE, "unknown cache dtype");
    const int D = kv->head_dim, Hkv = kv->num_kv_heads, B = kv->num_seqs;
    if (B <= 0 || Hkv <= 0 || D <= 0 || kv->block_size <= 0 || kv->max_blocks_per_seq <= 0 ||
        kv->num_blocks <= 0)
        return fail(TMLLM_INVALID_SHAPE, "paged KV dimensions must be positive");
    if (D % 2 != 0 || D > 512)
        return fail(TMLLM_INVALID_SHAPE, "head_dim must be even and <= 512, got %d", D);
    if (B > 65535)  // the sequences are the grid's y dimension
        return fail(TMLLM_INVALID_SHAPE, "at most 65535 sequences per decode call, got %d", B);
    if (q_heads <= 0 || q_heads % Hkv != 0)
        return fail(TMLLM_MODEL_FORMAT, "Q heads %d must be divisible by non-zero KV heads %d",
                    q_heads, Hkv);
    const int G = q_heads / Hkv;
    if (opts && (opts->variant < 0 || opts->variant > 2))
        return fail(TMLLM_INVALID_ARGUMENT, "unknown decode variant %d", opts->variant);
    if (opts && (opts->flags & ~TMLLM_DECODE_OVERLAP))
        return fail(TMLLM_INVALID_ARGUMENT, "unknown decode flags 0x%x", opts->flags);
    const bool mma_shape = kv->dtype == TMLLM_F16 && (D == 64 || D == 128) &&
                           !(opts && opts->variant == 1);
    if (opts && opts->variant == 2 && !mma_shape)
        return fail(TMLLM_INVALID_ARGUMENT, "the tensor-core decode needs F16 and head_dim 64/128");
    if (G > (mma_shape ? 16 : 8))
        return fail(TMLLM_INVALID_SHAPE, "GQA group size %d exceeds %d for this head size", G,
                    mma_shape ? 16 : 8);
    if ((k_new == nullptr) != (v_new == nullptr))
        return fail(TMLLM_INVALID_ARGUMENT, "k_new and v_new must both be given or both be NULL");
    if (!q || !out || !kv->k_cache || !kv->v_cache || !kv->block_table || !kv->seq_lens)
        return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    int64_t capacity;
    if (!mul_ok(kv->block_size, kv->max_blocks_per_seq, &capacity) || capacity > INT32_MAX - 1)
        return fail(TMLLM_INVALID_SHAPE, "sequence capacity exceeds i32");
    tmllm_decode_opts o{};
    if (opts) o = *opts;
    if (o.out_f32 != 0 && o.out_f32 != 1)
        return fail(TMLLM_INVALID_ARGUMENT, "out_f32 must be 0 or 1");
    if (o.rope_cos && (!o.rope_sin || o.rope_len <= 0))
        return fail(TMLLM_INVALID_ARGUMENT, "RoPE needs both tables and a positive length");
    const float scale = o.scale > 0.f ? o.scale : 1.0f / sqrtf(static_cast<float>(D));
    if (!std::isfinite(scale))
        return fail(TMLLM_INVALID_SHAPE, "attention scale must be positive and finite");

    int64_t hint = max_len_hint > 0 ? max_len_hint : capacity;
    if (hint > capacity) hint = capacity;
    int32_t splits = o.num_splits > 0 ? o.num_splits : auto_splits(B, Hkv, hint);
    if (splits > 1024) splits = 1024;
    // positions per split: a multiple of 32 (one positions-major item), so the splits of a
    // long sequence come out nearly equal (config 4 at 8 ranks: 37 x 448 instead of 33 x 512
    // with 4 of the 37 CTAs a KV head idle)
    int64_t chunk = (hint + splits - 1) / splits;
    chunk = ((chunk + 31) / 32) * 32;
    if (chunk_override > 0) {
        chunk = ((chunk_override + 31) / 32) * 32;
        int64_t s2 = (hint + chunk - 1) / chunk;
        if (s2 < 1) s2 = 1;
        if (s2 > 1024) s2 = 1024;
        splits = static_cast<int32_t>(s2);
    }
    if (chunk < 128) chunk = 128;
    if (chunk > INT32_MAX) chunk = INT32_MAX;

    int bs_shift = -1;
    if ((kv->block_size & (kv->block_size - 1)) == 0) {
        bs_shift = 0;
        while ((1 << bs_shift) < kv->block_size) ++bs_shift;
    }

    DecodeArgs a{};
    a.q = q;
    a.k_new = k_new;
    a.v_new = v_new;
    a.k_cache = kv->k_cache;
    a.v_cache = kv->v_cache;
    a.block_table = kv->block_table;
    a.seq_lens = kv->seq_lens;
    a.out = out;
    a.lse = lse;
    a.rope_cos = o.rope_cos;
    a.rope_sin = o.rope_sin;
    a.rope_len = o.rope_len;
    a.rope_off = o.rope_pos_offset;
    a.num_blocks = kv->num_blocks;
    a.q_heads = q_heads;
    a.kv_heads = Hkv;
    a.group = G;
    a.block_size = kv->block_size;
    a.bs_shift = bs_shift;
    a.max_blocks = kv->max_blocks_per_seq;
    a.chunk = static_cast<int32_t>(chunk);
    a.out_f32 = o.out_f32 || kv->dtype == TMLLM_F32;
    a.scale_log2 = scale * kLog2e;
    a.ex = ex;
    a.epoch = epoch;
    if (o.q_seq_stride < 0 || o.kv_seq_stride < 0 ||
        (o.q_seq_stride > 0 && o.q_seq_stride < static_cast<int64_t>(q_heads) * D) ||
        (o.kv_seq_stride > 0 && o.kv_seq_stride < static_cast<int64_t>(Hkv) * D))
        return fail(TMLLM_INVALID_SHAPE, "sequence strides of q / k_new must cover a sequence");
    a.q_stride = o.q_seq_stride > 0 ? o.q_seq_stride : static_cast<int64_t>(q_heads) * D;
    a.kv_stride = o.kv_seq_stride > 0 ? o.kv_seq_stride : static_cast<int64_t>(Hkv) * D;
    // the overlapped launch applies to the tensor-core kernel (the CUDA-core kernels always
    // launch plainly); with the exchange it lets a step's prologue run under the previous
    // step's exchange, whose cells alternate by step parity
    a.overlap = (o.flags & TMLLM_DECODE_OVERLAP) ? 1 : 0;
    a.clear_tickets = clear_tickets ? 1 : 0;
    if (ex && !(mma_shape && o.variant != 1))
        return fail(TMLLM_INVALID_ARGUMENT,
                    "the cross-GPU exchange needs the tensor-core decode (F16, head_dim 64/128)");

    const size_t es = dtype_size(kv->dtype);
    auto misaligned = [es](const void* p) {
        return p != nullptr && (reinterpret_cast<uintptr_t>(p) % es) != 0;
    };
    if (misaligned(kv->k_cache) || misaligned(kv->v_cache) || misaligned(q) ||
        misaligned(k_new) || misaligned(v_new) || misaligned(out) ||
        (reinterpret_cast<uintptr_t>(lse) & 3u) != 0)
        return fail(TMLLM_INVALID_ARGUMENT, "tensor pointers must be aligned to their element size");
    // The tiled kernel stages K/V with 16-byte copies: it needs 16-byte aligned arenas.
    const int tiled_ok = (D == 64 || D == 128 || D == 256) &&
                         !(kv->dtype == TMLLM_F32 && D == 256) && aligned16(kv->k_cache) &&
                         aligned16(kv->v_cache);
    if (tiled_ok) {
        if (splits > 1) {
            const WorkspaceLayout w = workspace_layout(B, q_heads, Hkv, D, splits);
            if (!workspace || workspace_bytes < w.total)
                return fail(TMLLM_INVALID_ARGUMENT,
                            "decode workspace too small: need %zu bytes, got %zu", w.total,
                            workspace_bytes);
            unsigned char* base = static_cast<unsigned char*>(workspace);
            a.counters = reinterpret_cast<int32_t*>(base + w.counters);
            a.part_ml = reinterpret_cast<float*>(base + w.part_ml);
            a.part_o = reinterpret_cast<float*>(base + w.part_o);
        }
        // splits are the slowest grid dimension: every sequence's first chunk is scheduled
        // before any second chunk, so the short remainders of long sequences run last
        dim3 grid(static_cast<unsigned>(Hkv), static_cast<unsigned>(B),
                  static_cast<unsigned>(splits));
        bool done = false;
        int st = launch_decode(kv->dtype, D, o.variant, a, grid, stream, &done);
        if (done) return st;
    }
    if (ex)
        return fail(TMLLM_INVALID_ARGUMENT,
                    "the cross-GPU exchange needs 16-byte aligned K/V arenas");
    // generic path: one CTA per (query head, sequence), no splits
    const size_t smem = (3 * static_cast<size_t>(D) + 128 + 4) * sizeof(float);
    dim3 grid(static_cast<unsigned>(q_heads), static_cast<unsigned>(B));
    if (kv->dtype == TMLLM_F16)
        decode_generic_kernel<__half><<<grid, 128, smem, stream>>>(a, D);
    else
        decode_generic_kernel<float><<<grid, 128, smem, stream>>>(a, D);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

size_t decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t splits) {
    if (splits <= 1) return 256;
    return workspace_layout(B, Hq, Hkv, D, splits).total;
}

int32_t decode_auto_splits(int64_t B, int64_t Hkv, int64_t max_len) {
    return auto_splits(B, Hkv, max_len);
}

int32_t decode_auto_splits_bound(int64_t B, int64_t Hkv) { return auto_splits_bound(B, Hkv); }

// Resident CTAs per SM of the decode kernel that runs for this configuration.
int decode_resident_ctas(int dtype, int head_dim, int variant, int group) {
    if (dtype == TMLLM_F16 && head_dim == 64 && variant != 1 && group <= 8) return kD64PtMinBlocks;
    if (dtype == TMLLM_F16 && head_dim == 64 && variant != 1 && group <= 16) return kD64MinBlocks;
    return 2;
}

// Split count for a batch whose lengths the host knows (the cache runtime): the largest count
// whose CTAs -- ceil(len / chunk) per sequence and KV head, chunk as decode_impl_ex derives
// it from `hint` -- still fit one wave of resident CTAs (`per_sm` per SM), so the long
// sequences of a mixed batch are cut without pushing work into a second wave.  The CTA
// count grows with the split count, so the largest fitting count is found by bisection.
// Positions per split for a batch whose lengths the host knows: the smallest multiple of
// 32 whose CTAs -- ceil(len / chunk) per sequence and KV head -- fit one wave of resident
// CTAs (`per_sm` per SM), so only the sequences longer than the chunk are cut and no work
// spills into a second wave.  The same floors as the split-count choice below: never under
// 256 positions, and >= 1024 once one CTA per (sequence, KV head) covers every SM.  Finer
// than choosing a split count (chunk = ceil(longest / s)): 64 sequences of 256-2048
// positions x 5 KV heads at 3 CTAs per SM fit chunks of 1440 (440 CTAs; 1536 in steps of
// 128), where 2 splits (chunks of 1152) would need a second wave.  Returns the chunk, or
// the longest length rounded up when even one chunk per sequence overflows the wave.
int64_t decode_auto_chunk_lens(const int64_t* lens, int64_t B, int64_t Hkv, int64_t hint,
                               int per_sm) {
    const int64_t slots = static_cast<int64_t>(device_sm_count()) * per_sm;
    if (hint < 1) hint = 1;
    auto ctas = [&](int64_t chunk) {
        int64_t n = 0;
        for (int64_t b = 0; b < B; ++b) {
            const int64_t L = lens[b] > 0 ? lens[b] : 1;
            n += (L + chunk - 1) / chunk;
        }
        return n * Hkv;
    };
    int64_t hi = (hint + 31) / 32;  // in units of 32 positions
    int64_t lo = 8;                 // never under 256 positions
    if (B * Hkv >= static_cast<int64_t>(device_sm_count())) lo = 32;  // >= 1024
    const int64_t lo_splits = ((hint + 1023) / 1024 + 31) / 32;  // at most 1024 splits
    if (lo < lo_splits) lo = lo_splits;
    if (lo > hi) lo = hi;
    if (ctas(hi * 32) > slots) return hi * 32;
    while (lo < hi) {  // smallest k in [lo, hi] with ctas(32 k) <= slots
        const int64_t mid = (lo + hi) / 2;
        if (ctas(mid * 32) <= slots) hi = mid;
        else lo = mid + 1;
    }
    return lo * 32;
}

int32_t decode_auto_splits_lens(const int64_t* lens, int64_t B, int64_t Hkv, int64_t hint,
                                int per_sm) {
    const int64_t slots = static_cast<int64_t>(device_sm_count()) * per_sm;
    if (hint < 1) hint = 1;
    auto ctas = [&](int64_t s) {
        int64_t chunk = (hint + s - 1) / s;
        chunk = ((chunk + 127) / 128) * 128;
        if (chunk < 128) chunk = 128;
        int64_t n = 0;
        for (int64_t b = 0; b < B; ++b) {
            const int64_t L = lens[b] > 0 ? lens[b] : 1;
            n += (L + chunk - 1) / chunk;
        }
        return n * Hkv;
    };
    // Never chunks under 256 positions; and when one CTA per (sequence, KV head) already
    // covers every SM, a split only adds a merge, so chunks keep >= 1024 positions there
    // (measured: 577 positions x 192 heads ran 12.7 us unsplit vs 13.9 us in 3 chunks; 64
    // sequences of 256-2048 positions x 5 heads stay best at 2 chunks of <= 1152).
    int64_t hi = (hint + 255) / 256;
    if (B * Hkv >= static_cast<int64_t>(device_sm_count())) hi = hint / 1024;
    if (hi > 1024) hi = 1024;
    if (hi < 1) hi = 1;
    int64_t lo = 1;
    if (ctas(1) > slots) return 1;
    while (lo < hi) {  // largest s in [lo, hi] with ctas(s) <= slots
        const int64_t mid = (lo + hi + 1) / 2;
        if (ctas(mid) <= slots) lo = mid;
        else hi = mid - 1;
    }
    return static_cast<int32_t>(lo);
}

}  // namespace tmllm

using namespace tmllm;

extern "C" {

size_t tmllm_decode_workspace_bytes(int32_t num_seqs, int32_t q_heads, int32_t kv_heads,
                                    int32_t head_dim, int32_t num_splits) {
    if (num_seqs <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0) return 0;
    int64_t s = num_splits > 0 ? num_splits : auto_splits_bound(num_seqs, kv_heads);
    return decode_workspace_bytes(num_seqs, q_heads, kv_heads, head_dim, s);
}

int tmllm_decode_workspace_init(void* workspace, size_t bytes, tmllm_stream stream) {
    clear_error();
    if (!workspace || bytes == 0) return fail(TMLLM_INVALID_ARGUMENT, "null workspace");
    TMLLM_CUDA_TRY(cudaMemsetAsync(workspace, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
    return TMLLM_OK;
}

int32_t tmllm_decode_auto_splits(int32_t num_seqs, int32_t kv_heads, int64_t max_len) {
    return decode_auto_splits(num_seqs, kv_heads, max_len);
}

int tmllm_gqa_decode(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                     const void* v_new, void* out, float* lse, int32_t q_heads,
                     const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                     tmllm_stream stream) {
    clear_error();
    return decode_impl(kv, q, k_new, v_new, out, lse, q_heads, opts, workspace, workspace_bytes,
                       opts ? opts->max_len_hint : 0, reinterpret_cast<cudaStream_t>(stream));
}

int tmllm_merge_lse(const float* parts_o, const float* parts_lse, int32_t num_parts,
                    int32_t rows, int32_t head_dim, int64_t o_stride, int64_t lse_stride,
                    void* out, int32_t out_dtype, float* out_lse, tmllm_stream stream) {
    clear_error();
    if (num_parts <= 0 || rows <= 0 || head_dim <= 0)
        return fail(TMLLM_INVALID_SHAPE, "merge dimensions must be positive");
    if (!valid_dtype(out_dtype)) return fail(TMLLM_UNSUPPORTED_DTYPE, "unknown dtype");
    if (!parts_o || !parts_lse || !out) return fail(TMLLM_INVALID_ARGUMENT, "null pointer");
    const int64_t os = o_stride > 0 ? o_stride : static_cast<int64_t>(rows) * head_dim;
    const int64_t ls = lse_stride > 0 ? lse_stride : rows;
    if (os < static_cast<int64_t>(rows) * head_dim || ls < rows)
        return fail(TMLLM_INVALID_SHAPE, "merge strides overlap the parts");
    auto s = reinterpret_cast<cudaStream_t>(stream);
    if (num_parts <= 32 && head_dim % 4 == 0 && os % 4 == 0 && aligned16(parts_o)) {
        const unsigned blocks = static_cast<unsigned>((rows + 3) / 4);
        if (out_dtype == TMLLM_F16)
            merge_lse_vec_kernel<__half><<<blocks, 128, 0, s>>>(
                parts_o, parts_lse, num_parts, rows, head_dim, os, ls, static_cast<__half*>(out),
                out_lse);
        else
            merge_lse_vec_kernel<float><<<blocks, 128, 0, s>>>(
                parts_o, parts_lse, num_parts, rows, head_dim, os, ls, static_cast<float*>(out),
                out_lse);
        TMLLM_LAUNCH_TRY();
        return TMLLM_OK;
    }
    const int threads = head_dim >= 128 ? 128 : 64;
    if (out_dtype == TMLLM_F16)
        merge_lse_kernel<__half><<<rows, threads, 0, s>>>(parts_o, parts_lse, num_parts, rows,
                                                          head_dim, os, ls,
                                                          static_cast<__half*>(out), out_lse);
    else
        merge_lse_kernel<float><<<rows, threads, 0, s>>>(parts_o, parts_lse, num_parts, rows,
                                                         head_dim, os, ls,
                                                         static_cast<float*>(out), out_lse);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

}  // extern "C"
