// Prefill: a chunk of new tokens per sequence is appended to the paged KV cache and attends
// causally over everything the sequence has cached, in two launches:
//
//   prefill_append_kernel   RoPE on the new keys, storage rounding, scatter of K and V rows
//                           into the paged arena (kernels/rope.metal:57-63 and
//                           kernels/kv_cache_write.metal:13-18 over the block table);
//   prefill_tc_kernel<D>    flash attention on the 5th-generation tensor cores: one CTA per
//                           (128 query rows, query head, sequence).  Q·Kᵀ and P·V are
//                           tcgen05.mma (F16 operands in 128-byte-swizzled shared memory, F32
//                           accumulators in tensor memory); K and V pages arrive by TMA
//                           straight from the paged arena; the online softmax runs in four
//                           warps, one thread per query row, reading S out of tensor memory.
//
// The attention equals the reference's chain for S > 1 new tokens
// (nn/attention.rs:216-247 with start = cached length, :303-315): scores = Q·Kᵀ, scale,
// causal mask j > start + i -> -inf (kernels/attention_scale_mask.metal:21-41), softmax over
// the row (kernels/softmax.metal), P·V (kernels/gqa_matmul.metal:323-629), with the F32
// accumulation of those kernels and one F16 rounding of P before the second product.
// F32 caches, other head sizes and small pages run a CUDA-core kernel with the same
// semantics (prefill_generic_kernel).
#include <atomic>
#include <cuda.h>  // CUtensorMap and its enums; the encoder is fetched from the driver at run time

#include <cmath>
#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace tmllm {

namespace {

constexpr float kLog2eP = 1.4426950408889634f;
constexpr int kTile = 128;            // query rows per CTA and keys per tile
constexpr int kSoftmaxThreads = 128;  // warps 0-3: one thread per query row
constexpr int kPrefillThreads = 192;  // + warp 4: TMA producer, warp 5: MMA issuer
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // bounded waits: 1 s

// Status word of the bounded waits (TMLLM_TIMEOUT after an expired wait); read and cleared by
// tmllm_prefill_status.
__device__ int g_prefill_status;

struct PrefillArgs {
    const void* q;
    const void* k_new;
    const void* v_new;
    void* k_cache;
    void* v_cache;
    void* out;
    void* q_rot;  // when set, the append kernel also writes RoPE'd q here ([rows, Hq*D] F16)
    const int32_t* block_table;
    const int32_t* seq_lens;  // cached length of each sequence before this chunk
    const int32_t* q_start;   // [num_seqs + 1] row offsets, or null: uniform rows per sequence
    const float* rope_cos;
    const float* rope_sin;
    int64_t num_blocks;
    int64_t arena_rows;  // rows of D elements in one arena (TMA coordinate bound)
    int64_t q_stride;    // elements between consecutive rows of q
    int64_t kv_stride;   // elements between consecutive rows of k_new / v_new
    int64_t out_stride;  // elements between consecutive rows of out (q_heads * D)
    int32_t uniform_rows, num_seqs, total_rows;
    int32_t q_heads, kv_heads, group, head_dim, block_size, bs_shift, max_blocks;
    int32_t rope_len, rope_off, out_f32;
    int32_t rope_vec;  // tables 16-byte aligned: 8 entries per two vector loads
    int32_t rope_tma;  // head_dim 64: a unit's 128 table rows are staged by TMA
    float scale_log2;
};

__device__ __forceinline__ int seq_rows(const PrefillArgs& a, int s, int* row0) {
    if (a.q_start) {
        *row0 = a.q_start[s];
        return a.q_start[s + 1] - a.q_start[s];
    }
    *row0 = s * a.uniform_rows;
    return a.uniform_rows;
}

// Sequence owning packed row `row` (rows are grouped by sequence in order).
__device__ __forceinline__ int seq_of_row(const PrefillArgs& a, int row) {
    if (!a.q_start) return row / a.uniform_rows;
    int lo = 0, hi = a.num_seqs - 1;
    while (lo < hi) {  // last s with q_start[s] <= row
        const int mid = (lo + hi + 1) >> 1;
        if (a.q_start[mid] <= row) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Physical block of position `pos` of sequence `s`, or -1 outside the table / pool.
__device__ __forceinline__ int64_t page_of(const PrefillArgs& a, int s, int pos) {
    const int idx = a.bs_shift >= 0 ? (pos >> a.bs_shift) : (pos / a.block_size);
    if (pos < 0 || idx >= a.max_blocks) return -1;
    const int64_t blk = a.block_table[static_cast<int64_t>(s) * a.max_blocks + idx];
    return (blk >= 0 && blk < a.num_blocks) ? blk : -1;
}

__device__ __forceinline__ int in_page(const PrefillArgs& a, int pos) {
    return a.bs_shift >= 0 ? (pos & (a.block_size - 1)) : (pos % a.block_size);
}

// kernels/rope.metal:57-63 without contraction; identity outside the table.
__device__ __forceinline__ void rope_rotate(const PrefillArgs& a, int pos, int i, int half,
                                            float& x1, float& x2) {
    if (a.rope_cos == nullptr || pos < 0 || pos >= a.rope_len) return;
    const float c = __ldg(&a.rope_cos[static_cast<int64_t>(pos) * half + i]);
    const float s = __ldg(&a.rope_sin[static_cast<int64_t>(pos) * half + i]);
    const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    x1 = y1;
    x2 = y2;
}

// ---- append: one thread per (row, KV head, rotation pair) -----------------------------
template <typename T>
__global__ void prefill_append_kernel(const PrefillArgs a) {
    const int half = a.head_dim / 2;
    const int64_t total = static_cast<int64_t>(a.total_rows) * a.kv_heads * half;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int i = static_cast<int>(idx % half);
        const int64_t t = idx / half;
        const int kvh = static_cast<int>(t % a.kv_heads);
        const int row = static_cast<int>(t / a.kv_heads);
        const int s = seq_of_row(a, row);
        int row0;
        seq_rows(a, s, &row0);
        const int pos = a.seq_lens[s] + (row - row0);
        const int64_t blk = page_of(a, s, pos);
        if (blk < 0) continue;
        const int64_t src = static_cast<int64_t>(row) * a.kv_stride +
                            static_cast<int64_t>(kvh) * a.head_dim;
        const int64_t dst =
            ((blk * a.kv_heads + kvh) * a.block_size + in_page(a, pos)) * a.head_dim;
        const T* kn = static_cast<const T*>(a.k_new) + src;
        const T* vn = static_cast<const T*>(a.v_new) + src;
        float x1 = to_f32<T>(kn[i]), x2 = to_f32<T>(kn[i + half]);
        rope_rotate(a, pos + a.rope_off, i, half, x1, x2);
        T* kd = static_cast<T*>(a.k_cache) + dst;
        T* vd = static_cast<T*>(a.v_cache) + dst;
        kd[i] = from_f32<T>(x1);
        kd[i + half] = from_f32<T>(x2);
        vd[i] = vn[i];
        vd[i + half] = vn[i + half];
    }
}

// Vectorised append: one thread per (row, KV head, 16-byte chunk of the first half), so
// every load and store is 16 bytes (needs D/2 a multiple of a chunk and 16-byte aligned
// rows, arenas and tables).  Same rotation and rounding as prefill_append_kernel.  With
// `q_rot` set it also rotates the query rows (one thread per row, query head and chunk)
// into q_rot, so the attention kernel can load them rotated; without k_new it does only
// that.
template <typename T>
__global__ void prefill_append_vec_kernel(const PrefillArgs a) {
    constexpr int EPC = 16 / sizeof(T);  // elements per chunk
    const int half = a.head_dim / 2;
    const int cph = half / EPC;  // chunks per half row
    const int64_t kv_items = a.k_new ? static_cast<int64_t>(a.total_rows) * a.kv_heads * cph : 0;
    const int64_t q_items = a.q_rot ? static_cast<int64_t>(a.total_rows) * a.q_heads * cph : 0;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
         idx < kv_items + q_items; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool is_q = idx >= kv_items;
        const int64_t id = is_q ? idx - kv_items : idx;
        const int heads = is_q ? a.q_heads : a.kv_heads;
        const int c = static_cast<int>(id % cph);
        const int64_t t = id / cph;
        const int hh = static_cast<int>(t % heads);
        const int row = static_cast<int>(t / heads);
        const int s = seq_of_row(a, row);
        int row0;
        seq_rows(a, s, &row0);
        const int pos = a.seq_lens[s] + (row - row0);
        const T* src;
        T* dst;
        int64_t blk = 0;
        if (is_q) {
            src = static_cast<const T*>(a.q) + static_cast<int64_t>(row) * a.q_stride +
                  static_cast<int64_t>(hh) * a.head_dim + c * EPC;
            dst = static_cast<T*>(a.q_rot) +
                  static_cast<int64_t>(row) * a.q_heads * a.head_dim +
                  static_cast<int64_t>(hh) * a.head_dim + c * EPC;
        } else {
            blk = page_of(a, s, pos);
            if (blk < 0) continue;
            src = static_cast<const T*>(a.k_new) + static_cast<int64_t>(row) * a.kv_stride +
                  static_cast<int64_t>(hh) * a.head_dim + c * EPC;
            dst = static_cast<T*>(a.k_cache) +
                  ((blk * a.kv_heads + hh) * a.block_size + in_page(a, pos)) * a.head_dim +
                  c * EPC;
        }
        const uint4 k1 = __ldg(reinterpret_cast<const uint4*>(src));
        const uint4 k2 = __ldg(reinterpret_cast<const uint4*>(src + half));
        float x1[EPC], x2[EPC];
        Chunk<T>::unpack(k1, x1);
        Chunk<T>::unpack(k2, x2);
        const int rp = pos + a.rope_off;
        if (a.rope_cos != nullptr && rp >= 0 && rp < a.rope_len) {
            const float* cp = a.rope_cos + static_cast<int64_t>(rp) * half + c * EPC;
            const float* sp = a.rope_sin + static_cast<int64_t>(rp) * half + c * EPC;
#pragma unroll
            for (int e = 0; e < EPC; ++e) {  // kernels/rope.metal:57-63 without contraction
                const float cs = __ldg(cp + e), sn = __ldg(sp + e);
                const float y1 = __fsub_rn(__fmul_rn(x1[e], cs), __fmul_rn(x2[e], sn));
                const float y2 = __fadd_rn(__fmul_rn(x2[e], cs), __fmul_rn(x1[e], sn));
                x1[e] = y1;
                x2[e] = y2;
            }
        }
        uint4 o1, o2;
        T* p1 = reinterpret_cast<T*>(&o1);
        T* p2 = reinterpret_cast<T*>(&o2);
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
            p1[e] = from_f32<T>(x1[e]);
            p2[e] = from_f32<T>(x2[e]);
        }
        *reinterpret_cast<uint4*>(dst) = o1;
        *reinterpret_cast<uint4*>(dst + half) = o2;
        if (!is_q) {  // the value row is copied as it is
            const int64_t vs = static_cast<int64_t>(row) * a.kv_stride +
                               static_cast<int64_t>(hh) * a.head_dim + c * EPC;
            const T* vn = static_cast<const T*>(a.v_new) + vs;
            T* vd = static_cast<T*>(a.v_cache) + (dst - static_cast<T*>(a.k_cache));
            *reinterpret_cast<uint4*>(vd) = __ldg(reinterpret_cast<const uint4*>(vn));
            *reinterpret_cast<uint4*>(vd + half) = __ldg(reinterpret_cast<const uint4*>(vn + half));
        }
    }
}

// ---- PTX wrappers of this kernel (the shared ones are in tc.cuh) -----------------------
// Waits for the phase of parity `parity` of barrier `bar` to complete.  Gives up (false)
// when another thread of the CTA already gave up or after kWaitLimitNs, recording
// TMLLM_TIMEOUT; nothing in a correct run waits longer than microseconds.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long t0) {
    for (uint32_t it = 0;; ++it) {
        if (mbar_test(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*abort_flag) return false;
            if (global_ns() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                atomicExch(&g_prefill_status, TMLLM_TIMEOUT);
                return false;
            }
        }
    }
}
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D>
struct TcCfg {
    static constexpr int BLK = 16384;               // one 64-column block of a 128-row tile
    static constexpr int NB = D / 64;               // 64-column blocks per row
    static constexpr int TILE = NB * BLK;           // Q, K or V tile
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = TILE;              // 2 stages
    static constexpr int OFF_V = 3 * TILE;          // 2 stages
    static constexpr int OFF_P = 5 * TILE;          // 128 x 128 F16, two 64-key blocks
    static constexpr int OFF_BAR = OFF_P + 2 * BLK;
    static constexpr int SMEM = OFF_BAR + 256;
    // S: columns [0, 128); two O buffers (consecutive units alternate): [128, 128 + D) and
    // [128 + D, 128 + 2D)
    static constexpr int TMEM_COLS = D == 64 ? 256 : 512;
    static constexpr int MIN_BLOCKS = D == 64 ? 2 : 1;
};

// mbarriers (8 bytes each) after the tiles, then the tensor-memory address and the abort
// flag.  Full/empty pairs form the rings between the roles:
//   QL  raw Q tile landed (TMA)            Q   rotated Q written (softmax warps)
//   QE  Q tile no longer read (MMA)        KF/VF[st]  K/V stage loaded (TMA)
//   KE[st] K/V stage no longer read (MMA)  S   S = Q K^T done (MMA)
//   F   S copied to registers (softmax)    P   P tile written (softmax)
//   O[b] O_b += P V done (MMA)             E[b] O_b copied out by the epilogue (softmax)
//   RL  the unit's RoPE table rows landed in the P buffer (TMA, head_dim 64)
enum : int {
    BAR_QL = 0, BAR_Q = 1, BAR_QE = 2, BAR_KF = 3, BAR_VF = 5, BAR_KE = 7, BAR_S = 9,
    BAR_F = 10, BAR_P = 11, BAR_O = 12, BAR_E = 14, BAR_RL = 16, NBARS = 17
};

// One unit of work: 128 query rows of one (query head, sequence).  Units are numbered
// longest first (last row tile of every head/sequence, then the one before, ...) and dealt
// to the persistent CTAs in a snake order, so every CTA gets a similar number of key tiles.
struct Unit {
    int h, s, kvh, row0, rows, q_lo, cached, kv_len, nt;
};
__device__ __forceinline__ bool unit_of(const PrefillArgs& a, int k, int num_units,
                                        int row_tiles, Unit& u) {
    const int G = gridDim.x;
    const int idx = (k & 1) ? (k + 1) * G - 1 - static_cast<int>(blockIdx.x)
                            : k * G + static_cast<int>(blockIdx.x);
    if (idx >= num_units) return false;
    const int hb = a.q_heads * a.num_seqs;
    const int tile = row_tiles - 1 - idx / hb;
    u.h = (idx % hb) % a.q_heads;
    u.s = (idx % hb) / a.q_heads;
    u.kvh = u.h / a.group;
    const int n = seq_rows(a, u.s, &u.row0);
    u.q_lo = tile * kTile;
    u.rows = n - u.q_lo < kTile ? n - u.q_lo : kTile;  // <= 0: nothing to do
    u.cached = a.seq_lens[u.s];
    u.kv_len = u.cached + u.q_lo + u.rows;
    u.nt = u.rows > 0 ? (u.kv_len + kTile - 1) / kTile : 0;
    return true;
}

template <int D>
__global__ void __launch_bounds__(kPrefillThreads, TcCfg<D>::MIN_BLOCKS)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap,
                      const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap cmap,
                      const __grid_constant__ CUtensorMap smap, const PrefillArgs a,
                      int num_units, int row_tiles) {
    using Cfg = TcCfg<D>;
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + Cfg::OFF_BAR;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::OFF_BAR + NBARS * 8);
    volatile int* abort_flag =
        reinterpret_cast<volatile int*>(smem + Cfg::OFF_BAR + NBARS * 8 + 4);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };

    if ((sbase & 1023u) != 0) {  // the swizzle atoms need 1024-byte alignment
        if (tid == 0) atomicExch(&g_prefill_status, TMLLM_INVALID_ARGUMENT);
        return;
    }
    if (tid == 0) {
        mbar_init(bar(BAR_QL), 1);
        mbar_init(bar(BAR_Q), kSoftmaxThreads);
        mbar_init(bar(BAR_QE), 1);
        for (int st = 0; st < 2; ++st) {
            mbar_init(bar(BAR_KF + st), 1);
            mbar_init(bar(BAR_VF + st), 1);
            mbar_init(bar(BAR_KE + st), 1);
        }
        mbar_init(bar(BAR_S), 1);
        mbar_init(bar(BAR_F), kSoftmaxThreads);
        mbar_init(bar(BAR_P), kSoftmaxThreads);
        for (int ob = 0; ob < 2; ++ob) {
            mbar_init(bar(BAR_O + ob), 1);
            mbar_init(bar(BAR_E + ob), kSoftmaxThreads);
        }
        mbar_init(bar(BAR_RL), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // warp 0 owns the tensor-memory allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(Cfg::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_s = tmem;
    auto tmem_o = [&](int ob) { return tmem + 128u + static_cast<uint32_t>(ob * D); };
    const unsigned long long t0 = global_ns();
    constexpr unsigned FULL = 0xffffffffu;

    if (warp == 4) {
        // ================= producer: raw Q tiles and K/V pages by TMA =================
        const int box_rows = a.block_size < kTile ? a.block_size : kTile;
        const int nbox = kTile / box_rows;  // <= 8: pages are >= 16 positions
        const uint32_t box_bytes = static_cast<uint32_t>(box_rows) * 128u;
        // Every box of a tile is loaded: a box past the keys or without a page reads rows
        // beyond the arena, which TMA fills with zeros, so masked keys never meet stale
        // shared memory (P = 0 times a non-finite V would not be 0).
        const uint32_t tile_bytes = static_cast<uint32_t>(nbox) * box_bytes * Cfg::NB;
        bool ok = true;
        int g = 0, it = 0;
        int pv[2] = {0, 0};  // P V products issued into each O buffer by earlier units
        Unit u;
        for (int k = 0; ok && unit_of(a, k, num_units, row_tiles, u); ++k) {
            if (u.nt == 0) continue;
            if (lane == 0) {
                if (it > 0) ok = mbar_wait(bar(BAR_QE), (it - 1) & 1, abort_flag, t0);
                if (ok) mbar_arrive_tx(bar(BAR_QL), static_cast<uint32_t>(Cfg::TILE));
                // the RoPE rows go to the P buffer, free once the previous unit's last P V
                // (into the other O buffer) has completed
                if (ok && a.rope_tma) {
                    const int pb = (it & 1) ^ 1;
                    if (it > 0) ok = mbar_wait(bar(BAR_O + pb), (pv[pb] - 1) & 1, abort_flag, t0);
                    if (ok) {
                        mbar_arrive_tx(bar(BAR_RL), 2u * Cfg::BLK);
                        const int y = u.cached + u.q_lo + a.rope_off;
                        tma_load_2d(sbase + Cfg::OFF_P, &cmap, 0, y, bar(BAR_RL));
                        tma_load_2d(sbase + Cfg::OFF_P + Cfg::BLK, &smap, 0, y, bar(BAR_RL));
                    }
                }
            }
            ok = __shfl_sync(FULL, ok, 0);
            if (!ok) break;
            if (lane < Cfg::NB)
                tma_load_2d(sbase + Cfg::OFF_Q + lane * Cfg::BLK, &qmap, u.h * D + lane * 64,
                            u.row0 + u.q_lo, bar(BAR_QL));
            for (int j = 0; j < u.nt; ++j, ++g) {
                const int st = g & 1;
                // arena row of box `lane` of this tile (all block-table reads in flight)
                const int pos = j * kTile + lane * box_rows;
                const int64_t blk = (lane < nbox && pos < u.kv_len) ? page_of(a, u.s, pos) : -1;
                const int y = blk < 0 ? static_cast<int>(a.arena_rows)
                                      : static_cast<int>((blk * a.kv_heads + u.kvh) * a.block_size +
                                                         in_page(a, pos));
                if (lane == 0) {
                    if (g >= 2) ok = mbar_wait(bar(BAR_KE + st), ((g >> 1) - 1) & 1, abort_flag, t0);
                    if (ok) {
                        mbar_arrive_tx(bar(BAR_KF + st), tile_bytes);
                        mbar_arrive_tx(bar(BAR_VF + st), tile_bytes);
                    }
                }
                ok = __shfl_sync(FULL, ok, 0);
                if (!ok) break;
                if (lane < nbox) {
                    const uint32_t kdst = sbase + Cfg::OFF_K + st * Cfg::TILE + lane * box_bytes;
                    const uint32_t vdst = sbase + Cfg::OFF_V + st * Cfg::TILE + lane * box_bytes;
#pragma unroll
                    for (int c = 0; c < Cfg::NB; ++c) {
                        tma_load_2d(kdst + c * Cfg::BLK, &kmap, c * 64, y, bar(BAR_KF + st));
                        tma_load_2d(vdst + c * Cfg::BLK, &vmap, c * 64, y, bar(BAR_VF + st));
                    }
                }
            }
            pv[it & 1] += u.nt;
            ++it;
        }
    } else if (warp == 5) {
        // ================= MMA issuer (one lane) =================
        if (lane == 0) {
            constexpr uint32_t IDESC_QK = f16_idesc(128, 128, false);
            constexpr uint32_t IDESC_PV = f16_idesc(128, D, true);
            auto issue_qk = [&](int st) {
                const uint32_t qa = sbase + Cfg::OFF_Q, ka = sbase + Cfg::OFF_K + st * Cfg::TILE;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * Cfg::BLK + (kk & 3) * 32;
                    tc_mma(tmem_s, sw128_desc(qa + off, 16, 1024), sw128_desc(ka + off, 16, 1024),
                           IDESC_QK, kk > 0);
                }
            };
            auto issue_pv = [&](int st, bool acc, int ob) {
                const uint32_t pa = sbase + Cfg::OFF_P, va = sbase + Cfg::OFF_V + st * Cfg::TILE;
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk) {
                    const uint32_t aoff = (kk >> 2) * Cfg::BLK + (kk & 3) * 32;
                    tc_mma(tmem_o(ob), sw128_desc(pa + aoff, 16, 1024),
                           sw128_desc(va + kk * 2048, Cfg::BLK, 1024), IDESC_PV, acc || kk > 0);
                }
            };
            // Without RoPE in this kernel the raw Q tile is the operand, so its TMA barrier
            // (QL) is enough, and a unit's first Q K^T is issued during the previous unit's
            // last softmax (as soon as S is copied out), not after its P.
            const bool q_by_tma = a.rope_cos == nullptr;
            const int qbar = q_by_tma ? BAR_QL : BAR_Q;
            bool ok = true;
            int g = 0, it = 0;
            bool qk0_issued = false;  // the current unit's first Q K^T is already issued
            Unit u, nxt;
            int kn = 0;  // unit search position for the look-ahead
            auto next_unit = [&](int from, Unit& out) -> int {  // index of the next non-empty unit
                for (int kk = from; unit_of(a, kk, num_units, row_tiles, out); ++kk)
                    if (out.nt > 0) return kk;
                return -1;
            };
            for (int k = next_unit(0, u); ok && k >= 0; k = kn) {
                kn = next_unit(k + 1, nxt);
                if (!qk0_issued) {
                    // S is free: the previous tile's P arrived, which follows its S copy
                    ok = mbar_wait(bar(qbar), it & 1, abort_flag, t0) &&
                         mbar_wait(bar(BAR_KF + (g & 1)), (g >> 1) & 1, abort_flag, t0);
                    if (!ok) break;
                    tc_fence_after();
                    issue_qk(g & 1);
                    tc_commit(bar(BAR_S));
                }
                qk0_issued = false;
                for (int j = 0; j < u.nt; ++j, ++g) {
                    const int st = g & 1;
                    if (j + 1 < u.nt) {
                        // S_{g+1} = Q K^T as soon as the softmax warps hold S_g in
                        // registers, so it runs while they exponentiate tile g
                        ok = mbar_wait(bar(BAR_F), g & 1, abort_flag, t0) &&
                             mbar_wait(bar(BAR_KF + (st ^ 1)), ((g + 1) >> 1) & 1, abort_flag, t0);
                        if (!ok) break;
                        tc_fence_after();
                        issue_qk(st ^ 1);
                        tc_commit(bar(BAR_S));
                    } else {
                        tc_commit(bar(BAR_QE));  // the Q tile is free once these QKs finish
                        if (q_by_tma && kn >= 0) {  // the next unit's first Q K^T, early
                            ok = mbar_wait(bar(BAR_F), g & 1, abort_flag, t0) &&
                                 mbar_wait(bar(BAR_QL), (it + 1) & 1, abort_flag, t0) &&
                                 mbar_wait(bar(BAR_KF + (st ^ 1)), ((g + 1) >> 1) & 1, abort_flag, t0);
                            if (!ok) break;
                            tc_fence_after();
                            issue_qk(st ^ 1);
                            tc_commit(bar(BAR_S));
                            qk0_issued = true;
                        }
                    }
                    ok = mbar_wait(bar(BAR_P), g & 1, abort_flag, t0) &&
                         mbar_wait(bar(BAR_VF + st), (g >> 1) & 1, abort_flag, t0);
                    // this unit's O buffer was last used two units ago: free once that
                    // unit's epilogue has read it
                    if (ok && j == 0 && it >= 2)
                        ok = mbar_wait(bar(BAR_E + (it & 1)), ((it >> 1) - 1) & 1, abort_flag, t0);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv(st, j > 0, it & 1);
                    tc_commit(bar(BAR_O + (it & 1)));
                    tc_commit(bar(BAR_KE + st));
                }
                ++it;
                u = nxt;
            }
            // every MMA and its barrier arrivals done before the CTA releases its memory
            if (ok && g > 0) mbar_wait(bar(BAR_KE + ((g - 1) & 1)), ((g - 1) >> 1) & 1, abort_flag, t0);
        }
    } else {
        // ================= softmax warps: thread r owns query row r =================
        const int r = tid;
        const int half = D / 2;
        const uint32_t lane_s = tmem_s + (static_cast<uint32_t>(warp * 32) << 16);
        auto lane_o = [&](int ob) { return tmem_o(ob) + (static_cast<uint32_t>(warp * 32) << 16); };
        unsigned char* prow_s = smem + Cfg::OFF_P + r * 128;
        unsigned char* qrow_s = smem + Cfg::OFF_Q + r * 128;
        bool ok = true;
        int g = 0, it = 0;
        int pv[2] = {0, 0};  // P V products into each O buffer by earlier units
        // The epilogue of a unit runs after the first tile of the next one, so the wait for
        // its last P V and the next unit's first Q K^T overlap.  It needs the unit's output
        // rows, its O buffer and each row's sum l.
        Unit prev{};
        float l_prev = 0.f;
        bool has_prev = false;
        auto epilogue = [&](const Unit& e, float le, int ob) {
            const bool lv = r < e.rows;
            const float inv = 1.f / le;
            const int64_t orow = static_cast<int64_t>(e.row0 + e.q_lo + (lv ? r : 0)) *
                                     a.out_stride + static_cast<int64_t>(e.h) * D;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                float o[32];
                tmem_ld32(lane_o(ob) + c * 32, o);  // warp-wide: every lane loads, live rows store
                if (c == D / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(bar(BAR_E + ob));  // the unit after next may overwrite O_ob
                }
                if (!lv) continue;
                if (a.out_f32) {
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv,
                                             o[4 * i + 2] * inv, o[4 * i + 3] * inv);
                } else {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + orow + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t pk[4];
#pragma unroll
                        for (int e2 = 0; e2 < 4; ++e2) {
                            __half2 hv = __floats2half2_rn(o[8 * i + 2 * e2] * inv,
                                                           o[8 * i + 2 * e2 + 1] * inv);
                            pk[e2] = *reinterpret_cast<uint32_t*>(&hv);
                        }
                        dst[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    }
                }
            }
        };
        Unit u;
        for (int k = 0; ok && unit_of(a, k, num_units, row_tiles, u); ++k) {
            if (u.nt == 0) continue;
            const int ob = it & 1;
            const bool live = r < u.rows;
            const int qpos = u.cached + u.q_lo + (live ? r : u.rows - 1);  // keys 0..qpos
            // ---- Q: the raw tile arrives by TMA; with RoPE in this kernel each thread
            // rotates its row in place (without, the MMA warp uses the tile as it lands and
            // these warps never touch it)
            const int rpos = qpos + a.rope_off;
            const bool rope_here = a.rope_cos != nullptr;
            const bool rot = live && rope_here && rpos >= 0 && rpos < a.rope_len;
            if (rope_here) {
                ok = mbar_wait(bar(BAR_QL), it & 1, abort_flag, t0);
                ok = __all_sync(FULL, ok);
                if (!ok) break;
            }
            if (a.rope_tma) {  // the table rows of this unit, staged in the P buffer
                ok = mbar_wait(bar(BAR_RL), it & 1, abort_flag, t0);
                ok = __all_sync(FULL, ok);
                if (!ok) break;
            }
            if (rot) {
                const float* ct = a.rope_cos + static_cast<int64_t>(rpos) * half;
                const float* stb = a.rope_sin + static_cast<int64_t>(rpos) * half;
                const unsigned char* cst = smem + Cfg::OFF_P + r * 128;  // 32 floats, swizzled
                const unsigned char* sst = cst + Cfg::BLK;
#pragma unroll
                for (int c0 = 0; c0 < D / 16; c0 += 4) {  // chunk c pairs with chunk c + D/16
                    float cs[32], sn[32];
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        float4 cv, sv;
                        if (a.rope_tma) {
                            cv = *reinterpret_cast<const float4*>(cst + ((q4 ^ (r & 7)) << 4));
                            sv = *reinterpret_cast<const float4*>(sst + ((q4 ^ (r & 7)) << 4));
                        } else if (a.rope_vec) {
                            cv = __ldg(reinterpret_cast<const float4*>(ct + c0 * 8) + q4);
                            sv = __ldg(reinterpret_cast<const float4*>(stb + c0 * 8) + q4);
                        } else {
                            const float* cp = ct + c0 * 8 + 4 * q4;
                            const float* sp = stb + c0 * 8 + 4 * q4;
                            cv = make_float4(__ldg(cp), __ldg(cp + 1), __ldg(cp + 2), __ldg(cp + 3));
                            sv = make_float4(__ldg(sp), __ldg(sp + 1), __ldg(sp + 2), __ldg(sp + 3));
                        }
                        cs[4 * q4] = cv.x; cs[4 * q4 + 1] = cv.y; cs[4 * q4 + 2] = cv.z; cs[4 * q4 + 3] = cv.w;
                        sn[4 * q4] = sv.x; sn[4 * q4 + 1] = sv.y; sn[4 * q4 + 2] = sv.z; sn[4 * q4 + 3] = sv.w;
                    }
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int c = c0 + q4, c2 = c + D / 16;
                        uint4* p1 = reinterpret_cast<uint4*>(qrow_s + (c >> 3) * Cfg::BLK +
                                                             (((c & 7) ^ (r & 7)) << 4));
                        uint4* p2 = reinterpret_cast<uint4*>(qrow_s + (c2 >> 3) * Cfg::BLK +
                                                             (((c2 & 7) ^ (r & 7)) << 4));
                        uint4 u1 = *p1, u2 = *p2;
                        __half2* h1 = reinterpret_cast<__half2*>(&u1);
                        __half2* h2 = reinterpret_cast<__half2*>(&u2);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            // kernels/rope.metal:57-63 without contraction, two pairs at once:
                            // x1' = x1 c - x2 s, x2' = x2 c + x1 s (each product rounded)
                            const float2 f1 = __half22float2(h1[e]), f2 = __half22float2(h2[e]);
                            const int i0 = q4 * 8 + 2 * e;
                            const float2 c2v = make_float2(cs[i0], cs[i0 + 1]);
                            const float2 s2v = make_float2(sn[i0], sn[i0 + 1]);
                            const float2 m1 = __fmul2_rn(f2, s2v), m2 = __fmul2_rn(f1, s2v);
                            const float2 x = __fadd2_rn(__fmul2_rn(f1, c2v), make_float2(-m1.x, -m1.y));
                            const float2 y = __fadd2_rn(__fmul2_rn(f2, c2v), m2);
                            h1[e] = __floats2half2_rn(x.x, x.y);
                            h2[e] = __floats2half2_rn(y.x, y.y);
                        }
                        *p1 = u1;
                        *p2 = u2;
                    }
                }
            }
            if (rope_here) {
                fence_async_smem();
                mbar_arrive(bar(BAR_Q));
            }

            float m_used = -INFINITY, l = 0.f;
            for (int j = 0; j < u.nt; ++j, ++g) {
                ok = mbar_wait(bar(BAR_S), g & 1, abort_flag, t0);
                ok = __all_sync(FULL, ok);
                if (!ok) break;
                tc_fence_after();
                const int lim = qpos - j * kTile;  // columns 0..lim of this tile are visible
                float v[128];
                tmem_ld128(lane_s, v);
                tc_fence_before();
                mbar_arrive(bar(BAR_F));  // S may be overwritten by the next Q K^T
                // On the diagonal, invisible columns become -inf once: the maximum then
                // ignores them and their exponentials are exactly 0.  32-column chunks that
                // no row of the warp can see are skipped altogether (warp-uniform).
                const bool wfull = __all_sync(FULL, lim >= kTile - 1);
                if (!wfull) {
#pragma unroll
                    for (int i = 0; i < 128; ++i) v[i] = i <= lim ? v[i] : -INFINITY;
                }
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < 128; ++i) mx = fmaxf(mx, v[i]);
                const float mt = mx * a.scale_log2;
                // the previous P V done: the P buffer is free (and, within a unit, O settled);
                // on a unit's first tile that is the previous unit's last P V, in its buffer
                if (j > 0 || has_prev) {
                    const int wb = j > 0 ? ob : (ob ^ 1);
                    const int idx = j > 0 ? pv[ob] + j - 1 : pv[ob ^ 1] - 1;
                    ok = mbar_wait(bar(BAR_O + wb), idx & 1, abort_flag, t0);
                    ok = __all_sync(FULL, ok);
                    if (!ok) break;
                    tc_fence_after();
                }
                // Rescale only when the running maximum grew by more than 2^8; otherwise
                // keep the stale maximum (P stays below 2^8 and the final 1/l makes it
                // exact).  Tensor-memory accesses are warp-wide, so a warp rescales when
                // any of its rows needs it (alpha = 1 for the others).
                const bool need = j > 0 && mt > m_used + 8.f;
                float alpha = 1.f;
                if (need) {
                    alpha = fast_exp2(m_used - mt);
                    l *= alpha;
                    m_used = mt;
                }
                if (j == 0) m_used = mt;
                const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
                const float2 neg2 = make_float2(-m_used, -m_used);
                float2 l2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const bool dark = __all_sync(FULL, c * 32 > lim);
#pragma unroll
                    for (int gq = 0; gq < 4; ++gq) {  // 8 keys -> one 16-byte chunk of P
                        uint32_t pk[4] = {0u, 0u, 0u, 0u};
                        if (!dark) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int i0 = c * 32 + gq * 8 + 2 * e;
                                const float2 x = __ffma2_rn(make_float2(v[i0], v[i0 + 1]), sc2, neg2);
                                const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
                                l2 = __fadd2_rn(l2, p);
                                __half2 hp = __floats2half2_rn(p.x, p.y);
                                pk[e] = *reinterpret_cast<uint32_t*>(&hp);
                            }
                        }
                        const int cc = c * 4 + gq;  // chunk 0..15 along the keys
                        *reinterpret_cast<uint4*>(prow_s + (cc >> 3) * Cfg::BLK +
                                                  (((cc & 7) ^ (r & 7)) << 4)) =
                            make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    }
                }
                l += l2.x + l2.y;
                if (__any_sync(FULL, need)) {  // after the exponentials: fewer live registers
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        float o[32];
                        tmem_ld32(lane_o(ob) + c * 32, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(lane_o(ob) + c * 32, o);
                    }
                }
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(bar(BAR_P));
                if (j == 0 && has_prev) {  // the previous unit's O is final: write it out
                    epilogue(prev, l_prev, ob ^ 1);
                    has_prev = false;
                }
            }
            if (!ok) break;
            pv[ob] += u.nt;
            prev = u;
            l_prev = l;
            has_prev = true;
            ++it;
        }
        if (ok && has_prev) {  // the last unit: wait for its last P V, then write it out
            const int ob = (it - 1) & 1;
            ok = mbar_wait(bar(BAR_O + ob), (pv[ob] - 1) & 1, abort_flag, t0);
            ok = __all_sync(FULL, ok);
            if (ok) {
                tc_fence_after();
                epilogue(prev, l_prev, ob);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(Cfg::TMEM_COLS)
                     : "memory");
    }
}

// ---- CUDA-core prefill: one warp per (query row, query head) ---------------------------
template <typename T>
__global__ void __launch_bounds__(128) prefill_generic_kernel(const PrefillArgs a) {
    constexpr int MAXP = 8;  // rotation pairs per lane: head_dim <= 512
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= a.total_rows * a.q_heads) return;
    const int h = warp % a.q_heads;
    const int row = warp / a.q_heads;
    const int s = seq_of_row(a, row);
    int row0;
    seq_rows(a, s, &row0);
    const int qpos = a.seq_lens[s] + (row - row0);
    const int D = a.head_dim, half = D / 2, kvh = h / a.group;
    float q1[MAXP], q2[MAXP], o1[MAXP], o2[MAXP];
    const T* qr = static_cast<const T*>(a.q) + static_cast<int64_t>(row) * a.q_stride +
                  static_cast<int64_t>(h) * D;
#pragma unroll
    for (int k = 0; k < MAXP; ++k) {
        const int i = lane + 32 * k;
        q1[k] = q2[k] = o1[k] = o2[k] = 0.f;
        if (i < half) {
            float x1 = to_f32<T>(qr[i]), x2 = to_f32<T>(qr[i + half]);
            rope_rotate(a, qpos + a.rope_off, i, half, x1, x2);
            q1[k] = round_store<T>(x1);
            q2[k] = round_store<T>(x2);
        }
    }
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j <= qpos; ++j) {
        const int64_t blk = page_of(a, s, j);
        if (blk < 0) continue;
        const int64_t off = ((blk * a.kv_heads + kvh) * a.block_size + in_page(a, j)) * D;
        const T* kr = static_cast<const T*>(a.k_cache) + off;
        const T* vr = static_cast<const T*>(a.v_cache) + off;
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < MAXP; ++k) {
            const int i = lane + 32 * k;
            if (i < half) dot += q1[k] * to_f32<T>(kr[i]) + q2[k] * to_f32<T>(kr[i + half]);
        }
        dot = warp_sum(dot) * a.scale_log2;
        const float mn = fmaxf(m, dot);
        const float corr = exp2f(m - mn), p = exp2f(dot - mn);
        l = l * corr + p;
        m = mn;
#pragma unroll
        for (int k = 0; k < MAXP; ++k) {
            const int i = lane + 32 * k;
            if (i < half) {
                o1[k] = o1[k] * corr + p * to_f32<T>(vr[i]);
                o2[k] = o2[k] * corr + p * to_f32<T>(vr[i + half]);
            }
        }
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t orow = static_cast<int64_t>(row) * a.out_stride + static_cast<int64_t>(h) * D;
#pragma unroll
    for (int k = 0; k < MAXP; ++k) {
        const int i = lane + 32 * k;
        if (i >= half) continue;
        if (a.out_f32) {
            static_cast<float*>(a.out)[orow + i] = o1[k] * inv;
            static_cast<float*>(a.out)[orow + i + half] = o2[k] * inv;
        } else {
            static_cast<T*>(a.out)[orow + i] = from_f32<T>(o1[k] * inv);
            static_cast<T*>(a.out)[orow + i + half] = from_f32<T>(o2[k] * inv);
        }
    }
}

// ---- host ----------------------------------------------------------------------------
}  // namespace

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        cudaGetLastError();
    });
    return fn;
}

// 2-D map over `rows` rows of `inner` elements, `row_bytes` apart; boxes of 128 bytes (64 F16
// or 32 F32 columns) x box_rows rows with the 128-byte swizzle (the layout the tensor-core
// descriptors read).
int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t row_bytes,
             int box_rows, bool f32) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return fail(TMLLM_DEVICE_ERROR, "cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {f32 ? 32u : 64u, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     2, const_cast<void*>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(TMLLM_DEVICE_ERROR, "tensor map encoding failed (CUresult %d)",
                    static_cast<int>(r));
    return TMLLM_OK;
}

namespace {

template <int D>
int launch_tc(const PrefillArgs& a, int64_t arena_rows, int max_rows, cudaStream_t s) {
    using Cfg = TcCfg<D>;
    const int box_rows = a.block_size < kTile ? a.block_size : kTile;
    CUtensorMap kmap, vmap, qmap;
    if (int st = make_map(&kmap, a.k_cache, D, arena_rows, D * 2, box_rows)) return st;
    if (int st = make_map(&vmap, a.v_cache, D, arena_rows, D * 2, box_rows)) return st;
    if (int st = make_map(&qmap, a.q, static_cast<int64_t>(a.q_heads) * D, a.total_rows,
                          a.q_stride * 2, kTile))
        return st;
    CUtensorMap cmap = qmap, smap = qmap;  // placeholders when the tables are not staged
    if (a.rope_tma) {
        if (int st = make_map(&cmap, a.rope_cos, D / 2, a.rope_len, D * 2, kTile, true)) return st;
        if (int st = make_map(&smap, a.rope_sin, D / 2, a.rope_len, D * 2, kTile, true)) return st;
    }
    // the shared-memory opt-in once per device (bit d of the mask; retried after a failure)
    static std::atomic<uint64_t> opted{0};
    int dev = 0;
    TMLLM_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (!bit || !(opted.load(std::memory_order_relaxed) & bit)) {
        TMLLM_CUDA_TRY(cudaFuncSetAttribute(prefill_tc_kernel<D>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            Cfg::SMEM));
        opted.fetch_or(bit, std::memory_order_relaxed);
    }
    const int row_tiles = (max_rows + kTile - 1) / kTile;
    const int64_t units = static_cast<int64_t>(row_tiles) * a.q_heads * a.num_seqs;
    if (units > INT32_MAX) return fail(TMLLM_INVALID_SHAPE, "too many prefill tiles");
    int64_t ctas = static_cast<int64_t>(device_sm_count()) * Cfg::MIN_BLOCKS;
    if (ctas > units) ctas = units;
    prefill_tc_kernel<D><<<static_cast<unsigned>(ctas), kPrefillThreads, Cfg::SMEM, s>>>(
        kmap, vmap, qmap, cmap, smap, a, static_cast<int>(units), row_tiles);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

}  // namespace

int prefill_impl(const tmllm_paged_kv* kv, const void* q, const void* k_new, const void* v_new,
                 const int32_t* q_start, int32_t rows_per_seq, int32_t max_rows,
                 int32_t total_rows, void* out, int32_t q_heads, const tmllm_decode_opts* opts,
                 cudaStream_t stream) {
    if (!kv) return fail(TMLLM_INVALID_ARGUMENT, "null paged KV descriptor");
    if (!valid_dtype(kv->dtype)) return fail(TMLLM_UNSUPPORTED_DTYPE, "unknown cache dtype");
    const int D = kv->head_dim, Hkv = kv->num_kv_heads, B = kv->num_seqs;
    if (B <= 0 || Hkv <= 0 || D <= 0 || kv->block_size <= 0 || kv->max_blocks_per_seq <= 0 ||
        kv->num_blocks <= 0)
        return fail(TMLLM_INVALID_SHAPE, "paged KV dimensions must be positive");
    if (D % 2 != 0 || D > 512)
        return fail(TMLLM_INVALID_SHAPE, "head_dim must be even and <= 512, got %d", D);
    if (q_heads <= 0 || q_heads % Hkv != 0)
        return fail(TMLLM_MODEL_FORMAT, "Q heads %d must be divisible by non-zero KV heads %d",
                    q_heads, Hkv);
    if (rows_per_seq < 0 || max_rows < 0 || total_rows < 0)
        return fail(TMLLM_INVALID_SHAPE, "row counts must be non-negative");
    if (!q_start) {
        int64_t tot;
        if (!mul_ok(rows_per_seq, B, &tot) || tot > INT32_MAX)
            return fail(TMLLM_INVALID_SHAPE, "total rows exceed i32");
        total_rows = static_cast<int32_t>(tot);
        max_rows = rows_per_seq;
    }
    if (total_rows == 0 || max_rows == 0) return TMLLM_OK;
    if ((k_new == nullptr) != (v_new == nullptr))
        return fail(TMLLM_INVALID_ARGUMENT, "k_new and v_new must both be given or both be NULL");
    if (!q || !out || !kv->k_cache || !kv->v_cache || !kv->block_table || !kv->seq_lens)
        return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    tmllm_decode_opts o{};
    if (opts) o = *opts;
    if (o.variant < 0 || o.variant > 2)
        return fail(TMLLM_INVALID_ARGUMENT, "unknown prefill variant %d", o.variant);
    if (o.out_f32 != 0 && o.out_f32 != 1)
        return fail(TMLLM_INVALID_ARGUMENT, "out_f32 must be 0 or 1");
    if (o.rope_cos && (!o.rope_sin || o.rope_len <= 0))
        return fail(TMLLM_INVALID_ARGUMENT, "RoPE needs both tables and a positive length");
    const float scale = o.scale > 0.f ? o.scale : 1.0f / sqrtf(static_cast<float>(D));
    if (!std::isfinite(scale))
        return fail(TMLLM_INVALID_SHAPE, "attention scale must be positive and finite");
    if (o.q_seq_stride < 0 || o.kv_seq_stride < 0 ||
        (o.q_seq_stride > 0 && o.q_seq_stride < static_cast<int64_t>(q_heads) * D) ||
        (o.kv_seq_stride > 0 && o.kv_seq_stride < static_cast<int64_t>(Hkv) * D))
        return fail(TMLLM_INVALID_SHAPE, "row strides of q / k_new must cover a row");
    const size_t es = dtype_size(kv->dtype);
    auto misaligned = [es](const void* p) { return (reinterpret_cast<uintptr_t>(p) % es) != 0; };
    if (misaligned(kv->k_cache) || misaligned(kv->v_cache) || misaligned(q) ||
        (k_new && misaligned(k_new)) || (v_new && misaligned(v_new)) || misaligned(out))
        return fail(TMLLM_INVALID_ARGUMENT, "tensor pointers must be aligned to their element size");

    int bs_shift = -1;
    if ((kv->block_size & (kv->block_size - 1)) == 0) {
        bs_shift = 0;
        while ((1 << bs_shift) < kv->block_size) ++bs_shift;
    }
    PrefillArgs a{};
    a.q = q;
    a.k_new = k_new;
    a.v_new = v_new;
    a.k_cache = kv->k_cache;
    a.v_cache = kv->v_cache;
    a.out = out;
    a.block_table = kv->block_table;
    a.seq_lens = kv->seq_lens;
    a.q_start = q_start;
    a.rope_cos = o.rope_cos;
    a.rope_sin = o.rope_sin;
    a.num_blocks = kv->num_blocks;
    a.q_stride = o.q_seq_stride > 0 ? o.q_seq_stride : static_cast<int64_t>(q_heads) * D;
    a.kv_stride = o.kv_seq_stride > 0 ? o.kv_seq_stride : static_cast<int64_t>(Hkv) * D;
    a.out_stride = static_cast<int64_t>(q_heads) * D;
    a.uniform_rows = rows_per_seq;
    a.num_seqs = B;
    a.total_rows = total_rows;
    a.q_heads = q_heads;
    a.kv_heads = Hkv;
    a.group = q_heads / Hkv;
    a.head_dim = D;
    a.block_size = kv->block_size;
    a.bs_shift = bs_shift;
    a.max_blocks = kv->max_blocks_per_seq;
    a.rope_len = o.rope_len;
    a.rope_off = o.rope_pos_offset;
    a.out_f32 = o.out_f32 || kv->dtype == TMLLM_F32;
    a.rope_vec = o.rope_cos && aligned16(o.rope_cos) && aligned16(o.rope_sin) && (D / 2) % 4 == 0;
    a.rope_tma = a.rope_vec && D == 64 && kv->dtype == TMLLM_F16;
    a.scale_log2 = scale * kLog2eP;

    // the attention path, decided before anything is enqueued
    int64_t arena_rows = 0;
    const bool rows_fit = mul_ok(kv->num_blocks, static_cast<int64_t>(Hkv) * kv->block_size,
                                 &arena_rows) && arena_rows <= INT32_MAX - kTile;
    const bool tc_shape = kv->dtype == TMLLM_F16 && (D == 64 || D == 128) && bs_shift >= 4 &&
                          rows_fit && aligned16(kv->k_cache) && aligned16(kv->v_cache) &&
                          aligned16(q) && aligned16(out) && (a.q_stride % 8) == 0 &&
                          o.variant != 1;
    if (o.variant == 2 && !tc_shape)
        return fail(TMLLM_INVALID_ARGUMENT,
                    "the tensor-core prefill needs F16, head_dim 64/128, power-of-two pages of "
                    ">= 16 positions and 16-byte aligned q/out/arenas");
    // 1. append (rotated keys, values) at each sequence's cached length.  On the tensor-core
    // path with RoPE and an F16 output, the query rows are rotated here as well, into the
    // output buffer: each unit of the attention kernel reads its own q rows from there (by
    // TMA, already rotated) before it overwrites them with its result.
    const bool pre_rotate = tc_shape && o.rope_cos != nullptr && !a.out_f32;
    {
        const int epc = static_cast<int>(16 / es);
        const bool vec = (D / 2) % epc == 0 && aligned16(kv->k_cache) && aligned16(kv->v_cache) &&
                         (!k_new || (aligned16(k_new) && aligned16(v_new) &&
                                     (a.kv_stride * static_cast<int64_t>(es)) % 16 == 0));
        auto grid_for = [&](int64_t work) {
            int64_t blocks = (work + 255) / 256;
            const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
            if (blocks > cap) blocks = cap;
            return static_cast<unsigned>(blocks < 1 ? 1 : blocks);
        };
        PrefillArgs ap = a;
        if (k_new && !vec) {  // scalar append of K and V, then (if asked) the q rotation
            const unsigned nb = grid_for(static_cast<int64_t>(total_rows) * Hkv * (D / 2));
            if (kv->dtype == TMLLM_F16)
                prefill_append_kernel<__half><<<nb, 256, 0, stream>>>(a);
            else
                prefill_append_kernel<float><<<nb, 256, 0, stream>>>(a);
            TMLLM_LAUNCH_TRY();
            ap.k_new = ap.v_new = nullptr;
        }
        ap.q_rot = pre_rotate ? out : nullptr;
        if (ap.k_new || ap.q_rot) {
            const int64_t heads = (ap.k_new ? Hkv : 0) + (ap.q_rot ? q_heads : 0);
            const unsigned nb = grid_for(static_cast<int64_t>(total_rows) * heads * (D / 2) / epc);
            if (kv->dtype == TMLLM_F16)
                prefill_append_vec_kernel<__half><<<nb, 256, 0, stream>>>(ap);
            else
                prefill_append_vec_kernel<float><<<nb, 256, 0, stream>>>(ap);
            TMLLM_LAUNCH_TRY();
        }
    }
    if (pre_rotate) {  // the attention kernel reads the rotated rows, without RoPE
        a.q = out;
        a.q_stride = static_cast<int64_t>(q_heads) * D;
        a.rope_cos = a.rope_sin = nullptr;
        a.rope_vec = a.rope_tma = 0;
    }
    // 2. attention over the cache, new rows included
    if (tc_shape) {
        a.arena_rows = arena_rows;
        const int64_t ctas = static_cast<int64_t>(q_heads) * B;
        if (ctas > INT32_MAX) return fail(TMLLM_INVALID_SHAPE, "too many sequences x heads");
        return D == 64 ? launch_tc<64>(a, arena_rows, max_rows, stream)
                       : launch_tc<128>(a, arena_rows, max_rows, stream);
    }
    const int64_t warps = static_cast<int64_t>(total_rows) * q_heads;
    if (warps > INT32_MAX) return fail(TMLLM_INVALID_SHAPE, "too many rows x heads");
    const unsigned blocks = static_cast<unsigned>((warps + 3) / 4);
    if (kv->dtype == TMLLM_F16)
        prefill_generic_kernel<__half><<<blocks, 128, 0, stream>>>(a);
    else
        prefill_generic_kernel<float><<<blocks, 128, 0, stream>>>(a);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}


}  // namespace tmllm

using namespace tmllm;

extern "C" {

int tmllm_gqa_prefill(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                      const void* v_new, const int32_t* q_start, int32_t rows_per_seq,
                      int32_t max_rows, int32_t total_rows, void* out, int32_t q_heads,
                      const tmllm_decode_opts* opts, tmllm_stream stream) {
    clear_error();
    return prefill_impl(kv, q, k_new, v_new, q_start, rows_per_seq, max_rows, total_rows, out,
                        q_heads, opts, reinterpret_cast<cudaStream_t>(stream));
}

int tmllm_prefill_status(int32_t* status) {
    clear_error();
    if (!status) return fail(TMLLM_INVALID_ARGUMENT, "null status pointer");
    int v = 0, zero = 0;
    TMLLM_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_prefill_status, sizeof(int)));
    TMLLM_CUDA_TRY(cudaMemcpyToSymbol(g_prefill_status, &zero, sizeof(int)));
    *status = v;
    return TMLLM_OK;
}

}  // extern "C"
