// Shared host/device helpers of libtmllm_b200.so: status handling, dtype helpers,
// 16-byte vector moves and cp.async wrappers for sm_100a.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <initializer_list>

#include "tmllm.h"

namespace tmllm {

// Records a formatted message for tmllm_last_error() and returns `status`.
int fail(int status, const char* fmt, ...);
// Records a CUDA runtime error and returns TMLLM_DEVICE_ERROR.
int cuda_fail(cudaError_t err, const char* what);
// Clears the calling thread's last error (message and fields).
void clear_error();
// TinyError::PositionOutOfRange {start_pos, seq_len, max_seq_len}: records the fields and
// the reference's message, returns TMLLM_POSITION_OUT_OF_RANGE.
int fail_position(int64_t start_pos, int64_t seq_len, int64_t max_seq_len);
// TinyError::ShapeMismatch {left, right}: records both shapes (up to TMLLM_MAX_RANK dims
// each) and a message, returns TMLLM_SHAPE_MISMATCH.
int fail_shapes(std::initializer_list<int64_t> left, std::initializer_list<int64_t> right,
                const char* fmt, ...);

inline bool valid_dtype(int dt) { return dt == TMLLM_F32 || dt == TMLLM_F16; }
inline size_t dtype_size(int dt) { return dt == TMLLM_F16 ? 2u : 4u; }
inline const char* dtype_name(int dt) { return dt == TMLLM_F16 ? "F16" : "F32"; }

// a*b with overflow detection (true when the product fits in int64 and is >= 0).
inline bool mul_ok(int64_t a, int64_t b, int64_t* out) {
    if (a < 0 || b < 0) return false;
    if (a != 0 && b > INT64_MAX / a) return false;
    *out = a * b;
    return true;
}
// Product of a list of non-negative sizes with overflow detection.
bool checked_numel(std::initializer_list<size_t> dims, int64_t* out);

// Number of SMs of the current device (cached per device ordinal).
int device_sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Cross-GPU exchange of a sequence split (device-resident; see exchange.cu).  Every rank
// owns one buffer of 8-byte cells {F32 value bits, step number}:
//   recv_o   [2 parities][world][rows][head_dim]   normalised partial outputs
//   recv_lse [2 parities][world][rows]             their natural-log log-sum-exp
// plus a status word (TMLLM_TIMEOUT after an expired wait), and holds device pointers to
// every rank's buffer.  A cell is written with one 8-byte store, so a reader that sees the
// current step number in a cell also sees its value: no fences or flags are needed.
constexpr int kMaxRanks = 8;
struct ExchangeArgs {
    uint2* recv_o[kMaxRanks];
    uint2* recv_lse[kMaxRanks];
    int* status;
    unsigned long long timeout_ns;
    int32_t rank, world, rows, groups, head_dim, pad;
};

}  // namespace tmllm

#define TMLLM_CUDA_TRY(expr)                                          \
    do {                                                              \
        cudaError_t tmllm_e_ = (expr);                                \
        if (tmllm_e_ != cudaSuccess) return ::tmllm::cuda_fail(tmllm_e_, #expr); \
    } while (0)

#define TMLLM_LAUNCH_TRY()                                            \
    do {                                                              \
        cudaError_t tmllm_e_ = cudaGetLastError();                    \
        if (tmllm_e_ != cudaSuccess) return ::tmllm::cuda_fail(tmllm_e_, "kernel launch"); \
    } while (0)

// ---- device helpers -------------------------------------------------------------------

namespace tmllm {

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Storage rounding: identity for F32, round-trip through binary16 for F16.
template <typename T> __device__ __forceinline__ float round_store(float x) {
    return to_f32<T>(from_f32<T>(x));
}

// 16-byte asynchronous global->shared copy; src_bytes == 0 zero-fills the destination
// without reading `src` (which must still be a valid address).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, int src_bytes) {
    unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem_src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Unpacks a 16-byte chunk into floats (8 halves or 4 floats).
template <typename T> struct Chunk;
template <> struct Chunk<__half> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
        const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 v = __half22float2(h[i]);
            f[2 * i] = v.x;
            f[2 * i + 1] = v.y;
        }
    }
};
template <> struct Chunk<float> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
        f[0] = __uint_as_float(r.x);
        f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z);
        f[3] = __uint_as_float(r.w);
    }
};

// Warp-level tensor-core helpers (ldmatrix, mma.sync m16n8k16 with F16 inputs and F32
// accumulators), shared by the decode kernel and the decoder's linear layers.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Programmatic dependent launch: a kernel launched with programmatic stream serialisation
// may start before the kernel ahead of it on the stream has finished; griddepcontrol.wait
// blocks until that kernel has completed and its writes are visible (immediately when
// there is no such dependency), launch_dependents lets the next such kernel start early.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace tmllm
