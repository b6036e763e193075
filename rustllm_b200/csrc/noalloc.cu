// Allocation-free form of the fused decode (tmllm_gqa_decode_noalloc).
//
// Some callers cannot call cudaMalloc at decode time: code running inside a CUDA stream
// capture that must not add allocation nodes, embedders whose memory is handed out by a
// pool they do not control, real-time loops that may not take the allocator's locks, and
// plug-in hosts that forbid a library from owning device memory at all.  For them the
// split-K scratch of the decode kernel lives in a fixed array compiled into this library.
//
// Facts a caller relies on:
//  * The array is TMLLM_NOALLOC_SCRATCH_BYTES (2 MiB) of device memory, created when the
//    library is loaded on a GPU and held until the process exits, on every GPU that loads
//    the library, whether or not this entry point is used.
//  * In host code the array's name is only a stand-in for the symbol, not a device
//    address.  The first call on each device (with that device current) looks up the real
//    address with cudaGetSymbolAddress and remembers it; make that first call before any
//    stream capture.
//  * Every call uses the same array and it keeps whatever the previous call left there.
//    When the call uses split-K, the ticket counters the kernel needs at zero are cleared
//    (cudaMemsetAsync, no allocation) on the caller's stream right before the launch, after
//    every argument check: a rejected call enqueues nothing.  Two calls whose work overlaps
//    on the GPU (different streams, or different host threads on the same device) race on
//    the array and produce wrong results; serialise them.
//  * A call whose split-K partials would not fit in the array is rejected before anything
//    is enqueued, with TMLLM_INVALID_SHAPE and a message naming the limit.
#include <mutex>

#include "common.cuh"

namespace tmllm {
int decode_impl_ex(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                   const void* v_new, void* out, float* lse, int32_t q_heads,
                   const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                   int64_t max_len_hint, const ExchangeArgs* ex, uint32_t epoch,
                   bool clear_tickets, cudaStream_t stream, int64_t chunk_override = 0);
size_t decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t splits);
int32_t decode_auto_splits(int64_t B, int64_t Hkv, int64_t max_len);
}  // namespace tmllm

using namespace tmllm;

static __device__ __align__(256) unsigned char g_noalloc_scratch[TMLLM_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    TMLLM_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(TMLLM_DEVICE_ERROR, "device ordinal %d outside the supported range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        TMLLM_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        if (p == nullptr) return fail(TMLLM_DEVICE_ERROR, "scratch array has no device address");
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return TMLLM_OK;
}

}  // namespace

extern "C" int tmllm_gqa_decode_noalloc(const tmllm_paged_kv* kv, const void* q,
                                        const void* k_new, const void* v_new, void* out,
                                        float* lse, int32_t q_heads,
                                        const tmllm_decode_opts* opts, tmllm_stream stream) {
    clear_error();
    if (!kv) return fail(TMLLM_INVALID_ARGUMENT, "null paged KV descriptor");
    if (kv->num_seqs <= 0 || kv->num_kv_heads <= 0 || kv->head_dim <= 0 || q_heads <= 0 ||
        kv->block_size <= 0 || kv->max_blocks_per_seq <= 0)
        return fail(TMLLM_INVALID_SHAPE, "paged KV dimensions must be positive");
    // Fix the split count here so the scratch size checked below is the one the kernel uses.
    tmllm_decode_opts o{};
    if (opts) o = *opts;
    int64_t capacity = static_cast<int64_t>(kv->block_size) * kv->max_blocks_per_seq;
    int64_t hint = o.max_len_hint > 0 && o.max_len_hint < capacity ? o.max_len_hint : capacity;
    if (o.num_splits <= 0) o.num_splits = decode_auto_splits(kv->num_seqs, kv->num_kv_heads, hint);
    if (o.num_splits > 1024) o.num_splits = 1024;
    const size_t need = decode_workspace_bytes(kv->num_seqs, q_heads, kv->num_kv_heads,
                                               kv->head_dim, o.num_splits);
    if (need > static_cast<size_t>(TMLLM_NOALLOC_SCRATCH_BYTES))
        return fail(TMLLM_INVALID_SHAPE,
                    "this decode needs %zu bytes of split scratch (%d sequences, %d query heads, "
                    "head_dim %d, %d splits) but the built-in scratch holds %d bytes; use "
                    "tmllm_gqa_decode with a workspace, or fewer splits",
                    need, kv->num_seqs, q_heads, kv->head_dim, o.num_splits,
                    TMLLM_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    if (int st = scratch_address(&scratch)) return st;
    // The ticket counters sit at the start of the scratch and must be zero at launch: the
    // decode clears them itself once every argument has been checked (never with a single
    // split, where no ticket is taken and `need` covers no counters).
    return decode_impl_ex(kv, q, k_new, v_new, out, lse, q_heads, &o, scratch,
                          static_cast<size_t>(TMLLM_NOALLOC_SCRATCH_BYTES), o.max_len_hint,
                          nullptr, 0, true, reinterpret_cast<cudaStream_t>(stream));
}
