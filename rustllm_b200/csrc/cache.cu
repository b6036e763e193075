// Paged KV cache runtime: block pool, per-sequence block tables and lengths, K/V arenas
// per layer, append / gather kernels and the cache-owned decode workspace.
//
// The reference keeps one contiguous [1, Hkv, max_seq, D] buffer per layer and a host-side
// length (src/model/kv_cache.rs:9-184).  Here every layer has a K and a V arena of
// fixed-size blocks [num_blocks, Hkv, block_size, D]; all layers of a sequence share one
// block table, so a block id addresses the same positions in every layer.  The host owns
// the truth (lengths, tables, free list) and mirrors tables and lengths to the device with
// small kernels enqueued on the caller's stream, so no host buffer is read asynchronously.
#include <algorithm>
#include <cstring>
#include <random>
#include <vector>

#include "common.cuh"

namespace tmllm {
int decode_impl(const tmllm_paged_kv* kv, const void* q, const void* k_new, const void* v_new,
                void* out, float* lse, int32_t q_heads, const tmllm_decode_opts* opts,
                void* workspace, size_t workspace_bytes, int64_t max_len_hint,
                cudaStream_t stream);
size_t decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t splits);
int32_t decode_auto_splits(int64_t B, int64_t Hkv, int64_t max_len);
int64_t decode_auto_chunk_lens(const int64_t* lens, int64_t B, int64_t Hkv, int64_t hint,
                               int per_sm);
int decode_impl_ex(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                   const void* v_new, void* out, float* lse, int32_t q_heads,
                   const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                   int64_t max_len_hint, const ExchangeArgs* ex, uint32_t epoch,
                   bool clear_tickets, cudaStream_t stream, int64_t chunk_override = 0);
int decode_resident_ctas(int dtype, int head_dim, int variant, int group);
int prefill_impl(const tmllm_paged_kv* kv, const void* q, const void* k_new, const void* v_new,
                 const int32_t* q_start, int32_t rows_per_seq, int32_t max_rows,
                 int32_t total_rows, void* out, int32_t q_heads, const tmllm_decode_opts* opts,
                 cudaStream_t stream);

namespace {

constexpr int kTableBatch = 32;
struct TableEntries {
    int32_t v[kTableBatch];
};

__global__ void set_entries_kernel(int32_t* dst, TableEntries e, int n) {
    if (threadIdx.x < n) dst[threadIdx.x] = e.v[threadIdx.x];
}

__global__ void fill_i32_kernel(int32_t* dst, int32_t value, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = value;
}

__global__ void add_lens_kernel(int32_t* lens, int first, int count, int32_t n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) lens[first + i] += n;
}

// Paged write/read of [Hkv, n, D] rows of one sequence at positions [start, start+n).
// kWrite: dense -> arena (LayerKvCache::append's kv_cache_write, kv_cache_write.metal:13-18
// with the paged address); !kWrite: arena -> dense (key()/value() + contiguous()).
template <typename V, bool kWrite>
__global__ void paged_rows_kernel(unsigned char* __restrict__ k_arena,
                                  unsigned char* __restrict__ v_arena,
                                  const int32_t* __restrict__ table, int64_t max_blocks,
                                  int32_t block_size, int32_t kv_heads, int64_t row_bytes,
                                  int64_t num_blocks, int seq, int64_t start, int64_t n,
                                  unsigned char* __restrict__ k_dense,
                                  unsigned char* __restrict__ v_dense) {
    const int64_t rv = row_bytes / static_cast<int64_t>(sizeof(V));
    const int64_t total = static_cast<int64_t>(kv_heads) * n * rv;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = i % rv, row = i / rv;
        const int64_t s = row % n, h = row / n;
        const int64_t pos = start + s;
        const int64_t bi = pos / block_size;
        if (bi >= max_blocks) continue;
        const int64_t blk = table[static_cast<int64_t>(seq) * max_blocks + bi];
        if (blk < 0 || blk >= num_blocks) continue;
        const int64_t aoff = ((blk * kv_heads + h) * block_size + pos % block_size) * row_bytes;
        const int64_t doff = (h * n + s) * row_bytes;
        V* ka = reinterpret_cast<V*>(k_arena + aoff);
        V* va = reinterpret_cast<V*>(v_arena + aoff);
        if (kWrite) {
            if (k_dense) ka[c] = reinterpret_cast<const V*>(k_dense + doff)[c];
            if (v_dense) va[c] = reinterpret_cast<const V*>(v_dense + doff)[c];
        } else {
            if (k_dense) reinterpret_cast<V*>(k_dense + doff)[c] = ka[c];
            if (v_dense) reinterpret_cast<V*>(v_dense + doff)[c] = va[c];
        }
    }
}

int grid_for(int64_t total) {
    int64_t blocks = (total + 255) / 256;
    int64_t cap = static_cast<int64_t>(device_sm_count()) * 32;
    return static_cast<int>(std::max<int64_t>(1, std::min(blocks, cap)));
}

// Makes `device` current for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != device) ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace
}  // namespace tmllm

using namespace tmllm;

struct tmllm_cache {
    tmllm_cache_config cfg{};
    int64_t num_blocks = 0;
    int32_t max_blocks = 0;   // per sequence
    int64_t layer_bytes = 0;  // one arena (K or V) of one layer
    unsigned char* arena = nullptr;
    int32_t* d_table = nullptr;
    int32_t* d_lens = nullptr;
    std::vector<int32_t> h_table;   // [num_seqs * max_blocks], -1 = none
    std::vector<int64_t> h_lens;    // [num_seqs]
    std::vector<int32_t> h_nblk;    // blocks held per sequence
    std::vector<int32_t> free_ids;  // pool, handed out from the back
    void* ws = nullptr;
    size_t ws_bytes = 0;

    unsigned char* k_layer(int l) const { return arena + static_cast<int64_t>(2 * l) * layer_bytes; }
    unsigned char* v_layer(int l) const {
        return arena + static_cast<int64_t>(2 * l + 1) * layer_bytes;
    }
    int64_t row_bytes() const { return static_cast<int64_t>(cfg.head_dim) * dtype_size(cfg.dtype); }
};

namespace {

int check_cache(const tmllm_cache* c) {
    if (!c) return fail(TMLLM_INVALID_ARGUMENT, "null cache handle");
    return TMLLM_OK;
}
int check_seq(const tmllm_cache* c, int32_t seq) {
    if (seq < 0 || seq >= c->cfg.num_seqs)
        return fail(TMLLM_INVALID_ARGUMENT, "sequence %d does not exist (num_seqs %d)", seq,
                    c->cfg.num_seqs);
    return TMLLM_OK;
}
int check_layer(const tmllm_cache* c, int32_t layer) {
    if (layer < 0 || layer >= c->cfg.num_layers)  // KvCache::layer_mut, kv_cache.rs:165-169
        return fail(TMLLM_MODEL_FORMAT, "KV cache layer %d does not exist", layer);
    return TMLLM_OK;
}

// Uploads table entries [first, first+count) of sequence `seq`.
int upload_entries(tmllm_cache* c, int32_t seq, int32_t first, int32_t count, cudaStream_t s) {
    if (count <= 0) return TMLLM_OK;
    int32_t* dst = c->d_table + static_cast<int64_t>(seq) * c->max_blocks + first;
    const int32_t* src = c->h_table.data() + static_cast<int64_t>(seq) * c->max_blocks + first;
    if (count <= kTableBatch) {
        TableEntries e{};
        std::memcpy(e.v, src, sizeof(int32_t) * count);
        set_entries_kernel<<<1, kTableBatch, 0, s>>>(dst, e, count);
        TMLLM_LAUNCH_TRY();
        return TMLLM_OK;
    }
    // Bulk (prefill-sized) update: synchronous so the host vector may change afterwards.
    TMLLM_CUDA_TRY(cudaMemcpyAsync(dst, src, sizeof(int32_t) * count, cudaMemcpyHostToDevice, s));
    TMLLM_CUDA_TRY(cudaStreamSynchronize(s));
    return TMLLM_OK;
}

// Blocks sequence `seq` still needs to hold positions [0, end).
int64_t blocks_needed(const tmllm_cache* c, int32_t seq, int64_t end) {
    const int64_t need = (end + c->cfg.block_size - 1) / c->cfg.block_size;
    return std::max<int64_t>(0, need - c->h_nblk[seq]);
}

// Assigns blocks so `seq` covers [0, end).  Caller has validated capacity and pool size.
int assign_blocks(tmllm_cache* c, int32_t seq, int64_t end, cudaStream_t s) {
    const int64_t need = blocks_needed(c, seq, end);
    if (need == 0) return TMLLM_OK;
    const int32_t first = c->h_nblk[seq];
    for (int64_t i = 0; i < need; ++i) {
        c->h_table[static_cast<int64_t>(seq) * c->max_blocks + first + i] = c->free_ids.back();
        c->free_ids.pop_back();
    }
    c->h_nblk[seq] = first + static_cast<int32_t>(need);
    return upload_entries(c, seq, first, static_cast<int32_t>(need), s);
}

int validate_extend(const tmllm_cache* c, int32_t seq, int64_t n) {
    if (n < 0) return fail(TMLLM_INVALID_ARGUMENT, "negative token count %lld",
                           static_cast<long long>(n));
    const int64_t len = c->h_lens[seq];
    if (n > c->cfg.max_seq_len - len)  // kv_cache.rs:40-51
        return fail_position(len, n, c->cfg.max_seq_len);
    if (blocks_needed(c, seq, len + n) > static_cast<int64_t>(c->free_ids.size()))
        return fail(TMLLM_OUT_OF_BLOCKS, "KV block pool exhausted (%zu free, %lld needed)",
                    c->free_ids.size(), static_cast<long long>(blocks_needed(c, seq, len + n)));
    return TMLLM_OK;
}

template <bool kWrite>
int launch_paged_rows(tmllm_cache* c, int32_t layer, int32_t seq, int64_t start, int64_t n,
                      const void* k_dense, const void* v_dense, cudaStream_t s) {
    if (n == 0 || (!k_dense && !v_dense)) return TMLLM_OK;
    const int64_t rb = c->row_bytes();
    const bool vec = rb % 16 == 0 && (!k_dense || aligned16(k_dense)) &&
                     (!v_dense || aligned16(v_dense));
    auto* kd = static_cast<unsigned char*>(const_cast<void*>(k_dense));
    auto* vd = static_cast<unsigned char*>(const_cast<void*>(v_dense));
    const int64_t units = vec ? rb / 16 : rb / static_cast<int64_t>(dtype_size(c->cfg.dtype));
    const int grid = grid_for(static_cast<int64_t>(c->cfg.num_kv_heads) * n * units);
    if (vec)
        paged_rows_kernel<uint4, kWrite><<<grid, 256, 0, s>>>(
            c->k_layer(layer), c->v_layer(layer), c->d_table, c->max_blocks, c->cfg.block_size,
            c->cfg.num_kv_heads, rb, c->num_blocks, seq, start, n, kd, vd);
    else if (c->cfg.dtype == TMLLM_F16)
        paged_rows_kernel<uint16_t, kWrite><<<grid, 256, 0, s>>>(
            c->k_layer(layer), c->v_layer(layer), c->d_table, c->max_blocks, c->cfg.block_size,
            c->cfg.num_kv_heads, rb, c->num_blocks, seq, start, n, kd, vd);
    else
        paged_rows_kernel<uint32_t, kWrite><<<grid, 256, 0, s>>>(
            c->k_layer(layer), c->v_layer(layer), c->d_table, c->max_blocks, c->cfg.block_size,
            c->cfg.num_kv_heads, rb, c->num_blocks, seq, start, n, kd, vd);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

void release(tmllm_cache* c) {
    if (c->arena) cudaFree(c->arena);
    if (c->d_table) cudaFree(c->d_table);
    if (c->d_lens) cudaFree(c->d_lens);
    if (c->ws) cudaFree(c->ws);
    c->arena = nullptr;
    c->d_table = c->d_lens = nullptr;
    c->ws = nullptr;
}

}  // namespace

extern "C" {

int tmllm_cache_create(const tmllm_cache_config* config, tmllm_cache** out) {
    clear_error();
    if (!config || !out) return fail(TMLLM_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    const tmllm_cache_config& cf = *config;
    if (!valid_dtype(cf.dtype)) return fail(TMLLM_UNSUPPORTED_DTYPE, "unknown dtype %d", cf.dtype);
    if (cf.num_kv_heads <= 0 || cf.max_seq_len <= 0 || cf.head_dim <= 0 || cf.num_layers <= 0 ||
        cf.num_seqs <= 0 || cf.block_size <= 0)  // kv_cache.rs:61-65
        return fail(TMLLM_INVALID_SHAPE, "KV cache dimensions must be positive");
    if (cf.num_blocks < 0) return fail(TMLLM_INVALID_SHAPE, "negative block count");
    const int64_t max_blocks = (static_cast<int64_t>(cf.max_seq_len) + cf.block_size - 1) / cf.block_size;
    int64_t num_blocks = cf.num_blocks;
    if (num_blocks == 0 && !mul_ok(max_blocks, cf.num_seqs, &num_blocks))
        return fail(TMLLM_INVALID_SHAPE, "block count overflow");
    if (num_blocks > INT32_MAX) return fail(TMLLM_INVALID_SHAPE, "more than 2^31 blocks");
    int64_t layer_bytes, total;
    if (!checked_numel({static_cast<size_t>(num_blocks), static_cast<size_t>(cf.num_kv_heads),
                        static_cast<size_t>(cf.block_size), static_cast<size_t>(cf.head_dim),
                        dtype_size(cf.dtype)},
                       &layer_bytes) ||
        !mul_ok(layer_bytes, 2 * static_cast<int64_t>(cf.num_layers), &total))
        return fail(TMLLM_INVALID_SHAPE, "KV cache size overflow");
    layer_bytes = (layer_bytes + 255) & ~static_cast<int64_t>(255);
    total = layer_bytes * 2 * cf.num_layers;

    DeviceGuard guard(cf.device);
    if (!guard.ok) return fail(TMLLM_DEVICE_ERROR, "cannot select CUDA device %d", cf.device);
    auto* c = new tmllm_cache();
    c->cfg = cf;
    c->num_blocks = num_blocks;
    c->max_blocks = static_cast<int32_t>(max_blocks);
    c->layer_bytes = layer_bytes;
    c->h_table.assign(static_cast<size_t>(cf.num_seqs) * max_blocks, -1);
    c->h_lens.assign(cf.num_seqs, 0);
    c->h_nblk.assign(cf.num_seqs, 0);
    c->free_ids.resize(num_blocks);
    // Handed out from the back: reverse pool order, or a seeded shuffle.
    for (int64_t i = 0; i < num_blocks; ++i) c->free_ids[i] = static_cast<int32_t>(num_blocks - 1 - i);
    if (cf.shuffle_seed != 0) {
        std::mt19937_64 rng(cf.shuffle_seed);
        for (int64_t i = num_blocks - 1; i > 0; --i) {
            std::uniform_int_distribution<int64_t> pick(0, i);
            std::swap(c->free_ids[i], c->free_ids[pick(rng)]);
        }
    }
    cudaError_t e = cudaMalloc(&c->arena, static_cast<size_t>(total));
    // zeroed once, so slots never written (a block's tail) hold finite values
    if (e == cudaSuccess) e = cudaMemset(c->arena, 0, static_cast<size_t>(total));
    if (e == cudaSuccess)
        e = cudaMalloc(&c->d_table, sizeof(int32_t) * c->h_table.size());
    if (e == cudaSuccess) e = cudaMalloc(&c->d_lens, sizeof(int32_t) * cf.num_seqs);
    if (e == cudaSuccess)
        e = cudaMemset(c->d_table, 0xff, sizeof(int32_t) * c->h_table.size());
    if (e == cudaSuccess) e = cudaMemset(c->d_lens, 0, sizeof(int32_t) * cf.num_seqs);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        release(c);
        delete c;
        return cuda_fail(e, "tmllm_cache_create allocation");
    }
    *out = c;
    return TMLLM_OK;
}

int tmllm_cache_destroy(tmllm_cache* cache) {
    clear_error();
    if (!cache) return TMLLM_OK;
    DeviceGuard guard(cache->cfg.device);
    cudaDeviceSynchronize();
    release(cache);
    delete cache;
    return TMLLM_OK;
}

int tmllm_cache_len(const tmllm_cache* cache, int32_t seq, int64_t* out) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_seq(cache, seq)) return st;
    if (!out) return fail(TMLLM_INVALID_ARGUMENT, "null output");
    *out = cache->h_lens[seq];
    return TMLLM_OK;
}

int tmllm_cache_capacity(const tmllm_cache* cache, int64_t* out) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (!out) return fail(TMLLM_INVALID_ARGUMENT, "null output");
    *out = cache->cfg.max_seq_len;
    return TMLLM_OK;
}

int tmllm_cache_storage_bytes(const tmllm_cache* cache, int64_t* out) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (!out) return fail(TMLLM_INVALID_ARGUMENT, "null output");
    *out = cache->layer_bytes * 2 * cache->cfg.num_layers;
    return TMLLM_OK;
}

int tmllm_cache_reset(tmllm_cache* cache, int32_t seq, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (seq >= 0)
        if (int st = check_seq(cache, seq)) return st;
    DeviceGuard guard(cache->cfg.device);
    auto s = reinterpret_cast<cudaStream_t>(stream);
    const int first = seq < 0 ? 0 : seq, last = seq < 0 ? cache->cfg.num_seqs : seq + 1;
    for (int i = first; i < last; ++i) {
        for (int32_t k = cache->h_nblk[i] - 1; k >= 0; --k) {
            int32_t& id = cache->h_table[static_cast<int64_t>(i) * cache->max_blocks + k];
            cache->free_ids.push_back(id);
            id = -1;
        }
        cache->h_nblk[i] = 0;
        cache->h_lens[i] = 0;
    }
    const int64_t off = static_cast<int64_t>(first) * cache->max_blocks;
    const int64_t n = static_cast<int64_t>(last - first) * cache->max_blocks;
    fill_i32_kernel<<<grid_for(n), 256, 0, s>>>(cache->d_table + off, -1, n);
    fill_i32_kernel<<<1, 256, 0, s>>>(cache->d_lens + first, 0, last - first);
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_cache_reserve(tmllm_cache* cache, int32_t seq, int64_t n, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_seq(cache, seq)) return st;
    if (int st = validate_extend(cache, seq, n)) return st;
    DeviceGuard guard(cache->cfg.device);
    return assign_blocks(cache, seq, cache->h_lens[seq] + n, reinterpret_cast<cudaStream_t>(stream));
}

int tmllm_cache_append(tmllm_cache* cache, int32_t layer, int32_t seq, const void* k,
                       const void* v, int64_t n, int32_t dtype, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (dtype != cache->cfg.dtype)  // kv_cache.rs:19-27
        return fail(TMLLM_UNSUPPORTED_DTYPE, "KV cache dtype mismatch: cache=%s, input=%s",
                    dtype_name(cache->cfg.dtype), valid_dtype(dtype) ? dtype_name(dtype) : "?");
    if (int st = check_layer(cache, layer)) return st;
    if (int st = check_seq(cache, seq)) return st;
    if (int st = validate_extend(cache, seq, n)) return st;
    if (n > 0 && (!k || !v)) return fail(TMLLM_INVALID_ARGUMENT, "null tensor pointer");
    DeviceGuard guard(cache->cfg.device);
    auto s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t start = cache->h_lens[seq];
    if (int st = assign_blocks(cache, seq, start + n, s)) return st;
    return launch_paged_rows<true>(cache, layer, seq, start, n, k, v, s);
}

int tmllm_cache_advance(tmllm_cache* cache, int32_t seq, int64_t n, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (seq >= 0)
        if (int st = check_seq(cache, seq)) return st;
    const int first = seq < 0 ? 0 : seq, last = seq < 0 ? cache->cfg.num_seqs : seq + 1;
    for (int i = first; i < last; ++i) {
        if (n < 0 || n > cache->cfg.max_seq_len - cache->h_lens[i])
            return fail_position(cache->h_lens[i], n, cache->cfg.max_seq_len);
        if (blocks_needed(cache, i, cache->h_lens[i] + n) > 0)
            return fail(TMLLM_NOT_RESERVED, "sequence %d has no block for position %lld", i,
                        static_cast<long long>(cache->h_lens[i] + n - 1));
    }
    if (n == 0) return TMLLM_OK;
    DeviceGuard guard(cache->cfg.device);
    for (int i = first; i < last; ++i) cache->h_lens[i] += n;
    const int count = last - first;
    add_lens_kernel<<<(count + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        cache->d_lens, first, count, static_cast<int32_t>(n));
    TMLLM_LAUNCH_TRY();
    return TMLLM_OK;
}

int tmllm_cache_view(const tmllm_cache* cache, int32_t layer, tmllm_paged_kv* out) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_layer(cache, layer)) return st;
    if (!out) return fail(TMLLM_INVALID_ARGUMENT, "null output");
    out->k_cache = cache->k_layer(layer);
    out->v_cache = cache->v_layer(layer);
    out->block_table = cache->d_table;
    out->seq_lens = cache->d_lens;
    out->num_blocks = cache->num_blocks;
    out->num_seqs = cache->cfg.num_seqs;
    out->num_kv_heads = cache->cfg.num_kv_heads;
    out->head_dim = cache->cfg.head_dim;
    out->block_size = cache->cfg.block_size;
    out->max_blocks_per_seq = cache->max_blocks;
    out->dtype = cache->cfg.dtype;
    return TMLLM_OK;
}

int tmllm_cache_block_table(const tmllm_cache* cache, int32_t seq, int32_t* out,
                            int64_t capacity, int64_t* n) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_seq(cache, seq)) return st;
    const int64_t cnt = cache->h_nblk[seq];
    if (n) *n = cnt;
    if (!out) return TMLLM_OK;
    if (capacity < cnt) return fail(TMLLM_INVALID_ARGUMENT, "output holds %lld of %lld entries",
                                    static_cast<long long>(capacity), static_cast<long long>(cnt));
    std::memcpy(out, cache->h_table.data() + static_cast<int64_t>(seq) * cache->max_blocks,
                sizeof(int32_t) * cnt);
    return TMLLM_OK;
}

int tmllm_cache_gather(const tmllm_cache* cache, int32_t layer, int32_t seq, void* k_out,
                       void* v_out, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_layer(cache, layer)) return st;
    if (int st = check_seq(cache, seq)) return st;
    DeviceGuard guard(cache->cfg.device);
    return launch_paged_rows<false>(const_cast<tmllm_cache*>(cache), layer, seq, 0,
                                    cache->h_lens[seq], k_out, v_out,
                                    reinterpret_cast<cudaStream_t>(stream));
}

int tmllm_cache_decode(tmllm_cache* cache, int32_t layer, const void* q, const void* k_new,
                       const void* v_new, void* out, float* lse, int32_t q_heads,
                       const tmllm_decode_opts* opts, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_layer(cache, layer)) return st;
    if (q_heads <= 0 || q_heads % cache->cfg.num_kv_heads != 0)
        return fail(TMLLM_MODEL_FORMAT, "Q heads %d must be divisible by non-zero KV heads %d",
                    q_heads, cache->cfg.num_kv_heads);
    const bool append = k_new != nullptr;
    int64_t max_len = 0, need_total = 0;
    for (int i = 0; i < cache->cfg.num_seqs; ++i) {
        const int64_t len = cache->h_lens[i];
        if (append && len >= cache->cfg.max_seq_len)
            return fail_position(len, 1, cache->cfg.max_seq_len);
        if (append) need_total += blocks_needed(cache, i, len + 1);
        max_len = std::max<int64_t>(max_len, len + (append ? 1 : 0));
    }
    if (need_total > static_cast<int64_t>(cache->free_ids.size()))
        return fail(TMLLM_OUT_OF_BLOCKS, "KV block pool exhausted");
    DeviceGuard guard(cache->cfg.device);
    auto s = reinterpret_cast<cudaStream_t>(stream);
    tmllm_paged_kv view;
    tmllm_cache_view(cache, layer, &view);
    tmllm_decode_opts o{};
    if (opts) o = *opts;
    if (o.rope_cos) {
        for (int i = 0; i < cache->cfg.num_seqs; ++i) {
            const int64_t pos = cache->h_lens[i] + o.rope_pos_offset;
            if (pos < 0 || pos >= o.rope_len)
                return fail_position(pos, 1, o.rope_len);  // rope.rs:121-127
        }
    }
    // a caller that knows lengths will grow (a captured graph replayed for several steps)
    // may ask for splits sized for the longest length it will see
    const int64_t hint = std::max<int64_t>(max_len, o.max_len_hint);
    int32_t splits = o.num_splits;
    int64_t chunk = 0;
    if (splits <= 0) {
        // positions per split from every sequence's length and the resident CTAs per SM of
        // the kernel that will run; the split count follows from the longest length
        const int G = q_heads / cache->cfg.num_kv_heads;
        const int per_sm = decode_resident_ctas(cache->cfg.dtype, cache->cfg.head_dim,
                                                o.variant, G);
        std::vector<int64_t> lens(cache->h_lens.begin(), cache->h_lens.end());
        if (append)
            for (auto& x : lens) ++x;
        chunk = decode_auto_chunk_lens(lens.data(), cache->cfg.num_seqs,
                                       cache->cfg.num_kv_heads, hint, per_sm);
        int64_t s2 = (hint + chunk - 1) / chunk;
        if (s2 > 1024) s2 = 1024;
        splits = static_cast<int32_t>(s2 < 1 ? 1 : s2);
    }
    o.num_splits = splits;
    const size_t need = decode_workspace_bytes(cache->cfg.num_seqs, q_heads,
                                               cache->cfg.num_kv_heads, cache->cfg.head_dim,
                                               splits);
    if (need > cache->ws_bytes) {
        if (cache->ws) {
            TMLLM_CUDA_TRY(cudaStreamSynchronize(s));
            cudaFree(cache->ws);
            cache->ws = nullptr;
            cache->ws_bytes = 0;
        }
        TMLLM_CUDA_TRY(cudaMalloc(&cache->ws, need));
        TMLLM_CUDA_TRY(cudaMemsetAsync(cache->ws, 0, need, s));
        cache->ws_bytes = need;
    }
    if (append)
        for (int i = 0; i < cache->cfg.num_seqs; ++i)
            if (int st = assign_blocks(cache, i, cache->h_lens[i] + 1, s)) return st;
    // A block assigned just now reaches the device table through a kernel queued right
    // ahead of the decode, which an overlapped launch would read before that kernel ends:
    // such a call launches plainly.
    if (need_total > 0) o.flags &= ~TMLLM_DECODE_OVERLAP;
    return decode_impl_ex(&view, q, k_new, v_new, out, lse, q_heads, &o, cache->ws,
                          cache->ws_bytes, hint, nullptr, 0, false, s, chunk);
}

int tmllm_cache_prefill(tmllm_cache* cache, int32_t layer, const void* q, const void* k_new,
                        const void* v_new, int64_t n, void* out, int32_t q_heads,
                        const tmllm_decode_opts* opts, tmllm_stream stream) {
    clear_error();
    if (int st = check_cache(cache)) return st;
    if (int st = check_layer(cache, layer)) return st;
    if (q_heads <= 0 || q_heads % cache->cfg.num_kv_heads != 0)
        return fail(TMLLM_MODEL_FORMAT, "Q heads %d must be divisible by non-zero KV heads %d",
                    q_heads, cache->cfg.num_kv_heads);
    if (n < 0) return fail(TMLLM_INVALID_ARGUMENT, "negative token count %lld",
                           static_cast<long long>(n));
    if (n == 0) return TMLLM_OK;
    if (!k_new || !v_new) return fail(TMLLM_INVALID_ARGUMENT, "prefill needs k_new and v_new");
    if (n > INT32_MAX / std::max(1, cache->cfg.num_seqs))
        return fail(TMLLM_INVALID_SHAPE, "prefill rows exceed i32");
    int64_t need_total = 0;
    for (int i = 0; i < cache->cfg.num_seqs; ++i) {
        const int64_t len = cache->h_lens[i];
        if (n > cache->cfg.max_seq_len - len)  // kv_cache.rs:40-51
            return fail_position(len, n, cache->cfg.max_seq_len);
        need_total += blocks_needed(cache, i, len + n);
    }
    if (need_total > static_cast<int64_t>(cache->free_ids.size()))
        return fail(TMLLM_OUT_OF_BLOCKS, "KV block pool exhausted");
    tmllm_decode_opts o{};
    if (opts) o = *opts;
    if (o.rope_cos) {
        for (int i = 0; i < cache->cfg.num_seqs; ++i) {
            const int64_t lo = cache->h_lens[i] + o.rope_pos_offset, hi = lo + n - 1;
            if (lo < 0 || hi >= o.rope_len)
                return fail_position(lo, n, o.rope_len);  // rope.rs:121-127
        }
    }
    DeviceGuard guard(cache->cfg.device);
    auto s = reinterpret_cast<cudaStream_t>(stream);
    for (int i = 0; i < cache->cfg.num_seqs; ++i)
        if (int st = assign_blocks(cache, i, cache->h_lens[i] + n, s)) return st;
    tmllm_paged_kv view;
    tmllm_cache_view(cache, layer, &view);
    return prefill_impl(&view, q, k_new, v_new, nullptr, static_cast<int32_t>(n), 0, 0, out,
                        q_heads, &o, s);
}

}  // extern "C"
