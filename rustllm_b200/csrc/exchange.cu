// Cross-GPU exchange for a sequence split (one process per GPU, or one process driving
// several GPUs).  Each rank allocates one buffer (receive cells for every rank's partial
// rows, a status word), shares it with CUDA IPC, and maps every other rank's buffer.  The fused decode kernel then pushes its final (O, lse) rows straight into
// every rank's buffer over NVLink and merges what arrives in its own: one launch per rank
// per decode step, no separate collective.
#include <cstring>
#include <vector>

#include "common.cuh"

namespace tmllm {
int decode_impl_ex(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                   const void* v_new, void* out, float* lse, int32_t q_heads,
                   const tmllm_decode_opts* opts, void* workspace, size_t workspace_bytes,
                   int64_t max_len_hint, const ExchangeArgs* ex, uint32_t epoch,
                   bool clear_tickets, cudaStream_t stream, int64_t chunk_override = 0);
}

using namespace tmllm;

struct tmllm_exchange {
    int world = 0, rank = 0, rows = 0, groups = 0, head_dim = 0, device = 0;
    size_t off_lse = 0, off_status = 0, bytes = 0;
    unsigned char* base = nullptr;                   // this rank's buffer
    unsigned char* peer[kMaxRanks] = {};             // every rank's buffer (own included)
    bool ipc_opened[kMaxRanks] = {};
    ExchangeArgs host{};
    ExchangeArgs* dev_args = nullptr;
    uint32_t epoch = 0;
    bool connected = false;
};

namespace {

size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int upload_args(tmllm_exchange* ex) {
    ExchangeArgs& h = ex->host;
    for (int p = 0; p < ex->world; ++p) {
        h.recv_o[p] = reinterpret_cast<uint2*>(ex->peer[p]);
        h.recv_lse[p] = reinterpret_cast<uint2*>(ex->peer[p] + ex->off_lse);
    }
    h.status = reinterpret_cast<int*>(ex->base + ex->off_status);
    h.rank = ex->rank;
    h.world = ex->world;
    h.rows = ex->rows;
    h.groups = ex->groups;
    h.head_dim = ex->head_dim;
    TMLLM_CUDA_TRY(cudaMemcpy(ex->dev_args, &h, sizeof(h), cudaMemcpyHostToDevice));
    ex->connected = true;
    return TMLLM_OK;
}

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int tmllm_exchange_create(int32_t world, int32_t rank, int32_t rows, int32_t groups,
                          int32_t head_dim, tmllm_exchange** out, void* ipc_handle_out) {
    clear_error();
    if (!out) return fail(TMLLM_INVALID_ARGUMENT, "null output");
    *out = nullptr;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(TMLLM_INVALID_ARGUMENT, "rank %d of world %d (at most %d ranks)", rank, world,
                    kMaxRanks);
    if (rows <= 0 || groups <= 0 || head_dim <= 0 || rows % groups != 0)
        return fail(TMLLM_INVALID_SHAPE, "exchange rows %d / groups %d / head_dim %d", rows, groups,
                    head_dim);
    auto* ex = new tmllm_exchange();
    ex->world = world;
    ex->rank = rank;
    ex->rows = rows;
    ex->groups = groups;
    ex->head_dim = head_dim;
    if (cudaGetDevice(&ex->device) != cudaSuccess) {
        delete ex;
        return fail(TMLLM_DEVICE_ERROR, "no current CUDA device");
    }
    ex->off_lse = up256(sizeof(uint2) * 2 * static_cast<size_t>(world) * rows * head_dim);
    ex->off_status = ex->off_lse + up256(sizeof(uint2) * 2 * static_cast<size_t>(world) * rows);
    ex->bytes = ex->off_status + 256;
    ex->host.timeout_ns = 2000000000ull;  // 2 s
    cudaError_t e = cudaMalloc(&ex->base, ex->bytes);
    if (e == cudaSuccess) e = cudaMemset(ex->base, 0, ex->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&ex->dev_args, sizeof(ExchangeArgs));
    if (e == cudaSuccess && ipc_handle_out) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, ex->base);
        if (e == cudaSuccess) std::memcpy(ipc_handle_out, &h, sizeof(h));
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (ex->base) cudaFree(ex->base);
        if (ex->dev_args) cudaFree(ex->dev_args);
        delete ex;
        return cuda_fail(e, "tmllm_exchange_create");
    }
    ex->peer[rank] = ex->base;
    *out = ex;
    return TMLLM_OK;
}

int tmllm_exchange_connect(tmllm_exchange* ex, const void* handles) {
    clear_error();
    if (!ex || !handles) return fail(TMLLM_INVALID_ARGUMENT, "null argument");
    DeviceScope scope(ex->device);
    const auto* hs = static_cast<const unsigned char*>(handles);
    for (int p = 0; p < ex->world; ++p) {
        if (p == ex->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + static_cast<size_t>(p) * TMLLM_IPC_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        TMLLM_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        ex->peer[p] = static_cast<unsigned char*>(ptr);
        ex->ipc_opened[p] = true;
    }
    return upload_args(ex);
}

int tmllm_exchange_connect_local(tmllm_exchange* ex, tmllm_exchange* const* ranks) {
    clear_error();
    if (!ex || !ranks) return fail(TMLLM_INVALID_ARGUMENT, "null argument");
    DeviceScope scope(ex->device);
    for (int p = 0; p < ex->world; ++p) {
        const tmllm_exchange* r = ranks[p];
        if (!r || r->world != ex->world || r->rank != p || r->rows != ex->rows ||
            r->groups != ex->groups || r->head_dim != ex->head_dim)
            return fail(TMLLM_INVALID_ARGUMENT, "rank %d's exchange does not match", p);
        if (p != ex->rank && r->device != ex->device) {
            int can = 0;
            TMLLM_CUDA_TRY(cudaDeviceCanAccessPeer(&can, ex->device, r->device));
            if (!can) return fail(TMLLM_DEVICE_ERROR, "device %d cannot reach device %d", ex->device,
                                  r->device);
            cudaError_t e = cudaDeviceEnablePeerAccess(r->device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
        }
        ex->peer[p] = r->base;
    }
    return upload_args(ex);
}

int tmllm_exchange_set_timeout(tmllm_exchange* ex, uint64_t timeout_ns) {
    clear_error();
    if (!ex) return fail(TMLLM_INVALID_ARGUMENT, "null exchange");
    ex->host.timeout_ns = timeout_ns;
    if (ex->connected) {
        DeviceScope scope(ex->device);
        TMLLM_CUDA_TRY(cudaMemcpy(&ex->dev_args->timeout_ns, &timeout_ns, sizeof(timeout_ns),
                                  cudaMemcpyHostToDevice));
    }
    return TMLLM_OK;
}

int tmllm_exchange_status(tmllm_exchange* ex, int32_t* status) {
    clear_error();
    if (!ex || !status) return fail(TMLLM_INVALID_ARGUMENT, "null argument");
    DeviceScope scope(ex->device);
    int v = 0;
    TMLLM_CUDA_TRY(cudaMemcpy(&v, ex->base + ex->off_status, sizeof(int), cudaMemcpyDeviceToHost));
    const int zero = 0;
    TMLLM_CUDA_TRY(cudaMemcpy(ex->base + ex->off_status, &zero, sizeof(int),
                              cudaMemcpyHostToDevice));
    *status = v;
    return TMLLM_OK;
}

int tmllm_exchange_destroy(tmllm_exchange* ex) {
    clear_error();
    if (!ex) return TMLLM_OK;
    DeviceScope scope(ex->device);
    cudaDeviceSynchronize();
    for (int p = 0; p < ex->world; ++p)
        if (ex->ipc_opened[p]) cudaIpcCloseMemHandle(ex->peer[p]);
    cudaFree(ex->base);
    cudaFree(ex->dev_args);
    delete ex;
    return TMLLM_OK;
}

int tmllm_gqa_decode_exchange(const tmllm_paged_kv* kv, const void* q, const void* k_new,
                              const void* v_new, void* out, float* lse, int32_t q_heads,
                              const tmllm_decode_opts* opts, void* workspace,
                              size_t workspace_bytes, tmllm_exchange* ex,
                              tmllm_stream stream) {
    clear_error();
    if (!ex || !ex->connected) return fail(TMLLM_INVALID_ARGUMENT, "exchange not connected");
    if (!kv) return fail(TMLLM_INVALID_ARGUMENT, "null paged KV descriptor");
    if (static_cast<int64_t>(kv->num_seqs) * q_heads != ex->rows ||
        static_cast<int64_t>(kv->num_seqs) * kv->num_kv_heads != ex->groups ||
        kv->head_dim != ex->head_dim)
        return fail_shapes({ex->rows, ex->groups, ex->head_dim},
                           {static_cast<int64_t>(kv->num_seqs) * q_heads,
                            static_cast<int64_t>(kv->num_seqs) * kv->num_kv_heads,
                            kv->head_dim},
                           "exchange sized for %d rows / %d groups / head_dim %d, call has "
                           "%d x %d / %d x %d / %d",
                           ex->rows, ex->groups, ex->head_dim, kv->num_seqs, q_heads,
                           kv->num_seqs, kv->num_kv_heads, kv->head_dim);
    const uint32_t epoch = ex->epoch + 1;
    int st = decode_impl_ex(kv, q, k_new, v_new, out, lse, q_heads, opts, workspace,
                            workspace_bytes, opts ? opts->max_len_hint : 0, ex->dev_args, epoch,
                            false, reinterpret_cast<cudaStream_t>(stream));
    if (st == TMLLM_OK) ex->epoch = epoch;
    return st;
}

}  // extern "C"
