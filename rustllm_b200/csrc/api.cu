// Library-level entry points: version, status names, per-thread error messages, sync.
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace tmllm {

namespace {
thread_local std::string g_last_error;
thread_local tmllm_error_fields g_fields{};

void set_message(const char* fmt, va_list ap) {
    char buf[1024];
    vsnprintf(buf, sizeof(buf), fmt, ap);
    g_last_error = buf;
}
}  // namespace

void clear_error() {
    g_last_error.clear();
    g_fields = tmllm_error_fields{};
}

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    set_message(fmt, ap);
    va_end(ap);
    g_fields = tmllm_error_fields{};
    g_fields.status = status;
    return status;
}

int fail_position(int64_t start_pos, int64_t seq_len, int64_t max_seq_len) {
    g_fields = tmllm_error_fields{};
    g_fields.status = TMLLM_POSITION_OUT_OF_RANGE;
    g_fields.start_pos = start_pos;
    g_fields.seq_len = seq_len;
    g_fields.max_seq_len = max_seq_len;
    // the reference's Display text (src/error.rs:86-95)
    char buf[160];
    snprintf(buf, sizeof(buf), "position range [%lld, %lld) exceeds max sequence length %lld",
             static_cast<long long>(start_pos), static_cast<long long>(start_pos + seq_len),
             static_cast<long long>(max_seq_len));
    g_last_error = buf;
    return TMLLM_POSITION_OUT_OF_RANGE;
}

int fail_shapes(std::initializer_list<int64_t> left, std::initializer_list<int64_t> right,
                const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    set_message(fmt, ap);
    va_end(ap);
    g_fields = tmllm_error_fields{};
    g_fields.status = TMLLM_SHAPE_MISMATCH;
    for (int64_t d : left)
        if (g_fields.left_rank < TMLLM_MAX_RANK) g_fields.left[g_fields.left_rank++] = d;
    for (int64_t d : right)
        if (g_fields.right_rank < TMLLM_MAX_RANK) g_fields.right[g_fields.right_rank++] = d;
    return TMLLM_SHAPE_MISMATCH;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(TMLLM_DEVICE_ERROR, "CUDA error in %s: %s (%s)", what, cudaGetErrorName(err),
                cudaGetErrorString(err));
}

bool checked_numel(std::initializer_list<size_t> dims, int64_t* out) {
    int64_t acc = 1;
    for (size_t d : dims) {
        if (d > static_cast<size_t>(INT64_MAX)) return false;
        if (!mul_ok(acc, static_cast<int64_t>(d), &acc)) return false;
    }
    *out = acc;
    return true;
}

int device_sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace tmllm

extern "C" {

int tmllm_version(void) { return 100; }

const char* tmllm_status_name(int status) {
    switch (status) {
        case TMLLM_OK: return "TMLLM_OK";
        case TMLLM_INVALID_ARGUMENT: return "TMLLM_INVALID_ARGUMENT";
        case TMLLM_INVALID_SHAPE: return "TMLLM_INVALID_SHAPE";
        case TMLLM_SHAPE_MISMATCH: return "TMLLM_SHAPE_MISMATCH";
        case TMLLM_INVALID_DIMENSION: return "TMLLM_INVALID_DIMENSION";
        case TMLLM_UNSUPPORTED_DTYPE: return "TMLLM_UNSUPPORTED_DTYPE";
        case TMLLM_NON_CONTIGUOUS: return "TMLLM_NON_CONTIGUOUS";
        case TMLLM_POSITION_OUT_OF_RANGE: return "TMLLM_POSITION_OUT_OF_RANGE";
        case TMLLM_MODEL_FORMAT: return "TMLLM_MODEL_FORMAT";
        case TMLLM_DEVICE_ERROR: return "TMLLM_DEVICE_ERROR";
        case TMLLM_OUT_OF_BLOCKS: return "TMLLM_OUT_OF_BLOCKS";
        case TMLLM_TIMEOUT: return "TMLLM_TIMEOUT";
        case TMLLM_NOT_RESERVED: return "TMLLM_NOT_RESERVED";
        default: return "TMLLM_UNKNOWN_STATUS";
    }
}

const char* tmllm_last_error(void) { return tmllm::g_last_error.c_str(); }

int tmllm_last_error_fields(tmllm_error_fields* out) {
    if (!out) return TMLLM_INVALID_ARGUMENT;  // leaves the recorded failure untouched
    *out = tmllm::g_fields;
    return TMLLM_OK;
}

int tmllm_sync(tmllm_stream stream) {
    tmllm::clear_error();
    TMLLM_CUDA_TRY(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
    return TMLLM_OK;
}

}  // extern "C"
