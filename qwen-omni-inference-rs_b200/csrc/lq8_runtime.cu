// lq8_runtime.cu -- context, errors, fault injection and device memory of liblq8.
#include "lq8_internal.cuh"

#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

namespace {
thread_local std::string g_init_error;  // lq_last_error(NULL)
}

namespace lq {

int set_error(lq_ctx* ctx, int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = buf;
    else g_init_error = buf;
    return code;
}

int check_cuda(lq_ctx* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return LQ_OK;
    int code = (e == cudaErrorMemoryAllocation) ? LQ_ERR_OOM : LQ_ERR_CUDA;
    return set_error(ctx, code, "CUDA error %d (%s) in %s", (int)e, cudaGetErrorString(e), what);
}

bool fault_injected(const char* entry) {
    const char* f = getenv("LQ_FAULT");
    if (!f || !*f) return false;
    // comma-separated list of entry names
    size_t n = strlen(entry);
    const char* p = f;
    while (*p) {
        const char* q = strchr(p, ',');
        size_t len = q ? (size_t)(q - p) : strlen(p);
        if (len == n && strncmp(p, entry, n) == 0) return true;
        if (!q) break;
        p = q + 1;
    }
    return false;
}

int ensure_scratch(lq_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->scratch_bytes) return LQ_OK;
    // LQ_FAULT=ensure_scratch turns every scratch allocation into an error (tests use it to
    // show that a path allocates nothing)
    if (fault_injected("ensure_scratch"))
        return set_error(ctx, LQ_ERR_INJECTED, "ensure_scratch: injected fault (LQ_FAULT), %zu bytes", bytes);
    // the old scratch may still be in use by queued work
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->scratch) LQ_CUDA(ctx, cudaFree(ctx->scratch));
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t sz = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;  // 1 MiB granularity
    LQ_CUDA(ctx, cudaMalloc(&ctx->scratch, sz));
    ctx->scratch_bytes = sz;
    return LQ_OK;
}

int ensure_wide(lq_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->wide_bytes) return LQ_OK;
    if (fault_injected("ensure_wide"))
        return set_error(ctx, LQ_ERR_INJECTED, "ensure_wide: injected fault (LQ_FAULT), %zu bytes", bytes);
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    LQ_CUDA(ctx, cudaStreamIsCapturing(ctx->stream, &st));
    if (st != cudaStreamCaptureStatusNone)
        return set_error(ctx, LQ_ERR_STATE, "fp16 operand buffer (%zu bytes) too small while capturing a graph", bytes);
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->wide) LQ_CUDA(ctx, cudaFree(ctx->wide));
    ctx->wide = nullptr;
    ctx->wide_bytes = 0;
    size_t sz = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;
    LQ_CUDA(ctx, cudaMalloc(&ctx->wide, sz));
    ctx->wide_bytes = sz;
    return LQ_OK;
}

int ensure_split(lq_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->split_bytes) return LQ_OK;
    if (fault_injected("ensure_split"))
        return set_error(ctx, LQ_ERR_INJECTED, "ensure_split: injected fault (LQ_FAULT), %zu bytes", bytes);
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    LQ_CUDA(ctx, cudaStreamIsCapturing(ctx->stream, &st));
    if (st != cudaStreamCaptureStatusNone)
        return set_error(ctx, LQ_ERR_STATE, "split-K buffer (%zu bytes) too small while capturing a graph", bytes);
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->split) LQ_CUDA(ctx, cudaFree(ctx->split));
    ctx->split = nullptr;
    ctx->split_bytes = 0;
    size_t sz = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;
    LQ_CUDA(ctx, cudaMalloc(&ctx->split, sz));
    ctx->split_bytes = sz;
    return LQ_OK;
}

int ensure_func_smem(lq_ctx* ctx, const void* func, size_t bytes) {
    // the attribute belongs to the function on one device; contexts on several devices (or
    // threads driving them) share this table
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> set_bytes;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = set_bytes[std::make_pair(func, ctx->device)];
    if (have >= bytes) return LQ_OK;
    LQ_CUDA(ctx, cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    have = bytes;
    return LQ_OK;
}

int consume_device_error(lq_ctx* ctx, const char* what) {
    int h[4];
    LQ_CUDA(ctx, cudaMemcpyAsync(h, ctx->err_flag, sizeof h, cudaMemcpyDeviceToHost, ctx->stream));
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (h[0] != 0) {
        LQ_CUDA(ctx, cudaMemsetAsync(ctx->err_flag, 0, sizeof h, ctx->stream));
        // a kernel that gave up may have left tile counters mid-count
        LQ_CUDA(ctx, cudaMemsetAsync(ctx->tile_cnt, 0, kTileCounters * sizeof(unsigned), ctx->stream));
        return set_error(ctx, LQ_ERR_INVALID_ARG, "%s: device check failed (code %d, value %d)",
                         what, h[0], h[1]);
    }
    return LQ_OK;
}

}  // namespace lq

extern "C" {

int lq_abi_version(void) { return LQ8_ABI_VERSION; }

int lq_init(int device, lq_ctx** out) {
    if (!out) return lq::set_error(nullptr, LQ_ERR_INVALID_ARG, "lq_init: out is NULL");
    *out = nullptr;
    if (lq::fault_injected("lq_init"))
        return lq::set_error(nullptr, LQ_ERR_INJECTED, "lq_init: injected fault (LQ_FAULT)");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return lq::set_error(nullptr, LQ_ERR_CUDA, "lq_init: no CUDA device (%s)",
                             cudaGetErrorString(e));
    if (device < 0 || device >= n)
        return lq::set_error(nullptr, LQ_ERR_INVALID_ARG, "lq_init: device %d of %d", device, n);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess)
        return lq::set_error(nullptr, LQ_ERR_CUDA, "lq_init: %s", cudaGetErrorString(e));
    if (prop.major != 10)
        return lq::set_error(nullptr, LQ_ERR_UNSUPPORTED,
                             "lq_init: device %d is sm_%d%d; this library is built for sm_100a",
                             device, prop.major, prop.minor);
    e = cudaSetDevice(device);
    if (e != cudaSuccess)
        return lq::set_error(nullptr, LQ_ERR_CUDA, "lq_init: %s", cudaGetErrorString(e));
    lq_ctx* c = new lq_ctx();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->err_flag, 4 * sizeof(int)) != cudaSuccess ||
        cudaMemset(c->err_flag, 0, 4 * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&c->tile_cnt, kTileCounters * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(c->tile_cnt, 0, kTileCounters * sizeof(unsigned)) != cudaSuccess) {
        if (c->err_flag) cudaFree(c->err_flag);
        if (c->tile_cnt) cudaFree(c->tile_cnt);
        if (c->own_stream) cudaStreamDestroy(c->own_stream);
        delete c;
        return lq::set_error(nullptr, LQ_ERR_CUDA, "lq_init: stream/flag allocation failed");
    }
    c->stream = c->own_stream;
    // LQ_NO_PDL=1 launches every kernel with plain stream ordering (no programmatic overlap)
    c->pdl = getenv("LQ_NO_PDL") == nullptr;
    *out = c;
    return LQ_OK;
}

int lq_destroy(lq_ctx* ctx) {
    if (!ctx) return LQ_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->split) cudaFree(ctx->split);
    if (ctx->wide) cudaFree(ctx->wide);
    if (ctx->err_flag) cudaFree(ctx->err_flag);
    if (ctx->tile_cnt) cudaFree(ctx->tile_cnt);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return LQ_OK;
}

const char* lq_last_error(const lq_ctx* ctx) {
    return ctx ? ctx->last_error.c_str() : g_init_error.c_str();
}

int lq_set_stream(lq_ctx* ctx, void* stream) {
    LQ_ENTRY(ctx, "lq_set_stream");
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return LQ_OK;
}

void* lq_get_stream(lq_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int lq_synchronize(lq_ctx* ctx) {
    LQ_ENTRY(ctx, "lq_synchronize");
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return LQ_OK;
}

int lq_device_info(lq_ctx* ctx, int* sm_count, int* cc_major, int* cc_minor, size_t* total_mem) {
    LQ_ENTRY(ctx, "lq_device_info");
    cudaDeviceProp p;
    LQ_CUDA(ctx, cudaGetDeviceProperties(&p, ctx->device));
    if (sm_count) *sm_count = p.multiProcessorCount;
    if (cc_major) *cc_major = p.major;
    if (cc_minor) *cc_minor = p.minor;
    if (total_mem) *total_mem = p.totalGlobalMem;
    return LQ_OK;
}

int lq_malloc(lq_ctx* ctx, size_t bytes, void** out) {
    LQ_ENTRY(ctx, "lq_malloc");
    LQ_REQUIRE(ctx, out != nullptr, "lq_malloc: out is NULL");
    *out = nullptr;
    if (bytes == 0) return LQ_OK;
    LQ_CUDA(ctx, cudaMalloc(out, bytes));
    return LQ_OK;
}

int lq_free(lq_ctx* ctx, void* p) {
    LQ_ENTRY(ctx, "lq_free");
    if (p) LQ_CUDA(ctx, cudaFree(p));
    return LQ_OK;
}

int lq_memcpy_h2d(lq_ctx* ctx, void* dst, const void* src, size_t bytes) {
    LQ_ENTRY(ctx, "lq_memcpy_h2d");
    if (!bytes) return LQ_OK;
    LQ_REQUIRE(ctx, dst && src, "lq_memcpy_h2d: NULL pointer");
    LQ_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return LQ_OK;
}

int lq_memcpy_d2h(lq_ctx* ctx, void* dst, const void* src, size_t bytes) {
    LQ_ENTRY(ctx, "lq_memcpy_d2h");
    if (!bytes) return LQ_OK;
    LQ_REQUIRE(ctx, dst && src, "lq_memcpy_d2h: NULL pointer");
    LQ_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return LQ_OK;
}

int lq_memset(lq_ctx* ctx, void* dst, int value, size_t bytes) {
    LQ_ENTRY(ctx, "lq_memset");
    if (!bytes) return LQ_OK;
    LQ_REQUIRE(ctx, dst != nullptr, "lq_memset: NULL pointer");
    LQ_CUDA(ctx, cudaMemsetAsync(dst, value, bytes, ctx->stream));
    return LQ_OK;
}

}  // extern "C"
