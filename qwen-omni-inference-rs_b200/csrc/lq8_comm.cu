// lq8_comm.cu -- NCCL communicator for tensor parallelism (one process per GPU).
//
// NCCL is opened at run time (dlopen of libnccl.so.2): the library loads without it, and a
// process that already loaded NCCL (PyTorch's) shares that copy. The bootstrap is NCCL's own:
// rank 0 makes a unique id (lq_comm_unique_id), the host side hands it to the other ranks
// (e.g. torch.distributed over gloo), every rank calls lq_comm_init. Collectives run on the
// context's stream, so they order with the kernels and can be captured in the decode graph.
#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_internal.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

struct lq_comm {
    lq_ctx* ctx = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
};

namespace lq {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

static NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
                 api.error_string;
    });
    return api;
}

static int nccl_check(lq_ctx* ctx, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return LQ_OK;
    return set_error(ctx, LQ_ERR_NCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

// (callers pass a valid communicator)
int comm_allreduce_sum_f32(lq_comm* c, const float* send, float* recv, int64_t count) {
    if (c->world == 1) {
        if (send != recv)
            LQ_CUDA(c->ctx, cudaMemcpyAsync(recv, send, (size_t)count * 4, cudaMemcpyDeviceToDevice, c->ctx->stream));
        return LQ_OK;
    }
    return nccl_check(c->ctx, nccl().all_reduce(send, recv, (size_t)count, ncclFloat32, ncclSum, c->comm, c->ctx->stream),
                      "ncclAllReduce");
}

int comm_allreduce_max_u64(lq_comm* c, unsigned long long* buf, int64_t count) {
    if (c->world == 1) return LQ_OK;
    return nccl_check(c->ctx, nccl().all_reduce(buf, buf, (size_t)count, ncclUint64, ncclMax, c->comm, c->ctx->stream),
                      "ncclAllReduce(max)");
}

int comm_allgather_f32(lq_comm* c, const float* send, float* recv, int64_t count) {
    if (c->world == 1) {
        LQ_CUDA(c->ctx, cudaMemcpyAsync(recv, send, (size_t)count * 4, cudaMemcpyDeviceToDevice, c->ctx->stream));
        return LQ_OK;
    }
    return nccl_check(c->ctx, nccl().all_gather(send, recv, (size_t)count, ncclFloat32, c->comm, c->ctx->stream),
                      "ncclAllGather");
}

// ---- one-shot all-reduce over the ranks' CUDA-IPC exchange regions (decode-sized rows) ----
//
// Each CTA owns a column slice of the rows: it stores its slice of this rank's partial sums
// into slot (parity, rank) of every rank's buffer with 16-byte peer stores, publishes them
// (system-scope fence, one counter increment per peer), waits (bounded) until every peer's CTA
// of the same index has done the same, and writes x = p_0 + p_1 + ... in rank order, so every
// rank holds the same sums. The buffer parity alternates per launch (each CTA counts its own
// launches): a rank can be at most one all-reduce ahead of a peer, so it never overwrites what
// the peer still reads.
struct ArDevice {
    float* buf[ALLREDUCE_MAX_TP];        // every rank's buffer [2][tp][ALLREDUCE_ROWS][H]
    unsigned* flags[ALLREDUCE_MAX_TP];   // every rank's counters [ALLREDUCE_CTAS]
    unsigned* done;                      // this rank's launches per CTA [ALLREDUCE_CTAS]
    int tp, rank;
};

__device__ __forceinline__ bool ar_wait(const unsigned* p, unsigned target, int* err) {
    const uint64_t t0 = global_ns();
    for (int i = 1;; i++) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if ((int)(v - target) >= 0) return true;
        if ((i & 63) == 0) {
            if (*reinterpret_cast<volatile const int*>(err) != 0) return false;
            if (global_ns() - t0 > 2000000000ull) {
                atomicCAS(err, 0, 60);
                return false;
            }
        }
    }
}

// The exchange of one launch, CTA c (column slice [c0, c0 + 4 w4)): this rank's slice of the
// partial sums into slot (parity, rank) of every rank's buffer, published by a system-scope
// fence and one counter increment per peer; then a bounded wait until every peer's CTA c has
// done the same. Leaves the launch count and the outcome in shared memory for the CTA.
__device__ __forceinline__ void ar_exchange(const float* __restrict__ part, int rows, int H, const ArDevice& a,
                                            int* err, int c, int c0, int w4, unsigned& sdone, int& ok) {
    const int T = a.tp;
    if (threadIdx.x == 0) sdone = a.done[c];
    __syncthreads();
    const unsigned done = sdone;
    const size_t slot = (size_t)ALLREDUCE_ROWS * H;  // floats per (parity, source rank)
    const size_t mine = ((size_t)(done & 1u) * T + a.rank) * slot;
    for (int i = threadIdx.x; i < rows * w4; i += blockDim.x) {
        const int r = i / w4, col = c0 + 4 * (i % w4);
        const float4 v = *reinterpret_cast<const float4*>(part + (size_t)r * H + col);
#pragma unroll
        for (int t = 0; t < ALLREDUCE_MAX_TP; t++)
            if (t < T) *reinterpret_cast<float4*>(a.buf[t] + mine + (size_t)r * H + col) = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();  // this CTA's peer stores, ordered before by the barrier
#pragma unroll
        for (int t = 0; t < ALLREDUCE_MAX_TP; t++)
            if (t < T && t != a.rank) asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.flags[t] + c) : "memory");
        ok = ar_wait(a.flags[a.rank] + c, (done + 1u) * (unsigned)(T - 1), err) ? 1 : 0;
        if (ok) a.done[c] = done + 1u;
    }
    __syncthreads();
}

// x[r][col] for one item (4 columns): the partial sums of every rank added in rank order
__device__ __forceinline__ float4 ar_sum(const ArDevice& a, int H, unsigned done, int r, int col) {
    const int T = a.tp;
    const size_t slot = (size_t)ALLREDUCE_ROWS * H;
    const float* b = a.buf[a.rank] + (size_t)(done & 1u) * T * slot;
    float4 v = __ldcg(reinterpret_cast<const float4*>(b + (size_t)r * H + col));
    for (int t = 1; t < T; t++) {
        const float4 u = __ldcg(reinterpret_cast<const float4*>(b + (size_t)t * slot + (size_t)r * H + col));
        v.x = __fadd_rn(v.x, u.x);
        v.y = __fadd_rn(v.y, u.y);
        v.z = __fadd_rn(v.z, u.z);
        v.w = __fadd_rn(v.w, u.w);
    }
    return v;
}

__global__ void __launch_bounds__(256) xchg_allreduce_kernel(const float* __restrict__ part, int rows, int H,
                                                               float* __restrict__ x, ArDevice a, int* err) {
    __shared__ unsigned sdone;
    __shared__ int ok;
    pdl_wait();  // the partial sums are the preceding kernel's
    const int c = blockIdx.x;
    const int per = ((H / 4 + (int)gridDim.x - 1) / (int)gridDim.x) * 4;
    const int c0 = c * per, c1 = min(H, c0 + per), w4 = max(0, c1 - c0) / 4;
    ar_exchange(part, rows, H, a, err, c, c0, w4, sdone, ok);
    pdl_trigger();
    if (!ok) return;
    for (int i = threadIdx.x; i < rows * w4; i += blockDim.x) {
        const int r = i / w4, col = c0 + 4 * (i % w4);
        *reinterpret_cast<float4*>(x + (size_t)r * H + col) = ar_sum(a, H, sdone, r, col);
    }
}

// The same all-reduce fused with the RMSNorm + Q8_0 quantization that follows it in the layer
// (post-attention norm after o_proj, the next layer's input norm or the final norm after down;
// rms_norm.rs:123-177). The 32 CTAs own column slices of whole Q8_0 blocks (H % 1024 == 0).
// Each CTA writes its slice of x, adds its slice's squares of the bf16-rounded values (items of 4
// in order, then the items in column order) into a per-row partial, and joins a counter of the
// launch's CTAs (bounded wait; every CTA of the launch is resident: 32 small CTAs). Every CTA then
// adds the 32 partials of a row in CTA order, so all use the same sum, and writes its slice of
// bf16(bf16(x) * inv_rms * w) as Q8_0 blocks. The sum is grouped differently from the unfused
// RMSNorm kernel's (a tolerance-level difference).
struct ArNorm {
    const uint16_t* w;   // [H] bf16 norm weights
    float eps;
    int8_t* xq;          // [rows][H]
    uint16_t* xd;        // [rows][H / 32] fp16
    float* sq;           // [2][ALLREDUCE_ROWS][ALLREDUCE_CTAS] per-row partial sums (this rank)
    unsigned* cnt;       // arrivals of the launches' CTAs (monotonic)
    unsigned* ndone;     // fused launches per CTA [ALLREDUCE_CTAS]
};

constexpr int ARN_ITEMS = 2;  // items of 4 columns per thread (8 rows x H/128 items <= 512)

__global__ void __launch_bounds__(256) xchg_allreduce_norm_kernel(const float* __restrict__ part, int rows, int H,
                                                                    float* __restrict__ x, ArDevice a, ArNorm n,
                                                                    int* err) {
    __shared__ unsigned sdone;
    __shared__ int ok, nok;
    __shared__ float sqi[256 * ARN_ITEMS];
    __shared__ float inv[ALLREDUCE_ROWS];
    pdl_wait();  // the partial sums are the preceding kernel's
    const int c = blockIdx.x, C = (int)gridDim.x, tid = threadIdx.x;
    const int per = H / C, c0 = c * per, w4 = per / 4, items = rows * w4;
    ar_exchange(part, rows, H, a, err, c, c0, w4, sdone, ok);
    pdl_trigger();
    const unsigned nd = n.ndone[c];  // the same count in every CTA of the launch
    float4 v[ARN_ITEMS];
#pragma unroll
    for (int k = 0; k < ARN_ITEMS; k++) {
        const int i = tid + 256 * k;
        v[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < items) {
            const int r = i / w4, col = c0 + 4 * (i % w4);
            if (ok) v[k] = ar_sum(a, H, sdone, r, col);
            *reinterpret_cast<float4*>(x + (size_t)r * H + col) = v[k];
            const float e0 = round_bf16(v[k].x), e1 = round_bf16(v[k].y), e2 = round_bf16(v[k].z), e3 = round_bf16(v[k].w);
            float q = __fmul_rn(e0, e0);
            q = __fadd_rn(q, __fmul_rn(e1, e1));
            q = __fadd_rn(q, __fmul_rn(e2, e2));
            q = __fadd_rn(q, __fmul_rn(e3, e3));
            sqi[i] = q;
        }
    }
    __syncthreads();
    float* sq = n.sq + (size_t)(nd & 1u) * ALLREDUCE_ROWS * ALLREDUCE_CTAS;
    if (tid < rows) {
        float ss = 0.0f;
        for (int k = 0; k < w4; k++) ss = __fadd_rn(ss, sqi[tid * w4 + k]);
        __stcg(sq + tid * ALLREDUCE_CTAS + c, ss);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(n.cnt) : "memory");
        const unsigned target = (nd + 1u) * (unsigned)C;
        const uint64_t t0 = global_ns();
        nok = 1;
        for (int it = 1;; it++) {
            unsigned got;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(got) : "l"(n.cnt) : "memory");
            if ((int)(got - target) >= 0) break;
            if ((it & 63) == 0 && global_ns() - t0 > 2000000000ull) {
                atomicCAS(err, 0, 61);
                nok = 0;
                break;
            }
        }
        n.ndone[c] = nd + 1u;
    }
    __syncthreads();
    if (!ok || !nok) return;
    if (tid < rows) {
        float tot = 0.0f;
        for (int q = 0; q < C; q++) tot = __fadd_rn(tot, __ldcg(sq + tid * ALLREDUCE_CTAS + q));
        const float mean = __fdiv_rn(tot, (float)H);
        inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, n.eps)));
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < ARN_ITEMS; k++) {
        const int i = tid + 256 * k;  // 8 consecutive items = one Q8_0 block (w4 % 8 == 0)
        const bool valid = i < items;
        float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int r = valid ? i / w4 : 0, col = c0 + 4 * (valid ? i % w4 : 0);
        if (valid) {
            const uint2 wt = *reinterpret_cast<const uint2*>(n.w + col);
            const float wv[4] = {bf16_to_f32((uint16_t)(wt.x & 0xFFFF)), bf16_to_f32((uint16_t)(wt.x >> 16)),
                                 bf16_to_f32((uint16_t)(wt.y & 0xFFFF)), bf16_to_f32((uint16_t)(wt.y >> 16))};
            const float e[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
            for (int j = 0; j < 4; j++)
                o[j] = bf16_to_f32(f32_to_bf16(__fmul_rn(__fmul_rn(round_bf16(e[j]), inv[r]), wv[j])));
        }
        if (256 * k < items) {  // uniform per warp group of 8: every lane joins the shuffles
            const size_t e0 = (size_t)r * H + col;
            const uint32_t q = quant_group8(o, tid & 7, valid ? n.xd + (e0 >> 5) : nullptr);
            if (valid) *reinterpret_cast<uint32_t*>(n.xq + e0) = q;
        }
    }
}

int launch_xchg_allreduce(lq_ctx* ctx, const AllreduceRegions& ar, const float* part, int64_t rows, int64_t H,
                          float* x) {
    if (rows < 1 || rows > ALLREDUCE_ROWS || H % 4 || ar.tp < 2 || ar.tp > ALLREDUCE_MAX_TP)
        return set_error(ctx, LQ_ERR_INVALID_ARG, "all-reduce over the exchange regions: %lld rows of %lld",
                         (long long)rows, (long long)H);
    size_t fo = 0, dn = 0;
    allreduce_layout(H, ar.tp, &fo, &dn);
    ArDevice a = {};
    a.tp = ar.tp;
    a.rank = ar.rank;
    for (int t = 0; t < ar.tp; t++) {
        a.buf[t] = static_cast<float*>(ar.region[t]);
        a.flags[t] = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ar.region[t]) + fo);
    }
    a.done = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ar.region[ar.rank]) + dn);
    return launch_kernel(ctx, xchg_allreduce_kernel, dim3(ALLREDUCE_CTAS), dim3(256), 0, "xchg_allreduce", part,
                         (int)rows, (int)H, x, a, ctx->err_flag);
}

size_t allreduce_layout(int64_t H, int tp, size_t* flags_off, size_t* done_off, size_t* norm_off) {
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t bbytes = al((size_t)2 * tp * ALLREDUCE_ROWS * (size_t)H * 4);
    *flags_off = bbytes;
    *done_off = bbytes + al(ALLREDUCE_CTAS * 4);
    const size_t no = *done_off + al(ALLREDUCE_CTAS * 4);
    if (norm_off) *norm_off = no;
    // fused norm (this rank only): row partials [2][ROWS][CTAS], a counter, launches per CTA
    return no + al((size_t)2 * ALLREDUCE_ROWS * ALLREDUCE_CTAS * 4) + al(4) + al(ALLREDUCE_CTAS * 4);
}

bool xchg_allreduce_norm_supported(int64_t rows, int64_t H) {
    return rows >= 1 && rows <= ALLREDUCE_ROWS && H % (32 * ALLREDUCE_CTAS) == 0 &&
           rows * (H / ALLREDUCE_CTAS / 4) <= 256 * ARN_ITEMS && getenv("LQ_AR_NORM") != nullptr;
}

int launch_xchg_allreduce_norm(lq_ctx* ctx, const AllreduceRegions& ar, const float* part, int64_t rows, int64_t H,
                               float* x, const uint16_t* w, float eps, int8_t* xq, uint16_t* xd) {
    if (!xchg_allreduce_norm_supported(rows, H) || ar.tp < 2 || ar.tp > ALLREDUCE_MAX_TP)
        return set_error(ctx, LQ_ERR_INVALID_ARG, "fused all-reduce + RMSNorm: %lld rows of %lld", (long long)rows,
                         (long long)H);
    size_t fo = 0, dn = 0, no = 0;
    allreduce_layout(H, ar.tp, &fo, &dn, &no);
    ArDevice a = {};
    a.tp = ar.tp;
    a.rank = ar.rank;
    for (int t = 0; t < ar.tp; t++) {
        a.buf[t] = static_cast<float*>(ar.region[t]);
        a.flags[t] = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ar.region[t]) + fo);
    }
    uint8_t* mine = static_cast<uint8_t*>(ar.region[ar.rank]);
    a.done = reinterpret_cast<unsigned*>(mine + dn);
    ArNorm n = {};
    n.w = w;
    n.eps = eps;
    n.xq = xq;
    n.xd = xd;
    n.sq = reinterpret_cast<float*>(mine + no);
    const size_t sqb = ((size_t)2 * ALLREDUCE_ROWS * ALLREDUCE_CTAS * 4 + 255) & ~(size_t)255;
    n.cnt = reinterpret_cast<unsigned*>(mine + no + sqb);
    n.ndone = reinterpret_cast<unsigned*>(mine + no + sqb + 256);
    return launch_kernel(ctx, xchg_allreduce_norm_kernel, dim3(ALLREDUCE_CTAS), dim3(256), 0, "xchg_allreduce_norm",
                         part, (int)rows, (int)H, x, a, n, ctx->err_flag);
}

int comm_rank(const lq_comm* c) { return c ? c->rank : 0; }
int comm_world(const lq_comm* c) { return c ? c->world : 1; }
lq_ctx* comm_ctx(const lq_comm* c) { return c ? c->ctx : nullptr; }

}  // namespace lq

extern "C" {

int lq_comm_unique_id(lq_ctx* ctx, uint8_t* id_out) {
    LQ_ENTRY(ctx, "lq_comm_unique_id");
    LQ_REQUIRE(ctx, id_out, "lq_comm_unique_id: NULL output");
    if (!lq::nccl().ok) return lq::set_error(ctx, LQ_ERR_UNSUPPORTED, "lq_comm_unique_id: libnccl.so.2 not found");
    ncclUniqueId id;
    int rc = lq::nccl_check(ctx, lq::nccl().get_unique_id(&id), "ncclGetUniqueId");
    if (rc) return rc;
    static_assert(sizeof(ncclUniqueId) == LQ_COMM_ID_BYTES, "NCCL unique id size");
    memcpy(id_out, &id, sizeof id);
    return LQ_OK;
}

int lq_comm_init(lq_ctx* ctx, const uint8_t* id, int rank, int world, lq_comm** out) {
    LQ_ENTRY(ctx, "lq_comm_init");
    LQ_REQUIRE(ctx, id && out, "lq_comm_init: NULL argument");
    LQ_REQUIRE(ctx, world >= 1 && rank >= 0 && rank < world, "lq_comm_init: rank %d of %d", rank, world);
    *out = nullptr;
    lq_comm* c = new lq_comm();
    c->ctx = ctx;
    c->rank = rank;
    c->world = world;
    if (world > 1) {
        if (!lq::nccl().ok) {
            delete c;
            return lq::set_error(ctx, LQ_ERR_UNSUPPORTED, "lq_comm_init: libnccl.so.2 not found");
        }
        ncclUniqueId uid;
        memcpy(&uid, id, sizeof uid);
        cudaSetDevice(ctx->device);
        int rc = lq::nccl_check(ctx, lq::nccl().comm_init_rank(&c->comm, world, uid, rank), "ncclCommInitRank");
        if (rc) {
            delete c;
            return rc;
        }
    }
    *out = c;
    return LQ_OK;
}

int lq_comm_destroy(lq_comm* comm) {
    if (!comm) return LQ_ERR_INVALID_ARG;
    if (comm->comm) {
        cudaStreamSynchronize(comm->ctx->stream);
        lq::nccl().comm_destroy(comm->comm);
    }
    delete comm;
    return LQ_OK;
}

int lq_comm_rank(lq_comm* comm, int* rank, int* world) {
    if (!comm || !rank || !world) return LQ_ERR_INVALID_ARG;
    *rank = comm->rank;
    *world = comm->world;
    return LQ_OK;
}

int lq_q8_0_matmul_allreduce(lq_ctx* ctx, lq_comm* comm, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                             int64_t m, float* y, const float* residual) {
    LQ_ENTRY(ctx, "lq_q8_0_matmul_allreduce");
    LQ_REQUIRE(ctx, comm && comm->ctx == ctx, "lq_q8_0_matmul_allreduce: communicator of another context");
    LQ_REQUIRE(ctx, w && w->n > 0 && w->k > 0 && w->k % 32 == 0 && w->qs && w->d,
               "lq_q8_0_matmul_allreduce: bad weight shard");
    LQ_REQUIRE(ctx, m >= 0 && (m == 0 || (xq && xd && y)), "lq_q8_0_matmul_allreduce: bad activations");
    if (m == 0) return LQ_OK;
    // rank 0 folds the residual into its partial; the sum over ranks is residual + x.W^T
    int rc = lq::launch_q8_matmul(ctx, w, xq, xd, m, y, comm->rank == 0 ? residual : nullptr, w->n, nullptr);
    if (rc) return rc;
    return lq::comm_allreduce_sum_f32(comm, y, y, m * w->n);
}

int lq_comm_allreduce_f32(lq_comm* comm, float* buf, int64_t count) {
    if (!comm) return LQ_ERR_INVALID_ARG;
    LQ_ENTRY(comm->ctx, "lq_comm_allreduce_f32");
    LQ_REQUIRE(comm->ctx, count >= 0 && (count == 0 || buf), "lq_comm_allreduce_f32: bad buffer");
    if (count == 0) return LQ_OK;
    return lq::comm_allreduce_sum_f32(comm, buf, buf, count);
}

}  // extern "C"
