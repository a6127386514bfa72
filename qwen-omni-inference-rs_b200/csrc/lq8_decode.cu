// lq8_decode.cu -- the whole decode step of a dense Qwen3 model (batch M <= 4) as one
// persistent kernel: every layer's q|k|v GEMV, attention, o GEMV, gate|up GEMV and down GEMV,
// then the LM head with the greedy argmax keys.
//
// One CTA per SM (cooperative launch, so every CTA is resident). Its producer warp streams the
// tiles of every weight matrix of the step, in step order, into an 8-stage shared-memory ring:
// a stage is 16 rows x up to 1 KiB of K plus their fp16 scales (17 KiB), two 2-D TMA boxes (the
// weights viewed as 8-byte elements, so one box carries 16 x 1 KiB). The producer never waits
// for activations: while the consumer warps sit at a grid barrier or in attention, the ring
// fills with the next matrix's tiles, so HBM keeps streaming across the phase boundaries that
// separate kernels elsewhere.
//
// The consumer warps walk the phases, with a grid barrier (a global counter, bounded spin;
// split into arrive and wait where work that reads nothing of other CTAs fits in between)
// wherever a phase reads what other CTAs wrote:
//   QKV  RMSNorm + Q8_0 of x (every CTA, redundantly), q|k|v rows                      | barrier
//   ATT  runs of 64-position chunks of one (row, kv head): q/k RMSNorm + RoPE once per run,
//        the new position's k/v appended to the caches, per chunk scores, softmax, P.V ->
//        published partials; then merge tasks (row, q head), taken by CTAs out of runs, each
//        waiting for its kv head's chunks: merge, Q8_0 of the head's output             | barrier
//   O    o rows + residual -> x                                                       | barrier
//   GU   RMSNorm prologue, gate|up rows, SiLU(gate)*up -> h, quantized per unit      | barrier
//   DN   h (Q8_0) as activations, down rows + residual -> x                           | barrier
//   LM   final RMSNorm, LM-head rows -> logits, greedy argmax keys
// GEMV units (16 output rows; 32 for gate|up, one Q8_0 block of h) are dealt to CTAs
// round-robin over one sequence that runs through all phases, so the CTAs' totals differ by
// one unit; the producer tags each stage with its unit and closes each phase with a marker
// stage. Attention runs are dealt statically (CTA c: runs c, c + gridDim.x, ...).
// Every arithmetic step is the one of the five-kernel decode path (the same row functions,
// the same per-lane block order and warp sums, the same attention order), so the logits are
// bit-identical to it. Data written by other CTAs is read through L2 (ld.cg / cp.async.cg).
#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_internal.cuh"
#include "lq8_tma.cuh"

#include <algorithm>
#include <cstdlib>
#include <vector>

namespace lq {

constexpr int PD_ROWS = 16;  // weight rows per stage (two per consumer warp)
constexpr int PD_KC = 1024;  // K bytes per stage (one Q8_0 block per lane and row)
constexpr int PD_STAGE = PD_ROWS * PD_KC + PD_ROWS * (PD_KC / 32) * 2;  // 17 KiB
constexpr int PD_MAX_STAGES = 8;  // ring depth: PdParams::ns stages (3..8, what shared memory allows)
constexpr int PD_CONS = 8;
constexpr int PD_CTHREADS = PD_CONS * 32;
constexpr int PD_THREADS = PD_CTHREADS + 32;
constexpr int PD_ATT_C = 64;
constexpr int PD_KS = 128 + 4;  // padded K row (floats): conflict-free float4 reads
constexpr int PD_MAX_SPLITS = 128;
constexpr int PD_MAX_G = 8;
constexpr int PD_MAX_M = 8;  // batch rows of one step (GEMV output lanes 8r + m: m < 8)
constexpr int PD_MAX_TP = 8;
constexpr int PD_XPAD = 32;  // batches of 5-8: activation row padding (conflict-free MMA token fragments)  // tensor-parallel ranks whose exchange slots a step addresses
constexpr uint64_t PD_WAIT_NS = 2000000000ull;

// one weight matrix: its Q8_0 rows viewed as [N][K/8] 8-byte elements and its scales [N][K/32]
struct alignas(64) PdMat {
    CUtensorMap wq;
    CUtensorMap wd;
    CUtensorMap wsw;  // the rows as bytes in [16][128 B] boxes with the 128-byte swizzle (batches 5-8)
};

// the device descriptor of one layer; the LM head is mat[0] of the entry after the last layer
struct alignas(64) PdLayer {
    PdMat mat[4];  // q|k|v, o, gate|up, down
    const uint16_t *in_norm, *post_norm, *q_norm, *k_norm;
    float *kc, *vc;  // [M][Hkv][ctx_max][128]
};

struct PdParams {
    const PdLayer* layers;  // [n_layers + 1]
    int n_layers;
    const uint16_t* final_norm;
    int H, Hq, Hkv, I, V, Nqkv, ctx_max;
    float eps;
    const float* cos_t;
    const float* sin_t;
    const int32_t* pos_dev;
    float* x;                  // [M][H]
    float* qkv;                // [M][Nqkv]
    int8_t* att_q;             // [M][Hq*128]
    uint16_t* att_d;
    int8_t* hq;                // [M][I] Q8_0 of SiLU(gate)*up
    uint16_t* hd;              // [M][I/32]
    float* part_o;             // [M][Hq][PD_MAX_SPLITS][128]
    float* part_ml;            // [M][Hq][PD_MAX_SPLITS][2]
    float* logits;             // [M][V]
    unsigned long long* keys;  // [M]
    unsigned* bar;             // [0] grid barrier, [1 + b*Hkv + kvh] published-chunk counters;
                               // zero at launch
    int* err;
    int ns;                    // ring stages
    int ring_off;              // byte offset of the ring in shared memory
    // tensor parallelism (tp > 1): o and down are row-parallel; each CTA pushes the partial
    // sums of its units to every rank's exchange buffer and adds all ranks' partials in rank
    // order (the same units fall to the same CTA index on every rank); the LM head's argmax
    // keys (global vocabulary index) go to every rank by 64-bit atomic max
    int tp, rank, vbase;
    float* xpeer[PD_MAX_TP];               // exchange buffers [2][tp][H/16][8 warps][16]
    unsigned* fpeer[PD_MAX_TP];            // counters [gridDim.x] per CTA, then [1] for the keys
    unsigned long long* kpeer[PD_MAX_TP];  // argmax keys [M] of every rank
    float* xself;                          // xpeer[rank]
    unsigned* fself;                       // fpeer[rank]
    unsigned* seq;                         // [0] exchanges and [1] steps completed before this one
};

// attention staging (the union area during ATT)
struct PdAtt {
    float ks[PD_ATT_C][PD_KS];
    float vs[PD_ATT_C][128];
    float qraw[PD_MAX_G][128];
    float qs[PD_MAX_G][PD_KS];  // padded like ks: the lanes of different heads hit different banks
    float kvraw[2][128];
    float knew[128];  // the new position's normed, rotated k
    uint16_t qn[128], kn[128];  // the layer's q/k RMSNorm weights (bf16)
    float cs[64], sn[64];       // the RoPE cos/sin row of the new position
    float ps[PD_MAX_G][PD_ATT_C + 4];  // padded: heads g and g' read position j in different banks
    float ml[PD_MAX_G][2];
    float cm[PD_MAX_G][PD_MAX_SPLITS];
    float cl[PD_MAX_G];
};

// 128-byte multiple: the union area behind it takes 16-byte vector and cp.async accesses
struct alignas(128) PdSmem {
    uint64_t full[PD_MAX_STAGES];
    uint64_t empty[PD_MAX_STAGES];
    float red[32];
    unsigned long long keys[PD_MAX_M];
    int tag[PD_MAX_STAGES];  // the unit a stage belongs to (-1: the phase has no more units for us)
    uint64_t hfull[2];     // gate|up: hbuf[b] written by the 8 consumer warps
    uint64_t hfree[2];     // gate|up: hbuf[b] quantized by warp 0
    float hbuf[2][PD_MAX_M][32];  // gate|up: one Q8_0 block of SiLU(gate)*up per row (two units in turn)
    int flag;  // grid barrier outcome
    int fail;  // a consumer warp gave up waiting for a stage
    int ns;        // ring stages
    int ring_off;  // byte offset of the ring (1024-aligned for the swizzled boxes of batches 5-8)
    uint64_t rfull[2];  // batches of 5-8: partial-sum buffer b written by the 8 consumer warps
    uint64_t rfree[2];  // ... and read by them
    // followed by the ring (ns stages of PD_STAGE bytes), then the union area: the GEMV
    // activations or PdAtt
};

__device__ __forceinline__ uint8_t* pd_align128(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 127) & ~(uintptr_t)127);
}

// the dynamic shared memory: PdSmem, the ring, the union area
extern __shared__ __align__(1024) uint8_t pd_dsmem[];
// a position in the ring, carried from stage to stage (no division by the run-time depth on the
// path of every stage): count of stages passed, slot, and the slot's mbarrier phase parity
struct PdRing {
    int it;
    int s;
    unsigned ph;
};
__device__ __forceinline__ void pd_next(PdRing& r, int ns) {
    r.it++;
    if (++r.s == ns) {
        r.s = 0;
        r.ph ^= 1u;
    }
}
__device__ __forceinline__ uint8_t* pd_ring(const PdSmem& S) { return pd_dsmem + S.ring_off; }
// batches of 5-8: the warps' partial sums of one 16-row group, two groups in turn (in the union
// area, after the GEMV activations)
typedef float PdRed[2][PD_CONS][PD_ROWS][8];

static_assert(sizeof(PdSmem) % 128 == 0 && PD_STAGE % 1024 == 0,
              "regions must stay 128-byte aligned, ring stages 1024-byte aligned (swizzled boxes)");

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DN = 3, PH_LM = 4 };

struct PdGemv {
    const PdMat* mat;
    int N, K;
    bool swi;
};

__device__ __forceinline__ PdGemv pd_gemv(const PdParams& p, int layer, int kind) {
    PdGemv g;
    g.swi = false;
    if (kind == PH_LM) {
        g.mat = &p.layers[p.n_layers].mat[0];
        g.N = p.V;
        g.K = p.H;
        return g;
    }
    g.mat = &p.layers[layer].mat[kind];
    switch (kind) {
        case PH_QKV: g.N = p.Nqkv; g.K = p.H; break;
        case PH_O: g.N = p.H; g.K = p.Hq * 128; break;
        case PH_GU: g.N = 2 * p.I; g.K = p.H; g.swi = true; break;
        default: g.N = p.H; g.K = p.I; break;
    }
    return g;
}

// a unit is PD_ROWS output rows; for gate|up 32 outputs (one Q8_0 block of h): two groups of
// 16 rows, each as its gate rows and then its up rows
__device__ __forceinline__ int pd_unit_rows(const PdGemv& g) { return g.swi ? 2 * PD_ROWS : PD_ROWS; }
__device__ __forceinline__ int pd_units(const PdGemv& g) {
    const int nout = g.swi ? g.N / 2 : g.N;
    return (nout + pd_unit_rows(g) - 1) / pd_unit_rows(g);
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// bounded mbarrier wait that also gives up once another CTA has flagged an error
__device__ __forceinline__ bool pd_wait(uint64_t* bar, unsigned parity, const int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (int i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 0 && (ld_volatile(err) != 0 || global_ns() - t0 > PD_WAIT_NS)) return false;
    }
}

// the first unit of this CTA in a phase whose units start at position `off` of the sequence
__device__ __forceinline__ int pd_first(unsigned off) {
    const unsigned G = gridDim.x;
    return (int)((blockIdx.x + G - off % G) % G);
}

// ---- producer: the units of one GEMV phase dealt to this CTA, their tiles streamed ----
// (Claiming units from a counter instead balanced worse: the producers claim ahead by up to a
// ring of tiles, so the first CTAs to reach a phase took most of its units.)
__device__ __forceinline__ bool pd_produce(PdSmem& S, const PdGemv& g, unsigned off, PdRing& r, int* err, bool sw) {
    const int K = g.K;
    const int kc = K < PD_KC ? K : PD_KC;
    const int nchunks = (K + kc - 1) / kc;
    const int nout = g.swi ? g.N / 2 : g.N;
    const int units = pd_units(g);
    const int halves = g.swi ? 2 : 1;
    const unsigned bytes = (unsigned)(PD_ROWS * kc + PD_ROWS * (kc / 16));  // whole boxes (OOB zero-filled)
    const int ns = S.ns;
    uint8_t* const ring = pd_ring(S);
    for (int u = pd_first(off);; u += gridDim.x) {
        const int s0 = r.s;
        if (u >= units) {
            // phase end marker: a stage without data
            if (!pd_wait(&S.empty[s0], r.ph ^ 1u, err)) {
                atomicCAS(err, 0, 41);
                return false;
            }
            S.tag[s0] = -1;
            mbar_arrive(&S.full[s0]);
            pd_next(r, ns);
            return true;
        }
        for (int grp = 0; grp < halves; grp++)
            for (int half = 0; half < halves; half++) {
                const int r0 = half * nout + u * pd_unit_rows(g) + grp * PD_ROWS;
                for (int c = 0; c < nchunks; c++, pd_next(r, ns)) {
                    const int s = r.s;
                    if (!pd_wait(&S.empty[s], r.ph ^ 1u, err)) {
                        atomicCAS(err, 0, 41);
                        return false;
                    }
                    uint8_t* st = ring + (size_t)s * PD_STAGE;
                    S.tag[s] = u;
                    if (sw) {
                        // one swizzled box per 128 bytes of K that exist (the consumers skip the rest)
                        const int nbox = min(kc, K - c * kc) / 128;
                        mbar_expect_tx(&S.full[s], (unsigned)(nbox * PD_ROWS * 128 + PD_ROWS * (kc / 16)));
                        for (int b = 0; b < nbox; b++)
                            tma_load_2d(st + b * (PD_ROWS * 128), &g.mat->wsw, c * kc + b * 128, r0, &S.full[s]);
                    } else {
                        mbar_expect_tx(&S.full[s], bytes);
                        tma_load_2d(st, &g.mat->wq, c * (kc / 8), r0, &S.full[s]);
                    }
                    tma_load_2d(st + PD_ROWS * kc, &g.mat->wd, c * (kc / 32), r0, &S.full[s]);
                }
            }
    }
}

// ---- consumers ----
__device__ __forceinline__ void pd_csync() { group_sync<PD_CTHREADS, 1>(); }

// grid barrier of the consumer groups, split in two: pd_grid_arrive publishes this CTA's
// writes (release) and counts it in; pd_grid_wait returns once every CTA has arrived (the k-th
// barrier completes when the counter reaches k * gridDim.x). Work that depends on no other
// CTA's writes may run between the two. The wait returns false when it gave up (~2 s) or
// another CTA flagged an error.
__device__ __forceinline__ void pd_grid_arrive(const PdParams& p, unsigned& epoch) {
    pd_csync();
    epoch++;
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
}

__device__ __forceinline__ bool pd_grid_wait(const PdParams& p, PdSmem& S, unsigned epoch) {
    if (threadIdx.x == 0) {
        const unsigned target = epoch * gridDim.x;
        const uint64_t t0 = global_ns();
        int ok = 1;
        for (int i = 1;; i++) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.bar) : "memory");
            if (v >= target) break;
            if ((i & 63) == 0) {
                if (ld_volatile(p.err) != 0) { ok = 0; break; }
                if (global_ns() - t0 > PD_WAIT_NS) { atomicCAS(p.err, 0, 42); ok = 0; break; }
            }
        }
        S.flag = ok;
    }
    pd_csync();
    return S.flag != 0;
}

__device__ __forceinline__ bool pd_grid_barrier(const PdParams& p, PdSmem& S, unsigned& epoch) {
    pd_grid_arrive(p, epoch);
    return pd_grid_wait(p, S, epoch);
}

// `bytes` (a multiple of 16) into shared memory through L2 with every 16-byte copy in flight;
// completes at the next cp_async_wait
__device__ __forceinline__ void pd_prefetch(void* dst, const void* src, int bytes, int tid) {
    for (int i = tid * 16; i < bytes; i += PD_CTHREADS * 16)
        cp_async16(static_cast<uint8_t*>(dst) + i, static_cast<const uint8_t*>(src) + i, true);
    cp_async_commit();
}

// f32 values written by other CTAs into shared memory through L2, every 16-byte copy in
// flight at once (one round trip); the caller syncs the consumers before reading dst
__device__ __forceinline__ void pd_stage_f32(float* dst, const float* src, int n, int tid) {
    for (int i = tid * 4; i < n; i += PD_CTHREADS * 4) cp_async16(dst + i, src + i, true);
    cp_async_commit();
    cp_async_wait<0>();
}

// Q8_0 of 32 values, one per lane (GGML's block quantization: d = amax/127, q = round(v/d))
__device__ __forceinline__ void pd_quant_warp32(float v, int lane, int8_t* q_out, uint16_t* d_out) {
    const float amax = warp_max(fabsf(v));
    float d, id;
    q8_scale(amax, d, id);
    q_out[lane] = (int8_t)q8_quant(v, id);
    if (lane == 0) *d_out = f2h(d);
}

// The integer sum of a Q8_0 block, w . x over 32 int8 pairs. Lanes 4-7 of each quarter-warp
// read the second 16 bytes first (sw = 1) and pair them with the same half of the other
// operand: the 16-byte shared-memory reads of a quarter-warp then cover all 32 banks once,
// and the (exact, integer) sum is the same in either order.
__device__ __forceinline__ int pd_block_sum(const int4 wa, const int4 wb, const int4 xa, const int4 xb) {
    int sum = 0;
    sum = __dp4a(wa.x, xa.x, sum); sum = __dp4a(wa.y, xa.y, sum);
    sum = __dp4a(wa.z, xa.z, sum); sum = __dp4a(wa.w, xa.w, sum);
    sum = __dp4a(wb.x, xb.x, sum); sum = __dp4a(wb.y, xb.y, sum);
    sum = __dp4a(wb.z, xb.z, sum); sum = __dp4a(wb.w, xb.w, sum);
    return sum;
}

// the residual a consumer lane adds in unit u of a phase with nout outputs (lane 8r + m: row
// 2w + r, token m); 0 for lanes without an output and for units past the phase's end
template <int M>
__device__ __forceinline__ float pd_res_lane(const float* out, int ldo, int nout, int u) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = u * PD_ROWS + 2 * warp + (lane >> 3);
    if (lane < 16 && (lane & 7) < M && row < nout) return __ldcg(out + (size_t)(lane & 7) * ldo + row);
    return 0.0f;
}

// the units of one GEMV phase that this CTA's producer claimed, against the activations
// xs/xds in shared memory: out[m][row] (+ the residual already in out), logits + argmax keys,
// or h = SiLU(gate)*up quantized to Q8_0 (hq, hd).
// A stage holds 16 rows x kc (<= 1 KiB) of K; warp w takes rows 2w and 2w+1 against one read
// of the activations, lane l block l of the chunk. Per output the lane accumulates the blocks
// l, 32+l, 64+l, ... in order and a butterfly sums the lanes: the decode GEMV's order.
// hn counts this CTA's gate|up units over the whole step (it indexes the h handoff buffers).
template <int M>
__device__ __forceinline__ bool pd_consume(PdSmem& S, const PdGemv& g, const int8_t* xs, const uint16_t* xds,
                                           PdRing& r, int& hn, float* out, int ldo, bool resid, bool keys,
                                           int8_t* hq, uint16_t* hd, int* err, int u_first = -1,
                                           float res_first = 0.0f, const PdParams* xp = nullptr, int xpar = 0,
                                           int kbase = 0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sw = (lane >> 2) & 1;
    const int K = g.K, nb = K >> 5;
    const int kc = K < PD_KC ? K : PD_KC;
    const int nchunks = (K + kc - 1) / kc;
    const int nout = g.swi ? g.N / 2 : g.N;
    const int halves = g.swi ? 2 : 1;
    const int ns = S.ns;
    const uint8_t* const ring = pd_ring(S);
    float acc[2][M], gate[2][M];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[r][m] = gate[r][m] = 0.0f;
    // a warp that gives up waiting leaves the phase at once; every warp then meets the others
    // at the closing consumer barrier (all waits below are bounded)
    bool failed = false;
    auto wait_full = [&](int s) {
        int ok = 1;
        if (lane == 0) ok = pd_wait(&S.full[s], r.ph, err);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();  // the other lanes read the stage after lane 0 saw it complete
        if (!ok) {
            if (lane == 0) {
                atomicCAS(err, 0, 43);
                S.fail = 1;
            }
            failed = true;
        }
        return ok != 0;
    };
    while (!failed) {
        const int s0 = r.s;
        if (!wait_full(s0)) break;
        int u = 0;
        if (lane == 0) u = S.tag[s0];
        u = __shfl_sync(0xffffffffu, u, 0);
        if (u < 0) {  // no more units: release the marker stage
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s0]);
            pd_next(r, ns);
            break;
        }
        const int hb = hn & 1, huse = hn >> 1;
        if (g.swi && huse > 0) {  // warp 0 is done with this buffer's previous unit
            int ok = 1;
            if (lane == 0) ok = pd_wait(&S.hfree[hb], (unsigned)(huse - 1) & 1u, err);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(err, 0, 45);
                    S.fail = 1;
                }
                failed = true;
            }
        }
        // the residual of the output this lane writes: loaded ahead (the caller loads the first
        // unit's before the phase, each unit the next one's), so no unit waits on its L2 round
        // trip; units arrive in the dealt order u_first, u_first + gridDim.x, ...
        float res = 0.0f;
        if (resid && !g.swi) {
            res = u == u_first ? res_first : pd_res_lane<M>(out, ldo, nout, u);
            u_first = u + (int)gridDim.x;
            res_first = pd_res_lane<M>(out, ldo, nout, u_first);
        }
        for (int grp = 0; grp < halves && !failed; grp++)
        for (int half = 0; half < halves && !failed; half++) {
            const int r0 = u * pd_unit_rows(g) + grp * PD_ROWS;
            const int rows = min(PD_ROWS, nout - r0);
            for (int c = 0; c < nchunks; c++, pd_next(r, ns)) {
                const int s = r.s;
                if ((grp | half | c) != 0 && !wait_full(s)) break;
                const int k0 = c * kc, nbc = min(kc, K - k0) >> 5;
                const bool act = lane < nbc;
                const int8_t* wst = reinterpret_cast<const int8_t*>((ring + (size_t)s * PD_STAGE)) + (2 * warp) * kc + lane * 32;
                const uint16_t* dst = reinterpret_cast<const uint16_t*>((ring + (size_t)s * PD_STAGE) + PD_ROWS * kc) + (2 * warp) * (kc / 32) + lane;
                int4 w[2][2];
                float dw[2] = {0.f, 0.f};
                if (act) {
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        w[r][0] = *reinterpret_cast<const int4*>(wst + r * kc + sw * 16);
                        w[r][1] = *reinterpret_cast<const int4*>(wst + r * kc + (sw ^ 1) * 16);
                        dw[r] = h2f(dst[r * (kc / 32)]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[s]);
                if (act) {
                    const int gb = (k0 >> 5) + lane;
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)m * K + (size_t)gb * 32);
                        const int4 xa = xp[sw], xb = xp[sw ^ 1];
                        const float dx = h2f(xds[(size_t)m * nb + gb]);
#pragma unroll
                        for (int r = 0; r < 2; r++) {
                            const int sum = pd_block_sum(w[r][0], w[r][1], xa, xb);
                            acc[r][m] = __fadd_rn(acc[r][m], __fmul_rn((float)sum, __fmul_rn(dw[r], dx)));
                        }
                    }
                }
                if (c == nchunks - 1) {
                    float xv[2][M];  // the unit's partial sums when they go to the exchange
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        const int rr = 2 * warp + r, row = r0 + rr;
#pragma unroll
                        for (int m = 0; m < M; m++) {
                            const float v = warp_sum(acc[r][m]);
                            acc[r][m] = 0.0f;
                            xv[r][m] = v;
                            if (g.swi) {
                                if (half == 0) gate[r][m] = v;
                                else if (lane == 0) S.hbuf[hb][m][grp * PD_ROWS + rr] = swiglu(gate[r][m], v);
                            } else if (rr < rows && !xp) {
                                if (lane == 8 * r + m) {
                                    const size_t o = (size_t)m * ldo + row;
                                    out[o] = resid ? __fadd_rn(res, v) : v;
                                }
                                if (keys && lane == 8 * r) atomicMax(&S.keys[m], argmax_key(v, row + kbase));
                            }
                        }
                    }
                    if (xp) {
                        // this warp's 2 rows x M tokens, 16 floats [token][row] at (unit, warp) of
                        // every rank's slot: lane q stores tokens 2q and 2q+1 as one 16-byte vector
#pragma unroll
                        for (int q = 0; q < (M + 1) / 2; q++) {
                            if (lane == q) {
                                const bool has1 = 2 * q + 1 < M;
                                const int m1 = has1 ? 2 * q + 1 : 2 * q;
                                const float4 f = make_float4(xv[0][2 * q], xv[1][2 * q], has1 ? xv[0][m1] : 0.0f,
                                                             has1 ? xv[1][m1] : 0.0f);
                                const size_t slot = (size_t)(g.N / PD_ROWS) * PD_CONS * 16;
                                const size_t off = ((size_t)xpar * xp->tp + xp->rank) * slot +
                                                   ((size_t)u * PD_CONS + warp) * 16 + 4 * q;
#pragma unroll
                                for (int t = 0; t < PD_MAX_TP; t++)
                                    if (t < xp->tp) *reinterpret_cast<float4*>(xp->xpeer[t] + off) = f;
                            }
                        }
                    }
                }
            }
        }
        if (g.swi && !failed) {
            // the unit's 32 outputs are one Q8_0 block of h per row (quant_row's arithmetic):
            // every warp hands its values over, warp 0 quantizes
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.hfull[hb]);
            if (warp == 0) {
                int ok = 1;
                if (lane == 0) ok = pd_wait(&S.hfull[hb], (unsigned)huse & 1u, err);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                __syncwarp();
                if (ok) {
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        const size_t e = (size_t)m * nout + (size_t)u * 32;
                        pd_quant_warp32(S.hbuf[hb][m][lane], lane, hq + e, hd + (e >> 5));
                    }
                } else if (lane == 0) {
                    atomicCAS(err, 0, 46);
                    S.fail = 1;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.hfree[hb]);
            }
        }
        if (g.swi) hn++;
    }
    pd_csync();
    return S.fail == 0;
}

// Batches of 5-8 rows on the tensor cores. The dp4a consumer above reads the activations of
// every token once per 2 weight rows, so at 8 tokens shared memory, not HBM, sets its pace;
// here each warp runs int8 MMAs that reuse a weight fragment across the 8 tokens and a token
// fragment across the 16 rows. The stage arrives as kc/128 boxes of [16 rows][128 B] with the
// 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7)); box w holds Q8_0 blocks
// 4w..4w+3 of the chunk and belongs to warp w. Per block one mma.sync m16n8k32 (s8; rows x
// tokens), its accumulator starting at 1.5*2^23 so the int32 dot read as a float is
// 1.5*2^23 + dot, then dot*(d_w*d_x) added per (row, token) with separately rounded operations
// in block order. At the end of each 16-row group the eight warps' partial sums meet in shared
// memory (double-buffered: one consumer barrier per group) and warp w finishes rows 2w, 2w+1
// (lanes 0-3: tokens 2q, 2q+1), adding the warps' sums in warp order: the output, the
// residual, the tensor-parallel exchange push (one 16-byte vector per lane), SwiGLU with the
// h handoff of the dp4a consumer, or the argmax keys. Activation rows are ldx = K + 32 bytes
// apart in shared memory (conflict-free token fragments), or, with GX (the down phase, whose h
// rows would take the ring's room), are read from global memory (L2: other CTAs wrote them)
// straight into the token fragments, two chunks ahead of the stage they serve: a warp's chunk
// sequence in a phase is 0, 1, ..., nchunks - 1 for every unit, so the next chunk is known
// before its stage arrives.
template <int M, bool GX>
__device__ __forceinline__ bool pd_consume_mma(PdSmem& S, const PdGemv& g, const int8_t* xs, int ldx,
                                               const uint16_t* xds, PdRed* mred, PdRing& r, int& hn, int& rn,
                                               float* out, int ldo, bool resid, bool keys, int8_t* hq, uint16_t* hd,
                                               int* err, const PdParams* xp, int xpar, int kbase) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, t = lane & 3;
    const int ns = S.ns;
    const uint8_t* const ring = pd_ring(S);
    const int K = g.K, nb = K >> 5;
    const int kc = K < PD_KC ? K : PD_KC;
    const int nchunks = (K + kc - 1) / kc;
    const int nout = g.swi ? g.N / 2 : g.N;
    const int halves = g.swi ? 2 : 1;
    bool failed = false;
    // the token fragments and scales of chunk c for this lane (zeros for tokens >= M)
    struct Frag {
        uint2 xv[4], dxa, dxb;
    };
    auto load_frag = [&](int c, Frag& f) {
        const int gb0 = c * (kc >> 5) + 4 * warp;
        const bool act = 4 * warp < (min(kc, K - c * kc) >> 5);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int8_t* src = xs + (size_t)gq * ldx + (gb0 + j) * 32 + 8 * t;
            f.xv[j] = (act && gq < M) ? (GX ? __ldcg(reinterpret_cast<const uint2*>(src))
                                            : *reinterpret_cast<const uint2*>(src))
                                      : make_uint2(0u, 0u);
        }
        const uint16_t* sa = xds + (size_t)(2 * t) * nb + gb0;
        const uint16_t* sb = sa + nb;
        f.dxa = (act && 2 * t < M) ? (GX ? __ldcg(reinterpret_cast<const uint2*>(sa)) : *reinterpret_cast<const uint2*>(sa))
                                   : make_uint2(0u, 0u);
        f.dxb = (act && 2 * t + 1 < M) ? (GX ? __ldcg(reinterpret_cast<const uint2*>(sb))
                                             : *reinterpret_cast<const uint2*>(sb))
                                       : make_uint2(0u, 0u);
    };
    Frag f0{}, f1{};
    if (GX) {  // the first two chunks, in flight while the first stage is awaited
        load_frag(0, f0);
        load_frag(1 % nchunks, f1);
    }
    auto wait_full = [&](int s) {
        int ok = 1;
        if (lane == 0) ok = pd_wait(&S.full[s], r.ph, err);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();
        if (!ok) {
            if (lane == 0) {
                atomicCAS(err, 0, 43);
                S.fail = 1;
            }
            failed = true;
        }
        return ok != 0;
    };
    float gate[4] = {0.f, 0.f, 0.f, 0.f};
    while (!failed) {
        const int s0 = r.s;
        if (!wait_full(s0)) break;
        int u = 0;
        if (lane == 0) u = S.tag[s0];
        u = __shfl_sync(0xffffffffu, u, 0);
        if (u < 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s0]);
            pd_next(r, ns);
            break;
        }
        const int hb = hn & 1, huse = hn >> 1;
        if (g.swi && huse > 0) {  // warp 0 is done with this buffer's previous unit
            int ok = 1;
            if (lane == 0) ok = pd_wait(&S.hfree[hb], (unsigned)(huse - 1) & 1u, err);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(err, 0, 45);
                    S.fail = 1;
                }
                failed = true;
            }
        }
        for (int grp = 0; grp < halves && !failed; grp++)
        for (int half = 0; half < halves && !failed; half++) {
            const int o0 = u * pd_unit_rows(g) + grp * PD_ROWS;  // first output of the group
            // this lane's outputs after the group: rows 2w, 2w+1 x tokens 2t, 2t+1 (lanes 0-3)
            float res[4] = {0.f, 0.f, 0.f, 0.f};
            if (resid && !xp && lane < 4) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int row = o0 + 2 * warp + (i & 1), tok = 2 * lane + (i >> 1);
                    if (tok < M && row < nout) res[i] = __ldcg(out + (size_t)tok * ldo + row);
                }
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int c = 0; c < nchunks; c++, pd_next(r, ns)) {
                const int s = r.s;
                if ((grp | half | c) != 0 && !wait_full(s)) break;
                const int k0 = c * kc, nbc = min(kc, K - k0) >> 5;
                const uint8_t* st = (ring + (size_t)s * PD_STAGE);
                const bool act = 4 * warp < nbc;
                uint2 wa[4], wb[4], swa = make_uint2(0u, 0u), swb = make_uint2(0u, 0u);
                if (act) {
                    const uint8_t* box = st + warp * (PD_ROWS * 128);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int ch = (((2 * j + (t >> 1)) ^ gq) << 4) + (t & 1) * 8;
                        wa[j] = *reinterpret_cast<const uint2*>(box + gq * 128 + ch);
                        wb[j] = *reinterpret_cast<const uint2*>(box + (gq + 8) * 128 + ch);
                    }
                    const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + PD_ROWS * kc);
                    swa = *reinterpret_cast<const uint2*>(sc + gq * (kc / 32) + 4 * warp);
                    swb = *reinterpret_cast<const uint2*>(sc + (gq + 8) * (kc / 32) + 4 * warp);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[s]);
                Frag fc;
                if (GX) {
                    fc = f0;
                    f0 = f1;
                    load_frag((c + 2) % nchunks, f1);  // the chunk two stages on (of this or the next unit)
                } else {
                    load_frag(c, fc);
                }
                if (act) {
                    const uint2 dxa = fc.dxa, dxb = fc.dxb;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        if (4 * warp + j >= nbc) break;
                        const uint32_t a[4] = {wa[j].x, wb[j].x, wa[j].y, wb[j].y};
                        const uint32_t b[2] = {fc.xv[j].x, fc.xv[j].y};
                        int d[4];
                        mma_s8_bias(d, a, b, 0x4B400000);
                        const uint32_t wsa = j < 2 ? swa.x : swa.y, wsb = j < 2 ? swb.x : swb.y;
                        const uint32_t xsa = j < 2 ? dxa.x : dxa.y, xsb = j < 2 ? dxb.x : dxb.y;
                        const float dwa = h2f((uint16_t)((j & 1) ? (wsa >> 16) : (wsa & 0xFFFFu)));
                        const float dwb = h2f((uint16_t)((j & 1) ? (wsb >> 16) : (wsb & 0xFFFFu)));
                        const float dx0 = h2f((uint16_t)((j & 1) ? (xsa >> 16) : (xsa & 0xFFFFu)));
                        const float dx1 = h2f((uint16_t)((j & 1) ? (xsb >> 16) : (xsb & 0xFFFFu)));
                        const float f0 = __fsub_rn(__int_as_float(d[0]), 12582912.0f);
                        const float f1 = __fsub_rn(__int_as_float(d[1]), 12582912.0f);
                        const float f2 = __fsub_rn(__int_as_float(d[2]), 12582912.0f);
                        const float f3 = __fsub_rn(__int_as_float(d[3]), 12582912.0f);
                        acc[0] = __fadd_rn(acc[0], __fmul_rn(f0, __fmul_rn(dwa, dx0)));
                        acc[1] = __fadd_rn(acc[1], __fmul_rn(f1, __fmul_rn(dwa, dx1)));
                        acc[2] = __fadd_rn(acc[2], __fmul_rn(f2, __fmul_rn(dwb, dx0)));
                        acc[3] = __fadd_rn(acc[3], __fmul_rn(f3, __fmul_rn(dwb, dx1)));
                    }
                }
            }
            if (failed) break;
            // the warps' partial sums: C fragment value i is (row gq + 8 (i >> 1), token 2t + (i & 1)).
            // Buffer b of the two holds every other group: written once all warps have read it
            // (rfree), read once all warps have written it (rfull); the waits are bounded
            const int buf = rn & 1, use = rn >> 1;  // rn: row groups of the step so far
            float(*red)[PD_ROWS][8] = (*mred)[buf];
            int rok = 1;
            if (use > 0) {
                if (lane == 0) rok = pd_wait(&S.rfree[buf], (unsigned)(use - 1) & 1u, err);
                rok = __shfl_sync(0xffffffffu, rok, 0);
            }
            if (rok) {
                red[warp][gq][2 * t] = acc[0];
                red[warp][gq][2 * t + 1] = acc[1];
                red[warp][gq + 8][2 * t] = acc[2];
                red[warp][gq + 8][2 * t + 1] = acc[3];
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.rfull[buf]);
                if (lane == 0) rok = pd_wait(&S.rfull[buf], (unsigned)use & 1u, err);
                rok = __shfl_sync(0xffffffffu, rok, 0);
                __syncwarp();
            }
            if (!rok) {
                if (lane == 0) {
                    atomicCAS(err, 0, 50);
                    S.fail = 1;
                }
                failed = true;
                break;
            }
            rn++;
            if (lane < 4) {
                float v[4];  // rows 2w + (i & 1), tokens 2 lane + (i >> 1)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int rr = 2 * warp + (i & 1), tok = 2 * lane + (i >> 1);
                    float a = red[0][rr][tok];
#pragma unroll
                    for (int w = 1; w < PD_CONS; w++) a = __fadd_rn(a, red[w][rr][tok]);
                    v[i] = a;
                }
                if (g.swi) {
                    if (half == 0) {
#pragma unroll
                        for (int i = 0; i < 4; i++) gate[i] = v[i];
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int tok = 2 * lane + (i >> 1);
                            if (tok < M) S.hbuf[hb][tok][grp * PD_ROWS + 2 * warp + (i & 1)] = swiglu(gate[i], v[i]);
                        }
                    }
                } else if (xp) {
                    // exchange layout per (unit, row pair w): 16 floats [token][row of the pair]
                    const size_t slot = (size_t)(g.N / PD_ROWS) * PD_CONS * 16;
                    const size_t off = ((size_t)xpar * xp->tp + xp->rank) * slot + ((size_t)u * PD_CONS + warp) * 16 +
                                       4 * lane;
                    const float4 f4 = make_float4(v[0], v[1], v[2], v[3]);
#pragma unroll
                    for (int tt = 0; tt < PD_MAX_TP; tt++)
                        if (tt < xp->tp) *reinterpret_cast<float4*>(xp->xpeer[tt] + off) = f4;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int row = o0 + 2 * warp + (i & 1), tok = 2 * lane + (i >> 1);
                        if (tok < M && row < nout) {
                            out[(size_t)tok * ldo + row] = resid ? __fadd_rn(res[i], v[i]) : v[i];
                            if (keys) atomicMax(&S.keys[tok], argmax_key(v[i], row + kbase));
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.rfree[buf]);  // this warp is done reading the buffer
        }
        if (g.swi && !failed) {
            // h's 32 values per token are one Q8_0 block: warp 0 quantizes once every warp
            // has written its rows
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.hfull[hb]);
            if (warp == 0) {
                int ok = 1;
                if (lane == 0) ok = pd_wait(&S.hfull[hb], (unsigned)huse & 1u, err);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                __syncwarp();
                if (ok) {
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        const size_t e = (size_t)m * nout + (size_t)u * 32;
                        pd_quant_warp32(S.hbuf[hb][m][lane], lane, hq + e, hd + (e >> 5));
                    }
                } else if (lane == 0) {
                    atomicCAS(err, 0, 46);
                    S.fail = 1;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.hfree[hb]);
            }
        }
        if (g.swi) hn++;
    }
    pd_csync();
    return S.fail == 0;
}

// RmsNorm::forward of one f32 row (written by other CTAs: read through L2) by one warp, with
// Q8_0 of the bf16 result (rms_norm.rs:144-176): the input rounded to bf16, lane l sums the
// squares of elements 128i + 4l .. +3 in pass order, a butterfly gives the total, inv =
// 1/sqrt(sum/dim + eps), out = bf16((x*inv)*w), quantized per 32-element block by the block's 8
// lanes. The second pass reads the row again (from L2). A row's arithmetic does not depend on
// the batch size.
__device__ __forceinline__ void pd_norm_row_warp(const float* __restrict__ xr, int dim, const uint16_t* nw, float eps,
                                                 int lane, int8_t* xq, uint16_t* xd) {
    float ss = 0.0f;
#pragma unroll 8
    for (int e = lane * 4; e < dim; e += 128) {
        const float4 t = __ldcg(reinterpret_cast<const float4*>(xr + e));
        const float v[4] = {round_bf16(t.x), round_bf16(t.y), round_bf16(t.z), round_bf16(t.w)};
#pragma unroll
        for (int i = 0; i < 4; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    }
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
#pragma unroll 8
    for (int e = lane * 4; e < dim; e += 128) {
        const float4 t = __ldcg(reinterpret_cast<const float4*>(xr + e));
        const uint2 wt = *reinterpret_cast<const uint2*>(nw + e);
        const float x4[4] = {t.x, t.y, t.z, t.w};
        const float wv[4] = {bf16_to_f32((uint16_t)(wt.x & 0xFFFF)), bf16_to_f32((uint16_t)(wt.x >> 16)),
                             bf16_to_f32((uint16_t)(wt.y & 0xFFFF)), bf16_to_f32((uint16_t)(wt.y >> 16))};
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = round_bf16(__fmul_rn(__fmul_rn(round_bf16(x4[i]), inv), wv[i]));
        const uint32_t q = quant_group8(v, lane & 7, xd + (e >> 5));
        *reinterpret_cast<uint32_t*>(xq + e) = q;
    }
}

// the GEMV of one phase: the dp4a consumer for batches of 1-4 (bit-identical to the per-layer
// decode path), the MMA consumer for 5-8 (activation rows K + PD_XPAD bytes apart)
template <int M>
__device__ __forceinline__ bool pd_phase(PdSmem& S, const PdGemv& g, const int8_t* xs, const uint16_t* xds,
                                         PdRed* mred, PdRing& r, int& hn, int& rn, float* out, int ldo, bool resid, bool keys, int8_t* hq,
                                         uint16_t* hd, int* err, int u_first = -1, float res_first = 0.0f,
                                         const PdParams* xp = nullptr, int xpar = 0, int kbase = 0) {
    if constexpr (M > 4)
        return pd_consume_mma<M, false>(S, g, xs, g.K + PD_XPAD, xds, mred, r, hn, rn, out, ldo, resid, keys, hq, hd, err,
                                        xp, xpar, kbase);
    else
        return pd_consume<M>(S, g, xs, xds, r, hn, out, ldo, resid, keys, hq, hd, err, u_first, res_first, xp, xpar,
                             kbase);
}

// ---- tensor parallelism: the row-parallel exchange ----

// bounded wait until the counter at p (written by other GPUs) reaches target (wrap-safe);
// false when it gave up (~2 s; error `code`) or another CTA flagged an error
__device__ __forceinline__ bool pd_wait_sys(const unsigned* p, unsigned target, int* err, int code) {
    const uint64_t t0 = global_ns();
    for (int i = 1;; i++) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if ((int)(v - target) >= 0) return true;
        if ((i & 63) == 0) {
            if (ld_volatile(err) != 0) return false;
            if (global_ns() - t0 > PD_WAIT_NS) {
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void pd_signal_sys(unsigned* p) {
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(p) : "memory");
}

// After a row-parallel phase (o or down) under tensor parallelism: this CTA has stored the
// partial sums of its units into slot (par, rank) of every rank's exchange buffer
// (pd_consume); it publishes them (system-scope fence, then one counter increment on every
// peer), waits until every peer's CTA of the same index -- which computed the same units --
// has done the same here, and adds x[m][row] += p_0 + p_1 + ... + p_{tp-1} (rank order, so
// every rank forms the same residual stream). The grid barrier that follows orders these
// writes before any CTA reads x. target: the counter's value once this exchange is complete.
template <int M>
__device__ bool pd_exchange_sum(const PdParams& p, PdSmem& S, int par, unsigned target, int u_first) {
    const int tid = threadIdx.x, T = p.tp, units = p.H / PD_ROWS;
    if (tid == 0) {
        __threadfence_system();  // the CTA's peer stores, ordered before by the consumer barrier
#pragma unroll
        for (int t = 0; t < PD_MAX_TP; t++)
            if (t < T && t != p.rank) pd_signal_sys(p.fpeer[t] + blockIdx.x);
        S.flag = pd_wait_sys(p.fself + blockIdx.x, target, p.err, 48) ? 1 : 0;
    }
    pd_csync();
    if (!S.flag) return false;
    const size_t slot = (size_t)units * PD_CONS * 16;  // floats per (par, source rank)
    const float* xb = p.xself + (size_t)par * T * slot;
    for (int u = u_first; u < units; u += (int)gridDim.x) {
        for (int idx = tid; idx < PD_ROWS * M; idx += PD_CTHREADS) {
            const int m = idx / PD_ROWS, rr = idx % PD_ROWS;
            const size_t off = ((size_t)u * PD_CONS + (rr >> 1)) * 16 + m * 2 + (rr & 1);
            float v = __ldcg(xb + off);
            for (int t = 1; t < T; t++) v = __fadd_rn(v, __ldcg(xb + (size_t)t * slot + off));
            float* xo = p.x + (size_t)m * p.H + (size_t)u * PD_ROWS + rr;
            *xo = __fadd_rn(__ldcg(xo), v);
        }
    }
    return true;
}

// the LM head's argmax keys under tensor parallelism: every CTA takes the maximum of its keys
// (global vocabulary indices) into every rank's key array, then counts itself in on every rank;
// CTA 0 waits for all CTAs of all ranks (the token is final) and advances the exchange counts
// the next step starts from
template <int M>
__device__ void pd_keys_exchange(const PdParams& p, PdSmem& S, unsigned seq0, unsigned steps0) {
    const int tid = threadIdx.x, T = p.tp;
    if (tid < M && S.keys[tid]) {
#pragma unroll
        for (int t = 0; t < PD_MAX_TP; t++)
            if (t < T) atomicMax(p.kpeer[t] + tid, S.keys[tid]);
    }
    pd_csync();
    if (tid == 0) {
        __threadfence_system();
#pragma unroll
        for (int t = 0; t < PD_MAX_TP; t++)
            if (t < T) pd_signal_sys(p.fpeer[t] + gridDim.x);
        if (blockIdx.x == 0 &&
            pd_wait_sys(p.fself + gridDim.x, (steps0 + 1u) * gridDim.x * (unsigned)T, p.err, 49)) {
            p.seq[0] = seq0 + 2u * (unsigned)p.n_layers;
            p.seq[1] = steps0 + 1u;
        }
    }
}

// ---- attention (the decode attention kernel's arithmetic, on 256 threads) ----

// Attention work is split into runs: run r covers chunks [c0, c1) of one (row b, kv head) pair.
// Runs are sized so that there are at most gridDim.x of them (about gridDim.x / (M * Hkv) runs
// per pair), and CTA c takes runs c, c + gridDim.x, ...: q is loaded, normed and rotated once per
// run, and the chunks of a run follow each other with the next chunk's cache rows copied in
// while the current one is computed.
struct PdRuns {
    int len;      // chunks per run (the last run of a pair may hold fewer)
    int per_seq;  // runs per (row, kv head) pair
    int n;        // runs in all
};
__device__ __forceinline__ PdRuns pd_runs(int M, int Hkv, int nsplit) {
    PdRuns r;
    const int pairs = M * Hkv;
    const int per_pair = max(1, (int)gridDim.x / pairs);
    r.len = (nsplit + per_pair - 1) / per_pair;
    r.per_seq = (nsplit + r.len - 1) / r.len;
    r.n = pairs * r.per_seq;
    return r;
}

// the K (which = 0) or V (which = 1) cache rows of earlier steps (those before the new
// position) of chunk `split` of (row b, kv head kvh) into the staging area, every copy in
// flight, issued by the consumer threads from t0 on; they depend on nothing this step
// computes. Every consumer thread commits one cp.async group per call (an empty one when it
// issues nothing), so the groups line up across threads and cp_async_wait<1> means "all but
// the most recent call's copies".
__device__ __forceinline__ void pd_chunk_rows(const PdParams& p, const PdLayer& L, PdAtt& A, int p0, int b, int kvh,
                                              int split, int which, int t0) {
    const int D = 128;
    const int j0 = split * PD_ATT_C;
    const int rows = min(PD_ATT_C, p0 - j0);  // the new position's row is computed, not copied
    const float* base =
        (which ? L.vc : L.kc) + ((int64_t)b * p.Hkv + kvh) * (int64_t)p.ctx_max * D + (int64_t)j0 * D;
    for (int i = threadIdx.x - t0; i >= 0 && i < rows * (D / 4); i += PD_CTHREADS - t0) {
        const int r = i / (D / 4), c = (i % (D / 4)) * 4;
        cp_async16(which ? &A.vs[r][c] : &A.ks[r][c], base + (int64_t)r * D + c, true);
    }
    cp_async_commit();
}

// the first chunk of run `run`: its K or V rows (an empty group when the run does not exist)
__device__ __forceinline__ void pd_run_rows(const PdParams& p, const PdLayer& L, PdAtt& A, int p0, const PdRuns& R,
                                            int run, int which, int t0) {
    if (run >= R.n) {
        cp_async_commit();
        return;
    }
    const int pair = run / R.per_seq;
    pd_chunk_rows(p, L, A, p0, pair / p.Hkv, pair % p.Hkv, (run % R.per_seq) * R.len, which, t0);
}

// this CTA's first run of the layer is run blockIdx.x; the layer's q/k norm weights, the new
// position's cos/sin row and the run's first chunk's cache rows start loading here, between
// the arrive and the wait of the grid barrier that precedes attention, so they overlap it
template <int M>
__device__ __forceinline__ void pd_attention_begin(const PdParams& p, const PdLayer& L, PdAtt& A, int p0,
                                                   int nsplit) {
    const PdRuns R = pd_runs(M, p.Hkv, nsplit);
    // the q/k norm weights and the new position's cos/sin row: one group committed before the
    // K and V groups, so the run waits for it with cp_async_wait<2>
    {
        const int t = threadIdx.x;
        if (t < 16) cp_async16(&A.qn[t * 8], L.q_norm + t * 8, true);
        else if (t < 32) cp_async16(&A.kn[(t - 16) * 8], L.k_norm + (t - 16) * 8, true);
        else if (t < 48) cp_async16(&A.cs[(t - 32) * 4], p.cos_t + (int64_t)p0 * 64 + (t - 32) * 4, true);
        else if (t < 64) cp_async16(&A.sn[(t - 48) * 4], p.sin_t + (int64_t)p0 * 64 + (t - 48) * 4, true);
        cp_async_commit();
    }
    pd_run_rows(p, L, A, p0, R, (int)blockIdx.x, 0, 0);
    pd_run_rows(p, L, A, p0, R, (int)blockIdx.x, 1, 0);
}

// target: the published-chunk counters' value once
// this layer's chunks are all published ((layer + 1) * nsplit). The first run's first chunk
// rows are already in flight (pd_attention_begin).
template <int M>
__device__ void pd_attention(const PdParams& p, const PdLayer& L, PdSmem& S, PdAtt& A, int p0, int nsplit,
                             unsigned target) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Hq = p.Hq, Hkv = p.Hkv, G = Hq / Hkv, D = 128;
    const int heads = Hq + 2 * Hkv;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    const PdRuns R = pd_runs(M, Hkv, nsplit);
    const int kt0 = G < PD_CONS ? G * 32 : 0;  // the softmax runs on warps 0..G-1
    for (int run = (int)blockIdx.x; run < R.n; run += (int)gridDim.x) {
        const int pair = run / R.per_seq, b = pair / Hkv, kvh = pair % Hkv;
        const int c0 = (run % R.per_seq) * R.len, c1 = min(nsplit, c0 + R.len);
        const bool has_new = c1 == nsplit;  // the run holds the chunk of the new position
        pd_csync();  // the previous run is done with q and the raw rows
        // this kv head's q heads (and, for the run holding the new position, its k and v) from
        // the q|k|v rows
        const float* qrow = p.qkv + (int64_t)b * heads * D;
        for (int i = tid; i < G * (D / 4); i += PD_CTHREADS) {
            const int g = i / (D / 4), c = (i % (D / 4)) * 4;
            *reinterpret_cast<float4*>(&A.qraw[g][c]) =
                __ldcg(reinterpret_cast<const float4*>(qrow + (int64_t)(kvh * G + g) * D + c));
        }
        if (has_new && tid < 2 * (D / 4)) {
            const int which = tid / (D / 4), c = (tid % (D / 4)) * 4;  // 0: k, 1: v
            *reinterpret_cast<float4*>(&A.kvraw[which][c]) =
                __ldcg(reinterpret_cast<const float4*>(qrow + (int64_t)(Hq + which * Hkv + kvh) * D + c));
        }
        cp_async_wait<2>();  // the norm weights and cos/sin (the first chunk's K and V may still fly)
        pd_csync();
        for (int g = warp; g < G; g += PD_CONS) head_norm_rope(A.qraw[g], A.qn, p.eps, A.cs, A.sn, lane, A.qs[g]);
        if (has_new) {
            // the new position's k (normed, rotated) and v: into the caches now, into the
            // staging rows when their chunk comes
            const int64_t prow = ((int64_t)b * Hkv + kvh) * (int64_t)p.ctx_max * D + (int64_t)p0 * D;
            if (warp == 0) {
                head_norm_rope(A.kvraw[0], A.kn, p.eps, A.cs, A.sn, lane, A.knew);
                __syncwarp();
                *reinterpret_cast<float4*>(L.kc + prow + lane * 4) = *reinterpret_cast<const float4*>(&A.knew[lane * 4]);
            } else if (warp == 1) {
                *reinterpret_cast<float4*>(L.vc + prow + lane * 4) = *reinterpret_cast<const float4*>(&A.kvraw[1][lane * 4]);
            }
        }
        for (int split = c0; split < c1; split++) {
            const int j0 = split * PD_ATT_C;
            const int cnt = min(PD_ATT_C, p0 + 1 - j0);
            const int fresh = p0 - j0;  // chunk row of the new position (when < cnt)
            cp_async_wait<1>();  // the chunk's K rows (its V rows, committed after them, may still fly)
            pd_csync();  // q (and the new k) ready, the chunk's K rows landed
            if (fresh < cnt && tid < 2 * (D / 4)) {
                const int which = tid / (D / 4), c = (tid % (D / 4)) * 4;
                const float4 v = *reinterpret_cast<const float4*>(which ? &A.kvraw[1][c] : &A.knew[c]);
                *reinterpret_cast<float4*>(which ? &A.vs[fresh][c] : &A.ks[fresh][c]) = v;
            }
            if (fresh < cnt) pd_csync();
            // scores: thread -> (position pp, head g), heads fastest, so the G lanes of a position
            // read the same K address and the lanes of a head the same q address (shared-memory
            // broadcasts: a K row is fetched once for all heads of the group); one multiply-add chain
            // over the 128 dims, then the scale. K and q are read 32 dims at a time into registers
            // ahead of the chain.
            for (int idx = tid; idx < PD_ATT_C * G; idx += PD_CTHREADS) {
                const int pp = idx / G, g = idx - pp * G;
                float s = 0.f;
                if (pp < cnt) {
#pragma unroll
                    for (int d0 = 0; d0 < D; d0 += 32) {
                        float4 kk[8], qq[8];
#pragma unroll
                        for (int i = 0; i < 8; i++) kk[i] = *reinterpret_cast<const float4*>(&A.ks[pp][d0 + 4 * i]);
#pragma unroll
                        for (int i = 0; i < 8; i++) qq[i] = *reinterpret_cast<const float4*>(&A.qs[g][d0 + 4 * i]);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            s = fmaf(qq[i].x, kk[i].x, s);
                            s = fmaf(qq[i].y, kk[i].y, s);
                            s = fmaf(qq[i].z, kk[i].z, s);
                            s = fmaf(qq[i].w, kk[i].w, s);
                        }
                    }
                }
                A.ps[g][pp] = pp < cnt ? __fmul_rn(s, scale) : -INFINITY;
            }
            pd_csync();
            // K is free: the next chunk's K rows start loading (this run's next chunk, else the
            // first chunk of this CTA's next run), issued by the warps the softmax leaves idle
            if (split + 1 < c1) pd_chunk_rows(p, L, A, p0, b, kvh, split + 1, 0, kt0);
            else pd_run_rows(p, L, A, p0, R, run + (int)gridDim.x, 0, kt0);
            // chunk softmax per head: max, exp(s - max), sum
            for (int g = warp; g < G; g += PD_CONS) {
                const float a = A.ps[g][lane], c = A.ps[g][lane + 32];
                const float mx = warp_max(fmaxf(a, c));
                const float ea = expf(__fsub_rn(a, mx)), ec = expf(__fsub_rn(c, mx));
                A.ps[g][lane] = ea;
                A.ps[g][lane + 32] = ec;
                const float sum = warp_sum(__fadd_rn(ea, ec));
                if (lane == 0) { A.ml[g][0] = mx; A.ml[g][1] = sum; }
            }
            cp_async_wait<1>();  // the chunk's V rows (the next chunk's K rows may still fly)
            pd_csync();
            // chunk P.V: thread -> (dims 4c..4c+3, head g), heads fastest, so the G lanes of a dim
            // group read the same V address and the lanes of a head the same P address; per output
            // one multiply-add chain over the positions in order, 8 at a time with their V and P
            // values read ahead
            const int64_t hb0 = ((int64_t)b * Hq + (int64_t)kvh * G) * PD_MAX_SPLITS;
            {
                for (int idx = tid; idx < (D / 4) * G; idx += PD_CTHREADS) {
                    const int c4 = idx / G, g = idx - c4 * G;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    int j0 = 0;
#pragma unroll 1
                    for (; j0 + 8 <= cnt; j0 += 8) {
                        float4 vv[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) vv[j] = *reinterpret_cast<const float4*>(&A.vs[j0 + j][4 * c4]);
                        const float4 pa = *reinterpret_cast<const float4*>(&A.ps[g][j0]);
                        const float4 pb = *reinterpret_cast<const float4*>(&A.ps[g][j0 + 4]);
                        const float pj[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            acc.x = fmaf(pj[j], vv[j].x, acc.x);
                            acc.y = fmaf(pj[j], vv[j].y, acc.y);
                            acc.z = fmaf(pj[j], vv[j].z, acc.z);
                            acc.w = fmaf(pj[j], vv[j].w, acc.w);
                        }
                    }
                    for (int j = j0; j < cnt; j++) {
                        const float4 vv = *reinterpret_cast<const float4*>(&A.vs[j][4 * c4]);
                        const float pj = A.ps[g][j];
                        acc.x = fmaf(pj, vv.x, acc.x);
                        acc.y = fmaf(pj, vv.y, acc.y);
                        acc.z = fmaf(pj, vv.z, acc.z);
                        acc.w = fmaf(pj, vv.w, acc.w);
                    }
                    *reinterpret_cast<float4*>(&p.part_o[(hb0 + (int64_t)g * PD_MAX_SPLITS + split) * D + 4 * c4]) = acc;
                }
                if (tid < G) {
                    p.part_ml[(hb0 + (int64_t)tid * PD_MAX_SPLITS + split) * 2] = A.ml[tid][0];
                    p.part_ml[(hb0 + (int64_t)tid * PD_MAX_SPLITS + split) * 2 + 1] = A.ml[tid][1];
                }
            }
            pd_csync();  // V is free: the next chunk's V rows start loading
            if (split + 1 < c1) pd_chunk_rows(p, L, A, p0, b, kvh, split + 1, 1, 0);
            else pd_run_rows(p, L, A, p0, R, run + (int)gridDim.x, 1, 0);
        }
        // publish the run's chunks: the (row, kv head)'s counter grows by nsplit per layer
        __threadfence();
        pd_csync();
        if (tid == 0) atomicAdd(p.bar + 1 + b * Hkv + kvh, (unsigned)(c1 - c0));
    }
    // merge tasks (row, q head), dealt from the highest CTA down (CTA c: task gridDim.x - 1 - c,
    // then every gridDim.x-th), so the CTAs without runs take the first ones and no CTA holds two
    // while another holds none: wait until the kv head's chunks of this layer are all published,
    // then merge them (rescale by exp(m_s - max), sum in chunk order, divide) and write the head's
    // Q8_0 output
    const int n_tasks = M * Hq;
    for (int task = (int)gridDim.x - 1 - (int)blockIdx.x; task < n_tasks; task += (int)gridDim.x) {
        const int b = task / Hq, head = task % Hq, kvh = head / G;
        const int64_t hb = ((int64_t)b * Hq + head) * PD_MAX_SPLITS;
        if (tid == 0) {
            const unsigned* cnt = p.bar + 1 + b * Hkv + kvh;
            const uint64_t t0 = global_ns();
            int ok = 1;
            for (int i = 1;; i++) {
                unsigned v;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
                if (v >= target) break;
                if ((i & 63) == 0) {
                    if (ld_volatile(p.err) != 0) { ok = 0; break; }
                    if (global_ns() - t0 > PD_WAIT_NS) { atomicCAS(p.err, 0, 47); ok = 0; break; }
                }
            }
            S.flag = ok;
        }
        pd_csync();
        if (S.flag) {
            // the head's chunk partials into the staging area, all copies in flight, landing
            // while warp 0 computes the merge weights
            float* po_s = &A.ks[0][0];
            for (int i = tid; i < nsplit * (D / 4); i += PD_CTHREADS)
                cp_async16(po_s + (size_t)i * 4, p.part_o + hb * D + (int64_t)i * 4, true);
            cp_async_commit();
            if (warp == 0) {
                // each lane's (m, l) pairs read at once, summed in the order s = lane, lane + 32, ...
                const float* ml = p.part_ml + hb * 2;
                float mv[PD_MAX_SPLITS / 32], lv[PD_MAX_SPLITS / 32];
#pragma unroll
                for (int i = 0; i < PD_MAX_SPLITS / 32; i++) {
                    const int s2 = lane + 32 * i;
                    mv[i] = s2 < nsplit ? __ldcg(ml + 2 * s2) : -INFINITY;
                    lv[i] = s2 < nsplit ? __ldcg(ml + 2 * s2 + 1) : 0.0f;
                }
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < PD_MAX_SPLITS / 32; i++) mx = fmaxf(mx, mv[i]);
                mx = warp_max(mx);
                float lsum = 0.0f;
#pragma unroll
                for (int i = 0; i < PD_MAX_SPLITS / 32; i++) {
                    const int s2 = lane + 32 * i;
                    if (s2 < nsplit) {
                        const float w = expf(__fsub_rn(mv[i], mx));
                        A.cm[0][s2] = w;
                        lsum = __fadd_rn(lsum, __fmul_rn(w, lv[i]));
                    }
                }
                lsum = warp_sum(lsum);
                if (lane == 0) A.cl[0] = lsum;
            }
            cp_async_wait<0>();
            pd_csync();
            if (tid < D) {
                const int d = tid;
                float o = 0.0f;
                for (int s2 = 0; s2 < nsplit; s2++) o = __fadd_rn(o, __fmul_rn(A.cm[0][s2], po_s[(size_t)s2 * D + d]));
                o = __fdiv_rn(o, A.cl[0]);
                const int64_t e = (int64_t)b * Hq * D + (int64_t)head * D + d;
                pd_quant_warp32(o, lane, p.att_q + (e - lane), p.att_d + (e >> 5));
            }
        }
        pd_csync();  // the staging area is free for the next task
    }
}

// ---- the kernel ----
template <int M>
__global__ void __launch_bounds__(PD_THREADS, 1) decode_step_kernel(const PdParams p) {
    PdSmem& S = *reinterpret_cast<PdSmem*>(pd_dsmem);
    uint8_t* area = pd_dsmem + p.ring_off + (size_t)p.ns * PD_STAGE;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int p0 = *p.pos_dev;
    // exchanges and steps completed before this launch (tensor parallelism): CTA 0 advances them
    // only after every CTA of every rank has contributed its last keys, long after this read
    const unsigned seq0 = p.tp > 1 ? p.seq[0] : 0u, steps0 = p.tp > 1 ? p.seq[1] : 0u;
    const bool xch = p.tp > 1;
    if (p0 < 0 || p0 >= p.ctx_max) {  // every CTA leaves before any copy or barrier
        if (tid == 0) atomicCAS(p.err, 0, 44);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < PD_MAX_STAGES; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], PD_CONS);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&S.hfull[b], PD_CONS);
            mbar_init(&S.hfree[b], 1);
            mbar_init(&S.rfull[b], PD_CONS);
            mbar_init(&S.rfree[b], PD_CONS);
        }
        mbar_fence_init();
    }
    if (tid < PD_MAX_M) S.keys[tid] = 0ull;
    if (tid == 0) {
        S.fail = 0;
        S.ns = p.ns;
        S.ring_off = p.ring_off;
    }
    __syncthreads();
    if (warp == PD_CONS) {
        // producer: every matrix of the step, in order, never waiting for activations
        if (lane == 0) {
            PdRing r = {0, 0, 0u};
            unsigned off = 0;
            bool ok = true;
            for (int l = 0; l < p.n_layers && ok; l++)
                for (int k = PH_QKV; k <= PH_DN && ok; k++) {
                    const PdGemv g = pd_gemv(p, l, k);
                    ok = pd_produce(S, g, off, r, p.err, M > 4);
                    off += (unsigned)pd_units(g);
                }
            if (ok) pd_produce(S, pd_gemv(p, 0, PH_LM), off, r, p.err, M > 4);
            // leave only after the copies in flight have landed (bounded)
            for (int j = max(0, r.it - p.ns); j < r.it; j++)
                mbar_wait_ns(&S.full[j % p.ns], (unsigned)(j / p.ns) & 1u, PD_WAIT_NS);
        }
        return;
    }
    const int nsplit = p0 / PD_ATT_C + 1;
    const int H = p.H, I = p.I;
    // the widest activation row kept in shared memory (batches of 5-8 stream h from L2)
    const int Kmax = M > 4 ? max(H, p.Hq * 128) : max(max(H, p.Hq * 128), I);
    // union area, GEMV phases: activations xs [M][K] int8 and xds [M][K/32] fp16, the norm
    // weight nws [H] bf16 (prefetched before the barrier that precedes its prologue) and the
    // f32 staging row xrow [H]
    constexpr int XP = M > 4 ? PD_XPAD : 0;  // activation row padding (MMA consumer)
    int8_t* xs = reinterpret_cast<int8_t*>(area);
    uint16_t* xds = reinterpret_cast<uint16_t*>(area + (size_t)M * (Kmax + XP));
    uint16_t* nws = reinterpret_cast<uint16_t*>(area + (size_t)M * (Kmax + XP) + (size_t)M * (Kmax / 32) * 2);
    // M rows of K bytes from global memory into xs (rows K + XP apart)
    auto stage_rows = [&](const int8_t* src, int K) {
        if (XP == 0) {
            pd_prefetch(xs, src, M * K, tid);
        } else {
            for (int m = 0; m < M; m++) pd_prefetch(xs + (size_t)m * (K + XP), src + (size_t)m * K, K, tid);
        }
    };
    float* xrow = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(nws) + (size_t)H * 2);
    PdRed* mred = M > 4 ? reinterpret_cast<PdRed*>(pd_align128(reinterpret_cast<uint8_t*>(xrow + H))) : nullptr;
    PdAtt& A = *reinterpret_cast<PdAtt*>(area);
    // RMSNorm + Q8_0 of the M rows of x (written by other CTAs) into xs/xds; the norm weight's
    // copies are already in flight
    auto norm_rows = [&]() {
        if constexpr (M > 4) {
            // batches of 5-8: warp w normalises row w on its own (warp sums only), all rows at once
            pd_csync();
            if (warp < M) pd_norm_row_warp(p.x + (size_t)warp * H, H, nws, p.eps, lane, xs + (size_t)warp * (H + XP),
                                           xds + (size_t)warp * (H / 32));
            pd_csync();
            return;
        }
        for (int m = 0; m < M; m++) {
            pd_csync();
            pd_stage_f32(xrow, p.x + (size_t)m * H, H, tid);
            pd_csync();
            rms_row<float, PD_CTHREADS, 1>(xrow, H, nws, p.eps, tid, S.red, nullptr, xs + (size_t)m * (H + XP),
                                           xds + (size_t)m * (H / 32));
        }
        pd_csync();
    };
    PdRing ring = {0, 0, 0u};
    int hn = 0, rn = 0;
    unsigned epoch = 0;
    // the consumers' copy of the producer's running unit offset (phase k of layer l starts at
    // position l * per_layer + before[k] of the dealt sequence)
    unsigned per_layer = 0, before[4];
    for (int k = PH_QKV; k <= PH_DN; k++) {
        before[k] = per_layer;
        per_layer += (unsigned)pd_units(pd_gemv(p, 0, k));
    }
    pd_prefetch(nws, p.layers[0].in_norm, H * 2, tid);
    for (int l = 0; l < p.n_layers; l++) {
        const PdLayer& L = p.layers[l];
        // QKV: input RMSNorm + Q8_0 of x, the q|k|v rows
        norm_rows();
        if (!pd_phase<M>(S, pd_gemv(p, l, PH_QKV), xs, xds, mred, ring, hn, rn, p.qkv, p.Nqkv, false, false, nullptr,
                           nullptr, p.err))
            return;
        // the first attention item's cache rows start loading before the barrier
        pd_grid_arrive(p, epoch);
        pd_attention_begin<M>(p, L, A, p0, nsplit);
        if (!pd_grid_wait(p, S, epoch)) return;
        // x is final until the o phase writes it: the first o unit's residual loads now
        const int u_o = pd_first((unsigned)l * per_layer + before[PH_O]);
        const float res_o = pd_res_lane<M>(p.x, H, H, u_o);
        // attention -> Q8_0 rows
        pd_attention<M>(p, L, S, A, p0, nsplit, (unsigned)((l + 1) * nsplit));
        if (!pd_grid_barrier(p, S, epoch)) return;
        // O: the attention output as activations, residual into x
        {
            const int Ko = p.Hq * 128;
            stage_rows(p.att_q, Ko);
            pd_prefetch(xds, p.att_d, M * (Ko / 32) * 2, tid);
            cp_async_wait<0>();
            pd_csync();
            if (!pd_phase<M>(S, pd_gemv(p, l, PH_O), xs, xds, mred, ring, hn, rn, p.x, H, !xch, false, nullptr, nullptr,
                               p.err, u_o, res_o, xch ? &p : nullptr, 0))
                return;
        }
        if (xch && !pd_exchange_sum<M>(p, S, 0, (seq0 + 2u * (unsigned)l + 1u) * (unsigned)(p.tp - 1), u_o))
            return;
        pd_grid_arrive(p, epoch);
        pd_prefetch(nws, L.post_norm, H * 2, tid);
        if (!pd_grid_wait(p, S, epoch)) return;
        // x is final until the down phase writes it: the first down unit's residual loads now
        const int u_dn = pd_first((unsigned)l * per_layer + before[PH_DN]);
        const float res_dn = pd_res_lane<M>(p.x, H, H, u_dn);
        // GU: post-attention RMSNorm, gate|up, SiLU(gate)*up -> h as Q8_0
        norm_rows();
        if (!pd_phase<M>(S, pd_gemv(p, l, PH_GU), xs, xds, mred, ring, hn, rn, nullptr, 0, false, false, p.hq, p.hd, p.err))
            return;
        if (!pd_grid_barrier(p, S, epoch)) return;
        // DN: h (already Q8_0) as activations, residual into x
        if (M <= 4) stage_rows(p.hq, I);
        pd_prefetch(xds, p.hd, M * (I / 32) * 2, tid);
        cp_async_wait<0>();
        pd_csync();
        bool dn_ok;
        if constexpr (M > 4)
            dn_ok = pd_consume_mma<M, true>(S, pd_gemv(p, l, PH_DN), p.hq, I, p.hd, mred, ring, hn, rn, p.x, H, !xch,
                                            false, nullptr, nullptr, p.err, xch ? &p : nullptr, 1, 0);
        else
            dn_ok = pd_phase<M>(S, pd_gemv(p, l, PH_DN), xs, xds, mred, ring, hn, rn, p.x, H, !xch, false, nullptr,
                                nullptr, p.err, u_dn, res_dn, xch ? &p : nullptr, 1);
        if (!dn_ok) return;
        if (xch && !pd_exchange_sum<M>(p, S, 1, (seq0 + 2u * (unsigned)l + 2u) * (unsigned)(p.tp - 1), u_dn))
            return;
        pd_grid_arrive(p, epoch);
        pd_prefetch(nws, l + 1 < p.n_layers ? p.layers[l + 1].in_norm : p.final_norm, H * 2, tid);
        if (!pd_grid_wait(p, S, epoch)) return;
    }
    // LM head: final RMSNorm, logits, greedy argmax keys
    norm_rows();
    if (!pd_phase<M>(S, pd_gemv(p, 0, PH_LM), xs, xds, mred, ring, hn, rn, p.logits, p.V, false, true, nullptr, nullptr,
                       p.err, -1, 0.0f, nullptr, 0, p.vbase))
        return;
    pd_csync();
    if (xch) pd_keys_exchange<M>(p, S, seq0, steps0);
    else if (tid < M && S.keys[tid]) atomicMax(p.keys + tid, S.keys[tid]);
}

// ---- host ----
static size_t pd_area_bytes(int64_t m, int64_t H, int64_t Hqd, int64_t I) {
    // GEMV phases: activations [m][Kmax (+ pad)], their scales, the norm weight, the f32 row and,
    // for batches of 5-8 (whose h streams from L2 instead), the partial-sum buffers
    const bool mma = m > 4;
    const int64_t Kmax = mma ? std::max(H, Hqd) : std::max({H, Hqd, I});
    size_t gemv = (size_t)(m * (Kmax + (mma ? PD_XPAD : 0)) + m * (Kmax / 32) * 2 + H * 2 + H * 4);
    if (mma) gemv = ((gemv + 127) & ~(size_t)127) + sizeof(PdRed);
    return std::max(gemv, sizeof(PdAtt));
}

constexpr size_t PD_SMEM_MAX = 227 * 1024;
constexpr int PD_MIN_STAGES = 3;

// the ring starts after PdSmem, 1024-aligned (the swizzled boxes of batches 5-8 need it)
static size_t pd_ring_off(int64_t m) {
    (void)m;
    return (sizeof(PdSmem) + 1023) & ~(size_t)1023;
}

// ring stages that fit beside the union area (at most PD_MAX_STAGES; 0 when fewer than
// PD_MIN_STAGES fit)
static int pd_ns(int64_t m, int64_t H, int64_t Hqd, int64_t I) {
    const size_t fixed = pd_ring_off(m) + pd_area_bytes(m, H, Hqd, I);
    if (fixed >= PD_SMEM_MAX) return 0;
    const int ns = (int)std::min<size_t>(PD_MAX_STAGES, (PD_SMEM_MAX - fixed) / PD_STAGE);
    return ns >= PD_MIN_STAGES ? ns : 0;
}

static size_t pd_smem_bytes(int64_t m, int64_t H, int64_t Hqd, int64_t I) {
    return pd_ring_off(m) + (size_t)pd_ns(m, H, Hqd, I) * PD_STAGE + pd_area_bytes(m, H, Hqd, I);
}

bool decode_persist_supported(lq_ctx* ctx, int64_t m, int64_t H, int64_t Hq, int64_t Hkv, int64_t I,
                              int64_t ctx_max) {
    if (m < 1 || m > PD_MAX_M || getenv("LQ_NO_PERSIST")) return false;
    if (H % 256 || I % 256 || Hq % Hkv || Hq / Hkv > PD_MAX_G) return false;
    if (ctx_max > (int64_t)PD_ATT_C * PD_MAX_SPLITS) return false;
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device);
    return coop && pd_ns(m, H, Hq * 128, I) > 0;
}

size_t decode_persist_xchg_layout(int64_t H, int tp, int sm_count, int64_t keys_n, size_t* flags_off,
                                  size_t* keys_off, size_t* seq_off) {
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t xbytes = al((size_t)2 * tp * (size_t)(H / PD_ROWS) * PD_CONS * 16 * 4);
    const size_t fbytes = al((size_t)(sm_count + 1) * 4);
    *flags_off = xbytes;
    *keys_off = xbytes + fbytes;
    *seq_off = *keys_off + al((size_t)std::max<int64_t>(PD_MAX_M, keys_n) * 8);
    return *seq_off + 256;
}

size_t decode_persist_desc_bytes(int64_t n_layers) { return (size_t)(n_layers + 1) * sizeof(PdLayer); }
size_t decode_persist_part_bytes(int64_t m, int64_t Hq) { return (size_t)(m * Hq * PD_MAX_SPLITS) * (128 + 2) * 4; }
size_t decode_persist_counter_bytes(int64_t m, int64_t Hkv, int64_t n_layers) {
    (void)n_layers;
    return (size_t)(1 + m * Hkv) * 4;
}

static int pd_map(lq_ctx* ctx, PdMat* out, const lq_q8_tensor& w) {
    const int64_t N = w.n, K = w.k, nb = K / 32;
    const uint32_t kc = (uint32_t)std::min<int64_t>(K, PD_KC);
    int rc = make_tensor_map_2d(ctx, &out->wq, CU_TENSOR_MAP_DATA_TYPE_UINT64, w.qs, (uint64_t)(K / 8), (uint64_t)N,
                                (uint64_t)K, kc / 8, PD_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = make_tensor_map_2d(ctx, &out->wsw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.qs, (uint64_t)K, (uint64_t)N, (uint64_t)K,
                            128, PD_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    return make_tensor_map_2d(ctx, &out->wd, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.d, (uint64_t)nb, (uint64_t)N,
                              (uint64_t)(nb * 2), kc / 32, PD_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int decode_persist_write_desc(lq_ctx* ctx, void* dev, const PdHostLayer* layers, int64_t n_layers,
                              const lq_q8_tensor* lm_head) {
    std::vector<PdLayer> h((size_t)n_layers + 1);
    memset(static_cast<void*>(h.data()), 0, h.size() * sizeof(PdLayer));
    for (int64_t l = 0; l < n_layers; l++) {
        const PdHostLayer& s = layers[l];
        const lq_q8_tensor* mats[4] = {s.qkv, s.o, s.gate_up, s.down};
        for (int k = 0; k < 4; k++) {
            for (const void* ptr : {(const void*)mats[k]->qs, (const void*)mats[k]->d})
                if ((uintptr_t)ptr % 16) return set_error(ctx, LQ_ERR_UNSUPPORTED, "decode_step: unaligned weights");
            int rc = pd_map(ctx, &h[l].mat[k], *mats[k]);
            if (rc) return rc;
        }
        h[l].in_norm = s.in_norm;
        h[l].post_norm = s.post_norm;
        h[l].q_norm = s.q_norm;
        h[l].k_norm = s.k_norm;
        h[l].kc = s.kc;
        h[l].vc = s.vc;
    }
    int rc = pd_map(ctx, &h[n_layers].mat[0], *lm_head);
    if (rc) return rc;
    LQ_CUDA(ctx, cudaMemcpy(dev, h.data(), h.size() * sizeof(PdLayer), cudaMemcpyHostToDevice));
    return LQ_OK;
}

template <int M>
static int launch_pd(lq_ctx* ctx, const PdParams& p, size_t smem) {
    auto kern = decode_step_kernel<M>;
    if (const int rc = ensure_func_smem(ctx, (const void*)kern, PD_SMEM_MAX)) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctx->sm_count);
    cfg.blockDim = dim3(PD_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident at once: the grid barriers rely on it
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return check_cuda(ctx, e, "decode_step (cooperative launch)");
    return LQ_OK;
}

int launch_decode_persist(lq_ctx* ctx, const PdLaunch& a) {
    if (a.m < 1 || a.m > PD_MAX_M)
        return set_error(ctx, LQ_ERR_INVALID_ARG, "decode_step: batch %lld > %d", (long long)a.m, PD_MAX_M);
    const int ns = pd_ns(a.m, a.H, a.Hq * 128, a.I);
    if (!ns) return set_error(ctx, LQ_ERR_UNSUPPORTED, "decode_step: shapes leave no room for the weight ring");
    PdParams p = {};
    p.layers = reinterpret_cast<const PdLayer*>(a.desc);
    p.n_layers = (int)a.n_layers;
    p.final_norm = a.final_norm;
    p.H = (int)a.H;
    p.Hq = (int)a.Hq;
    p.Hkv = (int)a.Hkv;
    p.I = (int)a.I;
    p.V = (int)a.V;
    p.Nqkv = (int)((a.Hq + 2 * a.Hkv) * 128);
    p.ctx_max = (int)a.ctx_max;
    p.eps = a.eps;
    p.cos_t = a.cos_t;
    p.sin_t = a.sin_t;
    p.pos_dev = a.pos_dev;
    p.x = a.x;
    p.qkv = a.qkv;
    p.att_q = a.att_q;
    p.att_d = a.att_d;
    p.hq = a.hq;
    p.hd = a.hd;
    p.part_o = a.part;
    p.part_ml = a.part + (size_t)(a.m * a.Hq * PD_MAX_SPLITS) * 128;
    p.logits = a.logits;
    p.keys = a.keys;
    p.bar = a.counters;
    p.err = ctx->err_flag;
    p.ns = ns;
    p.ring_off = (int)pd_ring_off(a.m);
    p.tp = a.tp;
    p.rank = a.rank;
    p.vbase = (int)a.vbase;
    if (a.tp > 1) {
        if (a.tp > PD_MAX_TP || a.rank < 0 || a.rank >= a.tp || a.H % PD_ROWS)
            return set_error(ctx, LQ_ERR_INVALID_ARG, "decode_step: tensor-parallel world %d (at most %d)", a.tp,
                             PD_MAX_TP);
        size_t fo = 0, ko = 0, so = 0;
        decode_persist_xchg_layout(a.H, a.tp, ctx->sm_count, a.keys_n, &fo, &ko, &so);
        for (int t = 0; t < a.tp; t++) {
            uint8_t* b = static_cast<uint8_t*>(a.xchg[t]);
            if (!b) return set_error(ctx, LQ_ERR_INVALID_ARG, "decode_step: exchange region of rank %d missing", t);
            p.xpeer[t] = reinterpret_cast<float*>(b);
            p.fpeer[t] = reinterpret_cast<unsigned*>(b + fo);
            p.kpeer[t] = reinterpret_cast<unsigned long long*>(b + ko);
        }
        p.xself = p.xpeer[a.rank];
        p.fself = p.fpeer[a.rank];
        p.seq = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(a.xchg[a.rank]) + so);
        if (a.keys != p.kpeer[a.rank])
            return set_error(ctx, LQ_ERR_INVALID_ARG, "decode_step: keys must be the exchange region's keys");
    }
    LQ_CUDA(ctx, cudaMemsetAsync(a.counters, 0, decode_persist_counter_bytes(a.m, a.Hkv, a.n_layers), ctx->stream));
    const size_t smem = pd_smem_bytes(a.m, a.H, a.Hq * 128, a.I);
    switch (a.m) {
        case 1: return launch_pd<1>(ctx, p, smem);
        case 2: return launch_pd<2>(ctx, p, smem);
        case 3: return launch_pd<3>(ctx, p, smem);
        case 4: return launch_pd<4>(ctx, p, smem);
        case 5: return launch_pd<5>(ctx, p, smem);
        case 6: return launch_pd<6>(ctx, p, smem);
        case 7: return launch_pd<7>(ctx, p, smem);
        default: return launch_pd<8>(ctx, p, smem);
    }
}

}  // namespace lq
