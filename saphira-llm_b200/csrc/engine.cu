// engine.cu -- the persistent I2_S GEMV engine for sm_100a (see engine.cuh).
//
// Per CTA (one per SM, 17 warps):
//   warp 16 (producer): walks the CTA's chunks of every stage in program
//     order and, for each, waits for a free ring slot and issues one TMA bulk
//     copy (two for a gate/up pair) of the chunk's contiguous weight rows into
//     it, with the slot's mbarrier counting the bytes. It never waits for
//     activations, so weights stream ahead across op and stage boundaries.
//   warps 0-15 (consumers): for each chunk, (re)build the int8 activations
//     of the chunk's input group when it changes (the certified RMSNorm +
//     absmax prologue of i2s_gemv.cu, shared by the 512 consumer threads),
//     wait for the slot, run the dp4a dots from shared memory, apply the
//     epilogue and release the slot.
//   At a stage boundary the consumers publish their outputs and meet every
//     other CTA at a grid barrier before reading the next stage's input.
//
// Exactness is the same as i2s_gemv.cu: integer dots in any order, the
// reference's float op order in the prologue and epilogues.
//
// Every wait is bounded by the global timer (2 s). A wait that gives up
// records why in *error and puts the CTA in a skip mode that still reaches
// every barrier, so the kernel always terminates; the producer then waits
// (bounded) for its own copies in flight before it exits.

#include "common.cuh"
#include "engine.cuh"

namespace sllm {

constexpr uint64_t kEngWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded: false when the phase did not complete within kEngWaitNs
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > kEngWaitNs) return false;
    }
    return true;
}

// one contiguous global -> shared copy on the TMA engine (no multicast)
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEngConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// reduction slots: one per consumer warp, padded to 16 with the identity
constexpr int kRed = 16;

struct EngSmem {
    uint64_t full[kEngSlots];
    uint64_t empty[kEngSlots];
    double dred[kRed];
    float fred[kRed];
    int ired[kRed];
    float fallback_mean;
    int abort_flag;
    int grid_ok;
};

// ---------------------------------------------------------------------------
// chunk walk: producer and consumers enumerate the same chunks
// ---------------------------------------------------------------------------
struct ChunkWalk {
    const EngOp* ops;        // the shared-memory copy
    int op, row;
    EngCursor end;
    __device__ __forceinline__ bool next(int& o, int& r, int& n) {
        while (true) {
            if (op > end.op || (op == end.op && row >= end.row)) return false;
            const int rows = ops[op].rows;
            if (row >= rows) { ++op; row = 0; continue; }
            const int stop = (op == end.op) ? end.row : rows;
            n = min(stop - row, ops[op].chunk_rows);
            o = op;
            r = row;
            row += n;
            return true;
        }
    }
};

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------
// consumer-side prologue (512 threads): int8 activations of a group into qs
// ---------------------------------------------------------------------------
__device__ __forceinline__ float cmax(float v, float* red, int warp, int lane) {
    v = warp_max(v);
    if (lane == 0) red[warp] = v;
    consumer_sync();
    v = red[lane & (kRed - 1)];
    for (int o = kRed / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int csum_i(int v, int* red, int warp, int lane) {
    v = __reduce_add_sync(0xffffffffu, v);
    if (lane == 0) red[warp] = v;
    consumer_sync();
    v = red[lane & (kRed - 1)];
    for (int o = kRed / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double csum_d(double v, double* red, int warp, int lane) {
    v = warp_sum_d(v);
    if (lane == 0) red[warp] = v;
    consumer_sync();
    v = red[lane & (kRed - 1)];
    for (int o = kRed / 2; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ sllm_cuda_act eng_prologue(const EngGroup& g, const EngParams& P, int8_t* qs, EngSmem& es, int tid,
                                      int warp, int lane) {
    constexpr int NT = kEngConsumerWarps * 32;
    constexpr int KPT = (8192 / 4 + NT - 1) / NT;     // float4 per thread for the widest K
    const int K = g.K, K4 = K >> 2;
    float4 x[KPT], w[KPT];
    if (g.pro == PRO_NORM) {
        #pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = tid + j * NT;
            w[j] = i < K4 ? __ldg(reinterpret_cast<const float4*>(g.norm_w) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    #pragma unroll
    for (int j = 0; j < KPT; ++j) {
        const int i = tid + j * NT;
        x[j] = i < K4 ? ldcg4(g.x + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (g.pro == PRO_NORM) {
        double ss = 0.0;
        #pragma unroll
        for (int j = 0; j < KPT; ++j) {
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].x, x[j].x));
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].y, x[j].y));
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].z, x[j].z));
            ss = __dadd_rn(ss, (double)__fmul_rn(x[j].w, x[j].w));
        }
        const double S = csum_d(ss, es.dred, warp, lane);
        float mean;
        const bool ok = certify_mean_mul(S, K, 1.0 / (double)K, &mean) && !P.force_fallback;
        if (!ok) {   // uniform: S is the same in every thread
            if (tid == 0) {
                // the reference's lane order, read straight from L2 (rare path)
                double l0 = 0.0, l1 = 0.0, l2 = 0.0, l3 = 0.0;
                for (int b = 0; b < K; b += 8) {
                    const float4 a = ldcg4(g.x + b), c = ldcg4(g.x + b + 4);
                    l0 = __dadd_rn(l0, (double)__fmul_rn(a.x, a.x));
                    l1 = __dadd_rn(l1, (double)__fmul_rn(a.y, a.y));
                    l2 = __dadd_rn(l2, (double)__fmul_rn(a.z, a.z));
                    l3 = __dadd_rn(l3, (double)__fmul_rn(a.w, a.w));
                    l0 = __dadd_rn(l0, (double)__fmul_rn(c.x, c.x));
                    l1 = __dadd_rn(l1, (double)__fmul_rn(c.y, c.y));
                    l2 = __dadd_rn(l2, (double)__fmul_rn(c.z, c.z));
                    l3 = __dadd_rn(l3, (double)__fmul_rn(c.w, c.w));
                }
                double ssr = 0.0;
                ssr = __dadd_rn(ssr, l0);
                ssr = __dadd_rn(ssr, l1);
                ssr = __dadd_rn(ssr, l2);
                ssr = __dadd_rn(ssr, l3);
                es.fallback_mean = __double2float_rn(__ddiv_rn(ssr, (double)K));
                if (P.fallback_count != nullptr && blockIdx.x == 0) atomicAdd(P.fallback_count, 1);
            }
            consumer_sync();
            mean = es.fallback_mean;
        }
        const float sc = rms_scale(mean, P.eps);
        #pragma unroll
        for (int j = 0; j < KPT; ++j) {
            x[j].x = __fmul_rn(__fmul_rn(sc, x[j].x), w[j].x);
            x[j].y = __fmul_rn(__fmul_rn(sc, x[j].y), w[j].y);
            x[j].z = __fmul_rn(__fmul_rn(sc, x[j].z), w[j].z);
            x[j].w = __fmul_rn(__fmul_rn(sc, x[j].w), w[j].w);
        }
    }
    float amax = 0.0f;
    #pragma unroll
    for (int j = 0; j < KPT; ++j)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x[j].x), fabsf(x[j].y)), fmaxf(fabsf(x[j].z), fabsf(x[j].w))));
    amax = cmax(amax, es.fred, warp, lane);
    const float s = quant_scale(amax);
    int sum = 0;
    #pragma unroll
    for (int j = 0; j < KPT; ++j) {
        const int i = tid + j * NT;
        if (i < K4) {
            const int a = quant_one(x[j].x, s), b = quant_one(x[j].y, s);
            const int c = quant_one(x[j].z, s), d = quant_one(x[j].w, s);
            sum += a + b + c + d;
            reinterpret_cast<uint32_t*>(qs)[i] = (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) |
                                                 ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
        }
    }
    sum = csum_i(sum, es.ired, warp, lane);     // its barrier also publishes qs
    sllm_cuda_act act;
    act.scale = s;
    act.sum = sum;
    return act;
}

// ---------------------------------------------------------------------------
// one chunk of rows from a ring slot
// ---------------------------------------------------------------------------
template <int WPL>
__device__ __forceinline__ void eng_chunk(const EngOp& op, int r0, int n, const uint8_t* slot, const int8_t* qs,
                                          int asum, float post, float post2, int warp, int lane) {
    const int K = op.K, W = K >> 4, rb = K >> 2;
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qs);
    int aq[WPL][4];
    #pragma unroll
    for (int i = 0; i < WPL; ++i) {
        const int wi = lane + 32 * i;
        #pragma unroll
        for (int f = 0; f < 4; ++f) aq[i][f] = wi < W ? (int)q32[(wi >> 3) * 32 + 8 * f + (wi & 7)] : 0;
    }
    if (op.epi == EPI_SILU) {
        const uint8_t* up = slot + (size_t)n * rb;
        for (int j = warp; j < n; j += kEngConsumerWarps) {
            const uint32_t* rg = reinterpret_cast<const uint32_t*>(slot + (size_t)j * rb);
            const uint32_t* ru = reinterpret_cast<const uint32_t*>(up + (size_t)j * rb);
            int ag = 0, au = 0;
            #pragma unroll
            for (int i = 0; i < WPL; ++i) {
                const int wi = lane + 32 * i;
                const uint32_t wg = wi < W ? rg[wi] : 0u, wu = wi < W ? ru[wi] : 0u;
                ag = i2s_dot_word(wg, aq[i][0], aq[i][1], aq[i][2], aq[i][3], ag);
                au = i2s_dot_word(wu, aq[i][0], aq[i][1], aq[i][2], aq[i][3], au);
            }
            ag = __reduce_add_sync(0xffffffffu, ag);
            au = __reduce_add_sync(0xffffffffu, au);
            if (lane == 0) {
                // h = silu(gate) * up (src/forward.c:765-778, src/ops.c:452-456)
                const float g = __fmul_rn(__int2float_rn(ag - asum), post);
                const float u = __fmul_rn(__int2float_rn(au - asum), post2);
                op.h[r0 + j] = __fmul_rn(silu_block(g), u);
            }
        }
        return;
    }
    for (int j = warp; j < n; j += kEngConsumerWarps) {
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(slot + (size_t)j * rb);
        int acc = 0;
        #pragma unroll
        for (int i = 0; i < WPL; ++i) {
            const int wi = lane + 32 * i;
            acc = i2s_dot_word(wi < W ? rw[wi] : 0u, aq[i][0], aq[i][1], aq[i][2], aq[i][3], acc);
        }
        acc = __reduce_add_sync(0xffffffffu, acc);
        if (lane == 0) {
            float v = __fmul_rn(__int2float_rn(acc - asum), post);
            if (op.epi == EPI_RESID) v = __fadd_rn(v, __ldcg(op.resid + r0 + j));
            op.y[r0 + j] = v;
        }
    }
}

__device__ __forceinline__ void eng_chunk_dispatch(const EngOp& op, int r0, int n, const uint8_t* slot,
                                                   const int8_t* qs, int asum, float post, float post2, int warp,
                                                   int lane) {
    const int wpl = ((op.K >> 4) + 31) >> 5;
    switch (wpl) {
#define SLLM_ENG_CASE(N) case N: eng_chunk<N>(op, r0, n, slot, qs, asum, post, post2, warp, lane); break;
        SLLM_ENG_CASE(1) SLLM_ENG_CASE(2) SLLM_ENG_CASE(3) SLLM_ENG_CASE(4)
        SLLM_ENG_CASE(5) SLLM_ENG_CASE(6) SLLM_ENG_CASE(7) SLLM_ENG_CASE(8)
        SLLM_ENG_CASE(9) SLLM_ENG_CASE(10) SLLM_ENG_CASE(11) SLLM_ENG_CASE(12)
        SLLM_ENG_CASE(13) SLLM_ENG_CASE(14) SLLM_ENG_CASE(15) SLLM_ENG_CASE(16)
#undef SLLM_ENG_CASE
        default: break;
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEngThreads, 1)
i2s_engine_kernel(const EngParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ EngSmem es;
    uint8_t* ring = smem;                                     // kEngSlots x kEngSlotBytes
    int8_t* qs = reinterpret_cast<int8_t*>(smem + kEngSlots * kEngSlotBytes);   // up to 8192 bytes
    EngOp* s_ops = reinterpret_cast<EngOp*>(smem + kEngSlots * kEngSlotBytes + 8192);
    EngGroup* s_groups = reinterpret_cast<EngGroup*>(s_ops + P.n_ops);
    EngCursor* s_cur = reinterpret_cast<EngCursor*>(s_groups + P.n_groups);   // [n_stages][2]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;

    // the program tables, once, into shared memory: no descriptor read on the
    // critical path ever goes to L2 again
    {
        static_assert(sizeof(EngOp) % 8 == 0 && sizeof(EngGroup) % 4 == 0, "table copy granularity");
        const int2* src = reinterpret_cast<const int2*>(P.ops);
        int2* dst = reinterpret_cast<int2*>(s_ops);
        for (int i = tid; i < (int)(P.n_ops * sizeof(EngOp) / 8); i += blockDim.x) dst[i] = __ldg(src + i);
        const int* gsrc = reinterpret_cast<const int*>(P.groups);
        int* gdst = reinterpret_cast<int*>(s_groups);
        for (int i = tid; i < (int)(P.n_groups * sizeof(EngGroup) / 4); i += blockDim.x) gdst[i] = __ldg(gsrc + i);
        for (int i = tid; i < 2 * P.n_stages; i += blockDim.x) {
            const int st = i >> 1;
            s_cur[i] = P.starts[(size_t)st * (G + 1) + c + (i & 1)];
        }
    }

    if (tid == 0) {
        for (int i = 0; i < kEngSlots; ++i) {
            mbar_init(&es.full[i], 1);
            mbar_init(&es.empty[i], kEngConsumerWarps);
        }
        for (int i = kEngConsumerWarps; i < kRed; ++i) { es.dred[i] = 0.0; es.fred[i] = 0.0f; es.ired[i] = 0; }
        es.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kEngConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t k = 0;
            for (int s = 0; s < P.n_stages; ++s) {
                ChunkWalk walk{s_ops, s_cur[2 * s].op, s_cur[2 * s].row, s_cur[2 * s + 1]};
                {
                    // the norm vectors this stage's prologues will read: into L2 now
                    ChunkWalk pw = walk;
                    int o, r, n, last = -1;
                    while (pw.next(o, r, n)) {
                        const int gi = s_ops[o].group;
                        if (gi != last && s_groups[gi].norm_w != nullptr)
                            prefetch_l2(s_groups[gi].norm_w, (uint32_t)s_groups[gi].K * 4u);
                        last = gi;
                    }
                }
                int o, r, n;
                while (walk.next(o, r, n)) {
                    const int slot = (int)(k % kEngSlots);
                    const uint32_t use = k / kEngSlots;
                    if (*(volatile int*)&es.abort_flag) break;
                    if (use > 0 && !mbar_wait(&es.empty[slot], (use - 1) & 1)) {
                        es.abort_flag = 1;
                        atomicExch(P.error, ENG_TIMEOUT_EMPTY);
                        break;
                    }
                    const EngOp& op = s_ops[o];
                    const uint32_t rb = (uint32_t)op.K >> 2;
                    const uint32_t bytes = (uint32_t)n * rb;
                    uint8_t* dst = ring + (size_t)slot * kEngSlotBytes;
                    if (op.epi == EPI_SILU) {
                        mbar_expect_tx(&es.full[slot], 2 * bytes);
                        bulk_copy(dst, op.w + (size_t)r * rb, bytes, &es.full[slot]);
                        bulk_copy(dst + bytes, op.w2 + (size_t)r * rb, bytes, &es.full[slot]);
                    } else {
                        mbar_expect_tx(&es.full[slot], bytes);
                        bulk_copy(dst, op.w + (size_t)r * rb, bytes, &es.full[slot]);
                    }
                    ++k;
                }
                if (*(volatile int*)&es.abort_flag) break;
            }
            // every copy this CTA issued lands before the CTA may exit
            const uint32_t first = k > (uint32_t)kEngSlots ? k - kEngSlots : 0;
            for (uint32_t j = first; j < k; ++j) mbar_wait(&es.full[j % kEngSlots], (j / kEngSlots) & 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    uint32_t k = 0;
    int cur_group = -1;
    sllm_cuda_act act{0.0f, 0};
    int cur_op = -1;
    float post = 0.0f, post2 = 0.0f;
    for (int s = 0; s < P.n_stages; ++s) {
        if (s > 0) {
            // the stage's input is the previous stage's output from every CTA
            if (tid == 0) {
                bool ok = true;
                if (!*(volatile int*)&es.abort_flag) {
                    const unsigned target = (unsigned)s * (unsigned)G;
                    const uint64_t t0 = gtimer();
                    while (ld_acquire(P.barrier) < target) {
                        if (gtimer() - t0 > kEngWaitNs) { ok = false; break; }
                        __nanosleep(20);
                    }
                }
                if (!ok) {
                    es.abort_flag = 1;
                    atomicExch(P.error, ENG_TIMEOUT_GRID);
                }
            }
            consumer_sync();
            cur_group = -1;
            cur_op = -1;
        }
        ChunkWalk walk{s_ops, s_cur[2 * s].op, s_cur[2 * s].row, s_cur[2 * s + 1]};
        int o, r, n;
        while (walk.next(o, r, n)) {
            const EngOp& op = s_ops[o];
            if (op.group != cur_group) {
                act = eng_prologue(s_groups[op.group], P, qs, es, tid, warp, lane);
                cur_group = op.group;
                cur_op = -1;
            }
            if (o != cur_op) {
                // per-tensor scales (src/quant.c:102-106), one division per tensor
                post = __fdiv_rn(op.ws, act.scale);
                post2 = op.epi == EPI_SILU ? __fdiv_rn(op.ws2, act.scale) : 0.0f;
                cur_op = o;
            }
            const int slot = (int)(k % kEngSlots);
            const uint32_t use = k / kEngSlots;
            bool have = !*(volatile int*)&es.abort_flag;
            if (have && !mbar_wait(&es.full[slot], use & 1)) {
                es.abort_flag = 1;
                atomicExch(P.error, ENG_TIMEOUT_FULL);
                have = false;
            }
            if (have)
                eng_chunk_dispatch(op, r, n, ring + (size_t)slot * kEngSlotBytes, qs, act.sum, post, post2, warp,
                                   lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&es.empty[slot]);
            ++k;
        }
        // publish this CTA's outputs of the stage, then arrive
        consumer_sync();
        if (tid == 0 && s + 1 < P.n_stages) red_release_add(P.barrier, 1u);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int engine_chunk_rows(int K, int epi) {
    // as many rows as fill a slot, in whole rounds of the consumer warps
    const int rb = (K / 4) * (epi == EPI_SILU ? 2 : 1);
    int rows = kEngSlotBytes / rb;
    if (rows > 4 * kEngConsumerWarps) rows = 4 * kEngConsumerWarps;
    if (rows >= kEngConsumerWarps) rows -= rows % kEngConsumerWarps;
    return rows < 1 ? 1 : rows;
}

int engine_smem_bytes(int n_groups, int n_ops, int n_stages) {
    const size_t b = (size_t)kEngSlots * kEngSlotBytes + 8192 + (size_t)n_ops * sizeof(EngOp) +
                     (size_t)n_groups * sizeof(EngGroup) + (size_t)n_stages * 2 * sizeof(EngCursor);
    const size_t limit = 227 * 1024 - sizeof(EngSmem) - 64;
    return b <= limit ? (int)b : 0;
}

int engine_grid(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) sms = 148;
    return sms;
}

cudaError_t prepare_engine() {
    // the largest dynamic shared memory any program may ask for
    return cudaFuncSetAttribute(i2s_engine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                227 * 1024 - (int)sizeof(EngSmem) - 64);
}

cudaError_t launch_engine(const EngParams& p, int grid, cudaStream_t st) {
    const int smem = engine_smem_bytes(p.n_groups, p.n_ops, p.n_stages);
    if (smem == 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kEngThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;     // all CTAs co-resident: they meet at grid barriers
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, i2s_engine_kernel, p);
}

}  // namespace sllm
