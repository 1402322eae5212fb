// engine.cu -- the persistent I2_S GEMV engine for sm_100a (see engine.cuh).
//
// Per CTA (one per SM, 16 warps):
//   warp 15 (producer): walks the CTA's chunks of every stage in program
//     order and, for each, waits for a free ring slot and issues one TMA bulk
//     copy (two for a gate/up pair) of the chunk's contiguous weight rows into
//     it, with the slot's mbarrier counting the bytes. It never waits for
//     activations, so weights stream ahead across op and stage boundaries.
//   warps 0-14 (consumers): for each op, (re)build the int8 activations of
//     the op's input group when it changes (the certified RMSNorm + absmax
//     prologue of i2s_gemv.cu, shared by the 480 consumer threads), load them
//     into registers, then for each chunk wait for its slot, run the dp4a
//     dots from shared memory (R rows per warp), apply the epilogue and
//     release the slot.
//   At a stage boundary the consumers publish their outputs and meet every
//     other CTA at a grid barrier before reading the next stage's input.
//
// Exactness is the same as i2s_gemv.cu: integer dots in any order, the
// reference's float op order in the prologue and epilogues.
//
// Every wait is bounded by the global timer (2 s; a test hook may shorten
// it). A wait that gives up
// records why in *error and puts the CTA in a skip mode that still reaches
// every barrier, so the kernel always terminates; the producer then waits
// (bounded) for its own copies in flight before it exits.

#include <type_traits>

#include "attn.cuh"
#include "common.cuh"
#include "engine.cuh"

namespace sllm {

constexpr uint64_t kEngWaitNs = 2000000000ull;

// Test hooks, read by every launch (so a context's captured graphs see them):
// the budget of every bounded wait, and a CTA that leaves out its first
// grid-barrier arrival (-1: none), so that a test can make the other CTAs'
// waits run out without faulting or hanging anything.
__device__ unsigned long long g_eng_wait_ns = kEngWaitNs;
__device__ int g_eng_skip_arrival = -1;

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
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 65536;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded: false when the phase did not complete within `budget` ns
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t budget) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > budget) return false;
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

struct ConsumerSync {
    __device__ __forceinline__ void operator()() const { consumer_sync(); }
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// unsigned bytes of a times signed bytes of b, summed into c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One 32-bit weight word against its four activation words, into four field
// accumulators: field f is masked in place (not shifted), so accumulator f
// collects 4^(3-f) times its dot; they are shifted down once per row.
// Every term is exact in int32 (|acc| < 64 * 2 * 128 * K/4 < 2^25).
__device__ __forceinline__ void i2s_word_fields(uint32_t w, const int4& a, int& f0, int& f1, int& f2, int& f3) {
    f0 = dp4a_us(w & 0xC0C0C0C0u, a.x, f0);
    f1 = dp4a_us(w & 0x30303030u, a.y, f1);
    f2 = dp4a_us(w & 0x0C0C0C0Cu, a.z, f2);
    f3 = dp4a_us(w & 0x03030303u, a.w, f3);
}

__device__ __forceinline__ int fields_total(int f0, int f1, int f2, int f3) {
    return (f0 >> 6) + (f1 >> 4) + (f2 >> 2) + f3;
}

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

// --- exchange with peers (XCH instances) -------------------------------------
__device__ __forceinline__ uint32_t x_ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void x_st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// system-scope release fence: orders this CTA's stores (into peers' memory
// too; the CTA barrier before it makes them this thread's) before its next
// release. acq_rel, not the sequentially consistent fence.sc.sys of
// __threadfence_system, which also waits for a global ordering point.
__device__ __forceinline__ void x_fence_release_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ unsigned x_atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// this rank has published exchange `kind` with value `val`: flag[kind][rank]
// of every rank's region (its own included)
__device__ __forceinline__ void x_signal(const EngX& x, int kind, uint32_t val) {
    for (int q = 0; q < x.n_peer; ++q) {
        uint32_t* f = reinterpret_cast<uint32_t*>(x.peer[q] + x.flag_off) + kind * kEngMaxPeers + x.rank;
        x_st_release_sys(f, val);
    }
}

// every rank has published `kind` up to `val` (bounded by the wait budget;
// at once false when an earlier wait of this context already gave up, so a
// dead peer costs one budget, not one per exchange)
__device__ __forceinline__ bool x_wait(const EngX& x, int kind, uint32_t val, uint64_t budget, const int* error) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(x.peer[x.rank] + x.flag_off) + kind * kEngMaxPeers;
    const uint64_t t0 = gtimer();
    for (int q = 0; q < x.n_peer; ++q) {
        while (x_ld_acquire_sys(f + q) < val) {
            if (gtimer() - t0 > budget || *(volatile const int*)error != 0) return false;
            __nanosleep(32);
        }
    }
    return true;
}

// the same float or int word at the same offset of every other rank's region
template <class T>
__device__ __forceinline__ void x_scatter(const EngX& x, const T* local, T v) {
    const ptrdiff_t off = reinterpret_cast<const char*>(local) - x.peer[x.rank];
    for (int q = 0; q < x.n_peer; ++q)
        if (q != x.rank) *reinterpret_cast<T*>(x.peer[q] + off) = v;
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
    if (g.pro == PRO_Q8) {
        // already quantised (a slice of a vector another kernel normalised and
        // quantised whole): only the lane-major layout is built here
        for (int i = tid; i < K4; i += NT) {
            const int wi = ((i >> 5) << 3) + (i & 7), f = (i >> 3) & 3;
            reinterpret_cast<uint32_t*>(qs)[wi * 4 + f] = __ldcg(reinterpret_cast<const unsigned int*>(g.q8) + i);
        }
        consumer_sync();
        sllm_cuda_act a;
        a.scale = __ldcg(&g.act8->scale);
        a.sum = __ldcg(&g.act8->sum);
        return a;
    }
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
            // activation word i pairs with field f = (i % 32) / 8 of weight word
            // wi = (i / 32) * 8 + i % 8; stored at [wi][f] so that a lane
            // fetches the four words of one weight word in one 16-byte load
            const int wi = ((i >> 5) << 3) + (i & 7), f = (i >> 3) & 3;
            reinterpret_cast<uint32_t*>(qs)[wi * 4 + f] = (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) |
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
// consumers: every chunk of one op, activations held in registers
// ---------------------------------------------------------------------------
// Rows per consumer warp per chunk: as many as a slot holds for the widest
// rows of that width (K = 512 * wpl), at most 8; two for widths 13 and 14
// (n_ff = 6912 has 1728-byte rows: 28 of the 30 fit a slot, the host gives
// the chunk 28 rows and two warps recompute a row they do not store).
__host__ __device__ constexpr int eng_rows_per_warp(int wpl, bool pair) {
    return pair ? (kEngSlotBytes / (2 * kEngConsumerWarps * 128 * wpl) >= 8
                       ? 8
                       : (kEngSlotBytes / (2 * kEngConsumerWarps * 128 * wpl) < 1
                              ? 1
                              : kEngSlotBytes / (2 * kEngConsumerWarps * 128 * wpl)))
                : (wpl == 13 || wpl == 14
                       ? 2
                       : (kEngSlotBytes / (kEngConsumerWarps * 128 * wpl) >= 8
                              ? 8
                              : (kEngSlotBytes / (kEngConsumerWarps * 128 * wpl) < 1
                                     ? 1
                                     : kEngSlotBytes / (kEngConsumerWarps * 128 * wpl))));
}

// the slow path of a consumer's wait for a full slot: bounded, and quick to
// give up once the CTA is aborting
__device__ __noinline__ bool consumer_wait_full_slow(EngSmem& es, const EngParams& P, uint64_t* bar,
                                                     uint32_t parity) {
    if (*(volatile int*)&es.abort_flag) return false;
    const uint64_t budget = *(volatile unsigned long long*)&g_eng_wait_ns;
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (*(volatile int*)&es.abort_flag) return false;
        if (gtimer() - t0 > budget) {
            es.abort_flag = 1;
            atomicExch(P.error, ENG_TIMEOUT_FULL);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool consumer_wait_full(EngSmem& es, const EngParams& P, uint32_t slot, uint32_t phase) {
    if (mbar_try_wait(&es.full[slot], phase)) return true;
    return consumer_wait_full_slow(es, P, &es.full[slot], phase);
}

// R rows per warp of a plain (one-tensor) chunk, branch-free. A warp whose
// row lies past the chunk's end (a short chunk) recomputes the chunk's last
// row and never stores it; a lane whose last word lies past a partial row
// width reads the bytes after the row (inside the slot: the host leaves that
// margin, see engine_chunk_rows) and masks them to zero codes. So no
// predicate sits in the loop.
template <int WPL, int R>
__device__ __forceinline__ void plain_rows(const int4 (&aq)[WPL], const uint8_t* base, int n, int rb,
                                           uint32_t last_mask, int warp, int lane, int (&dot)[R]) {
    int acc[R][4];
    #pragma unroll
    for (int t = 0; t < R; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
    const uint32_t* rp[R];
    #pragma unroll
    for (int t = 0; t < R; ++t)
        rp[t] = reinterpret_cast<const uint32_t*>(base + (size_t)min(warp + kEngConsumerWarps * t, n - 1) * rb) + lane;
    #pragma unroll
    for (int i = 0; i < WPL; ++i) {
        #pragma unroll
        for (int t = 0; t < R; ++t) {
            uint32_t w = rp[t][32 * i];
            if (i == WPL - 1) w &= last_mask;
            i2s_word_fields(w, aq[i], acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
        }
    }
    #pragma unroll
    for (int t = 0; t < R; ++t)
        dot[t] = __reduce_add_sync(0xffffffffu, fields_total(acc[t][0], acc[t][1], acc[t][2], acc[t][3]));
}

template <int WPL, int R>
__device__ __forceinline__ void pair_rows(const int4 (&aq)[WPL], const uint8_t* base, int n, int rb,
                                          uint32_t last_mask, int warp, int lane, int (&dg)[R], int (&du)[R]) {
    #pragma unroll
    for (int t = 0; t < R; ++t) {
        const int j = min(warp + kEngConsumerWarps * t, n - 1);
        int g0 = 0, g1 = 0, g2 = 0, g3 = 0, u0 = 0, u1 = 0, u2 = 0, u3 = 0;
        const uint32_t* rg = reinterpret_cast<const uint32_t*>(base + (size_t)j * rb) + lane;
        const uint32_t* ru = reinterpret_cast<const uint32_t*>(base + (size_t)(n + j) * rb) + lane;
        #pragma unroll
        for (int i = 0; i < WPL; ++i) {
            uint32_t wg = rg[32 * i], wu = ru[32 * i];
            if (i == WPL - 1) { wg &= last_mask; wu &= last_mask; }
            i2s_word_fields(wg, aq[i], g0, g1, g2, g3);
            i2s_word_fields(wu, aq[i], u0, u1, u2, u3);
        }
        dg[t] = __reduce_add_sync(0xffffffffu, fields_total(g0, g1, g2, g3));
        du[t] = __reduce_add_sync(0xffffffffu, fields_total(u0, u1, u2, u3));
    }
}

// The ring position of the consumers: chunk k sits in slot k % kEngSlots and
// completes phase (k / kEngSlots) & 1 of that slot's barriers.
struct RingPos {
    uint32_t slot = 0, phase = 0;
    __device__ __forceinline__ void advance() {
        if (++slot == (uint32_t)kEngSlots) { slot = 0; phase ^= 1u; }
    }
};

// Every chunk of op `o` that this CTA runs in the current stage, from row r0
// to r_end, activations loaded once into registers. The chunks follow the
// producer's order (ChunkWalk::next): n = min(chunk_rows, r_end - r).
template <int WPL, bool PAIR, bool XCH>
__device__ __forceinline__ void eng_run_op(const EngOp& op, int r0, int r_end, RingPos& rp, uint8_t* ring,
                                           EngSmem& es, const int8_t* qs, int asum, float post, float post2,
                                           const EngParams& P, int warp, int lane) {
    constexpr int R = eng_rows_per_warp(WPL, PAIR);
    const int K = op.K, W = K >> 4, rb = K >> 2, chunk_rows = op.chunk_rows;
    float* const out = PAIR ? op.h : op.y;
    const float* const resid = op.epi == EPI_RESID ? op.resid : nullptr;
    const bool dots_out = op.epi == EPI_DOTS;
    const bool scatter = XCH && (op.k0x & kOpScatter) != 0;
    // the op's slice of the activations (a contraction split over ranks reads
    // its columns of the whole quantised vector; 128-element blocks keep
    // their lane-major layout, so a block-aligned slice is a byte offset)
    const int8_t* qa = XCH ? qs + (op.k0x & kOpK0Mask) : qs;
    // this lane's last word lies in the row: else it reads past the row and is masked
    const uint32_t last_mask = lane + 32 * (WPL - 1) < W ? 0xffffffffu : 0u;
    int4 aq[WPL];
    #pragma unroll
    for (int i = 0; i < WPL; ++i) {
        const int wi = lane + 32 * i;
        aq[i] = wi < W ? reinterpret_cast<const int4*>(qa)[wi] : make_int4(0, 0, 0, 0);
    }
    for (int r = r0; r < r_end;) {
        const int n = min(chunk_rows, r_end - r);
        if (consumer_wait_full(es, P, rp.slot, rp.phase)) {
            const uint8_t* base = ring + (size_t)rp.slot * kEngSlotBytes;
            if (PAIR) {
                int dg[R], du[R];
                pair_rows<WPL, R>(aq, base, n, rb, last_mask, warp, lane, dg, du);
                // h = silu(gate) * up (src/forward.c:765-778, src/ops.c:452-456)
                int mg = dg[0], mu = du[0];
                #pragma unroll
                for (int t = 1; t < R; ++t)
                    if (lane == t) { mg = dg[t]; mu = du[t]; }
                const int j = warp + kEngConsumerWarps * lane;
                if (lane < R && j < n) {
                    const float g = __fmul_rn(__int2float_rn(mg - asum), post);
                    const float u = __fmul_rn(__int2float_rn(mu - asum), post2);
                    const float hv = __fmul_rn(silu_block(g), u);
                    out[r + j] = hv;
                    if (scatter) x_scatter(P.x, out + r + j, hv);
                }
            } else {
                int dot[R];
                plain_rows<WPL, R>(aq, base, n, rb, last_mask, warp, lane, dot);
                int mine = dot[0];
                #pragma unroll
                for (int t = 1; t < R; ++t)
                    if (lane == t) mine = dot[t];
                const int j = warp + kEngConsumerWarps * lane;
                if (lane < R && j < n) {
                    if (dots_out) {
                        int* dp = reinterpret_cast<int*>(out) + r + j;
                        *dp = mine;     // raw code dot (src/i2s_gemm.c:260-269)
                        if (scatter) x_scatter(P.x, dp, mine);
                    } else {
                        float v = __fmul_rn(__int2float_rn(mine - asum), post);
                        if (resid != nullptr) v = __fadd_rn(v, __ldcg(resid + r + j));
                        out[r + j] = v;
                        if (scatter) x_scatter(P.x, out + r + j, v);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&es.empty[rp.slot]);
        rp.advance();
        r += n;
    }
}

// an op whose width this instantiation does not carry: keep the ring moving
// and flag the program (the host never builds such a program)
__device__ __forceinline__ void eng_skip_op(const EngOp& op, int r0, int r_end, RingPos& rp, EngSmem& es,
                                            const EngParams& P, int lane) {
    if (lane == 0) atomicExch(P.error, ENG_BAD_PROGRAM);
    for (int r = r0; r < r_end;) {
        const int n = min(op.chunk_rows, r_end - r);
        consumer_wait_full(es, P, rp.slot, rp.phase);
        __syncwarp();
        if (lane == 0) mbar_arrive(&es.empty[rp.slot]);
        rp.advance();
        r += n;
    }
}

// ---------------------------------------------------------------------------
// the kernel: WA, WB are the two row widths (in 32-bit words per lane) of a
// model's programs -- n_embd (every projection but down) and n_ff (down)
// ---------------------------------------------------------------------------
template <int WA, int WB, bool KV16, bool XCH>
__global__ void __launch_bounds__(kEngThreads, 1)
i2s_engine_kernel(const __grid_constant__ EngParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ EngSmem es;
    // dependents may launch now: they take each SM as this kernel's CTA there
    // exits (a no-op unless the next launch asked for programmatic serialisation)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    uint8_t* ring = smem;                                     // kEngSlots x kEngSlotBytes
    int8_t* qs = reinterpret_cast<int8_t*>(smem + kEngSlots * kEngSlotBytes);   // up to 8192 bytes
    EngOp* s_ops = reinterpret_cast<EngOp*>(smem + kEngSlots * kEngSlotBytes + 8192);
    EngGroup* s_groups = reinterpret_cast<EngGroup*>(s_ops + P.n_ops);
    EngCursor* s_cur = reinterpret_cast<EngCursor*>(s_groups + P.n_groups);   // [n_stages][2]
    AttnParams* s_attn = reinterpret_cast<AttnParams*>(s_cur + 2 * P.n_stages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;

    // the program tables, once, into shared memory: no descriptor read on the
    // critical path ever goes to L2 again
    {
        static_assert(sizeof(EngOp) % 8 == 0 && sizeof(EngGroup) % 4 == 0, "table copy granularity");
        static_assert(sizeof(EngOp) == 72, "the op table's size bounds the programs that fit in shared memory");
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
        static_assert(sizeof(AttnParams) % 8 == 0 && sizeof(EngCursor) % 8 == 0, "table copy granularity");
        const int2* asrc = reinterpret_cast<const int2*>(P.attn);
        int2* adst = reinterpret_cast<int2*>(s_attn);
        for (int i = tid; i < (int)(P.n_attn * sizeof(AttnParams) / 8); i += blockDim.x) adst[i] = __ldg(asrc + i);
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
            const uint64_t budget = *(volatile unsigned long long*)&g_eng_wait_ns;
            uint32_t k = 0;
            for (int s = 0; s < P.n_stages; ++s) {
                ChunkWalk walk{s_ops, s_cur[2 * s].op, s_cur[2 * s].row, s_cur[2 * s + 1]};
                int o, r, n, last_group = -1;
                while (walk.next(o, r, n)) {
                    if (XCH && s_ops[o].epi == kEpiReduce) continue;     // no weights
                    if (s_ops[o].epi == kEpiAttention) {
                        // no weights to stream; instead the KV cache its heads
                        // will read (positions < pos), into L2 a stage ahead
                        const AttnParams& ap = s_attn[s_ops[o].group];
                        const int pos = *(volatile const int32_t*)ap.pos_ptr;
                        const uint32_t eb = (ap.kv_f16 & kAttnKvF16) ? 2u : 4u;     // bytes per cached value
                        for (int h = r; h < r + n && pos > 0; ++h) {
                            const int kvh = h / ap.group;
                            const char* vC = reinterpret_cast<const char*>(ap.v_cache) +
                                             (size_t)kvh * ap.n_ctx * 128 * eb;
                            prefetch_l2(vC, (uint32_t)pos * 128u * eb);
                            if (((size_t)ap.n_ctx * eb) % 16 == 0) {
                                const char* kT = reinterpret_cast<const char*>(ap.k_cache) +
                                                 (size_t)kvh * 128 * ap.n_ctx * eb;
                                const uint32_t bytes = ((uint32_t)pos * eb + 15u) & ~15u;
                                for (int d = 0; d < 128; ++d) prefetch_l2(kT + (size_t)d * ap.n_ctx * eb, bytes);
                            }
                        }
                        continue;
                    }
                    // the norm vector of a group this CTA reaches: into L2 as the
                    // producer gets to it, up to a ring ahead of the prologue
                    const int gi = s_ops[o].group;
                    if (gi != last_group && s_groups[gi].norm_w != nullptr)
                        prefetch_l2(s_groups[gi].norm_w, (uint32_t)s_groups[gi].K * 4u);
                    last_group = gi;
                    const int slot = (int)(k % kEngSlots);
                    const uint32_t use = k / kEngSlots;
                    if (*(volatile int*)&es.abort_flag) break;
                    if (use > 0 && !mbar_wait(&es.empty[slot], (use - 1) & 1, budget)) {
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
            for (uint32_t j = first; j < k; ++j) mbar_wait(&es.full[j % kEngSlots], (j / kEngSlots) & 1, budget);
        }
        return;
    }

    // ---------------- consumers ----------------
    // the previous kernel's results (this program's inputs) and its reads of
    // the buffers this program writes are complete from here on; the producer
    // streams only weights, which no kernel writes, and needs no such wait
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint64_t budget = 0;
    int skip_arrival = -1;
    uint32_t xval = 0;      // this layer's exchange value in this step (XCH)
    if (tid == 0) {
        budget = *(volatile unsigned long long*)&g_eng_wait_ns;
        skip_arrival = *(volatile int*)&g_eng_skip_arrival;
        if (XCH) xval = *(volatile const uint32_t*)P.x.steps * (uint32_t)P.x.n_layer + (uint32_t)P.x.layer + 1u;
    }
    RingPos rp;
    int cur_group = -1;
    sllm_cuda_act act{0.0f, 0};
    for (int s = 0; s < P.n_stages; ++s) {
        if (s > 0) {
            // the stage's input is the previous stage's output from every CTA
            if (tid == 0) {
                bool ok = true;
                if (!*(volatile int*)&es.abort_flag) {
                    const unsigned target = (unsigned)s * (unsigned)G;
                    const uint64_t t0 = gtimer();
                    while (ld_acquire(P.barrier) < target) {
                        if (gtimer() - t0 > budget) { ok = false; break; }
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
        }
        if (XCH && s < kEngMaxXStages && (P.x.xs[s] & kXsWaitMask) != 0) {
            // the stage reads what every rank published: after the local
            // barrier CTA 0 publishes this rank's part, then all CTAs wait
            // for every rank's flag (bounded)
            if (tid == 0 && !*(volatile int*)&es.abort_flag) {
                const int kind = (P.x.xs[s] & kXsWaitMask) - 1;
                const uint32_t want = (P.x.xs[s] & kXsPrev) != 0 ? xval - 1u : xval;
                if ((P.x.xs[s] & kXsSignal) != 0 && c == 0) x_signal(P.x, kind, want);
                // a peer may still be launching its step: five budgets
                if (!x_wait(P.x, kind, want, 5 * budget, P.error)) {
                    es.abort_flag = 1;
                    atomicExch(P.error, ENG_TIMEOUT_PEER);
                }
            }
            consumer_sync();
        }
        ChunkWalk walk{s_ops, s_cur[2 * s].op, s_cur[2 * s].row, s_cur[2 * s + 1]};
        int o, r, n;
        while (walk.next(o, r, n)) {
            const EngOp& op = s_ops[o];
            // this CTA's rows of op o in this stage: [r, r_end)
            const int r_end = o == walk.end.op ? walk.end.row : op.rows;
            walk.row = r_end;
            if (op.epi == kEpiAttention) {
                // decode attention, one query head per row; the scores use the
                // activation area, so the next op rebuilds its activations
                float* sc = reinterpret_cast<float*>(qs);
                float* hq = sc + kEngAttnMaxCtx;
                for (int head = r; head < r_end; ++head)
                    attention_head_t<kEngConsumerWarps * 32, typename std::conditional<KV16, __half, float>::type>(
                        s_attn[op.group], head, tid, sc, hq, hq + kHeadDim, es.fred, es.dred, ConsumerSync());
                consumer_sync();
                if (XCH && (op.k0x & kOpScatter) != 0) {
                    // this CTA's heads to every other rank's region (the
                    // outputs just stored are visible to the CTA after the barrier)
                    for (int i = r * kHeadDim + tid; i < r_end * kHeadDim; i += kEngConsumerWarps * 32)
                        x_scatter(P.x, op.y + i, __ldcg(op.y + i));
                }
                cur_group = -1;
                continue;
            }
            if (XCH && op.epi == kEpiReduce) {
                // the epilogue of a contraction split over ranks: integer sums
                // of the slots (exact in any order), then the single-GPU float
                // sequence (src/forward.c:739-750, 790-801)
                const sllm_cuda_act a = {__ldcg(&reinterpret_cast<const sllm_cuda_act*>(op.w2)->scale),
                                         __ldcg(&reinterpret_cast<const sllm_cuda_act*>(op.w2)->sum)};
                const float pr = __fdiv_rn(op.ws, a.scale);
                const int32_t* slots = reinterpret_cast<const int32_t*>(op.w);
                for (int i = r + tid; i < r_end; i += kEngConsumerWarps * 32) {
                    int d = 0;
                    for (int q = 0; q < op.K; ++q) d += __ldcg(slots + (size_t)q * op.rows + i);
                    float v = __fmul_rn(__int2float_rn(d - a.sum), pr);
                    if (op.resid != nullptr) v = __fadd_rn(v, __ldcg(op.resid + i));
                    op.y[i] = v;
                }
                continue;
            }
            if (op.group != cur_group) {
                act = eng_prologue(s_groups[op.group], P, qs, es, tid, warp, lane);
                cur_group = op.group;
                if (XCH && c == 0 && tid == 0 && s_groups[op.group].pro != PRO_Q8 && s_groups[op.group].act8 != nullptr)
                    *const_cast<sllm_cuda_act*>(s_groups[op.group].act8) = act;
            }
            // per-tensor scales (src/quant.c:102-106): one division per tensor
            const float post = __fdiv_rn(op.ws, act.scale);
            const float post2 = op.epi == EPI_SILU ? __fdiv_rn(op.ws2, act.scale) : 0.0f;
            const int wpl = ((op.K >> 4) + 31) >> 5;
            if (wpl == WA && op.epi == EPI_SILU)
                eng_run_op<WA, true, XCH>(op, r, r_end, rp, ring, es, qs, act.sum, post, post2, P, warp, lane);
            else if (wpl == WA)
                eng_run_op<WA, false, XCH>(op, r, r_end, rp, ring, es, qs, act.sum, post, post2, P, warp, lane);
            else if (wpl == WB && op.epi != EPI_SILU)
                eng_run_op<WB, false, XCH>(op, r, r_end, rp, ring, es, qs, act.sum, post, post2, P, warp, lane);
            else
                eng_skip_op(op, r, r_end, rp, es, P, lane);
        }
        // publish this CTA's outputs of the stage, then arrive
        consumer_sync();
        if (XCH && tid == 0 && s < kEngMaxXStages && (P.x.xs[s] & kXsFence) != 0)
            x_fence_release_sys();      // the stores into peers' regions, before the arrival that orders them
        if (tid == 0 && s + 1 < P.n_stages && !(s == 0 && c == skip_arrival)) red_release_add(P.barrier, 1u);
    }
    if (XCH && P.x.end_kind >= 0 && tid == 0) {
        // the last CTA to finish publishes the kernel's exchange
        x_fence_release_sys();
        if (x_atom_add_acq_rel(P.x.done, 1u) == (unsigned)G - 1u) {
            x_signal(P.x, P.x.end_kind, xval);
            atomicExch(P.x.done, 0u);
        }
    }
}

// the (WA, WB) pairs compiled in: the 2B-4T model and the widths the tests use
#define SLLM_ENGINE_SHAPES(X) \
    X(5, 14) X(1, 1) X(1, 2) X(1, 3) X(2, 6) X(3, 6) X(16, 16) X(16, 14) X(16, 7) X(16, 8) X(16, 4) X(16, 2)
// and the pairs with an fp16-KV instance (the single-GPU decode step's widths)
#define SLLM_ENGINE_KV16_SHAPES(X) X(5, 14) X(1, 1) X(1, 2) X(1, 3) X(2, 6) X(3, 6)
// and the pairs with an instance that exchanges with peers (tensor-parallel
// programs at n_embd 8192: the O slice at 2, 4 or 8 ranks, the down chunks)
#define SLLM_ENGINE_XCH_SHAPES(X) X(16, 16) X(16, 14) X(16, 7) X(16, 8) X(16, 4) X(16, 2)

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int engine_chunk_rows(int K, int epi) {
    // Whole rounds of the consumer warps (each warp computes R rows) when they
    // fit a slot; fewer rows for very wide gate/up pairs. A lane's last word
    // may lie past a partial row's end (rows are read as whole warp words):
    // those bytes must still lie in the slot, so they count here.
    const bool pair = epi == EPI_SILU;
    const int wpl = ((K / 16) + 31) / 32;
    const size_t rb = (size_t)(K / 4) * (pair ? 2 : 1);
    const size_t overhang = (size_t)wpl * 128 - (size_t)(K / 4);
    int rows = kEngConsumerWarps * eng_rows_per_warp(wpl, pair);
    while (rows > 1 && rows * rb + overhang > (size_t)kEngSlotBytes) --rows;
    return rows;
}

// The dynamic shared memory a program may use: 227 KB less the kernel's
// static shared memory (EngSmem plus the few __shared__ words of the inlined
// stage code; 256 bytes are reserved for the latter).
constexpr int kEngDynLimit = 227 * 1024 - (int)sizeof(EngSmem) - 256;

int engine_smem_bytes(int n_groups, int n_ops, int n_stages, int n_attn) {
    static_assert(kEngAttnMaxCtx * 4 + 2 * kHeadDim * 4 <= 8192, "attention scratch fits the activation area");
    const size_t b = (size_t)kEngSlots * kEngSlotBytes + 8192 + (size_t)n_ops * sizeof(EngOp) +
                     (size_t)n_groups * sizeof(EngGroup) + (size_t)n_stages * 2 * sizeof(EngCursor) +
                     (size_t)n_attn * sizeof(AttnParams);
    return b <= (size_t)kEngDynLimit ? (int)b : 0;
}

int engine_grid(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) sms = 148;
    return sms;
}

int engine_wpl(int K) { return ((K / 16) + 31) / 32; }

bool engine_supports(int wa, int wb) {
#define SLLM_ENG_SUP(A, B) if (wa == A && wb == B) return true;
    SLLM_ENGINE_SHAPES(SLLM_ENG_SUP)
#undef SLLM_ENG_SUP
    return false;
}

bool engine_supports_xch(int wa, int wb) {
#define SLLM_ENG_SUPX(A, B) if (wa == A && wb == B) return true;
    SLLM_ENGINE_XCH_SHAPES(SLLM_ENG_SUPX)
#undef SLLM_ENG_SUPX
    return false;
}

bool engine_supports_kv16(int wa, int wb) {
#define SLLM_ENG_SUP16(A, B) if (wa == A && wb == B) return true;
    SLLM_ENGINE_KV16_SHAPES(SLLM_ENG_SUP16)
#undef SLLM_ENG_SUP16
    return false;
}

cudaError_t engine_test_faults(int skip_arrival_cta, double wait_ms) {
    const unsigned long long ns =
        wait_ms > 0.0 ? (unsigned long long)(wait_ms * 1.0e6) : (unsigned long long)kEngWaitNs;
    cudaError_t e = cudaMemcpyToSymbol(g_eng_wait_ns, &ns, sizeof ns);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_eng_skip_arrival, &skip_arrival_cta, sizeof(int));
    return e;
}

bool engine_pair_for_width(int wpl, int* wa, int* wb) {
#define SLLM_ENG_FIND(A, B) if (wpl == A) { *wa = A; *wb = B; return true; }
    SLLM_ENGINE_SHAPES(SLLM_ENG_FIND)
#undef SLLM_ENG_FIND
    return false;
}

cudaError_t prepare_engine() {
    // the largest dynamic shared memory any program may ask for; the static
    // part must fit the reserve
    const int bytes = kEngDynLimit;
    cudaError_t e = cudaSuccess;
#define SLLM_ENG_PREP_ONE(A, B, KV, X)                                                                          \
    if (e == cudaSuccess) {                                                                                      \
        cudaFuncAttributes fa{};                                                                                 \
        e = cudaFuncGetAttributes(&fa, i2s_engine_kernel<A, B, KV, X>);                                          \
        if (e == cudaSuccess && fa.sharedSizeBytes + (size_t)bytes > 227u * 1024u) e = cudaErrorInvalidValue;    \
        if (e == cudaSuccess)                                                                                    \
            e = cudaFuncSetAttribute(i2s_engine_kernel<A, B, KV, X>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                     bytes);                                                                     \
    }
#define SLLM_ENG_PREP(A, B) SLLM_ENG_PREP_ONE(A, B, false, false)
#define SLLM_ENG_PREP16(A, B) SLLM_ENG_PREP_ONE(A, B, true, false)
#define SLLM_ENG_PREPX(A, B) SLLM_ENG_PREP_ONE(A, B, false, true)
    SLLM_ENGINE_SHAPES(SLLM_ENG_PREP)
    SLLM_ENGINE_KV16_SHAPES(SLLM_ENG_PREP16)
    SLLM_ENGINE_XCH_SHAPES(SLLM_ENG_PREPX)
#undef SLLM_ENG_PREPX
#undef SLLM_ENG_PREP16
#undef SLLM_ENG_PREP
#undef SLLM_ENG_PREP_ONE
    return e;
}

cudaError_t launch_engine(const EngParams& p, int grid, cudaStream_t st, int wa, int wb) {
    const int smem = engine_smem_bytes(p.n_groups, p.n_ops, p.n_stages, p.n_attn);
    if (smem == 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kEngThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (p.n_stages > 1) {
        attr[0].id = cudaLaunchAttributeCooperative;     // all CTAs co-resident: they meet at grid barriers
        attr[0].val.cooperative = 1;
    } else {
        // no grid barrier: a CTA of this launch may take an SM as soon as the
        // previous kernel's CTA there exits (its consumers wait for that
        // kernel's results before touching activations or outputs)
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.kv16) {
#define SLLM_ENG_LAUNCH16(A, B) \
        if (wa == A && wb == B) return cudaLaunchKernelEx(&cfg, i2s_engine_kernel<A, B, true, false>, p);
        SLLM_ENGINE_KV16_SHAPES(SLLM_ENG_LAUNCH16)
#undef SLLM_ENG_LAUNCH16
        return cudaErrorNotSupported;
    }
    if (p.xch) {
#define SLLM_ENG_LAUNCHX(A, B) \
        if (wa == A && wb == B) return cudaLaunchKernelEx(&cfg, i2s_engine_kernel<A, B, false, true>, p);
        SLLM_ENGINE_XCH_SHAPES(SLLM_ENG_LAUNCHX)
#undef SLLM_ENG_LAUNCHX
        return cudaErrorNotSupported;
    }
#define SLLM_ENG_LAUNCH(A, B) \
    if (wa == A && wb == B) return cudaLaunchKernelEx(&cfg, i2s_engine_kernel<A, B, false, false>, p);
    SLLM_ENGINE_SHAPES(SLLM_ENG_LAUNCH)
#undef SLLM_ENG_LAUNCH
    return cudaErrorNotSupported;
}

}  // namespace sllm
