// i2s_gemm.cu -- the multi-token I2_S GEMM (prefill) on the sm_100a tcgen05
// tensor cores, for configs[3]: 512 tokens through the gate/up and down
// projections of a 2B-4T layer.
//
// One CTA computes MT tiles of [128 tokens x BN weight rows] (each twice,
// gate and up, for the fused SiLU form) with the int32 accumulators in tensor
// memory; the weight tile is unpacked once per k-step and used by all MT
// token tiles:
//
//   warp 0 (one lane)   TMA: per k-step of 128 elements, the MT activation
//                       tiles [128 x 128 B] (128-byte swizzle, the UMMA K-major
//                       canonical layout) and the packed weight tile
//                       [BN x 32 B] into a stage of a shared-memory ring.
//   warps 2-9           unpack: each item turns 16 packed bytes of one weight
//                       row into 64 int8 codes {0, 1, 2} in the same swizzled
//                       K-major layout. The I2_S packing makes this two logic
//                       ops per output word: field f of packed word i holds
//                       elements 32f + 4i .. 32f + 4i + 3, i.e. exactly the int8
//                       word at element 32f + 4i of natural order.
//   warp 1 (one lane)   tcgen05.mma.cta_group::1.kind::i8 (s8 x s8 -> s32,
//                       M = 128, K = 32, N = BN or 2 BN: the gate and up tiles
//                       are one K-major tile of 2 BN rows) x 4 per k-step and
//                       token tile, the token tiles interleaved, then
//                       tcgen05.commit to the stage's "empty" barrier.
//   warps 2-9 again     epilogue: warps 2-5 take token tile 0, warps 6-9 tile
//                       1; tcgen05.ld of the accumulator (warp w reads TMEM
//                       lanes 32 (w % 4) ..), minus the token's code sum, times
//                       ws / scale, SiLU(gate) * up when fused.
//
// A long single-tensor contraction is split over a cluster of SK CTAs
// (blockIdx.z): each takes a contiguous share of the k-steps, the others
// store their int32 accumulators in their idle rings, and after a cluster
// barrier the first CTA adds them through distributed shared memory before
// its epilogue; a second barrier keeps the others resident until it has read
// them. Every thread of every CTA reaches both barriers (the waits before
// them are bounded).
//
// The integer sum is exact in any order, so every dot equals the reference's
// per-token sllm_i2s_gemv bit for bit; the epilogue is the GEMV epilogue's
// float sequence. Every wait is bounded by the global timer; a wait that
// gives up records an error, the CTA stops issuing work, drains what it has
// in flight (bounded) and frees its tensor memory before it exits.

#include <algorithm>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "gemm.cuh"

namespace sllm {
namespace {

constexpr int kBM = 128;          // tokens per tile (TMEM lanes)
constexpr int kBK = 128;          // elements (= activation bytes) per k-step
constexpr int kPK = kBK / 4;      // packed weight bytes per row per k-step
constexpr int kGmUnpackWarps = 8;
constexpr int kGmThreads = 64 + 32 * kGmUnpackWarps;   // TMA, MMA, 8 unpack / epilogue warps
constexpr uint64_t kGmWaitNs = 2000000000ull;

enum GemmError { GM_OK = 0, GM_TIMEOUT = 1 };

template <int BN, bool PAIR, int MT>
struct GemmCfg {
    static constexpr int NM = PAIR ? 2 : 1;
    static constexpr int A_BYTES = kBM * kBK;
    static constexpr int B_BYTES = BN * kBK;
    static constexpr int P_BYTES = BN * kPK;
    static constexpr int STAGE = MT * A_BYTES + NM * (B_BYTES + P_BYTES);   // a multiple of 1024
    static constexpr int S = (225280 / STAGE) > 6 ? 6 : (225280 / STAGE);
    static constexpr int SMEM = S * STAGE + 1024;                           // + room to align to 1024
    // a token tile's accumulator starts at a power-of-two column: gate at
    // +0, up at +BN, the next token tile at +TILE_COLS
    static constexpr int TILE_COLS = NM * BN <= 32 ? 32 : NM * BN <= 64 ? 64 : NM * BN <= 128 ? 128 : 256;
    static constexpr int TMEM_COLS = MT * TILE_COLS;                        // allocated: a power of two
    static_assert(STAGE % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "tile width");
    static_assert(MT == 1 || MT == 2, "token tiles per CTA (one epilogue warp group each)");
    static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
    static_assert(NM * BN <= 256, "one MMA covers the tensors' rows (N <= 256)");
    static_assert(S >= 2, "ring depth");
    static_assert(S * STAGE >= 8 * 8192, "the epilogue's staging boxes live in the ring");
    static_assert(NM * BN <= 256, "one MMA covers the tensors' rows (N <= 256)");
};

struct GemmKParams {
    const sllm_cuda_act* acts;
    const float* ws;       // the scale tail of w
    const float* ws2;      // ... of w2 (PAIR)
    int32_t* dots;
    float* y;
    int M, N, K;
    int* error;
    int tma_out;           // 1: outputs leave through the tensor maps tm_y / tm_d
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
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

// bounded wait: false when the phase did not complete in time, or when the
// CTA is aborting. The first check is inline: the single MMA-issuing thread
// waits once per k-step, and an out-of-line call there cost ~0.1 us each.
__device__ __noinline__ bool gm_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* error,
                                         bool sleep);
__device__ __forceinline__ bool gm_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* error,
                                        bool sleep = false) {
    if (mbar_try_wait(bar, parity)) return true;
    return gm_wait_slow(bar, parity, abort_flag, error, sleep);
}
__device__ __noinline__ bool gm_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* error,
                                         bool sleep) {
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (gtimer() - t0 > kGmWaitNs) {
            *abort_flag = 1;
            atomicExch(error, GM_TIMEOUT);
            return false;
        }
        // waits off the k-loop's critical path (the epilogue's, the
        // producer's) poll less often
        if (sleep) __nanosleep(32);
    }
    return true;
}

// a whole warp's wait, the same answer in every lane
__device__ __forceinline__ bool gm_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* error,
                                             bool sleep = false) {
    return __all_sync(0xffffffffu, gm_wait(bar, parity, abort_flag, error, sleep));
}

// drain: wait for a phase that must complete (work already in flight);
// bounded, never looks at the abort flag
__device__ __noinline__ void gm_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity))
        if (gtimer() - t0 > kGmWaitNs) return;
}

// a 2-D TMA tile load (no multicast) completing on bar
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// a 2-D TMA tile store from shared memory, tracked by the bulk-group counter
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }

// one warp's 32 rows x 32 four-byte values (lane = row) into a 4 KB staging
// box in the 128-byte swizzle the output tensor maps use: chunk j of row r
// at chunk j ^ (r % 8); eight consecutive lanes cover all 32 banks
__device__ __forceinline__ void stage_row32(uint8_t* box, int lane, const uint32_t (&v)[32]) {
    #pragma unroll
    for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor of a K-major tile in the 128-byte swizzle
// canonical layout: rows of 128 bytes, 8-row groups 1024 bytes apart
// (SBO), the 16-byte chunk index of row r XOR-ed with r % 8. LBO is unused
// for swizzled K-major layouts (1 by convention); version 1 (sm_100);
// layout type 2 = 128-byte swizzle. The tile base is 1024-byte aligned, so
// base_offset is 0 and a K offset inside the 128-byte row is added to the
// start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// instruction descriptor, kind::i8: D s32, A s8, B s8, both K-major, M, N
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 consecutive accumulator columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// the codes of one packed word, field f: four int8 codes of consecutive elements
__device__ __forceinline__ uint32_t field_codes(uint32_t w, int f) { return (w >> (6 - 2 * f)) & 0x03030303u; }

template <int BN, bool PAIR, int MT, int SK>
__global__ void __launch_bounds__(kGmThreads, 1)
i2s_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_y,
                const __grid_constant__ CUtensorMap tm_d, const GemmKParams p) {
    using C = GemmCfg<BN, PAIR, MT>;
    extern __shared__ uint8_t gsm_raw[];
    __shared__ uint64_t bar_loaded[C::S], bar_unpacked[C::S], bar_empty[C::S], bar_acc;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    uint8_t* const gsm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * (MT * kBM);
    // SK > 1: the CTAs of a cluster (blockIdx.z = 0..SK-1) split the
    // contraction; this CTA takes k-steps [kb0, kb0 + KB)
    const int KB_all = p.K / kBK;
    const int kb0 = (int)((long long)blockIdx.z * KB_all / SK);
    const int KB = (int)((long long)(blockIdx.z + 1) * KB_all / SK) - kb0;
    // token tiles of this CTA that hold tokens (the last CTA row may have fewer)
    const int mt_live = min(MT, (p.M - m0 + kBM - 1) / kBM);
    auto A = [&](int s, int mt) { return gsm + (size_t)s * C::STAGE + mt * C::A_BYTES; };
    auto B = [&](int s, int mat) { return gsm + (size_t)s * C::STAGE + MT * C::A_BYTES + mat * C::B_BYTES; };
    auto P = [&](int s, int mat) {
        return gsm + (size_t)s * C::STAGE + MT * C::A_BYTES + C::NM * C::B_BYTES + mat * C::P_BYTES;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&bar_loaded[s], 1);
            mbar_init(&bar_unpacked[s], kGmUnpackWarps);
            mbar_init(&bar_empty[s], 1);
        }
        mbar_init(&bar_acc, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int* const abort_v = &abort_flag;
    // launched with programmatic stream serialisation: the set-up above
    // overlaps the previous launch, whose outputs (the activation codes and
    // their scales) are complete and visible past this point; a no-op in an
    // ordinary launch
    asm volatile("griddepcontrol.wait;" ::: "memory");

    bool ep_ok = false;     // epilogue warps: the accumulators are complete and no CTA aborted
    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % C::S;
                const uint32_t use = (uint32_t)(kb / C::S);
                if (use > 0 && !gm_wait(&bar_empty[s], (use - 1) & 1u, abort_v, p.error, true)) break;
                mbar_expect_tx(&bar_loaded[s], (uint32_t)(mt_live * C::A_BYTES + C::NM * C::P_BYTES));
                for (int mt = 0; mt < mt_live; ++mt)
                    tma_load_2d(A(s, mt), &tm_a, (kb0 + kb) * kBK, m0 + mt * kBM, &bar_loaded[s]);
                tma_load_2d(P(s, 0), &tm_w, (kb0 + kb) * kPK, n0, &bar_loaded[s]);
                if (PAIR) tma_load_2d(P(s, 1), &tm_w2, (kb0 + kb) * kPK, n0, &bar_loaded[s]);
                ++issued;
            }
            // every copy issued lands before the CTA may exit
            for (int kb = issued > C::S ? issued - C::S : 0; kb < issued; ++kb)
                gm_drain(&bar_loaded[kb % C::S], (uint32_t)(kb / C::S) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // the gate and up tiles are adjacent in shared memory (rows 0..BN-1
            // and BN..2BN-1 of one K-major tile), so one MMA of N = 2 BN
            // computes both, into accumulator columns [0, BN) and [BN, 2 BN)
            constexpr uint32_t idesc = umma_idesc_i8(kBM, C::NM * BN);
            int issued = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % C::S;
                const uint32_t ph = (uint32_t)(kb / C::S) & 1u;
                // the unpack warps arrive only after the stage's copies landed,
                // so this one wait covers the activation tiles too
                if (!gm_wait(&bar_unpacked[s], ph, abort_v, p.error)) break;
                tc_fence_after();
                const uint32_t b0 = smem_u32(B(s, 0));
                #pragma unroll
                for (int kk = 0; kk < kBK / 32; ++kk) {
                    #pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        if (mt < mt_live)
                            umma_i8(tmem + (uint32_t)(mt * C::TILE_COLS), umma_desc_sw128(smem_u32(A(s, mt)) + 32u * kk),
                                    umma_desc_sw128(b0 + 32u * kk), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&bar_empty[s]);     // the stage may be refilled once these MMAs have read it
                ++issued;
            }
            umma_commit(&bar_acc);              // the accumulators are complete (or the CTA aborted)
            // the MMAs issued have finished reading shared memory before exit
            if (issued > 0) gm_drain(&bar_empty[(issued - 1) % C::S], (uint32_t)((issued - 1) / C::S) & 1u);
        }
        __syncwarp();
    } else {
        // ---------------- unpack, then epilogue (warps 2-9) ----------------
        constexpr int NT = 32 * kGmUnpackWarps;
        const int t = threadIdx.x - 64;     // 0..NT-1
        bool ok = true;
        for (int kb = 0; kb < KB && ok; ++kb) {
            const int s = kb % C::S;
            const uint32_t ph = (uint32_t)(kb / C::S) & 1u;
            ok = gm_wait_warp(&bar_loaded[s], ph, abort_v, p.error);
            if (ok) {
                // items: (matrix, half, row); eight consecutive threads take eight
                // consecutive rows, so their 16-byte stores hit eight distinct
                // swizzled chunks (no bank conflict)
                #pragma unroll
                for (int it = t; it < C::NM * 2 * BN; it += NT) {
                    const int row = it % BN, h = (it / BN) & 1, mat = it / (2 * BN);
                    const uint4 v = *reinterpret_cast<const uint4*>(P(s, mat) + row * kPK + h * 16);
                    uint8_t* brow = B(s, mat) + row * kBK;
                    #pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        uint4 o;
                        o.x = field_codes(v.x, f);
                        o.y = field_codes(v.y, f);
                        o.z = field_codes(v.z, f);
                        o.w = field_codes(v.w, f);
                        const int chunk = (2 * f + h) ^ (row & 7);
                        *reinterpret_cast<uint4*>(brow + chunk * 16) = o;
                    }
                }
                fence_proxy_async_smem();       // the tensor core reads through the async proxy
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_unpacked[s]);
            ok = __all_sync(0xffffffffu, ok);
        }
        // epilogue: warp group mt (warps 2-5: 0, warps 6-9: 1) takes token tile mt
        ep_ok = __all_sync(0xffffffffu, ok && gm_wait_warp(&bar_acc, 0u, abort_v, p.error, true)) &&
                __all_sync(0xffffffffu, *abort_v == 0);
    }
    const int mt = (warp - 2) >> 2;
    const int quarter = warp & 3;
    // SK > 1: a split CTA's accumulator columns, [col][lane] per epilogue warp
    // in its (now idle) ring, 32 lanes x BN columns
    uint32_t* const part = reinterpret_cast<uint32_t*>(gsm + (size_t)(warp >= 2 ? warp - 2 : 0) * (BN * 128));
    if constexpr (SK > 1) {
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        if (warp >= 2 && cl.block_rank() != 0 && ep_ok && mt < mt_live) {
            tc_fence_after();
            const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(mt * C::TILE_COLS);
            #pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t g[32];
                tmem_ld32(lane_base + (uint32_t)c0, g);
                tmem_ld_wait();
                #pragma unroll
                for (int j = 0; j < 32; ++j) part[(c0 + j) * 32 + lane] = g[j];
            }
        }
        cl.sync();      // every thread of every CTA of the cluster
    }
    bool lead = true;
    if constexpr (SK > 1) lead = cooperative_groups::this_cluster().block_rank() == 0;
    if (warp >= 2) {
        if (ep_ok && lead && mt < mt_live) {
            tc_fence_after();
            const int row0 = m0 + mt * kBM + 32 * quarter;      // this warp's first token
            const int m = row0 + lane;
            const bool live = m < p.M;
            sllm_cuda_act act{1.0f, 0};
            if (live) act = p.acts[m];
            // per-tensor scale over the token's activation scale (src/forward.c:653-655)
            const float post = __fdiv_rn(__ldg(p.ws), act.scale);
            const float post2 = PAIR ? __fdiv_rn(__ldg(p.ws2), act.scale) : 0.0f;
            const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(mt * C::TILE_COLS);
            // two 4 KB staging boxes per warp in the (now idle) ring: the store
            // of one drains while the other fills
            uint8_t* const stg = gsm + (size_t)(warp - 2) * 8192;
            int nst = 0;        // stores committed by this warp
            auto stage_out = [&](const CUtensorMap* tm, const uint32_t (&v)[32], int col) {
                uint8_t* box = stg + (nst & 1) * 4096;
                if (nst >= 2 && lane == 0) bulk_wait_read<1>();   // the store that last read this box
                __syncwarp();
                stage_row32(box, lane, v);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(tm, box, col, row0);    // rows >= M, columns >= N are clipped
                    bulk_commit();
                }
                ++nst;
            };
            #pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t g[32];
                tmem_ld32(lane_base + (uint32_t)c0, g);
                if (PAIR) {
                    uint32_t u[32];
                    tmem_ld32(lane_base + (uint32_t)(BN + c0), u);
                    tmem_ld_wait();
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        // h = silu(gate) * up (src/forward.c:765-778, src/ops.c:452-456)
                        const float gv = __fmul_rn(__int2float_rn((int)g[j] - act.sum), post);
                        const float uv = __fmul_rn(__int2float_rn((int)u[j] - act.sum), post2);
                        u[j] = __float_as_uint(__fmul_rn(silu_block(gv), uv));
                    }
                    if (p.tma_out) {
                        stage_out(&tm_y, u, n0 + c0);
                    } else if (live) {
                        float* yrow = p.y + (size_t)m * p.N;
                        #pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + c0 + j < p.N) yrow[n0 + c0 + j] = __uint_as_float(u[j]);
                    }
                } else {
                    tmem_ld_wait();
                    if constexpr (SK > 1) {
                        // the other CTAs' partial dots of these columns (int32: exact)
                        namespace cg = cooperative_groups;
                        cg::cluster_group cl = cg::this_cluster();
                        #pragma unroll 1
                        for (int r = 1; r < SK; ++r) {
                            const uint32_t* rp = cl.map_shared_rank(part, r);
                            #pragma unroll
                            for (int j = 0; j < 32; ++j) g[j] += rp[(c0 + j) * 32 + lane];
                        }
                    }
                    if (p.tma_out) {
                        if (p.dots != nullptr) stage_out(&tm_d, g, n0 + c0);
                        if (p.y != nullptr) {
                            #pragma unroll
                            for (int j = 0; j < 32; ++j)
                                g[j] = __float_as_uint(__fmul_rn(__int2float_rn((int)g[j] - act.sum), post));
                            stage_out(&tm_y, g, n0 + c0);
                        }
                    } else if (live) {
                        #pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int n = n0 + c0 + j;
                            if (n < p.N) {
                                if (p.dots != nullptr) p.dots[(size_t)m * p.N + n] = (int)g[j];
                                if (p.y != nullptr)
                                    p.y[(size_t)m * p.N + n] = __fmul_rn(__int2float_rn((int)g[j] - act.sum), post);
                            }
                        }
                    }
                }
            }
            // the staging boxes are read before the CTA exits
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
        }
    }
    if constexpr (SK > 1) cooperative_groups::this_cluster().sync();   // the leader has read the partials
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// The skinny form: at most 16 tokens (a decode step of a batch of sequences).
// The roles swap: 128 weight rows are the MMA's M operand, unpacked into
// shared memory as above, and the tokens are its N = 16 operand (one TMA box
// of 16 rows x 128 bytes, zero past m), so no MMA column is padding. The
// accumulator is 128 TMEM lanes (weight rows) x 16 columns (tokens).
//
// One launch covers up to four weight tensors ("segments") that share the
// activation matrix: Q, K and V, or the column chunks of down, each with its
// own column offset into the activations. A tile is 128 rows of one tensor,
// or, for the gate/up pair, 64 rows of gate over the same 64 rows of up
// (TMEM lanes 0-63 and 64-127). The grid is persistent: CTA c takes tiles
// c, c + G, ..., two CTAs per SM.
//
//   warp 0 (one lane)   TMA: per stage of four k-steps, the four activation
//                       boxes and the next 128 bytes of every weight row of
//                       the tile (128-byte swizzle), three stages in flight.
//   warps 2-9           unpack a k-step's packed bytes into one of two 16 KB
//                       operand stages (a quarter warp takes rows r, r + 2,
//                       r + 4, r + 6, both halves: its loads and stores land on
//                       eight distinct 16-byte chunks).
//   warp 1 (one lane)   tcgen05.mma kind::i8, M = 128, N = 16, K = 32, x 4 per
//                       k-step into one of two accumulators (tile parity);
//                       commits free the operand stage, the packed stage and,
//                       after a tile's last k-step, fill the accumulator.
//                       (Issuing from the unpack warps behind a named barrier
//                       measured slower.)
//   warps 10-13         epilogue: tcgen05.ld of the accumulator (warp w: TMEM
//                       lanes 32 (w % 4) ..), which then returns to the MMA
//                       warp, so a tile's epilogue overlaps the next tile's
//                       k-loop; one lane per weight row, the stores of a
//                       token's outputs coalesced. For the pair the up lanes
//                       hand their sums to the gate lanes through shared
//                       memory (bounded mbarrier hand-over).
//
// A grid shorter than two CTAs per SM instead splits the contraction over a
// cluster of SK CTAs, one tile each, as the 128-token form does.
// ---------------------------------------------------------------------------
constexpr int kSkM = 128;       // operand rows per tile (MMA M, TMEM lanes)
constexpr int kSkN = 16;        // tokens (MMA N)
constexpr int kSkMaxSeg = 4;
constexpr int kSkSp = 4;        // packed stages in shared memory
constexpr int kSkSa = 6;        // operand stages in tensor memory
constexpr int kSkG = 4;         // k-steps per packed stage: 128-byte segments of every weight row
constexpr int kSkPStage = kSkG * kSkN * kBK + kSkM * kSkG * kPK;    // 4 activation boxes + packed weights: 24 KB
constexpr int kSkACols = kBK / 4;                       // TMEM columns of one operand stage (4 codes each)
constexpr int kSkAcc = 2 * kSkN;                        // two accumulators of 16 columns at column 0
constexpr int kSkTmemCols = 256;                        // accumulators + operand stages; two CTAs per SM
__host__ __device__ constexpr int skinny_smem(bool) { return kSkSp * kSkPStage + 1024; }
constexpr int kSkEpiWarp0 = 2 + kGmUnpackWarps;        // warps 10-13
constexpr int kSkThreads = 32 * (kSkEpiWarp0 + 4);
static_assert(kSkPStage % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
static_assert(kSkAcc + kSkSa * kSkACols <= kSkTmemCols, "operand stages fit the allocation");
static_assert(kGmUnpackWarps == 8, "two unpack warps per TMEM lane quarter, one half of each row");
static_assert(kSkSp * kSkPStage >= kSkN * kSkM * 4, "a split CTA's partial sums fit the packed ring");

struct SkParams {
    CUtensorMap act;                    // [m][cols] int8, box 128 x 16, 128-byte swizzle
    CUtensorMap w[kSkMaxSeg];           // packed rows, box 32 B x (128 or 64 for the pair)
    CUtensorMap w2[kSkMaxSeg];          // the pair's up tensor
    int tile_end[kSkMaxSeg];            // cumulative tile counts
    int n_rows[kSkMaxSeg];
    int kx[kSkMaxSeg];                  // the segment's first activation column
    const float* ws[kSkMaxSeg];
    const float* ws2[kSkMaxSeg];
    int32_t* dots[kSkMaxSeg];
    float* y[kSkMaxSeg];
    const sllm_cuda_act* acts;
    int* error;
    int nseg, tiles, M, K;
};

// 16 consecutive accumulator columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void umma_commit_to(uint64_t* bar) { umma_commit(bar); }

// the MMA with its A operand (M = 128 lanes x K = 32 int8, four per column)
// in tensor memory
__device__ __forceinline__ void umma_i8_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// four consecutive 32-bit columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <bool PAIR, int SK>
__global__ void __launch_bounds__(kSkThreads, 2)
i2s_gemm_skinny_kernel(const __grid_constant__ SkParams P) {
    constexpr int TR = PAIR ? 64 : 128;          // weight rows per tile (of each tensor)
    constexpr int SP = kSkSp;
    extern __shared__ uint8_t gsm_raw[];
    __shared__ uint64_t bar_loaded[kSkSp], bar_pempty[kSkSp], bar_unpacked[kSkSa], bar_aempty[kSkSa];
    __shared__ uint64_t bar_full[2], bar_drained[2], bar_xfull, bar_xfree;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ float s_up[PAIR ? kSkN * 64 : 1];          // [token][64 rows]
    uint8_t* const gsm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto PS = [&](int sp) { return gsm + (size_t)sp * kSkPStage; };
    const int KB_all = P.K / kBK;
    const int kb0 = SK > 1 ? (int)((long long)blockIdx.z * KB_all / SK) : 0;
    const int KB = SK > 1 ? (int)((long long)(blockIdx.z + 1) * KB_all / SK) - kb0 : KB_all;   // >= 2
    const int t_first = blockIdx.x, t_step = SK > 1 ? P.tiles : gridDim.x;
    auto seg_of = [&](int t, int* row0) {
        int sg = 0;
        while (sg + 1 < P.nseg && t >= P.tile_end[sg]) ++sg;
        *row0 = (t - (sg > 0 ? P.tile_end[sg - 1] : 0)) * TR;
        return sg;
    };
    // each tile walks its packed stages (groups of four k-steps) starting at
    // group t % NG, so the CTAs running at one time read different columns of
    // the shared activation matrix (it sits in a few L2 slices otherwise);
    // the int32 sums do not depend on the order
    const int NG = (KB + kSkG - 1) / kSkG;
    auto group_of = [&](int t, int gi) { return (gi + t) % NG; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < SP; ++i) {
            mbar_init(&bar_loaded[i], 1);
            mbar_init(&bar_pempty[i], 1);
        }
        for (int i = 0; i < kSkSa; ++i) {
            mbar_init(&bar_unpacked[i], kGmUnpackWarps);
            mbar_init(&bar_aempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar_full[i], 1);
            mbar_init(&bar_drained[i], 4);
        }
        mbar_init(&bar_xfull, 2);
        mbar_init(&bar_xfree, 2);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)kSkTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int* const abort_v = &abort_flag;
    // no kernel writes the weights, so the weight boxes of the first SP packed
    // stages go out before the wait for the previous launch (programmatic
    // serialisation: that launch may still be running); each stage's barrier
    // expects the whole stage, so it completes only once the activation boxes
    // issued after the wait have landed too. The producer loop issues those
    // first SP stages' activations before its first wait, so every box sent
    // here lands before the CTA can exit.
    int pre = 0;
    if (warp == 0 && lane == 0) {
        for (int t = t_first; t < P.tiles && pre < SP; t += t_step) {
            int row0;
            const int sg = seg_of(t, &row0);
            for (int gi = 0; gi < NG && pre < SP; ++gi, ++pre) {
                const int kb = kb0 + kSkG * group_of(t, gi);
                mbar_expect_tx(&bar_loaded[pre], (uint32_t)kSkPStage);
                uint8_t* pw = PS(pre) + kSkG * kSkN * kBK;
                tma_load_2d(pw, &P.w[sg], kb * kPK, row0, &bar_loaded[pre]);
                if (PAIR) tma_load_2d(pw + 64 * kSkG * kPK, &P.w2[sg], kb * kPK, row0, &bar_loaded[pre]);
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int quarter = warp & 3;
    uint32_t g[16];                      // SK > 1: the epilogue warps' one tile
    bool ep_ok = false;

    // the outputs of tile t (j: this CTA's tile count, for the hand-over
    // buffer's parity) from this lane's 16 sums
    auto finish_tile = [&](int j, int t, const uint32_t (&v)[16]) -> bool {
        int row0;
        const int sg = seg_of(t, &row0);
        if (PAIR) {
            const uint32_t par = (uint32_t)j & 1u;
            float* up = s_up;
            if (quarter >= 2) {
                // up rows 0..63 of the tile are TMEM lanes 64..127
                if (j >= 1 && !gm_wait_warp(&bar_xfree, par ^ 1u, abort_v, P.error, true)) return false;
                #pragma unroll
                for (int jj = 0; jj < kSkN; ++jj) up[jj * 64 + 32 * (quarter - 2) + lane] = __int_as_float((int)v[jj]);
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_xfull);
                return true;
            }
            if (!gm_wait_warp(&bar_xfull, par, abort_v, P.error, true)) return false;
            const int n = row0 + 32 * quarter + lane;
            if (n < P.n_rows[sg]) {
                const float ws = __ldg(P.ws[sg]), ws2 = __ldg(P.ws2[sg]);
                float* y = P.y[sg];
                #pragma unroll
                for (int jj = 0; jj < kSkN; ++jj) {
                    if (jj < P.M) {
                        const sllm_cuda_act act = P.acts[jj];
                        // h = silu(gate) * up (src/forward.c:765-778, src/ops.c:452-456)
                        const float post = __fdiv_rn(ws, act.scale), post2 = __fdiv_rn(ws2, act.scale);
                        const int uv_i = __float_as_int(up[jj * 64 + 32 * quarter + lane]);
                        const float gv = __fmul_rn(__int2float_rn((int)v[jj] - act.sum), post);
                        const float uv = __fmul_rn(__int2float_rn(uv_i - act.sum), post2);
                        y[(size_t)jj * P.n_rows[sg] + n] = __fmul_rn(silu_block(gv), uv);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_xfree);
            return true;
        }
        const int n = row0 + 32 * quarter + lane;
        if (n < P.n_rows[sg]) {
            const float ws = __ldg(P.ws[sg]);
            int32_t* dots = P.dots[sg];
            float* y = P.y[sg];
            #pragma unroll
            for (int jj = 0; jj < kSkN; ++jj) {
                if (jj < P.M) {
                    const size_t o = (size_t)jj * P.n_rows[sg] + n;
                    if (dots != nullptr) dots[o] = (int)v[jj];
                    if (y != nullptr) {
                        const sllm_cuda_act act = P.acts[jj];
                        // per-tensor scale over the token's activation scale (src/forward.c:653-655)
                        y[o] = __fmul_rn(__int2float_rn((int)v[jj] - act.sum), __fdiv_rn(ws, act.scale));
                    }
                }
            }
        }
        return true;
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int gs = 0;      // packed stages issued
            bool ok = true;
            for (int t = t_first; t < P.tiles && ok; t += t_step) {
                int row0;
                const int sg = seg_of(t, &row0);
                for (int gi = 0; gi < NG; ++gi, ++gs) {
                    const int kb = kb0 + kSkG * group_of(t, gi);
                    const int sp = gs % SP;
                    const uint32_t use = (uint32_t)(gs / SP);
                    if (use > 0 && !gm_wait(&bar_pempty[sp], (use - 1) & 1u, abort_v, P.error, true)) { ok = false; break; }
                    if (gs >= pre) mbar_expect_tx(&bar_loaded[sp], (uint32_t)kSkPStage);
                    uint8_t* st = PS(sp);
                    #pragma unroll
                    for (int i = 0; i < kSkG; ++i)      // columns past the contraction read as zeros
                        tma_load_2d(st + i * (kSkN * kBK), &P.act, P.kx[sg] + (kb + i) * kBK, 0, &bar_loaded[sp]);
                    if (gs >= pre) {             // else its weights went out before the wait
                        uint8_t* pw = st + kSkG * kSkN * kBK;
                        tma_load_2d(pw, &P.w[sg], kb * kPK, row0, &bar_loaded[sp]);
                        if (PAIR) tma_load_2d(pw + 64 * kSkG * kPK, &P.w2[sg], kb * kPK, row0, &bar_loaded[sp]);
                    }
                }
            }
            for (int i = gs > SP ? gs - SP : 0; i < gs; ++i)
                gm_drain(&bar_loaded[i % SP], (uint32_t)(i / SP) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_i8(kSkM, kSkN);
            int gk = 0, gs = 0, j = 0;
            bool ok = true;
            for (int t = t_first; t < P.tiles && ok; t += t_step, ++j) {
                const int buf = j & 1;
                if (j >= 2 && !gm_wait(&bar_drained[buf], (uint32_t)((j >> 1) - 1) & 1u, abort_v, P.error)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * kSkN);
                for (int gi = 0; gi < NG && ok; ++gi) {
                    const int g = group_of(t, gi), nk = min(kSkG, KB - kSkG * g);
                    for (int sub = 0; sub < nk; ++sub, ++gk) {
                        const int sa = gk % kSkSa, sp = gs % SP;
                        if (!gm_wait(&bar_unpacked[sa], (uint32_t)(gk / kSkSa) & 1u, abort_v, P.error)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t a0 = tmem + (uint32_t)(kSkAcc + sa * kSkACols);
                        const uint32_t b0 = smem_u32(PS(sp) + sub * (kSkN * kBK));
                        #pragma unroll
                        for (int kk = 0; kk < kBK / 32; ++kk)
                            umma_i8_ta(d, a0 + 8u * kk, umma_desc_sw128(b0 + 32u * kk), idesc,
                                       (gi > 0 || sub > 0 || kk > 0) ? 1u : 0u);
                        umma_commit_to(&bar_aempty[sa]);
                        if (sub == nk - 1) {      // the packed stage's last k-step
                            umma_commit_to(&bar_pempty[sp]);
                            ++gs;
                        }
                    }
                }
                if (ok) umma_commit_to(&bar_full[buf]);
            }
            if (gk > 0) gm_drain(&bar_aempty[(gk - 1) % kSkSa], (uint32_t)((gk - 1) / kSkSa) & 1u);
        }
        __syncwarp();
    } else if (warp < kSkEpiWarp0) {
        // ---------------- unpack (warps 2-9) ----------------
        // warp w writes TMEM lanes 32 (w % 4) .. + 31 (rows of the tile), lane
        // i row 32 (w % 4) + i; warps 2-5 take the first 16 packed bytes of
        // each row, warps 6-9 the second. Packed word i, field f holds the
        // codes of natural word 8 f + i of the k-step (elements 32 f + 4 i ..),
        // so each field of the thread's four words is four consecutive
        // operand columns: four 32x32b.x4 stores per k-step. The eight lanes
        // of a quarter warp read eight consecutive rows' same logical chunk,
        // eight distinct swizzled chunks.
        const int row = 32 * (warp & 3) + lane, hh = (warp - 2) >> 2;
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        int gk = 0, gs = 0;
        bool ok = true;
        for (int t = t_first; t < P.tiles && ok; t += t_step) {
            for (int gi = 0; gi < NG && ok; ++gi) {
                const int g = group_of(t, gi), nk = min(kSkG, KB - kSkG * g);
                for (int sub = 0; sub < nk; ++sub, ++gk) {
                    const int sp = gs % SP, sa = gk % kSkSa;
                    if (sub == 0) ok = gm_wait_warp(&bar_loaded[sp], (uint32_t)(gs / SP) & 1u, abort_v, P.error);
                    if (ok && gk >= kSkSa)
                        ok = gm_wait_warp(&bar_aempty[sa], (uint32_t)((gk / kSkSa) - 1) & 1u, abort_v, P.error);
                    if (ok) {
                        tc_fence_after();
                        const int chunk = (2 * sub + hh) ^ (row & 7);
                        const uint4 v = *reinterpret_cast<const uint4*>(PS(sp) + kSkG * kSkN * kBK +
                                                                        row * (kSkG * kPK) + (chunk << 4));
                        const uint32_t col = lane_addr + (uint32_t)(kSkAcc + sa * kSkACols + 4 * hh);
                        #pragma unroll
                        for (int f = 0; f < 4; ++f)
                            tmem_st4(col + 8u * f, field_codes(v.x, f), field_codes(v.y, f), field_codes(v.z, f),
                                     field_codes(v.w, f));
                        tmem_st_wait();
                        tc_fence_before();
                    }
                    if (sub == nk - 1) ++gs;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_unpacked[sa]);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 10-13) ----------------
        const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
        int j = 0;
        bool ok = true;
        for (int t = t_first; t < P.tiles && ok; t += t_step, ++j) {
            const int buf = j & 1;
            ok = gm_wait_warp(&bar_full[buf], (uint32_t)(j >> 1) & 1u, abort_v, P.error, true);
            if (!ok) break;
            tc_fence_after();
            uint32_t v[16];
            tmem_ld16(lane_base + (uint32_t)(buf * kSkN), v);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_drained[buf]);
            if (SK > 1) {
                #pragma unroll
                for (int jj = 0; jj < kSkN; ++jj) g[jj] = v[jj];
                ep_ok = true;
            } else {
                ok = __all_sync(0xffffffffu, finish_tile(j, t, v));
            }
        }
        ep_ok = __all_sync(0xffffffffu, ep_ok && ok && *abort_v == 0);
    }
    if constexpr (SK > 1) {
        // one tile per CTA: the other CTAs' partial sums through distributed
        // shared memory (the operand ring is idle once the tile is complete)
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        uint32_t* const part = reinterpret_cast<uint32_t*>(gsm);
        const bool ep_warp = warp >= kSkEpiWarp0;
        if (ep_warp && cl.block_rank() != 0 && ep_ok) {
            #pragma unroll
            for (int jj = 0; jj < kSkN; ++jj) part[jj * kSkM + 32 * quarter + lane] = g[jj];
        }
        cl.sync();
        if (ep_warp && cl.block_rank() == 0 && ep_ok) {
            #pragma unroll 1
            for (int r = 1; r < SK; ++r) {
                const uint32_t* rp = cl.map_shared_rank(part, r);
                #pragma unroll
                for (int jj = 0; jj < kSkN; ++jj) g[jj] += rp[jj * kSkM + 32 * quarter + lane];
            }
            finish_tile(0, blockIdx.x, g);
        }
        cl.sync();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kSkTmemCols)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// a row-major [rows][cols] byte matrix, tiles of box_rows x box_cols bytes
bool encode_2d(CUtensorMap* tm, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
               CUtensorMapSwizzle swizzle, uint64_t row_bytes = 0) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_bytes != 0 ? row_bytes : cols};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// a row-major [rows][cols] matrix of 4-byte values for the epilogue's stores:
// boxes of 32 rows x 32 values (128 bytes) in the 128-byte swizzle
bool encode_out(CUtensorMap* tm, const void* base, uint64_t cols, uint64_t rows, CUtensorMapDataType type) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool PAIR, int MT, int SK>
cudaError_t launch_tile(const GemmArgs& a, int* error, cudaStream_t st) {
    using C = GemmCfg<BN, PAIR, MT>;
    static_assert(SK == 1 || (!PAIR && C::S * C::STAGE >= 4 * MT * BN * 128),
                  "a split CTA's partial accumulators (4 warps per token tile, 32 lanes x BN) fit its ring");
    CUtensorMap tm_a, tm_w, tm_w2;
    if (!encode_2d(&tm_a, a.q, (uint64_t)a.K, (uint64_t)a.m, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B,
                   (uint64_t)(a.lda > 0 ? a.lda : a.K)) ||
        !encode_2d(&tm_w, a.w, (uint64_t)(a.K / 4), (uint64_t)a.n_rows, kPK, BN, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    if (PAIR) {
        if (!encode_2d(&tm_w2, a.w2, (uint64_t)(a.K / 4), (uint64_t)a.n_rows, kPK, BN, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
    } else {
        tm_w2 = tm_w;
    }
    GemmKParams p{};
    p.acts = a.acts;
    const size_t tail = (size_t)a.n_rows * (size_t)(a.K / 4);
    p.ws = reinterpret_cast<const float*>(a.w + tail);
    p.ws2 = PAIR ? reinterpret_cast<const float*>(a.w2 + tail) : p.ws;
    p.dots = a.dots;
    p.y = a.y;
    p.M = a.m;
    p.N = a.n_rows;
    p.K = a.K;
    p.error = error;
    // the epilogue stores through tensor maps when the outputs allow it
    // (16-byte aligned rows); otherwise every thread stores its token's row
    CUtensorMap tm_y = tm_w, tm_d = tm_w;
    const bool rows16 = (a.n_rows % 4) == 0;
    const auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    p.tma_out = rows16 && (a.y == nullptr || al16(a.y)) && (a.dots == nullptr || al16(a.dots));
    if (p.tma_out && a.y != nullptr &&
        !encode_out(&tm_y, a.y, (uint64_t)a.n_rows, (uint64_t)a.m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32))
        p.tma_out = 0;
    if (p.tma_out && a.dots != nullptr &&
        !encode_out(&tm_d, a.dots, (uint64_t)a.n_rows, (uint64_t)a.m, CU_TENSOR_MAP_DATA_TYPE_INT32))
        p.tma_out = 0;
    cudaError_t e = cudaFuncSetAttribute(i2s_gemm_kernel<BN, PAIR, MT, SK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((a.n_rows + BN - 1) / BN), (unsigned)((a.m + MT * kBM - 1) / (MT * kBM)), SK);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kGmThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    // programmatic dependent launch: the CTAs may be scheduled while the
    // previous kernel runs (they wait for it after setting up); a CTA needs
    // more shared memory than two GEMM CTAs could share, so two GEMM launches
    // never hold one SM's tensor memory at once
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (SK > 1) {
        // the SK CTAs of one output tile form a cluster
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = SK;
        cfg.numAttrs = 2;
    }
    return cudaLaunchKernelEx(&cfg, i2s_gemm_kernel<BN, PAIR, MT, SK>, tm_a, tm_w, tm_w2, tm_y, tm_d, p);
}

template <bool PAIR, int SK>
cudaError_t launch_skinny(const SkParams& P, int grid, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(i2s_gemm_skinny_kernel<PAIR, SK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         skinny_smem(PAIR));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, 1, SK);
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = skinny_smem(PAIR);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (SK > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = SK;
        cfg.numAttrs = 2;
    }
    return cudaLaunchKernelEx(&cfg, i2s_gemm_skinny_kernel<PAIR, SK>, P);
}

template <bool PAIR>
cudaError_t launch_skinny_split(const SkParams& P, int grid, int sk, cudaStream_t st) {
    switch (sk) {
        case 8: return launch_skinny<PAIR, 8>(P, grid, st);
        case 4: return launch_skinny<PAIR, 4>(P, grid, st);
        case 2: return launch_skinny<PAIR, 2>(P, grid, st);
        default: return launch_skinny<PAIR, 1>(P, grid, st);
    }
}

int sm_count() {
    static int n[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (n[dev] == 0 && cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n[dev] = 148;
    return n[dev];
}

}  // namespace

int gemm_check(const GemmArgs& a, const char** why) {
    auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (a.w == nullptr || a.q == nullptr || a.acts == nullptr || a.m <= 0 || a.n_rows <= 0 || a.K <= 0) {
        *why = "gemm: null pointer or empty shape";
        return SLLM_CUDA_ERR_ARG;
    }
    if (a.K % kBK != 0) {
        *why = "gemm: K must be a multiple of 128";
        return SLLM_CUDA_ERR_ARG;
    }
    if (a.K > kMaxK) {
        *why = "gemm: K above the supported maximum";
        return SLLM_CUDA_ERR_UNSUPPORTED;
    }
    if (!al16(a.w) || !al16(a.q) || (a.w2 != nullptr && !al16(a.w2))) {
        *why = "gemm: w and q must be 16-byte aligned";
        return SLLM_CUDA_ERR_ARG;
    }
    if (a.lda != 0 && (a.lda < a.K || a.lda % 16 != 0)) {
        *why = "gemm: the row stride of q must be at least K and a multiple of 16 bytes";
        return SLLM_CUDA_ERR_ARG;
    }
    if (a.w2 != nullptr ? a.y == nullptr : (a.y == nullptr && a.dots == nullptr)) {
        *why = "gemm: no output";
        return SLLM_CUDA_ERR_ARG;
    }
    return SLLM_CUDA_OK;
}

// Tile shapes: the gate/up pair takes 96 weight rows x 256 tokens per CTA
// (MMAs of N = 192; the 6912 FFN rows make 72 column tiles, 144 CTAs at 512
// tokens: 51.6 us for both GEMMs against 55.8 us with 128-row tiles on 108
// CTAs). A single tensor with a long contraction (six k-steps or more) takes
// 128 rows x 256 tokens per CTA, the contraction split over a cluster of
// three CTAs whose partial int32 sums the first adds: the 2560-row down
// projection at 512 tokens runs on 120 CTAs (23.0 us, against 25.0 us for
// 128 x 128 tiles on 80 CTAs and 27.1 us for 256-row tiles on 120). Short
// contractions take 128 rows x 128 tokens, unsplit.
// The skinny form over up to four segments. Tiles: ceil(rows / 128) per
// tensor (64 for the pair). Two CTAs per SM are resident; with at least that
// many tiles the grid is persistent over them, otherwise the contraction is
// split over clusters of 2, 4 or 8 CTAs while that still fits (each CTA keeps
// at least two k-steps).
cudaError_t launch_i2s_gemm_skinny_segs(const SkinnySeg* segs, int nseg, const int8_t* q, int lda, int m, int K,
                                        const sllm_cuda_act* acts, int* error, cudaStream_t st) {
    if (nseg < 1 || nseg > kSkMaxSeg || m < 1 || m > kSkN || K < kBK || K % kBK != 0 || q == nullptr ||
        acts == nullptr)
        return cudaErrorInvalidValue;
    const bool pair = segs[0].w2 != nullptr;
    const int TR = pair ? 64 : kSkM;
    SkParams P{};
    int tiles = 0, cols = 0;
    for (int i = 0; i < nseg; ++i) {
        const SkinnySeg& sg = segs[i];
        if ((sg.w2 != nullptr) != pair || sg.w == nullptr || sg.n_rows < 1 || sg.kx < 0 || sg.kx % 16 != 0 ||
            (sg.dots == nullptr && sg.y == nullptr) || (pair && (sg.y == nullptr || sg.dots != nullptr)))
            return cudaErrorInvalidValue;
        if (!encode_2d(&P.w[i], sg.w, (uint64_t)(K / 4), (uint64_t)sg.n_rows, kSkG * kPK, TR,
                       CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        if (pair && !encode_2d(&P.w2[i], sg.w2, (uint64_t)(K / 4), (uint64_t)sg.n_rows, kSkG * kPK, TR,
                               CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        if (!pair) P.w2[i] = P.w[i];
        tiles += (sg.n_rows + TR - 1) / TR;
        P.tile_end[i] = tiles;
        P.n_rows[i] = sg.n_rows;
        P.kx[i] = sg.kx;
        const size_t tail = (size_t)sg.n_rows * (size_t)(K / 4);
        P.ws[i] = reinterpret_cast<const float*>(sg.w + tail);
        P.ws2[i] = pair ? reinterpret_cast<const float*>(sg.w2 + tail) : P.ws[i];
        P.dots[i] = sg.dots;
        P.y[i] = sg.y;
        cols = std::max(cols, sg.kx + K);
    }
    const int stride = lda > 0 ? lda : K;
    if (cols > stride) return cudaErrorInvalidValue;
    // the activation map spans exactly the columns the segments read
    if (!encode_2d(&P.act, q, (uint64_t)cols, (uint64_t)m, kBK, kSkN, CU_TENSOR_MAP_SWIZZLE_128B, (uint64_t)stride))
        return cudaErrorInvalidValue;
    P.acts = acts;
    P.error = error;
    P.nseg = nseg;
    P.tiles = tiles;
    P.M = m;
    P.K = K;
    const int slots = 2 * sm_count(), kb = K / kBK;
    int sk = 1;
    while (sk < 8 && tiles * sk * 2 <= slots && kb >= 4 * sk) sk *= 2;
    const int grid = sk > 1 ? tiles : std::min(tiles, slots);
    return pair ? launch_skinny_split<true>(P, grid, sk, st) : launch_skinny_split<false>(P, grid, sk, st);
}

cudaError_t launch_i2s_gemm_skinny(const GemmArgs& a, int* error, cudaStream_t st) {
    SkinnySeg sg{a.w, a.w2, a.n_rows, 0, a.w2 != nullptr ? nullptr : a.dots, a.y};
    return launch_i2s_gemm_skinny_segs(&sg, 1, a.q, a.lda, a.m, a.K, a.acts, error, st);
}

int g_gemm_form = 0;     // test hook: 0 by size, 1 the 128-token tiles, 2 the skinny form

void gemm_set_form(int form) { g_gemm_form = form; }

cudaError_t launch_i2s_gemm(const GemmArgs& a, int* error, cudaStream_t st) {
    if (g_gemm_form != 1 && a.m <= kSkN) return launch_i2s_gemm_skinny(a, error, st);
    if (g_gemm_form == 2) return cudaErrorInvalidValue;
    if (a.w2 != nullptr) return launch_tile<96, true, 2, 1>(a, error, st);
    if (a.K / kBK >= 6) return launch_tile<128, false, 2, 3>(a, error, st);
    return launch_tile<128, false, 1, 1>(a, error, st);
}

}  // namespace sllm
