// engine.cuh -- the persistent I2_S GEMV engine (engine.cu).
//
// One cooperative launch runs a whole program of GEMVs: a list of stages,
// each a list of ops whose rows are split over the CTAs by bytes. Inside a
// CTA a producer warp streams the weight rows of every chunk it will need, in
// program order, into a ring of shared-memory slots with TMA bulk copies,
// running ahead across op and stage boundaries (weights never depend on
// activations); fifteen consumer warps compute from shared memory. Stages are
// separated by a grid barrier, because a stage's input vector is the whole
// output of the stage before.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "decode.cuh"
#include "gemv.cuh"

namespace sllm {

constexpr int kEngConsumerWarps = 15;    // + 1 producer: 16 warps, 4 per SM sub-partition
constexpr int kEngThreads = (kEngConsumerWarps + 1) * 32;
constexpr int kEngSlotBytes = 48 * 1024;   // a slot holds one chunk: whole weight rows of one op
constexpr int kEngSlots = 4;

// An op of this kind is one layer's decode attention: its rows are the query
// heads, its `group` indexes EngParams::attn, and it streams no weights.
constexpr int kEpiAttention = 4;
// the longest context an attention op takes (its scores live in the CTA's
// 8 KB activation area, beside two 128-float vectors)
constexpr int kEngAttnMaxCtx = 1792;

// An op of this kind (tensor-parallel programs) streams no weights either:
// rows of y[i] = (float)(sum over slots q of s[q][i] - act.sum) * (ws /
// act.scale) + resid[i], the epilogue of a contraction split over ranks (and
// column chunks). Its EngOp fields: w = the int32 slots [K][rows], K = the
// number of slots, w2 = the act (sllm_cuda_act) of the quantised input, ws =
// the weight scale, y, resid (nullable).
constexpr int kEpiReduce = 5;

// Cross-GPU exchange inside a program (the XCH instances; tensor-parallel
// decode over peer memory). Every rank has an exchange region; all ranks map
// all regions. A stage may store its outputs into every rank's region as
// well as its own (EngOp::k0x & kOpScatter), then fence at system scope
// before its grid-barrier arrival; a later stage (or kernel) starts only when
// every rank has published that exchange: CTA 0 stores the exchange's flag
// value into flag[kind][rank] of every region after the local grid barrier,
// and every CTA waits (bounded) until flag[kind][r] of its own region reaches
// the value for every rank r. Values grow with every step: steps * n_layer +
// layer + 1, one exchange of each kind per layer.
constexpr int kEngMaxPeers = 8;
constexpr int kEngMaxXStages = 8;
constexpr int kOpScatter = 1 << 24;        // EngOp::k0x: store outputs to every rank's region too
constexpr int kOpK0Mask = (1 << 24) - 1;   // EngOp::k0x: byte offset of the op's slice of the activations
constexpr int kXsWaitMask = 0x0f;          // EngX::xs: kind + 1 to wait for at the stage's start
constexpr int kXsSignal = 0x10;            // EngX::xs: CTA 0 publishes that kind first (after the grid barrier)
constexpr int kXsFence = 0x20;             // EngX::xs: the stage stored to peers: system fence before arriving
constexpr int kXsPrev = 0x40;              // EngX::xs: the awaited exchange is the previous layer's

struct EngX {
    char* peer[kEngMaxPeers];   // every rank's exchange region; peer[rank] is this rank's
    uint32_t flag_off;          // byte offset of the flags [kind][kEngMaxPeers] (u32) in every region
    const uint32_t* steps;      // decode steps completed (device), for the flag values
    unsigned* done;             // end-of-kernel arrival counter (zero between launches)
    int n_peer, rank, layer, n_layer;
    int end_kind;               // kind the last CTA to finish publishes, -1 none
    int8_t xs[kEngMaxXStages];  // per stage: kXs* bits
};

// an input vector and how each CTA turns it into int8 activations
struct EngGroup {
    const float* x;          // input (read through L2: other CTAs may have written it)
    const float* norm_w;     // PRO_NORM weight (nullable for PRO_QUANT)
    int K;
    int pro;                 // PRO_NORM, PRO_QUANT or PRO_Q8
    const int8_t* q8;        // PRO_Q8: K int8 activations, natural order, already quantised
    const sllm_cuda_act* act8;   // PRO_Q8: their {scale, sum}; PRO_NORM in an XCH program: where CTA 0
                                 // stores the {scale, sum} it computed (nullable)
};

// one weight tensor (or a gate/up pair for EPI_SILU)
struct EngOp {
    const uint8_t* w;        // rows x K/4 bytes, scale tail after them
    const uint8_t* w2;       // EPI_SILU: the up tensor (same shape)
    float* y;                // EPI_F32 / EPI_RESID output; EPI_DOTS: int32 raw dots
    const float* resid;      // EPI_RESID: y = proj + resid
    float* h;                // EPI_SILU: h = silu(gate) * up
    int rows;
    int K;
    int epi;                 // EPI_F32, EPI_RESID, EPI_SILU or EPI_DOTS
    int group;               // index into the groups
    int chunk_rows;          // rows per slot
    float ws;                // the per-tensor scale of w (src/quant.c:102-106), read at upload
    float ws2;               // ... of w2
    int k0x;                 // XCH programs: kOpK0Mask bits = the op's activation slice offset, | kOpScatter
};

// a position in the op list: row `row` of op `op`
struct EngCursor {
    int op;
    int row;
};

struct EngParams {
    const EngGroup* groups;
    const EngOp* ops;
    const EngCursor* starts;     // [n_stages][grid + 1]: CTA c of stage s runs [starts[s][c], starts[s][c+1])
    int n_groups;
    int n_ops;
    int n_stages;
    unsigned int* barrier;       // zero at launch; counts CTA arrivals over all stages
    int* error;                  // 0, or why a bounded wait gave up
    float eps;
    int* fallback_count;         // nullable
    int force_fallback;
    const AttnParams* attn;      // [n_attn]: the attention ops' layers
    int n_attn;
    int kv16;                    // the attention ops' caches hold f16 (a separate kernel instance)
    int xch;                     // the program exchanges with peers (a separate kernel instance)
    EngX x;
};

enum EngError {
    ENG_OK = 0, ENG_TIMEOUT_FULL = 1, ENG_TIMEOUT_EMPTY = 2, ENG_TIMEOUT_GRID = 3, ENG_BAD_PROGRAM = 4,
    ENG_TIMEOUT_PEER = 5
};

// rows of an op per slot, so that a chunk fills at most one slot
int engine_chunk_rows(int K, int epi);
// dynamic shared memory of a program: the ring, the int8 activations, and the
// group / op / cursor tables every CTA copies in at start (0 when too large)
int engine_smem_bytes(int n_groups, int n_ops, int n_stages, int n_attn = 0);
int engine_grid(int device);
// the engine is compiled for pairs (wpl(n_embd), wpl(n_ff)) of row widths,
// wpl(K) = 32-bit words per lane = ceil(K / 512)
int engine_wpl(int K);
bool engine_supports(int wa, int wb);
// the pairs that also have an instance for f16 KV caches, and one for
// programs that exchange with peers
bool engine_supports_kv16(int wa, int wb);
bool engine_supports_xch(int wa, int wb);
// a compiled pair whose first width is `wpl` (for programs of one width)
bool engine_pair_for_width(int wpl, int* wa, int* wb);
cudaError_t prepare_engine();     // once, outside any stream capture
// test hook on the current device: every bounded wait gives up after wait_ms
// (<= 0: the default 2 s), and CTA skip_arrival_cta (-1: none) leaves out its
// first grid-barrier arrival
cudaError_t engine_test_faults(int skip_arrival_cta, double wait_ms);
cudaError_t launch_engine(const EngParams& p, int grid, cudaStream_t st, int wa, int wb);

}  // namespace sllm
