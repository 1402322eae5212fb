// backend.cu -- the C ABI of include/sllm_cuda.h: kernel-level entry points,
// device model upload, per-sequence contexts and the decode loop.
//
// One decode step (embedding, 30 x {QKV GEMV, attention, O GEMV, gate/up
// GEMV, down GEMV}, lm_head + argmax) is captured once per context into a
// CUDA graph. The token of each position, the position itself and the greedy
// feedback live in device memory, so a whole prompt + generation is a run of
// graph launches with no host round trip until the ids are copied back.

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"
#include "backend.cuh"
#include "engine.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "upload.cuh"
#include "../../include/sllm_cuda.h"
#include "../../include/sllm_cuda_testing.h"

using namespace sllm;

// ---------------------------------------------------------------------------
// status and errors
// ---------------------------------------------------------------------------
static thread_local std::string g_last_error;
static int g_force_fallback = 0;
static float g_engine_eps = 0.0f;          // set just before an engine program is captured
// Device words shared by every call in the process: one per device, since a
// kernel must never write another device's memory.
static std::mutex g_words_mu;
static std::vector<int*> g_fallback_counters;   // how often a certified sum fell back
static std::vector<int*> g_gemm_errors;         // why a GEMM's bounded wait gave up
static int* device_word(std::vector<int*>& words) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_words_mu);
    if ((int)words.size() <= dev) words.resize(dev + 1, nullptr);
    if (words[dev] == nullptr) {
        int* w = nullptr;
        if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            cudaFree(w);
            return nullptr;
        }
        words[dev] = w;
    }
    return words[dev];
}

// Kernels this library has put on a stream, for the benchmark's launch count:
// a graph adds its kernel nodes each time it is launched, a direct launch
// adds one.
static std::atomic<long long> g_kernel_launches{0};
static std::mutex g_graph_mu;
static std::unordered_map<cudaGraphExec_t, int> g_graph_kernels;

int sllm::fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int sllm::cuda_fail(cudaError_t e, const char* what) {
    const int st = (e == cudaErrorMemoryAllocation) ? SLLM_CUDA_ERR_NOMEM : SLLM_CUDA_ERR_DEVICE;
    cudaGetLastError();   // clear a sticky launch error where possible
    return fail(st, "%s: %s", what, cudaGetErrorString(e));
}



extern "C" const char* sllm_cuda_status_string(int st) {
    switch (st) {
        case SLLM_CUDA_OK: return "ok";
        case SLLM_CUDA_ERR_ARG: return "invalid argument";
        case SLLM_CUDA_ERR_NOMEM: return "out of memory";
        case SLLM_CUDA_ERR_IO: return "i/o error";
        case SLLM_CUDA_ERR_UNSUPPORTED: return "unsupported";
        case SLLM_CUDA_ERR_TRUNCATED: return "truncated";
        case SLLM_CUDA_ERR_KV_TYPE: return "wrong file type or version";
        case SLLM_CUDA_ERR_TENSOR_SHAPE: return "geometry mismatch";
        case SLLM_CUDA_ERR_TOO_LARGE: return "too large";
        case SLLM_CUDA_ERR_DEVICE: return "CUDA device error";
        case SLLM_CUDA_ERR_TIMEOUT: return "device wait timed out";
        case SLLM_CUDA_ERR_COMM: return "collective failed";
        default: return "unknown status";
    }
}

extern "C" const char* sllm_cuda_last_error(void) { return g_last_error.c_str(); }

// ---------------------------------------------------------------------------
// devices
// ---------------------------------------------------------------------------
int sllm::num_sms_of(int dev) {
    static std::mutex mu;
    static std::vector<int> cache;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

static int current_sms() {
    int dev = 0;
    cudaGetDevice(&dev);
    return num_sms_of(dev);
}

extern "C" int sllm_cuda_probe(int* n_devices, int* cc_major, int* cc_minor) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (n_devices) *n_devices = (e == cudaSuccess) ? n : 0;
    if (cc_major) *cc_major = 0;
    if (cc_minor) *cc_minor = 0;
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(e));
    }
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, 0), "cudaGetDeviceProperties");
    if (cc_major) *cc_major = prop.major;
    if (cc_minor) *cc_minor = prop.minor;
    if (prop.major != 10) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "device 0 is sm_%d%d, this build runs sm_100a",
                                      prop.major, prop.minor);
    return SLLM_CUDA_OK;
}

// Allocated on first use OUTSIDE any stream capture (ctx_new and the chain
// entry points call it before capturing); a graph then bakes the pointer in.
// instantiate a captured graph, remembering how many kernel nodes it holds
cudaError_t sllm::instantiate(cudaGraphExec_t* exec, cudaGraph_t g) {
    size_t n = 0;
    cudaError_t e = cudaGraphGetNodes(g, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    if (e == cudaSuccess && n > 0) e = cudaGraphGetNodes(g, nodes.data(), &n);
    int kernels = 0;
    for (size_t i = 0; e == cudaSuccess && i < n; ++i) {
        cudaGraphNodeType t;
        e = cudaGraphNodeGetType(nodes[i], &t);
        if (e == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
    }
    if (e != cudaSuccess) return e;
    e = cudaGraphInstantiate(exec, g, 0);
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(g_graph_mu);
        g_graph_kernels[*exec] = kernels;
    }
    return e;
}

void sllm::graph_exec_destroy(cudaGraphExec_t exec) {
    if (exec == nullptr) return;
    {
        std::lock_guard<std::mutex> lk(g_graph_mu);
        g_graph_kernels.erase(exec);
    }
    cudaGraphExecDestroy(exec);
}

cudaError_t sllm::graph_launch(cudaGraphExec_t exec, cudaStream_t st) {
    const cudaError_t e = cudaGraphLaunch(exec, st);
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(g_graph_mu);
        auto it = g_graph_kernels.find(exec);
        if (it != g_graph_kernels.end()) g_kernel_launches += it->second;
    }
    return e;
}

extern "C" long long sllm_cuda_test_kernel_launches(void) { return g_kernel_launches.load(); }

void sllm::count_launches(long long n) { g_kernel_launches += n; }
int sllm::force_fallback_flag() { return g_force_fallback; }

// host-side failure injection (tests): the next n device allocations of a
// model or context, or the next n communicator set-ups, fail as if the
// device or the library had refused them
static std::atomic<int> g_fail_alloc{0};
static std::atomic<int> g_fail_comm{0};

cudaError_t sllm::dev_malloc(void** p, size_t bytes) {
    int n = g_fail_alloc.load();
    while (n > 0 && !g_fail_alloc.compare_exchange_weak(n, n - 1)) {}
    if (n > 0) { *p = nullptr; return cudaErrorMemoryAllocation; }
    return cudaMalloc(p, bytes);
}

bool sllm::fail_next_comm_init() {
    int n = g_fail_comm.load();
    while (n > 0 && !g_fail_comm.compare_exchange_weak(n, n - 1)) {}
    return n > 0;
}

extern "C" void sllm_cuda_test_fail_next(int what, int count) {
    if (what == 1) g_fail_alloc = count;
    if (what == 2) g_fail_comm = count;
}

extern "C" int sllm_cuda_test_engine_faults(int device, int skip_arrival_cta, double wait_ms) {
    CK(cudaSetDevice(device), "cudaSetDevice");
    CK(engine_test_faults(skip_arrival_cta, wait_ms), "engine test hooks");
    return SLLM_CUDA_OK;
}

int* sllm::fallback_counter() { return device_word(g_fallback_counters); }

extern "C" void sllm_cuda_test_set_force_fallback(int on) { g_force_fallback = on; }

extern "C" int sllm_cuda_test_fallback_count(void) {
    int* p = fallback_counter();
    int v = -1;
    if (p != nullptr && cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) v = -1;
    return v;
}

// ---------------------------------------------------------------------------
// kernel level
// ---------------------------------------------------------------------------
bool sllm::aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

extern "C" int sllm_cuda_i2s_quant_act(const float* x, size_t n, int8_t* q_out, sllm_cuda_act* act_out,
                                       void* stream) {
    if (x == nullptr || q_out == nullptr || act_out == nullptr || n == 0 || n > (size_t)kMaxK)
        return fail(SLLM_CUDA_ERR_ARG, "quant_act: bad arguments (n=%zu)", n);
    CK(launch_quant_act(x, (int)n, q_out, act_out, (cudaStream_t)stream), "quant_act launch");
    ++g_kernel_launches;
    return SLLM_CUDA_OK;
}

static int check_gemv_shape(const void* w, size_t n_rows, size_t n, const void* out) {
    if (w == nullptr || out == nullptr || n_rows == 0 || n_rows > (1u << 30))
        return fail(SLLM_CUDA_ERR_ARG, "gemv: bad arguments");
    if (n % kQK != 0 || n == 0) return fail(SLLM_CUDA_ERR_ARG, "gemv: n=%zu is not a multiple of 128", n);
    if (n > (size_t)gemv_max_k()) return fail(SLLM_CUDA_ERR_UNSUPPORTED, "gemv: n=%zu above %d", n, gemv_max_k());
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_i2s_gemv(const uint8_t* w, size_t n_rows, size_t n, const int8_t* q, int32_t* rows_out,
                                  void* stream) {
    int rc = check_gemv_shape(w, n_rows, n, rows_out);
    if (rc != SLLM_CUDA_OK) return rc;
    if (q == nullptr || !aligned16(q)) return fail(SLLM_CUDA_ERR_ARG, "gemv: q must be 16-byte aligned");
    if (!aligned16(w)) return fail(SLLM_CUDA_ERR_ARG, "gemv: w must be 16-byte aligned");
    // The raw API has no act: an all-zero act makes the prologue a plain copy.
    // One per device (a kernel must not read another device's memory).
    static std::mutex zero_mu;
    static std::vector<sllm_cuda_act*> zero_acts;
    sllm_cuda_act* zero_act = nullptr;
    {
        int dev = 0;
        CK(cudaGetDevice(&dev), "cudaGetDevice");
        std::lock_guard<std::mutex> lk(zero_mu);
        if ((int)zero_acts.size() <= dev) zero_acts.resize(dev + 1, nullptr);
        if (zero_acts[dev] == nullptr) {
            CK(cudaMalloc(&zero_acts[dev], sizeof(sllm_cuda_act)), "cudaMalloc");
            CK(cudaMemset(zero_acts[dev], 0, sizeof(sllm_cuda_act)), "cudaMemset");
        }
        zero_act = zero_acts[dev];
    }
    GemvParams p{};
    p.K = (int)n;
    p.nseg = 1;
    p.seg[0] = GemvSeg{w, (int)n_rows, nullptr, rows_out};
    p.q_in = q;
    p.act_in = zero_act;
    // a dependent launch: it may start while the kernel before it finishes,
    // streams weights at once and waits for that kernel before it reads q
    CK(launch_gemv(p, PRO_Q8, EPI_DOTS, current_sms(), (cudaStream_t)stream, GEMV_DEPENDENT), "gemv launch");
    ++g_kernel_launches;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_i2s_gemv_f32(const uint8_t* w, size_t n_rows, size_t n, const float* x, float* y,
                                      int32_t* dots, void* stream) {
    int rc = check_gemv_shape(w, n_rows, n, y);
    if (rc != SLLM_CUDA_OK) return rc;
    if (x == nullptr || !aligned16(x) || !aligned16(w)) return fail(SLLM_CUDA_ERR_ARG, "gemv_f32: x and w must be 16-byte aligned");
    GemvParams p{};
    p.K = (int)n;
    p.nseg = 1;
    p.seg[0] = GemvSeg{w, (int)n_rows, y, dots};
    p.x = x;
    CK(launch_gemv(p, PRO_QUANT, EPI_F32, current_sms(), (cudaStream_t)stream, GEMV_DEPENDENT), "gemv_f32 launch");
    ++g_kernel_launches;
    return SLLM_CUDA_OK;
}

// ---------------------------------------------------------------------------
// multi-token (prefill) kernels
// ---------------------------------------------------------------------------
int* sllm::gemm_error_word() { return device_word(g_gemm_errors); }

extern "C" int sllm_cuda_test_gemm_error(void) {
    int* p = gemm_error_word();
    if (p == nullptr || cudaDeviceSynchronize() != cudaSuccess) return -1;
    int v = 0;
    if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    cudaMemset(p, 0, sizeof(int));
    return v;
}

extern "C" int sllm_cuda_i2s_quant_act_rows(const float* x, size_t m, size_t n, int8_t* q, sllm_cuda_act* acts,
                                            void* stream) {
    if (x == nullptr || q == nullptr || acts == nullptr || m == 0 || n == 0 || n > (size_t)kMaxK || m > (1u << 24))
        return fail(SLLM_CUDA_ERR_ARG, "quant_act_rows: bad arguments (m=%zu, n=%zu)", m, n);
    CK(launch_quant_act_rows(x, (int)m, (int)n, q, acts, (cudaStream_t)stream), "quant_act_rows launch");
    ++g_kernel_launches;
    return SLLM_CUDA_OK;
}

static int gemm_run(const GemmArgs& a, void* stream) {
    const char* why = nullptr;
    const int rc = gemm_check(a, &why);
    if (rc != SLLM_CUDA_OK) return fail(rc, "%s", why);
    int* err = gemm_error_word();
    if (err == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "gemm: error word");
    CK(launch_i2s_gemm(a, err, (cudaStream_t)stream), "gemm launch");
    ++g_kernel_launches;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_i2s_gemm(const uint8_t* w, size_t n_rows, size_t n, size_t m, const int8_t* q,
                                  const sllm_cuda_act* acts, int32_t* dots, float* y, void* stream) {
    if (n_rows == 0 || n_rows > (1u << 24) || m == 0 || m > (1u << 24) || n == 0 || n > (size_t)kMaxK)
        return fail(SLLM_CUDA_ERR_ARG, "gemm: bad shape (rows=%zu, n=%zu, m=%zu)", n_rows, n, m);
    GemmArgs a{};
    a.w = w; a.w2 = nullptr; a.q = q; a.acts = acts; a.dots = dots; a.y = y;
    a.m = (int)m; a.n_rows = (int)n_rows; a.K = (int)n;
    return gemm_run(a, stream);
}

extern "C" int sllm_cuda_i2s_gemm_silu(const uint8_t* w_gate, const uint8_t* w_up, size_t n_rows, size_t n, size_t m,
                                       const int8_t* q, const sllm_cuda_act* acts, float* h, void* stream) {
    if (w_up == nullptr || n_rows == 0 || n_rows > (1u << 24) || m == 0 || m > (1u << 24) || n == 0 ||
        n > (size_t)kMaxK)
        return fail(SLLM_CUDA_ERR_ARG, "gemm_silu: bad arguments (rows=%zu, n=%zu, m=%zu)", n_rows, n, m);
    GemmArgs a{};
    a.w = w_gate; a.w2 = w_up; a.q = q; a.acts = acts; a.dots = nullptr; a.y = h;
    a.m = (int)m; a.n_rows = (int)n_rows; a.K = (int)n;
    return gemm_run(a, stream);
}

extern "C" void sllm_cuda_test_gemm_form(int form) { gemm_set_form(form); }

extern "C" int sllm_cuda_test_gemm_strided(const uint8_t* w, int32_t n_rows, int32_t k, int32_t m, const int8_t* q,
                                           int32_t lda, const sllm_cuda_act* acts, int32_t* dots, float* y,
                                           void* stream) {
    GemmArgs a{};
    a.w = w; a.q = q; a.acts = acts; a.dots = dots; a.y = y;
    a.m = m; a.n_rows = n_rows; a.K = k; a.lda = lda;
    return gemm_run(a, stream);
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
struct DevLayer {
    const uint8_t *wq, *wk, *wv, *wo, *gate, *up, *down;
    const float *attn_norm, *attn_sub_norm, *ffn_norm, *ffn_sub_norm;
    // per-tensor scales, read from the host copies at upload (src/quant.c:102-106)
    float s_wq, s_wk, s_wv, s_wo, s_gate, s_up, s_down;
};

static float host_i2s_scale(const uint8_t* w, size_t rows, size_t cols) {
    float s;
    std::memcpy(&s, w + rows * cols / 4, sizeof s);
    return s;
}

struct sllm_cuda_model {
    int device = 0;
    int n_layer = 0, n_embd = 0, n_ff = 0, n_head = 0, n_head_kv = 0, n_vocab = 0, n_rot = 0, n_ctx_train = 0;
    int head_dim = 0, n_embd_gqa = 0;
    float eps = 0.0f, rope_base = 0.0f;
    uint8_t* blob = nullptr;        // every I2_S tensor and f32 norm, 256-byte aligned
    uint16_t* tok_embd = nullptr;   // f16 [V][E]
    float* output_norm = nullptr;
    std::vector<DevLayer> layers;
    size_t weight_bytes = 0;        // bytes one decode step streams
};

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

extern "C" int sllm_cuda_model_upload(const sllm_cuda_model_desc* d, int device, sllm_cuda_model** out) {
    if (d == nullptr || out == nullptr) return fail(SLLM_CUDA_ERR_ARG, "model_upload: NULL argument");
    *out = nullptr;
    if (d->n_layer <= 0 || d->n_embd <= 0 || d->n_head <= 0 || d->n_head_kv <= 0 || d->n_ff <= 0 ||
        d->n_vocab <= 0 || d->n_head % d->n_head_kv != 0 || d->n_embd % d->n_head != 0 || d->layers == nullptr ||
        d->tok_embd == nullptr || d->output_norm == nullptr)
        return fail(SLLM_CUDA_ERR_ARG, "model_upload: invalid hyperparameters or tensors");
    const int E = d->n_embd, F = d->n_ff, hd = E / d->n_head, G = hd * d->n_head_kv;
    if (hd != 128 || d->n_rot != hd || E % kQK != 0 || F % kQK != 0 || E > gemv_max_k() || F > gemv_max_k())
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "model_upload: shape E=%d F=%d head_dim=%d n_rot=%d not supported",
                    E, F, hd, d->n_rot);
    for (int l = 0; l < d->n_layer; ++l) {
        const sllm_cuda_layer_desc& L = d->layers[l];
        if (!L.wq || !L.wk || !L.wv || !L.wo || !L.ffn_gate || !L.ffn_up || !L.ffn_down || !L.attn_norm ||
            !L.attn_sub_norm || !L.ffn_norm || !L.ffn_sub_norm)
            return fail(SLLM_CUDA_ERR_ARG, "model_upload: layer %d has a NULL tensor", l);
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "model_upload: device %d not present", device);
    }
    CK(cudaSetDevice(device), "cudaSetDevice");

    auto* m = new sllm_cuda_model();
    m->device = device;
    m->n_layer = d->n_layer; m->n_embd = E; m->n_ff = F; m->n_head = d->n_head; m->n_head_kv = d->n_head_kv;
    m->n_vocab = d->n_vocab; m->n_rot = d->n_rot; m->n_ctx_train = d->n_ctx_train;
    m->head_dim = hd; m->n_embd_gqa = G; m->eps = d->f_rms_eps; m->rope_base = d->rope_freq_base;

    struct Item { const void* src; size_t bytes; size_t off; };
    std::vector<Item> items;
    size_t total = 0;
    auto add = [&](const void* src, size_t bytes) { items.push_back({src, bytes, total}); total += align256(bytes); return items.size() - 1; };
    auto i2s = [](int rows, int cols) { return (size_t)rows * (size_t)cols / 4 + 32; };
    std::vector<size_t> idx;
    for (int l = 0; l < d->n_layer; ++l) {
        const sllm_cuda_layer_desc& L = d->layers[l];
        idx.push_back(add(L.wq, i2s(E, E)));
        idx.push_back(add(L.wk, i2s(G, E)));
        idx.push_back(add(L.wv, i2s(G, E)));
        idx.push_back(add(L.wo, i2s(E, E)));
        idx.push_back(add(L.ffn_gate, i2s(F, E)));
        idx.push_back(add(L.ffn_up, i2s(F, E)));
        idx.push_back(add(L.ffn_down, i2s(E, F)));
        idx.push_back(add(L.attn_norm, (size_t)E * 4));
        idx.push_back(add(L.attn_sub_norm, (size_t)E * 4));
        idx.push_back(add(L.ffn_norm, (size_t)E * 4));
        idx.push_back(add(L.ffn_sub_norm, (size_t)F * 4));
    }
    const size_t out_norm = add(d->output_norm, (size_t)E * 4);
    cudaError_t e = dev_malloc((void**)&m->blob, total);
    if (e == cudaSuccess) e = dev_malloc((void**)&m->tok_embd, (size_t)d->n_vocab * (size_t)E * 2);
    if (e != cudaSuccess) { sllm_cuda_model_free(m); return cuda_fail(e, "model_upload: cudaMalloc"); }
    {
        // through pinned staging: host threads fill one buffer while the
        // device copies the other in
        Uploader up(device);
        for (const Item& it : items) {
            e = up.put(m->blob + it.off, it.src, it.bytes);
            if (e != cudaSuccess) break;
        }
        if (e == cudaSuccess) e = up.put(m->tok_embd, d->tok_embd, (size_t)d->n_vocab * (size_t)E * 2);
        if (e == cudaSuccess) e = up.finish();
        if (e != cudaSuccess) { sllm_cuda_model_free(m); return cuda_fail(e, "model_upload: weights"); }
    }
    m->layers.resize(d->n_layer);
    for (int l = 0; l < d->n_layer; ++l) {
        const size_t* ix = &idx[(size_t)l * 11];
        DevLayer& L = m->layers[l];
        L.wq = m->blob + items[ix[0]].off;  L.wk = m->blob + items[ix[1]].off;
        L.wv = m->blob + items[ix[2]].off;  L.wo = m->blob + items[ix[3]].off;
        L.gate = m->blob + items[ix[4]].off; L.up = m->blob + items[ix[5]].off;
        L.down = m->blob + items[ix[6]].off;
        L.attn_norm = (const float*)(m->blob + items[ix[7]].off);
        L.attn_sub_norm = (const float*)(m->blob + items[ix[8]].off);
        L.ffn_norm = (const float*)(m->blob + items[ix[9]].off);
        L.ffn_sub_norm = (const float*)(m->blob + items[ix[10]].off);
        const sllm_cuda_layer_desc& H = d->layers[l];
        L.s_wq = host_i2s_scale(H.wq, E, E);
        L.s_wk = host_i2s_scale(H.wk, G, E);
        L.s_wv = host_i2s_scale(H.wv, G, E);
        L.s_wo = host_i2s_scale(H.wo, E, E);
        L.s_gate = host_i2s_scale(H.ffn_gate, F, E);
        L.s_up = host_i2s_scale(H.ffn_up, F, E);
        L.s_down = host_i2s_scale(H.ffn_down, E, F);
    }
    m->output_norm = (float*)(m->blob + items[out_norm].off);
    for (const Item& it : items) m->weight_bytes += it.bytes;
    m->weight_bytes += (size_t)d->n_vocab * (size_t)E * 2;
    *out = m;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_model_free(sllm_cuda_model* m) {
    if (m == nullptr) return;
    cudaSetDevice(m->device);
    cudaFree(m->blob);
    cudaFree(m->tok_embd);
    delete m;
}

extern "C" size_t sllm_cuda_model_weight_bytes(const sllm_cuda_model* m) { return m ? m->weight_bytes : 0; }

// ---------------------------------------------------------------------------
// engine programs (engine.cu): device copies of the group / op / start tables
// ---------------------------------------------------------------------------
struct EngineProgram {
    EngGroup* groups = nullptr;
    EngOp* ops = nullptr;
    EngCursor* starts = nullptr;
    AttnParams* attn = nullptr;
    unsigned* barrier = nullptr;
    int* error = nullptr;
    int n_stages = 0;
    int grid = 0;
    cudaGraphExec_t exec = nullptr;  // multi-stage: barrier memset + cooperative launch
    bool built = false;
    EngParams params{};              // single-stage: launched directly (programmatic dependent launch)
    int wa = 0, wb = 0;
    // what the program was built for
    int key_begin = -1, key_n = -1;
    const void* key_x = nullptr;
    const void* key_y = nullptr;
};

static void engine_program_free(EngineProgram& p) {
    graph_exec_destroy(p.exec);
    cudaFree(p.groups); cudaFree(p.ops); cudaFree(p.starts); cudaFree(p.attn); cudaFree(p.barrier); cudaFree(p.error);
    p = EngineProgram();
}

// Split every stage's rows over `grid` CTAs so that each CTA costs the same:
// its weight bytes (a row of a gate/up pair weighs two rows), plus, for every
// input group whose rows it runs, the time of that group's prologue (the
// RMSNorm + quantisation every such CTA computes), counted in bytes the CTA
// could have streamed meanwhile. A CTA that spans several small ops builds
// several activation vectors, so it gets fewer bytes. The split is the
// greedy fill under the smallest feasible per-CTA cost (binary search).
static constexpr double kPrologueBytes = 192.0 * 1024.0;

std::vector<EngCursor> sllm::engine_starts(const std::vector<EngOp>& ops, const std::vector<int>& stage_first,
                                           int grid) {
    const int n_stages = (int)stage_first.size() - 1;
    std::vector<EngCursor> st((size_t)n_stages * (grid + 1));
    // an attention head costs about what 64 KB of weights take to stream, so
    // the heads of a layer spread over separate CTAs
    auto row_cost = [&](int o) {
        if (ops[o].epi == kEpiAttention) return 65536.0;
        if (ops[o].epi == kEpiReduce) return 4.0 * ops[o].K;       // its slots' int32 words
        return (double)(ops[o].K / 4) * (ops[o].epi == EPI_SILU ? 2 : 1);
    };
    for (int s = 0; s < n_stages; ++s) {
        const int o0 = stage_first[s], o1 = stage_first[s + 1];
        EngCursor* out = &st[(size_t)s * (grid + 1)];
        // greedy fill under budget M; returns the CTAs used, writes the cursors
        auto fill = [&](double M, bool write) {
            int cta = 0, group = -1;
            double cost = 0.0;
            if (write) out[0] = EngCursor{o0, 0};
            for (int o = o0; o < o1; ++o) {
                const double rc = row_cost(o);
                int row = 0;
                while (row < ops[o].rows) {
                    const double enter = (ops[o].group != group) ? kPrologueBytes : 0.0;
                    double room = M - cost - enter;
                    int take = room >= rc ? (int)std::min<double>(ops[o].rows - row, std::floor(room / rc)) : 0;
                    if (take == 0 && cost == 0.0) take = 1;          // an empty CTA always takes one row
                    if (take == 0) {                                  // this CTA is full: open the next one
                        ++cta;
                        if (write && cta < grid) out[cta] = EngCursor{o, row};
                        cost = 0.0;
                        group = -1;
                        continue;
                    }
                    cost += enter + take * rc;
                    group = ops[o].group;
                    row += take;
                }
            }
            return cta + 1;
        };
        double total = 0.0;
        for (int o = o0; o < o1; ++o) total += ops[o].rows * row_cost(o);
        double lo = total / grid, hi = total / grid + kPrologueBytes * (o1 - o0 + 1) + 4 * 65536.0;
        if (o1 > o0) {
            while (fill(hi, false) > grid) hi *= 2;
            for (int it = 0; it < 40; ++it) {
                const double mid = 0.5 * (lo + hi);
                if (fill(mid, false) <= grid) hi = mid; else lo = mid;
            }
        }
        for (int c = 0; c <= grid; ++c) out[c] = EngCursor{o1, 0};
        if (o1 > o0) {
            const int used = fill(hi, true);
            for (int c = used; c <= grid; ++c) out[c] = EngCursor{o1, 0};
        }
    }
    return st;
}

extern "C" int sllm_cuda_test_engine_split(const int32_t* rows, const int32_t* K, const int32_t* epi,
                                           const int32_t* group, int32_t n_ops, const int32_t* stage_first,
                                           int32_t n_stages, int32_t grid, int32_t* out) {
    if (rows == nullptr || K == nullptr || epi == nullptr || group == nullptr || stage_first == nullptr ||
        out == nullptr || n_ops < 0 || n_stages < 1 || grid < 1 || stage_first[0] != 0 ||
        stage_first[n_stages] != n_ops)
        return fail(SLLM_CUDA_ERR_ARG, "engine_split: bad arguments");
    for (int s = 0; s < n_stages; ++s)
        if (stage_first[s + 1] < stage_first[s]) return fail(SLLM_CUDA_ERR_ARG, "engine_split: stages out of order");
    std::vector<EngOp> ops((size_t)n_ops);
    for (int i = 0; i < n_ops; ++i) {
        if (rows[i] < 1 || K[i] < 1 || epi[i] < 0 || epi[i] > kEpiReduce || group[i] < 0 ||
            (K[i] < 4 && epi[i] != kEpiReduce))
            return fail(SLLM_CUDA_ERR_ARG, "engine_split: bad op %d", i);
        ops[i].rows = rows[i]; ops[i].K = K[i]; ops[i].epi = epi[i]; ops[i].group = group[i];
    }
    const std::vector<int> sf(stage_first, stage_first + n_stages + 1);
    const std::vector<EngCursor> st = engine_starts(ops, sf, grid);
    for (size_t i = 0; i < st.size(); ++i) {
        out[2 * i] = st[i].op;
        out[2 * i + 1] = st[i].row;
    }
    return SLLM_CUDA_OK;
}

static int engine_program_build(EngineProgram& p, const std::vector<EngGroup>& groups, const std::vector<EngOp>& ops,
                                const std::vector<int>& stage_first, int device, cudaStream_t capture_stream,
                                int* fallback, int wa, int wb, const std::vector<AttnParams>* attn = nullptr,
                                bool graph = true) {
    engine_program_free(p);
    p.grid = engine_grid(device);
    p.n_stages = (int)stage_first.size() - 1;
    const std::vector<EngCursor> st = engine_starts(ops, stage_first, p.grid);
    cudaError_t e = cudaMalloc(&p.groups, groups.size() * sizeof(EngGroup));
    if (e == cudaSuccess) e = cudaMalloc(&p.ops, ops.size() * sizeof(EngOp));
    if (e == cudaSuccess) e = cudaMalloc(&p.starts, st.size() * sizeof(EngCursor));
    if (e == cudaSuccess) e = cudaMalloc(&p.barrier, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMalloc(&p.error, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpy(p.groups, groups.data(), groups.size() * sizeof(EngGroup), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(p.ops, ops.data(), ops.size() * sizeof(EngOp), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(p.starts, st.data(), st.size() * sizeof(EngCursor), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(p.error, 0, sizeof(int));
    const int n_attn = attn != nullptr ? (int)attn->size() : 0;
    if (e == cudaSuccess && n_attn > 0) e = cudaMalloc(&p.attn, n_attn * sizeof(AttnParams));
    if (e == cudaSuccess && n_attn > 0)
        e = cudaMemcpy(p.attn, attn->data(), n_attn * sizeof(AttnParams), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { engine_program_free(p); return cuda_fail(e, "engine program"); }
    if (engine_smem_bytes((int)groups.size(), (int)ops.size(), p.n_stages, n_attn) == 0) {
        engine_program_free(p);
        return fail(SLLM_CUDA_ERR_TOO_LARGE, "engine program: %zu ops do not fit in shared memory", ops.size());
    }
    CK(prepare_engine(), "engine attributes");
    EngParams ep{};
    ep.groups = p.groups; ep.ops = p.ops; ep.starts = p.starts; ep.n_stages = p.n_stages;
    ep.n_groups = (int)groups.size(); ep.n_ops = (int)ops.size();
    ep.barrier = p.barrier; ep.error = p.error; ep.fallback_count = fallback; ep.force_fallback = g_force_fallback;
    ep.eps = g_engine_eps;     // every group of a program comes from one model
    ep.attn = p.attn;
    ep.n_attn = n_attn;
    p.params = ep;
    p.wa = wa;
    p.wb = wb;
    if (p.n_stages == 1 || !graph) {     // no grid barrier, or launched inside the caller's graph
        p.built = true;
        return SLLM_CUDA_OK;
    }
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(capture_stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    e = cudaMemsetAsync(p.barrier, 0, sizeof(unsigned), capture_stream);
    if (e == cudaSuccess) e = launch_engine(ep, p.grid, capture_stream, wa, wb);
    cudaError_t e2 = cudaStreamEndCapture(capture_stream, &g);
    if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); engine_program_free(p); return cuda_fail(e, "capture engine"); }
    if (e2 != cudaSuccess) { engine_program_free(p); return cuda_fail(e2, "end capture"); }
    e = instantiate(&p.exec, g);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { p.exec = nullptr; engine_program_free(p); return cuda_fail(e, "instantiate engine"); }
    p.built = true;
    return SLLM_CUDA_OK;
}

static int engine_error(const EngineProgram& p);

static cudaError_t engine_program_launch(const EngineProgram& p, cudaStream_t st) {
    if (p.exec != nullptr) return graph_launch(p.exec, st);
    const cudaError_t e = launch_engine(p.params, p.grid, st, p.wa, p.wb);
    if (e == cudaSuccess) count_launches(1);
    return e;
}

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
static constexpr int kProjPieces = 2;

struct sllm_cuda_ctx {
    const sllm_cuda_model* m = nullptr;
    int n_ctx = 0;
    int n_past = 0;
    bool have_logits = false;
    cudaStream_t stream = nullptr;
    float *k_cache = nullptr, *v_cache = nullptr;   // [layer][kvh][128][n_ctx], [layer][kvh][n_ctx][128]
    int kv_f16 = 0;                                  // the caches hold __half values (the fp16 KV option)
    float *rope_cos = nullptr, *rope_sin = nullptr;
    float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *ffn_inp = nullptr, *h = nullptr;
    float* logits = nullptr;
    float* chunk_logits = nullptr;
    size_t chunk_cap = 0;
    float* part_v = nullptr;
    int* part_i = nullptr;
    int* counter = nullptr;
    int* argmax = nullptr;
    int32_t *pos = nullptr, *tok_seq = nullptr, *prompt_end = nullptr, *argmax_hist = nullptr;
    int32_t* pinned = nullptr;                       // small host staging
    cudaGraphExec_t step = nullptr;
    int lm_grid = 0;
    // the layer chain as a graph, for the last (begin, n, x) it was asked for
    cudaGraphExec_t chain = nullptr;
    int chain_begin = -1, chain_n = -1;
    float* chain_x = nullptr;
    // the independent-input projections as a graph, likewise
    cudaGraphExec_t proj = nullptr;
    int proj_begin = -1, proj_n = -1;
    const float* proj_x = nullptr;
    float* proj_y = nullptr;
    void* io = nullptr;              // device staging of the host-buffer entry points
    size_t io_cap = 0;
    EngineProgram eng_chain;         // the layer chain on the persistent engine
    EngineProgram eng_proj;          // the independent projections on the persistent engine
    EngineProgram eng_decode;        // every layer of a decode step, attention included
    // the host-buffer projections in two pieces, the first piece's outputs
    // copied back on copy_stream behind the event its launch records
    EngineProgram eng_piece[kProjPieces];
    cudaEvent_t piece_done[kProjPieces] = {};
    cudaStream_t copy_stream = nullptr;
    // recorded on `stream` around the step launches of the last forward or
    // generate call (device time of the decode steps alone)
    cudaEvent_t run_ev[2] = {};
    // the multi-token chunk path (allocated at its first use): every token's
    // residual, projections, attention output and FFN state as row-major
    // [chunk][width] buffers, the per-token int8 activations and positions
    struct Chunk {
        int cap = 0;
        float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *proj = nullptr,
              *ffn_inp = nullptr, *h = nullptr;
        int8_t* qa = nullptr;
        sllm_cuda_act* acts = nullptr;
        int32_t* pos = nullptr;
        int32_t* pos_host = nullptr;      // pinned staging of the positions
    } ch;
};

// bytes of one cached value, and the cache of layer l
static size_t kv_elt(const sllm_cuda_ctx* c) { return c->kv_f16 ? 2 : 4; }
static float* kv_layer_ptr(const sllm_cuda_ctx* c, float* base, int l) {
    const size_t per = (size_t)c->m->n_embd_gqa * (size_t)c->n_ctx;
    return reinterpret_cast<float*>(reinterpret_cast<char*>(base) + (size_t)l * per * kv_elt(c));
}

// the reference's angle recurrence (src/ops.c:529-549), on the host libm
void sllm::rope_table(int n_ctx, int n_rot, float base, std::vector<float>& cs, std::vector<float>& sn) {
    const int half = n_rot / 2;
    cs.resize((size_t)n_ctx * half);
    sn.resize((size_t)n_ctx * half);
    volatile float vbase = base;                  // keep powf a run-time call
    volatile float vexp = -2.0f / (float)n_rot;
    const float theta_scale = powf(vbase, vexp);
    for (int pos = 0; pos < n_ctx; ++pos) {
        float th = (float)pos;
        for (int k = 0; k < half; ++k) {
            const float f = 1.0f * th;
            cs[(size_t)pos * half + k] = cosf(f);
            sn[(size_t)pos * half + k] = sinf(f);
            th *= theta_scale;
        }
    }
}

extern "C" void sllm_cuda_ctx_free(sllm_cuda_ctx* c) {
    if (c == nullptr) return;
    cudaSetDevice(c->m->device);
    graph_exec_destroy(c->step);
    graph_exec_destroy(c->chain);
    graph_exec_destroy(c->proj);
    if (c->stream) cudaStreamDestroy(c->stream);
    cudaFree(c->k_cache); cudaFree(c->v_cache); cudaFree(c->rope_cos); cudaFree(c->rope_sin);
    cudaFree(c->x); cudaFree(c->q); cudaFree(c->k); cudaFree(c->v); cudaFree(c->attn);
    cudaFree(c->ffn_inp); cudaFree(c->h); cudaFree(c->logits); cudaFree(c->chunk_logits);
    cudaFree(c->part_v); cudaFree(c->part_i); cudaFree(c->counter); cudaFree(c->argmax);
    cudaFree(c->pos); cudaFree(c->tok_seq); cudaFree(c->prompt_end); cudaFree(c->argmax_hist);
    cudaFreeHost(c->pinned);
    cudaFree(c->io);
    engine_program_free(c->eng_chain);
    engine_program_free(c->eng_proj);
    engine_program_free(c->eng_decode);
    for (int i = 0; i < kProjPieces; ++i) {
        engine_program_free(c->eng_piece[i]);
        if (c->piece_done[i]) cudaEventDestroy(c->piece_done[i]);
    }
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    for (cudaEvent_t ev : c->run_ev)
        if (ev) cudaEventDestroy(ev);
    for (void* p : {(void*)c->ch.x, (void*)c->ch.q, (void*)c->ch.k, (void*)c->ch.v, (void*)c->ch.attn,
                    (void*)c->ch.proj, (void*)c->ch.ffn_inp, (void*)c->ch.h, (void*)c->ch.qa, (void*)c->ch.acts,
                    (void*)c->ch.pos})
        cudaFree(p);
    if (c->ch.pos_host) cudaFreeHost(c->ch.pos_host);
    delete c;
}

extern "C" int sllm_cuda_ctx_new(const sllm_cuda_model* m, int32_t n_ctx, sllm_cuda_ctx** out) {
    return sllm_cuda_ctx_new_kv(m, n_ctx, SLLM_CUDA_KV_F32, out);
}

extern "C" int sllm_cuda_ctx_new_kv(const sllm_cuda_model* m, int32_t n_ctx, int32_t kv_type, sllm_cuda_ctx** out) {
    if (m == nullptr || out == nullptr || n_ctx <= 0) return fail(SLLM_CUDA_ERR_ARG, "ctx_new: bad arguments");
    if (kv_type != SLLM_CUDA_KV_F32 && kv_type != SLLM_CUDA_KV_F16)
        return fail(SLLM_CUDA_ERR_ARG, "ctx_new: kv_type %d is neither SLLM_CUDA_KV_F32 nor SLLM_CUDA_KV_F16", kv_type);
    *out = nullptr;
    if (n_ctx > attention_max_ctx())
        return fail(SLLM_CUDA_ERR_TOO_LARGE, "ctx_new: n_ctx %d above %d", n_ctx, attention_max_ctx());
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    CK(prepare_decode_kernels(), "kernel attributes");
    if (fallback_counter() == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "ctx_new: diagnostics counter");
    auto* c = new sllm_cuda_ctx();
    c->m = m;
    c->n_ctx = n_ctx;
    c->kv_f16 = kv_type == SLLM_CUDA_KV_F16 ? 1 : 0;
    const size_t kvb = (size_t)m->n_layer * (size_t)m->n_embd_gqa * (size_t)n_ctx * kv_elt(c);   // bytes of each cache
    const size_t E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa, V = m->n_vocab;
    c->lm_grid = lm_head_grid(num_sms_of(m->device));
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    auto A = [&](void** p, size_t bytes) { if (e == cudaSuccess) e = dev_malloc(p, bytes); };
    A((void**)&c->k_cache, kvb); A((void**)&c->v_cache, kvb);
    A((void**)&c->rope_cos, (size_t)n_ctx * 64 * 4); A((void**)&c->rope_sin, (size_t)n_ctx * 64 * 4);
    A((void**)&c->x, E * 4); A((void**)&c->q, E * 4); A((void**)&c->k, G * 4); A((void**)&c->v, G * 4);
    A((void**)&c->attn, E * 4); A((void**)&c->ffn_inp, E * 4); A((void**)&c->h, F * 4);
    A((void**)&c->logits, V * 4);
    A((void**)&c->part_v, (size_t)c->lm_grid * 4); A((void**)&c->part_i, (size_t)c->lm_grid * 4);
    A((void**)&c->counter, 4); A((void**)&c->argmax, 4);
    A((void**)&c->pos, 4); A((void**)&c->tok_seq, (size_t)n_ctx * 4 + 4); A((void**)&c->prompt_end, 4);
    A((void**)&c->argmax_hist, (size_t)n_ctx * 4);
    if (e == cudaSuccess) e = cudaMallocHost(&c->pinned, 64);
    if (e == cudaSuccess) e = cudaEventCreate(&c->run_ev[0]);
    if (e == cudaSuccess) e = cudaEventCreate(&c->run_ev[1]);
    if (e == cudaSuccess) e = cudaMemset(c->k_cache, 0, kvb);
    if (e == cudaSuccess) e = cudaMemset(c->v_cache, 0, kvb);
    if (e == cudaSuccess) e = cudaMemset(c->counter, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->pos, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->tok_seq, 0, (size_t)n_ctx * 4 + 4);
    if (e == cudaSuccess) e = cudaMemset(c->prompt_end, 0, 4);
    if (e != cudaSuccess) { sllm_cuda_ctx_free(c); return cuda_fail(e, "ctx_new"); }
    std::vector<float> cs, sn;
    rope_table(n_ctx, m->n_rot, m->rope_base, cs, sn);
    e = cudaMemcpy(c->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { sllm_cuda_ctx_free(c); return cuda_fail(e, "ctx_new: rope table"); }
    *out = c;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_ctx_reset(sllm_cuda_ctx* c) {
    if (c == nullptr) return;
    // Setting n_past = 0 is what makes a reset correct (every position is
    // written before it is read); clearing the cache is defence in depth,
    // as in src/forward.c:530-562.
    cudaSetDevice(c->m->device);
    const size_t kvb = (size_t)c->m->n_layer * (size_t)c->m->n_embd_gqa * (size_t)c->n_ctx * kv_elt(c);
    cudaMemsetAsync(c->k_cache, 0, kvb, c->stream);
    cudaMemsetAsync(c->v_cache, 0, kvb, c->stream);
    cudaStreamSynchronize(c->stream);
    c->n_past = 0;
    c->have_logits = false;
}

extern "C" int32_t sllm_cuda_ctx_n_past(const sllm_cuda_ctx* c) { return c ? c->n_past : 0; }

// The projection chain of one layer (four fused GEMV launches).
struct ChainBufs { float* x; float* q; float* k; float* v; float* ffn_inp; float* h; const float* attn; };

static cudaError_t launch_layer(const sllm_cuda_model* m, int l, const ChainBufs& b, int* fb, int force,
                                cudaStream_t st, bool with_attention, const AttnParams* ap) {
    const DevLayer& L = m->layers[l];
    const int E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa, sms = num_sms_of(m->device);
    GemvParams p{};
    p.eps = m->eps;
    p.fallback_count = fb;
    p.force_fallback = force;
    // attn_norm -> Q, K, V (src/forward.c:631-666)
    p.K = E; p.nseg = 3;
    p.seg[0] = GemvSeg{L.wq, E, b.q, nullptr};
    p.seg[1] = GemvSeg{L.wk, G, b.k, nullptr};
    p.seg[2] = GemvSeg{L.wv, G, b.v, nullptr};
    p.x = b.x; p.norm_w = L.attn_norm;
    cudaError_t e = launch_gemv(p, PRO_NORM, EPI_F32, sms, st, GEMV_DEPENDENT);
    if (e != cudaSuccess) return e;
    const float* attn_out = b.q;    // the benchmark chain feeds Q in place of attention
    if (with_attention) {
        e = launch_attention(*ap, m->n_head, st);
        if (e != cudaSuccess) return e;
        attn_out = b.attn;
    }
    // attn_sub_norm -> O, + residual (src/forward.c:728-750)
    GemvParams o = p;
    o.nseg = 1;
    o.seg[0] = GemvSeg{L.wo, E, b.ffn_inp, nullptr};
    o.x = attn_out; o.norm_w = L.attn_sub_norm; o.resid = b.x;
    e = launch_gemv(o, PRO_NORM, EPI_RESID, sms, st, GEMV_DEPENDENT);
    if (e != cudaSuccess) return e;
    // ffn_norm -> gate, up, silu(gate) * up (src/forward.c:752-779)
    GemvParams f = p;
    f.nseg = 2;
    f.seg[0] = GemvSeg{L.gate, F, nullptr, nullptr};
    f.seg[1] = GemvSeg{L.up, F, nullptr, nullptr};
    f.x = b.ffn_inp; f.norm_w = L.ffn_norm; f.h_out = b.h;
    e = launch_gemv(f, PRO_NORM, EPI_SILU, sms, st, GEMV_DEPENDENT);
    if (e != cudaSuccess) return e;
    // ffn_sub_norm -> down, + residual (src/forward.c:781-801)
    GemvParams dn = p;
    dn.K = F; dn.nseg = 1;
    dn.seg[0] = GemvSeg{L.down, E, b.x, nullptr};
    dn.x = b.h; dn.norm_w = L.ffn_sub_norm; dn.resid = b.ffn_inp;
    return launch_gemv(dn, PRO_NORM, EPI_RESID, sms, st, GEMV_DEPENDENT);
}

static cudaError_t enqueue_step(sllm_cuda_ctx* c, cudaStream_t st) {
    const sllm_cuda_model* m = c->m;
    int* fb = fallback_counter();
    // the embedding kernel also zeroes the engine's grid barrier, which the
    // engine launch behind it in the stream then counts up from
    cudaError_t e = launch_embed(m->tok_embd, c->tok_seq, c->pos, m->n_embd, m->n_vocab, c->x, st,
                                 c->eng_decode.built ? c->eng_decode.barrier : nullptr);
    if (e != cudaSuccess) return e;
    if (c->eng_decode.built) {
        // every layer in one engine launch: 5 stages each (Q/K/V, attention,
        // O, gate/up, down) behind grid barriers
        e = launch_engine(c->eng_decode.params, c->eng_decode.grid, st, c->eng_decode.wa, c->eng_decode.wb);
        if (e != cudaSuccess) return e;
        LmParams lp{};
        lp.x = c->x; lp.norm_w = m->output_norm; lp.eps = m->eps; lp.embd = m->tok_embd;
        lp.E = m->n_embd; lp.V = m->n_vocab; lp.logits = c->logits;
        lp.part_v = c->part_v; lp.part_i = c->part_i; lp.counter = c->counter; lp.argmax_out = c->argmax;
        lp.pos_ptr = c->pos; lp.tok_seq = c->tok_seq; lp.prompt_end = c->prompt_end; lp.argmax_hist = c->argmax_hist;
        lp.n_ctx = c->n_ctx; lp.fallback_count = fb; lp.force_fallback = g_force_fallback;
        return launch_lm_head(lp, c->lm_grid, st);
    }
    for (int l = 0; l < m->n_layer; ++l) {
        AttnParams ap{};
        ap.q = c->q; ap.k = c->k; ap.v = c->v;
        ap.k_cache = kv_layer_ptr(c, c->k_cache, l);
        ap.v_cache = kv_layer_ptr(c, c->v_cache, l);
        ap.kv_f16 = c->kv_f16;
        ap.rope_cos = c->rope_cos; ap.rope_sin = c->rope_sin;
        ap.pos_ptr = c->pos; ap.out = c->attn; ap.n_ctx = c->n_ctx;
        ap.group = m->n_head / m->n_head_kv;
        ap.attn_scale = 1.0f / sqrtf((float)m->head_dim);
        ap.fallback_count = fb; ap.force_fallback = g_force_fallback;
        ChainBufs b{c->x, c->q, c->k, c->v, c->ffn_inp, c->h, c->attn};
        e = launch_layer(m, l, b, fb, g_force_fallback, st, true, &ap);
        if (e != cudaSuccess) return e;
    }
    LmParams lp{};
    lp.x = c->x; lp.norm_w = m->output_norm; lp.eps = m->eps; lp.embd = m->tok_embd;
    lp.E = m->n_embd; lp.V = m->n_vocab; lp.logits = c->logits;
    lp.part_v = c->part_v; lp.part_i = c->part_i; lp.counter = c->counter; lp.argmax_out = c->argmax;
    lp.pos_ptr = c->pos; lp.tok_seq = c->tok_seq; lp.prompt_end = c->prompt_end; lp.argmax_hist = c->argmax_hist;
    lp.n_ctx = c->n_ctx; lp.fallback_count = fb; lp.force_fallback = g_force_fallback;
    return launch_lm_head(lp, c->lm_grid, st);
}

static int decode_program(sllm_cuda_ctx* c);

static int ensure_step_graph(sllm_cuda_ctx* c) {
    if (c->step != nullptr) return SLLM_CUDA_OK;
    const int rc = decode_program(c);
    if (rc != SLLM_CUDA_OK) return rc;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    cudaError_t e = enqueue_step(c, c->stream);
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); return cuda_fail(e, "capture decode step"); }
    if (e2 != cudaSuccess) return cuda_fail(e2, "end capture");
    e = instantiate(&c->step, g);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { c->step = nullptr; return cuda_fail(e, "instantiate decode step"); }
    return SLLM_CUDA_OK;
}

// Run positions [base, base + n) whose tokens are already in tok_seq.
static int run_steps(sllm_cuda_ctx* c, int base, int n, int prompt_end, float* chunk_logits_dev,
                     bool start_timer = true) {
    int rc = ensure_step_graph(c);
    if (rc != SLLM_CUDA_OK) return rc;
    c->pinned[0] = base;
    c->pinned[1] = prompt_end;
    CK(cudaMemcpyAsync(c->pos, &c->pinned[0], 4, cudaMemcpyHostToDevice, c->stream), "set pos");
    CK(cudaMemcpyAsync(c->prompt_end, &c->pinned[1], 4, cudaMemcpyHostToDevice, c->stream), "set prompt end");
    const size_t V = c->m->n_vocab;
    if (start_timer) CK(cudaEventRecord(c->run_ev[0], c->stream), "run timer");
    for (int t = 0; t < n; ++t) {
        CK(graph_launch(c->step, c->stream), "decode step");
        if (chunk_logits_dev != nullptr)
            CK(cudaMemcpyAsync(chunk_logits_dev + (size_t)t * V, c->logits, V * 4, cudaMemcpyDeviceToDevice, c->stream),
               "copy logits");
    }
    CK(cudaEventRecord(c->run_ev[1], c->stream), "run timer");
    return SLLM_CUDA_OK;
}

extern "C" float sllm_cuda_test_ctx_last_run_ms(const sllm_cuda_ctx* c) {
    float ms = -1.0f;
    if (c == nullptr || cudaSetDevice(c->m->device) != cudaSuccess) return -1.0f;
    if (cudaEventElapsedTime(&ms, c->run_ev[0], c->run_ev[1]) != cudaSuccess) {
        cudaGetLastError();
        return -1.0f;
    }
    return ms;
}

// ---------------------------------------------------------------------------
// The multi-token chunk (src/forward.c:589-835 with n > 1) on the tensor
// cores: per layer, every token's RMSNorm + quantisation, the projections of
// all tokens as tcgen05 GEMMs (each weight byte read once for the chunk
// instead of once per token), RoPE and the cache stores of every token, then
// causal attention for every (head, token). Every value equals the
// one-token-at-a-time path's: the same per-token prologue arithmetic, integer
// dots, epilogues, attention order. A chunk is not a semantic boundary
// (src/forward.c:572-588), and neither is this.
// ---------------------------------------------------------------------------
static constexpr int kChunkMax = 256;      // SLLM_MAX_CHUNK (include/saphira_llm/forward.h:90)

static int chunk_alloc(sllm_cuda_ctx* c) {
    if (c->ch.cap >= kChunkMax) return SLLM_CUDA_OK;
    const sllm_cuda_model* m = c->m;
    const size_t T = kChunkMax, E = m->n_embd, G = m->n_embd_gqa, F = m->n_ff;
    cudaError_t e = cudaSuccess;
    auto A = [&](void** p, size_t bytes) { if (e == cudaSuccess) e = dev_malloc(p, bytes); };
    A((void**)&c->ch.x, T * E * 4); A((void**)&c->ch.q, T * E * 4); A((void**)&c->ch.k, T * G * 4);
    A((void**)&c->ch.v, T * G * 4); A((void**)&c->ch.attn, T * E * 4); A((void**)&c->ch.proj, T * E * 4);
    A((void**)&c->ch.ffn_inp, T * E * 4); A((void**)&c->ch.h, T * F * 4);
    A((void**)&c->ch.qa, T * std::max(E, F)); A((void**)&c->ch.acts, T * sizeof(sllm_cuda_act));
    A((void**)&c->ch.pos, T * 4);
    if (e == cudaSuccess) e = cudaMallocHost(&c->ch.pos_host, T * 4);
    if (e != cudaSuccess) return cuda_fail(e, "chunk buffers");
    c->ch.cap = kChunkMax;
    return SLLM_CUDA_OK;
}

// the chunk path runs where the GEMM and the attention kernels do
static bool chunk_path_ok(const sllm_cuda_ctx* c) {
    const sllm_cuda_model* m = c->m;
    return m->head_dim == 128 && m->n_embd % 128 == 0 && m->n_ff % 128 == 0 && c->n_ctx <= attention_max_ctx();
}

// Positions [base, base + n) whose tokens are in tok_seq. heads: -1 every
// position's head (logits into logits_dev rows when it is not null), or the
// number of trailing positions whose head runs (0: none). The head of the
// last position leaves the greedy next token at tok_seq[base + n] when
// base + n >= prompt_end, as a decode step does.
static int run_chunk(sllm_cuda_ctx* c, int base, int n, int prompt_end, int heads, float* logits_dev) {
    const sllm_cuda_model* m = c->m;
    const cudaStream_t st = c->stream;
    const int E = m->n_embd, G = m->n_embd_gqa, F = m->n_ff;
    int rc = chunk_alloc(c);
    if (rc != SLLM_CUDA_OK) return rc;
    int* fb = fallback_counter();
    int* gerr = gemm_error_word();
    if (fb == nullptr || gerr == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "chunk: diagnostics words");
    CK(cudaStreamSynchronize(st), "chunk positions");        // the pinned staging is free again
    for (int t = 0; t < n; ++t) c->ch.pos_host[t] = base + t;
    CK(cudaMemcpyAsync(c->ch.pos, c->ch.pos_host, (size_t)n * 4, cudaMemcpyHostToDevice, st), "chunk positions");
    CK(launch_embed_rows(m->tok_embd, c->tok_seq + base, n, E, m->n_vocab, c->ch.x, st), "chunk embed");
    auto gemm = [&](const uint8_t* w, const uint8_t* w2, int rows, int K, float* y) {
        GemmArgs a{};
        a.w = w; a.w2 = w2; a.q = c->ch.qa; a.acts = c->ch.acts; a.dots = nullptr; a.y = y;
        a.m = n; a.n_rows = rows; a.K = K;
        const char* why = nullptr;
        const int r = gemm_check(a, &why);
        if (r != SLLM_CUDA_OK) return fail(r, "chunk gemm: %s", why);
        CK(launch_i2s_gemm(a, gerr, st), "chunk gemm");
        return (int)SLLM_CUDA_OK;
    };
    const int force = g_force_fallback;
    for (int l = 0; l < m->n_layer; ++l) {
        const DevLayer& L = m->layers[l];
        // attn_norm -> Q, K, V of every token (src/forward.c:631-666)
        CK(launch_norm_quant_rows(c->ch.x, L.attn_norm, E, m->eps, n, c->ch.qa, c->ch.acts, fb, force, st), "chunk norm");
        if ((rc = gemm(L.wq, nullptr, E, E, c->ch.q)) != SLLM_CUDA_OK) return rc;
        if ((rc = gemm(L.wk, nullptr, G, E, c->ch.k)) != SLLM_CUDA_OK) return rc;
        if ((rc = gemm(L.wv, nullptr, G, E, c->ch.v)) != SLLM_CUDA_OK) return rc;
        // RoPE, the cache stores of every token, then attention (src/forward.c:668-726)
        AttnParams ap{};
        ap.q = c->ch.q; ap.k = c->ch.k; ap.v = c->ch.v;
        ap.k_cache = kv_layer_ptr(c, c->k_cache, l);
        ap.v_cache = kv_layer_ptr(c, c->v_cache, l);
        ap.kv_f16 = c->kv_f16 ? kAttnKvF16 : 0;
        ap.rope_cos = c->rope_cos; ap.rope_sin = c->rope_sin;
        ap.out = c->ch.attn; ap.n_ctx = c->n_ctx;
        ap.group = m->n_head / m->n_head_kv;
        ap.attn_scale = 1.0f / sqrtf((float)m->head_dim);
        ap.fallback_count = fb; ap.force_fallback = force;
        CK(launch_chunk_kv_store(ap, c->ch.pos, n, m->n_head_kv, E, G, st), "chunk kv store");
        CK(launch_attention_chunk(ap, c->ch.pos, n, m->n_head, E, G, st), "chunk attention");
        // attn_sub_norm -> O, + x (src/forward.c:728-750)
        CK(launch_norm_quant_rows(c->ch.attn, L.attn_sub_norm, E, m->eps, n, c->ch.qa, c->ch.acts, fb, force, st),
           "chunk norm");
        if ((rc = gemm(L.wo, nullptr, E, E, c->ch.proj)) != SLLM_CUDA_OK) return rc;
        CK(launch_add(c->ch.proj, c->ch.x, c->ch.ffn_inp, (size_t)n * E, st), "chunk residual");
        // ffn_norm -> gate, up, silu(gate) * up (src/forward.c:752-779)
        CK(launch_norm_quant_rows(c->ch.ffn_inp, L.ffn_norm, E, m->eps, n, c->ch.qa, c->ch.acts, fb, force, st),
           "chunk norm");
        if ((rc = gemm(L.gate, L.up, F, E, c->ch.h)) != SLLM_CUDA_OK) return rc;
        // ffn_sub_norm -> down, + ffn_inp (src/forward.c:781-801)
        CK(launch_norm_quant_rows(c->ch.h, L.ffn_sub_norm, F, m->eps, n, c->ch.qa, c->ch.acts, fb, force, st),
           "chunk norm");
        if ((rc = gemm(L.down, nullptr, E, F, c->ch.proj)) != SLLM_CUDA_OK) return rc;
        CK(launch_add(c->ch.proj, c->ch.ffn_inp, c->ch.x, (size_t)n * E, st), "chunk residual");
    }
    count_launches((long long)m->n_layer * 15 + 1);
    // the heads: output_norm + the tied F16 head + argmax of each position
    // wanted, in position order (src/forward.c:803-833)
    const int h0 = heads < 0 ? 0 : n - std::min(heads, n);
    if (h0 < n) {
        // slots of the pinned staging of their own: a decode step enqueued
        // right after this may rewrite slots 0 and 1 before these copies run
        c->pinned[4] = base + h0;
        c->pinned[5] = prompt_end;
        CK(cudaMemcpyAsync(c->pos, &c->pinned[4], 4, cudaMemcpyHostToDevice, st), "set pos");
        CK(cudaMemcpyAsync(c->prompt_end, &c->pinned[5], 4, cudaMemcpyHostToDevice, st), "set prompt end");
        const size_t V = m->n_vocab;
        for (int t = h0; t < n; ++t) {
            LmParams lp{};
            lp.x = c->ch.x + (size_t)t * E; lp.norm_w = m->output_norm; lp.eps = m->eps; lp.embd = m->tok_embd;
            lp.E = E; lp.V = m->n_vocab; lp.logits = c->logits;
            lp.part_v = c->part_v; lp.part_i = c->part_i; lp.counter = c->counter; lp.argmax_out = c->argmax;
            lp.pos_ptr = c->pos; lp.tok_seq = c->tok_seq; lp.prompt_end = c->prompt_end;
            lp.argmax_hist = c->argmax_hist; lp.n_ctx = c->n_ctx; lp.fallback_count = fb; lp.force_fallback = force;
            CK(launch_lm_head(lp, c->lm_grid, st), "chunk head");
            count_launches(1);
            if (logits_dev != nullptr)
                CK(cudaMemcpyAsync(logits_dev + (size_t)t * V, c->logits, V * 4, cudaMemcpyDeviceToDevice, st),
                   "copy logits");
        }
    }
    return SLLM_CUDA_OK;
}

// a GEMM whose bounded wait gave up reports it once (the word is cleared)
static int chunk_error() {
    int* w = gemm_error_word();
    int v = 0;
    if (w != nullptr && cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && v != 0) {
        cudaMemset(w, 0, sizeof(int));
        return fail(SLLM_CUDA_ERR_TIMEOUT, "chunk: a GEMM's bounded wait gave up (code %d)", v);
    }
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_forward_chunk(const sllm_cuda_model* m, sllm_cuda_ctx* c, const int32_t* tokens, int32_t n,
                                       int32_t base, float* logits_out, int32_t* argmax_out) {
    if (m == nullptr || c == nullptr || tokens == nullptr || (logits_out == nullptr && argmax_out == nullptr) ||
        c->m != m)
        return fail(SLLM_CUDA_ERR_ARG, "forward_chunk: bad arguments");
    if (n < 1 || n > 256) return fail(SLLM_CUDA_ERR_ARG, "forward_chunk: n=%d outside [1, 256]", n);
    if (base < c->n_past || base + n > c->n_ctx)
        return fail(SLLM_CUDA_ERR_ARG, "forward_chunk: positions [%d, %d) outside [n_past=%d, n_ctx=%d]", base,
                    base + n, c->n_past, c->n_ctx);
    for (int t = 0; t < n; ++t)
        if (tokens[t] < 0 || tokens[t] >= m->n_vocab) return fail(SLLM_CUDA_ERR_ARG, "forward_chunk: token %d out of range", tokens[t]);
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    const size_t V = m->n_vocab;
    if (logits_out != nullptr && c->chunk_cap < (size_t)n) {
        cudaFree(c->chunk_logits);
        c->chunk_logits = nullptr;
        c->chunk_cap = 0;
        CK(cudaMalloc(&c->chunk_logits, (size_t)n * V * 4), "chunk logits");
        c->chunk_cap = n;
    }
    CK(cudaMemcpyAsync(c->tok_seq + base, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream), "tokens");
    int rc;
    if (n >= 2 && chunk_path_ok(c)) {
        // every position's head runs: each position's logits and argmax are outputs
        CK(cudaEventRecord(c->run_ev[0], c->stream), "run timer");
        rc = run_chunk(c, base, n, base + n, -1, logits_out ? c->chunk_logits : nullptr);
        if (rc == SLLM_CUDA_OK) CK(cudaEventRecord(c->run_ev[1], c->stream), "run timer");
    } else {
        rc = run_steps(c, base, n, base + n, logits_out ? c->chunk_logits : nullptr);
    }
    if (rc != SLLM_CUDA_OK) return rc;
    if (logits_out != nullptr)
        CK(cudaMemcpyAsync(logits_out, c->chunk_logits, (size_t)n * V * 4, cudaMemcpyDeviceToHost, c->stream), "logits");
    if (argmax_out != nullptr)
        CK(cudaMemcpyAsync(argmax_out, c->argmax_hist + base, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream), "argmax");
    CK(cudaStreamSynchronize(c->stream), "forward_chunk sync");
    if (c->eng_decode.built) {
        const int rc_e = engine_error(c->eng_decode);
        if (rc_e != SLLM_CUDA_OK) return rc_e;
    }
    if ((rc = chunk_error()) != SLLM_CUDA_OK) return rc;
    c->n_past = base + n;
    c->have_logits = true;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_generate_greedy(const sllm_cuda_model* m, sllm_cuda_ctx* c, const int32_t* prompt,
                                         int32_t n_prompt, int32_t n_new, int32_t* out) {
    if (m == nullptr || c == nullptr || out == nullptr || n_prompt < 0 || n_new < 0 || c->m != m ||
        (n_prompt > 0 && prompt == nullptr))
        return fail(SLLM_CUDA_ERR_ARG, "generate_greedy: bad arguments");
    if ((int64_t)n_prompt + n_new + c->n_past > c->n_ctx)
        return fail(SLLM_CUDA_ERR_TOO_LARGE, "generate_greedy: %d + %d tokens after %d exceed n_ctx %d", n_prompt,
                    n_new, c->n_past, c->n_ctx);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->n_vocab) return fail(SLLM_CUDA_ERR_ARG, "generate_greedy: token %d out of range", prompt[i]);
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    const int base = c->n_past;
    if (n_prompt == 0 && base == 0) {
        // no prompt and no history: the model's BOS (src/forward.c:909)
        if (n_new == 0) return SLLM_CUDA_OK;
        if (128000 >= m->n_vocab) return fail(SLLM_CUDA_ERR_ARG, "generate_greedy: BOS 128000 outside the vocabulary");
        c->pinned[2] = 128000;
        CK(cudaMemcpyAsync(c->tok_seq, &c->pinned[2], 4, cudaMemcpyHostToDevice, c->stream), "bos");
    } else if (n_prompt > 0) {
        CK(cudaMemcpyAsync(c->tok_seq + base, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, c->stream), "prompt");
    }
    // with no prompt and a history, tok_seq[base] already holds the argmax of
    // the last logits, written by the step that produced them
    const int steps = n_prompt + n_new;
    if (n_prompt >= 2 && chunk_path_ok(c)) {
        // the prompt as chunks of up to 256 tokens on the tensor cores; only
        // the last position's head matters (its logits and next token), then
        // one decode step per new token
        CK(cudaEventRecord(c->run_ev[0], c->stream), "run timer");
        for (int done = 0; done < n_prompt;) {
            const int take = std::min(kChunkMax, n_prompt - done);
            const bool last = done + take == n_prompt;
            int rc = run_chunk(c, base + done, take, base + n_prompt, last ? 1 : 0, nullptr);
            if (rc != SLLM_CUDA_OK) return rc;
            done += take;
        }
        if (n_new > 0) {
            int rc = run_steps(c, base + n_prompt, n_new, base + n_prompt, nullptr, false);
            if (rc != SLLM_CUDA_OK) return rc;
        } else {
            CK(cudaEventRecord(c->run_ev[1], c->stream), "run timer");
        }
    } else if (steps > 0) {
        int rc = run_steps(c, base, steps, base + n_prompt, nullptr);
        if (rc != SLLM_CUDA_OK) return rc;
    }
    if (n_new > 0)
        CK(cudaMemcpyAsync(out, c->tok_seq + base + n_prompt, (size_t)n_new * 4, cudaMemcpyDeviceToHost, c->stream), "ids");
    CK(cudaStreamSynchronize(c->stream), "generate sync");
    if (c->eng_decode.built) {
        const int rc_e = engine_error(c->eng_decode);
        if (rc_e != SLLM_CUDA_OK) return rc_e;
    }
    {
        const int rc_c = chunk_error();
        if (rc_c != SLLM_CUDA_OK) return rc_c;
    }
    c->n_past = base + steps;
    if (steps > 0) c->have_logits = true;
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_ctx_last_logits(const sllm_cuda_ctx* c, float* host_out) {
    if (c == nullptr || host_out == nullptr || !c->have_logits) return fail(SLLM_CUDA_ERR_ARG, "last_logits: nothing forwarded");
    CK(cudaSetDevice(c->m->device), "cudaSetDevice");
    CK(cudaMemcpy(host_out, c->logits, (size_t)c->m->n_vocab * 4, cudaMemcpyDeviceToHost), "last logits");
    return SLLM_CUDA_OK;
}

// ---------------------------------------------------------------------------
// the KV cache in the reference's layout, and state files (src/forward.c:963-1123)
// ---------------------------------------------------------------------------
// The device keeps K transposed ([layer][kvh][dim][n_ctx]) and V as
// [layer][kvh][n_ctx][dim]; the reference keeps both as [layer][kvh][pos][dim]
// (src/forward.c:81-83). These copy the live prefix between the two.
extern "C" int sllm_cuda_ctx_kv_export(const sllm_cuda_ctx* c, float* k_out, float* v_out) {
    if (c == nullptr || k_out == nullptr || v_out == nullptr) return fail(SLLM_CUDA_ERR_ARG, "kv_export: NULL argument");
    CK(cudaSetDevice(c->m->device), "cudaSetDevice");
    CK(cudaStreamSynchronize(c->stream), "kv_export sync");
    const sllm_cuda_model* m = c->m;
    const size_t D = m->head_dim, N = c->n_ctx, P = c->n_past;
    const size_t heads = (size_t)m->n_layer * (size_t)m->n_head_kv;
    if (P == 0) return SLLM_CUDA_OK;
    const size_t eb = kv_elt(c);
    std::vector<unsigned char> kt(D * P * eb), vt(P * D * eb);
    const char* kbase = reinterpret_cast<const char*>(c->k_cache);
    const char* vbase = reinterpret_cast<const char*>(c->v_cache);
    // an f16 cache's values widen exactly
    auto val = [&](const unsigned char* b, size_t i) {
        return eb == 4 ? reinterpret_cast<const float*>(b)[i] : __half2float(reinterpret_cast<const __half*>(b)[i]);
    };
    for (size_t lh = 0; lh < heads; ++lh) {
        const char* kd = kbase + lh * D * N * eb;          // [dim][n_ctx]
        const char* vd = vbase + lh * N * D * eb;          // [n_ctx][dim]
        CK(cudaMemcpy2D(kt.data(), P * eb, kd, N * eb, P * eb, D, cudaMemcpyDeviceToHost), "kv_export K");
        CK(cudaMemcpy(vt.data(), vd, P * D * eb, cudaMemcpyDeviceToHost), "kv_export V");
        float* kh = k_out + lh * N * D;                    // [pos][dim]
        float* vh = v_out + lh * N * D;
        for (size_t pos = 0; pos < P; ++pos)
            for (size_t d = 0; d < D; ++d) {
                kh[pos * D + d] = val(kt.data(), d * P + pos);
                vh[pos * D + d] = val(vt.data(), pos * D + d);
            }
    }
    return SLLM_CUDA_OK;
}

// the reference's sllm_argmax (src/forward.c:876-883): the first maximum by '>'
static int32_t host_argmax(const float* v, int32_t n) {
    int32_t best = 0;
    float bv = v[0];
    for (int32_t i = 1; i < n; ++i)
        if (v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

extern "C" int sllm_cuda_ctx_kv_import(sllm_cuda_ctx* c, const float* k_in, const float* v_in, int32_t n_past,
                                       const float* last_logits) {
    if (c == nullptr || (n_past > 0 && (k_in == nullptr || v_in == nullptr || last_logits == nullptr)))
        return fail(SLLM_CUDA_ERR_ARG, "kv_import: NULL argument");
    if (n_past < 0 || n_past > c->n_ctx)
        return fail(SLLM_CUDA_ERR_ARG, "kv_import: n_past %d outside [0, n_ctx=%d]", n_past, c->n_ctx);
    CK(cudaSetDevice(c->m->device), "cudaSetDevice");
    CK(cudaStreamSynchronize(c->stream), "kv_import sync");
    const sllm_cuda_model* m = c->m;
    const size_t D = m->head_dim, N = c->n_ctx, P = n_past;
    const size_t heads = (size_t)m->n_layer * (size_t)m->n_head_kv;
    const size_t eb = kv_elt(c);
    std::vector<unsigned char> kt(D * (P > 0 ? P : 1) * eb), vt((P > 0 ? P : 1) * D * eb);
    char* kbase = reinterpret_cast<char*>(c->k_cache);
    char* vbase = reinterpret_cast<char*>(c->v_cache);
    // an f16 cache stores each value rounded to the nearest half (ties to even)
    auto put = [&](unsigned char* b, size_t i, float v) {
        if (eb == 4) reinterpret_cast<float*>(b)[i] = v;
        else reinterpret_cast<__half*>(b)[i] = __float2half_rn(v);
    };
    for (size_t lh = 0; lh < heads; ++lh) {
        char* kd = kbase + lh * D * N * eb;
        char* vd = vbase + lh * N * D * eb;
        if (P > 0) {
            const float* kh = k_in + lh * N * D;
            const float* vh = v_in + lh * N * D;
            for (size_t pos = 0; pos < P; ++pos)
                for (size_t d = 0; d < D; ++d) {
                    put(kt.data(), d * P + pos, kh[pos * D + d]);
                    put(vt.data(), pos * D + d, vh[pos * D + d]);
                }
            CK(cudaMemcpy2D(kd, N * eb, kt.data(), P * eb, P * eb, D, cudaMemcpyHostToDevice), "kv_import K");
            CK(cudaMemcpy(vd, vt.data(), P * D * eb, cudaMemcpyHostToDevice), "kv_import V");
        }
        // positions past n_past read as absent (src/forward.c:1104-1118)
        if (P < N) {
            CK(cudaMemset2D(kd + P * eb, N * eb, 0, (N - P) * eb, D), "kv_import clear K");
            CK(cudaMemset(vd + P * D * eb, 0, (N - P) * D * eb), "kv_import clear V");
        }
    }
    if (P > 0) {
        CK(cudaMemcpy(c->logits, last_logits, (size_t)m->n_vocab * 4, cudaMemcpyHostToDevice), "kv_import logits");
        // a continuation without a prompt starts from the argmax of these
        // logits, which a decode step would have left at tok_seq[n_past]
        const int32_t next = host_argmax(last_logits, m->n_vocab);
        CK(cudaMemcpy(c->tok_seq + P, &next, 4, cudaMemcpyHostToDevice), "kv_import next token");
    }
    c->n_past = n_past;
    c->have_logits = n_past > 0;
    return SLLM_CUDA_OK;
}

// SLKV version 1, the reference's state format (src/forward.c:963-993): a
// header of eight 32-bit fields, then per layer and kv head the live K rows
// and V rows as [pos][dim] floats, then the last position's n_vocab logits.
static constexpr uint32_t kStateMagic = 0x564B4C53u;   // "SLKV"
static constexpr uint32_t kStateVersion = 1u;

extern "C" int sllm_cuda_state_save(const sllm_cuda_model* m, const sllm_cuda_ctx* c, const char* path) {
    if (m == nullptr || c == nullptr || path == nullptr || c->m != m) return fail(SLLM_CUDA_ERR_ARG, "state_save: bad arguments");
    const size_t D = m->head_dim, N = c->n_ctx, P = c->n_past, V = m->n_vocab;
    const size_t heads = (size_t)m->n_layer * (size_t)m->n_head_kv;
    std::vector<float> k(heads * N * D), v(heads * N * D), logits(V, 0.0f);
    int rc = sllm_cuda_ctx_kv_export(c, k.data(), v.data());
    if (rc != SLLM_CUDA_OK) return rc;
    // the reference writes whatever its last-logits buffer holds; a context
    // that never ran has none here, and zeros stand in for them
    if (c->have_logits) CK(cudaMemcpy(logits.data(), c->logits, V * 4, cudaMemcpyDeviceToHost), "state_save logits");
    FILE* f = fopen(path, "wb");
    if (f == nullptr) return fail(SLLM_CUDA_ERR_IO, "state_save: cannot open %s", path);
    const int32_t hdr[8] = {(int32_t)kStateMagic, (int32_t)kStateVersion, m->n_layer, c->n_ctx, m->n_head_kv,
                            m->head_dim, c->n_past, m->n_vocab};
    bool ok = fwrite(hdr, 4, 8, f) == 8;
    for (size_t lh = 0; ok && lh < heads; ++lh) {
        if (P > 0 && fwrite(k.data() + lh * N * D, 4, P * D, f) != P * D) ok = false;
        if (ok && P > 0 && fwrite(v.data() + lh * N * D, 4, P * D, f) != P * D) ok = false;
    }
    if (ok && fwrite(logits.data(), 4, V, f) != V) ok = false;
    if (fclose(f) != 0) ok = false;
    return ok ? SLLM_CUDA_OK : fail(SLLM_CUDA_ERR_IO, "state_save: write to %s failed", path);
}

extern "C" int sllm_cuda_state_load(const sllm_cuda_model* m, sllm_cuda_ctx* c, const char* path) {
    if (m == nullptr || c == nullptr || path == nullptr || c->m != m) return fail(SLLM_CUDA_ERR_ARG, "state_load: bad arguments");
    FILE* f = fopen(path, "rb");
    if (f == nullptr) return fail(SLLM_CUDA_ERR_IO, "state_load: cannot open %s", path);
    uint32_t hdr[8] = {};
    // the reference's status for each refusal (src/forward.c:1034-1068)
    if (fread(hdr, 4, 2, f) != 2 || hdr[0] != kStateMagic || hdr[1] != kStateVersion) {
        fclose(f);
        return fail(SLLM_CUDA_ERR_KV_TYPE, "state_load: %s is not an SLKV v1 file", path);
    }
    if (fread(hdr + 2, 4, 6, f) != 6) {
        fclose(f);
        return fail(SLLM_CUDA_ERR_TRUNCATED, "state_load: %s: truncated header", path);
    }
    const int32_t n_layer = (int32_t)hdr[2], n_ctx = (int32_t)hdr[3], n_head_kv = (int32_t)hdr[4];
    const int32_t head_dim = (int32_t)hdr[5], n_past = (int32_t)hdr[6], n_vocab = (int32_t)hdr[7];
    if (n_layer != m->n_layer || n_head_kv != m->n_head_kv || head_dim != m->head_dim || n_ctx != c->n_ctx ||
        n_vocab != m->n_vocab || n_past < 0 || n_past > c->n_ctx) {
        fclose(f);
        return fail(SLLM_CUDA_ERR_TENSOR_SHAPE, "state_load: %s was saved for another geometry", path);
    }
    const size_t D = head_dim, N = n_ctx, P = n_past, V = n_vocab;
    const size_t heads = (size_t)n_layer * (size_t)n_head_kv;
    std::vector<float> k(heads * N * D, 0.0f), v(heads * N * D, 0.0f), logits(V);
    bool ok = true;
    for (size_t lh = 0; ok && lh < heads; ++lh) {
        if (P > 0 && fread(k.data() + lh * N * D, 4, P * D, f) != P * D) ok = false;
        if (ok && P > 0 && fread(v.data() + lh * N * D, 4, P * D, f) != P * D) ok = false;
    }
    if (ok && fread(logits.data(), 4, V, f) != V) ok = false;
    fclose(f);
    if (!ok) return fail(SLLM_CUDA_ERR_TRUNCATED, "state_load: %s is truncated", path);
    return sllm_cuda_ctx_kv_import(c, k.data(), v.data(), n_past, logits.data());
}

// The decode step's layers as one engine program: per layer Q/K/V, attention,
// O + residual, gate/up, down + residual, each a stage behind a grid barrier
// (src/forward.c:628-801). Built when the model's widths are compiled into
// the engine, the context fits the attention scratch, and the tables fit in
// shared memory; otherwise the step runs the per-GEMV kernels.
static int decode_program(sllm_cuda_ctx* c) {
    const sllm_cuda_model* m = c->m;
    if (c->eng_decode.built) return SLLM_CUDA_OK;
    const int E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa;
    if (!engine_supports(engine_wpl(E), engine_wpl(F)) || c->n_ctx > kEngAttnMaxCtx || m->head_dim != 128 ||
        (c->kv_f16 && !engine_supports_kv16(engine_wpl(E), engine_wpl(F))))
        return SLLM_CUDA_OK;
    int* fb = fallback_counter();
    std::vector<EngGroup> groups;
    std::vector<EngOp> ops;
    std::vector<int> stage_first;
    std::vector<AttnParams> attn;
    auto op = [&](const uint8_t* w, const uint8_t* w2, float* y, const float* resid, float* h, int rows, int K,
                  int epi, int group, float ws, float ws2) {
        EngOp o{};
        o.w = w; o.w2 = w2; o.y = y; o.resid = resid; o.h = h; o.rows = rows; o.K = K; o.epi = epi; o.group = group;
        o.chunk_rows = epi == kEpiAttention ? 1 : engine_chunk_rows(K, epi);
        o.ws = ws; o.ws2 = ws2;
        ops.push_back(o);
    };
    for (int l = 0; l < m->n_layer; ++l) {
        const DevLayer& L = m->layers[l];
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->x, L.attn_norm, E, PRO_NORM});
        op(L.wq, nullptr, c->q, nullptr, nullptr, E, E, EPI_F32, (int)groups.size() - 1, L.s_wq, 0.f);
        op(L.wk, nullptr, c->k, nullptr, nullptr, G, E, EPI_F32, (int)groups.size() - 1, L.s_wk, 0.f);
        op(L.wv, nullptr, c->v, nullptr, nullptr, G, E, EPI_F32, (int)groups.size() - 1, L.s_wv, 0.f);
        stage_first.push_back((int)ops.size());
        AttnParams ap{};
        ap.q = c->q; ap.k = c->k; ap.v = c->v;
        ap.k_cache = kv_layer_ptr(c, c->k_cache, l);
        ap.v_cache = kv_layer_ptr(c, c->v_cache, l);
        ap.kv_f16 = c->kv_f16;
        ap.rope_cos = c->rope_cos; ap.rope_sin = c->rope_sin;
        ap.pos_ptr = c->pos; ap.out = c->attn; ap.n_ctx = c->n_ctx;
        ap.group = m->n_head / m->n_head_kv;
        ap.attn_scale = 1.0f / sqrtf((float)m->head_dim);
        ap.fallback_count = fb; ap.force_fallback = g_force_fallback;
        attn.push_back(ap);
        op(nullptr, nullptr, c->attn, nullptr, nullptr, m->n_head, c->n_ctx, kEpiAttention, l, 0.f, 0.f);
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->attn, L.attn_sub_norm, E, PRO_NORM});
        op(L.wo, nullptr, c->ffn_inp, c->x, nullptr, E, E, EPI_RESID, (int)groups.size() - 1, L.s_wo, 0.f);
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->ffn_inp, L.ffn_norm, E, PRO_NORM});
        op(L.gate, L.up, nullptr, nullptr, c->h, F, E, EPI_SILU, (int)groups.size() - 1, L.s_gate, L.s_up);
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->h, L.ffn_sub_norm, F, PRO_NORM});
        op(L.down, nullptr, c->x, c->ffn_inp, nullptr, E, F, EPI_RESID, (int)groups.size() - 1, L.s_down, 0.f);
    }
    stage_first.push_back((int)ops.size());
    if (engine_smem_bytes((int)groups.size(), (int)ops.size(), (int)stage_first.size() - 1, (int)attn.size()) == 0)
        return SLLM_CUDA_OK;       // too many layers for the tables: the per-GEMV step
    g_engine_eps = m->eps;
    const int rc = engine_program_build(c->eng_decode, groups, ops, stage_first, m->device, c->stream, fb,
                                        engine_wpl(E), engine_wpl(F), &attn, false);
    c->eng_decode.params.kv16 = c->kv_f16;     // the instance whose attention reads f16 caches
    return rc;
}

// ---------------------------------------------------------------------------
// the layer projection chain (benchmark configuration 1)
// ---------------------------------------------------------------------------
// The chain as an engine program: per layer four stages (Q/K/V, O, gate/up,
// down), each behind a grid barrier because its input is the whole output of
// the stage before.
static int chain_program(const sllm_cuda_model* m, sllm_cuda_ctx* c, int begin, int n, float* x, int* fb) {
    const int E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa;
    std::vector<EngGroup> groups;
    std::vector<EngOp> ops;
    std::vector<int> stage_first;
    auto op = [&](const uint8_t* w, const uint8_t* w2, float* y, const float* resid, float* h, int rows, int K,
                  int epi, int group, float ws, float ws2) {
        EngOp o{};
        o.w = w; o.w2 = w2; o.y = y; o.resid = resid; o.h = h; o.rows = rows; o.K = K; o.epi = epi; o.group = group;
        o.chunk_rows = engine_chunk_rows(K, epi);
        o.ws = ws; o.ws2 = ws2;
        ops.push_back(o);
    };
    for (int l = begin; l < begin + n; ++l) {
        const DevLayer& L = m->layers[l];
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{x, L.attn_norm, E, PRO_NORM});
        op(L.wq, nullptr, c->q, nullptr, nullptr, E, E, EPI_F32, (int)groups.size() - 1, L.s_wq, 0.f);
        op(L.wk, nullptr, c->k, nullptr, nullptr, G, E, EPI_F32, (int)groups.size() - 1, L.s_wk, 0.f);
        op(L.wv, nullptr, c->v, nullptr, nullptr, G, E, EPI_F32, (int)groups.size() - 1, L.s_wv, 0.f);
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->q, L.attn_sub_norm, E, PRO_NORM});
        op(L.wo, nullptr, c->ffn_inp, x, nullptr, E, E, EPI_RESID, (int)groups.size() - 1, L.s_wo, 0.f);
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->ffn_inp, L.ffn_norm, E, PRO_NORM});
        op(L.gate, L.up, nullptr, nullptr, c->h, F, E, EPI_SILU, (int)groups.size() - 1, L.s_gate, L.s_up);
        stage_first.push_back((int)ops.size());
        groups.push_back(EngGroup{c->h, L.ffn_sub_norm, F, PRO_NORM});
        op(L.down, nullptr, x, c->ffn_inp, nullptr, E, F, EPI_RESID, (int)groups.size() - 1, L.s_down, 0.f);
    }
    stage_first.push_back((int)ops.size());
    g_engine_eps = m->eps;
    return engine_program_build(c->eng_chain, groups, ops, stage_first, m->device, c->stream, fb,
                                engine_wpl(E), engine_wpl(F));
}

// A program's error word after its launches have completed: a bounded wait
// that gave up is reported once and the word cleared, so the context's next
// call starts clean.
static int engine_error(const EngineProgram& p) {
    int err = 0;
    if (p.error != nullptr && cudaMemcpy(&err, p.error, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && err != 0) {
        cudaMemset(p.error, 0, sizeof(int));
        return fail(SLLM_CUDA_ERR_TIMEOUT, "engine: a bounded device wait gave up (code %d)", err);
    }
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_layer_chain_device(const sllm_cuda_model* m, sllm_cuda_ctx* c, int32_t layer_begin,
                                            int32_t n_layers, float* x, void* stream) {
    if (m == nullptr || c == nullptr || x == nullptr || c->m != m || layer_begin < 0 || n_layers < 0 ||
        layer_begin + n_layers > m->n_layer || !aligned16(x))
        return fail(SLLM_CUDA_ERR_ARG, "layer_chain: bad arguments");
    if (n_layers == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    int* fb = fallback_counter();
    if (fb == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "layer_chain: diagnostics counter");
    if (!engine_supports(engine_wpl(m->n_embd), engine_wpl(m->n_ff))) {
        // widths the engine is not compiled for: one fused GEMV launch per
        // projection, programmatically chained, captured as a graph
        if (c->chain == nullptr || c->chain_begin != layer_begin || c->chain_n != n_layers || c->chain_x != x) {
            graph_exec_destroy(c->chain); c->chain = nullptr;
            ChainBufs b{x, c->q, c->k, c->v, c->ffn_inp, c->h, nullptr};
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
            cudaError_t e = cudaSuccess;
            for (int l = layer_begin; l < layer_begin + n_layers && e == cudaSuccess; ++l)
                e = launch_layer(m, l, b, fb, g_force_fallback, c->stream, false, nullptr);
            cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
            if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); return cuda_fail(e, "capture layer chain"); }
            if (e2 != cudaSuccess) return cuda_fail(e2, "end capture");
            e = instantiate(&c->chain, g);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) { c->chain = nullptr; return cuda_fail(e, "instantiate layer chain"); }
            c->chain_begin = layer_begin; c->chain_n = n_layers; c->chain_x = x;
        }
        CK(graph_launch(c->chain, (cudaStream_t)stream), "layer chain");
        return SLLM_CUDA_OK;
    }
    EngineProgram& p = c->eng_chain;
    if (!p.built || p.key_begin != layer_begin || p.key_n != n_layers || p.key_x != x) {
        int rc = chain_program(m, c, layer_begin, n_layers, x, fb);
        if (rc != SLLM_CUDA_OK) return rc;
        p.key_begin = layer_begin; p.key_n = n_layers; p.key_x = x;
    }
    CK(engine_program_launch(p, (cudaStream_t)stream), "layer chain");
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_layer_chain(const sllm_cuda_model* m, sllm_cuda_ctx* c, int32_t layer_begin,
                                     int32_t n_layers, const float* x_in, float* x_out) {
    if (m == nullptr || c == nullptr || x_in == nullptr || x_out == nullptr || c->m != m)
        return fail(SLLM_CUDA_ERR_ARG, "layer_chain: bad arguments");
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    const size_t bytes = (size_t)m->n_embd * 4;
    CK(cudaMemcpyAsync(c->x, x_in, bytes, cudaMemcpyHostToDevice, c->stream), "chain input");
    int rc = sllm_cuda_layer_chain_device(m, c, layer_begin, n_layers, c->x, c->stream);
    if (rc != SLLM_CUDA_OK) return rc;
    CK(cudaMemcpyAsync(x_out, c->x, bytes, cudaMemcpyDeviceToHost, c->stream), "chain output");
    CK(cudaStreamSynchronize(c->stream), "chain sync");
    return engine_error(c->eng_chain);
}

// ---------------------------------------------------------------------------
// the seven projections of a layer on independent inputs (configuration 1 as
// the benchmark states it: each GEMV has its own f32 activation, RMSNorm'd
// with its layer norm and quantised per token)
// ---------------------------------------------------------------------------
extern "C" size_t sllm_cuda_layer_projections_sizes(const sllm_cuda_model* m, size_t* y_floats_per_layer) {
    if (m == nullptr) return 0;
    const size_t E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa;
    if (y_floats_per_layer) *y_floats_per_layer = 3 * E + 2 * G + 2 * F;
    return 6 * E + F;
}

// The seven projections of a layer as seven independent fused GEMV launches
// (the fallback for widths the engine is not compiled for).
static cudaError_t launch_projections(const sllm_cuda_model* m, int l, const float* x, float* y, int* fb,
                                      cudaStream_t st) {
    const DevLayer& L = m->layers[l];
    const int E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa, sms = num_sms_of(m->device);
    struct P { const uint8_t* w; int rows; int K; const float* norm; size_t xoff; size_t yoff; };
    const P ps[7] = {
        {L.wq, E, E, L.attn_norm, 0 * (size_t)E, 0},
        {L.wk, G, E, L.attn_norm, 1 * (size_t)E, (size_t)E},
        {L.wv, G, E, L.attn_norm, 2 * (size_t)E, (size_t)E + G},
        {L.wo, E, E, L.attn_sub_norm, 3 * (size_t)E, (size_t)E + 2 * G},
        {L.gate, F, E, L.ffn_norm, 4 * (size_t)E, 2 * (size_t)E + 2 * G},
        {L.up, F, E, L.ffn_norm, 5 * (size_t)E, 2 * (size_t)E + 2 * G + F},
        {L.down, E, F, L.ffn_sub_norm, 6 * (size_t)E, 2 * (size_t)E + 2 * G + 2 * (size_t)F},
    };
    for (const P& q : ps) {
        GemvParams p{};
        p.K = q.K;
        p.nseg = 1;
        p.seg[0] = GemvSeg{q.w, q.rows, y + q.yoff, nullptr};
        p.x = x + q.xoff;
        p.norm_w = q.norm;
        p.eps = m->eps;
        p.fallback_count = fb;
        p.force_fallback = g_force_fallback;
        cudaError_t e = launch_gemv(p, PRO_NORM, EPI_F32, sms, st, GEMV_INDEPENDENT);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// The seven projections of each layer as one engine stage: every GEMV has its
// own input, so nothing waits for anything and the weights stream back to back.
static int projections_program(const sllm_cuda_model* m, sllm_cuda_ctx* c, EngineProgram& prog, int begin, int n,
                               const float* x, float* y, int* fb) {
    const int E = m->n_embd, F = m->n_ff, G = m->n_embd_gqa;
    size_t ystride = 0;
    sllm_cuda_layer_projections_sizes(m, &ystride);
    std::vector<EngGroup> groups;
    std::vector<EngOp> ops;
    for (int l = 0; l < n; ++l) {
        const DevLayer& L = m->layers[begin + l];
        float* yl = y + (size_t)l * ystride;
        struct P { const uint8_t* w; int rows; int K; const float* norm; size_t xoff; size_t yoff; float ws; };
        const P ps[7] = {
            {L.wq, E, E, L.attn_norm, 0 * (size_t)E, 0, L.s_wq},
            {L.wk, G, E, L.attn_norm, 1 * (size_t)E, (size_t)E, L.s_wk},
            {L.wv, G, E, L.attn_norm, 2 * (size_t)E, (size_t)E + G, L.s_wv},
            {L.wo, E, E, L.attn_sub_norm, 3 * (size_t)E, (size_t)E + 2 * G, L.s_wo},
            {L.gate, F, E, L.ffn_norm, 4 * (size_t)E, 2 * (size_t)E + 2 * G, L.s_gate},
            {L.up, F, E, L.ffn_norm, 5 * (size_t)E, 2 * (size_t)E + 2 * G + F, L.s_up},
            {L.down, E, F, L.ffn_sub_norm, 6 * (size_t)E, 2 * (size_t)E + 2 * G + 2 * (size_t)F, L.s_down},
        };
        for (const P& q : ps) {
            groups.push_back(EngGroup{x + q.xoff, q.norm, q.K, PRO_NORM});
            EngOp o{};
            o.w = q.w; o.y = yl + q.yoff; o.rows = q.rows; o.K = q.K; o.epi = EPI_F32; o.ws = q.ws;
            o.group = (int)groups.size() - 1;
            o.chunk_rows = engine_chunk_rows(q.K, EPI_F32);
            ops.push_back(o);
        }
    }
    std::vector<int> stage_first{0, (int)ops.size()};
    g_engine_eps = m->eps;
    return engine_program_build(prog, groups, ops, stage_first, m->device, c->stream, fb,
                                engine_wpl(E), engine_wpl(F));
}

extern "C" int sllm_cuda_layer_projections_device(const sllm_cuda_model* m, sllm_cuda_ctx* c, int32_t layer_begin,
                                                  int32_t n_layers, const float* x, float* y, void* stream) {
    if (m == nullptr || c == nullptr || x == nullptr || y == nullptr || c->m != m || layer_begin < 0 ||
        n_layers < 0 || layer_begin + n_layers > m->n_layer || !aligned16(x) || !aligned16(y))
        return fail(SLLM_CUDA_ERR_ARG, "layer_projections: bad arguments");
    if (n_layers == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    int* fb = fallback_counter();
    if (fb == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "layer_projections: diagnostics counter");
    if (!engine_supports(engine_wpl(m->n_embd), engine_wpl(m->n_ff))) {
        size_t ystride = 0;
        sllm_cuda_layer_projections_sizes(m, &ystride);
        if (c->proj == nullptr || c->proj_begin != layer_begin || c->proj_n != n_layers || c->proj_x != x ||
            c->proj_y != y) {
            graph_exec_destroy(c->proj); c->proj = nullptr;
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
            cudaError_t e = cudaSuccess;
            for (int l = 0; l < n_layers && e == cudaSuccess; ++l)
                e = launch_projections(m, layer_begin + l, x, y + (size_t)l * ystride, fb, c->stream);
            cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
            if (e != cudaSuccess) { if (g) cudaGraphDestroy(g); return cuda_fail(e, "capture projections"); }
            if (e2 != cudaSuccess) return cuda_fail(e2, "end capture");
            e = instantiate(&c->proj, g);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) { c->proj = nullptr; return cuda_fail(e, "instantiate projections"); }
            c->proj_begin = layer_begin; c->proj_n = n_layers; c->proj_x = x; c->proj_y = y;
        }
        CK(graph_launch(c->proj, (cudaStream_t)stream), "projections");
        return SLLM_CUDA_OK;
    }
    EngineProgram& p = c->eng_proj;
    if (!p.built || p.key_begin != layer_begin || p.key_n != n_layers || p.key_x != x || p.key_y != y) {
        int rc = projections_program(m, c, p, layer_begin, n_layers, x, y, fb);
        if (rc != SLLM_CUDA_OK) return rc;
        p.key_begin = layer_begin; p.key_n = n_layers; p.key_x = x; p.key_y = y;
    }
    CK(engine_program_launch(p, (cudaStream_t)stream), "projections");
    return SLLM_CUDA_OK;
}

// Where the host-buffer projections split into two pieces; 0 = run as one.
// The first piece's outputs go back to the host on the copy stream while the
// second piece computes, so only the second piece's copy is exposed. It is
// made just large enough that the first piece's copy (host link, ~54 GB/s
// measured) hides behind its compute (weights streamed at ~5.6 TB/s). Every
// piece boundary costs about 11 us of engine tail and ramp, more than a
// third piece would save, and below 16 layers more than the split saves.
static int projection_split_widths(int n_embd, int n_ff, int n_embd_gqa, int n_layers) {
    if (!engine_supports(engine_wpl(n_embd), engine_wpl(n_ff)) || n_layers < 16) return 0;
    const double E = n_embd, F = n_ff, G = n_embd_gqa;
    const double weight_bytes = (2.0 * E * E + 2.0 * G * E + 3.0 * E * F) / 4.0;   // 2-bit codes of a layer
    const double out_bytes = 4.0 * (3.0 * E + 2.0 * G + 2.0 * F);                  // f32 outputs of a layer
    const double copy_s = out_bytes / 54e9, compute_s = weight_bytes / 5.6e12;
    int last = (int)std::ceil(copy_s / (copy_s + compute_s) * n_layers);
    last = std::max(1, std::min(last, n_layers / 2));
    return n_layers - last;
}

static int projection_split(const sllm_cuda_model* m, int n_layers) {
    return projection_split_widths(m->n_embd, m->n_ff, m->n_embd_gqa, n_layers);
}

extern "C" int sllm_cuda_test_projection_split(int32_t n_embd, int32_t n_ff, int32_t n_embd_gqa,
                                               int32_t n_layers) {
    if (n_embd < 1 || n_ff < 1 || n_embd_gqa < 1 || n_layers < 0) return -1;
    return projection_split_widths(n_embd, n_ff, n_embd_gqa, n_layers);
}

static int projections_in_pieces(const sllm_cuda_model* m, sllm_cuda_ctx* c, int begin, int n, int split,
                                 const float* dx, float* dy, float* y_host, size_t ystride) {
    const int bound[kProjPieces + 1] = {0, split, n};
    const int pieces = kProjPieces;
    if (c->copy_stream == nullptr) {     // created last: a stream means the events exist
        for (int i = 0; i < kProjPieces; ++i)
            if (c->piece_done[i] == nullptr)
                CK(cudaEventCreateWithFlags(&c->piece_done[i], cudaEventDisableTiming), "piece events");
        CK(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking), "copy stream");
    }
    int* fb = fallback_counter();
    if (fb == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "layer_projections: diagnostics counter");
    for (int i = 0; i < pieces; ++i) {
        const int lo = bound[i], hi = bound[i + 1];
        EngineProgram& p = c->eng_piece[i];
        float* y = dy + (size_t)lo * ystride;
        if (!p.built || p.key_begin != begin + lo || p.key_n != hi - lo || p.key_x != dx || p.key_y != y) {
            const int rc = projections_program(m, c, p, begin + lo, hi - lo, dx, y, fb);
            if (rc != SLLM_CUDA_OK) return rc;
            p.key_begin = begin + lo; p.key_n = hi - lo; p.key_x = dx; p.key_y = y;
        }
        if (p.exec != nullptr) return fail(SLLM_CUDA_ERR_ARG, "layer_projections: a piece needs one stage");
    }
    // every piece reports a gave-up wait into the first piece's error word,
    // which comes back behind the last copy
    int* err = c->eng_piece[0].error;
    for (int i = 0; i < pieces; ++i) {
        const EngineProgram& p = c->eng_piece[i];
        EngParams ep = p.params;
        ep.error = err;
        CK(launch_engine(ep, p.grid, c->stream, p.wa, p.wb), "projections piece");
        count_launches(1);
        CK(cudaEventRecord(c->piece_done[i], c->stream), "piece event");
    }
    for (int i = 0; i < pieces; ++i) {
        const int lo = bound[i], hi = bound[i + 1];
        CK(cudaStreamWaitEvent(c->copy_stream, c->piece_done[i], 0), "piece wait");
        CK(cudaMemcpyAsync(y_host + (size_t)lo * ystride, dy + (size_t)lo * ystride, (size_t)(hi - lo) * ystride * 4,
                           cudaMemcpyDeviceToHost, c->copy_stream), "projection outputs");
    }
    int32_t* err_host = &c->pinned[8];
    CK(cudaMemcpyAsync(err_host, err, sizeof(int), cudaMemcpyDeviceToHost, c->copy_stream), "engine status");
    CK(cudaStreamSynchronize(c->copy_stream), "projections sync");
    if (*err_host != 0)
        return fail(SLLM_CUDA_ERR_TIMEOUT, "engine: a bounded device wait gave up (code %d)", (int)*err_host);
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_layer_projections(const sllm_cuda_model* m, sllm_cuda_ctx* c, int32_t layer_begin,
                                           int32_t n_layers, const float* x_host, float* y_host) {
    if (m == nullptr || c == nullptr || x_host == nullptr || y_host == nullptr || c->m != m || n_layers < 0 ||
        layer_begin < 0 || layer_begin + n_layers > m->n_layer)
        return fail(SLLM_CUDA_ERR_ARG, "layer_projections: bad arguments");
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    size_t ystride = 0;
    const size_t xn = sllm_cuda_layer_projections_sizes(m, &ystride);
    const size_t xbytes = xn * 4, ybytes = ystride * 4 * (size_t)n_layers;
    if (c->io_cap < xbytes + ybytes) {
        cudaFree(c->io);
        c->io = nullptr;
        c->io_cap = 0;
        CK(cudaMalloc(&c->io, xbytes + ybytes), "projection buffers");
        c->io_cap = xbytes + ybytes;
    }
    float* dx = (float*)c->io;
    float* dy = (float*)((uint8_t*)c->io + ((xbytes + 255) & ~(size_t)255));
    if (((xbytes + 255) & ~(size_t)255) + ybytes > c->io_cap) {
        cudaFree(c->io);
        c->io = nullptr;
        c->io_cap = 0;
        CK(cudaMalloc(&c->io, xbytes + ybytes + 256), "projection buffers");
        c->io_cap = xbytes + ybytes + 256;
        dx = (float*)c->io;
        dy = (float*)((uint8_t*)c->io + ((xbytes + 255) & ~(size_t)255));
    }
    CK(cudaMemcpyAsync(dx, x_host, xbytes, cudaMemcpyHostToDevice, c->stream), "projection inputs");
    const int split = projection_split(m, n_layers);
    if (split > 0) return projections_in_pieces(m, c, layer_begin, n_layers, split, dx, dy, y_host, ystride);
    int rc = sllm_cuda_layer_projections_device(m, c, layer_begin, n_layers, dx, dy, c->stream);
    if (rc != SLLM_CUDA_OK) return rc;
    CK(cudaMemcpyAsync(y_host, dy, ybytes, cudaMemcpyDeviceToHost, c->stream), "projection outputs");
    if (c->eng_proj.built && n_layers > 0) {
        // the engine's status word comes back behind the outputs: one wait
        int32_t* err_host = &c->pinned[8];
        CK(cudaMemcpyAsync(err_host, c->eng_proj.error, sizeof(int), cudaMemcpyDeviceToHost, c->stream),
           "engine status");
        CK(cudaStreamSynchronize(c->stream), "projections sync");
        if (*err_host != 0)
            return fail(SLLM_CUDA_ERR_TIMEOUT, "engine: a bounded device wait gave up (code %d)", (int)*err_host);
        return SLLM_CUDA_OK;
    }
    CK(cudaStreamSynchronize(c->stream), "projections sync");
    return engine_error(c->eng_proj);
}

// ---------------------------------------------------------------------------
// A batch of independent GEMVs of one shape as one persistent engine launch.
// ---------------------------------------------------------------------------
struct sllm_cuda_gemv_batch {
    int device = 0;
    int rows = 0, K = 0, count = 0, wa = 0, wb = 0;
    std::vector<const uint8_t*> w;
    std::vector<float> ws;
    EngineProgram prog;
    size_t key_stride = 0;
};

extern "C" int sllm_cuda_gemv_batch_new(const uint8_t* const* w, size_t count, size_t n_rows, size_t n, int device,
                                        sllm_cuda_gemv_batch** out) {
    if (out == nullptr) return fail(SLLM_CUDA_ERR_ARG, "gemv_batch_new: NULL out");
    *out = nullptr;
    if (w == nullptr || count == 0 || count > 256) return fail(SLLM_CUDA_ERR_ARG, "gemv_batch_new: count %zu outside [1, 256]", count);
    int rc = check_gemv_shape(w[0], n_rows, n, w[0]);
    if (rc != SLLM_CUDA_OK) return rc;
    for (size_t i = 0; i < count; ++i)
        if (w[i] == nullptr || !aligned16(w[i])) return fail(SLLM_CUDA_ERR_ARG, "gemv_batch_new: tensor %zu NULL or unaligned", i);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "gemv_batch_new: no device %d", device);
    }
    CK(cudaSetDevice(device), "cudaSetDevice");
    auto* b = new sllm_cuda_gemv_batch();
    b->device = device;
    b->rows = (int)n_rows;
    b->K = (int)n;
    b->count = (int)count;
    if (!engine_pair_for_width(engine_wpl(b->K), &b->wa, &b->wb)) {
        delete b;
        return fail(SLLM_CUDA_ERR_UNSUPPORTED, "gemv_batch_new: no engine instance for width %zu", n);
    }
    b->w.assign(w, w + count);
    b->ws.resize(count);
    for (size_t i = 0; i < count; ++i) {
        // the per-tensor scale after the packed codes (src/quant.c:102-106)
        const cudaError_t e = cudaMemcpy(&b->ws[i], w[i] + n_rows * (n / 4), 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) { delete b; return cuda_fail(e, "gemv_batch_new: read scale"); }
    }
    *out = b;
    return SLLM_CUDA_OK;
}

extern "C" void sllm_cuda_gemv_batch_free(sllm_cuda_gemv_batch* b) {
    if (b == nullptr) return;
    cudaSetDevice(b->device);
    engine_program_free(b->prog);
    delete b;
}

extern "C" int sllm_cuda_gemv_batch_run(sllm_cuda_gemv_batch* b, const float* x, size_t x_stride, float* y,
                                        void* stream) {
    if (b == nullptr || x == nullptr || y == nullptr || !aligned16(x) || !aligned16(y) ||
        (x_stride != 0 && (x_stride < (size_t)b->K || x_stride % 4 != 0)) || b->rows % 4 != 0)
        return fail(SLLM_CUDA_ERR_ARG, "gemv_batch_run: bad arguments");
    CK(cudaSetDevice(b->device), "cudaSetDevice");
    EngineProgram& p = b->prog;
    if (!p.built || p.key_x != x || p.key_y != y || b->key_stride != x_stride) {
        int* fb = fallback_counter();
        if (fb == nullptr) return fail(SLLM_CUDA_ERR_NOMEM, "gemv_batch_run: diagnostics counter");
        std::vector<EngGroup> groups;
        std::vector<EngOp> ops;
        for (int i = 0; i < b->count; ++i) {
            if (i == 0 || x_stride != 0)
                groups.push_back(EngGroup{x + (size_t)i * x_stride, nullptr, b->K, PRO_QUANT});
            EngOp o{};
            o.w = b->w[i]; o.y = y + (size_t)i * b->rows; o.rows = b->rows; o.K = b->K; o.epi = EPI_F32;
            o.ws = b->ws[i]; o.group = (int)groups.size() - 1;
            o.chunk_rows = engine_chunk_rows(b->K, EPI_F32);
            ops.push_back(o);
        }
        std::vector<int> stage_first{0, (int)ops.size()};
        g_engine_eps = 0.0f;            // PRO_QUANT: no norm
        const int rc = engine_program_build(p, groups, ops, stage_first, b->device, nullptr, fb, b->wa, b->wb);
        if (rc != SLLM_CUDA_OK) return rc;
        p.key_x = x; p.key_y = y; b->key_stride = x_stride;
    }
    CK(engine_program_launch(p, (cudaStream_t)stream), "gemv_batch launch");
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_test_gemv_batch_error(sllm_cuda_gemv_batch* b) {
    if (b == nullptr || !b->prog.built) return -1;
    if (cudaSetDevice(b->device) != cudaSuccess) return -1;
    return engine_error(b->prog);
}

// ---------------------------------------------------------------------------
// The layer chain with no allocation at all.
//
// For callers that must not allocate device memory: code recording into a
// CUDA graph under a strict capture mode (cudaMalloc is illegal while the
// stream captures), hosts whose own allocator has already reserved the
// device's memory (a late cudaMalloc fails or fragments it), and real-time
// loops that cannot afford cudaMalloc's implicit device synchronisation. They
// have a model but no context, so the chain's five scratch vectors (q, k, v,
// ffn_inp: n_embd / n_embd_gqa floats; h: n_ff floats) live in this file-scope
// device array instead of a context. The array is loaded with the library and
// every device that loads it holds it until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchFloats = 32768;   // 128 KB: 2*n_embd + 2*n_embd_gqa + n_ff must fit
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// The array's device address, looked up once per device with that device
// current (the host-side symbol is only a stand-in and must never reach a
// kernel). The first call on a device does this lookup.
static int noalloc_scratch(int dev, float** out) {
    static std::mutex mu;
    static std::vector<float*> ptrs;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)ptrs.size() <= dev) ptrs.resize(dev + 1, nullptr);
    if (ptrs[dev] == nullptr) {
        float* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void**)&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "layer_chain_noalloc: cudaGetSymbolAddress");
        ptrs[dev] = p;
    }
    *out = ptrs[dev];
    return SLLM_CUDA_OK;
}

extern "C" int sllm_cuda_layer_chain_device_noalloc(const sllm_cuda_model* m, int32_t layer_begin,
                                                    int32_t n_layers, float* x, void* stream) {
    if (m == nullptr || x == nullptr || layer_begin < 0 || n_layers < 0 || layer_begin + n_layers > m->n_layer ||
        !aligned16(x))
        return fail(SLLM_CUDA_ERR_ARG, "layer_chain_noalloc: bad arguments");
    const size_t E = m->n_embd, G = m->n_embd_gqa, F = m->n_ff;
    const size_t need = 2 * E + 2 * G + F;
    if (need > kNoAllocScratchFloats)
        return fail(SLLM_CUDA_ERR_TOO_LARGE,
                    "layer_chain_noalloc: the model needs %zu scratch floats (2*n_embd + 2*n_embd_gqa + n_ff); "
                    "the static scratch holds %zu", need, kNoAllocScratchFloats);
    if (n_layers == 0) return SLLM_CUDA_OK;
    CK(cudaSetDevice(m->device), "cudaSetDevice");
    float* s = nullptr;
    int rc = noalloc_scratch(m->device, &s);
    if (rc != SLLM_CUDA_OK) return rc;
    // every scratch vector is written before it is read within one call
    // (Q/K/V -> q, k, v; O -> ffn_inp; gate/up -> h), so nothing is cleared
    ChainBufs b{x, s, s + E, s + E + G, s + E + 2 * G, s + 2 * E + 2 * G, nullptr};
    // the fallback counter stays null (the kernels skip a null counter); the
    // forced-fallback test switch is a host int and is honoured as elsewhere
    for (int l = layer_begin; l < layer_begin + n_layers; ++l) {
        CK(launch_layer(m, l, b, nullptr, g_force_fallback, (cudaStream_t)stream, false, nullptr),
           "layer_chain_noalloc");
        g_kernel_launches += 4;
    }
    return SLLM_CUDA_OK;
}
