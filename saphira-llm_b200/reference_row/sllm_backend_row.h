/*
 * sllm_backend_row.h -- the CUDA row of saphira-llm's dispatch, on the
 * reference's side of the boundary.
 *
 * saphira-llm's dispatch (include/saphira_llm/dispatch.h) decides from
 * measured evidence WHETHER a model may execute, and refuses explicitly when
 * it may not. The backend rows add WHERE it executes, under the same
 * contract: a measured capability, an exact selection, an explicit refusal,
 * and no fallback once a row is selected.
 *
 *   CPU row   always executable (the reference's own kernels).
 *   CUDA row  executable when the architecture evidence resolves to
 *             SLLM_PROFILE_DENSE_ATTENTION, libsllm_cuda.so reports a device
 *             of compute capability 10.x, and the widths are ones that
 *             library runs (head dim 128, n_embd and n_ff multiples of 128 up
 *             to 8192).
 *
 * The row is chosen when a model is loaded (sllm_model_load). The request
 * comes from sllm_backend_request() (the CLI's --backend flag) or else from
 * the environment variable SAPHIRA_LLM_BACKEND: "cpu" (the default), "cuda"
 * (refuse to load when the CUDA row is not executable) or "auto" (the CUDA row
 * when it is executable, else the CPU row). SAPHIRA_LLM_CUDA_DEVICE picks the
 * device (default 0).
 *
 * This header and sllm_backend_row.c are compiled into the reference library
 * beside the two insertion-only patches (forward.c.patch, dispatch.c.patch).
 */
#ifndef SLLM_BACKEND_ROW_H
#define SLLM_BACKEND_ROW_H

#include <saphira_llm/dispatch.h>
#include <saphira_llm/status.h>

#include <stdint.h>

#include "sllm_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    SLLM_BACKEND_CPU = 0,
    SLLM_BACKEND_CUDA = 1,
    SLLM_BACKEND_AUTO = 2
} sllm_backend;

/* Parse "cpu", "cuda" or "auto"; SLLM_ERR_ARG for anything else. */
sllm_status sllm_backend_parse(const char * s, sllm_backend * out);

/* Override the environment for the rest of the process (the CLI flag). */
void sllm_backend_request(sllm_backend b);

/* The row asked for: the override, else SAPHIRA_LLM_BACKEND, else CPU. */
sllm_backend sllm_backend_requested(void);

/* The CUDA device the CUDA row uses (SAPHIRA_LLM_CUDA_DEVICE, default 0). */
int sllm_backend_cuda_device(void);

/* The measured device capability: SLLM_OK when libsllm_cuda.so sees a device
 * of compute capability 10.x; otherwise its status, with `reason` filled. */
sllm_status sllm_backend_cuda_capability(char * reason, size_t cap);

/*
 * The dispatch question for a backend (src/dispatch.c, after
 * sllm_dispatch_resolve): may `requested` execute a model with this evidence
 * and these widths? SLLM_DISPATCH_EXECUTABLE with the row in *row_out, or
 * SLLM_DISPATCH_REFUSED with ev->reason saying why. "auto" resolves to the
 * CUDA row when it is executable and to the CPU row otherwise.
 */
sllm_dispatch_result sllm_dispatch_resolve_backend(sllm_arch_evidence * ev, sllm_backend requested,
                                                   int32_t n_embd, int32_t n_ff, int32_t head_dim,
                                                   sllm_backend * row_out);

/* The row a loaded model runs on (forward.c, added by forward.c.patch). */
struct sllm_model;
sllm_backend sllm_model_backend(const struct sllm_model * m);

#ifdef __cplusplus
}
#endif

#endif /* SLLM_BACKEND_ROW_H */
