/*
 * sllm_backend_row.c -- how the CUDA row is requested and how its capability
 * is measured (see sllm_backend_row.h). Plain C11, compiled with the
 * reference's own flags into the reference library.
 */
#include "sllm_backend_row.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int g_override = -1;     /* -1: none; else an sllm_backend */

sllm_status sllm_backend_parse(const char * s, sllm_backend * out) {
    if (s == NULL || out == NULL) { return SLLM_ERR_ARG; }
    if (strcmp(s, "cpu") == 0)  { *out = SLLM_BACKEND_CPU;  return SLLM_OK; }
    if (strcmp(s, "cuda") == 0) { *out = SLLM_BACKEND_CUDA; return SLLM_OK; }
    if (strcmp(s, "auto") == 0) { *out = SLLM_BACKEND_AUTO; return SLLM_OK; }
    return SLLM_ERR_ARG;
}

void sllm_backend_request(sllm_backend b) { g_override = (int) b; }

sllm_backend sllm_backend_requested(void) {
    if (g_override >= 0) { return (sllm_backend) g_override; }
    sllm_backend b = SLLM_BACKEND_CPU;
    const char * e = getenv("SAPHIRA_LLM_BACKEND");
    if (e != NULL && e[0] != '\0' && sllm_backend_parse(e, &b) != SLLM_OK) {
        /* an unknown request is not silently read as the CPU: it is refused
         * at load, where the caller sees a status */
        return (sllm_backend) -1;
    }
    return b;
}

int sllm_backend_cuda_device(void) {
    const char * e = getenv("SAPHIRA_LLM_CUDA_DEVICE");
    return (e != NULL && e[0] != '\0') ? atoi(e) : 0;
}

sllm_status sllm_backend_cuda_capability(char * reason, size_t cap) {
    int n = 0, major = 0, minor = 0;
    const int rc = sllm_cuda_probe(&n, &major, &minor);
    if (rc != SLLM_CUDA_OK) {
        if (reason != NULL && cap > 0) {
            snprintf(reason, cap, "CUDA row: no device of compute capability 10.x (%s: %s)",
                     sllm_cuda_status_string(rc), sllm_cuda_last_error());
        }
        return (sllm_status) rc;
    }
    const int dev = sllm_backend_cuda_device();
    if (dev < 0 || dev >= n) {
        if (reason != NULL && cap > 0) {
            snprintf(reason, cap, "CUDA row: device %d requested, %d present", dev, n);
        }
        return SLLM_ERR_UNSUPPORTED;
    }
    return SLLM_OK;
}
