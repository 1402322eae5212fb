/*
 * A C11 caller of the library, as saphira-llm's own C host code would be:
 * it includes only the public and testing headers, links libsllm_cuda.so,
 * and exercises the calls that need no device -- status strings, argument
 * errors, and the host-side plans (engine work split, tensor-parallel shard,
 * host-buffer projection pieces). Prints "ok" and exits 0 when every check
 * holds; otherwise prints the failed check and exits 1.
 */
#include <stdio.h>
#include <string.h>

#include "sllm_cuda.h"
#include "sllm_cuda_testing.h"

static int failures = 0;

#define CHECK(cond)                                                   \
    do {                                                              \
        if (!(cond)) {                                                \
            fprintf(stderr, "failed: %s (line %d)\n", #cond, __LINE__); \
            ++failures;                                               \
        }                                                             \
    } while (0)

int main(void) {
    sllm_cuda_model* model = NULL;
    int32_t plan[8];
    const int32_t rows[2] = {2560, 640}, K[2] = {2560, 2560}, epi[2] = {1, 1}, group[2] = {0, 1};
    const int32_t stage_first[2] = {0, 2};
    int32_t cursors[2 * 5];

    CHECK(strcmp(sllm_cuda_status_string(SLLM_CUDA_ERR_TIMEOUT), "device wait timed out") == 0);
    CHECK(sllm_cuda_model_upload(NULL, 0, &model) == SLLM_CUDA_ERR_ARG && model == NULL);
    CHECK(strstr(sllm_cuda_last_error(), "model_upload") != NULL);

    /* configs[4] (80 layers, 8192 wide, 64/8 heads, 28672 FFN) on rank 3 of 8 */
    CHECK(sllm_cuda_test_tp_plan(80, 8192, 28672, 64, 8, 128256, 8, 3, plan) == SLLM_CUDA_OK);
    CHECK(plan[0] == 8 && plan[1] == 1 && plan[2] == 1024 && plan[3] == 3584);
    CHECK(plan[4] * plan[5] == 3584 && plan[6] == 3 * 16032 && plan[7] == 16032);
    CHECK(sllm_cuda_test_tp_plan(30, 2560, 6912, 20, 5, 128256, 2, 0, plan) == SLLM_CUDA_ERR_UNSUPPORTED);

    /* two ops of one stage over four CTAs: the first starts at row 0, the last ends past the ops */
    CHECK(sllm_cuda_test_engine_split(rows, K, epi, group, 2, stage_first, 1, 4, cursors) == SLLM_CUDA_OK);
    CHECK(cursors[0] == 0 && cursors[1] == 0 && cursors[8] == 2 && cursors[9] == 0);

    CHECK(sllm_cuda_test_projection_split(2560, 6912, 640, 32) == 20);
    CHECK(sllm_cuda_test_projection_split(2560, 6912, 640, 8) == 0);

    if (failures != 0) return 1;
    puts("ok");
    return 0;
}
