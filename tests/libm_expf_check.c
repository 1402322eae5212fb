/* Checks saphira-llm_b200/csrc/libm_expf.h against the host libm's expf over
 * every one of the 2^32 float bit patterns (tests/test_libm_expf.py builds and
 * runs it). Exit status 0 and "mismatch 0" when every result is bit-identical. */
#include <stdio.h>
#include <stdint.h>
#include <math.h>
#include <string.h>
#include "../saphira-llm_b200/csrc/libm_expf.h"

int main(void) {
    unsigned long long bad = 0;
    uint32_t first = 0;
    #pragma omp parallel for reduction(+:bad) schedule(static, 65536)
    for (long long i = 0; i < 4294967296LL; ++i) {
        uint32_t u = (uint32_t) i;
        float x;
        memcpy(&x, &u, 4);
        volatile float xv = x;
        float a = expf(xv), b = sllm_libm_expf(xv);
        uint32_t ua, ub;
        memcpy(&ua, &a, 4);
        memcpy(&ub, &b, 4);
        if (ua != ub && !(isnan(a) && isnan(b))) {
            bad++;
            if (!first) { first = u; }
        }
    }
    printf("mismatch %llu first %08x\n", bad, first);
    return bad != 0;
}
