/* host_model_sanitize.c - loads GGUF files through the library's host
 * runtime (lmc_b200/host/lmc_model.c, built with AddressSanitizer and
 * UndefinedBehaviorSanitizer by tests/test_host_model_sanitize.py) on a
 * machine without a GPU: malformed files stop in the GGUF reader, a
 * well-formed one stops at its first device allocation, and each call must
 * return a status code and release what it took.  Prints one line per call:
 * the status, then lmc_last_error(). */
#include <stdio.h>

#include "../include/lmc_cuda.h"

static void report(int rc) { printf("%d %s\n", rc, lmc_last_error()); }

int main(int argc, char **argv) {
    for (int i = 1; i < argc; i++) {
        lmc_model *m = NULL;
        int rc = lmc_model_load(argv[i], 2, LMC_KV_F16, &m);
        report(rc);
        if (!rc) lmc_model_free(m);
        m = NULL;
        rc = lmc_model_load_paged(argv[i], 2, 4, LMC_KV_Q8, 16, 3, 0, 1, NULL, &m);
        report(rc);
        if (!rc) lmc_model_free(m);
    }
    report(lmc_model_free(NULL));
    return 0;
}
