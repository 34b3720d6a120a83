/* A plain C99 caller of the C ABI (include/sparse_attn_b200.h), as a non-Python runtime would bind
 * it: version, the selection workspace size query, and argument checks that reject bad calls before
 * any device work (so it runs without a GPU).  Prints one line per check; exit code 0 when all pass. */
#include <stdio.h>
#include <string.h>

#include "sparse_attn_b200.h"

static int fails = 0;

static void check(int ok, const char* what) {
    printf("%s %s\n", ok ? "ok" : "FAIL", what);
    if (!ok) ++fails;
}

int main(void) {
    check(sa_version() == 1, "sa_version");
    /* 64 heads x 64 q blocks x 512 key blocks of fp32 logits, rows padded to 32 blocks */
    size_t ws = sa_select_workspace_bytes(64, 64, 512);
    check(ws >= (size_t)64 * 64 * 512 * 4, "sa_select_workspace_bytes covers the logits");
    check(sa_select_workspace_bytes(-1, 64, 512) == 0, "sa_select_workspace_bytes rejects bad sizes");
    /* null pointers and unsupported sizes come back as error codes with a message */
    int rc = sa_quantize_e4m3(NULL, 0, 0, 16, 2, 128, NULL, 0, SA_QUANT_MUL, NULL, 0, 0, 0, 0, NULL);
    check(rc == SA_ERR_ARG && strlen(sa_last_error()) > 0, "sa_quantize_e4m3 rejects null pointers");
    rc = sa_attn_fwd_bf16(NULL, 0, 0, NULL, 0, 0, NULL, 0, 0, NULL, 0, 0, 16, 2, 1, 96, 16, 0, 0, NULL, NULL, 0,
                          128, 64, 0.1f, NULL, NULL);
    check(rc < 0 && strlen(sa_last_error()) > 0, "sa_attn_fwd_bf16 rejects head_dim 96");
    rc = sa_add_rmsnorm_bf16(NULL, 0, NULL, 0, NULL, NULL, 0, 4, 100, 1e-6f, NULL);
    check(rc == SA_ERR_ARG, "sa_add_rmsnorm_bf16 rejects hidden % 8 != 0");
    printf("%d failures\n", fails);
    return fails != 0;
}
