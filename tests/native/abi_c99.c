/* The C ABI as a C binding (cgo, N-API, JNI glue) sees it: include/ctu_b200.h compiled as
 * strict C99 and linked against the built libctu_b200.so, with calls that need no GPU
 * (argument contracts, host-side plans and sizes).  Exits 0 when every check holds,
 * otherwise prints the failing check and exits 1. */
#include <stdio.h>
#include <string.h>

#include "ctu_b200.h"

static int failures = 0;

#define CHECK(cond)                                                        \
    do {                                                                   \
        if (!(cond)) {                                                     \
            fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            ++failures;                                                    \
        }                                                                  \
    } while (0)

static int error_mentions(const char *text) { return strstr(ctu_last_error(), text) != NULL; }

int main(void) {
    int kind = -1, warps = -1, rows = -1, prev;
    void *const fake = (void *)0x10000; /* aligned, never dereferenced: a contract check fails first */

    CHECK(ctu_version() >= ((0 << 16) | (1 << 8)));

    /* Quantizer: K must be a multiple of the 256-column rotation group; no rows is a no-op. */
    CHECK(ctu_convrot_quantize(NULL, 4, 300, CTU_ACT_NONE, 8, NULL, NULL, NULL) == CTU_ERR_INVALID_ARGUMENT);
    CHECK(error_mentions("divisible by 256"));
    CHECK(ctu_convrot_quantize(NULL, 0, 512, CTU_ACT_NONE, 8, NULL, NULL, NULL) == CTU_OK);

    /* W8A8 linear: K % 16 (reference: bindings.cpp's TORCH_CHECK). */
    CHECK(ctu_int8_linear(NULL, NULL, NULL, NULL, 8, NULL, NULL, 4, 8, 24, NULL) == CTU_ERR_INVALID_ARGUMENT);
    CHECK(error_mentions("K%16=0"));

    /* One-call linear: its synchronisation words and its N % 8 contract. */
    CHECK(ctu_convrot_int8_linear_sync_words(0) == 1);
    CHECK(ctu_convrot_int8_linear_sync_words(129) == 3);
    CHECK(ctu_convrot_int8_linear_sync_words(32760) == 257);
    CHECK(ctu_convrot_int8_linear((const void *)fake, (const int8_t *)fake, (const float *)fake, 12, NULL, fake,
                                  (int8_t *)fake, (float *)fake, (uint32_t *)fake, 4, 12, 512, NULL) ==
          CTU_ERR_INVALID_ARGUMENT);
    CHECK(error_mentions("N%8=0"));

    /* Per-group linears: K a multiple of the 128-column group. */
    CHECK(ctu_asym_w4a8_g128_linear(NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 4, 8, 192, NULL) ==
          CTU_ERR_INVALID_ARGUMENT);
    CHECK(ctu_w4a4_g128_linear(NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 4, 12, 128, NULL) ==
          CTU_ERR_INVALID_ARGUMENT);

    /* Test hooks: out-of-range selectors are refused, valid ones return the previous value. */
    CHECK(ctu_debug_set_fused_linear(3) == CTU_ERR_INVALID_ARGUMENT);
    prev = ctu_debug_set_gemm_kernel(2);
    CHECK(prev >= 0);
    CHECK(ctu_debug_set_gemm_kernel(prev) == 2);

    /* The quantizer plan is host logic: a K = 5120 int8 row has one. */
    CHECK(ctu_debug_quant_plan(5120, CTU_ACT_NONE, 8, 232448, &kind, &warps, &rows) == CTU_OK);
    CHECK(kind >= 0 && warps > 0 && rows > 0);

    if (failures == 0) printf("C99 ABI checks passed\n");
    return failures == 0 ? 0 : 1;
}
