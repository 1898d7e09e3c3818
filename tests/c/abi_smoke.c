/* C99 consumer of include/gguf_b200.h: checks that the header compiles as C and that the
 * entry points that need no GPU behave as documented (sizes, status codes, argument
 * checks before any CUDA call).  Built and run by tests/test_c_abi.py. */
#include <stdio.h>
#include <string.h>

#include "gguf_b200.h"

#define CHECK(cond)                                                   \
    do {                                                              \
        if (!(cond)) {                                                \
            fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                 \
        }                                                             \
    } while (0)

int main(void) {
    gq_layout_t lay;
    gq_tensor_t t;
    CHECK(gq_version() == GQ_ABI_VERSION);
    CHECK(strcmp(gq_strerror(GQ_OK), "success") == 0);
    CHECK(gq_strerror(GQ_ERR_SIZE) != NULL && strlen(gq_strerror(GQ_ERR_SIZE)) > 0);

    /* Q4_K 11008 x 4096: 176128 super-blocks of 144 bytes */
    CHECK(gq_query(GQ_TYPE_Q4_K, 11008, 4096, &lay) == GQ_OK);
    CHECK(lay.n_units == 176128 && lay.src_bytes == 176128LL * 144);
    CHECK(lay.codes_bytes == 11008LL * 4096 && lay.scales_count == 11008LL * 4096 / 32);
    CHECK(lay.block_values == 32 && lay.unit_values == 256);
    /* Q6_K keeps blocks of 16; Q8_0 4096 x 4096 (config 1) */
    CHECK(gq_query(GQ_TYPE_Q6_K, 256, 256, &lay) == GQ_OK && lay.block_values == 16);
    CHECK(gq_query(GQ_TYPE_Q8_0, 4096, 4096, &lay) == GQ_OK && lay.src_bytes == 524288LL * 34);
    CHECK(gq_query(GQ_TYPE_F32, 7, 1, &lay) == GQ_OK && lay.values_bytes == 28 && lay.block_values == 0);
    /* errors: unknown type, columns off the block grid, NULL out */
    CHECK(gq_query(99, 1, 32, &lay) == GQ_ERR_TYPE);
    CHECK(gq_query(GQ_TYPE_Q4_K, 1, 100, &lay) == GQ_ERR_SIZE);
    CHECK(gq_query(GQ_TYPE_Q4_K, 1, 256, NULL) == GQ_ERR_NULL);

    /* argument checks happen before any CUDA call */
    memset(&t, 0, sizeof t);
    t.type = GQ_TYPE_Q4_K;
    t.rows = 1;
    t.cols = 256;
    t.src_bytes = 144;
    CHECK(gq_convert(&t, GQ_OUT_CODES, NULL) == GQ_ERR_NULL);
    CHECK(gq_convert(NULL, GQ_OUT_CODES, NULL) == GQ_ERR_NULL);
    CHECK(gq_convert(&t, 0, NULL) == GQ_ERR_ARG);
    t.src_bytes = 143;
    CHECK(gq_convert(&t, GQ_OUT_CODES, NULL) == GQ_ERR_SIZE);
    t.perm_heads = 3;   /* rows must be a multiple of 2 * heads */
    t.src_bytes = 144;
    CHECK(gq_convert(&t, GQ_OUT_CODES, NULL) == GQ_ERR_ARG);
    CHECK(gq_convert_batch(NULL, 0, GQ_OUT_CODES, NULL) == GQ_OK);
    CHECK(gq_requantize_symmetric(NULL, NULL, 1, 32, 9, NULL, NULL, NULL, NULL) == GQ_ERR_ARG);
    CHECK(gq_unpack_fields(GQ_TYPE_Q8_0, NULL, 0, 1, NULL, NULL, NULL, NULL) == GQ_ERR_TYPE);
    CHECK(gq_remove_superblocks(NULL, NULL, 4, 1, 8, 2, NULL, NULL, NULL) == GQ_ERR_ARG);
    t.perm_heads = 0;
    t.cols = 512;       /* fused layout: cols must be whole 256-channel tiles (512 is) */
    t.src_bytes = 288;
    CHECK(gq_convert_modalix(&t, 0, NULL) == GQ_ERR_SIZE);   /* rows_padded < rows */
    CHECK(gq_session_create(0, 1000, NULL) == GQ_ERR_NULL);
    printf("abi_smoke: ok\n");
    return 0;
}
