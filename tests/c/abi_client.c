/* SPDX-License-Identifier: MIT
 *
 * abi_client.c -- a plain C17 client of the C-ABI, as the reference (itself
 * C17) would link it: every public header included, only host-side entry
 * points called, so it runs without a GPU. Built and run by
 * tests/test_c_client.py; prints "ok" and exits 0, or names the failed check.
 *
 * Checks: the headers compile as C; status codes instead of aborts on bad
 * arguments (the reference's matmul_dispatch aborts, slm/model.c:259-261);
 * activation-layout size queries; deterministic synthetic data; a synthetic
 * model written as GGUF and read back (slm/gguf.c format) with identical
 * tensors; the sampler's generator seeding.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qh_backend.h"
#include "qh_gguf.h"
#include "qh_kernels.h"
#include "qh_sampler.h"
#include "qh_slm.h"
#include "qh_synth.h"

#define CHECK(cond)                                              \
    do {                                                         \
        if (!(cond)) {                                           \
            fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                            \
        }                                                        \
    } while (0)

int main(int argc, char **argv) {
    const char *gguf_path = argc > 1 ? argv[1] : "abi_client.gguf";

    CHECK(strstr(qh_version(), "sm_100a") != NULL);

    /* bad arguments come back as statuses with a message */
    CHECK(qh_matmul(12, NULL, 1024, 3072, NULL, 1, NULL, NULL, 0, NULL) == QH_ERR_INVALID);
    CHECK(strlen(qh_last_error()) > 0);
    CHECK(qh_quantize_q8k(NULL, 1024, 1, NULL, NULL) == QH_ERR_INVALID);
    CHECK(qh_gdn_chunked(NULL, NULL, NULL, NULL, 1, 1, 1, 128, NULL, NULL) == QH_ERR_INVALID);

    /* split Q8_K layout of 3 rows of 1024: qs, then 16-byte scale rows, then block sums */
    CHECK(qh_q8k_d_offset(1024, 3) == 3072);
    CHECK(qh_q8k_bsums_offset(1024, 3) == 3072 + 48);
    CHECK(qh_q8k_bytes(1024, 3) == 3072 + 48 + 384);

    /* synthetic inputs are reproducible */
    uint8_t *a = (uint8_t *)malloc(144 * 8), *b = (uint8_t *)malloc(144 * 8);
    CHECK(a && b);
    CHECK(qh_synth_blocks(12, 8, 0x5EED, a) == 0 && qh_synth_blocks(12, 8, 0x5EED, b) == 0);
    CHECK(memcmp(a, b, 144 * 8) == 0);
    free(a);
    free(b);
    float x0[64], x1[64];
    CHECK(qh_synth_normal(7, 64, 0.0f, 1.0f, x0) == 0 && qh_synth_normal(7, 64, 0.0f, 1.0f, x1) == 0);
    CHECK(memcmp(x0, x1, sizeof(x0)) == 0);

    /* a small synthetic model through the GGUF writer and reader */
    qh_slm_config cfg;
    qh_slm_config_default(&cfg, 64);
    cfg.n_layers = 4;
    cfg.vocab = 512;
    qh_blob *blob = NULL, *back = NULL;
    CHECK(qh_blob_synthetic(&cfg, 0x51A11, &blob) == 0 && blob != NULL);
    CHECK(qh_gguf_write(gguf_path, &cfg, blob) == 0);
    qh_slm_config cfg2;
    CHECK(qh_gguf_load(gguf_path, 0, &cfg2, &back) == 0 && back != NULL);
    CHECK(cfg2.n_layers == cfg.n_layers && cfg2.hidden == cfg.hidden && cfg2.vocab == cfg.vocab);
    CHECK(qh_blob_count(back) == qh_blob_count(blob));
    for (int i = 0; i < qh_blob_count(blob); ++i) {
        const char *name;
        int32_t type, type2;
        int64_t shape[2], shape2[2], nb, nb2;
        const void *d, *d2;
        CHECK(qh_blob_tensor(blob, i, &name, &type, shape, &d, &nb) == 0);
        const int j = qh_blob_find(back, name);
        CHECK(j >= 0);
        const char *name2;
        CHECK(qh_blob_tensor(back, j, &name2, &type2, shape2, &d2, &nb2) == 0);
        CHECK(type == type2 && shape[0] == shape2[0] && shape[1] == shape2[1] && nb == nb2);
        CHECK(memcmp(d, d2, (size_t)nb) == 0);
    }
    qh_blob_free(back);
    qh_blob_free(blob);
    remove(gguf_path);

    /* sampler defaults and the generator's seeding */
    qh_sampler sp;
    qh_sampler_defaults(&sp);
    uint64_t s0[2], s1[2];
    qh_rng_seed(42, s0);
    qh_rng_seed(42, s1);
    CHECK(s0[0] == s1[0] && s0[1] == s1[1] && (s0[0] | s0[1]) != 0);

    printf("ok\n");
    return 0;
}
