/*
 * c_abi_host.c -- the C ABI of libabra_b200.so used from plain C, as a
 * caller that binds the header directly (no ctypes) would.  It makes only
 * calls that need no GPU: the version and error strings, the candidate
 * tables and the tuning table, the launch-plan query, the prompt-lookup
 * draft, the tensor-parallel split, and argument checks that fail before
 * any launch.  Built and run by tests/test_c_abi.py; exits 0 when every
 * check holds, else prints the first failure and exits 1.
 */
#include <stdio.h>
#include <string.h>

#include "abra_b200.h"

#define CHECK(cond)                                                        \
    do {                                                                   \
        if (!(cond)) {                                                     \
            fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
            return 1;                                                      \
        }                                                                  \
    } while (0)

int main(void) {
    CHECK(strncmp(abra_version(), "abra_b200", 9) == 0);

    /* candidate tables */
    const int n = abra_candidate_count();
    CHECK(n >= 8);
    int32_t id, mode, ks, ncw, cps, kb;
    CHECK(abra_candidate_info(0, &id, &mode, &ks, &ncw, &cps, &kb) == ABRA_OK);
    CHECK(id > 0 && mode >= 0 && mode <= 2 && (ks == 1 || ks == 2 || ks == 4 || ks == 8));
    CHECK(abra_candidate_info(n, &id, &mode, &ks, &ncw, &cps, &kb) == ABRA_E_INVALID);
    CHECK(strlen(abra_last_error()) > 0);
    CHECK(abra_q6k_candidate_count() >= 8);

    /* tuning table: set, get, clear */
    CHECK(abra_tune_set(777, 2560, 1, 1, id) == ABRA_OK);
    CHECK(abra_tune_get(777, 2560, 1, 1) == id);
    CHECK(abra_tune_set(777, 2560, 1, 1, 999999) == ABRA_E_INVALID);
    CHECK(abra_tune_clear() == ABRA_OK);

    /* launch plan of the gate shape on 148 SMs, without a GPU */
    int64_t plan[8];
    CHECK(abra_mmvq_plan_info(ABRA_GGML_Q4_K, 0, 9728, 2560, 1, 1, 0, 0, 0, 8, 148, plan) ==
          ABRA_OK);
    CHECK(plan[0] >= 1 && plan[0] <= 4 * 148 && plan[6] == 1216 && plan[5] <= 227 * 1024);
    CHECK(abra_mmvq_plan_info(ABRA_GGML_Q6_K, 0, 151936, 2560, 1, 1, 0, 0, 0, 8, 148, plan) ==
          ABRA_OK);
    CHECK(plan[6] == 18992);

    /* prompt-lookup draft (host only) */
    const int32_t hist[6] = {1, 2, 3, 4, 1, 2};
    int32_t draft[4];
    CHECK(abra_lookup_draft(hist, 6, 2, 4, draft) == 2 && draft[0] == 3 && draft[1] == 4);
    CHECK(abra_lookup_draft(hist, 3, 2, 4, draft) == 0);

    /* tensor-parallel split of the default Qwen3-4B shape */
    abra_model_config cfg;
    CHECK(abra_model_default_config(&cfg) == ABRA_OK);
    CHECK(cfg.n_layers == 36 && cfg.hidden == 2560 && cfg.vocab == 151936);
    abra_tp_shard sh;
    CHECK(abra_tp_shard_info(&cfg, 1, 2, &sh) == ABRA_OK);
    CHECK(sh.vocab_lo == 75968 && sh.vocab_hi == 151936 && sh.sl_base == 4 && sh.sl_cnt == 4);
    CHECK(abra_tp_shard_info(&cfg, 0, 3, &sh) != ABRA_OK);
    /* rank 1 of 2 keeps canonical K-slices 4..7 of every attn_output row:
     * superblocks 8..15 of 16, bytes [1152, 2304) of each 2304-byte row */
    int64_t sl[8];
    CHECK(abra_tp_tensor_slice(&cfg, 1, 2, 0, ABRA_TENSOR_ATTN_OUTPUT, sl) == ABRA_OK);
    CHECK(sl[0] == ABRA_GGML_Q4_K && sl[1] == 2560 && sl[2] == 4096 && sl[3] == 2304);
    CHECK(sl[4] == 0 && sl[5] == 2560 && sl[6] == 1152 && sl[7] == 1152);
    CHECK(abra_tp_tensor_slice(&cfg, 1, 2, 0, 11, sl) == ABRA_E_INVALID);

    /* the adapter's host functions: a row quantized to Q4_K and back */
    {
        float xr[512], yr[512];
        unsigned char qb[2 * 144];
        for (int i = 0; i < 512; ++i) xr[i] = (float)((i * 37) % 101 - 50) / 25.0f;
        quantize_row_q4_K_upstream_cpu(xr, qb, 512);
        dequantize_row_q4_K_upstream_cpu(qb, yr, 512);
        double se = 0.0, sx = 0.0;
        for (int i = 0; i < 512; ++i) {
            se += (double)(xr[i] - yr[i]) * (xr[i] - yr[i]);
            sx += (double)xr[i] * xr[i];
        }
        CHECK(se < 0.01 * sx);
    }

    /* argument checks that fail before any launch */
    CHECK(abra_q4k_mmvq(NULL, NULL, NULL, 64, 2560, 1, NULL) == ABRA_E_INVALID);
    CHECK(abra_q4k_mmvq((void *)16, (void *)16, (float *)16, 64, 300, 1, NULL) == ABRA_E_INVALID);
    CHECK(strstr(abra_last_error(), "QK_K") != NULL);
    CHECK(abra_q6k_mmvq((void *)16, (void *)16, (float *)16, 64, 2560, 9, NULL) ==
          ABRA_E_UNSUPPORTED);
    CHECK(abra_model_prefill(NULL, 32) == ABRA_E_INVALID);
    printf("c abi host checks: ok\n");
    return 0;
}
