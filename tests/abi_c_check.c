/* A plain C caller of the library's C ABI (include/crosslane_b200.h), built and run by
 * tests/test_abi_compiled.py: the host-only entry points (lane config, placement parsing,
 * routing, packing) and the error convention (status code + message, NULL handles,
 * out-of-range ids). With a CUDA device it also creates a bank and checks contains /
 * geometry / destroy; without one, bank creation must fail with a CUDA error code and a
 * message. Prints "abi ok" and exits 0 when every check holds. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "crosslane_b200.h"

static int failures = 0;
#define CHECK(cond, what)                                      \
    do {                                                       \
        if (!(cond)) {                                         \
            fprintf(stderr, "FAILED: %s (%s:%d)\n", what, __FILE__, __LINE__); \
            ++failures;                                        \
        }                                                      \
    } while (0)

int main(int argc, char** argv) {
    const int expect_gpu = argc > 1 && strcmp(argv[1], "gpu") == 0;
    clb_error_v1 err;

    CHECK(clb_abi_version() == CLB_ABI_VERSION, "abi version");

    /* lane config: the reference parser's strictness (common.hpp:55-125) */
    clb_lane_config_v1 lc;
    memset(&err, 0, sizeof err);
    CHECK(clb_lane_config_parse("warm_cuda_experts=stack-v1\ncuda_expert_math=cpu-q8k-v1\n", &lc, &err) == CLB_OK,
          "lane config parse");
    CHECK(lc.experts == 2 && lc.exact_math == 1 && (lc.bank_flags & CLB_BANK_EXACT_ORDER), "lane config values");
    memset(&err, 0, sizeof err);
    CHECK(clb_lane_config_parse("warm_cuda_experts=stack-v1\nwarm_cuda_experts=off\n", &lc, &err) == CLB_E_INVALID,
          "duplicate key rejected");
    CHECK(err.code == CLB_E_INVALID && strlen(err.message) > 0, "error struct filled");

    /* frozen placement: 1 layer, 2 experts, lane 3 = CUDA */
    const char* text = "STRATA_WARM_PLACEMENT_V1 1 2 7\n0 0 3\n0 1 0\n";
    int32_t lanes[2] = {-1, -1};
    uint64_t tag = 0;
    CHECK(clb_placement_parse(text, strlen(text), 1, 2, lanes, &tag, &err) == CLB_OK, "placement parse");
    CHECK(lanes[0] == CLB_LANE_CUDA && lanes[1] == CLB_LANE_CPU && tag == 7, "placement values");
    const char* bad = "STRATA_WARM_PLACEMENT_V1 1 2 7\n0 0 3\n";
    CHECK(clb_placement_parse(bad, strlen(bad), 1, 2, lanes, &tag, &err) == CLB_E_INVALID, "missing row rejected");

    /* host routing, mode A (top-k by logit, ties to the lower id, sigmoid weights) */
    float logits[4] = {0.5f, 2.0f, -1.0f, 2.0f};
    int32_t ids[2];
    float w[2];
    CHECK(clb_route_host(0, logits, NULL, 4, 2, 1.0f, ids, w) == CLB_OK, "route host");
    CHECK(ids[0] == 1 && ids[1] == 3 && w[0] == w[1] && w[0] > 0.49f && w[0] < 0.51f, "route host picks");

    /* null handles */
    CHECK(clb_bank_contains(NULL, 0, 0) == 0, "contains on a null bank");
    CHECK(clb_bank_weight_bytes(NULL) == 0, "weight bytes of a null bank");
    CHECK(clb_bank_create(NULL, NULL, &err) == CLB_E_INVALID, "create with null config");

    clb_bank_config_v1 cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.device = 0;
    cfg.n_layers = 2;
    cfg.n_experts = 8;
    cfg.dim = 512;
    cfg.ff = 256;
    cfg.max_picks = 2;
    clb_bank* bank = NULL;
    memset(&err, 0, sizeof err);
    const int32_t rc = clb_bank_create(&cfg, &bank, &err);
    if (expect_gpu) {
        CHECK(rc == CLB_OK && bank != NULL, "bank create on a GPU");
        if (bank) {
            int32_t nl = 0, ne = 0, dim = 0, ff = 0;
            CHECK(clb_bank_geometry(bank, &nl, &ne, &dim, &ff) == CLB_OK && nl == 2 && ne == 8 && dim == 512 && ff == 256,
                  "geometry");
            CHECK(clb_bank_contains(bank, 0, 3) == 0, "nothing resident yet");
            CHECK(clb_bank_contains(bank, 5, 3) == 0 && clb_bank_contains(bank, 0, 99) == 0, "out of range ids");
            float x[512] = {0}, y[512];
            memset(&err, 0, sizeof err);
            CHECK(clb_bank_compute(bank, 0, 3, x, y, &err) == CLB_E_INVALID && strlen(err.message) > 0,
                  "compute of a non-resident expert");
            clb_bank_destroy(bank);
        }
    } else {
        CHECK(rc != CLB_OK && bank == NULL && err.code == rc && strlen(err.message) > 0, "bank create without a GPU");
    }
    clb_bank_destroy(NULL);

    if (failures) return 1;
    printf("abi ok\n");
    return 0;
}
