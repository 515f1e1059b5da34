/* tests/cpp/c_abi_cpu_test.c - the C ABI from plain C (host only).
 *
 * include/strata_kv.h is a C header: this file is compiled as C99 with -Wall -Wextra -pedantic -Werror and linked
 * against libstrata_kv.so.  It calls the entry points that need no GPU - the version, argument refusals with
 * their error text, the block-table expansion and the many-to-many hand-off order - and checks the results.
 * Exit 0 = pass. */
#include "strata_kv.h"

#include <stdio.h>
#include <string.h>

static int checks = 0, failures = 0;

static void check(int ok, const char* what) {
    ++checks;
    if (!ok) {
        ++failures;
        fprintf(stderr, "FAIL: %s\n", what);
    }
}

int main(void) {
    check(skv_version() >= 1, "a version");

    /* refusals carry a message */
    check(skv_pool_create(0, 0, 1024, NULL) == SKV_EINVAL, "a null output is refused");
    check(strlen(skv_last_error()) > 0, "with an error message");

    /* the reference page_table format from a block table: page p of block b -> slot * 128 + offset + p */
    {
        const int32_t blocks[3] = {7, 0, 2};
        int32_t table[3 * 64];
        check(skv_expand_block_table(blocks, 3, 64, 128, 64, table) == SKV_OK, "expand a block table");
        check(table[0] == 7 * 128 + 64 && table[63] == 7 * 128 + 127 && table[64] == 64 && table[128] == 2 * 128 + 64,
              "V pages of each slot, in block order");
        check(skv_expand_block_table(blocks, 3, 64, 128, 65, table) == SKV_EINVAL, "an offset past the slot");
    }

    /* the hand-off order: 2 sources x 2 destinations, destination 1 reads both sources */
    {
        const uint64_t demand[4] = {100, 300, 0, 200}; /* s0->d0 100, s0->d1 300, s1->d1 200 */
        skv_sched_run runs[2 * 4];
        int n_runs[2] = {0, 0};
        uint64_t bound = 0;
        int phases = 0;
        uint64_t moved[2][2] = {{0, 0}, {0, 0}};
        int d, j;
        check(skv_schedule_phases(demand, 2, 2, runs, 4, n_runs, &bound, &phases) == SKV_OK, "schedule a batch");
        check(bound == 500, "the bound is destination 1's ingress (300 + 200)");
        check(phases >= 1 && phases <= 4, "at most n * n phases");
        for (d = 0; d < 2; ++d)
            for (j = 0; j < n_runs[d]; ++j) {
                const skv_sched_run* r = &runs[d * 4 + j];
                check(r->src >= 0 && r->src < 2 && r->hi > r->lo, "a run reads a real source");
                check(r->lo == moved[r->src][d], "runs of one flow are consecutive");
                moved[r->src][d] = r->hi;
                if (r->wait >= 0) check(r->wait == j, "a destination waits on the flag of its own run index");
            }
        check(moved[0][0] == 100 && moved[0][1] == 300 && moved[1][1] == 200 && moved[1][0] == 0,
              "every flow is moved exactly");
        check(skv_schedule_phases(demand, 0, 2, runs, 4, n_runs, &bound, &phases) == SKV_EINVAL,
              "an empty side is refused");
    }

    printf("c_abi_cpu_test: %d checks, %s\n", checks, failures ? "FAILED" : "OK");
    return failures ? 1 : 0;
}
