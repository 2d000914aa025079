/* abi_cpu.c -- the C ABI from C, with no GPU: compile a KIR graph read from a file, describe
 * it, read its algorithmic work and shard split, print a pointwise graph's kernel source length,
 * and check a malformed graph's refusal code. Prints "ok" and exits 0, or names what failed.
 * Built and run by tests/test_c_abi.py:  abi_cpu <pointwise.kir> <bad.kir> */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "irx.h"

static char *slurp(const char *path, size_t *len)
{
    FILE *f = fopen(path, "rb");
    char *buf;
    long n;
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    n = ftell(f);
    fseek(f, 0, SEEK_SET);
    buf = (char *)malloc((size_t)n + 1);
    if (!buf || fread(buf, 1, (size_t)n, f) != (size_t)n) { fclose(f); free(buf); return NULL; }
    fclose(f);
    buf[n] = 0;
    *len = (size_t)n;
    return buf;
}

int main(int argc, char **argv)
{
    irx_plan_t plan;
    char desc[512], err[256];
    double bytes = 0, flops = 0;
    long long u0, u1;
    int comb, n;
    size_t len;
    char *kir;
    if (argc != 3) { fprintf(stderr, "usage: abi_cpu good.kir bad.kir\n"); return 2; }
    irx_quiet(1);
    if (!(kir = slurp(argv[1], &len))) { puts("cannot read the good KIR"); return 1; }
    if (irx_compile(kir, len, &plan)) { irx_last_error(err, sizeof err); printf("compile failed: %s\n", err); return 1; }
    free(kir);
    if (irx_plan_family(&plan) != IRX_FAM_POINTWISE) { puts("family is not pointwise"); return 1; }
    irx_plan_describe(&plan, desc, sizeof desc);
    if (strncmp(desc, "pointwise n=4099", 16)) { printf("describe: %s\n", desc); return 1; }
    if (irx_plan_work(&plan, &bytes, &flops) || bytes != 3.0 * 4 * 4099) { printf("work: %g\n", bytes); return 1; }
    if (irx_plan_shard(&plan, 1, 2, &u0, &u1, &comb) || u0 != 257 || u1 != 513 || comb != IRX_COMBINE_NONE) {
        printf("shard: %lld %lld %d\n", u0, u1, comb);
        return 1;
    }
    n = irx_plan_source(&plan, NULL, 0);
    if (irx_jit(-1) && n < 100) { printf("source length %d\n", n); return 1; }
    if (!(kir = slurp(argv[2], &len))) { puts("cannot read the bad KIR"); return 1; }
    if (irx_compile(kir, len, &plan) != 1) { puts("a malformed graph compiled"); return 1; }
    free(kir);
    n = irx_last_error(err, sizeof err);
    if (n <= 0 || strncmp(err, "error[E", 7)) { printf("refusal: %d %s\n", n, err); return 1; }
    if (irx_plan_family(&plan) != 0) { puts("a refused plan has a family"); return 1; }
    printf("ok %s\n", irx_version());
    return 0;
}
