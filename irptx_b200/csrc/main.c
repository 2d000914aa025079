/* main.c -- the `irx` command: the reference's `irptx [file] | --version` process contract
 * (src/main.c:1-6, 48-76) over the sm_100a selector.
 *
 *   irx [file]          KIR from the file, or stdin: exit 0 with the selected template's
 *                       one-line description on stdout, or exit 1 with exactly one
 *                       `error[E0NN]: irptx: cannot lower ...` line on stderr and nothing on
 *                       stdout
 *   irx --version
 *   irx --work [file]   the description plus the plan's algorithmic bytes and flops
 *   irx --source [file] the CUDA source of a pointwise graph's own sm_100a kernel, the
 *                       counterpart of the reference's printed PTX (exit 1, E093, for plans
 *                       of the families that run prebuilt kernels) */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "irx_int.h"
#include "../../include/irx.h"

static char BUF[KIR_MAX_TEXT + 1];

int main(int argc, char **argv)
{
    FILE *fp = stdin;
    size_t n;
    int work = 0, src = 0, ai = 1;
    static irx_plan_t plan;
    char desc[1024];

    if (argc == 2 && !strcmp(argv[1], "--version")) { puts(irx_version()); return 0; }
    if (argc > 1 && !strcmp(argv[1], "--work")) { work = 1; ai = 2; }
    if (argc > 1 && !strcmp(argv[1], "--source")) { src = 1; ai = 2; }
    if (argc > ai + 1) return irx_fail(E001, "more than one input file argument");
    if (argc == ai + 1 && !(fp = fopen(argv[ai], "rb"))) return irx_fail(E001, "an input file that could be opened");
    n = fread(BUF, 1, sizeof BUF, fp);
    if (fp != stdin) fclose(fp);
    if (n > KIR_MAX_TEXT) return irx_fail(E080, "input larger than the KIR limit");
    if (irx_compile(BUF, n, &plan)) return 1;
    if (src) {
        int len = irx_plan_source(&plan, NULL, 0);
        char *text;
        if (len < 0) return 1;
        if (!(text = (char *)malloc((size_t)len + 1))) return irx_fail(E094, "host memory for the kernel source");
        irx_plan_source(&plan, text, (size_t)len + 1);
        fputs(text, stdout);
        free(text);
        return fflush(stdout) ? 1 : 0;
    }
    irx_plan_describe(&plan, desc, sizeof desc);
    if (work) {
        double b = 0, f = 0;
        irx_plan_work(&plan, &b, &f);
        printf("%s bytes=%.0f flops=%.0f\n", desc, b, f);
    } else {
        printf("%s\n", desc);
    }
    return fflush(stdout) ? 1 : 0;
}
