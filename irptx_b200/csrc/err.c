/* err.c -- the E-code table and the one-line refusal.
 *
 * The refusal format, exit discipline and code ranges are the reference's contract
 * (src/err.c:96-114, docs/ARCHITECTURE.md:85-92): exactly one
 * `error[E0NN]: irptx: cannot lower <what>` line on stderr, nothing on stdout, and the
 * first failure wins. Codes E000-E034 keep the reference's meanings so a caller that
 * switches on them sees no change; E040-E043 (selection) and E090-E094 (device) are this
 * backend's additions inside the reference's ranges.
 *
 * The last message is also kept per thread, so a C-ABI caller (ctypes, cgo) can read it
 * back with irx_last_error() instead of scraping stderr. */

#include <stdio.h>
#include <string.h>
#include "irx_int.h"

typedef struct { int code; const char *text; } etab_t;

static const etab_t ETAB[] = {
    { E000, "internal error, a bug in irptx-b200 rather than in the input" },
    { E001, "input file missing or unreadable" },
    { E002, "meta.json missing or without the requested kernel entry" },
    { E003, "KIR dump not printable ASCII" },
    { E004, "core library missing and could not be built" },
    { E005, "core timed out or could not be run" },
    { E009, "front end: other load failure" },
    { E010, "KIR syntax error, truncated input or unsupported format version" },
    { E011, "index out of range (node, item, field or string offset past its table)" },
    { E012, "kernel or buffer name is not a valid identifier" },
    { E013, "KIR string not printable ASCII, or over 63 characters" },
    { E014, "malformed number (integer or hex float)" },
    { E015, "required KIR field missing" },
    { E019, "KIR reader: other malformed input" },
    { E020, "unsupported node kind" },
    { E021, "unsupported op, or the body is not exactly one Tile" },
    { E022, "name not bound in any enclosing scope" },
    { E024, "dtype other than f32 or bf16" },
    { E025, "launch uses y or z beyond 1" },
    { E026, "StridedLoop step that is not a constant above 0" },
    { E027, "combine_states statement other than an Assign" },
    { E028, "accumulator or Init name declared twice" },
    { E029, "one name used for both an integer loop variable and an f32 value" },
    { E034, "warp shuffle whose length is not a power of two" },
    { E040, "graph matches no op family with an sm_100a kernel template" },
    { E041, "an index does not cover its buffer the way the family's template needs" },
    { E042, "a shape or dtype outside what the family's template takes" },
    { E043, "an op program longer or wider than the template's register file" },
    { E059, "selection: other unsupported construct" },
    { E080, "input larger than the KIR limit" },
    { E081, "a fixed table is full (nodes, fields, args)" },
    { E082, "nesting deeper than the limit" },
    { E090, "CUDA driver missing or failed to initialise" },
    { E091, "sm_100a kernel module failed to load, or a kernel is missing from it" },
    { E092, "a launch failed or a device-side wait ran out" },
    { E093, "bad argument at the C ABI" },
    { E094, "device or host memory could not be allocated or copied" },
    { E099, "limits: other" }
};

#define NETAB (sizeof ETAB / sizeof ETAB[0])

static _Thread_local char last_msg[400];
static _Thread_local int last_code = -1;
static _Thread_local int deferred;     /* 1: record refusals without printing them (irx_defer) */
static int quiet;

const char *irx_etext(int code)
{
    size_t i;
    for (i = 0; i < NETAB; i++)
        if (ETAB[i].code == code) return ETAB[i].text;
    return NULL;
}

void irx_set_quiet(int q) { quiet = q; }

const char *irx_last_msg(void) { return last_msg; }

int irx_last_code(void) { return last_code; }

void irx_clear_error(void) { last_code = -1; last_msg[0] = '\0'; }

int irx_fail(int code, const char *what)
{
    char w[300];
    if (!irx_etext(code)) code = E000;
    if (!what) what = irx_etext(code);
    snprintf(w, sizeof w, "%s", what);
    last_code = code;
    snprintf(last_msg, sizeof last_msg, "error[E%03d]: irptx: cannot lower %s", code, w);
    if (!quiet && !deferred) {
        fputs(last_msg, stderr);
        fputc('\n', stderr);
        fflush(stderr);
    }
    return 1;
}

/* While deferred, refusals are recorded on this thread but not printed: the selector tries the
 * templates, then the generic per-graph kernel, and prints only the refusal that stands. */
void irx_defer(int on) { deferred = on; }

void irx_emit_last(void)
{
    if (!quiet && last_code >= 0) {
        fputs(last_msg, stderr);
        fputc('\n', stderr);
        fflush(stderr);
    }
}

/* Keep a recorded refusal aside and put it back (the first refusal wins when both attempts fail). */
void irx_save_error(int *code, char *msg, size_t cap)
{
    *code = last_code;
    snprintf(msg, cap, "%s", last_msg);
}

void irx_restore_error(int code, const char *msg)
{
    last_code = code;
    snprintf(last_msg, sizeof last_msg, "%s", msg);
}
