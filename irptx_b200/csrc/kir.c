/* kir.c -- the KIR text reader.
 *
 * Reads the reference's wire format (BhuvanB404/IRptx 0.1.0): the header lines `kir 1`,
 * `kernel`, `launch gx gy gz bx by bz smem`, `arg i name in|const|out dtype rank dims...`,
 * `zero name`, `body`, then one S-expression and `end` (src/kir.c:553-675,
 * fe/kirdump.py:90-103). Node fields are `name=value`; values are ints, hex floats with an
 * `f` suffix (narrowed to f32 bits once, src/kir.c:187-205), quoted strings, `none`,
 * `true`/`false`, `op:<name>`, `dt:<name>`, lists `[...]` and nodes `(Kind ...)`. The same
 * inputs are refused with the same codes (E010 syntax, E012 names, E013 strings, E014
 * numbers, E015 missing header, E080-E082 limits).
 *
 * The number and atom lexer follows the reference's checks one for one (src/kir.c:124-205:
 * string append, decimal integers, the hex-float shape test and the f32 narrowing), because
 * the grammar fixes what is accepted and with which code; the reader around it is this file's
 * own design.
 *
 * One difference from the reference reader: argument dtypes. The reference types only
 * `f32` and turns every other name into a refusal at selection time (src/kir.c:587,
 * src/isel.c:315); this reader also types `bf16`, which the sm_100a templates lower.
 *
 * Parsing is iterative. Values that belong to a still-open node or list sit on a pending
 * stack; when the bracket closes they are copied, contiguously, into the field or item
 * pool, so every node's fields and every list's items are one slice. */

#include <ctype.h>
#include <float.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "irx_int.h"

#define PEND_MAX (KIR_MAX_FLD + KIR_MAX_ITEM)

typedef struct {
    uint8_t  is_node;
    uint32_t node;          /* node id for a node frame */
    uint32_t pend0;         /* first pending entry of this frame */
    uint32_t fname;         /* field name waiting for its value (node frames) */
} frame_t;

typedef struct { uint32_t name; kv_t val; } pend_t;

static pend_t PEND[PEND_MAX];

static int bad_at(int code, const char *msg, size_t at)
{
    char b[200];
    snprintf(b, sizeof b, "%s (at byte %lu)", msg, (unsigned long)at);
    return irx_fail(code, b);
}

static int is_ws(int c) { return c == ' ' || c == '\t' || c == '\r' || c == '\n'; }
static int is_delim(int c) { return is_ws(c) || c == '(' || c == ')' || c == '[' || c == ']' || c == '"'; }
static int is_id0(int c) { return (c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || c == '_'; }
static int is_id(int c) { return is_id0(c) || (c >= '0' && c <= '9'); }

static int str_put(kir_t *k, const char *s, size_t n, uint32_t *off)
{
    if (n > KIR_MAX_NAME) return irx_fail(E013, "a KIR string over 63 characters");
    if ((size_t)k->nstr + n + 1u >= KIR_MAX_STR) return irx_fail(E081, "more KIR string bytes than the pool holds");
    memcpy(k->str + k->nstr, s, n);
    k->str[k->nstr + n] = '\0';
    *off = k->nstr;
    k->nstr += (uint32_t)n + 1u;
    return 0;
}

static int parse_int(const char *s, size_t n, int64_t *out)
{
    int neg = n > 0 && s[0] == '-';
    size_t i = neg ? 1u : 0u;
    uint64_t v = 0, lim = neg ? (uint64_t)INT64_MAX + 1u : (uint64_t)INT64_MAX;

    if (i >= n || n - i > 19) return irx_fail(E014, "an integer that is empty or too long");
    for (; i < n; i++) {
        unsigned d;
        if (s[i] < '0' || s[i] > '9') return irx_fail(E014, "an integer with a non-digit in it");
        d = (unsigned)(s[i] - '0');
        if (v > (lim - d) / 10u) return irx_fail(E014, "an integer outside the int64 range");
        v = v * 10u + d;
    }
    *out = neg ? (int64_t)(0u - v) : (int64_t)v;
    return 0;
}

/* [-]0x<hex>[.<hex>]p[+-]<dec>f: the only float spelling float.hex() produces. */
static int hexfloat_ok(const char *s, size_t n)
{
    size_t i = (n > 0 && s[0] == '-') ? 1u : 0u, digits = 0;

    if (n < i + 5 || s[n - 1] != 'f' || s[i] != '0' || s[i + 1] != 'x') return 0;
    n--;
    for (i += 2; i < n && isxdigit((unsigned char)s[i]); i++) digits++;
    if (i < n && s[i] == '.')
        for (i++; i < n && isxdigit((unsigned char)s[i]); i++) digits++;
    if (!digits || i >= n || s[i] != 'p') return 0;
    i++;
    if (i < n && (s[i] == '+' || s[i] == '-')) i++;
    if (i >= n) return 0;
    for (; i < n; i++)
        if (!isdigit((unsigned char)s[i])) return 0;
    return 1;
}

static int parse_flt(const char *s, size_t n, uint32_t *bits)
{
    char buf[KIR_MAX_NAME + 1];
    char *end = NULL;
    double d;
    float f;

    if (n > KIR_MAX_NAME || !hexfloat_ok(s, n)) return irx_fail(E014, "a malformed hex float");
    memcpy(buf, s, n - 1u);
    buf[n - 1u] = '\0';
    d = strtod(buf, &end);
    if (end != buf + (n - 1u)) return irx_fail(E014, "a hex float strtod would not take whole");
    if (d > FLT_MAX || d < -FLT_MAX) return irx_fail(E014, "a hex float outside the f32 range");
    f = (float)d;
    memcpy(bits, &f, sizeof *bits);
    return 0;
}

static int parse_atom(kir_t *k, const char *s, size_t n, kv_t *v, size_t at)
{
    size_t i;
    for (i = 0; i < n; i++)
        if ((unsigned char)s[i] < 0x21 || (unsigned char)s[i] >= 0x7f)
            return bad_at(E010, "a non-ASCII byte in a KIR token", at + i);
    if (n == 0) return bad_at(E010, "a bracket or quote where a value should be", at);
    if (n == 4 && !memcmp(s, "none", 4)) { v->tag = KV_NONE; return 0; }
    if (n == 4 && !memcmp(s, "true", 4)) { v->tag = KV_BOOL; v->i = 1; return 0; }
    if (n == 5 && !memcmp(s, "false", 5)) { v->tag = KV_BOOL; v->i = 0; return 0; }
    if (n > 3 && (!memcmp(s, "op:", 3) || !memcmp(s, "dt:", 3))) {
        v->tag = s[0] == 'o' ? KV_OP : KV_DT;
        return str_put(k, s + 3, n - 3u, &v->ref);
    }
    if (isdigit((unsigned char)s[0]) || s[0] == '-') {
        size_t j = s[0] == '-' ? 1u : 0u;
        if (n > j + 1 && s[j] == '0' && s[j + 1] == 'x') {
            v->tag = KV_FLT;
            return parse_flt(s, n, &v->fbits);
        }
        v->tag = KV_INT;
        return parse_int(s, n, &v->i);
    }
    return bad_at(E010, "an unknown bare word in the KIR body", at);
}

/* Push one finished value for the innermost open frame (or make it the root). */
static int push_val(kir_t *k, frame_t *fr, int depth, uint32_t *npend, const kv_t *v, kv_t *root, int *done)
{
    (void)k;
    if (depth == 0) { *root = *v; *done = 1; return 0; }
    if (*npend >= PEND_MAX) return irx_fail(E081, "more KIR values than the pools hold");
    PEND[*npend].name = fr[depth - 1].is_node ? fr[depth - 1].fname : 0u;
    PEND[*npend].val = *v;
    (*npend)++;
    return 0;
}

static int close_frame(kir_t *k, frame_t *fr, int *depth, uint32_t *npend, kv_t *out)
{
    frame_t *f = &fr[*depth - 1];
    uint32_t m = *npend - f->pend0, i;

    memset(out, 0, sizeof *out);
    if (f->is_node) {
        kn_t *nd = &k->node[f->node];
        if (k->nfld + m >= KIR_MAX_FLD) return irx_fail(E081, "more node fields than the field pool holds");
        nd->fld0 = k->nfld + 1u;
        nd->nfld = m;
        for (i = 0; i < m; i++) {
            k->fld[k->nfld + 1u + i].name = PEND[f->pend0 + i].name;
            k->fld[k->nfld + 1u + i].val = PEND[f->pend0 + i].val;
        }
        k->nfld += m;
        out->tag = KV_NODE;
        out->ref = f->node;
    } else {
        if (k->nitem + m >= KIR_MAX_ITEM) return irx_fail(E081, "more list items than the item pool holds");
        out->tag = KV_LIST;
        out->ref = m ? k->nitem + 1u : 0u;
        out->n = m;
        for (i = 0; i < m; i++) k->item[k->nitem + 1u + i] = PEND[f->pend0 + i].val;
        k->nitem += m;
    }
    *npend = f->pend0;
    (*depth)--;
    return 0;
}

static int parse_body(kir_t *k, const char *t, size_t n, size_t *pos)
{
    frame_t fr[KIR_MAX_DEP];
    int depth = 0, done = 0;
    uint32_t npend = 0;
    kv_t root, v;
    size_t p = *pos;

    memset(&root, 0, sizeof root);
    while (!done) {
        int c;
        while (p < n && is_ws((unsigned char)t[p])) p++;
        if (p >= n) return bad_at(E010, "truncated KIR body", p);
        c = (unsigned char)t[p];
        if (depth > 0 && (c == ')' || c == ']')) {
            if ((c == ')') != (fr[depth - 1].is_node != 0)) return bad_at(E010, "mismatched brackets", p);
            p++;
            if (close_frame(k, fr, &depth, &npend, &v)) return 1;
            if (push_val(k, fr, depth, &npend, &v, &root, &done)) return 1;
            continue;
        }
        if (depth > 0 && fr[depth - 1].is_node) {           /* a field: name=value */
            size_t b = p;
            if (!is_id0(c)) return bad_at(E010, "a malformed field token (no name)", p);
            while (p < n && is_id((unsigned char)t[p])) p++;
            if (p >= n || t[p] != '=') return bad_at(E010, "a malformed field token (no '=')", p);
            if (str_put(k, t + b, p - b, &fr[depth - 1].fname)) return 1;
            p++;
            if (p >= n || is_ws((unsigned char)t[p]) || t[p] == ')' || t[p] == ']')
                return bad_at(E010, "a field with no value after '='", p);
            c = (unsigned char)t[p];
        }
        memset(&v, 0, sizeof v);
        if (c == '(' || c == '[') {
            frame_t *f;
            if (depth >= (int)KIR_MAX_DEP) return irx_fail(E082, "KIR nested deeper than 64 levels");
            f = &fr[depth];
            memset(f, 0, sizeof *f);
            f->is_node = c == '(';
            f->pend0 = npend;
            p++;
            if (f->is_node) {
                size_t b = p;
                if (p >= n || !is_id0((unsigned char)t[p])) return bad_at(E010, "a '(' without a node kind after it", p);
                while (p < n && is_id((unsigned char)t[p])) p++;
                if (p < n && !is_ws((unsigned char)t[p]) && t[p] != ')') return bad_at(E010, "junk after a node kind", p);
                if (k->nnode + 1u >= KIR_MAX_NODE) return irx_fail(E081, "more KIR nodes than the node pool holds");
                f->node = ++k->nnode;
                if (str_put(k, t + b, p - b, &k->node[f->node].kname)) return 1;
                k->node[f->node].fld0 = 0;
                k->node[f->node].nfld = 0;
            }
            depth++;
            continue;
        }
        if (c == '"') {
            size_t b = ++p;
            while (p < n && t[p] != '"') {
                unsigned char ch = (unsigned char)t[p];
                if (ch < 0x20 || ch >= 0x7f || ch == '\\')
                    return bad_at(E013, "a KIR string with an unprintable or backslash character", p);
                p++;
            }
            if (p >= n) return bad_at(E010, "truncated KIR string", p);
            v.tag = KV_STR;
            if (str_put(k, t + b, p - b, &v.ref)) return 1;
            p++;
            if (p < n && !is_ws((unsigned char)t[p]) && t[p] != ')' && t[p] != ']')
                return bad_at(E013, "a KIR string followed by junk (a quote inside it?)", p);
        } else {
            size_t b = p;
            while (p < n && !is_delim((unsigned char)t[p])) p++;
            if (parse_atom(k, t + b, p - b, &v, b)) return 1;
        }
        if (push_val(k, fr, depth, &npend, &v, &root, &done)) return 1;
    }
    if (root.tag == KV_NODE) k->root = root.ref;
    else if (root.tag == KV_LIST && root.n == 1 && k->item[root.ref].tag == KV_NODE)
        k->root = k->item[root.ref].ref;
    while (p < n && is_ws((unsigned char)t[p])) p++;
    if (n - p < 3 || memcmp(t + p, "end", 3)) return bad_at(E010, "KIR body not followed by 'end'", p);
    p += 3;
    while (p < n && is_ws((unsigned char)t[p])) p++;
    if (p < n) return bad_at(E010, "text after the KIR 'end' line", p);
    *pos = p;
    return 0;
}

/* ---- header ---- */

typedef struct { const char *t; size_t p, end; } line_t;

static int next_tok(line_t *ln, const char **s, size_t *n)
{
    while (ln->p < ln->end && is_ws((unsigned char)ln->t[ln->p])) ln->p++;
    if (ln->p >= ln->end) return 0;
    *s = ln->t + ln->p;
    while (ln->p < ln->end && !is_ws((unsigned char)ln->t[ln->p])) ln->p++;
    *n = (size_t)(ln->t + ln->p - *s);
    return 1;
}

static int hdr_int(line_t *ln, int64_t lo, int64_t hi, int32_t *out)
{
    const char *s;
    size_t n;
    int64_t v;
    if (!next_tok(ln, &s, &n)) return bad_at(E010, "a header line with a missing number", ln->p);
    if (parse_int(s, n, &v)) return 1;
    if (v < lo || v > hi) return bad_at(E014, "a header number outside its range", ln->p);
    *out = (int32_t)v;
    return 0;
}

static int hdr_name(kir_t *k, line_t *ln, uint32_t *off, char *copy)
{
    const char *s;
    size_t n, i;
    if (!next_tok(ln, &s, &n)) return bad_at(E010, "a header line with a missing name", ln->p);
    if (n > KIR_MAX_NAME || !is_id0((unsigned char)s[0])) return bad_at(E012, "a name that is not a valid identifier", ln->p);
    for (i = 1; i < n; i++)
        if (!is_id((unsigned char)s[i])) return bad_at(E012, "a name that is not a valid identifier", ln->p);
    if (copy) { memcpy(copy, s, n); copy[n] = '\0'; }
    return str_put(k, s, n, off);
}

static int hdr_end(line_t *ln)
{
    const char *s;
    size_t n;
    return next_tok(ln, &s, &n) ? bad_at(E010, "extra text at the end of a header line", ln->p) : 0;
}

dt_t kir_dtype(const char *s)
{
    if (!strcmp(s, "f32")) return DT_F32;
    if (!strcmp(s, "bf16")) return DT_BF16;
    return DT_OTHER;
}

static int hdr_arg(kir_t *k, line_t *ln)
{
    ka_t *a;
    const char *s;
    size_t n;
    int32_t idx, rank, d;
    char dts[KIR_MAX_NAME + 1];

    if (k->narg >= KIR_MAX_ARG) return irx_fail(E081, "more kernel arguments than 32");
    a = &k->arg[k->narg];
    memset(a, 0, sizeof *a);
    if (hdr_int(ln, 0, INT32_MAX, &idx)) return 1;
    if ((uint32_t)idx != k->narg) return bad_at(E010, "an arg line out of order", ln->p);
    if (hdr_name(k, ln, &a->name, NULL)) return 1;
    if (!next_tok(ln, &s, &n)) return bad_at(E010, "an arg line without a kind", ln->p);
    if (n == 2 && !memcmp(s, "in", 2)) a->kind = KA_IN;
    else if (n == 3 && !memcmp(s, "out", 3)) a->kind = KA_OUT;
    else if (n == 5 && !memcmp(s, "const", 5)) a->kind = KA_CONST;
    else return bad_at(E010, "an arg kind other than in, const or out", ln->p);
    if (!next_tok(ln, &s, &n)) return bad_at(E010, "an arg line without a dtype", ln->p);
    if (n > KIR_MAX_NAME) n = KIR_MAX_NAME;
    memcpy(dts, s, n);
    dts[n] = '\0';
    a->dt = (uint8_t)kir_dtype(dts);
    if (hdr_int(ln, 0, INT32_MAX, &rank)) return 1;
    if ((uint32_t)rank > KIR_MAX_DIM) return irx_fail(E081, "a buffer of rank over 8");
    a->rank = (uint8_t)rank;
    for (d = 0; d < rank; d++)
        if (hdr_int(ln, 1, INT32_MAX, &a->dim[d])) return 1;
    k->narg++;
    return hdr_end(ln);
}

/* 0 go on, 2 `body` seen, 1 error. `have`: bit 0 kernel, bit 1 launch. */
static int hdr_line(kir_t *k, line_t *ln, unsigned *have)
{
    const char *s;
    size_t n;
    int i;
    uint32_t off;

    if (!next_tok(ln, &s, &n)) return 0;
    if (n == 6 && !memcmp(s, "kernel", 6) && !(*have & 1u)) {
        *have |= 1u;
        if (hdr_name(k, ln, &off, k->name)) return 1;
        return hdr_end(ln);
    }
    if (n == 6 && !memcmp(s, "launch", 6) && !(*have & 2u)) {
        *have |= 2u;
        for (i = 0; i < 3; i++) if (hdr_int(ln, 1, INT32_MAX, &k->grid[i])) return 1;
        for (i = 0; i < 3; i++) if (hdr_int(ln, 1, INT32_MAX, &k->block[i])) return 1;
        if (hdr_int(ln, 0, INT32_MAX, &k->smem)) return 1;
        return hdr_end(ln);
    }
    if (n == 3 && !memcmp(s, "arg", 3)) return hdr_arg(k, ln);
    if (n == 4 && !memcmp(s, "zero", 4)) {
        if (k->nzero >= KIR_MAX_ARG) return irx_fail(E081, "more zero lines than 32");
        if (hdr_name(k, ln, &k->zero[k->nzero], NULL)) return 1;
        k->nzero++;
        return hdr_end(ln);
    }
    if (n == 4 && !memcmp(s, "body", 4)) {
        if (*have != 3u) return bad_at(E015, "a KIR body before its kernel or launch line", ln->p);
        return hdr_end(ln) ? 1 : 2;
    }
    return bad_at(E010, "an unknown or repeated KIR header line", ln->p);
}

int kir_load(kir_t *k, const char *txt, size_t len)
{
    size_t p = 0;
    unsigned have = 0;
    int rc = 0;
    line_t ln;
    const char *s;
    size_t n;

    if (!k || !txt) return irx_fail(E010, "no KIR text");
    if (len > KIR_MAX_TEXT) return irx_fail(E080, "KIR text over 1 MiB");
    memset(k->name, 0, sizeof k->name);
    memset(k->grid, 0, sizeof k->grid);
    memset(k->block, 0, sizeof k->block);
    k->smem = 0;
    k->narg = k->nzero = k->root = 0;
    k->nnode = k->nfld = k->nitem = 0;
    k->nstr = 1u;
    k->str[0] = '\0';
    memset(&k->node[0], 0, sizeof k->node[0]);
    memset(&k->item[0], 0, sizeof k->item[0]);
    /* first line: exactly `kir 1` */
    ln.t = txt; ln.p = 0; ln.end = 0;
    while (ln.end < len && txt[ln.end] != '\n') ln.end++;
    if (!next_tok(&ln, &s, &n) || n != 3 || memcmp(s, "kir", 3)) return bad_at(E010, "KIR text without a 'kir 1' first line", 0);
    if (!next_tok(&ln, &s, &n) || n != 1 || s[0] != '1') return bad_at(E010, "a KIR format version other than 1", ln.p);
    if (hdr_end(&ln)) return 1;
    p = ln.end < len ? ln.end + 1 : len;
    while (rc == 0) {
        if (p >= len) return bad_at(E010, "KIR text ends before its body", p);
        ln.t = txt; ln.p = p; ln.end = p;
        while (ln.end < len && txt[ln.end] != '\n') ln.end++;
        p = ln.end < len ? ln.end + 1 : len;
        rc = hdr_line(k, &ln, &have);
    }
    if (rc != 2) return 1;
    return parse_body(k, txt, len, &p);
}

/* ---- lookup ---- */

const char *kir_str(const kir_t *k, uint32_t off)
{
    return off >= k->nstr ? "" : k->str + off;
}

const kn_t *kir_node(const kir_t *k, const kv_t *v)
{
    if (!v || v->tag != KV_NODE || v->ref == 0 || v->ref > k->nnode) return NULL;
    return &k->node[v->ref];
}

const kv_t *kir_fld(const kir_t *k, const kn_t *nd, const char *name)
{
    uint32_t i;
    if (!nd || !name || !nd->nfld || nd->fld0 == 0 || nd->fld0 + nd->nfld - 1u > k->nfld) return NULL;
    for (i = 0; i < nd->nfld; i++) {
        const kf_t *f = &k->fld[nd->fld0 + i];
        if (strcmp(kir_str(k, f->name), name) == 0) return &f->val;
    }
    return NULL;
}

const kv_t *kir_item(const kir_t *k, const kv_t *lst, uint32_t i)
{
    if (!lst || lst->tag != KV_LIST || i >= lst->n || lst->ref == 0 || lst->ref + i > k->nitem) return NULL;
    return &k->item[lst->ref + i];
}

int kir_is(const kir_t *k, const kn_t *nd, const char *kind)
{
    return nd && strcmp(kir_str(k, nd->kname), kind) == 0;
}
