/* mm_attn.c -- launchers for the matmul and attention templates: tensor maps for the TMA
 * loads, the tcgen05 path when the shape and alignment allow it, the SIMT path otherwise. */
#include <string.h>
#include "irx_int.h"
#include "irx_kparams.h"
#include "launch.h"

#define MM_BN 256
#define MM_STAGES 4
#define MM_SMEM (MM_STAGES * (128 * 64 * 2 + 256 * 64 * 2) + 1024 + 256)
#define M2_SMEM(st) ((st) * 2 * (128 * 64 * 2) + 1024 + 256)
#define MW_SMEM (4 * 3 * (128 * 64 * 2) + 8 * 32 * 128 + 1024 + 256)

static int a16(const void *p) { return ((unsigned long long)(size_t)p & 15u) == 0; }

static int grid_for(irx_dev_t *d, int k, int block, size_t smem, long long want)
{
    int occ = 1;
    long long g;
    if (irx_dev_occupancy(d, k, block, smem, &occ)) occ = 1;
    g = (long long)d->sms * occ;
    if (want < g) g = want;
    return (int)(g < 1 ? 1 : g);
}

/* Failure injection for tests (irx_inject): the next tcgen05 matmul launch issues none of its
 * loads and bounds its device waits by INJ_WAIT_NS, so its waits run out with no copy in flight
 * and no fault; the kernel stops, frees TMEM and returns, and irx_check reports E092. Read and
 * cleared under the launch lock. */
static int INJ_NO_LOADS;
static unsigned long long INJ_WAIT_NS;

void irx_inject_mm(int on, unsigned long long wait_ns)
{
    INJ_NO_LOADS = on;
    INJ_WAIT_NS = wait_ns;
}

int irx_launch_mm(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    const irx_mm_t *m = &p->u.mm;
    static irx_kmm_t k;
    long long units = (m->n + MM_BN - 1) / MM_BN, u0, u1;
    memset(&k, 0, sizeof k);
    irx_unit_range(units, s, ns, &u0, &u1);
    if (u0 >= u1) return 0;
    k.a = args[m->a_arg];
    k.b = args[m->b_arg];
    k.c = args[m->c_arg];
    k.m = m->m; k.n = m->n; k.k = m->k;
    k.n0 = u0 * MM_BN;
    k.n1 = u1 * MM_BN < m->n ? u1 * MM_BN : m->n;
    k.err = (unsigned *)(size_t)d->err;
    k.b_kmajor = m->b_kmajor;
    if (INJ_NO_LOADS && m->dt == DT_BF16) {
        k.no_loads = 1;
        k.wait_ns = INJ_WAIT_NS;
        INJ_NO_LOADS = 0;
    }
    if (m->dt != DT_BF16) {
        long long tiles = ((m->m + 63) / 64) * ((k.n1 - k.n0 + 63) / 64);
        return irx_dev_launch(d, K_MM_F32, (unsigned)grid_for(d, K_MM_F32, 256, 0, tiles), 256, 0, 1, st, &k);
    }
    if ((m->k % 8) || (!m->b_kmajor && (m->n % 8)) || !a16(k.a) || !a16(k.b) || m->m > 0x7fffffff || m->n > 0x7fffffff) {
        long long tiles = ((m->m + 63) / 64) * ((k.n1 - k.n0 + 63) / 64);
        return irx_dev_launch(d, K_MM_BF16_SIMT, (unsigned)grid_for(d, K_MM_BF16_SIMT, 256, 0, tiles), 256, 0, 1, st, &k);
    }
    {
        /* CTA pairs (256x256 tiles, cta_group::2) unless one 128-row tile covers M */
        const int pair = m->m > 128;
        cuuint64_t dims[2], strides[1];
        cuuint32_t box[2];
        long long tiles;
        dims[0] = (cuuint64_t)m->k; dims[1] = (cuuint64_t)m->m;
        strides[0] = (cuuint64_t)m->k * 2;
        box[0] = 64; box[1] = 128;
        if (irx_dev_tmap(&k.tma_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)k.a, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)) return 1;
        if (m->b_kmajor) {
            dims[0] = (cuuint64_t)m->k; dims[1] = (cuuint64_t)m->n;
            strides[0] = (cuuint64_t)m->k * 2;
            box[0] = 64; box[1] = pair ? 128 : 256;
        } else {
            dims[0] = (cuuint64_t)m->n; dims[1] = (cuuint64_t)m->k;
            strides[0] = (cuuint64_t)m->n * 2;
            box[0] = 64; box[1] = 64;
        }
        if (irx_dev_tmap(&k.tma_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)k.b, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)) return 1;
        if (pair) {
            /* 256x512 tiles with a TMA-store epilogue when C's rows can be stored by TMA (16-byte
             * aligned rows); else the 256x256 pair tile with per-thread stores. Measured on B200
             * (10-launch bursts, A-B-B-A): 256x512 1546-1562 / 1575-1588 TFLOP/s at 8192^3 /
             * 16384x4096x14336 against 1455-1493 / 1486-1494 for 256x256; raster groups of 16
             * tile rows were best or within 1% (cuBLAS 1566-1594 / 1601-1612 in the same runs). */
            int fit = d->sms / 2;
            const int stg = 6, grp = 16, wide = (m->n % 8) == 0 && a16(k.c);
            if (wide) {
                k.group = (uint8_t)grp;
                dims[0] = (cuuint64_t)k.n1; dims[1] = (cuuint64_t)m->m;      /* this launch's columns only */
                strides[0] = (cuuint64_t)m->n * 2;
                box[0] = 64; box[1] = 32;
                if (irx_dev_tmap(&k.tma_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k.c, dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B)) return 1;
                tiles = ((m->m + 255) / 256) * ((k.n1 - k.n0 + 511) / 512);
                if (irx_dev_max_clusters(d, K_MM_BF16_WIDE, (unsigned)(2 * fit), 192, MW_SMEM, 2, &fit)) return 1;
                if (tiles < fit) fit = (int)tiles;
                return irx_dev_launch(d, K_MM_BF16_WIDE, (unsigned)(2 * fit), 192, MW_SMEM, 2, st, &k);
            }
            k.stages = (uint8_t)stg;
            k.group = (uint8_t)grp;
            tiles = ((m->m + 255) / 256) * ((k.n1 - k.n0 + MM_BN - 1) / MM_BN);
            if (irx_dev_max_clusters(d, K_MM_BF16_PAIR, (unsigned)(2 * fit), 192, M2_SMEM(stg), 2, &fit)) return 1;
            if (tiles < fit) fit = (int)tiles;
            return irx_dev_launch(d, K_MM_BF16_PAIR, (unsigned)(2 * fit), 192, M2_SMEM(stg), 2, st, &k);
        }
        tiles = ((m->m + 127) / 128) * ((k.n1 - k.n0 + MM_BN - 1) / MM_BN);
        return irx_dev_launch(d, K_MM_BF16, (unsigned)(tiles < d->sms ? tiles : d->sms), 192, MM_SMEM, 1, st, &k);
    }
}

#define AT_SMEM (6 * 32768 + 1024)     /* Q x2, K x2, V x2 tiles; barriers and the TMEM slot */

int irx_launch_attn(const irx_plan_int_t *p, irx_dev_t *d, unsigned s, unsigned ns, void *const *args, void *st)
{
    const irx_at_t *a = &p->u.at;
    static irx_kat_t k;
    long long units = a->b * a->h, u0, u1;
    float sc;
    memset(&k, 0, sizeof k);
    irx_unit_range(units, s, ns, &u0, &u1);
    if (u0 >= u1) return 0;
    memcpy(&sc, &a->scale_bits, 4);
    k.q = args[a->q_arg]; k.k = args[a->k_arg]; k.v = args[a->v_arg]; k.o = args[a->o_arg];
    k.b = a->b; k.h = a->h; k.s = a->s; k.d = a->d;
    k.sq = a->sq; k.sk = a->sk; k.dqk = a->dqk; k.dv = a->dv; k.k_t = a->k_t;
    k.bh0 = u0; k.bh1 = u1;
    k.scale = sc;
    memcpy(&k.divisor, &a->div_bits, 4);
    k.scale_div = a->scale_div;
    k.causal = a->causal;
    k.err = (unsigned *)(size_t)d->err;
    if (a->dt == DT_BF16 && a->sq == a->sk && a->dqk == 128 && a->dv == 128 && !a->k_t && a->s % 128 == 0 &&
        a->b * a->h * a->s < 0x7fffffffLL &&
        a16(k.q) && a16(k.k) && a16(k.v) && a16(k.o)) {
        cuuint64_t dims[2], strides[1];
        cuuint32_t box[2];
        dims[0] = (cuuint64_t)a->d; dims[1] = (cuuint64_t)(a->b * a->h * a->s);
        strides[0] = (cuuint64_t)a->d * 2;
        box[0] = 64; box[1] = 128;
        if (irx_dev_tmap(&k.tma_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)k.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
            irx_dev_tmap(&k.tma_k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)k.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
            irx_dev_tmap(&k.tma_v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)k.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return 1;
        {
            /* One CTA per SM; the CTAs take (batch*head, 256-query) units from a counter in
             * global memory: this launch's own scratch slot, zeroed here on the launch's stream. */
            const long long units = (a->s / 128 + 1) / 2 * (u1 - u0);
            const unsigned grid = (unsigned)(units < d->sms ? units : d->sms);
            irx_slot_t sl;
            irx_dev_slot(d, &sl);
            k.sched = (unsigned *)(size_t)sl.sched;
            if (irx_dev_memset32(sl.sched, 0, 1, st)) return 1;
            return irx_dev_launch(d, K_ATTN_BF16, grid, 384, AT_SMEM, 1, st, &k);
        }
    }
    if (a->dqk > 128 || a->dv > 128) return irx_fail(E042, "an attention with a head size over 128");
    {
        int kk = a->dt == DT_BF16 ? K_ATTN_BF16_SIMT : K_ATTN_F32;
        long long work = (u1 - u0) * ((a->sq + 127) / 128);
        return irx_dev_launch(d, kk, (unsigned)grid_for(d, kk, 128, 0, work), 128, 0, 1, st, &k);
    }
}
