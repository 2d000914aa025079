// attn.cu -- the attention templates: O = softmax(Q K^T * scale [causal]) V over [B, H, S, D].
//
// irx_attn_bf16: flash attention on the 5th-generation tensor cores, D = 128, S a multiple of 128.
// One CTA per SM takes units of (batch*head, 256 queries) = two 128-query tiles from a global
// counter, head by head so the CTAs running at once share K and V in L2; within a head the
// heaviest causal blocks go first. 384 threads in three warpgroups (setmaxnreg: 216 registers
// for the two softmax warpgroups, 72 for the third):
//   * warp 8 (TMA): both Q tiles of a unit, then K_j and V_j tiles of 128 keys into two 2-deep
//     rings (128-byte swizzle, 64-column boxes); each CTA loads its own tiles;
//   * warp 9 (MMA): S_t = Q_t K_j^T into TMEM (128 f32 columns per tile t) and O_t += P_t V_j into
//     a TMEM accumulator per tile, P_t read from TMEM. Issued as P0 V, S0', P1 V, S1' per key
//     tile, so each tile's softmax runs under the other tile's MMAs;
//   * warps 0-3 / 4-7 (softmax of tile 0 / 1): one thread per query row reads the row's 128
//     scores from TMEM, keeps the running max m and sum l (log2 domain, scale folded in), and
//     writes P = 2^(s - m) as bf16 over the scores' first 64 TMEM columns; three exp pairs in
//     four on the MUFU, the fourth on the FMA pipe. At the end it writes O / l. O is rescaled in
//     TMEM only when a row's max grows by more than 8 (a factor of 256): until then the stale
//     max is kept for that row's P and l alike, which the final division cancels exactly.
// Every wait is bounded; a timeout sets the error word and the roles stop.
//
// irx_attn_f32 / irx_attn_bf16_simt: one thread per query row, keys streamed through shared
// memory, the online softmax of the KIR graph statement by statement (dot product by ascending
// d, max, two exps, rescaled sum and output; src/isel.c:1301-1319), for f32 graphs and for
// shapes the tensor-core path does not take.

#include "tc.cuh"

#define AT_BM 128
#define AT_BN 128
#define AT_D 128
#define AT_TILE_BYTES (128 * AT_D * 2)      // 32 KiB: a 128-row x 128-col bf16 tile
#define AT_HALF (AT_TILE_BYTES / 2)         // one 64-column swizzle block

__device__ __forceinline__ int at_wait(uint64_t *bar, uint32_t parity, unsigned *err)
{
    if (irx_mbar_wait(bar, parity)) return 1;
    if (err) atomicOr(err, IRX_KERR_TIMEOUT);
    return 0;
}

// A 128x128 tile in two 64-column blocks: the 16-column K-step k starts at block k/4, +32 bytes
// per step inside the 128-byte swizzled row.
__device__ __forceinline__ uint64_t at_kmajor_desc(uint32_t base, int k)
{
    return umma_desc_sw128(base + (k >> 2) * AT_HALF + (k & 3) * 32, 16, 1024);
}

// 2^x on the MUFU unit (ex2.approx, flush to zero).
__device__ __forceinline__ float at_ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float at_max3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// All 128 f32 columns of this thread's TMEM lane, with the wait in the same statement so no
// use of the registers can be scheduled before the load has landed.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&v)[128])
{
    uint32_t r[128];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
                 "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                 "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
                 "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
                 "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, "
                 "%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, "
                 "%80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, "
                 "%96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, "
                 "%112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"
                 "tcgen05.wait::ld.sync.aligned;"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
                   "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
                   "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
                   "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
                   "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
                   "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
                   "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
                   "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
                   "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
                   "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
                   "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
                   "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
                   "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
                 : "r"(taddr) : "memory");
#pragma unroll
    for (int i = 0; i < 128; i++) v[i] = __uint_as_float(r[i]);
}

// 64 packed columns (128 bf16 of P) into this thread's TMEM lane, then wait for the stores.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&v)[64])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {"
                 "%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
                 "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, "
                 "%33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, "
                 "%49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};\n\t"
                 "tcgen05.wait::st.sync.aligned;"
                 :: "r"(taddr),
                    "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                    "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
                    "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
                    "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]),
                    "r"(v[32]), "r"(v[33]), "r"(v[34]), "r"(v[35]), "r"(v[36]), "r"(v[37]), "r"(v[38]), "r"(v[39]),
                    "r"(v[40]), "r"(v[41]), "r"(v[42]), "r"(v[43]), "r"(v[44]), "r"(v[45]), "r"(v[46]), "r"(v[47]),
                    "r"(v[48]), "r"(v[49]), "r"(v[50]), "r"(v[51]), "r"(v[52]), "r"(v[53]), "r"(v[54]), "r"(v[55]),
                    "r"(v[56]), "r"(v[57]), "r"(v[58]), "r"(v[59]), "r"(v[60]), "r"(v[61]), "r"(v[62]), "r"(v[63])
                 : "memory");
}

// D (TMEM) += A (TMEM, K-major: lane = row, 2 bf16 per column) x B (shared-memory descriptor).
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ uint32_t at_pack_bf16(float lo, float hi)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// a * b + c, clamped to [0, 1] (NaN gives 0).
__device__ __forceinline__ float at_ffma_sat(float a, float b, float c)
{
    float d;
    asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// One score row of a tile: P = 2^(s * sl2 - m) packed as bf16 pairs into pk, returns the sum of
// P (f32). Three pairs in four go to the MUFU (ex2, then cvt to bf16), the fourth to the FMA pipe.
// Measured on B200, 3:1 beats both 1:1 and all-MUFU: the cubic costs issue slots that a 1:1
// split runs short of.
//
// The FMA-pipe pair: x = s * sl2 - m is clamped to [-126, 127] by a saturating FMA that maps it
// to y = (x + 126) / 253 in [0, 1] (one instruction per element, both bounds, and -inf gives 0).
// t = 253 y + (1.5 * 2^23 - 126) = 1.5 * 2^23 + n rounds x to the integer n, and f = x - n in
// [-1/2, 1/2] comes from the same y. 2^f is a cubic fitted here for minimum relative error on
// [-1/2, 1/2] (max 7.5e-5, far below the bf16 P it feeds, 2^-9), and n goes into the exponent
// field: the low bits of t hold n, so shifting them up by 23 adds n to the exponent. With
// n >= -126 the exponent never wraps into the sign bit, so no integer clamp is needed; a masked
// score (-inf) gives 2^-126 (1.2e-38), which no sum of P can notice. Rounding to bf16 is by
// integer adds: round half up, which differs from round-to-nearest-even only at exact ties.
__device__ __forceinline__ float at_softmax_row(const float (&v)[128], float sl2, float m, uint32_t (&pk)[64])
{
    float2 sa = make_float2(0.0f, 0.0f), sb = make_float2(0.0f, 0.0f);
    const float2 s2 = make_float2(sl2, sl2), nm = make_float2(-m, -m);
    const float ks = sl2 * (1.0f / 253.0f), kc = (126.0f - m) * (1.0f / 253.0f);
    const float2 k253 = make_float2(253.0f, 253.0f), kmg = make_float2(12582912.0f - 126.0f, 12582912.0f - 126.0f);
#pragma unroll
    for (int i = 0; i < 64; i++) {
        if ((i & 3) != 3) {
            const float2 x = __ffma2_rn(make_float2(v[2 * i], v[2 * i + 1]), s2, nm);
            const float p0 = at_ex2(x.x), p1 = at_ex2(x.y);
            pk[i] = at_pack_bf16(p0, p1);
            sa = __fadd2_rn(sa, make_float2(p0, p1));
        } else {
            const float2 y = make_float2(at_ffma_sat(v[2 * i], ks, kc), at_ffma_sat(v[2 * i + 1], ks, kc));
            const float2 t = __ffma2_rn(y, k253, kmg);
            const float2 nn = __fadd2_rn(kmg, make_float2(-t.x, -t.y));
            const float2 f = __ffma2_rn(y, k253, nn);
            float2 q = __ffma2_rn(make_float2(0.055171319384097875f, 0.055171319384097875f), f,
                                  make_float2(0.2426105373823389f, 0.2426105373823389f));
            q = __ffma2_rn(q, f, make_float2(0.6932609854947172f, 0.6932609854947172f));
            q = __ffma2_rn(q, f, make_float2(0.9999281096694117f, 0.9999281096694117f));
            const uint32_t r0 = __float_as_uint(q.x) + (__float_as_uint(t.x) << 23);
            const uint32_t r1 = __float_as_uint(q.y) + (__float_as_uint(t.y) << 23);
            pk[i] = __byte_perm(r0 + 0x8000u, r1 + 0x8000u, 0x7632);
            sb = __fadd2_rn(sb, make_float2(__uint_as_float(r0), __uint_as_float(r1)));
        }
    }
    return (sa.x + sa.y) + (sb.x + sb.y);
}

#define AT_THREADS 384      // two softmax warpgroups (one per query tile), then TMA warp, MMA warp, 2 idle
#define AT_REG_SOFTMAX 216  // setmaxnreg split of the launch's 384 x 168 registers:
#define AT_REG_OTHER 72     //   2 x 128 x 216 + 128 x 72 = 384 x 168 (and 216 + 216 + 72 per SM quarter)

__device__ __forceinline__ void at_reg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(AT_REG_OTHER)); }
__device__ __forceinline__ void at_reg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(AT_REG_SOFTMAX)); }

// TMEM columns: S_t (scores of query tile t, 128 f32; P_t overwrites its first 64 columns as
// packed bf16) at 128 t, O_t (the output accumulator) at 256 + 128 t.
// ---- the tcgen05 kernel: one CTA per SM (persistent) over all units ----
//
// A unit is (batch*head, block of 256 queries): two 128-query tiles of one head, each with its
// own softmax warpgroup, sharing every K and V tile. Units are numbered head-major and heaviest
// causal block first. CTAs take units dynamically: the TMA thread claims the next unit index from
// a counter in global memory (p.sched, zeroed by the host before the launch) and hands it to the
// MMA thread and the softmax warps through a two-slot ring in shared memory; -1 ends the CTA. A
// CTA that drew light causal blocks thus takes more of them, and the order stays head-major, so
// the CTAs at work share a few heads' K and V through L2. The K/V ring and every barrier's phase
// count run on across units. Q is released as soon as the unit's last score MMA has read it
// (q_empty), so the next unit's Q loads while this unit's last softmax, P V products and output
// write-back run; the next unit's first P V waits until this unit's O has been read out of TMEM
// (o_free). Measured on B200 against one unit per CTA (the form this replaced), A-B-B-A order:
// [16, 32, 4096, 128] 1196-1223 against 1169-1202 TFLOP/s non-causal, 997-1031 against 922-950
// causal.

extern "C" __global__ void __launch_bounds__(AT_THREADS, 1) irx_attn_bf16(const __grid_constant__ irx_kat_t p)
{
    irx_pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw;
    if (irx_smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0 && p.err) atomicOr(p.err, IRX_KERR_TIMEOUT);
        return;
    }
    unsigned char *sq = smem;                                 // Q tiles 0 and 1
    unsigned char *sk = smem + 2 * AT_TILE_BYTES;             // K ring, 2 slots
    unsigned char *sv = smem + 4 * AT_TILE_BYTES;             // V ring, 2 slots
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 6 * AT_TILE_BYTES);
    uint64_t *q_full = bars, *k_full = bars + 1, *k_empty = bars + 3, *v_full = bars + 5, *v_empty = bars + 7;
    uint64_t *s_full = bars + 9, *p_full = bars + 11, *pv_done = bars + 13, *done = bars + 15;
    uint64_t *q_empty = bars + 16, *o_free = bars + 17;
    uint64_t *u_full = bars + 20, *u_empty = bars + 22;       // the unit handout ring, 2 slots
    volatile int *u_id = reinterpret_cast<volatile int *>(bars + 24);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 25);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (int)p.s;
    const int nqt = S / AT_BM, nqb = (nqt + 1) / 2;
    const int nunits = (int)(p.bh1 - p.bh0) * nqb;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 24; i++)                        // u_empty: the MMA thread and 8 softmax warps
            irx_mbar_init(&bars[i], (i == 11 || i == 12 || i == 17 || i == 18) ? 128 : (i >= 22 ? 9 : 1));
        irx_fence_mbar_init();
        tma_prefetch_desc(&p.tma_q);
        tma_prefetch_desc(&p.tma_k);
        tma_prefetch_desc(&p.tma_v);
    }
    if (warp == 9) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    // Each warpgroup sets its register budget at the top of its own branch, and the branches
    // never rejoin: warpgroup 2 frees TMEM once the softmax warps have arrived on barrier 1.
    if (warp >= 8) {
      at_reg_dec();
      if (warp == 8) {
        if (elect_one()) {                                    // TMA
            bool ok = true;
            int kv = 0, uq = 0;
            for (int uc = 0; ok; uc++) {
                const int us = uc & 1;
                if (!(ok = at_wait(&u_empty[us], ((uc >> 1) & 1) ^ 1, p.err))) break;
                int w = (int)atomicAdd(p.sched, 1u);
                if (w >= nunits) w = -1;
                u_id[us] = w;
                irx_mbar_arrive(&u_full[us]);
                if (w < 0) break;
                const int qb = nqb - 1 - w % nqb, bh = (int)p.bh0 + w / nqb, qt0 = 2 * qb;
                const int has1 = qt0 + 1 < nqt;
                const int nmax = p.causal ? qt0 + 1 + has1 : nqt;
                const int krow0 = bh * S;
                if (uq > 0 && !(ok = at_wait(q_empty, (uq - 1) & 1, p.err))) break;
                irx_mbar_expect_tx(q_full, has1 ? 2 * AT_TILE_BYTES : AT_TILE_BYTES);
                for (int t = 0; t < 1 + has1; t++) {
                    tma_load_2d(sq + t * AT_TILE_BYTES, &p.tma_q, 0, krow0 + (qt0 + t) * AT_BM, q_full);
                    tma_load_2d(sq + t * AT_TILE_BYTES + AT_HALF, &p.tma_q, 64, krow0 + (qt0 + t) * AT_BM, q_full);
                }
                for (int t = 0; t <= nmax && ok; t++) {
                    if (t < nmax) {
                        const int g = kv + t, sl = g & 1;
                        if (!(ok = at_wait(&k_empty[sl], ((g >> 1) & 1) ^ 1, p.err))) break;
                        irx_mbar_expect_tx(&k_full[sl], AT_TILE_BYTES);
                        tma_load_2d(sk + sl * AT_TILE_BYTES, &p.tma_k, 0, krow0 + t * AT_BN, &k_full[sl]);
                        tma_load_2d(sk + sl * AT_TILE_BYTES + AT_HALF, &p.tma_k, 64, krow0 + t * AT_BN, &k_full[sl]);
                    }
                    if (t >= 1) {
                        const int g = kv + t - 1, sl = g & 1;
                        if (!(ok = at_wait(&v_empty[sl], ((g >> 1) & 1) ^ 1, p.err))) break;
                        irx_mbar_expect_tx(&v_full[sl], AT_TILE_BYTES);
                        tma_load_2d(sv + sl * AT_TILE_BYTES, &p.tma_v, 0, krow0 + (t - 1) * AT_BN, &v_full[sl]);
                        tma_load_2d(sv + sl * AT_TILE_BYTES + AT_HALF, &p.tma_v, 64, krow0 + (t - 1) * AT_BN, &v_full[sl]);
                    }
                }
                kv += nmax;
                uq++;
            }
        }
      } else if (warp == 9) {
        if (elect_one()) {                                    // MMA
            // Order per key tile j: P0_j V_j, S0_{j+1}, P1_j V_j, S1_{j+1}. S_t of tile j+1 goes into
            // the columns P_t of tile j occupies, issued after the MMA that reads them (tcgen05.mma
            // from one thread execute in issue order). Query tile 1's softmax runs under tile 0's
            // MMAs and the other way round.
            const uint32_t id_qk = umma_idesc_bf16(AT_BM, AT_BN, 0);
            const uint32_t id_pv = umma_idesc_bf16(AT_BM, AT_D, 1);
            const uint32_t sq_a = irx_smem_u32(sq), sk_a = irx_smem_u32(sk), sv_a = irx_smem_u32(sv);
            bool ok = true;
            int kv = 0, uq = 0, it0 = 0, it1 = 0, uo0 = 0, uo1 = 0;
            for (int uc = 0; ok; uc++) {
                const int us = uc & 1;
                if (!(ok = at_wait(&u_full[us], (uc >> 1) & 1, p.err))) break;
                const int w = u_id[us];
                irx_mbar_arrive(&u_empty[us]);
                if (w < 0) break;
                const int qb = nqb - 1 - w % nqb, qt0 = 2 * qb;
                const int has1 = qt0 + 1 < nqt;
                const int n0 = p.causal ? qt0 + 1 : nqt, n1 = has1 ? (p.causal ? qt0 + 2 : nqt) : 0;
                const int nmax = n0 > n1 ? n0 : n1;
                int sleft = n0 + n1;                          // score MMAs of this unit still to issue
                if (!(ok = at_wait(q_full, uq & 1, p.err))) break;
                for (int j = -1; j < nmax && ok; j++) {
                    // j = -1: the first scores; then per key tile j: P_t V_j and S_t of tile j + 1
#pragma unroll
                    for (int t = 0; t < 2; t++) {
                        const int nt = t ? n1 : n0;
                        if (!ok) break;
                        if (j >= 0 && j < nt) {               // O_t (+)= P_t V_j
                            const int g = kv + j;
                            if (j == 0 && (t ? uo1 : uo0) > 0 &&
                                !(ok = at_wait(&o_free[t], ((t ? uo1 : uo0) - 1) & 1, p.err))) break;
                            if (!(ok = at_wait(&p_full[t], ((t ? it1 : it0) + j) & 1, p.err))) break;
                            if (!(ok = at_wait(&v_full[g & 1], (g >> 1) & 1, p.err))) break;
                            tc_fence_after();
                            const uint32_t bv = sv_a + (g & 1) * AT_TILE_BYTES;
#pragma unroll
                            for (int kk = 0; kk < AT_BN / 16; kk++)
                                umma_bf16_tmem_a(tbase + 256 + t * AT_D, tbase + t * AT_BN + kk * 8,
                                                 umma_desc_sw128(bv + kk * 16 * 128, AT_HALF, 1024), id_pv, (j | kk) != 0);
                            umma_commit(&pv_done[t]);
                        }
                        if (j + 1 < nt) {                     // S_t = Q_t K_{j+1}^T
                            const int g = kv + j + 1;
                            if (!(ok = at_wait(&k_full[g & 1], (g >> 1) & 1, p.err))) break;
                            tc_fence_after();
                            const uint32_t aq = sq_a + t * AT_TILE_BYTES, bk = sk_a + (g & 1) * AT_TILE_BYTES;
#pragma unroll
                            for (int kk = 0; kk < AT_D / 16; kk++)
                                umma_bf16(tbase + t * AT_BN, at_kmajor_desc(aq, kk), at_kmajor_desc(bk, kk), id_qk, kk > 0);
                            umma_commit(&s_full[t]);
                            if (--sleft == 0) umma_commit(q_empty);   // Q is free once these scores land
                        }
                    }
                    if (!ok) break;
                    if (j >= 0) umma_commit(&v_empty[(kv + j) & 1]);
                    if (j + 1 < nmax) umma_commit(&k_empty[(kv + j + 1) & 1]);
                }
                if (!ok) break;
                if (n0 > 0) { it0 += n0; uo0++; }
                if (n1 > 0) { it1 += n1; uo1++; }
                kv += nmax;
                uq++;
            }
            umma_commit(done);
            at_wait(done, 0, p.err);
        }
        asm volatile("bar.sync 1, 288;" ::: "memory");         // the softmax warps are done with TMEM
        tc_fence_after();
        tmem_dealloc(tbase, 512);
      }
    } else {                                                   // softmax: warps 0-3 tile 0, 4-7 tile 1
        at_reg_inc();
        // One thread per query row (TMEM lane): it reads the row's 128 scores, keeps the running
        // max m and sum l (log2 domain, scale folded in), writes P = 2^(s - m) as bf16 over the
        // scores' first 64 columns for the P V MMA, and at the end writes O / l. O is rescaled
        // in TMEM only when the row's max grows by more than 8 (a factor of 256): until then the
        // stale max is kept for the row's P and l alike, which the final division cancels.
        const int t = warp >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t tl = (uint32_t)(q * 32) << 16;
        const uint32_t tS = tbase + tl + t * AT_BN, tO = tbase + tl + 256 + t * AT_D;
        const float sl2 = p.scale * 1.4426950408889634f;
        bool ok = true;
        int it = 0;
        for (int uc = 0; ok; uc++) {
            const int us = uc & 1;
            ok = __all_sync(0xffffffffu, at_wait(&u_full[us], (uc >> 1) & 1, p.err));
            if (!ok) break;
            const int w = u_id[us];
            __syncwarp();
            if (lane == 0) irx_mbar_arrive(&u_empty[us]);
            if (w < 0) break;
            const int qtile = 2 * (nqb - 1 - w % nqb) + t;
            if (qtile >= nqt) continue;                       // the missing second tile of S = 128 (mod 256)
            const int nj = p.causal ? qtile + 1 : nqt;
            const int qrow = qtile * AT_BM + r;
            float m = -1e30f, l = 0.0f;
            for (int j = 0; j < nj; j++) {
                ok = __all_sync(0xffffffffu, at_wait(&s_full[t], (it + j) & 1, p.err));
                if (!ok) break;
                tc_fence_after();
                float v[128];
                tmem_ld128(tS, v);
                if (p.causal && j == qtile) {
#pragma unroll
                    for (int cc = 0; cc < 128; cc++)
                        if (j * AT_BN + cc > qrow) v[cc] = -INFINITY;
                }
                float mk[4];
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    mk[kk] = fmaxf(v[kk * 32], v[kk * 32 + 1]);
#pragma unroll
                    for (int cc = 2; cc < 32; cc += 2) mk[kk] = at_max3(mk[kk], v[kk * 32 + cc], v[kk * 32 + cc + 1]);
                }
                const float mnew = fmaxf(m, at_max3(mk[0], mk[1], fmaxf(mk[2], mk[3])) * sl2);
                if (j == 0) {
                    m = mnew;
                } else if (__any_sync(0xffffffffu, mnew > m + 8.0f)) {
                    ok = __all_sync(0xffffffffu, at_wait(&pv_done[t], (it + j - 1) & 1, p.err));
                    if (!ok) break;
                    tc_fence_after();
                    const float alpha = at_ex2(m - mnew);
                    m = mnew;
                    l *= alpha;
#pragma unroll 1
                    for (int cc = 0; cc < 4; cc++) {
                        float o[32];
                        tmem_ld32(tO + cc * 32, o);
#pragma unroll
                        for (int e = 0; e < 32; e++) o[e] *= alpha;
                        tmem_st32(tO + cc * 32, o);
                    }
                }
                uint32_t pk[64];
                l += at_softmax_row(v, sl2, m, pk);
                tmem_st64(tS, pk);
                tc_fence_before();
                irx_mbar_arrive(&p_full[t]);
            }
            if (!ok) break;
            it += nj;
            ok = __all_sync(0xffffffffu, at_wait(&pv_done[t], (it - 1) & 1, p.err));
            if (!ok) break;
            tc_fence_after();
            {
                const float inv = 1.0f / l;
                __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.o) +
                                      (size_t)(((int)p.bh0 + w / nqb) * S + qrow) * AT_D;
#pragma unroll 1
                for (int cc = 0; cc < 4; cc++) {
                    float o[32];
                    tmem_ld32(tO + cc * 32, o);
#pragma unroll
                    for (int j8 = 0; j8 < 4; j8++) {
                        uint4 pk;
                        pk.x = at_pack_bf16(o[j8 * 8 + 0] * inv, o[j8 * 8 + 1] * inv);
                        pk.y = at_pack_bf16(o[j8 * 8 + 2] * inv, o[j8 * 8 + 3] * inv);
                        pk.z = at_pack_bf16(o[j8 * 8 + 4] * inv, o[j8 * 8 + 5] * inv);
                        pk.w = at_pack_bf16(o[j8 * 8 + 6] * inv, o[j8 * 8 + 7] * inv);
                        *reinterpret_cast<uint4 *>(orow + cc * 32 + j8 * 8) = pk;
                    }
                }
            }
            tc_fence_before();
            irx_mbar_arrive(&o_free[t]);
        }
        tc_fence_before();
        asm volatile("bar.arrive 1, 288;" ::: "memory");
    }
}

// ---- SIMT fallback: one thread per query row ----

#define AS_KT 32          // keys per shared tile
#define AS_DMAX 128

template <typename T>
__device__ __forceinline__ float at_ld(const T *p, int64_t i);
template <>
__device__ __forceinline__ float at_ld<float>(const float *p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float at_ld<__nv_bfloat16>(const __nv_bfloat16 *p, int64_t i) { return __bfloat162float(p[i]); }

template <typename T>
__device__ __forceinline__ void at_st(T *p, int64_t i, float v);
template <>
__device__ __forceinline__ void at_st<float>(float *p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void at_st<__nv_bfloat16>(__nv_bfloat16 *p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

template <typename T>
__device__ __forceinline__ void attn_simt(const irx_kat_t &p)
{
    __shared__ float Ks[AS_KT][AS_DMAX + 1], Vs[AS_KT][AS_DMAX + 1];
    const int64_t Sq = p.sq, Sk = p.sk, Dqk = p.dqk, Dv = p.dv;
    const int64_t nqb = (Sq + blockDim.x - 1) / blockDim.x;
    const T *Q = reinterpret_cast<const T *>(p.q);
    const T *Kp = reinterpret_cast<const T *>(p.k);
    const T *Vp = reinterpret_cast<const T *>(p.v);
    T *O = reinterpret_cast<T *>(p.o);
    for (int64_t w = blockIdx.x; w < (p.bh1 - p.bh0) * nqb; w += gridDim.x) {
        const int64_t bh = p.bh0 + w / nqb, q = (w % nqb) * blockDim.x + threadIdx.x;
        float qv[AS_DMAX], o[AS_DMAX];
#pragma unroll
        for (int d = 0; d < AS_DMAX; d++) {
            qv[d] = (q < Sq && d < Dqk) ? at_ld<T>(Q, (bh * Sq + q) * Dqk + d) : 0.0f;
            o[d] = 0.0f;
        }
        float m = -1e30f, l = 0.0f;            // the reference's finite identity for maximum
        const int64_t qmax = (w % nqb) * blockDim.x + blockDim.x - 1;
        const int64_t kend = p.causal ? min(Sk, qmax + 1) : Sk;
        for (int64_t k0 = 0; k0 < kend; k0 += AS_KT) {
            __syncthreads();
            for (int64_t e = threadIdx.x; e < AS_KT * AS_DMAX; e += blockDim.x) {
                const int64_t kk = e / AS_DMAX, d = e % AS_DMAX, key = k0 + kk;
                const bool in = key < Sk;
                // K is [.., key, d] or, transposed, [.., d, key]
                Ks[kk][d] = in && d < Dqk ? at_ld<T>(Kp, p.k_t ? (bh * Dqk + d) * Sk + key : (bh * Sk + key) * Dqk + d) : 0.0f;
                Vs[kk][d] = in && d < Dv ? at_ld<T>(Vp, (bh * Sk + key) * Dv + d) : 0.0f;
            }
            __syncthreads();
            if (q >= Sq) continue;
            for (int kk = 0; kk < AS_KT; kk++) {
                const int64_t key = k0 + kk;
                if (key >= Sk || (p.causal && key > q)) break;
                float dot = 0.0f;
#pragma unroll
                for (int d = 0; d < AS_DMAX; d++)
                    if (d < Dqk) dot = __fadd_rn(dot, __fmul_rn(qv[d], Ks[kk][d]));
                const float sc = p.scale_div ? __fdiv_rn(dot, p.divisor) : __fmul_rn(dot, p.scale);
                const float mn = fmaxf(m, sc);
                const float alpha = expf(__fsub_rn(m, mn));
                const float pj = expf(__fsub_rn(sc, mn));
                l = __fadd_rn(__fmul_rn(l, alpha), pj);
#pragma unroll
                for (int d = 0; d < AS_DMAX; d++)
                    if (d < Dv) o[d] = __fadd_rn(__fmul_rn(o[d], alpha), __fmul_rn(pj, Vs[kk][d]));
                m = mn;
            }
        }
        if (q < Sq) {
#pragma unroll
            for (int d = 0; d < AS_DMAX; d++)
                if (d < Dv) at_st<T>(O, (bh * Sq + q) * Dv + d, __fdiv_rn(o[d], l));
        }
    }
}

extern "C" __global__ void __launch_bounds__(128) irx_attn_f32(const __grid_constant__ irx_kat_t p) { irx_pdl_enter(); attn_simt<float>(p); }
extern "C" __global__ void __launch_bounds__(128) irx_attn_bf16_simt(const __grid_constant__ irx_kat_t p) { irx_pdl_enter(); attn_simt<__nv_bfloat16>(p); }
