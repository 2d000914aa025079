// attn.cu -- the attention templates: O = softmax(Q K^T * scale [causal]) V over [B, H, S, D].
//
// irx_attn_bf16: flash attention on the 5th-generation tensor cores, D = 128, S a multiple of 128.
// One CTA per (batch*head, 128-query tile), ordered head by head so the CTAs running at once
// share K and V in L2; within a head the heaviest causal query tiles launch first. Per CTA:
//   * warp 0 (TMA): the Q tile once, then K_j and V_j tiles of 128 keys into a 2-deep ring
//     (128-byte swizzle, 64-column boxes, no multicast);
//   * warp 1 (MMA): S_j = Q K_j^T into one of two TMEM score buffers (128x128 f32), and, once
//     the softmax warps have written P_j, O += P_j V_j into a TMEM output accumulator. S_{j+1}
//     is issued before P_j V_j, so the next scores compute under this tile's softmax;
//   * warps 2-9 (softmax): two threads own one query row, 64 score columns each: they read the
//     scores from TMEM, agree on the row max through shared memory,
//     keeps the running max m and sum l (log2 domain, scale folded in), writes P = 2^(s - m) as
//     bf16 into shared memory in the MMA's 128-byte-swizzled K-major layout, and at the end
//     writes O / l. O is rescaled in TMEM only when a row's max grows by more than 8 (a factor
//     of 256): until then the stale max is kept for that row's P and l alike, which the final
//     division cancels exactly.
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

// 2^x on the FMA pipe, for x <= 8: x = n + f with n = floor(x), 2^f from a cubic fitted here to
// 2^f on [0, 1) (weighted least squares toward equal relative error, max 7.5e-5 in f32), then
// n added to the exponent field. Below -126 the result is flushed to 0. Accurate far beyond
// the bf16 P it feeds (2^-9). Half of the scores go this way so the MUFU unit, which would
// otherwise take as long as the two MMAs of a tile, carries only the other half.
__device__ __forceinline__ float at_ex2_poly(float x)
{
    const float xc = fmaxf(x, -126.0f);
    const float n = floorf(xc);
    const float f = xc - n;
    float q = fmaf(0.07802446186542511f, f, 0.22606727480888367f);
    q = fmaf(q, f, 0.6958335041999817f);
    q = fmaf(q, f, 0.9999251961708069f);
    const float r = __int_as_float(__float_as_int(q) + ((int)n << 23));
    return x < -126.0f ? 0.0f : r;
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

// 64 f32 columns of this thread's TMEM lane, the wait in the same statement.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64])
{
    uint32_t r[64];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
                 "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                 "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
                 "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
                 "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
                 "tcgen05.wait::ld.sync.aligned;"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
                   "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
                   "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
                   "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
                   "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
                 : "r"(taddr) : "memory");
#pragma unroll
    for (int i = 0; i < 64; i++) v[i] = __uint_as_float(r[i]);
}

#define AT_THREADS 320      // TMA warp, MMA warp, 8 softmax warps

extern "C" __global__ void __launch_bounds__(AT_THREADS, 1) irx_attn_bf16(const __grid_constant__ irx_kat_t p)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // The launch reserves no alignment slack: the declared 1024-byte alignment of the dynamic
    // shared base is relied on, and checked here before anything touches shared memory.
    unsigned char *smem = smem_raw;
    if (irx_smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0 && p.err) atomicOr(p.err, IRX_KERR_TIMEOUT);
        return;
    }
    unsigned char *sq = smem;
    unsigned char *sk = smem + AT_TILE_BYTES;                 // 2 slots
    unsigned char *sv = smem + 3 * AT_TILE_BYTES;             // 2 slots
    unsigned char *sp = smem + 5 * AT_TILE_BYTES;             // 2 P buffers
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 7 * AT_TILE_BYTES);
    uint64_t *q_full = bars, *k_full = bars + 1, *v_full = bars + 3, *k_empty = bars + 5;
    uint64_t *s_full = bars + 7, *s_free = bars + 9, *p_full = bars + 11, *pv_done = bars + 13, *done = bars + 15;
    uint64_t *mx_bar = bars + 16, *l_bar = bars + 18;      // row-max and final-sum exchanges
    uint64_t *v_empty = bars + 19;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 21);
    float *xch = reinterpret_cast<float *>(bars + 24);     // [2 tiles][2 halves][128 rows]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (int)p.s;
    const int nqt = S / AT_BM;
    // Head-major order: the query tiles of one head are consecutive blocks, so the CTAs resident
    // at once share each head's K and V through L2 (read from HBM about once per head rather
    // than once per query tile); within a head the heaviest causal tiles go first.
    const int qt = nqt - 1 - (int)(blockIdx.x % nqt);
    const int bh = (int)p.bh0 + (int)(blockIdx.x / nqt);
    const int nkv = p.causal ? qt + 1 : S / AT_BN;
    const int row0 = bh * S + qt * AT_BM;                     // first row of Q / O in [B*H*S, D]
    const int krow0 = bh * S;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 21; i++) irx_mbar_init(&bars[i], ((i >= 9 && i <= 12) || (i >= 16 && i <= 18)) ? 256 : 1);
        irx_fence_mbar_init();
        tma_prefetch_desc(&p.tma_q);
        tma_prefetch_desc(&p.tma_k);
        tma_prefetch_desc(&p.tma_v);
    }
    if (warp == 1) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    const uint32_t t_o = tbase + 256;

    if (warp == 0) {
        if (elect_one()) {                                    // TMA
            irx_mbar_expect_tx(q_full, AT_TILE_BYTES);
            tma_load_2d(sq, &p.tma_q, 0, row0, q_full);
            tma_load_2d(sq + AT_HALF, &p.tma_q, 64, row0, q_full);
            // K runs one tile ahead of V: a K slot frees when its S = Q K^T is done, a V slot only
            // when its P V is, so K_{t} loads while P_{t-2} V_{t-2} is still pending
            bool ok = true;
            for (int t = 0; t <= nkv && ok; t++) {
                if (t < nkv) {
                    const int s = t & 1;
                    if (!(ok = at_wait(&k_empty[s], ((t >> 1) & 1) ^ 1, p.err))) break;
                    irx_mbar_expect_tx(&k_full[s], AT_TILE_BYTES);
                    tma_load_2d(sk + s * AT_TILE_BYTES, &p.tma_k, 0, krow0 + t * AT_BN, &k_full[s]);
                    tma_load_2d(sk + s * AT_TILE_BYTES + AT_HALF, &p.tma_k, 64, krow0 + t * AT_BN, &k_full[s]);
                }
                if (t >= 1) {
                    const int i = t - 1, s = i & 1;
                    if (!(ok = at_wait(&v_empty[s], ((i >> 1) & 1) ^ 1, p.err))) break;
                    irx_mbar_expect_tx(&v_full[s], AT_TILE_BYTES);
                    tma_load_2d(sv + s * AT_TILE_BYTES, &p.tma_v, 0, krow0 + i * AT_BN, &v_full[s]);
                    tma_load_2d(sv + s * AT_TILE_BYTES + AT_HALF, &p.tma_v, 64, krow0 + i * AT_BN, &v_full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {                                    // MMA
            const uint32_t id_qk = umma_idesc_bf16(AT_BM, AT_BN, 0);   // K tile: keys x d, d contiguous
            const uint32_t id_pv = umma_idesc_bf16(AT_BM, AT_D, 1);    // V tile: keys x d, read MN-major
            const uint32_t aq = irx_smem_u32(sq);
            bool ok = at_wait(q_full, 0, p.err);
            for (int j = 0; j <= nkv && ok; j++) {
                if (j < nkv) {                                // S_j = Q K_j^T
                    const int s = j & 1;
                    if (!(ok = at_wait(&k_full[s], (j >> 1) & 1, p.err))) break;
                    if (!(ok = at_wait(&s_free[s], ((j >> 1) & 1) ^ 1, p.err))) break;
                    tc_fence_after();
                    const uint32_t bk = irx_smem_u32(sk + s * AT_TILE_BYTES);
#pragma unroll
                    for (int k = 0; k < AT_D / 16; k++)
                        umma_bf16(tbase + s * AT_BN, at_kmajor_desc(aq, k), at_kmajor_desc(bk, k), id_qk, k > 0);
                    umma_commit(&s_full[s]);
                    umma_commit(&k_empty[s]);
                }
                if (j >= 1) {                                 // O += P_{j-1} V_{j-1}
                    const int i = j - 1, s = i & 1;
                    if (!(ok = at_wait(&p_full[s], (i >> 1) & 1, p.err))) break;
                    if (!(ok = at_wait(&v_full[s], (i >> 1) & 1, p.err))) break;
                    tc_fence_after();
                    const uint32_t ap = irx_smem_u32(sp + s * AT_TILE_BYTES);
                    const uint32_t bv = irx_smem_u32(sv + s * AT_TILE_BYTES);
#pragma unroll
                    for (int k = 0; k < AT_BN / 16; k++)
                        umma_bf16(t_o, at_kmajor_desc(ap, k), umma_desc_sw128(bv + k * 16 * 128, AT_HALF, 1024), id_pv,
                                  (i | k) != 0);
                    umma_commit(&v_empty[s]);
                    umma_commit(&pv_done[s]);
                }
            }
            umma_commit(done);                    // every MMA issued above has finished once this lands
            at_wait(done, 0, p.err);
        }
    } else {                                                   // softmax: warps 2-9
        // Two threads per query row: warps 2-5 take score columns 0-63, warps 6-9 columns 64-127
        // of the same rows (warp w reads TMEM lane quarter w % 4). They agree on the row max
        // through shared memory each tile, keep partial sums, rescale and write half of O each.
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r = q * 32 + lane;                          // row within the tile = TMEM lane
        const int qrow = qt * AT_BM + r;                      // query position in the sequence
        const int c0 = half * 64;                             // this thread's first score / O column
        const uint32_t tl = (uint32_t)(q * 32) << 16;
        const float sl2 = p.scale * 1.4426950408889634f;      // scale * log2(e)
        float m = -1e30f, l = 0.0f;                           // running max (log2 units), partial sum
        bool ok = true;
        for (int j = 0; j < nkv; j++) {
            const int s = j & 1;
            ok = __all_sync(0xffffffffu, at_wait(&s_full[s], (j >> 1) & 1, p.err));
            if (!ok) break;
            tc_fence_after();
            float v[64];
            tmem_ld64(tbase + tl + s * AT_BN + c0, v);
            tc_fence_before();
            irx_mbar_arrive(&s_free[s]);
            if (p.causal && j == qt) {                         // the diagonal tile: keys after the query
#pragma unroll
                for (int c = 0; c < 64; c++)
                    if (j * AT_BN + c0 + c > qrow) v[c] = -INFINITY;
            }
            float m4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
            for (int c = 4; c < 64; c++) m4[c & 3] = fmaxf(m4[c & 3], v[c]);
            const float mine = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;
            float *xm = xch + s * 256;
            xm[half * 128 + r] = mine;
            irx_mbar_arrive(&mx_bar[s]);
            ok = __all_sync(0xffffffffu, at_wait(&mx_bar[s], (j >> 1) & 1, p.err));
            if (!ok) break;
            const float mnew = fmaxf(m, fmaxf(mine, xm[(half ^ 1) * 128 + r]));
            if (j >= 2) {                                      // P buffer s is free once P_{j-2} V_{j-2} is done
                ok = __all_sync(0xffffffffu, at_wait(&pv_done[s], ((j >> 1) & 1) ^ 1, p.err));
                if (!ok) break;
            }
            if (j == 0) {
                m = mnew;
            } else if (__any_sync(0xffffffffu, mnew > m + 8.0f)) {
                // rescale this half of O: it must hold every earlier P V first
                ok = __all_sync(0xffffffffu, at_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err));
                if (!ok) break;
                tc_fence_after();
                const float alpha = at_ex2(m - mnew);
                m = mnew;
                l *= alpha;
#pragma unroll 1
                for (int c = 0; c < 2; c++) {
                    float o[32];
                    tmem_ld32(t_o + tl + c0 + c * 32, o);
#pragma unroll
                    for (int e = 0; e < 32; e++) o[e] *= alpha;
                    tmem_st32(t_o + tl + c0 + c * 32, o);
                }
            }
            float sum4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            unsigned char *prow = sp + s * AT_TILE_BYTES + half * AT_HALF + r * 128;
#pragma unroll
            for (int cb = 0; cb < 8; cb++) {                  // 8 chunks of 8 keys: this half's swizzle block
                uint4 pk;
                __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float x0 = fmaf(v[cb * 8 + 2 * e], sl2, -m), x1 = fmaf(v[cb * 8 + 2 * e + 1], sl2, -m);
                    const float p0 = (cb & 3) == 3 ? at_ex2_poly(x0) : at_ex2(x0);
                    const float p1 = (cb & 3) == 3 ? at_ex2_poly(x1) : at_ex2(x1);
                    sum4[e] += p0 + p1;
                    h[e] = __floats2bfloat162_rn(p0, p1);
                }
                *reinterpret_cast<uint4 *>(prow + ((cb ^ (r & 7)) << 4)) = pk;
            }
            l += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
            fence_proxy_async_smem();                         // P visible to the tensor core
            tc_fence_before();
            irx_mbar_arrive(&p_full[s]);
        }
        // the row's total sum, both halves: through the max buffer of the tile before the last,
        // which every thread has finished reading once it passed the last tile's exchange
        float *xl = xch + (((nkv - 1) & 1) ^ 1) * 256;
        if (ok) {
            xl[half * 128 + r] = l;
            irx_mbar_arrive(l_bar);
            ok = __all_sync(0xffffffffu, at_wait(l_bar, 0, p.err));
        }
        if (ok && __all_sync(0xffffffffu, at_wait(&pv_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1, p.err))) {
            tc_fence_after();
            const float inv = 1.0f / (l + xl[(half ^ 1) * 128 + r]);
            __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.o) + (size_t)(row0 + r) * AT_D + c0;
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                float o[32];
                tmem_ld32(t_o + tl + c0 + c * 32, o);
#pragma unroll
                for (int j8 = 0; j8 < 4; j8++) {
                    uint4 pk;
                    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                    for (int e = 0; e < 4; e++) h[e] = __floats2bfloat162_rn(o[j8 * 8 + 2 * e] * inv, o[j8 * 8 + 2 * e + 1] * inv);
                    *reinterpret_cast<uint4 *>(orow + c * 32 + j8 * 8) = pk;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
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
    const int64_t S = p.s, D = p.d;
    const int64_t nqb = (S + blockDim.x - 1) / blockDim.x;
    const T *Q = reinterpret_cast<const T *>(p.q);
    const T *Kp = reinterpret_cast<const T *>(p.k);
    const T *Vp = reinterpret_cast<const T *>(p.v);
    T *O = reinterpret_cast<T *>(p.o);
    for (int64_t w = blockIdx.x; w < (p.bh1 - p.bh0) * nqb; w += gridDim.x) {
        const int64_t bh = p.bh0 + w / nqb, q = (w % nqb) * blockDim.x + threadIdx.x;
        const int64_t base = bh * S * D;
        float qv[AS_DMAX], o[AS_DMAX];
#pragma unroll
        for (int d = 0; d < AS_DMAX; d++) {
            qv[d] = (q < S && d < D) ? at_ld<T>(Q, base + q * D + d) : 0.0f;
            o[d] = 0.0f;
        }
        float m = -1e30f, l = 0.0f;            // the reference's finite identity for maximum
        const int64_t qmax = (w % nqb) * blockDim.x + blockDim.x - 1;
        const int64_t kend = p.causal ? min(S, qmax + 1) : S;
        for (int64_t k0 = 0; k0 < kend; k0 += AS_KT) {
            __syncthreads();
            for (int64_t e = threadIdx.x; e < AS_KT * D; e += blockDim.x) {
                const int64_t kk = e / D, d = e % D;
                const bool in = k0 + kk < S;
                Ks[kk][d] = in ? at_ld<T>(Kp, base + (k0 + kk) * D + d) : 0.0f;
                Vs[kk][d] = in ? at_ld<T>(Vp, base + (k0 + kk) * D + d) : 0.0f;
            }
            __syncthreads();
            if (q >= S) continue;
            for (int kk = 0; kk < AS_KT; kk++) {
                const int64_t key = k0 + kk;
                if (key >= S || (p.causal && key > q)) break;
                float dot = 0.0f;
#pragma unroll
                for (int d = 0; d < AS_DMAX; d++)
                    if (d < D) dot = __fadd_rn(dot, __fmul_rn(qv[d], Ks[kk][d]));
                const float sc = __fmul_rn(dot, p.scale);
                const float mn = fmaxf(m, sc);
                const float alpha = expf(__fsub_rn(m, mn));
                const float pj = expf(__fsub_rn(sc, mn));
                l = __fadd_rn(__fmul_rn(l, alpha), pj);
#pragma unroll
                for (int d = 0; d < AS_DMAX; d++)
                    if (d < D) o[d] = __fadd_rn(__fmul_rn(o[d], alpha), __fmul_rn(pj, Vs[kk][d]));
                m = mn;
            }
        }
        if (q < S) {
#pragma unroll
            for (int d = 0; d < AS_DMAX; d++)
                if (d < D) at_st<T>(O, base + q * D + d, __fdiv_rn(o[d], l));
        }
    }
}

extern "C" __global__ void __launch_bounds__(128) irx_attn_f32(const __grid_constant__ irx_kat_t p) { attn_simt<float>(p); }
extern "C" __global__ void __launch_bounds__(128) irx_attn_bf16_simt(const __grid_constant__ irx_kat_t p) { attn_simt<__nv_bfloat16>(p); }
