// attn.cu -- the attention templates: O = softmax(Q K^T * scale [causal]) V over [B, H, S, D].
//
// irx_attn_bf16: flash attention on the 5th-generation tensor cores, D = 128, S a multiple of 128.
// One CTA per (batch*head, 128-query tile); for causal graphs the heaviest query tiles launch
// first. Per CTA:
//   * warp 0 (TMA): the Q tile once, then K_j and V_j tiles of 128 keys into a 2-deep ring
//     (128-byte swizzle, 64-column boxes, no multicast);
//   * warp 1 (MMA): S_j = Q K_j^T into one of two TMEM score buffers (128x128 f32), and, once
//     the softmax warps have written P_j, O += P_j V_j into a TMEM output accumulator. S_{j+1}
//     is issued before P_j V_j, so the next scores compute under this tile's softmax;
//   * warps 2-5 (softmax): each thread owns one query row: it reads its 128 scores from TMEM,
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

extern "C" __global__ void __launch_bounds__(192, 1) irx_attn_bf16(const __grid_constant__ irx_kat_t p)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *sq = smem;
    unsigned char *sk = smem + AT_TILE_BYTES;                 // 2 slots
    unsigned char *sv = smem + 3 * AT_TILE_BYTES;             // 2 slots
    unsigned char *sp = smem + 5 * AT_TILE_BYTES;             // P (one buffer)
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 6 * AT_TILE_BYTES);
    uint64_t *q_full = bars, *k_full = bars + 1, *v_full = bars + 3, *kv_empty = bars + 5;
    uint64_t *s_full = bars + 7, *s_free = bars + 9, *p_full = bars + 11, *o_done = bars + 12, *done = bars + 13;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 16);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (int)p.s;
    const int nqt = S / AT_BM;
    const int nbh = (int)(p.bh1 - p.bh0);
    const int qt = nqt - 1 - (int)(blockIdx.x / nbh);         // heaviest (causal) tiles first
    const int bh = (int)p.bh0 + (int)(blockIdx.x % nbh);
    const int nkv = p.causal ? qt + 1 : S / AT_BN;
    const int row0 = bh * S + qt * AT_BM;                     // first row of Q / O in [B*H*S, D]
    const int krow0 = bh * S;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 16; i++) irx_mbar_init(&bars[i], (i == 9 || i == 10 || i == 11) ? 128 : 1);
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
            for (int j = 0; j < nkv; j++) {
                const int s = j & 1;
                if (!at_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, p.err)) break;
                irx_mbar_expect_tx(&k_full[s], AT_TILE_BYTES);
                tma_load_2d(sk + s * AT_TILE_BYTES, &p.tma_k, 0, krow0 + j * AT_BN, &k_full[s]);
                tma_load_2d(sk + s * AT_TILE_BYTES + AT_HALF, &p.tma_k, 64, krow0 + j * AT_BN, &k_full[s]);
                irx_mbar_expect_tx(&v_full[s], AT_TILE_BYTES);
                tma_load_2d(sv + s * AT_TILE_BYTES, &p.tma_v, 0, krow0 + j * AT_BN, &v_full[s]);
                tma_load_2d(sv + s * AT_TILE_BYTES + AT_HALF, &p.tma_v, 64, krow0 + j * AT_BN, &v_full[s]);
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {                                    // MMA
            const uint32_t id_qk = umma_idesc_bf16(AT_BM, AT_BN, 0);   // K tile: keys x d, d contiguous
            const uint32_t id_pv = umma_idesc_bf16(AT_BM, AT_D, 1);    // V tile: keys x d, read MN-major
            const uint32_t aq = irx_smem_u32(sq), ap = irx_smem_u32(sp);
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
                }
                if (j >= 1) {                                 // O += P_{j-1} V_{j-1}
                    const int i = j - 1, s = i & 1;
                    if (!(ok = at_wait(p_full, i & 1, p.err))) break;
                    if (!(ok = at_wait(&v_full[s], (i >> 1) & 1, p.err))) break;
                    tc_fence_after();
                    const uint32_t bv = irx_smem_u32(sv + s * AT_TILE_BYTES);
#pragma unroll
                    for (int k = 0; k < AT_BN / 16; k++)
                        umma_bf16(t_o, at_kmajor_desc(ap, k), umma_desc_sw128(bv + k * 16 * 128, AT_HALF, 1024), id_pv,
                                  (i | k) != 0);
                    umma_commit(&kv_empty[s]);
                    umma_commit(o_done);
                }
            }
            umma_commit(done);                    // every MMA issued above has finished once this lands
            at_wait(done, 0, p.err);
        }
    } else {                                                   // softmax: warps 2-5
        const int q = warp & 3;
        const int r = q * 32 + lane;                          // row within the tile = TMEM lane
        const int qrow = qt * AT_BM + r;                      // query position in the sequence
        const uint32_t tl = (uint32_t)(q * 32) << 16;
        const float sl2 = p.scale * 1.4426950408889634f;      // scale * log2(e)
        float m = -1e30f, l = 0.0f;
        bool ok = true;
        unsigned char *prow = sp + r * 128;
        for (int j = 0; j < nkv; j++) {
            const int s = j & 1;
            ok = __all_sync(0xffffffffu, at_wait(&s_full[s], (j >> 1) & 1, p.err));
            if (!ok) break;
            tc_fence_after();
            float sc[AT_BN];
#pragma unroll
            for (int c = 0; c < AT_BN / 32; c++) {
                float v[32];
                tmem_ld32(tbase + tl + s * AT_BN + c * 32, v);
#pragma unroll
                for (int e = 0; e < 32; e++) sc[c * 32 + e] = v[e] * sl2;
            }
            tc_fence_before();
            irx_mbar_arrive(&s_free[s]);
            if (p.causal && j == qt) {                         // the diagonal tile: keys after the query
#pragma unroll
                for (int c = 0; c < AT_BN; c++)
                    if (j * AT_BN + c > qrow) sc[c] = -INFINITY;
            }
            float mx = sc[0];
#pragma unroll
            for (int c = 1; c < AT_BN; c++) mx = fmaxf(mx, sc[c]);
            const float mnew = fmaxf(m, mx);
            if (j > 0) {
                ok = __all_sync(0xffffffffu, at_wait(o_done, (j - 1) & 1, p.err));   // P free, O current
                if (!ok) break;
                tc_fence_after();
            }
            if (j == 0) {
                m = mnew;
            } else if (__any_sync(0xffffffffu, mnew > m + 8.0f)) {
                const float alpha = exp2f(m - mnew);
                m = mnew;
                l *= alpha;
#pragma unroll 1
                for (int c = 0; c < AT_D / 32; c++) {
                    float v[32];
                    tmem_ld32(t_o + tl + c * 32, v);
#pragma unroll
                    for (int e = 0; e < 32; e++) v[e] *= alpha;
                    tmem_st32(t_o + tl + c * 32, v);
                }
            }
            float sum = 0.0f;
#pragma unroll
            for (int cb = 0; cb < AT_BN / 8; cb++) {          // 16 chunks of 8 keys
                uint4 pk;
                __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float p0 = exp2f(sc[cb * 8 + 2 * e] - m), p1 = exp2f(sc[cb * 8 + 2 * e + 1] - m);
                    const __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);
                    const float2 f = __bfloat1622float2(b);
                    sum += f.x + f.y;                          // l sums the P the MMA will see
                    h[e] = b;
                }
                const int blk = cb >> 3, ch = cb & 7;
                *reinterpret_cast<uint4 *>(prow + blk * AT_HALF + ((ch ^ (r & 7)) << 4)) = pk;
            }
            l += sum;
            fence_proxy_async_smem();                         // P visible to the tensor core
            tc_fence_before();
            irx_mbar_arrive(p_full);
        }
        if (ok && __all_sync(0xffffffffu, at_wait(o_done, (nkv - 1) & 1, p.err))) {
            tc_fence_after();
            const float inv = 1.0f / l;
            __nv_bfloat16 *orow = reinterpret_cast<__nv_bfloat16 *>(p.o) + (size_t)(row0 + r) * AT_D;
#pragma unroll 1
            for (int c = 0; c < AT_D / 32; c++) {
                float v[32];
                tmem_ld32(t_o + tl + c * 32, v);
#pragma unroll
                for (int j8 = 0; j8 < 4; j8++) {
                    uint4 pk;
                    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                    for (int e = 0; e < 4; e++) h[e] = __floats2bfloat162_rn(v[j8 * 8 + 2 * e] * inv, v[j8 * 8 + 2 * e + 1] * inv);
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
