// gemm.cu -- the matmul templates: C[M,N] = A[M,K] B (B stored [K,N] or [N,K]).
//
// irx_mm_bf16: bf16 operands, f32 accumulation in TMEM, bf16 result, on the 5th-generation
// tensor cores (tcgen05.mma kind::f16, cta_group::1, 128x256x16 per instruction).
//   * persistent: one CTA per SM walks output tiles of 128x256 in a grouped order (8 tile rows
//     at a time) so the tiles in flight share A rows and B columns in L2;
//   * warp 0 is the TMA producer: per K-block of 64, a 128x64 A tile and a 64x256 B tile, both
//     128-byte swizzled, into a 4-deep ring of shared-memory stages (48 KiB each). Each CTA
//     fetches its own tiles;
//   * warp 1 allocates 512 TMEM columns (two 128x256 f32 accumulators) and one elected thread
//     issues the MMAs; tcgen05.commit frees a stage when the MMAs reading it finish, and marks
//     an accumulator full when its tile's last K-block is done;
//   * warps 2-5 are the epilogue: each thread owns one accumulator row (its TMEM lane), reads
//     it 32 columns at a time, rounds to bf16 and stores it. The two accumulators let the
//     epilogue of one tile run under the mainloop of the next.
//   B stored [K, N] is read through an MN-major descriptor, B stored [N, K] through a K-major
//   one. Every mbarrier wait is bounded (p.wait_ns, else IRX_WAIT_NS); a wait that runs out sets
//   the error word and ends that role's loop, and the CTA still drains its MMAs before it frees
//   TMEM. `no_loads` (failure injection for tests, set by irx_inject) makes the producer issue
//   nothing, so the MMA and epilogue waits run out with no copy in flight.
//
// irx_mm_f32 / irx_mm_bf16_simt: SIMT tiles for f32 graphs and for shapes the TMA path cannot
// address (a row stride that is not a multiple of 16 bytes). Each output is accumulated over k
// in ascending order with round-to-nearest multiply then add, the reference's per-element
// order (src/isel.c:1848-1870, src/ops.c:128-135), so f32 results equal the reference's bit
// for bit.

#include "tc.cuh"

#define MM_BM 128
#define MM_BN 256
#define MM_BK 64
#define MM_STAGES 4
#define MM_A_BYTES (MM_BM * MM_BK * 2)
#define MM_B_BYTES (MM_BN * MM_BK * 2)
#define MM_STAGE_BYTES (MM_A_BYTES + MM_B_BYTES)
#define MM_GROUP 8

struct MmTile { int m0, n0; };

__device__ __forceinline__ MmTile mm_tile(int t, int ntm, int ntn, int n_tile0)
{
    const int per_group = MM_GROUP * ntn;
    const int g = t / per_group;
    const int first = g * MM_GROUP;
    const int gsize = min(ntm - first, MM_GROUP);
    const int r = t % per_group;
    MmTile x;
    x.m0 = (first + r % gsize) * MM_BM;
    x.n0 = (n_tile0 + r / gsize) * MM_BN;
    return x;
}

__device__ __forceinline__ int mm_wait(uint64_t *bar, uint32_t parity, const irx_kmm_t &p)
{
    if (irx_mbar_wait(bar, parity, IRX_WAIT_LIMIT, p.wait_ns ? p.wait_ns : IRX_WAIT_NS)) return 1;
    if (p.err) atomicOr(p.err, IRX_KERR_TIMEOUT);
    return 0;
}

extern "C" __global__ void __launch_bounds__(192, 1) irx_mm_bf16(const __grid_constant__ irx_kmm_t p)
{
    irx_pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *sa = smem;
    unsigned char *sb = smem + MM_STAGES * MM_A_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + MM_STAGES * MM_STAGE_BYTES);
    uint64_t *empty = full + MM_STAGES;
    uint64_t *tfull = empty + MM_STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *done = tempty + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    const int n_tile0 = (int)(p.n0 / MM_BN);
    const int ntm = (M + MM_BM - 1) / MM_BM;
    const int ntn = (int)((p.n1 + MM_BN - 1) / MM_BN) - n_tile0;
    const int tiles = ntm * ntn;
    const int nk = (K + MM_BK - 1) / MM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < MM_STAGES; s++) { irx_mbar_init(&full[s], 1); irx_mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { irx_mbar_init(&tfull[b], 1); irx_mbar_init(&tempty[b], 128); }
        irx_mbar_init(done, 1);
        irx_fence_mbar_init();
        tma_prefetch_desc(&p.tma_a);
        tma_prefetch_desc(&p.tma_b);
    }
    if (warp == 1) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (elect_one() && !p.no_loads) {                    // TMA producer
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const MmTile x = mm_tile(t, ntm, ntn, n_tile0);
                for (int kb = 0; kb < nk && ok; kb++) {
                    if (!(ok = mm_wait(&empty[s], ph ^ 1, p))) break;
                    irx_mbar_expect_tx(&full[s], MM_STAGE_BYTES);
                    tma_load_2d(sa + s * MM_A_BYTES, &p.tma_a, kb * MM_BK, x.m0, &full[s]);
                    if (p.b_kmajor) {
                        tma_load_2d(sb + s * MM_B_BYTES, &p.tma_b, kb * MM_BK, x.n0, &full[s]);
                    } else {
#pragma unroll
                        for (int j = 0; j < MM_BN / 64; j++)
                            tma_load_2d(sb + s * MM_B_BYTES + j * (64 * MM_BK * 2), &p.tma_b, x.n0 + j * 64, kb * MM_BK, &full[s]);
                    }
                    if (++s == MM_STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {                                   // MMA issuer
            const uint32_t idesc = umma_idesc_bf16(MM_BM, MM_BN, p.b_kmajor ? 0 : 1);
            int s = 0, acc = 0;
            uint32_t ph = 0, aph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                if (!(ok = mm_wait(&tempty[acc], aph ^ 1, p))) break;
                tc_fence_after();
                const uint32_t tacc = tbase + (uint32_t)(acc * MM_BN);
                for (int kb = 0; kb < nk && ok; kb++) {
                    if (!(ok = mm_wait(&full[s], ph, p))) break;
                    tc_fence_after();
                    const uint32_t a0 = irx_smem_u32(sa + s * MM_A_BYTES);
                    const uint32_t b0 = irx_smem_u32(sb + s * MM_B_BYTES);
#pragma unroll
                    for (int k = 0; k < MM_BK / 16; k++) {
                        const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
                        const uint64_t bd = p.b_kmajor ? umma_desc_sw128(b0 + k * 32, 16, 1024)
                                                       : umma_desc_sw128(b0 + k * 16 * 128, 64 * MM_BK * 2, 1024);
                        umma_bf16(tacc, ad, bd, idesc, (kb | k) != 0);
                    }
                    umma_commit(&empty[s]);
                    if (++s == MM_STAGES) { s = 0; ph ^= 1; }
                }
                if (ok) umma_commit(&tfull[acc]);
                if (++acc == 2) { acc = 0; aph ^= 1; }
            }
            umma_commit(done);                   // every MMA issued above has finished once this lands
            mm_wait(done, 0, p);
        }
    } else {                                                  // epilogue: warps 2-5
        const int q = warp & 3;                               // this warp's TMEM lane quarter
        const int nend = (int)p.n1;
        const bool vec = (N % 8) == 0 && ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0);
        int acc = 0;
        uint32_t aph = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const MmTile x = mm_tile(t, ntm, ntn, n_tile0);
            if (!__all_sync(0xffffffffu, mm_wait(&tfull[acc], aph, p))) break;   // warp-uniform: tcgen05.ld is collective
            tc_fence_after();
            const int row = x.m0 + q * 32 + lane;
            __nv_bfloat16 *crow = reinterpret_cast<__nv_bfloat16 *>(p.c) + (size_t)row * N;
#pragma unroll 1
            for (int c = 0; c < MM_BN / 32; c++) {
                float v[32];
                tmem_ld32(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * MM_BN + c * 32), v);
                const int col = x.n0 + c * 32;
                if (row < M) {
                    if (vec && col + 32 <= nend) {
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            uint4 pk;
                            __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                            for (int e = 0; e < 4; e++) h[e] = __floats2bfloat162_rn(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
                            *reinterpret_cast<uint4 *>(crow + col + j * 8) = pk;
                        }
                    } else {
                        for (int j = 0; j < 32; j++)
                            if (col + j < nend) crow[col + j] = __float2bfloat16_rn(v[j]);
                    }
                }
            }
            tc_fence_before();
            irx_mbar_arrive(&tempty[acc]);
            if (++acc == 2) { acc = 0; aph ^= 1; }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ---- irx_mm_bf16_pair: the same product on CTA pairs (cta_group::2), 256x256 tiles ----
//
// A cluster of two CTAs (one TPC) owns a 256x256 output tile: CTA r of the pair loads rows
// m0 + 128r .. +128 of A and columns n0 + 128r .. +128 of B into its own shared memory (each CTA
// fetches only its own tiles: no multicast load), and one thread of the leader CTA (r = 0) issues
// tcgen05.mma.cta_group::2 with M = 256, N = 256, which reads A from each CTA's shared memory and
// B from both, and writes each CTA's 128 rows of D into that CTA's TMEM. Per CTA and K-step of 16
// that is 8 KB of shared-memory operand reads and 32 KB of TMA writes per 64-deep K-block, where
// the 128x256 single-CTA tile needs 12 KB and 48 KB, for the same tensor time per SM: the pair
// form leaves shared-memory bandwidth for both streams.
//   * both CTAs' TMA producers count their bytes on the leader's `full` barrier; the leader's
//     producer posts the expected byte count for the pair;
//   * the leader's MMA commits arrive on the `empty` (stage free) and `tfull` (accumulator ready)
//     barriers of both CTAs at once (commit multicast, a completion signal, not a load);
//   * each CTA's epilogue warps read its own TMEM rows and arrive on the leader's `tempty`
//     (one arrival per warp, eight per tile);
//   * TMEM (512 columns, two 256-column accumulators) is allocated and freed by warp 1 of both
//     CTAs together; the CTAs meet at a cluster barrier after set-up and before the free, so no
//     CTA exits while its peer can still signal it. Each producer waits, at its end, until the
//     MMAs have consumed every stage it loaded.
// Every wait is bounded, as in irx_mm_bf16.

#define M2_BN 256
#define M2_BK 64
#define M2_MAX_STAGES 7                              // the ring's depth is p.stages (launcher), at most this
#define M2_HALF_BYTES (128 * M2_BK * 2)              // 16 KB: one CTA's A tile, and its B half
#define M2_STAGE_BYTES (2 * M2_HALF_BYTES)

__device__ __forceinline__ MmTile mm2_tile(int t, int ntm, int ntn, int n_tile0, int group)
{
    const int per_group = group * ntn;
    const int g = t / per_group;
    const int first = g * group;
    const int gsize = min(ntm - first, group);
    const int r = t % per_group;
    MmTile x;
    x.m0 = (first + r % gsize) * 256;
    x.n0 = (n_tile0 + r / gsize) * M2_BN;
    return x;
}

extern "C" __global__ void __launch_bounds__(192, 1) irx_mm_bf16_pair(const __grid_constant__ irx_kmm_t p)
{
    irx_pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *sa = smem;
    const int stages = p.stages, group = p.group;
    unsigned char *sb = smem + stages * M2_HALF_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + stages * M2_STAGE_BYTES);
    uint64_t *empty = full + stages;
    uint64_t *tfull = empty + stages;
    uint64_t *tempty = tfull + 2;
    uint64_t *done = tempty + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    const int n_tile0 = (int)(p.n0 / M2_BN);
    const int ntm = (M + 255) / 256;
    const int ntn = (int)((p.n1 + M2_BN - 1) / M2_BN) - n_tile0;
    const int tiles = ntm * ntn;
    const int nk = (K + M2_BK - 1) / M2_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) { irx_mbar_init(&full[s], 1); irx_mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { irx_mbar_init(&tfull[b], 1); irx_mbar_init(&tempty[b], 8); }
        irx_mbar_init(done, 1);
        irx_fence_mbar_init();
        tma_prefetch_desc(&p.tma_a);
        tma_prefetch_desc(&p.tma_b);
    }
    if (warp == 1) tmem_alloc_pair(tslot, 512);
    tc_fence_before();
    __syncthreads();
    cluster_sync();                        // both CTAs' barriers exist before either signals the other
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (elect_one() && !p.no_loads) {                    // TMA producer, both CTAs
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                const MmTile x = mm2_tile(t, ntm, ntn, n_tile0, group);
                for (int kb = 0; kb < nk && ok; kb++) {
                    if (!(ok = mm_wait(&empty[s], ph ^ 1, p))) break;
                    const uint32_t fl = cluster_addr(&full[s], 0);
                    if (leader) irx_mbar_expect_tx(&full[s], 2 * M2_STAGE_BYTES);
                    tma_load_2d_pair(sa + s * M2_HALF_BYTES, &p.tma_a, kb * M2_BK, x.m0 + (int)rank * 128, fl);
                    if (p.b_kmajor) {
                        tma_load_2d_pair(sb + s * M2_HALF_BYTES, &p.tma_b, kb * M2_BK, x.n0 + (int)rank * 128, fl);
                    } else {
#pragma unroll
                        for (int j = 0; j < 2; j++)
                            tma_load_2d_pair(sb + s * M2_HALF_BYTES + j * (64 * M2_BK * 2), &p.tma_b,
                                             x.n0 + (int)rank * 128 + j * 64, kb * M2_BK, fl);
                    }
                    if (++s == stages) { s = 0; ph ^= 1; }
                }
            }
            // the tail: every stage loaded above has been consumed by the MMAs (its `empty`
            // arrival has landed) before this CTA can reach the exit barrier
            for (int i = 0; i < stages && ok; i++) {
                ok = mm_wait(&empty[s], ph ^ 1, p);
                if (++s == stages) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (leader && elect_one()) {                         // MMA issuer: the leader CTA only
            const uint32_t idesc = umma_idesc_bf16(256, M2_BN, p.b_kmajor ? 0 : 1);
            int s = 0, acc = 0;
            uint32_t ph = 0, aph = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                if (!(ok = mm_wait(&tempty[acc], aph ^ 1, p))) break;
                tc_fence_after();
                const uint32_t tacc = tbase + (uint32_t)(acc * M2_BN);
                for (int kb = 0; kb < nk && ok; kb++) {
                    if (!(ok = mm_wait(&full[s], ph, p))) break;
                    tc_fence_after();
                    const uint32_t a0 = irx_smem_u32(sa + s * M2_HALF_BYTES);
                    const uint32_t b0 = irx_smem_u32(sb + s * M2_HALF_BYTES);
#pragma unroll
                    for (int k = 0; k < M2_BK / 16; k++) {
                        const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
                        const uint64_t bd = p.b_kmajor ? umma_desc_sw128(b0 + k * 32, 16, 1024)
                                                       : umma_desc_sw128(b0 + k * 16 * 128, 64 * M2_BK * 2, 1024);
                        umma_bf16_pair(tacc, ad, bd, idesc, (kb | k) != 0);
                    }
                    umma_commit_pair(&empty[s], 0x3);
                    if (++s == stages) { s = 0; ph ^= 1; }
                }
                if (ok) umma_commit_pair(&tfull[acc], 0x3);
                if (++acc == 2) { acc = 0; aph ^= 1; }
            }
            umma_commit_pair(done, 0x1);         // every MMA issued above has finished once this lands
            mm_wait(done, 0, p);
        }
    } else {                                                  // epilogue: warps 2-5 of both CTAs
        const int q = warp & 3;                               // this warp's TMEM lane quarter
        const int nend = (int)p.n1;
        const bool vec = (N % 8) == 0 && ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0);
        int acc = 0;
        uint32_t aph = 0;
        const uint32_t te0 = cluster_addr(&tempty[0], 0), te1 = cluster_addr(&tempty[1], 0);
        for (int t = pair; t < tiles; t += npairs) {
            const MmTile x = mm2_tile(t, ntm, ntn, n_tile0, group);
            if (!__all_sync(0xffffffffu, mm_wait(&tfull[acc], aph, p))) break;   // warp-uniform: tcgen05.ld is collective
            tc_fence_after();
            const int row = x.m0 + (int)rank * 128 + q * 32 + lane;
            __nv_bfloat16 *crow = reinterpret_cast<__nv_bfloat16 *>(p.c) + (size_t)row * N;
#pragma unroll 1
            for (int c = 0; c < M2_BN / 32; c++) {
                float v[32];
                tmem_ld32(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * M2_BN + c * 32), v);
                const int col = x.n0 + c * 32;
                if (row < M) {
                    if (vec && col + 32 <= nend) {
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            uint4 pk;
                            __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                            for (int e = 0; e < 4; e++) h[e] = __floats2bfloat162_rn(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
                            *reinterpret_cast<uint4 *>(crow + col + j * 8) = pk;
                        }
                    } else {
                        for (int j = 0; j < 32; j++)
                            if (col + j < nend) crow[col + j] = __float2bfloat16_rn(v[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? te1 : te0);
            if (++acc == 2) { acc = 0; aph ^= 1; }
        }
    }
    tc_fence_before();
    __syncthreads();
    __syncwarp();
    cluster_sync();                        // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tbase, 512);
    }
}

// ---- irx_mm_bf16_wide: CTA pairs over 256x512 tiles, TMA-store epilogue ----
//
// The pair scheme of irx_mm_bf16_pair, with each A stage used for 512 columns: per K-step of 16
// the leader issues two tcgen05.mma.cta_group::2 of M = 256, N = 256 (columns n0 .. n0+255 and
// n0+256 .. n0+511 of the tile), both reading the same A tile. So each CTA loads per 64-deep
// K-block its 128 A rows (16 KB) and two 128-column chunks of B (32 KB): 48 KB for 4 MMAs of
// 128 cycles, where the 256x256 pair tile loads 32 KB for 2 -- a quarter less L2-to-SM traffic,
// which under the power cap is clock. The accumulator is the whole of TMEM (two 256-column
// halves), so the epilogue must drain it before the next tile's first MMA; the producer keeps
// loading the next tile's stages meanwhile. Epilogue: each warp reads its 32 TMEM lanes 32
// columns at a time, packs bf16 into a 128-byte-swizzled staging box (32 rows x 64 columns,
// two per warp, alternating), and one lane stores the box with a TMA store, whose map covers
// only this launch's columns (a shard's tile that reaches past its last column is clipped).
// It arrives on the leader's `tempty` as soon as its last TMEM load has landed.

#define MW_BN 512
#define MW_STAGES 4
#define MW_A_BYTES (128 * 64 * 2)                     // 16 KB: this CTA's 128 A rows x 64 k
#define MW_B_BYTES (256 * 64 * 2)                     // 32 KB: this CTA's two 128-column B chunks
#define MW_STAGE_BYTES (MW_A_BYTES + MW_B_BYTES)
#define MW_STG_BYTES (32 * 128)                       // one staging box: 32 rows x 64 bf16

__device__ __forceinline__ MmTile mw_tile(int t, int ntm, int ntn, int n0, int group)
{
    const int per_group = group * ntn;
    const int g = t / per_group;
    const int first = g * group;
    const int gsize = min(ntm - first, group);
    const int r = t % per_group;
    MmTile x;
    x.m0 = (first + r % gsize) * 256;
    x.n0 = n0 + (r / gsize) * MW_BN;
    return x;
}

extern "C" __global__ void __launch_bounds__(192, 1) irx_mm_bf16_wide(const __grid_constant__ irx_kmm_t p)
{
    irx_pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *sa = smem;
    unsigned char *sb = smem + MW_STAGES * MW_A_BYTES;
    unsigned char *stg = smem + MW_STAGES * MW_STAGE_BYTES;          // 4 warps x 2 boxes
    uint64_t *full = reinterpret_cast<uint64_t *>(stg + 8 * MW_STG_BYTES);
    uint64_t *empty = full + MW_STAGES;
    uint64_t *tfull = empty + MW_STAGES;
    uint64_t *tempty = tfull + 1;
    uint64_t *done = tempty + 1;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const int M = (int)p.m, K = (int)p.k;
    const int n0 = (int)p.n0;
    const int ntm = (M + 255) / 256;
    const int ntn = (int)((p.n1 - p.n0 + MW_BN - 1) / MW_BN);
    const int tiles = ntm * ntn;
    const int nk = (K + 63) / 64;
    const int group = p.group;

    if (threadIdx.x == 0) {
        for (int s = 0; s < MW_STAGES; s++) { irx_mbar_init(&full[s], 1); irx_mbar_init(&empty[s], 1); }
        irx_mbar_init(tfull, 1);
        irx_mbar_init(tempty, 8);
        irx_mbar_init(done, 1);
        irx_fence_mbar_init();
        tma_prefetch_desc(&p.tma_a);
        tma_prefetch_desc(&p.tma_b);
        tma_prefetch_desc(&p.tma_c);
    }
    if (warp == 1) tmem_alloc_pair(tslot, 512);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (elect_one() && !p.no_loads) {                    // TMA producer, both CTAs
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                const MmTile x = mw_tile(t, ntm, ntn, n0, group);
                for (int kb = 0; kb < nk && ok; kb++) {
                    if (!(ok = mm_wait(&empty[s], ph ^ 1, p))) break;
                    const uint32_t fl = cluster_addr(&full[s], 0);
                    if (leader) irx_mbar_expect_tx(&full[s], 2 * MW_STAGE_BYTES);
                    tma_load_2d_pair(sa + s * MW_A_BYTES, &p.tma_a, kb * 64, x.m0 + (int)rank * 128, fl);
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        unsigned char *dst = sb + s * MW_B_BYTES + h * (MW_B_BYTES / 2);
                        const int col = x.n0 + h * 256 + (int)rank * 128;
                        if (p.b_kmajor) {
                            tma_load_2d_pair(dst, &p.tma_b, kb * 64, col, fl);
                        } else {
                            tma_load_2d_pair(dst, &p.tma_b, col, kb * 64, fl);
                            tma_load_2d_pair(dst + 64 * 64 * 2, &p.tma_b, col + 64, kb * 64, fl);
                        }
                    }
                    if (++s == MW_STAGES) { s = 0; ph ^= 1; }
                }
            }
            for (int i = 0; i < MW_STAGES && ok; i++) {      // every loaded stage consumed
                ok = mm_wait(&empty[s], ph ^ 1, p);
                if (++s == MW_STAGES) { s = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        if (leader && elect_one()) {                         // MMA issuer: the leader CTA only
            const uint32_t idesc = umma_idesc_bf16(256, 256, p.b_kmajor ? 0 : 1);
            int s = 0;
            uint32_t ph = 0, tph = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                if (!(ok = mm_wait(tempty, tph ^ 1, p))) break;       // the epilogues drained TMEM
                tc_fence_after();
                for (int kb = 0; kb < nk && ok; kb++) {
                    if (!(ok = mm_wait(&full[s], ph, p))) break;
                    tc_fence_after();
                    const uint32_t a0 = irx_smem_u32(sa + s * MW_A_BYTES);
                    const uint32_t b0 = irx_smem_u32(sb + s * MW_B_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t bh = b0 + h * (MW_B_BYTES / 2);
                            const uint64_t bd = p.b_kmajor ? umma_desc_sw128(bh + k * 32, 16, 1024)
                                                           : umma_desc_sw128(bh + k * 16 * 128, 64 * 64 * 2, 1024);
                            umma_bf16_pair(tbase + (uint32_t)(h * 256), ad, bd, idesc, (kb | k) != 0);
                        }
                    }
                    umma_commit_pair(&empty[s], 0x3);
                    if (++s == MW_STAGES) { s = 0; ph ^= 1; }
                }
                if (ok) umma_commit_pair(tfull, 0x3);
                tph ^= 1;
            }
            umma_commit_pair(done, 0x1);
            mm_wait(done, 0, p);
        }
    } else {                                                  // epilogue: warps 2-5 of both CTAs
        const int q = warp & 3;                               // this warp's TMEM lane quarter
        unsigned char *box0 = stg + (q * 2) * MW_STG_BYTES;
        const uint32_t te = cluster_addr(tempty, 0);
        uint32_t tph = 0, sc = 0;
        for (int t = pair; t < tiles; t += npairs) {
            const MmTile x = mw_tile(t, ntm, ntn, n0, group);
            if (!__all_sync(0xffffffffu, mm_wait(tfull, tph, p))) break;
            tc_fence_after();
            const int row0 = x.m0 + (int)rank * 128 + q * 32;
#pragma unroll 1
            for (int b = 0; b < MW_BN / 64; b++, sc++) {
                unsigned char *box = box0 + (sc & 1) * MW_STG_BYTES;
                if (sc >= 2) {                                // the store two boxes back has read this one
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
                }
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    float v[32];
                    tmem_ld32(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 64 + h * 32), v);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        uint4 pk;
                        __nv_bfloat162 *hh = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                        for (int e = 0; e < 4; e++) hh[e] = __floats2bfloat162_rn(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
                        const int chunk = (h * 4 + j) ^ (lane & 7);         // the 128-byte swizzle
                        *reinterpret_cast<uint4 *>(box + lane * 128 + chunk * 16) = pk;
                    }
                }
                if (b == MW_BN / 64 - 1) {                    // every TMEM load of this tile has landed
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(te);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&p.tma_c, box, x.n0 + b * 64, row0);
                    bulk_commit();
                }
            }
            tph ^= 1;
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    __syncwarp();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tbase, 512);
    }
}

// ---- SIMT fallback: 64x64 output tiles, 4x4 per thread, k ascending ----

template <typename T>
__device__ __forceinline__ float mm_ld(const T *p, int64_t i);
template <>
__device__ __forceinline__ float mm_ld<float>(const float *p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float mm_ld<__nv_bfloat16>(const __nv_bfloat16 *p, int64_t i) { return __bfloat162float(p[i]); }

template <typename T>
__device__ __forceinline__ void mm_st(T *p, int64_t i, float v);
template <>
__device__ __forceinline__ void mm_st<float>(float *p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void mm_st<__nv_bfloat16>(__nv_bfloat16 *p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

template <typename T>
__device__ __forceinline__ void mm_simt(const irx_kmm_t &p)
{
    __shared__ float As[16][65], Bs[16][65];
    const int64_t M = p.m, N = p.n, K = p.k;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t ncol = p.n1 - p.n0;
    const int64_t tn = (ncol + 63) / 64, tm = (M + 63) / 64;
    const T *A = reinterpret_cast<const T *>(p.a);
    const T *B = reinterpret_cast<const T *>(p.b);
    T *C = reinterpret_cast<T *>(p.c);
    for (int64_t t = blockIdx.x; t < tm * tn; t += gridDim.x) {
        const int64_t m0 = (t / tn) * 64, n0 = p.n0 + (t % tn) * 64;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
        for (int64_t k0 = 0; k0 < K; k0 += 16) {
            for (int e = threadIdx.x; e < 16 * 64; e += 256) {
                const int kk = e / 64, mm = e % 64;
                const int64_t gm = m0 + mm, gk = k0 + kk, gn = n0 + mm;
                As[kk][mm] = (gm < M && gk < K) ? mm_ld<T>(A, gm * K + gk) : 0.0f;
                float bv = 0.0f;
                if (gn < p.n1 && gk < K) bv = p.b_kmajor ? mm_ld<T>(B, gn * K + gk) : mm_ld<T>(B, gk * N + gn);
                Bs[kk][mm] = bv;
            }
            __syncthreads();
            const int kmax = (int)min((int64_t)16, K - k0);
            for (int kk = 0; kk < kmax; kk++) {
                float a[4], b[4];
#pragma unroll
                for (int i = 0; i < 4; i++) { a[i] = As[kk][ty * 4 + i]; b[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
                if (gm < M && gn < p.n1) mm_st<T>(C, gm * N + gn, acc[i][j]);
            }
    }
}

extern "C" __global__ void __launch_bounds__(256) irx_mm_f32(const __grid_constant__ irx_kmm_t p) { irx_pdl_enter(); mm_simt<float>(p); }
extern "C" __global__ void __launch_bounds__(256) irx_mm_bf16_simt(const __grid_constant__ irx_kmm_t p) { irx_pdl_enter(); mm_simt<__nv_bfloat16>(p); }
