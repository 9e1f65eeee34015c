// Int8 stage-1 IVF scan on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Same contract as the reference's `_first8c` / `_emit8c` (`throughput/ivf8c_kern.py:2-36`): one CTA owns a tile of
// 128 code rows of one cell, starting on a global 32-row boundary so that epilogue warp w covers exactly the
// reference's 32-row block blk = row0/32 + w (`src/s1cell.py:161-168`).
//
// Persistent kernel: one CTA per SM walks the tiles b, b + G, b + 2G, ... of the static work list (skipping cells no
// query probes).  A tile is split into sub-tiles of up to 64 of the cell's queries; sub-tiles are numbered in walk
// order (nb).  Warp roles (672 threads):
//   warp 0      : TMA loads of the 128 x 256 B code tiles (two 128 B-wide boxes, 128 B swizzle), A_STAGES (4) ahead
//   warp 1      : TMEM allocation; lane 0 issues tcgen05.mma.kind::i8 (M=128 rows, N=16..64 queries, K=32 x 8) per
//                 sub-tile into one of T_STAGES accumulators, and releases a code tile when its last MMA completes
//                 and a query tile as soon as its own MMAs complete
//   warps 2-4   : gather: warp 2+g fills the sub-tiles nb = g (mod 3) -- the rows of q8 picked by qid, in the
//                 canonical K-major 128 B-swizzled layout, into query-tile stage g, and the sub-tile's scales / pair
//                 constants / thresholds / row scales into the metadata slot of its accumulator stage (nb mod
//                 T_STAGES, freed by the epilogue together with the accumulator) -- so three sub-tiles' dependent
//                 loads are in flight at once and a query tile is not held through the epilogue
//   warps 5-20  : four epilogue warpgroups, group e on the sub-tiles nb = e (mod 4): tcgen05.ld of the warp's 32 TMEM
//                 lanes (= code rows) 32 columns (queries) at a time, est = ((acc * qs) * zs) + qcp in fp32 with
//                 explicit rounding, then first pass: per-query block maximum by one redux.sync.max, or emit:
//                 per-row kept-column masks transposed across the warp (lane j: the rows keeping column j), lane j
//                 reserving space for column j with one atomicAdd (a chunk's 32 atomics in flight together), prefix
//                 positions by popc, each row's kept estimates picked from registers by a select tree.
// So the loads and MMAs of the next sub-tiles and tiles overlap the epilogues of the current ones.
// Every mbarrier wait is bounded; on expiry the CTA raises `status`, drains what it issued, frees TMEM and returns.
#include <cuda.h>

#include "fvs_common.cuh"
#include "fvs_tcgen05.cuh"

namespace fvs {
namespace tc {
using namespace fvs::tcg;

#ifndef FVS_TC_A_STAGES
#define FVS_TC_A_STAGES 4
#endif
#ifndef FVS_TC_GATHER_WARPS
#define FVS_TC_GATHER_WARPS 3
#endif
#ifndef FVS_TC_MAXT
#define FVS_TC_MAXT 512
#endif
constexpr int TILE_ROWS = 128;
constexpr int QN = 64;  // queries per sub-tile
constexpr int RB = 256;
constexpr int A_STAGES = FVS_TC_A_STAGES;
constexpr int GATHER_WARPS = FVS_TC_GATHER_WARPS;
constexpr int B_STAGES = GATHER_WARPS;  // gather warp g owns B stage g
constexpr int T_STAGES = 8;
constexpr int EPI_GROUPS = 4;
constexpr int NTHREADS = 32 * (2 + GATHER_WARPS + 4 * EPI_GROUPS);
constexpr uint32_t TMEM_COLS = T_STAGES * QN;  // int32 accumulator columns

// shared-memory carve-up (offsets from a 1024-byte aligned base)
constexpr int A_BYTES = 2 * TILE_ROWS * 128;               // one code tile: 2 K-halves x 16 KB
constexpr int B_BYTES = 2 * QN * 128;                      // one query sub-tile: 2 K-halves x 8 KB
constexpr int A_OFF = 0;
constexpr int B_OFF = A_OFF + A_STAGES * A_BYTES;
constexpr int META_OFF = B_OFF + B_STAGES * B_BYTES;       // T_STAGES x 4 x QN x 4 B (per accumulator stage)
constexpr int ZS_OFF = META_OFF + T_STAGES * 4 * QN * 4;   // T_STAGES x TILE_ROWS x 4 B (row scales of the sub-tile)
constexpr int MAXT = FVS_TC_MAXT;                          // tiles of one round of a CTA's walk
constexpr int LIST_OFF = ZS_OFF + T_STAGES * TILE_ROWS * 4; // 5 x MAXT int32: row0, cs, ce, qoff, qn
constexpr int COL_OFF = LIST_OFF + 5 * MAXT * 4;           // per epilogue warp: 32 column masks + 32 bases
constexpr int BAR_OFF = COL_OFF + 16 * 64 * 4;             // mbarriers
constexpr int NBAR = 2 * A_STAGES + 2 * B_STAGES + 3 * T_STAGES + 1;  // + the MMA drain barrier
constexpr int MISC_OFF = BAR_OFF + NBAR * 8;               // tmem base, abort flag, list length, scan scratch
constexpr int SMEM_BYTES = MISC_OFF + 16 + 128 + 1024;     // + alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(NTHREADS / 32 <= 32, "per-warp scratch holds 32 warps");

struct Params {
    const int8_t* q8;
    const float* qs;
    const int32_t* qid;
    const int32_t* coff;
    const int32_t* ccnt;
    const float* qcp;
    const int32_t* tile_cell;
    const int32_t* tile_row0;
    const int64_t* off;
    const float* zs;
    const float* t0;
    int32_t* cnt;
    float* bval;
    int32_t* bpos;
    float* bmc;
    int32_t* status;
    int M, MB;
    uint32_t wait_limit;  // polls of every pipeline wait (fvs_set_wait_limit)
};

// 32 x 32 bit-matrix transpose across a warp: lane r holds row r (bit c = entry (r, c)); returns row `lane` of the
// transpose (bit r = entry (r, lane)).  Five butterfly stages swap the off-diagonal blocks of width 16, 8, 4, 2, 1.
__device__ __forceinline__ uint32_t transpose32(uint32_t x) {
    const int lane = threadIdx.x & 31;
    const uint32_t ms[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
    for (int k = 0; k < 5; k++) {
        const int j = 16 >> k;
        const uint32_t m = ms[k];
        const uint32_t y = __shfl_xor_sync(0xffffffffu, x, j);
        x = (lane & j) ? ((x & ~m) | ((y >> j) & m)) : ((x & m) | ((y & m) << j));
    }
    return x;
}

// a[jj] for a run-time jj without local memory: a five-level select tree on the index bits (31 selects)
__device__ __forceinline__ uint32_t select32(const uint32_t (&a)[32], int jj) {
    uint32_t t16[16], t8[8], t4[4], t2[2];
#pragma unroll
    for (int i = 0; i < 16; i++) t16[i] = (jj & 1) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
    for (int i = 0; i < 8; i++) t8[i] = (jj & 2) ? t16[2 * i + 1] : t16[2 * i];
#pragma unroll
    for (int i = 0; i < 4; i++) t4[i] = (jj & 4) ? t8[2 * i + 1] : t8[2 * i];
#pragma unroll
    for (int i = 0; i < 2; i++) t2[i] = (jj & 8) ? t4[2 * i + 1] : t4[2 * i];
    return (jj & 16) ? t2[1] : t2[0];
}

template <int MODE>
__global__ void __launch_bounds__(NTHREADS, 1) scan_tc_kernel(const __grid_constant__ CUtensorMap zmap, Params p,
                                                              int ntiles) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = saddr(smem);
    auto a_full = [&](int s) { return sbase + BAR_OFF + 8 * s; };
    auto a_empty = [&](int s) { return sbase + BAR_OFF + 8 * (A_STAGES + s); };
    auto b_full = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + s); };
    auto b_empty = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + B_STAGES + s); };
    auto t_full = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + s); };
    auto t_empty = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + T_STAGES + s); };
    auto m_full = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 2 * T_STAGES + s); };
    const uint32_t d_bar = sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 3 * T_STAGES);
    const uint32_t WL = p.wait_limit;
    int* meta_qid = reinterpret_cast<int*>(smem + META_OFF);          // [T_STAGES][QN]
    float* meta_qs = reinterpret_cast<float*>(meta_qid + T_STAGES * QN);
    float* meta_qc = meta_qs + T_STAGES * QN;
    float* meta_th = meta_qc + T_STAGES * QN;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + MISC_OFF);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);

    if (tid == 0) {
        for (int s = 0; s < A_STAGES; s++) {
            mbar_init(a_full(s), 1);
            mbar_init(a_empty(s), 1);
        }
        for (int s = 0; s < B_STAGES; s++) {
            mbar_init(b_full(s), 1);
            mbar_init(b_empty(s), 1);  // released by the MMA commit of its sub-tile
        }
        for (int s = 0; s < T_STAGES; s++) {
            mbar_init(t_full(s), 1);
            mbar_init(t_empty(s), 4);  // accumulator + metadata slot, released by the epilogue
            mbar_init(m_full(s), 1);   // metadata slot written by its gather warp
        }
        mbar_init(d_bar, 1);           // every MMA this CTA issued has completed (before TMEM is freed)
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int G = gridDim.x;
    int* L_row0 = reinterpret_cast<int*>(smem + LIST_OFF);
    int* L_cs = L_row0 + MAXT;
    int* L_ce = L_cs + MAXT;
    int* L_qoff = L_ce + MAXT;
    int* L_qn = L_qoff + MAXT;
    volatile int* L_len = reinterpret_cast<volatile int*>(smem + MISC_OFF + 8);
    int* wsum = reinterpret_cast<int*>(smem + MISC_OFF + 16);  // one slot per warp, up to 32 warps
    float* zsm = reinterpret_cast<float*>(smem + ZS_OFF);
    const int nlocal = ntiles > blockIdx.x ? (ntiles - blockIdx.x + G - 1) / G : 0;

    // per-role pipeline counters persist across rounds
    int na_tma = 0, na_mma = 0, nb_mma = 0, nb_g = 0, nb_e = 0;
    bool mma_issued = false;
    for (int r0 = 0; r0 < nlocal; r0 += MAXT) {
        // ---- stage this round's tiles (skipping cells no query probes) in shared memory, in walk order
        {
            const int cnt_r = min(MAXT, nlocal - r0);
            // NTHREADS >= MAXT is not required: loop in chunks of NTHREADS
            int base = 0;
            for (int c0 = 0; c0 < cnt_r; c0 += NTHREADS) {
                const int li = c0 + tid;
                int qn = 0, row0 = 0, cs = 0, ce = 0, qoff = 0;
                if (li < cnt_r) {
                    const int tile = blockIdx.x + (r0 + li) * G;
                    const int c = p.tile_cell[tile];
                    row0 = p.tile_row0[tile];
                    qn = p.ccnt[c];
                    cs = (int)p.off[c];
                    ce = (int)p.off[c + 1];
                    qoff = p.coff[c];
                }
                const bool act = qn > 0;
                const unsigned bal = __ballot_sync(0xffffffffu, act);
                if (lane == 0) wsum[warp] = __popc(bal);
                __syncthreads();
                int before = base;
                for (int w = 0; w < warp; w++) before += wsum[w];
                int tot = 0;
                for (int w = 0; w < NTHREADS / 32; w++) tot += wsum[w];
                if (act) {
                    const int at = before + __popc(bal & ((1u << lane) - 1u));
                    L_row0[at] = row0;
                    L_cs[at] = cs;
                    L_ce[at] = ce;
                    L_qoff[at] = qoff;
                    L_qn[at] = qn;
                }
                base += tot;
                __syncthreads();
            }
            if (tid == 0) *L_len = base;
            __syncthreads();
        }
        const int len = *L_len;

        if (warp == 0) {
            // ---- code tiles by TMA
            if (lane == 0) {
                if (r0 == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&zmap) : "memory");
                for (int t = 0; t < len && !*abort; t++) {
                    const int s = na_tma % A_STAGES;
                    if (!mbar_wait(a_empty(s), ((na_tma / A_STAGES) & 1) ^ 1, abort, WL)) break;
                    const int row0 = L_row0[t];
                    mbar_expect_tx(a_full(s), A_BYTES);
                    tma_load_2d(sbase + A_OFF + s * A_BYTES, &zmap, 0, row0, a_full(s));
                    tma_load_2d(sbase + A_OFF + s * A_BYTES + TILE_ROWS * 128, &zmap, 128, row0, a_full(s));
                    na_tma++;
                }
            }
        } else if (warp == 1) {
            // ---- MMA issue
            if (lane == 0) {
                for (int t = 0; t < len && !*abort; t++) {
                    const int qn = L_qn[t];
                    const int sa = na_mma % A_STAGES;
                    if (!mbar_wait(a_full(sa), (na_mma / A_STAGES) & 1, abort, WL)) break;
                    tc_fence_after();
                    const uint32_t abase = sbase + A_OFF + sa * A_BYTES;
                    bool ok = true;
                    for (int i = 0; i * QN < qn; i++, nb_mma++) {
                        const int sb = nb_mma % B_STAGES, st = nb_mma % T_STAGES;
                        if (!mbar_wait(b_full(sb), (nb_mma / B_STAGES) & 1, abort, WL) ||
                            !mbar_wait(t_empty(st), ((nb_mma / T_STAGES) & 1) ^ 1, abort, WL)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const int nq = min(QN, qn - i * QN);
                        const uint32_t idesc = i8_idesc((nq + 15) & ~15);
                        const uint32_t d = tmem + (uint32_t)(st * QN);
                        const uint32_t bb = sbase + B_OFF + sb * B_BYTES;
#pragma unroll
                        for (int ks = 0; ks < RB / 32; ks++) {
                            const int h = ks >> 2, kofs = (ks & 3) * 32;
                            mma_i8(d, sw128_desc(abase + h * TILE_ROWS * 128 + kofs),
                                   sw128_desc(bb + h * QN * 128 + kofs), idesc, ks > 0 ? 1u : 0u);
                        }
                        mma_issued = true;
                        mma_commit(t_full(st));
                        mma_commit(b_empty(sb));  // the query tile is free once these MMAs complete
                    }
                    if (!ok) break;
                    mma_commit(a_empty(sa));  // the code tile is free once these MMAs complete
                    na_mma++;
                }
            }
            __syncwarp();
        } else if (warp < 2 + GATHER_WARPS) {
            // ---- query gather: warp gw fills the sub-tiles nb = gw (mod GATHER_WARPS); lane l fills rows l, l + 32
            const int gw = warp - 2;
            for (int t = 0; t < len && !*abort; t++) {
                const int qn = L_qn[t], qoff = L_qoff[t], row0 = L_row0[t], cs = L_cs[t], ce = L_ce[t];
                bool ok = true;
                for (int i = 0; i * QN < qn; i++, nb_g++) {
                    if (nb_g % GATHER_WARPS != gw) continue;
                    const int s = nb_g % B_STAGES;
                    const int st = nb_g % T_STAGES;
                    const int nq = min(QN, qn - i * QN);
                    const int n16 = (nq + 15) & ~15;
                    // the sub-tile's scalars are loaded before waiting for its slots (they do not depend on them), so
                    // their latency overlaps the wait: row scales (rows outside the cell read as 0), query ids, then
                    // the per-query scale / pair constant / threshold
                    float zv[TILE_ROWS / 32];
#pragma unroll
                    for (int rr = 0; rr < TILE_ROWS / 32; rr++) {
                        const int row = row0 + 32 * rr + lane;
                        zv[rr] = (row >= cs && row < ce) ? p.zs[row] : 0.f;
                    }
                    int qq[2];
                    float qsv[2], qcv[2], thv[2];
#pragma unroll
                    for (int rr = 0; rr < 2; rr++) {
                        const int g = lane + 32 * rr;
                        qq[rr] = -1;
                        qsv[rr] = qcv[rr] = thv[rr] = 0.f;
                        if (g < nq) {
                            const int pi = qoff + i * QN + g;
                            qq[rr] = p.qid[pi];
                            qcv[rr] = p.qcp[pi];
                        }
                    }
#pragma unroll
                    for (int rr = 0; rr < 2; rr++)
                        if (qq[rr] >= 0) {
                            qsv[rr] = p.qs[qq[rr]];
                            thv[rr] = MODE ? p.t0[qq[rr]] : 0.f;
                        }
                    if (!warp_wait(b_empty(s), ((nb_g / B_STAGES) & 1) ^ 1, abort, WL) ||
                        !warp_wait(t_empty(st), ((nb_g / T_STAGES) & 1) ^ 1, abort, WL)) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int rr = 0; rr < TILE_ROWS / 32; rr++) zsm[st * TILE_ROWS + 32 * rr + lane] = zv[rr];
#pragma unroll
                    for (int rr = 0; rr < 2; rr++) {
                        const int g = lane + 32 * rr;
                        if (g < nq) {
                            meta_qid[st * QN + g] = qq[rr];
                            meta_qs[st * QN + g] = qsv[rr];
                            meta_qc[st * QN + g] = qcv[rr];
                            meta_th[st * QN + g] = thv[rr];
                        }
                    }
#pragma unroll
                    for (int rr = 0; rr < 2; rr++) {
                        const int g = lane + 32 * rr;
                        if (g >= n16) continue;
                        const int q = qq[rr];
                        const uint4* src = reinterpret_cast<const uint4*>(p.q8 + (int64_t)(q >= 0 ? q : 0) * RB);
                        uint8_t* bs = smem + B_OFF + s * B_BYTES + (g >> 3) * 1024 + (g & 7) * 128;
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            uint4 v[8];
#pragma unroll
                            for (int cc = 0; cc < 8; cc++)
                                v[cc] = q >= 0 ? __ldg(src + 8 * h + cc) : make_uint4(0, 0, 0, 0);
#pragma unroll
                            for (int cc = 0; cc < 8; cc++)
                                *reinterpret_cast<uint4*>(bs + h * QN * 128 + ((cc ^ (g & 7)) << 4)) = v[cc];
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(b_full(s));
                        mbar_arrive(m_full(st));
                    }
                }
                if (!ok) break;
            }
        } else {
            // ---- epilogue: group eg = sub-tiles nb = eg (mod EPI_GROUPS); warp ew = warp % 4 reads TMEM lanes
            //      32*ew .. 32*ew+31 (tile rows)
            const int eg = (warp - 2 - GATHER_WARPS) / 4;
            const int ew = warp & 3;
            for (int t = 0; t < len && !*abort; t++) {
                const int qn = L_qn[t], qoff = L_qoff[t], row0 = L_row0[t], cs = L_cs[t], ce = L_ce[t];
                const int row = row0 + 32 * ew + lane;
                const bool rvalid = row >= cs && row < ce;
                const bool wactive = row0 + 32 * ew < ce;
                const int blk_rel = (row0 + 32 * ew) / 32 - cs / 32;
                bool ok = true;
                for (int i = 0; i * QN < qn; i++, nb_e++) {
                    if (nb_e % EPI_GROUPS != eg) continue;
                    const int st = nb_e % T_STAGES;
                    if (!warp_wait(t_full(st), (nb_e / T_STAGES) & 1, abort, WL) ||
                        !warp_wait(m_full(st), (nb_e / T_STAGES) & 1, abort, WL)) {  // m_full: acquire the metadata
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int nq = min(QN, qn - i * QN);
                    const uint32_t ta = tmem + ((uint32_t)(32 * ew) << 16) + (uint32_t)(st * QN);
                    const int* mq = meta_qid + st * QN;
                    const float* ms = meta_qs + st * QN;
                    const float* mc = meta_qc + st * QN;
                    const float* mt = meta_th + st * QN;
                    const float zr = zsm[st * TILE_ROWS + 32 * ew + lane];
                    uint32_t* colm = reinterpret_cast<uint32_t*>(smem + COL_OFF) + (warp - 2 - GATHER_WARPS) * 64;
                    int* colb = reinterpret_cast<int*>(colm + 32);
                    for (int h = 0; h * 32 < nq; h++) {
                        uint32_t acc[32];
                        tmem_ld32(ta + 32 * h, acc);
                        tmem_ld_wait();
                        if (!wactive) continue;
                        const int nc = min(32, nq - h * 32);
                        const float4* ms4 = reinterpret_cast<const float4*>(ms + 32 * h);
                        const float4* mc4 = reinterpret_cast<const float4*>(mc + 32 * h);
                        if (MODE == 0) {
#pragma unroll
                            for (int j4 = 0; j4 < 8; j4++) {
                                if (4 * j4 >= nc) break;
                                const float4 sv = ms4[j4], cv = mc4[j4];
                                const float s4[4] = {sv.x, sv.y, sv.z, sv.w}, c4[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
                                for (int u = 0; u < 4; u++) {
                                    const int jj = 4 * j4 + u;
                                    if (jj < nc) {
                                        const float est =
                                            __fadd_rn(__fmul_rn(__fmul_rn((float)(int32_t)acc[jj], s4[u]), zr), c4[u]);
                                        const uint32_t m = __reduce_max_sync(0xffffffffu, rvalid ? f2o(est) : 0u);
                                        if (lane == 0)
                                            p.bmc[(int64_t)(qoff + i * QN + 32 * h + jj) * p.MB + blk_rel] = o2f(m);
                                    }
                                }
                            }
                        } else {
                            // every row its kept columns (a bit mask), their transpose (lane jj: the rows keeping
                            // column jj), then lane jj reserves space for column jj: the chunk's atomics are in
                            // flight together; finally every row writes only its own kept entries
                            const float4* mt4 = reinterpret_cast<const float4*>(mt + 32 * h);
                            uint32_t mymask = 0, rowmask = 0;
#pragma unroll
                            for (int j4 = 0; j4 < 8; j4++) {
                                if (4 * j4 >= nc) break;
                                const float4 sv = ms4[j4], cv = mc4[j4], tv = mt4[j4];
                                const float s4[4] = {sv.x, sv.y, sv.z, sv.w}, c4[4] = {cv.x, cv.y, cv.z, cv.w};
                                const float t4[4] = {tv.x, tv.y, tv.z, tv.w};
#pragma unroll
                                for (int u = 0; u < 4; u++) {
                                    const int jj = 4 * j4 + u;
                                    if (jj < nc) {
                                        const float est =
                                            __fadd_rn(__fmul_rn(__fmul_rn((float)(int32_t)acc[jj], s4[u]), zr), c4[u]);
                                        const bool keep = rvalid && est >= t4[u];
                                        acc[jj] = __float_as_uint(est);  // the column's estimate from here on
                                        rowmask |= (uint32_t)keep << jj;
                                    }
                                }
                            }
                            mymask = transpose32(rowmask);  // lane jj: the rows keeping column jj
                            int mybase = 0;
                            if (mymask) mybase = atomicAdd(p.cnt + mq[32 * h + lane], __popc(mymask));
                            colm[lane] = mymask;
                            colb[lane] = mybase;
                            __syncwarp();
                            while (rowmask) {
                                const int jj = __ffs(rowmask) - 1;
                                rowmask &= rowmask - 1;
                                const int j = 32 * h + jj;
                                const float est = __uint_as_float(select32(acc, jj));
                                const int idx = colb[jj] + __popc(colm[jj] & ((1u << lane) - 1u));
                                if (idx < p.M) {
                                    const int64_t o = (int64_t)mq[j] * p.M + idx;
                                    p.bval[o] = est;
                                    p.bpos[o] = row;
                                }
                            }
                            __syncwarp();
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(t_empty(st));
                    }
                }
                if (!ok) break;
            }
        }
        __syncthreads();  // the round's list is consumed by every role before it is overwritten
    }
    // drain (waits that ignore the abort flag): the most recent load of every A stage has landed, and one commit
    // after the last MMA this thread issued has arrived, i.e. every MMA of this CTA has completed
    if (warp == 0 && lane == 0)
        for (int u = na_tma - 1; u >= 0 && u >= na_tma - A_STAGES; u--) mbar_drain(a_full(u % A_STAGES), (u / A_STAGES) & 1);
    if (warp == 1 && lane == 0 && mma_issued) {
        mma_commit(d_bar);
        mbar_drain(d_bar, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    if (tid == 0 && *abort && p.status) atomicExch(p.status, 1);
}

}  // namespace tc
}  // namespace fvs

extern "C" int fvs_i8_scan_tc(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                              const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                              const int32_t* tile_cell, const int32_t* tile_row0, int ntiles, const int64_t* off,
                              int NC, const int8_t* Z, int64_t N, const float* zs, const float* t0, int32_t* cnt,
                              float* bval, int32_t* bpos, int M, float* bmc, int MB, int32_t* status) {
    using namespace fvs::tc;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(R == RB && B >= 0 && ntiles >= 0 && NC > 0 && N > 0);
    FVS_CHECK_ARG(q8 && qs && qid && coff && ccnt && qcp && tile_cell && tile_row0 && off && Z && zs);
    FVS_CHECK_ARG(((uintptr_t)Z & 15) == 0 && ((uintptr_t)q8 & 15) == 0);
    if (mode == 0) FVS_CHECK_ARG(bmc && MB > 0);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (ntiles == 0 || B == 0) return FVS_OK;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)RB, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)RB};
    const cuuint32_t box[2] = {128, (cuuint32_t)TILE_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)Z, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return FVS_EINVAL;
    Params p{q8,  qs,  qid, coff, ccnt, qcp,    tile_cell, tile_row0, off, zs,
             t0,  cnt, bval, bpos, bmc, status, M,         MB,        pipeline_wait_limit()};
    cudaError_t e = mode ? fvs_ensure_smem((const void*)scan_tc_kernel<1>, SMEM_BYTES)
                         : fvs_ensure_smem((const void*)scan_tc_kernel<0>, SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    static int nsm = 0;
    if (nsm == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 148;
    }
    const int grid = ntiles < nsm ? ntiles : nsm;
    if (mode == 0)
        scan_tc_kernel<0><<<grid, NTHREADS, SMEM_BYTES, stream>>>(map, p, ntiles);
    else
        scan_tc_kernel<1><<<grid, NTHREADS, SMEM_BYTES, stream>>>(map, p, ntiles);
    return fvs_launch_status();
}
