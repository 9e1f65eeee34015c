// Int8 stage-1 IVF scan (first pass / threshold emit) for sm_100a.
//
// Replaces `_first8c` / `_emit8c` (`throughput/ivf8c_kern.py:2-36`) and `ivf8` (`throughput/civf8.py:15-83`).
// One CTA owns one tile of TILE_ROWS (=128) code rows of one cell: the tile starts on a global 32-row boundary, so
// warp w covers exactly the reference's global block blk = row0/32 + w (`src/s1cell.py:161-168`), which keeps the
// first-pass block maxima identical to the reference's.  The code tile is staged once in shared memory with cp.async
// and reused for every query of the cell; queries come in tiles of QT (=64), gathered by qid from q8 (L2-resident).
// Scores: int8 x int8 -> int32 on the tensor cores (mma m16n8k32), then the reference's fp32 sequence
// est = ((float(acc) * qs[q]) * zs[n]) + qcp[pair] with explicit round-to-nearest operations (no FMA contraction).
// Epilogue (emit): per (query, 32-row block) the 4 lanes holding that query's 32 scores count their kept entries,
// one lane reserves space with a single atomicAdd, and every lane writes its entries at base + prefix.
#include "fvs_common.cuh"

namespace fvs {
namespace i8scan {

constexpr int TILE_ROWS = 128;
constexpr int QT = 64;        // queries per query tile
constexpr int RB = 256;       // code bytes per row (R = 256)
constexpr int RS = RB + 16;   // padded shared-memory row stride (bank-conflict-free ldmatrix)
constexpr int NTHREADS = 128;

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
    const int8_t* Z;
    const float* zs;
    const float* t0;
    int32_t* cnt;
    float* bval;
    int32_t* bpos;
    float* bmc;
    int M, MB;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    const int sz = valid ? 16 : 0;  // src-size 0 zero-fills the 16 destination bytes
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::);
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int MODE>
__global__ void __launch_bounds__(NTHREADS) scan_kernel(Params p) {
    extern __shared__ __align__(16) uint8_t smem[];
    int8_t* zt = reinterpret_cast<int8_t*>(smem);            // TILE_ROWS x RS
    int8_t* qt = zt + TILE_ROWS * RS;                          // QT x RS
    float* zsc = reinterpret_cast<float*>(qt + QT * RS);       // TILE_ROWS
    float* qsc = zsc + TILE_ROWS;                               // QT
    float* qcs = qsc + QT;                                      // QT
    float* thr = qcs + QT;                                      // QT
    int* qids = reinterpret_cast<int*>(thr + QT);               // QT

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x;
    const int c = p.tile_cell[tile];
    const int qn = p.ccnt[c];
    if (qn == 0) return;
    const int64_t cs = p.off[c], ce = p.off[c + 1];
    const int64_t row0 = p.tile_row0[tile];
    const int qoff = p.coff[c];

    // ---- stage the code tile (rows outside the cell are zero) and its scales
    for (int i = tid; i < TILE_ROWS * (RB / 16); i += NTHREADS) {
        const int r = i >> 4, ch = i & 15;
        const int64_t n = row0 + r;
        const bool v = n >= cs && n < ce;
        cp_async16(zt + r * RS + ch * 16, p.Z + (v ? n : 0) * RB + ch * 16, v);
    }
    for (int r = tid; r < TILE_ROWS; r += NTHREADS) {
        const int64_t n = row0 + r;
        zsc[r] = (n >= cs && n < ce) ? p.zs[n] : 0.f;
    }

    const int64_t wrow0 = row0 + 32 * warp;          // first row of this warp's global block
    const bool warp_active = wrow0 < ce;             // the block intersects the cell (row0 >= floor(cs/32)*32)
    const int blk_rel = (int)(wrow0 / 32 - cs / 32);  // block index within the cell
    const int g = lane >> 2, t4 = lane & 3;

    for (int qb = 0; qb < qn; qb += QT) {
        const int nq = min(QT, qn - qb);
        __syncthreads();  // previous query tile fully consumed
        if (tid < QT) {
            if (tid < nq) {
                const int pi = qoff + qb + tid;
                const int q = p.qid[pi];
                qids[tid] = q;
                qsc[tid] = p.qs[q];
                qcs[tid] = p.qcp[pi];
                thr[tid] = MODE ? p.t0[q] : 0.f;
            } else {
                qids[tid] = -1;
            }
        }
        __syncthreads();
        const int mt = (nq + 15) >> 4;  // 16-query MMA tiles actually needed
        for (int i = tid; i < mt * 16 * (RB / 16); i += NTHREADS) {
            const int r = i >> 4, ch = i & 15;
            const int q = qids[r];
            cp_async16(qt + r * RS + ch * 16, p.q8 + (int64_t)(q >= 0 ? q : 0) * RB + ch * 16, q >= 0);
        }
        cp_async_wait_all();
        __syncthreads();
        if (!warp_active) continue;

        int acc[4][4][4];
#pragma unroll
        for (int m = 0; m < 4; m++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[m][j][e] = 0;

#pragma unroll
        for (int kk = 0; kk < RB; kk += 32) {
            uint32_t b[4][2];
#pragma unroll
            for (int jp = 0; jp < 2; jp++) {
                const int nrow = 32 * warp + 16 * jp + (lane & 7) + ((lane >> 4) << 3);
                const int kb = kk + ((lane >> 3) & 1) * 16;
                ldsm_x4(b[2 * jp][0], b[2 * jp][1], b[2 * jp + 1][0], b[2 * jp + 1][1], zt + nrow * RS + kb);
            }
#pragma unroll
            for (int m = 0; m < 4; m++) {
                if (m < mt) {
                    uint32_t a[4];
                    const int qrow = 16 * m + (lane & 15);
                    ldsm_x4(a[0], a[1], a[2], a[3], qt + qrow * RS + kk + (lane >> 4) * 16);
#pragma unroll
                    for (int j = 0; j < 4; j++) mma_s8(acc[m][j], a, b[j][0], b[j][1]);
                }
            }
        }

        // ---- epilogue: thread holds queries (16m + g + 8h) x rows (32w + 8j + 2*t4 + e)
        float zr[4][2];
        bool rv[4][2];
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int r = 32 * warp + 8 * j + 2 * t4 + e;
                const int64_t n = row0 + r;
                rv[j][e] = n >= cs && n < ce;
                zr[j][e] = zsc[r];
            }
#pragma unroll
        for (int m = 0; m < 4; m++) {
            if (m >= mt) break;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int ql = 16 * m + g + 8 * h;
                const bool qv = ql < nq;
                const float qsv = qv ? qsc[ql] : 0.f, qcv = qv ? qcs[ql] : 0.f;
                float est[4][2];
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int e = 0; e < 2; e++)
                        est[j][e] = __fadd_rn(__fmul_rn(__fmul_rn((float)acc[m][j][2 * h + e], qsv), zr[j][e]), qcv);
                if (MODE == 0) {
                    float mx = -INFINITY;
#pragma unroll
                    for (int j = 0; j < 4; j++)
#pragma unroll
                        for (int e = 0; e < 2; e++)
                            if (rv[j][e]) mx = fmaxf(mx, est[j][e]);
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                    if (qv && t4 == 0) p.bmc[(int64_t)(qoff + qb + ql) * p.MB + blk_rel] = mx;
                } else {
                    const float th = qv ? thr[ql] : INFINITY;
                    unsigned kmask = 0;
#pragma unroll
                    for (int j = 0; j < 4; j++)
#pragma unroll
                        for (int e = 0; e < 2; e++)
                            if (qv && rv[j][e] && est[j][e] >= th) kmask |= 1u << (2 * j + e);
                    if (__any_sync(0xffffffffu, kmask != 0)) {
                        const int s = __popc(kmask);
                        int incl = s;
                        int v = __shfl_up_sync(0xffffffffu, incl, 1, 4);
                        if (t4 >= 1) incl += v;
                        v = __shfl_up_sync(0xffffffffu, incl, 2, 4);
                        if (t4 >= 2) incl += v;
                        const int total = __shfl_sync(0xffffffffu, incl, 3, 4);
                        int base = 0;
                        const int q = qv ? qids[ql] : 0;
                        if (t4 == 0 && total > 0) base = atomicAdd(p.cnt + q, total);
                        base = __shfl_sync(0xffffffffu, base, 0, 4) + incl - s;
#pragma unroll
                        for (int j = 0; j < 4; j++)
#pragma unroll
                            for (int e = 0; e < 2; e++)
                                if (kmask & (1u << (2 * j + e))) {
                                    if (base < p.M) {
                                        const int64_t o = (int64_t)q * p.M + base;
                                        p.bval[o] = est[j][e];
                                        p.bpos[o] = (int32_t)(row0 + 32 * warp + 8 * j + 2 * t4 + e);
                                    }
                                    base++;
                                }
                    }
                }
            }
        }
    }
}

constexpr size_t smem_bytes() {
    return (size_t)TILE_ROWS * RS + (size_t)QT * RS + TILE_ROWS * 4 + QT * 4 * 4;
}

}  // namespace i8scan
}  // namespace fvs

extern "C" int fvs_i8_tile_rows(void) { return fvs::i8scan::TILE_ROWS; }

extern "C" int fvs_i8_scan(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                           const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                           const int32_t* tile_cell, const int32_t* tile_row0, int ntiles, const int64_t* off, int NC,
                           const int8_t* Z, const float* zs, const float* t0, int32_t* cnt, float* bval, int32_t* bpos,
                           int M, float* bmc, int MB) {
    using namespace fvs::i8scan;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(R == RB && B >= 0 && ntiles >= 0 && NC > 0);
    FVS_CHECK_ARG(q8 && qs && qid && coff && ccnt && qcp && tile_cell && tile_row0 && off && Z && zs);
    if (mode == 0) FVS_CHECK_ARG(bmc && MB > 0);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (ntiles == 0 || B == 0) return FVS_OK;
    Params p{q8, qs, qid, coff, ccnt, qcp, tile_cell, tile_row0, off, Z, zs, t0, cnt, bval, bpos, bmc, M, MB};
    const size_t sm = smem_bytes();
    cudaError_t e = mode ? fvs_ensure_smem((const void*)scan_kernel<1>, sm) : fvs_ensure_smem((const void*)scan_kernel<0>, sm);
    if (e != cudaSuccess) return (int)e;
    if (mode == 0)
        scan_kernel<0><<<ntiles, NTHREADS, sm, stream>>>(p);
    else
        scan_kernel<1><<<ntiles, NTHREADS, sm, stream>>>(p);
    return fvs_launch_status();
}
