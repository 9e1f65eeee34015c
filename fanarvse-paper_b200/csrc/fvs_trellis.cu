// Default engine (cell-residual trellis code): stage-1 scan, tiered gather stage 2, fp32-keyed routing, and the
// build-time Viterbi encoder.
//
// fvs_trellis_scan replaces `_first_compact_s` / `_emit_loop_s` (`src/s1cell.py:121-154`) with the decoder of
// `src/decode2.py:5-17`: value_j = tab[state_j], state_j = ((w[j/32] << 32 | w[j/32+1]) >> (64 - L - j%32)) & (2^L-1)
// (bits MSB-first per uint32 word, `src/trellis_scan.py:10-18`), rounded to fp16 as the reference's `.to(fp16)`.
// One CTA owns 128 code rows of one cell (four of the reference's 32-row blocks): each thread decodes one row into an
// fp16 tile through a shared-memory table of fp16 value pairs indexed by (L+1)-bit windows (two states per lookup);
// queries (fp16 Q @ W1) come in tiles of 64; the dot products run on the tensor cores (mma m16n8k16, fp16 in, fp32
// accumulate) and the epilogue computes est = scale1[n] * dot + qcp (fp32, unfused) with the same first-pass /
// threshold-emit logic as the int8 scan.
#include <cuda.h>

#include "fvs_common.cuh"

namespace fvs {
namespace trellis {

constexpr int TILE_ROWS = 128;
constexpr int QT = 64;
constexpr int R = 256;
constexpr int RS = R * 2 + 16;  // fp16 row stride in bytes (ldmatrix bank-conflict free)
constexpr int NTHREADS = 256;  // two threads decode a row; warp w: rows 32*(w%4).., queries of half w/4
constexpr int MAXW = 16;         // words per row (R + L - 1 <= 512 bits)

struct Params {
    const __half* Qh;
    const int32_t* qid;
    const int32_t* coff;
    const int32_t* ccnt;
    const float* qcp;
    const int32_t* tile_cell;
    const int32_t* tile_row0;
    const int64_t* off;
    const uint32_t* words;
    const float* tab;
    const __half* scale1;
    const float* t0;
    int32_t* cnt;
    float* bval;
    int32_t* bpos;
    float* bmc;
    int W, L, M, MB, ntiles;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int MODE>
__global__ void __launch_bounds__(NTHREADS) trellis_scan_kernel(Params p) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* vt = smem;                                        // TILE_ROWS x RS (decoded fp16 values)
    uint8_t* qt = vt + TILE_ROWS * RS;                         // QT x RS (fp16 queries)
    uint32_t* tab2 = reinterpret_cast<uint32_t*>(qt + QT * RS);  // 2^(L+1): fp16 value pairs of (L+1)-bit windows
    float* ssc = reinterpret_cast<float*>(tab2 + (2 << p.L));  // TILE_ROWS row scales
    float* qcs = ssc + TILE_ROWS;                              // QT
    float* thr = qcs + QT;                                     // QT
    int* qids = reinterpret_cast<int*>(thr + QT);              // QT

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L = p.L, W = p.W;

    // pair table: window w of L+1 bits covers two consecutive states (w >> 1, w & (2^L - 1)); entry = their two
    // values rounded to fp16, first value in the low half (memory order of the decoded row)
    {
        const uint32_t mask = (1u << L) - 1u;
        for (int w = tid; w < (2 << L); w += NTHREADS) {
            const uint32_t h0 = __half_as_ushort(__float2half_rn(__ldg(p.tab + (w >> 1))));
            const uint32_t h1 = __half_as_ushort(__float2half_rn(__ldg(p.tab + (w & mask))));
            tab2[w] = h0 | (h1 << 16);
        }
    }
    __syncthreads();
    // the CTA walks tiles blockIdx.x, + gridDim.x, ... (with one CTA per tile: exactly one)
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
        const int c = p.tile_cell[tile];
        const int qn = p.ccnt[c];
        if (qn == 0) continue;  // uniform over the CTA
        const int64_t cs = p.off[c], ce = p.off[c + 1];
        const int64_t row0 = p.tile_row0[tile];
        const int qoff = p.coff[c];
        // ---- decode: thread pair (2r, 2r+1) decodes row r, halves [0, R/2) and [R/2, R) (rows outside the cell: 0)
        {
            const int r = tid >> 1, hf = tid & 1;
            const int64_t n = row0 + r;
            uint32_t* dst = reinterpret_cast<uint32_t*>(vt + r * RS) + hf * (R / 4);
            if (n >= cs && n < ce) {
                uint32_t w[R / 64 + 1];
#pragma unroll
                for (int i = 0; i <= R / 64; i++) {
                    const int wi = hf * (R / 64) + i;
                    w[i] = (wi < W) ? p.words[n * W + wi] : 0u;
                }
                const uint32_t mask2 = (2u << L) - 1u;
#pragma unroll
                for (int wi = 0; wi < R / 64; wi++) {
                    const unsigned long long comb = ((unsigned long long)w[wi] << 32) | w[wi + 1];
#pragma unroll
                    for (int o = 0; o < 32; o += 2)  // states o and o+1 = the L+1 bits starting at bit o
                        dst[(wi * 32 + o) >> 1] = tab2[(uint32_t)(comb >> (64 - L - 1 - o)) & mask2];
                }
                if (hf == 0) ssc[r] = __half2float(p.scale1[n]);
            } else {
                for (int j = 0; j < R / 4; j++) dst[j] = 0u;
                if (hf == 0) ssc[r] = 0.f;
            }
        }
        const int rw = warp & 3, qh = warp >> 2;
        const int64_t wrow0 = row0 + 32 * rw;
        const bool warp_active = wrow0 < ce;
        const int blk_rel = (int)(wrow0 / 32 - cs / 32);
        const int g = lane >> 2, t4 = lane & 3;

        for (int qb = 0; qb < qn; qb += QT) {
            const int nq = min(QT, qn - qb);
            __syncthreads();
            if (tid < QT) {
                if (tid < nq) {
                    const int pi = qoff + qb + tid;
                    const int q = p.qid[pi];
                    qids[tid] = q;
                    qcs[tid] = p.qcp[pi];
                    thr[tid] = MODE == 1 ? p.t0[q] : 0.f;
                } else {
                    qids[tid] = -1;
                }
            }
            __syncthreads();
            const int mt = (nq + 15) >> 4;
            for (int i = tid; i < mt * 16 * (R * 2 / 16); i += NTHREADS) {
                const int r = i >> 5, ch = i & 31;
                const int q = qids[r];
                uint4 v = make_uint4(0, 0, 0, 0);
                if (q >= 0) v = reinterpret_cast<const uint4*>(p.Qh + (int64_t)q * R)[ch];
                *reinterpret_cast<uint4*>(qt + r * RS + ch * 16) = v;
            }
            __syncthreads();
            const int m0 = 2 * qh;  // this warp's two 16-query m-tiles
            if (!warp_active || m0 >= mt) continue;

            float acc[2][4][4];
#pragma unroll
            for (int m = 0; m < 2; m++)
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int e = 0; e < 4; e++) acc[m][j][e] = 0.f;
#pragma unroll 4
            for (int kb = 0; kb < R * 2; kb += 32) {  // 16 fp16 = 32 bytes per k-step
                uint32_t b[4][2];
#pragma unroll
                for (int jp = 0; jp < 2; jp++) {
                    const int nrow = 32 * rw + 16 * jp + (lane & 7) + ((lane >> 4) << 3);
                    ldsm_x4(b[2 * jp][0], b[2 * jp][1], b[2 * jp + 1][0], b[2 * jp + 1][1],
                            vt + nrow * RS + kb + ((lane >> 3) & 1) * 16);
                }
#pragma unroll
                for (int mm = 0; mm < 2; mm++) {
                    const int m = m0 + mm;
                    if (m < mt) {
                        uint32_t a[4];
                        ldsm_x4(a[0], a[1], a[2], a[3], qt + (16 * m + (lane & 15)) * RS + kb + (lane >> 4) * 16);
#pragma unroll
                        for (int j = 0; j < 4; j++) mma_f16(acc[mm][j], a, b[j][0], b[j][1]);
                    }
                }
            }
            float sr[4][2];
            bool rv[4][2];
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int r = 32 * rw + 8 * j + 2 * t4 + e;
                    const int64_t n = row0 + r;
                    rv[j][e] = n >= cs && n < ce;
                    sr[j][e] = ssc[r];
                }
#pragma unroll
            for (int mm = 0; mm < 2; mm++) {
                const int m = m0 + mm;
                if (m >= mt) break;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int ql = 16 * m + g + 8 * h;
                    const bool qv = ql < nq;
                    const float qcv = qv ? qcs[ql] : 0.f;
                    float est[4][2];
#pragma unroll
                    for (int j = 0; j < 4; j++)
#pragma unroll
                        for (int e = 0; e < 2; e++) est[j][e] = __fadd_rn(__fmul_rn(sr[j][e], acc[mm][j][2 * h + e]), qcv);
                    if (MODE != 1) {
                        float mx = -INFINITY;
#pragma unroll
                        for (int j = 0; j < 4; j++)
#pragma unroll
                            for (int e = 0; e < 2; e++)
                                if (rv[j][e]) mx = fmaxf(mx, est[j][e]);
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                        if (qv && t4 == 0) {
                            if (MODE == 0)
                                p.bmc[(int64_t)(qoff + qb + ql) * p.MB + blk_rel] = mx;
                            else  // small-batch rule: global block maxima; MB holds the blocks per query row
                                atomic_max_float(p.bmc + (int64_t)qids[ql] * p.MB + wrow0 / 32, mx);
                        }
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
                                            p.bpos[o] = (int32_t)(row0 + 32 * rw + 8 * j + 2 * t4 + e);
                                        }
                                        base++;
                                    }
                        }
                    }
                }
            }
        }
        __syncthreads();  // every warp is done with this tile's shared memory before the next decode
    }
}

constexpr size_t smem_bytes(int L) {
    return (size_t)TILE_ROWS * RS + (size_t)QT * RS + ((size_t)2 << L) * 4 + TILE_ROWS * 4 + QT * 4 * 3;
}

}  // namespace trellis

// ------------------------------------------------------------------------------------------------ small batches
// `_small_scan` (`src/s1small_cell.py:7-28`) for B <= 8: est = (sum_j tab[state_j] * q'[j]) * scale1[n] + qcp with
// fp32 table values and the fp32 query projection q' = Q @ W1 (no fp16 rounding, no tensor core), work taken straight
// from the probe list like fvs_i8_scan_small: one CTA per (query, probe column, 4 blocks), a warp per 32-row block,
// lane = row (its words in registers, the query and the table in shared memory); mode 0 merges the block maximum into
// bm[q * NBg + global block] with an atomic max (as the reference's `tl.atomic_max` into bm [B, NB]: a block shared by
// two adjacent first-pass cells holds one value), mode 1 emits est >= t0[q].
namespace tsmall {
constexpr int WARPS = 4;
constexpr int R = 256;
}

template <int MODE>
__global__ void __launch_bounds__(32 * tsmall::WARPS) trellis_small_kernel(
    const float* __restrict__ Qr, const int64_t* __restrict__ probe, int nprobe, int ncols,
    const __half* __restrict__ QM, int NC, const int64_t* __restrict__ off, const uint32_t* __restrict__ words, int W,
    const float* __restrict__ tab, int L, const __half* __restrict__ scale1, const float* __restrict__ t0,
    int32_t* __restrict__ cnt, float* __restrict__ bval, int32_t* __restrict__ bpos, int M, float* __restrict__ bm,
    int NBg, int groups) {
    using namespace tsmall;
    extern __shared__ __align__(16) uint8_t smem[];
    float* qv = reinterpret_cast<float*>(smem);  // R
    float* tb = qv + R;                           // 2^L
    const int pair = blockIdx.x / groups, grp = blockIdx.x - pair * groups;
    const int q = pair / ncols, j = pair - q * ncols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = (int)probe[(int64_t)q * nprobe + j];
    const int64_t cs = off[c], ce = off[c + 1];
    if (ce <= cs) return;  // uniform over the CTA
    const int64_t b0 = cs / 32, nb = (ce - 1) / 32 - b0 + 1;
    if ((int64_t)grp * WARPS >= nb) return;  // uniform over the CTA
    for (int i = threadIdx.x; i < R; i += blockDim.x) qv[i] = Qr[(int64_t)q * R + i];
    for (int i = threadIdx.x; i < (1 << L); i += blockDim.x) tb[i] = tab[i];
    __syncthreads();
    const int64_t blk = b0 + (int64_t)grp * WARPS + warp;
    if (blk - b0 >= nb) return;
    const float qcp = __half2float(QM[(int64_t)q * NC + c]);
    const int64_t n = blk * 32 + lane;
    const bool valid = n >= cs && n < ce;
    float est = -INFINITY;
    if (valid) {
        uint32_t w[R / 32 + 1];
#pragma unroll
        for (int i = 0; i <= R / 32; i++) w[i] = i < W ? words[n * W + i] : 0u;
        const uint32_t mask = (1u << L) - 1u;
        float acc = 0.f;
#pragma unroll
        for (int wi = 0; wi < R / 32; wi++) {
            const unsigned long long comb = ((unsigned long long)w[wi] << 32) | w[wi + 1];
#pragma unroll
            for (int o = 0; o < 32; o++)
                acc = __fmaf_rn(tb[(uint32_t)(comb >> (64 - L - o)) & mask], qv[wi * 32 + o], acc);
        }
        est = __fadd_rn(__fmul_rn(acc, __half2float(scale1[n])), qcp);
    }
    if (MODE == 0) {
        float mx = est;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) atomic_max_float(bm + (int64_t)q * NBg + blk, mx);
    } else {
        const bool keep = valid && est >= t0[q];
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        if (m) {
            int base = 0;
            if (lane == 0) base = atomicAdd(cnt + q, __popc(m));
            base = __shfl_sync(0xffffffffu, base, 0) + __popc(m & ((1u << lane) - 1u));
            if (keep && base < M) {
                bval[(int64_t)q * M + base] = est;
                bpos[(int64_t)q * M + base] = (int32_t)n;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ tiered gather
// est = qc + sum_t scale_t <q_t, cb_t[code]>, var = sum_t ||q_t||^2 sig_t^2 (`src/tiered_fused.py:8-41`); code of
// coordinate 8j+k of tier t = sum_p bit(7-k) of byte j of plane p << (b-1-p).  One CTA per query holds the rotated
// query and every tier's codebook in shared memory; the query is stored interleaved by coordinate-within-byte
// (zqk[s_t + k*kb_t + j] = Zq[s_t + 8j + k], the reference's qk[8, B, KB] layout) so that lanes over consecutive byte
// positions j read consecutive words.  Each warp scores one candidate at a time, lane l owning byte positions l,
// l+32, ... of the candidate over all tiers; the bytes of all b planes of a position are loaded together, then decoded;
// scale_t is folded into the partial sums so that a candidate needs one reduction for the estimate and one for the
// variance.
constexpr int TG_MAXT = 8;
struct TieredSet {
    int T, nbytes;  // nbytes: byte positions per candidate over all tiers = D / 8
    int s[TG_MAXT], kb[TG_MAXT], bits[TG_MAXT], cboff[TG_MAXT], pbase[TG_MAXT + 1];
    int toff[TG_MAXT];  // byte offset of the tier in a packed record (sum of the earlier tiers' b * KB)
    const uint8_t* planes[TG_MAXT];
    const float* cb[TG_MAXT];
    const uint8_t* rec;  // packed records [N, RB] (`src/tiered_fused.py:112-125`), or null: separate planes
    int RB, soff;
};

// codes of the 8 coordinates of one byte position from NB bit planes, as 8 bytes (lo: coordinates 0-3, hi: 4-7):
// a nibble's 4 bits are spread into 4 bytes by one multiply (n * 0x00204081 places bit i at bit 8i, the partial
// products do not overlap) and put in coordinate order by a byte permute; planes are combined MSB-first by
// shift-or (codes < 2^NB <= 256 never carry into the next byte)
template <int NB>
__device__ __forceinline__ float tier_pos_dot(const uint8_t* __restrict__ pb, int64_t pstride,
                                              const float* __restrict__ cbt, const float* __restrict__ z, int kb) {
    uint32_t by[NB];
#pragma unroll
    for (int pl = 0; pl < NB; pl++) by[pl] = pb[pl * pstride];  // global planes or the warp's staged record
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int pl = 0; pl < NB; pl++) {
        lo = (lo << 1) | __byte_perm(((by[pl] >> 4) * 0x00204081u) & 0x01010101u, 0, 0x0123);
        hi = (hi << 1) | __byte_perm(((by[pl] & 15u) * 0x00204081u) & 0x01010101u, 0, 0x0123);
    }
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < 4; k++) a += cbt[(lo >> (8 * k)) & 255u] * z[k * kb];
#pragma unroll
    for (int k = 0; k < 4; k++) a += cbt[(hi >> (8 * k)) & 255u] * z[(k + 4) * kb];
    return a;
}

__global__ void __launch_bounds__(256) tiered_score_kernel(const int64_t* __restrict__ pos, int B, int K,
                                                          const float* __restrict__ qc, const float* __restrict__ Zq,
                                                          int ldz, int D, TieredSet ts, const __half* __restrict__ scale,
                                                          const __half* __restrict__ sig, int64_t N,
                                                          float* __restrict__ est, float* __restrict__ sd) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_qn2[TG_MAXT];
    __shared__ float s_scl[8][TG_MAXT];  // per warp: this candidate's scale of every tier
    __shared__ const uint8_t* s_planes[TG_MAXT];
    __shared__ int s_s[TG_MAXT], s_kb[TG_MAXT], s_bits[TG_MAXT], s_cbo[TG_MAXT], s_pbase[TG_MAXT], s_toff[TG_MAXT];
    float* zqk = reinterpret_cast<float*>(smem);  // D, interleaved per tier
    float* cbs = zqk + D;                         // sum_t 2^b_t
    const int q = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    if (tid < ts.T) {
        s_planes[tid] = ts.planes[tid];
        s_s[tid] = ts.s[tid];
        s_kb[tid] = ts.kb[tid];
        s_bits[tid] = ts.bits[tid];
        s_cbo[tid] = ts.cboff[tid];
        s_pbase[tid] = ts.pbase[tid];
        s_toff[tid] = ts.toff[tid];
    }
    __syncthreads();
    uint8_t* ptier = reinterpret_cast<uint8_t*>(cbs + ts.cboff[ts.T - 1] + (1 << ts.bits[ts.T - 1]));  // nbytes
    for (int i = tid; i < D; i += blockDim.x) {
        int t = 0;
        while (t + 1 < ts.T && i >= s_s[t + 1]) t++;
        const int loc = i - s_s[t];
        if (loc < 8 * s_kb[t]) zqk[s_s[t] + (loc & 7) * s_kb[t] + (loc >> 3)] = Zq[(int64_t)q * ldz + i];
    }
    for (int t = 0; t < ts.T; t++)
        for (int i = tid; i < (1 << s_bits[t]); i += blockDim.x) cbs[s_cbo[t] + i] = ts.cb[t][i];
    for (int gp = tid; gp < ts.nbytes; gp += blockDim.x) {
        int t = 0;
        while (t + 1 < ts.T && gp >= s_pbase[t + 1]) t++;
        ptier[gp] = (uint8_t)t;
    }
    __syncthreads();
    if (warp < ts.T) {
        float a = 0.f;
        for (int i = s_s[warp] + lane; i < s_s[warp] + 8 * s_kb[warp]; i += 32) a += zqk[i] * zqk[i];
        a = warp_sum(a);
        if (lane == 0) s_qn2[warp] = a;
    }
    __syncthreads();
    const float qcv = qc[q];
    const int tl = lane < ts.T ? lane : 0;
    const float qn2l = s_qn2[tl];
    // packed records of at most 512 bytes are staged per warp in shared memory: the next candidate's record (one
    // coalesced 16-byte load per lane, held in registers) is in flight while the current one is scored
    const bool staged = ts.rec && ts.RB <= 512;
    uint8_t* wrec = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ptier + ts.nbytes) + 15) & ~uintptr_t(15)) +
                    warp * 512;
    uint4 nxt = make_uint4(0, 0, 0, 0);
    if (staged && warp < K) {
        const int64_t n0 = pos[(int64_t)q * K + warp];
        if (lane * 16 < ts.RB) nxt = __ldg(reinterpret_cast<const uint4*>(ts.rec + n0 * ts.RB) + lane);
        if (lane * 16 < ts.RB) *reinterpret_cast<uint4*>(wrec + lane * 16) = nxt;
        __syncwarp();
    }
    for (int i = warp; i < K; i += nw) {
        const int64_t n = pos[(int64_t)q * K + i];
        const uint8_t* rb = wrec;
        if (staged && i + nw < K && lane * 16 < ts.RB)
            nxt = __ldg(reinterpret_cast<const uint4*>(ts.rec + pos[(int64_t)q * K + i + nw] * ts.RB) + lane);
        float scl = 0.f, sgl = 0.f;
        if (lane < ts.T) {
            if (ts.rec) {
                const uint32_t sp = staged ? reinterpret_cast<const uint32_t*>(rb + ts.soff)[lane]
                                           : __ldg(reinterpret_cast<const uint32_t*>(ts.rec + n * ts.RB + ts.soff) + lane);
                scl = __half2float(__ushort_as_half((unsigned short)(sp & 0xffffu)));
                sgl = __half2float(__ushort_as_half((unsigned short)(sp >> 16)));
            } else {
                scl = __half2float(scale[(int64_t)lane * N + n]);
                sgl = __half2float(sig[(int64_t)lane * N + n]);
            }
        }
        if (lane < ts.T) s_scl[warp][lane] = scl;
        __syncwarp();
        float part = 0.f;
        for (int gp = lane; gp < ts.nbytes; gp += 32) {
            const int t = ptier[gp];
            const int j = gp - s_pbase[t], b = s_bits[t], kb = s_kb[t];
            const uint8_t* pb = staged ? rb + s_toff[t] + j
                                       : ts.rec ? ts.rec + n * ts.RB + s_toff[t] + j : s_planes[t] + n * kb + j;
            const int64_t pstride = ts.rec ? (int64_t)kb : N * kb;
            const float* cbt = cbs + s_cbo[t];
            const float* z = zqk + s_s[t] + j;
            float a;
            switch (b) {
                case 1: a = tier_pos_dot<1>(pb, pstride, cbt, z, kb); break;
                case 2: a = tier_pos_dot<2>(pb, pstride, cbt, z, kb); break;
                case 3: a = tier_pos_dot<3>(pb, pstride, cbt, z, kb); break;
                case 4: a = tier_pos_dot<4>(pb, pstride, cbt, z, kb); break;
                case 5: a = tier_pos_dot<5>(pb, pstride, cbt, z, kb); break;
                case 6: a = tier_pos_dot<6>(pb, pstride, cbt, z, kb); break;
                case 7: a = tier_pos_dot<7>(pb, pstride, cbt, z, kb); break;
                default: a = tier_pos_dot<8>(pb, pstride, cbt, z, kb); break;
            }
            part += a * s_scl[warp][t];
        }
        __syncwarp();  // every lane is done with the staged record
        if (staged && i + nw < K) {
            if (lane * 16 < ts.RB) *reinterpret_cast<uint4*>(wrec + lane * 16) = nxt;
            __syncwarp();
        }
        part = warp_sum(part);
        const float var = warp_sum(lane < ts.T ? qn2l * sgl * sgl : 0.f);
        if (lane == 0) {
            est[(int64_t)q * K + i] = qcv + part;
            sd[(int64_t)q * K + i] = sqrtf(var);
        }
    }
}

// Tiered gather on packed records with one candidate per thread: the same estimate as tiered_score_kernel, organised
// so that every lane of a warp runs the same tier, position and plane at each step (no divergence, no warp
// reductions).  A CTA of TC_THREADS scores TC_THREADS candidates of one query; each warp stages its 32 records in
// shared memory with coalesced 16-byte loads, at a word stride SW = RB/4 rounded up to odd, so that the 32 lanes
// reading the same byte offset of their own records hit 32 different banks.  The rotated query sits in natural order
// (the four coordinates a byte half covers are one 16-byte broadcast read) and the tiers' codebooks after it (a code
// of b <= 5 bits indexes at most 32 words: conflict-free).  Per candidate the work is about 6 instructions per
// coordinate, against ~25 per coordinate in the warp-per-candidate kernel.
constexpr int TC_THREADS = 128;

template <int NB>
__device__ __forceinline__ float tier_cand_dot(const uint8_t* __restrict__ pt, int kb, const float* __restrict__ cbt,
                                               const float* __restrict__ zt) {
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 2
    for (int j = 0; j < kb; j++) {
        uint32_t by[NB];
#pragma unroll
        for (int pl = 0; pl < NB; pl++) by[pl] = pt[pl * kb + j];
        // codes of coordinates 8j .. 8j+7, one per byte of lo (0-3) and hi (4-7): bit 7-k of every plane's byte, planes
        // combined MSB-first (as tier_pos_dot)
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int pl = 0; pl < NB; pl++) {
            lo = (lo << 1) | __byte_perm(((by[pl] >> 4) * 0x00204081u) & 0x01010101u, 0, 0x0123);
            hi = (hi << 1) | __byte_perm(((by[pl] & 15u) * 0x00204081u) & 0x01010101u, 0, 0x0123);
        }
        const float4 za = *reinterpret_cast<const float4*>(zt + 8 * j);
        const float4 zb = *reinterpret_cast<const float4*>(zt + 8 * j + 4);
        a0 += cbt[lo & 255u] * za.x;
        a1 += cbt[(lo >> 8) & 255u] * za.y;
        a0 += cbt[(lo >> 16) & 255u] * za.z;
        a1 += cbt[lo >> 24] * za.w;
        a0 += cbt[hi & 255u] * zb.x;
        a1 += cbt[(hi >> 8) & 255u] * zb.y;
        a0 += cbt[(hi >> 16) & 255u] * zb.z;
        a1 += cbt[hi >> 24] * zb.w;
    }
    return a0 + a1;
}

__global__ void __launch_bounds__(TC_THREADS) tiered_cand_kernel(const int64_t* __restrict__ pos, int K,
                                                                 const float* __restrict__ qc,
                                                                 const float* __restrict__ Zq, int ldz, int D,
                                                                 TieredSet ts, float* __restrict__ est,
                                                                 float* __restrict__ sd) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_qn2[TG_MAXT];
    const int T = ts.T;
    const int cbn = ts.cboff[T - 1] + (1 << ts.bits[T - 1]);
    float* z = reinterpret_cast<float*>(smem);             // D (rounded up to 4)
    float* cbs = z + ((D + 3) & ~3);                       // the tiers' codebooks
    uint32_t* recs = reinterpret_cast<uint32_t*>(cbs + ((cbn + 3) & ~3));  // TC_THREADS records at word stride SW
    const int SW = (ts.RB / 4) | 1;
    const int q = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t qK = (int64_t)q * K;
    for (int k = tid; k < D; k += TC_THREADS) z[k] = Zq[(int64_t)q * ldz + k];
    for (int t = 0; t < T; t++)
        for (int v = tid; v < (1 << ts.bits[t]); v += TC_THREADS) cbs[ts.cboff[t] + v] = ts.cb[t][v];
    // the warp's 32 records, chunk c of record r by lane (32 r + c) mod 32 of step (32 r + c) / 32
    const int RC = ts.RB / 16;
    const int base = blockIdx.y * TC_THREADS + warp * 32;
    for (int e = lane; e < 32 * RC; e += 32) {
        const int r = e / RC, c = e - r * RC;
        if (base + r < K) {
            const int64_t n = pos[qK + base + r];
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(ts.rec + n * ts.RB) + c);
            uint32_t* d = recs + (warp * 32 + r) * SW + 4 * c;
            d[0] = v.x;
            d[1] = v.y;
            d[2] = v.z;
            d[3] = v.w;
        }
    }
    __syncthreads();
    for (int t = warp; t < T; t += TC_THREADS / 32) {  // ||q_t||^2 per tier
        float a = 0.f;
        for (int k = ts.s[t] + lane; k < ts.s[t] + 8 * ts.kb[t]; k += 32) a += z[k] * z[k];
        a = warp_sum(a);
        if (lane == 0) s_qn2[t] = a;
    }
    __syncthreads();
    const int i = blockIdx.y * TC_THREADS + tid;
    if (i >= K) return;
    const uint8_t* rb = reinterpret_cast<const uint8_t*>(recs + tid * SW);
    float acc = qc[q], var = 0.f;
    for (int t = 0; t < T; t++) {
        const int kb = ts.kb[t];
        const uint8_t* pt = rb + ts.toff[t];
        const float* cbt = cbs + ts.cboff[t];
        const float* zt = z + ts.s[t];
        float a;
        switch (ts.bits[t]) {  // uniform over the CTA
            case 1: a = tier_cand_dot<1>(pt, kb, cbt, zt); break;
            case 2: a = tier_cand_dot<2>(pt, kb, cbt, zt); break;
            case 3: a = tier_cand_dot<3>(pt, kb, cbt, zt); break;
            case 4: a = tier_cand_dot<4>(pt, kb, cbt, zt); break;
            case 5: a = tier_cand_dot<5>(pt, kb, cbt, zt); break;
            case 6: a = tier_cand_dot<6>(pt, kb, cbt, zt); break;
            case 7: a = tier_cand_dot<7>(pt, kb, cbt, zt); break;
            default: a = tier_cand_dot<8>(pt, kb, cbt, zt); break;
        }
        // the tier's fp16 (scale, sigma) pair at soff + 4t, read bytewise (soff need not be 4-aligned)
        const uint8_t* sp = rb + ts.soff + 4 * t;
        const float scl = __half2float(__ushort_as_half((unsigned short)(sp[0] | (sp[1] << 8))));
        const float sgl = __half2float(__ushort_as_half((unsigned short)(sp[2] | (sp[3] << 8))));
        acc += a * scl;
        var += s_qn2[t] * sgl * sgl;
    }
    est[qK + i] = acc;
    sd[qK + i] = sqrtf(var);
}

// ------------------------------------------------------------------------------------------------ routing (fp32)
// probe = the nprobe largest float(QM[q, c]) * scale[c] (`src/engine_cell.py:40-42`), ordered (score desc, cell asc).
__global__ void __launch_bounds__(512) route_topk_scaled_kernel(const __half* __restrict__ QM, const float* __restrict__ sc,
                                                               int NC, int nprobe, int kp, int64_t* __restrict__ probe) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectScratch ss;
    __shared__ int s_fill;
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem);  // NC
    unsigned long long* sb = keys + NC;                                      // kp
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    for (int c = tid; c < NC; c += nt) {
        const float v = __fmul_rn(__half2float(QM[(int64_t)q * NC + c]), sc[c]);
        keys[c] = ((unsigned long long)f2o(v) << 32) | (0xffffffffu - (uint32_t)c);
    }
    if (tid == 0) s_fill = 0;
    __syncthreads();
    const uint32_t Th = block_select_rth_largest<32, uint32_t>([&](int i) { return (uint32_t)(keys[i] >> 32); }, NC,
                                                               nprobe, ss);
    // ties at the boundary score: by cell index (keys are unique)
    int gt = 0;
    for (int c = tid; c < NC; c += nt) gt += (uint32_t)(keys[c] >> 32) > Th;
    __shared__ int s_red[32];
    gt = block_sum_int(gt, s_red);
    const uint32_t Tl = block_select_rth_largest<32, uint32_t>(
        [&](int i) { return (uint32_t)(keys[i] >> 32) == Th ? (uint32_t)keys[i] : 0u; }, NC, nprobe - gt, ss);
    const unsigned long long T = ((unsigned long long)Th << 32) | Tl;
    for (int c = tid; c < NC; c += nt)
        if (keys[c] >= T) {
            const int slot = atomicAdd(&s_fill, 1);
            if (slot < nprobe) sb[slot] = keys[c];
        }
    __syncthreads();
    if (nprobe <= 1024) {  // unique keys: place each by its rank, no sorting network
        for (int i = tid; i < nprobe; i += nt) {
            const unsigned long long ki = sb[i];
            int rank = 0;
            for (int j = 0; j < nprobe; j++) rank += sb[j] > ki;
            probe[(int64_t)q * nprobe + rank] = (int64_t)(0xffffffffu - (uint32_t)ki);
        }
        return;
    }
    for (int i = nprobe + tid; i < kp; i += nt) sb[i] = 0ull;
    __syncthreads();
    block_bitonic_desc(sb, kp);
    for (int i = tid; i < nprobe; i += nt) probe[(int64_t)q * nprobe + i] = (int64_t)(0xffffffffu - (uint32_t)sb[i]);
}

// Register-resident variant for NC <= 2048 * V (NC a multiple of 8, 16-byte aligned QM rows and scales) and
// nprobe <= 512: each of 256 threads holds the order keys of 8 * V scaled scores, the nprobe-th largest score key is
// found by histogram passes below the keys' common prefix (block_rth_largest_reg), the cell half of the cut only
// where scores tied with it straddle it.  Same keys, same result as route_topk_scaled_kernel.
constexpr int RSR_THREADS = 256;
constexpr int RSR_MAXP = 512;
template <int V>
__global__ void __launch_bounds__(RSR_THREADS) route_topk_scaled_reg_kernel(const __half* __restrict__ QM,
                                                                            const float* __restrict__ sc, int NC,
                                                                            int nprobe, int64_t* __restrict__ probe) {
    __shared__ RegSelectScratch rs;
    __shared__ SelectScratch ss;
    __shared__ int s_fill;
    __shared__ unsigned long long s_sel[RSR_MAXP];
    const int q = blockIdx.x, tid = threadIdx.x;
    const __half* qrow = QM + (int64_t)q * NC;
    uint32_t hk[8 * V];  // 0 = no cell (a finite score's key is never 0)
#pragma unroll
    for (int v = 0; v < V; v++) {
        const int u = tid + v * RSR_THREADS;
        const bool in = u * 8 < NC;
        const uint4 w = in ? __ldg(reinterpret_cast<const uint4*>(qrow) + u) : make_uint4(0u, 0u, 0u, 0u);
        const float4 s0 = in ? __ldg(reinterpret_cast<const float4*>(sc) + 2 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 s1 = in ? __ldg(reinterpret_cast<const float4*>(sc) + 2 * u + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const float ss8[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const __half h = __ushort_as_half((unsigned short)((ws[e >> 1] >> (16 * (e & 1))) & 0xffffu));
            hk[8 * v + e] = in ? f2o(__fmul_rn(__half2float(h), ss8[e])) : 0u;
        }
    }
    if (tid == 0) s_fill = 0;
    int gt, eq;
    const uint32_t Th = block_rth_largest_reg<8 * V>(hk, nprobe, rs, &gt, &eq);
    uint32_t Tl = 0u;
    if (eq > nprobe - gt)
        Tl = block_select_rth_largest<32, uint32_t>(
            [&](int i) {
                return f2o(__fmul_rn(__half2float(qrow[i]), sc[i])) == Th ? (0xffffffffu - (uint32_t)i) : 0u;
            },
            NC, nprobe - gt, ss);
    const unsigned long long T = ((unsigned long long)Th << 32) | Tl;
#pragma unroll
    for (int v = 0; v < V; v++)
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint32_t h = hk[8 * v + e];
            if (h != 0u && h >= Th) {
                const int c = 8 * (tid + v * RSR_THREADS) + e;
                const unsigned long long k = ((unsigned long long)h << 32) | (0xffffffffu - (uint32_t)c);
                if (k >= T) {  // unique keys: exactly nprobe of them
                    const int slot = atomicAdd(&s_fill, 1);
                    if (slot < nprobe) s_sel[slot] = k;
                }
            }
        }
    __syncthreads();
    if (nprobe > 128 && nprobe <= RSR_THREADS) {
        // order by a bitonic sort, one key per thread (the O(nprobe^2) rank loop costs more at these sizes)
        int kp = 1;
        while (kp < nprobe) kp <<= 1;
        unsigned long long v = tid < nprobe ? s_sel[tid] : 0ull;
        __syncthreads();
        v = block_bitonic_desc_u64(v, kp, s_sel);
        if (tid < nprobe) probe[(int64_t)q * nprobe + tid] = (int64_t)(0xffffffffu - (uint32_t)v);
        return;
    }
    for (int i = tid; i < nprobe; i += RSR_THREADS) {
        const unsigned long long ki = s_sel[i];
        int rank = 0;
        for (int j = 0; j < nprobe; j++) rank += s_sel[j] > ki;
        probe[(int64_t)q * nprobe + rank] = (int64_t)(0xffffffffu - (uint32_t)ki);
    }
}

// ------------------------------------------------------------------------------------------------ Viterbi (build)
// Encoder of the bitshift trellis (k = 1) as `src/trellis_scan.py:21-32`: predecessors of state s are
// (s >> 1) | (u << (L-1)); entering s emits vals[s]; ties keep predecessor u = 0 and the lowest final state.  One CTA
// per vector: path costs in shared memory, backpointers one bit per (step, state).
__global__ void __launch_bounds__(256) viterbi_kernel(const float* __restrict__ Zs, int n, int R,
                                                      const float* __restrict__ vals, int L, int32_t* __restrict__ path) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int S = 1 << L, tid = threadIdx.x;
    float* cost = reinterpret_cast<float*>(smem);          // 2 x S
    float* v = cost + 2 * S;                                // S
    uint32_t* back = reinterpret_cast<uint32_t*>(v + S);   // (R-1) x S/32
    __shared__ float s_best[256];
    __shared__ int s_arg[256];
    const int vec = blockIdx.x;
    const float* x = Zs + (int64_t)vec * R;
    for (int s = tid; s < S; s += blockDim.x) {
        v[s] = vals[s];
        const float d = __fsub_rn(x[0], vals[s]);
        cost[s] = __fmul_rn(d, d);
    }
    __syncthreads();
    for (int j = 1; j < R; j++) {
        const float* src = cost + ((j - 1) & 1) * S;
        float* dst = cost + (j & 1) * S;
        const float xj = x[j];
        for (int s = tid; s < S; s += blockDim.x) {  // S is a multiple of 32: whole warps per iteration
            const int p0 = s >> 1, p1 = p0 | (1 << (L - 1));
            const float c0 = src[p0], c1 = src[p1];
            const bool take1 = c1 < c0;
            const float d = __fsub_rn(xj, v[s]);
            dst[s] = __fadd_rn(take1 ? c1 : c0, __fmul_rn(d, d));  // no contraction: same rounding as separate ops
            const uint32_t bits = __ballot_sync(0xffffffffu, take1);
            if ((tid & 31) == 0) back[(j - 1) * (S / 32) + (s >> 5)] = bits;
        }
        __syncthreads();
    }
    // argmin of the final costs (lowest state on ties)
    const float* fin = cost + ((R - 1) & 1) * S;
    float best = INFINITY;
    int arg = 0;
    for (int s = tid; s < S; s += blockDim.x)
        if (fin[s] < best) {
            best = fin[s];
            arg = s;
        }
    s_best[tid] = best;
    s_arg[tid] = arg;
    __syncthreads();
    if (tid == 0) {
        for (int i = 1; i < (int)blockDim.x; i++)
            if (s_best[i] < best || (s_best[i] == best && s_arg[i] < arg)) {
                best = s_best[i];
                arg = s_arg[i];
            }
        int s = arg;
        int32_t* out = path + (int64_t)vec * R;
        out[R - 1] = s;
        for (int j = R - 1; j >= 1; j--) {
            const uint32_t take1 = (back[(j - 1) * (S / 32) + (s >> 5)] >> (s & 31)) & 1u;
            s = (s >> 1) | ((int)take1 << (L - 1));
            out[j - 1] = s;
        }
    }
}

}  // namespace fvs

extern "C" int fvs_trellis_tile_rows(void) { return fvs::trellis::TILE_ROWS; }

extern "C" int fvs_trellis_scan(fvs_stream_t stream, int mode, const uint16_t* Qh, int B, int R, const int32_t* qid,
                                const int32_t* coff, const int32_t* ccnt, const float* qcp, const int32_t* tile_cell,
                                const int32_t* tile_row0, int ntiles, const int64_t* off, int NC, const int32_t* words,
                                int W, const float* tab, int L, const uint16_t* scale1, const float* t0, int32_t* cnt,
                                float* bval, int32_t* bpos, int M, float* bmc, int MB) {
    using namespace fvs::trellis;
    FVS_CHECK_ARG(mode == 0 || mode == 1 || mode == 2);
    FVS_CHECK_ARG(R == fvs::trellis::R && B >= 0 && ntiles >= 0 && NC > 0 && L >= 2 && L <= 12);
    FVS_CHECK_ARG(W >= (R + L - 1 + 31) / 32 && W <= MAXW);
    FVS_CHECK_ARG(Qh && qid && coff && ccnt && qcp && tile_cell && tile_row0 && off && words && tab && scale1);
    if (mode != 1) FVS_CHECK_ARG(bmc && MB > 0);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (ntiles == 0 || B == 0) return FVS_OK;
    Params p{(const __half*)Qh, qid, coff, ccnt, qcp, tile_cell, tile_row0, off, (const uint32_t*)words, tab,
             (const __half*)scale1, t0, cnt, bval, bpos, bmc, W, L, M, MB, ntiles};
    const size_t sm = smem_bytes(L);
    const void* fn = mode == 0 ? (const void*)trellis_scan_kernel<0>
                               : mode == 1 ? (const void*)trellis_scan_kernel<1> : (const void*)trellis_scan_kernel<2>;
    cudaError_t e = fvs_ensure_smem(fn, sm);
    if (e != cudaSuccess) return (int)e;
    // one CTA per tile (a persistent walk measured slower: the per-tile phases do not overlap within a CTA, so
    // more resident CTAs hide more latency)
    const int grid = ntiles;
    if (mode == 0)
        trellis_scan_kernel<0><<<grid, NTHREADS, sm, stream>>>(p);
    else if (mode == 1)
        trellis_scan_kernel<1><<<grid, NTHREADS, sm, stream>>>(p);
    else
        trellis_scan_kernel<2><<<grid, NTHREADS, sm, stream>>>(p);
    return fvs_launch_status();
}

extern "C" int fvs_trellis_scan_small(fvs_stream_t stream, int mode, const float* Qr, int B, int R,
                                      const int64_t* probe, int nprobe, int ncols, const uint16_t* QM, int NC,
                                      const int64_t* off, const int32_t* words, int W, const float* tab, int L,
                                      const uint16_t* scale1, const float* t0, int32_t* cnt, float* bval,
                                      int32_t* bpos, int M, float* bm, int NBg, int MB) {
    using namespace fvs::tsmall;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(R == fvs::tsmall::R && B >= 0 && nprobe >= 1 && ncols >= 1 && ncols <= nprobe && NC > 0 && MB > 0);
    FVS_CHECK_ARG(L >= 2 && L <= 12 && W >= (R + L - 1 + 31) / 32 && W <= 16);
    FVS_CHECK_ARG(Qr && probe && QM && off && words && tab && scale1);
    if (mode == 0) FVS_CHECK_ARG(bm && NBg > 0);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (B == 0) return FVS_OK;
    const int groups = (MB + WARPS - 1) / WARPS;
    const int64_t grid = (int64_t)B * ncols * groups;
    if (grid > INT32_MAX) return FVS_ERANGE;
    const size_t sm = (size_t)(R + (1 << L)) * 4;
    cudaError_t e = mode ? fvs_ensure_smem((const void*)fvs::trellis_small_kernel<1>, sm)
                         : fvs_ensure_smem((const void*)fvs::trellis_small_kernel<0>, sm);
    if (e != cudaSuccess) return (int)e;
    if (mode == 0)
        fvs::trellis_small_kernel<0><<<(unsigned)grid, 32 * WARPS, sm, stream>>>(
            Qr, probe, nprobe, ncols, (const __half*)QM, NC, off, (const uint32_t*)words, W, tab, L,
            (const __half*)scale1, t0, cnt, bval, bpos, M, bm, NBg, groups);
    else
        fvs::trellis_small_kernel<1><<<(unsigned)grid, 32 * WARPS, sm, stream>>>(
            Qr, probe, nprobe, ncols, (const __half*)QM, NC, off, (const uint32_t*)words, W, tab, L,
            (const __half*)scale1, t0, cnt, bval, bpos, M, bm, NBg, groups);
    return fvs_launch_status();
}

namespace fvs {
static int make_tiered_set(TieredSet& ts, int T, int D, const int32_t* tier_s, const int32_t* tier_e,
                           const int32_t* tier_bits, const float* const* tier_cb, const uint8_t* const* tier_planes,
                           const uint8_t* rec, int RB, int soff) {
    if (T < 1 || T > TG_MAXT) return FVS_ERANGE;
    ts.T = T;
    int pb = 0, cbo = 0, to = 0;
    for (int t = 0; t < T; t++) {
        FVS_CHECK_ARG(tier_e[t] > tier_s[t] && (tier_e[t] - tier_s[t]) % 8 == 0 && tier_e[t] <= D);
        FVS_CHECK_ARG(tier_bits[t] >= 1 && tier_bits[t] <= 8 && tier_cb[t] && (rec || tier_planes[t]));
        ts.s[t] = tier_s[t];
        ts.kb[t] = (tier_e[t] - tier_s[t]) / 8;
        ts.bits[t] = tier_bits[t];
        ts.planes[t] = tier_planes ? tier_planes[t] : nullptr;
        ts.cb[t] = tier_cb[t];
        ts.cboff[t] = cbo;
        cbo += 1 << tier_bits[t];
        ts.pbase[t] = pb;
        pb += ts.kb[t];
        ts.toff[t] = to;
        to += tier_bits[t] * ts.kb[t];
    }
    ts.pbase[T] = pb;
    ts.nbytes = pb;
    ts.rec = rec;
    ts.RB = RB;
    ts.soff = soff;
    if (rec) FVS_CHECK_ARG(soff == to && soff + 4 * T <= RB && RB % 4 == 0 && ((uintptr_t)rec & 3) == 0);
    return FVS_OK;
}
}  // namespace fvs

extern "C" int fvs_tiered_score(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const float* Zq,
                                int ldz, int D, int T, const int32_t* tier_s, const int32_t* tier_e,
                                const int32_t* tier_bits, const float* const* tier_cb,
                                const uint8_t* const* tier_planes, const uint16_t* scale, const uint16_t* sig,
                                int64_t N, float* est, float* sd) {
    FVS_CHECK_ARG(pos && qc && Zq && tier_s && tier_e && tier_bits && tier_cb && tier_planes && scale && sig && est && sd);
    FVS_CHECK_ARG(B >= 0 && K >= 1 && N > 0 && D > 0 && ldz >= D);
    if (T < 1 || T > fvs::TG_MAXT) return FVS_ERANGE;
    fvs::TieredSet ts;
    int rc = fvs::make_tiered_set(ts, T, D, tier_s, tier_e, tier_bits, tier_cb, tier_planes, nullptr, 0, 0);
    if (rc) return rc;
    const int pb = ts.nbytes, cbo = ts.cboff[T - 1] + (1 << ts.bits[T - 1]);
    const size_t sm = (size_t)(D + cbo) * 4 + (size_t)((pb + 15) & ~15);
    if (sm > 200 * 1024) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::tiered_score_kernel, sm);  // 256 threads = 8 warps (s_scl)
    if (e != cudaSuccess) return (int)e;
    fvs::tiered_score_kernel<<<B, 256, sm, stream>>>(pos, B, K, qc, Zq, ldz, D, ts, (const __half*)scale,
                                                     (const __half*)sig, N, est, sd);
    return fvs_launch_status();
}

extern "C" int fvs_route_topk_scaled(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe,
                                     const float* cell_scale, int64_t* probe) {
    FVS_CHECK_ARG(QM && cell_scale && probe && B >= 0 && NC > 0 && nprobe >= 1 && nprobe <= NC);
    if (nprobe > 4096) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    if (NC % 8 == 0 && NC <= 8 * fvs::RSR_THREADS * 4 && nprobe <= fvs::RSR_MAXP &&
        (((uintptr_t)QM | (uintptr_t)cell_scale) & 15) == 0) {
        const int V = (NC + 8 * fvs::RSR_THREADS - 1) / (8 * fvs::RSR_THREADS);
        if (V <= 1)
            fvs::route_topk_scaled_reg_kernel<1>
                <<<B, fvs::RSR_THREADS, 0, stream>>>((const __half*)QM, cell_scale, NC, nprobe, probe);
        else if (V <= 2)
            fvs::route_topk_scaled_reg_kernel<2>
                <<<B, fvs::RSR_THREADS, 0, stream>>>((const __half*)QM, cell_scale, NC, nprobe, probe);
        else
            fvs::route_topk_scaled_reg_kernel<4>
                <<<B, fvs::RSR_THREADS, 0, stream>>>((const __half*)QM, cell_scale, NC, nprobe, probe);
        return fvs_launch_status();
    }
    int kp = 1;
    while (kp < nprobe) kp <<= 1;
    const size_t sm = (size_t)(NC + kp) * 8;
    if (sm > 200 * 1024) return FVS_ERANGE;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::route_topk_scaled_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    fvs::route_topk_scaled_kernel<<<B, 512, sm, stream>>>((const __half*)QM, cell_scale, NC, nprobe, kp, probe);
    return fvs_launch_status();
}

extern "C" int fvs_viterbi_encode(fvs_stream_t stream, const float* Zs, int n, int R, const float* vals, int L,
                                  int32_t* path) {
    FVS_CHECK_ARG(Zs && vals && path && n >= 0 && R >= 2 && L >= 5 && L <= 12);
    if (n == 0) return FVS_OK;
    const int S = 1 << L;
    const size_t sm = (size_t)3 * S * 4 + (size_t)(R - 1) * (S / 32) * 4;
    if (sm > 200 * 1024) return FVS_ERANGE;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::viterbi_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    fvs::viterbi_kernel<<<n, 256, sm, stream>>>(Zs, n, R, vals, L, path);
    return fvs_launch_status();
}

extern "C" int fvs_tiered_score_rec(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc,
                                    const float* Zq, int ldz, int D, int T, const int32_t* tier_s,
                                    const int32_t* tier_e, const int32_t* tier_bits, const float* const* tier_cb,
                                    const uint8_t* rec, int RB, int soff, int64_t N, float* est, float* sd) {
    FVS_CHECK_ARG(pos && qc && Zq && tier_s && tier_e && tier_bits && tier_cb && rec && est && sd);
    FVS_CHECK_ARG(B >= 0 && K >= 1 && N > 0 && D > 0 && ldz >= D);
    fvs::TieredSet ts;
    int rc = fvs::make_tiered_set(ts, T, D, tier_s, tier_e, tier_bits, tier_cb, nullptr, rec, RB, soff);
    if (rc) return rc;
    const int cbo = ts.cboff[T - 1] + (1 << ts.bits[T - 1]);
    if (B == 0) return FVS_OK;
    FVS_CHECK_ARG(RB % 16 == 0 && ((uintptr_t)rec & 15) == 0);   // 16-byte record chunks
    // one candidate per thread (tiered_cand_kernel): the query, the codebooks and TC_THREADS records in shared memory
    const size_t sm = (size_t)(((D + 3) & ~3) + ((cbo + 3) & ~3)) * 4 +
                      (size_t)fvs::TC_THREADS * (size_t)((RB / 4) | 1) * 4;
    if (sm > 200 * 1024) return FVS_ERANGE;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::tiered_cand_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    const dim3 grid(B, (K + fvs::TC_THREADS - 1) / fvs::TC_THREADS);
    fvs::tiered_cand_kernel<<<grid, fvs::TC_THREADS, sm, stream>>>(pos, K, qc, Zq, ldz, D, ts, est, sd);
    return fvs_launch_status();
}
