// Stage 2 of the throughput mode: per-query nibble lookup tables and the LUT-scored tiered refinement.
//
// `fvs_lut_build` replaces `_lut_kernel` + the tier sums of `luts_fused` (`throughput/s2lut.py:108-126`).
// `fvs_lut_score` replaces `_score_lut` / `_tier_lut` (`throughput/s2lut.py:48-106`): one CTA per query holds the
// query's table (D/4 x 16 entries, 12 KB at D = 1536 in fp16) in shared memory; each warp scores one candidate at a
// time, its lanes striding over the tier's (plane, byte) pairs; the per-tier dot products are warp-reduced.
#include <type_traits>

#include "fvs_common.cuh"

namespace fvs {

constexpr int MAX_TIERS = 8;

struct TierSet {
    int T, nwords;  // nwords: 4-byte plane words per candidate over all tiers
    int s[MAX_TIERS], e[MAX_TIERS], bits[MAX_TIERS], kb[MAX_TIERS], loff[MAX_TIERS], wbase[MAX_TIERS + 1];
    float delta[MAX_TIERS], mid[MAX_TIERS], pw[MAX_TIERS][8];
    const uint8_t* planes[MAX_TIERS];
};

// ------------------------------------------------------------------------------------------------ LUT build
template <bool HALF>
__global__ void lut_build_kernel(const float* __restrict__ Zq, int ldz, int D, void* __restrict__ Lout, TierSet ts,
                                 int B, float* __restrict__ qsum, float* __restrict__ qn2) {
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const float* z = Zq + (int64_t)q * ldz;
    const int nent = (D / 4) * 16;
    for (int idx = tid; idx < nent; idx += nt) {
        const int n = idx >> 4, v = idx & 15;
        // sum of the selected coordinates in order i = 0..3 (bits 3..0 of v), as acc += z_i * bit_i
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++)
            if ((v >> (3 - i)) & 1) acc = __fadd_rn(acc, z[4 * n + i]);
        if (HALF)
            reinterpret_cast<__half*>(Lout)[(int64_t)q * nent + idx] = __float2half_rn(acc);
        else
            reinterpret_cast<float*>(Lout)[(int64_t)q * nent + idx] = acc;
    }
    __shared__ float red[2][32];
    const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
    for (int t = 0; t < ts.T; t++) {
        float a = 0.f, b = 0.f;
        for (int i = ts.s[t] + tid; i < ts.e[t]; i += nt) {
            const float x = z[i];
            a += x;
            b += x * x;
        }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
            red[0][warp] = a;
            red[1][warp] = b;
        }
        __syncthreads();
        if (tid == 0) {
            float sa = 0.f, sb = 0.f;
            for (int w = 0; w < nw; w++) {
                sa += red[0][w];
                sb += red[1][w];
            }
            qsum[(int64_t)t * B + q] = sa;
            qn2[(int64_t)t * B + q] = sb;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------ LUT score
template <bool HALF>
__global__ void __launch_bounds__(256) lut_score_kernel(const int64_t* __restrict__ pos, int B, int K,
                                                        const float* __restrict__ qc, const void* __restrict__ L, int LW,
                                                        TierSet ts, const __half* __restrict__ scale,
                                                        const __half* __restrict__ sig, int64_t N,
                                                        const float* __restrict__ qsum, const float* __restrict__ qn2,
                                                        const int32_t* __restrict__ ncnt, float* __restrict__ est,
                                                        float* __restrict__ sd) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int q = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int lim = ncnt ? min(max(ncnt[q], 0), K) : K;
    // dead candidates first (no table needed)
    for (int i = lim + tid; i < K; i += blockDim.x) {
        est[(int64_t)q * K + i] = kNeg;
        sd[(int64_t)q * K + i] = 0.f;
    }
    if (lim == 0) return;
    // stage the query's table
    using E = typename std::conditional<HALF, __half, float>::type;
    E* lut = reinterpret_cast<E*>(smem);
    {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(L) + (int64_t)q * LW);
        uint4* dst = reinterpret_cast<uint4*>(lut);
        const int nv = LW * (int)sizeof(E) / 16;
        for (int i = tid; i < nv; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    const float qcv = qc[q];
    float qs_t[MAX_TIERS], qn_t[MAX_TIERS];
#pragma unroll
    for (int t = 0; t < MAX_TIERS; t++) {
        qs_t[t] = t < ts.T ? qsum[(int64_t)t * B + q] : 0.f;
        qn_t[t] = t < ts.T ? qn2[(int64_t)t * B + q] : 0.f;
    }
    for (int i = warp; i < lim; i += nw) {
        const int64_t n = pos[(int64_t)q * K + i];
        float acc = qcv, var = 0.f;
#pragma unroll 1
        for (int t = 0; t < ts.T; t++) {
            const int kb = ts.kb[t], nbytes = ts.bits[t] * kb;
            const uint8_t* pl = ts.planes[t];
            const E* lt = lut + ts.loff[t];
            float a = 0.f;
            for (int idx = lane; idx < nbytes; idx += 32) {
                const int p = idx / kb, j = idx - p * kb;
                const uint32_t byt = __ldg(pl + ((int64_t)p * N + n) * kb + j);
                const float h = (float)lt[(2 * j) * 16 + (byt >> 4)];
                const float l = (float)lt[(2 * j + 1) * 16 + (byt & 15u)];
                a += (h + l) * ts.pw[t][p];
            }
            a = warp_sum(a);
            const float at = ts.delta[t] * (a - ts.mid[t] * qs_t[t]);
            const float s = __half2float(scale[(int64_t)t * N + n]);
            const float g = __half2float(sig[(int64_t)t * N + n]);
            acc = acc + at * s;
            var = var + qn_t[t] * g * g;
        }
        if (lane == 0) {
            est[(int64_t)q * K + i] = acc;
            sd[(int64_t)q * K + i] = sqrtf(var);
        }
    }
}


// ------------------------------------------------------------------------------------------------ fused LUT score
// One CTA per query: the query's table and tier sums are built in shared memory from Zq, then each warp scores
// candidates.  A candidate's plane bytes are read as 4-byte words (every plane segment is a multiple of 4 bytes): lane
// l owns words l, l+32, ... of the candidate's word list (tier-major, then plane, then position), issues all its loads
// before any lookup, and folds delta_t * 2^(b-1-p) * scale_t into its partial sum, so a candidate needs one warp
// reduction for the estimate and one for the variance.  Two candidates are in flight per warp.
// Table layout: a plane word covers one block of 32 coordinates, ga = coordinate / 32 (tiers are contiguous 32-wide
// groups from coordinate 0), and its byte c4 / nibble h select LUT group c = 2*c4 + h (4 coordinates).  Entry
// (c, v, ga) sits at (c*16 + v)*GA + ga with GA a multiple of 32, so the 32 lanes of a warp, which hold consecutive
// words, read 32 different banks.  Entries are fp32 slots holding the fp16-rounded value when HALF (the reference's
// `LUTH` table), otherwise the fp32 value.
// REC: the candidate's plane words and (scale, sigma) pairs come from its packed record (`src/tiered_fused.py:112-125`:
// tier t plane p at byte toff[t] + p*KB_t = 4 * word index, then fp16 (scale, sigma) per tier at soff + 4t), one
// contiguous RB-byte row per vector, instead of b_t separate plane rows and two [T, N] arrays
struct RecSet {
    const uint8_t* rec;
    int RB, soff;
};

// GAC: the table stride GA as a compile-time constant (32 or 64), so that a lookup's address is a shift and a mask of
// the plane word plus an immediate; 0 = GA from the argument.
// WCOL: one table column per plane word instead of one per 32-coordinate block.  Column w (stride GA = 32 * WPL)
// holds the 8 x 16 entries of the block that word w covers, so a block coded with b planes appears in b columns.  In
// the per-block layout the lanes holding different planes of one block read the same bank at different entries
// (up to b-way conflicts per lookup); with a column per word, lane l's word lane + 32u sits in bank l and every
// lookup instruction is conflict-free.  The entries are the same numbers, so the estimates are unchanged.
// the 4-bit field of w at bits p..p+3, moved to bits 9..12 (p a compile-time constant after unrolling)
__device__ __forceinline__ uint32_t nibble_at9(uint32_t w, int p) {
    return (p >= 9 ? (w >> (p - 9)) : (w << (9 - p))) & (15u << 9);
}

template <bool HALF, int WPL, bool REC, int GAC, bool WCOL = false>
__global__ void __launch_bounds__(256, 3) lut_score_zq_kernel(const int64_t* __restrict__ pos, int B, int K,
                                                           const float* __restrict__ qc, const void* __restrict__ Zq,
                                                           int ldz, int zh, int D, int GA_, TierSet ts,
                                                           const __half* __restrict__ scale,
                                                           const __half* __restrict__ sig, int64_t N,
                                                           const int32_t* __restrict__ ncnt, float* __restrict__ est,
                                                           float* __restrict__ sd, RecSet rs) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_qsum[MAX_TIERS], s_qn2[MAX_TIERS];
    static_assert(!WCOL || WPL == 4, "the column-per-word table is laid out for 4 words per lane (stride 2^9 B)");
    const int GA = WCOL ? 32 * WPL : (GAC ? GAC : GA_);
    float* lut = reinterpret_cast<float*>(smem);
    int32_t* s_pos = reinterpret_cast<int32_t*>(lut + 128 * GA);  // the query's candidate positions (K)
    const int q = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int lim = ncnt ? min(max(ncnt[q], 0), K) : K;
    if (blockIdx.y == 0)
        for (int i = lim + tid; i < K; i += blockDim.x) {
            est[(int64_t)q * K + i] = kNeg;
            sd[(int64_t)q * K + i] = 0.f;
        }
    if (lim == 0) return;
    // the rotated query row: fp32, or the fp16 product itself (converted here, the same values as its .float())
    const float* z = zh ? nullptr : reinterpret_cast<const float*>(Zq) + (int64_t)q * ldz;
    const __half* zhr = zh ? reinterpret_cast<const __half*>(Zq) + (int64_t)q * ldz : nullptr;
    auto zat = [&](int i) { return zhr ? __half2float(zhr[i]) : z[i]; };
    const int nblk = D / 32;
    // positions staged once (coalesced), so that each candidate round trip is the plane words alone
    for (int i = tid; i < lim; i += blockDim.x) s_pos[i] = (int32_t)pos[(int64_t)q * K + i];
    // entry v of a 4-coordinate group sums the selected coordinates left to right in fp32, as acc += z_i * bit_i does
    auto entries = [&](int ga, int cgrp, float (&e16)[16]) {
        float z0 = 0.f, z1 = 0.f, z2 = 0.f, z3 = 0.f;
        if (ga < nblk) {
            if (zhr) {
                const uint2 u = *reinterpret_cast<const uint2*>(zhr + 32 * ga + 4 * cgrp);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                z0 = a.x;
                z1 = a.y;
                z2 = b.x;
                z3 = b.y;
            } else {
                const float4 zz = *reinterpret_cast<const float4*>(z + 32 * ga + 4 * cgrp);
                z0 = zz.x;
                z1 = zz.y;
                z2 = zz.z;
                z3 = zz.w;
            }
        }
#pragma unroll
        for (int v = 0; v < 16; v++) {
            float acc = 0.f;
            if (v & 8) acc = __fadd_rn(acc, z0);
            if (v & 4) acc = __fadd_rn(acc, z1);
            if (v & 2) acc = __fadd_rn(acc, z2);
            if (v & 1) acc = __fadd_rn(acc, z3);
            e16[v] = HALF ? __half2float(__float2half_rn(acc)) : acc;
        }
    };
    if (WCOL) {
        // one (block, group) per thread, block fastest across lanes; its 16 entries are stored in the column of every
        // plane word covering the block (tier t, plane p, block j of the tier: column wbase[t] + p * blocks_t + j)
        for (int gi = tid; gi < 8 * nblk; gi += blockDim.x) {
            const int ga = gi % nblk, cgrp = gi / nblk;
            int t = 0;
            while (t + 1 < ts.T && 32 * ga >= ts.e[t]) t++;
            if (32 * ga < ts.s[t] || 32 * ga >= ts.e[t]) continue;  // past the last tier: no word reads it
            float e16[16];
            entries(ga, cgrp, e16);
            const int nbt = ts.kb[t] / 4, c0 = ts.wbase[t] + ga - ts.s[t] / 32;
            for (int pl = 0; pl < ts.bits[t]; pl++) {
                float* out = lut + (cgrp * 16) * GA + c0 + pl * nbt;
#pragma unroll
                for (int v = 0; v < 16; v++) out[v * GA] = e16[v];
            }
        }
    } else {
        // one 4-coordinate group per thread (ga fastest across lanes: conflict-free stores)
        for (int gi = tid; gi < 8 * GA; gi += blockDim.x) {
            const int ga = gi % GA, cgrp = gi / GA;
            float e16[16];
            entries(ga, cgrp, e16);
            float* out = lut + (cgrp * 16) * GA + ga;
#pragma unroll
            for (int v = 0; v < 16; v++) out[v * GA] = e16[v];
        }
    }
    if (warp < ts.T) {  // warp t reduces tier t
        float a = 0.f, b = 0.f;
        for (int i = ts.s[warp] + lane; i < ts.e[warp]; i += 32) {
            const float x = zat(i);
            a += x;
            b += x * x;
        }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
            s_qsum[warp] = a;
            s_qn2[warp] = b;
        }
    }
    __syncthreads();
    // per-lane word descriptors (same for every candidate): tier, plane, byte offset in the plane segment, block ga
    int wt[WPL], wp[WPL], wj[WPL], wg[WPL];
    float wsc[WPL];  // 2^(b-1-p) * delta_t of the word's plane
#pragma unroll
    for (int u = 0; u < WPL; u++) {
        const int w = lane + 32 * u;
        int t = 0;
        while (t + 1 < ts.T && w >= ts.wbase[t + 1]) t++;
        const int r = w - ts.wbase[t], wpp = ts.kb[t] / 4;
        wt[u] = w < ts.nwords ? t : -1;
        wp[u] = r / wpp;
        wj[u] = (r - wp[u] * wpp) * 4;
        wg[u] = ts.s[t] / 32 + wj[u] / 4;
        wsc[u] = ts.pw[t][wp[u] < 8 ? wp[u] : 0] * ts.delta[t];
    }
    const int tl = lane < ts.T ? lane : 0;
    const float dmq = ts.delta[tl] * ts.mid[tl] * s_qsum[tl], qn2l = s_qn2[tl];
    const float qcv = qc[q];
    // a small batch splits each query's candidates over gridDim.y CTAs (rounds of 2 * nw candidates, round-robin),
    // each with its own copy of the table
    // each warp scores two candidates per round; the next round's plane words are fetched before this round's
    // lookups, so that a round's load latency overlaps the previous round's table work
    uint32_t wv[2][WPL], wn[2][WPL];
    float scl[2], sgl[2], scn[2], sgn[2];
    const int step = gridDim.y * 2 * nw;
    auto fetch = [&](int r0, uint32_t (&w)[2][WPL], float (&sc)[2], float (&sg)[2]) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int i = r0 + c * nw;
            const bool lv = i < lim;
            const int64_t n = lv ? s_pos[i] : 0;
#pragma unroll
            for (int u = 0; u < WPL; u++) {
                w[c][u] = 0;
                if (lv && wt[u] >= 0) {
                    const int t = wt[u];
                    if (REC)
                        w[c][u] = __ldg(reinterpret_cast<const uint32_t*>(rs.rec + n * rs.RB) + lane + 32 * u);
                    else
                        w[c][u] = __ldg(reinterpret_cast<const uint32_t*>(
                            ts.planes[t] + ((int64_t)wp[u] * N + n) * ts.kb[t] + wj[u]));
                }
            }
            if (REC) {
                const uint32_t sp = (lv && lane < ts.T)
                                        ? __ldg(reinterpret_cast<const uint32_t*>(rs.rec + n * rs.RB + rs.soff) + lane)
                                        : 0u;
                sc[c] = __half2float(__ushort_as_half((unsigned short)(sp & 0xffffu)));
                sg[c] = __half2float(__ushort_as_half((unsigned short)(sp >> 16)));
            } else {
                sc[c] = (lv && lane < ts.T) ? __half2float(scale[(int64_t)lane * N + n]) : 0.f;
                sg[c] = (lv && lane < ts.T) ? __half2float(sig[(int64_t)lane * N + n]) : 0.f;
            }
        }
    };
    // (with more than 4 words per lane the second set of registers would spill: fetch and score in turn)
    constexpr bool PREFETCH = WPL <= 4;
    int i0 = warp + blockIdx.y * 2 * nw;
    if (PREFETCH && i0 < lim) fetch(i0, wn, scn, sgn);
    for (; i0 < lim; i0 += step) {
        if (PREFETCH) {
#pragma unroll
            for (int c = 0; c < 2; c++) {
                scl[c] = scn[c];
                sgl[c] = sgn[c];
#pragma unroll
                for (int u = 0; u < WPL; u++) wv[c][u] = wn[c][u];
            }
            if (i0 + step < lim) fetch(i0 + step, wn, scn, sgn);
        } else {
            fetch(i0, wv, scl, sgl);
        }
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const bool live = i0 + c * nw < lim;
            float part = lane < ts.T ? -dmq * scl[c] : 0.f;
            float var = lane < ts.T ? qn2l * sgl[c] * sgl[c] : 0.f;
#pragma unroll
            for (int u = 0; u < WPL; u++) {
                const int t = wt[u];
                const float st = __shfl_sync(0xffffffffu, scl[c], t < 0 ? 0 : t);
                if (t >= 0) {
                    const uint32_t w = wv[c][u];
                    float a = 0.f;
                    if (WCOL) {
                        // byte offset of entry (c, v, column) = (c * 16 + v) * GA * 4 + column * 4 with GA * 4 = 2^9:
                        // the nibble shifted to bits 9..12 and or-ed with the lane's column offset
                        const uint32_t cb = (uint32_t)(lane + 32 * u) * 4u;
                        const char* tb = reinterpret_cast<const char*>(lut);
#pragma unroll
                        for (int bi = 0; bi < 4; bi++) {
                            const float xh = *reinterpret_cast<const float*>(
                                tb + (2 * bi) * 16 * GA * 4 + (nibble_at9(w, 8 * bi + 4) | cb));
                            const float xl = *reinterpret_cast<const float*>(
                                tb + (2 * bi + 1) * 16 * GA * 4 + (nibble_at9(w, 8 * bi) | cb));
                            a += xh + xl;
                        }
                    } else {
                        const float* lt = lut + wg[u];
#pragma unroll
                        for (int bi = 0; bi < 4; bi++) {
                            const uint32_t byt = (w >> (8 * bi)) & 0xffu;
                            a += lt[((2 * bi) * 16 + (byt >> 4)) * GA] + lt[((2 * bi + 1) * 16 + (byt & 15u)) * GA];
                        }
                    }
                    part += a * wsc[u] * st;
                }
            }
            part = warp_sum(part);
            var = warp_sum(var);
            if (lane == 0 && live) {
                est[(int64_t)q * K + i0 + c * nw] = qcv + part;
                sd[(int64_t)q * K + i0 + c * nw] = sqrtf(var);
            }
        }
    }
}

// Fused LUT score with one candidate per thread (large batches): the same estimate as lut_score_zq_kernel on packed
// records, organised so that every lane of a warp scores its own candidate and all lanes take the same plane word at
// each step.  The CTA builds the query's table once (entry (block ga, group c, nibble v) at ga*128 + c*16 + v: the 32
// lanes reading one (ga, c) touch at most 16 consecutive words, conflict-free) and a per-word list (table block,
// tier, plane weight); each lane then streams its record in 32-byte steps (two steps in flight) and folds each
// finished tier as delta_t * (a_t - mid_t * qsum_t) * scale_t, the reference's per-tier form.  No warp reduction per
// candidate.
constexpr int LC_THREADS = 128;

// fp32 load from a 32-bit address in the shared window
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}

template <bool HALF>
__global__ void __launch_bounds__(LC_THREADS) lut_cand_kernel(const int64_t* __restrict__ pos, int K,
                                                              const float* __restrict__ qc,
                                                              const void* __restrict__ Zq, int ldz, int zh, int D,
                                                              TierSet ts, const int32_t* __restrict__ ncnt,
                                                              float* __restrict__ est, float* __restrict__ sd,
                                                              RecSet rs) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_qsum[MAX_TIERS], s_qn2[MAX_TIERS];
    const int nblk = D / 32, nwords = ts.nwords;
    // the table starts on a 256-byte boundary of the shared window (the launch reserves 256 bytes for it), so that
    // every lookup address is one byte permutation of a block base and the word's nibble offsets
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
    const uint32_t pad = (256u - (sbase & 255u)) & 255u;
    const uint32_t tab_s = sbase + pad;
    float* tab = reinterpret_cast<float*>(smem + pad);             // nblk * 128
    uint2* wmeta = reinterpret_cast<uint2*>(tab + nblk * 128);  // per word: (table byte offset | tier << 24, 2^(b-1-p))
    const int q = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t qK = (int64_t)q * K;
    for (int w = tid; w < nwords; w += LC_THREADS) {
        int t = 0;
        while (t + 1 < ts.T && w >= ts.wbase[t + 1]) t++;
        const int r = w - ts.wbase[t], wpp = ts.kb[t] / 4;
        const int p = r / wpp, j4 = r - p * wpp;
        wmeta[w] = make_uint2((uint32_t)((ts.s[t] / 32 + j4) * 128 * 4) | ((uint32_t)t << 24),
                              __float_as_uint(ts.pw[t][p]));
    }
    // group g = 4-coordinate group (block g / 8, group g % 8) holds coordinates 4g .. 4g+3.  Entry v sums the selected
    // coordinates left to right in fp32 from 0, as acc += z_i * bit_i does (bit 8 of v selects z0, 4 z1, 2 z2, 1 z3).
    // Four threads build a group, thread x its entries 4x .. 4x+3 (z0, z1 selected by x): the prefix p over z0, z1,
    // then p, p + z3, p + z2, (p + z2) + z3 -- the same additions in the same order; consecutive threads store
    // consecutive 16-byte quarters (conflict-free).
    for (int gx = tid; gx < nblk * 32; gx += LC_THREADS) {
        const int g = gx >> 2, x = gx & 3;
        float z[4];
        if (zh) {
            const uint2 h = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(Zq) +
                                                                  (int64_t)q * ldz + 4 * g));
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
            z[0] = a.x, z[1] = a.y, z[2] = b.x, z[3] = b.y;
        } else {
            const float4 f = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(Zq) +
                                                                    (int64_t)q * ldz + 4 * g));
            z[0] = f.x, z[1] = f.y, z[2] = f.z, z[3] = f.w;
        }
        float p = 0.f;
        if (x & 2) p = __fadd_rn(p, z[0]);
        if (x & 1) p = __fadd_rn(p, z[1]);
        const float p2 = __fadd_rn(p, z[2]);
        float o[4] = {p, __fadd_rn(p, z[3]), p2, __fadd_rn(p2, z[3])};
        if (HALF) {
#pragma unroll
            for (int u = 0; u < 4; u++) o[u] = __half2float(__float2half_rn(o[u]));
        }
        reinterpret_cast<float4*>(tab)[gx] = make_float4(o[0], o[1], o[2], o[3]);
    }
    for (int t = warp; t < ts.T; t += LC_THREADS / 32) {
        float a = 0.f, b = 0.f;
        for (int k = ts.s[t] + lane; k < ts.e[t]; k += 32) {
            const float x = zh ? __half2float(reinterpret_cast<const __half*>(Zq)[(int64_t)q * ldz + k])
                                    : reinterpret_cast<const float*>(Zq)[(int64_t)q * ldz + k];
            a += x;
            b += x * x;
        }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
            s_qsum[t] = a;
            s_qn2[t] = b;
        }
    }
    __syncthreads();
    const int i = blockIdx.y * LC_THREADS + tid;
    if (i >= K) return;
    const int lim = ncnt ? min(max(ncnt[q], 0), K) : K;
    if (i >= lim) {
        est[qK + i] = kNeg;
        sd[qK + i] = 0.f;
        return;
    }
    const int64_t n = pos[qK + i];
    const uint8_t* rec = rs.rec + n * rs.RB;
    float sc[MAX_TIERS];
    float var = 0.f;
#pragma unroll
    for (int t = 0; t < MAX_TIERS; t++) {
        sc[t] = 0.f;
        if (t < ts.T) {
            const uint32_t sp = __ldg(reinterpret_cast<const uint32_t*>(rec + rs.soff) + t);
            sc[t] = __half2float(__ushort_as_half((unsigned short)(sp & 0xffffu)));
            const float g = __half2float(__ushort_as_half((unsigned short)(sp >> 16)));
            var = var + s_qn2[t] * g * g;
        }
    }
    float acc = qc[q], at = 0.f;
    int ct = 0;
    auto fold = [&](int t, float a) {  // t uniform over the warp
        float s = 0.f;
#pragma unroll
        for (int u = 0; u < MAX_TIERS; u++)
            if (u == t) s = sc[u];
        acc = acc + ts.delta[t] * (a - ts.mid[t] * s_qsum[t]) * s;
    };
    // the record streams in 32-byte steps (two 16-byte chunks, a whole sector), two steps in flight ahead of the one
    // being scored
    const uint4* rp = reinterpret_cast<const uint4*>(rec);
    const int nst = (nwords + 7) / 8;
    auto ld = [&](int st, uint4& a, uint4& b) {
        a = st < nst ? __ldg(rp + 2 * st) : make_uint4(0u, 0u, 0u, 0u);
        b = st < nst && 8 * st + 4 < nwords ? __ldg(rp + 2 * st + 1) : make_uint4(0u, 0u, 0u, 0u);
    };
    uint4 n1a, n1b, n2a, n2b;
    ld(0, n1a, n1b);
    ld(1, n2a, n2b);
    for (int k = 0; k < nst; k++) {
        const uint32_t wd8[8] = {n1a.x, n1a.y, n1a.z, n1a.w, n1b.x, n1b.y, n1b.z, n1b.w};
        n1a = n2a;
        n1b = n2b;
        ld(k + 2, n2a, n2b);
        uint4 mp;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int w = 8 * k + u;
            if (w >= nwords) break;
            if ((u & 1) == 0) mp = reinterpret_cast<const uint4*>(wmeta)[w >> 1];   // the entries of words w, w + 1
            const uint2 m = (u & 1) ? make_uint2(mp.z, mp.w) : make_uint2(mp.x, mp.y);
            const int t = (int)(m.x >> 24);
            if (t != ct) {
                fold(ct, at);
                ct = t;
                at = 0.f;
            }
            // the word's table block (512 bytes, groups 0..7 of 16 entries) starts at A, a multiple of 256; the
            // entries of byte bi sit at A + 128 bi + (high nibble: 4 v, low nibble: 64 + 4 v).  Byte bi of ho / lo is
            // that offset's low 8 bits (128 (bi & 1) + [64] + 4 v < 256) and A + 256 (bi >> 1) supplies the rest, so
            // one byte permutation forms each lookup address
            const uint32_t A = tab_s + (m.x & 0xffffffu);
            const uint32_t wd = wd8[u];
            const uint32_t ho = ((wd >> 2) & 0x3C3C3C3Cu) | 0x80008000u, lo = ((wd << 2) & 0x3C3C3C3Cu) | 0xC040C040u;
            float a = 0.f;
#pragma unroll
            for (int bi = 0; bi < 4; bi++) {
                const uint32_t base = bi < 2 ? A : A + 256u;
                a += lds_f32(__byte_perm(ho, base, 0x7650u | bi)) + lds_f32(__byte_perm(lo, base, 0x7650u | bi));
            }
            at += a * __uint_as_float(m.y);
        }
    }
    fold(ct, at);
    est[qK + i] = acc;
    sd[qK + i] = sqrtf(var);
}

// CTAs per query of the fused LUT kernel: enough for about two per SM when the batch is small, at most one per 16
// candidates (two rounds of its 8 warps)
static int lut_split(int B, int K) {
    if (B <= 0) return 1;
    const int want = (2 * fvs_sm_count() + B - 1) / B;
    const int cap = (K + 15) / 16;
    return want < 1 ? 1 : (want < cap ? want : cap);
}

static int make_tiers(TierSet& ts, int T, const int32_t* s, const int32_t* e, const int32_t* bits,
                      const float* delta, const uint8_t* const* planes) {
    if (T < 1 || T > MAX_TIERS) return FVS_ERANGE;
    ts.T = T;
    int loff = 0;
    for (int t = 0; t < T; t++) {
        if (e[t] <= s[t] || (e[t] - s[t]) % 8 != 0) return FVS_EINVAL;
        ts.s[t] = s[t];
        ts.e[t] = e[t];
        ts.bits[t] = bits ? bits[t] : 0;
        if (bits && (bits[t] < 1 || bits[t] > 8)) return FVS_EINVAL;
        ts.kb[t] = (e[t] - s[t]) / 8;
        ts.loff[t] = loff;
        loff += (e[t] - s[t]) / 4 * 16;
        ts.delta[t] = delta ? delta[t] : 0.f;
        ts.mid[t] = bits ? ((1 << bits[t]) - 1) * 0.5f : 0.f;
        for (int p = 0; p < 8; p++) ts.pw[t][p] = (bits && p < bits[t]) ? (float)(1 << (bits[t] - 1 - p)) : 0.f;
        ts.planes[t] = planes ? planes[t] : nullptr;
    }
    int w = 0;
    for (int t = 0; t < T; t++) {
        ts.wbase[t] = w;
        w += ts.bits[t] * ts.kb[t] / 4;
    }
    ts.wbase[T] = w;
    ts.nwords = w;
    return FVS_OK;
}

}  // namespace fvs

extern "C" int fvs_lut_build(fvs_stream_t stream, const float* Zq, int B, int ldz, int D, int half, void* L, int T,
                             const int32_t* tier_s, const int32_t* tier_e, float* qsum, float* qn2) {
    FVS_CHECK_ARG(Zq && L && tier_s && tier_e && qsum && qn2 && B >= 0 && D > 0 && D % 4 == 0 && ldz >= D);
    fvs::TierSet ts;
    int rc = fvs::make_tiers(ts, T, tier_s, tier_e, nullptr, nullptr, nullptr);
    if (rc) return rc;
    for (int t = 0; t < T; t++)
        if (tier_e[t] > D) return FVS_EINVAL;
    if (B == 0) return FVS_OK;
    if (half)
        fvs::lut_build_kernel<true><<<B, 256, 0, stream>>>(Zq, ldz, D, L, ts, B, qsum, qn2);
    else
        fvs::lut_build_kernel<false><<<B, 256, 0, stream>>>(Zq, ldz, D, L, ts, B, qsum, qn2);
    return fvs_launch_status();
}

extern "C" int fvs_lut_score(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const void* L,
                             int half, int LW, int T, const int32_t* tier_s, const int32_t* tier_e,
                             const int32_t* tier_bits, const float* tier_delta, const uint8_t* const* tier_planes,
                             const uint16_t* scale, const uint16_t* sig, int64_t N, const float* qsum, const float* qn2,
                             const int32_t* ncnt, float* est, float* sd) {
    FVS_CHECK_ARG(pos && qc && L && tier_s && tier_e && tier_bits && tier_delta && tier_planes && scale && sig);
    FVS_CHECK_ARG(qsum && qn2 && est && sd && B >= 0 && K >= 1 && N > 0 && LW > 0);
    fvs::TierSet ts;
    int rc = fvs::make_tiers(ts, T, tier_s, tier_e, tier_bits, tier_delta, tier_planes);
    if (rc) return rc;
    for (int t = 0; t < T; t++) FVS_CHECK_ARG(tier_planes[t] != nullptr);
    if (ts.loff[T - 1] + (tier_e[T - 1] - tier_s[T - 1]) / 4 * 16 > LW) return FVS_EINVAL;
    const size_t esz = half ? 2 : 4;
    if ((LW * esz) % 16 != 0) return FVS_EINVAL;
    const size_t sm = (size_t)LW * esz;
    if (sm > 200 * 1024) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    cudaError_t e;
    if (half) {
        e = fvs_ensure_smem((const void*)fvs::lut_score_kernel<true>, sm);
        if (e != cudaSuccess) return (int)e;
        fvs::lut_score_kernel<true><<<B, 256, sm, stream>>>(pos, B, K, qc, L, LW, ts, (const __half*)scale,
                                                            (const __half*)sig, N, qsum, qn2, ncnt, est, sd);
    } else {
        e = fvs_ensure_smem((const void*)fvs::lut_score_kernel<false>, sm);
        if (e != cudaSuccess) return (int)e;
        fvs::lut_score_kernel<false><<<B, 256, sm, stream>>>(pos, B, K, qc, L, LW, ts, (const __half*)scale,
                                                             (const __half*)sig, N, qsum, qn2, ncnt, est, sd);
    }
    return fvs_launch_status();
}

extern "C" int fvs_lut_score_zq(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const void* Zq,
                                int ldz, int zq_half, int D, int half, int T, const int32_t* tier_s, const int32_t* tier_e,
                                const int32_t* tier_bits, const float* tier_delta, const uint8_t* const* tier_planes,
                                const uint16_t* scale, const uint16_t* sig, int64_t N, const int32_t* ncnt, float* est,
                                float* sd) {
    FVS_CHECK_ARG(pos && qc && Zq && tier_s && tier_e && tier_bits && tier_delta && tier_planes && scale && sig);
    FVS_CHECK_ARG(est && sd && B >= 0 && K >= 1 && N > 0 && D > 0 && D % 4 == 0 && ldz >= D && ldz % 4 == 0);
    FVS_CHECK_ARG(((uintptr_t)Zq & 15) == 0);
    fvs::TierSet ts;
    int rc = fvs::make_tiers(ts, T, tier_s, tier_e, tier_bits, tier_delta, tier_planes);
    if (rc) return rc;
    for (int t = 0; t < T; t++) {
        FVS_CHECK_ARG(tier_planes[t] != nullptr && tier_e[t] <= D && (tier_e[t] - tier_s[t]) % 32 == 0);
        if (t > 0) FVS_CHECK_ARG(tier_s[t] == tier_e[t - 1]);
    }
    FVS_CHECK_ARG(tier_s[0] == 0);
    const int wpl = (ts.nwords + 31) / 32;
    if (wpl > 12) return FVS_ERANGE;
    const int GA = ((D / 32) + 31) / 32 * 32;
    FVS_CHECK_ARG(D % 32 == 0);
    // up to 128 plane words: one table column per word (conflict-free lookups, 64 KB); more: one column per block
    const bool wcol = wpl <= 4;
    const size_t sm = (size_t)128 * (wcol ? 128 : GA) * 4 + (size_t)K * 4;
    if (sm > 200 * 1024) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    const fvs::RecSet rs{nullptr, 0, 0};
    const int S = fvs::lut_split(B, K);
#define FVS_LZ(H, W, C)                                                                                            \
    do {                                                                                                           \
        cudaError_t e = fvs_ensure_smem((const void*)fvs::lut_score_zq_kernel<H, W, false, 0, C>, sm);            \
        if (e != cudaSuccess) return (int)e;                                                                       \
        fvs::lut_score_zq_kernel<H, W, false, 0, C><<<dim3(B, S), 256, sm, stream>>>(                              \
            pos, B, K, qc, Zq, ldz, zq_half, D, GA, ts, (const __half*)scale, (const __half*)sig, N, ncnt, est, sd,   \
            rs);                                                                                                   \
    } while (0)
    if (half) {
        if (wcol) FVS_LZ(true, 4, true); else if (wpl <= 8) FVS_LZ(true, 8, false); else FVS_LZ(true, 12, false);
    } else {
        if (wcol) FVS_LZ(false, 4, true); else if (wpl <= 8) FVS_LZ(false, 8, false); else FVS_LZ(false, 12, false);
    }
#undef FVS_LZ
    return fvs_launch_status();
}

extern "C" int fvs_lut_score_rec(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc,
                                 const void* Zq, int ldz, int zq_half, int D, int half, int T, const int32_t* tier_s,
                                 const int32_t* tier_e, const int32_t* tier_bits, const float* tier_delta,
                                 const uint8_t* rec, int RB, int soff, int64_t N, const int32_t* ncnt, float* est,
                                 float* sd) {
    FVS_CHECK_ARG(pos && qc && Zq && tier_s && tier_e && tier_bits && tier_delta && rec && est && sd);
    FVS_CHECK_ARG(B >= 0 && K >= 1 && N > 0 && D > 0 && D % 32 == 0 && ldz >= D && ldz % 4 == 0);
    FVS_CHECK_ARG(((uintptr_t)Zq & 15) == 0 && ((uintptr_t)rec & 15) == 0 && RB > 0 && RB % 16 == 0);
    fvs::TierSet ts;
    int rc = fvs::make_tiers(ts, T, tier_s, tier_e, tier_bits, tier_delta, nullptr);
    if (rc) return rc;
    for (int t = 0; t < T; t++) {
        FVS_CHECK_ARG(tier_e[t] <= D && (tier_e[t] - tier_s[t]) % 32 == 0);
        if (t > 0) FVS_CHECK_ARG(tier_s[t] == tier_e[t - 1]);
    }
    FVS_CHECK_ARG(tier_s[0] == 0);
    FVS_CHECK_ARG(soff == 4 * ts.nwords && soff + 4 * T <= RB);
    const int wpl = (ts.nwords + 31) / 32;
    if (wpl > 12) return FVS_ERANGE;
    const int GA = ((D / 32) + 31) / 32 * 32;
    // up to 128 plane words: one table column per word (conflict-free lookups, 64 KB); more: one column per block
    const bool wcol = wpl <= 4;
    const size_t sm = (size_t)128 * (wcol ? 128 : GA) * 4 + (size_t)K * 4;
    if (sm > 200 * 1024) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    const fvs::RecSet rs{rec, RB, soff};
    if (B >= fvs_sm_count() && ts.T <= fvs::MAX_TIERS && ts.nwords <= 4 * RB / 16) {
        // large batch: one candidate per thread
        // the table, the word list padded to whole 8-word steps (read in pairs), the table's alignment
        const size_t smc = (size_t)(D / 32) * 128 * 4 + (size_t)((ts.nwords + 7) & ~7) * 8 + 256;
        const dim3 grid(B, (K + fvs::LC_THREADS - 1) / fvs::LC_THREADS);
        cudaError_t e = half ? fvs_ensure_smem((const void*)fvs::lut_cand_kernel<true>, smc)
                             : fvs_ensure_smem((const void*)fvs::lut_cand_kernel<false>, smc);
        if (e != cudaSuccess) return (int)e;
        if (half)
            fvs::lut_cand_kernel<true><<<grid, fvs::LC_THREADS, smc, stream>>>(pos, K, qc, Zq, ldz, zq_half, D, ts,
                                                                                ncnt, est, sd, rs);
        else
            fvs::lut_cand_kernel<false><<<grid, fvs::LC_THREADS, smc, stream>>>(pos, K, qc, Zq, ldz, zq_half, D, ts,
                                                                                 ncnt, est, sd, rs);
        return fvs_launch_status();
    }
    const int S = fvs::lut_split(B, K);
#define FVS_LRG(H, W, G, C)                                                                                        \
    do {                                                                                                           \
        cudaError_t e = fvs_ensure_smem((const void*)fvs::lut_score_zq_kernel<H, W, true, G, C>, sm);             \
        if (e != cudaSuccess) return (int)e;                                                                       \
        fvs::lut_score_zq_kernel<H, W, true, G, C><<<dim3(B, S), 256, sm, stream>>>(                               \
            pos, B, K, qc, Zq, ldz, zq_half, D, GA, ts, nullptr, nullptr, N, ncnt, est, sd, rs);                   \
    } while (0)
#define FVS_LR(H, W)                                                                                               \
    do {                                                                                                           \
        if (GA == 64) FVS_LRG(H, W, 64, false); else if (GA == 32) FVS_LRG(H, W, 32, false);                      \
        else FVS_LRG(H, W, 0, false);                                                                              \
    } while (0)
    if (half) {
        if (wcol) FVS_LRG(true, 4, 0, true); else if (wpl <= 8) FVS_LR(true, 8); else FVS_LR(true, 12);
    } else {
        if (wcol) FVS_LRG(false, 4, 0, true); else if (wpl <= 8) FVS_LR(false, 8); else FVS_LR(false, 12);
    }
#undef FVS_LR
#undef FVS_LRG
    return fvs_launch_status();
}
