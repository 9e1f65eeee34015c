// Int8 stage-1 scan for small batches: an HBM-streaming kernel with 16-byte coalesced loads and dp4a.
//
// Same contract and arithmetic as the tensor-core scan (`_first8c` / `_emit8c`, `throughput/ivf8c_kern.py:2-36`):
// est = ((float(acc) * qs[q]) * zs[n]) + qcp with explicit rounding, block maxima per global 32-row block (mode 0), and
// every row with est >= t0[q] appended to the query's buffer (mode 1).  With few queries a cell is scanned by one or
// two queries only, so there is no tile to share on the tensor cores; instead the work is one CTA per
// (query, probe column, group of four 32-row blocks) straight from the probe list, with no pair sort:
//   * the pair constant is float(QM[q, c]) * mnorm[c] (`throughput/enginei8.py:11-16`),
//   * the first-pass block maxima go to bmc[(q * ncols + j) * MB + blk - cs/32], i.e. the pair slot is q * ncols + j.
// Each warp takes one 32-row block; each half-warp one row per step (16 lanes x 16 bytes = a 256-byte code row), four
// rows per half-warp in flight; the row's dot product is reduced over the 16 lanes by shuffles.
#include "fvs_common.cuh"

namespace fvs {
namespace small {

constexpr int R = 256;
constexpr int WARPS = 4;
constexpr int UNROLL = 4;  // rows per half-warp per step

__device__ __forceinline__ int dot16(const uint4 a, const uint4 b) {
    int s = __dp4a((int)a.x, (int)b.x, 0);
    s = __dp4a((int)a.y, (int)b.y, s);
    s = __dp4a((int)a.z, (int)b.z, s);
    return __dp4a((int)a.w, (int)b.w, s);
}

template <int MODE>
__global__ void __launch_bounds__(32 * WARPS) scan_small_kernel(
    const int8_t* __restrict__ q8, const float* __restrict__ qs, const int64_t* __restrict__ probe, int nprobe,
    int ncols, const __half* __restrict__ QM, int NC, const float* __restrict__ mnorm, const int64_t* __restrict__ off,
    const int8_t* __restrict__ Z, const float* __restrict__ zs, const float* __restrict__ t0, int32_t* __restrict__ cnt,
    float* __restrict__ bval, int32_t* __restrict__ bpos, int M, float* __restrict__ bmc, int MB, int groups) {
    const int pair = blockIdx.x / groups, grp = blockIdx.x - pair * groups;
    const int q = pair / ncols, j = pair - q * ncols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
    const int c = (int)probe[(int64_t)q * nprobe + j];
    const int64_t cs = off[c], ce = off[c + 1];
    if (ce <= cs) return;
    const int64_t b0 = cs / 32, nb = (ce - 1) / 32 - b0 + 1;
    const int64_t blk = b0 + (int64_t)grp * WARPS + warp;
    if (blk - b0 >= nb) return;
    const float v = __half2float(QM[(int64_t)q * NC + c]);
    const float qcp = mnorm ? __fmul_rn(v, mnorm[c]) : v;
    const float sq = qs[q];
    const uint4 qv = reinterpret_cast<const uint4*>(q8 + (int64_t)q * R)[hl];
    const float th = MODE ? t0[q] : 0.f;
    const int64_t lo = blk * 32 > cs ? blk * 32 : cs, hi = blk * 32 + 32 < ce ? blk * 32 + 32 : ce;
    float mx = -INFINITY;
    // a block has at most 32 rows: 32 / (2 * UNROLL) steps; in the emit pass the rows kept over the whole block are
    // reserved with one atomicAdd per warp (the candidate counters of a small batch are shared by thousands of CTAs)
    constexpr int STEPS = 32 / (2 * UNROLL);
    float kest[STEPS * UNROLL];
    uint32_t kmask = 0;
#pragma unroll
    for (int st = 0; st < STEPS; st++) {
        const int64_t r0 = lo + (int64_t)st * 2 * UNROLL;
        uint4 zv[UNROLL];
        float zr[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int64_t r = r0 + 2 * u + half;
            if (r < hi) {
                zv[u] = __ldg(reinterpret_cast<const uint4*>(Z + r * R) + hl);
                zr[u] = __ldg(zs + r);
            } else {
                zv[u] = make_uint4(0, 0, 0, 0);
                zr[u] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int64_t r = r0 + 2 * u + half;
            int acc = dot16(qv, zv[u]);
            acc += __shfl_xor_sync(0xffffffffu, acc, 8);
            acc += __shfl_xor_sync(0xffffffffu, acc, 4);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            const bool valid = r < hi;
            const float est = __fadd_rn(__fmul_rn(__fmul_rn((float)acc, sq), zr[u]), qcp);
            if (MODE == 0) {
                if (valid) mx = fmaxf(mx, est);
            } else {
                kest[st * UNROLL + u] = est;
                if (valid && est >= th) kmask |= 1u << (st * UNROLL + u);
            }
        }
    }
    if (MODE == 1) {
        // lanes 0 and 16 (one per half-warp) hold the kept rows of their half
        const int mine = hl == 0 ? __popc(kmask) : 0;
        const int other = __shfl_xor_sync(0xffffffffu, mine, 16);
        int base = 0;
        if (lane == 0 && mine + other > 0) base = atomicAdd(cnt + q, mine + other);
        base = __shfl_sync(0xffffffffu, base, 0);
        if (hl == 0 && kmask) {
            int idx = base + (half ? other : 0);
#pragma unroll
            for (int e = 0; e < STEPS * UNROLL; e++)
                if ((kmask >> e) & 1u) {
                    if (idx < M) {
                        const int64_t r = lo + (int64_t)(e / UNROLL) * 2 * UNROLL + 2 * (e % UNROLL) + half;
                        bval[(int64_t)q * M + idx] = kest[e];
                        bpos[(int64_t)q * M + idx] = (int32_t)r;
                    }
                    idx++;
                }
        }
    }
    if (MODE == 0) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        if (lane == 0) bmc[(int64_t)pair * MB + (blk - b0)] = mx;
    }
}

}  // namespace small
}  // namespace fvs

extern "C" int fvs_i8_scan_small(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                                 const int64_t* probe, int nprobe, int ncols, const uint16_t* QM, int NC,
                                 const float* mnorm, const int64_t* off, const int8_t* Z, const float* zs,
                                 const float* t0, int32_t* cnt, float* bval, int32_t* bpos, int M, float* bmc, int MB) {
    using namespace fvs::small;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(R == fvs::small::R && B >= 0 && nprobe >= 1 && ncols >= 1 && ncols <= nprobe && NC > 0 && MB > 0);
    FVS_CHECK_ARG(q8 && qs && probe && QM && off && Z && zs);
    FVS_CHECK_ARG(((uintptr_t)Z & 15) == 0 && ((uintptr_t)q8 & 15) == 0);
    if (mode == 0) FVS_CHECK_ARG(bmc);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (B == 0) return FVS_OK;
    // blocks per cell <= MB (MB = ceil(largest cell / 32) + 1: a cell may start inside a block)
    const int groups = (MB + WARPS - 1) / WARPS;
    const int64_t grid = (int64_t)B * ncols * groups;
    if (grid > INT32_MAX) return FVS_ERANGE;
    if (mode == 0)
        scan_small_kernel<0><<<(unsigned)grid, 32 * WARPS, 0, stream>>>(q8, qs, probe, nprobe, ncols, (const __half*)QM,
                                                                        NC, mnorm, off, Z, zs, t0, cnt, bval, bpos, M,
                                                                        bmc, MB, groups);
    else
        scan_small_kernel<1><<<(unsigned)grid, 32 * WARPS, 0, stream>>>(q8, qs, probe, nprobe, ncols, (const __half*)QM,
                                                                        NC, mnorm, off, Z, zs, t0, cnt, bval, bpos, M,
                                                                        bmc, MB, groups);
    return fvs_launch_status();
}
