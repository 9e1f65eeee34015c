// Routing selection and pairing in two launches (the reference's routing top-n_p and `pairs_fast`,
// `throughput/enginei8.py:11-16, 64-70`, which it runs as torch topk + a stable sort + scatter_add + cumsum + gathers).
//
// Launch 1, one CTA per query: the nprobe cells of largest fp16 routing score, ordered by (score desc, cell asc) as
// fvs_route_topk orders them.  The keys (score, cell) sit in registers; a lower bound on the nprobe-th key comes from
// the lanes' maxima (small nprobe) or four subset maxima per thread (larger nprobe), the keys above it are compacted
// into shared memory and ranked by count, and rank < nprobe selects; with more than CAND_CAP keys above the bound the
// cut is found by histogram passes instead.  While placing selected cell c at rank j, the CTA also takes the
// pair's rank inside the cell's list with one atomicAdd on a per-cell cursor (first-pass columns j < n1 on cur1, the
// others on cur2).  The probe row holds (rank in cell << 32 | cell) until launch 2 rewrites it.
// Launch 2, a grid over the pairs: every CTA scans the per-cell counts (cur1 + cur2) into offsets in shared memory,
// then places its pairs: first-pass pairs of cell c at coff[c] + r, the others at coff[c] + cur1[c] + r (each cell's
// first-pass pairs first, the layout of fvs_pairs_split), writes qid, the pair constant float(QM[q, c]) * mnorm[c] and
// the first pass's pair slots, and the plain cell into probe.  One more CTA (the last) places no pairs: it writes
// coff / ccnt / ccnt1, the two passes' work lists for the cell-major scans (the cell-part entries of the order given
// whose cells have pairs) and clears the caller's counters, beside the placing CTAs.  The last CTA to finish clears
// the cursors, so every call leaves them zero for the next.
#include "fvs_common.cuh"

namespace fvs {
namespace rp {

__device__ __forceinline__ uint32_t h2o(uint16_t u) { return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u); }

constexpr int THREADS = 256;
constexpr int MAXP = 512;
constexpr int CAND_CAP = 1024;  // candidates above the lower bound ranked by count; more: histogram passes
constexpr int LANE_BOUND_MAXP = 128;  // routing bound from the lanes' maxima up to this many probes, subset maxima beyond
constexpr int PLACE_THREADS = 1024;
constexpr int LB = 4;  // cells per thread whose loads the bookkeeping CTA issues together
constexpr int MAX_CELLS = 16384;  // per-cell offsets held in shared memory by every placing CTA

template <int V>
__global__ void __launch_bounds__(THREADS) route_rank_kernel(const uint16_t* __restrict__ QM, int NC, int nprobe,
                                                             int n1, int32_t* __restrict__ cur1,
                                                             int32_t* __restrict__ cur2, int64_t* __restrict__ probe) {
    __shared__ RegSelectScratch rs;
    __shared__ int s_fill;
    __shared__ int s_red[32];
    __shared__ uint32_t s_wb[THREADS / 32];
    __shared__ __align__(16) uint32_t s_sel[CAND_CAP + 4];  // candidates (fast path) or the selected keys (radix path)
    const int q = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint4* row = reinterpret_cast<const uint4*>(QM + (int64_t)q * NC);
    uint32_t key[8 * V];  // (order-preserving score << 16) | (65535 - cell); 0 = no cell
#pragma unroll
    for (int v = 0; v < V; v++) {
        const int u = tid + v * THREADS;
        const bool in = u * 8 < NC;
        const uint4 w = in ? __ldg(row + u) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint32_t h = (ws[e >> 1] >> (16 * (e & 1))) & 0xffffu;
            key[8 * v + e] = in ? ((h2o((uint16_t)h) << 16) | (uint32_t)(0xffff - (u * 8 + e))) : 0u;
        }
    }
    if (tid == 0) s_fill = 0;
    // Lower bound T0 on the nprobe-th largest key, each bound being a key value that at least nprobe distinct keys
    // reach.  Up to LANE_BOUND_MAXP probes: every warp takes the r-th largest of its lanes' maxima (r = ceil(nprobe /
    // warps), r rounds of redux.max), T0 the smallest over the warps (0 when a warp has fewer than r lanes with keys).
    // Beyond: every thread keeps the maxima of four disjoint subsets of its keys and T0 is the nprobe-th largest of
    // those 4 * THREADS maxima (histogram passes over four keys per thread; 0 when fewer than nprobe maxima exist),
    // tighter when r is large (nprobe 192 of 8192 cells: 0.123 -> 0.086 ms for both launches; at nprobe 72 of 4096 the
    // lane bound is the faster, 0.053 against 0.060 ms).
    uint32_t T0 = 0u;
    if (nprobe <= LANE_BOUND_MAXP) {
        uint32_t mx = 0u;
#pragma unroll
        for (int i = 0; i < 8 * V; i++) mx = max(mx, key[i]);
        const int r = (nprobe + THREADS / 32 - 1) / (THREADS / 32);
        uint32_t b = 0u;
        for (int it = 0; it < r; it++) {
            b = __reduce_max_sync(0xffffffffu, mx);
            if (mx == b) mx = 0u;
        }
        if (lane == 0) s_wb[warp] = b;
        __syncthreads();
        T0 = 0xffffffffu;
#pragma unroll
        for (int w = 0; w < THREADS / 32; w++) T0 = min(T0, s_wb[w]);
    } else {
        uint32_t mx[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < 8 * V; i++) mx[i & 3] = max(mx[i & 3], key[i]);
        const int nz = block_sum_int(
            (int)(mx[0] != 0u) + (int)(mx[1] != 0u) + (int)(mx[2] != 0u) + (int)(mx[3] != 0u), s_red);
        if (nz >= nprobe) {
            int gt, eq;
            T0 = block_rth_largest_reg<4>(mx, nprobe, rs, &gt, &eq);
        }
    }
#pragma unroll
    for (int i = 0; i < 8 * V; i++)
        if (key[i] != 0u && key[i] >= T0) {
            const int slot = atomicAdd(&s_fill, 1);
            if (slot < CAND_CAP) s_sel[slot] = key[i];
        }
    __syncthreads();
    const int C = s_fill;
    if (C <= CAND_CAP) {
        // the candidates' ranks by count (keys are unique): rank < nprobe selects, and the rank is the probe column
        if (tid < 4) s_sel[C + tid] = 0u;  // pads the last group of four; 0 ranks below every key
        __syncthreads();
        const uint4* s4 = reinterpret_cast<const uint4*>(s_sel);
        const int C4 = (C + 3) >> 2;
        for (int i = tid; i < C; i += THREADS) {
            const uint32_t ki = s_sel[i];
            int rank = 0;
            for (int j = 0; j < C4; j++) {
                const uint4 o = s4[j];
                rank += (int)(o.x > ki) + (int)(o.y > ki) + (int)(o.z > ki) + (int)(o.w > ki);
            }
            if (rank < nprobe) {
                const int c = 0xffff - (int)(ki & 0xffffu);
                const int rr = atomicAdd(rank < n1 ? cur1 + c : cur2 + c, 1);
                probe[(int64_t)q * nprobe + rank] = ((int64_t)rr << 32) | (int64_t)c;
            }
        }
        return;
    }
    // too many candidates above the bound: the exact cut by histogram passes over the register keys
    __syncthreads();
    if (tid == 0) s_fill = 0;
    int above, equal;
    const uint32_t T = block_rth_largest_reg<8 * V>(key, nprobe, rs, &above, &equal);  // keys are unique
#pragma unroll
    for (int i = 0; i < 8 * V; i++)
        if (key[i] != 0u && key[i] >= T) {
            const int slot = atomicAdd(&s_fill, 1);
            if (slot < nprobe) s_sel[slot] = key[i];
        }
    __syncthreads();
    for (int i = tid; i < nprobe; i += THREADS) {
        const uint32_t ki = s_sel[i];
        int rank = 0;
        for (int j = 0; j < nprobe; j++) rank += s_sel[j] > ki;
        const int c = 0xffff - (int)(ki & 0xffffu);
        const int r = atomicAdd(rank < n1 ? cur1 + c : cur2 + c, 1);
        probe[(int64_t)q * nprobe + rank] = ((int64_t)r << 32) | (int64_t)c;
    }
}

// Launch 1 with a per-cell routing scale (the default engine's routing, `src/engine_cell.py:40-42`): the nprobe cells
// of largest float(QM[q, c]) * sc[c] (fp32 product, as fvs_route_topk_scaled), ordered by (score desc, cell asc), on
// 64-bit keys (score key << 32 | ~cell).  The lower bound comes from four subset maxima per thread (one per cell
// index mod 4), its K-th largest over the block found by histogram passes; the cells at or above it are compacted and
// ranked by count.  More than CAND_CAP cells above the bound (many equal scores): the exact cut by histogram passes
// over the score keys, then over the cell keys of the scores tied with it.  Cursors and probe rows as launch 1.
template <int V>
__global__ void __launch_bounds__(THREADS) route_rank_scaled_kernel(const uint16_t* __restrict__ QM,
                                                                    const float* __restrict__ sc, int NC, int nprobe,
                                                                    int n1, int32_t* __restrict__ cur1,
                                                                    int32_t* __restrict__ cur2,
                                                                    int64_t* __restrict__ probe) {
    __shared__ RegSelectScratch rs;
    __shared__ SelectScratch ss;
    __shared__ int s_red[32];
    __shared__ int s_fill;
    __shared__ __align__(16) unsigned long long s_key[CAND_CAP + 2];  // read as 16-byte pairs
    const int q = blockIdx.x, tid = threadIdx.x;
    const uint16_t* qrow = QM + (int64_t)q * NC;
    uint32_t hk[8 * V];  // score keys; 0 = no cell (a finite score's key is never 0)
#pragma unroll
    for (int v = 0; v < V; v++) {
        const int u = tid + v * THREADS;
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
    uint32_t mx[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 8 * V; i++) mx[i & 3] = max(mx[i & 3], hk[i]);
    const int nz =
        block_sum_int((int)(mx[0] != 0u) + (int)(mx[1] != 0u) + (int)(mx[2] != 0u) + (int)(mx[3] != 0u), s_red);
    uint32_t T0 = 0u;
    if (nz >= nprobe) {
        int gt, eq;
        T0 = block_rth_largest_reg<4>(mx, nprobe, rs, &gt, &eq);
    }
#pragma unroll
    for (int v = 0; v < V; v++)
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint32_t h = hk[8 * v + e];
            if (h != 0u && h >= T0) {
                const int slot = atomicAdd(&s_fill, 1);
                if (slot < CAND_CAP)
                    s_key[slot] = ((unsigned long long)h << 32) | (0xffffffffu - (uint32_t)(8 * (tid + v * THREADS) + e));
            }
        }
    __syncthreads();
    const int C = s_fill;
    if (C <= CAND_CAP) {
        if (tid == 0) s_key[C] = 0ull;  // pads an odd count; 0 ranks below every key
        __syncthreads();
        const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(s_key);
        const int C2 = (C + 1) >> 1;
        for (int i = tid; i < C; i += THREADS) {
            const unsigned long long ki = s_key[i];
            int rank = 0;
            for (int j = 0; j < C2; j++) {
                const ulonglong2 o = k2[j];
                rank += (int)(o.x > ki) + (int)(o.y > ki);
            }
            if (rank < nprobe) {
                const int c = (int)(0xffffffffu - (uint32_t)ki);
                const int rr = atomicAdd(rank < n1 ? cur1 + c : cur2 + c, 1);
                probe[(int64_t)q * nprobe + rank] = ((int64_t)rr << 32) | (int64_t)c;
            }
        }
        return;
    }
    __syncthreads();
    if (tid == 0) s_fill = 0;
    int gt, eq;
    const uint32_t Th = block_rth_largest_reg<8 * V>(hk, nprobe, rs, &gt, &eq);
    uint32_t Tl = 0u;
    if (eq > nprobe - gt)  // scores equal to the cut straddle it: the smallest cells among them fill the places left
        Tl = block_select_rth_largest<32, uint32_t>(
            [&](int i) {
                return f2o(__fmul_rn(__half2float(__ushort_as_half(qrow[i])), sc[i])) == Th ? (0xffffffffu - (uint32_t)i)
                                                                                           : 0u;
            },
            NC, nprobe - gt, ss);
    const unsigned long long T = ((unsigned long long)Th << 32) | Tl;
#pragma unroll
    for (int v = 0; v < V; v++)
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint32_t h = hk[8 * v + e];
            if (h != 0u && h >= Th) {
                const unsigned long long k =
                    ((unsigned long long)h << 32) | (0xffffffffu - (uint32_t)(8 * (tid + v * THREADS) + e));
                if (k >= T) {  // unique keys: exactly nprobe of them
                    const int slot = atomicAdd(&s_fill, 1);
                    if (slot < nprobe) s_key[slot] = k;
                }
            }
        }
    __syncthreads();
    for (int i = tid; i < nprobe; i += THREADS) {
        const unsigned long long ki = s_key[i];
        int rank = 0;
        for (int j = 0; j < nprobe; j++) rank += s_key[j] > ki;
        const int c = (int)(0xffffffffu - (uint32_t)ki);
        const int rr = atomicAdd(rank < n1 ? cur1 + c : cur2 + c, 1);
        probe[(int64_t)q * nprobe + rank] = ((int64_t)rr << 32) | (int64_t)c;
    }
}

// exclusive scan of cur1[c] + cur2[c] over the NC cells into coff (shared memory), by one block of PLACE_THREADS
__device__ void scan_counts(const int32_t* __restrict__ cur1, const int32_t* __restrict__ cur2, int NC, int* coff) {
    __shared__ int wsum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (NC + PLACE_THREADS - 1) / PLACE_THREADS;
    const int b0 = tid * per;
    int local = 0;
    // the thread's cells' counts, loads issued four at a time, kept in coff until the offsets replace them
    for (int i0 = 0; i0 < per; i0 += 4) {
        int cnt[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int c = b0 + i0 + u;
            cnt[u] = (i0 + u < per && c < NC) ? cur1[c] + cur2[c] : 0;
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u < per && b0 + i0 + u < NC) {
                coff[b0 + i0 + u] = cnt[u];
                local += cnt[u];
            }
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += v;
        }
        wsum[lane] = w;
    }
    __syncthreads();
    int run = incl - local + (warp > 0 ? wsum[warp - 1] : 0);
    for (int i = 0; i < per; i++)
        if (b0 + i < NC) {
            const int cnt = coff[b0 + i];
            coff[b0 + i] = run;
            run += cnt;
        }
    __syncthreads();
}

struct PlaceOut {
    int32_t *qid, *coff, *ccnt, *ccnt1, *slot, *list1, *list, *nlist, *zero, *done;
    float* qcp;
    int nzero;
};

__global__ void __launch_bounds__(PLACE_THREADS) pairs_place_kernel(int64_t* __restrict__ probe, int B, int nprobe,
                                                                    int n1, int NC, const __half* __restrict__ QM,
                                                                    const float* __restrict__ mnorm,
                                                                    const int32_t* __restrict__ order, int norder,
                                                                    int32_t* __restrict__ cur1,
                                                                    int32_t* __restrict__ cur2, PlaceOut o) {
    extern __shared__ int s_coff[];  // NC
    __shared__ int s_last;
    const int tid = threadIdx.x;
    scan_counts(cur1, cur2, NC, s_coff);
    const int64_t n = (int64_t)B * nprobe;
    const int nplace = gridDim.x - 1;  // placing CTAs; the last one keeps the books
    for (int64_t i = (int64_t)blockIdx.x * PLACE_THREADS + tid; blockIdx.x < nplace && i < n;
         i += (int64_t)nplace * PLACE_THREADS) {
        const int64_t v = probe[i];
        const int c = (int)(v & 0xffff), r = (int)(v >> 32);
        const int q = (int)(i / nprobe), j = (int)(i - (int64_t)q * nprobe);
        const int pos = s_coff[c] + (j < n1 ? r : cur1[c] + r);
        o.qid[pos] = q;
        const float s = __half2float(QM[(int64_t)q * NC + c]);
        o.qcp[pos] = mnorm ? __fmul_rn(s, mnorm[c]) : s;
        if (j < n1 && o.slot) o.slot[(int64_t)q * n1 + j] = pos;
        probe[i] = c;
    }
    if (blockIdx.x == nplace) {
        for (int c0 = 0; c0 < NC; c0 += LB * PLACE_THREADS) {
            int a[LB], b[LB];
#pragma unroll
            for (int u = 0; u < LB; u++) {
                const int c = c0 + u * PLACE_THREADS + tid;
                a[u] = c < NC ? cur1[c] : 0;
                b[u] = c < NC ? cur2[c] : 0;
            }
#pragma unroll
            for (int u = 0; u < LB; u++) {
                const int c = c0 + u * PLACE_THREADS + tid;
                if (c < NC) {
                    o.coff[c] = s_coff[c];
                    o.ccnt[c] = a[u] + b[u];
                    o.ccnt1[c] = a[u];
                }
            }
        }
        for (int i = tid; i < o.nzero; i += PLACE_THREADS) o.zero[i] = 0;
        if (o.list) {
            // the entries (cell | part << 16) of `order` whose cell has first-pass pairs / any pairs, in that order
            __shared__ int wsum[2][32];
            __shared__ int base[2];
            const int lane = tid & 31, warp = tid >> 5;
            if (tid == 0) base[0] = base[1] = 0;
            __syncthreads();
            for (int c0 = 0; c0 < norder; c0 += LB * PLACE_THREADS) {
                // the chunk's order entries, then their cells' counts, loaded together; then one pass per 1024
                int cc[LB], a1[LB], a2[LB];
#pragma unroll
                for (int u = 0; u < LB; u++) {
                    const int ii = c0 + u * PLACE_THREADS + tid;
                    cc[u] = ii < norder ? order[ii] : -1;
                }
#pragma unroll
                for (int u = 0; u < LB; u++) {
                    a1[u] = cc[u] >= 0 ? cur1[cc[u] & 0xffff] : 0;
                    a2[u] = cc[u] >= 0 ? cur2[cc[u] & 0xffff] : 0;
                }
#pragma unroll
                for (int u = 0; u < LB; u++) {
                    if (c0 + u * PLACE_THREADS >= norder) break;  // uniform over the block
                    const int e = cc[u];  // cell | part << 16
                    const bool k1 = e >= 0 && a1[u] > 0;
                    const bool k2 = e >= 0 && a1[u] + a2[u] > 0;
                    const unsigned m1 = __ballot_sync(0xffffffffu, k1), m2 = __ballot_sync(0xffffffffu, k2);
                    if (lane == 0) {
                        wsum[0][warp] = __popc(m1);
                        wsum[1][warp] = __popc(m2);
                    }
                    __syncthreads();
                    int b1 = base[0], b2 = base[1], t1 = 0, t2 = 0;
                    for (int w = 0; w < PLACE_THREADS / 32; w++) {
                        if (w < warp) {
                            b1 += wsum[0][w];
                            b2 += wsum[1][w];
                        }
                        t1 += wsum[0][w];
                        t2 += wsum[1][w];
                    }
                    const unsigned below = (1u << lane) - 1u;
                    if (k1) o.list1[b1 + __popc(m1 & below)] = e;
                    if (k2) o.list[b2 + __popc(m2 & below)] = e;
                    __syncthreads();
                    if (tid == 0) {
                        base[0] += t1;
                        base[1] += t2;
                    }
                    __syncthreads();
                }
            }
            if (tid == 0) {
                o.nlist[0] = base[0];
                o.nlist[1] = base[1];
            }
        }
    }
    // the last CTA out clears the cursors for the next call (every CTA has read them by then)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(o.done, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        for (int c = tid; c < NC; c += PLACE_THREADS) {
            cur1[c] = 0;
            cur2[c] = 0;
        }
        if (tid == 0) *o.done = 0;
    }
}

}  // namespace rp
}  // namespace fvs

static int route_pairs_run(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int n1,
                           const float* sc, const float* mnorm, const int32_t* order, int norder, int64_t* probe,
                           int32_t* qid,
                           float* qcp, int32_t* coff, int32_t* ccnt, int32_t* ccnt1, int32_t* slot, int32_t* list1,
                           int32_t* list, int32_t* nlist, int32_t* zero, int nzero, int32_t* work) {
    using namespace fvs::rp;
    FVS_CHECK_ARG(QM && probe && qid && qcp && coff && ccnt && ccnt1 && work && B >= 0 && NC > 0);
    FVS_CHECK_ARG(nprobe >= 1 && nprobe <= NC && n1 >= 1 && n1 <= nprobe && nzero >= 0);
    FVS_CHECK_ARG(order == nullptr || (list1 && list && nlist && norder >= 0));
    FVS_CHECK_ARG(nzero == 0 || zero != nullptr);
    if (NC % 8 != 0 || ((uintptr_t)QM & 15) != 0 || nprobe > MAXP || NC > MAX_CELLS) return FVS_ERANGE;
    if (sc != nullptr && ((uintptr_t)sc & 15) != 0) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    int32_t *cur1 = work, *cur2 = work + NC, *done = work + 2 * NC;
    const int V = (NC + THREADS * 8 - 1) / (THREADS * 8);
#define FVS_RR(VV)                                                                                                    \
    do {                                                                                                              \
        if (sc)                                                                                                       \
            route_rank_scaled_kernel<VV><<<B, THREADS, 0, stream>>>(QM, sc, NC, nprobe, n1, cur1, cur2, probe);       \
        else                                                                                                          \
            route_rank_kernel<VV><<<B, THREADS, 0, stream>>>(QM, NC, nprobe, n1, cur1, cur2, probe);                  \
    } while (0)
    if (V <= 1)
        FVS_RR(1);
    else if (V <= 2)
        FVS_RR(2);
    else if (V <= 4)
        FVS_RR(4);
    else
        FVS_RR(8);
#undef FVS_RR
    const int64_t npairs = (int64_t)B * nprobe;
    const int nsm = fvs_sm_count();
    int grid = (int)((npairs + PLACE_THREADS * 2 - 1) / (PLACE_THREADS * 2));
    grid = grid > nsm - 1 ? nsm - 1 : grid;
    grid = grid < 1 ? 1 : grid;  // placing CTAs, plus the bookkeeping one
    const size_t sm = (size_t)NC * sizeof(int);
    cudaError_t e = fvs_ensure_smem((const void*)pairs_place_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    PlaceOut o{qid, coff, ccnt, ccnt1, slot, list1, list, nlist, zero, done, qcp, nzero};
    pairs_place_kernel<<<grid + 1, PLACE_THREADS, sm, stream>>>(probe, B, nprobe, n1, NC, (const __half*)QM, mnorm, order,
                                                            order ? norder : 0, cur1, cur2, o);
    return fvs_launch_status();
}

extern "C" int fvs_route_pairs(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int n1,
                               const float* mnorm, const int32_t* order, int norder, int64_t* probe, int32_t* qid,
                               float* qcp, int32_t* coff, int32_t* ccnt, int32_t* ccnt1, int32_t* slot,
                               int32_t* list1, int32_t* list, int32_t* nlist, int32_t* zero, int nzero,
                               int32_t* work) {
    return route_pairs_run(stream, QM, B, NC, nprobe, n1, nullptr, mnorm, order, norder, probe, qid, qcp, coff, ccnt,
                           ccnt1, slot, list1, list, nlist, zero, nzero, work);
}

extern "C" int fvs_route_pairs_scaled(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int n1,
                                      const float* sc, const float* mnorm, const int32_t* order, int norder,
                                      int64_t* probe, int32_t* qid, float* qcp, int32_t* coff, int32_t* ccnt,
                                      int32_t* ccnt1, int32_t* slot, int32_t* list1, int32_t* list, int32_t* nlist,
                                      int32_t* zero, int nzero, int32_t* work) {
    FVS_CHECK_ARG(sc != nullptr);
    return route_pairs_run(stream, QM, B, NC, nprobe, n1, sc, mnorm, order, norder, probe, qid, qcp, coff, ccnt,
                           ccnt1, slot, list1, list, nlist, zero, nzero, work);
}
