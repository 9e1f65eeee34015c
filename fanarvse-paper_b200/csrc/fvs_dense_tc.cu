// Routing-free int8 scan on the 5th-generation tensor cores (tcgen05, sm_100a): the dense [B x R] x [R x N]
// contraction of every query code with every row code, fused with the reference's score and threshold-emit epilogue.
//
// Contract of `_scan` in `throughput/brute.py:7-39` (MODE 0: dense scores of a row sample; MODE 1: emit every row with
// est >= t0[q] into the query's buffer, one atomic per (query, 32-row group) of kept rows):
//     est[q, n] = (float(acc[q, n]) * qs[q]) * float(zs[n]),   acc = sum_k q8[q, k] * Z[n, k]  (exact int32)
// with explicit round-to-nearest multiplies (no contraction), as the reference's expression evaluates.
//
// Persistent kernel, one CTA per SM, walking output tiles of 128 rows x QB queries (QB = min(256, B rounded up to
// 16)), tile t = (row block t / nqb, query block t % nqb), so the CTAs running at one time share row blocks through L2
// and the queries stay L2-resident.  Warp roles (320 threads):
//   warp 0    : TMA producer: per K-chunk of 128 bytes, the 128-row code box and the QB-row query box (128 B swizzle)
//               into one of STAGES shared-memory stages
//   warp 1    : TMEM allocation (2 x 256 columns); lane 0 issues tcgen05.mma.kind::i8 (M=128, N=QB, K=32 x 4 per
//               chunk) into accumulator buffer (tile & 1), releasing each stage when its MMAs complete
//   warps 2-9 : two epilogue warpgroups; warp w reads TMEM lanes 32*(w%4).. (its 32 rows), group g the columns
//               [128 g, 128 g + 128) of the tile, 32 at a time (tcgen05.ld), while the MMAs of the next tile run into
//               the other buffer.
// Every mbarrier wait is bounded; on expiry the CTA raises `status`, drains what it issued, frees TMEM and returns.
#include <cuda.h>

#include "fvs_common.cuh"
#include "fvs_tcgen05.cuh"

namespace fvs {
namespace dense {
using namespace fvs::tcg;

constexpr int TM = 128;     // code rows per tile (MMA M)
constexpr int QBMAX = 256;  // queries per tile (MMA N)
constexpr int KC = 128;     // K bytes per stage (one 128 B swizzle atom wide)
constexpr int STAGES = 4;
constexpr int A_BYTES = TM * KC;
constexpr int B_BYTES = QBMAX * KC;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int NTHREADS = 32 * (2 + EPI_WARPS);
constexpr uint32_t TMEM_COLS = 2 * QBMAX;
constexpr int COL_OFF = STAGES * STAGE_BYTES;          // per epilogue warp: 32 column masks + 32 bases
constexpr int BAR_OFF = COL_OFF + EPI_WARPS * 64 * 4;
constexpr int NBAR = 2 * STAGES + 4;
constexpr int MISC_OFF = BAR_OFF + NBAR * 8;           // tmem base, abort flag
constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;       // + alignment slack

struct Params {
    const float* qs;
    const __half* zs;
    const float* t0;
    int32_t* cnt;
    float* bval;
    int32_t* bpos;
    float* out;
    int32_t* status;
    int64_t ldo;
    int B, N, NK, QB, nqb, M;
    uint32_t wait_limit;  // polls of every pipeline wait (fvs_set_wait_limit)
};

template <int MODE>
__global__ void __launch_bounds__(NTHREADS, 1) dense_tc_kernel(const __grid_constant__ CUtensorMap zmap,
                                                               const __grid_constant__ CUtensorMap qmap, Params p,
                                                               int ntiles) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = saddr(smem);
    auto full = [&](int s) { return sbase + BAR_OFF + 8 * s; };
    auto empty = [&](int s) { return sbase + BAR_OFF + 8 * (STAGES + s); };
    auto t_full = [&](int b) { return sbase + BAR_OFF + 8 * (2 * STAGES + b); };
    auto t_empty = [&](int b) { return sbase + BAR_OFF + 8 * (2 * STAGES + 2 + b); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + MISC_OFF);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);
    const uint32_t WL = p.wait_limit;

    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(t_full(b), 1);
            mbar_init(t_empty(b), EPI_WARPS);
        }
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
    const uint32_t stage_tx = (uint32_t)(A_BYTES + p.QB * KC);
    int last_load = -1, last_commit = -1;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&zmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&qmap) : "memory");
            int it = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort; t += G) {
                const int row0 = (t / p.nqb) * TM, q0 = (t % p.nqb) * p.QB;
                bool ok = true;
                for (int kc = 0; kc < p.NK; kc++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1, abort, WL)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = sbase + s * STAGE_BYTES;
                    mbar_expect_tx(full(s), stage_tx);
                    tma_load_2d(sa, &zmap, kc * KC, row0, full(s));
                    tma_load_2d(sa + A_BYTES, &qmap, kc * KC, q0, full(s));
                    last_load = it;
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int it = 0, tc = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort; t += G, tc++) {
                const int q0 = (t % p.nqb) * p.QB;
                const int nq16 = (min(p.QB, p.B - q0) + 15) & ~15;
                const uint32_t idesc = i8_idesc(nq16, TM);
                const int b = tc & 1;
                if (!mbar_wait(t_empty(b), ((tc >> 1) & 1) ^ 1, abort, WL)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * QBMAX);
                bool ok = true;
                for (int kc = 0; kc < p.NK; kc++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(full(s), (it / STAGES) & 1, abort, WL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = sbase + s * STAGE_BYTES;
#pragma unroll
                    for (int kk = 0; kk < KC / 32; kk++)
                        mma_i8(d, sw128_desc(sa + kk * 32), sw128_desc(sa + A_BYTES + kk * 32), idesc,
                               (kc | kk) ? 1u : 0u);
                    mma_commit(empty(s));
                    last_commit = it;
                }
                if (!ok) break;
                mma_commit(t_full(b));
            }
        }
        __syncwarp();
    } else {
        const int ew = warp & 3, eg = (warp - 2) >> 2;
        uint32_t* colm = reinterpret_cast<uint32_t*>(smem + COL_OFF) + (warp - 2) * 64;
        int* colb = reinterpret_cast<int*>(colm + 32);
        int tc = 0;
        for (int t = blockIdx.x; t < ntiles && !*abort; t += G, tc++) {
            const int row0 = (t / p.nqb) * TM, q0 = (t % p.nqb) * p.QB;
            const int nq = min(p.QB, p.B - q0);
            const int b = tc & 1;
            if (!warp_wait(t_full(b), (tc >> 1) & 1, abort, WL)) break;
            tc_fence_after();
            const int row = row0 + 32 * ew + lane;
            const bool rvalid = row < p.N;
            const float zr = rvalid ? __half2float(p.zs[row]) : 0.f;
            for (int h = 0; h < 4; h++) {
                const int c0 = eg * 128 + 32 * h;
                if (c0 >= nq) break;
                uint32_t acc[32];
                tmem_ld32(tmem + ((uint32_t)(32 * ew) << 16) + (uint32_t)(b * QBMAX + c0), acc);
                tmem_ld_wait();
                const int nc = min(32, nq - c0);
                const bool cv = lane < nc;
                const float myqs = cv ? p.qs[q0 + c0 + lane] : 0.f;
                if (MODE == 0) {
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        const float s = __shfl_sync(0xffffffffu, myqs, jj);
                        if (jj < nc && rvalid)
                            p.out[(int64_t)(q0 + c0 + jj) * p.ldo + row] =
                                __fmul_rn(__fmul_rn((float)(int32_t)acc[jj], s), zr);
                    }
                } else {
                    const float myt = cv ? p.t0[q0 + c0 + lane] : INFINITY;
                    uint32_t mymask = 0, rowmask = 0;
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        const float s = __shfl_sync(0xffffffffu, myqs, jj);
                        const float th = __shfl_sync(0xffffffffu, myt, jj);
                        const float est = __fmul_rn(__fmul_rn((float)(int32_t)acc[jj], s), zr);
                        const bool keep = rvalid && est >= th;
                        rowmask |= (uint32_t)keep << jj;
                        const uint32_t m = __ballot_sync(0xffffffffu, keep);
                        if (lane == jj) mymask = m;
                    }
                    int mybase = 0;
                    if (mymask) mybase = atomicAdd(p.cnt + q0 + c0 + lane, __popc(mymask));
                    colm[lane] = mymask;
                    colb[lane] = mybase;
                    __syncwarp();
                    while (rowmask) {
                        const int jj = __ffs(rowmask) - 1;
                        rowmask &= rowmask - 1;
                        float accj = 0.f;
#pragma unroll
                        for (int u = 0; u < 32; u++)
                            if (u == jj) accj = (float)(int32_t)acc[u];
                        const int q = q0 + c0 + jj;
                        const float est = __fmul_rn(__fmul_rn(accj, p.qs[q]), zr);
                        const int idx = colb[jj] + __popc(colm[jj] & ((1u << lane) - 1u));
                        if (idx < p.M) {
                            const int64_t o = (int64_t)q * p.M + idx;
                            p.bval[o] = est;
                            p.bpos[o] = row;
                        }
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(t_empty(b));
        }
    }
    // drain what this CTA issued (only pending when a wait gave up; these waits ignore the abort flag): the last load
    // of every stage, and the commit after the last MMA issued (an MMA is only issued right before such a commit)
    if (warp == 0 && lane == 0)
        for (int u = last_load; u >= 0 && u > last_load - STAGES; u--) mbar_drain(full(u % STAGES), (u / STAGES) & 1);
    if (warp == 1 && lane == 0 && last_commit >= 0)
        mbar_drain(empty(last_commit % STAGES), (last_commit / STAGES) & 1);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    if (tid == 0 && *abort && p.status) atomicExch(p.status, 1);
}

// r-th largest of each row of vals [B, ld] over its first n entries (one CTA per row, radix select on
// order-preserving keys, staged in shared memory when they fit)
__global__ void __launch_bounds__(512) rth_largest_kernel(const float* __restrict__ vals, int n, int64_t ld, int r,
                                                          int staged, float* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectScratch ss;
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
    const int q = blockIdx.x;
    const float* v = vals + (int64_t)q * ld;
    uint32_t k;
    if (staged) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = f2o(v[i]);
        __syncthreads();
        k = block_select_rth_largest<32, uint32_t>([&](int i) { return keys[i]; }, n, r, ss);
    } else {
        k = block_select_rth_largest<32, uint32_t>([&](int i) { return f2o(__ldg(v + i)); }, n, r, ss);
    }
    if (threadIdx.x == 0) out[q] = o2f(k);
}

// Same result for r <= RM: every thread keeps the RM largest of its strided share in registers (branch-free insertion,
// taken only by values above its current RM-th), the threads' r best go to shared memory, and one radix select over
// those blockDim * r candidates (a superset of the row's r largest) gives the answer.
template <int RM>
__global__ void __launch_bounds__(512) rth_largest_small_kernel(const float* __restrict__ vals, int n, int64_t ld,
                                                                int r, float* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectScratch ss;
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem);  // blockDim * r
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const float* v = vals + (int64_t)q * ld;
    float top[RM];
#pragma unroll
    for (int j = 0; j < RM; j++) top[j] = -INFINITY;
    constexpr int U = 8;  // independent loads in flight per thread
    for (int i0 = tid; i0 < n; i0 += U * nt) {
        float xs[U];
#pragma unroll
        for (int u = 0; u < U; u++) xs[u] = i0 + u * nt < n ? __ldg(v + i0 + u * nt) : -INFINITY;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const float x = xs[u];
            if (x > top[RM - 1]) {
#pragma unroll
                for (int j = RM - 1; j > 0; j--) top[j] = x > top[j - 1] ? top[j - 1] : fmaxf(top[j], x);
                top[0] = fmaxf(top[0], x);
            }
        }
    }
    // lower bound: a thread's r-th largest (its r values are all >= it, so the row's r-th largest is too); only
    // entries >= the largest such bound can matter, and the threads' top-r lists hold at least r of them
    __shared__ float s_lb[32];
    __shared__ int s_n;
    float kth = INFINITY;  // top[] is sorted descending: its r-th entry is the minimum of the first r
#pragma unroll
    for (int j = 0; j < RM; j++)
        if (j < r) kth = fminf(kth, top[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kth = fmaxf(kth, __shfl_xor_sync(0xffffffffu, kth, o));
    if ((tid & 31) == 0) s_lb[tid >> 5] = kth;
    if (tid == 0) s_n = 0;
    __syncthreads();
    float lb = -INFINITY;
    for (int w = 0; w < (nt >> 5); w++) lb = fmaxf(lb, s_lb[w]);
#pragma unroll
    for (int j = 0; j < RM; j++)
        if (j < r && top[j] >= lb) keys[atomicAdd(&s_n, 1)] = f2o(top[j]);
    __syncthreads();
    const uint32_t k = block_select_rth_largest<32, uint32_t>([&](int i) { return keys[i]; }, s_n, r, ss);
    if (tid == 0) out[q] = o2f(k);
}

}  // namespace dense
}  // namespace fvs

extern "C" int fvs_dense_scan_tc(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                                 const int8_t* Z, const uint16_t* zs, int64_t N, const float* t0, int32_t* cnt,
                                 float* bval, int32_t* bpos, int M, float* out, int64_t ldo, int32_t* status) {
    using namespace fvs::dense;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(q8 && qs && Z && zs && B >= 0 && N >= 0 && N < (int64_t)1 << 31);
    FVS_CHECK_ARG(R >= KC && R % KC == 0 && R <= 8192);
    FVS_CHECK_ARG(((uintptr_t)Z & 15) == 0 && ((uintptr_t)q8 & 15) == 0);
    if (mode == 0) FVS_CHECK_ARG(out && ldo >= N);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (B == 0 || N == 0) return FVS_OK;
    fvs::tcg::EncodeTiledFn enc = fvs::tcg::encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    const int QB = B >= QBMAX ? QBMAX : ((B + 15) & ~15);
    CUtensorMap zmap, qmap;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)R, (cuuint64_t)N};
        const cuuint64_t strides[1] = {(cuuint64_t)R};
        const cuuint32_t box[2] = {(cuuint32_t)KC, (cuuint32_t)TM};
        const cuuint32_t estr[2] = {1, 1};
        if (enc(&zmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)Z, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return FVS_EINVAL;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)R, (cuuint64_t)B};
        const cuuint64_t strides[1] = {(cuuint64_t)R};
        const cuuint32_t box[2] = {(cuuint32_t)KC, (cuuint32_t)QB};
        const cuuint32_t estr[2] = {1, 1};
        if (enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)q8, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return FVS_EINVAL;
    }
    const int nqb = (B + QB - 1) / QB;
    const int64_t nrb = (N + TM - 1) / TM;
    if (nrb * nqb > INT32_MAX) return FVS_ERANGE;
    const int ntiles = (int)(nrb * nqb);
    Params p{qs, (const __half*)zs, t0, cnt, bval, bpos, out, status, ldo, B, (int)N, R / KC, QB, nqb, M,
             pipeline_wait_limit()};
    cudaError_t e = mode ? fvs_ensure_smem((const void*)dense_tc_kernel<1>, SMEM_BYTES)
                         : fvs_ensure_smem((const void*)dense_tc_kernel<0>, SMEM_BYTES);
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
        dense_tc_kernel<0><<<grid, NTHREADS, SMEM_BYTES, stream>>>(zmap, qmap, p, ntiles);
    else
        dense_tc_kernel<1><<<grid, NTHREADS, SMEM_BYTES, stream>>>(zmap, qmap, p, ntiles);
    return fvs_launch_status();
}

extern "C" int fvs_rth_largest(fvs_stream_t stream, const float* vals, int B, int n, int64_t ld, int r, float* out) {
    FVS_CHECK_ARG(vals && out && B >= 0 && n >= 1 && ld >= n && r >= 1 && r <= n);
    if (B == 0) return FVS_OK;
    if (r <= 32) {
        const size_t sk = (size_t)512 * r * 4;
        if (r <= 16) {
            cudaError_t e = fvs_ensure_smem((const void*)fvs::dense::rth_largest_small_kernel<16>, sk);
            if (e != cudaSuccess) return (int)e;
            fvs::dense::rth_largest_small_kernel<16><<<B, 512, sk, stream>>>(vals, n, ld, r, out);
        } else {
            cudaError_t e = fvs_ensure_smem((const void*)fvs::dense::rth_largest_small_kernel<32>, sk);
            if (e != cudaSuccess) return (int)e;
            fvs::dense::rth_largest_small_kernel<32><<<B, 512, sk, stream>>>(vals, n, ld, r, out);
        }
        return fvs_launch_status();
    }
    const size_t want = (size_t)n * 4;
    const int staged = want <= 200 * 1024;
    const size_t sm = staged ? want : 0;
    if (staged) {
        cudaError_t e = fvs_ensure_smem((const void*)fvs::dense::rth_largest_kernel, sm);
        if (e != cudaSuccess) return (int)e;
    }
    fvs::dense::rth_largest_kernel<<<B, 512, sm, stream>>>(vals, n, ld, r, staged, out);
    return fvs_launch_status();
}
