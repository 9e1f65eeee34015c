// Classification, exact re-rank of the ambiguous candidates and final top-k, fused in one kernel (one CTA per query).
//
// Replaces `_finish` lines 92-95 (`throughput/enginei8.py`), `Engine8._s3` (`src/engine3.py:143-146`) and the zero-copy
// stage-3 kernel `_stage3` (`src/stage3_zc.py:11-27`).  The fp16 store H stays in HBM (the reference reads it from
// pinned host memory over PCIe): each ambiguous candidate's row (d x 2 bytes) is read once by one warp with 16-byte
// loads and dotted with the fp32 query in fp32.
#include "fvs_common.cuh"

namespace fvs {

// NT threads per CTA at 2048 / NT CTAs per SM (32 registers): the re-rank is memory-latency bound, and occupancy hides
// the row loads better than more loads per warp (measured 0.083 -> 0.070 ms at 2000 queries, NT = 256); a small batch
// (fewer CTAs than SMs) takes NT = 1024, so that each query's ambiguous rows are spread over 32 warps.

// exact fp32 dot of one fp16 row with the query: lane l owns coordinates 8l + 256c (c = 0..NCH-1, d = 256 NCH), summed
// in c order with the expression of the generic loop in refine_kernel (so both give the same sums); the row's loads go
// out in batches of three 16-byte loads, so that a row costs two load latencies instead of one per chunk
template <int NCH>
__device__ __forceinline__ float row_dot_fixed(const __half* __restrict__ h, const float* __restrict__ qrow, int lane) {
    float acc = 0.f;
#pragma unroll
    for (int c0 = 0; c0 < NCH; c0 += 3) {
        uint4 hv[3];
#pragma unroll
        for (int u = 0; u < 3; u++)
            if (c0 + u < NCH) hv[u] = __ldg(reinterpret_cast<const uint4*>(h + (c0 + u) * 256 + lane * 8));
#pragma unroll
        for (int u = 0; u < 3; u++) {
            if (c0 + u >= NCH) break;
            const int cc = (c0 + u) * 256 + lane * 8;
            const float4 qa = *reinterpret_cast<const float4*>(qrow + cc);
            const float4 qb = *reinterpret_cast<const float4*>(qrow + cc + 4);
            const __half2* h2 = reinterpret_cast<const __half2*>(&hv[u]);
            float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
            float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
            acc += f0.x * qa.x + f0.y * qa.y + f1.x * qa.z + f1.y * qa.w;
            acc += f2.x * qb.x + f2.y * qb.y + f3.x * qb.z + f3.y * qb.w;
        }
    }
    return acc;
}

// the keys of entries 0..K-1 sorted in descending order by one warp (K <= 32 * PER; missing entries are key 0, below
// every key of a float), then key number r (0-based) written to *out by the lane holding it
template <int PER, typename T, typename KeyFn>
__device__ __forceinline__ void warp_rth_sorted(KeyFn key, int K, int r, T* out) {
    const int lane = threadIdx.x & 31;
    T v[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = lane * PER + j;
        v[j] = i < K ? key(i) : (T)0;
    }
    warp_sort_regs_desc<PER>(v);
#pragma unroll
    for (int j = 0; j < PER; j++)
        if (lane * PER + j == r) *out = v[j];
}

template <int NT>
__global__ void __launch_bounds__(NT, 2048 / NT) refine_kernel(const __half* __restrict__ H, int d,
                                                            const int32_t* __restrict__ order,
                                                            const int64_t* __restrict__ pos,
                                                            const float* __restrict__ est, const float* __restrict__ sd,
                                                            int K, float z, int k, int kp, const float* __restrict__ Q,
                                                            int ldq, int32_t* __restrict__ ids, int32_t* __restrict__ I,
                                                            int32_t* __restrict__ reads, float* __restrict__ score_k) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ unsigned hist[2][256];
    __shared__ uint32_t s_bounds[2];
    __shared__ int s_namb;
    uint32_t* klo = reinterpret_cast<uint32_t*>(smem);       // K
    uint32_t* khi = klo + K;                                  // K
    float* score = reinterpret_cast<float*>(khi + K);         // K
    int32_t* cid = reinterpret_cast<int32_t*>(score + K);     // K candidate ids
    int32_t* amb_list = cid + K;                              // K
    unsigned long long* sb = reinterpret_cast<unsigned long long*>(amb_list + K + (K & 1));  // kp
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
    const int64_t qK = (int64_t)q * K;
    for (int i = tid; i < K; i += nt) {
        const float e = est[qK + i], s = sd[qK + i];
        const float zs = __fmul_rn(z, s);
        klo[i] = f2o(__fsub_rn(e, zs));
        khi[i] = f2o(__fadd_rn(e, zs));
        const int32_t id = order[pos[qK + i]];
        cid[i] = id;
        ids[qK + i] = id;
    }
    if (tid == 0) s_namb = 0;
    __syncthreads();
    // (k+1)-th largest hi, k-th largest lo: by register sorts of one warp each when K <= 128, by ranks when K <= 256,
    // else warp selects
    if (K <= 128) {
        if (warp == 0) warp_rth_sorted<4, uint32_t>([&](int i) { return khi[i]; }, K, k, &s_bounds[0]);
        if (warp == 1) warp_rth_sorted<4, uint32_t>([&](int i) { return klo[i]; }, K, k - 1, &s_bounds[1]);
    } else if (K <= 256) {  // ranks, every thread (O(K^2))
        for (int i = tid; i < K; i += nt) {
            const uint32_t hi = khi[i], lo = klo[i];
            int rh = 0, rl = 0;
            for (int j = 0; j < K; j++) {
                const uint32_t hj = khi[j], lj = klo[j];
                rh += (hj > hi) || (hj == hi && j < i);
                rl += (lj > lo) || (lj == lo && j < i);
            }
            if (rh == k) s_bounds[0] = hi;
            if (rl == k - 1) s_bounds[1] = lo;
        }
    } else if (warp == 0) {
        const uint32_t v = warp_select_rth_largest<32, uint32_t>([&](int i) { return khi[i]; }, K, k + 1, hist[0]);
        if (lane == 0) s_bounds[0] = v;
    } else if (warp == 1) {
        const uint32_t v = warp_select_rth_largest<32, uint32_t>([&](int i) { return klo[i]; }, K, k, hist[1]);
        if (lane == 0) s_bounds[1] = v;
    }
    __syncthreads();
    const uint32_t hk1 = s_bounds[0], lk = s_bounds[1];
    // sure: lo > (k+1)-th hi; ambiguous: hi >= k-th lo and not sure (key order == float order)
    for (int i = tid; i < K; i += nt) {
        const bool sure = klo[i] > hk1;
        const bool amb = !sure && khi[i] >= lk;
        score[i] = sure ? __fadd_rn(est[qK + i], 10.f) : -1e9f;
        if (amb) amb_list[atomicAdd(&s_namb, 1)] = i;
    }
    __syncthreads();
    const int namb = s_namb;
    // exact fp32 dot products of the ambiguous rows (one warp per row, 8 halves per lane per step)
    const float* qrow = Q + (int64_t)q * ldq;
    const int nch = (d & 255) == 0 ? d >> 8 : 0;
    for (int a = warp; a < namb; a += nw) {
        const int i = amb_list[a];
        const __half* h = H + (int64_t)cid[i] * d;
        if (nch >= 1 && nch <= 8) {
            float acc;
            switch (nch) {
                case 1: acc = row_dot_fixed<1>(h, qrow, lane); break;
                case 2: acc = row_dot_fixed<2>(h, qrow, lane); break;
                case 3: acc = row_dot_fixed<3>(h, qrow, lane); break;
                case 4: acc = row_dot_fixed<4>(h, qrow, lane); break;
                case 5: acc = row_dot_fixed<5>(h, qrow, lane); break;
                case 6: acc = row_dot_fixed<6>(h, qrow, lane); break;
                case 7: acc = row_dot_fixed<7>(h, qrow, lane); break;
                default: acc = row_dot_fixed<8>(h, qrow, lane); break;
            }
            acc = warp_sum(acc);
            if (lane == 0) score[i] = acc;
            continue;
        }
        float acc = 0.f;
        for (int c0 = lane * 8; c0 < d; c0 += 256) {
            const uint4 hv = *reinterpret_cast<const uint4*>(h + c0);
            const float4 qa = *reinterpret_cast<const float4*>(qrow + c0);
            const float4 qb = *reinterpret_cast<const float4*>(qrow + c0 + 4);
            const __half2* h2 = reinterpret_cast<const __half2*>(&hv);
            float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
            float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
            acc += f0.x * qa.x + f0.y * qa.y + f1.x * qa.z + f1.y * qa.w;
            acc += f2.x * qb.x + f2.y * qb.y + f3.x * qb.z + f3.y * qb.w;
        }
        acc = warp_sum(acc);
        if (lane == 0) score[i] = acc;
    }
    __syncthreads();
    // final top-k by (score desc, id asc; keys are unique): a register sort of one warp when K <= 128, by ranks when
    // K <= 256, else on warp 0 the k-th largest score key, then id order among ties
    auto fkey = [&](int i) {
        return ((unsigned long long)f2o(score[i]) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)cid[i]);
    };
    if (K <= 128) {
        if (warp == 0) {
            {
                unsigned long long v[4];
#pragma unroll
                for (int j = 0; j < 4; j++) v[j] = lane * 4 + j < K ? fkey(lane * 4 + j) : 0ull;
                warp_sort_regs_desc<4>(v);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int r = lane * 4 + j;
                    if (r < k) {
                        I[(int64_t)q * k + r] = (int32_t)(0xffffffffu - (uint32_t)v[j]);
                        if (score_k) score_k[(int64_t)q * k + r] = o2f((uint32_t)(v[j] >> 32));
                    }
                }
            }
        }
    } else if (K <= 256) {
        for (int i = tid; i < K; i += nt) {
            const unsigned long long ki = fkey(i);
            int r = 0;
            for (int j = 0; j < K && r < k; j++) {
                const unsigned long long kj = fkey(j);
                r += (kj > ki) || (kj == ki && j < i);
            }
            if (r < k) {
                I[(int64_t)q * k + r] = cid[i];
                if (score_k) score_k[(int64_t)q * k + r] = score[i];
            }
        }
    } else if (warp == 0) {
        auto key = [&](int i) {
            return ((unsigned long long)f2o(score[i]) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)cid[i]);
        };
        const uint32_t Th = warp_select_rth_largest<32, uint32_t>([&](int i) { return f2o(score[i]); }, K, k, hist[0]);
        int gt = 0, eq = 0;
        for (int i = lane; i < K; i += 32) {
            const uint32_t h = f2o(score[i]);
            gt += h > Th;
            eq += h == Th;
        }
        gt = warp_sum_int(gt);
        eq = warp_sum_int(eq);
        unsigned long long T = (unsigned long long)Th << 32;
        if (eq > k - gt)
            T |= warp_select_rth_largest<32, uint32_t>(
                [&](int i) { return f2o(score[i]) == Th ? (0xffffffffu - (uint32_t)cid[i]) : 0u; }, K, k - gt, hist[0]);
        // keys above T first, then keys equal to T (fillers can repeat a key) up to k
        int fill = 0;
        for (int pass = 0; pass < 2; pass++) {
            for (int b = 0; b < K; b += 32) {
                const int i = b + lane;
                unsigned long long kk = 0;
                bool take = false;
                if (i < K) {
                    kk = key(i);
                    take = pass == 0 ? kk > T : kk == T;
                }
                const unsigned m = __ballot_sync(0xffffffffu, take);
                const int at = fill + __popc(m & ((1u << lane) - 1u));
                if (take && at < k) sb[at] = kk;
                fill += __popc(m);
            }
        }
        for (int i = k + lane; i < kp; i += 32) sb[i] = 0ull;
        __syncwarp();
        warp_bitonic_desc(sb, kp);
        for (int i = lane; i < k; i += 32) {
            I[(int64_t)q * k + i] = (int32_t)(0xffffffffu - (uint32_t)sb[i]);
            if (score_k) score_k[(int64_t)q * k + i] = o2f((uint32_t)(sb[i] >> 32));
        }
    }
    if (tid == 0) reads[q] = namb;
}

// One warp per (query, listed id): exact fp32 dot of the fp16 row with the query.
__global__ void exact_scores_kernel(const __half* __restrict__ H, int d, const int32_t* __restrict__ ids, int B, int k,
                                    const float* __restrict__ Q, int ldq, float* __restrict__ score) {
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= B * k) return;
    const int q = w / k;
    const int32_t id = ids[w];
    if (id < 0) {
        if (lane == 0) score[w] = kNeg;
        return;
    }
    const __half* h = H + (int64_t)id * d;
    const float* qrow = Q + (int64_t)q * ldq;
    float acc = 0.f;
    for (int c0 = lane * 8; c0 < d; c0 += 256) {
        const uint4 hv = *reinterpret_cast<const uint4*>(h + c0);
        const float4 qa = *reinterpret_cast<const float4*>(qrow + c0);
        const float4 qb = *reinterpret_cast<const float4*>(qrow + c0 + 4);
        const __half2* h2 = reinterpret_cast<const __half2*>(&hv);
        float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
        float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
        acc += f0.x * qa.x + f0.y * qa.y + f1.x * qa.z + f1.y * qa.w;
        acc += f2.x * qb.x + f2.y * qb.y + f3.x * qb.z + f3.y * qb.w;
    }
    acc = warp_sum(acc);
    if (lane == 0) score[w] = acc;
}

}  // namespace fvs

extern "C" int fvs_exact_scores(fvs_stream_t stream, const uint16_t* H, int d, const int32_t* ids, int B, int k,
                                const float* Q, int ldq, float* score) {
    FVS_CHECK_ARG(H && ids && Q && score && d > 0 && d % 8 == 0 && ldq >= d && ldq % 4 == 0 && B >= 0 && k >= 1);
    FVS_CHECK_ARG(((uintptr_t)Q & 15) == 0 && ((uintptr_t)H & 15) == 0);   // 16-byte row loads
    if (B == 0) return FVS_OK;
    const int64_t warps = (int64_t)B * k;
    fvs::exact_scores_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>((const __half*)H, d, ids, B, k, Q, ldq,
                                                                             score);
    return fvs_launch_status();
}

extern "C" int fvs_refine(fvs_stream_t stream, const uint16_t* H, int d, const int32_t* order, const int64_t* pos,
                          const float* est, const float* sd, int B, int K, float z, int k, const float* Q, int ldq,
                          int32_t* ids, int32_t* I, int32_t* reads, float* score_k) {
    FVS_CHECK_ARG(H && order && pos && est && sd && Q && ids && I && reads);
    FVS_CHECK_ARG(d > 0 && d % 8 == 0 && ldq >= d && ldq % 4 == 0 && B >= 0 && k >= 1 && K > k);
    FVS_CHECK_ARG(((uintptr_t)Q & 15) == 0 && ((uintptr_t)H & 15) == 0);   // 16-byte row loads
    if (K > 4096 || k > 256) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    int kp = 1;
    while (kp < k) kp <<= 1;
    const size_t sm = (size_t)K * 4 * 5 + 8 + (size_t)kp * 8;
    if (B < fvs_sm_count()) {
        cudaError_t e = fvs_ensure_smem((const void*)fvs::refine_kernel<1024>, sm);
        if (e != cudaSuccess) return (int)e;
        fvs::refine_kernel<1024><<<B, 1024, sm, stream>>>((const __half*)H, d, order, pos, est, sd, K, z, k, kp, Q, ldq,
                                                          ids, I, reads, score_k);
    } else {
        cudaError_t e = fvs_ensure_smem((const void*)fvs::refine_kernel<256>, sm);
        if (e != cudaSuccess) return (int)e;
        fvs::refine_kernel<256><<<B, 256, sm, stream>>>((const __half*)H, d, order, pos, est, sd, K, z, k, kp, Q, ldq,
                                                        ids, I, reads, score_k);
    }
    return fvs_launch_status();
}
