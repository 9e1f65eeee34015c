// Selection kernels: first-pass threshold, stage-1 top-K (+ delta rule), top-k merge across shards.
// One CTA per query; candidates are staged in shared memory, the k-th bound is found by a block-wide MSB-first radix
// select on order-preserving integer keys, the winners are compacted and sorted with a bitonic network.
#include <cstddef>

#include "fvs_common.cuh"

namespace fvs {

// ------------------------------------------------------------------------------------------------ threshold
// t0[q] = r-th largest of the block maxima of q's first-pass pairs (`throughput/enginei8.py:53-55`).
__global__ void threshold_kernel(const float* __restrict__ bmc, int MB, const int32_t* __restrict__ slot,
                                 const int64_t* __restrict__ probe, int nprobe, int n1, const int64_t* __restrict__ off,
                                 int r, float* __restrict__ t0) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectScratch ss;
    __shared__ int s_base[1024 + 1];
    __shared__ int s_cnt_valid;
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
    const int q = blockIdx.x, tid = threadIdx.x;
    // exclusive prefix of the first-pass cells' block counts (n1 <= 1024), one cell per thread
    {
        int nb = 0;
        for (int j = tid; j < n1; j += blockDim.x) {
            const int64_t c = probe[(int64_t)q * nprobe + j];
            const int64_t s = off[c], e = off[c + 1];
            nb = (e > s) ? (int)((e - 1) / 32 - s / 32 + 1) : 0;
            s_base[j + 1] = nb;  // counts first, scanned below
        }
        if (tid == 0) s_cnt_valid = 0;
        __syncthreads();
        if (tid == 0) {
            int acc = 0;
            s_base[0] = 0;
            for (int j = 1; j <= n1; j++) {
                acc += s_base[j];
                s_base[j] = acc;
            }
        }
        __syncthreads();
    }
    const int n = s_base[n1];
    int nvalid = 0;
    for (int j = 0; j < n1; j++) {
        const int b0 = s_base[j], nb = s_base[j + 1] - b0;
        const float* row = bmc + (int64_t)slot[(int64_t)q * n1 + j] * MB;
        for (int b = tid; b < nb; b += blockDim.x) {
            const float v = row[b];
            keys[b0 + b] = f2o(v);
            nvalid += v > -1e29f;
        }
    }
    atomicAdd(&s_cnt_valid, nvalid);
    __syncthreads();
    const int cv = s_cnt_valid;
    float res;
    if (cv >= r && r >= 1) {
        res = o2f(block_select_rth_largest<32, uint32_t>([&](int i) { return keys[i]; }, n, r, ss));
    } else if (cv > 0) {
        // fewer valid maxima than r: the smallest valid one
        __shared__ unsigned s_min;
        if (tid == 0) s_min = 0xffffffffu;
        __syncthreads();
        unsigned m = 0xffffffffu;
        for (int i = tid; i < n; i += blockDim.x)
            if (o2f(keys[i]) > -1e29f) m = min(m, keys[i]);
        atomicMin(&s_min, m);
        __syncthreads();
        res = o2f(s_min);
    } else {
        res = 1e30f;
    }
    if (tid == 0) t0[q] = res;
}

// ------------------------------------------------------------------------------------------------ stage-1 top-K
constexpr int SEL_SMEM_KEYS = 6144;  // keys staged in shared memory; larger buffers are read from global memory

__device__ __forceinline__ unsigned long long cand_key(float v, int32_t pos) {
    return ((unsigned long long)f2o(v) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)pos);
}

__global__ void select_topk_kernel(const float* __restrict__ bval, const int32_t* __restrict__ bpos,
                                   const int32_t* __restrict__ cnt, int M, int K, int Kp, int64_t* __restrict__ pos,
                                   float* __restrict__ est1, uint8_t* __restrict__ ok, int32_t* __restrict__ ncnt,
                                   float delta, int didx) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectScratch ss;
    __shared__ int s_fill, s_ncnt, s_red[32];
    unsigned long long* sb = reinterpret_cast<unsigned long long*>(smem);   // Kp sort buffer
    unsigned long long* sk = sb + Kp;                                        // staged keys (<= SEL_SMEM_KEYS)
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const int c = cnt[q];
    const int n = min(max(c, 0), M);
    const float* bv = bval + (int64_t)q * M;
    const int32_t* bp = bpos + (int64_t)q * M;
    const bool staged = n <= SEL_SMEM_KEYS;
    if (staged)
        for (int i = tid; i < n; i += nt) sk[i] = cand_key(bv[i], bp[i]);
    if (tid == 0) s_fill = 0;
    __syncthreads();
    auto key = [&](int i) { return staged ? sk[i] : cand_key(bv[i], bp[i]); };
    const unsigned long long filler = cand_key(kNeg, 0);
    if (n <= K) {
        for (int i = tid; i < Kp; i += nt) sb[i] = i < n ? key(i) : (i < K ? filler : 0ull);
        __syncthreads();
    } else {
        // K-th largest score key; ties at it are resolved by position only when they straddle the K-th place
        const uint32_t Th = block_select_rth_largest<32, uint32_t>([&](int i) { return (uint32_t)(key(i) >> 32); }, n,
                                                                   K, ss);
        int gt = 0, eq = 0;
        for (int i = tid; i < n; i += nt) {
            const uint32_t h = (uint32_t)(key(i) >> 32);
            gt += h > Th;
            eq += h == Th;
        }
        gt = block_sum_int(gt, s_red);
        eq = block_sum_int(eq, s_red);
        unsigned long long T = (unsigned long long)Th << 32;
        if (eq > K - gt) {
            const uint32_t Tl = block_select_rth_largest<32, uint32_t>(
                [&](int i) {
                    const unsigned long long k = key(i);
                    return (uint32_t)(k >> 32) == Th ? (uint32_t)k : 0u;
                },
                n, K - gt, ss);
            T |= Tl;
        }
        for (int i = tid; i < n; i += nt) {
            const unsigned long long k = key(i);
            if (k >= T) {  // keys are unique (one entry per probed row): exactly K of them
                const int slot = atomicAdd(&s_fill, 1);
                if (slot < K) sb[slot] = k;
            }
        }
        for (int i = K + tid; i < Kp; i += nt) sb[i] = 0ull;
        __syncthreads();
    }
    __shared__ float s_dval;
    if (K <= 1024) {
        // order by rank: entry i goes to place #{greater} + #{equal before it} (the fill entries are equal); no
        // sorting network
        for (int i = tid; i < K; i += nt) {
            const unsigned long long ki = sb[i];
            int rank = 0;
            for (int j = 0; j < K; j++) {
                const unsigned long long kj = sb[j];
                rank += (kj > ki) || (kj == ki && j < i);
            }
            est1[(int64_t)q * K + rank] = o2f((uint32_t)(ki >> 32));
            pos[(int64_t)q * K + rank] = (int64_t)(0xffffffffu - (uint32_t)ki);
            if (rank == didx) s_dval = o2f((uint32_t)(ki >> 32));
        }
    } else {
        block_bitonic_desc(sb, Kp);
        for (int i = tid; i < K; i += nt) {
            const unsigned long long k = sb[i];
            est1[(int64_t)q * K + i] = o2f((uint32_t)(k >> 32));
            pos[(int64_t)q * K + i] = (int64_t)(0xffffffffu - (uint32_t)k);
        }
        if (tid == 0 && ncnt != nullptr) s_dval = o2f((uint32_t)(sb[didx] >> 32));
    }
    if (tid == 0) ok[q] = (c >= K && c <= M) ? 1 : 0;
    if (ncnt != nullptr) {
        if (tid == 0) s_ncnt = 0;
        __syncthreads();
        const float thr = __fsub_rn(s_dval, delta);
        int m = 0;
        for (int i = tid; i < K; i += nt) m += o2f((uint32_t)(sb[i] >> 32)) >= thr;
        atomicAdd(&s_ncnt, m);
        __syncthreads();
        if (tid == 0) ncnt[q] = s_ncnt;
    }
}


// Register-resident variant (same contract) for M a multiple of 4 and K <= NT (NT = 256 threads, 512 for K up to 512,
// 1024 for batches smaller than the SM count): for a query with at most 8192 candidates each thread holds the order keys of 4 * W candidate scores, loaded as
// 16-byte words, where W (chunks of 4 * NT keys) is the smallest power of two that covers its cnt (more candidates:
// radix passes over global memory, select_glob_cut); the K-th largest score key is found by histogram passes below
// the keys' common prefix (block_rth_largest_reg); positions are read only for the keys at or above it, and where
// scores tied with the cut straddle it, the cut's position half comes from the block radix select over those ties;
// the K winners are placed by rank, one per thread.
constexpr int SELR_MAXK = 512;
constexpr int SELR_MAXM = 8192;
constexpr int SELR_CAND_CAP = 2048;
template <int NT>
struct SelRegShared {
    SelectScratch ss;
    RegSelectScratch rs;
    int red[32];
    int fill, ncnt;
    float dval;
    unsigned long long sb[NT];
    // candidates above the lane-maxima bound (select_rank_bound), read as 16-byte pairs
    alignas(16) unsigned long long cb[SELR_CAND_CAP + 2];
};

// the K largest (score key, position key) pairs of the n > K candidates, unordered, into sh.sb
template <int NT, int W>
__device__ __forceinline__ void select_reg_cut(const float* __restrict__ bv, const int32_t* __restrict__ bp, int n,
                                               int K, SelRegShared<NT>& sh) {
    const int tid = threadIdx.x;
    uint32_t hk[4 * W];  // 0 = no candidate (a finite score's key is never 0)
#pragma unroll
    for (int v = 0; v < W; v++) {
        const int u = tid + v * NT;
        const bool in = 4 * u < n;
        const float4 w = in ? __ldcg(reinterpret_cast<const float4*>(bv) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
        hk[4 * v + 0] = in ? f2o(w.x) : 0u;
        hk[4 * v + 1] = 4 * u + 1 < n ? f2o(w.y) : 0u;
        hk[4 * v + 2] = 4 * u + 2 < n ? f2o(w.z) : 0u;
        hk[4 * v + 3] = 4 * u + 3 < n ? f2o(w.w) : 0u;
    }
    int gt, eq;
    const uint32_t Th = block_rth_largest_reg<4 * W>(hk, K, sh.rs, &gt, &eq);
    uint32_t Tl = 0u;
    if (eq > K - gt) {
        // scores equal to the cut straddle it: the largest position keys among them fill the remaining places
        Tl = block_select_rth_largest<32, uint32_t>(
            [&](int i) { return f2o(bv[i]) == Th ? (0xffffffffu - (uint32_t)bp[i]) : 0u; }, n, K - gt, sh.ss);
    }
    const unsigned long long T = ((unsigned long long)Th << 32) | Tl;
#pragma unroll
    for (int v = 0; v < W; v++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t h = hk[4 * v + e];
            if (h != 0u && h >= Th) {
                const int i = 4 * (tid + v * NT) + e;
                const unsigned long long k = ((unsigned long long)h << 32) | (0xffffffffu - (uint32_t)bp[i]);
                if (k >= T) {  // keys are unique (one entry per probed row): exactly K of them
                    const int slot = atomicAdd(&sh.fill, 1);
                    if (slot < K) sh.sb[slot] = k;
                }
            }
        }
}

// The K <= NT largest of n > K candidates, placed in order: est1 / pos at each key's rank, the keys at sh.sb[rank],
// sh.dval at rank didx.  A lower bound on the K-th largest score key: every thread keeps the maxima of four disjoint
// subsets of its scores (one per float4 component), each a distinct candidate, so at least K candidates reach the
// K-th largest of those 4 * NT maxima (found by histogram passes over four keys per thread; 0 when fewer than K
// maxima exist).  With 4 * NT well above K the candidates at or above it number about 1.1 K; they are compacted into
// sh.cb and ranked by count on the unique (score key, position key) pairs.  Two strided passes over the scores (the
// second from L2), for any n.  Returns false, with nothing written, when more than SELR_CAND_CAP candidates reach
// the bound (many equal scores).
template <int NT>
__device__ __forceinline__ bool select_rank_bound(const float* __restrict__ bv, const int32_t* __restrict__ bp, int n,
                                                  int K, SelRegShared<NT>& sh, float* __restrict__ est1q,
                                                  int64_t* __restrict__ posq, int didx) {
    const int tid = threadIdx.x;
    const float4* bv4 = reinterpret_cast<const float4*>(bv);
    uint32_t mx[4] = {0u, 0u, 0u, 0u};  // subset maxima (0 = empty subset; a finite score's key is never 0)
    for (int u = tid; 4 * u < n; u += NT) {
        const float4 w = __ldcg(bv4 + u);
        mx[0] = max(mx[0], f2o(w.x));
        if (4 * u + 1 < n) mx[1] = max(mx[1], f2o(w.y));
        if (4 * u + 2 < n) mx[2] = max(mx[2], f2o(w.z));
        if (4 * u + 3 < n) mx[3] = max(mx[3], f2o(w.w));
    }
    const int nz = block_sum_int((int)(mx[0] != 0u) + (int)(mx[1] != 0u) + (int)(mx[2] != 0u) + (int)(mx[3] != 0u),
                                 sh.red);
    uint32_t T0 = 0u;
    if (nz >= K) {
        int gt, eq;
        T0 = block_rth_largest_reg<4>(mx, K, sh.rs, &gt, &eq);
    }
    // the scores again, the ones at or above the bound compacted with their positions
    for (int u = tid; 4 * u < n; u += NT) {
        const float4 w = __ldcg(bv4 + u);
        const float f4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t h = f2o(f4[e]);
            if (4 * u + e < n && h >= T0) {
                const int slot = atomicAdd(&sh.fill, 1);
                if (slot < SELR_CAND_CAP)
                    sh.cb[slot] = ((unsigned long long)h << 32) | (0xffffffffu - (uint32_t)bp[4 * u + e]);
            }
        }
    }
    __syncthreads();
    const int C = sh.fill;
    if (C > SELR_CAND_CAP) return false;  // uniform over the block
    if (tid == 0) sh.cb[C] = 0ull;        // pads an odd count; 0 ranks below every key
    __syncthreads();
    const ulonglong2* c2 = reinterpret_cast<const ulonglong2*>(sh.cb);
    const int C2 = (C + 1) >> 1;
    for (int i = tid; i < C; i += NT) {
        const unsigned long long ki = sh.cb[i];
        int rank = 0;
        for (int j = 0; j < C2; j++) {
            const ulonglong2 o = c2[j];
            rank += (int)(o.x > ki) + (int)(o.y > ki);
        }
        if (rank < K) {
            est1q[rank] = o2f((uint32_t)(ki >> 32));
            posq[rank] = (int64_t)(0xffffffffu - (uint32_t)ki);
            sh.sb[rank] = ki;
            if (rank == didx) sh.dval = o2f((uint32_t)(ki >> 32));
        }
    }
    return true;
}

// the same for n > SELR_MAXM candidates: keys read from global memory in every radix pass
template <int NT>
__device__ __forceinline__ void select_glob_cut(const float* __restrict__ bv, const int32_t* __restrict__ bp, int n,
                                                int K, SelRegShared<NT>& sh) {
    const int tid = threadIdx.x;
    const uint32_t Th = block_select_rth_largest<32, uint32_t>([&](int i) { return f2o(bv[i]); }, n, K, sh.ss);
    int gt = 0, eq = 0;
    for (int i = tid; i < n; i += NT) {
        const uint32_t h = f2o(bv[i]);
        gt += h > Th;
        eq += h == Th;
    }
    gt = block_sum_int(gt, sh.red);
    eq = block_sum_int(eq, sh.red);
    unsigned long long T = (unsigned long long)Th << 32;
    if (eq > K - gt)
        T |= block_select_rth_largest<32, uint32_t>(
            [&](int i) { return f2o(bv[i]) == Th ? (0xffffffffu - (uint32_t)bp[i]) : 0u; }, n, K - gt, sh.ss);
    for (int i = tid; i < n; i += NT) {
        const float v = bv[i];
        if (f2o(v) >= Th) {
            const unsigned long long k = cand_key(v, bp[i]);
            if (k >= T) {  // unique keys: exactly K of them
                const int slot = atomicAdd(&sh.fill, 1);
                if (slot < K) sh.sb[slot] = k;
            }
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(NT, 1024 / NT) select_topk_reg_kernel(
    const float* __restrict__ bval, const int32_t* __restrict__ bpos, const int32_t* __restrict__ cnt, int M, int K,
    int64_t* __restrict__ pos, float* __restrict__ est1, uint8_t* __restrict__ ok, int32_t* __restrict__ ncnt,
    float delta, int didx) {
    static_assert(offsetof(SelRegShared<NT>, cb) % 16 == 0, "the candidates are read as 16-byte pairs");
    __shared__ SelRegShared<NT> sh;
    const int q = blockIdx.x, tid = threadIdx.x;
    const int c = cnt[q];
    const int n = min(max(c, 0), M);
    const float* bv = bval + (int64_t)q * M;
    const int32_t* bp = bpos + (int64_t)q * M;
    if (tid == 0) sh.fill = 0;
    bool placed = false;  // est1 / pos / sh.sb already in rank order
    if (n <= K) {
        const unsigned long long filler = cand_key(kNeg, 0);
        for (int i = tid; i < K; i += NT) sh.sb[i] = i < n ? cand_key(bv[i], bp[i]) : filler;
    } else {
        if (K <= NT) {
            placed = select_rank_bound<NT>(bv, bp, n, K, sh, est1 + (int64_t)q * K, pos + (int64_t)q * K, didx);
            if (!placed) {
                __syncthreads();  // every thread has read the candidate count
                if (tid == 0) sh.fill = 0;
            }
        }
    }
    if (!placed && n > K) {
        const int nv = (n + 4 * NT - 1) / (4 * NT);  // uniform over the block
        if (n > SELR_MAXM || n > 32 * NT)  // more than 8 keys per thread: from global memory
            select_glob_cut<NT>(bv, bp, n, K, sh);
        else if (nv <= 1)
            select_reg_cut<NT, 1>(bv, bp, n, K, sh);
        else if (nv <= 2)
            select_reg_cut<NT, 2>(bv, bp, n, K, sh);
        else if (nv <= 4 || NT >= 512)
            select_reg_cut<NT, 4>(bv, bp, n, K, sh);
        else
            select_reg_cut<NT, 8>(bv, bp, n, K, sh);
    }
    if (K <= 128) {
        // order by rank: entry i goes to place #{greater} + #{equal before it} (the fill entries are equal); the
        // bound-and-rank selection has placed its keys already
        __syncthreads();
        for (int i = tid; i < K && !placed; i += NT) {
            const unsigned long long ki = sh.sb[i];
            int rank = 0;
            for (int j = 0; j < K; j++) {
                const unsigned long long kj = sh.sb[j];
                rank += (kj > ki) || (kj == ki && j < i);
            }
            est1[(int64_t)q * K + rank] = o2f((uint32_t)(ki >> 32));
            pos[(int64_t)q * K + rank] = (int64_t)(0xffffffffu - (uint32_t)ki);
            if (rank == didx) sh.dval = o2f((uint32_t)(ki >> 32));
        }
    } else if (!placed) {
        // larger K: a bitonic sort of the K keys (descending; real keys are unique, the fill entries are equal), padded
        // to a power of two kp <= NT with key 0, thread t holding position t: exchanges at distances below 32 go
        // through warp shuffles, the longer ones through shared memory (10 barrier pairs at kp = 512 instead of a
        // barrier after each of the 45 stages)
        int kp = 1;
        while (kp < K) kp <<= 1;
        __syncthreads();  // the selection's keys are in sh.sb
        unsigned long long v = tid < K ? sh.sb[tid] : 0ull;
        __syncthreads();
        v = block_bitonic_desc_u64(v, kp, sh.sb);
        if (tid < K) {
            est1[(int64_t)q * K + tid] = o2f((uint32_t)(v >> 32));
            pos[(int64_t)q * K + tid] = (int64_t)(0xffffffffu - (uint32_t)v);
            if (tid == didx) sh.dval = o2f((uint32_t)(v >> 32));
        }
        if (ncnt != nullptr) {  // the delta rule below reads the sorted keys from sh.sb
            __syncthreads();
            if (tid < K) sh.sb[tid] = v;
        }
    }
    if (tid == 0) ok[q] = (c >= K && c <= M) ? 1 : 0;
    if (ncnt != nullptr) {
        if (tid == 0) sh.ncnt = 0;
        __syncthreads();
        const float thr = __fsub_rn(sh.dval, delta);
        int m = 0;
        for (int i = tid; i < K; i += NT) m += o2f((uint32_t)(sh.sb[i] >> 32)) >= thr;
        atomicAdd(&sh.ncnt, m);
        __syncthreads();
        if (tid == 0) ncnt[q] = sh.ncnt;
    }
}

// threshold (same contract as threshold_kernel) for small batches: one CTA of 256 threads per query; the block
// maxima of its first-pass cells are located through a prefix of the cells' block counts and loaded all at once
// (one key per thread and step of NK), then the r-th largest valid key comes from block_rth_largest_reg.
constexpr int THR_THREADS = 256;
template <int NK>
__global__ void __launch_bounds__(THR_THREADS) threshold_reg_kernel(const float* __restrict__ bmc, int MB,
                                                                    const int32_t* __restrict__ slot,
                                                                    const int64_t* __restrict__ probe, int nprobe,
                                                                    int n1, const int64_t* __restrict__ off, int r,
                                                                    float* __restrict__ t0) {
    __shared__ int s_base[1024 + 1];
    __shared__ int s_red[32];
    __shared__ RegSelectScratch rs;
    const int q = blockIdx.x, tid = threadIdx.x;
    // block counts of the first-pass cells, then their exclusive prefix (n1 <= 1024, four cells per thread)
    int nbl[4], tot = 0;
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int j = 4 * tid + u;
        nbl[u] = 0;
        if (j < n1) {
            const int64_t c = probe[(int64_t)q * nprobe + j];
            const int64_t cs = off[c], ce = off[c + 1];
            nbl[u] = ce > cs ? (int)((ce - 1) / 32 - cs / 32 + 1) : 0;
        }
        tot += nbl[u];
    }
    const int lane = tid & 31, warp = tid >> 5;
    int incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_red[warp] = incl;
    __syncthreads();
    int before = 0, n = 0;
#pragma unroll
    for (int w = 0; w < THR_THREADS / 32; w++) {
        if (w < warp) before += s_red[w];
        n += s_red[w];
    }
    int run = before + incl - tot;
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int j = 4 * tid + u;
        if (j < n1) s_base[j] = run;
        run += nbl[u];
    }
    if (tid == 0) s_base[n1] = n;
    __syncthreads();
    // key i belongs to the cell j with s_base[j] <= i < s_base[j + 1]
    uint32_t hk[NK];  // 0 = no key or an empty block (-1e30)
    int nvalid = 0;
#pragma unroll
    for (int u = 0; u < NK; u++) {
        const int i = tid + THR_THREADS * u;
        hk[u] = 0u;
        if (i < n) {
            int lo = 0, hi = n1 - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (s_base[mid] <= i) lo = mid; else hi = mid - 1;
            }
            const float v = bmc[(int64_t)slot[(int64_t)q * n1 + lo] * MB + (i - s_base[lo])];
            if (v > -1e29f) {
                hk[u] = f2o(v);
                nvalid++;
            }
        }
    }
    nvalid = block_sum_int(nvalid, s_red);
    float res;
    if (nvalid >= r) {
        int above, equal;
        res = o2f(block_rth_largest_reg<NK>(hk, r, rs, &above, &equal));
    } else if (nvalid > 0) {
        uint32_t m = 0xffffffffu;
#pragma unroll
        for (int u = 0; u < NK; u++)
            if (hk[u] != 0u) m = min(m, hk[u]);
        m = __reduce_min_sync(0xffffffffu, m);
        if (lane == 0) s_red[warp] = (int)m;
        __syncthreads();
        m = __reduce_min_sync(0xffffffffu, lane < THR_THREADS / 32 ? (uint32_t)s_red[lane] : 0xffffffffu);
        res = o2f(m);
    } else {
        res = 1e30f;
    }
    if (tid == 0) t0[q] = res;
}

// ------------------------------------------------------------------------------------------------ warp-per-query
constexpr int WQ_WARPS = 8;  // queries per CTA in the warp-per-query kernels

// threshold (same contract as threshold_kernel), one warp per query; keys staged in the warp's shared slice
__global__ void __launch_bounds__(32 * WQ_WARPS) threshold_warp_kernel(const float* __restrict__ bmc, int MB,
                                                                      const int32_t* __restrict__ slot,
                                                                      const int64_t* __restrict__ probe, int nprobe,
                                                                      int n1, const int64_t* __restrict__ off, int B,
                                                                      int r, int cap, float* __restrict__ t0) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * WQ_WARPS + warp;
    if (q >= B) return;
    unsigned* hist = reinterpret_cast<unsigned*>(smem) + warp * (256 + cap);
    uint32_t* keys = hist + 256;
    int base = 0, nvalid = 0;
    for (int j0 = 0; j0 < n1; j0 += 32) {
        const int j = j0 + lane;
        int nb = 0;
        int64_t srow = 0;
        if (j < n1) {
            const int64_t c = probe[(int64_t)q * nprobe + j];
            const int64_t s = off[c], e = off[c + 1];
            nb = (e > s) ? (int)((e - 1) / 32 - s / 32 + 1) : 0;
            srow = (int64_t)slot[(int64_t)q * n1 + j] * MB;
        }
        int incl = nb;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        const int tot = __shfl_sync(0xffffffffu, incl, 31);
        // each lane copies its cell's block maxima (short rows), then the warp continues
        int kb = base + incl - nb;
        for (int b = 0; b < nb; b++) {
            const float v = bmc[srow + b];
            keys[kb + b] = f2o(v);
            nvalid += v > -1e29f;
        }
        base += tot;
    }
    __syncwarp();
    nvalid = warp_sum_int(nvalid);
    const int n = base;
    float res;
    if (nvalid >= r) {
        res = o2f(warp_select_rth_largest<32, uint32_t>([&](int i) { return keys[i]; }, n, r, hist));
    } else if (nvalid > 0) {
        unsigned m = 0xffffffffu;
        for (int i = lane; i < n; i += 32)
            if (o2f(keys[i]) > -1e29f) m = min(m, keys[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
        res = o2f(m);
    } else {
        res = 1e30f;
    }
    if (lane == 0) t0[q] = res;
}

// stage-1 top-K (same contract as select_topk_kernel) for K <= 512, one warp per query; keys read from global
__global__ void __launch_bounds__(32 * WQ_WARPS) select_topk_warp_kernel(
    const float* __restrict__ bval, const int32_t* __restrict__ bpos, const int32_t* __restrict__ cnt, int B, int M,
    int K, int Kp, int64_t* __restrict__ pos, float* __restrict__ est1, uint8_t* __restrict__ ok,
    int32_t* __restrict__ ncnt, float delta, int didx) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * WQ_WARPS + warp;
    if (q >= B) return;
    unsigned long long* sb = reinterpret_cast<unsigned long long*>(smem) + (int64_t)warp * (Kp + 128);
    unsigned* hist = reinterpret_cast<unsigned*>(sb + Kp);
    const int c = cnt[q];
    const int n = min(max(c, 0), M);
    const float* bv = bval + (int64_t)q * M;
    const int32_t* bp = bpos + (int64_t)q * M;
    auto key = [&](int i) { return cand_key(bv[i], bp[i]); };
    if (n <= K) {
        const unsigned long long filler = cand_key(kNeg, 0);
        for (int i = lane; i < Kp; i += 32) sb[i] = i < n ? key(i) : (i < K ? filler : 0ull);
    } else {
        const uint32_t Th =
            warp_select_rth_largest<32, uint32_t>([&](int i) { return f2o(bv[i]); }, n, K, hist);
        int gt = 0, eq = 0;
        for (int i = lane; i < n; i += 32) {
            const uint32_t h = f2o(bv[i]);
            gt += h > Th;
            eq += h == Th;
        }
        gt = warp_sum_int(gt);
        eq = warp_sum_int(eq);
        unsigned long long T = (unsigned long long)Th << 32;
        if (eq > K - gt) {
            const uint32_t Tl = warp_select_rth_largest<32, uint32_t>(
                [&](int i) { return f2o(bv[i]) == Th ? (0xffffffffu - (uint32_t)bp[i]) : 0u; }, n, K - gt, hist);
            T |= Tl;
        }
        int fill = 0;
        for (int b = 0; b < n; b += 32) {
            const int i = b + lane;
            unsigned long long k = 0;
            bool take = false;
            if (i < n) {
                k = key(i);
                take = k >= T;
            }
            const unsigned m = __ballot_sync(0xffffffffu, take);
            const int at = fill + __popc(m & ((1u << lane) - 1u));
            if (take && at < K) sb[at] = k;
            fill += __popc(m);
        }
        for (int i = K + lane; i < Kp; i += 32) sb[i] = 0ull;
    }
    __syncwarp();
    warp_bitonic_desc(sb, Kp);
    for (int i = lane; i < K; i += 32) {
        const unsigned long long k = sb[i];
        est1[(int64_t)q * K + i] = o2f((uint32_t)(k >> 32));
        pos[(int64_t)q * K + i] = (int64_t)(0xffffffffu - (uint32_t)k);
    }
    if (lane == 0) ok[q] = (c >= K && c <= M) ? 1 : 0;
    if (ncnt != nullptr) {
        const float thr = __fsub_rn(o2f((uint32_t)(sb[didx] >> 32)), delta);
        int m = 0;
        for (int i = lane; i < K; i += 32) m += o2f((uint32_t)(sb[i] >> 32)) >= thr;
        m = warp_sum_int(m);
        if (lane == 0) ncnt[q] = m;
    }
}

// ------------------------------------------------------------------------------------------------ merge
// Keys hold (score, slot): the order-preserving score bits above, 0xffffffff - slot below, so equal scores order by
// slot.  The tie order the merge needs is by the int64 global id (a -1 "no result" id included), which is read back
// through the slot; ids are never squeezed into the key.
__device__ __forceinline__ bool merge_before(float si, int64_t ii, int i, float sj, int64_t ij, int j) {
    // true when entry j ranks ahead of entry i: larger score, then smaller id, then smaller slot
    return sj > si || (sj == si && (ij < ii || (ij == ii && j < i)));
}

__global__ void merge_kernel(const int64_t* __restrict__ ids_g, const float* __restrict__ score_g, int G, int B,
                             int kin, int k, int Kp, int64_t* __restrict__ I, float* __restrict__ S) {
    extern __shared__ __align__(16) uint8_t smem[];
    unsigned long long* sb = reinterpret_cast<unsigned long long*>(smem);
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const int n = G * kin;
    auto src = [&](int i) {  // global offset of slot i of this query: shard g = i / kin, entry j = i % kin
        const int g = i / kin, j = i - g * kin;
        return ((int64_t)g * B + q) * kin + j;
    };
    if (n <= 1024) {  // place the k best by rank, no sorting network
        float* ss = reinterpret_cast<float*>(smem);
        int64_t* si = reinterpret_cast<int64_t*>(smem + 1024 * 4);
        for (int i = tid; i < n; i += nt) {
            const int64_t o = src(i);
            ss[i] = score_g[o];
            si[i] = ids_g[o];
        }
        __syncthreads();
        for (int i = tid; i < n; i += nt) {
            const float s = ss[i];
            const int64_t id = si[i];
            int rank = 0;
            for (int j = 0; j < n; j++) rank += merge_before(s, id, i, ss[j], si[j], j);
            if (rank < k) {
                I[(int64_t)q * k + rank] = id;
                if (S) S[(int64_t)q * k + rank] = s;
            }
        }
        return;
    }
    for (int i = tid; i < Kp; i += nt)
        sb[i] = i < n ? ((unsigned long long)f2o(score_g[src(i)]) << 32) | (0xffffffffu - (uint32_t)i) : 0ull;
    __syncthreads();
    block_bitonic_desc(sb, Kp);  // by score desc, slot asc
    // Only entries whose score reaches the k-th best can be kept: sorted positions [0, b), b the end of the run of
    // entries equal in score to position k-1.  Within a run of equal scores (sorted positions [a, e)) an entry's
    // final rank is a + #(run entries ahead of it by (id, slot)).
    const uint32_t sk = (uint32_t)(sb[k - 1] >> 32);
    for (int i = tid; i < n; i += nt) {
        const uint32_t si = (uint32_t)(sb[i] >> 32);
        if (si < sk) continue;
        int a = i, e = i + 1;
        while (a > 0 && (uint32_t)(sb[a - 1] >> 32) == si) a--;
        while (e < n && (uint32_t)(sb[e] >> 32) == si) e++;
        if (a >= k) continue;
        const int slot_i = (int)(0xffffffffu - (uint32_t)sb[i]);
        const int64_t id_i = ids_g[src(slot_i)];
        int rank = a;
        for (int j = a; j < e; j++) {
            if (j == i) continue;
            const int slot_j = (int)(0xffffffffu - (uint32_t)sb[j]);
            const int64_t id_j = ids_g[src(slot_j)];
            rank += id_j < id_i || (id_j == id_i && slot_j < slot_i);
        }
        if (rank < k) {
            I[(int64_t)q * k + rank] = id_i;
            if (S) S[(int64_t)q * k + rank] = o2f(si);
        }
    }
}

static int pow2_at_least(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

}  // namespace fvs

extern "C" int fvs_threshold(fvs_stream_t stream, const float* bmc, int MB, const int32_t* slot, const int64_t* probe,
                             int nprobe, int n1, const int64_t* off, int B, int r, float* t0) {
    FVS_CHECK_ARG(bmc && slot && probe && off && t0 && MB > 0 && nprobe > 0 && B >= 0);
    FVS_CHECK_ARG(n1 >= 1 && n1 <= nprobe && r >= 1);
    if (n1 > 1024) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    const int cap = n1 * MB;
    const size_t smw = (size_t)fvs::WQ_WARPS * (256 + cap) * 4;
    // one CTA per query for a small batch, and for any batch whose key capacity is too large for the warp kernel
    if ((B < fvs_sm_count() || smw > 96 * 1024) && cap <= 16 * fvs::THR_THREADS) {
        const int NK = (cap + fvs::THR_THREADS - 1) / fvs::THR_THREADS;
        if (NK <= 1)
            fvs::threshold_reg_kernel<1><<<B, fvs::THR_THREADS, 0, stream>>>(bmc, MB, slot, probe, nprobe, n1, off, r, t0);
        else if (NK <= 2)
            fvs::threshold_reg_kernel<2><<<B, fvs::THR_THREADS, 0, stream>>>(bmc, MB, slot, probe, nprobe, n1, off, r, t0);
        else if (NK <= 4)
            fvs::threshold_reg_kernel<4><<<B, fvs::THR_THREADS, 0, stream>>>(bmc, MB, slot, probe, nprobe, n1, off, r, t0);
        else if (NK <= 8)
            fvs::threshold_reg_kernel<8><<<B, fvs::THR_THREADS, 0, stream>>>(bmc, MB, slot, probe, nprobe, n1, off, r, t0);
        else
            fvs::threshold_reg_kernel<16><<<B, fvs::THR_THREADS, 0, stream>>>(bmc, MB, slot, probe, nprobe, n1, off, r,
                                                                               t0);
        return fvs_launch_status();
    }
    if (smw <= 96 * 1024) {
        cudaError_t e = fvs_ensure_smem((const void*)fvs::threshold_warp_kernel, smw);
        if (e != cudaSuccess) return (int)e;
        fvs::threshold_warp_kernel<<<(B + fvs::WQ_WARPS - 1) / fvs::WQ_WARPS, 32 * fvs::WQ_WARPS, smw, stream>>>(
            bmc, MB, slot, probe, nprobe, n1, off, B, r, cap, t0);
        return fvs_launch_status();
    }
    const size_t sm = (size_t)n1 * MB * sizeof(uint32_t);
    if (sm > 200 * 1024) return FVS_ERANGE;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::threshold_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    fvs::threshold_kernel<<<B, 256, sm, stream>>>(bmc, MB, slot, probe, nprobe, n1, off, r, t0);
    return fvs_launch_status();
}

extern "C" int fvs_select_topk(fvs_stream_t stream, const float* bval, const int32_t* bpos, const int32_t* cnt, int B,
                               int M, int K, int64_t* pos, float* est1, uint8_t* ok, int32_t* ncnt, float delta,
                               int delta_idx) {
    FVS_CHECK_ARG(bval && bpos && cnt && pos && est1 && ok && B >= 0 && M > 0 && K >= 1);
    if (ncnt) FVS_CHECK_ARG(delta_idx >= 0 && delta_idx < K);
    if (K > 4096) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    const int Kp = fvs::pow2_at_least(K);
    if (Kp <= 512 && M < 0) {  // warp-per-query variant: slower than the staged block version; kept disabled
        const size_t smw = (size_t)fvs::WQ_WARPS * (Kp + 128) * 8;
        cudaError_t e = fvs_ensure_smem((const void*)fvs::select_topk_warp_kernel, smw);
        if (e != cudaSuccess) return (int)e;
        fvs::select_topk_warp_kernel<<<(B + fvs::WQ_WARPS - 1) / fvs::WQ_WARPS, 32 * fvs::WQ_WARPS, smw, stream>>>(
            bval, bpos, cnt, B, M, K, Kp, pos, est1, ok, ncnt, delta, delta_idx);
        return fvs_launch_status();
    }
    if (K <= fvs::SELR_MAXK && M % 4 == 0 && ((uintptr_t)bval & 15) == 0) {
        if (B < fvs_sm_count())  // a small batch: 32 warps per query
            fvs::select_topk_reg_kernel<1024><<<B, 1024, 0, stream>>>(bval, bpos, cnt, M, K, pos, est1, ok, ncnt,
                                                                      delta, delta_idx);
        else if (K <= 128)
            fvs::select_topk_reg_kernel<128><<<B, 128, 0, stream>>>(bval, bpos, cnt, M, K, pos, est1, ok, ncnt, delta,
                                                                    delta_idx);
        else if (K <= 256)
            fvs::select_topk_reg_kernel<256><<<B, 256, 0, stream>>>(bval, bpos, cnt, M, K, pos, est1, ok, ncnt, delta,
                                                                    delta_idx);
        else
            fvs::select_topk_reg_kernel<512><<<B, 512, 0, stream>>>(bval, bpos, cnt, M, K, pos, est1, ok, ncnt, delta,
                                                                    delta_idx);
        return fvs_launch_status();
    }
    const size_t sm = (size_t)(Kp + fvs::SEL_SMEM_KEYS) * 8;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::select_topk_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    fvs::select_topk_kernel<<<B, 512, sm, stream>>>(bval, bpos, cnt, M, K, Kp, pos, est1, ok, ncnt, delta, delta_idx);
    return fvs_launch_status();
}

extern "C" int fvs_merge_topk(fvs_stream_t stream, const int64_t* ids_g, const float* score_g, int G, int B, int kin,
                              int k, int64_t* I, float* S) {
    FVS_CHECK_ARG(ids_g && score_g && I && G >= 1 && B >= 0 && kin >= 1 && k >= 1 && k <= G * kin);
    if (G * kin > 4096) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    const int Kp = fvs::pow2_at_least(G * kin);
    const size_t sm = G * kin <= 1024 ? (size_t)1024 * 12 : (size_t)Kp * 8;
    fvs::merge_kernel<<<B, 256, sm, stream>>>(ids_g, score_g, G, B, kin, k, Kp, I, S);
    return fvs_launch_status();
}
