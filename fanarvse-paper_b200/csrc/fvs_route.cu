// Routing and pairing: the probe list of each query and the cell-sorted pair list (CSR) the scan consumes.
//
// fvs_route_topk replaces `QM.topk(nprobe, 1).indices` on the fp16 routing product (`throughput/enginei8.py:67-68`):
// one CTA per query selects the nprobe largest 32-bit keys (ordered fp16 score << 16 | (65535 - cell)), so the order
// is (score desc, cell asc) -- the reference leaves the order of equal scores to torch.topk.  Up to 16384 cells the
// keys stay in registers and the cut is found by a bitwise binary search (route_topk_reg_kernel); beyond that they are
// staged in shared memory for a block radix select (route_topk_kernel).
// fvs_pairs replaces `pairs_fast` (`throughput/enginei8.py:11-16`): a counting sort of the (query, cell) pairs by cell
// (histogram, exclusive scan, atomic scatter).  Within a cell the query order is the scatter order; nothing downstream
// depends on it (block maxima are addressed through `slot`, emitted sets are sets).
#include "fvs_common.cuh"

namespace fvs {

__device__ __forceinline__ uint32_t h2o(uint16_t u) { return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u); }

#ifndef FVS_RT_THREADS
#define FVS_RT_THREADS 512
#endif
constexpr int RT_THREADS = FVS_RT_THREADS;

__global__ void __launch_bounds__(RT_THREADS) route_topk_kernel(const uint16_t* __restrict__ QM, int NC, int nprobe,
                                                                int kp, int64_t* __restrict__ probe) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectScratch ss;
    __shared__ int s_fill;
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem);        // NC
    unsigned long long* sb = reinterpret_cast<unsigned long long*>(keys + NC + (NC & 1));  // kp (as 64-bit slots)
    const int q = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const uint16_t* row = QM + (int64_t)q * NC;
    for (int c = tid; c < NC; c += nt) keys[c] = (h2o(row[c]) << 16) | (uint32_t)(0xffff - c);
    if (tid == 0) s_fill = 0;
    __syncthreads();
    // the nprobe-th largest score (16-bit order key, two radix passes); the cell half of the key only where scores
    // tied with it straddle the cut
    const uint32_t Th = block_select_rth_largest<16, uint32_t>([&](int i) { return keys[i] >> 16; }, NC, nprobe, ss);
    int gt = 0, eq = 0;
    for (int c = tid; c < NC; c += nt) {
        gt += (keys[c] >> 16) > Th;
        eq += (keys[c] >> 16) == Th;
    }
    __shared__ int s_red[32];
    gt = block_sum_int(gt, s_red);
    eq = block_sum_int(eq, s_red);
    uint32_t T = Th << 16;
    if (eq > nprobe - gt)
        T |= block_select_rth_largest<16, uint32_t>(
            [&](int i) { return (keys[i] >> 16) == Th ? (keys[i] & 0xffffu) : 0u; }, NC, nprobe - gt, ss);
    for (int c = tid; c < NC; c += nt)
        if (keys[c] >= T) {
            const int slot = atomicAdd(&s_fill, 1);
            if (slot < nprobe) sb[slot] = keys[c];
        }
    __syncthreads();
    if (nprobe <= 1024) {
        // order by rank (keys are unique): entry i goes to place #{keys greater than it}; no sorting network
        for (int i = tid; i < nprobe; i += nt) {
            const unsigned long long ki = sb[i];
            int rank = 0;
            for (int j = 0; j < nprobe; j++) rank += sb[j] > ki;
            probe[(int64_t)q * nprobe + rank] = 0xffff - (int64_t)(ki & 0xffffu);
        }
    } else {
        for (int i = nprobe + tid; i < kp; i += nt) sb[i] = 0ull;
        __syncthreads();
        block_bitonic_desc(sb, kp);
        for (int i = tid; i < nprobe; i += nt) probe[(int64_t)q * nprobe + i] = 0xffff - (int64_t)(sb[i] & 0xffffu);
    }
}

// Register-resident variant for NC <= 256 * 8 * V (NC a multiple of 8, 16-byte aligned rows) and nprobe <= 512: each
// of 256 threads holds 8 * V keys loaded as 16-byte words, the nprobe-th largest key is found by histogram passes
// below the keys' common prefix (block_rth_largest_reg), and the selected keys are ordered by rank.  Same keys, same
// result as route_topk_kernel.
constexpr int RTR_THREADS = 256;
constexpr int RTR_MAXP = 512;
template <int V>
__global__ void __launch_bounds__(RTR_THREADS) route_topk_reg_kernel(const uint16_t* __restrict__ QM, int NC,
                                                                     int nprobe, int64_t* __restrict__ probe) {
    __shared__ RegSelectScratch rs;
    __shared__ int s_fill;
    __shared__ uint32_t s_sel[RTR_MAXP];
    const int q = blockIdx.x, tid = threadIdx.x;
    const uint4* row = reinterpret_cast<const uint4*>(QM + (int64_t)q * NC);
    uint32_t key[8 * V];  // 0 = no cell (real keys are >= 1: a score's order half is 0 only for the NaN 0xffff)
#pragma unroll
    for (int v = 0; v < V; v++) {
        const int u = tid + v * RTR_THREADS;
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
    int above, equal;
    const uint32_t T = block_rth_largest_reg<8 * V>(key, nprobe, rs, &above, &equal);  // keys are unique
#pragma unroll
    for (int i = 0; i < 8 * V; i++)
        if (key[i] != 0u && key[i] >= T) {
            const int slot = atomicAdd(&s_fill, 1);
            if (slot < nprobe) s_sel[slot] = key[i];
        }
    __syncthreads();
    // order by rank (keys are unique): entry i goes to place #{keys greater than it}
    for (int i = tid; i < nprobe; i += RTR_THREADS) {
        const uint32_t ki = s_sel[i];
        int rank = 0;
        for (int j = 0; j < nprobe; j++) rank += s_sel[j] > ki;
        probe[(int64_t)q * nprobe + rank] = 0xffff - (int64_t)(ki & 0xffffu);
    }
}

__global__ void pair_hist_kernel(const int64_t* __restrict__ probe, int B, int nprobe, int ncols,
                                 int32_t* __restrict__ ccnt) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * ncols) return;
    const int q = (int)(i / ncols), j = (int)(i - (int64_t)q * ncols);
    atomicAdd(ccnt + probe[(int64_t)q * nprobe + j], 1);
}

// both counts of fvs_pairs_split: all nprobe columns, and the first n1 of them
__global__ void pair_hist_split_kernel(const int64_t* __restrict__ probe, int B, int nprobe, int n1,
                                       int32_t* __restrict__ ccnt, int32_t* __restrict__ ccnt1) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * nprobe) return;
    const int j = (int)(i % nprobe);
    const int64_t c = probe[i];
    atomicAdd(ccnt + c, 1);
    if (j < n1) atomicAdd(ccnt1 + c, 1);
}

// columns < n1 fill the front of their cell's range, the others the back
__global__ void pair_scatter_split_kernel(const int64_t* __restrict__ probe, int B, int nprobe, int n1, int NC,
                                          const __half* __restrict__ QM, const float* __restrict__ mnorm,
                                          const int32_t* __restrict__ coff, const int32_t* __restrict__ ccnt1,
                                          int32_t* __restrict__ cur1, int32_t* __restrict__ cur2,
                                          int32_t* __restrict__ qid, float* __restrict__ qcp,
                                          int32_t* __restrict__ slot) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * nprobe) return;
    const int q = (int)(i / nprobe), j = (int)(i - (int64_t)q * nprobe);
    const int c = (int)probe[i];
    int pos;
    if (j < n1) {
        pos = coff[c] + atomicAdd(cur1 + c, 1);
        if (slot) slot[(int64_t)q * n1 + j] = pos;
    } else {
        pos = coff[c] + ccnt1[c] + atomicAdd(cur2 + c, 1);
    }
    qid[pos] = q;
    const float v = __half2float(QM[(int64_t)q * NC + c]);
    qcp[pos] = mnorm ? __fmul_rn(v, mnorm[c]) : v;
}

// exclusive scan of NC counts in one CTA of 1024 threads
__global__ void __launch_bounds__(1024) pair_scan_kernel(const int32_t* __restrict__ ccnt, int NC,
                                                         int32_t* __restrict__ coff) {
    __shared__ int wsum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (NC + 1023) / 1024;
    const int b0 = tid * per;
    int local = 0;
    for (int i = 0; i < per; i++)
        if (b0 + i < NC) local += ccnt[b0 + i];
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
            coff[b0 + i] = run;
            run += ccnt[b0 + i];
        }
}

__global__ void pair_scatter_kernel(const int64_t* __restrict__ probe, int B, int nprobe, int ncols, int NC,
                                    const __half* __restrict__ QM, const float* __restrict__ mnorm,
                                    const int32_t* __restrict__ coff, int32_t* __restrict__ cursor,
                                    int32_t* __restrict__ qid, float* __restrict__ qcp, int32_t* __restrict__ slot) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * ncols) return;
    const int q = (int)(i / ncols), j = (int)(i - (int64_t)q * ncols);
    const int c = (int)probe[(int64_t)q * nprobe + j];
    const int pos = coff[c] + atomicAdd(cursor + c, 1);
    qid[pos] = q;
    const float v = __half2float(QM[(int64_t)q * NC + c]);
    qcp[pos] = mnorm ? __fmul_rn(v, mnorm[c]) : v;
    if (slot) slot[i] = pos;
}

// q8, qs from the projected queries z [B, ldz] (`throughput/enginei8.py:38`): qs = max(max|z|, 1e-12) / 127,
// q8 = clamp(round_half_even(z / qs), -127, 127); one warp per query.  The division by the constant 127 is evaluated as
// torch evaluates a tensor-by-scalar division on the GPU, a multiplication by the fp32 reciprocal; z / qs is a true
// division.
__global__ void quantize_kernel(const float* __restrict__ z, int B, int R, int ldz, int8_t* __restrict__ q8,
                                float* __restrict__ qs) {
    const int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (q >= B) return;
    const float* zr = z + (int64_t)q * ldz;
    float m = 0.f;
    for (int i = lane; i < R; i += 32) m = fmaxf(m, fabsf(zr[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float sc = __fmul_rn(fmaxf(m, 1e-12f), 1.0f / 127.0f);
    for (int i = lane; i < R; i += 32) {
        const float v = rintf(__fdiv_rn(zr[i], sc));
        q8[(int64_t)q * R + i] = (int8_t)fminf(fmaxf(v, -127.f), 127.f);
    }
    if (lane == 0) qs[q] = sc;
}

// One warp per query row: the row is read once as float4 (16-byte loads), written back as fp16 (round to nearest
// even, as a tensor's .half() conversion), and dotted with c in fp32 (per-lane partial sums, then a warp reduction).
__global__ void query_prep_kernel(const float* __restrict__ Q, int B, int d, int ldq, const float* __restrict__ c,
                                  __half* __restrict__ Qh, float* __restrict__ qc) {
    const int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (q >= B) return;
    const float4* row = reinterpret_cast<const float4*>(Q + (int64_t)q * ldq);
    const float4* cv = reinterpret_cast<const float4*>(c);
    uint2* out = reinterpret_cast<uint2*>(Qh + (int64_t)q * d);
    float acc = 0.f;
    const int nv = d / 4;
    // four 16-byte slices of the row in flight per lane (the lane's slices are summed in the same order as one at a time)
    for (int i0 = lane; i0 < nv; i0 += 4 * 32) {
        float4 x[4], y[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = i0 + 32 * u;
            if (i < nv) {
                x[u] = row[i];
                y[u] = cv[i];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = i0 + 32 * u;
            if (i >= nv) break;
            acc = fmaf(x[u].x, y[u].x, acc);
            acc = fmaf(x[u].y, y[u].y, acc);
            acc = fmaf(x[u].z, y[u].z, acc);
            acc = fmaf(x[u].w, y[u].w, acc);
            const __half2 lo = __floats2half2_rn(x[u].x, x[u].y), hi = __floats2half2_rn(x[u].z, x[u].w);
            out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
        }
    }
    acc = warp_sum(acc);
    if (lane == 0 && qc) qc[q] = acc;
}

}  // namespace fvs

extern "C" int fvs_query_prep(fvs_stream_t stream, const float* Q, int B, int d, int ldq, const float* c, uint16_t* Qh,
                              float* qc) {
    FVS_CHECK_ARG(Q && c && Qh && B >= 0 && d > 0 && d % 4 == 0 && ldq >= d && ldq % 4 == 0);
    FVS_CHECK_ARG(((uintptr_t)Q & 15) == 0 && ((uintptr_t)c & 15) == 0 && ((uintptr_t)Qh & 7) == 0);
    if (B == 0) return FVS_OK;
    fvs::query_prep_kernel<<<(B + 7) / 8, 256, 0, stream>>>(Q, B, d, ldq, c, (__half*)Qh, qc);
    return fvs_launch_status();
}

extern "C" int fvs_quantize(fvs_stream_t stream, const float* z, int B, int R, int ldz, int8_t* q8, float* qs) {
    FVS_CHECK_ARG(z && q8 && qs && B >= 0 && R > 0 && ldz >= R);
    if (B == 0) return FVS_OK;
    fvs::quantize_kernel<<<(B + 7) / 8, 256, 0, stream>>>(z, B, R, ldz, q8, qs);
    return fvs_launch_status();
}

extern "C" int fvs_route_topk(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int64_t* probe) {
    FVS_CHECK_ARG(QM && probe && B >= 0 && NC > 0 && nprobe >= 1 && nprobe <= NC);
    if (NC > 65535 || nprobe > 4096) return FVS_ERANGE;
    if (B == 0) return FVS_OK;
    if (NC % 8 == 0 && ((uintptr_t)QM & 15) == 0 && nprobe <= fvs::RTR_MAXP) {
        const int V = (NC + fvs::RTR_THREADS * 8 - 1) / (fvs::RTR_THREADS * 8);
        if (V <= 8) {
            const int Vp = V <= 1 ? 1 : V <= 2 ? 2 : V <= 4 ? 4 : 8;
            if (Vp == 1) fvs::route_topk_reg_kernel<1><<<B, fvs::RTR_THREADS, 0, stream>>>(QM, NC, nprobe, probe);
            if (Vp == 2) fvs::route_topk_reg_kernel<2><<<B, fvs::RTR_THREADS, 0, stream>>>(QM, NC, nprobe, probe);
            if (Vp == 4) fvs::route_topk_reg_kernel<4><<<B, fvs::RTR_THREADS, 0, stream>>>(QM, NC, nprobe, probe);
            if (Vp == 8) fvs::route_topk_reg_kernel<8><<<B, fvs::RTR_THREADS, 0, stream>>>(QM, NC, nprobe, probe);
            return fvs_launch_status();
        }
    }
    int kp = 1;
    while (kp < nprobe) kp <<= 1;
    const size_t sm = (size_t)(NC + (NC & 1)) * 4 + (size_t)kp * 8;
    if (sm > 200 * 1024) return FVS_ERANGE;
    cudaError_t e = fvs_ensure_smem((const void*)fvs::route_topk_kernel, sm);
    if (e != cudaSuccess) return (int)e;
    fvs::route_topk_kernel<<<B, fvs::RT_THREADS, sm, stream>>>(QM, NC, nprobe, kp, probe);
    return fvs_launch_status();
}

extern "C" int fvs_pairs(fvs_stream_t stream, const int64_t* probe, int B, int nprobe, int ncols, int NC,
                         const uint16_t* QM, const float* mnorm, int32_t* qid, int32_t* coff, int32_t* ccnt,
                         float* qcp, int32_t* slot, int32_t* work) {
    FVS_CHECK_ARG(probe && QM && qid && coff && ccnt && qcp && work && B >= 0 && NC > 0);
    FVS_CHECK_ARG(ncols >= 1 && ncols <= nprobe);
    cudaError_t e = cudaMemsetAsync(ccnt, 0, (size_t)NC * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(work, 0, (size_t)NC * 4, stream);
    if (e != cudaSuccess) return (int)e;
    const int64_t n = (int64_t)B * ncols;
    const unsigned grid = (unsigned)((n + 255) / 256);
    if (n > 0) fvs::pair_hist_kernel<<<grid, 256, 0, stream>>>(probe, B, nprobe, ncols, ccnt);
    fvs::pair_scan_kernel<<<1, 1024, 0, stream>>>(ccnt, NC, coff);
    if (n > 0)
        fvs::pair_scatter_kernel<<<grid, 256, 0, stream>>>(probe, B, nprobe, ncols, NC, (const __half*)QM, mnorm, coff,
                                                           work, qid, qcp, slot);
    return fvs_launch_status();
}

extern "C" int fvs_pairs_split(fvs_stream_t stream, const int64_t* probe, int B, int nprobe, int n1, int NC,
                               const uint16_t* QM, const float* mnorm, int32_t* qid, int32_t* coff, int32_t* ccnt,
                               int32_t* ccnt1, float* qcp, int32_t* slot, int32_t* work) {
    FVS_CHECK_ARG(probe && QM && qid && coff && ccnt && ccnt1 && qcp && work && B >= 0 && NC > 0);
    FVS_CHECK_ARG(n1 >= 1 && n1 <= nprobe);
    cudaError_t e = cudaMemsetAsync(ccnt, 0, (size_t)NC * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ccnt1, 0, (size_t)NC * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(work, 0, (size_t)NC * 8, stream);
    if (e != cudaSuccess) return (int)e;
    const int64_t n = (int64_t)B * nprobe;
    const unsigned grid = (unsigned)((n + 255) / 256);
    if (n > 0) fvs::pair_hist_split_kernel<<<grid, 256, 0, stream>>>(probe, B, nprobe, n1, ccnt, ccnt1);
    fvs::pair_scan_kernel<<<1, 1024, 0, stream>>>(ccnt, NC, coff);
    if (n > 0)
        fvs::pair_scatter_split_kernel<<<grid, 256, 0, stream>>>(probe, B, nprobe, n1, NC, (const __half*)QM, mnorm,
                                                                 coff, ccnt1, work, work + NC, qid, qcp, slot);
    return fvs_launch_status();
}

// ------------------------------------------------------------------------------------------------ allocation-free
// fvs_pairs_noalloc: fvs_pairs for callers that cannot allocate device memory (the per-cell cursors live in this
// file-scope array instead of a caller-provided `work` buffer).  The array is allocated once per GPU when the library
// is loaded there and stays allocated until the process exits.
static __device__ __align__(256) int32_t g_pairs_cursor[FVS_PAIRS_NOALLOC_MAX_CELLS];

// Device address of g_pairs_cursor on the current device, looked up once per device.  The host-side symbol is only a
// handle: a kernel must be given the address cudaGetSymbolAddress returns for the device it runs on.
static cudaError_t pairs_cursor_address(int32_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    constexpr int MAXDEV = 256;
    static std::mutex mu;
    static int32_t* addr[MAXDEV] = {};
    if (dev < 0 || dev >= MAXDEV) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_pairs_cursor);
        if (e != cudaSuccess) return e;
        addr[dev] = reinterpret_cast<int32_t*>(ptr);
    }
    *out = addr[dev];
    return cudaSuccess;
}

extern "C" int fvs_pairs_noalloc(fvs_stream_t stream, const int64_t* probe, int B, int nprobe, int ncols, int NC,
                                 const uint16_t* QM, const float* mnorm, int32_t* qid, int32_t* coff, int32_t* ccnt,
                                 float* qcp, int32_t* slot) {
    FVS_CHECK_ARG(probe && QM && qid && coff && ccnt && qcp && B >= 0 && NC > 0);
    FVS_CHECK_ARG(ncols >= 1 && ncols <= nprobe);
    if (NC > FVS_PAIRS_NOALLOC_MAX_CELLS) return FVS_ERANGE;
    int32_t* cursor = nullptr;
    cudaError_t e = pairs_cursor_address(&cursor);
    if (e != cudaSuccess) return (int)e;
    // the array keeps the previous call's cursors: clear the part this call uses
    e = cudaMemsetAsync(ccnt, 0, (size_t)NC * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(cursor, 0, (size_t)NC * 4, stream);
    if (e != cudaSuccess) return (int)e;
    const int64_t n = (int64_t)B * ncols;
    const unsigned grid = (unsigned)((n + 255) / 256);
    if (n > 0) fvs::pair_hist_kernel<<<grid, 256, 0, stream>>>(probe, B, nprobe, ncols, ccnt);
    fvs::pair_scan_kernel<<<1, 1024, 0, stream>>>(ccnt, NC, coff);
    if (n > 0)
        fvs::pair_scatter_kernel<<<grid, 256, 0, stream>>>(probe, B, nprobe, ncols, NC, (const __half*)QM, mnorm, coff,
                                                           cursor, qid, qcp, slot);
    return fvs_launch_status();
}
