// Query codes for the int8 stage 1: z = Q @ Vr in fp32 accuracy on the tensor cores, then q8 / qs exactly as
// fvs_quantize (the reference's `throughput/enginei8.py:38`: qs = max|z| / 127, q8 = clamp(round(z / qs), +-127)).
//
// The product is a [B x d] x [d x 256] fp32 GEMM (B = 2000, d = 1536 at the headline: 1.6 GFLOP, 45 us as a SIMT
// GEMM).  Here it runs as three TF32 products per K-step (the "3xTF32" split): every fp32 x is written as
// big(x) + small(x), big = x rounded to nearest at 10 mantissa bits (exactly representable in TF32), small = x - big
// (exact, of either sign, at most half a TF32 step); z = Qbig.Vbig + Qbig.Vsmall + Qsmall.Vbig accumulated in fp32
// in TMEM.  The dropped Qsmall.Vsmall term and the TF32 conversion of the small parts are ~2^-22 relative to each
// product and of either sign; the tensor cores' fp32 accumulation over a split's K-steps is the larger term (measured
// on B = 2000, d = 1536: qs within 2.2e-6 relative of the float64 product, against ~1e-7 for a SIMT fp32 GEMM).
// Vr's two parts are made once per index (transposed, K-major); the query's parts are made in shared memory by the
// converter warps as each tile lands.
// Kernel 1 (split-K): CTA (m-tile of 128 queries, K-split ks) accumulates its K range into one 128 x 256 TMEM tile
// and writes the partial sums to part[ks][B][256].  Warp 0 issues the TMA loads (query box 128 x 32 fp32, Vr boxes
// 256 x 32 of each part, 128-byte swizzle, 2 stages), warps 1-4 split the query tile in place and later read TMEM
// back, warp 5 issues tcgen05.mma.kind::tf32 (M = 128, N = 256, K = 8; three per K-step).
// Kernel 2: one warp per query sums the KS partials in a fixed order and quantizes the row.
// Every mbarrier wait is bounded; on expiry the CTA raises `status`, drains its MMAs, frees TMEM and returns.
#include <cuda.h>

#include "fvs_common.cuh"
#include "fvs_tcgen05.cuh"

namespace fvs {
namespace proj {
using namespace fvs::tcg;

constexpr int TM = 128;   // queries per tile
constexpr int TN = 256;   // code dimensions (N)
constexpr int KC = 32;    // fp32 elements per 128-byte row of a K-chunk
constexpr int STAGES = 2;
constexpr int A_BYTES = TM * 128;   // 16 KB
constexpr int B_BYTES = TN * 128;   // 32 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;  // query (split in place), query small part, Vr big, Vr small
constexpr int BAR_OFF = STAGES * STAGE_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 8 * (3 * STAGES + 1) + 16 + 1024;
constexpr int NTHREADS = 6 * 32;
constexpr uint32_t TMEM_COLS = TN;

// instruction descriptor of tcgen05.mma.kind::tf32: f32 accumulate, TF32 A and B, both K-major
__device__ __forceinline__ uint32_t tf32_idesc(int N, int M) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// x rounded to nearest (ties away from zero) at 10 mantissa bits: a carry out of the mantissa moves into the exponent,
// which is the correct rounded value; finite inputs far from the fp32 range limits are assumed (query values)
__device__ __forceinline__ uint32_t tf32_big(uint32_t x) { return (x + 0x1000u) & 0xffffe000u; }

__global__ void __launch_bounds__(NTHREADS, 1)
    project_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap bbmap,
                   const __grid_constant__ CUtensorMap bsmap, int B, int nchunks, int chunks_per_split,
                   float* __restrict__ part, int32_t* __restrict__ status, uint32_t wait_limit) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = saddr(smem);
    auto full = [&](int s) { return sbase + BAR_OFF + 8 * s; };
    auto conv = [&](int s) { return sbase + BAR_OFF + 8 * (STAGES + s); };
    auto empty = [&](int s) { return sbase + BAR_OFF + 8 * (2 * STAGES + s); };
    const uint32_t done = sbase + BAR_OFF + 8 * (3 * STAGES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BAR_OFF + 8 * (3 * STAGES + 1));
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int m0 = blockIdx.x * TM, ks = blockIdx.y;
    const int c0 = ks * chunks_per_split, c1 = min(nchunks, c0 + chunks_per_split);
    const int nc = c1 - c0;

    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(conv(s), 4);   // the four converter warps
            mbar_init(empty(s), 1);  // MMA commit
        }
        mbar_init(done, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int nload = 0;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&qmap) : "memory");
            for (int i = 0; i < nc; i++) {
                const int s = i % STAGES;
                if (!mbar_wait(empty(s), ((i / STAGES) & 1) ^ 1, abort, wait_limit)) break;
                const uint32_t st = sbase + s * STAGE_BYTES;
                mbar_expect_tx(full(s), (uint32_t)(A_BYTES + 2 * B_BYTES));
                const int k = (c0 + i) * KC;
                tma_load_2d(st, &qmap, k, m0, full(s));
                tma_load_2d(st + 2 * A_BYTES, &bbmap, k, 0, full(s));
                tma_load_2d(st + 2 * A_BYTES + B_BYTES, &bsmap, k, 0, full(s));
                nload++;
            }
        }
    } else if (warp <= 4) {
        // ---- converters: split the landed query tile (in place: big part; beside it: small part)
        const int ct = tid - 32;
        bool ok = true;
        for (int i = 0; i < nc && ok; i++) {
            const int s = i % STAGES;
            if (!warp_wait(full(s), (i / STAGES) & 1, abort, wait_limit)) {
                ok = false;
                break;
            }
            uint4* a = reinterpret_cast<uint4*>(smem + s * STAGE_BYTES);
            uint4* as = reinterpret_cast<uint4*>(smem + s * STAGE_BYTES + A_BYTES);
#pragma unroll 4
            for (int j = ct; j < A_BYTES / 16; j += 128) {
                const uint4 v = a[j];
                const uint4 b = make_uint4(tf32_big(v.x), tf32_big(v.y), tf32_big(v.z), tf32_big(v.w));
                a[j] = b;
                as[j] = make_uint4(__float_as_uint(__uint_as_float(v.x) - __uint_as_float(b.x)),
                                   __float_as_uint(__uint_as_float(v.y) - __uint_as_float(b.y)),
                                   __float_as_uint(__uint_as_float(v.z) - __uint_as_float(b.z)),
                                   __float_as_uint(__uint_as_float(v.w) - __uint_as_float(b.w)));
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(conv(s));
        }
        // ---- epilogue: TMEM lanes 32 (warp % 4) .. + 31 = tile rows; 256 fp32 columns to the partial-sum buffer
        if (ok && warp_wait(done, 0, abort, wait_limit)) {
            tc_fence_after();
            const int r = 32 * (warp & 3) + lane;
            const int row = m0 + r;
            const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
            float* out = part + ((int64_t)ks * B + row) * TN;
            for (int j = 0; j < TN / 32; j++) {
                uint32_t acc[32];
                tmem_ld32(ta + 32 * j, acc);
                tmem_ld_wait();
                if (row < B) {
#pragma unroll
                    for (int v = 0; v < 8; v++)
                        reinterpret_cast<uint4*>(out + 32 * j)[v] =
                            make_uint4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
                }
            }
        }
    } else {
        // ---- MMA issuer: per K-step of 8, Qbig.Vbig + Qbig.Vsmall + Qsmall.Vbig
        if (lane == 0) {
            const uint32_t idesc = tf32_idesc(TN, TM);
            for (int i = 0; i < nc; i++) {
                const int s = i % STAGES;
                if (!mbar_wait(conv(s), (i / STAGES) & 1, abort, wait_limit)) break;
                tc_fence_after();
                const uint32_t st = sbase + s * STAGE_BYTES;
                const uint32_t ab = st, asm_ = st + A_BYTES, bb = st + 2 * A_BYTES, bs = bb + B_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t o = kk * 32;
                    mma_tf32(tmem, sw128_desc(ab + o), sw128_desc(bb + o), idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    mma_tf32(tmem, sw128_desc(ab + o), sw128_desc(bs + o), idesc, 1u);
                    mma_tf32(tmem, sw128_desc(asm_ + o), sw128_desc(bb + o), idesc, 1u);
                }
                mma_issued = true;
                mma_commit(empty(s));
            }
            if (mma_issued) mma_commit(done);  // the epilogue's signal; also the drain below
        }
        __syncwarp();
    }
    // drain: the last loads of every stage have landed and the MMAs have completed before the CTA exits
    if (warp == 0 && lane == 0)
        for (int u = nload - 1; u >= 0 && u >= nload - STAGES; u--) mbar_drain(full(u % STAGES), (u / STAGES) & 1);
    if (warp == 5 && lane == 0 && mma_issued) mbar_drain(done, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    if (tid == 0 && *abort && status) atomicExch(status, 1);
}

// one warp per query: z = sum of the KS partials (in order ks = 0, 1, ...), then the quantisation of quantize_kernel
__global__ void reduce_quantize_kernel(const float* __restrict__ part, int KS, int B, int8_t* __restrict__ q8,
                                       float* __restrict__ qs) {
    const int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (q >= B) return;
    float z[8];
#pragma unroll
    for (int v = 0; v < 8; v++) z[v] = 0.f;
    for (int ks = 0; ks < KS; ks++) {
        const float4* p = reinterpret_cast<const float4*>(part + ((int64_t)ks * B + q) * TN) + 2 * lane;
        const float4 a = p[0], b = p[1];
        z[0] += a.x;
        z[1] += a.y;
        z[2] += a.z;
        z[3] += a.w;
        z[4] += b.x;
        z[5] += b.y;
        z[6] += b.z;
        z[7] += b.w;
    }
    float m = 0.f;
#pragma unroll
    for (int v = 0; v < 8; v++) m = fmaxf(m, fabsf(z[v]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float sc = __fmul_rn(fmaxf(m, 1e-12f), 1.0f / 127.0f);
    uint32_t pk[2] = {0u, 0u};
#pragma unroll
    for (int v = 0; v < 8; v++) {
        const float r = fminf(fmaxf(rintf(__fdiv_rn(z[v], sc)), -127.f), 127.f);
        pk[v >> 2] |= ((uint32_t)(uint8_t)(int8_t)r) << (8 * (v & 3));
    }
    reinterpret_cast<uint2*>(q8 + (int64_t)q * TN)[lane] = make_uint2(pk[0], pk[1]);
    if (lane == 0) qs[q] = sc;
}

}  // namespace proj
}  // namespace fvs

extern "C" int fvs_project_quantize(fvs_stream_t stream, const float* Q, int B, int d, int ldq, const float* vt_big,
                                    const float* vt_small, int R, int8_t* q8, float* qs, float* part, int ks_max,
                                    int32_t* status) {
    using namespace fvs::proj;
    FVS_CHECK_ARG(Q && vt_big && vt_small && q8 && qs && part && B >= 0 && d > 0 && ldq >= d && ks_max >= 1);
    FVS_CHECK_ARG(R == TN && d % 4 == 0 && ldq % 4 == 0);
    FVS_CHECK_ARG((((uintptr_t)Q | (uintptr_t)vt_big | (uintptr_t)vt_small | (uintptr_t)part) & 15) == 0);
    if (B == 0) return FVS_OK;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    const int mt = (B + TM - 1) / TM;
    const int nchunks = (d + KC - 1) / KC;
    // K-splits: enough CTAs for the SMs, at most ks_max (the partial buffer holds ks_max x B x 256 floats)
    int KS = fvs_sm_count() / mt;
    KS = KS < 1 ? 1 : KS > nchunks ? nchunks : KS;
    KS = KS > ks_max ? ks_max : KS;
    const int per = (nchunks + KS - 1) / KS;
    KS = (nchunks + per - 1) / per;
    CUtensorMap qmap, bbmap, bsmap;
    const cuuint32_t estr[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)B};
        const cuuint64_t strides[1] = {(cuuint64_t)ldq * 4};
        const cuuint32_t box[2] = {KC, TM};
        if (enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)Q, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return FVS_EINVAL;
    }
    for (int which = 0; which < 2; which++) {
        const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)TN};
        const cuuint64_t strides[1] = {(cuuint64_t)d * 4};
        const cuuint32_t box[2] = {KC, TN};
        if (enc(which ? &bsmap : &bbmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)(which ? vt_small : vt_big), dims,
                strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return FVS_EINVAL;
    }
    cudaError_t e = fvs_ensure_smem((const void*)project_kernel, SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    project_kernel<<<dim3(mt, KS), NTHREADS, SMEM_BYTES, stream>>>(qmap, bbmap, bsmap, B, nchunks, per, part, status,
                                                                   pipeline_wait_limit());
    reduce_quantize_kernel<<<(B + 7) / 8, 256, 0, stream>>>(part, KS, B, q8, qs);
    return fvs_launch_status();
}
