// Row compaction / gather / scatter for the in-graph recompute of flagged queries (new; the reference recomputes
// flagged rows from the host, `throughput/enginei8.py:108-111`).
//
// fvs_flagged_gather: one CTA compacts the rows whose flag is 0 (stable order; the first FB of them), writes their
// indices (B for unused slots) and the number of flagged rows, then copies those rows of up to 8 arrays into dense
// [FB, row] buffers (unused slots copy row 0, so that the recompute runs on valid inputs).
// fvs_rows_scatter: copies the recomputed rows back to their places and sets their flags to 1.
#include "fvs_common.cuh"

namespace fvs {
namespace rows {

constexpr int MAXG = 8;
struct RowSet {
    int G;
    const uint8_t* src[MAXG];
    uint8_t* dst[MAXG];
    int rb[MAXG];  // bytes per row (multiple of 4)
};

__device__ __forceinline__ void copy_row(uint8_t* __restrict__ d, const uint8_t* __restrict__ s, int rb, int t, int nt) {
    if ((((uintptr_t)d | (uintptr_t)s | (uintptr_t)rb) & 15) == 0) {
        for (int i = t; i < rb / 16; i += nt) reinterpret_cast<uint4*>(d)[i] = reinterpret_cast<const uint4*>(s)[i];
    } else {
        for (int i = t; i < rb / 4; i += nt) reinterpret_cast<uint32_t*>(d)[i] = reinterpret_cast<const uint32_t*>(s)[i];
    }
}

__global__ void __launch_bounds__(1024) flagged_gather_kernel(const uint8_t* __restrict__ ok, int B, int FB,
                                                              int32_t* __restrict__ rows, int32_t* __restrict__ nflag,
                                                              RowSet rs) {
    __shared__ int wsum[32];
    __shared__ int s_rows[1024];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = blockDim.x;
    for (int i = tid; i < FB; i += nt) s_rows[i] = B;
    // chunked stable compaction: each thread owns a contiguous run of rows
    const int per = (B + nt - 1) / nt;
    const int b0 = tid * per, b1 = min(B, b0 + per);
    int local = 0;
    for (int i = b0; i < b1; i++) local += ok[i] == 0;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < (nt >> 5); w++) {
        if (w < warp) before += wsum[w];
        total += wsum[w];
    }
    int at = before + incl - local;
    for (int i = b0; i < b1 && at < FB; i++)
        if (ok[i] == 0) s_rows[at++] = i;
    __syncthreads();
    for (int i = tid; i < FB; i += nt) rows[i] = s_rows[i];
    if (tid == 0) *nflag = total;
    // one (slot, array) row per warp at a time: the copies are independent, so they are in flight together
    for (int pg = warp; pg < FB * rs.G; pg += (nt >> 5)) {
        const int slot = pg / rs.G, g = pg - slot * rs.G;
        const int r = s_rows[slot] < B ? s_rows[slot] : 0;
        copy_row(rs.dst[g] + (int64_t)slot * rs.rb[g], rs.src[g] + (int64_t)r * rs.rb[g], rs.rb[g], lane, 32);
    }
}

__global__ void __launch_bounds__(256) rows_scatter_kernel(const int32_t* __restrict__ rows, int B,
                                                           uint8_t* __restrict__ ok, RowSet rs) {
    const int slot = blockIdx.x;
    const int r = rows[slot];
    if (r < 0 || r >= B) return;
    for (int g = 0; g < rs.G; g++)
        copy_row(rs.dst[g] + (int64_t)r * rs.rb[g], rs.src[g] + (int64_t)slot * rs.rb[g], rs.rb[g], threadIdx.x,
                 blockDim.x);
    if (threadIdx.x == 0 && ok) ok[r] = 1;
}

static int make_rowset(RowSet& rs, int G, const void* const* src, void* const* dst, const int32_t* rb) {
    if (G < 0 || G > MAXG) return FVS_ERANGE;
    rs.G = G;
    for (int g = 0; g < G; g++) {
        if (!src[g] || !dst[g] || rb[g] <= 0 || rb[g] % 4 != 0) return FVS_EINVAL;
        if ((((uintptr_t)src[g]) | ((uintptr_t)dst[g])) & 3) return FVS_EINVAL;
        rs.src[g] = (const uint8_t*)src[g];
        rs.dst[g] = (uint8_t*)dst[g];
        rs.rb[g] = rb[g];
    }
    return FVS_OK;
}

}  // namespace rows
}  // namespace fvs

extern "C" int fvs_flagged_gather(fvs_stream_t stream, const uint8_t* ok, int B, int FB, int32_t* rows, int32_t* nflag,
                                  int G, const void* const* src, void* const* dst, const int32_t* row_bytes) {
    FVS_CHECK_ARG(ok && rows && nflag && B >= 1 && FB >= 1 && FB <= 1024 && (G == 0 || (src && dst && row_bytes)));
    fvs::rows::RowSet rs;
    int rc = fvs::rows::make_rowset(rs, G, src, dst, row_bytes);
    if (rc) return rc;
    fvs::rows::flagged_gather_kernel<<<1, 1024, 0, stream>>>(ok, B, FB, rows, nflag, rs);
    return fvs_launch_status();
}

extern "C" int fvs_rows_scatter(fvs_stream_t stream, const int32_t* rows, int FB, int B, uint8_t* ok, int G,
                                const void* const* src, void* const* dst, const int32_t* row_bytes) {
    FVS_CHECK_ARG(rows && B >= 1 && FB >= 1 && (G == 0 || (src && dst && row_bytes)));
    fvs::rows::RowSet rs;
    int rc = fvs::rows::make_rowset(rs, G, src, dst, row_bytes);
    if (rc) return rc;
    fvs::rows::rows_scatter_kernel<<<FB, 256, 0, stream>>>(rows, B, ok, rs);
    return fvs_launch_status();
}
