// Row compaction / gather / scatter for the in-graph recompute of flagged queries (new; the reference recomputes
// flagged rows from the host, `throughput/enginei8.py:108-111`).
//
// fvs_flagged_gather: compacts the rows whose flag is 0 (stable order; the first FB of them), writes their indices (B
// for unused slots) and the number of flagged rows, and copies those rows of up to 8 arrays into dense [FB, row]
// buffers (unused slots copy row 0, so that the recompute runs on valid inputs); one CTA per (slot, array).
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

// grid (FB, max(G, 1)): CTA (slot, g) finds the slot-th row with flag 0 (stable order) by a block-wide count over the
// flags -- every CTA repeats this small scan, so that the copies of all (slot, array) rows run in parallel -- and
// copies that row of array g; CTAs (slot, 0) write rows[slot], CTA (0, 0) the number of flagged rows.
constexpr int GATHER_THREADS = 256;
__global__ void __launch_bounds__(GATHER_THREADS) flagged_gather_kernel(const uint8_t* __restrict__ ok, int B, int FB,
                                                                        int32_t* __restrict__ rows,
                                                                        int32_t* __restrict__ nflag, RowSet rs) {
    __shared__ int wsum[GATHER_THREADS / 32];
    __shared__ int s_row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int slot = blockIdx.x, g = blockIdx.y;
    if (tid == 0) s_row = B;
    // each thread owns a contiguous run of rows; exclusive prefix of the flagged counts over the block
    const int per = (B + GATHER_THREADS - 1) / GATHER_THREADS;
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
#pragma unroll
    for (int w = 0; w < GATHER_THREADS / 32; w++) {
        if (w < warp) before += wsum[w];
        total += wsum[w];
    }
    const int start = before + incl - local;  // flagged rows before this thread's run
    if (slot >= start && slot < start + local) {
        int at = start;
        for (int i = b0; i < b1; i++)
            if (ok[i] == 0) {
                if (at == slot) s_row = i;
                at++;
            }
    }
    __syncthreads();
    const int r = s_row;  // B when fewer than slot + 1 rows are flagged
    if (tid == 0 && g == 0) {
        rows[slot] = r;
        if (slot == 0) *nflag = total;
    }
    if (g < rs.G)
        copy_row(rs.dst[g] + (int64_t)slot * rs.rb[g], rs.src[g] + (int64_t)(r < B ? r : 0) * rs.rb[g], rs.rb[g], tid,
                 GATHER_THREADS);
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
    fvs::rows::flagged_gather_kernel<<<dim3(FB, G > 0 ? G : 1), fvs::rows::GATHER_THREADS, 0, stream>>>(ok, B, FB, rows,
                                                                                                        nflag, rs);
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
