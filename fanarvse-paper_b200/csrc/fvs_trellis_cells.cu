// Default-engine stage-1 scan (cell-residual trellis code) on the 5th-generation tensor cores (tcgen05, sm_100a),
// cell-major.
//
// Same contract and arithmetic as fvs_trellis_scan modes 0 / 1 (the reference's `_first_compact_s` / `_emit_loop_s`
// with the decoder `_decode_tile2`, `src/s1cell.py:121-154`, `src/decode2.py:5-17`):
//   value_j = fp16(tab[state_j]),  state_j = ((w[j/32] << 32 | w[j/32+1]) >> (64 - L - j%32)) & (2^L - 1),
//   est = scale1[n] * dot(fp16 q', value) + qcp   (dot accumulated in fp32, product and sum rounded separately),
// then block maxima per 32-row block (mode 0, first pass) or the threshold emit est >= t0[q] (mode 1).
// Work items are (cell part, group of up to QN = 128 of its queries), handed out dynamically (cells largest first;
// list entries `cell | part << 16`, part p covering tiles 8p .. 8p+7 of the cell, so that several CTAs share a large
// cell).  An item's queries are gathered once and held while the part's 128-row tiles pass; each tile x item is ONE sequence of
// 16 tcgen05.mma.kind::f16 (M = 128 rows, N = the item's queries rounded up to 16, K = 16 each), since the issue cost
// of an MMA hardly depends on N.  The code tile is not copied but decoded in the CTA: two sets of four decode warps,
// one tile row per lane, read the row's words (prefetched one tile ahead) and write its fp16 values, two per lookup of
// a table of fp16 value pairs indexed by (L+1)-bit windows, straight into the canonical K-major 128 B-swizzled layout
// the MMA reads; set 0 writes values 0-127 of every row (words 0-4), set 1 values 128-255 (words 4-8).  The tile moves
// in K-chunks of 64 values through a ring of AC chunk slots, so decode and MMAs overlap chunk by chunk.
// Warp roles (768 threads):
//   warps 0-7   : decode (warps 0-3 chunks 0-1, warps 4-7 chunks 2-3 of every tile)
//   warp 8      : TMEM allocation; lane 0 issues the MMAs per chunk, commits a chunk slot back once its MMAs are done
//                 and an accumulator after the tile's last chunk
//   warps 9-10  : gather, items alternating: fp16 query rows picked by qid, copied with cp.async (an item's rows in
//                 flight at once) into the swizzled layout; column metadata (qid, pair constant, threshold)
//   warp 11     : lane 0 takes cell parts (atomicAdd on sched[0], cell fields loaded ahead in stages) and publishes the
//                 work items in a ring of I_STAGES slots
//   warps 12-23 : three epilogue warpgroups, tiles alternating between them
// The last CTA to finish resets sched[0..1].  Every mbarrier wait is bounded; on expiry the CTA raises `status`,
// drains the MMAs it issued, frees TMEM and returns.
#include <cuda.h>

#include "fvs_common.cuh"
#include "fvs_tcgen05.cuh"

namespace fvs {
namespace tcells {
using namespace fvs::tcg;

constexpr int TILE_ROWS = 128;
constexpr int QN = 128;     // queries per work item (one B operand, one accumulator per tile)
constexpr int R = 256;      // decoded values per row
constexpr int KCH = 4;      // K-chunks of 64 fp16 values (128 B per row) per tile
constexpr int DEC_SETS = 2;  // decode warp sets, each decoding KCH / DEC_SETS chunks of every tile
constexpr int SWORDS = 2 * (KCH / DEC_SETS) + 1;  // words a lane of a set reads for its row (from word 4 * set)
constexpr int AC = 5;       // chunk slots
constexpr int B_STAGES = 2;
constexpr int T_STAGES = 4;
constexpr int I_STAGES = 8;
constexpr int MS = 4;       // column-metadata slots (one per item, held until the item's last tile is done)
constexpr int EPI_GROUPS = 3;
constexpr int GATHER_WARPS = 2;
constexpr int DEC_WARPS = 8;
constexpr int MAX_L = 10;
constexpr int W_MMA = 8, W_GATHER = 9, W_PROD = 11, W_EPI = 12;
constexpr int NWARPS = W_EPI + 4 * EPI_GROUPS;
constexpr int NTHREADS = 32 * NWARPS;
constexpr uint32_t TMEM_COLS = T_STAGES * QN;
static_assert(W_EPI % 4 == 0, "epilogue warpgroups start on a TMEM lane quarter");
static_assert(DEC_WARPS / DEC_SETS * 32 == TILE_ROWS, "one lane of each decode set per tile row");
static_assert(W_MMA == DEC_WARPS, "decode warps first");
static_assert(B_STAGES == GATHER_WARPS, "gather warp g fills B stage g");
static_assert(TMEM_COLS <= 512, "tensor memory columns");

struct Item {
    int cell, cs, ce, first, ntiles, qoff, nq, live;  // live == 0: no more work
};

// shared-memory carve-up (offsets from a 1024-byte aligned base)
constexpr int CH_BYTES = TILE_ROWS * 128;  // one K-chunk of a decoded tile
constexpr int B_BYTES = KCH * QN * 128;    // one item's queries: 4 K-chunks x 16 KB
constexpr int A_OFF = 0;
constexpr int B_OFF = A_OFF + AC * CH_BYTES;
constexpr int META_OFF = B_OFF + B_STAGES * B_BYTES;  // per item slot: qid, qcp, t0 of QN columns
constexpr int META_W = 3 * QN * 4;
constexpr int COL_OFF = META_OFF + MS * META_W;               // per epilogue warp: 32 column masks + 32 bases
constexpr int MCNT_OFF = COL_OFF + 4 * EPI_GROUPS * 64 * 4;   // per metadata slot: epilogue warps done with it
constexpr int TAB_OFF = MCNT_OFF + MS * 4;                    // pair table: 2^(L+1) fp16 value pairs
constexpr int ITEM_OFF = TAB_OFF + (2 << MAX_L) * 4;
constexpr int BAR_OFF = ITEM_OFF + I_STAGES * (int)sizeof(Item);
constexpr int NBAR = 2 * AC + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + 2 * MS + 1;
constexpr int MISC_OFF = BAR_OFF + NBAR * 8;  // tmem base, abort flag
constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
// MMA thread, gather warps, decode warps, epilogue warps
constexpr uint32_t I_CONSUMERS = 1 + GATHER_WARPS + DEC_WARPS + 4 * EPI_GROUPS;

struct Params {
    const __half* Qh;
    const uint32_t* words;
    const float* tab;
    const __half* scale1;
    const int32_t* qid;
    const int32_t* coff;
    const int32_t* ccnt;
    const float* qcp;
    const int32_t* list;
    const int32_t* nlist;
    const int64_t* off;
    const float* t0;
    int32_t* cnt;
    float* bval;
    int32_t* bpos;
    float* bmc;
    int32_t* sched;
    int32_t* status;
    int M, MB, W, L;
    uint32_t wait_limit;
};

// instruction descriptor of tcgen05.mma.kind::f16: f32 accumulate, fp16 A and B, both K-major, M rows, N columns
__device__ __forceinline__ uint32_t f16_idesc(int N, int M = 128) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ uint32_t transpose32(uint32_t x) {
    const int lane = threadIdx.x & 31;
    const uint32_t ms[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
    for (int k = 0; k < 5; k++) {
        const int j = 16 >> k;
        const uint32_t m = ms[k];
        const uint32_t y = __shfl_xor_sync(0xffffffffu, x, j);
        x = (lane & j) ? ((x & ~m) | ((y >> j) & m)) : ((x & m) | ((y & m) << j));
    }
    return x;
}

__device__ __forceinline__ uint32_t select32(const uint32_t (&a)[32], int jj) {
    uint32_t t16[16], t8[8], t4[4], t2[2];
#pragma unroll
    for (int i = 0; i < 16; i++) t16[i] = (jj & 1) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
    for (int i = 0; i < 8; i++) t8[i] = (jj & 2) ? t16[2 * i + 1] : t16[2 * i];
#pragma unroll
    for (int i = 0; i < 4; i++) t4[i] = (jj & 4) ? t8[2 * i + 1] : t8[2 * i];
#pragma unroll
    for (int i = 0; i < 2; i++) t2[i] = (jj & 8) ? t4[2 * i + 1] : t4[2 * i];
    return (jj & 16) ? t2[1] : t2[0];
}

// the fields of one cell the producer needs, loaded in stages so that no load is waited on in the iteration that
// issues it
struct CellInfo {
    int cell, cs, ce, qn, qoff, part;
};

template <int MODE>
__global__ void __launch_bounds__(NTHREADS, 1) trellis_cells_kernel(Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = saddr(smem);
    auto bar = [&](int i) { return sbase + BAR_OFF + 8 * i; };
    auto c_full = [&](int s) { return bar(s); };
    auto c_empty = [&](int s) { return bar(AC + s); };
    auto b_full = [&](int s) { return bar(2 * AC + s); };
    auto b_empty = [&](int s) { return bar(2 * AC + B_STAGES + s); };
    auto t_full = [&](int s) { return bar(2 * AC + 2 * B_STAGES + s); };
    auto t_empty = [&](int s) { return bar(2 * AC + 2 * B_STAGES + T_STAGES + s); };
    auto i_full = [&](int s) { return bar(2 * AC + 2 * B_STAGES + 2 * T_STAGES + s); };
    auto i_empty = [&](int s) { return bar(2 * AC + 2 * B_STAGES + 2 * T_STAGES + I_STAGES + s); };
    auto m_full = [&](int s) { return bar(2 * AC + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + s); };
    auto m_empty = [&](int s) { return bar(2 * AC + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + MS + s); };
    const uint32_t d_bar = bar(2 * AC + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + 2 * MS);
    auto meta = [&](int slot) { return reinterpret_cast<int*>(smem + META_OFF + slot * META_W); };
    Item* items = reinterpret_cast<Item*>(smem + ITEM_OFF);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + MISC_OFF);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);
    const uint32_t WL = p.wait_limit;

    if (tid == 0) {
        for (int s = 0; s < AC; s++) {
            mbar_init(c_full(s), DEC_WARPS / DEC_SETS);  // every warp of the chunk's decode set has written its rows
            mbar_init(c_empty(s), 1);  // the MMAs reading the chunk have completed
        }
        for (int s = 0; s < B_STAGES; s++) {
            mbar_init(b_full(s), 1);
            mbar_init(b_empty(s), 1);
        }
        for (int s = 0; s < T_STAGES; s++) {
            mbar_init(t_full(s), 1);
            mbar_init(t_empty(s), 4);
        }
        for (int s = 0; s < I_STAGES; s++) {
            mbar_init(i_full(s), 1);
            mbar_init(i_empty(s), I_CONSUMERS);
        }
        for (int s = 0; s < MS; s++) {
            mbar_init(m_full(s), 1);   // written by the item's gather warp
            mbar_init(m_empty(s), 1);  // released by the last epilogue warp to finish a tile of the item
            reinterpret_cast<int*>(smem + MCNT_OFF)[s] = 0;
        }
        mbar_init(d_bar, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    {
        // pair table: window w of L+1 bits covers two consecutive states (w >> 1, w & (2^L - 1)); entry = their two
        // values rounded to fp16, the first in the low half (the memory order of the decoded row)
        uint32_t* tab2 = reinterpret_cast<uint32_t*>(smem + TAB_OFF);
        const uint32_t mask = (1u << p.L) - 1u;
        for (int w = tid; w < (2 << p.L); w += NTHREADS) {
            const uint32_t h0 = __half_as_ushort(__float2half_rn(__ldg(p.tab + (w >> 1))));
            const uint32_t h1 = __half_as_ushort(__float2half_rn(__ldg(p.tab + (w & mask))));
            tab2[w] = h0 | (h1 << 16);
        }
    }
    if (warp == W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // every consumer role reads the items in order: item n sits in slot n % I_STAGES (the MMA thread alone, the
    // other roles with all lanes and one outcome per warp)
    auto read_item = [&](int n, Item& it, bool whole_warp) -> bool {
        const int s = n % I_STAGES;
        const bool r = whole_warp ? warp_wait(i_full(s), (n / I_STAGES) & 1, abort, WL)
                                  : mbar_wait(i_full(s), (n / I_STAGES) & 1, abort, WL);
        if (r) it = items[s];
        return r;
    };
    auto take_item = [&](int n, Item& it) -> bool {  // whole warp: read and release
        const bool r = read_item(n, it, true);
        if (r && lane == 0) mbar_arrive(i_empty(n % I_STAGES));
        return r;
    };

    bool mma_issued = false;

    if (warp < W_MMA) {
        // ---- decode: set ds = warp / 4 writes chunks KCH / DEC_SETS * ds .. of every tile; warp w % 4, rows
        //      32 (w % 4) + lane
        const uint32_t* tab2 = reinterpret_cast<const uint32_t*>(smem + TAB_OFF);
        const int sh = 31 - p.L;  // a window is the top L+1 bits of a 32-bit funnel shift
        const int ds = warp / (DEC_WARPS / DEC_SETS);
        constexpr int SCH = KCH / DEC_SETS;  // chunks per set
        const int c0 = SCH * ds;             // the set's first chunk; its words start at 2 * c0
        const int r = 32 * (warp % (DEC_WARPS / DEC_SETS)) + lane;
        const int sw = r & 7;
        const uint32_t row_off = (uint32_t)((r >> 3) * 1024 + sw * 128);
        auto load_words = [&](const Item& it, int t, uint32_t (&w)[SWORDS]) {
            const int row = it.first + t * TILE_ROWS + r;
            const bool v = it.live && row >= it.cs && row < it.ce;
            const uint32_t* src = p.words + (int64_t)(v ? row : 0) * p.W + 2 * c0;
#pragma unroll
            for (int i = 0; i < SWORDS; i++) w[i] = v ? __ldg(src + i) : 0u;
        };
        int n = 0;
        uint32_t gtile = 0;  // tiles decoded so far: chunk c of tile gtile is chunk KCH * gtile + c of the ring
        Item it;
        bool ok = take_item(0, it);
        uint32_t w[SWORDS], wn[SWORDS];
        if (ok) load_words(it, 0, w);
        while (ok && it.live) {
            Item itn;
            if (!take_item(n + 1, itn)) break;
            for (int t = 0; t < it.ntiles; t++, gtile++) {
                // words of the tile after this one (this item's next tile, else the next item's first)
                if (t + 1 < it.ntiles)
                    load_words(it, t + 1, wn);
                else
                    load_words(itn, 0, wn);
                const int row = it.first + t * TILE_ROWS + r;
                const bool v = row >= it.cs && row < it.ce;
#pragma unroll
                for (int cc = 0; cc < SCH; cc++) {
                    // the other set fills the ring's other chunks: a set's wait for chunk g starts after its wait
                    // for its previous chunk (g - 1 or g - KCH + SCH - 1) passed, i.e. after every chunk up to g - 8
                    // was consumed, so the slot's barrier is never two phases behind the parity waited on
                    const uint32_t g = KCH * gtile + (uint32_t)(c0 + cc);
                    const int cslot = (int)(g % AC);
                    if (!warp_wait(c_empty(cslot), ((g / AC) & 1u) ^ 1u, abort, WL)) {
                        ok = false;
                        break;
                    }
                    if (v) {
                        uint8_t* dst = smem + A_OFF + cslot * CH_BYTES + row_off;
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t hi = w[2 * cc + h], lo = w[2 * cc + h + 1];
#pragma unroll
                            for (int uu = 0; uu < 4; uu++) {
                                uint4 q;
                                q.x = tab2[__funnelshift_l(lo, hi, 8 * uu + 0) >> sh];
                                q.y = tab2[__funnelshift_l(lo, hi, 8 * uu + 2) >> sh];
                                q.z = tab2[__funnelshift_l(lo, hi, 8 * uu + 4) >> sh];
                                q.w = tab2[__funnelshift_l(lo, hi, 8 * uu + 6) >> sh];
                                *reinterpret_cast<uint4*>(dst + (((h * 4 + uu) ^ sw) << 4)) = q;
                            }
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(c_full(cslot));
                }
                if (!ok) break;
#pragma unroll
                for (int i = 0; i < SWORDS; i++) w[i] = wn[i];
            }
            if (!ok) break;
            it = itn;
            n++;
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            int nu = 0, cslot = 0;
            uint32_t cph = 0;
            for (int n = 0;; n++) {
                Item it;
                if (!read_item(n, it, false)) break;
                mbar_arrive(i_empty(n % I_STAGES));
                if (!it.live) break;
                const int sb = n % B_STAGES;
                const uint32_t idesc = f16_idesc((it.nq + 15) & ~15);
                const uint32_t bbase = sbase + B_OFF + sb * B_BYTES;
                bool ok = true;
                for (int t = 0; t < it.ntiles && ok; t++, nu++) {
                    const int st = nu % T_STAGES;
                    const uint32_t d = tmem + (uint32_t)(st * QN);
                    for (int c = 0; c < KCH; c++) {
                        if (!mbar_wait(c_full(cslot), cph, abort, WL) ||
                            (c == 0 && t == 0 && !mbar_wait(b_full(sb), (n / B_STAGES) & 1, abort, WL)) ||
                            (c == 0 && !mbar_wait(t_empty(st), ((nu / T_STAGES) & 1) ^ 1, abort, WL))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t abase = sbase + A_OFF + cslot * CH_BYTES;
                        const uint32_t bb = bbase + c * QN * 128;
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            mma_f16(d, sw128_desc(abase + kk * 32), sw128_desc(bb + kk * 32), idesc,
                                    (c > 0 || kk > 0) ? 1u : 0u);
                        mma_issued = true;
                        if (c == KCH - 1) mma_commit(t_full(st));
                        mma_commit(c_empty(cslot));  // the chunk slot is free once these MMAs complete
                        if (++cslot == AC) {
                            cslot = 0;
                            cph ^= 1u;
                        }
                    }
                }
                if (!ok) break;
                mma_commit(b_empty(sb));  // the item's queries are free once its last MMAs complete
            }
        }
        __syncwarp();
    } else if (warp < W_PROD) {
        // ---- query gather: items alternate between the gather warps (warp g fills B stage g); lane l fills rows
        //      l + 32 rr
        const int gw = warp - W_GATHER;
        for (int n = 0;; n++) {
            Item it;
            if (!take_item(n, it)) break;
            if (!it.live) break;
            if (n % GATHER_WARPS != gw) continue;
            const int sb = n % B_STAGES, sm = n % MS;
            const int nq = it.nq, n16 = (it.nq + 15) & ~15;
            // the item's query ids and pair constants; its rows are copied with cp.async (all of them in flight at
            // once, zero rows past nq) while the thresholds load and the metadata slot is filled
            int qq[4];
            float qcv[4], thv[4];
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                const int gq = lane + 32 * rr;
                qq[rr] = gq < nq ? p.qid[it.qoff + gq] : -1;
                qcv[rr] = gq < nq ? p.qcp[it.qoff + gq] : 0.f;
            }
            if (!warp_wait(b_empty(sb), ((n / B_STAGES) & 1) ^ 1, abort, WL)) break;
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                const int gq = lane + 32 * rr;
                if (gq >= n16) continue;
                const int q = qq[rr];
                const uint4* src = reinterpret_cast<const uint4*>(p.Qh + (int64_t)(q >= 0 ? q : 0) * R);
                const uint32_t bs = sbase + B_OFF + sb * B_BYTES + (gq >> 3) * 1024 + (gq & 7) * 128;
#pragma unroll
                for (int c = 0; c < KCH; c++)
#pragma unroll
                    for (int cc = 0; cc < 8; cc++)
                        cp_async16(bs + c * QN * 128 + ((cc ^ (gq & 7)) << 4), src + 8 * c + cc, q >= 0);
            }
#pragma unroll
            for (int rr = 0; rr < 4; rr++) thv[rr] = (MODE && qq[rr] >= 0) ? p.t0[qq[rr]] : 0.f;
            if (!warp_wait(m_empty(sm), ((n / MS) & 1) ^ 1, abort, WL)) {
                cp_async_wait_all();  // no copy into shared memory stays in flight
                break;
            }
            int* mq = meta(sm);
            float* mc = reinterpret_cast<float*>(mq + QN);
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                const int gq = lane + 32 * rr;
                mq[gq] = qq[rr];
                mc[gq] = qcv[rr];
                mc[QN + gq] = thv[rr];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(m_full(sm));
            cp_async_wait_all();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(b_full(sb));
        }
    } else if (warp == W_PROD) {
        if (lane == 0) {
            const int nl = *p.nlist;
            // cell pipeline, refilled by every next_cell(): `pre` (bounds and pair range of the next cell), `cn` (the
            // cell after it), `idxn` (the list index after that); each call only uses values loaded by the previous
            // call, so the producer never waits for a load it just issued
            auto grab = [&]() { return atomicAdd(p.sched, 1); };
            auto cell_of = [&](int idx) { return idx < nl ? p.list[idx] : -1; };
            auto fields = [&](int e) {  // a list entry: cell | part << 16
                const int c = e >= 0 ? (e & 0xffff) : -1;
                CellInfo ci{c, 0, 0, 0, 0, e >= 0 ? e >> 16 : 0};
                if (c >= 0) {
                    ci.cs = (int)p.off[c];
                    ci.ce = (int)p.off[c + 1];
                    ci.qn = p.ccnt[c];
                    ci.qoff = p.coff[c];
                }
                return ci;
            };
            CellInfo pre = fields(cell_of(grab()));
            int cn = cell_of(grab());
            int idxn = grab();
            auto next_cell = [&]() {
                const CellInfo c = pre;
                pre = fields(cn);
                cn = cell_of(idxn);
                idxn = grab();
                return c;
            };
            // cells with no pairs (not listed) or no rows (probed, but nothing to scan) are skipped
            auto idle = [&](const CellInfo& ci) {  // no pairs, no rows, or a part past the cell's last tile
                return ci.cell >= 0 && (ci.qn <= 0 || ci.ce <= ci.cs ||
                                        (ci.cs & ~31) + ci.part * CELL_PART_TILES * TILE_ROWS >= ci.ce);
            };
            CellInfo cur;
            do {
                cur = next_cell();
            } while (idle(cur));
            int g = 0;  // group of `cur` the next item covers
            for (int ni = 0;; ni++) {
                Item it{-1, 0, 0, 0, 0, 0, 0, 0};
                if (cur.cell >= 0) {
                    // the part's tiles of the cell's tile grid (which starts at the cell's first 32-row block)
                    const int first = (cur.cs & ~31) + cur.part * CELL_PART_TILES * TILE_ROWS;
                    it = Item{cur.cell, cur.cs, cur.ce, first,
                              min(CELL_PART_TILES, (cur.ce - first + TILE_ROWS - 1) / TILE_ROWS), cur.qoff + g * QN,
                              min(QN, cur.qn - g * QN), 1};
                }
                const int s = ni % I_STAGES;
                if (!mbar_wait(i_empty(s), ((ni / I_STAGES) & 1) ^ 1, abort, WL)) break;
                items[s] = it;
                mbar_arrive(i_full(s));  // release: the item's fields are visible to whoever acquires the phase
                if (!it.live) break;
                if (++g * QN >= cur.qn) {
                    g = 0;
                    do {
                        cur = next_cell();
                    } while (idle(cur));
                }
            }
        }
    } else {
        // ---- epilogue: group eg takes the tiles nu = eg (mod EPI_GROUPS); warp ew = warp % 4 reads TMEM lanes
        //      32*ew .. 32*ew+31 (tile rows)
        const int we = warp - W_EPI;
        const int eg = we / 4;
        const int ew = warp & 3;
        uint32_t* colm = reinterpret_cast<uint32_t*>(smem + COL_OFF) + we * 64;
        int* colb = reinterpret_cast<int*>(colm + 32);
        int nu = 0;
        for (int n = 0;; n++) {
            Item it;
            if (!take_item(n, it)) break;
            if (!it.live) break;
            bool ok = true;
            const int nq = it.nq, sm = n % MS;
            for (int t = 0; t < it.ntiles; t++, nu++) {
                if (nu % EPI_GROUPS != eg) continue;
                const int row0 = it.first + t * TILE_ROWS;
                const int row = row0 + 32 * ew + lane;
                const bool rvalid = row >= it.cs && row < it.ce;
                const bool wactive = row0 + 32 * ew < it.ce;
                const int blk_rel = (row0 + 32 * ew) / 32 - it.cs / 32;
                const int st = nu % T_STAGES;
                const float sc = rvalid ? __half2float(p.scale1[row]) : 0.f;  // loaded before the waits
                if (!warp_wait(m_full(sm), (n / MS) & 1, abort, WL) ||
                    !warp_wait(t_full(st), (nu / T_STAGES) & 1, abort, WL)) {
                    ok = false;
                    break;
                }
                const int* mq = meta(sm);
                const float* mc = reinterpret_cast<const float*>(mq + QN);
                const float* mt = mc + QN;
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(32 * ew) << 16) + (uint32_t)(st * QN);
                for (int h = 0; h * 32 < nq; h++) {
                    uint32_t acc[32];
                    tmem_ld32(ta + 32 * h, acc);
                    tmem_ld_wait();
                    if ((h + 1) * 32 >= nq) {
                        // accumulator in registers: the TMEM stage goes back to the MMA before the scoring
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(t_empty(st));
                    }
                    if (!wactive) continue;
                    const int nc = min(32, nq - h * 32);
                    const float4* mc4 = reinterpret_cast<const float4*>(mc + 32 * h);
                    if (MODE == 0) {
#pragma unroll
                        for (int j4 = 0; j4 < 8; j4++) {
                            if (4 * j4 >= nc) break;
                            const float4 cv = mc4[j4];
                            const float c4[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const int jj = 4 * j4 + u;
                                if (jj < nc) {
                                    const float est = __fadd_rn(__fmul_rn(sc, __uint_as_float(acc[jj])), c4[u]);
                                    const uint32_t m = __reduce_max_sync(0xffffffffu, rvalid ? f2o(est) : 0u);
                                    if (lane == 0) p.bmc[(int64_t)(it.qoff + 32 * h + jj) * p.MB + blk_rel] = o2f(m);
                                }
                            }
                        }
                    } else {
                        const float4* mt4 = reinterpret_cast<const float4*>(mt + 32 * h);
                        uint32_t rowmask = 0;
#pragma unroll
                        for (int j4 = 0; j4 < 8; j4++) {
                            if (4 * j4 >= nc) break;
                            const float4 cv = mc4[j4], tv = mt4[j4];
                            const float c4[4] = {cv.x, cv.y, cv.z, cv.w};
                            const float t4[4] = {tv.x, tv.y, tv.z, tv.w};
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const int jj = 4 * j4 + u;
                                if (jj < nc) {
                                    const float est = __fadd_rn(__fmul_rn(sc, __uint_as_float(acc[jj])), c4[u]);
                                    const bool keep = rvalid && est >= t4[u];
                                    acc[jj] = __float_as_uint(est);
                                    rowmask |= (uint32_t)keep << jj;
                                }
                            }
                        }
                        const uint32_t mymask = transpose32(rowmask);  // lane jj: the rows keeping column jj
                        int mybase = 0;
                        if (mymask) mybase = atomicAdd(p.cnt + mq[32 * h + lane], __popc(mymask));
                        colm[lane] = mymask;
                        colb[lane] = mybase;
                        __syncwarp();
                        while (rowmask) {
                            const int jj = __ffs(rowmask) - 1;
                            rowmask &= rowmask - 1;
                            const int j = 32 * h + jj;
                            const float est = __uint_as_float(select32(acc, jj));
                            const int idx = colb[jj] + __popc(colm[jj] & ((1u << lane) - 1u));
                            if (idx < p.M) {
                                const int64_t o = (int64_t)mq[j] * p.M + idx;
                                p.bval[o] = est;
                                p.bpos[o] = row;
                            }
                        }
                        __syncwarp();
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    // the item's tiles are spread over the warpgroups, which finish in any order: the metadata slot is
                    // free once all 4 * ntiles warps are done with it; the last one to count itself resets the count
                    // and releases the slot
                    __threadfence_block();
                    int* mcount = reinterpret_cast<int*>(smem + MCNT_OFF);
                    if (atomicAdd(mcount + sm, 1) == 4 * it.ntiles - 1) {
                        mcount[sm] = 0;
                        mbar_arrive(m_empty(sm));
                    }
                }
            }
            if (!ok) break;
        }
    }
    // drain (a wait that ignores the abort flag): one commit after the last MMA issued has arrived, i.e. every MMA of
    // this CTA has completed before its tensor memory is freed and its shared memory released
    if (warp == W_MMA && lane == 0 && mma_issued) {
        mma_commit(d_bar);
        mbar_drain(d_bar, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == W_MMA)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    if (tid == 0) {
        if (*abort && p.status) atomicExch(p.status, 1);
        // the last CTA out resets the work counter for the next launch (every CTA took its last cell before this)
        __threadfence();
        if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(p.sched, 0);
            atomicExch(p.sched + 1, 0);
        }
    }
}

}  // namespace tcells
}  // namespace fvs

extern "C" int fvs_trellis_scan_cells(fvs_stream_t stream, int mode, const uint16_t* Qh, int B, int R,
                                      const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                                      const int32_t* list, const int32_t* nlist, int maxlist, const int64_t* off,
                                      int NC, const int32_t* words, int W, const float* tab, int L,
                                      const uint16_t* scale1, const float* t0, int32_t* cnt, float* bval,
                                      int32_t* bpos, int M, float* bmc, int MB, int32_t* sched, int32_t* status) {
    using namespace fvs::tcells;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(R == fvs::tcells::R && B >= 0 && maxlist >= 0 && NC > 0);
    FVS_CHECK_ARG(L >= 2 && W >= (R + L - 1 + 31) / 32);
    FVS_CHECK_ARG(Qh && qid && coff && ccnt && qcp && list && nlist && off && words && tab && scale1 && sched);
    FVS_CHECK_ARG(((uintptr_t)Qh & 15) == 0);
    if (mode == 0) FVS_CHECK_ARG(bmc && MB > 0);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (L > MAX_L) return FVS_ERANGE;
    if (maxlist == 0 || B == 0) return FVS_OK;
    Params p{(const __half*)Qh, (const uint32_t*)words, tab, (const __half*)scale1, qid, coff, ccnt, qcp, list, nlist,
             off, t0, cnt, bval, bpos, bmc, sched, status, M, MB, W, L, pipeline_wait_limit()};
    cudaError_t e = mode ? fvs_ensure_smem((const void*)trellis_cells_kernel<1>, SMEM_BYTES)
                         : fvs_ensure_smem((const void*)trellis_cells_kernel<0>, SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    const int nsm = fvs_sm_count();
    const int grid = maxlist < nsm ? maxlist : nsm;
    if (mode == 0)
        trellis_cells_kernel<0><<<grid, NTHREADS, SMEM_BYTES, stream>>>(p);
    else
        trellis_cells_kernel<1><<<grid, NTHREADS, SMEM_BYTES, stream>>>(p);
    return fvs_launch_status();
}
