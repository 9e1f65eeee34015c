// Int8 stage-1 IVF scan on the 5th-generation tensor cores, cell-major (tcgen05, sm_100a).
//
// Same contract and arithmetic as fvs_i8_scan_tc (the reference's `_first8c` / `_emit8c`,
// `throughput/ivf8c_kern.py:2-36`), organised around cells instead of 128-row tiles:
//   * work items are cell parts, handed out dynamically: the producer thread of a CTA takes the next entry of a
//     compact list of the pass's non-empty cells (largest first) with one atomicAdd, so CTAs finish together whatever
//     the cells' sizes and query counts; an entry is `cell | part << 16`, part p covering tiles 8p .. 8p+7 of the
//     cell, so that a large cell (the index's largest hold thousands of rows) is shared by several CTAs instead of
//     setting the pass's tail;
//   * a part's queries (the cell's, up to RSUB sub-tiles of QN) are gathered ONCE into shared memory and stay there
//     while the part's 128-row code tiles stream past them (a cell of ~250 rows spans 2-3 tiles; the tile scan
//     gathered them once per tile); cells with more queries are split into groups of RSUB sub-tiles, each group
//     streaming the part's tiles again (from L2);
//   * a code tile is fetched as the 32-row blocks the cell occupies, one TMA copy per K-half with a box of 32, 64, 96
//     or 128 rows (four tensor maps), so the rows past the cell's end are not moved; K-half 1 lands right after
//     K-half 0's blocks.
// Warp roles (640 threads, one CTA per SM; see Shape):
//   warp 0      : lane 0 takes cell parts (atomicAdd on sched[0]; the list entry, bounds and pair range of a cell are
//                 loaded ahead in stages), publishes each work item (cell, group of sub-tiles) in a ring of I_STAGES
//                 slots up to AHEAD items ahead, and issues the TMA loads of the item's code tiles into A_STAGES stages
//   warp 1      : TMEM allocation; lane 0 issues tcgen05.mma.kind::i8 (M=128 rows, N=16..64 queries, K=256 as 8 x 32)
//                 for every (tile, sub-tile) unit into one of T_STAGES accumulators; releases a code tile after its
//                 units and the item's query sub-tiles after its last tile
//   warps 2-3   : gather: the item's sub-tiles alternate between the two warps; rows of q8 picked by qid, copied with
//                 cp.async (a sub-tile's rows in flight at once) into the canonical K-major 128 B-swizzled layout,
//                 and the sub-tile's column metadata (qid, qs, pair constant, threshold) into one of MS slots,
//                 released when every epilogue warp is done with the sub-tile
//   warps 4-    : EPI_GROUPS epilogue warpgroups, units alternating between them; each warp loads its rows' scales before
//                 waiting for the accumulator, returns the TMEM stage as soon as the accumulator is in registers, then
//                 as fvs_i8_scan_tc: est = ((acc * qs) * zs) + qcp with explicit rounding, first pass: block maximum
//                 per query by redux.sync.max; emit: kept-column masks transposed across the warp, one atomicAdd per
//                 column.
// The last CTA to finish resets sched[0..1], so the next launch starts from zero.
// Every mbarrier wait is bounded; on expiry the CTA raises `status`, drains what it issued, frees TMEM and returns.
#include <cuda.h>

#include "fvs_common.cuh"
#include "fvs_tcgen05.cuh"

namespace fvs {
namespace cells {
using namespace fvs::tcg;

constexpr int TILE_ROWS = 128;
constexpr int QN = 64;  // queries per sub-tile
constexpr int RB = 256;
constexpr int I_STAGES = 8;
constexpr int MS = 8;    // column-metadata slots (one per sub-tile, held until the sub-tile's last unit is done)
constexpr int GATHER_WARPS = 2;
constexpr int AHEAD = 4;  // work items published beyond the one whose tiles are being loaded
constexpr int W_TMA = 0, W_MMA = 1, W_GATHER = 2, W_EPI = W_GATHER + GATHER_WARPS;
static_assert(W_EPI % 4 == 0, "epilogue warpgroups cover TMEM lane quarters 0..3 in order");
static_assert(AHEAD + 2 <= I_STAGES, "an item's slot is not reused before the producer has loaded its tiles");

// Pipeline shape per pass: one CTA per SM with 4 code-tile stages, 4 query sub-tile stages (two sub-tiles per item),
// 8 TMEM accumulators and 4 epilogue warpgroups.  (Two CTAs per SM with half of each, measured for the first pass:
// 82 -> 68 us at 1M rows and 4096 cells, but 0.19 -> 0.28 ms at 2M rows and 8192 cells, where the last CTAs' parts
// set the pass time and half a pipeline lengthens that tail.)
template <int MODE>
struct Shape;
template <>
struct Shape<0> {
    static constexpr int A_STAGES = 4, B_STAGES = 4, RSUB = 2, T_STAGES = 8, EPI_GROUPS = 4, CTAS_PER_SM = 1;
};
template <>
struct Shape<1> {
    static constexpr int A_STAGES = 4, B_STAGES = 4, RSUB = 2, T_STAGES = 8, EPI_GROUPS = 4, CTAS_PER_SM = 1;
};

struct Item {
    int cell, cs, ce, first, ntiles, qoff, nq, nsub;  // nsub == 0: no more work
};

constexpr int A_BYTES = 2 * TILE_ROWS * 128;  // one code tile: 2 K-halves x 16 KB
constexpr int BLK_BYTES = 32 * 128;           // one 32-row block of one K-half

// the code matrix as 2D tensor maps whose boxes are one K-half (128 B) of 32, 64, 96 or 128 rows: a tile of nblk
// 32-row blocks moves as two copies (one per K-half) with map nblk - 1
struct ZMaps {
    CUtensorMap m[4];
};
constexpr int B_BYTES = 2 * QN * 128;         // one query sub-tile: 2 K-halves x 8 KB
constexpr int META_W = 4 * QN * 4;

// the pass's warps, tensor memory and shared-memory carve-up (offsets from a 1024-byte aligned base)
template <int MODE>
struct Layout : Shape<MODE> {
    using S = Shape<MODE>;
    static constexpr int NWARPS = W_EPI + 4 * S::EPI_GROUPS;
    static constexpr int NTHREADS = 32 * NWARPS;
    static constexpr uint32_t TMEM_COLS = S::T_STAGES * QN;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + S::A_STAGES * A_BYTES;
    static constexpr int META_OFF = B_OFF + S::B_STAGES * B_BYTES;   // per sub-tile slot: qid, qs, qcp, t0 of QN columns
    static constexpr int COL_OFF = META_OFF + MS * META_W;           // per epilogue warp: 32 column masks + 32 bases
    static constexpr int MCNT_OFF = COL_OFF + 4 * S::EPI_GROUPS * 64 * 4;  // per metadata slot: warps done with it
    static constexpr int ITEM_OFF = MCNT_OFF + MS * 4;
    static constexpr int BAR_OFF = ITEM_OFF + I_STAGES * (int)sizeof(Item);
    static constexpr int NBAR = 2 * S::A_STAGES + 2 * S::B_STAGES + 2 * S::T_STAGES + 2 * I_STAGES + 2 * MS + 1;
    static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;  // tmem base, abort flag
    static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
    static constexpr uint32_t I_CONSUMERS = 1 + GATHER_WARPS + 4 * S::EPI_GROUPS;  // MMA thread, gather, epilogue
    static_assert(S::B_STAGES >= 2 * S::RSUB, "a work item's sub-tiles and the next item's fit together");
    static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS >= 32 && TMEM_COLS * S::CTAS_PER_SM <= 512,
                  "tensor memory columns: a power of two, the SM's CTAs together within 512");
    static_assert(SMEM_BYTES * S::CTAS_PER_SM <= 232448 - 1024 * (S::CTAS_PER_SM - 1), "shared memory per SM");
    static_assert(NTHREADS * S::CTAS_PER_SM <= 2048, "threads per SM");
};

struct Params {
    const int8_t* q8;
    const float* qs;
    const int32_t* qid;
    const int32_t* coff;
    const int32_t* ccnt;
    const float* qcp;
    const int32_t* list;
    const int32_t* nlist;
    const int64_t* off;
    const float* zs;
    const float* t0;
    int32_t* cnt;
    float* bval;
    int32_t* bpos;
    float* bmc;
    int32_t* sched;
    int32_t* status;
    int M, MB;
    uint32_t wait_limit;
};

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
__global__ void __launch_bounds__(Layout<MODE>::NTHREADS, Layout<MODE>::CTAS_PER_SM)
    scan_cells_kernel(const __grid_constant__ ZMaps zm, Params p) {
    using LY = Layout<MODE>;
    constexpr int A_STAGES = LY::A_STAGES, B_STAGES = LY::B_STAGES, RSUB = LY::RSUB, T_STAGES = LY::T_STAGES;
    constexpr int EPI_GROUPS = LY::EPI_GROUPS;
    constexpr uint32_t TMEM_COLS = LY::TMEM_COLS, I_CONSUMERS = LY::I_CONSUMERS;
    constexpr int A_OFF = LY::A_OFF, B_OFF = LY::B_OFF, META_OFF = LY::META_OFF, COL_OFF = LY::COL_OFF;
    constexpr int MCNT_OFF = LY::MCNT_OFF, ITEM_OFF = LY::ITEM_OFF, BAR_OFF = LY::BAR_OFF, MISC_OFF = LY::MISC_OFF;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = saddr(smem);
    auto a_full = [&](int s) { return sbase + BAR_OFF + 8 * s; };
    auto a_empty = [&](int s) { return sbase + BAR_OFF + 8 * (A_STAGES + s); };
    auto b_full = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + s); };
    auto b_empty = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + B_STAGES + s); };
    auto t_full = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + s); };
    auto t_empty = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + T_STAGES + s); };
    auto i_full = [&](int s) { return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 2 * T_STAGES + s); };
    auto i_empty = [&](int s) {
        return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 2 * T_STAGES + I_STAGES + s);
    };
    auto m_full = [&](int s) {
        return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + s);
    };
    auto m_empty = [&](int s) {
        return sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + MS + s);
    };
    const uint32_t d_bar = sbase + BAR_OFF + 8 * (2 * A_STAGES + 2 * B_STAGES + 2 * T_STAGES + 2 * I_STAGES + 2 * MS);
    auto meta = [&](int slot) { return reinterpret_cast<int*>(smem + META_OFF + slot * META_W); };
    Item* items = reinterpret_cast<Item*>(smem + ITEM_OFF);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + MISC_OFF);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);
    const uint32_t WL = p.wait_limit;

    if (tid == 0) {
        for (int s = 0; s < A_STAGES; s++) {
            mbar_init(a_full(s), 1);
            mbar_init(a_empty(s), 1);
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
            mbar_init(m_full(s), 1);   // written by the sub-tile's gather warp
            mbar_init(m_empty(s), 1);  // released by the last epilogue warp to finish a unit of the sub-tile
            reinterpret_cast<int*>(smem + MCNT_OFF)[s] = 0;
        }
        mbar_init(d_bar, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
    // gather and epilogue warps with all lanes and one outcome per warp)
    auto read_item = [&](int n, Item& it, bool whole_warp) -> bool {
        const int s = n % I_STAGES;
        const bool r = whole_warp ? warp_wait(i_full(s), (n / I_STAGES) & 1, abort, WL)
                                  : mbar_wait(i_full(s), (n / I_STAGES) & 1, abort, WL);
        if (r) it = items[s];
        return r;
    };

    int na_load = 0, na_mma = 0;  // code tiles loaded / consumed
    bool mma_issued = false;

    if (warp == W_TMA) {
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 4; k++) asm volatile("prefetch.tensormap [%0];" ::"l"(&zm.m[k]) : "memory");
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
            int g = 0;  // group of `cur` the next item covers
            int ni = 0;
            auto make_item = [&](const CellInfo& ci, int grp) {
                Item it;
                if (ci.cell < 0) {
                    it = Item{-1, 0, 0, 0, 0, 0, 0, 0};
                } else {
                    // the part's tiles of the cell's tile grid (which starts at the cell's first 32-row block)
                    const int grid0 = ci.cs & ~31;
                    const int first = grid0 + ci.part * CELL_PART_TILES * TILE_ROWS;
                    const int ntiles = min(CELL_PART_TILES, (ci.ce - first + TILE_ROWS - 1) / TILE_ROWS);
                    const int q0 = grp * RSUB * QN;
                    const int nq = min(RSUB * QN, ci.qn - q0);
                    it = Item{ci.cell, ci.cs, ci.ce, first, ntiles, ci.qoff + q0, nq, (nq + QN - 1) / QN};
                }
                return it;
            };
            auto push = [&](const Item& it) -> bool {
                const int s = ni % I_STAGES;
                if (!mbar_wait(i_empty(s), ((ni / I_STAGES) & 1) ^ 1, abort, WL)) return false;
                items[s] = it;
                mbar_arrive(i_full(s));  // release: the item's fields are visible to whoever acquires the phase
                ni++;
                return true;
            };
            // cells with no pairs (not listed) or no rows (probed, but nothing to scan: the reference launches no
            // program for them) are skipped
            auto idle = [&](const CellInfo& ci) {  // no pairs, no rows, or a part past the cell's last tile
                return ci.cell >= 0 && (ci.qn <= 0 || ci.ce <= ci.cs ||
                                        (ci.cs & ~31) + ci.part * CELL_PART_TILES * TILE_ROWS >= ci.ce);
            };
            auto advance = [&](CellInfo& ci, int& grp) {
                grp++;
                if (ci.cell >= 0 && grp * RSUB * QN < ci.qn) return;
                grp = 0;
                do {
                    ci = next_cell();
                } while (idle(ci));
            };
            // items are published up to AHEAD beyond the one whose tiles are being loaded, so that the gathers of the
            // next items start early; the producer reads its own items back from the ring (a slot is reused only
            // AHEAD + 1 < I_STAGES items later)
            CellInfo cur{-1, 0, 0, 0, 0};
            bool more = true, started = false, ok = true;
            auto publish_until = [&](int upto) -> bool {
                while (more && ni <= upto) {
                    if (!started) {
                        started = true;
                        cur = next_cell();
                        while (idle(cur)) cur = next_cell();
                    } else {
                        advance(cur, g);
                    }
                    const Item nx = make_item(cur, g);
                    if (!push(nx)) return false;
                    if (nx.nsub == 0) more = false;
                }
                return true;
            };
            for (int n = 0; ok; n++) {
                if (!publish_until(n + AHEAD)) break;
                const Item it = items[n % I_STAGES];
                if (it.nsub == 0) break;
                for (int t = 0; t < it.ntiles && ok; t++) {
                    const int s = na_load % A_STAGES;
                    if (!mbar_wait(a_empty(s), ((na_load / A_STAGES) & 1) ^ 1, abort, WL)) {
                        ok = false;
                        break;
                    }
                    const int row0 = it.first + t * TILE_ROWS;
                    const int nblk = min(4, (it.ce - row0 + 31) / 32);
                    mbar_expect_tx(a_full(s), (uint32_t)(nblk * 2 * BLK_BYTES));
                    const uint32_t dst = sbase + A_OFF + s * A_BYTES;
                    // K-half 0 at dst, K-half 1 right after it (nblk * 4 KB on, 1024-byte aligned)
                    tma_load_2d(dst, &zm.m[nblk - 1], 0, row0, a_full(s));
                    tma_load_2d(dst + nblk * BLK_BYTES, &zm.m[nblk - 1], 128, row0, a_full(s));
                    na_load++;
                }
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            int nb = 0, nu = 0;
            for (int n = 0;; n++) {
                Item it;
                if (!read_item(n, it, false)) break;
                mbar_arrive(i_empty(n % I_STAGES));
                if (it.nsub == 0) break;
                bool ok = true;
                for (int t = 0; t < it.ntiles && ok; t++) {
                    const int sa = na_mma % A_STAGES;
                    if (!mbar_wait(a_full(sa), (na_mma / A_STAGES) & 1, abort, WL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t abase = sbase + A_OFF + sa * A_BYTES;
                    // K-half 1 follows the tile's nblk blocks of K-half 0; the MMA's 128 rows reach past them only in
                    // rows beyond the cell's end, which the epilogue does not read, and stay inside the stage
                    const int row0 = it.first + t * TILE_ROWS;
                    const uint32_t half1 = (uint32_t)(min(4, (it.ce - row0 + 31) / 32) * BLK_BYTES);
                    for (int s = 0; s < it.nsub; s++) {
                        const int sb = (nb + s) % B_STAGES, st = nu % T_STAGES;
                        if ((t == 0 && !mbar_wait(b_full(sb), ((nb + s) / B_STAGES) & 1, abort, WL)) ||
                            !mbar_wait(t_empty(st), ((nu / T_STAGES) & 1) ^ 1, abort, WL)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const int nq = min(QN, it.nq - s * QN);
                        const uint32_t idesc = i8_idesc((nq + 15) & ~15);
                        const uint32_t d = tmem + (uint32_t)(st * QN);
                        const uint32_t bb = sbase + B_OFF + sb * B_BYTES;
#pragma unroll
                        for (int ks = 0; ks < RB / 32; ks++) {
                            const int h = ks >> 2, kofs = (ks & 3) * 32;
                            mma_i8(d, sw128_desc(abase + h * half1 + kofs),
                                   sw128_desc(bb + h * QN * 128 + kofs), idesc, ks > 0 ? 1u : 0u);
                        }
                        mma_issued = true;
                        mma_commit(t_full(st));
                        nu++;
                    }
                    if (!ok) break;
                    mma_commit(a_empty(sa));  // the code tile is free once these MMAs complete
                    na_mma++;
                }
                if (!ok) break;
                for (int s = 0; s < it.nsub; s++) mma_commit(b_empty((nb + s) % B_STAGES));
                nb += it.nsub;
            }
        }
        __syncwarp();
    } else if (warp < W_EPI) {
        // ---- query gather: the item's sub-tiles alternate between the gather warps; lane l fills rows l, l + 32
        const int gw = warp - W_GATHER;
        int nb = 0;
        for (int n = 0;; n++) {
            Item it;
            if (!read_item(n, it, true)) break;
            if (lane == 0) mbar_arrive(i_empty(n % I_STAGES));
            if (it.nsub == 0) break;
            bool ok = true;
            for (int s = 0; s < it.nsub; s++, nb++) {
                if (nb % GATHER_WARPS != gw) continue;
                const int sb = nb % B_STAGES, sm = nb % MS;
                const int nq = min(QN, it.nq - s * QN);
                const int n16 = (nq + 15) & ~15;
                // the sub-tile's query ids and pair constants; its rows are copied with cp.async (all of them in flight
                // at once, zero rows past nq) while the scales and thresholds load and the metadata slot is filled
                int qq[2];
                float qcv[2], qsv[2], thv[2];
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    const int gq = lane + 32 * rr;
                    qq[rr] = gq < nq ? p.qid[it.qoff + s * QN + gq] : -1;
                    qcv[rr] = gq < nq ? p.qcp[it.qoff + s * QN + gq] : 0.f;
                }
                if (!warp_wait(b_empty(sb), ((nb / B_STAGES) & 1) ^ 1, abort, WL)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    const int gq = lane + 32 * rr;
                    if (gq >= n16) continue;
                    const int q = qq[rr];
                    const uint4* src = reinterpret_cast<const uint4*>(p.q8 + (int64_t)(q >= 0 ? q : 0) * RB);
                    const uint32_t bs = sbase + B_OFF + sb * B_BYTES + (gq >> 3) * 1024 + (gq & 7) * 128;
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int cc = 0; cc < 8; cc++)
                            cp_async16(bs + h * QN * 128 + ((cc ^ (gq & 7)) << 4), src + 8 * h + cc, q >= 0);
                }
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    qsv[rr] = qq[rr] >= 0 ? p.qs[qq[rr]] : 0.f;
                    thv[rr] = (MODE && qq[rr] >= 0) ? p.t0[qq[rr]] : 0.f;
                }
                if (!warp_wait(m_empty(sm), ((nb / MS) & 1) ^ 1, abort, WL)) {
                    cp_async_wait_all();  // no copy into shared memory stays in flight
                    ok = false;
                    break;
                }
                int* mq = meta(sm);
                float* msc = reinterpret_cast<float*>(mq + QN);
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    const int gq = lane + 32 * rr;
                    mq[gq] = qq[rr];
                    msc[gq] = qsv[rr];
                    msc[QN + gq] = qcv[rr];
                    msc[2 * QN + gq] = thv[rr];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(m_full(sm));
                cp_async_wait_all();
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(b_full(sb));
            }
            if (!ok) break;
        }
    } else {
        // ---- epilogue: group eg takes the units nu = eg (mod EPI_GROUPS); warp ew = warp % 4 reads TMEM lanes
        //      32*ew .. 32*ew+31 (tile rows)
        const int we = warp - W_EPI;
        const int eg = we / 4;
        const int ew = warp & 3;
        uint32_t* colm = reinterpret_cast<uint32_t*>(smem + COL_OFF) + we * 64;
        int* colb = reinterpret_cast<int*>(colm + 32);
        int nu = 0, nb = 0;
        for (int n = 0;; n++) {
            Item it;
            if (!read_item(n, it, true)) break;
            if (lane == 0) mbar_arrive(i_empty(n % I_STAGES));
            if (it.nsub == 0) break;
            bool ok = true;
            for (int t = 0; t < it.ntiles && ok; t++) {
                const int row0 = it.first + t * TILE_ROWS;
                const int row = row0 + 32 * ew + lane;
                const bool rvalid = row >= it.cs && row < it.ce;
                const bool wactive = row0 + 32 * ew < it.ce;
                const int blk_rel = (row0 + 32 * ew) / 32 - it.cs / 32;
                for (int s = 0; s < it.nsub; s++, nu++) {
                    if (nu % EPI_GROUPS != eg) continue;
                    const int st = nu % T_STAGES;
                    const int nq = min(QN, it.nq - s * QN);
                    const int pair0 = it.qoff + s * QN;
                    const int sm = (nb + s) % MS;
                    const float zr = rvalid ? p.zs[row] : 0.f;  // loaded before the waits
                    if (!warp_wait(m_full(sm), ((nb + s) / MS) & 1, abort, WL) ||
                        !warp_wait(t_full(st), (nu / T_STAGES) & 1, abort, WL)) {
                        ok = false;
                        break;
                    }
                    const int* mq = meta(sm);
                    const float* ms = reinterpret_cast<const float*>(mq + QN);
                    const float* mc = ms + QN;
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
                        const float4* ms4 = reinterpret_cast<const float4*>(ms + 32 * h);
                        const float4* mc4 = reinterpret_cast<const float4*>(mc + 32 * h);
                        if (MODE == 0) {
#pragma unroll
                            for (int j4 = 0; j4 < 8; j4++) {
                                if (4 * j4 >= nc) break;
                                const float4 sv = ms4[j4], cv = mc4[j4];
                                const float s4[4] = {sv.x, sv.y, sv.z, sv.w}, c4[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
                                for (int u = 0; u < 4; u++) {
                                    const int jj = 4 * j4 + u;
                                    if (jj < nc) {
                                        const float est =
                                            __fadd_rn(__fmul_rn(__fmul_rn((float)(int32_t)acc[jj], s4[u]), zr), c4[u]);
                                        const uint32_t m = __reduce_max_sync(0xffffffffu, rvalid ? f2o(est) : 0u);
                                        if (lane == 0) p.bmc[(int64_t)(pair0 + 32 * h + jj) * p.MB + blk_rel] = o2f(m);
                                    }
                                }
                            }
                        } else {
                            const float4* mt4 = reinterpret_cast<const float4*>(mt + 32 * h);
                            uint32_t rowmask = 0;
#pragma unroll
                            for (int j4 = 0; j4 < 8; j4++) {
                                if (4 * j4 >= nc) break;
                                const float4 sv = ms4[j4], cv = mc4[j4], tv = mt4[j4];
                                const float s4[4] = {sv.x, sv.y, sv.z, sv.w}, c4[4] = {cv.x, cv.y, cv.z, cv.w};
                                const float t4[4] = {tv.x, tv.y, tv.z, tv.w};
#pragma unroll
                                for (int u = 0; u < 4; u++) {
                                    const int jj = 4 * j4 + u;
                                    if (jj < nc) {
                                        const float est =
                                            __fadd_rn(__fmul_rn(__fmul_rn((float)(int32_t)acc[jj], s4[u]), zr), c4[u]);
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
                        // the sub-tile's units (one per tile) are spread over the warpgroups, which finish in any
                        // order: the slot is free once all 4 * ntiles warps are done with it; the last one to count
                        // itself resets the count and releases the slot
                        __threadfence_block();
                        int* mcount = reinterpret_cast<int*>(smem + MCNT_OFF);
                        if (atomicAdd(mcount + sm, 1) == 4 * it.ntiles - 1) {
                            mcount[sm] = 0;
                            mbar_arrive(m_empty(sm));
                        }
                    }
                }
            }
            if (!ok) break;
            nb += it.nsub;
        }
    }
    // drain (waits that ignore the abort flag): the most recent load of every A stage has landed, and one commit
    // after the last MMA issued has arrived, i.e. every MMA of this CTA has completed
    if (warp == W_TMA && lane == 0)
        for (int u = na_load - 1; u >= 0 && u >= na_load - A_STAGES; u--)
            mbar_drain(a_full(u % A_STAGES), (u / A_STAGES) & 1);
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

// Compact lists of the cells a pass visits, in the order given (largest first): cells with ccnt1 > 0 (first pass) and
// with ccnt > 0 (emit pass).  One CTA; nlist[0], nlist[1] = the lengths; zero[0..nzero) is cleared on the way (the
// emit pass's counters, so that they need no fill of their own).
__global__ void __launch_bounds__(1024) cell_lists_kernel(const int32_t* __restrict__ order, int NC,
                                                          const int32_t* __restrict__ ccnt1,
                                                          const int32_t* __restrict__ ccnt, int32_t* __restrict__ list1,
                                                          int32_t* __restrict__ list, int32_t* __restrict__ nlist,
                                                          int32_t* __restrict__ zero, int nzero) {
    __shared__ int wsum[2][32];
    __shared__ int base[2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < nzero; i += 1024) zero[i] = 0;
    if (tid == 0) base[0] = base[1] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < NC; c0 += 1024) {
        const int i = c0 + tid;
        const int e = i < NC ? order[i] : -1;  // cell | part << 16
        const int c = e >= 0 ? (e & 0xffff) : -1;
        const bool k1 = c >= 0 && ccnt1 && ccnt1[c] > 0;
        const bool k2 = c >= 0 && ccnt[c] > 0;
        const unsigned m1 = __ballot_sync(0xffffffffu, k1), m2 = __ballot_sync(0xffffffffu, k2);
        if (lane == 0) {
            wsum[0][warp] = __popc(m1);
            wsum[1][warp] = __popc(m2);
        }
        __syncthreads();
        int b1 = base[0], b2 = base[1], t1 = 0, t2 = 0;
        for (int w = 0; w < 32; w++) {
            if (w < warp) {
                b1 += wsum[0][w];
                b2 += wsum[1][w];
            }
            t1 += wsum[0][w];
            t2 += wsum[1][w];
        }
        const unsigned below = (1u << lane) - 1u;
        if (k1) list1[b1 + __popc(m1 & below)] = e;
        if (k2) list[b2 + __popc(m2 & below)] = e;
        __syncthreads();
        if (tid == 0) {
            base[0] += t1;
            base[1] += t2;
        }
        __syncthreads();
    }
    if (tid == 0) {
        nlist[0] = base[0];
        nlist[1] = base[1];
    }
}

}  // namespace cells
}  // namespace fvs

extern "C" int fvs_cell_lists(fvs_stream_t stream, const int32_t* order, int NC, const int32_t* ccnt1,
                              const int32_t* ccnt, int32_t* list1, int32_t* list, int32_t* nlist, int32_t* zero,
                              int nzero) {
    FVS_CHECK_ARG(order && ccnt && list && nlist && NC > 0 && nzero >= 0);
    FVS_CHECK_ARG(ccnt1 == nullptr || list1 != nullptr);
    FVS_CHECK_ARG(nzero == 0 || zero != nullptr);
    fvs::cells::cell_lists_kernel<<<1, 1024, 0, stream>>>(order, NC, ccnt1, ccnt, list1, list, nlist, zero, nzero);
    return fvs_launch_status();
}

extern "C" int fvs_cell_part_tiles(void) { return FVS_CELL_PART_TILES; }

extern "C" int fvs_i8_scan_cells(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                                 const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                                 const int32_t* list, const int32_t* nlist, int maxlist, const int64_t* off, int NC,
                                 const int8_t* Z, int64_t N, const float* zs, const float* t0, int32_t* cnt,
                                 float* bval, int32_t* bpos, int M, float* bmc, int MB, int32_t* sched,
                                 int32_t* status) {
    using namespace fvs::cells;
    FVS_CHECK_ARG(mode == 0 || mode == 1);
    FVS_CHECK_ARG(R == RB && B >= 0 && maxlist >= 0 && NC > 0 && N > 0);
    FVS_CHECK_ARG(q8 && qs && qid && coff && ccnt && qcp && list && nlist && off && Z && zs && sched);
    FVS_CHECK_ARG(((uintptr_t)Z & 15) == 0 && ((uintptr_t)q8 & 15) == 0);
    if (mode == 0) FVS_CHECK_ARG(bmc && MB > 0);
    if (mode == 1) FVS_CHECK_ARG(t0 && cnt && bval && bpos && M > 0);
    if (maxlist == 0 || B == 0) return FVS_OK;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    ZMaps zm;
    const cuuint64_t dims[2] = {(cuuint64_t)RB, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)RB};
    const cuuint32_t estr[2] = {1, 1};
    for (int k = 0; k < 4; k++) {
        const cuuint32_t box[2] = {128, (cuuint32_t)(32 * (k + 1))};  // one K-half of k + 1 32-row blocks
        CUresult cr = enc(&zm.m[k], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)Z, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return FVS_EINVAL;
    }
    Params p{q8, qs, qid, coff, ccnt, qcp, list, nlist, off, zs, t0, cnt, bval, bpos, bmc, sched, status, M, MB,
             pipeline_wait_limit()};
    cudaError_t e = mode ? fvs_ensure_smem((const void*)scan_cells_kernel<1>, Layout<1>::SMEM_BYTES)
                         : fvs_ensure_smem((const void*)scan_cells_kernel<0>, Layout<0>::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    const int nsm = fvs_sm_count();
    const int slots = nsm * (mode ? Layout<1>::CTAS_PER_SM : Layout<0>::CTAS_PER_SM);  // persistent CTAs
    const int grid = maxlist < slots ? maxlist : slots;
    if (mode == 0)
        scan_cells_kernel<0><<<grid, Layout<0>::NTHREADS, Layout<0>::SMEM_BYTES, stream>>>(zm, p);
    else
        scan_cells_kernel<1><<<grid, Layout<1>::NTHREADS, Layout<1>::SMEM_BYTES, stream>>>(zm, p);
    return fvs_launch_status();
}
