/*
 * libfanar_b200 -- the C ABI of the B200 (sm_100a) query path of FanarVSE.
 *
 * Conventions (all entry points):
 *   - every pointer argument is a DEVICE pointer unless the comment says "host"; the caller allocates every buffer;
 *   - kernels are enqueued on `stream` (a cudaStream_t); no entry point allocates, synchronises or reads device memory
 *     on the host, so every call can be captured into a CUDA graph;
 *   - return 0 on success, a negative FVS_E* code for a bad argument, or a positive cudaError_t from the launch;
 *   - data conditions are not errors: overflow / underflow of the emit buffer is reported through cnt / ok exactly as
 *     the reference reports it (`throughput/enginei8.py:60`), and handled by the caller's recompute path.
 * Index layout is the reference's (sorted-position order; see `throughput/enginei8.py:19-27`, `src/tiered.py:29-44`).
 */
#ifndef FANAR_B200_H
#define FANAR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fvs_stream_t; /* == cudaStream_t */

#define FVS_OK 0
#define FVS_EINVAL (-1)   /* null pointer, negative size, unsupported shape */
#define FVS_ERANGE (-2)   /* a size above what the kernel supports (e.g. K > 4096) */

/* Library version (major*10000 + minor*100 + patch) and build target ("sm_100a"). */
int fvs_version(void);
const char* fvs_arch(void);

/*
 * Polls allowed to each pipeline wait (an mbarrier wait between the roles of a CTA) of the tcgen05 kernels
 * (fvs_i8_scan_tc, fvs_dense_scan_tc) launched from now on in this process; returns the previous value.  No
 * counterpart in the reference (its Triton kernels have no waits of their own).  When a wait's polls run out, the
 * CTA stops its work, waits (with the default limit, whatever this setting) for the copies and MMAs it already issued,
 * frees its tensor memory, sets the call's `status` word to 1 and returns: the search raises instead of hanging.
 * This knob exists so that tests can make that path run (0: every pipeline wait gives up at once); production code
 * leaves it at FVS_WAIT_LIMIT_DEFAULT.  Takes effect at launch, so a captured graph keeps the value it was captured with.
 */
#define FVS_WAIT_LIMIT_DEFAULT 4194304u
uint32_t fvs_set_wait_limit(uint32_t polls);

/*
 * Per-batch query preparation in one pass over the fp32 queries Q [B, ldq]: Qh [B, d] = fp16(Q) (round to nearest
 * even: the `Qb.half()` operand of the routing and rotation products, `throughput/enginei8.py:67`,
 * `throughput/s2lut.py:122`) and qc[q] = <Q[q, :d], c> in fp32 (`QC = Qb @ s1["c"]`, `throughput/enginei8.py:63`;
 * summation order differs from the BLAS product).  qc may be NULL.  d % 4 == 0; Q, c 16-byte aligned, Qh 8-byte.
 */
int fvs_query_prep(fvs_stream_t stream, const float* Q, int B, int d, int ldq, const float* c, uint16_t* Qh,
                   float* qc);

/*
 * Query quantisation (`throughput/enginei8.py:38`): qs[q] = max(max_r |z[q,r]|, 1e-12) / 127,
 * q8[q,r] = clamp(round_half_even(z[q,r] / qs[q]), -127, 127); z [B, ldz] f32 = Q @ Vr.
 */
int fvs_quantize(fvs_stream_t stream, const float* z, int B, int R, int ldz, int8_t* q8, float* qs);

/*
 * Routing selection (`throughput/enginei8.py:67-68`, `QM.topk(nprobe, 1).indices`): probe[q, :] = the nprobe cells of
 * largest fp16 score QM[q, :] (QM [B, NC] fp16, the routing product q . m_c / |m_c|), ordered by (score desc, cell asc).
 * NC <= 65535, nprobe <= 4096.
 */
int fvs_route_topk(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int64_t* probe);

/*
 * Pair list by cell (`throughput/enginei8.py:11-16`, `pairs_fast`) over the first ncols columns of probe [B, nprobe]:
 * ccnt[c] = #pairs in cell c, coff = exclusive prefix of ccnt, qid[coff[c] .. coff[c]+ccnt[c]) = the queries probing c,
 * qcp[i] = float(QM[qid, c]) * mnorm[c] (mnorm nullable: 1), slot[q*ncols + j] = position of pair (q, j) (nullable).
 * work: NC int32 of scratch.  The order of queries within a cell is unspecified.
 */
int fvs_pairs(fvs_stream_t stream, const int64_t* probe, int B, int nprobe, int ncols, int NC, const uint16_t* QM,
              const float* mnorm, int32_t* qid, int32_t* coff, int32_t* ccnt, float* qcp, int32_t* slot,
              int32_t* work);

/*
 * Both pair lists of the int8 stage 1 (`throughput/enginei8.py:42,56`: `pairs_fast` over the first n1 columns for
 * the first pass, over all nprobe columns for the emit pass) as ONE list by cell over all nprobe columns, in which
 * each cell's pairs from columns < n1 come first: ccnt[c] = #pairs in cell c, ccnt1[c] = #of them from columns < n1,
 * coff = exclusive prefix of ccnt, qid / qcp as fvs_pairs, slot[q*n1 + j] (j < n1) = position of pair (q, j).  The
 * first pass reads (coff, ccnt1), the emit pass (coff, ccnt); one histogram, scan and scatter serve both.
 * 1 <= n1 <= nprobe.  work: 2*NC int32 of scratch.
 */
int fvs_pairs_split(fvs_stream_t stream, const int64_t* probe, int B, int nprobe, int n1, int NC, const uint16_t* QM,
                    const float* mnorm, int32_t* qid, int32_t* coff, int32_t* ccnt, int32_t* ccnt1, float* qcp,
                    int32_t* slot, int32_t* work);

/*
 * fvs_pairs without the `work` argument, for callers that cannot allocate device memory: host programs that drive
 * the search through a foreign-function binding and own no CUDA allocator, or plugins inside another application
 * (a database engine, a serving process) whose device memory belongs to that application's own pool and may not be
 * taken behind its back with cudaMalloc.  No counterpart in the reference (its pairing is torch code that
 * allocates freely).  The per-cell scratch is a file-scope device array of FVS_PAIRS_NOALLOC_MAX_CELLS int32 inside
 * this library, held on every GPU that loads the library until the process exits; NC above that returns FVS_ERANGE.
 * This call allocates nothing: it clears the part of the array it uses, then runs the same kernels as fvs_pairs.
 * The first call on a device looks up the array's device address (once per device): make it before capturing a
 * stream.  All calls share the one array, so calls whose kernels overlap on the GPU (concurrent streams, other host
 * threads) race on it and must be serialised by the caller.
 */
#define FVS_PAIRS_NOALLOC_MAX_CELLS 65536
int fvs_pairs_noalloc(fvs_stream_t stream, const int64_t* probe, int B, int nprobe, int ncols, int NC,
                      const uint16_t* QM, const float* mnorm, int32_t* qid, int32_t* coff, int32_t* ccnt, float* qcp,
                      int32_t* slot);

/*
 * Cell parts: the cell-major scans (fvs_i8_scan_cells, fvs_trellis_scan_cells) take their work from lists whose
 * entries are `cell | part << 16`: part p of a cell covers its 128-row tiles p*FVS_CELL_PART_TILES ..
 * (p+1)*FVS_CELL_PART_TILES - 1 (tiles start at the cell's first 32-row block), so that several CTAs share a large
 * cell.  An order that lists every cell once with part 0 (plain cell ids) is a valid order for cells of at most
 * FVS_CELL_PART_TILES tiles.  Cell ids below 65536.
 */
#define FVS_CELL_PART_TILES 8
int fvs_cell_part_tiles(void);

/*
 * Routing selection and both pair lists in two launches (replaces fvs_route_topk + fvs_pairs_split + fvs_cell_lists
 * on the throughput path: the reference's `QM.topk(nprobe)` and `pairs_fast`, `throughput/enginei8.py:11-16, 67-70`).
 * probe [B, nprobe] as fvs_route_topk; qid / qcp / coff / ccnt / ccnt1 / slot as fvs_pairs_split with first-pass
 * columns j < n1; when order is given (norder cell-part entries, largest cells first), list1 / list / nlist as
 * fvs_cell_lists (list capacity norder).  zero[0..nzero)
 * is cleared.  work: 2*NC + 1 int32 that are zero before the first call; every call leaves them zero (a call's cursors
 * are cleared by its last CTA), so calls on one stream can share them.  NC % 8 == 0, NC <= 16384, nprobe <= 512, QM
 * 16-byte aligned; other shapes return FVS_ERANGE (the three separate entry points take them).
 */
int fvs_route_pairs(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int n1, const float* mnorm,
                    const int32_t* order, int norder, int64_t* probe, int32_t* qid, float* qcp, int32_t* coff,
                    int32_t* ccnt, int32_t* ccnt1, int32_t* slot, int32_t* list1, int32_t* list, int32_t* nlist,
                    int32_t* zero, int nzero, int32_t* work);

/*
 * fvs_route_pairs with a per-cell routing scale: the nprobe cells of largest float(QM[q, c]) * sc[c] (fp32 product,
 * ties by smaller cell), as fvs_route_topk_scaled (the default engine's routing `(QM.float() * inv_mnorm).topk(nprobe)`,
 * `src/engine_cell.py:40-42`), then the pair lists, cell lists and cleared counters exactly as fvs_route_pairs (pair
 * constant float(QM[q, c]) * mnorm[c], or float(QM[q, c]) when mnorm is NULL: the default engine's `_pairs_static`
 * for both passes, `src/s1cell.py:170-175, 184, 192`).  sc 16-byte aligned; the other conditions and the work buffer
 * as fvs_route_pairs.
 */
int fvs_route_pairs_scaled(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, int n1, const float* sc,
                           const float* mnorm, const int32_t* order, int norder, int64_t* probe, int32_t* qid,
                           float* qcp, int32_t* coff, int32_t* ccnt, int32_t* ccnt1, int32_t* slot, int32_t* list1,
                           int32_t* list, int32_t* nlist, int32_t* zero, int nzero, int32_t* work);

/* Rows per tile of the int8 scan (a multiple of the reference's 32-row block).  Host-side helper. */
int fvs_i8_tile_rows(void);

/*
 * Int8 stage-1 scan over the probed cells: first pass (mode 0) or threshold emit (mode 1).
 * Replaces the Triton kernels `_first8c` / `_emit8c` (`throughput/ivf8c_kern.py:2-36`) and the CUDA WMMA kernel
 * `ivf8` (`throughput/civf8.py:15-91`, launched by `civf8.launch(mode, P, q8, qs, qid, coff, ccnt, pcell, pblk, ps, pe,
 * Z, zs, qcp, t0, cnt, bval, bpos, bmc, CAP, MB)`).
 *   q8 [B,R] int8, qs [B]           quantised queries and their scales (`throughput/enginei8.py:38`)
 *   qid, qcp [npairs]; coff, ccnt [NC]  pairs sorted by cell (`throughput/enginei8.py:11-16`)
 *   tile_cell, tile_row0 [ntiles]   static work list: tiles of fvs_i8_tile_rows() rows of one cell, row0 a multiple of 32
 *   off [NC+1] int64                cell boundaries in sorted positions
 *   Z [N,R] int8, zs [N] f32        stage-1 codes and scales
 *   mode 0: bmc[(coff[c]+i)*MB + (blk - off[c]/32)] = max over the cell's rows of global 32-row block blk of
 *           est = ((float(q8.z) * qs) * zs) + qcp; slots of blocks a cell does not have are not written.
 *   mode 1: every (q, n) with est >= t0[q]: i = atomicAdd(cnt[q], 1); if i < M: bval[q*M+i] = est, bpos[q*M+i] = n.
 *   R must be 256.  Unused outputs of a mode may be NULL.
 */
int fvs_i8_scan(fvs_stream_t stream, int mode,
                const int8_t* q8, const float* qs, int B, int R,
                const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                const int32_t* tile_cell, const int32_t* tile_row0, int ntiles,
                const int64_t* off, int NC,
                const int8_t* Z, const float* zs,
                const float* t0, int32_t* cnt, float* bval, int32_t* bpos, int M,
                float* bmc, int MB);

/*
 * fvs_i8_scan on the 5th-generation tensor cores (tcgen05.mma.kind::i8, TMEM accumulators, TMA-staged code tiles).
 * Same inputs, outputs and semantics as fvs_i8_scan, plus N (rows of Z, for the tensor map; Z and q8 16-byte aligned)
 * and status (nullable): set to 1 if a bounded internal wait expired (the outputs of that launch are then incomplete).
 */
int fvs_i8_scan_tc(fvs_stream_t stream, int mode,
                   const int8_t* q8, const float* qs, int B, int R,
                   const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                   const int32_t* tile_cell, const int32_t* tile_row0, int ntiles,
                   const int64_t* off, int NC,
                   const int8_t* Z, int64_t N, const float* zs,
                   const float* t0, int32_t* cnt, float* bval, int32_t* bpos, int M,
                   float* bmc, int MB, int32_t* status);

/*
 * First-pass threshold (`throughput/enginei8.py:53-55`): t0[q] = the r-th largest block maximum over the blocks of the
 * n1 first-pass cells probe[q*nprobe + j] (j < n1) of query q, read at bmc[slot[q*n1+j]*MB + b]; the smallest one if
 * there are fewer than r; 1e30 if none.  slot[q*n1+j] is the cell-sorted position of pair (q, j) (`inv` in the
 * reference).
 */
int fvs_threshold(fvs_stream_t stream, const float* bmc, int MB, const int32_t* slot,
                  const int64_t* probe, int nprobe, int n1, const int64_t* off, int B, int r, float* t0);

/*
 * Stage-1 top-K and exactness flag (`throughput/enginei8.py:60`, `bval.topk(K)` + `K <= cnt <= M`) fused with the
 * delta rule (`throughput/enginei8.py:87-90`).  Per query: the K best of the first min(cnt, M) buffer entries by
 * (est desc, pos asc), written sorted; slots beyond cnt read as (-1e30, position 0) as the reference's initialised
 * buffers do.  ok[q] = K <= cnt[q] <= M.  If ncnt != NULL: ncnt[q] = #{i : est1[q,i] >= est1[q,delta_idx] - delta}.
 * K <= 4096.
 */
int fvs_select_topk(fvs_stream_t stream, const float* bval, const int32_t* bpos, const int32_t* cnt, int B, int M,
                    int K, int64_t* pos, float* est1, uint8_t* ok, int32_t* ncnt, float delta, int delta_idx);

/*
 * Per-query nibble lookup tables (`throughput/s2lut.py:108-126`, `_lut_kernel` + `luts_fused`):
 *   L[q, n*16 + v] = sum_{i<4} Zq[q, 4n+i] * ((v >> (3-i)) & 1) over the leading D coordinates (fp16 if half else f32),
 *   qsum[t*B+q] = sum Zq[q, s_t:e_t], qn2[t*B+q] = sum Zq[q, s_t:e_t]^2 for the T tiers (host arrays tier_s / tier_e).
 */
int fvs_lut_build(fvs_stream_t stream, const float* Zq, int B, int ldz, int D, int half, void* L,
                  int T, const int32_t* tier_s, const int32_t* tier_e, float* qsum, float* qn2);

/*
 * LUT-scored tiered refinement (`throughput/s2lut.py:48-106`, `_score_lut` / `_tier_lut`).  For candidate i of query q
 * (row n = pos[q*K+i]; live if i < ncnt[q], or all when ncnt == NULL):
 *   est = qc[q] + sum_t delta_t (sum_p 2^(b_t-1-p) sum_j (L[2j][hi(byte)] + L[2j+1][lo(byte)]) - mid_t qsum[t,q])
 *                   * scale[t*N+n],      sd = sqrt(sum_t qn2[t,q] sig[t*N+n]^2);   dead: est = -1e30, sd = 0.
 * Host arrays of length T: tier_s, tier_e, tier_bits, tier_delta, tier_planes (device pointers to planes_t
 * [b_t, N, (e_t-s_t)/8] uint8).  T <= 8.
 */
int fvs_lut_score(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc,
                  const void* L, int half, int LW, int T, const int32_t* tier_s, const int32_t* tier_e,
                  const int32_t* tier_bits, const float* tier_delta, const uint8_t* const* tier_planes,
                  const uint16_t* scale, const uint16_t* sig, int64_t N, const float* qsum, const float* qn2,
                  const int32_t* ncnt, float* est, float* sd);

/*
 * fvs_lut_score with the table built in shared memory: takes the rotated tier query Zq [B, ldz] (the input of
 * fvs_lut_build) instead of L/qsum/qn2, and computes the same est / sd (same fp16 / f32 table rounding).  Zq is f32, or
 * with zq_half = 1 the fp16 product `Qb.half() @ VP16` itself (`throughput/s2lut.py:122` takes its .float(): the same
 * values, without the conversion pass); ldz % 4 == 0, Zq 16-byte aligned.  Tiers must be contiguous from coordinate 0
 * with widths multiples of 32 (the reference's 32-dim allocation groups, `src/tiered.py:19-27`).  Replaces
 * `luts_fused` + `score_lut` (`throughput/s2lut.py:92-126`) in one launch.
 */
int fvs_lut_score_zq(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const void* Zq, int ldz,
                     int zq_half, int D, int half, int T, const int32_t* tier_s, const int32_t* tier_e, const int32_t* tier_bits,
                     const float* tier_delta, const uint8_t* const* tier_planes, const uint16_t* scale,
                     const uint16_t* sig, int64_t N, const int32_t* ncnt, float* est, float* sd);

/*
 * Classification, exact re-rank and final top-k (`throughput/enginei8.py:92-95`, `src/engine3.py:143-146`,
 * `src/stage3_zc.py:11-27`):  lo/hi = est -/+ z*sd;  sure = lo > (k+1)-th largest hi;  amb = hi >= k-th largest lo
 * and not sure;  score = est + 10 if sure, the exact fp32 dot <H[id], Q[q]> of the fp16 row id = order[pos] if
 * ambiguous, -1e9 otherwise;  I[q] = the k ids of largest score (ties by smaller id).
 * Outputs: ids [B,K] (candidate ids, int32), I [B,k] int32, reads [B] int32 (#ambiguous), score_k [B,k] (nullable).
 * H [Nfull, d] fp16 in original-id order; d a multiple of 8.  K <= 4096, k <= 256.
 */
int fvs_refine(fvs_stream_t stream, const uint16_t* H, int d, const int32_t* order, const int64_t* pos,
               const float* est, const float* sd, int B, int K, float z, int k, const float* Q, int ldq,
               int32_t* ids, int32_t* I, int32_t* reads, float* score_k);

/*
 * Exact fp32 inner products of given rows: score[q*k+i] = <H[ids[q*k+i]], Q[q]> (fp16 rows, fp32 accumulate), as the
 * exact read of `src/stage3_zc.py:11-22` but for every listed id.  Used by the row-sharded search so that each shard's
 * local top-k carries exact scores before the cross-shard merge (a "sure" candidate is ranked by est + 10 without a
 * read, `src/engine3.py:144-145`, which is not comparable across shards).  ids < 0 give -1e30.
 */
int fvs_exact_scores(fvs_stream_t stream, const uint16_t* H, int d, const int32_t* ids, int B, int k, const float* Q,
                     int ldq, float* score);

/*
 * Query codes of the int8 stage 1 (`throughput/enginei8.py:38`: z = Q @ Vr, qs = max|z| / 127,
 * q8 = clamp(round(z / qs), +-127), the rounding and clamp of fvs_quantize): z is computed on the tensor cores as
 * three TF32 products (Q and Vr each split into a TF32 part and an exact remainder; error ~2^-21 relative per product,
 * fp32 accumulation), split over K into ks_max x B x R partial sums in `part` (16-byte aligned; a fixed-order sum then
 * quantises each row).  vt_big / vt_small: Vr transposed [R, d] row-major, vt_big = Vr^T with the low 13 mantissa bits
 * cleared, vt_small = Vr^T - vt_big.  R = 256, d % 4 == 0, ldq % 4 == 0, Q 16-byte aligned.  `status` as
 * fvs_i8_scan_tc.
 */
int fvs_project_quantize(fvs_stream_t stream, const float* Q, int B, int d, int ldq, const float* vt_big,
                         const float* vt_small, int R, int8_t* q8, float* qs, float* part, int ks_max,
                         int32_t* status);

/* Rows per work tile of fvs_trellis_scan (tiles start on the cell's first global 32-row boundary). */
int fvs_trellis_tile_rows(void);

/*
 * The int8 stage-1 scan organised by cells (same contract and results as fvs_i8_scan_tc; replaces the same reference
 * kernels, `throughput/ivf8c_kern.py:2-36`): the CTAs take the cell parts of `list` (nlist[0] entries
 * `cell | part << 16`, a device count; see FVS_CELL_PART_TILES) one at a time with an atomicAdd on sched[0]; a part's
 * queries (the cell's) are gathered once and held while its code tiles are scanned; a tile is fetched as the 32-row
 * blocks the cell occupies.  maxlist >= the count (sizes the grid: the list's capacity).
 * sched: 2 int32, zero before the first launch; every launch leaves them zero (the last CTA resets them), so calls on
 * one stream can share them, while calls that may run at the same time need their own.  Other arguments as
 * fvs_i8_scan_tc (mode 0 reads the first pass's per-cell counts, mode 1 the emit pass's).
 */
int fvs_i8_scan_cells(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                      const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                      const int32_t* list, const int32_t* nlist, int maxlist, const int64_t* off, int NC,
                      const int8_t* Z, int64_t N, const float* zs, const float* t0, int32_t* cnt, float* bval,
                      int32_t* bpos, int M, float* bmc, int MB, int32_t* sched, int32_t* status);

/*
 * The work lists of fvs_i8_scan_cells for both passes (new; the reference launches one program per (cell, block)):
 * the entries of `order` [NC] (cell-part entries, see FVS_CELL_PART_TILES: every part of every cell once, largest
 * cells first) whose cell c has ccnt1[c] > 0 into list1 and ccnt[c] > 0 into list, in that order; nlist[0], nlist[1]
 * = their lengths (device), the lists' capacity NC entries.  ccnt1 may be NULL (no list1).
 * zero[0..nzero) is set to 0 in the same launch (the emit pass's per-query counters; zero may be NULL when nzero = 0).
 */
int fvs_cell_lists(fvs_stream_t stream, const int32_t* order, int NC, const int32_t* ccnt1, const int32_t* ccnt,
                   int32_t* list1, int32_t* list, int32_t* nlist, int32_t* zero, int nzero);

/*
 * Small-batch int8 scan (B <= 32): same contract and arithmetic as fvs_i8_scan_tc, streamed from HBM with 16-byte loads
 * and dp4a, one CTA per (query, probe column, 4 blocks), taking the work straight from probe [B, nprobe] (columns
 * 0..ncols-1) without a pair list: the pair constant is float(QM[q, c]) * mnorm[c] (mnorm may be NULL: the constant is
 * float(QM[q, c])) and mode 0 writes bmc[(q * ncols + j) * MB + blk - cs/32] (pair slot q * ncols + j, so
 * fvs_threshold takes slot[i] = i).  Replaces `_first8c` / `_emit8c` (`throughput/ivf8c_kern.py:2-36`) for batches where
 * a cell is probed by one or two queries.
 */
int fvs_i8_scan_small(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R,
                      const int64_t* probe, int nprobe, int ncols, const uint16_t* QM, int NC, const float* mnorm,
                      const int64_t* off, const int8_t* Z, const float* zs, const float* t0, int32_t* cnt, float* bval,
                      int32_t* bpos, int M, float* bmc, int MB);

/*
 * Default engine, stage 1 (`src/s1cell.py:121-154`, `_first_compact_s` / `_emit_loop_s`): same contract as
 * fvs_i8_scan with the score est = scale1[n] * dot(Qh[q], v_n) + qcp, where v_n is row n's trellis code decoded as
 * `src/decode2.py:5-17` (words [N, W] uint32, bits MSB-first; value = tab[L-bit window], rounded to fp16) and
 * Qh [B, 256] = fp16(Q @ W1); fp16 products accumulated in fp32 on the tensor cores.  R = 256, W >= ceil((R+L-1)/32).
 * mode 2 (the first pass of `search_mask`, `src/s1small_cell.py:44-71`, batches 9..32): block maxima merged into
 * bmc[q * MB + global 32-row block] by atomic max, MB then being the blocks per query row (ceil(N / 32)).
 */
int fvs_trellis_scan(fvs_stream_t stream, int mode, const uint16_t* Qh, int B, int R,
                     const int32_t* qid, const int32_t* coff, const int32_t* ccnt, const float* qcp,
                     const int32_t* tile_cell, const int32_t* tile_row0, int ntiles, const int64_t* off, int NC,
                     const int32_t* words, int W, const float* tab, int L, const uint16_t* scale1,
                     const float* t0, int32_t* cnt, float* bval, int32_t* bpos, int M, float* bmc, int MB);

/*
 * fvs_trellis_scan modes 0 / 1 on the 5th-generation tensor cores, organised by cells (same contract and values;
 * replaces the same reference kernels, `src/s1cell.py:121-154` with `src/decode2.py:5-17`): the CTAs take the cells of
 * `list` (nlist[0] of them) with an atomicAdd on sched[0], gather a cell's queries once, decode each 128-row tile of the
 * cell in shared memory (fp16 values in the tensor cores' operand layout) and run tcgen05.mma.kind::f16 on it.  Lists,
 * maxlist and sched as fvs_i8_scan_cells (the lists come from fvs_cell_lists); status as fvs_i8_scan_tc.  L above
 * FVS_TRELLIS_CELLS_MAX_L returns FVS_ERANGE (fvs_trellis_scan takes it).
 */
#define FVS_TRELLIS_CELLS_MAX_L 10
int fvs_trellis_scan_cells(fvs_stream_t stream, int mode, const uint16_t* Qh, int B, int R, const int32_t* qid,
                           const int32_t* coff, const int32_t* ccnt, const float* qcp, const int32_t* list,
                           const int32_t* nlist, int maxlist, const int64_t* off, int NC, const int32_t* words, int W,
                           const float* tab, int L, const uint16_t* scale1, const float* t0, int32_t* cnt,
                           float* bval, int32_t* bpos, int M, float* bmc, int MB, int32_t* sched, int32_t* status);

/*
 * Default engine, stage 1 for B <= 8 (`src/s1small_cell.py:7-42`, `_small_scan` / `search_small`): est =
 * (sum_j tab[state_j] * Qr[q, j]) * scale1[n] + float(QM[q, c]) in fp32 (Qr = Q @ W1 in fp32, table values not rounded
 * to fp16), work taken straight from probe [B, nprobe] (columns 0..ncols-1): mode 0 merges the block maxima into
 * bm[q * NBg + global 32-row block] with an atomic max (bm filled with -1e30 by the caller, NBg = ceil(N / 32); the
 * reference's `tl.atomic_max` into bm [B, NB]), mode 1 appends est >= t0[q].  MB = ceil(largest cell / 32) + 1.
 */
int fvs_trellis_scan_small(fvs_stream_t stream, int mode, const float* Qr, int B, int R, const int64_t* probe,
                           int nprobe, int ncols, const uint16_t* QM, int NC, const int64_t* off, const int32_t* words,
                           int W, const float* tab, int L, const uint16_t* scale1, const float* t0, int32_t* cnt,
                           float* bval, int32_t* bpos, int M, float* bm, int NBg, int MB);

/*
 * Default engine, stage 2 (`src/tiered_fused.py:8-41, 54-72`): est = qc[q] + sum_t scale[t*N+n] * sum_x
 * cb_t[code_x] * Zq[q, x] over the tier's coordinates x (code_x from the tier's bit planes, plane p giving bit b-1-p),
 * sd = sqrt(sum_t ||Zq[q, s_t:e_t]||^2 * sig[t*N+n]^2); Zq = Q @ VP (f32).  Host arrays of length T: tier_s, tier_e,
 * tier_bits, tier_cb (device pointers to 2^b codebook levels), tier_planes.  T <= 8.
 */
int fvs_tiered_score(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const float* Zq, int ldz,
                     int D, int T, const int32_t* tier_s, const int32_t* tier_e, const int32_t* tier_bits,
                     const float* const* tier_cb, const uint8_t* const* tier_planes, const uint16_t* scale,
                     const uint16_t* sig, int64_t N, float* est, float* sd);

/*
 * Default engine routing (`src/engine_cell.py:40-42`): probe[q, :] = the nprobe cells of largest
 * float(QM[q, c]) * cell_scale[c] (QM fp16 = fp16(Q) @ means16^T, cell_scale = 1/|m_c|), ordered (score desc, cell asc).
 */
int fvs_route_topk_scaled(fvs_stream_t stream, const uint16_t* QM, int B, int NC, int nprobe, const float* cell_scale,
                          int64_t* probe);

/*
 * Index build (not the query path): Viterbi encoding of n segments Zs [n, R] f32 with the bitshift trellis (k = 1) of
 * `src/trellis_scan.py:21-32` (predecessors (s >> 1) | (u << (L-1)), emitted value vals[s], ties to u = 0 and to the
 * lowest final state) -> path [n, R] int32 of states.
 */
int fvs_viterbi_encode(fvs_stream_t stream, const float* Zs, int n, int R, const float* vals, int L, int32_t* path);

/*
 * Routing-free int8 scan (`throughput/brute.py:7-39`, `_scan`): the dense contraction of q8 [B, R] with every row code
 * Z [N, R] (int32 accumulate on the tensor cores), est[q, n] = (float(acc) * qs[q]) * float(zs[n]) (zs fp16).
 *   mode 0: out[q * ldo + n] = est (dense scores, used on the fixed row sample), ldo >= N
 *   mode 1: every n with est >= t0[q] is appended to query q's buffer (bval/bpos [B, M], counter cnt[q]; entries past M
 *           are counted, not stored), as MODE=1 of the reference.
 * R a multiple of 128 (<= 8192); q8 and Z 16-byte aligned; N < 2^31.  status: set to 1 if a bounded wait expired.
 */
int fvs_dense_scan_tc(fvs_stream_t stream, int mode, const int8_t* q8, const float* qs, int B, int R, const int8_t* Z,
                      const uint16_t* zs, int64_t N, const float* t0, int32_t* cnt, float* bval, int32_t* bpos, int M,
                      float* out, int64_t ldo, int32_t* status);

/*
 * out[q] = the r-th largest of vals[q * ld + 0 .. n-1] (`throughput/brute.py:56-57`: `scores(...).topk(r).values[:, -1]`),
 * 1 <= r <= n.
 */
int fvs_rth_largest(fvs_stream_t stream, const float* vals, int B, int n, int64_t ld, int r, float* out);

/*
 * fvs_lut_score_zq reading each candidate from its packed record instead of the separate planes / scale / sig arrays:
 * rec [N, RB] uint8 as `tiered_fused.pack` (`src/tiered_fused.py:112-125`) lays it out -- tier t plane p at byte
 * toff[t] + p * KB_t, then fp16 (scale, sigma) per tier at soff + 4t, RB a multiple of 16 (64 in the reference).  One
 * coalesced row read per candidate; same arithmetic and results as fvs_lut_score_zq.
 */
int fvs_lut_score_rec(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const void* Zq,
                      int ldz, int zq_half, int D, int half, int T, const int32_t* tier_s, const int32_t* tier_e,
                      const int32_t* tier_bits, const float* tier_delta, const uint8_t* rec, int RB, int soff,
                      int64_t N, const int32_t* ncnt, float* est, float* sd);

/*
 * fvs_tiered_score reading each candidate from its packed record (layout as fvs_lut_score_rec; the reference's
 * `score_rec` / `_tiered_score_rec`, `src/tiered_fused.py:74-111, 127-142`).
 */
int fvs_tiered_score_rec(fvs_stream_t stream, const int64_t* pos, int B, int K, const float* qc, const float* Zq,
                         int ldz, int D, int T, const int32_t* tier_s, const int32_t* tier_e,
                         const int32_t* tier_bits, const float* const* tier_cb, const uint8_t* rec, int RB, int soff,
                         int64_t N, float* est, float* sd);

/*
 * Compaction of flagged rows for a recompute inside the batch's own graph (new; the reference recomputes them from the
 * host, `throughput/enginei8.py:108-111`): rows[0..FB) = the first FB indices i with ok[i] == 0 in order (B for unused
 * slots), *nflag = the number of flagged rows; then row rows[s] (row 0 for an unused slot) of each of the G <= 8
 * arrays src[g] (row_bytes[g] bytes per row, a multiple of 4) is copied to row s of dst[g].  B >= 1, 1 <= FB <= 1024.
 */
int fvs_flagged_gather(fvs_stream_t stream, const uint8_t* ok, int B, int FB, int32_t* rows, int32_t* nflag, int G,
                       const void* const* src, void* const* dst, const int32_t* row_bytes);

/*
 * Inverse of fvs_flagged_gather's copies: for every slot s with 0 <= rows[s] < B, row s of src[g] goes to row rows[s] of
 * dst[g] for each array, and ok[rows[s]] = 1 (ok may be NULL).
 */
int fvs_rows_scatter(fvs_stream_t stream, const int32_t* rows, int FB, int B, uint8_t* ok, int G, const void* const* src,
                     void* const* dst, const int32_t* row_bytes);

/*
 * Exact top-k of each query over G shards' local top-k (new: the row-sharded multi-GPU search).
 * ids_g [G,B,kin] int64 global ids, score_g [G,B,kin] f32 -> I [B,k], S [B,k] by (score desc, id asc).  G*kin <= 4096.
 * Any int64 id is kept as given (ids of 2^32 and above, and -1 for "no result", come back unchanged).
 */
int fvs_merge_topk(fvs_stream_t stream, const int64_t* ids_g, const float* score_g, int G, int B, int kin, int k,
                   int64_t* I, float* S);

#ifdef __cplusplus
}
#endif
#endif /* FANAR_B200_H */
