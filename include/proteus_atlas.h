/*
 * proteus_atlas.h — C ABI of the B200 (sm_100a) streaming-atlas kernels.
 *
 * Plain pointers and sizes only: every pointer is CUDA device memory unless stated otherwise, and
 * every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream). The caller
 * owns every buffer; no entry point allocates or frees device memory, and none keeps a pointer
 * beyond the call. Return value: 0 on success, otherwise an ATLAS_ERR_* code with a message from
 * atlas_last_error(). Data never raises an error: candidate-buffer overflow is reported through the
 * device counters the reference uses (count > cap), exactly as filter_triton.py:66-68 does.
 *
 * Each entry point names the reference (haelyons/proteus) interface whose behaviour it provides.
 * Layouts of the atlas state are the reference's (atlas/core.py:173-196):
 *   top_s  f32 [G, K]   top_t i64 [G, K]   top_k i64 [G, K]   (G = L*2*D groups; sorted by top_k desc)
 *   res_s  i64 [G*B, Kr] (= -key)  res_t i64 [G*B, Kr]  res_v f32 [G*B, Kr]   (sorted by res_s desc)
 *   top_seed f32 [G]   res_seed i64 [G*B]   E f32 [L, 2, D, B]
 */
#ifndef PROTEUS_ATLAS_H
#define PROTEUS_ATLAS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum atlas_dtype { ATLAS_F32 = 0, ATLAS_BF16 = 1, ATLAS_F16 = 2 };

enum atlas_status {
  ATLAS_OK = 0,
  ATLAS_ERR_ARG = 1,      /* invalid argument (shape, stride, alignment, null pointer) */
  ATLAS_ERR_CUDA = 2,     /* a CUDA runtime call or kernel launch failed */
  ATLAS_ERR_UNSUPPORTED = 3
};

/* Device status word of the kernels that wait on mbarriers (the tensor-core kernels and the TMA-fed
 * filter): 0, or the code of the first bounded wait that gave up (a kernel never hangs; it records
 * the failure here and finishes). Synchronous read; `reset` clears it. No counterpart in the
 * reference (its Triton kernels have no waits). */
int atlas_device_status(int* status_host, int reset);
/* Test hook: writes `code` into the device status word (synchronous), so that a host can exercise
 * its handling of a failed wait (refusing results and checkpoints) without making a wait give up.
 * No counterpart in the reference. */
int atlas_device_status_set(int code);

/* Message of the last error raised on the calling host thread ("" if none). */
const char* atlas_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int atlas_abi_version(void);

/* ------------------------------------------------------------------------------------------------
 * K1 compare-and-compact — replaces filter_candidates (atlas/filter_triton.py:65-86).
 * survivor (t, d) <=> rowmap[t] >= 0 && (h > thr_pos[d] || -h > thr_neg[d]).
 * H: [T, D] of `dtype` with row stride ld elements (unit column stride). rowmap i32 [T]: valid-row
 * index or -1. Survivors are written as (val = h as fp32, row = rowmap[t], col = d) in arbitrary
 * order into out_* [cap]; *count (must be 0 on entry) receives the exact survivor count even when it
 * exceeds cap, and nothing is written past cap.
 */
int atlas_filter_compact(const void* H, int dtype, int64_t T, int64_t D, int64_t ld,
                         const int32_t* rowmap, const float* thr_pos, const float* thr_neg,
                         float* out_val, int32_t* out_row, int32_t* out_col, int32_t* count,
                         int64_t cap, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Batch context on the device — replaces the row-level decisions of Atlas.make_ctx
 * (atlas/core.py:210-237), so a batch needs only its raw valid rows, token ids and annotation ids.
 * atlas_ctx_rows: valid_rows int64 [n_v] (rows of H, < T), tok int64 [n_v] (in [0, 2^32); a bad one
 *   sets *err and is skipped). Writes key int64 [n_v] = lowbias32((tok ^ seed) mod 2^32)
 *   (core.py:46-55); rowmap int32 [T] (-1 for padding rows); the subsample {i : key < U_sub} in
 *   increasing i as sub_idx int64 and sub_rows32 = valid_rows[sub_idx]; within it the bulk rows
 *   {j : key[sub_idx[j]] < U_res} as res_in_sub int64 (positions j), res_rows32 and res_vidx32
 *   (valid index); key_order int32 [n_v] = valid indices by ascending key; counts int64 [2] =
 *   (n_s, n_r), on the device. Index outputs are sized n_v (the first n_s / n_r entries are set).
 *   ws: device bytes >= atlas_ctx_ws_bytes(n_v). Asynchronous on `stream`.
 * atlas_ctx_annotations: ann int64 [n_v, m_a] (class ids, -1 padded); writes annT int8
 *   [A_pad, n_pad] with annT[a, j] = 1 when a is among the ids of subsample row j (zero elsewhere;
 *   n_pad >= n_s) and ann_totals int64 [n_a] = per-class row counts of the subsample (the
 *   ann_sub / ann_sub_i8 of the reference's make_ctx, transposed for the enrichment contraction).
 */
int64_t atlas_ctx_ws_bytes(int64_t n_v);
int atlas_ctx_rows(const int64_t* valid_rows, const int64_t* tok, int64_t n_v, int64_t T, int64_t seed, int64_t U_sub,
                   int64_t U_res, int64_t* key, int32_t* rowmap, int64_t* sub_idx, int64_t* res_in_sub,
                   int32_t* sub_rows32, int32_t* res_rows32, int32_t* res_vidx32, int32_t* key_order, int64_t* counts,
                   int32_t* err, void* ws, int64_t ws_bytes, void* stream);
int atlas_ctx_annotations(const int64_t* sub_idx, const int64_t* counts, const int64_t* ann, int64_t n_v, int64_t m_a,
                          int64_t n_a, int8_t* annT, int64_t A_pad, int64_t n_pad, int64_t* ann_totals, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Per-batch compaction thresholds — replaces the device math of Atlas.begin_batch
 * (atlas/core.py:250-259):
 *   tau_top = max(nextafter(top_s[g, K-1], -inf), top_seed[g])
 *   kth     = max(res_s[g*B+b, Kr-1], res_seed[g*B+b]);  underfilled = kth < -U_res
 *   eps     = nextafter(min_b{E[g, b] : underfilled}, -inf)  (inf when none)
 *   thr[g]  = reservoir ? min(tau_top, eps) : tau_top            for g in [0, G)
 * Optionally (non-NULL) it also keeps the batch's admission thresholds in compact arrays for
 * atlas_admit: top_kth[g] = top_k[g, K-1] (top_k required) and, with reservoir,
 * res_thr[g*B+b] = kth. They stay valid until the state is next merged (end of the batch).
 */
int atlas_thresholds(const float* top_s, int64_t K, const int64_t* res_s, int64_t Kr,
                     const float* top_seed, const int64_t* res_seed, const float* E,
                     int64_t G, int64_t B, int64_t U_res, int reservoir, float* thr,
                     const int64_t* top_k, int64_t* top_kth, int64_t* res_thr, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Subsample row gathers — replace H.index_select(0, sub_rows) and Hn.index_select(0, res_in_sub)
 * (atlas/core.py:289, :292).
 * atlas_gather_transpose: XT[d, col0 + i] = H[rows[i], d] for i < n, zero for n <= i < round8(n);
 *   XT has leading dimension ldx (elements, multiple of 8), same dtype as H.
 * atlas_gather_rows: R[i, d] = H[rows[i], d] (R row stride D, same dtype as H).
 */
int atlas_gather_transpose(const void* H, int dtype, int64_t T, int64_t D, int64_t ld,
                           const int32_t* rows, int64_t n, void* XT, int64_t ldx, int64_t col0,
                           void* stream);
int atlas_gather_rows(const void* H, int dtype, int64_t T, int64_t D, int64_t ld, const int32_t* rows,
                      int64_t n, void* R, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Subsample statistics — replaces sub_stats (atlas/stats_triton.py:77-117) and the accumulation
 * of Atlas._subsample_stats_v3 / _v1 (atlas/core.py:312-338, :378-399).
 * Input XT [D, n] (columns col0..col0+n of a transposed staging buffer, leading dim ldx).
 * Accumulates in place, per column d:
 *   sum[d] += sum_i x,  sq[d] += sum_i x^2          (fp32 within 8-row groups, fp64 across)
 *   bins[(p*D + d)*B + b] += #{i : s_p >= E_p[d, b]} - #{i : s_p >= E_p[d, b+1]}   (int64; s_0 = x, s_1 = -x)
 * and, when NL > 0, writes masks i8 [2, NL, D, n_pad]: masks[p, j, d, i] = (s_p >= E_p[d, levels[j]])
 * for i < n, 0 for n <= i < n_pad (the layout of an exact int8 GEMM against [n_pad, A] one-hots).
 * E0, E1: [D, B] fp32 (pole 0 / pole 1 lower edges). levels: host array of NL ints.
 */
int atlas_sub_stats(const void* XT, int dtype, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                    const float* E0, const float* E1, int64_t B, const int32_t* levels_host, int64_t NL,
                    double* sum, double* sq, int64_t* bins, int8_t* masks, int64_t n_pad, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Exact int8 contingency GEMM on tcgen05 tensor cores — replaces _count_mm_i8 / torch._int_mm
 * (atlas/core.py:762-774) and the accumulation enr[l] += c (core.py:398-399).
 * masks i8 [M, n_pad] (row-major, K-major), annT i8 [A_pad, n_pad] (annotation one-hots transposed,
 * zero padded), out i64 [M, A] accumulated in place: out[m, a] += sum_k masks[m, k] * annT[a, k].
 * n_pad % 128 == 0, A_pad % 16 == 0, 16 <= A_pad <= 256, A <= A_pad, M % 128 == 0.
 */
int atlas_count_gemm_i8(const int8_t* masks, int64_t M, int64_t n_pad, const int8_t* annT, int64_t A_pad,
                        int64_t* out, int64_t A, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Subsample statistics and enrichment in one pass — replaces sub_stats followed by _count_mm_i8
 * (atlas/stats_triton.py:77-117, atlas/core.py:378-399, :762-774) without materialising the int8
 * masks: the same accumulations as atlas_sub_stats (sum, sq, bins; masks are not written) and as
 * atlas_count_gemm_i8 on those masks (enr [2, NL, D, A] int64 += masks . annT^T), read from XT once.
 * The 0/1 mask tiles are built in shared memory and contracted on tcgen05 (kind::i8, exact int32).
 * Supported when atlas_stats_enrich_supported(dtype, B, NL, A_pad) != 0 (bf16 staging, B <= 8,
 * 1 <= NL <= 3, A_pad in {16, 32, 48}); otherwise use the two kernels. annT [A_pad, n_pad] int8
 * (n_pad % 128 == 0, zero past the n subsample rows). ws: device workspace of
 * atlas_stats_enrich_ws_bytes(D, n) bytes, zero-filled before its first use (the kernel leaves it
 * reusable); calls sharing one ws must not overlap. Sums are fp32 per 8 rows and fp64 across, in
 * an order that does not depend on CTA timing.
 */
int atlas_stats_enrich_supported(int dtype, int64_t B, int64_t NL, int64_t A_pad);
int64_t atlas_stats_enrich_ws_bytes(int64_t D, int64_t n);
int atlas_sub_stats_enrich(const void* XT, int dtype, int64_t ldx, int64_t col0, int64_t n, int64_t D,
                           const float* E0, const float* E1, int64_t B, const int32_t* levels_host, int64_t NL,
                           double* sum, double* sq, int64_t* bins, const int8_t* annT, int64_t A_pad, int64_t n_pad,
                           int64_t* enr, int64_t A, void* ws, int64_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Upper-block-triangle Gram on tcgen05 tensor cores — replaces gram_accumulate
 * (atlas/stats_triton.py:148-169): C[D, D] (fp32, row-major, contiguous) += X^T X on the 128x128
 * blocks with block row <= block column; lower blocks untouched. X is supplied transposed:
 * XT [D, n] bf16 or fp16 (tcgen05, fp32 accumulation) or fp32 (exact fp32 FMA on CUDA cores) with
 * leading dimension ldx (elements; ldx % 8 == 0, 16-byte aligned base).
 */
int atlas_gram_upper(const void* XT, int dtype, int64_t ldx, int64_t n, int64_t D, float* C, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Per-batch counters of end_batch — the bookkeeping of _merge_filtered_impl's counts read
 * (atlas/core.py:458-470), kept on the device instead of read on the host: one thread adds
 *   stats[0] += sum of count[l] over filtered layers (filtered_host[l] != 0) with count[l] <= cap(l)
 *   stats[1] += *n_top,  stats[2] += *n_res  (records admitted this batch)
 *   stats[3] += number of filtered layers with count[l] > cap(l) (each took the dense path)
 * cap(l) = l < early_layers ? cap_early : cap_main. filtered_host is a HOST array of L bytes (may be
 * NULL: no filtered layer); L <= 64. stats: int64[4] on the device.
 */
int atlas_batch_counters(const int32_t* count, int64_t L, const int8_t* filtered_host, int64_t cap_main,
                         int64_t cap_early, int64_t early_layers, const int32_t* n_top, const int32_t* n_res,
                         int64_t* stats, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Candidate admission for the filtered layers of a batch — replaces _merge_filtered_impl's
 * candidate tests and the bulk-row paths _bulk_loop / _bulk_stacked (atlas/core.py:482-590).
 * top_kth [G] and res_thr [G*B] are the batch's compact thresholds from atlas_thresholds
 * (top_k[g, K-1] and max(res_s[g*B+b, Kr-1], res_seed[g*B+b])).
 * For every layer l with layer_mode[l] == 1 and count[l] <= cap(l):
 *   compacted candidate (h, row, col), pole p (s = +-h), g = (l*2+p)*D + col:
 *     top:  s > top_seed[g] && top_key(s, tok[row]) > top_kth[g]         -> record (g, top_key, tok, s)
 *     res:  b = bin(s, E[l,p,col]) >= 0 && key[row] >= U_res && -key > res_thr[g*B+b]
 *                                                                        -> record (g*B+b, -key, tok, h)
 *   bulk rows R[l] [n_r, D] (rows with key < U_res; bulk_vidx = their valid-row indices):
 *     every (row, col, pole) with bin >= 0 and -key > res_thr[g*B+bin] -> res record.
 * cap(l) = l < early_layers ? cap_early : cap_main. Candidate buffers are [L, cand_stride].
 * Records are appended to SoA lists (group i32, score i64, tok i64, val f32) with device counters
 * n_top / n_res; an append past the list capacity sets err[0] and is dropped.
 */
int atlas_admit(int64_t L, int64_t D, int64_t B, int64_t K, int64_t Kr, int64_t U_res, int reservoir,
                const int8_t* layer_mode_host, const int32_t* count, int64_t cap_main, int64_t cap_early,
                int64_t early_layers, const float* cand_val, const int32_t* cand_row, const int32_t* cand_col,
                int64_t cand_stride, const int64_t* tok, const int64_t* key,
                const void* R, int dtype, int64_t n_r, int64_t r_stride, const int32_t* bulk_vidx,
                const float* top_seed, const int64_t* top_kth, const int64_t* res_thr, const float* E,
                int32_t* top_g, int64_t* top_sc, int64_t* top_tok, float* top_val, int32_t* n_top, int64_t top_cap,
                int32_t* res_g, int64_t* res_sc, int64_t* res_tok, float* res_val, int32_t* n_res, int64_t res_cap,
                int32_t* err, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Dense burst path for one layer — replaces Atlas._dense (atlas/core.py:407-446) without a forward
 * re-run: runs on the live hook output when force != 0 or *count > cap (the 0.5%-fill overflow of
 * the compaction buffer), otherwise returns immediately on the device.
 * Per column and pole it selects, from the n_v valid rows, the exact top-K by top_key (the only
 * batch elements that can enter the state's top-K) and, per bin, the Kr smallest keys among rows in
 * the bin under the bin's key ceiling; admitted records are appended to the same lists as
 * atlas_admit. key_order: valid-row indices sorted by key ascending. scratch: device bytes,
 * >= atlas_dense_scratch_bytes(n_v, D, B, dtype) (per-column partial counts of the row ranges, the
 * per-column decisions and hard-column lists, the keys in key order), ZERO-FILLED before its first
 * use: the call counts arrivals in some of its words and leaves them at zero, so a buffer kept for
 * later calls needs no further clearing.
 * `flag` is unused (kept for ABI stability); K <= 256, Kr <= 256, 2K + 2*B*Kr <= 1024.
 */
int64_t atlas_dense_scratch_bytes(int64_t n_v, int64_t D, int64_t B, int dtype);
int atlas_dense_select(const void* H, int dtype, int64_t T, int64_t D, int64_t ld, int64_t layer,
                       const int32_t* valid_rows, int64_t n_v, const int64_t* tok, const int64_t* key,
                       const int32_t* key_order, int64_t B, int64_t K, int64_t Kr, int reservoir,
                       const float* top_seed, const int64_t* top_k, const int64_t* res_s, const int64_t* res_seed,
                       const float* E, const int32_t* count, int64_t cap, int force,
                       int32_t* top_g, int64_t* top_sc, int64_t* top_tok, float* top_val, int32_t* n_top, int64_t top_cap,
                       int32_t* res_g, int64_t* res_sc, int64_t* res_tok, float* res_val, int32_t* n_res, int64_t res_cap,
                       void* scratch, int64_t scratch_bytes, int32_t* flag, int32_t* err, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Exact grouped top-K merge — replaces grouped_merge (atlas/core.py:75-104).
 * state_sc i64 [G, K] sorted descending with payloads state_tok i64 [G, K], state_val f32 [G, K];
 * candidates: *n_dev records (g i32, sc i64, tok i64, val f32), n_max a host upper bound on *n_dev.
 * Afterwards each touched row holds the K largest scores of (row U its candidates), descending,
 * with their payloads. Scores must be unique within a group (the atlas keys are).
 * Workspace (device): ws_i32 of atlas_merge_ws_i32(G, n_max) ints, ws_bytes of
 * atlas_merge_ws_bytes(n_max) bytes.
 */
int64_t atlas_merge_ws_i32(int64_t G, int64_t n_max);
int64_t atlas_merge_ws_bytes(int64_t n_max);
int atlas_grouped_merge(int64_t* state_sc, int64_t* state_tok, float* state_val, int64_t G, int64_t K,
                        const int32_t* g, const int64_t* sc, const int64_t* tok, const float* val,
                        const int32_t* n_dev, int64_t n_max, int32_t* ws_i32, void* ws_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Allocation-free grouped merge. No counterpart in the reference. Same inputs, outputs and result
 * as atlas_grouped_merge, but the workspace is a fixed device array inside this library instead of
 * caller memory, for callers that cannot allocate device memory themselves: a host runtime that owns
 * every device byte through its own pool and forbids side allocations, or a call site that must not
 * pay for cudaMalloc's implicit device synchronisation in the middle of a stream.
 * Limits: G <= 262144 groups and n_max <= 262144 records per call (larger requests are rejected
 * with ATLAS_ERR_ARG). Each GPU has its own copy of the array (about 11 MB). It is created when the
 * library's device code is first loaded on that GPU (under lazy module loading, the CUDA default,
 * that is this entry point's first call there) and stays until the process exits. Make one warm-up
 * call per GPU at initialisation, before any stream capture on it. Calls on one GPU share its copy:
 * calls on that GPU that can overlap (different streams, or several host threads) race and must be
 * serialised by the caller; calls on different GPUs do not race. The library must not be used across
 * a cudaDeviceReset of the calling context's device while a call is in flight. Nothing is allocated
 * by this call or by anything it calls beyond that one array.
 */
int atlas_grouped_merge_static(int64_t* state_sc, int64_t* state_tok, float* state_val, int64_t G, int64_t K,
                               const int32_t* g, const int64_t* sc, const int64_t* tok, const float* val,
                               const int32_t* n_dev, int64_t n_max, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Row-wise merge of two sorted states — replaces the top-K / reservoir part of Atlas.merge_from
 * (atlas/core.py:636-643): for each of G rows, (sc, tok, val) <- the K largest of
 * (sc U other_sc) with payloads (keys unique across the two states).
 */
int atlas_merge_rows(int64_t* sc, int64_t* tok, float* val, const int64_t* other_sc, const int64_t* other_tok,
                     const float* other_val, int64_t G, int64_t K, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Pilot pass — replaces the sorts and top-k selections of pilot_edges / pilot_seeds
 * (atlas/reference.py:55-122) with exact order statistics and integer counts on the device.
 *
 * atlas_column_select: out[d, t] = the value at ascending rank ranks_host[t] (0-based, < n) of the
 *   n elements XT[d, 0..n) (transposed activations, leading dimension ldx % 8 == 0, 16-byte aligned
 *   base), for every d < D; 1 <= R <= 32 ranks; -0.0 ranks below +0.0 (the order of a radix sort of
 *   the float bits). Values are returned as fp32 (exact for every dtype).
 * atlas_pilot_edges: sel [D, 2B] holds, per column, the values at ranks r_b = round(q_b (n-1)) and
 *   at n-1-r_b; writes E [2, D, B] with E[0, d, b] = sel[d, b], E[1, d, b] = -sel[d, B + b], each
 *   then raised to nextafter(E[p, d, b-1], +inf) where not above it (strictly increasing edges).
 * atlas_pilot_counts: for the rows visited in the order `order` (int32 row indices, NULL = 0..n-1),
 *   per pole p (s = +h, -h), column d and bin b (bin = #{b : s >= E[p, d, b]} - 1):
 *     cnt[(p*D + d)*B + b]   += #{rows in the bin}
 *     sumsq[(p*D + d)*B + b] += sum over runs of (#{rows of the run in the bin})^2
 *   where a run ends at every visited position i with run_last[i] != 0 (run_last NULL: no runs,
 *   sumsq untouched). chunk_start (device int64 [n_chunks + 1], 0 = first, n = last) splits the
 *   visiting order into pieces of whole runs worked on in parallel. cnt, sumsq: int64 [2, D, B].
 * atlas_pilot_seeds: per pole and column, top_seed[p*D + d] = nextafter(v, -inf) with v = sel2[d, 0]
 *   (p = 0) or -sel2[d, 1] (p = 1), sel2 [D, 2] the values at ascending ranks n-kk and kk-1
 *   (kk = min(2K, n)); per bin the key ceiling
 *     grouped:   n_eff = cnt^2 / max(sumsq, 1); m_lo = (cnt / n) * max(1 - z / sqrt(max(n_eff, 1e-9)), 0)
 *     otherwise: m_lo = max(cnt - z * sqrt(cnt), 0) / n
 *     res_seed_key = floor(min(m_lo > 0 ? c*Kr*2^32 / (n_total * m_lo) : 2^32, 2^32))
 *   in fp64 with the reference's operation order (each operation correctly rounded).
 */
int atlas_column_select(const void* XT, int dtype, int64_t ldx, int64_t n, int64_t D, const int64_t* ranks_host,
                        int64_t R, float* out, void* stream);
int atlas_pilot_edges(const float* sel, int64_t D, int64_t B, float* E, void* stream);
int atlas_pilot_counts(const void* H, int dtype, int64_t ld, int64_t n, int64_t D, const int32_t* order,
                       const uint8_t* run_last, const int64_t* chunk_start, int64_t n_chunks, const float* E,
                       int64_t B, int64_t* cnt, int64_t* sumsq, void* stream);
int atlas_pilot_seeds(const int64_t* cnt, const int64_t* sumsq, const float* sel2, int64_t D, int64_t B, int64_t n,
                      int64_t Kr, int64_t n_total, double c, double z, int grouped, float* top_seed,
                      int64_t* res_seed_key, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PROTEUS_ATLAS_H */
