/*
 * p2p_b200.h -- C ABI of the B200 (sm_100a) replica hot path of p2pLLM.
 *
 * Every entry point takes plain device pointers, element counts, strides (in elements) and a CUDA stream passed as
 * `void*` (a cudaStream_t; NULL is the legacy default stream). Nothing here allocates device memory unless its comment
 * says so: scratch space is passed in by the caller, sized by the matching *_workspace() query. Entry points launch
 * asynchronously on the given stream and never synchronise the host, except where a comment says they read a status
 * word back.
 *
 * Return value: P2P_OK (0) or a negative P2P_E* code; p2p_last_error() then holds a message for this host thread.
 *
 * Reference interfaces are cited as path:line inside the p2pLLM source tree.
 */
#ifndef P2P_B200_H
#define P2P_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of weights, activations and outputs. */
enum { P2P_BF16 = 0, P2P_F16 = 1, P2P_F32 = 2 };

/* Status codes. */
enum {
    P2P_OK = 0,
    P2P_EINVAL = -1,      /* a null pointer, a negative size, a stride below the row length, misalignment */
    P2P_EUNSUPPORTED = -2,/* a dtype or a size this build does not handle (the message names the limit) */
    P2P_ECUDA = -3,       /* a CUDA runtime error at launch */
    P2P_EDATA = -4        /* the data broke a format rule (rows of unequal length, a column index out of range) */
};

/* The message of the last failed call on this host thread ("" if none). */
const char* p2p_last_error(void);
/* ABI version: bumped when a signature changes. */
int p2p_abi_version(void);

/* ------------------------------------------------------------------------------------------------------------------
 * (1) Wanda calibration and selection
 * ------------------------------------------------------------------------------------------------------------------ */

/* Bytes of workspace p2p_sumsq_cols needs for this shape (0 if none). */
size_t p2p_sumsq_workspace(int64_t tokens, int64_t cols, int dtype);

/* sums[c] += (double)(float)(sum_t x[t, c]^2) for x [tokens, cols] (row stride ldx) of `dtype`: each square in fp32,
 * the column total accumulated in fp64 and rounded to fp32 once per call, as the reference's hook does.
 * Deterministic: a fixed reduction order, whatever the launch shape.
 * Replaces p2p/wanda.py:37-40 (Calibration._linear: x.float().pow(2).sum(0).double()) and wanda.py:34-35 (_add).
 * workspace: p2p_sumsq_workspace() bytes of device memory, zeroed once before its first use (the kernel leaves it
 * zeroed again); calls that share a workspace must not overlap on the GPU. */
int p2p_sumsq_cols(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, double* sums,
                   void* workspace, size_t workspace_bytes, void* stream);

/* p2p_sumsq_cols for callers that cannot allocate device memory: the same reduction (deterministic, each column
 * total rounded to fp32 once), with its scratch held inside the library in one fixed device array of 4 MiB + 4 KiB per
 * GPU (kept until the process exits) instead of a caller-provided workspace. It allocates nothing. For a calibration
 * hook running inside a serving engine that has already reserved its share of GPU memory (SGLang's static fraction for
 * weights and the KV pool), where a fresh allocation can fail or fragment what is left. cols <= 16,384
 * (P2P_EUNSUPPORTED above).
 * Every call looks up the array's device address in the current context. With CUDA's lazy module loading the
 * library's device module -- and with it the array -- is committed on a device the first time any of its kernels
 * or this array is used there: make a first call (tokens = 1 is enough) before the engine reserves its memory, and
 * before any stream capture. Every call uses the same array: calls that overlap on the GPU (other streams, other
 * host threads) race and must be ordered by the caller.
 * Rounding: when tokens x cols is large enough that p2p_sumsq_cols would split the rows into more slabs than the
 * fixed array holds (more than 4 MiB / (8 cols) slabs), this call uses fewer, taller slabs, so the fp64 partials are
 * added in another grouping; the column totals then agree with p2p_sumsq_cols to within one fp32 rounding of the
 * total, and are still deterministic. No counterpart in the reference (p2pLLM allocates through torch). */
int p2p_sumsq_cols_noalloc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, double* sums,
                           void* stream);

/* Per-expert sums of squares of the tokens routed to each expert: into[e, c] += (double)(float)sum over the tokens t
 * whose ids row holds e (each token once per expert) of x[t, c]^2. order: the `tokens * topk` (token, slot) pairs
 * sorted by expert and then token (order[i] = token * topk + slot), seg: [n_experts + 1] offsets into order per expert.
 * Replaces the `into` half of p2p/wanda.py:10-20 (expert_inputs). */
int p2p_expert_sumsq(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const int64_t* order,
                     const int64_t* seg, int64_t topk, int64_t n_experts, double* into, void* stream);

/* norms[g, c] = (float)sqrt(sums[g, c]) for `groups` rows of `cols` sums; with experts != 0 a row whose fp32 norms
 * add up to 0 becomes all ones (an expert no token reached).
 * Replaces p2p/wanda.py:63-73 (channel_norms; the rank slice is taken by the caller). */
int p2p_channel_norms(const double* sums, int64_t groups, int64_t cols, int experts, float* norms, void* stream);

/* Per-row Wanda top-k of w [rows, cols] (row stride ldw): score[r, c] = |float(w[r, c])| * norms[g(r), c] in fp32,
 * g(r) = r / norm_group_rows (norm_group_rows 0: one norms row for all rows). Keeps the k highest scores of each row,
 * ties going to the lower column, and writes any of:
 *   vals [rows, k] (row stride ldo, dtype of w) and idx [rows, k] (int16 if idx_bytes == 2, int32 if 4): the kept
 *     weights and their columns, in ascending column order;
 *   words [rows, ceil(cols/32)] int32 (row stride ldwords): bit c%32 of word c/32 set where kept (the reference's
 *     mask words, p2p/compact.py:36-45);
 *   mask [rows, cols] uint8 (row stride ldm): 1 where kept;
 *   pruned [rows, cols] (row stride ldp, dtype of w): w where kept, w * 0.0f elsewhere.
 * Null outputs are skipped. cols <= 52,000.
 * Replaces p2p/wanda.py:76-87 (prune, with_mask) and p2p/compact.py:36-45 (pack). */
int p2p_wanda_select(const void* w, int dtype, int64_t rows, int64_t cols, int64_t ldw, const float* norms,
                     int64_t norm_group_rows, int64_t k, void* vals, void* idx, int idx_bytes, int64_t ldo,
                     int32_t* words, int64_t ldwords, uint8_t* mask, int64_t ldm, void* pruned, int64_t ldp,
                     void* stream);

/* ------------------------------------------------------------------------------------------------------------------
 * Compact formats: reference mask words <-> values + column indices <-> dense
 * ------------------------------------------------------------------------------------------------------------------ */

/* idx [rows, k] (ascending columns) from the reference's mask words [rows, ceil(cols/32)] int32. Checks that every
 * row sets exactly k bits below `cols`; otherwise P2P_EDATA (this call reads one status word back, so it syncs the
 * stream). Used to load p2p/compact.py:36-45 blocks and p2p/prepare.py:42-73 files. */
int p2p_words_to_idx(const int32_t* words, int64_t rows, int64_t cols, int64_t ldwords, int64_t k, void* idx,
                     int idx_bytes, int64_t ldi, void* stream);

/* values [rows, k] + mask words from w [rows, cols] and a uint8 mask that keeps k weights in each row (P2P_EDATA,
 * after a status read-back, if a row keeps another number). Replaces p2p/compact.py:36-45 (pack). */
int p2p_pack_mask(const void* w, int dtype, int64_t rows, int64_t cols, int64_t ldw, const uint8_t* mask,
                  int64_t ldm, int64_t k, void* vals, int64_t ldo, int32_t* words, int64_t ldwords, void* stream);

/* dense [rows, cols] (row stride ldd) from values [rows, k] and either mask words (idx == NULL) or column indices:
 * kept weights in place, zeros elsewhere. Replaces p2p/compact.py:48-61 (unpack) and the Triton kernel _unpack
 * (p2p/compact.py:64-85); p2p/compact.py:88-97 (expand) calls it per expert. */
int p2p_unpack(const void* vals, int dtype, int64_t rows, int64_t k, int64_t ldv, const int32_t* words,
               int64_t ldwords, const void* idx, int idx_bytes, int64_t ldi, int64_t cols, void* dense, int64_t ldd,
               void* stream);

/* P2P_OK if every row of idx [rows, k] (row stride ldi) holds strictly ascending columns in [0, cols), else P2P_EDATA
 * (reads one status word back, so it syncs the stream). The GEMMs clamp indices instead of checking them; the host
 * checks once, at load. Guards what p2p/compact.py:113-166 (Tiles.__init__) assumes of the blocks it is given. */
int p2p_check_idx(const void* idx, int idx_bytes, int64_t rows, int64_t k, int64_t ldi, int64_t cols, void* stream);

/* ------------------------------------------------------------------------------------------------------------------
 * (2) Compact sparse GEMM  y[t, r] = sum_j vals[r, j] * x[t, idx[r, j]]
 * ------------------------------------------------------------------------------------------------------------------ */

/* One row block of a module: rows [row0, row0 + rows) of y read values [rows, k] (row stride ld, dtype of x) and
 * column indices [rows, k] (same stride; idx == NULL means a dense block, k == cols, column j = j). */
typedef struct {
    const void* vals;
    const void* idx;
    int64_t row0;
    int64_t rows;
    int64_t k;
    int64_t ld;
} p2p_row_block;

/* y [tokens, ldy] (columns row0.. of each block) = x [tokens, cols] (row stride ldx) times the blocks' rows, fp32
 * sums, on CUDA cores straight from the row layout (values + column indices). Any token count. bf16, f16 or f32;
 * idx_bytes 2 or 4. cols * element size <= 200 KiB. Up to 32 tokens whose x fits 200 KiB, one block an SM stages all
 * of x; otherwise blocks stage token tiles.
 * Replaces p2p/compact.cu:265-278 (spmm) for row-layout weights; p2p/compact.py:192-199 (Tiles.__call__). */
int p2p_spmm_rows(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const p2p_row_block* blocks,
                  int nblocks, int idx_bytes, void* y, int64_t ldy, void* stream);

/* The tensor-core layout of a module (bf16 / f16 weights): rows in tiles of 128, columns in tiles of 64; each
 * (row tile, column tile) segment holds its kept weights as 32-bit words (value bits << 16 | row << 6 | column, bit 13
 * marking fillers), padded to a multiple of 4 words; seg [row_tiles * col_tiles + 1] holds where each starts.
 * Same 4 bytes per kept weight as values + int16 indices. The B200 counterpart of p2p/compact.py:124-166
 * (Tiles.__init__ re-tiling a module into 8 x 8 pieces), run once at load:
 *   p2p_tiles_workspace: bytes of scratch both calls need;
 *   p2p_tiles_plan: fills seg and returns the total words through *total_words (reads it back: syncs the stream);
 *   p2p_tiles_fill: writes the words [total_words]. Row blocks as for p2p_spmm_rows, column indices ascending. */
size_t p2p_tiles_workspace(const p2p_row_block* blocks, int nblocks, int64_t cols);
int p2p_tiles_plan(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int64_t* seg,
                   int64_t* total_words, void* workspace, size_t workspace_bytes, void* stream);
int p2p_tiles_fill(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int dtype, const int64_t* seg,
                   uint32_t* words, int64_t n_words, void* workspace, size_t workspace_bytes, void* stream);

/* The bitmask layout of a module (values + one bit a weight, the reference's storage of p2p/compact.py:36-45) for
 * p2p_spmm_mask, built on the GPU from row blocks as for p2p_tiles_*: 128-row x 64-column segments, each a 16-byte
 * header of cumulative 16-row block counts, 1024 bytes of piece masks (8 blocks x 16 pieces x 64 bits) and the kept
 * values piece by piece, padded to 16 bytes; seg[n_seg + 1] holds byte offsets. Load time, syncs.
 *   p2p_mask_workspace: bytes of scratch p2p_mask_plan needs;
 *   p2p_mask_plan: fills seg and returns the total bytes through *total_bytes;
 *   p2p_mask_fill: writes the layout [total_bytes] (16-byte aligned); refuses indices out of ascending order.
 * Replaces p2p/compact.py:124-174 (Tiles.__init__: the re-tiling into 8 x 8 pieces of masks and values). */
size_t p2p_mask_workspace(const p2p_row_block* blocks, int nblocks, int64_t cols);
int p2p_mask_plan(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int64_t* seg,
                  int64_t* total_bytes, void* workspace, size_t workspace_bytes, void* stream);
int p2p_mask_fill(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int dtype, const int64_t* seg,
                  void* data, int64_t total_bytes, void* stream);

/* Bytes of workspace p2p_spmm_mask needs for this shape (0 if it does not split the columns). */
size_t p2p_spmm_mask_workspace(int64_t rows, int64_t cols, int64_t tokens);

/* y [tokens, ldy] = x [tokens, cols] (row stride ldx, 16-byte aligned rows) times the module in the bitmask layout, on
 * tcgen05 tensor cores: segments streamed into shared memory by bulk copies, each 128 x 64 weight tile rebuilt in
 * registers and stored into tensor memory, the MMAs reading it from there (fp32 accumulation in TMEM, x by TMA).
 * bf16 or f16; cols a multiple of 8; any token count (288 a launch). workspace: zeroed once before its first use (left
 * zeroed again); calls sharing it must not overlap on the GPU. Each launch is a programmatic dependent of the stream's
 * previous kernel, as p2p_spmm_tc (x may be that kernel's output; data and seg must not be).
 * Replaces p2p/compact.cu:82-278 (spmm_kernel, sum_parts, spmm) on the reference's own storage format. */
int p2p_spmm_mask(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const void* data,
                  const int64_t* seg, int64_t rows, void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                  void* stream);

/* p2p_spmm_mask with the all-gather of a row-sharded module fused into its epilogue: this rank's `rows` rows of y go
 * to columns y_col0 .. y_col0 + rows - 1 of each of the n_ys (1..8) buffers ys[k] [tokens, ldy] -- the y of every
 * rank of the node, peers' buffers addressed through CUDA IPC / symmetric memory, written with plain stores over
 * NVLink. The other ranks read their y only after a p2p_peer_barrier that follows this launch on every rank.
 * Replaces the NCCL all-gather that p2p/wanda.py:81's column split needs in SGLang (here rows are split, so each rank's
 * rows are final and only need placing). */
int p2p_spmm_mask_peers(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const void* data,
                        const int64_t* seg, int64_t rows, void* const* ys, int n_ys, int64_t y_col0, int64_t ldy,
                        void* workspace, size_t workspace_bytes, void* stream);

/* P2P_OK unless a p2p_spmm_mask launch since the last reset gave up waiting on its pipeline (then P2P_ECUDA, naming
 * the site); reset != 0 clears it. Syncs the stream. After a give-up the launch's workspace is undefined: zero it
 * again before the next launch that uses it. */
int p2p_spmm_mask_status(int reset, void* stream);

/* Bytes of workspace p2p_spmm_tc needs for this shape: 0 if one CTA takes each row tile whole; ticket counters and
 * fp32 partials when the columns are split (and not added in a cluster), or when the module runs as persistent runs
 * (more row tiles than SMs at up to 128 tokens: the partials of row tiles two runs share). */
size_t p2p_spmm_tc_workspace(int64_t rows, int64_t cols, int64_t tokens);

/* y [tokens, ldy] = x [tokens, cols] (row stride ldx, 16-byte aligned rows) times the module in the tensor-core
 * layout, on tcgen05 tensor cores (fp32 accumulation in TMEM, x staged by TMA). bf16 or f16; cols a multiple of 8;
 * seg_cap_words: the largest segment's word count. Any token count (512 a launch). workspace: zeroed once before its
 * first use (left zeroed again); calls sharing it must not overlap on the GPU.
 * Each launch is a programmatic dependent of the stream's previous kernel: it may start while that kernel finishes,
 * reading words and seg (and setting up) at once, but it reads x and writes y / the workspace only after that kernel
 * has completed. So x may be the previous kernel's output; words and seg must not be (build them, then synchronize,
 * as p2p_tiles_fill does). Column splits of a row tile may run as a thread-block cluster reducing over DSMEM; a module
 * of more row tiles than SMs at up to 128 tokens runs as one CTA an SM, each a contiguous run of (row tile, column
 * tile) units. Results are deterministic for a shape on a device (fixed reduction orders, whatever the scheduling).
 * Replaces p2p/compact.cu:82-278 (spmm_kernel, sum_parts, spmm) and p2p/compact.py:192-199 (Tiles.__call__). */
int p2p_spmm_tc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* y, int64_t ldy, void* workspace,
                size_t workspace_bytes, void* stream);

/* Routed experts in one launch: y [x_rows, ldy] row x_row0 + t = x row x_row0 + t times its expert's matrix, for every
 * item {expert, x_row0, tokens (1..256), 0} of items [n_items][4] (device memory, int32, 16-byte aligned;
 * p2p_moe_route writes them). The layout stacks the experts' matrices, expert e starting at row tile
 * e * item_row_tiles (layout_row_tiles row tiles in all, item_row_tiles = ceil(rows / 128)); x holds each expert's
 * tokens contiguously (sorted by expert); max_tokens bounds every item's tokens. Items that point past the layout or x
 * are skipped. No workspace: an item takes whole rows.
 * Replaces p2p/compact.py:241-256 (CompactMoE.apply, which expands every used expert to dense each pass) for the
 * routed experts' GEMMs. */
int p2p_spmm_tc_grouped(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx, const uint32_t* words,
                        const int64_t* seg, int64_t layout_row_tiles, int64_t rows, int64_t item_row_tiles,
                        int64_t seg_cap_words, const int32_t* items, int64_t n_items, int64_t max_tokens, void* y,
                        int64_t ldy, void* stream);

/* p2p_spmm_tc with the all-gather of a row-sharded module fused into its epilogue: this rank's `rows` rows of y go
 * to columns y_col0 .. y_col0 + rows - 1 of each of the n_ys (1..8) buffers ys[k] [tokens, ldy] -- the y of every
 * rank of the node, peers' buffers addressed through CUDA IPC / symmetric memory -- by plain stores over NVLink (8-byte
 * stores when ldy, y_col0 and the buffers allow). The other ranks read their y only after a p2p_peer_barrier that
 * follows this launch on every rank. The counterpart of p2p_spmm_mask_peers for the tensor-core layout; no
 * counterpart in the reference (it all-gathers through NCCL, p2p/wanda.py:81 on the scores). */
int p2p_spmm_tc_peers(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                      const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* const* ys, int n_ys,
                      int64_t y_col0, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* The gated forms: a gate + up module whose rows are interleaved 64 and 64 (row tile k: gate rows 64k..64k+63, then
 * up rows 64k..64k+63; rows = 2R, R a multiple of 64), and y [tokens, ldy >= R] = dtype(silu(g) * u), g and u the two
 * projections' outputs rounded to dtype, computed in the GEMM's epilogue (the accumulators of a row tile meet in
 * shared memory, in the cluster's, or in the workspace's partials first). Otherwise as p2p_spmm_tc /
 * p2p_spmm_tc_grouped (the workspace as p2p_spmm_tc_workspace(rows, cols, tokens) gives). Replaces
 * p2p/compact.py:205-224's gate_up projection followed by the model's SiluAndMul (two kernels and [T, 2R] in HBM). */
int p2p_spmm_tc_gated(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                      const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* y, int64_t ldy, void* workspace,
                      size_t workspace_bytes, void* stream);
int p2p_spmm_tc_grouped_gated(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx,
                              const uint32_t* words, const int64_t* seg, int64_t layout_row_tiles, int64_t rows,
                              int64_t item_row_tiles, int64_t seg_cap_words, const int32_t* items, int64_t n_items,
                              int64_t max_tokens, void* y, int64_t ldy, void* stream);

/* The gated half of expert calibration on the grouped launch: for routed experts whose gate + up rows are interleaved
 * as above (dense rows work too: a keep-100 layout), sums [n_items, ld_sums >= rows / 2] fp32 receives, per item and
 * unit j, the sum over the item's tokens of (silu(g) * u)^2 with g and u the unrounded fp32 products (bf16 / f16
 * inputs multiply exactly in fp32). Nothing else is written. Replaces p2p/wanda.py:16-19's loop (an fp32 GEMM, SiLU
 * and a sum of squares per expert). */
int p2p_spmm_tc_grouped_gated_sums(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx,
                                   const uint32_t* words, const int64_t* seg, int64_t layout_row_tiles, int64_t rows,
                                   int64_t item_row_tiles, int64_t seg_cap_words, const int32_t* items,
                                   int64_t n_items, int64_t max_tokens, float* sums, int64_t ld_sums, void* stream);

/* The routing of a routed-experts pass, on the GPU: ids [n_pairs] int64 (a token's slots consecutive; < 0: no expert).
 * order [n_pairs]: the routed pairs sorted by expert, and within an expert by pair index (stable); where [n_pairs]:
 * each pair's place in order, or -1; counts [experts] int32; items [max_items][4] int32: {expert, first place,
 * places (1..256), 0} for the grouped GEMM (max_items >= ceil(n_pairs / 256) + experts); meta [3] int64: {routed
 * pairs, items, most places in an item}. One block; experts <= 8192.
 * Replaces the routing CompactMoE leaves to torch and SGLang (p2p/compact.py:241-256: unique, renumbering). */
int p2p_moe_route(const int64_t* ids, int64_t n_pairs, int experts, int64_t* order, int64_t* where, int32_t* counts,
                  int32_t* items, int64_t max_items, int64_t* meta, void* stream);

/* out [tokens, ldo] row t = dtype(sum over slots j = 0.. k-1, in order, of weights[t k + j] * y[where[t k + j]]),
 * the fp32 weights and y [*, ldy] (bf16 or f16) in the pair order of p2p_moe_route; pairs with where < 0 add nothing.
 * The weighted sum a fused MoE ends with (SGLang's, which CompactMoE hands the experts to). */
int p2p_moe_combine(const void* y, int dtype, int64_t ldy, const int64_t* where, const float* weights, int64_t tokens,
                    int k, int64_t hidden, void* out, int64_t ldo, void* stream);

/* P2P_OK unless a p2p_spmm_tc launch since the last reset gave up waiting on its pipeline (then P2P_ECUDA, naming
 * the site); reset != 0 clears the flag. Syncs the stream. A launch that gives up issues no further loads or MMAs,
 * drains what it issued and exits; its y is then undefined, and so is its workspace (a run or column split that stopped
 * may leave its row tile's ticket counter taken): zero the workspace again before the next launch that uses it. */
int p2p_spmm_tc_status(int reset, void* stream);

/* Test of that give-up path: p2p_spmm_tc (one launch, tokens <= 512) in which every CTA withholds the x tile of local
 * index hold_tile (never loads it), so the waits for it run out after wait_us (1 ms .. 2 s) of %globaltimer and the
 * launch gives up; p2p_spmm_tc_status then reports the site. y is undefined. No counterpart in the reference (its
 * kernel has no waits to bound). */
int p2p_spmm_tc_withhold(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                         const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* y, int64_t ldy, void* workspace,
                         size_t workspace_bytes, int64_t hold_tile, int64_t wait_us, void* stream);

/* A barrier of the node's ranks over peer memory, on `stream`, after which every store this rank's stream made before
 * it (into its own or peers' memory) is visible to every rank. flags[r]: rank r's array of 8 uint32 slots, as this GPU
 * addresses it (zeroed before first use; epochs start at 1 and grow by one a barrier). Each wait is bounded by
 * timeout_us (1 ms .. 60 s): past it the barrier gives up and p2p_peer_status reports the rank it waited for.
 * The ranks' barriers wait on each other, so they must run on different GPUs, one process each.
 * No counterpart in the reference (its hops go through NCCL send/recv, p2p/route.py:798-831). */
int p2p_peer_barrier(void* const* flags, int n_ranks, int me, uint32_t epoch, int64_t timeout_us, void* stream);

/* The all-gather of a row-sharded module as a push: columns col0 .. col0 + width - 1 of the first `tokens` rows of
 * this rank's y [.., ldy] (its own rows of the module, written there by its GEMM) stored into the same place of each
 * of the n_peers (0..7) other ranks' y buffers (peer memory), 16-byte loads and stores over all SMs. Column offsets,
 * width and ldy in elements, 16-byte aligned. The peers read the columns after a p2p_peer_barrier that follows on
 * every rank. The form of the fused all-gather for many ranks, where storing every value to every rank from the
 * GEMM's epilogue would lengthen it N-fold. No counterpart in the reference. */
int p2p_peer_push(const void* y, void* const* peers, int n_peers, int64_t tokens, int64_t col0, int64_t width,
                  int64_t ldy, int dtype, void* stream);

/* P2P_OK unless a p2p_peer_barrier since the last reset gave up (P2P_ECUDA, naming the rank); reset != 0 clears it.
 * Syncs the stream. */
int p2p_peer_status(int reset, void* stream);

/* ------------------------------------------------------------------------------------------------------------------
 * (3) Group combine epilogue
 * ------------------------------------------------------------------------------------------------------------------ */

/* out = dtype(float(parts[0]) + sum_{0<k<n-1} dtype(float(parts[k]) - float(h))
 *                             + dtype(float(parts[n-1]) - float(h_copy)))       (n >= 2; fp32 sums in member order)
 * over n_elem elements: a group of n layers run in parallel, member k's output parts[k], the last member having
 * read the replica's h_copy. Replaces p2p/replica.py:81-85 (_member's combine). */
int p2p_combine(const void* const* parts, int n, const void* h, const void* h_copy, void* out, int dtype,
                int64_t n_elem, void* stream);

/* out = dtype(sum_k float(parts[k])) in member order (fp32). Replaces p2p/route.py:825-831 (_summed). */
int p2p_sum_parts(const void* const* parts, int n, void* out, int dtype, int64_t n_elem, void* stream);

/* out = dtype(float(y) - float(x)): a middle or last member's part of a spread step.
 * Replaces p2p/route.py:1268-1274 (_member's part). */
int p2p_member_part(const void* y, const void* x, void* out, int dtype, int64_t n_elem, void* stream);

/* ------------------------------------------------------------------------------------------------------------------
 * (3b) The step hop of a layer-parallel plan over NVLink peer memory, part and sum fused in
 * ------------------------------------------------------------------------------------------------------------------ */

/* What p2p_hop_send stores: P2P_PART_SUM: dtype(sum of float(parts)) in member order (one part: the part itself);
 * P2P_PART_DIFF: dtype(float(parts[0]) - float(h)), a middle or last member's part; P2P_PART_COMBINE: the whole group
 * combine of p2p_combine over parts, h and h_copy. */
enum { P2P_PART_SUM = 0, P2P_PART_DIFF = 1, P2P_PART_COMBINE = 2 };

/* Bytes of one rank's hop inbox: 256 bytes of counters, then n_ranks x ring slots of cap_elems elements (each 32 bits
 * of a part stored as a 64-bit word with the pass's flag, so a slot takes twice the part's bytes, rounded up to 256). Allocate it where every rank of the node addresses it (symmetric memory or CUDA IPC),
 * zeroed before the first hop; 0 for arguments out of range (1..8 ranks, 1..64 slots). */
size_t p2p_hop_inbox_bytes(int n_ranks, int64_t cap_elems, int dtype, int ring);

/* Sender side of the hop of pass `pass` (0, 1, 2, ... per sender and receiver pair; read from device memory at
 * *pass_at instead when pass_at is not null, so a CUDA graph can replay the hop pass after pass): computes this
 * rank's part (mode above) of n_elem elements and stores it into slot [me][pass % ring] of the inbox of every rank in dsts
 * (inboxes[r]: rank r's inbox as this GPU addresses it) as flagged words, so no separate signal follows. Before
 * storing it waits until each destination has consumed pass - ring of this rank. n_elem * element size a multiple of 16 bytes, at most
 * cap_elems; parts, h, h_copy 16-byte aligned. Waits are bounded by wait_us (1 ms .. 60 s); a wait that gives up is
 * reported by p2p_hop_status. Replaces p2p/route.py:800-810 (_send_piece, one NCCL isend per destination) with the
 * part of p2p/route.py:1268-1274 (_member) or the combine of p2p/replica.py:81-85 computed in the same pass. */
int p2p_hop_send(int mode, const void* const* parts, int n_parts, const void* h, const void* h_copy, int dtype,
                 int64_t n_elem, void* const* inboxes, int n_ranks, int me, const int* dsts, int n_dst, uint32_t pass,
                 const uint32_t* pass_at, int ring, int64_t cap_elems, int64_t wait_us, void* stream);

/* Receiver side: waits until every rank in srcs (member order) has stored its part of pass `pass` (or *pass_at)
 * into this rank's inbox, writes out = dtype(sum of float(parts)) in member order, and frees the slots for the senders. The same
 * n_elem, ring and cap_elems as the senders'. Replaces p2p/route.py:365-402 (_recv) with p2p/route.py:825-831
 * (_summed) in the same pass. A sender and receiver run on different GPUs, one process each, or on one GPU in stream
 * order with the sends first. */
int p2p_hop_recv(void* const* inboxes, int n_ranks, int me, const int* srcs, int n_src, uint32_t pass,
                 const uint32_t* pass_at, int ring, int64_t cap_elems, int dtype, int64_t n_elem, void* out,
                 int64_t wait_us, void* stream);

/* Adds 1 to each of the n (1..32) uint32 counters in device memory, on `stream`: the pass number a graphed pass reads
 * through pass_at moves on after the pass. No counterpart in the reference (it launches every pass from the host). */
int p2p_hop_advance(uint32_t* counters, int n, void* stream);

/* P2P_OK unless a hop wait since the last reset gave up (P2P_ECUDA, naming the side and the rank); reset != 0 clears
 * it. Syncs the stream. */
int p2p_hop_status(int reset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* P2P_B200_H */
