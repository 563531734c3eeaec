/*
 * fack_gemm.h -- C ABI of the B200 (sm_100a) FP8 block-scaled GEMM library.
 *
 * Computes, for e4m3 activations XQ[M,K] and weights WQ[N,K] (both K-major),
 *
 *   Y[m,n] (bf16) = sum_kb ( sum_{k in block kb} XQ[m,k] * WQ[n,k] )
 *                        * x_scale[m,kb] * w_scale[n/128,kb]
 *
 * with one fp32 activation scale per token per 128-wide K block and one fp32
 * weight scale per 128x128 weight block.  This is the arithmetic of the
 * reference's fp32 oracle, client/aiter/hsa/gfx942/driver.py:18-20, and of the
 * aiter operator it times, gemm_a8w8_blockscale_bpreshuffle_asm
 * (client/aiter/hsa/gfx942/driver.py:26-29; signature observed at
 * client/aiter/hsa/gfx942/dispatch_driver.py:62-63).
 *
 * Contract shared by every entry point:
 *   - plain pointers and sizes only; `stream` is a cudaStream_t (NULL = legacy
 *     default stream) passed as void*;
 *   - every argument is validated on the host and a non-zero status is
 *     returned before anything is launched; nothing aborts the process;
 *   - no entry point allocates, frees or synchronises, so every launch can be
 *     captured in a CUDA graph (the caller sizes and owns the workspace);
 *   - the device must be sm_100 (B200); other devices return
 *     FACK_ERR_UNSUPPORTED_ARCH;
 *   - the calling thread's current device (cudaGetDevice) must be the device
 *     that owns `stream` and the operands: per-device state (the plan's
 *     occupancy queries, the no-allocation scratch, the status word) is
 *     looked up for the current device, not derived from `stream`.
 */
#ifndef FACK_GEMM_H
#define FACK_GEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum fack_status {
  FACK_OK = 0,
  FACK_ERR_BAD_SHAPE = 1,       /* M<1 or M>8388480, N or K not a positive multiple of 128 */
  FACK_ERR_BAD_ALIGN = 2,       /* a pointer is NULL or misaligned */
  FACK_ERR_BAD_STRIDE = 3,      /* leading dimension / scale stride invalid */
  FACK_ERR_WS_TOO_SMALL = 4,    /* split-K workspace missing or too small */
  FACK_ERR_LAUNCH = 5,          /* the CUDA launch itself failed */
  FACK_ERR_UNSUPPORTED_ARCH = 6,/* current device is not sm_100 */
  FACK_ERR_BAD_ARG = 7,         /* other invalid argument (split_k, layout, g) */
  FACK_ERR_DEVICE_TIMEOUT = 8,  /* a kernel gave up waiting (device status) */
  FACK_ERR_CUDA = 9,            /* a CUDA runtime query failed */
  FACK_ERR_SCRATCH_LIMIT = 10   /* fack_gemm_bs_noalloc: built-in scratch too small */
};

/* Weight layouts accepted by fack_gemm_bs (argument `wq_packed`). */
enum fack_w_layout {
  FACK_W_ROW_MAJOR = 0,  /* WQ[N,K], row stride K bytes                       */
  FACK_W_PACKED = 1      /* output of fack_gemm_bs_prepack_w                   */
};

/* Sibling GEMM families of fack_gemm_tn (argument `kind`). */
enum fack_gemm_kind {
  FACK_GEMM_BF16 = 0,    /* bf16 A, B; fp32 accumulation                        */
  FACK_GEMM_I8 = 1       /* int8 A, B; s32 accumulation, per-row/column scales  */
};

/* Element types of the activation input to fack_quant_act (argument `x_dtype`). */
enum fack_dtype {
  FACK_DTYPE_F32 = 0,    /* fp32                                               */
  FACK_DTYPE_BF16 = 1    /* bf16                                               */
};

/* Status and version helpers: no counterpart in the reference, whose errors
 * are Python exceptions (client/aiter/runner.py:208-212 reports them). */

/* Human-readable text for a status code (static storage, never NULL). */
const char* fack_status_string(int status);

/* Library ABI version: 100 * major + minor. */
int fack_version(void);

/* Detail of the last failure on the calling thread (CUDA error name and
 * text where one was involved); empty if none.  Static per-thread storage. */
const char* fack_last_error(void);

/*
 * Full plan for an (M,N,K) problem: the token tile (128 = one CTA per tile;
 * 256 = a pair of CTAs sharing each tensor-core MMA through a 2-SM cluster,
 * each loading half of the weight rows; 16, 32 or 64 = swapped small-M tiles
 * for M <= the tile: 128 weight rows on the MMA's M side x all M tokens on its
 * N side, weight tile 128, at most 128 K blocks per slice, split-K always
 * through distributed shared memory, no workspace), the weight-tile width
 * (64, 128, 224 or 256), split-K (1..8; 2 x split <= 8 for pairs) -- 0 for any of them = the
 * library's choice; a 224-wide weight tile (four per 896 columns: one rank's
 * shard of a 7168-wide layer over 8 GPUs) is valid with 128-token tiles and
 * one K slice only, runs on the persistent kernel, and is chosen by request
 * or by a tuned-table row, never by the cost model; a 16-wide weight tile
 * (tile_m 16 or 0, split-K 1 or 0, M <= 16, K <= 256 x 128) is the small-M
 * kernel -- 16 weight rows per CTA, K split among the CTA's warps, no
 * workspace -- which the library picks for M <= 8, and for M <= 16 when
 * N > 4096 -- and the workspace bytes
 * fack_gemm_bs_ex needs for that plan when the caller supplies a workspace
 * (0 for a single K slice).  A
 * library choice of split-K queries the current device (cluster occupancy); an
 * explicit split does not.  When all three requests are 0, an exact-shape row
 * of the tuned table (fack_gemm_bs_tuned_*) for the current device's SM count
 * takes precedence over the cost model.  Plays the role of aiter's per-shape
 * kernelName/splitK selection (client/aiter/dispatch.py:142-150).
 */
int fack_gemm_bs_plan(int M, int N, int K, int tile_m_request, int tile_n_request,
                      int split_k_request, int* tile_m, int* tile_n, int* split_k,
                      size_t* workspace_bytes);

/*
 * Tile / split-K plan the library uses for an (M,N,K) problem.  Every CTA
 * computes a 128-token x tile_n-weight-row block of Y (tile_n = 64, 128 or
 * 256) over split_k slices of K.  split_k_request = 0 asks for the library's
 * own choice on the current device (the stand-in for aiter's tuned-CSV lookup
 * get_CKGEMM_config, client/aiter/dispatch.py:23-35 and
 * unittests/test_aiter_dispatch.py:472-477); a positive value is validated,
 * echoed, and paired with a tile chosen from the shape alone (no device
 * query).
 */
int fack_gemm_bs_select(int M, int N, int K, int split_k_request,
                        int* tile_n, int* split_k);

/*
 * The planner's cost-model estimate for one explicit plan (tile_m, tile_n,
 * split_k all given, valid for the shape as for fack_gemm_bs_tuned_set), in
 * SM cycles on the current device; 1e30 if the model would not offer it
 * (e.g. swapped small-M tiles whose clusters are not all resident at once).
 * For calibrating the model against measured times (python -m fack_b200.tune
 * --log); it launches nothing.  No counterpart in the reference, which
 * chooses kernels from tuned tables only.
 */
int fack_gemm_bs_plan_estimate(int M, int N, int K, int tile_m, int tile_n, int split_k, double* cycles);

/*
 * fack_gemm_bs_ex that also stores every bf16 result to n_peers (0..7) more
 * copies of the output block, peer_outs[i] + (row * ldo + column), with the
 * same ldo: the fused compute + all-gather of the column-sharded multi-GPU
 * path, where rank r writes its [M, N/g] block straight into every rank's
 * row-major Y[M, N] (out and each peer_outs[i] point at column r * N/g of a
 * rank's Y).  peer_outs are this process's mappings of other GPUs' memory
 * (fack_ipc_open_handle), 16-byte aligned; plain stores over NVLink, no
 * multicast.  The caller orders the launch between two barriers across the
 * ranks (e.g. a one-element all-reduce on the same stream): before it, so no
 * rank overwrites a Y another rank still reads; after it, so every rank's Y is
 * complete.  The kernel ends its peer stores with a system-scope fence.
 * No counterpart in the reference, which runs one GPU per process with no
 * collective (client/aiter/docs/validation.md:42-46).
 */
int fack_gemm_bs_bcast(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                       int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo,
                       void* const* peer_outs, int n_peers, int M, int N, int K, int tile_m, int tile_n, int split_k,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * Bytes of one rank's exchange state for fack_gemm_bs_allgather and
 * fack_xchg_barrier: device memory, 16-byte aligned, zero before its first
 * use, mapped into every other rank like the outputs (fack_ipc_*).
 */
#define FACK_XCHG_BYTES 128

/*
 * The fused compute + all-gather with its own completion: fack_gemm_bs_bcast
 * to the world - 1 peers (peer_outs, in rank order without `rank`), where
 * each CTA, once its blocks have landed, adds its share of the step to every
 * peer's exchange state over NVLink (peer_xchg[i] in the same order; the
 * shares of one launch sum to one step whatever its grid size) and CTA 0
 * waits, bounded by 10 s, until every peer's shares for this step have
 * arrived in this rank's state.  When the launch completes on `stream`,
 * this rank's Y holds every rank's block: no barrier or collective is needed
 * around it.  2 <= world <= 8.  On a wait that runs out the device status word
 * gets FACK_DEVICE_EXCHANGE (fack_device_status) and the launch still ends.
 *
 * Ordering contract: every rank makes the same sequence of allgather and
 * barrier calls on one stream with its exchange state.  A peer may store into
 * this rank's output as soon as every rank has completed the previous
 * exchange, so an output buffer must not be passed to two consecutive calls
 * while work that reads it may still be queued behind the first one; either
 * alternate between two registered outputs (work queued on `stream` before a
 * call is complete before any peer stores into the buffer of the call after
 * it) or put fack_xchg_barrier before the second call.
 * No counterpart in the reference (one GPU per process, no collective:
 * client/aiter/docs/validation.md:42-46).
 */
int fack_gemm_bs_allgather(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                           int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo,
                           void* const* peer_outs, void* xchg, void* const* peer_xchg, int rank, int world,
                           int M, int N, int K, int tile_m, int tile_n, int split_k,
                           void* workspace, size_t workspace_bytes, void* stream);

/*
 * One exchange step alone (a one-thread kernel on `stream`): signals every
 * peer, then waits (bounded by 10 s) until every peer has signalled, so that
 * no rank's next fack_gemm_bs_allgather stores into an output before every
 * rank's earlier work on its stream is complete.  Same arguments and
 * ordering contract as fack_gemm_bs_allgather.
 */
int fack_xchg_barrier(void* xchg, void* const* peer_xchg, int rank, int world, void* stream);

/* Device status bits (fack_device_status). */
#define FACK_DEVICE_PRODUCER 1u   /* a TMA producer's wait for a free stage ran out */
#define FACK_DEVICE_MMA 2u        /* the MMA issuer's wait ran out */
#define FACK_DEVICE_EPILOGUE 8u   /* a rescale / epilogue warp's wait ran out */
#define FACK_DEVICE_DRAIN 16u     /* draining in-flight copies or MMAs ran out */
#define FACK_DEVICE_EXCHANGE 32u  /* a peer's exchange signal did not arrive */
#define FACK_DEVICE_QUANT 64u     /* a wait in the activation quantiser ran out */
#define FACK_DEVICE_TN 128u       /* a wait in the sibling GEMM (fack_gemm_tn) ran out */

/*
 * CUDA IPC for the peer outputs.  fack_ipc_get_handle: the IPC handle (64
 * bytes into `handle`, handle_bytes >= 64) of the allocation holding `ptr` and
 * ptr's byte offset inside it (allocators hand out sub-ranges).  Another
 * process on the node opens the handle with fack_ipc_open_handle, adds the
 * offset, and releases it with fack_ipc_close_handle.  No counterpart in
 * the reference (one GPU per process, no exchange between them).
 */
int fack_ipc_get_handle(const void* ptr, void* handle, size_t handle_bytes, size_t* offset);
int fack_ipc_open_handle(const void* handle, void** base);
int fack_ipc_close_handle(void* base);

/*
 * Exact-shape plan table, the B200 counterpart of aiter's tuned GEMM CSV
 * (rows keyed by cu_num, M, N, K with kernelName and splitK;
 * client/aiter/dispatch.py:23-35, exact match only, dispatch.py:3-6).  Rows
 * are keyed by (SM count, M, N, K) and fix tile_m, tile_n and split_k of the
 * automatic plan for exactly that shape; other shapes keep the cost model.
 * The table is process-wide and thread-safe.
 *
 * fack_gemm_bs_tuned_set: add or replace one row (BAD_SHAPE / BAD_ARG if the
 *   plan is not valid for the shape, as for an explicit request).
 * fack_gemm_bs_tuned_lookup: the row for a key, or 0, 0, 0 if there is none.
 * fack_gemm_bs_tuned_count / _clear: number of rows / remove all rows.
 * fack_gemm_bs_tuned_load: merge a CSV file.  '#' lines are comments, the
 *   first other line is a header, columns are found by name: cu_num, M, N, K,
 *   kernelName (fack_bs_sm100_t{128|256}x{64|128|256}_s{S}, or the swapped
 *   small-M fack_bs_sm100_t{16|32|64}x128_s{S}) are required, splitK (= S)
 *   and errRatio (= 0) are checked when present.  Rows naming another
 *   library's kernel are skipped and counted in *rows_skipped; a name with
 *   this library's prefix that is not in that canonical form is a bad row.  The
 *   whole file is checked before any row is added; on a bad row the table is
 *   unchanged, BAD_ARG is returned and fack_last_error gives "path:line: why".
 *   A later row for the same key replaces an earlier one.
 */
int fack_gemm_bs_tuned_set(int cu_num, int M, int N, int K, int tile_m, int tile_n, int split_k);
int fack_gemm_bs_tuned_lookup(int cu_num, int M, int N, int K, int* tile_m, int* tile_n,
                              int* split_k);
int fack_gemm_bs_tuned_count(void);
int fack_gemm_bs_tuned_clear(void);
int fack_gemm_bs_tuned_load(const char* path, int* rows_loaded, int* rows_skipped);

/*
 * The same exact-shape table for the sibling families (fack_gemm_tn), the
 * counterpart of aiter's bf16 and a8w8 tuned GEMM tables that the reference
 * names beside the blockscale one (client/aiter/dispatch.py:24-27): rows
 * keyed by (kind = FACK_GEMM_BF16 | FACK_GEMM_I8, SM count, M, N, K) fix
 * tile_m, tile_n and split_k of fack_gemm_tn_plan's fully automatic plan (all
 * three requests 0).  Rows are checked by fack_gemm_tn_plan's rules for an
 * explicit plan.  The CSV form is the FP8 table's, with kernelName
 * fack_tn_sm100_{bf16|i8}_t{128|256}x{64|128|256}_s{S} (the name gives the
 * kind); rows naming other kernels, the FP8 ones included, are skipped.
 * _count / _clear touch the sibling rows only (and the FP8 functions the FP8
 * rows only).
 */
int fack_gemm_tn_tuned_set(int kind, int cu_num, int M, int N, int K, int tile_m, int tile_n, int split_k);
int fack_gemm_tn_tuned_lookup(int kind, int cu_num, int M, int N, int K, int* tile_m, int* tile_n,
                              int* split_k);
int fack_gemm_tn_tuned_count(void);
int fack_gemm_tn_tuned_clear(void);
int fack_gemm_tn_tuned_load(const char* path, int* rows_loaded, int* rows_skipped);

/*
 * Bytes of workspace fack_gemm_bs needs for this problem and split (0 when the
 * plan has a single K slice).  Replaces the allocation the aiter launcher does
 * internally (csrc/py_itfs_cu/asm_a8w8_blockscale_bpreshuffle.cu, a missing
 * upstream file named at client/aiter/hsa/gfx942/manifest.json:12).
 */
int fack_gemm_bs_workspace_size(int M, int N, int K, int split_k, size_t* bytes);

/*
 * Optional weight pre-pack, the stand-in for aiter's BpreShuffle
 * (shuffle_weight(b, layout=(16,16)), client/aiter/hsa/gfx942/driver.py:21).
 * Rewrites WQ[N,K] (row stride ldw bytes) into 128x128 tiles, tile (nb,kb) at
 * ((nb*K/128)+kb)*16384 bytes, each tile stored in the exact 128-byte-swizzled
 * image the kernel's shared-memory stage expects, so one TMA box per tile is a
 * straight 16 KB copy.  wq_packed must hold N*K bytes.  w_scale needs no
 * repacking: ws_packed may be NULL; when it is not, the [N/128,K/128] fp32
 * scales are copied there unchanged.
 */
int fack_gemm_bs_prepack_w(const void* wq, int64_t ldw, const float* w_scale,
                           int N, int K, void* wq_packed, float* ws_packed,
                           void* stream);

/*
 * The GEMM.  Replaces aiter's gemm_a8w8_blockscale_bpreshuffle_asm(a, b, out,
 * x_scale, w_scale, bias=None, splitK, kernelName, bpreshuffle, zero_bias_buf)
 * (client/aiter/hsa/gfx942/dispatch_driver.py:62-63; positional launch tuple
 * pinned at unittests/test_aiter_dispatch.py:504-505).
 *
 *   M, N, K   1 <= M <= 8388480 (65535 tiles of 128 tokens); N and K positive
 *             multiples of 128
 *   xq        e4m3 activations, row m at xq + m*ldx (ldx >= K, ldx % 16 == 0)
 *   wq        e4m3 weights, FACK_W_ROW_MAJOR ([N,K], row stride K) or
 *             FACK_W_PACKED (fack_gemm_bs_prepack_w output)
 *   x_scale   fp32, element (m,kb) at x_scale[m*xs_stride_m + kb*xs_stride_kb];
 *             the reference's transposed-contiguous view
 *             (sa.T.contiguous().view_as(sa), driver.py:22) is
 *             xs_stride_m = 1, xs_stride_kb = M; logical row-major is
 *             xs_stride_m = K/128, xs_stride_kb = 1
 *   w_scale   fp32 [N/128, K/128] row-major
 *   out       bf16 [M,N], row stride ldo elements (ldo >= N, ldo % 8 == 0);
 *             every element of the MxN block is written exactly once
 *   split_k   0 = library choice, else 1..8 (and <= K/128)
 *   workspace fp32 partials for split_k > 1, at least
 *             fack_gemm_bs_workspace_size() bytes, 16-byte aligned; NULL
 *             combines the K slices through distributed shared memory
 *
 * The split-K reduction is deterministic: slices are summed in a fixed order,
 * so repeated calls give bitwise-identical outputs.
 */
int fack_gemm_bs(const void* xq, int64_t ldx, const void* wq, int wq_packed,
                 const float* x_scale, int64_t xs_stride_m, int64_t xs_stride_kb,
                 const float* w_scale, void* out, int64_t ldo,
                 int M, int N, int K, int split_k,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Optional workspace of a single-slice plan (split_k resolves to 1, 128-token
 * tiles) whose tiles outnumber the current device's SMs.  Such a plan runs on
 * one persistent CTA per SM, and T tiles on G SMs leave a last round of
 * T mod G tiles (1792 = 12 x 148 + 16 for the prefill layer) during which
 * most SMs idle.  Given a workspace of at least *bytes (16-byte aligned) in
 * fack_gemm_bs / fack_gemm_bs_ex, those last tiles are cut into 2..8 K slices
 * spread over the idle SMs; each slice writes an fp32 partial there and a
 * second, small launch in the same stream sums the slices in a fixed order
 * (deterministic) and stores the bf16 tiles.  Without the workspace (NULL or
 * smaller) the plan runs unsplit.  The two results differ only in the fp32
 * summation order of those tiles.  *bytes = 0 when the plan has no such tail.
 * Same tile / split requests as fack_gemm_bs_plan; queries the current device.
 * No counterpart in the reference (its tile kernels are not persistent).
 */
int fack_gemm_bs_tail_workspace_size(int M, int N, int K, int tile_m_request, int tile_n_request,
                                     int split_k_request, size_t* bytes);

/*
 * fack_gemm_bs with an explicit plan (tile_m, tile_n, split_k; 0 = library
 * choice), the counterpart of aiter selecting one tile kernel by kernelName
 * (client/aiter/hsa/gfx942/driver.py:26-29 passes kernelName=symbol).
 * For split_k > 1 the K slices of a tile are combined either through the
 * caller's workspace (when `workspace` is not NULL; at least the plan's
 * workspace bytes) or, with workspace = NULL, through the distributed shared
 * memory of the tile's thread-block cluster (no global memory).  For a
 * single-slice plan the workspace is optional and enables the tail split of
 * fack_gemm_bs_tail_workspace_size when it is large enough.
 */
int fack_gemm_bs_ex(const void* xq, int64_t ldx, const void* wq, int wq_packed,
                    const float* x_scale, int64_t xs_stride_m, int64_t xs_stride_kb,
                    const float* w_scale, void* out, int64_t ldo,
                    int M, int N, int K, int tile_m, int tile_n, int split_k,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * fack_gemm_bs without a workspace argument, for callers that cannot call
 * cudaMalloc when they run the GEMM: an engine plugin whose enqueue path must
 * neither allocate nor synchronise (cudaMalloc may synchronise the device), or
 * a process whose device memory is wholly owned by another allocator with a
 * fixed budget.  No counterpart in the
 * reference (aiter's launcher allocates its own buffers).
 *
 * The split-K partial sums go to one 16 MiB buffer compiled into this library
 * (every GPU that loads the library keeps it until the process exits).  With
 * split_k = 0 the library picks its best plan whose partials fit the buffer;
 * an explicit split_k whose partials do not fit returns FACK_ERR_SCRATCH_LIMIT
 * before anything is launched (a smaller split_k, or fack_gemm_bs with your
 * own workspace, avoids that).  Nothing in the buffer has to start at zero: each
 * call writes every partial it later reads.
 *
 * The buffer is shared by all calls on a device and keeps the last call's
 * contents, so calls whose kernels may overlap on the GPU (for example on
 * two streams without an ordering between them) race and corrupt each other;
 * order them on one stream.  The first call on each device looks up the
 * buffer's device address (a runtime query, no allocation): make that first
 * call before any stream capture.  The buffer used is the current device's
 * (cudaGetDevice), so make the device that owns `stream` current before the
 * call.  It calls no cudaMalloc or cudaFree.
 */
int fack_gemm_bs_noalloc(const void* xq, int64_t ldx, const void* wq, int wq_packed,
                         const float* x_scale, int64_t xs_stride_m, int64_t xs_stride_kb,
                         const float* w_scale, void* out, int64_t ldo,
                         int M, int N, int K, int split_k, void* stream);

/*
 * Column interleave for the N-sharded multi-GPU path: `gathered` holds g
 * contiguous bf16 shards [g][M][n_shard] (the layout an all-gather of each
 * rank's [M, n_shard] output produces); writes out[m, r*n_shard + c] =
 * gathered[r][m][c] with row stride ldo.  n_shard % 8 == 0, ldo % 8 == 0.
 * No reference counterpart: the reference runs one GPU per process
 * (client/aiter/docs/validation.md:42-46).
 */
int fack_gather_interleave(const void* gathered, int g, int M, int n_shard,
                           void* out, int64_t ldo, void* stream);

/*
 * Fused activation quantisation producing the GEMM's XQ and x_scale in one
 * pass over X (fp32 or bf16 [M, K], row stride ldx elements):
 *   x_scale[m, kb] = amax(|X[m, kb*128 .. kb*128+127]|) / 240  (1 if all zero)
 *   xq[m, k]       = e4m3fn(clamp(X[m, k] / x_scale[m, k/128], -240, 240))
 * (round to nearest even), the construction of the benchmark inputs; bf16
 * input is widened to fp32 first.  x_scale element (m, kb) is written at
 * x_scale[m*xs_stride_m + kb*xs_stride_kb], so the reference's
 * transposed-contiguous view sa.T.contiguous().view_as(sa)
 * (client/aiter/hsa/gfx942/driver.py:22) is xs_stride_m = 1,
 * xs_stride_kb = M.  K % 128 == 0; x 16-byte aligned with ldx % 8 == 0;
 * xq 16-byte aligned with ldq % 16 == 0.  The reference takes X already
 * quantised (driver.py:14-17); this is the step before the GEMM, fused.
 */
int fack_quant_act(const void* x, int x_dtype, int64_t ldx, int M, int K, void* xq, int64_t ldq,
                   float* x_scale, int64_t xs_stride_m, int64_t xs_stride_kb, void* stream);

/*
 * The sibling GEMM families the reference drives through the same client
 * (client/aiter/hsa/gfx942/gemm_driver.py:32-79), both "TN" (A[M,K] and
 * B[N,K] row-major, K contiguous), bf16 output Y[M,N] with row stride ldo:
 *
 *   kind = FACK_GEMM_BF16: Y = bf16(A . B^T (+ bias)), A and B bf16, fp32
 *     accumulation; a_scale and b_scale must be NULL (gemm_driver.py:50,
 *     aiter's gemm_a16w16_asm).
 *   kind = FACK_GEMM_I8: Y = bf16((float(A . B^T) * a_scale[m]) * b_scale[n]
 *     (+ bias[n])), A and B int8, exact s32 accumulation, each product and
 *     the sum rounded in fp32 in that order (gemm_driver.py:73, aiter's
 *     gemm_a8w8_asm with per-token scales and an fp32 bias).
 *
 * lda / ldb / ldo are in elements; A and B rows 16-byte aligned (lda, ldb
 * times the element size a multiple of 16; the reference pads int8 rows to
 * K + 128); ldo % 8 == 0.  K x element size % 128 == 0 (bf16: K % 64, int8:
 * K % 128); N % 64 == 0; 1 <= M <= 8388480.  b_packed = 1 takes B from
 * fack_gemm_bs_prepack_w applied to B's bytes (N rows of K x element size
 * bytes; ldb is then ignored).  bias is optional (NULL).  tile_m (128 = one
 * CTA per 128-row tile, 256 = a pair of CTAs sharing each MMA through
 * cta_group::2), tile_n (64, 128, 256) and split_k (1..8; 2 x split <= 8 for
 * pairs): 0 = the library's choice (fack_gemm_tn_plan, which queries the
 * current device unless all three are given).  Capturable; allocates nothing.
 */
int fack_gemm_tn_plan(int kind, int M, int N, int K, int tile_m_request, int tile_n_request, int split_k_request,
                      int* tile_m, int* tile_n, int* split_k);
int fack_gemm_tn(int kind, const void* a, int64_t lda, const void* b, int b_packed, int64_t ldb,
                 const float* a_scale, const float* b_scale, const float* bias, void* out, int64_t ldo, int M,
                 int N, int K, int tile_m, int tile_n, int split_k, void* stream);

/*
 * Reads (and with reset != 0 clears) the current device's error word, which a
 * kernel sets when a bounded wait inside it gives up.  Synchronises `stream`.
 * *flags == 0 means no kernel has reported a problem.  Returns
 * FACK_ERR_DEVICE_TIMEOUT when flags are set, FACK_OK otherwise.  No
 * counterpart in the reference (its kernels have no bounded waits to report).
 */
int fack_device_status(void* stream, unsigned int* flags, int reset);

#ifdef __cplusplus
}
#endif

#endif /* FACK_GEMM_H */
