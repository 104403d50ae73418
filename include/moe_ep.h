/*
 * moe_ep.h — C ABI of the B200 fused MoE expert-parallel layer
 * (libmoe_ep.so, built from nvshmem_testing_b200/csrc).
 *
 * Every entry point is extern "C", takes plain pointers and sizes, and
 * returns an int status (MOE_EP_OK on success).  Device pointers are CUDA
 * device addresses; `stream` is a cudaStream_t passed as void*.  No call
 * synchronises the stream unless stated.
 *
 * Which reference interface each entry point replaces (paths are within the
 * jy1534/nvshmem_testing project):
 *   moe_route, moe_pack_padded  utils.py:28-69  (bucketize, pad, coalesce)
 *   moe_publish_i32             utils.py:45-49  (the largest bucket, read on
 *                               the host to size the padded chunk)
 *   moe_symm_*                  alltoall_persistent_gemm.py:161-204
 *                               (_get_symm_buffers: symmetric receive and
 *                               signal buffers, rendezvous)
 *   moe_ep_workspace_layout     alltoall_persistent_gemm.py:187-195
 *                               (receive [W*transmit, H] + signal [W] shapes)
 *   moe_ep_read_status          (status word; the reference has no error path)
 *   moe_ep_run_noalloc          no counterpart (see its declaration)
 *   moe_ep_run                  alltoall_persistent_gemm.py:207-309 (run:
 *                               peer copies + flags + fused grouped GEMM) and
 *                               baseline.py:8-56 (same output contract)
 *   moe_swiglu,                 the full expert MLP's activation, separate or
 *   moe_ep_run_compact_swiglu   in the first GEMM's epilogue (the reference's
 *                               expert is one GEMM, baseline.py:50)
 *   moe_router                  utils.py:17-25 (router logits einsum, softmax,
 *                               top-k: the step before the reference's path)
 *   moe_pack_compact,           the general (unbalanced) all-to-all that
 *   moe_ep_run_compact          alltoall_persistent_gemm.py:221-222 and
 *                               baseline.py:15-16 leave as stubs: unpadded
 *                               send buffer and output
 *   moe_route_slots,            the step after the reference's path: the
 *   moe_ep_workspace_layout_ret, return of expert outputs to their source
 *   moe_ep_run_combine          ranks and the top-k weighted sum with the
 *                               router weights that utils.py:24-25 computes
 *                               (top_vals) and the reference never uses
 */
#ifndef MOE_EP_H
#define MOE_EP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  Device-side errors are also latched in the workspace status
 * word as (code << 24) | (site << 16) | detail. */
#define MOE_EP_OK 0
#define MOE_EP_BAD_ARG 1
#define MOE_EP_CUDA_ERR 2
#define MOE_EP_TIMEOUT 3
#define MOE_EP_CAPACITY 4
#define MOE_EP_BAD_ROUTE 5

#define MOE_EP_ABI_VERSION 3

int moe_ep_abi_version(void);
const char* moe_ep_status_string(int code);
/* Number of SMs of `device`. */
int moe_ep_num_sms(int device, int* out);

/* ---------------------------------------------------------------- routing
 * Replaces the per-expert mask loop of utils.py:28-41.
 *   top_idxs  [T, K] int32 (ids_are_int64 = 0) or int64 (= 1) expert ids
 *   counts    [E]    tokens per expert; a token counts once per expert even
 *                    if the id repeats in its row (utils.py:31 `.any(-1)`);
 *                    ids outside [0, E) match no expert.
 *   offsets   [E+1]  exclusive scan of counts
 *   perm      [T*K]  perm[offsets[e] + j] = j-th token (ascending) of expert e
 *   max_count [1]    max over e of counts[e] (utils.py:45, local max)
 * E <= 1024, K <= 32.  One cluster of 8 CTAs, each routing a contiguous
 * token range; they find their bucket offsets from each other's counts
 * through distributed shared memory (no scratch memory). */
int moe_route(const void* top_idxs, int ids_are_int64, int64_t T, int K, int E, int32_t* counts, int32_t* offsets,
              int32_t* perm, int32_t* max_count, void* stream);

/* Replaces the router of utils.py:17-25 (the step before the path):
 *   logits [T, E] bf16 = x [T, H] @ router_w [H, E]   (bf16 in, fp32
 *                        accumulation rounded once to bf16)
 *   probs              = softmax over E in fp32, rounded to bf16
 *   top_idxs [T, K]    = the K most probable experts, descending, equal
 *                        probabilities by ascending id (int64 or int32)
 *   top_vals [T, K]    = their probabilities (bf16 values as float32)
 * `logits` receives the bf16 logits (16-byte aligned).  Requires H % 8 == 0,
 * 8 <= E <= 1024 with E % 8 == 0, 1 <= K <= min(E, 32).  Allocates nothing.
 * E <= 256: one kernel (split-K clusters on the tensor cores, the partial
 * logits reduced through distributed shared memory, softmax and top-k in its
 * epilogue); it keeps no state between calls, so calls may overlap.
 * E > 256: the fused layer kernel's GEMM, whose control words live in a
 * fixed 2 KB array inside the library, then a softmax/top-k kernel; such
 * calls must not overlap each other on the GPU, and the first one on a
 * device looks the array up (make it before any stream capture).
 * status_host: optional mapped pinned word that receives a device-side error
 * (a pipeline wait that exceeded its bound), encoded as the workspace status
 * word; NULL discards it. */
int moe_router(const void* x, int64_t T, int32_t H, const void* router_w, int32_t E, int32_t K, void* logits,
               void* top_idxs, int32_t ids_are_int64, float* top_vals, int32_t* status_host, void* stream);

/* moe_route plus, for the return path,
 *   slots     [T, K] int32: j such that perm[offsets[e] + j] = t for
 *                    e = top_idxs[t, k] (the token's row inside bucket e,
 *                    i.e. padded send row e*gm + j); -1 where the id is
 *                    outside [0, E) or repeats an earlier id of the row. */
int moe_route_slots(const void* top_idxs, int ids_are_int64, int64_t T, int K, int E, int32_t* counts,
                    int32_t* offsets, int32_t* perm, int32_t* slots, int32_t* max_count, void* stream);

/* Copies n int32 words from src (device) to dst with a kernel, in stream
 * order.  For sizes computed on the device that the host must read before
 * it can size the next buffers (utils.py:45-49: the largest bucket decides
 * the padded chunk): dst may be pinned host memory, which the GPU writes over
 * PCIe without a copy engine, so the host's wait (an event after this call)
 * does not queue behind a bulk device-to-host copy on another stream.
 * n <= 2^20. */
int moe_publish_i32(const int32_t* src, int64_t n, int32_t* dst, void* stream);

/* Replaces utils.py:54-69: out[e*gm + j, :] = tokens[perm[offsets[e] + j], :]
 * for j < counts[e] and zero rows for counts[e] <= j < gm.  Requires
 * H * elem_bytes % 16 == 0 and gm >= max(counts). */
int moe_pack_padded(const void* tokens, int64_t H, int elem_bytes, const int32_t* counts, const int32_t* offsets,
                    const int32_t* perm, int E, int64_t gm, void* out, void* stream);

/* The general all-to-all's send buffer (no counterpart in the reference,
 * whose general_a2a path is a stub): out[r, :] = tokens[perm[r], :] for
 * r < rows, with rows = offsets[E] of moe_route, i.e. every bucket back to
 * back in expert order without padding. */
int moe_pack_compact(const void* tokens, int64_t H, int elem_bytes, const int32_t* perm, int64_t rows, void* out,
                     void* stream);

/* ---------------------------------------------------------------- symmetric memory
 * Replaces the torch symmetric-memory allocation + rendezvous of
 * alltoall_persistent_gemm.py:161-204 with cuMem VMM: the owner allocates
 * device memory exportable as a POSIX file descriptor; each peer imports the
 * descriptor (passed over a Unix socket by the host) and maps it. */
int moe_symm_alloc(int device, size_t bytes, size_t* mapped_bytes, uint64_t* ptr, int* fd, uint64_t* handle);
int moe_symm_import(int device, int fd, size_t bytes, uint64_t* ptr, uint64_t* handle);
int moe_symm_free(uint64_t ptr, size_t bytes, uint64_t handle);

/* Byte layout of one rank's symmetric workspace (identical on every rank). */
typedef struct moe_ep_layout {
  uint64_t off_cmat;   /* int32 [2][W owner][W src][El]: published recv counts  */
  uint64_t off_cflag;  /* uint32 [2][W owner]: count arrival epochs            */
  uint64_t off_dflag;  /* uint32 [2][W src][El][max_chunks]: row-chunk epochs  */
  uint64_t off_free;   /* uint32 [W peer]: last epoch the peer finished        */
  uint64_t off_local;  /* uint32 [8]: work counters and the status word        */
  uint64_t ctrl_bytes; /* bytes [0, ctrl_bytes) must start zeroed              */
  uint64_t off_data;   /* element [2][cap_rows][H]: compact remote rows        */
  uint64_t total_bytes;
  uint64_t off_rflag;  /* uint32 [W peer]: last epoch the peer returned rows   */
  uint64_t off_ret;    /* bf16 [ret_rows][ret_cols]: returned expert outputs   */
  uint64_t ret_bytes;  /* 0 without a return region                            */
} moe_ep_layout;

int moe_ep_workspace_layout(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks,
                            moe_ep_layout* out);
/* The same layout with a return region of ret_rows x ret_cols bf16 (for
 * moe_ep_run_combine: ret_rows >= W*El*gm, ret_cols = out_dim). */
int moe_ep_workspace_layout_ret(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks,
                                int64_t ret_rows, int64_t ret_cols, moe_ep_layout* out);

/* Zero the control region [0, ctrl_bytes) of a freshly allocated workspace
 * (counts, flags, epochs, counters).  Every rank must do this, and all ranks
 * must have done it, before the first moe_ep_run on the workspace. */
int moe_ep_workspace_reset(uint64_t local_base, const moe_ep_layout* layout, void* stream);

/* ---------------------------------------------------------------- fused layer
 * Replaces alltoall_persistent_gemm.run (alltoall_persistent_gemm.py:207-309):
 *   out[le, src*gm + i, :] = tokens_src[(rank*El + le)*gm + i, :] @ weights[le]
 * for i < recv_counts[src, le]; rows i >= recv_counts[src, le] are written as
 * zeros.  bf16 in, fp32 accumulate, bf16 out.
 * Collective: every rank calls with the same W, El, gm, H, N, epoch. */
typedef struct moe_ep_run_params {
  int32_t world_size;          /* W                                                  */
  int32_t rank;                /* this rank                                          */
  int32_t local_experts;       /* El                                                 */
  int32_t hidden;              /* H: GEMM K, multiple of 8                           */
  int32_t out_dim;             /* N: multiple of 8                                   */
  int32_t elem_bytes;          /* 2 (bf16)                                           */
  int64_t gm;                  /* padded rows per (rank, expert) slot                */
  const void* tokens;          /* [W*El*gm, H] this rank's padded send buffer        */
  const void* weights;         /* [El, H, N] local experts, N contiguous             */
  const int32_t* recv_counts;  /* [W, El] rows this rank receives per (src, expert)  */
  void* out;                   /* [El, W*gm, N]                                      */
  const uint64_t* peer_bases;  /* device array [W]: every rank's workspace, mapped  */
  uint64_t local_base;         /* this rank's workspace base address                */
  int64_t cap_rows;            /* remote receive capacity (rows) per parity          */
  int32_t push_rows;           /* rows per push item and arrival flag                */
  int32_t max_chunks;          /* flag slots per (src, expert)                       */
  uint32_t epoch;              /* call counter: 1, 2, 3, ... identical on all ranks  */
  uint32_t num_ctas;           /* 0 = one CTA per SM                                 */
  uint64_t timeout_ns;         /* bound on every wait for a peer                     */
  int32_t* status_host;        /* optional mapped pinned word for device errors      */
  uint64_t* trace;             /* optional device timeline, MOE_EP_TRACE_WORDS per  */
                               /* CTA (NULL = off); see MOE_EP_TRACE_* below         */
  int32_t push_ctas;           /* CTAs (even, at the end of the grid) that only     */
                               /* move rows to peers and zero padded rows, with all */
                               /* their warps; 0 = two push warps in every CTA      */
  int32_t local_first;         /* experts whose local tiles all run before any      */
                               /* remote tile (0 = expert-major order throughout)   */
  int32_t counts_are_send;     /* 1: recv_counts holds this rank's SEND counts      */
                               /* [W dst, El] (the routing's per-expert counts)     */
                               /* instead of its receive counts; the kernel's own   */
                               /* count exchange then replaces the host-side count  */
                               /* all-to-all of benchmark.py:114-118                */
  int32_t push_warps;          /* push_ctas == 0: warps of every CTA that move rows */
                               /* (1..6; 0 = 2)                                     */
  int32_t push_mode;           /* MOE_EP_PUSH_* bits                                */
  int32_t sched_mode;          /* MOE_EP_SCHED_* bits (0: one fixed tile order)     */
} moe_ep_run_params;

/* sched_mode bits.  READY_FIRST (more than one rank): a CTA pair takes the
 * next remote tile when every row it reads has landed and a local tile
 * otherwise (local tiles from their own counter), so that local work fills
 * the waits for rows in flight; local_first is then ignored. */
#define MOE_EP_SCHED_READY_FIRST 1
/* MERGED (more than one rank): an expert whose local rows (padded to 8) and
 * remote rows together fit 128 rows gets one tile per weight slice covering
 * both, instead of a local and a remote tile that each stream the slice
 * (small experts are weight-bound: decode shapes); larger experts keep
 * separate local and remote tiles. */
#define MOE_EP_SCHED_MERGED 2
/* Bits 4-7: row groups G for the remote tiles of each expert (more than one
 * rank).  Feature-major order (every row tile of a weight slice, then the
 * next slice) needs all of an expert's remote rows within the first slices;
 * with G > 1 the expert's remote row tiles are split into G contiguous
 * groups, taken one after another, each feature-major, so the tiles of rows
 * that land first (sources arrive in order me+1, me+2, ...) run first, at
 * the cost of reading each weight slice from HBM once per group.  0 chooses:
 * W-1 groups for an expert whose remote tiles per group would still fill
 * every computing pair (large experts: Mixtral's shapes), else 1. */
#define MOE_EP_SCHED_ROW_GROUPS_SHIFT 4
#define MOE_EP_SCHED_ROW_GROUPS_MASK 0xF0

/* push_mode bits.  BULK: push CTAs move rows with TMA bulk copies (local rows
 * through a ring of shared-memory pieces to the peer) instead of loads and
 * stores.  BY_DESTINATION: senders go through destinations one at a time
 * (me-1, me-2, ...; experts in order within each) instead of finishing each
 * expert for every destination before the next. */
#define MOE_EP_PUSH_BULK 1
#define MOE_EP_PUSH_BY_DESTINATION 2
/* HYBRID: with push CTAs, the computing CTAs' push_warps warps move rows too
 * (all take items from one counter). */
#define MOE_EP_PUSH_HYBRID 4
/* L2_STREAM: the push's loads of the send buffer and the stores of the
 * output mark their lines evict-first in L2 (each is touched once), so that
 * L2 keeps the weight slices and rows that several tiles read. */
#define MOE_EP_PUSH_L2_STREAM 8

/* Device timeline (globaltimer ns, or counts), one record per CTA. */
#define MOE_EP_TRACE_WORDS 24
#define MOE_EP_TRACE_START 0          /* kernel entry                                */
#define MOE_EP_TRACE_COUNTS 1         /* all count blocks arrived                    */
#define MOE_EP_TRACE_SCHED 2          /* schedule built                              */
#define MOE_EP_TRACE_PRODUCER_END 3   /* TMA producer finished its tiles             */
#define MOE_EP_TRACE_MMA_END 4        /* MMA issuer finished (leader CTAs)           */
#define MOE_EP_TRACE_EPI_END 5        /* epilogue finished                           */
#define MOE_EP_TRACE_PUSH_END 6       /* this CTA's last NVLink push item done       */
#define MOE_EP_TRACE_ZERO_END 7       /* padded-row zeroing done                     */
#define MOE_EP_TRACE_END 8            /* teardown done                               */
#define MOE_EP_TRACE_TILES 9          /* tiles processed (count)                     */
#define MOE_EP_TRACE_FLAG_WAIT 10     /* ns the producer spent waiting for rows      */
#define MOE_EP_TRACE_FULL_WAIT 11     /* ns the MMA issuer spent waiting for stages  */
#define MOE_EP_TRACE_PUSH_ITEMS 12    /* push items done (count)                     */
#define MOE_EP_TRACE_PUSH_BYTES 13    /* bytes pushed over NVLink                    */
#define MOE_EP_TRACE_EMPTY_WAIT 14    /* ns the producer spent waiting for free stages */
#define MOE_EP_TRACE_EPI_WAIT 15      /* ns the epilogue spent waiting for accumulators */
#define MOE_EP_TRACE_ACC_WAIT 16      /* ns the MMA issuer waited for a free accumulator */
#define MOE_EP_TRACE_MMA_ISSUE 17     /* ns the MMA issuer spent issuing (not waiting) */
#define MOE_EP_TRACE_KBLOCKS 18       /* k-blocks issued by the MMA issuer (count)    */

int moe_ep_run(const moe_ep_run_params* params, void* stream);

/* The general (unbalanced) all-to-all: moe_ep_run without padding, for the
 * general_a2a=True path that the reference leaves unimplemented
 * (alltoall_persistent_gemm.py:221-222, baseline.py:15-16).
 *   tokens [send_rows, H]: the cells (d, le) — rows for rank d's local expert
 *          le — back to back in (d, le) order, recv_counts_d[rank, le] rows
 *          each (moe_pack_compact output);
 *   out    [out_rows, N]: the cells (le, src) back to back in (le, src)
 *          order, recv_counts[src, le] rows each: row
 *          sum_{(le',s') < (le,src)} recv_counts[s', le'] + i is
 *          tokens_src[that cell's row i] @ weights[le].
 * gm is a bound on every count (the workspace is sized by it); nothing is
 * zero-filled.  A cell layout larger than send_rows or out_rows latches
 * MOE_EP_BAD_ARG on the device instead of touching memory beyond them. */
int moe_ep_run_compact(const moe_ep_run_params* params, int64_t send_rows, int64_t out_rows, void* stream);

/* No counterpart in the reference.  The single-rank form of moe_ep_run for
 * callers that cannot allocate device memory: a host that reaches the library
 * only through this C ABI and owns no CUDA allocator, a process whose device
 * memory is fixed after start-up, or a one-GPU user who does not want the
 * exportable cuMem workspace that moe_ep_run needs.  The kernel's control
 * words live in a fixed __device__ array inside the library
 * (MOE_EP_NOALLOC_SCRATCH_BYTES on every GPU that loads it, held until the
 * process exits); the caller still passes tokens, weights, recv_counts and
 * out.  Requires world_size == 1 and rank == 0; peer_bases, local_base,
 * cap_rows, push_rows, max_chunks and epoch are ignored.  More than
 * MOE_EP_NOALLOC_MAX_EXPERTS local experts returns MOE_EP_SCRATCH_LIMIT.
 * Allocates nothing: no cudaMalloc/cudaFree, no allocating library call.
 * The first call on a device looks up the array's address (a host-side
 * lookup), so make that call before any stream capture; every call then
 * prepares the array in stream order (a one-block kernel writes the one-entry
 * peer table and clears the control words the previous call left) and
 * launches the layer.  Every call reuses the same array, so calls whose
 * kernels overlap on the GPU (different streams, or several threads) race and
 * must not be made; calls queued on one stream are fine.  Device-side errors
 * (a count above gm, a timed-out wait) are reported only through the mapped
 * pinned word status_host, which is therefore required (NULL returns
 * MOE_EP_BAD_ARG); the caller clears it between calls. */
#define MOE_EP_SCRATCH_LIMIT 6
#define MOE_EP_NOALLOC_MAX_EXPERTS 64
#define MOE_EP_NOALLOC_SCRATCH_BYTES 2048
int moe_ep_run_noalloc(const moe_ep_run_params* params, void* stream);

/* ---------------------------------------------------------------- return path
 * The layer with its combine step (no counterpart in the reference, whose
 * path ends at the expert outputs):
 *   y[t, :] = sum over k of top_vals[t, k] * (x_t @ weights_e)
 * for e = top_idxs[t, k] of this rank's tokens, counting each distinct valid
 * id of a row once (like the routing) and skipping ids outside [0, E).
 * One call launches the fused kernel of moe_ep_run in return mode — every
 * output row is stored (bf16) into its source rank's return region over
 * NVLink, at the row its padded send buffer holds the token in, and the
 * last CTA releases a per-source flag — and then a combine kernel that
 * waits (bounded by timeout_ns) for all W flags and forms y in fp32,
 * rounded to bf16 (tokens with no valid id get a zero row).
 * `run` is as for moe_ep_run except that run->out is not used; the
 * workspace must have a return region (moe_ep_workspace_layout_ret) of
 * ret_rows >= W*El*gm rows and out_dim columns.  Collective like moe_ep_run;
 * all ranks use this call or moe_ep_run for the same epoch. */
typedef struct moe_ep_combine_params {
  const void* top_idxs;  /* [T, K] this rank's expert ids (the moe_route_slots input) */
  const void* top_vals;  /* [T, K] router weights, fp32 (vals_are_bf16 = 0) or bf16   */
  const int32_t* slots;  /* [T, K] from moe_route_slots                               */
  void* y;               /* [T, out_dim] bf16                                         */
  int64_t T;             /* tokens of this rank                                       */
  int64_t ret_rows;      /* rows of the workspace's return region                     */
  int32_t K;             /* ids per token, <= 32                                      */
  int32_t ids_are_int64;
  int32_t vals_are_bf16;
  int32_t reserved;
} moe_ep_combine_params;

int moe_ep_run_combine(const moe_ep_run_params* run, const moe_ep_combine_params* combine, void* stream);

/* ---------------------------------------------------------------- expert MLP
 * The activation between the expert MLP's two GEMMs (the reference's expert
 * is a single GEMM, baseline.py:50): a [rows, 2F] bf16 holds [gate | up] per
 * row; h [rows, F] bf16 = silu(gate) * up, computed in fp32 with
 * silu(g) = g / (1 + exp(-g)).  Requires F % 8 == 0 and 16-byte aligned
 * buffers.  The GEMMs around it are moe_ep_run_compact calls (the exchange
 * with w13 [El, H, 2F], then one rank's local call with w2 [El, F, H]). */
int moe_swiglu(const void* a, int64_t rows, int32_t F, void* h, void* stream);

/* moe_ep_run_compact with the activation in the GEMM's epilogue: the first
 * GEMM of the expert MLP writing h = silu(gate) * up directly, so the
 * [gate | up] rows never reach memory.  `weights` is w13 in the fused layout
 * (mlp.fuse_gate_up): per 256 columns, 64 gate, the 64 matching up, 64
 * gate, 64 up (one CTA's 128 features each); out_dim = 2F with
 * 2F % 256 == 0; out is [out_rows, F], same row order as moe_ep_run_compact.
 * Each value equals moe_swiglu applied to moe_ep_run_compact's output. */
int moe_ep_run_compact_swiglu(const moe_ep_run_params* params, int64_t send_rows, int64_t out_rows, void* stream);

/* Copy the workspace status word to the host (synchronous). */
int moe_ep_read_status(uint64_t local_base, const moe_ep_layout* layout, uint32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* MOE_EP_H */
