// Fused expert-parallel layer for sm_100a: count exchange, NVLink dispatch
// with per-chunk arrival flags, and a persistent grouped GEMM on CTA pairs
// (tcgen05 cta_group::2, TMEM accumulators, TMA) whose tiles start as soon as
// the rows they read have landed.
//
// Reference behaviour (paths within jy1534/nvshmem_testing):
//   alltoall_persistent_gemm.py:207-309  run(): peer copies of each rank's
//       padded chunk, a per-source signal, and a Triton grouped GEMM that
//       spins on the signal, skips rows >= recv_counts[src, e], and stores
//       out[e, src*gm + m, :] in bf16 (fp32 accumulation).
//   baseline.py:18-50                    same output contract through NCCL
//       all_to_all_single + view/permute/flatten + bmm; padded rows are zero.
//
// B200 design.  The GEMM is computed transposed, D^T[features, rows] =
// W^T[features, K] . X^T[K, rows]: expert weights are the MMA A operand
// (N-contiguous in memory, so "MN-major"), token rows the B operand
// (K-major), and a tile's row count becomes the MMA N, which can be any
// multiple of 16 up to 256 — experts with ~130 rows waste at most 15 rows,
// not a whole 128-row M tile.  Two CTAs of a cluster form a pair: one
// tcgen05.mma.cta_group::2 (M = 256 features, N = rows, K = 16) reads each
// CTA's 128 features of A and half of the rows of B from that CTA's shared
// memory and accumulates into each CTA's TMEM, so each CTA stages 64 KB per
// 128-deep k-stage (3 stages).  Loads use few, large TMA boxes (one 32 KB box
// for a CTA's weights per stage): the TMA engine overlaps a limited number of
// boxes, so box size sets the bytes in flight.
//
// Warp roles (both CTAs of a pair, 256 threads):
//   warp 0      TMA producer.  The leader CTA takes the next tile from a
//               global counter (dynamic scheduling), waits for the arrival
//               flags of its rows and publishes it to every role of both
//               CTAs; both then stream their halves; pair loads complete on
//               the leader's full barrier.
//   warp 1      MMA issuer (leader only): one thread issues the pair MMAs and
//               commits to both CTAs' barriers.
//   warps 2-5   epilogue: tcgen05.ld of this CTA's 128 features, bf16,
//               transposed through shared memory, 16-byte stores of the valid
//               rows to out[le, src*gm + m, :].
//   warps 6-7   dispatch: copy this rank's valid rows for every peer straight
//               into the peer's receive buffer over NVLink (16-byte vectors),
//               then release a per-(src, expert, chunk) flag with the call's
//               epoch; afterwards zero the padded output rows.
// Rows this rank sends to itself are never copied: local tiles read them in
// place from the padded send buffer.  Remote rows land in a compact,
// expert-major receive buffer (per expert, sources in the order rank+1,
// rank+2, ...), so a tile can span several sources.  Receive buffers, counts
// and flags are double-buffered by epoch parity; a peer reuses parity p only
// after this rank has published that it finished the call that last used it
// ("free" epochs), so no per-call barrier or flag reset exists.  Every wait is
// bounded by timeout_ns; on expiry the kernel latches MOE_EP_TIMEOUT, drains
// its in-flight copies and MMAs, frees TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "moe_ep.h"
#include "moe_ep_internal.h"
#include "ptx.cuh"

namespace moe {

constexpr int BK = 64;                          // K of one 128-byte swizzle atom (bf16)
constexpr int KB = 128;                         // K per pipeline stage (two atoms)
constexpr int kStages = 3;
constexpr int kFeatPair = 256;                  // output features per pair tile (MMA M)
constexpr int kFeatCta = 128;                   // features per CTA (TMEM lanes)
constexpr int kMaxTileRows = 256;               // rows per tile (MMA N)
constexpr int kEpiWarps = 4;
constexpr int kMaxPushWarps = 6;                // push warps present in every CTA (Params::push_warps of them work)
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpEpi0 = 2, kWarpPush0 = 2 + kEpiWarps;
constexpr int kThreads = (2 + kEpiWarps + kMaxPushWarps) * 32;
constexpr int kZeroWarps = 2;                   // computing CTAs' warps that zero padded rows when push CTAs exist
// Push CTAs in bulk mode: kBulkStreams warps, each with a ring of
// kBulkSlots pieces of kBulkPiece bytes in the CTA's stage memory; loads run
// kBulkLead pieces ahead of the stores.
constexpr int kBulkStreams = 3;
constexpr int kBulkSlots = 8;
constexpr uint32_t kBulkPiece = 8192;
constexpr int kBulkLead = 6;
constexpr uint32_t kABox = 64 * KB * 2;                       // 16 KB: 64 features x 128 K
constexpr uint32_t kABytes = kFeatCta * KB * 2;               // 32 KB
constexpr uint32_t kBHalf = (kMaxTileRows / 2) * BK * 2;      // 16 KB: 128 rows x 64 K
constexpr uint32_t kBBytesMax = 2 * kBHalf;                   // 32 KB: 128 rows x 128 K
constexpr uint32_t kStageBytes = kABytes + kBBytesMax;        // 64 KB
constexpr int kMaxCells = 512;                  // W * El
constexpr int kMaxLocalExperts = 256;
constexpr uint32_t kAccCols = kMaxTileRows;
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr int kMergeMaxRows = 128;             // merged tiles only for experts this small (local padded + remote)
constexpr int kGoSlots = 8;                     // > kStages: the leader runs at most kStages k-blocks ahead
constexpr int kRowMaps = 5;                     // B boxes of 8, 16, 32, 64, 128 rows
constexpr int kNamedBarPush = 1;
constexpr int kNamedBarEpi = 2;                 // the epilogue warps (SwiGLU mode)
constexpr int kNamedBarZero = 3;                // zero warps working beside the push warps
// A pair whose first tile waits for remote rows prefetches the tile's first
// weight k-blocks into L2 meanwhile: at most this many bytes over the grid.
constexpr int64_t kPrefetchBudget = 64ll << 20;
constexpr uint32_t kEpiStageBytes = kEpiWarps * 32 * 32 * 2;  // 32 rows x 32 features bf16 per warp

struct Params {
  int W, me, El, H, N;
  int64_t gm;
  const __nv_bfloat16* tokens;
  const __nv_bfloat16* weights;
  const int32_t* recv_counts;
  __nv_bfloat16* out;
  const uint64_t* peers;
  unsigned char* local;
  int64_t cap_rows;
  int push_rows, max_chunks;
  int w4;  // weights also described by the 4-D map (N % 128 == 0)
  uint32_t epoch;
  uint64_t timeout_ns;
  uint64_t off_cmat, off_cflag, off_dflag, off_free, off_local, off_data;
  // Return mode (combine): instead of out, each output row goes to its
  // source rank's return region, row (me*El + le)*gm + i, and the last CTA
  // releases off_rflag[me] at every rank.
  int ret;
  uint64_t off_ret, off_rflag;
  // Compact mode (general all-to-all): tokens is [send_rows, H] with the
  // cells (d, le) back to back, unpadded; out is [out_rows, N] with the
  // cells (le, src) back to back.  Nothing is padded or zero-filled.
  int general;
  int64_t send_rows, out_rows;
  int tile_cap;  // most rows per tile (multiple of 16, <= kMaxTileRows)
  // SwiGLU mode (compact only): the weights hold, per 128 features of a CTA,
  // 64 gate columns then the 64 matching up columns; the epilogue writes
  // h = silu(gate) * up, N/2 columns per row.
  int glu;
  int out_cols;  // columns of an output row: N, or N/2 in SwiGLU mode
  int kstagger;  // tile t walks K from k-block t % kblocks (many tiles sharing one weight slice)
  // Dispatch placement: the last push_ctas CTAs of the grid (whole clusters)
  // only move rows to peers and zero padded rows, with all their warps; the
  // others only compute.  0: two push warps in every CTA.
  int push_ctas;
  int push_warps;  // push warps per computing CTA when push_ctas == 0 (1..kMaxPushWarps)
  int push_bulk;   // push CTAs copy through the TMA engine (bulk copies) instead of loads and stores
  // Push order: 0 = expert-major (every sender finishes expert le for all
  // destinations before le+1); 1 = destination-major (q = 1..W-1, destination
  // me - q, experts in order within each).
  int push_phased;
  // With push CTAs, the computing CTAs' push_warps warps push as well
  // (both take items from the same counter).
  int push_hybrid;
  // Send-buffer loads of the push and the output's stores marked evict-first
  // in L2 (each byte is touched once), keeping L2 for weights and rows.
  int l2_stream;
  // Tile order: the local tiles of experts [0, local_first) come before any
  // remote tile, so the GEMM starts on rows that need no NVLink transfer.
  int local_first;
  // Ready-first scheduling (local_first = El): a leader takes the next
  // remote tile if every row chunk it reads has landed, otherwise a local
  // tile from a second counter, so local work fills the waits for NVLink.
  int ready_first;
  // Merged tiles: an expert's local rows and its remote rows form one row
  // space (local rows, padded to 8, then remote rows), cut into tiles
  // together, so that each weight slice is read by as few tiles as the rows
  // need (one, where local + remote rows fit 256) instead of separate local
  // and remote tiles.  local_first and ready_first are then off.
  int merged;
  // Remote row groups per expert (0: chosen per expert, see decode_tile).
  int row_groups;
  // recv_counts holds this rank's send counts [W dst][El] instead of its
  // receive counts [W src][El]; every rank publishes its block either way,
  // so the exchanged matrix is read transposed and no host-side count
  // all-to-all is needed.
  int send_counts;
  int32_t* status_host;
  uint64_t* trace;  // MOE_EP_TRACE_WORDS per CTA, or null
};

// Timeline hooks (no effect when the caller passed no trace buffer).
#define TRACE_SET(p, i, v)                                                     \
  do {                                                                         \
    if ((p).trace) (p).trace[size_t(blockIdx.x) * MOE_EP_TRACE_WORDS + (i)] = (v); \
  } while (0)
#define TRACE_NOW(p) ((p).trace ? globaltimer_ns() : 0ull)

struct RowMaps {
  CUtensorMap m[kRowMaps];  // box {64, 8 << i}
};

// Sched and Smem sit back to back in shared memory; both are 16-byte
// aligned (Smem holds the 8-byte mbarriers) whatever their arrays add up to.
struct alignas(16) Sched {
  int nfeat, kblocks;
  int row_groups, npairs;  // Params::row_groups; computing CTA pairs
  int tiles_total, push_total, zero_total, pad_;
  int cnt[kMaxCells];                     // [src][le] rows this rank receives
  int seg[kMaxCells + kMaxLocalExperts];  // [le][q], q = 0..W: compact start of position q (seg[.][1] = 0)
  int rbase[kMaxLocalExperts + 1];        // compact base row of expert le in this rank's receive buffer
  int loc_tr[kMaxLocalExperts];           // rows per local tile of expert le (multiple of 16)
  int rem_tr[kMaxLocalExperts];           // rows per remote tile of expert le
  int push_off[kMaxCells];                // [d][le] first destination row at rank d
  int push_cnt[kMaxCells];                // [d][le] rows this rank sends to (d, le)
  int push_pfx[kMaxCells + 1];            // prefix of push items over cells le*(W-1) + (q-1)
  int tile_pfx[kMaxLocalExperts + 1];     // prefix of tiles over experts (after the local-first tiles)
  int lf_pfx[kMaxLocalExperts + 1];       // prefix of the local-first tiles over experts [0, local_first)
  int loc_nt[kMaxLocalExperts];           // local row tiles of expert le
  int rem_nt[kMaxLocalExperts];           // remote row tiles of expert le
  int tmp[kMaxCells];                     // scratch while building
  int soff[kMaxCells + 1];                // compact mode: [d][le] first row of my cell in tokens
  int ooff[kMaxCells + 1];                // compact mode: [le][src] first output row of the cell
};

struct alignas(16) Smem {
  uint64_t full[kStages];   // leader: both CTAs' bytes for the stage landed
  uint64_t empty[kStages];  // each CTA: the pair MMA finished reading the stage
  uint64_t tfull[2];        // each CTA: accumulator ready
  uint64_t tempty[2];       // leader: both CTAs' epilogues drained the accumulator
  uint64_t go[kGoSlots];    // peer: the leader's verdict for a tile
  uint64_t drain;
  uint64_t bulk[kBulkStreams][kBulkSlots];  // push CTAs, bulk mode: a ring slot's load landed
  int go_tile[kGoSlots];    // the tile the leader handed out for this slot, or -1 (stop)
  uint32_t tmem_base;
  int abort_flag;
  int push_item;
  int zero_item;
  unsigned long long push_items, push_bytes, push_end;  // this CTA's dispatch (timeline)
  uint32_t fills[kStages];
  uint32_t cons[kStages];
};

__device__ __forceinline__ uint32_t* at_u32(unsigned char* base, uint64_t off) {
  return reinterpret_cast<uint32_t*>(base + off);
}

__device__ __forceinline__ bool aborted(Smem& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0;
}

// Latch the first error (device word + mapped host word) and stop both CTAs
// of the pair.
__device__ void raise_error(const Params& p, Smem& sm, int code, int site, int detail) {
  LocalWords* lw = reinterpret_cast<LocalWords*>(p.local + p.off_local);
  const uint32_t w = status_word(code, site, detail);
  // Only the first error is kept; its writer alone also posts it to the
  // mapped host word (a plain store: no atomics on host memory).
  if (atomicCAS(&lw->status, 0u, w) == 0u && p.status_host != nullptr) {
    *reinterpret_cast<volatile int32_t*>(p.status_host) = int32_t(w);
    __threadfence_system();
  }
  atomicExch(&sm.abort_flag, 1);
  st_shared_cluster_u32(mapa_shared(smem_u32(&sm.abort_flag), cluster_ctarank() ^ 1u), 1u);
}

// Wait until a flag written by a peer reaches `epoch` (wrap-safe compare).
__device__ bool wait_epoch(const uint32_t* flag, uint32_t epoch, uint64_t timeout_ns, Smem& sm) {
  uint64_t deadline = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (int32_t(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((spin & 31) == 31) {
      if (aborted(sm)) return false;
      const uint64_t now = globaltimer_ns();
      if (deadline == 0) deadline = now + timeout_ns;
      else if (now > deadline) return false;
    }
  }
}

// Bounded mbarrier wait; pipeline waits only end early on abort or after a
// hard bound well above the peer timeout (a bug guard).
__device__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t bound_ns, Smem& sm, bool cluster_scope = false) {
  uint64_t deadline = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (cluster_scope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((spin & 63) == 63) {
      if (aborted(sm)) return false;
      const uint64_t now = globaltimer_ns();
      if (deadline == 0) deadline = now + bound_ns;
      else if (now > deadline) return false;
    }
  }
}

// The leader's producer hands tiles out dynamically: it takes the next tile
// of the call from a global counter and publishes it, in slot ti % kGoSlots,
// to both CTAs of the pair; every role of both CTAs reads the same sequence.
// The leader runs at most kStages k-blocks ahead of its MMA, which runs at
// most two tiles ahead of the epilogues, so kGoSlots slots are never
// overwritten before all readers are past them.
__device__ int wait_tile(Smem& sm, uint32_t ti, uint64_t bound_ns);

__device__ __forceinline__ int find_cell(const int* pfx, int ncells, int t) {
  // largest c with pfx[c] <= t (pfx[0] = 0, pfx[ncells] = total > t)
  int lo = 0, hi = ncells - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pfx[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Push items are counted per cell (expert le, position q = 1..W-1 where the
// destination is me - q), then per chunk; the cell order is expert-major or
// destination-major (Params::push_phased).
__device__ __forceinline__ int push_cell(const Params& p, int le, int qi) {
  return p.push_phased ? qi * p.El + le : le * (p.W - 1) + qi;
}
__device__ __forceinline__ void push_cell_decode(const Params& p, int c, int& le, int& q) {
  if (p.push_phased) {
    le = c % p.El;
    q = c / p.El + 1;
  } else {
    le = c / (p.W - 1);
    q = c % (p.W - 1) + 1;
  }
}

__device__ int wait_tile(Smem& sm, uint32_t ti, uint64_t bound_ns) {
  const int slot = int(ti % kGoSlots);
  if (!mbar_wait(&sm.go[slot], (ti / kGoSlots) & 1, bound_ns, sm, true)) return -1;
  return *reinterpret_cast<volatile int*>(&sm.go_tile[slot]);
}

struct Tile {
  int le, feat, remote;
  int row0, row1;  // rows [row0, row1) of the expert's local slot or compact remote rows
  int n;           // MMA N: row1 - row0 rounded up to 16
  // Merged tiles: rows [row0, row1) of the expert's merged row space; rows
  // below lr are local, [lr, lr8) padding (computed, never stored), rows
  // from lr8 on are remote row (row - lr8).  remote: the tile holds remote rows.
  int merged, lr, lr8;
};

// The remote rows [lo, hi) a tile reads (empty when hi <= lo).
__device__ __forceinline__ void tile_remote_rows(const Tile& tl, int& lo, int& hi) {
  if (tl.merged) {
    lo = max(tl.row0, tl.lr8) - tl.lr8;
    hi = tl.row1 - tl.lr8;
  } else if (tl.remote) {
    lo = tl.row0;
    hi = tl.row1;
  } else {
    lo = hi = 0;
  }
}

// Tiles are expert-major: expert le's cell holds nfeat feature slices, each
// followed by all of its row tiles (local first, then remote), so the tiles
// that share a weight slice run back to back on neighbouring clusters and
// read it once from HBM.  With local_first = X > 0 the local tiles of
// experts [0, X) come first of all (same order among themselves), and those
// experts' cells then hold only their remote tiles.  A merged expert (merged
// mode, small experts with remote rows: no separate remote tiles) counts its
// merged tiles as its local tiles.
//
// Row groups: with G > 1 groups for an expert, its cell holds first its
// local tiles (feature-major) and then its remote row tiles cut into G
// contiguous groups, each group feature-major, so the tiles whose rows land
// first (sources arrive in segment order) do not wait behind tiles of rows
// still in flight.  G = row_groups if set, else W-1 for an expert whose
// remote tiles per group still cover every computing pair, else 1.
__device__ __forceinline__ int remote_groups(const Sched& s, int W, int rem_nt) {
  int g = s.row_groups;
  if (g == 0) g = (W > 1 && s.nfeat * rem_nt >= (W - 1) * s.npairs) ? W - 1 : 1;
  return max(1, min(g, rem_nt));
}

__device__ __forceinline__ Tile decode_tile(const Sched& s, int W, int El, int me, int lf, int t, bool merged) {
  const int lf_total = s.lf_pfx[lf];
  const bool in_lf = t < lf_total;
  int c, r, lnt, nrt;
  if (in_lf) {
    c = find_cell(s.lf_pfx, lf, t);
    r = t - s.lf_pfx[c];
    lnt = nrt = s.loc_nt[c];
  } else {
    t -= lf_total;
    c = find_cell(s.tile_pfx, El, t);
    r = t - s.tile_pfx[c];
    lnt = c < lf ? 0 : s.loc_nt[c];
    nrt = lnt + s.rem_nt[c];
  }
  Tile tl;
  tl.le = c;
  tl.feat = r / nrt;
  int i = r % nrt;
  const int run = s.seg[c * (W + 1) + W];
  if (merged && s.rem_nt[c] == 0 && run > 0) {
    // One row space: local rows, padding to an 8-row boundary, remote rows.
    tl.merged = 1;
    tl.lr = s.cnt[me * El + c];
    tl.lr8 = (tl.lr + 7) & ~7;
    tl.row0 = i * s.loc_tr[c];
    tl.row1 = min(tl.row0 + s.loc_tr[c], tl.lr8 + run);
    tl.remote = tl.row1 > tl.lr8;
    tl.n = (tl.row1 - tl.row0 + 15) & ~15;
    return tl;
  }
  tl.merged = 0;
  tl.lr = tl.lr8 = 0;
  const int rn = s.rem_nt[c];
  const int g = in_lf ? 1 : remote_groups(s, W, rn);
  if (g > 1) {
    // Local tiles feature-major, then the remote row groups (see above).
    const int nf = s.nfeat;
    if (r < nf * lnt) {
      tl.feat = r / lnt;
      i = r % lnt;
      tl.remote = 0;
    } else {
      int r2 = r - nf * lnt, start = 0, gi = 0;
      const int base = rn / g, extra = rn % g;
      int gs = base + (extra > 0);
      while (r2 >= nf * gs) {
        r2 -= nf * gs;
        start += gs;
        ++gi;
        gs = base + (gi < extra);
      }
      tl.feat = r2 / gs;
      i = start + r2 % gs;
      tl.remote = 1;
    }
  } else {
    tl.remote = i >= lnt;
    if (tl.remote) i -= lnt;
  }
  const int rows = tl.remote ? run : s.cnt[me * El + tl.le];
  const int tr = tl.remote ? s.rem_tr[tl.le] : s.loc_tr[tl.le];
  tl.row0 = i * tr;
  tl.row1 = min(tl.row0 + tr, rows);
  tl.n = (tl.row1 - tl.row0 + 15) & ~15;
  return tl;
}

// Ready-first: whether every row chunk a remote tile reads has landed (one
// acquire load per chunk, no waiting).
__device__ bool tile_rows_landed(const Params& p, const Sched& s, const Tile& tl) {
  const int W = p.W, El = p.El;
  const uint32_t par = p.epoch & 1u;
  const int* sg = s.seg + tl.le * (W + 1);
  int rlo, rhi;
  tile_remote_rows(tl, rlo, rhi);
  for (int q = 1; q < W && rlo < rhi; ++q) {
    const int lo = max(rlo, sg[q]), hi = min(rhi, sg[q + 1]);
    if (lo >= hi) continue;
    const int src = (p.me + q) % W;
    const uint32_t* fl =
        reinterpret_cast<const uint32_t*>(p.local + p.off_dflag) + ((size_t(par) * W + src) * El + tl.le) * p.max_chunks;
    for (int c = (lo - sg[q]) / p.push_rows; c <= (hi - 1 - sg[q]) / p.push_rows; ++c)
      if (int32_t(ld_acquire_sys(fl + c) - p.epoch) < 0) return false;
  }
  return true;
}

// Rows per tile for `rows` rows: the fewest tiles of at most `cap` rows
// (a multiple of 16, at most 256), balanced, rounded up to a multiple of 16.
__device__ __forceinline__ int tile_rows(int rows, int cap) {
  if (rows <= 0) return 16;
  const int nt = (rows + cap - 1) / cap;
  return ((rows + nt - 1) / nt + 15) & ~15;
}

// In-place exclusive scan of a[0..n) by one warp; a[n] receives the total.
__device__ void warp_exclusive_scan(int* a, int n, int lane) {
  int carry = 0;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const int v = i < n ? a[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (i < n) a[i] = carry + x - v;
    carry += __shfl_sync(0xffffffffu, x, 31);
  }
  if (lane == 0) a[n] = carry;
  __syncwarp();
}

// Build the schedule for this call from the full count matrix.  All ranks
// hold identical matrices, so every validation failure is seen by all ranks.
// Every step is parallel over (rank, expert) cells; prefix sums are warp
// scans over shared memory.  The matrix is first copied in one coalesced
// pass into `scratch` (the stage memory, unused until the schedule exists),
// so the per-cell loops below read shared memory, not dependent L2 loads.
__device__ void build_schedule(const Params& p, Sched& s, Smem& sm, int32_t* scratch) {
  const int W = p.W, El = p.El, me = p.me, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t par = p.epoch & 1u;
  // One rank reads its own recv_counts (nothing was exchanged).
  const int32_t* cm_g = W == 1 ? p.recv_counts
                               : reinterpret_cast<const int32_t*>(p.local + p.off_cmat) + size_t(par) * W * W * El;
  const int ncm = W * W * El;
  for (int i = tid; i < ncm; i += kThreads) scratch[i] = cm_g[i];
  __syncthreads();
  const int32_t* cm = scratch;
  // C(owner, src, le): rows src sends to owner's local expert le.  The
  // matrix holds every rank's published block: receive counts (block =
  // owner) or send counts (block = src).
  const bool by_src = p.send_counts != 0;
  auto C = [&](int owner, int src, int le) {
    return by_src ? cm[(size_t(src) * W + owner) * El + le] : cm[(size_t(owner) * W + src) * El + le];
  };
  const int nfeat = (p.N + kFeatPair - 1) / kFeatPair;

  if (tid == 0) {
    s.nfeat = nfeat;
    s.kblocks = (p.H + KB - 1) / KB;
    s.row_groups = p.row_groups;
    s.npairs = max(1, (int(gridDim.x) - p.push_ctas) / 2);
    s.zero_total = (p.ret || p.general) ? 0 : W * El;  // no padded output in return or compact mode
  }
  // Validation: 0 <= count <= gm everywhere, chunk slots suffice.
  for (int i = tid; i < W * W * El; i += kThreads) {
    const int v = cm[i];
    if (v < 0 || int64_t(v) > p.gm || (v + p.push_rows - 1) / p.push_rows > p.max_chunks)
      raise_error(p, sm, kBadArg, kSiteTable, i);
  }
  // Per (d, le): rows this rank receives from d (cnt), rows it sends to d
  // (push_cnt), d's total remote rows for le (push_off, scanned below) and
  // the rows that precede this rank's segment at d (tmp).
  for (int i = tid; i < W * El; i += kThreads) {
    const int d = i / El, le = i % El;
    s.cnt[i] = C(me, d, le);
    const int q_me = (me - d + W) % W;  // my position at d (0 means d == me)
    int before = 0, total = 0;
    for (int q = 1; q < W; ++q) {
      const int v = C(d, (d + q) % W, le);
      if (q < q_me) before += v;
      total += v;
    }
    const int sc = (d == me) ? 0 : C(d, me, le);
    s.push_cnt[i] = sc;
    s.push_off[i] = total;
    s.tmp[i] = before;
    if (p.general) {
      s.soff[i] = C(d, me, le);          // scanned below (cells d-major)
      s.ooff[le * W + d] = s.cnt[i];     // scanned below (cells le-major)
    }
    if (d != me) s.push_pfx[push_cell(p, le, q_me - 1)] = (sc + p.push_rows - 1) / p.push_rows;
  }
  __syncthreads();

  // Per local expert: compact segment starts (positions 1..W-1), tile sizes.
  for (int le = tid; le < El; le += kThreads) {
    int* sg = s.seg + le * (W + 1);
    sg[0] = 0;
    int run = 0;
    for (int q = 1; q < W; ++q) {
      sg[q] = run;
      run += s.cnt[((me + q) % W) * El + le];
    }
    sg[W] = run;
    const int lr = s.cnt[me * El + le];
    // Merged mode merges small experts only: their tiles are weight-bound, so
    // one tile instead of a local and a remote one halves their weight
    // reads; larger experts keep separate tiles (whole boxes, and local rows
    // that need no NVLink wait).
    if (p.merged && run > 0 && ((lr + 7) & ~7) + run <= kMergeMaxRows) {
      const int v = ((lr + 7) & ~7) + run;
      s.loc_tr[le] = tile_rows(v, p.tile_cap);
      s.loc_nt[le] = (v + s.loc_tr[le] - 1) / s.loc_tr[le];
      s.rem_tr[le] = 16;
      s.rem_nt[le] = 0;
    } else {
      s.loc_tr[le] = tile_rows(lr, p.tile_cap);
      s.rem_tr[le] = tile_rows(run, p.tile_cap);
      s.loc_nt[le] = (lr + s.loc_tr[le] - 1) / s.loc_tr[le];
      s.rem_nt[le] = (run + s.rem_tr[le] - 1) / s.rem_tr[le];
    }
    s.rbase[le] = run;                                   // scanned below
    const bool lf = le < p.local_first;
    s.tile_pfx[le] = ((lf ? 0 : s.loc_nt[le]) + s.rem_nt[le]) * nfeat;  // scanned below
    s.lf_pfx[le] = lf ? s.loc_nt[le] * nfeat : 0;                     // scanned below
  }
  __syncthreads();

  // Prefix sums, one warp each:
  //  * rbase: compact base of each expert in this rank's receive buffer;
  //  * tile_pfx: tiles, expert-major (see decode_tile);
  //  * push_pfx: push items per cell (push_cell), then row chunks.  In the
  //    expert-major order every sender finishes an expert's rows for all
  //    destinations before the next expert, matching the expert-major order
  //    of the receivers' tiles;
  //  * push_off (per destination d, warps 3..): where my rows for (d, le)
  //    land at d = d's compact base of le + the rows that precede mine.
  if (warp == 0) {
    warp_exclusive_scan(s.rbase, El, lane);
    if (p.general) {
      warp_exclusive_scan(s.soff, W * El, lane);
      if (lane == 0 && int64_t(s.soff[W * El]) > p.send_rows) raise_error(p, sm, kBadArg, kSiteTable, 0xFFFE);
    }
  }
  if (warp == 1) {
    warp_exclusive_scan(s.tile_pfx, El, lane);
    warp_exclusive_scan(s.lf_pfx, p.local_first, lane);
    if (lane == 0) s.tiles_total = s.tile_pfx[El] + s.lf_pfx[p.local_first];
    if (p.general) {
      warp_exclusive_scan(s.ooff, W * El, lane);
      if (lane == 0 && int64_t(s.ooff[W * El]) > p.out_rows) raise_error(p, sm, kBadArg, kSiteTable, 0xFFFF);
    }
  }
  if (warp == 2) {
    warp_exclusive_scan(s.push_pfx, El * (W - 1), lane);
    if (lane == 0) s.push_total = s.push_pfx[El * (W - 1)];
  }
  for (int d = warp - 3; d >= 0 && d < W; d += kThreads / 32 - 3) {
    int* row = s.push_off + d * El;
    const int last = row[El - 1];
    warp_exclusive_scan(row, El - 1, lane);  // row[El-1] receives the sum of the first El-1 totals
    const int total = row[El - 1] + last;
    __syncwarp();
    for (int le = lane; le < El; le += 32) {
      if (le == El - 1) row[le] = total - last;  // exclusive prefix of the last expert
    }
    __syncwarp();
    for (int le = lane; le < El; le += 32) row[le] += s.tmp[d * El + le];
    if (lane == 0 && int64_t(total) > p.cap_rows) raise_error(p, sm, kCapacity, kSiteTable, d);
  }
  __syncthreads();
}

__device__ __forceinline__ int64_t out_row_of(const Sched& s, const Params& p, const Tile& tl, int row) {
  const int W = p.W;
  int src = p.me, i = row;
  if (tl.remote) {
    const int* sg = s.seg + tl.le * (W + 1);
    int q = 1;
    while (q < W - 1 && row >= sg[q + 1]) ++q;
    src = (p.me + q) % W;
    i = row - sg[q];
  }
  if (p.general) return int64_t(s.ooff[tl.le * W + src]) + i;
  return (int64_t(tl.le) * W + src) * p.gm + i;
}

// Return mode: where output row `row` of tile tl goes — the source rank's
// return region, at the row the source's padded send buffer holds it in.
__device__ __forceinline__ unsigned char* ret_row_ptr(const Sched& s, const Params& p, const Tile& tl, int row) {
  int src = p.me, i = row;
  if (tl.remote) {
    const int* sg = s.seg + tl.le * (p.W + 1);
    int q = 1;
    while (q < p.W - 1 && row >= sg[q + 1]) ++q;
    src = (p.me + q) % p.W;
    i = row - sg[q];
  }
  return reinterpret_cast<unsigned char*>(p.peers[src]) + p.off_ret +
         ((int64_t(p.me) * p.El + tl.le) * p.gm + i) * int64_t(p.N) * 2;
}

// Zero one padded output cell's rows past its count (padded mode): z =
// le * W + src; np threads, pt = this thread.
__device__ void zero_fill(const Params& p, const Sched& s, int z, int pt, int np) {
  const int W = p.W, El = p.El;
  const int le = z / W, src = z % W;
  const int64_t c0 = s.cnt[src * El + le];
  const int64_t nvec = (p.gm - c0) * int64_t(p.N) / 8;
  uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t(le) * W * p.gm + int64_t(src) * p.gm + c0) * p.N);
  const uint4 zv = make_uint4(0, 0, 0, 0);
  for (int64_t v = pt; v < nvec; v += np) dst[v] = zv;
}

// One push item's rows: nvec 16-byte vectors from this GPU's send buffer to
// a peer's receive region, U loads in flight per thread before their stores.
// With `stream`, the loads of the send buffer (read once) are marked
// evict-first in L2, so they do not push the GEMM's weights and rows out.
template <int U>
__device__ __forceinline__ void copy_rows(const uint4* src, uint4* dst, int64_t nvec, int pt, int np, bool stream) {
  const uint64_t pol = l2_policy_evict_first();
  int64_t v = pt;
  for (; v + (U - 1) * np < nvec; v += U * np) {
    uint4 a[U];
    if (stream) {
#pragma unroll
      for (int u = 0; u < U; ++u) a[u] = ld_nc_v4_hint(src + v + u * np, pol);
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) a[u] = ld_nc_v4(src + v + u * np);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) st_v4(dst + v + u * np, a[u]);
  }
  for (; v < nvec; v += np) st_v4(dst + v, stream ? ld_nc_v4_hint(src + v, pol) : ld_nc_v4(src + v));
}

// Zero-fill items (padded output cells) from the shared zero counter until
// none is left: np threads of one group (pt = this thread), `slot` the
// group's shared-memory word for the claimed item, `bar` its named barrier.
__device__ void zero_items(const Params& p, const Sched& s, Smem& sm, LocalWords* lw, uint32_t par, int* slot,
                           int bar, int np, int pt) {
  for (;;) {
    if (pt == 0) *slot = aborted(sm) ? 0x7fffffff : int(atomicAdd(&lw->zero_ctr[par], 1u));
    named_bar_sync(bar, np);
    const int z = *slot;
    named_bar_sync(bar, np);
    if (z >= s.zero_total) break;
    zero_fill(p, s, z, pt, np);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    fused_ep_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w4,
                    const __grid_constant__ RowMaps rows_local,
                    const __grid_constant__ RowMaps rows_remote, const Params p) {
  extern __shared__ unsigned char smem_dyn[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  unsigned char* stage_mem = base;  // kStages * kStageBytes, 1024-aligned
  unsigned char* epi_mem = base + kStages * kStageBytes;
  Sched& s = *reinterpret_cast<Sched*>(epi_mem + kEpiStageBytes);
  Smem& sm = *reinterpret_cast<Smem*>(epi_mem + kEpiStageBytes + sizeof(Sched));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int W = p.W, El = p.El, me = p.me;
  const uint32_t par = p.epoch & 1u;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  // Whole clusters at the end of the grid only push (see Params::push_ctas).
  const bool push_cta = p.push_ctas > 0 && int(blockIdx.x) >= int(gridDim.x) - p.push_ctas;
  const uint64_t pipe_bound = 2 * p.timeout_ns + 1000000000ull;
  LocalWords* lw = reinterpret_cast<LocalWords*>(p.local + p.off_local);
  if (tid == 0) TRACE_SET(p, MOE_EP_TRACE_START, TRACE_NOW(p));

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
      sm.fills[i] = 0;
      sm.cons[i] = 0;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], 2 * kEpiWarps);
    }
    for (int i = 0; i < kGoSlots; ++i) {
      mbar_init(&sm.go[i], 1);
      sm.go_tile[i] = -1;
    }
    mbar_init(&sm.drain, 1);
    for (int i = 0; i < kBulkStreams; ++i)
      for (int j = 0; j < kBulkSlots; ++j) mbar_init(&sm.bulk[i][j], 1);
    sm.abort_flag = 0;
    sm.push_items = sm.push_bytes = sm.push_end = 0ull;
    fence_mbar_init();
    prefetch_tensormap(&tm_w);
  }
  cluster_sync();  // the peer's barriers exist before any remote arrive
  if (warp == kWarpMma && !push_cta) {
    __syncwarp();
    tmem_alloc_pair(&sm.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = sm.tmem_base;

  // ---- count exchange: CTA 0 publishes this rank's recv_counts block to
  // every rank; every CTA then waits for all W blocks.  One rank has nothing
  // to exchange: the schedule reads recv_counts directly, and each CTA only
  // waits until the call that last used this epoch parity has finished.
  // Warp w of CTA 0 publishes to ranks w, w + 12, ...: the W system-scope
  // fences run side by side.
  if (W > 1 && blockIdx.x == 0) {
    for (int d = warp; d < W; d += kThreads / 32) {
      unsigned char* peer = reinterpret_cast<unsigned char*>(p.peers[d]);
      int go = 1;
      if (lane == 0) {
        const uint32_t* fr = at_u32(p.local, p.off_free) + d;
        if (p.epoch > 2 && !wait_epoch(fr, p.epoch - 2, p.timeout_ns, sm)) raise_error(p, sm, kTimeout, kSiteFree, d);
        go = !aborted(sm);
      }
      go = __shfl_sync(0xffffffffu, go, 0);
      if (!go) break;
      int32_t* dst = reinterpret_cast<int32_t*>(peer + p.off_cmat) + (size_t(par) * W + me) * W * El;
      for (int i = lane; i < W * El; i += 32) dst[i] = p.recv_counts[i];
      fence_acq_rel_sys();
      __syncwarp();
      if (lane == 0) st_release_sys(at_u32(peer, p.off_cflag) + par * W + me, p.epoch);
    }
  }
  if (tid == 0) {
    if (W == 1) {
      if (p.epoch > 2 && !wait_epoch(at_u32(p.local, p.off_free), p.epoch - 2, p.timeout_ns, sm))
        raise_error(p, sm, kTimeout, kSiteFree, 0);
    }
    for (int q = 0; q < W && W > 1; ++q) {
      if (!wait_epoch(at_u32(p.local, p.off_cflag) + par * W + q, p.epoch, p.timeout_ns, sm)) {
        raise_error(p, sm, kTimeout, kSiteCounts, q);
        break;
      }
    }
    TRACE_SET(p, MOE_EP_TRACE_COUNTS, TRACE_NOW(p));
  }
  __syncthreads();
  if (!aborted(sm)) build_schedule(p, s, sm, reinterpret_cast<int32_t*>(stage_mem));
  __syncthreads();
  // The stage memory held the count matrix (generic proxy); TMA writes it next.
  fence_proxy_async_smem();
  const bool run_main = !aborted(sm);
  if (tid == 0) TRACE_SET(p, MOE_EP_TRACE_SCHED, TRACE_NOW(p));

  // Rows are pushed by push_warps warps of every CTA, or by the push CTAs
  // (every warp, or kBulkStreams bulk-copy streams).
  const bool pusher = push_cta || ((p.push_ctas == 0 || p.push_hybrid) && warp >= kWarpPush0 &&
                                   warp < kWarpPush0 + p.push_warps);
  if (run_main && !push_cta && warp == kWarpProducer) {
    if (lane == 0) {
      const uint32_t bar_leader0 = mapa_shared(smem_u32(&sm.full[0]), 0);
      uint32_t it = 0, ti = 0;
      uint64_t flag_ns = 0, empty_ns = 0;
      // The leader claims one tile ahead, so the counter's round trip
      // overlaps the current tile's loads.
      // Ready-first: local tiles [0, nloc), remote tiles [nloc, tiles_total)
      // from separate counters; `claimed` is then the pending remote tile.
      const int nloc = s.lf_pfx[p.local_first];
      auto claim_remote = [&]() {
        const int r = int(atomicAdd(&lw->tile_ctr[par], 1u));
        return r < s.tiles_total - nloc ? nloc + r : s.tiles_total;
      };
      int claimed = !leader ? -1 : p.ready_first ? claim_remote() : int(atomicAdd(&lw->tile_ctr[par], 1u));
      for (;; ++ti) {
        const int slot = int(ti % kGoSlots);
        int t;
        Tile tl{};
        if (leader) {
          if (p.ready_first) {
            t = -1;
            if (!aborted(sm)) {
              if (claimed < s.tiles_total) {
                if (tile_rows_landed(p, s, decode_tile(s, W, El, me, p.local_first, claimed, p.merged))) {
                  t = claimed;
                  claimed = claim_remote();
                } else {
                  const int l = int(atomicAdd(&lw->local_ctr[par], 1u));
                  if (l < nloc) {
                    t = l;
                  } else {  // no local work left: wait for the pending tile's rows
                    t = claimed;
                    claimed = claim_remote();
                  }
                }
              } else {
                const int l = int(atomicAdd(&lw->local_ctr[par], 1u));
                t = l < nloc ? l : -1;
              }
            }
          } else {
            t = (aborted(sm) || claimed >= s.tiles_total) ? -1 : claimed;
            if (t >= 0) claimed = int(atomicAdd(&lw->tile_ctr[par], 1u));
          }
          bool ok = t >= 0;
          if (ok) tl = decode_tile(s, W, El, me, p.local_first, t, p.merged);
          if (ok && ti == 0 && p.w4 && tl.remote && !tile_rows_landed(p, s, tl)) {
            // The pair's first tile waits for rows in flight (decode shapes:
            // one tile per pair): stream the start of its weight slice into
            // L2 meanwhile, both CTAs' feature halves, within the budget.
            const int busy = max(1, min(s.npairs, s.tiles_total));
            const int64_t fit = kPrefetchBudget / (int64_t(busy) * 2 * kABytes);
            const int nk = fit < s.kblocks ? int(fit) : s.kblocks;
            const int fa = tl.feat * kFeatPair;
            const int rot0 = p.kstagger ? t % s.kblocks : 0;  // the k-block the tile starts at
            for (int kb = 0; kb < nk; ++kb) {
              const int kc = kb + rot0 < s.kblocks ? kb + rot0 : kb + rot0 - s.kblocks;
              if (fa < p.N) tma_prefetch_l2_4d(&tm_w4, 0, kc * KB, fa / 64, tl.le);
              if (fa + kFeatCta < p.N) tma_prefetch_l2_4d(&tm_w4, 0, kc * KB, (fa + kFeatCta) / 64, tl.le);
            }
          }
          const uint64_t tw0 = TRACE_NOW(p);
          if (ok && tl.remote) {
            const int* sg = s.seg + tl.le * (W + 1);
            int rlo, rhi;
            tile_remote_rows(tl, rlo, rhi);
            for (int q = 1; q < W && ok; ++q) {
              const int lo = max(rlo, sg[q]), hi = min(rhi, sg[q + 1]);
              if (lo >= hi) continue;
              const int src = (me + q) % W;
              const uint32_t* fl = at_u32(p.local, p.off_dflag) + ((size_t(par) * W + src) * El + tl.le) * p.max_chunks;
              for (int c = (lo - sg[q]) / p.push_rows; c <= (hi - 1 - sg[q]) / p.push_rows; ++c) {
                if (!wait_epoch(fl + c, p.epoch, p.timeout_ns, sm)) {
                  if (!aborted(sm)) raise_error(p, sm, kTimeout, kSiteTileFlag, src);
                  ok = false;
                  break;
                }
              }
            }
          }
          flag_ns += TRACE_NOW(p) - tw0;
          if (!ok) t = -1;
          for (uint32_t r = 0; r < 2; ++r) {
            st_shared_cluster_u32(mapa_shared(smem_u32(&sm.go_tile[slot]), r), uint32_t(t));
            mbar_arrive_cluster(mapa_shared(smem_u32(&sm.go[slot]), r));
          }
          if (t < 0) break;
        } else {
          t = wait_tile(sm, ti, pipe_bound);
          if (t < 0) break;
          tl = decode_tile(s, W, El, me, p.local_first, t, p.merged);
        }
        if (tl.remote) fence_proxy_async_global();
        const int half = tl.n >> 1;
        const int64_t local_cell = p.general ? int64_t(s.soff[me * El + tl.le]) : (int64_t(me) * El + tl.le) * p.gm;
        const int64_t row_base = tl.remote ? int64_t(par) * p.cap_rows + s.rbase[tl.le] + tl.row0 + crank * half
                                           : local_cell + tl.row0 + crank * half;
        const RowMaps& rm = tl.remote ? rows_remote : rows_local;
        // Feature boxes of 64 that exist (trailing features beyond N are not loaded).
        const int f_mine = tl.feat * kFeatPair + int(crank) * kFeatCta;
        const int f_peer = tl.feat * kFeatPair + int(crank ^ 1u) * kFeatCta;
        const int nb_mine = max(0, min(2, (p.N - f_mine + 63) / 64));
        const int nb_peer = max(0, min(2, (p.N - f_peer + 63) / 64));
        // Rows go in one box of the smallest height >= half (rows past the
        // tile land in unused shared memory).  A merged tile's half is one
        // or two segments (local rows from the send buffer, remote rows from
        // the receive region), each 8-row aligned and loaded as exact
        // power-of-two boxes so that neither overwrites the other.
        int bm = 0;
        while ((8 << bm) < half) ++bm;
        const uint32_t b_bytes = tl.merged ? 2 * uint32_t(half) * BK * 2 : 2 * uint32_t(8 << bm) * BK * 2;
        int nseg = 0;
        int64_t seg_row[2];
        int seg_off[2], seg_len[2], seg_rem[2];
        if (tl.merged) {
          const int h0 = tl.row0 + int(crank) * half, h1 = h0 + half;
          if (h0 < tl.lr8) {
            seg_row[nseg] = local_cell + h0;
            seg_off[nseg] = 0;
            seg_len[nseg] = min(h1, tl.lr8) - h0;
            seg_rem[nseg++] = 0;
          }
          if (h1 > tl.lr8) {
            const int v0 = max(h0, tl.lr8);
            seg_row[nseg] = int64_t(par) * p.cap_rows + s.rbase[tl.le] + (v0 - tl.lr8);
            seg_off[nseg] = v0 - h0;
            seg_len[nseg] = h1 - v0;
            seg_rem[nseg++] = 1;
          }
        }
        const uint32_t tx = uint32_t(nb_mine + nb_peer) * kABox + 2 * b_bytes;
        bool stop = false;
        // With k staggering, tile t starts its K loop at k-block t % kblocks
        // (the MMA's accumulate flag follows the iteration, not the block).
        const int rot = p.kstagger ? t % s.kblocks : 0;
        for (int kb = 0; kb < s.kblocks; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t round = it / kStages;
          const int kc = kb + rot < s.kblocks ? kb + rot : kb + rot - s.kblocks;
          const uint64_t te0 = TRACE_NOW(p);
          if (!mbar_wait(&sm.empty[st], (round & 1) ^ 1, pipe_bound, sm)) {
            if (!aborted(sm)) raise_error(p, sm, kTimeout, kSitePipe, 0);
            stop = true;
            break;
          }
          empty_ns += TRACE_NOW(p) - te0;
          unsigned char* a_dst = stage_mem + st * kStageBytes;
          unsigned char* b_dst = a_dst + kABytes;
          const uint32_t bar = bar_leader0 + uint32_t(st) * sizeof(uint64_t);
          if (leader) mbar_arrive_expect_tx(&sm.full[st], tx);
          // One 16 KB box for both 64-feature atoms when N is a multiple
          // of 128, one box for the rows: the TMA engine overlaps few boxes
          // at a time, so fewer, larger boxes keep more bytes in flight.
          if (p.w4) {
            if (nb_mine) tma_load_4d_pair(&tm_w4, bar, a_dst, 0, kc * KB, f_mine / 64, tl.le);
          } else {
            for (int j = 0; j < nb_mine; ++j)
              tma_load_3d_pair(&tm_w, bar, a_dst + j * kABox, f_mine + 64 * j, kc * KB, tl.le);
          }
          if (tl.merged) {
            for (int g = 0; g < nseg; ++g) {
              const RowMaps& sm_rows = seg_rem[g] ? rows_remote : rows_local;
              int off = seg_off[g], left = seg_len[g];
              for (int b = kRowMaps - 1; b >= 0; --b) {
                const int bh = 8 << b;
                if (left < bh) continue;
                const int r0 = int(seg_row[g] + (off - seg_off[g]));
                tma_load_2d_pair(&sm_rows.m[b], bar, b_dst + off * 128, kc * KB, r0);
                tma_load_2d_pair(&sm_rows.m[b], bar, b_dst + kBHalf + off * 128, kc * KB + BK, r0);
                off += bh;
                left -= bh;
              }
            }
          } else {
            tma_load_2d_pair(&rm.m[bm], bar, b_dst, kc * KB, int(row_base));
            tma_load_2d_pair(&rm.m[bm], bar, b_dst + kBHalf, kc * KB + BK, int(row_base));
          }
          sm.fills[st] += 1;
        }
        if (stop) break;
      }
      TRACE_SET(p, MOE_EP_TRACE_PRODUCER_END, TRACE_NOW(p));
      TRACE_SET(p, MOE_EP_TRACE_TILES, ti);
      TRACE_SET(p, MOE_EP_TRACE_FLAG_WAIT, flag_ns);
      TRACE_SET(p, MOE_EP_TRACE_EMPTY_WAIT, empty_ns);
    }
  } else if (run_main && !push_cta && warp == kWarpMma) {
    if (leader && lane == 0) {
      uint32_t it = 0, lt = 0;
      uint64_t full_ns = 0, acc_ns = 0, issue_ns = 0;
      for (;; ++lt) {
        const int t = wait_tile(sm, lt, pipe_bound);
        if (t < 0) break;
        const Tile tl = decode_tile(s, W, El, me, p.local_first, t, p.merged);
        const uint32_t acc = lt & 1, use = lt >> 1;
        const uint64_t ta0 = TRACE_NOW(p);
        if (!mbar_wait(&sm.tempty[acc], (use & 1) ^ 1, pipe_bound, sm, true)) break;
        acc_ns += TRACE_NOW(p) - ta0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        const uint32_t idesc = make_idesc_mn(/*bf16*/ 1, kFeatPair, uint32_t(tl.n), /*A MN-major*/ 1, /*B K-major*/ 0);
        bool stop = false;
        for (int kb = 0; kb < s.kblocks; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t round = it / kStages;
          const uint64_t tf0 = TRACE_NOW(p);
          if (!mbar_wait(&sm.full[st], round & 1, pipe_bound, sm)) {
            stop = true;
            break;
          }
          const uint64_t tf1 = TRACE_NOW(p);
          full_ns += tf1 - tf0;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_mem + st * kStageBytes);
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int k = 0; k < KB / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(a_addr + k * 2048, kABox, 1024);  // MN-major: 16 K = 2 x 8-row groups
            // K-major rows: 16 K = 32 bytes inside a 64-K atom; the second atom is kBHalf further.
            const uint64_t bd = smem_desc_sw128(b_addr + (k >> 2) * kBHalf + (k & 3) * 32, 16, 1024);
            tc_mma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit_pair_mc(&sm.empty[st], 0x3);
          sm.cons[st] += 1;
          issue_ns += TRACE_NOW(p) - tf1;
        }
        if (stop) break;
        tc_commit_pair_mc(&sm.tfull[acc], 0x3);
      }
      TRACE_SET(p, MOE_EP_TRACE_MMA_END, TRACE_NOW(p));
      TRACE_SET(p, MOE_EP_TRACE_FULL_WAIT, full_ns);
      TRACE_SET(p, MOE_EP_TRACE_ACC_WAIT, acc_ns);
      TRACE_SET(p, MOE_EP_TRACE_MMA_ISSUE, issue_ns);
      TRACE_SET(p, MOE_EP_TRACE_KBLOCKS, it);
    }
  } else if (run_main && !push_cta && warp >= kWarpEpi0 && warp < kWarpPush0) {
    const int quarter = warp & 3;
    __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(epi_mem) + (warp - kWarpEpi0) * 32 * 32;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&sm.tempty[0]), 0);
    uint32_t lt = 0;
    uint64_t epi_ns = 0;
    const uint64_t out_pol = l2_policy_evict_first();
    // SwiGLU mode: quarters 0 and 1 hold gate features, 2 and 3 the matching
    // up features; a gate warp reads its partner's staged values.  The four
    // warps meet at named barriers, so they decide together whether to go on
    // (bar.red.and) and never leave one of them waiting.
    const __nv_bfloat16* partner =
        reinterpret_cast<const __nv_bfloat16*>(epi_mem) + (quarter + 2 - (kWarpEpi0 & 3)) % 4 * 32 * 32;
    for (;; ++lt) {
      int t = wait_tile(sm, lt, pipe_bound);
      if (p.glu && !named_bar_and(kNamedBarEpi, kEpiWarps * 32, t >= 0)) t = -1;
      if (t < 0) break;
      const Tile tl = decode_tile(s, W, El, me, p.local_first, t, p.merged);
      const uint32_t acc = lt & 1, use = lt >> 1;
      const uint64_t tp0 = TRACE_NOW(p);
      bool full = mbar_wait(&sm.tfull[acc], use & 1, pipe_bound, sm);
      if (p.glu) full = named_bar_and(kNamedBarEpi, kEpiWarps * 32, full);
      if (!full) break;
      epi_ns += TRACE_NOW(p) - tp0;
      tc_fence_after();
      const int fbase = p.glu ? tl.feat * (kFeatPair / 2) + int(crank) * (kFeatCta / 2) + quarter * 32
                              : tl.feat * kFeatPair + int(crank) * kFeatCta + quarter * 32;
      const bool stores = !p.glu || quarter < 2;
      for (int jc = 0; jc * 32 < tl.n; ++jc) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tmem_base + acc * kAccCols + (uint32_t(quarter * 32) << 16) + jc * 32, r);
        tmem_ld_wait();
        if (p.glu) named_bar_sync(kNamedBarEpi, kEpiWarps * 32);  // partners done with the last chunk
        // stage[i][lane] = D[feature fbase + lane][row jc*32 + i]
#pragma unroll
        for (int i = 0; i < 32; ++i) stage[i * 32 + lane] = __float2bfloat16_rn(__uint_as_float(r[i]));
        __syncwarp();
        if (p.glu) {
          named_bar_sync(kNamedBarEpi, kEpiWarps * 32);  // every warp's chunk is staged
          if (quarter < 2) {
#pragma unroll 8
            for (int i = 0; i < 32; ++i) {
              const float g = __bfloat162float(stage[i * 32 + lane]);
              const float u = __bfloat162float(partner[i * 32 + lane]);
              stage[i * 32 + lane] = __float2bfloat16_rn((g / (1.f + expf(-g))) * u);
            }
            __syncwarp();
          }
        }
        if (stores) {
#pragma unroll
          for (int step = 0; step < 4; ++step) {
            const int c = lane + 32 * step;
            const int i = c >> 2, part = c & 3;
            const int row = tl.row0 + jc * 32 + i;
            const int f = fbase + part * 8;
            if (row < tl.row1 && f + 8 <= p.out_cols) {
              Tile ts = tl;  // the row's own part (merged tiles hold local and remote rows)
              int rr = row;
              bool keep = true;
              if (tl.merged) {
                ts.remote = row >= tl.lr8;
                rr = ts.remote ? row - tl.lr8 : row;
                keep = ts.remote || row < tl.lr;  // [lr, lr8) is padding
              }
              if (keep) {
                const uint4 v = *reinterpret_cast<const uint4*>(stage + i * 32 + part * 8);
                if (p.ret) st_v4(ret_row_ptr(s, p, ts, rr) + size_t(f) * 2, v);  // NVLink for remote rows
                else if (p.l2_stream) st_v4_hint(p.out + out_row_of(s, p, ts, rr) * p.out_cols + f, v, out_pol);
                else *reinterpret_cast<uint4*>(p.out + out_row_of(s, p, ts, rr) * p.out_cols + f) = v;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + acc * sizeof(uint64_t));
    }
    if (p.ret) fence_acq_rel_sys();  // this thread's return rows before the CTA's completion count
    if (warp == kWarpEpi0 && lane == 0) {
      TRACE_SET(p, MOE_EP_TRACE_EPI_END, TRACE_NOW(p));
      TRACE_SET(p, MOE_EP_TRACE_EPI_WAIT, epi_ns);
    }
  } else if (run_main && pusher && !(push_cta && p.push_bulk)) {
    // Loads and stores: push_warps warps of every computing CTA, or every
    // warp of a push CTA.  Without push CTAs the same warps then help the
    // zero warps zero the padded output rows (the zero counter); computing
    // CTAs that push beside push CTAs zero after their pushes (items after
    // the push items).
    const int np = push_cta ? kThreads : p.push_warps * 32;  // threads taking part in each item
    const int pt = push_cta ? tid : tid - kWarpPush0 * 32;
    const bool zero_counter = p.push_ctas == 0;
    const int last = (push_cta || zero_counter) ? s.push_total : s.push_total + s.zero_total;
    const size_t row_bytes = size_t(p.H) * 2;
    bool pushes_done = false;
    for (;;) {
      if (pt == 0) {
        int it = aborted(sm) ? 0x7fffffff : int(atomicAdd(&lw->push_ctr[par], 1u));
        if (it < s.push_total && p.epoch > 2) {
          int le, q;
          push_cell_decode(p, find_cell(s.push_pfx, (W - 1) * El, it), le, q);
          const int d = (me - q + W) % W;
          if (!wait_epoch(at_u32(p.local, p.off_free) + d, p.epoch - 2, p.timeout_ns, sm)) {
            raise_error(p, sm, kTimeout, kSiteFree, d);
            it = 0x7fffffff;
          }
        }
        sm.push_item = it;
      }
      named_bar_sync(kNamedBarPush, np);
      const int item = sm.push_item;
      named_bar_sync(kNamedBarPush, np);
      if (item < s.push_total) {
        const int c = find_cell(s.push_pfx, (W - 1) * El, item);
        int le, q;
        push_cell_decode(p, c, le, q);
        const int d = (me - q + W) % W;
        const int chunk = item - s.push_pfx[c];
        const int j0 = chunk * p.push_rows;
        const int j1 = min(j0 + p.push_rows, s.push_cnt[d * El + le]);
        unsigned char* peer = reinterpret_cast<unsigned char*>(p.peers[d]);
        const int64_t cell = p.general ? int64_t(s.soff[d * El + le]) : (int64_t(d) * El + le) * p.gm;
        const uint4* src = reinterpret_cast<const uint4*>(p.tokens + (cell + j0) * p.H);
        uint4* dst = reinterpret_cast<uint4*>(peer + p.off_data +
                                              (size_t(par) * p.cap_rows + s.push_off[d * El + le] + j0) * row_bytes);
        const int64_t nvec = int64_t(j1 - j0) * int64_t(row_bytes / 16);
        // More loads in flight per thread where a whole CTA pushes.
        if (push_cta) copy_rows<16>(src, dst, nvec, pt, np, p.l2_stream);
        else copy_rows<4>(src, dst, nvec, pt, np, p.l2_stream);
        fence_acq_rel_sys();
        named_bar_sync(kNamedBarPush, np);
        if (pt == 0) {
          uint32_t* fl = at_u32(peer, p.off_dflag) + ((size_t(par) * W + me) * El + le) * p.max_chunks + chunk;
          st_release_sys(fl, p.epoch);
          atomicAdd(&sm.push_items, 1ull);
          atomicAdd(&sm.push_bytes, static_cast<unsigned long long>(nvec) * 16ull);
        }
      } else if (item < last) {
        if (pt == 0 && !pushes_done) {
          pushes_done = true;
          atomicMax(&sm.push_end, static_cast<unsigned long long>(TRACE_NOW(p)));
        }
        zero_fill(p, s, item - s.push_total, pt, np);
      } else {
        break;
      }
    }
    if (pt == 0 && !pushes_done) atomicMax(&sm.push_end, static_cast<unsigned long long>(TRACE_NOW(p)));
    if (zero_counter) zero_items(p, s, sm, lw, par, &sm.push_item, kNamedBarPush, np, pt);
  } else if (run_main && p.push_ctas == 0 && p.push_warps + kZeroWarps <= kMaxPushWarps &&
             warp >= kWarpPush0 + p.push_warps && warp < kWarpPush0 + p.push_warps + kZeroWarps) {
    // Without push CTAs, kZeroWarps otherwise idle warps zero the padded
    // output rows from the start, beside the push warps.
    zero_items(p, s, sm, lw, par, &sm.zero_item, kNamedBarZero, kZeroWarps * 32,
               tid - (kWarpPush0 + p.push_warps) * 32);
  } else if (run_main && push_cta && p.push_bulk && warp < kBulkStreams) {
    // Bulk copies: lane 0 of each stream warp moves its items through the
    // TMA engine — local rows into a ring of shared-memory pieces, each
    // piece out to the peer's receive region — loads kBulkLead pieces ahead
    // of the stores.  An item's flag is released once every store of the
    // item has completed.
    unsigned char* ring = stage_mem + size_t(warp) * kBulkSlots * kBulkPiece;
    const size_t row_bytes = size_t(p.H) * 2;
    uint32_t gp = 0;  // pieces this stream has loaded (ring slot and phase)
    bool ok = true;
    if (lane == 0) {
      for (;;) {
        int it = (!ok || aborted(sm)) ? 0x7fffffff : int(atomicAdd(&lw->push_ctr[par], 1u));
        if (it >= s.push_total) break;
        const int c = find_cell(s.push_pfx, (W - 1) * El, it);
        int le, q;
        push_cell_decode(p, c, le, q);
        const int d = (me - q + W) % W;
        if (p.epoch > 2 && !wait_epoch(at_u32(p.local, p.off_free) + d, p.epoch - 2, p.timeout_ns, sm)) {
          raise_error(p, sm, kTimeout, kSiteFree, d);
          break;
        }
        const int chunk = it - s.push_pfx[c];
        const int j0 = chunk * p.push_rows;
        const int j1 = min(j0 + p.push_rows, s.push_cnt[d * El + le]);
        unsigned char* peer = reinterpret_cast<unsigned char*>(p.peers[d]);
        const int64_t cell = p.general ? int64_t(s.soff[d * El + le]) : (int64_t(d) * El + le) * p.gm;
        const unsigned char* src = reinterpret_cast<const unsigned char*>(p.tokens + (cell + j0) * p.H);
        unsigned char* dst = peer + p.off_data + (size_t(par) * p.cap_rows + s.push_off[d * El + le] + j0) * row_bytes;
        const uint32_t nbytes = uint32_t(j1 - j0) * uint32_t(row_bytes);
        const int npieces = int((nbytes + kBulkPiece - 1) / kBulkPiece);
        auto piece_len = [&](int k) { return min(kBulkPiece, nbytes - uint32_t(k) * kBulkPiece); };
        int stored = 0;
        for (int k = 0; k < npieces + kBulkLead && ok; ++k) {
          const int jst = k - kBulkLead;  // piece to store: its load was issued kBulkLead iterations ago
          if (jst >= 0 && jst < npieces) {
            const uint32_t g = gp + uint32_t(jst);
            if (!mbar_wait(&sm.bulk[warp][g % kBulkSlots], (g / kBulkSlots) & 1, pipe_bound, sm)) {
              if (!aborted(sm)) raise_error(p, sm, kTimeout, kSitePipe, 20);
              ok = false;
              break;
            }
            bulk_s2g(dst + size_t(jst) * kBulkPiece, ring + (g % kBulkSlots) * kBulkPiece, piece_len(jst));
            bulk_commit();
            stored = jst + 1;
          }
          if (k < npieces) {
            // The slot's previous store (kBulkSlots pieces back) has been
            // read out: at most kBulkSlots - kBulkLead newer stores pending.
            bulk_wait_read<kBulkSlots - kBulkLead>();
            const uint32_t g = gp + uint32_t(k);
            uint64_t* bar = &sm.bulk[warp][g % kBulkSlots];
            mbar_arrive_expect_tx(bar, piece_len(k));
            bulk_g2s(ring + (g % kBulkSlots) * kBulkPiece, src + size_t(k) * kBulkPiece, piece_len(k), bar);
          }
        }
        if (!ok) {
          // Wait (bounded) for the loads issued but not stored, then stop.
          const uint64_t until = globaltimer_ns() + 1000000000ull;
          for (int k = stored; k < npieces && k < stored + kBulkLead; ++k) {
            const uint32_t g = gp + uint32_t(k);
            while (!mbar_try_wait(&sm.bulk[warp][g % kBulkSlots], (g / kBulkSlots) & 1) && globaltimer_ns() < until) {
            }
          }
          bulk_wait<0>();
          break;
        }
        gp += uint32_t(npieces);
        bulk_wait<0>();  // every store of the item is complete
        fence_proxy_async_global();
        fence_acq_rel_sys();
        uint32_t* fl = at_u32(peer, p.off_dflag) + ((size_t(par) * W + me) * El + le) * p.max_chunks + chunk;
        st_release_sys(fl, p.epoch);
        atomicAdd(&sm.push_items, 1ull);
        atomicAdd(&sm.push_bytes, static_cast<unsigned long long>(nbytes));
      }
      atomicMax(&sm.push_end, static_cast<unsigned long long>(TRACE_NOW(p)));
    }
    __syncwarp();
  } else if (run_main && p.push_ctas > 0 && !p.push_hybrid && !push_cta && warp >= kWarpPush0 &&
             warp < kWarpPush0 + kZeroWarps) {
    // With push CTAs, the computing CTAs' first push warps zero the padded
    // output rows (their own counter).
    zero_items(p, s, sm, lw, par, &sm.zero_item, kNamedBarPush, kZeroWarps * 32, tid - kWarpPush0 * 32);
  }

  // ---- teardown: drain in-flight copies and MMAs, free TMEM, publish "free".
  __syncthreads();
  if (tid == 0) {
    TRACE_SET(p, MOE_EP_TRACE_PUSH_END, sm.push_end);
    TRACE_SET(p, MOE_EP_TRACE_ZERO_END, TRACE_NOW(p));
    TRACE_SET(p, MOE_EP_TRACE_PUSH_ITEMS, sm.push_items);
    TRACE_SET(p, MOE_EP_TRACE_PUSH_BYTES, sm.push_bytes);
  }
  if (aborted(sm) && !leader && tid == 0) {
    // Pair loads issued by this CTA complete on the leader's barrier; after an
    // abort give them time to land before the pair tears down (bug guard).
    const uint64_t until = globaltimer_ns() + 200000ull;
    while (globaltimer_ns() < until) {
    }
  }
  cluster_sync();
  if (leader && tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      if (sm.fills[i] != sm.cons[i]) {
        // A fill that the MMA warp never consumed (abort): wait for its bytes.
        const uint32_t parity = (sm.fills[i] - 1) & 1;
        const uint64_t deadline = globaltimer_ns() + 1000000000ull;
        while (!mbar_try_wait(&sm.full[i], parity)) {
          if (globaltimer_ns() > deadline) {
            raise_error(p, sm, kTimeout, kSiteDrain, i);
            break;
          }
        }
      }
    }
  }
  if (leader && !push_cta && warp == kWarpMma && lane == 0) {
    tc_commit_pair(&sm.drain);
    const uint64_t deadline = globaltimer_ns() + 1000000000ull;
    while (!mbar_try_wait(&sm.drain, 0)) {
      if (globaltimer_ns() > deadline) {
        raise_error(p, sm, kTimeout, kSiteDrain, 99);
        break;
      }
    }
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == kWarpMma && !push_cta) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (warp == 0) {
    uint32_t old = 0;
    if (lane == 0) {
      if (p.ret) __threadfence_system();
      else __threadfence();
      old = atomicAdd(&lw->done_ctr[par], 1u);
      if (old == gridDim.x - 1) {
        if (p.ret) __threadfence_system();
        else __threadfence();
        lw->push_ctr[par ^ 1] = 0;
        lw->zero_ctr[par ^ 1] = 0;
        lw->local_ctr[par ^ 1] = 0;
        lw->tile_ctr[par ^ 1] = 0;
        lw->done_ctr[par ^ 1] = 0;
        __threadfence();
      }
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    __syncwarp();
    if (old == gridDim.x - 1) {
      // The last CTA: lane q releases "free" (and, with return rows, "rows
      // returned") to rank q, so the W system-scope releases run side by
      // side instead of one NVLink round trip after another.  After an error
      // the return flags stay unset and the sources' combine waits time out.
      const bool returned = p.ret && ld_volatile_u32(&lw->status) == 0;
      for (int q = lane; q < W; q += 32) {
        unsigned char* peer = reinterpret_cast<unsigned char*>(p.peers[q]);
        st_release_sys(at_u32(peer, p.off_free) + me, p.epoch);
        if (returned) st_release_sys(at_u32(peer, p.off_rflag) + me, p.epoch);
      }
    }
  }
  if (tid == 0) TRACE_SET(p, MOE_EP_TRACE_END, TRACE_NOW(p));
  cluster_sync();  // neither CTA leaves while its peer may still address it
}

// ------------------------------------------------------------------ host side

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int workspace_layout(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks, int64_t ret_rows,
                     int64_t ret_cols, moe_ep_layout* L) {
  size_t off = 0;
  L->off_cmat = off;
  off = align_up(off + size_t(2) * W * W * El * 4, 256);
  L->off_cflag = off;
  off = align_up(off + size_t(2) * W * 4, 256);
  L->off_dflag = off;
  off = align_up(off + size_t(2) * W * El * max_chunks * 4, 256);
  L->off_free = off;
  L->off_rflag = off + align_up(size_t(W) * 4, 16);  // same 256-byte block for W <= 31
  off = align_up(L->off_rflag + size_t(W) * 4, 256);
  L->off_local = off;
  off = align_up(off + sizeof(LocalWords), 256);
  L->ctrl_bytes = off;
  off = align_up(off, 4096);
  L->off_data = off;
  off += size_t(2) * cap_rows * H * elem_bytes;
  off = align_up(off, 4096);
  L->off_ret = off;
  L->ret_bytes = size_t(ret_rows) * size_t(ret_cols) * 2;
  off += L->ret_bytes;
  L->total_bytes = align_up(off, 4096);
  return kOk;
}

static int encode_2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                     uint32_t box_inner, uint32_t box_rows) {
  const Driver& d = driver();
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = d.cuTensorMapEncodeTiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kCudaErr;
}

static int encode_3d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                     uint64_t s2_bytes, uint32_t b0, uint32_t b1) {
  const Driver& d = driver();
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = d.cuTensorMapEncodeTiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kCudaErr;
}

static int encode_4d_atoms(CUtensorMap* m, const void* ptr, uint64_t N, uint64_t H, uint64_t El) {
  const Driver& d = driver();
  cuuint64_t dims[4] = {64, H, N / 64, El};
  cuuint64_t strides[3] = {N * 2, 128, H * N * 2};
  cuuint32_t box[4] = {64, uint32_t(KB), 2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = d.cuTensorMapEncodeTiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides,
                                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kCudaErr;
}

static int encode_rows(RowMaps* rm, const void* ptr, uint64_t H, uint64_t rows) {
  for (int i = 0; i < kRowMaps; ++i)
    if (encode_2d(&rm->m[i], ptr, H, rows, H * 2, BK, 8u << i)) return kCudaErr;
  return kOk;
}

// Per-device launch facts, computed on the first launch on each device.
constexpr int kMaxDevices = 64;
struct DeviceLaunchInfo {
  bool ready;
  int grid;
};
static DeviceLaunchInfo g_launch_info[kMaxDevices];

// The count matrix (W <= 64 ranks, W * El <= kMaxCells) fits the stage
// memory that build_schedule copies it into.
static_assert(size_t(64) * kMaxCells * 4 <= size_t(kStages) * kStageBytes, "count matrix exceeds the stage memory");
static_assert(sizeof(Sched) % 16 == 0 && kEpiStageBytes % 16 == 0 && (kStages * kStageBytes) % 1024 == 0,
              "Sched and Smem must start on 16-byte boundaries");
// The whole shared-memory plan must fit the 227 KB a CTA may opt in to.
static_assert(1024 + size_t(kStages) * kStageBytes + kEpiStageBytes + sizeof(Sched) + sizeof(Smem) <= 227 * 1024,
              "shared memory plan exceeds 227 KB");

size_t fused_smem_bytes() {
  return 1024 + size_t(kStages) * kStageBytes + kEpiStageBytes + sizeof(Sched) + sizeof(Smem);
}

// m.ret_rows > 0 selects return mode: output rows go to the source ranks'
// return regions (ret_rows rows of out_dim bf16 each, at least W*El*gm) and
// `out` is not used.  m.general selects compact mode (send_rows rows of
// tokens, out_rows rows of out, no padding).
int launch_fused(const moe_ep_run_params* a, const FusedMode& m, cudaStream_t stream) {
  const int W = a->world_size, El = a->local_experts;
  const int64_t ret_rows = m.ret_rows;
  if (W < 1 || W > 64 || a->rank < 0 || a->rank >= W || El < 1 || El > kMaxLocalExperts || W * El > kMaxCells)
    return kBadArg;
  if (a->elem_bytes != 2 || a->hidden <= 0 || a->out_dim <= 0 || a->hidden % 8 || a->out_dim % 8 || a->gm < 0)
    return kBadArg;
  if (a->push_rows <= 0 || a->max_chunks <= 0 || a->cap_rows < 0 || a->epoch == 0) return kBadArg;
  const bool ret = ret_rows > 0;
  if (!a->tokens || !a->weights || (!ret && !a->out) || !a->peer_bases || !a->local_base || !a->recv_counts)
    return kBadArg;
  if (ret && ret_rows < int64_t(W) * El * a->gm) return kBadArg;
  if (m.general && (ret || m.send_rows < 0 || m.out_rows < 0)) return kBadArg;
  if (m.tile_cap < 0 || m.tile_cap > kMaxTileRows || m.tile_cap % 16) return kBadArg;
  if (m.glu && (!m.general || ret || a->out_dim % kFeatPair)) return kBadArg;
  if ((reinterpret_cast<uintptr_t>(a->tokens) | reinterpret_cast<uintptr_t>(a->weights) |
       reinterpret_cast<uintptr_t>(a->out)) & 15)
    return kBadArg;
  if (a->num_ctas & 1u) return kBadArg;  // CTA pairs
  if (a->push_ctas < 0 || (a->push_ctas & 1) || a->local_first < 0 || a->local_first > El) return kBadArg;
  if (a->push_warps < 0 || a->push_warps > kMaxPushWarps || (a->push_mode & ~15) || (a->sched_mode & ~(3 | MOE_EP_SCHED_ROW_GROUPS_MASK)))
    return kBadArg;
  // Rows of the token buffer (the local TMA map's extent).
  const int64_t rows_in = m.general ? m.send_rows : int64_t(W) * El * a->gm;
  if (rows_in + kMaxTileRows > (int64_t(1) << 31) || 2 * a->cap_rows + kMaxTileRows > (int64_t(1) << 31) ||
      m.out_rows + kMaxTileRows > (int64_t(1) << 31))
    return kBadArg;
  if (!driver().ok) return kCudaErr;

  moe_ep_layout L;
  workspace_layout(W, El, a->hidden, a->elem_bytes, a->cap_rows, a->max_chunks, ret ? ret_rows : 0, a->out_dim, &L);
  unsigned char* local = reinterpret_cast<unsigned char*>(a->local_base);

  CUtensorMap tw;
  RowMaps rl, rr;
  const uint64_t H = uint64_t(a->hidden), N = uint64_t(a->out_dim);
  if (encode_3d(&tw, a->weights, N, H, uint64_t(El), N * 2, H * N * 2, 64, KB)) return kCudaErr;
  // Weights as (64 features, K, 64-feature atom, expert): one box holds both
  // atoms of a CTA's 128 features.
  CUtensorMap tw4 = tw;
  const int w4 = (N % 128) == 0;
  if (w4 && encode_4d_atoms(&tw4, a->weights, N, H, uint64_t(El))) return kCudaErr;
  if (encode_rows(&rl, a->tokens, H, rows_in > 0 ? uint64_t(rows_in) : 1)) return kCudaErr;
  // With no remote capacity (one rank) no remote tile exists; the maps then
  // describe the token buffer so that they never name unbacked memory.
  if (a->cap_rows > 0) {
    if (encode_rows(&rr, local + L.off_data, H, uint64_t(2 * a->cap_rows))) return kCudaErr;
  } else {
    rr = rl;
  }

  Params p;
  p.W = W;
  p.me = a->rank;
  p.El = El;
  p.H = a->hidden;
  p.N = a->out_dim;
  p.gm = a->gm;
  p.tokens = static_cast<const __nv_bfloat16*>(a->tokens);
  p.weights = static_cast<const __nv_bfloat16*>(a->weights);
  p.recv_counts = a->recv_counts;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.peers = a->peer_bases;
  p.local = local;
  p.cap_rows = a->cap_rows;
  p.push_rows = a->push_rows;
  p.w4 = w4;
  p.max_chunks = a->max_chunks;
  p.epoch = a->epoch;
  p.timeout_ns = a->timeout_ns;
  p.off_cmat = L.off_cmat;
  p.off_cflag = L.off_cflag;
  p.off_dflag = L.off_dflag;
  p.off_free = L.off_free;
  p.off_local = L.off_local;
  p.off_data = L.off_data;
  p.ret = ret;
  p.off_ret = L.off_ret;
  p.off_rflag = L.off_rflag;
  p.general = m.general;
  p.tile_cap = m.tile_cap > 0 ? m.tile_cap : kMaxTileRows;
  p.kstagger = m.kstagger;
  p.glu = m.glu;
  p.out_cols = m.glu ? a->out_dim / 2 : a->out_dim;
  p.send_rows = m.send_rows;
  p.out_rows = m.out_rows;
  p.status_host = a->status_host;
  p.trace = a->trace;
  p.push_ctas = a->push_ctas;
  p.push_warps = a->push_warps > 0 ? a->push_warps : 2;
  p.push_bulk = (a->push_mode & MOE_EP_PUSH_BULK) != 0;
  p.push_phased = (a->push_mode & MOE_EP_PUSH_BY_DESTINATION) != 0;
  p.push_hybrid = (a->push_mode & MOE_EP_PUSH_HYBRID) != 0;
  p.l2_stream = (a->push_mode & MOE_EP_PUSH_L2_STREAM) != 0;
  p.merged = (a->sched_mode & MOE_EP_SCHED_MERGED) != 0 && W > 1;
  p.ready_first = (a->sched_mode & MOE_EP_SCHED_READY_FIRST) != 0 && W > 1;
  p.local_first = p.ready_first ? El : a->local_first;
  p.send_counts = a->counts_are_send != 0;
  p.row_groups = (a->sched_mode & MOE_EP_SCHED_ROW_GROUPS_MASK) >> MOE_EP_SCHED_ROW_GROUPS_SHIFT;

  const size_t smem = fused_smem_bytes();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kCudaErr;
  DeviceLaunchInfo& info = g_launch_info[dev];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!info.ready) {
    // Once per device: opt in to the shared memory size and size the
    // persistent grid to the CTA pairs that can be resident together.
    int sms = 0, clusters = 0;
    if (cudaFuncSetAttribute(fused_ep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return kCudaErr;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
    cfg.gridDim = dim3(unsigned(sms & ~1), 1, 1);
    if (cudaOccupancyMaxActiveClusters(&clusters, fused_ep_kernel, &cfg) != cudaSuccess || clusters < 1)
      return kCudaErr;
    info.grid = 2 * std::min(clusters, sms / 2);
    info.ready = true;
  }
  const int grid = a->num_ctas > 0 ? int(a->num_ctas) : info.grid;
  if (a->push_ctas > grid - 2) return kBadArg;  // at least one computing pair
  cfg.gridDim = dim3(unsigned(grid), 1, 1);
  if (cudaLaunchKernelEx(&cfg, fused_ep_kernel, tw, tw4, rl, rr, p) != cudaSuccess) return kCudaErr;
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

}  // namespace moe
