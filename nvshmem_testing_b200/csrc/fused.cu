// Fused expert-parallel layer for sm_100a: count exchange, NVLink dispatch
// with per-chunk arrival flags, and a persistent tcgen05/TMEM grouped GEMM
// whose tiles start as soon as the rows they read have landed.
//
// Reference behaviour (paths within jy1534/nvshmem_testing):
//   alltoall_persistent_gemm.py:207-309  run(): peer copies of each rank's
//       padded chunk, a per-source signal, and a Triton grouped GEMM that
//       spins on the signal, skips rows >= recv_counts[src, e], and stores
//       out[e, src*gm + m, :] in bf16 (fp32 accumulation).
//   baseline.py:18-50                    same output contract through NCCL
//       all_to_all_single + view/permute/flatten + bmm; padded rows are zero.
//
// B200 design (one CTA per SM, 320 threads):
//   warp 0      TMA producer: waits for the arrival flags of a tile's rows,
//               then streams A (token rows, K-major) and B (expert weights,
//               N-major) k-blocks into a 4-stage shared-memory ring.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256,
//               K=16, bf16 -> f32) into one of two TMEM accumulators.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator, bf16 convert, store
//               of the valid rows to out[le, src*gm + m, :].
//   warps 6-9   dispatch: copy this rank's valid rows for every peer straight
//               into the peer's receive buffer over NVLink (16-byte vectors),
//               then release a per-(src, expert, chunk) flag with the call's
//               epoch; afterwards zero the padded output rows.
// Rows this rank sends to itself are never copied: local tiles read them in
// place from the padded send buffer.  Remote rows land in a compact,
// expert-major receive buffer (per expert, sources in the order rank+1,
// rank+2, ...), so one 128-row tile can span several sources.
// Receive buffers, counts and flags are double-buffered by epoch parity; a
// peer reuses parity p only after this rank has published that it finished
// the call that last used it (the "free" epochs), so no per-call barrier or
// flag reset exists.  Every wait is bounded by timeout_ns; on expiry the
// kernel latches MOE_EP_TIMEOUT, drains its in-flight copies and MMAs, frees
// TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "moe_ep.h"
#include "moe_ep_internal.h"
#include "ptx.cuh"

namespace moe {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 4;
constexpr int kEpiWarps = 4;
constexpr int kPushWarps = 4;
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpEpi0 = 2, kWarpPush0 = 2 + kEpiWarps;
constexpr int kThreads = (2 + kEpiWarps + kPushWarps) * 32;
constexpr int kPushThreads = kPushWarps * 32;
constexpr uint32_t kABytes = BM * BK * 2;       // 16 KB
constexpr uint32_t kBBoxBytes = BK * 64 * 2;    // 8 KB: 64 K-rows x 64 N (128 B)
constexpr uint32_t kBBytes = BK * BN * 2;       // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kMaxCells = 512;                  // W * El
constexpr int kMaxLocalExperts = 256;
constexpr uint32_t kAccCols = BN;
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr uint32_t kIdesc = make_idesc(/*bf16*/ 1, BM, BN, /*B N-major*/ 1);
constexpr int kNamedBarPush = 1;

// Where an error was detected (status word "site" byte).
enum Site : int {
  kSiteCounts = 1,
  kSiteTable = 2,
  kSiteTileFlag = 3,
  kSiteFree = 4,
  kSitePipe = 5,
  kSiteDrain = 6,
};

struct Params {
  int W, me, El, H, N;
  int64_t gm;
  const __nv_bfloat16* tokens;
  const int32_t* recv_counts;
  __nv_bfloat16* out;
  const uint64_t* peers;
  unsigned char* local;
  int64_t cap_rows;
  int push_rows, max_chunks;
  uint32_t epoch;
  uint64_t timeout_ns;
  uint64_t off_cmat, off_cflag, off_dflag, off_free, off_local, off_data;
  int32_t* status_host;
};

// Local (never remote-accessed) words at off_local.
struct LocalWords {
  uint32_t push_ctr[2];
  uint32_t done_ctr[2];
  uint32_t status;
  uint32_t pad[3];
};

struct Sched {
  int ntiles_n, kblocks;
  int tiles_total, push_total, zero_total;
  int cnt[kMaxCells];             // [src][le] rows this rank receives
  int seg[kMaxCells + kMaxLocalExperts];  // [le][p], p = 0..W: compact start of position p (seg[.][1] = 0)
  int rbase[kMaxLocalExperts + 1];  // compact base row of expert le in this rank's receive buffer
  int push_off[kMaxCells];        // [d][le] first destination row at rank d
  int push_cnt[kMaxCells];        // [d][le] rows this rank sends to (d, le)
  int push_pfx[kMaxCells + 1];    // prefix of push items over cells (p-1)*El + le
  int tile_pfx[kMaxCells + 1];    // prefix of tiles over cells: local le, then El + (p-1)*El + le
  int tile_mlo[kMaxCells];
};

struct Smem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int push_item;
  uint32_t fills[kStages];
  uint32_t cons[kStages];
};

__device__ __forceinline__ uint32_t* at_u32(unsigned char* base, uint64_t off) {
  return reinterpret_cast<uint32_t*>(base + off);
}

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
}

__device__ __forceinline__ bool aborted(Smem& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0;
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
__device__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t bound_ns, Smem& sm) {
  uint64_t deadline = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63) == 63) {
      if (aborted(sm)) return false;
      const uint64_t now = globaltimer_ns();
      if (deadline == 0) deadline = now + bound_ns;
      else if (now > deadline) return false;
    }
  }
}

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

struct Tile {
  int le, m, n, remote;
};

__device__ __forceinline__ Tile decode_tile(const Sched& s, int W, int El, int t) {
  const int ncells = W * El;
  const int c = find_cell(s.tile_pfx, ncells, t);
  const int r = t - s.tile_pfx[c];
  Tile tile;
  tile.remote = c >= El;
  tile.le = tile.remote ? (c - El) % El : c;
  tile.m = s.tile_mlo[c] + r / s.ntiles_n;
  tile.n = r % s.ntiles_n;
  return tile;
}

// m-tile index of the first tile whose last valid row is >= x (x < R).
__device__ __forceinline__ int first_mtile_reaching(int x) { return x < BM ? 0 : (x - (BM - 1) + BM - 1) / BM; }

// Build the schedule for this call from the full count matrix.  All ranks
// hold identical matrices, so every validation failure is seen by all ranks.
__device__ void build_schedule(const Params& p, Sched& s, Smem& sm) {
  const int W = p.W, El = p.El, me = p.me, tid = threadIdx.x;
  const uint32_t par = p.epoch & 1u;
  const int32_t* cm = reinterpret_cast<const int32_t*>(p.local + p.off_cmat) + size_t(par) * W * W * El;
  // cmat[owner][src][le]: rows src sends to owner's local expert le.
  auto C = [&](int owner, int src, int le) { return cm[(size_t(owner) * W + src) * El + le]; };

  if (tid == 0) {
    s.ntiles_n = (p.N + BN - 1) / BN;
    s.kblocks = (p.H + BK - 1) / BK;
  }
  for (int i = tid; i < W * El; i += kThreads) {
    const int src = i / El, le = i % El;
    s.cnt[i] = C(me, src, le);
  }
  __syncthreads();

  // Validation: 0 <= count <= gm everywhere, chunk slots suffice.
  for (int i = tid; i < W * W * El; i += kThreads) {
    const int v = cm[i];
    if (v < 0 || int64_t(v) > p.gm || (v + p.push_rows - 1) / p.push_rows > p.max_chunks) {
      raise_error(p, sm, kBadArg, kSiteTable, i);
    }
  }

  // Per local expert: compact segment starts (positions 1..W-1) and rows.
  for (int le = tid; le < El; le += kThreads) {
    int* sg = s.seg + le * (W + 1);
    sg[0] = 0;
    sg[1] = 0;
    int run = 0;
    for (int q = 1; q < W; ++q) {
      sg[q] = run;
      run += s.cnt[((me + q) % W) * El + le];
    }
    sg[W] = run;
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int le = 0; le < El; ++le) {
      s.rbase[le] = run;
      run += s.seg[le * (W + 1) + W];
    }
    s.rbase[El] = run;
  }
  // Push offsets: where my rows for (d, le) land at rank d.
  for (int d = tid; d < W; d += kThreads) {
    const int q_me = (me - d + W) % W;  // my position at d (0 means d == me)
    int base = 0;
    for (int le = 0; le < El; ++le) {
      int before = 0, total = 0;
      for (int q = 1; q < W; ++q) {
        const int v = C(d, (d + q) % W, le);
        if (q < q_me) before += v;
        total += v;
      }
      s.push_off[d * El + le] = base + before;
      s.push_cnt[d * El + le] = (d == me) ? 0 : C(d, me, le);
      base += total;
    }
    if (int64_t(base) > p.cap_rows) raise_error(p, sm, kCapacity, kSiteTable, d);
  }
  __syncthreads();

  if (tid == 0) {
    // Push items: positions p = 1..W-1 (destination d = me - p), experts, chunks.
    int run = 0;
    for (int q = 1; q < W; ++q) {
      const int d = (me - q + W) % W;
      for (int le = 0; le < El; ++le) {
        s.push_pfx[(q - 1) * El + le] = run;
        run += (s.push_cnt[d * El + le] + p.push_rows - 1) / p.push_rows;
      }
    }
    s.push_pfx[(W - 1) * El] = run;
    s.push_total = run;
    s.zero_total = W * El;

    // Tiles: local cells first, then remote cells by the latest position
    // their rows depend on, so work follows data arrival.
    const int nn = s.ntiles_n;
    int t = 0;
    for (int le = 0; le < El; ++le) {
      s.tile_pfx[le] = t;
      s.tile_mlo[le] = 0;
      t += ((s.cnt[me * El + le] + BM - 1) / BM) * nn;
    }
    for (int q = 1; q < W; ++q) {
      for (int le = 0; le < El; ++le) {
        const int c = El + (q - 1) * El + le;
        const int* sg = s.seg + le * (W + 1);
        const int R = sg[W];
        const int mtiles = (R + BM - 1) / BM;
        const int lo = sg[q] < R ? first_mtile_reaching(sg[q]) : mtiles;
        const int hi = (q + 1 <= W - 1 && sg[q + 1] < R) ? first_mtile_reaching(sg[q + 1]) : mtiles;
        const int lo_c = (sg[q] < sg[q + 1]) ? lo : hi;  // empty segment: no tiles
        s.tile_pfx[c] = t;
        s.tile_mlo[c] = lo_c;
        t += (hi > lo_c ? hi - lo_c : 0) * nn;
      }
    }
    s.tile_pfx[W * El] = t;
    s.tiles_total = t;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1)
    fused_ep_kernel(const __grid_constant__ CUtensorMap tm_a_local, const __grid_constant__ CUtensorMap tm_a_remote,
                    const __grid_constant__ CUtensorMap tm_b, const Params p) {
  extern __shared__ unsigned char smem_dyn[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  unsigned char* stage_mem = base;  // kStages * kStageBytes, 1024-aligned
  Sched& s = *reinterpret_cast<Sched*>(base + kStages * kStageBytes);
  Smem& sm = *reinterpret_cast<Smem*>(base + kStages * kStageBytes + sizeof(Sched));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int W = p.W, El = p.El, me = p.me;
  const uint32_t par = p.epoch & 1u;
  const uint64_t pipe_bound = 2 * p.timeout_ns + 1000000000ull;
  LocalWords* lw = reinterpret_cast<LocalWords*>(p.local + p.off_local);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
      sm.fills[i] = 0;
      sm.cons[i] = 0;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], kEpiWarps);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_a_local);
    prefetch_tensormap(&tm_a_remote);
    prefetch_tensormap(&tm_b);
  }
  if (warp == kWarpMma) {
    __syncwarp();
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sm.tmem_base;

  // ---- count exchange: CTA 0 publishes this rank's recv_counts block to
  // every rank; every CTA then waits for all W blocks.
  if (blockIdx.x == 0 && warp == kWarpPush0) {
    for (int d = 0; d < W; ++d) {
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
    for (int q = 0; q < W; ++q) {
      if (!wait_epoch(at_u32(p.local, p.off_cflag) + par * W + q, p.epoch, p.timeout_ns, sm)) {
        raise_error(p, sm, kTimeout, kSiteCounts, q);
        break;
      }
    }
  }
  __syncthreads();
  if (!aborted(sm)) build_schedule(p, s, sm);
  __syncthreads();
  const bool run_main = !aborted(sm);

  if (run_main && warp == kWarpProducer) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < s.tiles_total; t += gridDim.x) {
        const Tile tl = decode_tile(s, W, El, t);
        int arow;
        const CUtensorMap* amap;
        if (!tl.remote) {
          arow = int((int64_t(me) * El + tl.le) * p.gm + int64_t(tl.m) * BM);
          amap = &tm_a_local;
        } else {
          const int* sg = s.seg + tl.le * (W + 1);
          const int R = sg[W];
          const int r0 = tl.m * BM, r1 = min(r0 + BM, R);
          bool ok = true;
          for (int q = 1; q < W && ok; ++q) {
            const int lo = max(r0, sg[q]), hi = min(r1, sg[q + 1]);
            if (lo >= hi) continue;
            const int src = (me + q) % W;
            const uint32_t* fl = at_u32(p.local, p.off_dflag) + ((size_t(par) * W + src) * El + tl.le) * p.max_chunks;
            for (int c = (lo - sg[q]) / p.push_rows; c <= (hi - 1 - sg[q]) / p.push_rows; ++c) {
              if (!wait_epoch(fl + c, p.epoch, p.timeout_ns, sm)) {
                raise_error(p, sm, kTimeout, kSiteTileFlag, src);
                ok = false;
                break;
              }
            }
          }
          if (!ok) break;
          fence_proxy_async_global();
          arow = int(int64_t(par) * p.cap_rows + s.rbase[tl.le] + r0);
          amap = &tm_a_remote;
        }
        const int n0 = tl.n * BN;
        const int nb = min(4, (p.N - n0 + 63) / 64);
        const uint32_t tx = kABytes + uint32_t(nb) * kBBoxBytes;
        bool stop = false;
        for (int kb = 0; kb < s.kblocks; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t round = it / kStages;
          if (!mbar_wait(&sm.empty[st], (round & 1) ^ 1, pipe_bound, sm)) {
            stop = true;
            break;
          }
          unsigned char* a_dst = stage_mem + st * kStageBytes;
          unsigned char* b_dst = a_dst + kABytes;
          mbar_arrive_expect_tx(&sm.full[st], tx);
          tma_load_2d(amap, &sm.full[st], a_dst, kb * BK, arow);
          for (int j = 0; j < nb; ++j) tma_load_3d(&tm_b, &sm.full[st], b_dst + j * kBBoxBytes, n0 + 64 * j, kb * BK, tl.le);
          sm.fills[st] += 1;
        }
        if (stop) break;
      }
    }
  } else if (run_main && warp == kWarpMma) {
    if (lane == 0) {
      uint32_t it = 0, local_tile = 0;
      for (int t = blockIdx.x; t < s.tiles_total; t += gridDim.x, ++local_tile) {
        const uint32_t acc = local_tile & 1;
        const uint32_t use = local_tile >> 1;
        if (!mbar_wait(&sm.tempty[acc], (use & 1) ^ 1, pipe_bound, sm)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        bool stop = false;
        for (int kb = 0; kb < s.kblocks; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t round = it / kStages;
          if (!mbar_wait(&sm.full[st], round & 1, pipe_bound, sm)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_mem + st * kStageBytes);
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b_addr + k * 2048, kBBoxBytes, 1024);
            tc_mma_f16(d_tmem, ad, bd, kIdesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&sm.empty[st]);
          sm.cons[st] += 1;
        }
        if (stop) break;
        tc_commit(&sm.tfull[acc]);
      }
    }
  } else if (run_main && warp >= kWarpEpi0 && warp < kWarpPush0) {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    uint32_t local_tile = 0;
    for (int t = blockIdx.x; t < s.tiles_total; t += gridDim.x, ++local_tile) {
      const Tile tl = decode_tile(s, W, El, t);
      const uint32_t acc = local_tile & 1;
      const uint32_t use = local_tile >> 1;
      if (!mbar_wait(&sm.tfull[acc], use & 1, pipe_bound, sm)) break;
      tc_fence_after();
      // Output row of this thread's accumulator lane (-1: not a valid row).
      int64_t orow = -1;
      if (!tl.remote) {
        const int m = tl.m * BM + row;
        if (m < s.cnt[me * El + tl.le]) orow = int64_t(tl.le) * W * p.gm + int64_t(me) * p.gm + m;
      } else {
        const int* sg = s.seg + tl.le * (W + 1);
        const int r = tl.m * BM + row;
        if (r < sg[W]) {
          int q = 1;
          while (q < W - 1 && r >= sg[q + 1]) ++q;
          const int src = (me + q) % W;
          orow = int64_t(tl.le) * W * p.gm + int64_t(src) * p.gm + (r - sg[q]);
        }
      }
      const int n0 = tl.n * BN;
      __nv_bfloat16* orow_ptr = p.out + (orow < 0 ? 0 : orow) * p.N;
#pragma unroll 1
      for (int j = 0; j < BN / 32; ++j) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tmem_base + acc * kAccCols + (uint32_t(quarter * 32) << 16) + j * 32, r);
        tmem_ld_wait();
        if (orow >= 0) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int col = n0 + j * 32 + c8 * 8;
            if (col + 8 <= p.N) {
              uint4 v;
              __nv_bfloat162 h0 = __floats2bfloat162_rn(__uint_as_float(r[c8 * 8 + 0]), __uint_as_float(r[c8 * 8 + 1]));
              __nv_bfloat162 h1 = __floats2bfloat162_rn(__uint_as_float(r[c8 * 8 + 2]), __uint_as_float(r[c8 * 8 + 3]));
              __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(r[c8 * 8 + 4]), __uint_as_float(r[c8 * 8 + 5]));
              __nv_bfloat162 h3 = __floats2bfloat162_rn(__uint_as_float(r[c8 * 8 + 6]), __uint_as_float(r[c8 * 8 + 7]));
              v.x = *reinterpret_cast<uint32_t*>(&h0);
              v.y = *reinterpret_cast<uint32_t*>(&h1);
              v.z = *reinterpret_cast<uint32_t*>(&h2);
              v.w = *reinterpret_cast<uint32_t*>(&h3);
              *reinterpret_cast<uint4*>(orow_ptr + col) = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tempty[acc]);
    }
  } else if (run_main && warp >= kWarpPush0) {
    const int pt = tid - kWarpPush0 * 32;
    const size_t row_bytes = size_t(p.H) * 2;
    for (;;) {
      if (pt == 0) {
        int it = aborted(sm) ? 0x7fffffff : int(atomicAdd(&lw->push_ctr[par], 1u));
        if (it < s.push_total && p.epoch > 2) {
          const int c = find_cell(s.push_pfx, (W - 1) * El, it);
          const int d = (me - (c / El + 1) + W) % W;
          if (!wait_epoch(at_u32(p.local, p.off_free) + d, p.epoch - 2, p.timeout_ns, sm)) {
            raise_error(p, sm, kTimeout, kSiteFree, d);
            it = 0x7fffffff;
          }
        }
        sm.push_item = it;
      }
      named_bar_sync(kNamedBarPush, kPushThreads);
      const int item = sm.push_item;
      named_bar_sync(kNamedBarPush, kPushThreads);
      if (item < s.push_total) {
        const int c = find_cell(s.push_pfx, (W - 1) * El, item);
        const int q = c / El + 1, le = c % El;
        const int d = (me - q + W) % W;
        const int chunk = item - s.push_pfx[c];
        const int j0 = chunk * p.push_rows;
        const int j1 = min(j0 + p.push_rows, s.push_cnt[d * El + le]);
        unsigned char* peer = reinterpret_cast<unsigned char*>(p.peers[d]);
        const uint4* src = reinterpret_cast<const uint4*>(p.tokens + ((int64_t(d) * El + le) * p.gm + j0) * p.H);
        uint4* dst = reinterpret_cast<uint4*>(peer + p.off_data +
                                              (size_t(par) * p.cap_rows + s.push_off[d * El + le] + j0) * row_bytes);
        const int64_t nvec = int64_t(j1 - j0) * int64_t(row_bytes / 16);
        int64_t v = pt;
        for (; v + 3 * kPushThreads < nvec; v += 4 * kPushThreads) {
          const uint4 a0 = ld_nc_v4(src + v);
          const uint4 a1 = ld_nc_v4(src + v + kPushThreads);
          const uint4 a2 = ld_nc_v4(src + v + 2 * kPushThreads);
          const uint4 a3 = ld_nc_v4(src + v + 3 * kPushThreads);
          st_v4(dst + v, a0);
          st_v4(dst + v + kPushThreads, a1);
          st_v4(dst + v + 2 * kPushThreads, a2);
          st_v4(dst + v + 3 * kPushThreads, a3);
        }
        for (; v < nvec; v += kPushThreads) st_v4(dst + v, ld_nc_v4(src + v));
        fence_acq_rel_sys();
        named_bar_sync(kNamedBarPush, kPushThreads);
        if (pt == 0) {
          uint32_t* fl = at_u32(peer, p.off_dflag) + ((size_t(par) * W + me) * El + le) * p.max_chunks + chunk;
          st_release_sys(fl, p.epoch);
        }
      } else if (item < s.push_total + s.zero_total) {
        const int z = item - s.push_total;
        const int le = z / W, src = z % W;
        const int64_t c0 = s.cnt[src * El + le];
        const int64_t nvec = (p.gm - c0) * int64_t(p.N) / 8;
        uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t(le) * W * p.gm + int64_t(src) * p.gm + c0) * p.N);
        const uint4 zv = make_uint4(0, 0, 0, 0);
        for (int64_t v = pt; v < nvec; v += kPushThreads) dst[v] = zv;
      } else {
        break;
      }
    }
  }

  // ---- teardown: drain in-flight copies and MMAs, free TMEM, publish "free".
  __syncthreads();
  if (tid == 0) {
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
  if (warp == kWarpMma && lane == 0) {
    tc_commit(&sm.drain);
    const uint64_t deadline = globaltimer_ns() + 1000000000ull;
    while (!mbar_try_wait(&sm.drain, 0)) {
      if (globaltimer_ns() > deadline) {
        raise_error(p, sm, kTimeout, kSiteDrain, 99);
        break;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (tid == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(&lw->done_ctr[par], 1u);
    if (old == gridDim.x - 1) {
      __threadfence();
      lw->push_ctr[par ^ 1] = 0;
      lw->done_ctr[par ^ 1] = 0;
      __threadfence();
      for (int q = 0; q < W; ++q) {
        unsigned char* peer = reinterpret_cast<unsigned char*>(p.peers[q]);
        st_release_sys(at_u32(peer, p.off_free) + me, p.epoch);
      }
    }
  }
}

// ------------------------------------------------------------------ host side

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int workspace_layout(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks, moe_ep_layout* L) {
  size_t off = 0;
  L->off_cmat = off;
  off = align_up(off + size_t(2) * W * W * El * 4, 256);
  L->off_cflag = off;
  off = align_up(off + size_t(2) * W * 4, 256);
  L->off_dflag = off;
  off = align_up(off + size_t(2) * W * El * max_chunks * 4, 256);
  L->off_free = off;
  off = align_up(off + size_t(W) * 4, 256);
  L->off_local = off;
  off = align_up(off + sizeof(LocalWords), 256);
  L->ctrl_bytes = off;
  off = align_up(off, 4096);
  L->off_data = off;
  off += size_t(2) * cap_rows * H * elem_bytes;
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

size_t fused_smem_bytes() { return 1024 + size_t(kStages) * kStageBytes + sizeof(Sched) + sizeof(Smem); }

int launch_fused(const moe_ep_run_params* a, cudaStream_t stream) {
  const int W = a->world_size, El = a->local_experts;
  if (W < 1 || W > 64 || a->rank < 0 || a->rank >= W || El < 1 || El > kMaxLocalExperts || W * El > kMaxCells)
    return kBadArg;
  if (a->elem_bytes != 2 || a->hidden <= 0 || a->out_dim <= 0 || a->hidden % 8 || a->out_dim % 8 || a->gm < 0)
    return kBadArg;
  if (a->push_rows <= 0 || a->max_chunks <= 0 || a->cap_rows < 0 || a->epoch == 0) return kBadArg;
  if (!a->tokens || !a->weights || !a->out || !a->peer_bases || !a->local_base || !a->recv_counts) return kBadArg;
  if ((reinterpret_cast<uintptr_t>(a->tokens) | reinterpret_cast<uintptr_t>(a->weights) |
       reinterpret_cast<uintptr_t>(a->out)) & 15)
    return kBadArg;
  const int64_t rows_in = int64_t(W) * El * a->gm;
  if (rows_in + BM > (int64_t(1) << 31) || 2 * a->cap_rows + BM > (int64_t(1) << 31)) return kBadArg;
  if (!driver().ok) return kCudaErr;

  moe_ep_layout L;
  workspace_layout(W, El, a->hidden, a->elem_bytes, a->cap_rows, a->max_chunks, &L);
  unsigned char* local = reinterpret_cast<unsigned char*>(a->local_base);

  CUtensorMap ta_local, ta_remote, tb;
  const uint64_t H = uint64_t(a->hidden), N = uint64_t(a->out_dim);
  if (rows_in == 0) {
    // No rows at all: map a single dummy row so the descriptor stays valid.
    if (encode_2d(&ta_local, a->tokens, H, 1, H * 2, BK, BM)) return kCudaErr;
  } else if (encode_2d(&ta_local, a->tokens, H, uint64_t(rows_in), H * 2, BK, BM)) {
    return kCudaErr;
  }
  // With no remote capacity (one rank) no remote tile exists; the map then
  // describes the token buffer so that it never names unbacked memory.
  if (a->cap_rows > 0) {
    if (encode_2d(&ta_remote, local + L.off_data, H, uint64_t(2 * a->cap_rows), H * 2, BK, BM)) return kCudaErr;
  } else {
    ta_remote = ta_local;
  }
  if (encode_3d(&tb, a->weights, N, H, uint64_t(El), N * 2, H * N * 2, 64, BK)) return kCudaErr;

  Params p;
  p.W = W;
  p.me = a->rank;
  p.El = El;
  p.H = a->hidden;
  p.N = a->out_dim;
  p.gm = a->gm;
  p.tokens = static_cast<const __nv_bfloat16*>(a->tokens);
  p.recv_counts = a->recv_counts;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.peers = a->peer_bases;
  p.local = local;
  p.cap_rows = a->cap_rows;
  p.push_rows = a->push_rows;
  p.max_chunks = a->max_chunks;
  p.epoch = a->epoch;
  p.timeout_ns = a->timeout_ns;
  p.off_cmat = L.off_cmat;
  p.off_cflag = L.off_cflag;
  p.off_dflag = L.off_dflag;
  p.off_free = L.off_free;
  p.off_local = L.off_local;
  p.off_data = L.off_data;
  p.status_host = a->status_host;

  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  const int grid = a->num_ctas > 0 ? int(a->num_ctas) : sms;
  const size_t smem = fused_smem_bytes();
  if (cudaFuncSetAttribute(fused_ep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return kCudaErr;
  fused_ep_kernel<<<grid, kThreads, smem, stream>>>(ta_local, ta_remote, tb, p);
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

}  // namespace moe
