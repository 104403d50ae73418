// Router: the step before the path (utils.py:17-25 of the reference:
// logits = einsum('bh,he->be', tokens, router) in bf16, softmax over the
// experts, top-k).
//
// E <= 256: one kernel, router_kernel.  Each cluster of S CTAs (S = 1, 2, 4
// or 8, chosen so that the grid fills the SMs) computes one 128-token tile:
// CTA r of the cluster multiplies the tile by the r-th 1/S of the hidden
// dimension on the tensor cores (tcgen05.mma kind::f16, M = 128 tokens,
// N = E, fp32 accumulators in TMEM, TMA-fed 4-stage pipeline).  The S
// partial tiles are then reduced through distributed shared memory: CTA r
// owns rows [r*128/S, (r+1)*128/S) of the tile, every CTA sends each row's
// partial sums to the row's owner, and the owner adds the S partials in CTA
// order (deterministic), rounds the logits once to bf16 (the reference's
// einsum dtype), writes them, and takes the softmax and top-k of each row
// (S threads per row): fp32 softmax of the bf16 logits rounded to bf16
// (the reference's softmax output dtype), the K largest probabilities in
// descending order, equal probabilities by ascending expert id (torch.topk
// leaves their order unspecified).  No control words, nothing allocated.
//
// E > 256: the logits GEMM runs on the fused layer kernel as a one-rank,
// one-expert layer (tokens = x [T, H], weights = the router [H, E], out =
// logits [T, E]) whose control words live in a fixed array of this file, and
// a second kernel takes the softmax and top-k (the same arithmetic); calls of
// this form must not overlap on the GPU, and the first one on a device looks
// the array's address up (make it before any stream capture).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <climits>
#include <mutex>

#include "moe_ep.h"
#include "moe_ep_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

constexpr size_t kRouterScratchBytes = 2048;
constexpr size_t kPeerTable = 256;                          // [0, 256): control base of the one rank
constexpr size_t kCountOffset = kRouterScratchBytes - 16;   // int32 rows of the one (rank, expert) cell
constexpr int kMaxDevices = 64;
constexpr int kTopkThreads = 256;
constexpr int kTopkWarps = kTopkThreads / 32;

__device__ __align__(256) unsigned char g_router_scratch[kRouterScratchBytes];

uint64_t g_router_addr[kMaxDevices];
std::mutex g_router_setup;

// Once per device, with `dev` current: the array's device address, and the
// control base stored in its peer-table slot.
int router_scratch(int dev, uint64_t* out) {
  std::lock_guard<std::mutex> lock(g_router_setup);
  if (g_router_addr[dev] == 0) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_router_scratch) != cudaSuccess || ptr == nullptr) return kCudaErr;
    const uint64_t control_base = reinterpret_cast<uint64_t>(ptr) + kPeerTable;
    if (cudaMemcpyToSymbol(g_router_scratch, &control_base, sizeof(control_base), 0, cudaMemcpyHostToDevice) !=
        cudaSuccess)
      return kCudaErr;
    g_router_addr[dev] = reinterpret_cast<uint64_t>(ptr);
  }
  *out = g_router_addr[dev];
  return kOk;
}

__global__ void set_count_kernel(int32_t* p, int32_t v) { *p = v; }

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// ---------------------------------------------------------------- E <= 256: split-K cluster kernel
constexpr int kRtThreads = 512;                 // 16 warps; warp w reads TMEM lane quarter w % 4
constexpr int kRtStages = 4;
constexpr int kRtKB = 64;                       // K per stage (one 128-byte swizzle atom of bf16)
constexpr int kRtTile = 128;                    // tokens per tile (MMA M)
constexpr int kRtMaxE = 256;                    // MMA N and TMEM columns
constexpr uint32_t kRtXBytes = kRtTile * kRtKB * 2;           // 16 KB
constexpr uint32_t kRtAtomBytes = 64 * kRtKB * 2;             // 8 KB: 64 experts x 64 K
constexpr uint32_t kRtStageBytes = kRtXBytes + 4 * kRtAtomBytes;  // 48 KB
constexpr uint64_t kRtBoundNs = 2000000000ull;  // bug guard on every pipeline wait

struct RouterArgs {
  int64_t T;
  int H, E, K, S;          // S: CTAs per cluster (split of the hidden dimension)
  int kblocks, kb_per;     // k-blocks of the whole H, per CTA
  int n_mma, tmem_cols, ep;  // MMA N (E rounded to 16), TMEM columns, floats per exchanged row
  int r3d;                   // the router map is 3-D: one box holds every 64-expert atom of a stage
  __nv_bfloat16* logits;
  void* ids;
  float* vals;
  int32_t* status_host;
};

struct alignas(16) RtSmem {
  uint64_t full[kRtStages];
  uint64_t empty[kRtStages];
  uint64_t acc;
  uint64_t drain;
  uint32_t tmem_base;
  int err;
  uint32_t fills[kRtStages];
};

__device__ __forceinline__ bool rt_wait(uint64_t* bar, uint32_t parity, RtSmem& sm) {
  uint64_t deadline = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63) == 63) {
      if (*reinterpret_cast<volatile int*>(&sm.err)) return false;
      const uint64_t now = globaltimer_ns();
      if (deadline == 0) deadline = now + kRtBoundNs;
      else if (now > deadline) return false;
    }
  }
}

__device__ void rt_fail(RtSmem& sm, const RouterArgs& a, int detail) {
  if (atomicExch(&sm.err, 1) == 0 && a.status_host)
    *reinterpret_cast<volatile int32_t*>(a.status_host) = int32_t(status_word(kTimeout, kSitePipe, detail));
}

__device__ __forceinline__ void st_shared_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Float index of (row, col) in one source's block of the exchange buffer:
// rows of `ep` floats, 16-byte chunks XOR-swizzled by the row so that both
// the senders (one row per lane) and the owner's readers (one row per warp,
// consecutive columns per lane) touch distinct banks.
__device__ __forceinline__ int rt_xidx(int row, int col, int ep) {
  return row * ep + ((((col >> 2) ^ (row & 7))) << 2) + (col & 3);
}

// One owner row's softmax and top-k with its VPT values per thread held in
// registers (TPR threads per row, thread `part` holding experts part,
// part + TPR, ...): the same arithmetic, in the same order, as the shared-
// memory form below.  The S partial sums are read one source block at a
// time, all VPT loads of a block in flight together, before any store (a
// store between them would order every later load behind it).  Each
// probability then becomes one 32-bit key, its bf16 bits above
// (0xFFFF - expert), kept in the same registers: probabilities are >= 0, so
// the keys order like the values, and equal values order by ascending
// expert id.  A top-k pick is one max over the thread's keys and one shuffle
// max over the row; the picked key is unique and is cleared where it is held.
template <int VPT, typename IdT>
__device__ __forceinline__ void rt_row_topk_regs(const RouterArgs& a, const float* xbuf, int S, int R, int TPR,
                                                 int lr, int part, int64_t t, bool live) {
  const int E = a.E, K = a.K;
  float lv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) lv[j] = 0.f;
  for (int q = 0; q < S; ++q) {
    const float* blk = xbuf + q * R * a.ep;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int e = part + j * TPR;
      if (e < E) lv[j] += blk[rt_xidx(lr, e, a.ep)];
    }
  }
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = part + j * TPR;
    if (e < E) {
      const __nv_bfloat16 lb = __float2bfloat16_rn(lv[j]);
      if (live) a.logits[t * E + e] = lb;
      lv[j] = __bfloat162float(lb);
      m = fmaxf(m, lv[j]);
    }
  }
  for (int o = 1; o < TPR; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if (part + j * TPR < E) z += expf(lv[j] - m);
  for (int o = 1; o < TPR; o <<= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = part + j * TPR;
    uint32_t key = 0u;
    if (e < E) {
      const __nv_bfloat16 pb = __float2bfloat16_rn(expf(lv[j] - m) / z);
      key = (uint32_t(__bfloat16_as_ushort(pb)) << 16) | uint32_t(0xFFFF - e);
    }
    lv[j] = __uint_as_float(key);  // the key's bits, never used as a number
  }
  IdT* ids = static_cast<IdT*>(a.ids);
  for (int k = 0; k < K; ++k) {
    uint32_t b = 0u;
#pragma unroll
    for (int j = 0; j < VPT; ++j) b = max(b, __float_as_uint(lv[j]));
    for (int o = 1; o < TPR; o <<= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
#pragma unroll
    for (int j = 0; j < VPT; ++j) lv[j] = __float_as_uint(lv[j]) == b ? 0.f : lv[j];
    if (part == 0 && live) {
      ids[t * K + k] = static_cast<IdT>(0xFFFF - int(b & 0xFFFFu));
      a.vals[t * K + k] = __uint_as_float(b & 0xFFFF0000u);
    }
  }
}

template <typename IdT>
__global__ void __launch_bounds__(kRtThreads, 1)
    router_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_r,
                  const RouterArgs a) {
  extern __shared__ unsigned char rt_dyn[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(rt_dyn) + 1023) & ~uintptr_t(1023));
  RtSmem& sm = *reinterpret_cast<RtSmem*>(base + kRtStages * kRtStageBytes);
  float* xbuf = reinterpret_cast<float*>(base);  // exchange buffer [S][128/S][ep], reuses the stages

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.S;
  const int r = S > 1 ? int(cluster_ctarank()) : 0;
  const int64_t m0 = int64_t(blockIdx.x / S) * kRtTile;
  const int kb0 = r * a.kb_per;
  const int kb1 = min(a.kblocks, kb0 + a.kb_per);
  const int nk = max(0, kb1 - kb0);
  const int atoms = (a.n_mma + 63) / 64;
  const uint32_t tx = kRtXBytes + uint32_t(atoms) * kRtAtomBytes;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRtStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
      sm.fills[i] = 0;
    }
    mbar_init(&sm.acc, 1);
    mbar_init(&sm.drain, 1);
    sm.err = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_r);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(&sm.tmem_base, uint32_t(a.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0 && lane == 0) {
    // TMA producer: the tile's 128 tokens and the router rows of this CTA's k-blocks.
    for (int i = 0; i < nk; ++i) {
      const int st = i % kRtStages;
      if (i >= kRtStages && !rt_wait(&sm.empty[st], ((i / kRtStages) & 1) ^ 1, sm)) {
        rt_fail(sm, a, 1);
        break;
      }
      unsigned char* dst = base + st * kRtStageBytes;
      const int kc = (kb0 + i) * kRtKB;
      mbar_arrive_expect_tx(&sm.full[st], tx);
      tma_load_2d(&tm_x, &sm.full[st], dst, kc, int(m0));
      if (a.r3d) {
        tma_load_3d(&tm_r, &sm.full[st], dst + kRtXBytes, 0, kc, 0);
      } else {
        for (int at = 0; at < atoms; ++at)
          tma_load_2d(&tm_r, &sm.full[st], dst + kRtXBytes + at * kRtAtomBytes, at * 64, kc);
      }
      sm.fills[st] += 1;
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: D[128 tokens, N] (+)= X[128, 64] . R[64, N] per stage.
    const uint32_t idesc = make_idesc_mn(/*bf16*/ 1, kRtTile, uint32_t(a.n_mma), /*A K-major*/ 0, /*B N-major*/ 1);
    int i = 0;
    for (; i < nk; ++i) {
      const int st = i % kRtStages;
      if (!rt_wait(&sm.full[st], (i / kRtStages) & 1, sm)) {
        rt_fail(sm, a, 2);
        break;
      }
      tc_fence_after();
      const uint32_t xa = smem_u32(base + st * kRtStageBytes);
      const uint32_t ra = xa + kRtXBytes;
#pragma unroll
      for (int k = 0; k < kRtKB / 16; ++k) {
        const uint64_t ad = smem_desc_sw128(xa + k * 32, 16, 1024);                 // K-major: 16 K = 32 bytes
        const uint64_t bd = smem_desc_sw128(ra + k * 2048, kRtAtomBytes, 1024);     // N-major: 16 K = 2 x 8 rows
        tc_mma_f16(tmem, ad, bd, idesc, (i | k) != 0 ? 1u : 0u);
      }
      tc_commit(&sm.empty[st]);
    }
    tc_commit(nk > 0 && i == nk ? &sm.acc : &sm.drain);  // accumulator ready (or: every issued MMA done)
  }
  __syncwarp();

  // This CTA's partial tile: wait for the accumulator (none without k-blocks).
  if (nk > 0 && !rt_wait(&sm.acc, 0, sm)) rt_fail(sm, a, 3);
  __syncthreads();
  tc_fence_after();
  const bool ok = nk > 0 && !*reinterpret_cast<volatile int*>(&sm.err);  // uniform over the CTA
  // Every CTA of the cluster is done reading its stages: they become the
  // exchange buffer.
  if (S > 1) cluster_sync();

  // Exchange: row (32*(warp % 4) + lane) of the partial tile goes to its
  // owner, into block r of the owner's buffer; the four warps of a lane
  // quarter take every fourth 64-column group.
  const int R = kRtTile / S;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int owner = row / R, lrow = row % R;
  const uint32_t blk = smem_u32(xbuf) + uint32_t(r * R * a.ep) * 4u;
  const uint32_t dst_blk = S > 1 ? mapa_shared(blk, uint32_t(owner)) : blk;
  // 64 columns per round: two TMEM loads behind one wait.  Rows past T (the
  // last tile, small decode batches) are not sent; a warp none of whose 32
  // rows is a token skips its TMEM loads too.
  const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16);
  const bool row_live = m0 + row < a.T;
  const bool warp_live = __any_sync(0xffffffffu, row_live);
  for (int c0 = (warp >> 2) * 64; warp_live && c0 < a.ep; c0 += (kRtThreads / 128) * 64) {
    uint32_t v0[32], v1[32];
    const bool l0 = ok && c0 < a.n_mma, l1 = ok && c0 + 32 < a.n_mma;
    if (l0) tmem_ld_32x32b_x32(trow + uint32_t(c0), v0);
    if (l1) tmem_ld_32x32b_x32(trow + uint32_t(c0 + 32), v1);
    if (l0 || l1) tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (!l0) v0[j] = 0u;
      if (!l1) v1[j] = 0u;
    }
#pragma unroll
    for (int j = 0; j < 32 && row_live; j += 4) {
      st_shared_cluster_v4(dst_blk + uint32_t(rt_xidx(lrow, c0 + j, a.ep)) * 4u, v0[j], v0[j + 1], v0[j + 2],
                           v0[j + 3]);
      if (c0 + 32 < a.ep)
        st_shared_cluster_v4(dst_blk + uint32_t(rt_xidx(lrow, c0 + 32 + j, a.ep)) * 4u, v1[j], v1[j + 1], v1[j + 2],
                             v1[j + 3]);
    }
  }
  tc_fence_before();
  if (S > 1) cluster_sync();  // every partial has reached its owner
  else __syncthreads();

  // Owner: rows [r*R, (r+1)*R) of the tile; TPR = kRtThreads / R
  // neighbouring threads per row, thread `part` holding experts part,
  // part + TPR, ...
  // The partials are summed in CTA order, the bf16 logit written out and
  // kept in block 0 of the buffer (then replaced by its probability); the
  // row's max, sum and each top-k pick combine the S threads by shuffles.
  const int E = a.E, K = a.K;
  const int TPR = kRtThreads / R;  // 4 * S: 4..32, a power of two dividing 32
  const int lr = int(threadIdx.x) / TPR, part = int(threadIdx.x) % TPR;
  const int64_t t = m0 + int64_t(r) * R + lr;
  // Rows past T were not exchanged: a warp with no live row skips them; in
  // a warp with some, they compute on stale values and write nothing.
  const bool live = t < a.T;
  const int vpt = (E + TPR - 1) / TPR;
  if (!__any_sync(0xffffffffu, live)) {
  } else if (vpt <= 8) rt_row_topk_regs<8, IdT>(a, xbuf, S, R, TPR, lr, part, t, live);
  else if (vpt <= 16) rt_row_topk_regs<16, IdT>(a, xbuf, S, R, TPR, lr, part, t, live);
  else if (vpt <= 32) rt_row_topk_regs<32, IdT>(a, xbuf, S, R, TPR, lr, part, t, live);
  else {
  // More than 32 values per thread (one CTA per tile and E > 128): the
  // values stay in the exchange buffer.
  float m = -INFINITY;
  for (int e = part; e < E; e += TPR) {
    const int xi = rt_xidx(lr, e, a.ep);
    float sum = 0.f;
    for (int q = 0; q < S; ++q) sum += xbuf[q * R * a.ep + xi];
    const __nv_bfloat16 lb = __float2bfloat16_rn(sum);
    if (live) a.logits[t * E + e] = lb;
    const float v = __bfloat162float(lb);
    xbuf[xi] = v;
    m = fmaxf(m, v);
  }
  for (int o = 1; o < TPR; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
  for (int e = part; e < E; e += TPR) z += expf(xbuf[rt_xidx(lr, e, a.ep)] - m);
  for (int o = 1; o < TPR; o <<= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  // Probabilities are >= 0; -2 marks one already taken.
  for (int e = part; e < E; e += TPR) {
    const int xi = rt_xidx(lr, e, a.ep);
    xbuf[xi] = __bfloat162float(__float2bfloat16_rn(expf(xbuf[xi] - m) / z));
  }
  IdT* ids = static_cast<IdT*>(a.ids);
  for (int k = 0; k < K; ++k) {
    float best = -3.f;
    int be = INT_MAX;
    for (int e = part; e < E; e += TPR) {  // ascending ids: a strict > keeps the lowest id of equal values
      const float v = xbuf[rt_xidx(lr, e, a.ep)];
      if (v > best) {
        best = v;
        be = e;
      }
    }
    for (int o = 1; o < TPR; o <<= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ob > best || (ob == best && oe < be)) {
        best = ob;
        be = oe;
      }
    }
    if (be % TPR == part) xbuf[rt_xidx(lr, be, a.ep)] = -2.f;
    if (part == 0 && live) {
      ids[t * K + k] = static_cast<IdT>(be);
      a.vals[t * K + k] = best;
    }
  }
  }

  // Teardown: after an abort, wait (bounded) for every issued load and MMA.
  if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(&sm.err)) {
    const uint64_t until = globaltimer_ns() + kRtBoundNs;
    for (int st = 0; st < kRtStages; ++st) {
      const uint32_t f = sm.fills[st];
      if (f == 0) continue;
      while (!mbar_try_wait(&sm.full[st], (f - 1) & 1) && globaltimer_ns() < until) {
      }
    }
    while (!mbar_try_wait(&sm.drain, 0) && globaltimer_ns() < until) {
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, uint32_t(a.tmem_cols));
  }
}

int encode_router_maps(CUtensorMap* mx, CUtensorMap* mr, const void* x, int64_t T, int H, const void* rw, int E,
                       bool r3d) {
  const Driver& d = driver();
  if (!d.ok) return kCudaErr;
  {
    cuuint64_t dims[2] = {cuuint64_t(H), cuuint64_t(T)};
    cuuint64_t strides[1] = {cuuint64_t(H) * 2};
    cuuint32_t box[2] = {cuuint32_t(kRtKB), cuuint32_t(kRtTile)};
    cuuint32_t estr[2] = {1, 1};
    if (d.cuTensorMapEncodeTiled(mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return kCudaErr;
  }
  if (r3d) {
    // Router rows [H, E] seen as (64 experts, K, E/64 atoms): one box of
    // every atom of a 64-deep stage (few, large boxes keep more bytes in
    // flight); rows past H read as zeros.
    cuuint64_t dims[3] = {64, cuuint64_t(H), cuuint64_t(E / 64)};
    cuuint64_t strides[2] = {cuuint64_t(E) * 2, 128};
    cuuint32_t box[3] = {64, cuuint32_t(kRtKB), cuuint32_t(E / 64)};
    cuuint32_t estr[3] = {1, 1, 1};
    if (d.cuTensorMapEncodeTiled(mr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(rw), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return kCudaErr;
  } else {
    // Router rows [H, E], E contiguous: boxes of 64 experts x 64 K (columns
    // past E and rows past H read as zeros).
    cuuint64_t dims[2] = {cuuint64_t(E), cuuint64_t(H)};
    cuuint64_t strides[1] = {cuuint64_t(E) * 2};
    cuuint32_t box[2] = {64, cuuint32_t(kRtKB)};
    cuuint32_t estr[2] = {1, 1};
    if (d.cuTensorMapEncodeTiled(mr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(rw), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return kCudaErr;
  }
  return kOk;
}

size_t router_smem_bytes() { return 1024 + size_t(kRtStages) * kRtStageBytes + sizeof(RtSmem); }
static_assert(1024 + size_t(kRtStages) * kRtStageBytes + sizeof(RtSmem) <= 227 * 1024, "router smem plan");
static_assert(size_t(kRtTile) * kRtMaxE * 4 <= size_t(kRtStages) * kRtStageBytes, "exchange buffer fits the stages");

template <typename IdT>
int launch_router_cluster(const void* x, int64_t T, int H, const void* rw, int E, int K, void* logits, void* ids,
                          float* vals, int32_t* status_host, int sms, cudaStream_t s) {
  CUtensorMap mx, mr;
  const bool r3d = E % 64 == 0;
  if (encode_router_maps(&mx, &mr, x, T, H, rw, E, r3d) != kOk) return kCudaErr;
  RouterArgs a;
  a.r3d = r3d;
  a.T = T;
  a.H = H;
  a.E = E;
  a.K = K;
  a.kblocks = (H + kRtKB - 1) / kRtKB;
  const int64_t tiles = (T + kRtTile - 1) / kRtTile;
  int S = 1;
  while (S < 8 && tiles * (S * 2) <= sms && S * 2 <= a.kblocks) S *= 2;  // fill the SMs, at most 8 per cluster
  a.S = S;
  a.kb_per = (a.kblocks + S - 1) / S;
  a.n_mma = (E + 15) / 16 * 16;
  int cols = 32;
  while (cols < a.n_mma) cols *= 2;
  a.tmem_cols = cols;
  a.ep = (E + 31) / 32 * 32;
  a.logits = static_cast<__nv_bfloat16*>(logits);
  a.ids = ids;
  a.vals = vals;
  a.status_host = status_host;
  const size_t smem = router_smem_bytes();
  if (cudaFuncSetAttribute(router_kernel<IdT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return kCudaErr;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(S);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(unsigned(tiles * S), 1, 1);
  cfg.blockDim = dim3(kRtThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, router_kernel<IdT>, mx, mr, a) != cudaSuccess) return kCudaErr;
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

// PER = probabilities held per lane (E <= 32 * PER).
template <typename IdT, int PER>
__global__ void __launch_bounds__(kTopkThreads)
    router_topk_kernel(const __nv_bfloat16* __restrict__ logits, int64_t T, int E, int K, IdT* __restrict__ ids,
                       float* __restrict__ vals) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = int64_t(gridDim.x) * kTopkWarps;
  for (int64_t t = int64_t(blockIdx.x) * kTopkWarps + (threadIdx.x >> 5); t < T; t += stride) {
    const __nv_bfloat16* row = logits + t * E;
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? __bfloat162float(row[e]) : -INFINITY;
      m = fmaxf(m, v[j]);
    }
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      v[j] = (lane + 32 * j) < E ? expf(v[j] - m) : 0.f;
      sum += v[j];
    }
    sum = warp_sum(sum);
    // Probabilities are >= 0; -1 marks a slot past E, -2 a slot already taken.
#pragma unroll
    for (int j = 0; j < PER; ++j)
      v[j] = (lane + 32 * j) < E ? __bfloat162float(__float2bfloat16_rn(v[j] / sum)) : -1.f;
    for (int k = 0; k < K; ++k) {
      float best = -3.f;
      int be = INT_MAX;
#pragma unroll
      for (int j = 0; j < PER; ++j) {  // ids ascend with j: a strict > keeps the lowest id of equal values
        if (v[j] > best) {
          best = v[j];
          be = lane + 32 * j;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
#pragma unroll
      for (int j = 0; j < PER; ++j)
        if (lane + 32 * j == be) v[j] = -2.f;
      if (lane == 0) {
        ids[t * K + k] = static_cast<IdT>(be);
        vals[t * K + k] = best;
      }
    }
  }
}

template <typename IdT>
int launch_topk(const __nv_bfloat16* logits, int64_t T, int E, int K, void* ids, float* vals, cudaStream_t s) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  int64_t blocks = (T + kTopkWarps - 1) / kTopkWarps;
  const int64_t cap = int64_t(sms) * 8;
  if (blocks > cap) blocks = cap;
  IdT* out = static_cast<IdT*>(ids);
  const unsigned g = unsigned(blocks);
  if (E <= 32) router_topk_kernel<IdT, 1><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 64) router_topk_kernel<IdT, 2><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 128) router_topk_kernel<IdT, 4><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 256) router_topk_kernel<IdT, 8><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 512) router_topk_kernel<IdT, 16><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else router_topk_kernel<IdT, 32><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_router(const void* x, int64_t T, int32_t H, const void* router_w, int32_t E, int32_t K,
                          void* logits, void* top_idxs, int32_t ids_are_int64, float* top_vals, int32_t* status_host,
                          void* stream) {
  if (T < 0 || T > (int64_t(1) << 30) || H <= 0 || H % 8 || E < 8 || E % 8 || E > kMaxExperts || K < 1 ||
      K > kMaxRouteK || K > E)
    return kBadArg;
  if (T == 0) return kOk;
  if (!x || !router_w || !logits || !top_idxs || !top_vals) return kBadArg;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w) | reinterpret_cast<uintptr_t>(logits)) &
      15)
    return kBadArg;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  if (E <= kRtMaxE)
    return ids_are_int64 ? launch_router_cluster<long long>(x, T, H, router_w, E, K, logits, top_idxs, top_vals,
                                                            status_host, sms, s)
                         : launch_router_cluster<int32_t>(x, T, H, router_w, E, K, logits, top_idxs, top_vals,
                                                          status_host, sms, s);

  moe_ep_layout L;
  if (workspace_layout(1, 1, H, 2, 0, 1, 0, 0, &L) != kOk) return kBadArg;
  if (kPeerTable + L.ctrl_bytes > kCountOffset) return kBadArg;
  uint64_t base = 0;
  if (router_scratch(dev, &base) != kOk) return kCudaErr;
  // The array keeps the previous call's words: zero the control region and
  // set this call's row count, in stream order.
  if (cudaMemsetAsync(reinterpret_cast<void*>(base + kPeerTable), 0, L.ctrl_bytes, s) != cudaSuccess) return kCudaErr;
  int32_t* count = reinterpret_cast<int32_t*>(base + kCountOffset);
  set_count_kernel<<<1, 1, 0, s>>>(count, int32_t(T));
  if (cudaGetLastError() != cudaSuccess) return kCudaErr;

  moe_ep_run_params p = {};
  p.world_size = 1;
  p.rank = 0;
  p.local_experts = 1;
  p.hidden = H;
  p.out_dim = E;
  p.elem_bytes = 2;
  p.gm = T;
  p.tokens = x;
  p.weights = router_w;
  p.recv_counts = count;
  p.out = logits;
  p.peer_bases = reinterpret_cast<const uint64_t*>(base);
  p.local_base = base + kPeerTable;
  p.cap_rows = 0;
  p.push_rows = int32_t(T);
  p.max_chunks = 1;
  p.epoch = 1;
  p.timeout_ns = 1000000000ull;  // one rank: it only waits for itself
  p.status_host = status_host;
  // One expert and few features: spread the rows over every CTA pair
  // (tiles of 16..256 rows, at least one per pair where T allows).
  const int64_t pairs = sms / 2 > 0 ? sms / 2 : 1;
  const int64_t feat_slices = (E + 255) / 256;
  int64_t cap = (T * feat_slices + pairs - 1) / pairs;
  cap = (cap + 15) / 16 * 16;
  FusedMode m;
  m.tile_cap = int(cap < 16 ? 16 : (cap > 256 ? 256 : cap));
  // Every tile reads the same router matrix: start each one at a different
  // k-block so the CTAs do not all request the same lines at once.
  m.kstagger = 1;
  const int rc = launch_fused(&p, m, s);
  if (rc != kOk) return rc;
  const auto* lg = static_cast<const __nv_bfloat16*>(logits);
  return ids_are_int64 ? launch_topk<long long>(lg, T, E, K, top_idxs, top_vals, s)
                       : launch_topk<int32_t>(lg, T, E, K, top_idxs, top_vals, s);
}
