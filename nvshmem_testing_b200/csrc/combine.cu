// Return path, second half: the top-k weighted combine.
//
// The fused kernel in return mode stores every expert output row into the
// return region of the rank that sent the token, at the row the sender's
// padded send buffer holds it in (expert e, bucket row j -> row e*gm + j),
// and releases off_rflag[owner] at every rank when all its rows are out.
// This kernel waits (bounded) for all W flags and forms, per token t,
//   y[t, :] = sum_k top_vals[t, k] * ret[e_k*gm + slots[t, k], :]
// over the distinct valid ids e_k of the row, in fp32, rounded to bf16.
// The reference computes top_vals (utils.py:24-25) but ends its path at the
// expert outputs; the selection rule (a repeated id counts once, ids outside
// [0, E) are skipped) is the routing's (utils.py:31 `.any(-1)`).
//
// One warp per token: the warp reads the token's K ids, weights and slots
// once, compacts the valid entries into shared memory, and then each lane
// streams 16-byte vectors of the K rows (K independent loads in flight per
// vector) and writes one 16-byte vector of y.  HBM-bound: reads
// valid_k * N * 2 bytes and writes N * 2 bytes per token.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "moe_ep.h"
#include "moe_ep_internal.h"
#include "ptx.cuh"

namespace moe {

constexpr int kCombThreads = 256;
constexpr int kCombWarps = kCombThreads / 32;

struct CombineArgs {
  const void* ids;
  const void* vals;
  const int32_t* slots;
  __nv_bfloat16* y;
  const unsigned char* ret;  // this rank's return region [ret_rows][N] bf16
  const uint32_t* rflag;     // [W]
  LocalWords* lw;
  int32_t* status_host;
  int64_t T, gm, ret_rows;
  int K, E, N, W;
  int ids64, vals_bf16;
  uint32_t epoch;
  uint64_t timeout_ns;
};

__device__ void latch_error(const CombineArgs& a, int code, int site, int detail) {
  const uint32_t w = status_word(code, site, detail);
  if (atomicCAS(&a.lw->status, 0u, w) == 0u && a.status_host != nullptr) {
    *reinterpret_cast<volatile int32_t*>(a.status_host) = int32_t(w);
    __threadfence_system();
  }
}

__global__ void __launch_bounds__(kCombThreads) combine_kernel(const CombineArgs a) {
  __shared__ int go;
  __shared__ int64_t rows[kCombWarps][kMaxRouteK];
  __shared__ float wts[kCombWarps][kMaxRouteK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // Nothing was returned if this rank's own fused kernel failed.
    int ok = ld_volatile_u32(&a.lw->status) == 0;
    for (int q = 0; q < a.W && ok; ++q) {
      uint64_t deadline = 0;
      for (uint32_t spin = 0;; ++spin) {
        if (int32_t(ld_acquire_sys(a.rflag + q) - a.epoch) >= 0) break;
        if ((spin & 31) == 31) {
          if (ld_volatile_u32(&a.lw->status) != 0) {  // another CTA gave up
            ok = 0;
            break;
          }
          const uint64_t now = globaltimer_ns();
          if (deadline == 0) deadline = now + a.timeout_ns;
          else if (now > deadline) {
            latch_error(a, kTimeout, kSiteReturn, q);
            ok = 0;
            break;
          }
        }
      }
    }
    go = ok;
  }
  __syncthreads();
  if (!go) return;

  const int nvec = a.N / 8;
  const int64_t stride = int64_t(gridDim.x) * kCombWarps;
  for (int64_t t = int64_t(blockIdx.x) * kCombWarps + warp; t < a.T; t += stride) {
    int e = -1, slot = -1;
    float w = 0.f;
    if (lane < a.K) {
      const int64_t i = t * a.K + lane;
      const long long v = a.ids64 ? static_cast<const long long*>(a.ids)[i]
                                  : static_cast<long long>(static_cast<const int32_t*>(a.ids)[i]);
      e = (v >= 0 && v < a.E) ? int(v) : -1;
      slot = a.slots[i];
      w = a.vals_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.vals)[i])
                      : static_cast<const float*>(a.vals)[i];
    }
    bool dup = false;
    for (int j = 0; j < a.K; ++j) {
      const int ej = __shfl_sync(0xffffffffu, e, j);
      dup |= (j < lane && ej == e);
    }
    const int64_t row = int64_t(e) * a.gm + slot;
    const bool valid = e >= 0 && !dup && slot >= 0 && slot < a.gm && row < a.ret_rows;
    const uint32_t mask = __ballot_sync(0xffffffffu, valid);
    const int nv = __popc(mask);
    if (valid) {
      const int pos = __popc(mask & ((1u << lane) - 1u));
      rows[warp][pos] = row * a.N;
      wts[warp][pos] = w;
    }
    __syncwarp();
    __nv_bfloat16* yt = a.y + t * a.N;
    for (int v = lane; v < nvec; v += 32) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int k0 = 0; k0 < nv; k0 += 4) {
        uint4 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          x[j] = (k0 + j < nv) ? ld_cg_v4(a.ret + (rows[warp][k0 + j] + int64_t(v) * 8) * 2) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float wk = (k0 + j < nv) ? wts[warp][k0 + j] : 0.f;
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x[j]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            acc[2 * i] = fmaf(wk, f.x, acc[2 * i]);
            acc[2 * i + 1] = fmaf(wk, f.y, acc[2 * i + 1]);
          }
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      st_v4(yt + int64_t(v) * 8, o);
    }
    __syncwarp();
  }
}

int launch_combine(const moe_ep_run_params* run, const moe_ep_combine_params* c, const moe_ep_layout& L,
                   cudaStream_t stream) {
  if (run->out_dim % 8) return kBadArg;
  CombineArgs a;
  unsigned char* local = reinterpret_cast<unsigned char*>(run->local_base);
  a.ids = c->top_idxs;
  a.vals = c->top_vals;
  a.slots = c->slots;
  a.y = static_cast<__nv_bfloat16*>(c->y);
  a.ret = local + L.off_ret;
  a.rflag = reinterpret_cast<const uint32_t*>(local + L.off_rflag);
  a.lw = reinterpret_cast<LocalWords*>(local + L.off_local);
  a.status_host = run->status_host;
  a.T = c->T;
  a.gm = run->gm;
  a.ret_rows = c->ret_rows;
  a.K = c->K;
  a.E = run->world_size * run->local_experts;
  a.N = run->out_dim;
  a.W = run->world_size;
  a.ids64 = c->ids_are_int64 != 0;
  a.vals_bf16 = c->vals_are_bf16 != 0;
  a.epoch = run->epoch;
  a.timeout_ns = run->timeout_ns;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  // At least one CTA even without tokens: it still waits for the peers, so
  // the call returns only after every peer is done with this rank's region.
  int64_t blocks = (c->T + kCombWarps - 1) / kCombWarps;
  blocks = blocks < 1 ? 1 : blocks;
  const int64_t cap = int64_t(sms) * 8;
  if (blocks > cap) blocks = cap;
  combine_kernel<<<unsigned(blocks), kCombThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

}  // namespace moe
