// Routing kernels: per-expert counts, expert offsets, the stable token
// permutation (and, optionally, each (token, k)'s index inside its bucket, the
// key of the return path), and the padded expert-major pack.
//
// These restate, on the device, the host loop of the reference's router
// post-processing (utils.py:28-69):
//   for ex in range(E): mask = (top_idxs == ex).any(-1); bucket = tokens[mask]
// i.e. a token joins bucket e at most once however often e appears in its
// top-k row, buckets keep ascending token order, ids outside [0, E) never
// match any bucket, and every bucket is zero-padded to gm rows and
// concatenated expert-major.
#include <cuda_runtime.h>
#include <cstdint>

#include "ptx.cuh"
#include "moe_ep_internal.h"

namespace moe {

// One cluster of kRouteCtas CTAs; CTA c routes the contiguous token range
// [c*per, (c+1)*per), so ascending CTA order is ascending token order.  The
// CTAs find where their tokens go in every bucket from each other's
// histograms through distributed shared memory: no global scratch.
constexpr int kRouteCtas = 8;             // a portable cluster size
constexpr int kRouteThreads = 512;        // one token per thread per chunk
constexpr int kRouteWords = kRouteThreads / 32;

template <typename IdT>
__device__ __forceinline__ int load_id(const IdT* ids, int64_t i, int E) {
  const long long v = static_cast<long long>(ids[i]);
  return (v >= 0 && v < E) ? static_cast<int>(v) : -1;
}

__device__ __forceinline__ uint32_t ld_shared_cluster_u32(uint32_t addr_cluster) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr_cluster) : "memory");
  return v;
}

// Block-wide exclusive scan of one int per thread (kRouteThreads threads).
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < kRouteThreads / 32 ? warp_sums[lane] : 0;
    int t = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < kRouteThreads / 32) warp_sums[lane] = t - s;  // exclusive prefix of warp sums
    if (lane == 31) *total = t;
  }
  __syncthreads();
  const int r = x - v + warp_sums[warp];
  __syncthreads();
  return r;
}

// Routing: counts, offsets (exclusive scan), permutation, max, slots.
// Dynamic shared memory per CTA: E * (4 * 4 + 4 * kRouteWords + 2 * kRouteWords)
// bytes.  The chunk bitmap is word-major (bits[w][e]) so that threads walking
// experts touch consecutive banks.
template <typename IdT>
__global__ void __launch_bounds__(kRouteThreads, 1)
    route_kernel(const IdT* __restrict__ ids, int64_t T, int K, int E, int32_t* __restrict__ counts,
                 int32_t* __restrict__ offsets, int32_t* __restrict__ perm, int32_t* __restrict__ slots,
                 int32_t* __restrict__ max_count) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* hist = reinterpret_cast<int*>(smem_raw);                      // [E] this CTA's tokens per expert
  int* off = hist + E;                                               // [E] expert offsets (all tokens)
  int* cursor = off + E;                                             // [E] next slot of this CTA in bucket e
  int* tot = cursor + E;                                             // [E] tokens per expert (all CTAs)
  uint32_t* bits = reinterpret_cast<uint32_t*>(tot + E);             // [kRouteWords][E]
  uint16_t* wpre = reinterpret_cast<uint16_t*>(bits + size_t(E) * kRouteWords);  // [kRouteWords][E]
  __shared__ int warp_sums[32];
  __shared__ int scan_total;

  const int tid = threadIdx.x;
  const int c = int(cluster_ctarank());
  const int64_t per = (T + kRouteCtas - 1) / kRouteCtas;
  const int64_t t_begin = min(T, int64_t(c) * per), t_end = min(T, t_begin + per);
  for (int e = tid; e < E; e += kRouteThreads) hist[e] = 0;
  __syncthreads();

  // Pass 1: this CTA's counts with per-row de-duplication (the reference's
  // .any(-1)): a slot whose id repeats an earlier slot of its row is skipped.
  for (int64_t t = t_begin + tid; t < t_end; t += kRouteThreads) {
    const IdT* row = ids + t * K;
    int seen[kMaxRouteK];
    for (int k = 0; k < K; ++k) {
      const int e = load_id(row, k, E);
      bool dup = false;
      for (int j = 0; j < k; ++j) dup |= (seen[j] == e);
      seen[k] = e;
      if (e >= 0 && !dup) atomicAdd(&hist[e], 1);
    }
  }
  __syncthreads();
  cluster_sync();  // every CTA's histogram is complete and visible to the cluster

  // Per expert: the tokens of all CTAs (tot) and of the CTAs before this one.
  for (int e = tid; e < E; e += kRouteThreads) {
    const uint32_t a = smem_u32(&hist[e]);
    int before = 0, all = 0;
    for (int q = 0; q < kRouteCtas; ++q) {
      const int v = int(ld_shared_cluster_u32(mapa_shared(a, uint32_t(q))));
      before += q < c ? v : 0;
      all += v;
    }
    tot[e] = all;
    cursor[e] = before;
  }
  cluster_sync();  // no CTA reads a peer's histogram after this point
  __syncthreads();

  // Exclusive scan of the totals over experts (in slabs of kRouteThreads).
  int carry = 0, mx = 0;
  for (int base = 0; base < E; base += kRouteThreads) {
    const int e = base + tid;
    const int v = e < E ? tot[e] : 0;
    mx = max(mx, v);
    const int ex = block_exclusive_scan(v, warp_sums, &scan_total);
    if (e < E) {
      off[e] = carry + ex;
      cursor[e] += carry + ex;
      if (c == 0) {
        offsets[e] = carry + ex;
        counts[e] = v;
      }
    }
    carry += scan_total;
    __syncthreads();
  }
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) warp_sums[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0 && c == 0) {
    int m = 0;
    for (int w = 0; w < kRouteThreads / 32; ++w) m = max(m, warp_sums[w]);
    *max_count = m;
    offsets[E] = carry;
  }
  __syncthreads();

  // Pass 2: stable scatter of this CTA's tokens, one chunk of kRouteThreads
  // tokens at a time.  A token's rank inside its bucket is the number of
  // earlier tokens in the chunk holding that expert (popcount of a
  // per-expert bitmap) plus the cursor carried over from earlier chunks and
  // earlier CTAs.
  for (int64_t c0 = t_begin; c0 < t_end; c0 += kRouteThreads) {
    for (int i = tid; i < E * kRouteWords; i += kRouteThreads) bits[i] = 0u;
    __syncthreads();
    const int64_t t = c0 + tid;
    const int w = tid >> 5, b = tid & 31;
    int seen[kMaxRouteK];
    if (t < t_end) {
      const IdT* row = ids + t * K;
      for (int k = 0; k < K; ++k) {
        const int e = load_id(row, k, E);
        seen[k] = e;
        if (e >= 0) atomicOr(&bits[size_t(w) * E + e], 1u << b);
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kRouteThreads) {
      int run = 0;
      for (int j = 0; j < kRouteWords; ++j) {
        wpre[size_t(j) * E + e] = static_cast<uint16_t>(run);
        run += __popc(bits[size_t(j) * E + e]);
      }
    }
    __syncthreads();
    if (t < t_end) {
      const uint32_t below = (1u << b) - 1u;
      for (int k = 0; k < K; ++k) {
        const int e = seen[k];
        bool dup = false;
        for (int j = 0; j < k; ++j) dup |= (seen[j] == e);
        if (e < 0 || dup) {
          if (slots) slots[t * K + k] = -1;
          continue;
        }
        const size_t s = size_t(w) * E + e;
        const int pos = cursor[e] + wpre[s] + __popc(bits[s] & below);
        perm[pos] = static_cast<int32_t>(t);
        if (slots) slots[t * K + k] = pos - off[e];  // index inside bucket e
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kRouteThreads) {
      const size_t s = size_t(kRouteWords - 1) * E + e;
      cursor[e] += wpre[s] + __popc(bits[s]);
    }
    __syncthreads();
  }
}

// Padded expert-major pack: out[e*gm + j] = tokens[perm[offsets[e] + j]] for
// j < counts[e], zero rows for counts[e] <= j < gm.  One warp per output row,
// 16-byte vectors (row bytes must be a multiple of 16).
__global__ void pack_padded_kernel(const uint4* __restrict__ tokens, int64_t row_vecs,
                                   const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
                                   const int32_t* __restrict__ perm, int E, int64_t gm, uint4* __restrict__ out) {
  const int64_t warps_total = int64_t(gridDim.x) * (blockDim.x >> 5);
  const int64_t rows = int64_t(E) * gm;
  const int lane = threadIdx.x & 31;
  for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps_total) {
    const int e = static_cast<int>(r / gm);
    const int64_t j = r - int64_t(e) * gm;
    uint4* dst = out + r * row_vecs;
    if (j < counts[e]) {
      const uint4* src = tokens + int64_t(perm[offsets[e] + j]) * row_vecs;
      for (int64_t v = lane; v < row_vecs; v += 32) dst[v] = ld_nc_v4(src + v);
    } else {
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int64_t v = lane; v < row_vecs; v += 32) dst[v] = z;
    }
  }
}

// Compact expert-major pack (the general all-to-all's send buffer):
// out[r] = tokens[perm[r]] for r < rows (rows = offsets[E]).  One warp per row.
__global__ void pack_compact_kernel(const uint4* __restrict__ tokens, int64_t row_vecs,
                                    const int32_t* __restrict__ perm, int64_t rows, uint4* __restrict__ out) {
  const int64_t warps_total = int64_t(gridDim.x) * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps_total) {
    const uint4* src = tokens + int64_t(perm[r]) * row_vecs;
    uint4* dst = out + r * row_vecs;
    for (int64_t v = lane; v < row_vecs; v += 32) dst[v] = ld_nc_v4(src + v);
  }
}

// n int32 words from src to dst by one warp (dst may be mapped pinned host
// memory: the stores cross PCIe without a copy engine).
__global__ void publish_i32_kernel(const int32_t* __restrict__ src, int64_t n, int32_t* dst) {
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) *reinterpret_cast<volatile int32_t*>(dst + i) = src[i];
  __threadfence_system();
}

int launch_publish_i32(const int32_t* src, int64_t n, int32_t* dst, cudaStream_t stream) {
  if (n == 0) return kOk;
  publish_i32_kernel<<<1, 32, 0, stream>>>(src, n, dst);
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

size_t route_smem_bytes(int E) { return size_t(E) * (4 * 4 + 4 * kRouteWords + 2 * kRouteWords); }

template <typename IdT>
static int launch_route_t(const IdT* ids, int64_t T, int K, int E, int32_t* counts, int32_t* offsets, int32_t* perm,
                          int32_t* slots, int32_t* max_count, cudaStream_t stream) {
  const size_t smem = route_smem_bytes(E);
  if (cudaFuncSetAttribute(route_kernel<IdT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return kCudaErr;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRouteCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(kRouteCtas, 1, 1);
  cfg.blockDim = dim3(kRouteThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, route_kernel<IdT>, ids, T, K, E, counts, offsets, perm, slots, max_count) !=
      cudaSuccess)
    return kCudaErr;
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

int launch_route(const void* ids, int ids_are_int64, int64_t T, int K, int E, int32_t* counts, int32_t* offsets,
                 int32_t* perm, int32_t* slots, int32_t* max_count, cudaStream_t stream) {
  if (ids_are_int64)
    return launch_route_t(static_cast<const long long*>(ids), T, K, E, counts, offsets, perm, slots, max_count, stream);
  return launch_route_t(static_cast<const int32_t*>(ids), T, K, E, counts, offsets, perm, slots, max_count, stream);
}

int launch_pack_padded(const void* tokens, int64_t H, int elem_bytes, const int32_t* counts, const int32_t* offsets,
                       const int32_t* perm, int E, int64_t gm, void* out, int num_sms, cudaStream_t stream) {
  const int64_t row_vecs = H * elem_bytes / 16;
  const int64_t rows = int64_t(E) * gm;
  if (rows == 0) return kOk;
  const int threads = 256;
  int64_t blocks = (rows + (threads / 32) - 1) / (threads / 32);
  const int64_t cap = int64_t(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  pack_padded_kernel<<<int(blocks), threads, 0, stream>>>(static_cast<const uint4*>(tokens), row_vecs, counts,
                                                          offsets, perm, E, gm, static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

int launch_pack_compact(const void* tokens, int64_t H, int elem_bytes, const int32_t* perm, int64_t rows, void* out,
                        int num_sms, cudaStream_t stream) {
  if (rows == 0) return kOk;
  const int64_t row_vecs = H * elem_bytes / 16;
  const int threads = 256;
  int64_t blocks = (rows + (threads / 32) - 1) / (threads / 32);
  const int64_t cap = int64_t(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  pack_compact_kernel<<<int(blocks), threads, 0, stream>>>(static_cast<const uint4*>(tokens), row_vecs, perm, rows,
                                                           static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

}  // namespace moe
