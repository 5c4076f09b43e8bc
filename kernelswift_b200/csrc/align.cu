// moe_align_block_size: groups the flat (token, slot) -> expert assignments by
// expert, pads each expert's group to a multiple of block_m and emits the
// per-block expert id. Replaces the per-expert boolean masks of
// kernels/track1-triton/fused_moe/base.py:64-68 with a stable counting sort.
//
// Determinism: an element's slot is its expert's offset + the number of
// elements of the same expert before it in flat order. The rank inside a
// warp comes from __match_any_sync + popc, the rank across warps from a
// per-(warp, expert) count table in shared memory, the rank across chunks
// from an exclusive scan of per-chunk histograms. No atomic decides an
// element's position, so the output is bit-identical run to run.
//
// Paths:
//   numel <= small_max: one CTA does fill + histogram + scan + scatter.
//   otherwise: three launches over chunks of `chunk` ids:
//     hist (per-chunk histogram, sentinel fill) -> scan (one CTA: offsets,
//     expert_ids, num_tokens_post_pad, per-chunk bases) -> scatter.
// moe_align_block_size and moe_fused_experts take the single CTA up to 2048
// ids and chunks of 1024 above (the single CTA handles its ids in 1024-id
// passes of a few block barriers each, so larger problems are faster spread
// over CTAs); moe_align_block_size_noalloc keeps 8192 / 4096, the limits its
// header documents for the static scratch.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace ksw {
namespace {

constexpr int kThreads = 1024;
constexpr int kChunk = 1024;          // ids per CTA on the multi-CTA path
constexpr int64_t kSmallMax = 2048;   // single-CTA path up to this many ids
constexpr int kChunkNoAlloc = 4096;   // the same for moe_align_block_size_noalloc
constexpr int64_t kSmallMaxNoAlloc = 8192;
constexpr int kMaxExperts = 1024;

// Flat ids at or past the valid count are dropped: *valid_dev * mult of the
// numel ids when the caller gives a device-side count (the rows an
// expert-parallel receive buffer actually got this step), else all of them.
__device__ __forceinline__ int64_t valid_ids(int64_t numel, const int32_t* valid_dev, int mult) {
  if (valid_dev == nullptr) return numel;
  const int64_t v = int64_t(max(*valid_dev, 0)) * mult;
  return v < numel ? v : numel;
}

template <typename IdT>
__device__ __forceinline__ int load_id(const IdT* ids, int64_t i, int E) {
  const long long v = static_cast<long long>(ids[i]);
  return (v >= 0 && v < E) ? static_cast<int>(v) : -1;
}

// Exclusive prefix sum across a 1024-thread block. `tmp` holds >= 33 ints.
__device__ __forceinline__ int block_excl_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = tmp[lane];
    int s = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    tmp[lane] = s - w;
    if (lane == 31) tmp[32] = s;
  }
  __syncthreads();
  const int excl = x - v + tmp[warp];
  *total = tmp[32];
  __syncthreads();
  return excl;
}

// Adds ids[base, min(base + 1024, end)) (one per thread) to the expert
// histogram with one shared-memory atomic per distinct expert per warp (the
// warp's lanes with the same expert are grouped by __match_any_sync), instead
// of one per id: with few experts per-id atomics all contend on a handful of
// counters. `base` is the same for every thread of the block.
template <typename IdT>
__device__ __forceinline__ void count_subchunk(const IdT* ids, int64_t base, int64_t end,
                                               int E, int* counts) {
  const int lane = threadIdx.x & 31;
  const int64_t i = base + threadIdx.x;
  const int e = (i < end) ? load_id(ids, i, E) : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  if (e >= 0 && lane == __ffs(peers) - 1) atomicAdd(&counts[e], __popc(peers));
}

// Places ids[base, min(base + 1024, end)) (one per thread) at their final
// slots. running[e] is expert e's next free slot; warp_cnt[32][E] must be
// all zero on entry and is all zero again on exit.
//
// An id's slot = running[e] + (ids of e in the warps before its warp) + (its
// rank among the lanes of its warp with the same expert). The warp leader of
// each expert group stores the group size in warp_cnt[warp][e]; one thread
// per expert then turns its 32-entry column into absolute bases (an
// exclusive scan over the warps, starting at running[e]; loads are issued eight
// at a time, independent of one another), and every id reads its base
// with one shared-memory load. Entries of warps without the expert stay
// zero, and each leader zeroes its own entry after its warp has read it.
// inv (optional) receives each id's slot, -1 for an id outside [0, E).
template <typename IdT>
__device__ __forceinline__ void scatter_subchunk(const IdT* ids, int64_t base,
                                                 int64_t end, int E,
                                                 int* running, int* warp_cnt,
                                                 int32_t* sorted, int32_t* inv) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t i = base + tid;
  const int e = (i < end) ? load_id(ids, i, E) : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & lanemask_lt());
  const bool leader = e >= 0 && lane == __ffs(peers) - 1;
  if (leader) warp_cnt[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int ee = tid; ee < E; ee += kThreads) {
    int s = running[ee];
#pragma unroll
    for (int w0 = 0; w0 < 32; w0 += 8) {
      int c[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) c[u] = warp_cnt[(w0 + u) * E + ee];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (c[u] != 0) warp_cnt[(w0 + u) * E + ee] = s;
        s += c[u];
      }
    }
    running[ee] = s;
  }
  __syncthreads();
  if (e >= 0) {
    const int slot = warp_cnt[warp * E + e] + rank;
    sorted[slot] = static_cast<int32_t>(i);
    if (inv) inv[i] = slot;
  } else if (inv && i < end) {
    inv[i] = -1;
  }
  __syncwarp();
  if (leader) warp_cnt[warp * E + e] = 0;
  __syncthreads();
}

// Writes expert_ids for the blocks of expert `e` (thread e) and -1 for the
// blocks past the padded total.
__device__ __forceinline__ void write_expert_ids(int e, int E, int off,
                                                 int padded, int total, int BM,
                                                 int64_t num_blocks,
                                                 int32_t* expert_ids) {
  if (e < E) {
    for (int b = off / BM; b < (off + padded) / BM; ++b) expert_ids[b] = e;
  }
  for (int64_t b = total / BM + threadIdx.x; b < num_blocks; b += kThreads)
    expert_ids[b] = -1;
}

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    align_small_kernel(const IdT* __restrict__ ids, int64_t numel, int E,
                       int BM, int64_t L, int32_t* __restrict__ sorted,
                       int32_t* __restrict__ expert_ids,
                       int32_t* __restrict__ num_post_pad, const int32_t* valid_dev,
                       int valid_mult, int32_t* __restrict__ inv) {
  pdl_wait();
  pdl_trigger();
  const int64_t nv = valid_ids(numel, valid_dev, valid_mult);
  extern __shared__ int sm[];
  int* counts = sm;                 // E
  int* running = counts + E;        // E
  int* scan_tmp = running + E;      // 64
  int* warp_cnt = scan_tmp + 64;    // 32 * E
  const int tid = threadIdx.x;

  for (int64_t p = tid; p < L; p += kThreads) sorted[p] = static_cast<int32_t>(numel);
  for (int e = tid; e < E; e += kThreads) counts[e] = 0;
  for (int p = tid; p < 32 * E; p += kThreads) warp_cnt[p] = 0;
  __syncthreads();

  for (int64_t base = 0; base < nv; base += kThreads)
    count_subchunk(ids, base, nv, E, counts);
  __syncthreads();

  const int cnt = tid < E ? counts[tid] : 0;
  const int padded = (cnt + BM - 1) / BM * BM;
  int total = 0;
  const int off = block_excl_scan(padded, scan_tmp, &total);
  if (tid < E) running[tid] = off;
  write_expert_ids(tid, E, off, padded, total, BM, L / BM, expert_ids);
  if (tid == 0) *num_post_pad = total;
  __syncthreads();

  for (int64_t base = 0; base < nv; base += kThreads)
    scatter_subchunk(ids, base, nv, E, running, warp_cnt, sorted, inv);
}

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    align_hist_kernel(const IdT* __restrict__ ids, int64_t numel, int E,
                      int64_t L, int chunk, int32_t* __restrict__ sorted,
                      int32_t* __restrict__ chunk_counts, const int32_t* valid_dev,
                      int valid_mult) {
  pdl_wait();
  pdl_trigger();
  const int64_t nv = valid_ids(numel, valid_dev, valid_mult);
  extern __shared__ int sm[];
  int* counts = sm;  // E
  const int tid = threadIdx.x;
  for (int64_t p = int64_t(blockIdx.x) * kThreads + tid; p < L;
       p += int64_t(gridDim.x) * kThreads)
    sorted[p] = static_cast<int32_t>(numel);
  for (int e = tid; e < E; e += kThreads) counts[e] = 0;
  __syncthreads();
  const int64_t begin = int64_t(blockIdx.x) * chunk;
  const int64_t end = min(nv, begin + chunk);
  for (int64_t base = begin; base < end; base += kThreads)
    count_subchunk(ids, base, end, E, counts);
  __syncthreads();
  for (int e = tid; e < E; e += kThreads)
    chunk_counts[int64_t(blockIdx.x) * E + e] = counts[e];
}

// One CTA. chunk_counts[c][e] is replaced by the first slot of chunk c's
// elements of expert e.
__global__ void __launch_bounds__(kThreads)
    align_scan_kernel(int nchunks, int E, int BM, int64_t L,
                      int32_t* __restrict__ chunk_counts,
                      int32_t* __restrict__ expert_ids,
                      int32_t* __restrict__ num_post_pad) {
  pdl_wait();
  pdl_trigger();
  __shared__ int scan_tmp[64];
  const int tid = threadIdx.x;
  int cnt = 0;
  if (tid < E)
    for (int c = 0; c < nchunks; ++c) cnt += chunk_counts[int64_t(c) * E + tid];
  const int padded = (cnt + BM - 1) / BM * BM;
  int total = 0;
  const int off = block_excl_scan(padded, scan_tmp, &total);
  if (tid < E) {
    int run = off;
    for (int c = 0; c < nchunks; ++c) {
      const int v = chunk_counts[int64_t(c) * E + tid];
      chunk_counts[int64_t(c) * E + tid] = run;
      run += v;
    }
  }
  write_expert_ids(tid, E, off, padded, total, BM, L / BM, expert_ids);
  if (tid == 0) *num_post_pad = total;
}

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    align_scatter_kernel(const IdT* __restrict__ ids, int64_t numel, int E, int chunk,
                         const int32_t* __restrict__ chunk_base,
                         int32_t* __restrict__ sorted, const int32_t* valid_dev,
                         int valid_mult, int32_t* __restrict__ inv) {
  pdl_wait();
  pdl_trigger();
  const int64_t nv = valid_ids(numel, valid_dev, valid_mult);
  extern __shared__ int sm[];
  int* running = sm;           // E
  int* warp_cnt = running + E; // 32 * E
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += kThreads)
    running[e] = chunk_base[int64_t(blockIdx.x) * E + e];
  for (int p = tid; p < 32 * E; p += kThreads) warp_cnt[p] = 0;
  __syncthreads();
  const int64_t begin = int64_t(blockIdx.x) * chunk;
  const int64_t end = min(nv, begin + chunk);
  if (begin >= end) return;  // nothing valid in this chunk
  for (int64_t base = begin; base < end; base += kThreads)
    scatter_subchunk(ids, base, end, E, running, warp_cnt, sorted, inv);
}

template <typename IdT>
int launch_align(const IdT* ids, int64_t numel, int E, int BM, int64_t L,
                 int32_t* sorted, int32_t* expert_ids, int32_t* num_post_pad,
                 int32_t* ws, int chunk, int64_t small_max, cudaStream_t s,
                 const int32_t* valid_dev, int valid_mult, int32_t* inv) {
  if (numel <= small_max) {
    const size_t smem = size_t(2 * E + 64 + 32 * E) * sizeof(int);
    auto k = align_small_kernel<IdT>;
    if (smem > 48 * 1024)
      KSW_CUDA(cudaFuncSetAttribute(
          k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    KSW_LAUNCH(k, dim3(1), dim3(kThreads), smem, s, ids, numel, E, BM, L, sorted,
               expert_ids, num_post_pad, valid_dev, valid_mult, inv);
    return MOE_OK;
  }
  const int nchunks = static_cast<int>(ceil_div(numel, chunk));
  KSW_LAUNCH(align_hist_kernel<IdT>, dim3(nchunks), dim3(kThreads),
             size_t(E) * sizeof(int), s, ids, numel, E, L, chunk, sorted, ws, valid_dev,
             valid_mult);
  KSW_LAUNCH(align_scan_kernel, dim3(1), dim3(kThreads), 0, s, nchunks, E, BM, L, ws,
             expert_ids, num_post_pad);
  const size_t smem = size_t(E + 32 * E) * sizeof(int);
  auto k = align_scatter_kernel<IdT>;
  if (smem > 48 * 1024)
    KSW_CUDA(cudaFuncSetAttribute(
        k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  KSW_LAUNCH(k, dim3(nchunks), dim3(kThreads), smem, s, ids, numel, E, chunk,
             static_cast<const int32_t*>(ws), sorted, valid_dev, valid_mult, inv);
  return MOE_OK;
}

size_t workspace_bytes(int64_t numel, int E, int chunk, int64_t small_max) {
  if (numel <= small_max) return 0;
  return align256(size_t(ceil_div(numel, chunk)) * size_t(E) * sizeof(int32_t));
}

// align_launch with the given path thresholds.
int align_launch_cfg(const void* ids, int ids_dtype, int64_t numel, int E, int BM,
                     int32_t* sorted, int32_t* expert_ids, int32_t* num_post_pad,
                     void* workspace, size_t ws_bytes, int chunk, int64_t small_max,
                     cudaStream_t s, const int32_t* valid_dev = nullptr,
                     int valid_mult = 1, int32_t* inv = nullptr) {
  int st = align_validate(numel, E, BM);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(ids_dtype == MOE_DTYPE_I32 || ids_dtype == MOE_DTYPE_I64,
              MOE_ERR_INVALID_ARG, "topk_ids dtype must be int32 or int64");
  KSW_REQUIRE(sorted && expert_ids && num_post_pad, MOE_ERR_INVALID_ARG,
              "null output pointer");
  KSW_REQUIRE(numel == 0 || ids != nullptr, MOE_ERR_INVALID_ARG,
              "null topk_ids");
  const size_t need = workspace_bytes(numel, E, chunk, small_max);
  KSW_REQUIRE(ws_bytes >= need && (need == 0 || workspace != nullptr),
              MOE_ERR_WORKSPACE, "align workspace too small");
  const int64_t L = align_buffer_len(numel, E, BM);
  if (ids_dtype == MOE_DTYPE_I32)
    return launch_align(static_cast<const int32_t*>(ids), numel, E, BM, L,
                        sorted, expert_ids, num_post_pad,
                        static_cast<int32_t*>(workspace), chunk, small_max, s, valid_dev,
                        valid_mult, inv);
  return launch_align(static_cast<const int64_t*>(ids), numel, E, BM, L, sorted,
                      expert_ids, num_post_pad,
                      static_cast<int32_t*>(workspace), chunk, small_max, s, valid_dev,
                      valid_mult, inv);
}

}  // namespace

int64_t align_small_max() { return kSmallMax; }

int64_t align_buffer_len(int64_t numel, int E, int BM) {
  return round_up(numel + int64_t(E) * (BM - 1), BM);
}

size_t align_workspace_bytes(int64_t numel, int E) {
  return workspace_bytes(numel, E, kChunk, kSmallMax);
}

int align_validate(int64_t numel, int E, int BM) {
  KSW_REQUIRE(numel >= 0, MOE_ERR_INVALID_ARG, "numel must be >= 0");
  KSW_REQUIRE(E >= 1 && E <= kMaxExperts, MOE_ERR_UNSUPPORTED,
              "num_experts must be in [1, 1024]");
  KSW_REQUIRE(BM == 16 || BM == 32 || BM == 64 || BM == 128 || BM == 256,
              MOE_ERR_UNSUPPORTED, "block_m must be one of 16/32/64/128/256");
  KSW_REQUIRE(align_buffer_len(numel, E, BM) < (int64_t(1) << 31),
              MOE_ERR_UNSUPPORTED, "numel too large for int32 indices");
  return MOE_OK;
}

int align_launch(const void* ids, int ids_dtype, int64_t numel, int E, int BM,
                 int32_t* sorted, int32_t* expert_ids, int32_t* num_post_pad,
                 void* workspace, size_t ws_bytes, cudaStream_t s, const int32_t* valid_dev,
                 int valid_mult, int32_t* inv) {
  return align_launch_cfg(ids, ids_dtype, numel, E, BM, sorted, expert_ids, num_post_pad,
                          workspace, ws_bytes, kChunk, kSmallMax, s, valid_dev, valid_mult,
                          inv);
}

}  // namespace ksw

extern "C" {

int64_t moe_align_buffer_len(int64_t numel, int num_experts, int block_m) {
  if (numel < 0 || num_experts < 1 || block_m < 1) return -1;
  return ksw::align_buffer_len(numel, num_experts, block_m);
}

int moe_align_workspace_size(int64_t numel, int num_experts, int block_m,
                             size_t* bytes) {
  KSW_REQUIRE(bytes != nullptr, MOE_ERR_INVALID_ARG, "null bytes pointer");
  int st = ksw::align_validate(numel, num_experts, block_m);
  if (st != MOE_OK) return st;
  *bytes = ksw::align_workspace_bytes(numel, num_experts);
  return MOE_OK;
}

int moe_align_block_size(const void* topk_ids, int ids_dtype, int64_t numel,
                         int num_experts, int block_m,
                         int32_t* sorted_token_ids, int32_t* expert_ids,
                         int32_t* num_tokens_post_pad, void* workspace,
                         size_t workspace_bytes, void* stream) {
  int st = ksw::check_device(nullptr);
  if (st != MOE_OK) return st;
  return ksw::align_launch(topk_ids, ids_dtype, numel, num_experts, block_m,
                           sorted_token_ids, expert_ids, num_tokens_post_pad,
                           workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant: moe_align_block_size_noalloc
//
// For callers that cannot allocate device memory: a serving runtime that has
// handed all free HBM to its own pool (KV cache, activations) and gives an
// operator no workspace hook, or a latency-critical path that must not call
// cudaMalloc because it can synchronise the device. The per-chunk histograms
// of the multi-CTA path live in one static device array instead of a caller
// workspace.
//
//   - The array has a fixed size (kNoAllocScratchBytes, 1 MiB) and exists once
//     on every GPU that loads this library, until the process exits.
//   - Host code cannot pass the array's name to a kernel: in host code that
//     name is only a stand-in for the symbol. Its device address is looked up
//     with cudaGetSymbolAddress the first time the entry point runs on a
//     device (with that device current) and cached per device. That first
//     call on each device therefore does the look-up and should come before
//     any stream capture.
//   - Every call on a device shares the array and it keeps the previous
//     call's contents. Nothing in it needs to start at zero: every entry the
//     kernels read is written earlier in the same call. Calls whose work
//     overlaps on the GPU (different streams, no ordering between them) race
//     on the array; order them on one stream or with events.
//   - No cudaMalloc, cudaFree or other allocating call is made.
// ---------------------------------------------------------------------------
namespace ksw {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) int32_t g_align_noalloc_scratch[kNoAllocScratchBytes / 4];

std::mutex g_noalloc_mu;
int32_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the static scratch on the current device.
int noalloc_scratch_address(int32_t** out) {
  int dev = 0;
  KSW_CUDA(cudaGetDevice(&dev));
  KSW_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, MOE_ERR_DEVICE,
              "moe_align_block_size_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    int32_t* ptr = nullptr;
    KSW_CUDA(cudaGetSymbolAddress((void**)&ptr, g_align_noalloc_scratch));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return MOE_OK;
}

}  // namespace
}  // namespace ksw

extern "C" int moe_align_block_size_noalloc(const void* topk_ids, int ids_dtype,
                                            int64_t numel, int num_experts, int block_m,
                                            int32_t* sorted_token_ids, int32_t* expert_ids,
                                            int32_t* num_tokens_post_pad, void* stream) {
  using namespace ksw;
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  st = align_validate(numel, num_experts, block_m);
  if (st != MOE_OK) return st;
  const size_t need = workspace_bytes(numel, num_experts, kChunkNoAlloc, kSmallMaxNoAlloc);
  if (need > kNoAllocScratchBytes)
    return fail(MOE_ERR_UNSUPPORTED,
                "moe_align_block_size_noalloc: this problem needs " + std::to_string(need) +
                    " bytes of scratch but the static scratch holds " +
                    std::to_string(kNoAllocScratchBytes) +
                    " (numel * num_experts too large); use moe_align_block_size with a "
                    "workspace");
  int32_t* scratch = nullptr;
  st = noalloc_scratch_address(&scratch);
  if (st != MOE_OK) return st;
  return align_launch_cfg(topk_ids, ids_dtype, numel, num_experts, block_m, sorted_token_ids,
                          expert_ids, num_tokens_post_pad, scratch, kNoAllocScratchBytes,
                          kChunkNoAlloc, kSmallMaxNoAlloc, static_cast<cudaStream_t>(stream));
}
