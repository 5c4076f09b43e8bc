// Expert-parallel dispatch plan: one launch that turns this rank's routing
// into everything the token exchange needs (replacing a sort, a bincount, two
// gathers and an inverse-permutation scatter of torch ops).
//
// Experts are sharded in contiguous blocks of e_local per rank, so slot r
// (= token * top_k + j) goes to rank dest[r] = topk_ids[r] / e_local; ids
// outside [0, num_experts) go to an extra bucket `world` that is never sent.
// Above 8192 slots moe_ep_plan_ws splits the same sort over CTAs (below).
// The send order is a stable counting sort of the slots by destination:
//   order[p]      = the slot at send position p (slots ascending within a rank)
//   send_eid[p]   = topk_ids[order[p]] - dest * e_local (id local to the rank)
//   inv[r]        = the send position of slot r (-1 for the extra bucket)
//   counts[d]     = slots for rank d, d <= world (counts[world] = invalid ids)
// Positions come from the same warp-match / per-warp-count / running-offset
// scheme as moe_align_block_size, so the plan is deterministic.
#include "common.cuh"

namespace ksw {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxBuckets = 129;  // world <= 128 ranks, plus the invalid bucket

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    ep_plan_kernel(const IdT* __restrict__ ids, int64_t numel, int num_experts, int e_local,
                   int world, int32_t* __restrict__ order, int32_t* __restrict__ send_eid,
                   int32_t* __restrict__ inv, int64_t* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  __shared__ int cnt[kMaxBuckets];
  __shared__ int running[kMaxBuckets];
  __shared__ int warp_cnt[32 * kMaxBuckets];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = world + 1;
  for (int b = tid; b < B; b += kThreads) cnt[b] = 0;
  for (int i = tid; i < 32 * B; i += kThreads) warp_cnt[i] = 0;
  __syncthreads();
  auto bucket_of = [&](int64_t i, int* local) -> int {
    const long long v = static_cast<long long>(ids[i]);
    if (v < 0 || v >= num_experts) {
      *local = -1;
      return world;
    }
    const int d = static_cast<int>(v / e_local);
    *local = static_cast<int>(v - int64_t(d) * e_local);
    return d;
  };
  // histogram with one shared-memory atomic per distinct bucket per warp
  for (int64_t base = 0; base < numel; base += kThreads) {
    const int64_t i = base + tid;
    int loc;
    const int d = i < numel ? bucket_of(i, &loc) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    if (d >= 0 && lane == __ffs(peers) - 1) atomicAdd(&cnt[d], __popc(peers));
  }
  __syncthreads();
  // exclusive scan over the (<= 129) buckets by warp 0..4
  if (tid == 0) {
    int run = 0;
    for (int b = 0; b < B; ++b) {
      running[b] = run;
      run += cnt[b];
    }
  }
  for (int b = tid; b < B; b += kThreads) counts[b] = cnt[b];
  __syncthreads();
  for (int64_t base = 0; base < numel; base += kThreads) {
    const int64_t i = base + tid;
    int loc = -1;
    const int d = i < numel ? bucket_of(i, &loc) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int rank = __popc(peers & lanemask_lt());
    if (d >= 0 && lane == __ffs(peers) - 1) warp_cnt[warp * B + d] = __popc(peers);
    __syncthreads();
    if (d >= 0) {
      int prefix = 0;
      for (int w = 0; w < warp; ++w) prefix += warp_cnt[w * B + d];
      const int pos = running[d] + prefix + rank;
      if (d < world) {
        order[pos] = static_cast<int32_t>(i);
        send_eid[pos] = loc;
        inv[i] = pos;
      } else {
        inv[i] = -1;
      }
    }
    __syncthreads();
    for (int b = tid; b < B; b += kThreads) {
      int s = 0;
      for (int w = 0; w < 32; ++w) {
        s += warp_cnt[w * B + b];
        warp_cnt[w * B + b] = 0;
      }
      running[b] += s;
    }
    __syncthreads();
  }
}

// ---- the same plan over many CTAs (moe_ep_plan_ws, more than kPlanSmallMax
// slots): per-chunk histograms, one scan for the chunk bases, then every
// chunk places its slots from its bases exactly as the single CTA does ----
constexpr int kPlanChunk = 1024;
constexpr int64_t kPlanSmallMax = 8192;

template <typename IdT>
__device__ __forceinline__ int plan_bucket(const IdT* ids, int64_t i, int num_experts,
                                           int e_local, int world, int* local) {
  const long long v = static_cast<long long>(ids[i]);
  if (v < 0 || v >= num_experts) {
    *local = -1;
    return world;
  }
  const int d = static_cast<int>(v / e_local);
  *local = static_cast<int>(v - int64_t(d) * e_local);
  return d;
}

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    ep_plan_hist_kernel(const IdT* __restrict__ ids, int64_t numel, int num_experts,
                        int e_local, int world, int32_t* __restrict__ chunk_counts) {
  pdl_wait();
  pdl_trigger();
  __shared__ int cnt[kMaxBuckets];
  const int tid = threadIdx.x, lane = tid & 31;
  const int B = world + 1;
  for (int b = tid; b < B; b += kThreads) cnt[b] = 0;
  __syncthreads();
  const int64_t begin = int64_t(blockIdx.x) * kPlanChunk;
  const int64_t end = min(numel, begin + kPlanChunk);
  for (int64_t base = begin; base < end; base += kThreads) {
    const int64_t i = base + tid;
    int loc;
    const int d = i < end ? plan_bucket(ids, i, num_experts, e_local, world, &loc) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    if (d >= 0 && lane == __ffs(peers) - 1) atomicAdd(&cnt[d], __popc(peers));
  }
  __syncthreads();
  for (int b = tid; b < B; b += kThreads) chunk_counts[int64_t(blockIdx.x) * B + b] = cnt[b];
}

// One CTA: counts[b] = slots of bucket b; chunk_counts[c][b] becomes the first
// position of chunk c's slots of bucket b.
__global__ void __launch_bounds__(kThreads)
    ep_plan_scan_kernel(int nchunks, int world, int32_t* __restrict__ chunk_counts,
                        int64_t* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  __shared__ int total[kMaxBuckets];
  __shared__ int start[kMaxBuckets];
  const int tid = threadIdx.x;
  const int B = world + 1;
  for (int b = tid; b < B; b += kThreads) {
    int t = 0;
    for (int c = 0; c < nchunks; ++c) t += chunk_counts[int64_t(c) * B + b];
    total[b] = t;
    counts[b] = t;
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int b = 0; b < B; ++b) {
      start[b] = run;
      run += total[b];
    }
  }
  __syncthreads();
  for (int b = tid; b < B; b += kThreads) {
    int run = start[b];
    for (int c = 0; c < nchunks; ++c) {
      const int v = chunk_counts[int64_t(c) * B + b];
      chunk_counts[int64_t(c) * B + b] = run;
      run += v;
    }
  }
}

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    ep_plan_scatter_kernel(const IdT* __restrict__ ids, int64_t numel, int num_experts,
                           int e_local, int world, const int32_t* __restrict__ chunk_base,
                           int32_t* __restrict__ order, int32_t* __restrict__ send_eid,
                           int32_t* __restrict__ inv) {
  pdl_wait();
  pdl_trigger();
  __shared__ int running[kMaxBuckets];
  __shared__ int warp_cnt[32 * kMaxBuckets];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = world + 1;
  for (int b = tid; b < B; b += kThreads) running[b] = chunk_base[int64_t(blockIdx.x) * B + b];
  for (int i = tid; i < 32 * B; i += kThreads) warp_cnt[i] = 0;
  __syncthreads();
  const int64_t begin = int64_t(blockIdx.x) * kPlanChunk;
  const int64_t end = min(numel, begin + kPlanChunk);
  for (int64_t base = begin; base < end; base += kThreads) {
    const int64_t i = base + tid;
    int loc = -1;
    const int d = i < end ? plan_bucket(ids, i, num_experts, e_local, world, &loc) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int rank = __popc(peers & lanemask_lt());
    if (d >= 0 && lane == __ffs(peers) - 1) warp_cnt[warp * B + d] = __popc(peers);
    __syncthreads();
    if (d >= 0) {
      int prefix = 0;
      for (int w = 0; w < warp; ++w) prefix += warp_cnt[w * B + d];
      const int pos = running[d] + prefix + rank;
      if (d < world) {
        order[pos] = static_cast<int32_t>(i);
        send_eid[pos] = loc;
        inv[i] = pos;
      } else {
        inv[i] = -1;
      }
    }
    __syncthreads();
    for (int b = tid; b < B; b += kThreads) {
      int sum = 0;
      for (int w = 0; w < 32; ++w) {
        sum += warp_cnt[w * B + b];
        warp_cnt[w * B + b] = 0;
      }
      running[b] += sum;
    }
    __syncthreads();
  }
}

size_t plan_workspace_bytes(int64_t numel, int world) {
  if (numel <= kPlanSmallMax) return 0;
  return size_t(ceil_div(numel, kPlanChunk)) * size_t(world + 1) * sizeof(int32_t);
}

template <typename IdT>
int launch_plan_multi(const IdT* ids, int64_t numel, int num_experts, int world,
                      int32_t* order, int32_t* send_eid, int32_t* inv, int64_t* counts,
                      int32_t* ws, cudaStream_t s) {
  const int e_local = num_experts / world;
  const int nchunks = int(ceil_div(numel, kPlanChunk));
  KSW_LAUNCH(ep_plan_hist_kernel<IdT>, dim3(nchunks), dim3(kThreads), 0, s, ids, numel,
             num_experts, e_local, world, ws);
  KSW_LAUNCH(ep_plan_scan_kernel, dim3(1), dim3(kThreads), 0, s, nchunks, world, ws, counts);
  KSW_LAUNCH(ep_plan_scatter_kernel<IdT>, dim3(nchunks), dim3(kThreads), 0, s, ids, numel,
             num_experts, e_local, world, static_cast<const int32_t*>(ws), order, send_eid, inv);
  return MOE_OK;
}

}  // namespace
}  // namespace ksw

extern "C" int moe_ep_plan(const void* topk_ids, int ids_dtype, int64_t numel, int num_experts,
                           int world, int32_t* order, int32_t* send_eid, int32_t* inv_index,
                           int64_t* counts, void* stream) {
  using namespace ksw;
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(world >= 1 && world + 1 <= kMaxBuckets, MOE_ERR_UNSUPPORTED,
              "ep_plan: world must be in [1, 128]");
  KSW_REQUIRE(num_experts >= world && num_experts % world == 0, MOE_ERR_INVALID_ARG,
              "ep_plan: num_experts must be a positive multiple of world");
  KSW_REQUIRE(numel >= 0 && numel < (int64_t(1) << 31), MOE_ERR_UNSUPPORTED,
              "ep_plan: numel out of range");
  KSW_REQUIRE(ids_dtype == MOE_DTYPE_I32 || ids_dtype == MOE_DTYPE_I64, MOE_ERR_INVALID_ARG,
              "ep_plan: ids dtype must be int32 or int64");
  KSW_REQUIRE(counts && (numel == 0 || (topk_ids && order && send_eid && inv_index)),
              MOE_ERR_INVALID_ARG, "ep_plan: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int e_local = num_experts / world;
  if (ids_dtype == MOE_DTYPE_I32)
    KSW_LAUNCH(ep_plan_kernel<int32_t>, dim3(1), dim3(kThreads), 0, s,
               static_cast<const int32_t*>(topk_ids), numel, num_experts, e_local, world,
               order, send_eid, inv_index, counts);
  else
    KSW_LAUNCH(ep_plan_kernel<int64_t>, dim3(1), dim3(kThreads), 0, s,
               static_cast<const int64_t*>(topk_ids), numel, num_experts, e_local, world,
               order, send_eid, inv_index, counts);
  return MOE_OK;
}

extern "C" int moe_ep_plan_workspace_size(int64_t numel, int world, size_t* bytes) {
  using namespace ksw;
  KSW_REQUIRE(bytes != nullptr, MOE_ERR_INVALID_ARG, "ep_plan: null bytes pointer");
  KSW_REQUIRE(world >= 1 && world + 1 <= kMaxBuckets, MOE_ERR_UNSUPPORTED,
              "ep_plan: world must be in [1, 128]");
  KSW_REQUIRE(numel >= 0 && numel < (int64_t(1) << 31), MOE_ERR_UNSUPPORTED,
              "ep_plan: numel out of range");
  *bytes = plan_workspace_bytes(numel, world);
  return MOE_OK;
}

extern "C" int moe_ep_plan_ws(const void* topk_ids, int ids_dtype, int64_t numel,
                              int num_experts, int world, int32_t* order, int32_t* send_eid,
                              int32_t* inv_index, int64_t* counts, void* workspace,
                              size_t workspace_bytes, void* stream) {
  using namespace ksw;
  if (numel <= kPlanSmallMax)
    return moe_ep_plan(topk_ids, ids_dtype, numel, num_experts, world, order, send_eid,
                       inv_index, counts, stream);
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(world >= 1 && world + 1 <= kMaxBuckets, MOE_ERR_UNSUPPORTED,
              "ep_plan: world must be in [1, 128]");
  KSW_REQUIRE(num_experts >= world && num_experts % world == 0, MOE_ERR_INVALID_ARG,
              "ep_plan: num_experts must be a positive multiple of world");
  KSW_REQUIRE(numel < (int64_t(1) << 31), MOE_ERR_UNSUPPORTED, "ep_plan: numel out of range");
  KSW_REQUIRE(ids_dtype == MOE_DTYPE_I32 || ids_dtype == MOE_DTYPE_I64, MOE_ERR_INVALID_ARG,
              "ep_plan: ids dtype must be int32 or int64");
  KSW_REQUIRE(counts && topk_ids && order && send_eid && inv_index, MOE_ERR_INVALID_ARG,
              "ep_plan: null pointer");
  const size_t need = plan_workspace_bytes(numel, world);
  KSW_REQUIRE(workspace != nullptr && workspace_bytes >= need, MOE_ERR_WORKSPACE,
              "ep_plan: workspace smaller than moe_ep_plan_workspace_size");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* ws = static_cast<int32_t*>(workspace);
  if (ids_dtype == MOE_DTYPE_I32)
    return launch_plan_multi(static_cast<const int32_t*>(topk_ids), numel, num_experts, world,
                             order, send_eid, inv_index, counts, ws, s);
  return launch_plan_multi(static_cast<const int64_t*>(topk_ids), numel, num_experts, world,
                           order, send_eid, inv_index, counts, ws, s);
}
