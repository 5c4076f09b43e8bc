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

// ---- the deduplicated plan (moe_ep_plan_dedup): one send row per (token,
// destination rank) holding any of the token's slots. Rows are grouped by
// rank, tokens ascending inside a rank. One CTA per 1024-token chunk: every
// CTA first counts the rows of ALL tokens per rank (the ids are a few hundred
// KB, read from L2), keeping apart the counts of the chunks before its own;
// its rows for rank d then start at (rows of ranks < d) + (rows of rank d in
// earlier chunks), and a token's position inside the chunk is the ballot
// count of earlier lanes in its warp plus the totals of earlier warps. No
// atomic decides a position, so the plan is deterministic, and it is the
// same whatever the number of CTAs. ----
constexpr int kDedupMaxWorld = 32;

__device__ __forceinline__ float weight_as_f32(const void* w, int dtype, int64_t i) {
  if (dtype == MOE_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]);
  if (dtype == MOE_DTYPE_F16) return __half2float(static_cast<const __half*>(w)[i]);
  return static_cast<const float*>(w)[i];
}

// Bit d of the result: the token has a slot on rank d; bit `world`: it has a
// slot whose id is outside [0, num_experts).
template <typename IdT>
__device__ __forceinline__ uint64_t token_ranks(const IdT* ids, int64_t t, int k, int E,
                                                int e_local, int world) {
  uint64_t m = 0;
  for (int j = 0; j < k; ++j) {
    const long long v = static_cast<long long>(ids[t * k + j]);
    m |= (v >= 0 && v < E) ? (uint64_t(1) << (v / e_local)) : (uint64_t(1) << world);
  }
  return m;
}

template <typename IdT>
__global__ void __launch_bounds__(kThreads)
    ep_plan_dedup_kernel(const IdT* __restrict__ ids, const void* __restrict__ w, int w_dtype,
                         int64_t T, int k, int E, int e_local, int world,
                         int32_t* __restrict__ send_token, int32_t* __restrict__ send_eid,
                         float* __restrict__ send_w, int32_t* __restrict__ inv,
                         int64_t* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  __shared__ int cnt[kDedupMaxWorld + 1];
  __shared__ int pre[kDedupMaxWorld];
  __shared__ int running[kDedupMaxWorld];
  __shared__ int warp_tot[32][kDedupMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t my_base = int64_t(blockIdx.x) * kThreads;
  if (tid <= world) cnt[tid] = 0;
  if (tid < world) pre[tid] = 0;
  __syncthreads();
  // pass 1 (every CTA, all tokens): rows per rank, tokens with an invalid
  // slot, and the rows of the chunks before this CTA's
  for (int64_t base = 0; base < T; base += kThreads) {
    const int64_t t = base + tid;
    const uint64_t m = t < T ? token_ranks(ids, t, k, E, e_local, world) : 0;
    for (int d = 0; d <= world; ++d) {
      const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
      if (lane == 0 && b) {
        atomicAdd(&cnt[d], __popc(b));
        if (base < my_base && d < world) atomicAdd(&pre[d], __popc(b));
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int d = 0; d < world; ++d) {
      running[d] = run + pre[d];
      run += cnt[d];
    }
  }
  if (blockIdx.x == 0 && tid <= world) counts[tid] = cnt[tid];
  __syncthreads();
  // pass 2: placement of this CTA's chunk
  const int64_t t = my_base + tid;
  const uint64_t m = t < T ? token_ranks(ids, t, k, E, e_local, world) : 0;
  for (int d = 0; d < world; ++d) {
    const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
    if (lane == 0) warp_tot[warp][d] = __popc(b);
  }
  __syncthreads();
  for (int d = 0; d < world; ++d) {  // warp-uniform: every lane takes each ballot
    const bool on = (m >> d) & 1u;
    const unsigned b = __ballot_sync(0xffffffffu, on);
    if (t >= T) continue;
    if (!on) {
      inv[t * world + d] = -1;
      continue;
    }
    int prefix = 0;
    for (int w2 = 0; w2 < warp; ++w2) prefix += warp_tot[w2][d];
    const int pos = running[d] + prefix + __popc(b & lanemask_lt());
    send_token[pos] = static_cast<int32_t>(t);
    inv[t * world + d] = pos;
    for (int j = 0; j < k; ++j) {
      const long long v = static_cast<long long>(ids[t * k + j]);
      const bool here = v >= 0 && v < E && v / e_local == d;
      send_eid[int64_t(pos) * k + j] = here ? static_cast<int32_t>(v - int64_t(d) * e_local) : -1;
      send_w[int64_t(pos) * k + j] = here ? weight_as_f32(w, w_dtype, t * k + j) : 0.0f;
    }
  }
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

extern "C" int moe_ep_plan_dedup(const void* topk_ids, int ids_dtype, const void* topk_weights,
                                 int weights_dtype, int64_t num_tokens, int top_k,
                                 int num_experts, int world, int32_t* send_token,
                                 int32_t* send_eid, float* send_w, int32_t* inv_index,
                                 int64_t* counts, void* stream) {
  using namespace ksw;
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(world >= 1 && world <= kDedupMaxWorld, MOE_ERR_UNSUPPORTED,
              "ep_plan_dedup: world must be in [1, 32]");
  KSW_REQUIRE(num_experts >= world && num_experts % world == 0, MOE_ERR_INVALID_ARG,
              "ep_plan_dedup: num_experts must be a positive multiple of world");
  KSW_REQUIRE(top_k >= 1 && top_k <= 64, MOE_ERR_INVALID_ARG, "ep_plan_dedup: top_k in [1, 64]");
  KSW_REQUIRE(num_tokens >= 0 && num_tokens * world < (int64_t(1) << 31), MOE_ERR_UNSUPPORTED,
              "ep_plan_dedup: num_tokens out of range");
  KSW_REQUIRE(ids_dtype == MOE_DTYPE_I32 || ids_dtype == MOE_DTYPE_I64, MOE_ERR_INVALID_ARG,
              "ep_plan_dedup: ids dtype must be int32 or int64");
  KSW_REQUIRE(weights_dtype == MOE_DTYPE_F32 || weights_dtype == MOE_DTYPE_BF16 ||
                  weights_dtype == MOE_DTYPE_F16,
              MOE_ERR_INVALID_ARG, "ep_plan_dedup: weights must be f32, bf16 or f16");
  KSW_REQUIRE(counts && (num_tokens == 0 || (topk_ids && topk_weights && send_token &&
                                             send_eid && send_w && inv_index)),
              MOE_ERR_INVALID_ARG, "ep_plan_dedup: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int e_local = num_experts / world;
  const dim3 grid(unsigned(std::max<int64_t>(1, ceil_div(num_tokens, int64_t(kThreads)))));
  if (ids_dtype == MOE_DTYPE_I32)
    KSW_LAUNCH(ep_plan_dedup_kernel<int32_t>, grid, dim3(kThreads), 0, s,
               static_cast<const int32_t*>(topk_ids), topk_weights, weights_dtype, num_tokens,
               top_k, num_experts, e_local, world, send_token, send_eid, send_w, inv_index,
               counts);
  else
    KSW_LAUNCH(ep_plan_dedup_kernel<int64_t>, grid, dim3(kThreads), 0, s,
               static_cast<const int64_t*>(topk_ids), topk_weights, weights_dtype, num_tokens,
               top_k, num_experts, e_local, world, send_token, send_eid, send_w, inv_index,
               counts);
  return MOE_OK;
}
