// Expert parallelism over NVLink peer memory: token dispatch and result
// combine as kernels that store into / load from the other GPUs' buffers
// (mapped with CUDA IPC), with per-rank flags for the hand-offs instead of a
// host-synchronised collective. A token goes to a rank once, however many of
// its k slots that rank holds (moe_ep_plan_dedup): its row carries the k
// expert ids local to that rank (-1 for slots held elsewhere) and their
// weights, the receiving rank returns one weighted row (the sum over its
// slots), and the source adds the rows of the ranks it used.
//
// Buffer of one rank (identical layout on every rank; capacity = token rows):
//   [ctrl: EpCtrl, 4 KB][recv ids: capacity x k int32][recv weights:
//    capacity x k f32][recv rows: capacity x H][result rows: capacity x H]
//
// One step, epoch e = ctrl.epoch + 1 (ctrl.epoch counts finished steps and
// is advanced on the device by the last kernel of the step; the host keeps
// no per-step state):
//   dispatch  CTA 0 writes this rank's per-destination row counts into row
//             `me` of every rank's counts matrix, then arrive[me] = e on every
//             rank. Every CTA waits for arrive[s] >= e from all ranks (this
//             also means every rank finished step e-1, so the buffers are
//             free), derives from the counts matrix where its rows go
//             (dst_off[d] = rows that lower ranks send to d), and copies its
//             rows, ids and weights into the destination buffers; ctrl.n_recv
//             = the rows this rank receives. The last CTA to finish sets
//             sent[me] = e on every rank and waits for sent[s] >= e from all.
//   experts   moe_fused_experts over the first n_recv received rows (the
//             caller's launch, with num_tokens_dev = &ctrl.n_recv): result
//             row i = sum_j w[i, j] * expert_{ids[i, j]}(row i)
//   combine   one CTA sets done[me] = e on every rank; the combine CTAs wait
//             for done[d] >= e from all ranks, then out[t] = the sum over the
//             ranks d that got token t, in rank order, of d's result row; a
//             last kernel sets ctrl.epoch = e.
// Stores that publish data are followed by a system-scope fence and a
// release store of the flag; flags are read with acquire loads. Every wait
// is bounded (5 s of %globaltimer by default); on expiry the kernel records
// MOE_ERR_TIMEOUT and skips its work instead of hanging.
#include <cstring>

#include "common.cuh"

struct moe_ep_peer {
  int world = 0, rank = 0, device = 0, top_k = 0;
  int64_t capacity = 0, hidden = 0;
  int act_dtype = 0, esize = 2;
  size_t bytes = 0;
  char* base = nullptr;                      // this rank's buffer
  char* peers[MOE_EP_MAX_RANKS] = {};        // every rank's buffer in this address space
  bool opened[MOE_EP_MAX_RANKS] = {};
  bool connected = false;
  uint64_t wait_limit_ns = 0;
};

namespace ksw {
namespace {

constexpr int kMaxRanks = MOE_EP_MAX_RANKS;
constexpr size_t kCtrlBytes = 4096;
constexpr int kThreadsEp = 256;

struct EpCtrl {
  uint32_t epoch;     // finished steps (local)
  uint32_t cta_done;  // dispatch CTAs finished this step (local)
  int32_t n_recv;     // token rows received this step (local; the expert pass's count)
  uint32_t dispatched;  // last step whose dispatch offsets are valid (local)
  uint32_t arrive[kMaxRanks];  // [s]: last step rank s started (written by s)
  uint32_t sent[kMaxRanks];    // [s]: last step whose rows s delivered here
  uint32_t done[kMaxRanks];    // [s]: last step whose result rows s finished
  int32_t counts[kMaxRanks][kMaxRanks];  // [s][d]: rows rank s sends to d
  int32_t dst_off[kMaxRanks];            // local: first row of mine in d's buffer
  int32_t send_start[kMaxRanks + 1];     // local: prefix sums of my counts
};
static_assert(sizeof(EpCtrl) <= kCtrlBytes, "control block");

struct EpView {
  char* base[kMaxRanks];
  int world, me, top_k;
  int64_t capacity, hidden;
  int esize;
  int64_t off_ids, off_w, off_recv, off_res;
  uint64_t wait_limit_ns;
};

__device__ __forceinline__ EpCtrl* ctrl_of(const EpView& v, int r) {
  return reinterpret_cast<EpCtrl*>(v.base[r]);
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t x;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(x) : "l"(p) : "memory");
  return x;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t x) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(x) : "memory");
}

// Waits until flags[s] >= e for every rank s (wrap-around ignored: 2^32
// steps). One thread calls it; returns false after the wait limit.
__device__ bool wait_flags(const uint32_t* flags, int world, uint32_t e, uint64_t limit) {
  const uint64_t t0 = globaltimer_ns();
  for (int s = 0; s < world; ++s) {
    while (ld_acquire_sys(flags + s) < e) {
      if (globaltimer_ns() - t0 > limit) return false;
    }
  }
  return true;
}

// The counts matrix is written by other GPUs during the kernel that reads
// it: read it past the (non-coherent) L1.
__device__ __forceinline__ int32_t count_of(const EpCtrl* c, int s, int d) {
  return *reinterpret_cast<const volatile int32_t*>(&c->counts[s][d]);
}

__device__ __forceinline__ int bucket_of(const int32_t* start, int world, int64_t p) {
  int d = 0;
  while (d + 1 < world && p >= start[d + 1]) ++d;
  return d;
}

// ---------------- dispatch ----------------
__global__ void __launch_bounds__(kThreadsEp)
    ep_dispatch_kernel(EpView v, const uint8_t* __restrict__ hidden,
                       const int32_t* __restrict__ send_token,
                       const int32_t* __restrict__ send_eid, const float* __restrict__ send_w,
                       const int64_t* __restrict__ counts, int32_t* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok;
  __shared__ int32_t s_dst_off[kMaxRanks];
  __shared__ int32_t s_start[kMaxRanks + 1];
  __shared__ int32_t s_dok[kMaxRanks];  // rank d can take all rows sent to it
  EpCtrl* my = ctrl_of(v, v.me);
  const uint32_t e = my->epoch + 1;
  const int tid = threadIdx.x;

  if (blockIdx.x == 0) {
    // publish my counts row to every rank, then my arrival
    if (tid < v.world * v.world) {
      const int p = tid / v.world, d = tid % v.world;
      ctrl_of(v, p)->counts[v.me][d] = static_cast<int32_t>(counts[d]);
    }
    __syncthreads();
    __threadfence_system();
    __syncthreads();
    if (tid < v.world) st_release_sys(&ctrl_of(v, tid)->arrive[v.me], e);
  }
  if (tid == 0) {
    const bool ok = wait_flags(my->arrive, v.world, e, v.wait_limit_ns);
    if (!ok) report_status(status, MOE_ERR_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;

  // offsets from the counts matrix (now complete on this rank)
  if (tid == 0) {
    int32_t run = 0;
    for (int d = 0; d < v.world; ++d) {
      s_start[d] = run;
      run += count_of(my, v.me, d);
      int32_t off = 0, total = 0;
      for (int s = 0; s < v.world; ++s) {
        const int32_t c = count_of(my, s, d);
        if (s < v.me) off += c;
        total += c;
      }
      s_dst_off[d] = off;
      // a destination that would overflow reports it itself; its senders
      // skip their rows for it
      s_dok[d] = total <= v.capacity;
    }
    s_start[v.world] = run;
    int32_t n_recv = 0;
    for (int s = 0; s < v.world; ++s) n_recv += count_of(my, s, v.me);
    if (n_recv > v.capacity) report_status(status, MOE_ERR_WORKSPACE);
    if (blockIdx.x == 0) {
      // the expert pass reads this many rows; after an overflow (reported
      // above, its senders skipped their rows) it reads none
      my->n_recv = n_recv <= v.capacity ? n_recv : 0;
      for (int d = 0; d <= v.world; ++d) my->send_start[d] = s_start[d];
      for (int d = 0; d < v.world; ++d) my->dst_off[d] = s_dst_off[d];
      my->dispatched = e;  // combine reads the offsets only for this step
    }
  }
  __syncthreads();

  // copy rows: one warp per send position, 16-byte vectors
  const int warp = tid >> 5, lane = tid & 31;
  const int64_t n_send = s_start[v.world];
  const int64_t row_bytes = v.hidden * v.esize;
  for (int64_t p = int64_t(blockIdx.x) * (kThreadsEp / 32) + warp; p < n_send;
       p += int64_t(gridDim.x) * (kThreadsEp / 32)) {
    const int d = bucket_of(s_start, v.world, p);
    if (!s_dok[d]) continue;
    const int64_t dst = int64_t(s_dst_off[d]) + (p - s_start[d]);
    const int64_t src_row = send_token[p];
    const uint4* src = reinterpret_cast<const uint4*>(hidden + src_row * row_bytes);
    uint4* out = reinterpret_cast<uint4*>(v.base[d] + v.off_recv + dst * row_bytes);
    const int64_t nvec = row_bytes / 16;
    // four 16-byte loads in flight per lane before the (remote) stores
    for (int64_t c0 = lane; c0 < nvec; c0 += 4 * 32) {
      uint4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u * 32 < nvec) x[u] = src[c0 + u * 32];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u * 32 < nvec) out[c0 + u * 32] = x[u];
    }
    // the row's k local ids and weights
    for (int j = lane; j < v.top_k; j += 32) {
      reinterpret_cast<int32_t*>(v.base[d] + v.off_ids)[dst * v.top_k + j] =
          send_eid[p * v.top_k + j];
      reinterpret_cast<float*>(v.base[d] + v.off_w)[dst * v.top_k + j] = send_w[p * v.top_k + j];
    }
  }

  // the last CTA publishes "sent" and waits for every rank's rows
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&my->cta_done, 1u);
    if (prev == gridDim.x - 1) {
      my->cta_done = 0;
      __threadfence_system();
      for (int d = 0; d < v.world; ++d) st_release_sys(&ctrl_of(v, d)->sent[v.me], e);
      if (!wait_flags(my->sent, v.world, e, v.wait_limit_ns))
        report_status(status, MOE_ERR_TIMEOUT);
    }
  }
}

// ---------------- combine ----------------
__global__ void ep_signal_done_kernel(EpView v) {
  pdl_wait();
  pdl_trigger();
  EpCtrl* my = ctrl_of(v, v.me);
  const uint32_t e = my->epoch + 1;
  __threadfence_system();
  if (threadIdx.x < v.world) st_release_sys(&ctrl_of(v, threadIdx.x)->done[v.me], e);
}

// out[t] = sum over ranks d (ascending) of d's result row for token t, for
// the ranks the token was sent to (inv[t * world + d] >= 0), in fp32.
template <typename T>
__global__ void __launch_bounds__(kThreadsEp)
    ep_combine_kernel(EpView v, const int32_t* __restrict__ inv, int64_t T_tokens,
                      T* __restrict__ out, int32_t* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok;
  __shared__ int32_t s_dst_off[kMaxRanks];
  __shared__ int32_t s_start[kMaxRanks + 1];
  EpCtrl* my = ctrl_of(v, v.me);
  const uint32_t e = my->epoch + 1;
  if (threadIdx.x == 0) {
    // this rank's dispatch of the step must have completed its offsets
    bool ok = my->dispatched == e;
    if (ok) ok = wait_flags(my->done, v.world, e, v.wait_limit_ns);
    if (!ok) report_status(status, MOE_ERR_TIMEOUT);
    s_ok = ok;
    for (int d = 0; d < v.world; ++d) s_dst_off[d] = my->dst_off[d];
    for (int d = 0; d <= v.world; ++d) s_start[d] = my->send_start[d];
  }
  __syncthreads();
  if (!s_ok) return;
  const int64_t vec_per_row = v.hidden / 8;
  const int64_t total = T_tokens * vec_per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int64_t h = (i - t * vec_per_row) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // up to four ranks' rows in flight before the adds
    for (int d0 = 0; d0 < v.world; d0 += 4) {
      float val[4][8];
      bool on[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = d0 + u;
        int64_t row = -1;
        if (d < v.world) {
          const int p = __ldg(inv + t * v.world + d);
          if (p >= s_start[d] && p < s_start[d + 1]) row = int64_t(s_dst_off[d]) + (p - s_start[d]);
        }
        on[u] = row >= 0 && row < v.capacity;
        if (on[u]) {
          const T* src = reinterpret_cast<const T*>(v.base[d] + v.off_res) + row * v.hidden + h;
          const uint4 raw = *reinterpret_cast<const uint4*>(src);
          const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int q = 0; q < 8; ++q) val[u][q] = to_f32(x[q]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (on[u]) {
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += val[u][q];
        }
    }
    uint4 packed;
    uint32_t* pk = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
    for (int q = 0; q < 4; ++q) pk[q] = pack2<T>(acc[2 * q], acc[2 * q + 1]);
    *reinterpret_cast<uint4*>(out + t * v.hidden + h) = packed;
  }
}

__global__ void ep_step_end_kernel(EpView v) {
  pdl_wait();
  pdl_trigger();
  EpCtrl* my = ctrl_of(v, v.me);
  my->epoch = my->epoch + 1;
}

int esize_of(int dtype) {
  return (dtype == MOE_DTYPE_BF16 || dtype == MOE_DTYPE_F16) ? 2 : 0;
}

void layout(int64_t capacity, int64_t hidden, int esize, int top_k, int64_t* off_ids,
            int64_t* off_w, int64_t* off_recv, int64_t* off_res, size_t* total) {
  *off_ids = kCtrlBytes;
  *off_w = *off_ids + int64_t(align256(size_t(capacity) * top_k * 4));
  *off_recv = *off_w + int64_t(align256(size_t(capacity) * top_k * 4));
  const int64_t rows = int64_t(align256(size_t(capacity * hidden * esize)));
  *off_res = *off_recv + rows;
  *total = size_t(*off_res + rows);
}

EpView view_of(const moe_ep_peer* ep) {
  EpView v{};
  for (int r = 0; r < ep->world; ++r) v.base[r] = ep->peers[r];
  v.world = ep->world;
  v.me = ep->rank;
  v.top_k = ep->top_k;
  v.capacity = ep->capacity;
  v.hidden = ep->hidden;
  v.esize = ep->esize;
  size_t total;
  layout(ep->capacity, ep->hidden, ep->esize, ep->top_k, &v.off_ids, &v.off_w, &v.off_recv,
         &v.off_res, &total);
  v.wait_limit_ns = ep->wait_limit_ns;
  return v;
}

int check_ep(const moe_ep_peer* ep) {
  KSW_REQUIRE(ep != nullptr, MOE_ERR_INVALID_ARG, "ep_peer: null handle");
  KSW_REQUIRE(ep->connected, MOE_ERR_INVALID_ARG, "ep_peer: not connected");
  int dev = 0;
  KSW_CUDA(cudaGetDevice(&dev));
  KSW_REQUIRE(dev == ep->device, MOE_ERR_INVALID_ARG,
              "ep_peer: the current device is not the one the buffer was created on");
  return MOE_OK;
}

}  // namespace
}  // namespace ksw

extern "C" int moe_ep_peer_create(int world, int rank, int64_t capacity, int64_t hidden_size,
                                  int top_k, int act_dtype, int wait_limit_ms,
                                  moe_ep_peer_t** out, void* handle_out) {
  using namespace ksw;
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(out && handle_out, MOE_ERR_INVALID_ARG, "ep_peer_create: null pointer");
  KSW_REQUIRE(world >= 2 && world <= kMaxRanks && rank >= 0 && rank < world,
              MOE_ERR_UNSUPPORTED, "ep_peer_create: world must be in [2, 8], rank in [0, world)");
  KSW_REQUIRE(top_k >= 1 && top_k <= 64, MOE_ERR_INVALID_ARG,
              "ep_peer_create: top_k must be in [1, 64]");
  KSW_REQUIRE(capacity >= 1 && capacity * top_k < (int64_t(1) << 31), MOE_ERR_INVALID_ARG,
              "ep_peer_create: capacity out of range");
  KSW_REQUIRE(hidden_size > 0 && hidden_size % 8 == 0, MOE_ERR_UNSUPPORTED,
              "ep_peer_create: hidden_size must be a positive multiple of 8");
  const int es = esize_of(act_dtype);
  KSW_REQUIRE(es == 2, MOE_ERR_UNSUPPORTED, "ep_peer_create: act dtype must be f16 or bf16");
  KSW_REQUIRE(wait_limit_ms >= 0 && wait_limit_ms <= 600000, MOE_ERR_INVALID_ARG,
              "ep_peer_create: wait_limit_ms must be in [0, 600000]");
  auto* ep = new moe_ep_peer();
  ep->world = world;
  ep->rank = rank;
  ep->top_k = top_k;
  ep->capacity = capacity;
  ep->hidden = hidden_size;
  ep->act_dtype = act_dtype;
  ep->esize = es;
  ep->wait_limit_ns = uint64_t(wait_limit_ms > 0 ? wait_limit_ms : 5000) * 1000000ull;
  int64_t a, b, c, d;
  layout(capacity, hidden_size, es, top_k, &a, &b, &c, &d, &ep->bytes);
  cudaError_t err = cudaGetDevice(&ep->device);
  if (err == cudaSuccess) err = cudaMalloc(&ep->base, ep->bytes);
  if (err == cudaSuccess) err = cudaMemset(ep->base, 0, kCtrlBytes);
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, ep->base);
  if (err != cudaSuccess) {
    if (ep->base) cudaFree(ep->base);
    delete ep;
    return check_cuda(err, "moe_ep_peer_create");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == MOE_EP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  ep->peers[rank] = ep->base;
  *out = ep;
  return MOE_OK;
}

extern "C" int moe_ep_peer_connect(moe_ep_peer_t* ep, const void* handles) {
  using namespace ksw;
  KSW_REQUIRE(ep && handles, MOE_ERR_INVALID_ARG, "ep_peer_connect: null pointer");
  KSW_REQUIRE(!ep->connected, MOE_ERR_INVALID_ARG, "ep_peer_connect: already connected");
  const auto* hs = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < ep->world; ++r) {
    if (r == ep->rank) continue;
    void* p = nullptr;
    cudaError_t err = cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (ep->opened[q]) {
          cudaIpcCloseMemHandle(ep->peers[q]);
          ep->opened[q] = false;
          ep->peers[q] = nullptr;
        }
      return check_cuda(err, "cudaIpcOpenMemHandle");
    }
    ep->peers[r] = static_cast<char*>(p);
    ep->opened[r] = true;
  }
  ep->connected = true;
  return MOE_OK;
}

extern "C" int moe_ep_peer_buffers(const moe_ep_peer_t* ep, void** recv_rows,
                                   int32_t** recv_ids, float** recv_weights, void** result_rows,
                                   int32_t** recv_count) {
  using namespace ksw;
  KSW_REQUIRE(ep != nullptr, MOE_ERR_INVALID_ARG, "ep_peer_buffers: null handle");
  int64_t a, b, c, d;
  size_t total;
  layout(ep->capacity, ep->hidden, ep->esize, ep->top_k, &a, &b, &c, &d, &total);
  if (recv_ids) *recv_ids = reinterpret_cast<int32_t*>(ep->base + a);
  if (recv_weights) *recv_weights = reinterpret_cast<float*>(ep->base + b);
  if (recv_rows) *recv_rows = ep->base + c;
  if (result_rows) *result_rows = ep->base + d;
  if (recv_count) *recv_count = &reinterpret_cast<EpCtrl*>(ep->base)->n_recv;
  return MOE_OK;
}

extern "C" int moe_ep_peer_dispatch(moe_ep_peer_t* ep, const void* hidden, int64_t num_tokens,
                                    const int32_t* send_token, const int32_t* send_eid,
                                    const float* send_w, const int64_t* counts, int32_t* status,
                                    void* stream) {
  using namespace ksw;
  int st = check_ep(ep);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(num_tokens >= 0, MOE_ERR_INVALID_ARG, "ep_peer_dispatch: bad sizes");
  KSW_REQUIRE(counts && (num_tokens == 0 || (hidden && send_token && send_eid && send_w)),
              MOE_ERR_INVALID_ARG, "ep_peer_dispatch: null pointer");
  KSW_REQUIRE(aligned16(hidden), MOE_ERR_INVALID_ARG,
              "ep_peer_dispatch: hidden must be 16-byte aligned");
  // at most one row per (token, rank)
  const int64_t max_rows = num_tokens * ep->world;
  const int64_t rows_per_cta = kThreadsEp / 32;
  const int grid = int(std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(std::max<int64_t>(max_rows, 1), rows_per_cta), 148 * 4)));
  KSW_LAUNCH(ep_dispatch_kernel, dim3(grid), dim3(kThreadsEp), 0,
             static_cast<cudaStream_t>(stream), view_of(ep),
             static_cast<const uint8_t*>(hidden), send_token, send_eid, send_w, counts, status);
  return MOE_OK;
}

extern "C" int moe_ep_peer_combine(moe_ep_peer_t* ep, const int32_t* inv_index,
                                   int64_t num_tokens, void* out, int32_t* status,
                                   void* stream) {
  using namespace ksw;
  int st = check_ep(ep);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(num_tokens >= 0, MOE_ERR_INVALID_ARG, "ep_peer_combine: bad sizes");
  KSW_REQUIRE(num_tokens == 0 || (inv_index && out), MOE_ERR_INVALID_ARG,
              "ep_peer_combine: null pointer");
  KSW_REQUIRE(aligned16(out), MOE_ERR_INVALID_ARG, "ep_peer_combine: out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const EpView v = view_of(ep);
  KSW_LAUNCH(ep_signal_done_kernel, dim3(1), dim3(32), 0, s, v);
  const int64_t total = num_tokens * (ep->hidden / 8);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, kThreadsEp),
                                                              148 * 8)));
  if (ep->act_dtype == MOE_DTYPE_BF16)
    KSW_LAUNCH(ep_combine_kernel<__nv_bfloat16>, dim3(grid), dim3(kThreadsEp), 0, s, v,
               inv_index, num_tokens, static_cast<__nv_bfloat16*>(out), status);
  else
    KSW_LAUNCH(ep_combine_kernel<__half>, dim3(grid), dim3(kThreadsEp), 0, s, v, inv_index,
               num_tokens, static_cast<__half*>(out), status);
  KSW_LAUNCH(ep_step_end_kernel, dim3(1), dim3(1), 0, s, v);
  return MOE_OK;
}

extern "C" int moe_ep_peer_disconnect(moe_ep_peer_t* ep) {
  using namespace ksw;
  KSW_REQUIRE(ep != nullptr, MOE_ERR_INVALID_ARG, "ep_peer_disconnect: null handle");
  int dev = 0;
  KSW_CUDA(cudaGetDevice(&dev));
  if (dev != ep->device) KSW_CUDA(cudaSetDevice(ep->device));
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < ep->world; ++r)
    if (ep->opened[r]) {
      const cudaError_t e = cudaIpcCloseMemHandle(ep->peers[r]);
      if (first == cudaSuccess) first = e;
      ep->opened[r] = false;
      ep->peers[r] = nullptr;
    }
  ep->connected = false;
  if (dev != ep->device) cudaSetDevice(dev);
  return check_cuda(first, "cudaIpcCloseMemHandle");
}

extern "C" int moe_ep_peer_destroy(moe_ep_peer_t* ep) {
  using namespace ksw;
  if (ep == nullptr) return MOE_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != ep->device) cudaSetDevice(ep->device);
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < ep->world; ++r)
    if (ep->opened[r]) {
      const cudaError_t e = cudaIpcCloseMemHandle(ep->peers[r]);
      if (first == cudaSuccess) first = e;
    }
  if (ep->base) {
    const cudaError_t e = cudaFree(ep->base);
    if (first == cudaSuccess) first = e;
  }
  if (dev != ep->device) cudaSetDevice(dev);
  delete ep;
  return check_cuda(first, "moe_ep_peer_destroy");
}
