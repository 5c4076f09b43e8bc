// Decode path of moe_fused_experts for a handful of routed rows (T*k <= 16,
// 16-bit activations, unquantised weights): the expert MLP of
// kernels/track1-triton/fused_moe/base.py:64-76 as two weight-streaming
// kernels on the CUDA cores instead of align -> gather -> two grouped GEMMs
// -> reduce -> sum. At these sizes every weight element is used by one or
// two rows, so the work is a stream of the hit experts' weights through the
// SMs and the tensor-core path is bound by its fixed costs (seven launches,
// pipeline fill, 128-row tiles that are almost all padding).
//
//   decode_gate_up_kernel  item = (routed slot, one 32-row slice of the
//                          regrouped w13, i.e. 16 gate rows and their 16 up
//                          rows); each warp dots 4 weight rows with the
//                          slot's token row (staged in shared memory), 16
//                          16-byte loads in flight per lane, then SiLU(gate)
//                          * up for 16 act columns, rounded to the activation
//                          dtype. With fp32 router logits it first routes the
//                          item's token itself (routing.cuh: the routing
//                          kernel's code, so the same experts and weights bit
//                          for bit); the CTA holding the first item of a
//                          token writes that token's ids and weights.
//   decode_down_kernel     item = (token, 8 rows of w2): warp j streams slot
//                          j's 8 rows (one contiguous run of its expert) and
//                          dots them with the slot's act row (the token's act
//                          rows are staged); w_j * dot_j is then summed over
//                          the slots in slot order, in fp32.
//
// Both run persistent grids (the CTAs that fit at once walk the items).
// Loads are 16-byte vectors, several in flight per lane. Slots whose id is
// outside [0, E) contribute nothing. Deterministic: fixed reduction order.
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "routing.cuh"

namespace ksw {
namespace {

constexpr int kThreadsDec = 256;
constexpr int kRowsDn = 8;    // w2 rows per down CTA (one per warp)

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& raw, float (&f)[8]) {
  const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int q = 0; q < 8; ++q) f[q] = to_f32(x[q]);
}

template <typename IdT>
__device__ __forceinline__ int valid_expert(const IdT* ids, int64_t r, int E) {
  const long long e = static_cast<long long>(ids[r]);
  return (e >= 0 && e < E) ? static_cast<int>(e) : -1;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Copies `n` 16-bit elements (n % 8 == 0) into shared memory.
template <typename T>
__device__ __forceinline__ void stage_row(T* dst, const T* src, int64_t n) {
  for (int64_t c = threadIdx.x; c < n / 8; c += blockDim.x)
    reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
}

constexpr int kGuRouteMaxE = 256;  // in-kernel routing: 8 logits per lane

// ---------------- gate-up ----------------
// item = (slot, 32-row slice); one CTA per item while they fit, each warp
// dots 4 weight rows with the token row (staged in shared memory), 16
// 16-byte loads in flight per lane. With router logits warp 0 routes the
// item's token first (routing.cuh); the CTA holding slice 0 of a token's
// first slot writes that token's ids and weights.
constexpr int kRowsGuD = 32;

template <typename T, typename IdT, typename Tw>
__global__ void __launch_bounds__(kThreadsDec)
    decode_gate_up_kernel(const T* __restrict__ hidden, const T* __restrict__ w13,
                                 IdT* __restrict__ ids, Tw* __restrict__ weights,
                                 const float* __restrict__ logits, int renorm, int64_t numel,
                                 int top_k, int E, int64_t H, int64_t I, T* __restrict__ act) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint4 smem_dec[];
  T* a = reinterpret_cast<T*>(smem_dec);  // [H] token row of the current slot
  __shared__ float res[kRowsGuD];
  __shared__ int s_sel[64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunks = 2 * I / kRowsGuD;
  int64_t staged = -1;  // token whose row (and routing) is in shared memory
  for (int64_t item = blockIdx.x; item < numel * chunks; item += gridDim.x) {
    const int64_t slot = item / chunks;
    const int64_t chunk = item - slot * chunks;
    const int64_t tok = slot / top_k;
    if (tok != staged) {
      __syncthreads();  // everyone is done with the previous row
      if (logits != nullptr && warp == 0) {
        float sel_w;
        int sel_i;
        route_token_warp<kGuRouteMaxE / 32>(logits + tok * E, E, top_k, renorm, lane, sel_w,
                                            sel_i);
        if (lane < top_k) {
          s_sel[lane] = sel_i;
          if (chunk == 0 && slot == tok * top_k) {
            weights[tok * top_k + lane] = from_f32<Tw>(sel_w);
            ids[tok * top_k + lane] = static_cast<IdT>(sel_i);
          }
        }
      }
      stage_row(a, hidden + tok * H, H);
      staged = tok;
      __syncthreads();
    }
    const int e = logits != nullptr ? s_sel[slot - tok * top_k] : valid_expert(ids, slot, E);
    if (e < 0) continue;  // the act row of a dropped slot is never read
    const T* w = w13 + (int64_t(e) * 2 * I + chunk * kRowsGuD + warp * 4) * H;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // four 256-column steps of the 4 rows per iteration: 16 weight loads in
    // flight per lane
    for (int64_t k0 = int64_t(lane) * 8; k0 < H; k0 += 1024) {
      uint4 wv[4][4];
#pragma unroll
      for (int st = 0; st < 4; ++st)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (k0 + 256 * st < H) wv[st][r] = *reinterpret_cast<const uint4*>(w + r * H + k0 + 256 * st);
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        if (k0 + 256 * st >= H) break;
        float x[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(a + k0 + 256 * st), x);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float f[8];
          unpack8<T>(wv[st][r], f);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[r] = fmaf(f[q], x[q], acc[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float v = warp_sum(acc[r]);
      if (lane == 0) res[warp * 4 + r] = v;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
      const float g = res[threadIdx.x], u = res[16 + threadIdx.x];
      act[slot * I + chunk * 16 + threadIdx.x] = from_f32<T>(g / (1.0f + __expf(-g)) * u);
    }
    __syncthreads();  // res is reused by the next item
  }
}

// item = (token t, kRowsDn consecutive output rows h0 .. h0 + 7). Warp w
// takes the token's slot j = w (and j = w + 8 for top-16): the 8 rows
// w2[e_j][h0 .. h0 + 8) are one contiguous run of 8 * I elements, which the
// warp streams with two 256-column steps of all 8 rows per iteration (16
// sixteen-byte loads in flight per lane), dotting each row with slot j's act
// row (staged in shared memory). The dots go to shared memory and thread r
// sums row r over the slots in slot order, out = sum_j w_j * dot_j, in fp32.
// Per dot the lane sums its columns in order and the warp then reduces, as
// the gate-up kernel does. KMAX >= top_k.
template <typename T, typename IdT, typename Tw, int KMAX>
__global__ void __launch_bounds__(kThreadsDec)
    decode_down_kernel(const T* __restrict__ act, const T* __restrict__ w2,
                       const IdT* __restrict__ ids, const Tw* __restrict__ weights,
                       int64_t T_tokens, int top_k, int E, int64_t H, int64_t I,
                       T* __restrict__ out) {
  constexpr int kWarps = kThreadsDec / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row_blocks = H / kRowsDn;
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint4 smem_dec[];
  T* a = reinterpret_cast<T*>(smem_dec);  // [top_k, I] act rows of the current token
  __shared__ int s_e[KMAX];
  __shared__ float s_dot[KMAX][kRowsDn];
  int64_t staged = -1;
  for (int64_t item = blockIdx.x; item < T_tokens * row_blocks; item += gridDim.x) {
    const int64_t t = item / row_blocks;
    const int64_t h0 = (item - t * row_blocks) * kRowsDn;
    if (t != staged) {
      __syncthreads();
      if (threadIdx.x < KMAX)
        s_e[threadIdx.x] = threadIdx.x < top_k ? valid_expert(ids, t * top_k + threadIdx.x, E) : -1;
      for (int j = 0; j < top_k; ++j)
        if (valid_expert(ids, t * top_k + j, E) >= 0)
          stage_row(a + int64_t(j) * I, act + (t * top_k + j) * I, I);
      staged = t;
      __syncthreads();
    }
    for (int j = warp; j < top_k; j += kWarps) {
      const int e = s_e[j];
      if (e < 0) continue;  // a dropped slot contributes nothing
      const T* base = w2 + (int64_t(e) * H + h0) * I;
      const T* x = a + int64_t(j) * I;
      float acc[kRowsDn];
#pragma unroll
      for (int r = 0; r < kRowsDn; ++r) acc[r] = 0.f;
      for (int64_t k0 = int64_t(lane) * 8; k0 < I; k0 += 512) {
        const bool second = k0 + 256 < I;
        uint4 wv[2][kRowsDn];
#pragma unroll
        for (int r = 0; r < kRowsDn; ++r) {
          wv[0][r] = *reinterpret_cast<const uint4*>(base + r * I + k0);
          if (second) wv[1][r] = *reinterpret_cast<const uint4*>(base + r * I + k0 + 256);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (u == 1 && !second) break;
          float xv[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(x + k0 + 256 * u), xv);
#pragma unroll
          for (int r = 0; r < kRowsDn; ++r) {
            float f[8];
            unpack8<T>(wv[u][r], f);
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[r] = fmaf(f[q], xv[q], acc[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRowsDn; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == 0) s_dot[j][r] = v;
      }
    }
    __syncthreads();
    if (threadIdx.x < kRowsDn) {
      const int r = threadIdx.x;
      float total = 0.f;
      for (int j = 0; j < top_k; ++j)
        if (s_e[j] >= 0) total = fmaf(to_f32(weights[t * top_k + j]), s_dot[j][r], total);
      out[t * H + h0 + r] = from_f32<T>(total);
    }
    __syncthreads();  // s_dot is reused by the next item
  }
}

// CTAs of `kern` that fit on the GPU at once with `smem` bytes of dynamic
// shared memory each: the persistent grid of the decode kernels.
template <typename Kern>
int grid_cap(Kern kern, size_t smem, int64_t* cap) {
  int sms = 148, per_sm = 0;
  int st = check_device(&sms);
  if (st != MOE_OK) return st;
  KSW_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreadsDec, smem));
  *cap = int64_t(sms) * std::max(per_sm, 1);
  return MOE_OK;
}

// Raises a kernel's dynamic shared-memory limit when a launch needs more
// than the default 48 KB (once per size and kernel; the attribute is per
// function and device, and every device here is the same part).
template <typename Kern>
int ensure_smem(Kern k, size_t bytes, std::atomic<size_t>& granted) {
  if (bytes <= 48 * 1024 || bytes <= granted.load(std::memory_order_acquire)) return MOE_OK;
  KSW_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)));
  size_t cur = granted.load();
  while (cur < bytes && !granted.compare_exchange_weak(cur, bytes)) {
  }
  return MOE_OK;
}

template <typename T, typename IdT, typename Tw, int KMAX>
int launch_down(const DecodeArgs& d, cudaStream_t s) {
  const size_t smem = size_t(d.top_k) * size_t(d.I) * sizeof(T);
  auto k = decode_down_kernel<T, IdT, Tw, KMAX>;
  static std::atomic<size_t> granted{0};
  const int st = ensure_smem(k, smem, granted);
  if (st != MOE_OK) return st;
  const int64_t items = d.T * (d.H / kRowsDn);
  int64_t cap = 0;
  const int stc = grid_cap(k, smem, &cap);
  if (stc != MOE_OK) return stc;
  KSW_LAUNCH(k, dim3(unsigned(std::min<int64_t>(items, cap))), dim3(kThreadsDec),
             smem, s, static_cast<const T*>(d.act), static_cast<const T*>(d.w2),
             static_cast<const IdT*>(d.ids), static_cast<const Tw*>(d.weights), d.T, d.top_k,
             d.E, d.H, d.I, static_cast<T*>(d.out));
  return MOE_OK;
}

template <typename T, typename IdT, typename Tw>
int launch_decode(const DecodeArgs& d, int stage, cudaStream_t s) {
  if (stage == 0) {
    KSW_REQUIRE(d.logits == nullptr || d.E <= kGuRouteMaxE, MOE_ERR_UNSUPPORTED,
                "decode path: in-kernel routing takes at most 256 experts");
    const size_t smem = size_t(d.H) * sizeof(T);
    auto k = decode_gate_up_kernel<T, IdT, Tw>;
    static std::atomic<size_t> granted{0};
    const int st = ensure_smem(k, smem, granted);
    if (st != MOE_OK) return st;
    const int64_t items = d.T * d.top_k * (2 * d.I / kRowsGuD);
    int64_t cap = 0;
    const int stc = grid_cap(k, smem, &cap);
    if (stc != MOE_OK) return stc;
    KSW_LAUNCH(k, dim3(unsigned(std::min<int64_t>(items, cap))), dim3(kThreadsDec), smem, s,
               static_cast<const T*>(d.hidden), static_cast<const T*>(d.w13),
               static_cast<IdT*>(const_cast<void*>(d.ids)),
               static_cast<Tw*>(const_cast<void*>(d.weights)),
               static_cast<const float*>(d.logits), d.renorm, d.T * d.top_k, d.top_k, d.E, d.H,
               d.I, static_cast<T*>(d.act));
    return MOE_OK;
  }
  if (d.top_k <= 1) return launch_down<T, IdT, Tw, 1>(d, s);
  if (d.top_k <= 2) return launch_down<T, IdT, Tw, 2>(d, s);
  if (d.top_k <= 4) return launch_down<T, IdT, Tw, 4>(d, s);
  if (d.top_k <= 8) return launch_down<T, IdT, Tw, 8>(d, s);
  return launch_down<T, IdT, Tw, 16>(d, s);
}

template <typename T, typename IdT>
int dispatch_w(const DecodeArgs& d, int stage, cudaStream_t s) {
  switch (d.weights_dtype) {
    case MOE_DTYPE_F32: return launch_decode<T, IdT, float>(d, stage, s);
    case MOE_DTYPE_BF16: return launch_decode<T, IdT, __nv_bfloat16>(d, stage, s);
    case MOE_DTYPE_F16: return launch_decode<T, IdT, __half>(d, stage, s);
    default: return fail(MOE_ERR_UNSUPPORTED, "decode path: weights dtype");
  }
}

}  // namespace

bool decode_path_fits(int64_t T, int top_k, int64_t H, int64_t I, int act_dtype) {
  const int64_t numel = T * top_k;
  // Large experts stream better through the TMA-fed GEMMs (Mixtral-sized
  // experts at T=1: 0.153 ms there against 0.168 ms here); the decode
  // kernels win where the fixed costs dominate (Qwen3-sized experts at T=1:
  // 35 us against 51 us). Split at 256 MB of weights streamed per call.
  const double weight_bytes = double(numel) * 3.0 * double(H) * double(I) * 2.0;
  return numel >= 1 && numel <= kDecodeMaxRows && weight_bytes <= 256.0 * 1024 * 1024 &&
         (act_dtype == MOE_DTYPE_BF16 || act_dtype == MOE_DTYPE_F16) && H % kRowsDn == 0 &&
         H % 8 == 0 && I % 16 == 0 && H * 2 <= 200 * 1024 &&
         int64_t(top_k) * I * 2 <= 200 * 1024;
}

int decode_launch(const DecodeArgs& d, int stage, cudaStream_t s) {
  KSW_REQUIRE(decode_path_fits(d.T, d.top_k, d.H, d.I, d.act_dtype), MOE_ERR_UNSUPPORTED,
              "decode path: problem does not fit");
  const bool i64 = d.ids_dtype == MOE_DTYPE_I64;
  if (d.act_dtype == MOE_DTYPE_BF16)
    return i64 ? dispatch_w<__nv_bfloat16, int64_t>(d, stage, s)
               : dispatch_w<__nv_bfloat16, int32_t>(d, stage, s);
  return i64 ? dispatch_w<__half, int64_t>(d, stage, s) : dispatch_w<__half, int32_t>(d, stage, s);
}

bool decode_path_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_NO_DECODE_PATH");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

}  // namespace ksw
