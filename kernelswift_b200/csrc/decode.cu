// Decode path of moe_fused_experts for a handful of routed rows (T*k <= 16,
// 16-bit activations, unquantised weights): the expert MLP of
// kernels/track1-triton/fused_moe/base.py:64-76 as two weight-streaming
// kernels on the CUDA cores instead of align -> gather -> two grouped GEMMs
// -> reduce -> sum. At these sizes every weight element is used by one or
// two rows, so the work is a stream of the hit experts' weights through the
// SMs and the tensor-core path is bound by its fixed costs (seven launches,
// pipeline fill, 128-row tiles that are almost all padding).
//
//   decode_gate_up_kernel  CTA = (routed slot, 32 rows of the regrouped w13):
//                          16 gate rows and their 16 up rows; each warp dots
//                          4 weight rows with the slot's token row (staged in
//                          shared memory), then SiLU(gate) * up for 16 act
//                          columns, rounded to the activation dtype
//   decode_down_kernel     CTA = (token, 8 rows of w2): each warp dots one
//                          w2 row of every slot's expert with that slot's act
//                          row (all of the token's act rows staged) and sums
//                          w_j * dot_j over the slots in slot order, in fp32
//
// Loads are 16-byte vectors, several in flight per lane. Slots whose id is
// outside [0, E) contribute nothing. Deterministic: fixed reduction order.
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace ksw {
namespace {

constexpr int kThreadsDec = 256;
constexpr int kRowsGu = 32;   // w13 rows per gate-up CTA (one 32-row regroup slice)
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

template <typename T, typename IdT>
__global__ void __launch_bounds__(kThreadsDec)
    decode_gate_up_kernel(const T* __restrict__ hidden, const T* __restrict__ w13,
                          const IdT* __restrict__ ids, int top_k, int E, int64_t H, int64_t I,
                          T* __restrict__ act) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint4 smem_dec[];
  T* a = reinterpret_cast<T*>(smem_dec);  // [H] token row
  __shared__ float res[kRowsGu];
  const int64_t chunks = 2 * I / kRowsGu;
  const int64_t slot = blockIdx.x / chunks;
  const int64_t chunk = blockIdx.x - slot * chunks;
  const int e = valid_expert(ids, slot, E);
  if (e < 0) return;  // the act row of a dropped slot is never read
  stage_row(a, hidden + (slot / top_k) * H, H);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* w = w13 + (int64_t(e) * 2 * I + chunk * kRowsGu + warp * 4) * H;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // two 256-column steps per iteration: 8 weight loads in flight per lane
  for (int64_t k0 = int64_t(lane) * 8; k0 < H; k0 += 512) {
    uint4 wv[2][4];
    const bool second = k0 + 256 < H;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      wv[0][r] = *reinterpret_cast<const uint4*>(w + r * H + k0);
      if (second) wv[1][r] = *reinterpret_cast<const uint4*>(w + r * H + k0 + 256);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (s == 1 && !second) break;
      float x[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(a + k0 + 256 * s), x);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float f[8];
        unpack8<T>(wv[s][r], f);
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
  // rows 0-15 of the slice are gate rows, 16-31 the matching up rows
  if (threadIdx.x < 16) {
    const float g = res[threadIdx.x], u = res[16 + threadIdx.x];
    act[slot * I + chunk * 16 + threadIdx.x] = from_f32<T>(g / (1.0f + __expf(-g)) * u);
  }
}

template <typename T, typename IdT, typename Tw>
__global__ void __launch_bounds__(kThreadsDec)
    decode_down_kernel(const T* __restrict__ act, const T* __restrict__ w2,
                       const IdT* __restrict__ ids, const Tw* __restrict__ weights, int top_k,
                       int E, int64_t H, int64_t I, T* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint4 smem_dec[];
  T* a = reinterpret_cast<T*>(smem_dec);  // [top_k, I] the token's act rows
  const int64_t row_blocks = H / kRowsDn;
  const int64_t t = blockIdx.x / row_blocks;
  const int64_t h0 = (blockIdx.x - t * row_blocks) * kRowsDn;
  for (int j = 0; j < top_k; ++j)
    if (valid_expert(ids, t * top_k + j, E) >= 0)
      stage_row(a + int64_t(j) * I, act + (t * top_k + j) * I, I);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t h = h0 + warp;
  float total = 0.f;
  for (int j = 0; j < top_k; ++j) {
    const int e = valid_expert(ids, t * top_k + j, E);
    if (e < 0) continue;
    const T* w = w2 + (int64_t(e) * H + h) * I;
    const T* x = a + int64_t(j) * I;
    float acc = 0.f;
    for (int64_t k0 = int64_t(lane) * 8; k0 < I; k0 += 4 * 256) {
      uint4 wv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (k0 + u * 256 < I) wv[u] = *reinterpret_cast<const uint4*>(w + k0 + u * 256);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (k0 + u * 256 >= I) break;
        float f[8], xv[8];
        unpack8<T>(wv[u], f);
        unpack8<T>(*reinterpret_cast<const uint4*>(x + k0 + u * 256), xv);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc = fmaf(f[q], xv[q], acc);
      }
    }
    acc = warp_sum(acc);
    total = fmaf(to_f32(weights[t * top_k + j]), acc, total);
  }
  if (lane == 0) out[t * H + h] = from_f32<T>(total);
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

template <typename T, typename IdT, typename Tw>
int launch_decode(const DecodeArgs& d, int stage, cudaStream_t s) {
  if (stage == 0) {
    const size_t smem = size_t(d.H) * sizeof(T);
    auto k = decode_gate_up_kernel<T, IdT>;
    static std::atomic<size_t> granted{0};
    const int st = ensure_smem(k, smem, granted);
    if (st != MOE_OK) return st;
    KSW_LAUNCH(k, dim3(unsigned(d.T * d.top_k * (2 * d.I / kRowsGu))), dim3(kThreadsDec), smem,
               s, static_cast<const T*>(d.hidden), static_cast<const T*>(d.w13),
               static_cast<const IdT*>(d.ids), d.top_k, d.E, d.H, d.I, static_cast<T*>(d.act));
    return MOE_OK;
  }
  const size_t smem = size_t(d.top_k) * size_t(d.I) * sizeof(T);
  auto k = decode_down_kernel<T, IdT, Tw>;
  static std::atomic<size_t> granted{0};
  const int st = ensure_smem(k, smem, granted);
  if (st != MOE_OK) return st;
  KSW_LAUNCH(k, dim3(unsigned(d.T * (d.H / kRowsDn))), dim3(kThreadsDec), smem, s,
             static_cast<const T*>(d.act), static_cast<const T*>(d.w2),
             static_cast<const IdT*>(d.ids), static_cast<const Tw*>(d.weights), d.top_k, d.E,
             d.H, d.I, static_cast<T*>(d.out));
  return MOE_OK;
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
  return numel >= 1 && numel <= kDecodeMaxRows &&
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
