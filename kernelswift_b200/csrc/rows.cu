// Row-wise kernels around the grouped GEMMs (all HBM-bound, one warp per row):
//   gather_rows: A[m] = hidden[sorted_ids[m] / top_k] in expert-sorted order
//                (the replicate + boolean gather of base.py:52-58,68), with
//                an optional cast (f32 -> bf16) or quantisation (e4m3 per
//                128-column group with an fp32 or a power-of-two scale, int8
//                per row). Given the align's slot map, moe_fused_experts
//                gathers token by token instead (gather_tokens_kernel: each
//                source row read and converted once, stored into its top_k
//                operand rows).
//   quant_rows:  the same quantisations for the gate-up output (the second
//                GEMM's operand).
//   sum_topk:    out[t] = sum_s sum_j part[s, t*k + j] (the top-k reduction of
//                base.py:75-76), in fixed order, fp32, then cast.
#include <type_traits>

#include "common.cuh"
#include "rows.h"

namespace ksw {
namespace {

constexpr int kWarps = 8;  // rows per CTA
constexpr int kBatch = 4;  // loads in flight per lane in the row loops
constexpr float kInt8Max = 127.0f;

// Loads 8 consecutive elements as floats (16-byte aligned source).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p,
                                                     float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p,
                                                      const float (&v)[8]) {
  uint4 o;
  o.x = pack2<__nv_bfloat16>(v[0], v[1]);
  o.y = pack2<__nv_bfloat16>(v[2], v[3]);
  o.z = pack2<__nv_bfloat16>(v[4], v[5]);
  o.w = pack2<__nv_bfloat16>(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = o;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  uint4 o;
  o.x = pack2<__half>(v[0], v[1]);
  o.y = pack2<__half>(v[2], v[3]);
  o.z = pack2<__half>(v[4], v[5]);
  o.w = pack2<__half>(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = o;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Activation quantisation arithmetic (the oracle's quant_fp8_group /
// quant_int8_rows restate it): scale = absmax / qmax (1 when the group is all
// zero), inv = 1 / scale (one IEEE division per group),
// q = clamp(x * inv, -qmax, qmax) rounded to nearest-even in the target
// format. Multiplying by the reciprocal keeps the per-element work to a
// multiply, a clamp and a conversion, which these HBM-bound kernels need.
__device__ __forceinline__ float quant_scale(float absmax, float qmax) {
  const float s = absmax / qmax;
  return s > 0.0f ? s : 1.0f;
}

__device__ __forceinline__ int8_t to_i8(float x, float inv) {
  const float q = fminf(fmaxf(x * inv, -kInt8Max), kInt8Max);
  return static_cast<int8_t>(__float2int_rn(q));
}

// Source row of operand row m, or -1 for a padding slot. top_k == 0 maps a
// valid row to itself (quantising an operand that is already in sorted order).
__device__ __forceinline__ int64_t source_row(const int32_t* sorted, int64_t m,
                                              int64_t numel, int top_k) {
  const int r = __ldg(sorted + m);
  if (r >= numel) return -1;
  return top_k > 0 ? int64_t(r / top_k) : m;
}

// ---------------- plain gather (+ cast) ----------------
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kWarps * 32)
    gather_cast_kernel(const Tin* __restrict__ src, int64_t H, int top_k,
                       const int32_t* __restrict__ sorted,
                       const int32_t* __restrict__ num_post_pad, int64_t max_rows,
                       int64_t numel, int64_t src_rows, Tout* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = min(int64_t(__ldg(num_post_pad)), max_rows);
  for (int64_t m = int64_t(blockIdx.x) * kWarps + warp; m < rows;
       m += int64_t(gridDim.x) * kWarps) {
    const int64_t sr = source_row(sorted, m, numel, top_k);
    if (sr < 0 || sr >= src_rows) continue;
    const Tin* s = src + sr * H;
    Tout* d = dst + m * H;
    // kBatch 16-byte loads in flight per lane before the stores
    for (int64_t h0 = int64_t(lane) * 8; h0 < H; h0 += kBatch * 256) {
      float v[kBatch][8];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (h0 + u * 256 < H) load8(s + h0 + u * 256, v[u]);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if constexpr (std::is_same<Tout, float>::value) {
          // fp32 operand rows of the tf32 GEMMs: rounded to tf32 here
#pragma unroll
          for (int i = 0; i < 8; ++i) v[u][i] = round_tf32(v[u][i]);
        }
        if (h0 + u * 256 < H) store8(d + h0 + u * 256, v[u]);
      }
    }
  }
}

// ---------------- gather + e4m3 per (row, 128 columns) ----------------
// Each lane handles 8 consecutive columns (one 16-byte load for 16-bit
// sources); 16 lanes cover one 128-column group, so the group's absmax is a
// 16-lane shuffle reduction. Requires H % 8 == 0 (checked on the host); a
// partial last group is handled by masking lanes past H (pack_e4m3x8 is in
// common.cuh, shared with the UE8M0 gate-up epilogue).

template <typename Tin>
__global__ void __launch_bounds__(kWarps * 32)
    gather_fp8_kernel(const Tin* __restrict__ src, int64_t H, int top_k,
                      const int32_t* __restrict__ sorted,
                      const int32_t* __restrict__ num_post_pad, int64_t max_rows,
                      int64_t numel, int64_t src_rows, uint8_t* __restrict__ dst,
                      float* __restrict__ scale) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = min(int64_t(__ldg(num_post_pad)), max_rows);
  const int64_t groups = (H + 127) / 128;
  for (int64_t m = int64_t(blockIdx.x) * kWarps + warp; m < rows;
       m += int64_t(gridDim.x) * kWarps) {
    const int64_t sr = sorted ? source_row(sorted, m, numel, top_k) : m;
    if (sr < 0 || sr >= src_rows) continue;
    const Tin* s = src + sr * H;
    // two groups per warp step: lanes 0-15 group g, lanes 16-31 group g+1;
    // kBatch steps' loads are issued before any of them is quantised
    for (int64_t gb = 0; gb < groups; gb += 2 * kBatch) {
      float v[kBatch][8];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t g = gb + 2 * u + (lane >> 4);
        const int64_t h = g * 128 + (lane & 15) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
        if (g < groups && h < H) load8(s + h, v[u]);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t g = gb + 2 * u + (lane >> 4);
        const int64_t h = g * 128 + (lane & 15) * 8;
        const bool in = g < groups && h < H;
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[u][i]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1)
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float sc = quant_scale(amax, kFp8Max);
        const float inv = 1.0f / sc;
        if (in) *reinterpret_cast<uint2*>(dst + m * H + h) = pack_e4m3x8(v[u], inv);
        if (in && (lane & 15) == 0) scale[m * groups + g] = sc;
      }
    }
  }
}

// ---------------- gather + e4m3 with UE8M0 scales per (row, 128 columns) ---
// The gather_fp8_kernel scheme with a power-of-two scale per group (H % 128
// == 0): the scale byte goes into the scale-factor image of the operand rows
// (row_slices = max_rows / 128 chunks per 4 column groups).
template <typename Tin>
__global__ void __launch_bounds__(kWarps * 32)
    gather_ue8m0_kernel(const Tin* __restrict__ src, int64_t H, int top_k,
                        const int32_t* __restrict__ sorted,
                        const int32_t* __restrict__ num_post_pad, int64_t max_rows,
                        int64_t numel, int64_t src_rows, uint8_t* __restrict__ dst,
                        uint8_t* __restrict__ sf, int64_t q_blocks, int64_t row_slices) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = min(int64_t(__ldg(num_post_pad)), max_rows);
  const int64_t groups = H / 128;
  for (int64_t m = int64_t(blockIdx.x) * kWarps + warp; m < rows;
       m += int64_t(gridDim.x) * kWarps) {
    const int64_t sr = sorted ? source_row(sorted, m, numel, top_k) : m;
    if (sr < 0 || sr >= src_rows) continue;
    const Tin* s = src + sr * H + (lane & 15) * 8;
    uint8_t* d = dst + m * H + (lane & 15) * 8;
    // this row's bytes in the image: group g at sf_row + (g / 4) * q_stride + g % 4
    // (the sf_image_offset layout)
    uint8_t* sf_row = sf + (m >> 7) * 512 + 16 * (m & 31) + 4 * ((m & 127) >> 5);
    const int64_t q_stride = row_slices * 512;
    for (int64_t gb = 0; gb < groups; gb += 2 * kBatch) {
      float v[kBatch][8];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t g = gb + 2 * u + (lane >> 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
        if (g < groups) load8(s + g * 128, v[u]);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t g = gb + 2 * u + (lane >> 4);
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[u][i]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1)
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const uint32_t b = ue8m0_byte(amax);
        const float inv = ue8m0_inv_scale(b);
        if (g < groups) {
          *reinterpret_cast<uint2*>(d + g * 128) = pack_e4m3x8(v[u], inv);
          if ((lane & 15) == 0) sf_row[(g >> 2) * q_stride + (g & 3)] = static_cast<uint8_t>(b);
        }
      }
    }
  }
}

// ---------------- token-major gather ----------------
// The rows of the three kernels above, visited from the source side. With
// the align's slot map (inv[t * top_k + j] = operand row of token t's slot
// j, -1 for a dropped slot) one warp reads a 1024-column chunk of a token
// once, converts or quantises it once, and stores the result into each of
// the token's top_k operand rows: the source is read, and the e4m3
// arithmetic done, once per token instead of once per routed row. Lane
// geometry and per-element arithmetic are the row-major kernels' (pass u
// covers columns c0 + 256 u + 8 lane; in fp8 modes lanes 0-15 and 16-31
// hold two 128-column groups), so the operand rows and scales written are
// the same bytes. Needs top_k <= 32 (one slot position per lane).
enum { kTokCast = 0, kTokFp8 = 1, kTokUe8m0 = 2 };

template <int MODE, typename Tin, typename Tout>
__global__ void __launch_bounds__(kWarps * 32)
    gather_tokens_kernel(const Tin* __restrict__ src, int64_t H, int top_k,
                         const int32_t* __restrict__ inv,
                         const int32_t* __restrict__ src_count, int64_t src_rows,
                         int64_t max_rows, Tout* __restrict__ dst, void* __restrict__ scale,
                         int64_t row_slices) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tokens = src_count ? min(int64_t(__ldg(src_count)), src_rows) : src_rows;
  constexpr int64_t kCols = kBatch * 256;
  const int64_t chunks = (H + kCols - 1) / kCols;
  const int64_t groups = (H + 127) / 128;
  const int64_t q_stride = row_slices * 512;
  for (int64_t task = int64_t(blockIdx.x) * kWarps + warp; task < tokens * chunks;
       task += int64_t(gridDim.x) * kWarps) {
    const int64_t t = task / chunks;
    const int64_t c0 = (task - t * chunks) * kCols;
    const int my_pos = lane < top_k ? __ldg(inv + t * top_k + lane) : -1;
    const Tin* s = src + t * H;
    float v[kBatch][8];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t h = c0 + u * 256 + lane * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
      if (h < H) load8(s + h, v[u]);
    }
    // converted once: 16-bit rows packed, fp32 rows rounded to tf32, fp8
    // rows packed to e4m3 with their group scale
    uint4 packed[kBatch];
    float sc[kBatch];
    uint32_t sb[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if constexpr (MODE == kTokCast) {
        if constexpr (std::is_same<Tout, float>::value) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[u][i] = round_tf32(v[u][i]);
        } else {
          packed[u] = make_uint4(pack2<Tout>(v[u][0], v[u][1]), pack2<Tout>(v[u][2], v[u][3]),
                                 pack2<Tout>(v[u][4], v[u][5]), pack2<Tout>(v[u][6], v[u][7]));
        }
      } else {
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[u][i]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1)
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        float inv_s;
        if constexpr (MODE == kTokFp8) {
          sc[u] = quant_scale(amax, kFp8Max);
          inv_s = 1.0f / sc[u];
        } else {
          sb[u] = ue8m0_byte(amax);
          inv_s = ue8m0_inv_scale(sb[u]);
        }
        const uint2 q = pack_e4m3x8(v[u], inv_s);
        packed[u] = make_uint4(q.x, q.y, 0u, 0u);
      }
    }
    for (int j = 0; j < top_k; ++j) {
      const int64_t m = __shfl_sync(0xffffffffu, my_pos, j);
      if (m < 0 || m >= max_rows) continue;  // dropped slot (warp-uniform)
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t h = c0 + u * 256 + lane * 8;
        if (h >= H) continue;
        if constexpr (MODE == kTokCast) {
          Tout* d = dst + m * H + h;
          if constexpr (std::is_same<Tout, float>::value) {
            reinterpret_cast<float4*>(d)[0] = make_float4(v[u][0], v[u][1], v[u][2], v[u][3]);
            reinterpret_cast<float4*>(d)[1] = make_float4(v[u][4], v[u][5], v[u][6], v[u][7]);
          } else {
            *reinterpret_cast<uint4*>(d) = packed[u];
          }
        } else {
          uint8_t* d = reinterpret_cast<uint8_t*>(dst) + m * H + h;
          *reinterpret_cast<uint2*>(d) = make_uint2(packed[u].x, packed[u].y);
          if ((lane & 15) == 0) {
            const int64_t g = (c0 + u * 256) / 128 + (lane >> 4);
            if constexpr (MODE == kTokFp8) {
              static_cast<float*>(scale)[m * groups + g] = sc[u];
            } else {
              uint8_t* sf_row = static_cast<uint8_t*>(scale) + (m >> 7) * 512 +
                                16 * (m & 31) + 4 * ((m & 127) >> 5);
              sf_row[(g >> 2) * q_stride + (g & 3)] = static_cast<uint8_t>(sb[u]);
            }
          }
        }
      }
    }
  }
}

// ---------------- gather + int8 per row ----------------
template <typename Tin>
__global__ void __launch_bounds__(kWarps * 32)
    gather_i8_kernel(const Tin* __restrict__ src, int64_t H, int top_k,
                     const int32_t* __restrict__ sorted,
                     const int32_t* __restrict__ num_post_pad, int64_t max_rows,
                     int64_t numel, int64_t src_rows, int8_t* __restrict__ dst,
                     float* __restrict__ scale) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = min(int64_t(__ldg(num_post_pad)), max_rows);
  for (int64_t m = int64_t(blockIdx.x) * kWarps + warp; m < rows;
       m += int64_t(gridDim.x) * kWarps) {
    const int64_t sr = sorted ? source_row(sorted, m, numel, top_k) : m;
    if (sr < 0 || sr >= src_rows) continue;
    const Tin* s = src + sr * H;
    float amax = 0.0f;
    for (int64_t h0 = int64_t(lane) * 8; h0 < H; h0 += kBatch * 256) {
      float v[kBatch][8];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
        if (h0 + u * 256 < H) load8(s + h0 + u * 256, v[u]);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[u][i]));
    }
    amax = warp_max(amax);
    const float sc = quant_scale(amax, kInt8Max);
    const float inv = 1.0f / sc;
    for (int64_t h0 = int64_t(lane) * 8; h0 < H; h0 += kBatch * 256) {
      float v[kBatch][8];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (h0 + u * 256 < H) load8(s + h0 + u * 256, v[u]);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t h = h0 + u * 256;
        if (h >= H) continue;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lo |= uint32_t(uint8_t(to_i8(v[u][i], inv))) << (8 * i);
          hi |= uint32_t(uint8_t(to_i8(v[u][4 + i], inv))) << (8 * i);
        }
        *reinterpret_cast<uint2*>(dst + m * H + h) = make_uint2(lo, hi);
      }
    }
    if (lane == 0) scale[m] = sc;
  }
}

// ---------------- top-k (and K-split) reduction ----------------
template <typename Tout, typename IdT, typename Tp>
__global__ void __launch_bounds__(256)
    sum_topk_kernel(const Tp* __restrict__ part, int splits, int64_t T,
                    int top_k, int64_t H, int64_t numel, const IdT* __restrict__ ids,
                    int E, Tout* __restrict__ out, const int32_t* count_dev) {
  pdl_wait();
  pdl_trigger();
  const int64_t vec_per_row = H / 8;
  // rows past the device-side count (the rows a receive buffer actually got)
  // are neither read nor written
  const int64_t rows = count_dev != nullptr ? min(T, int64_t(max(*count_dev, 0))) : T;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int64_t h = (i - t * vec_per_row) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // Four top-k slots at a time: their ids first, then for each K split
    // the four partial rows, all in flight before the adds (at decode sizes
    // each thread has few rows to visit and the reduction is bound by load
    // latency). Dropped slots add exact zeros.
    for (int j0 = 0; j0 < top_k; j0 += 4) {
      int64_t rr[4];
      bool ok[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        rr[u] = t * top_k + j0 + u;
        ok[u] = j0 + u < top_k;
        if (ok[u] && ids != nullptr) {
          const long long e = static_cast<long long>(ids[rr[u]]);
          ok[u] = e >= 0 && e < E;
        }
      }
      for (int sp = 0; sp < splits; ++sp) {
        float v[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (ok[u]) {
            load8(part + (int64_t(sp) * numel + rr[u]) * H + h, v[u]);
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) v[u][q] = 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += v[u][q];
      }
    }
    store8(out + t * H + h, acc);
  }
}

// ---------------- split-K gate-up: sum the splits, SiLU(gate) * up ----------------
// part [S, numel, 2I] in the regrouped column order (32-column groups: 16
// gate, then the 16 matching up columns); act[m, 16g + c] for operand row m
// whose flat row r = sorted[m] is valid.
template <typename Tout>
__global__ void __launch_bounds__(256)
    swiglu_reduce_kernel(const float* __restrict__ part, int splits, int64_t numel, int64_t I,
                         const int32_t* __restrict__ sorted,
                         const int32_t* __restrict__ num_post_pad, int64_t max_rows,
                         Tout* __restrict__ act) {
  pdl_wait();
  pdl_trigger();
  const int64_t rows = min(int64_t(__ldg(num_post_pad)), max_rows);
  const int64_t vec_per_row = I / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / vec_per_row;
    const int r = __ldg(sorted + m);
    if (r >= numel) continue;
    const int64_t a0 = (i - m * vec_per_row) * 8;     // first act column
    const int64_t g = a0 / 16, c0 = a0 % 16;          // 8 columns stay in one group
    const int64_t gate_col = 32 * g + c0, up_col = gate_col + 16;
    float gsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float usum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // four splits' loads in flight at a time; sums in split order
    for (int s0 = 0; s0 < splits; s0 += 4) {
      float gv[4][8], uv[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (s0 + u < splits) {
          const float* row = part + (int64_t(s0 + u) * numel + r) * (2 * I);
          load8(row + gate_col, gv[u]);
          load8(row + up_col, uv[u]);
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) gv[u][q] = uv[u][q] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          gsum[q] += gv[u][q];
          usum[q] += uv[u][q];
        }
    }
    float out[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      out[q] = gsum[q] / (1.0f + __expf(-gsum[q])) * usum[q];
      // fp32 act rows are the down GEMM's tf32 operand: rounded here
      if constexpr (std::is_same<Tout, float>::value) out[q] = round_tf32(out[q]);
    }
    store8(act + m * I + a0, out);
  }
}

// ---------------- combine rows computed elsewhere ----------------
template <typename Tin, typename Tw, typename Tout>
__global__ void __launch_bounds__(256)
    combine_rows_kernel(const Tin* __restrict__ rows, const int32_t* __restrict__ inv,
                        const Tw* __restrict__ w, int64_t T, int top_k, int64_t H,
                        Tout* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t vec_per_row = H / 8;
  const int64_t total = T * vec_per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int64_t h = (i - t * vec_per_row) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // four slots at a time, loads first (as in sum_topk_kernel); slots that
    // were not sent contribute 0 * 0
    for (int j0 = 0; j0 < top_k; j0 += 4) {
      float v[4][8], wj[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t r = t * top_k + j0 + u;
        const int src = j0 + u < top_k ? __ldg(inv + r) : -1;
        if (src >= 0) {
          wj[u] = to_f32(w[r]);
          load8(rows + int64_t(src) * H + h, v[u]);
        } else {
          wj[u] = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) v[u][q] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = fmaf(wj[u], v[u][q], acc[q]);
    }
    store8(out + t * H + h, acc);
  }
}

int grid_for_rows(int64_t rows) {
  return int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, kWarps), 148 * 16)));
}

template <int MODE, typename Tin, typename Tout>
int launch_tokens_typed(const GatherArgs& a, cudaStream_t s) {
  const int64_t tasks = a.src_rows * ceil_div(a.H, int64_t(kBatch * 256));
  KSW_LAUNCH(gather_tokens_kernel<MODE, Tin, Tout>, dim3(grid_for_rows(tasks)),
             dim3(kWarps * 32), 0, s, static_cast<const Tin*>(a.src), a.H, a.top_k, a.inv,
             a.src_count, a.src_rows, a.max_rows, static_cast<Tout*>(a.dst),
             static_cast<void*>(a.scale), a.max_rows / 128);
  return MOE_OK;
}

template <int MODE, typename Tout>
int launch_tokens(const GatherArgs& a, cudaStream_t s) {
  switch (a.src_dtype) {
    case MOE_DTYPE_F32: return launch_tokens_typed<MODE, float, Tout>(a, s);
    case MOE_DTYPE_BF16: return launch_tokens_typed<MODE, __nv_bfloat16, Tout>(a, s);
    case MOE_DTYPE_F16: return launch_tokens_typed<MODE, __half, Tout>(a, s);
    default: return fail(MOE_ERR_UNSUPPORTED, "gather: unsupported source dtype");
  }
}

// The token-major gather, for the argument sets it covers; -1 otherwise.
int gather_tokens_launch(const GatherArgs& a, cudaStream_t s) {
  if (!a.inv || a.top_k < 1 || a.top_k > 32) return -1;
  if (a.quant == MOE_QUANT_NONE) {
    const int in = a.src_dtype, out = a.dst_dtype;
    if (in == MOE_DTYPE_F32 && out == MOE_DTYPE_BF16)
      return launch_tokens_typed<kTokCast, float, __nv_bfloat16>(a, s);
    if (in == MOE_DTYPE_F32 && out == MOE_DTYPE_F16)
      return launch_tokens_typed<kTokCast, float, __half>(a, s);
    if (in == MOE_DTYPE_F32 && out == MOE_DTYPE_F32)
      return launch_tokens_typed<kTokCast, float, float>(a, s);
    if (in == MOE_DTYPE_BF16 && out == MOE_DTYPE_BF16)
      return launch_tokens_typed<kTokCast, __nv_bfloat16, __nv_bfloat16>(a, s);
    if (in == MOE_DTYPE_F16 && out == MOE_DTYPE_F16)
      return launch_tokens_typed<kTokCast, __half, __half>(a, s);
    return -1;
  }
  if (a.quant == MOE_QUANT_FP8_BLOCK && a.scale) return launch_tokens<kTokFp8, uint8_t>(a, s);
  if (a.quant == MOE_QUANT_FP8_UE8M0 && a.scale && a.H % 128 == 0 && a.max_rows % 128 == 0)
    return launch_tokens<kTokUe8m0, uint8_t>(a, s);
  return -1;
}

}  // namespace

int gather_launch(const GatherArgs& a, cudaStream_t s) {
  KSW_REQUIRE(a.src && a.dst && a.num_post_pad, MOE_ERR_INVALID_ARG, "gather: null pointer");
  KSW_REQUIRE(aligned16(a.src) && aligned16(a.dst), MOE_ERR_INVALID_ARG,
              "gather: src and dst must be 16-byte aligned");
  KSW_REQUIRE(a.sorted || a.quant != MOE_QUANT_NONE, MOE_ERR_INVALID_ARG,
              "gather: null sorted ids");
  KSW_REQUIRE(a.sorted || a.top_k == 0, MOE_ERR_INVALID_ARG,
              "gather: sorted ids needed when top_k > 0");
  KSW_REQUIRE(a.H % 16 == 0 && a.H > 0, MOE_ERR_UNSUPPORTED, "gather: H % 16 != 0");
  KSW_REQUIRE(a.top_k >= 0, MOE_ERR_INVALID_ARG, "gather: top_k < 0");
  const int tok = gather_tokens_launch(a, s);
  if (tok >= 0) {
    if (tok != MOE_OK) return tok;
    KSW_CUDA(cudaGetLastError());
    return MOE_OK;
  }
  const int grid = grid_for_rows(a.max_rows);
  const int block = kWarps * 32;
  if (a.quant == MOE_QUANT_NONE) {
    if (a.src_dtype == MOE_DTYPE_F32 && a.dst_dtype == MOE_DTYPE_BF16)
      KSW_LAUNCH(gather_cast_kernel<float, __nv_bfloat16>, dim3(grid), dim3(block), 0, s,
          static_cast<const float*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<__nv_bfloat16*>(a.dst));
    else if (a.src_dtype == MOE_DTYPE_F32 && a.dst_dtype == MOE_DTYPE_F16)
      KSW_LAUNCH(gather_cast_kernel<float, __half>, dim3(grid), dim3(block), 0, s,
          static_cast<const float*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<__half*>(a.dst));
    else if (a.src_dtype == MOE_DTYPE_F32 && a.dst_dtype == MOE_DTYPE_F32)
      KSW_LAUNCH(gather_cast_kernel<float, float>, dim3(grid), dim3(block), 0, s,
          static_cast<const float*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<float*>(a.dst));
    else if (a.src_dtype == MOE_DTYPE_BF16 && a.dst_dtype == MOE_DTYPE_BF16)
      KSW_LAUNCH(gather_cast_kernel<__nv_bfloat16, __nv_bfloat16>, dim3(grid), dim3(block), 0, s,
          static_cast<const __nv_bfloat16*>(a.src), a.H, a.top_k, a.sorted,
          a.num_post_pad, a.max_rows, a.numel, a.src_rows,
          static_cast<__nv_bfloat16*>(a.dst));
    else if (a.src_dtype == MOE_DTYPE_F16 && a.dst_dtype == MOE_DTYPE_F16)
      KSW_LAUNCH(gather_cast_kernel<__half, __half>, dim3(grid), dim3(block), 0, s,
          static_cast<const __half*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<__half*>(a.dst));
    else
      return fail(MOE_ERR_UNSUPPORTED, "gather: unsupported dtype pair");
  } else if (a.quant == MOE_QUANT_FP8_BLOCK) {
    KSW_REQUIRE(a.scale != nullptr, MOE_ERR_INVALID_ARG, "gather: null scale");
    if (a.src_dtype == MOE_DTYPE_F32)
      KSW_LAUNCH(gather_fp8_kernel<float>, dim3(grid), dim3(block), 0, s,
          static_cast<const float*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<uint8_t*>(a.dst), a.scale);
    else if (a.src_dtype == MOE_DTYPE_BF16)
      KSW_LAUNCH(gather_fp8_kernel<__nv_bfloat16>, dim3(grid), dim3(block), 0, s,
          static_cast<const __nv_bfloat16*>(a.src), a.H, a.top_k, a.sorted,
          a.num_post_pad, a.max_rows, a.numel, a.src_rows,
          static_cast<uint8_t*>(a.dst), a.scale);
    else if (a.src_dtype == MOE_DTYPE_F16)
      KSW_LAUNCH(gather_fp8_kernel<__half>, dim3(grid), dim3(block), 0, s,
          static_cast<const __half*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<uint8_t*>(a.dst), a.scale);
    else
      return fail(MOE_ERR_UNSUPPORTED, "gather: unsupported source dtype");
  } else if (a.quant == MOE_QUANT_FP8_UE8M0) {
    KSW_REQUIRE(a.scale != nullptr, MOE_ERR_INVALID_ARG, "gather: null scale-factor image");
    KSW_REQUIRE(a.H % 128 == 0 && a.max_rows % 128 == 0, MOE_ERR_UNSUPPORTED,
                "gather: fp8 ue8m0 needs H and the buffer length divisible by 128");
    uint8_t* sf = reinterpret_cast<uint8_t*>(a.scale);
    const int64_t qb = ceil_div(a.H / 128, 4), rs = a.max_rows / 128;
    if (a.src_dtype == MOE_DTYPE_F32)
      KSW_LAUNCH(gather_ue8m0_kernel<float>, dim3(grid), dim3(block), 0, s,
          static_cast<const float*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<uint8_t*>(a.dst), sf, qb, rs);
    else if (a.src_dtype == MOE_DTYPE_BF16)
      KSW_LAUNCH(gather_ue8m0_kernel<__nv_bfloat16>, dim3(grid), dim3(block), 0, s,
          static_cast<const __nv_bfloat16*>(a.src), a.H, a.top_k, a.sorted,
          a.num_post_pad, a.max_rows, a.numel, a.src_rows,
          static_cast<uint8_t*>(a.dst), sf, qb, rs);
    else if (a.src_dtype == MOE_DTYPE_F16)
      KSW_LAUNCH(gather_ue8m0_kernel<__half>, dim3(grid), dim3(block), 0, s,
          static_cast<const __half*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<uint8_t*>(a.dst), sf, qb, rs);
    else
      return fail(MOE_ERR_UNSUPPORTED, "gather: unsupported source dtype");
  } else if (a.quant == MOE_QUANT_INT8_CHANNEL) {
    KSW_REQUIRE(a.scale != nullptr, MOE_ERR_INVALID_ARG, "gather: null scale");
    if (a.src_dtype == MOE_DTYPE_F32)
      KSW_LAUNCH(gather_i8_kernel<float>, dim3(grid), dim3(block), 0, s,
          static_cast<const float*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<int8_t*>(a.dst), a.scale);
    else if (a.src_dtype == MOE_DTYPE_BF16)
      KSW_LAUNCH(gather_i8_kernel<__nv_bfloat16>, dim3(grid), dim3(block), 0, s,
          static_cast<const __nv_bfloat16*>(a.src), a.H, a.top_k, a.sorted,
          a.num_post_pad, a.max_rows, a.numel, a.src_rows,
          static_cast<int8_t*>(a.dst), a.scale);
    else if (a.src_dtype == MOE_DTYPE_F16)
      KSW_LAUNCH(gather_i8_kernel<__half>, dim3(grid), dim3(block), 0, s,
          static_cast<const __half*>(a.src), a.H, a.top_k, a.sorted, a.num_post_pad,
          a.max_rows, a.numel, a.src_rows, static_cast<int8_t*>(a.dst), a.scale);
    else
      return fail(MOE_ERR_UNSUPPORTED, "gather: unsupported source dtype");
  } else {
    return fail(MOE_ERR_UNSUPPORTED, "gather: unknown quant mode");
  }
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

int sum_topk_launch(const SumArgs& a, cudaStream_t s) {
  KSW_REQUIRE(a.part && a.out, MOE_ERR_INVALID_ARG, "sum_topk: null pointer");
  KSW_REQUIRE(aligned16(a.part) && aligned16(a.out), MOE_ERR_INVALID_ARG,
              "sum_topk: partial and out must be 16-byte aligned");
  KSW_REQUIRE(a.H % 8 == 0, MOE_ERR_UNSUPPORTED, "sum_topk: H % 8 != 0");
  KSW_REQUIRE(a.splits >= 1 && a.top_k >= 1, MOE_ERR_INVALID_ARG, "sum_topk: bad sizes");
  KSW_REQUIRE(a.part_dtype == MOE_DTYPE_F32 || a.part_dtype == a.out_dtype, MOE_ERR_UNSUPPORTED,
              "sum_topk: partial rows must be f32 or the output dtype");
  if (a.T == 0) return MOE_OK;
  const int64_t total = a.T * (a.H / 8);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), 148 * 32)));
  const int64_t numel = a.T * a.top_k;
#define KSW_SUM(TOUT, IDT)                                                                   \
  if (a.part_dtype == MOE_DTYPE_F32)                                                         \
    KSW_LAUNCH(sum_topk_kernel<TOUT, IDT, float>, dim3(grid), dim3(256), 0, s,                                   \
        static_cast<const float*>(a.part), a.splits, a.T, a.top_k, a.H, numel,               \
        static_cast<const IDT*>(a.ids), a.E, static_cast<TOUT*>(a.out), a.count_dev);        \
  else                                                                                       \
    KSW_LAUNCH(sum_topk_kernel<TOUT, IDT, TOUT>, dim3(grid), dim3(256), 0, s,                                    \
        static_cast<const TOUT*>(a.part), a.splits, a.T, a.top_k, a.H, numel,                \
        static_cast<const IDT*>(a.ids), a.E, static_cast<TOUT*>(a.out), a.count_dev)
  const bool i64 = a.ids_dtype == MOE_DTYPE_I64;
  if (a.out_dtype == MOE_DTYPE_BF16) {
    if (i64) { KSW_SUM(__nv_bfloat16, int64_t); } else { KSW_SUM(__nv_bfloat16, int32_t); }
  } else if (a.out_dtype == MOE_DTYPE_F16) {
    if (i64) { KSW_SUM(__half, int64_t); } else { KSW_SUM(__half, int32_t); }
  } else if (a.out_dtype == MOE_DTYPE_F32) {
    if (i64) { KSW_SUM(float, int64_t); } else { KSW_SUM(float, int32_t); }
  } else {
    return fail(MOE_ERR_UNSUPPORTED, "sum_topk: unsupported output dtype");
  }
#undef KSW_SUM
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

int swiglu_reduce_launch(const float* part, int splits, int64_t numel, int64_t I,
                         const int32_t* sorted, const int32_t* num_post_pad, int64_t max_rows,
                         void* act, int act_dtype, cudaStream_t s) {
  KSW_REQUIRE(part && sorted && num_post_pad && act, MOE_ERR_INVALID_ARG,
              "swiglu_reduce: null pointer");
  KSW_REQUIRE(I % 16 == 0 && splits >= 1, MOE_ERR_UNSUPPORTED, "swiglu_reduce: bad sizes");
  const int64_t total = max_rows * (I / 8);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), 148 * 16)));
  if (act_dtype == MOE_DTYPE_BF16)
    KSW_LAUNCH(swiglu_reduce_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s,
        part, splits, numel, I, sorted, num_post_pad, max_rows, static_cast<__nv_bfloat16*>(act));
  else if (act_dtype == MOE_DTYPE_F16)
    KSW_LAUNCH(swiglu_reduce_kernel<__half>, dim3(grid), dim3(256), 0, s,
        part, splits, numel, I, sorted, num_post_pad, max_rows, static_cast<__half*>(act));
  else if (act_dtype == MOE_DTYPE_F32)
    KSW_LAUNCH(swiglu_reduce_kernel<float>, dim3(grid), dim3(256), 0, s,
        part, splits, numel, I, sorted, num_post_pad, max_rows, static_cast<float*>(act));
  else
    return fail(MOE_ERR_UNSUPPORTED, "swiglu_reduce: act dtype must be bf16/f16/f32");
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

int combine_launch(const CombineArgs& a, cudaStream_t s) {
  KSW_REQUIRE(a.inv && a.weights && a.out && (a.rows || a.T == 0), MOE_ERR_INVALID_ARG,
              "combine: null pointer");
  KSW_REQUIRE(a.H % 8 == 0 && a.top_k >= 1, MOE_ERR_UNSUPPORTED, "combine: bad sizes");
  KSW_REQUIRE(aligned16(a.rows) && aligned16(a.out), MOE_ERR_INVALID_ARG,
              "combine: rows and out must be 16-byte aligned");
  if (a.T == 0) return MOE_OK;
  const int64_t total = a.T * (a.H / 8);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), 148 * 32)));
#define KSW_COMB(TIN, TW, TOUT)                                                         \
  KSW_LAUNCH(combine_rows_kernel<TIN, TW, TOUT>, dim3(grid), dim3(256), 0, s,                               \
      static_cast<const TIN*>(a.rows), a.inv, static_cast<const TW*>(a.weights), a.T,   \
      a.top_k, a.H, static_cast<TOUT*>(a.out))
#define KSW_COMB_W(TIN, TOUT)                                                           \
  if (a.weights_dtype == MOE_DTYPE_F32) KSW_COMB(TIN, float, TOUT);                     \
  else if (a.weights_dtype == MOE_DTYPE_BF16) KSW_COMB(TIN, __nv_bfloat16, TOUT);       \
  else if (a.weights_dtype == MOE_DTYPE_F16) KSW_COMB(TIN, __half, TOUT);               \
  else return fail(MOE_ERR_INVALID_ARG, "combine: bad weights dtype")
  if (a.rows_dtype != a.out_dtype)
    return fail(MOE_ERR_UNSUPPORTED, "combine: rows and out must share a dtype");
  if (a.out_dtype == MOE_DTYPE_BF16) {
    KSW_COMB_W(__nv_bfloat16, __nv_bfloat16);
  } else if (a.out_dtype == MOE_DTYPE_F16) {
    KSW_COMB_W(__half, __half);
  } else if (a.out_dtype == MOE_DTYPE_F32) {
    KSW_COMB_W(float, float);
  } else {
    return fail(MOE_ERR_UNSUPPORTED, "combine: unsupported dtype");
  }
#undef KSW_COMB_W
#undef KSW_COMB
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

}  // namespace ksw
