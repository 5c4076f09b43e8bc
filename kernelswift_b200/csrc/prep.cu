// One-time weight preparation. base.py:60-61 casts the fp32 master weights to
// the activation dtype on every forward call; here the cast (or quantisation)
// runs once per weight version and also regroups the gate/up rows of w1 so
// that every 32-row slice of the gate-up GEMM's B operand holds 16 gate rows
// followed by the 16 matching up rows (the SwiGLU epilogue then finds gate
// and up of one output column in the same TMEM tile).
//
// Quantisation arithmetic (shared with the oracle):
//   fp8 block: per 128x128 block of the ORIGINAL [rows, cols] layout,
//              scale = absmax / 448 (1 if the block is zero),
//              q = e4m3_rn(clamp(x / scale, -448, 448))
//   int8 channel: per row, scale = absmax / 127 (1 if zero),
//              q = rint(clamp(x / scale, -127, 127))
//   fp8 UE8M0: per 128x128 block of the ORIGINAL layout, scale = the
//              smallest power of two with absmax / scale <= 448 (1 if the
//              block is zero), q = e4m3_rn(x / scale) (exact scaling); the
//              scale byte is written into the scale-factor image at every
//              row of the block (its regrouped row for w13)
#include <type_traits>

#include "common.cuh"

namespace ksw {
namespace {

// Destination row of source row `rs` (of 2I rows) in the regrouped w13.
__device__ __forceinline__ int64_t w13_row(int64_t rs, int64_t I) {
  if (rs < I) return (rs >> 4) * 32 + (rs & 15);
  const int64_t ru = rs - I;
  return (ru >> 4) * 32 + 16 + (ru & 15);
}

__device__ __forceinline__ int64_t map_row(int64_t rs, int64_t I, bool regroup) {
  return regroup ? w13_row(rs, I) : rs;
}

template <typename T>
__device__ __forceinline__ float ld(const T* p) { return to_f32(*p); }

// Cast with row regrouping: one warp per source row.
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256)
    prep_cast_kernel(const Tin* __restrict__ src, int64_t E, int64_t R, int64_t C,
                     int64_t I, bool regroup, Tout* __restrict__ dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = E * R;
  for (int64_t row = int64_t(blockIdx.x) * 8 + warp; row < rows;
       row += int64_t(gridDim.x) * 8) {
    const int64_t e = row / R, rs = row - e * R;
    const Tin* s = src + row * C;
    Tout* d = dst + (e * R + map_row(rs, I, regroup)) * C;
    for (int64_t c = lane; c < C; c += 32) {
      if constexpr (std::is_same<Tout, float>::value)
        d[c] = round_tf32(ld(s + c));  // fp32 weights of the tf32 GEMMs
      else
        d[c] = from_f32<Tout>(ld(s + c));
    }
  }
}

// fp8 block quantisation: one CTA of 256 threads per 128x128 block.
template <typename Tin>
__global__ void __launch_bounds__(256)
    prep_fp8_kernel(const Tin* __restrict__ src, int64_t E, int64_t R, int64_t C,
                    int64_t I, bool regroup, uint8_t* __restrict__ dst,
                    float* __restrict__ scale) {
  __shared__ float red[8];
  const int64_t RB = (R + 127) / 128, CB = (C + 127) / 128;
  const int64_t blk = blockIdx.x;
  const int64_t e = blk / (RB * CB);
  const int64_t rb = (blk / CB) % RB;
  const int64_t cb = blk % CB;
  const int t = threadIdx.x;
  const int r_in = t >> 4;          // 0..15
  const int c_in = (t & 15) * 8;    // 0..120
  float amax = 0.0f;
  for (int i = 0; i < 8; ++i) {
    const int64_t r = rb * 128 + r_in + 16 * i;
    if (r >= R) break;
    for (int j = 0; j < 8; ++j) {
      const int64_t c = cb * 128 + c_in + j;
      if (c < C) amax = fmaxf(amax, fabsf(ld(src + (e * R + r) * C + c)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();
  amax = red[0];
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  float sc = amax / 448.0f;
  sc = sc > 0.0f ? sc : 1.0f;
  for (int i = 0; i < 8; ++i) {
    const int64_t r = rb * 128 + r_in + 16 * i;
    if (r >= R) break;
    uint8_t* d = dst + (e * R + map_row(r, I, regroup)) * C;
    for (int j = 0; j < 8; ++j) {
      const int64_t c = cb * 128 + c_in + j;
      if (c < C) {
        const float q = fminf(fmaxf(ld(src + (e * R + r) * C + c) / sc, -448.0f), 448.0f);
        d[c] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3));
      }
    }
  }
  if (t == 0) scale[(e * RB + rb) * CB + cb] = sc;
}

// fp8 block quantisation with power-of-two scales: one CTA of 256 threads per
// 128x128 block (R and C multiples of 128); the block's scale byte goes into
// the scale-factor image at each of its 128 rows.
template <typename Tin>
__global__ void __launch_bounds__(256)
    prep_ue8m0_kernel(const Tin* __restrict__ src, int64_t E, int64_t R, int64_t C,
                      int64_t I, bool regroup, uint8_t* __restrict__ dst,
                      uint8_t* __restrict__ sf, int64_t q_blocks) {
  __shared__ float red[8];
  const int64_t RB = R / 128, CB = C / 128;
  const int64_t blk = blockIdx.x;
  const int64_t e = blk / (RB * CB);
  const int64_t rb = (blk / CB) % RB;
  const int64_t cb = blk % CB;
  const int t = threadIdx.x;
  const int r_in = t >> 4;          // 0..15
  const int c_in = (t & 15) * 8;    // 0..120
  float amax = 0.0f;
  for (int i = 0; i < 8; ++i) {
    const int64_t r = rb * 128 + r_in + 16 * i;
    for (int j = 0; j < 8; ++j)
      amax = fmaxf(amax, fabsf(ld(src + (e * R + r) * C + cb * 128 + c_in + j)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();
  amax = red[0];
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const uint32_t b = ue8m0_byte(amax);
  const float inv = ue8m0_inv_scale(b);
  for (int i = 0; i < 8; ++i) {
    const int64_t r = rb * 128 + r_in + 16 * i;
    uint8_t* d = dst + (e * R + map_row(r, I, regroup)) * C;
    for (int j = 0; j < 8; ++j) {
      const int64_t c = cb * 128 + c_in + j;
      const float q = fminf(fmaxf(ld(src + (e * R + r) * C + c) * inv, -448.0f), 448.0f);
      d[c] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3));
    }
  }
  if (t < 128) {
    const int64_t rr = map_row(rb * 128 + t, I, regroup);
    sf[sf_image_offset(e, rr, cb, q_blocks, RB)] = static_cast<uint8_t>(b);
  }
}

// int8 per-row quantisation: one warp per source row; the scale follows the
// row to its regrouped position.
template <typename Tin>
__global__ void __launch_bounds__(256)
    prep_i8_kernel(const Tin* __restrict__ src, int64_t E, int64_t R, int64_t C,
                   int64_t I, bool regroup, int8_t* __restrict__ dst,
                   float* __restrict__ scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = E * R;
  for (int64_t row = int64_t(blockIdx.x) * 8 + warp; row < rows;
       row += int64_t(gridDim.x) * 8) {
    const int64_t e = row / R, rs = row - e * R;
    const Tin* s = src + row * C;
    float amax = 0.0f;
    for (int64_t c = lane; c < C; c += 32) amax = fmaxf(amax, fabsf(ld(s + c)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float sc = amax / 127.0f;
    sc = sc > 0.0f ? sc : 1.0f;
    const int64_t rd = e * R + map_row(rs, I, regroup);
    int8_t* d = dst + rd * C;
    for (int64_t c = lane; c < C; c += 32) {
      const float q = fminf(fmaxf(ld(s + c) / sc, -127.0f), 127.0f);
      d[c] = static_cast<int8_t>(__float2int_rn(q));
    }
    if (lane == 0) scale[rd] = sc;
  }
}

// Row regrouping of an already-quantised byte matrix.
__global__ void __launch_bounds__(256)
    prep_copy_rows_kernel(const uint8_t* __restrict__ src, int64_t E, int64_t R,
                          int64_t C, int64_t I, bool regroup,
                          uint8_t* __restrict__ dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = E * R;
  for (int64_t row = int64_t(blockIdx.x) * 8 + warp; row < rows;
       row += int64_t(gridDim.x) * 8) {
    const int64_t e = row / R, rs = row - e * R;
    const uint8_t* s = src + row * C;
    uint8_t* d = dst + (e * R + map_row(rs, I, regroup)) * C;
    for (int64_t c = lane; c < C; c += 32) d[c] = s[c];
  }
}

int grid_rows(int64_t rows) {
  return int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, 8), 148 * 64)));
}

template <typename Tin>
int prep_typed(const Tin* src, int64_t E, int64_t R, int64_t C, int64_t I,
               bool regroup, int quant, void* dst, int dst_dtype, float* scale,
               cudaStream_t s) {
  const int64_t rows = E * R;
  if (quant == MOE_QUANT_NONE) {
    if (dst_dtype == MOE_DTYPE_BF16)
      prep_cast_kernel<Tin, __nv_bfloat16><<<grid_rows(rows), 256, 0, s>>>(
          src, E, R, C, I, regroup, static_cast<__nv_bfloat16*>(dst));
    else if (dst_dtype == MOE_DTYPE_F16)
      prep_cast_kernel<Tin, __half><<<grid_rows(rows), 256, 0, s>>>(
          src, E, R, C, I, regroup, static_cast<__half*>(dst));
    else if (dst_dtype == MOE_DTYPE_F32)
      prep_cast_kernel<Tin, float><<<grid_rows(rows), 256, 0, s>>>(
          src, E, R, C, I, regroup, static_cast<float*>(dst));
    else
      return fail(MOE_ERR_INVALID_ARG, "prepare: dst dtype must be bf16/f16/f32");
  } else if (quant == MOE_QUANT_FP8_BLOCK) {
    KSW_REQUIRE(dst_dtype == MOE_DTYPE_E4M3 && scale, MOE_ERR_INVALID_ARG,
                "prepare: fp8 needs an e4m3 destination and a scale buffer");
    const int64_t nblk = E * ceil_div(R, 128) * ceil_div(C, 128);
    KSW_REQUIRE(nblk < (int64_t(1) << 31), MOE_ERR_UNSUPPORTED, "prepare: too many blocks");
    prep_fp8_kernel<Tin><<<unsigned(nblk), 256, 0, s>>>(
        src, E, R, C, I, regroup, static_cast<uint8_t*>(dst), scale);
  } else if (quant == MOE_QUANT_FP8_UE8M0) {
    KSW_REQUIRE(dst_dtype == MOE_DTYPE_E4M3 && scale, MOE_ERR_INVALID_ARG,
                "prepare: fp8 ue8m0 needs an e4m3 destination and a scale-factor image");
    KSW_REQUIRE(R % 128 == 0 && C % 128 == 0 && (!regroup || I % 128 == 0),
                MOE_ERR_UNSUPPORTED,
                "prepare: fp8 ue8m0 needs rows and columns (and I) divisible by 128");
    const int64_t nblk = E * (R / 128) * (C / 128);
    KSW_REQUIRE(nblk < (int64_t(1) << 31), MOE_ERR_UNSUPPORTED, "prepare: too many blocks");
    prep_ue8m0_kernel<Tin><<<unsigned(nblk), 256, 0, s>>>(
        src, E, R, C, I, regroup, static_cast<uint8_t*>(dst), reinterpret_cast<uint8_t*>(scale),
        ceil_div(C / 128, 4));
  } else if (quant == MOE_QUANT_INT8_CHANNEL) {
    KSW_REQUIRE(dst_dtype == MOE_DTYPE_I8 && scale, MOE_ERR_INVALID_ARG,
                "prepare: int8 needs an int8 destination and a scale buffer");
    prep_i8_kernel<Tin><<<grid_rows(rows), 256, 0, s>>>(
        src, E, R, C, I, regroup, static_cast<int8_t*>(dst), scale);
  } else {
    return fail(MOE_ERR_INVALID_ARG, "prepare: unknown quant mode");
  }
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

int prepare(const void* src, int src_dtype, const float* scale_in, int64_t E,
            int64_t R, int64_t C, int64_t I, bool regroup, int quant, void* dst,
            int dst_dtype, float* scale_out, cudaStream_t s) {
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(src && dst, MOE_ERR_INVALID_ARG, "prepare: null pointer");
  KSW_REQUIRE(E >= 1 && R >= 1 && C >= 1, MOE_ERR_INVALID_ARG, "prepare: bad sizes");
  KSW_REQUIRE(C % 16 == 0 && (!regroup || I % 16 == 0), MOE_ERR_UNSUPPORTED,
              "prepare: sizes must be multiples of 16");
  if (src_dtype == MOE_DTYPE_E4M3) {
    KSW_REQUIRE(quant == MOE_QUANT_FP8_BLOCK && dst_dtype == MOE_DTYPE_E4M3,
                MOE_ERR_INVALID_ARG, "prepare: e4m3 source only for fp8 block quant");
    KSW_REQUIRE(scale_in && scale_out, MOE_ERR_INVALID_ARG,
                "prepare: e4m3 source needs scale_in and scale_out");
    prep_copy_rows_kernel<<<grid_rows(E * R), 256, 0, s>>>(
        static_cast<const uint8_t*>(src), E, R, C, I, regroup, static_cast<uint8_t*>(dst));
    KSW_CUDA(cudaGetLastError());
    const size_t n = size_t(E * ceil_div(R, 128) * ceil_div(C, 128)) * sizeof(float);
    KSW_CUDA(cudaMemcpyAsync(scale_out, scale_in, n, cudaMemcpyDeviceToDevice, s));
    return MOE_OK;
  }
  switch (src_dtype) {
    case MOE_DTYPE_F32:
      return prep_typed(static_cast<const float*>(src), E, R, C, I, regroup, quant, dst,
                        dst_dtype, scale_out, s);
    case MOE_DTYPE_BF16:
      return prep_typed(static_cast<const __nv_bfloat16*>(src), E, R, C, I, regroup, quant,
                        dst, dst_dtype, scale_out, s);
    case MOE_DTYPE_F16:
      return prep_typed(static_cast<const __half*>(src), E, R, C, I, regroup, quant, dst,
                        dst_dtype, scale_out, s);
    default:
      return fail(MOE_ERR_INVALID_ARG, "prepare: unsupported source dtype");
  }
}

}  // namespace
}  // namespace ksw

extern "C" {

int64_t moe_ue8m0_scale_bytes(int64_t groups, int64_t rows, int64_t cols) {
  if (groups < 0 || rows < 0 || cols < 0) return -1;
  return groups * ksw::ceil_div(ksw::ceil_div(cols, 128), 4) * ksw::ceil_div(rows, 128) * 512;
}

int moe_prepare_w13(const void* w1, int src_dtype, const float* scale_in,
                    int64_t num_experts, int64_t inter_size, int64_t hidden_size,
                    int quant, void* w13_out, int dst_dtype, float* scale_out,
                    void* stream) {
  return ksw::prepare(w1, src_dtype, scale_in, num_experts, 2 * inter_size, hidden_size,
                      inter_size, true, quant, w13_out, dst_dtype, scale_out,
                      static_cast<cudaStream_t>(stream));
}

int moe_prepare_w2(const void* w2, int src_dtype, const float* scale_in,
                   int64_t num_experts, int64_t hidden_size, int64_t inter_size,
                   int quant, void* w2_out, int dst_dtype, float* scale_out,
                   void* stream) {
  return ksw::prepare(w2, src_dtype, scale_in, num_experts, hidden_size, inter_size, 0,
                      false, quant, w2_out, dst_dtype, scale_out,
                      static_cast<cudaStream_t>(stream));
}

}  // extern "C"
