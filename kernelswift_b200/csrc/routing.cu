// Fused routing: softmax over the router logits, top-k, optional
// renormalisation and the cast of the weights to the activation dtype, in one
// launch (kernels/track1-triton/fused_moe/base.py:44-48, which takes five
// to six torch launches).
//
// One warp per token; lane l holds logits l, l+32, l+64, ... in registers.
// Selection is by logit (softmax is strictly increasing in the logit), ties
// broken by the lower expert index; weight_j = exp(l_j - max) / sum_e
// exp(l_e - max), then divided by the sum of the k selected weights when
// renormalising. All arithmetic is fp32.
#include "common.cuh"

namespace ksw {
namespace {

constexpr int kWarpsPerBlock = 8;

// Warp-wide argmax of (value, index): larger value wins, then lower index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

template <typename Tin>
__device__ __forceinline__ float ld_logit(const Tin* p) {
  return to_f32(*p);
}

template <int PER_LANE, typename Tin, typename Tw, typename Tid>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    topk_softmax_kernel(const Tin* __restrict__ logits, int64_t T, int E, int k, int renorm,
                        Tw* __restrict__ weights, Tid* __restrict__ ids) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t t = int64_t(blockIdx.x) * kWarpsPerBlock + warp; t < T;
       t += int64_t(gridDim.x) * kWarpsPerBlock) {
    const Tin* row = logits + t * E;
    float v[PER_LANE];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? ld_logit(row + e) : -INFINITY;
      mx = fmaxf(mx, v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j)
      if (lane + 32 * j < E) sum += expf(v[j] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);

    uint32_t taken = 0;  // bit j: this lane's j-th logit already selected
    float sel_w = 0.0f;  // lane j < k keeps the j-th selected weight
    int sel_i = 0;
    float wsum = 0.0f;
    for (int s = 0; s < k; ++s) {
      float bv = -INFINITY;
      int bi = INT32_MAX;
#pragma unroll
      for (int j = 0; j < PER_LANE; ++j) {
        const int e = lane + 32 * j;
        if (e < E && !(taken >> j & 1u) && (v[j] > bv || (v[j] == bv && e < bi))) {
          bv = v[j];
          bi = e;
        }
      }
      warp_argmax(bv, bi);
      if (bi < E && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      const float w = expf(bv - mx) / sum;
      wsum += w;
      if (lane == s) {
        sel_w = w;
        sel_i = bi;
      }
    }
    if (lane < k) {
      const float w = renorm ? sel_w / wsum : sel_w;
      weights[t * k + lane] = from_f32<Tw>(w);
      ids[t * k + lane] = static_cast<Tid>(sel_i);
    }
  }
}

template <int PER_LANE, typename Tin, typename Tw>
int launch_ids(const Tin* logits, int64_t T, int E, int k, int renorm, Tw* w, void* ids,
               int ids_dtype, cudaStream_t s) {
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(T, kWarpsPerBlock),
                                                               148 * 16)));
  if (ids_dtype == MOE_DTYPE_I32)
    KSW_LAUNCH(topk_softmax_kernel<PER_LANE, Tin, Tw, int32_t>, dim3(grid),
               dim3(kWarpsPerBlock * 32), 0, s, logits, T, E, k, renorm, w,
               static_cast<int32_t*>(ids));
  else
    KSW_LAUNCH(topk_softmax_kernel<PER_LANE, Tin, Tw, int64_t>, dim3(grid),
               dim3(kWarpsPerBlock * 32), 0, s, logits, T, E, k, renorm, w,
               static_cast<int64_t*>(ids));
  return MOE_OK;
}

template <int PER_LANE, typename Tin>
int launch_w(const Tin* logits, int64_t T, int E, int k, int renorm, void* w, int w_dtype,
             void* ids, int ids_dtype, cudaStream_t s) {
  switch (w_dtype) {
    case MOE_DTYPE_F32:
      return launch_ids<PER_LANE>(logits, T, E, k, renorm, static_cast<float*>(w), ids,
                                  ids_dtype, s);
    case MOE_DTYPE_BF16:
      return launch_ids<PER_LANE>(logits, T, E, k, renorm, static_cast<__nv_bfloat16*>(w), ids,
                                  ids_dtype, s);
    case MOE_DTYPE_F16:
      return launch_ids<PER_LANE>(logits, T, E, k, renorm, static_cast<__half*>(w), ids,
                                  ids_dtype, s);
    default:
      return fail(MOE_ERR_INVALID_ARG, "topk_softmax: weights dtype must be f32/bf16/f16");
  }
}

template <typename Tin>
int launch_e(const Tin* logits, int64_t T, int E, int k, int renorm, void* w, int w_dtype,
             void* ids, int ids_dtype, cudaStream_t s) {
  const int per = (E + 31) / 32;
  if (per <= 1) return launch_w<1>(logits, T, E, k, renorm, w, w_dtype, ids, ids_dtype, s);
  if (per <= 2) return launch_w<2>(logits, T, E, k, renorm, w, w_dtype, ids, ids_dtype, s);
  if (per <= 4) return launch_w<4>(logits, T, E, k, renorm, w, w_dtype, ids, ids_dtype, s);
  if (per <= 8) return launch_w<8>(logits, T, E, k, renorm, w, w_dtype, ids, ids_dtype, s);
  if (per <= 16) return launch_w<16>(logits, T, E, k, renorm, w, w_dtype, ids, ids_dtype, s);
  return launch_w<32>(logits, T, E, k, renorm, w, w_dtype, ids, ids_dtype, s);
}

}  // namespace
}  // namespace ksw

extern "C" int moe_topk_softmax(const void* router_logits, int logits_dtype, int64_t num_tokens,
                                int num_experts, int top_k, int renormalize,
                                void* topk_weights, int weights_dtype, void* topk_ids,
                                int ids_dtype, void* stream) {
  using namespace ksw;
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(num_tokens >= 0, MOE_ERR_INVALID_ARG, "topk_softmax: num_tokens < 0");
  KSW_REQUIRE(num_experts >= 1 && num_experts <= 1024, MOE_ERR_UNSUPPORTED,
              "topk_softmax: num_experts must be in [1, 1024]");
  KSW_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= num_experts, MOE_ERR_UNSUPPORTED,
              "topk_softmax: top_k must be in [1, min(32, num_experts)]");
  KSW_REQUIRE(ids_dtype == MOE_DTYPE_I32 || ids_dtype == MOE_DTYPE_I64, MOE_ERR_INVALID_ARG,
              "topk_softmax: ids dtype must be int32 or int64");
  if (num_tokens == 0) return MOE_OK;
  KSW_REQUIRE(router_logits && topk_weights && topk_ids, MOE_ERR_INVALID_ARG,
              "topk_softmax: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (logits_dtype) {
    case MOE_DTYPE_F32:
      return launch_e(static_cast<const float*>(router_logits), num_tokens, num_experts, top_k,
                      renormalize, topk_weights, weights_dtype, topk_ids, ids_dtype, s);
    case MOE_DTYPE_BF16:
      return launch_e(static_cast<const __nv_bfloat16*>(router_logits), num_tokens, num_experts,
                      top_k, renormalize, topk_weights, weights_dtype, topk_ids, ids_dtype, s);
    case MOE_DTYPE_F16:
      return launch_e(static_cast<const __half*>(router_logits), num_tokens, num_experts, top_k,
                      renormalize, topk_weights, weights_dtype, topk_ids, ids_dtype, s);
    default:
      return fail(MOE_ERR_INVALID_ARG, "topk_softmax: logits dtype must be f32/bf16/f16");
  }
}
