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
#include "routing.cuh"

namespace ksw {
namespace {

constexpr int kWarpsPerBlock = 8;

template <int PER_LANE, typename Tin, typename Tw, typename Tid>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    topk_softmax_kernel(const Tin* __restrict__ logits, int64_t T, int E, int k, int renorm,
                        Tw* __restrict__ weights, Tid* __restrict__ ids) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t t = int64_t(blockIdx.x) * kWarpsPerBlock + warp; t < T;
       t += int64_t(gridDim.x) * kWarpsPerBlock) {
    float sel_w;
    int sel_i;
    route_token_warp<PER_LANE>(logits + t * E, E, k, renorm, lane, sel_w, sel_i);
    if (lane < k) {
      weights[t * k + lane] = from_f32<Tw>(sel_w);
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

// ---------------------------------------------------------------------------
// Grouped top-k routing (kernels/track1-triton/groupedtopk/base.py:31-72):
// scores = softmax or sigmoid of the logits; the experts form G equal groups;
// the topk_group groups with the best maximum score are kept and the top-k
// experts are chosen among them; weights = their scores, renormalised over
// the k when asked, times routed_scaling_factor; fp32 weights, int32 ids.
// Both score functions are strictly increasing, so groups and experts are
// ranked by logit (ties to the lower index), and only the chosen experts'
// scores are evaluated.
// ---------------------------------------------------------------------------
template <int PER_LANE, typename Tin>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    grouped_topk_kernel(const Tin* __restrict__ logits, int64_t T, int E, int k, int renorm,
                        int G, int topk_group, int sigmoid, float scale,
                        float* __restrict__ weights, int32_t* __restrict__ ids) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int EG = E / G;
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
    if (!sigmoid) {
#pragma unroll
      for (int j = 0; j < PER_LANE; ++j)
        if (lane + 32 * j < E) sum += expf(v[j] - mx);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    // lane g < G ends up with the best logit of group g
    float gbest = -INFINITY;
    for (int g = 0; g < G; ++g) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < PER_LANE; ++j) {
        const int e = lane + 32 * j;
        if (e < E && e / EG == g) m = fmaxf(m, v[j]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == g) gbest = m;
    }
    uint32_t gsel = 0;  // bit g: group g kept
    bool gtaken = false;
    for (int s = 0; s < topk_group; ++s) {
      float bv = (lane < G && !gtaken) ? gbest : -INFINITY;
      int bi = (lane < G && !gtaken) ? lane : INT32_MAX;
      warp_argmax(bv, bi);
      if (bi < G) gsel |= 1u << bi;
      if (lane == bi) gtaken = true;
    }
    uint32_t taken = 0;
    float sel_w = 0.0f;
    int sel_i = 0;
    float wsum = 0.0f;
    for (int s = 0; s < k; ++s) {
      float bv = -INFINITY;
      int bi = INT32_MAX;
#pragma unroll
      for (int j = 0; j < PER_LANE; ++j) {
        const int e = lane + 32 * j;
        if (e < E && ((gsel >> (e / EG)) & 1u) && !(taken >> j & 1u) &&
            (v[j] > bv || (v[j] == bv && e < bi))) {
          bv = v[j];
          bi = e;
        }
      }
      warp_argmax(bv, bi);
      if (bi < E && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      const float w = sigmoid ? 1.0f / (1.0f + expf(-bv)) : expf(bv - mx) / sum;
      wsum += w;
      if (lane == s) {
        sel_w = w;
        sel_i = bi;
      }
    }
    if (lane < k) {
      float w = renorm ? sel_w / wsum : sel_w;
      if (scale != 1.0f) w *= scale;
      weights[t * k + lane] = w;
      ids[t * k + lane] = sel_i;
    }
  }
}

template <int PER_LANE, typename Tin>
int launch_grouped(const Tin* logits, int64_t T, int E, int k, int renorm, int G,
                   int topk_group, int sigmoid, float scale, float* w, int32_t* ids,
                   cudaStream_t s) {
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(T, kWarpsPerBlock),
                                                               148 * 16)));
  KSW_LAUNCH(grouped_topk_kernel<PER_LANE, Tin>, dim3(grid), dim3(kWarpsPerBlock * 32), 0, s,
             logits, T, E, k, renorm, G, topk_group, sigmoid, scale, w, ids);
  return MOE_OK;
}

template <typename Tin>
int launch_grouped_e(const Tin* logits, int64_t T, int E, int k, int renorm, int G,
                     int topk_group, int sigmoid, float scale, float* w, int32_t* ids,
                     cudaStream_t s) {
  const int per = (E + 31) / 32;
#define KSW_GTK(P) \
  return launch_grouped<P>(logits, T, E, k, renorm, G, topk_group, sigmoid, scale, w, ids, s)
  if (per <= 1) KSW_GTK(1);
  if (per <= 2) KSW_GTK(2);
  if (per <= 4) KSW_GTK(4);
  if (per <= 8) KSW_GTK(8);
  if (per <= 16) KSW_GTK(16);
  KSW_GTK(32);
#undef KSW_GTK
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

extern "C" int moe_grouped_topk(const void* gating_output, int logits_dtype, int64_t num_tokens,
                                int num_experts, int top_k, int renormalize,
                                int num_expert_group, int topk_group, int scoring_func,
                                float routed_scaling_factor, float* topk_weights,
                                int32_t* topk_ids, void* stream) {
  using namespace ksw;
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(num_tokens >= 0, MOE_ERR_INVALID_ARG, "grouped_topk: num_tokens < 0");
  KSW_REQUIRE(num_experts >= 1 && num_experts <= 1024, MOE_ERR_UNSUPPORTED,
              "grouped_topk: num_experts must be in [1, 1024]");
  KSW_REQUIRE(num_expert_group >= 1 && num_expert_group <= 32 &&
                  num_experts % num_expert_group == 0,
              MOE_ERR_UNSUPPORTED,
              "grouped_topk: num_expert_group must be in [1, 32] and divide num_experts");
  KSW_REQUIRE(topk_group >= 1 && topk_group <= num_expert_group, MOE_ERR_INVALID_ARG,
              "grouped_topk: topk_group must be in [1, num_expert_group]");
  KSW_REQUIRE(top_k >= 1 && top_k <= 32 &&
                  top_k <= topk_group * (num_experts / num_expert_group),
              MOE_ERR_UNSUPPORTED,
              "grouped_topk: top_k must be in [1, 32] and fit in the kept groups");
  KSW_REQUIRE(scoring_func == 0 || scoring_func == 1, MOE_ERR_INVALID_ARG,
              "grouped_topk: scoring_func must be 0 (softmax) or 1 (sigmoid)");
  if (num_tokens == 0) return MOE_OK;
  KSW_REQUIRE(gating_output && topk_weights && topk_ids, MOE_ERR_INVALID_ARG,
              "grouped_topk: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (logits_dtype) {
    case MOE_DTYPE_F32:
      return launch_grouped_e(static_cast<const float*>(gating_output), num_tokens, num_experts,
                              top_k, renormalize, num_expert_group, topk_group, scoring_func,
                              routed_scaling_factor, topk_weights, topk_ids, s);
    case MOE_DTYPE_BF16:
      return launch_grouped_e(static_cast<const __nv_bfloat16*>(gating_output), num_tokens,
                              num_experts, top_k, renormalize, num_expert_group, topk_group,
                              scoring_func, routed_scaling_factor, topk_weights, topk_ids, s);
    case MOE_DTYPE_F16:
      return launch_grouped_e(static_cast<const __half*>(gating_output), num_tokens, num_experts,
                              top_k, renormalize, num_expert_group, topk_group, scoring_func,
                              routed_scaling_factor, topk_weights, topk_ids, s);
    default:
      return fail(MOE_ERR_INVALID_ARG, "grouped_topk: logits dtype must be f32/bf16/f16");
  }
}
