// Routing of one token by one warp: softmax over the router logits, top-k,
// optional renormalisation (kernels/track1-triton/fused_moe/base.py:44-47).
// Shared by the routing kernel (moe_topk_softmax) and the fused decode
// kernel, so both select the same experts with the same weights bit for bit.
//
// Lane l holds logits l, l+32, l+64, ... in registers. Selection is by logit
// (softmax is strictly increasing in the logit), ties broken by the lower
// expert index; weight_j = exp(l_j - max) / sum_e exp(l_e - max), then
// divided by the sum of the k selected weights when renormalising. All
// arithmetic is fp32. The per-lane sums skip experts >= E, so the result
// does not depend on PER_LANE as long as 32 * PER_LANE >= E.
#pragma once

#include "common.cuh"

namespace ksw {

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

// All 32 lanes call it for the same token row; lane j < k receives the j-th
// selected expert (descending logit) and its weight (renormalised over the k
// when `renorm`).
template <int PER_LANE, typename Tin>
__device__ __forceinline__ void route_token_warp(const Tin* __restrict__ row, int E, int k,
                                                 int renorm, int lane, float& sel_w,
                                                 int& sel_i) {
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
  sel_w = 0.0f;        // lane j < k keeps the j-th selected weight
  sel_i = 0;
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
  if (renorm) sel_w = sel_w / wsum;
}

}  // namespace ksw
