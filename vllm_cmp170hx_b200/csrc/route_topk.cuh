// Router top-k of one token per warp (router.cu, and the fused route + dispatch of sp_comm.cu).
//
//   mode 0  softmax over all experts, top-k, renormalise over the k picked
//   mode 1  sigmoid scores, select by score + bias, weights = score / sum (GLM)
//   mode 2  sqrt(softplus(logit)), select by score + bias, weights = s / (sum + 1e-20)
// then every weight is multiplied by `scale`.  Ties pick the lowest expert id.
#pragma once
#include <cfloat>

#include "common.cuh"

namespace b200 {

constexpr int kMaxExpertsPerLane = 16;  // E <= 512

// One warp routes one token: its row of E logits -> lane j < k holds the j-th pick (*id, *w: the
// weight after the mode's renormalisation and `scale`).  Lanes >= k get id -1.
B200_DEVICE void route_topk_warp(const float* __restrict__ row, int E, int k, int mode,
                                 const float* __restrict__ bias, float scale, int renorm, int* id_out,
                                 float* w_out) {
  const int lane = threadIdx.x % 32;
  float score[kMaxExpertsPerLane];  // value used for the weight
  float key[kMaxExpertsPerLane];    // value used for selection
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    float l = e < E ? row[e] : -INFINITY;
    score[i] = l;
    mx = fmaxf(mx, l);
  }
  float denom = 1.f;
  if (mode == 0) {
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = lane + 32 * i;
      score[i] = e < E ? __expf(score[i] - mx) : 0.f;
      s += score[i];
    }
    denom = warp_sum(s);
  }
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    if (e >= E) {
      key[i] = -INFINITY;
      continue;
    }
    if (mode == 0) {
      score[i] = score[i] / denom;
      key[i] = score[i];
    } else if (mode == 1) {
      score[i] = sigmoidf_(score[i]);
      key[i] = score[i] + (bias ? bias[e] : 0.f);
    } else {
      const float l = score[i];
      const float sp = l > 20.f ? l : log1pf(__expf(l));
      score[i] = sqrtf(sp);
      key[i] = score[i] + (bias ? bias[e] : 0.f);
    }
    // a NaN key (a failed row) ranks below every real score but stays selectable, so every row
    // gets k distinct valid expert ids (its weights carry the NaN on to the output row)
    if (key[i] != key[i]) key[i] = -FLT_MAX;
  }
  float picked_sum = 0.f;
  float my_w = 0.f;
  int my_id = -1;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
    float best_s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = lane + 32 * i;
      if (key[i] > best || (key[i] == best && e < best_e)) {
        best = key[i];
        best_e = e;
        best_s = score[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      const float os = __shfl_xor_sync(0xffffffffu, best_s, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
        best_s = os;
      }
    }
    // remove the pick
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      if (lane + 32 * i == best_e) key[i] = -INFINITY;
    picked_sum += best_s;
    if (lane == j) {
      my_w = best_s;
      my_id = best_e;
    }
  }
  float w = my_w;
  if (lane < k && renorm) w = mode == 2 ? w / (picked_sum + 1e-20f) : w / picked_sum;
  *id_out = lane < k ? my_id : -1;
  *w_out = lane < k ? w * scale : 0.f;
}

}  // namespace b200
