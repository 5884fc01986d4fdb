// Per-head RMSNorm + rotate-half RoPE for head_dim 128, one warp per head:
// lane l owns elements [4l, 4l+4); its rotate-half partner lives in lane l ^ 16.
// Shared by the QK-norm+RoPE kernel and the decode attention kernel so that
// both write bit-identical rotated keys.  HF order (Qwen3MoeAttention):
// q_norm / k_norm over the head, times the norm weight, then
// x * cos + rotate_half(x) * sin with inv_freq = 1 / theta^(2i/128).
#pragma once

#include "common.cuh"

namespace nkimoe {

constexpr int kHeadDim = 128;

__device__ __forceinline__ void head_load4(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}

__device__ __forceinline__ float head_wload(const void* w, int w_dtype, int i) {
  return w_dtype == 0 ? static_cast<const float*>(w)[i] : __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]);
}

// cos / sin of the RoPE angle at position `pos` for frequency index fi
// (0..63): inv_freq = 1 / theta^(2 fi / 128), angle = pos * inv_freq in fp32.
__device__ __forceinline__ void rope_cs(float pos, int fi, float theta, float& c, float& s) {
  const float inv_freq = 1.0f / powf(theta, static_cast<float>(2 * fi) / static_cast<float>(kHeadDim));
  sincosf(pos * inv_freq, &s, &c);
}

// RMSNorm over the head (all 32 lanes call it) times the norm weight.
__device__ __forceinline__ void head_rmsnorm(const float (&v_in)[4], const void* w, int w_dtype, float eps, int lane,
                                             float (&v)[4]) {
  float ss = v_in[0] * v_in[0] + v_in[1] * v_in[1] + v_in[2] * v_in[2] + v_in[3] * v_in[3];
  ss = warp_sum(ss);
  const float rinv = rsqrtf(ss / static_cast<float>(kHeadDim) + eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = v_in[j] * rinv * head_wload(w, w_dtype, lane * 4 + j);
}

// Rotate-half RoPE of a normalised head given this lane's cos / sin.
__device__ __forceinline__ void head_rope(const float (&v)[4], const float (&cs)[4], const float (&sn)[4], int lane,
                                          float (&o)[4]) {
  // rotate-half partner: element i pairs with i + 64 (first half) / i - 64
  float pv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) pv[j] = __shfl_xor_sync(0xffffffffu, v[j], 16);
  const bool first = lane < 16;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float rot = first ? -pv[j] : pv[j];
    o[j] = fmaf(v[j], cs[j], __fmul_rn(rot, sn[j]));
  }
}

// cos / sin of this lane's 4 elements at position `pos` (the same for every
// head of a token).
__device__ __forceinline__ void rope_cs_lane(float pos, float theta, int lane, float (&cs)[4], float (&sn)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) rope_cs(pos, (lane * 4 + j) & (kHeadDim / 2 - 1), theta, cs[j], sn[j]);
}

// norm_rope_head128 with the lane's cos / sin given (computed once per token).
__device__ __forceinline__ void norm_rope_head128_cs(const float (&v_in)[4], const void* w, int w_dtype, float eps,
                                                     int lane, const float (&cs)[4], const float (&sn)[4],
                                                     float (&o)[4]) {
  float v[4];
  head_rmsnorm(v_in, w, w_dtype, eps, lane, v);
  head_rope(v, cs, sn, lane, o);
}

// v: this lane's 4 elements of one head; returns the normalised, weighted and
// rotated values in o.  All 32 lanes of the warp must call it.
__device__ __forceinline__ void norm_rope_head128(const float (&v_in)[4], const void* w, int w_dtype, float pos,
                                                  float theta, float eps, int lane, float (&o)[4]) {
  float cs[4], sn[4];
  rope_cs_lane(pos, theta, lane, cs, sn);
  norm_rope_head128_cs(v_in, w, w_dtype, eps, lane, cs, sn, o);
}

__device__ __forceinline__ void head_store4(__nv_bfloat16* p, const float (&o)[4]) {
  uint2 u;
  u.x = pack_bf16x2(o[0], o[1]);
  u.y = pack_bf16x2(o[2], o[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

}  // namespace nkimoe
