// Per-element arithmetic of the decoder-layer stages, shared by the standalone
// elementwise kernels (layer_ops.cu) and the projection epilogues
// (linear.cu), so both round at the same points as the transformers ops.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace rt {

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct alignas(16) Vec8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const Vec8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __bfloat1622float2(v.h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ Vec8 pack8(const float* f) {
  Vec8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ void unpack4(uint2 raw, float* x) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  x[0] = a.x, x[1] = a.y, x[2] = b.x, x[3] = b.y;
}

__device__ __forceinline__ uint2 pack4(const float* y) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(y[0], y[1]);
  const __nv_bfloat162 b = __floats2bfloat162_rn(y[2], y[3]);
  uint2 r;
  r.x = *reinterpret_cast<const uint32_t*>(&a);
  r.y = *reinterpret_cast<const uint32_t*>(&b);
  return r;
}

// silu(g) * u with the rounding of act_fn(gate) * up on bf16 tensors
// (Qwen3MLP.forward, modeling_qwen3.py:81-83): silu evaluated in fp32 as
// x / (1 + exp(-x)), rounded to bf16, then the bf16 product.
__device__ __forceinline__ float silu_mul_bf16(float g, float u) {
  return round_bf16(g / (1.0f + expf(-g))) * u;
}

// One 128-wide query/key head row held by a warp, lane l owning features
// 4l..4l+3 (bf16 values in x).  Per-head RMSNorm with weight `norm_w` (skipped
// when NULL; Qwen3RMSNorm on the head dim, modeling_qwen3.py:269-270) and the
// rotary embedding q*cos + rotate_half(q)*sin (:151-181) with the bf16 cos/sin
// rows of this token's position.  Returns the lane's 4 output values, packed.
__device__ __forceinline__ uint2 qk_norm_rope4(float* x, const __nv_bfloat16* norm_w, float eps,
                                               const __nv_bfloat16* cos_row, const __nv_bfloat16* sin_row,
                                               int lane) {
  constexpr int D = 128;
  if (norm_w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float r = rsqrtf(ss * (1.0f / D) + eps);
    float w[4];
    unpack4(reinterpret_cast<const uint2*>(norm_w)[lane], w);
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = round_bf16(w[e] * round_bf16(x[e] * r));
  }
  float c[4], sn[4], y[4];
  unpack4(reinterpret_cast<const uint2*>(cos_row)[lane], c);
  unpack4(reinterpret_cast<const uint2*>(sin_row)[lane], sn);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float other = __shfl_xor_sync(0xFFFFFFFFu, x[e], 16);
    const float rot = lane < 16 ? -other : other;
    y[e] = round_bf16(x[e] * c[e]) + round_bf16(rot * sn[e]);
  }
  return pack4(y);
}

}  // namespace rt
