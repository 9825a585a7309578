// Elementwise stages of the target's verify forward, fused around the
// projections (cuBLAS) and the tree-attention kernel.
//
// A Qwen3 decoder layer (transformers models/qwen3/modeling_qwen3.py:305-334,
// :273-299) runs, per verify round, over n = 1 + budget tree nodes:
//
//   residual += o_proj(attn)            \  one launch: rt_add_rmsnorm
//   x = rmsnorm(residual) * w           /
//   qkv = x @ [Wq; Wk; Wv]^T            (cuBLAS)
//   q, k = rope(rmsnorm_head(q|k) * w)  \  one launch: rt_qk_norm_rope_append
//   cache[offset + i] = k, v            /
//   attn = tree_attention(q, cache)     (rt_tree_attn)
//   ...
//   act = silu(gate) * up               one launch: rt_silu_mul
//
// Each kernel reproduces the rounding steps of the unfused PyTorch ops it
// replaces: every intermediate the model materialises as a bf16 tensor is
// rounded to bf16 at the same point (the residual sum, the normalised row
// before the weight multiply, q*cos and rot(q)*sin before their sum, silu(g)
// before the multiply by up; squares are rounded to fp32 before they are
// summed, as x.pow(2).mean() does).  The only difference is the order of that
// fp32 sum, which moves a result by one bf16 unit in rare elements.
//
// All of it is HBM- and launch-bound (a few MB per launch at tree sizes);
// rows move as 16-byte vectors.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_util.h"
#include "layer_math.cuh"

namespace rt {
namespace {

constexpr int kNormThreads = 128;
constexpr int kNormMaxVec = 16;  // hidden <= 128 threads * 16 vectors * 8 = 16384

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) s += red[w];
  return s;
}

// One CTA per token row, V 16-byte vectors per thread.  mode 0: residual =
// embed[ids[row]];  mode 1: residual = bf16(residual + delta);  mode 2: the
// row is `residual` as is.  out = bf16(weight * bf16(x * rsqrt(mean(x^2) +
// eps)))  (Qwen3RMSNorm.forward, modeling_qwen3.py:59-64, and the residual
// adds at :327 and :333).  Every load of the row (input, delta, weight) is
// issued before the first store, so a launch costs one memory round trip.
template <int V>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    int mode, const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ embed, int64_t vocab,
    const __nv_bfloat16* __restrict__ delta, __nv_bfloat16* __restrict__ residual,
    const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ out, int hidden, float eps,
    int* status) {
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  const int nvec = hidden >> 3;
  pdl_launch_dependents();
  // the norm weights are not written by the round: fetch them before waiting
  const Vec8* wv = reinterpret_cast<const Vec8*>(weight);
  Vec8 wr[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) wr[j] = wv[v];
  }
  pdl_wait();
  const Vec8* src;
  bool zero = false;
  if (mode == 0) {
    const int64_t id = ids[row];
    if (id < 0 || id >= vocab) {
      zero = true;
      if (threadIdx.x == 0) set_status(status, RT_DEV_BAD_INDEX);
    }
    src = reinterpret_cast<const Vec8*>(embed + (zero ? 0 : id) * hidden);
  } else {
    src = reinterpret_cast<const Vec8*>(residual + static_cast<int64_t>(row) * hidden);
  }
  const Vec8* dsrc = reinterpret_cast<const Vec8*>(delta + static_cast<int64_t>(row) * hidden);
  Vec8 xr[V], dr[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      xr[j] = src[v];
      if (mode == 1) dr[j] = dsrc[v];
    }
  }
  Vec8* rdst = reinterpret_cast<Vec8*>(residual + static_cast<int64_t>(row) * hidden);
  float x[V][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      unpack8(xr[j], x[j]);
      if (zero) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[j][e] = 0.f;
      }
      if (mode == 1) {
        float d[8];
        unpack8(dr[j], d);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[j][e] = round_bf16(x[j][e] + d[e]);
      }
      if (mode != 2) rdst[v] = pack8(x[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(x[j][e], x[j][e]));
    }
  }
  const float var = block_sum(ss, red) * (1.0f / static_cast<float>(hidden));
  const float r = rsqrtf(var + eps);
  Vec8* o = reinterpret_cast<Vec8*>(out + static_cast<int64_t>(row) * hidden);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v < nvec) {
      float w[8], y[8];
      unpack8(wr[j], w);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = w[e] * round_bf16(x[j][e] * r);
      o[v] = pack8(y);
    }
  }
}

template <int V>
void launch_norm(int mode, const int64_t* ids, const void* embed, int64_t vocab, const void* delta, void* residual,
                 const void* weight, void* out, int rows, int hidden, float eps, int* status, cudaStream_t s) {
  launch_ex(add_rmsnorm_kernel<V>, dim3(rows), dim3(kNormThreads), 0, s, 1, mode, ids,
            static_cast<const __nv_bfloat16*>(embed), vocab, static_cast<const __nv_bfloat16*>(delta),
            static_cast<__nv_bfloat16*>(residual), static_cast<const __nv_bfloat16*>(weight),
            static_cast<__nv_bfloat16*>(out), hidden, eps, status);
}

void dispatch_norm(int mode, const int64_t* ids, const void* embed, int64_t vocab, const void* delta,
                   void* residual, const void* weight, void* out, int rows, int hidden, float eps, int* status,
                   cudaStream_t s) {
  const int per = (hidden / 8 + kNormThreads - 1) / kNormThreads;
  if (per <= 1) launch_norm<1>(mode, ids, embed, vocab, delta, residual, weight, out, rows, hidden, eps, status, s);
  else if (per <= 2) launch_norm<2>(mode, ids, embed, vocab, delta, residual, weight, out, rows, hidden, eps, status, s);
  else if (per <= 3) launch_norm<3>(mode, ids, embed, vocab, delta, residual, weight, out, rows, hidden, eps, status, s);
  else if (per <= 4) launch_norm<4>(mode, ids, embed, vocab, delta, residual, weight, out, rows, hidden, eps, status, s);
  else if (per <= 8) launch_norm<8>(mode, ids, embed, vocab, delta, residual, weight, out, rows, hidden, eps, status, s);
  else launch_norm<kNormMaxVec>(mode, ids, embed, vocab, delta, residual, weight, out, rows, hidden, eps, status, s);
}

// One warp per (token, head slot); slots [0, hq) are query heads, [hq, hq+hkv)
// key heads, [hq+hkv, hq+2hkv) value heads of the packed qkv row.  Lane l holds
// elements 4l..4l+3 of the 128-wide head; rotate_half pairs lane l with l^16.
// Query/key: per-head RMSNorm with its weight (modeling_qwen3.py:269-270), then
// rotary embedding q*cos + rotate_half(q)*sin (:151-181) with cos/sin rows from
// bf16 tables indexed by position.  Keys and values are stored at cache row
// offset + token (DynamicLayer.update's append, cache_utils.py:102-121).
__global__ void __launch_bounds__(256) qk_norm_rope_append_kernel(
    const __nv_bfloat16* __restrict__ qkv, int n, int hq, int hkv, const __nv_bfloat16* __restrict__ q_norm_w,
    const __nv_bfloat16* __restrict__ k_norm_w, float eps, const __nv_bfloat16* __restrict__ cos_t,
    const __nv_bfloat16* __restrict__ sin_t, int64_t table_len, const int64_t* __restrict__ positions,
    __nv_bfloat16* __restrict__ q_out, char* k_cache, char* v_cache, int64_t c_head_stride, int64_t c_row_stride,
    int64_t capacity, int64_t offset, const int64_t* offset_dev, int* status) {
  constexpr int D = 128;
  pdl_launch_dependents();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int slots = hq + 2 * hkv;
  if (warp >= n * slots) return;
  const int t = warp / slots, s = warp - t * slots;
  const __nv_bfloat16* row = qkv + static_cast<int64_t>(t) * slots * D + static_cast<int64_t>(s) * D;
  const uint2 raw = reinterpret_cast<const uint2*>(row)[lane];
  const bool is_v = s >= hq + hkv;
  uint2 res = raw;
  if (!is_v) {
    float x[4];
    unpack4(raw, x);
    int64_t p = positions[t];
    if (p < 0 || p >= table_len) {
      if (lane == 0) set_status(status, RT_DEV_BAD_INDEX);
      p = 0;
    }
    res = qk_norm_rope4(x, s < hq ? q_norm_w : k_norm_w, eps, cos_t + p * D, sin_t + p * D, lane);
  }
  if (s < hq) {
    reinterpret_cast<uint2*>(q_out + (static_cast<int64_t>(t) * hq + s) * D)[lane] = res;
    return;
  }
  const int64_t off = (offset_dev != nullptr ? *offset_dev : 0) + offset;
  const int64_t dst_row = off + t;
  if (off < 0 || dst_row >= capacity) {
    if (lane == 0) set_status(status, RT_DEV_OVERFLOW);
    return;
  }
  const int g = is_v ? s - hq - hkv : s - hq;
  char* base = (is_v ? v_cache : k_cache) + g * c_head_stride + dst_row * c_row_stride;
  reinterpret_cast<uint2*>(base)[lane] = res;
}

// act = bf16(bf16(silu(gate)) * up) over gate_up = [gate | up] per row
// (Qwen3MLP.forward, modeling_qwen3.py:81-83; silu(x) = x / (1 + exp(-x)) in
// fp32 as torch's CUDA kernel evaluates it).
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up,
                                                       __nv_bfloat16* __restrict__ out, int rows, int inter) {
  pdl_launch_dependents();
  pdl_wait();
  const int vpr = inter >> 3;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(rows) * vpr) return;
  const int64_t r = i / vpr;
  const int v = static_cast<int>(i - r * vpr);
  const Vec8* g = reinterpret_cast<const Vec8*>(gate_up + r * 2 * inter);
  float a[8], b[8], y[8];
  unpack8(g[v], a);
  unpack8(g[vpr + v], b);
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = silu_mul_bf16(a[e], b[e]);
  reinterpret_cast<Vec8*>(out + r * inter)[v] = pack8(y);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" int rt_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, void* residual,
                                const void* weight, void* out, int rows, int hidden, float eps, int* status,
                                rt_stream_t stream) {
  if (rows < 0 || hidden <= 0 || hidden % 8 || hidden > kNormThreads * kNormMaxVec * 8 || vocab <= 0) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  if (rows == 0) return RT_OK;
  if (!ids || !table || !residual || !weight || !out || !aligned16(table) || !aligned16(residual) ||
      !aligned16(weight) || !aligned16(out)) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  dispatch_norm(0, ids, table, vocab, nullptr, residual, weight, out, rows, hidden, eps, status,
                static_cast<cudaStream_t>(stream));
  return check_launch();
}

extern "C" int rt_add_rmsnorm(const void* delta, void* residual, const void* weight, void* out, int rows,
                              int hidden, float eps, rt_stream_t stream) {
  if (rows < 0 || hidden <= 0 || hidden % 8 || hidden > kNormThreads * kNormMaxVec * 8) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  if (rows == 0) return RT_OK;
  if (!residual || !weight || !out || !aligned16(residual) || !aligned16(weight) || !aligned16(out) ||
      (delta && !aligned16(delta))) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  dispatch_norm(delta ? 1 : 2, nullptr, nullptr, 0, delta, residual, weight, out, rows, hidden, eps, nullptr,
                static_cast<cudaStream_t>(stream));
  return check_launch();
}

extern "C" int rt_qk_norm_rope_append(const void* qkv, int n, int num_q_heads, int num_kv_heads, int head_dim,
                                      const void* q_norm_weight, const void* k_norm_weight, float eps,
                                      const void* cos_table, const void* sin_table, int64_t table_len,
                                      const int64_t* positions, void* q_out, void* k_cache, void* v_cache,
                                      int64_t cache_head_stride, int64_t cache_row_stride, int64_t capacity,
                                      int64_t offset, const int64_t* offset_dev, int* status,
                                      rt_stream_t stream) {
  if (n < 0 || head_dim != 128 || num_q_heads <= 0 || num_kv_heads <= 0 || table_len <= 0 || capacity <= 0) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  if ((q_norm_weight == nullptr) != (k_norm_weight == nullptr)) return RT_ERR_INVALID_ARGUMENT;
  if (n == 0) return RT_OK;
  if (!qkv || !cos_table || !sin_table || !positions || !q_out || !k_cache || !v_cache) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  if (reinterpret_cast<uintptr_t>(qkv) % 8 || reinterpret_cast<uintptr_t>(q_out) % 8 ||
      reinterpret_cast<uintptr_t>(k_cache) % 8 || reinterpret_cast<uintptr_t>(v_cache) % 8 ||
      reinterpret_cast<uintptr_t>(cos_table) % 8 || reinterpret_cast<uintptr_t>(sin_table) % 8 ||
      cache_head_stride % 8 || cache_row_stride % 8 ||
      (q_norm_weight && (reinterpret_cast<uintptr_t>(q_norm_weight) % 8 ||
                         reinterpret_cast<uintptr_t>(k_norm_weight) % 8))) {
    return RT_ERR_INVALID_ARGUMENT;
  }
  const int64_t warps = static_cast<int64_t>(n) * (num_q_heads + 2 * num_kv_heads);
  const int blocks = static_cast<int>((warps * 32 + 255) / 256);
  launch_ex(qk_norm_rope_append_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1,
      static_cast<const __nv_bfloat16*>(qkv), n, num_q_heads, num_kv_heads,
      static_cast<const __nv_bfloat16*>(q_norm_weight), static_cast<const __nv_bfloat16*>(k_norm_weight), eps,
      static_cast<const __nv_bfloat16*>(cos_table), static_cast<const __nv_bfloat16*>(sin_table), table_len,
      positions, static_cast<__nv_bfloat16*>(q_out), static_cast<char*>(k_cache), static_cast<char*>(v_cache),
      cache_head_stride, cache_row_stride, capacity, offset, offset_dev, status);
  return check_launch();
}

extern "C" int rt_silu_mul(const void* gate_up, void* out, int rows, int inter, rt_stream_t stream) {
  if (rows < 0 || inter <= 0 || inter % 8) return RT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return RT_OK;
  if (!gate_up || !out || !aligned16(gate_up) || !aligned16(out)) return RT_ERR_INVALID_ARGUMENT;
  const int64_t total = static_cast<int64_t>(rows) * (inter / 8);
  launch_ex(silu_mul_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0,
            static_cast<cudaStream_t>(stream), 1, static_cast<const __nv_bfloat16*>(gate_up),
            static_cast<__nv_bfloat16*>(out), rows, inter);
  return check_launch();
}

