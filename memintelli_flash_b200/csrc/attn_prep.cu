// Attention input preparation for the Qwen3 prefill driver (not part of the reference's CIM path):
// per-head RMSNorm of q and k, rotary position embedding, and bf16 casts of q, k and v, in one pass
// over the fused q/k/v crossbar output.  The torch sequence it replaces is
//   q = rope(rms_norm(q, q_norm)), k = rope(rms_norm(k, k_norm)), then q/k/v.bfloat16()
// with rms_norm(x, w) = x * rsqrt(mean(x^2) + eps) * w and rope(x) = x * cos + rotate_half(x) * sin,
// rotate_half(x) = cat(-x[D/2:], x[:D/2]) (the Hugging Face Qwen3 convention).
#include "common.cuh"
#include "kernels.cuh"

#include <cuda_bf16.h>

namespace mib {

// One warp per (token, head); lane l holds elements [EPL*l, EPL*l + EPL) of the head (EPL = D/32), so the
// rotate_half partner of element i (i +- D/2) sits in lane l ^ 16.
template <int EPL>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const float* __restrict__ qkv, int64_t tokens,
                                                           int64_t ld_token, int seq_len, int q_heads, int kv_heads,
                                                           const float* __restrict__ q_norm,
                                                           const float* __restrict__ k_norm, float eps,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, __nv_bfloat16* q_out,
                                                           __nv_bfloat16* k_out, __nv_bfloat16* v_out) {
  constexpr int D = 32 * EPL;
  const int lane = threadIdx.x & 31;
  const int heads = q_heads + 2 * kv_heads;
  const int64_t items = tokens * heads;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; item < items;
       item += nwarps) {
    const int64_t tok = item / heads;
    const int h = static_cast<int>(item - tok * heads);
    const float* src = qkv + tok * ld_token + static_cast<int64_t>(h) * D + lane * EPL;
    float x[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) x[e] = __ldg(src + e);
    __nv_bfloat16* dst;
    if (h >= q_heads + kv_heads) {  // v: cast only
      dst = v_out + (tok * kv_heads + (h - q_heads - kv_heads)) * D + lane * EPL;
    } else {
      const bool is_q = h < q_heads;
      const float* w = (is_q ? q_norm : k_norm) + lane * EPL;
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float r = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
      for (int e = 0; e < EPL; ++e) x[e] = x[e] * r * __ldg(w + e);
      const int t = static_cast<int>(tok % seq_len);
      const float* c = cos_t + static_cast<int64_t>(t) * D + lane * EPL;
      const float* s = sin_t + static_cast<int64_t>(t) * D + lane * EPL;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        const float rot = lane < 16 ? -partner : partner;
        x[e] = x[e] * __ldg(c + e) + rot * __ldg(s + e);
      }
      dst = is_q ? q_out + (tok * q_heads + h) * D + lane * EPL
                 : k_out + (tok * kv_heads + (h - q_heads)) * D + lane * EPL;
    }
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      __nv_bfloat162 pair = __floats2bfloat162_rn(x[e], x[e + 1]);
      *reinterpret_cast<__nv_bfloat162*>(dst + e) = pair;
    }
  }
}

cudaError_t qk_norm_rope(const float* qkv, int64_t tokens, int64_t ld_token, int seq_len, int q_heads, int kv_heads,
                         int head_dim, const float* q_norm, const float* k_norm, float eps, const float* cos_t,
                         const float* sin_t, void* q_out, void* k_out, void* v_out, cudaStream_t stream) {
  const int64_t items = tokens * (q_heads + 2 * kv_heads);
  int64_t blocks = (items + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  auto* q = static_cast<__nv_bfloat16*>(q_out);
  auto* k = static_cast<__nv_bfloat16*>(k_out);
  auto* v = static_cast<__nv_bfloat16*>(v_out);
  switch (head_dim) {
    case 64:
      qk_norm_rope_kernel<2><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
          qkv, tokens, ld_token, seq_len, q_heads, kv_heads, q_norm, k_norm, eps, cos_t, sin_t, q, k, v);
      break;
    case 128:
      qk_norm_rope_kernel<4><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
          qkv, tokens, ld_token, seq_len, q_heads, kv_heads, q_norm, k_norm, eps, cos_t, sin_t, q, k, v);
      break;
    case 256:
      qk_norm_rope_kernel<8><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
          qkv, tokens, ld_token, seq_len, q_heads, kv_heads, q_norm, k_norm, eps, cos_t, sin_t, q, k, v);
      break;
    default:
      return cudaErrorNotSupported;
  }
  count_launch();
  return cudaGetLastError();
}

}  // namespace mib
