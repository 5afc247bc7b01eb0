// Row log-sum-exp for the Qwen3 prefill driver's loss (not part of the reference's CIM path): for every row
// of a (rows, cols) logit block, its maximum m, the sum of exp(x - m) over the row, and the logit at the
// row's target column when the target falls inside this block.  One read of the logits replaces torch's
// max / subtract / exp / sum passes; several blocks (vocabulary shards) combine as
// M = max_r m_r, S = sum_r s_r exp(m_r - M), loss = log S + M - target.
#include "common.cuh"
#include "kernels.cuh"

namespace mib {

// Online maximum and rescaled sum of one value stream: (m, s) with s = sum exp(x - m).
__device__ __forceinline__ void lse_push(float v, float& m, float& s) {
  if (v > m) {
    s = s * __expf(m - v) + 1.0f;
    m = v;
  } else {
    s += __expf(v - m);
  }
}

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
  m = mm;
}

// One warp per row; lane l reads float4 l, l + 32, ... of the row (16-byte aligned rows, cols % 4 == 0),
// else scalars.
__global__ void __launch_bounds__(256) row_lse_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                                      int64_t ld, const int64_t* __restrict__ targets,
                                                      int64_t target_offset, float* __restrict__ row_max,
                                                      float* __restrict__ row_sumexp,
                                                      float* __restrict__ target_logit, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const float* p = x + r * ld;
    float m = -INFINITY, s = 0.0f;
    if (vec) {
      const float4* p4 = reinterpret_cast<const float4*>(p);
      const int64_t n4 = cols / 4;
      for (int64_t i = lane; i < n4; i += 32) {
        const float4 v = __ldg(p4 + i);
        lse_push(v.x, m, s);
        lse_push(v.y, m, s);
        lse_push(v.z, m, s);
        lse_push(v.w, m, s);
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) lse_push(__ldg(p + c), m, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      lse_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      row_max[r] = m;
      row_sumexp[r] = s;
      if (target_logit) {
        const int64_t t = targets[r] - target_offset;
        target_logit[r] = (t >= 0 && t < cols) ? __ldg(p + t) : 0.0f;
      }
    }
  }
}

cudaError_t row_lse(const float* x, int64_t rows, int64_t cols, int64_t ld, const int64_t* targets,
                    int64_t target_offset, float* row_max, float* row_sumexp, float* target_logit,
                    cudaStream_t stream) {
  const bool vec = cols % 4 == 0 && ld % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
  row_lse_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, rows, cols, ld, targets, target_offset,
                                                                    row_max, row_sumexp, target_logit, vec);
  count_launch();
  return cudaGetLastError();
}

}  // namespace mib
