// Quantise + bit-slice + level-map kernels (inputs and weights) and the per-call
// noise pre-passes.  All are HBM-bound element-wise/reduction kernels.
//
// Reference arithmetic (zhuizhou/memintelli_flash):
//   block abs-max and tiling      memintelli/pimpy/data_formats.py:141-184
//   INT quantise + slice          memintelli/pimpy/utils.py:44-83
//   BFP quantise + slice          memintelli/pimpy/utils.py:86-128
//   weight levels, faults         memintelli/pimpy/memmat_tensor.py:160-202
//   DAC levels                    memintelli/pimpy/memmat_tensor.py:295-297, 358-360
//   read variation                memintelli/pimpy/memmat_tensor.py:204-236
//   voltage noise                 memintelli/pimpy/memmat_tensor.py:297-299
#include "common.cuh"
#include "kernels.cuh"

#include <type_traits>

namespace mib {

static unsigned long long g_launches = 0;
void count_launch(int n) { __atomic_add_fetch(&g_launches, static_cast<unsigned long long>(n), __ATOMIC_RELAXED); }
unsigned long long launch_count() { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

// ---------------------------------------------------------------------------
// element loaders: matmul coordinates (batch b, row r, col c) -> value
// ---------------------------------------------------------------------------
struct DenseLoader {
  const float* x;
  int64_t ld_batch, ld_row, ld_col, rows, cols;
  __device__ __forceinline__ float operator()(int64_t b, int64_t r, int64_t c) const {
    if (r >= rows || c >= cols) return 0.0f;
    return __ldg(x + b * ld_batch + r * ld_row + c * ld_col);
  }
};

// F.unfold order: column c = ci*kh*kw + i*kw + j, row r = oh*Wo + ow (per image b).
struct ConvLoader {
  const float* x;
  int64_t C, H, W, Ho, Wo, rows, cols;
  int kh, kw, sh, sw, ph, pw, dh, dw;
  __device__ __forceinline__ float operator()(int64_t b, int64_t r, int64_t c) const {
    if (r >= rows || c >= cols) return 0.0f;
    const int64_t khw = static_cast<int64_t>(kh) * kw;
    const int64_t ci = c / khw;
    const int rem = static_cast<int>(c - ci * khw);
    const int i = rem / kw, j = rem - (rem / kw) * kw;
    const int64_t oh = r / Wo, ow = r - (r / Wo) * Wo;
    const int64_t ih = oh * sh - ph + static_cast<int64_t>(i) * dh;
    const int64_t iw = ow * sw - pw + static_cast<int64_t>(j) * dw;
    if (ih < 0 || ih >= H || iw < 0 || iw >= W) return 0.0f;
    return __ldg(x + ((b * C + ci) * H + ih) * W + iw);
  }
};

// ---------------------------------------------------------------------------
// generic block abs-max: one warp per quant block (b, rb, cb)
// ---------------------------------------------------------------------------
template <class Loader>
__global__ void block_absmax_kernel(Loader ld, int64_t batch, int64_t rows, int64_t cols, int qg0, int qg1,
                                    int64_t nbr, int64_t nbc, float* __restrict__ bmax) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t nblocks = batch * nbr * nbc;
  for (int64_t wb = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; wb < nblocks;
       wb += nwarps) {
    const int64_t b = wb / (nbr * nbc);
    const int64_t rb = (wb / nbc) % nbr;
    const int64_t cb = wb % nbc;
    const int64_t r0 = rb * qg0, c0 = cb * qg1;
    const int64_t nr = max(static_cast<int64_t>(0), min(static_cast<int64_t>(qg0), rows - r0));
    const int64_t nc = max(static_cast<int64_t>(0), min(static_cast<int64_t>(qg1), cols - c0));
    const int64_t total = nr * nc;
    float m = 0.0f;
    for (int64_t e = lane; e < total; e += 32) {
      const int64_t t = e / nc, c = e - (e / nc) * nc;
      m = fmaxf(m, fabsf(ld(b, r0 + t, c0 + c)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) bmax[wb] = m;
  }
}

// ---------------------------------------------------------------------------
// input slicing: one warp per (b, row, column quant block).  When `have_max`
// is false the block is one row high (quant_gran[0] == 1) and the warp computes
// its max itself, making the kernel a single pass over x.
//
// The DAC level of slice t is round(code_t / m_t * (rdac - 1)) with the
// reference's fp32 steps; it depends only on the packed code q (< 2^bits), so
// each CTA tabulates q -> encoded level of every slice once in shared memory.
// ---------------------------------------------------------------------------
// Quantise one value to its packed code given the block maximum / exponent.
// inv_p2e = 2^-e when that is a normal float (e <= 126): v / 2^e == v * 2^-e then, both being one
// correctly rounded operation on the same real value.  Otherwise inv_p2e is 0 and the division runs.
__device__ __forceinline__ int quantize_fast(float v, float bmax, int e, float inv_p2e, int bits, bool bfp) {
  int q;
  if (bfp) {
    const float s = inv_p2e != 0.0f ? __fmul_rn(v, inv_p2e) : __fdiv_rn(v, pow2f(e));
    float t = __fmul_rn(s, static_cast<float>(1 << (bits - 2)));
    float r = rintf(t);
    r = fminf(fmaxf(r, -static_cast<float>(1 << (bits - 1))), static_cast<float>((1 << (bits - 1)) - 1));
    q = static_cast<int>(r);
  } else {
    if (bmax == 0.0f) return 0;
    q = static_cast<int>(rintf(__fmul_rn(__fdiv_rn(v, bmax), static_cast<float>((1 << (bits - 1)) - 1))));
  }
  if (q < 0) q += (1 << bits);
  return q;
}

// Per-CTA table: packed code q -> encoded level of every slice.  E4M3 keeps slice t in byte t&3 of
// word t>>2; FP16 keeps it in half t&1 of word t>>1.
template <int KIND>
struct alignas(16) LevelLut {
  static constexpr int kWords = KIND == MIB_OPERAND_E4M3 ? 2 : 4;
  uint32_t w[256][kWords];
};

template <int KIND>
__device__ __forceinline__ void build_level_lut(LevelLut<KIND>& lut, const SliceArgs& a) {
  for (int q = threadIdx.x; q < (1 << a.bits); q += blockDim.x) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    for (int t = 0; t < a.n_slices; ++t) {
      const int code = (q >> a.offs[t]) & a.maxes[t];
      const float lv = static_cast<float>(level_map(code, a.maxes[t], a.lm1));
      if constexpr (KIND == MIB_OPERAND_E4M3) {
        w[t >> 2] |= static_cast<uint32_t>(enc_e4m3(lv)) << (8 * (t & 3));
      } else {
        const __half h = __float2half_rn(lv);
        w[t >> 1] |= static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&h)) << (16 * (t & 1));
      }
    }
#pragma unroll
    for (int k = 0; k < LevelLut<KIND>::kWords; ++k) lut.w[q][k] = w[k];
  }
  __syncthreads();
}

// Voltage noise of one plane element (memmat_tensor.py:297-299): level * (1 + vnoise * z), with explicit
// roundings so that the fused (slicing) and separate (input_noise_kernel) passes give the same bits.
__device__ __forceinline__ float apply_vnoise(float v, float z, float vnoise) {
  return __fmul_rn(v, __fmaf_rn(z, vnoise, 1.0f));
}

// Voltage noise on 4 FP16 plane elements starting at linear plane index idx (idx % 4 == 0): they are
// Philox group idx / 4 of the call's input-noise stream, as in input_noise_kernel.
__device__ __forceinline__ uint2 vnoise4(uint2 o, const SliceArgs& a, int64_t idx) {
  float z[4];
  normal4(a.noise_seed, a.noise_stream, static_cast<uint64_t>(idx >> 2), z);
  const __half2 h0 = *reinterpret_cast<const __half2*>(&o.x), h1 = *reinterpret_cast<const __half2*>(&o.y);
  const __half2 n0 = __floats2half2_rn(apply_vnoise(__low2float(h0), z[0], a.vnoise),
                                       apply_vnoise(__high2float(h0), z[1], a.vnoise));
  const __half2 n1 = __floats2half2_rn(apply_vnoise(__low2float(h1), z[2], a.vnoise),
                                       apply_vnoise(__high2float(h1), z[3], a.vnoise));
  uint2 r;
  r.x = *reinterpret_cast<const uint32_t*>(&n0);
  r.y = *reinterpret_cast<const uint32_t*>(&n1);
  return r;
}

// Write the planes of 4 consecutive positions (codes q0..q3) starting at element offset dst.
// S > 0 fixes the slice count at compile time; S == 0 reads it from the arguments.
template <int KIND, int S>
__device__ __forceinline__ void store_planes4(const LevelLut<KIND>& lut, const SliceArgs& a, int64_t dst, int q0,
                                              int q1, int q2, int q3) {
  const int ns = S > 0 ? S : a.n_slices;
  if constexpr (KIND == MIB_OPERAND_E4M3) {
    // one 8-byte shared load per code: the encoded levels of all slices
    const uint2 e0 = *reinterpret_cast<const uint2*>(lut.w[q0]), e1 = *reinterpret_cast<const uint2*>(lut.w[q1]);
    const uint2 e2 = *reinterpret_cast<const uint2*>(lut.w[q2]), e3 = *reinterpret_cast<const uint2*>(lut.w[q3]);
    const uint32_t lo0 = e0.x, lo1 = e1.x, lo2 = e2.x, lo3 = e3.x;
    const uint32_t hi0 = e0.y, hi1 = e1.y, hi2 = e2.y, hi3 = e3.y;
    uint8_t* base = static_cast<uint8_t*>(a.planes) + dst;
#pragma unroll
    for (int t = 0; t < (S > 0 ? S : 8); ++t) {
      if (S == 0 && t >= ns) break;
      const uint32_t k = static_cast<uint32_t>(t & 3);
      const bool lo = t < 4;
      const uint32_t p01 = __byte_perm(lo ? lo0 : hi0, lo ? lo1 : hi1, k | ((k + 4) << 4));
      const uint32_t p23 = __byte_perm(lo ? lo2 : hi2, lo ? lo3 : hi3, k | ((k + 4) << 4));
      *reinterpret_cast<uint32_t*>(base + t * a.plane_stride) = __byte_perm(p01, p23, 0x5410);
    }
  } else {
    __half* base = static_cast<__half*>(a.planes) + dst;
    // one 16-byte shared load per code: the FP16 levels of all slices
    const uint4 e0 = *reinterpret_cast<const uint4*>(lut.w[q0]), e1 = *reinterpret_cast<const uint4*>(lut.w[q1]);
    const uint4 e2 = *reinterpret_cast<const uint4*>(lut.w[q2]), e3 = *reinterpret_cast<const uint4*>(lut.w[q3]);
    const uint32_t w0[4] = {e0.x, e0.y, e0.z, e0.w}, w1[4] = {e1.x, e1.y, e1.z, e1.w};
    const uint32_t w2[4] = {e2.x, e2.y, e2.z, e2.w}, w3[4] = {e3.x, e3.y, e3.z, e3.w};
#pragma unroll
    for (int t = 0; t < (S > 0 ? S : 8); ++t) {
      if (S == 0 && t >= ns) break;
      const int wk = t >> 1;
      const uint32_t sel = (t & 1) ? 0x7632u : 0x5410u;
      uint2 o;
      o.x = __byte_perm(w0[wk], w1[wk], sel);
      o.y = __byte_perm(w2[wk], w3[wk], sel);
      if (a.vnoise != 0.0f) o = vnoise4(o, a, t * a.plane_stride + dst);
      *reinterpret_cast<uint2*>(base + t * a.plane_stride) = o;
    }
  }
}

template <class Loader, int KIND>
__global__ void slice_rows_kernel(Loader ld, SliceArgs a, bool have_max) {
  __shared__ LevelLut<KIND> lut;
  build_level_lut<KIND>(lut, a);

  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t nitems = a.batch * a.rows * a.nbc;
  const int tiles_per_block = a.qg1 / a.p;
  for (int64_t item = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; item < nitems;
       item += nwarps) {
    const int64_t cb = item % a.nbc;
    const int64_t br = item / a.nbc;  // b * rows + r
    const int64_t b = br / a.rows, r = br - (br / a.rows) * a.rows;
    const int64_t blk = (b * a.nbr + r / a.qg0) * a.nbc + cb;
    float bm;
    if (have_max) {
      bm = a.block_max[blk];
    } else {
      float m = 0.0f;
      const int64_t c0 = cb * a.qg1;
      for (int c = lane; c < a.qg1; c += 32) m = fmaxf(m, fabsf(ld(b, r, c0 + c)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      bm = m;
      if (lane == 0) a.block_max[blk] = bm;
    }
    const int e = a.bfp ? bfp_exponent(bm) : 0;
    if (a.bfp && lane == 0 && !have_max && a.block_exp) a.block_exp[blk] = static_cast<float>(e);
    const float inv_p2e = (a.bfp && e <= 126) ? pow2f(-e) : 0.0f;
    const float scale = a.bfp ? pow2f(e + 2 - a.bits) : bm / static_cast<float>((1 << (a.bits - 1)) - 1);
    const int64_t tile0 = cb * tiles_per_block;
    const int64_t npos = static_cast<int64_t>(tiles_per_block) * a.pp;
    const int64_t row_idx = b * a.rows + r;
    const int64_t plane_row = row_idx * a.row_pitch;
    for (int64_t pos = 4 * lane; pos < npos; pos += 128) {
      int q[4];
      const int64_t tt = pos / a.pp;                    // 4 positions never straddle a tile (pp % 4 == 0)
      const int o0 = static_cast<int>(pos - tt * a.pp);
      const int64_t c0 = (tile0 + tt) * a.p + o0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool real = o0 + u < a.p;
        q[u] = real ? quantize_fast(ld(b, r, c0 + u), bm, e, inv_p2e, a.bits, a.bfp) : 0;
      }
      if (o0 == 0) a.tile_scale[(tile0 + tt) * a.scale_ld + row_idx] = scale;
      if (a.packed) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (o0 + u < a.p) a.packed[row_idx * a.kp + c0 + u] = static_cast<uint8_t>(q[u]);
      }
      store_planes4<KIND, 0>(lut, a, plane_row + tile0 * a.pp + pos, q[0], q[1], q[2], q[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Vectorised input slicing for dense rows: unit column stride, 16-byte aligned rows, K % 4 == 0
// and unpadded tiles (pp == p, so plane positions are columns).  Work item = (row, group of
// kChunks chunks of 128 columns); lane l of a chunk holds columns 4l..4l+3 as one float4, so a
// warp keeps kChunks * 512 bytes of x in flight.  Without precomputed maxima (one-row quant
// blocks, qg1 dividing 128) the block max is a butterfly over the qg1/4 lanes of the block.
// The BFP exponent (a double-precision log2) is evaluated by one lane per block and broadcast.
// ---------------------------------------------------------------------------
constexpr int kSliceVecChunks = 4;

// rne(t) for |t| < 2^22 on the FMA pipe: adding 1.5 * 2^23 leaves the rounded integer in the low mantissa bits.
__device__ __forceinline__ int rne_small(float t) {
  return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}

// fl(v / b) for |v| <= b and 2^-60 <= b < 2^126, given rb = RN(1/b), without a per-element division.
// y0 = RN(v * rb) is within 1.5 ulp of v/b; one residual correction y1 = RN(y0 + rb * (v - b * y0)) brings it
// well within one ulp, and the same step once more is Markstein's final correction (P. Markstein, IBM J. Res.
// Dev. 34(1):111-119, 1990), which returns RN(v / b) when rb = RN(1/b) and the estimate is within one ulp.
// The residuals v - b * y are exact under FMA for these magnitudes (no underflow since b >= 2^-60).
__device__ __forceinline__ float div_markstein(float v, float b, float rb) {
  float y = __fmul_rn(v, rb);
  float r = __fmaf_rn(-b, y, v);
  y = __fmaf_rn(r, rb, y);
  r = __fmaf_rn(-b, y, v);
  return __fmaf_rn(r, rb, y);
}

// quantize() for the vector path.  INT: rne(fl(fl(v / bmax) * qmax)), |t| <= qmax; the division uses
// div_markstein when rb != 0 (bmax in its range), else __fdiv_rn.  BFP: v / 2^e as quantize_fast,
// |t| <= 2^(bits-1).  Both stay far below 2^22, so rne_small rounds exactly.
__device__ __forceinline__ int quantize_vec(float v, float bmax, float rb, float qmax, int e, float inv_p2e, int bits,
                                            bool bfp) {
  int q;
  if (bfp) {
    const float s = inv_p2e != 0.0f ? __fmul_rn(v, inv_p2e) : __fdiv_rn(v, pow2f(e));
    q = rne_small(__fmul_rn(s, static_cast<float>(1 << (bits - 2))));
    q = min(max(q, -(1 << (bits - 1))), (1 << (bits - 1)) - 1);
  } else if (rb != 0.0f) {
    q = rne_small(__fmul_rn(div_markstein(v, bmax, rb), qmax));
  } else {
    q = bmax == 0.0f ? 0 : rne_small(__fmul_rn(__fdiv_rn(v, bmax), qmax));
  }
  return q & ((1 << bits) - 1);
}

// Element sources of the vector kernel.  row(b, r) prepares a per-row context once per work item;
// load4(row, col) returns columns col..col+3 of that row, zero beyond the matrix.

// Dense rows: unit column stride, 16-byte aligned rows, cols % 4 == 0 (one float4 per call).
struct DenseRowSrc {
  const float* x;
  int64_t ld_batch, ld_row;
  int cols;
  struct Row {
    const float* p;
  };
  __device__ __forceinline__ Row row(int b, int r) const {
    return {x + b * ld_batch + static_cast<int64_t>(r) * ld_row};
  }
  __device__ __forceinline__ float4 load4(const Row& w, int col) const {
    return col < cols ? __ldg(reinterpret_cast<const float4*>(w.p + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
};

// Convolution patches in F.unfold order: column c = ci*kh*kw + i*kw + j of output pixel r = oh*Wo + ow
// of image b reads x[b, ci, oh*sh - ph + i*dh, ow*sw - pw + j*dw] (zero outside the image).  One
// image holds fewer than 2^31 elements.  KH > 0 fixes a square KH x KH kernel at compile time, so the
// column decomposition is a multiply-shift; the next three columns follow by incrementing (ci, i, j).
template <int KH>
struct ConvRowSrc {
  const float* x;
  int C, H, W, Wo, kh, kw, sh, sw, ph, pw, dh, dw, cols;
  struct Row {
    const float* p;
    int ih0, iw0;
  };
  __device__ __forceinline__ Row row(int b, int r) const {
    const int oh = r / Wo, ow = r - (r / Wo) * Wo;
    return {x + static_cast<int64_t>(b) * C * H * W, oh * sh - ph, ow * sw - pw};
  }
  __device__ __forceinline__ float4 load4(const Row& w, int col) const {
    const unsigned k_h = KH > 0 ? KH : kh, k_w = KH > 0 ? KH : kw;
    const unsigned c0 = static_cast<unsigned>(col);
    unsigned ci = c0 / (k_h * k_w);
    const unsigned rem = c0 - ci * (k_h * k_w);
    unsigned i = rem / k_w, j = rem - (rem / k_w) * k_w;
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int ih = w.ih0 + static_cast<int>(i) * dh, iw = w.iw0 + static_cast<int>(j) * dw;
      const bool in = col + u < cols && static_cast<unsigned>(ih) < static_cast<unsigned>(H) &&
                      static_cast<unsigned>(iw) < static_cast<unsigned>(W);
      // unsigned: the offset of a column past the end (not loaded) may wrap
      const unsigned off = (ci * static_cast<unsigned>(H) + static_cast<unsigned>(ih)) * static_cast<unsigned>(W) +
                           static_cast<unsigned>(iw);
      v[u] = in ? __ldg(w.p + off) : 0.0f;
      if (++j == k_w) {
        j = 0;
        if (++i == k_h) {
          i = 0;
          ++ci;
        }
      }
    }
    return make_float4(v[0], v[1], v[2], v[3]);
  }
};

// Fused producers (no reference counterpart: they replace a torch pass before the slicing).

// RMSNorm of each row, y = x * rsqrt(mean(x^2) + eps) * w, evaluated in that order.  row() is
// warp-collective: the warp reduces the row's sum of squares (cols % 4 == 0, 16-byte aligned rows).
struct RmsNormRowSrc {
  const float* x;
  const float* w;
  int64_t ld_batch, ld_row;
  int cols;
  float eps;
  struct Row {
    const float* p;
    float rstd;
  };
  __device__ __forceinline__ Row row(int b, int r) const {
    const float* p = x + b * ld_batch + static_cast<int64_t>(r) * ld_row;
    float ss = 0.0f;
    for (int c = 4 * (threadIdx.x & 31); c < cols; c += 128) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p + c));
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    return {p, rsqrtf(ss / static_cast<float>(cols) + eps)};
  }
  __device__ __forceinline__ float4 load4(const Row& rw, int col) const {
    if (col >= cols) return make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 v = __ldg(reinterpret_cast<const float4*>(rw.p + col));
    const float4 g = __ldg(reinterpret_cast<const float4*>(w + col));
    return make_float4(v.x * rw.rstd * g.x, v.y * rw.rstd * g.y, v.z * rw.rstd * g.z, v.w * rw.rstd * g.w);
  }
};

// SwiGLU of a fused gate/up row, y[c] = silu(gate[c]) * up[c] with silu(g) = g / (1 + exp(-g)); gate
// columns start at 0 and up columns at up_offset of the same row (cols and up_offset % 4 == 0).
struct SwigluRowSrc {
  const float* x;
  int64_t ld_batch, ld_row, up_offset;
  int cols;
  struct Row {
    const float* p;
  };
  __device__ __forceinline__ Row row(int b, int r) const {
    return {x + b * ld_batch + static_cast<int64_t>(r) * ld_row};
  }
  __device__ __forceinline__ static float swish(float g, float u) { return g / (1.0f + expf(-g)) * u; }
  __device__ __forceinline__ float4 load4(const Row& rw, int col) const {
    if (col >= cols) return make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 g = __ldg(reinterpret_cast<const float4*>(rw.p + col));
    const float4 u = __ldg(reinterpret_cast<const float4*>(rw.p + up_offset + col));
    return make_float4(swish(g.x, u.x), swish(g.y, u.y), swish(g.z, u.z), swish(g.w, u.w));
  }
};

template <int KIND, int S, class Src>
__global__ void __launch_bounds__(256, 4) slice_vec_kernel(Src src, SliceArgs a, bool have_max) {
  __shared__ LevelLut<KIND> lut;
  build_level_lut<KIND>(lut, a);

  const int lane = threadIdx.x & 31;
  const int nwarps = static_cast<int>(gridDim.x * (blockDim.x >> 5));
  const int nrows = static_cast<int>(a.batch * a.rows);
  const int rows = static_cast<int>(a.rows);
  const int kp = static_cast<int>(a.kp);
  const int nchunks = (kp + 127) / 128;
  const int ngroups = (nchunks + kSliceVecChunks - 1) / kSliceVecChunks;
  const int nitems = nrows * ngroups;
  const int lp = __ffs(a.p) - 1, lq = __ffs(a.qg1) - 1;  // p and qg1 are powers of two here
  // lanes sharing one quant block inside a chunk: qg1/4 when qg1 divides 128, else the whole warp
  const int glanes = a.qg1 <= 128 ? a.qg1 / 4 : 32;
  const int leader = lane & ~(glanes - 1);
  const float qmax = static_cast<float>((1 << (a.bits - 1)) - 1);
  const float inv_qmax = 1.0f / qmax;
  for (int item = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; item < nitems; item += nwarps) {
    const int row_idx = item / ngroups;
    const int ch0 = (item - row_idx * ngroups) * kSliceVecChunks;
    const int b = row_idx / rows, r = row_idx - b * rows;
    const typename Src::Row rw = src.row(b, r);
    const int64_t blk_row = (static_cast<int64_t>(b) * a.nbr + (a.qg0 == 1 ? r : r / a.qg0)) * a.nbc;
    float4 v[kSliceVecChunks];
#pragma unroll
    for (int u = 0; u < kSliceVecChunks; ++u) {
      const int col = (ch0 + u) * 128 + 4 * lane;
      v[u] = src.load4(rw, col);
    }
#pragma unroll
    for (int u = 0; u < kSliceVecChunks; ++u) {
      if (ch0 + u >= nchunks) break;  // warp-uniform
      const int col = (ch0 + u) * 128 + 4 * lane;
      const bool valid = col < kp;
      const int cb = col >> lq;
      float bm;
      if (have_max) {
        bm = valid ? a.block_max[blk_row + cb] : 0.0f;
      } else {
        float m = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
          if (o < glanes) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bm = m;
      }
      int e = 0;
      float scale, rb = 0.0f;
      if (a.bfp) {
        if (lane == leader) e = bfp_exponent(bm);
        e = __shfl_sync(0xffffffffu, e, leader);
        scale = pow2f(e + 2 - a.bits);
      } else {
        scale = __fmul_rn(bm, inv_qmax);   // dequantisation factor (within one ulp of bm / qmax)
        if (bm >= 0x1p-60f && bm < 0x1p126f) rb = __frcp_rn(bm);
      }
      if (!valid) continue;
      if (!have_max && (col & (a.qg1 - 1)) == 0) {
        a.block_max[blk_row + cb] = bm;
        if (a.bfp && a.block_exp) a.block_exp[blk_row + cb] = static_cast<float>(e);
      }
      if ((col & (a.p - 1)) == 0) a.tile_scale[static_cast<int64_t>(col >> lp) * a.scale_ld + row_idx] = scale;
      const float inv_p2e = (a.bfp && e <= 126) ? pow2f(-e) : 0.0f;
      const int q0 = quantize_vec(v[u].x, bm, rb, qmax, e, inv_p2e, a.bits, a.bfp);
      const int q1 = quantize_vec(v[u].y, bm, rb, qmax, e, inv_p2e, a.bits, a.bfp);
      const int q2 = quantize_vec(v[u].z, bm, rb, qmax, e, inv_p2e, a.bits, a.bfp);
      const int q3 = quantize_vec(v[u].w, bm, rb, qmax, e, inv_p2e, a.bits, a.bfp);
      if (a.packed)
        *reinterpret_cast<uint32_t*>(a.packed + static_cast<int64_t>(row_idx) * kp + col) =
            static_cast<uint32_t>(q0) | (static_cast<uint32_t>(q1) << 8) | (static_cast<uint32_t>(q2) << 16) |
            (static_cast<uint32_t>(q3) << 24);
      store_planes4<KIND, S>(lut, a, static_cast<int64_t>(row_idx) * kp + col, q0, q1, q2, q3);
    }
  }
}

// ---------------------------------------------------------------------------
// weight programming: one thread per (column n, crossbar tile t)
// ---------------------------------------------------------------------------
template <int KIND>
__global__ void program_weight_kernel(DenseLoader ld, ProgramArgs a) {
  const int64_t total = a.n * a.kt;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = idx % a.n;
    const int64_t t = idx / a.n;
    const int64_t k0 = t * a.p;
    const int64_t blk = (k0 / a.qg0) * a.nbc + n / a.qg1;
    const float bm = a.block_max[blk];
    const int e = a.bfp ? bfp_exponent(bm) : 0;
    const float scale = a.bfp ? pow2f(e + 2 - a.bits) : bm / static_cast<float>((1 << (a.bits - 1)) - 1);
    a.tile_scale[t * a.n + n] = scale;
    const int64_t np_tiles = a.np_pad / a.p1;  // reference G layout: (Kp/p0, Np/p1, S, p0, p1)
    for (int o0 = 0; o0 < a.pp; o0 += 16) {
      int q[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int o = o0 + u;
        const int64_t k = k0 + o;
        const float v = (o < a.p) ? ld(0, k, n) : 0.0f;
        q[u] = (o < a.p) ? quantize(v, bm, e, a.bits, a.bfp) : 0;
        if (a.packed && o < a.p) a.packed[n * a.kp + k] = static_cast<uint8_t>(q[u]);
      }
      for (int j = 0; j < a.n_slices; ++j) {
        float lv[16];
        float gv[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int o = o0 + u;
          const int64_t k = k0 + o;
          const int code = (q[u] >> a.offs[j]) & a.maxes[j];
          int level = level_map(code, a.maxes[j], a.g_level - 1);
          // reference order: G = level*Q_G + LGS, write variation, then stuck-at (memmat_tensor.py:171-197)
          float g = __fadd_rn(__fmul_rn(static_cast<float>(level), a.qg_f), a.lgs_f);
          if (o < a.p && (a.stuck_field || a.write_field)) {
            const int64_t fi = (((k / a.p0) * np_tiles + n / a.p1) * a.n_slices + j) * (a.p0 * a.p1) +
                               (k % a.p0) * a.p1 + (n % a.p1);
            if (a.write_field) g = __fadd_rn(g, __fmul_rn(g, a.write_field[fi]));
            if (a.stuck_field) {
              const float rv = a.stuck_field[fi];
              if (a.rate_h > 0.0f && rv < a.rate_h) {
                level = a.g_level - 1;
                g = a.hgs_f;
              } else if (a.rate_l > 0.0f && rv >= a.rate_h && rv < a.rate_hl) {
                level = 0;
                g = a.lgs_f;
              }
            }
          }
          lv[u] = (o < a.p) ? static_cast<float>(level) : 0.0f;
          gv[u] = (o < a.p) ? g : a.lgs_f;
        }
        const int64_t dst = (j * a.n + n) * a.row_pitch + t * a.pp + o0;
        if constexpr (KIND == MIB_OPERAND_E4M3) {
          uint32_t w4[4];
#pragma unroll
          for (int v = 0; v < 4; ++v)
            w4[v] = static_cast<uint32_t>(enc_e4m3(lv[4 * v])) | (static_cast<uint32_t>(enc_e4m3(lv[4 * v + 1])) << 8) |
                    (static_cast<uint32_t>(enc_e4m3(lv[4 * v + 2])) << 16) |
                    (static_cast<uint32_t>(enc_e4m3(lv[4 * v + 3])) << 24);
          *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.planes) + dst) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        } else {
          __half2* p2 = reinterpret_cast<__half2*>(static_cast<__half*>(a.planes) + dst);
#pragma unroll
          for (int v = 0; v < 8; ++v) p2[v] = __floats2half2_rn(lv[2 * v], lv[2 * v + 1]);
        }
        if (a.g_planes) {
          float4* g4 = reinterpret_cast<float4*>(a.g_planes + dst);
#pragma unroll
          for (int v = 0; v < 4; ++v) g4[v] = make_float4(gv[4 * v], gv[4 * v + 1], gv[4 * v + 2], gv[4 * v + 3]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// per-call noise pre-passes
// ---------------------------------------------------------------------------
// 8 elements per thread: E4M3 levels in, FP16 levels * (1 + vnoise*N) out.
__global__ void input_noise_kernel(const uint8_t* __restrict__ in, __half* __restrict__ out, int64_t n8, float vnoise,
                                   uint64_t seed, uint64_t stream) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint2 raw = reinterpret_cast<const uint2*>(in)[i];
    float v[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = dec_e4m3(static_cast<uint8_t>(raw.x >> (8 * u)));
      v[4 + u] = dec_e4m3(static_cast<uint8_t>(raw.y >> (8 * u)));
    }
    if (vnoise != 0.0f) {
      float z0[4], z1[4];
      normal4(seed, stream, 2 * static_cast<uint64_t>(i), z0);
      normal4(seed, stream, 2 * static_cast<uint64_t>(i) + 1, z1);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        v[u] = apply_vnoise(v[u], z0[u], vnoise);
        v[4 + u] = apply_vnoise(v[4 + u], z1[u], vnoise);
      }
    }
    __half2 h[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) h[u] = __floats2half2_rn(v[2 * u], v[2 * u + 1]);
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(h);
  }
}

// Read variation of one group of 4 cells (memmat_tensor.py:204-236): G' = G exp(sigma z) with one standard
// normal z per cell (Philox group `grp`), output (G' - LGS) / Q_G as FP16.  From an E4M3 level L
// (G = L Q_G + LGS) the output is L e + (LGS / Q_G)(e - 1) with e = exp(sigma z): no division, and L
// itself indexes a per-level sigma (the reference recovers it as round((G - LGS) / Q_G)).  Conductance
// planes (write variation present) go through G directly.
__device__ __forceinline__ void read_noise_group(uint32_t lv_raw, const float* __restrict__ gp, int64_t grp,
                                                 const ReadNoiseArgs& a, uint64_t seed, uint64_t stream,
                                                 float (&o)[4]) {
  float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (a.any_sigma) normal4(seed, stream, static_cast<uint64_t>(grp), z);
  if (gp) {
    const float4 g4 = reinterpret_cast<const float4*>(gp)[grp];
    const float g[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float gg = g[u];
      if (a.any_sigma) {
        float sigma = a.sigma[0];
        if (a.per_level) {
          int lv = static_cast<int>(rintf((gg - a.lgs_f) / a.qg_f));
          sigma = a.sigma[min(max(lv, 0), a.g_level - 1)];
        }
        gg = gg * __expf(z[u] * sigma);  // approximate hardware exp: the noise is statistical
      }
      o[u] = (gg - a.lgs_f) * a.inv_qg;
    }
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float L = dec_e4m3(static_cast<uint8_t>(lv_raw >> (8 * u)));
      if (a.any_sigma) {
        const float sigma = a.per_level ? a.sigma[min(static_cast<int>(L), a.g_level - 1)] : a.sigma[0];
        const float e = __expf(z[u] * sigma);
        o[u] = fmaf(L, e, a.lgs_over_qg * (e - 1.0f));
      } else {
        o[u] = L;
      }
    }
  }
}

// FP16 of 4 values, and (lo) of what that rounding left out: hi + lo carries 22 significand bits.
__device__ __forceinline__ uint2 half4_hi(const float (&o)[4]) {
  const __half2 h0 = __floats2half2_rn(o[0], o[1]), h1 = __floats2half2_rn(o[2], o[3]);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
}
__device__ __forceinline__ uint2 half4_lo(const float (&o)[4], uint2 hi) {
  const __half2 h0 = *reinterpret_cast<const __half2*>(&hi.x), h1 = *reinterpret_cast<const __half2*>(&hi.y);
  const __half2 l0 = __floats2half2_rn(o[0] - __low2float(h0), o[1] - __high2float(h0));
  const __half2 l1 = __floats2half2_rn(o[2] - __low2float(h1), o[3] - __high2float(h1));
  return make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
}

// Two 4-cell groups per thread (8 B of levels in, 16 B of FP16 out) when the buffers allow the wide
// accesses, else one group per thread.  Group g always draws Philox block g, so both forms give the
// same values.
// With out_lo (the weight operand split into FP16 hi and lo planes), the residual of every value's FP16
// rounding goes to out_lo at the same index.
template <bool WIDE>
__global__ void read_noise_kernel(const uint8_t* __restrict__ levels, const float* __restrict__ gp,
                                  __half* __restrict__ out, __half* __restrict__ out_lo, int64_t n4, ReadNoiseArgs a,
                                  uint64_t seed, uint64_t stream) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  float o0[4], o1[4];
  if constexpr (WIDE) {
    const int64_t n8 = n4 / 2;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += step) {
      uint2 raw = make_uint2(0u, 0u);
      if (!gp) raw = reinterpret_cast<const uint2*>(levels)[i];
      read_noise_group(raw.x, gp, 2 * i, a, seed, stream, o0);
      read_noise_group(raw.y, gp, 2 * i + 1, a, seed, stream, o1);
      const uint2 h0 = half4_hi(o0), h1 = half4_hi(o1);
      reinterpret_cast<uint4*>(out)[i] = make_uint4(h0.x, h0.y, h1.x, h1.y);
      if (out_lo) {
        const uint2 l0 = half4_lo(o0, h0), l1 = half4_lo(o1, h1);
        reinterpret_cast<uint4*>(out_lo)[i] = make_uint4(l0.x, l0.y, l1.x, l1.y);
      }
    }
    if ((n4 & 1) && blockIdx.x == 0 && threadIdx.x == 0) {
      const int64_t g = n4 - 1;
      const uint32_t raw = gp ? 0u : reinterpret_cast<const uint32_t*>(levels)[g];
      read_noise_group(raw, gp, g, a, seed, stream, o0);
      const uint2 h0 = half4_hi(o0);
      reinterpret_cast<uint2*>(out)[g] = h0;
      if (out_lo) reinterpret_cast<uint2*>(out_lo)[g] = half4_lo(o0, h0);
    }
  } else {
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < n4; g += step) {
      const uint32_t raw = gp ? 0u : reinterpret_cast<const uint32_t*>(levels)[g];
      read_noise_group(raw, gp, g, a, seed, stream, o0);
      const uint2 h0 = half4_hi(o0);
      reinterpret_cast<uint2*>(out)[g] = h0;
      if (out_lo) reinterpret_cast<uint2*>(out_lo)[g] = half4_lo(o0, h0);
    }
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
static int grid_for(int64_t work_items, int per_block) {
  int64_t g = (work_items + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > 148 * 64) g = 148 * 64;
  return static_cast<int>(g);
}

template <int KIND, class Src>
static void launch_slice_vec_k(const Src& src, const SliceArgs& a, int grid, bool have_max, cudaStream_t stream) {
  switch (a.n_slices) {
    case 1: slice_vec_kernel<KIND, 1, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    case 2: slice_vec_kernel<KIND, 2, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    case 3: slice_vec_kernel<KIND, 3, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    case 4: slice_vec_kernel<KIND, 4, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    case 5: slice_vec_kernel<KIND, 5, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    case 6: slice_vec_kernel<KIND, 6, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    case 7: slice_vec_kernel<KIND, 7, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
    default: slice_vec_kernel<KIND, 8, Src><<<grid, 256, 0, stream>>>(src, a, have_max); break;
  }
}

template <class Src>
static void launch_slice_vec(const Src& src, const SliceArgs& a, int grid, bool have_max, cudaStream_t stream) {
  if (a.kind == MIB_OPERAND_E4M3)
    launch_slice_vec_k<MIB_OPERAND_E4M3>(src, a, grid, have_max, stream);
  else
    launch_slice_vec_k<MIB_OPERAND_FP16>(src, a, grid, have_max, stream);
}

// The vector kernel needs unpadded power-of-two tiles and power-of-two quant blocks, index ranges that
// fit 32-bit arithmetic, and a fused max only when a quant block fits one 128-column chunk.
static bool slice_vec_eligible(const SliceArgs& a) {
  auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
  const int64_t groups = ((a.kp + 127) / 128 + kSliceVecChunks - 1) / kSliceVecChunks;
  return a.p == a.pp && a.p >= 4 && pow2(a.p) && pow2(a.qg1) && a.kp == a.row_pitch &&
         a.kp < (int64_t{1} << 30) && a.batch * a.rows * groups < (int64_t{1} << 30) &&
         (a.qg0 != 1 || a.qg1 <= 128);
}

template <class Loader, class Src>
static cudaError_t launch_slice_vec_path(const Loader& ld, const Src& src, SliceArgs a, cudaStream_t stream) {
  const bool one_row = (a.qg0 == 1);
  if (!one_row) {
    block_absmax_kernel<<<grid_for(a.batch * a.nbr * a.nbc, 8), 256, 0, stream>>>(ld, a.batch, a.rows, a.cols, a.qg0,
                                                                                   a.qg1, a.nbr, a.nbc, a.block_max);
    count_launch();
  }
  const int64_t groups = ((a.kp + 127) / 128 + kSliceVecChunks - 1) / kSliceVecChunks;
  int64_t g = (a.batch * a.rows * groups + 7) / 8;
  g = g < 1 ? 1 : (g > 148 * 4 ? 148 * 4 : g);
  launch_slice_vec(src, a, static_cast<int>(g), !one_row, stream);
  count_launch();
  if (!one_row && a.bfp && a.block_exp) launch_block_exp(a.block_max, a.block_exp, a.batch * a.nbr * a.nbc, stream);
  return cudaGetLastError();
}

template <class Loader>
static cudaError_t launch_slice(const Loader& ld, SliceArgs a, cudaStream_t stream) {
  const bool one_row = (a.qg0 == 1);
  if constexpr (std::is_same<Loader, DenseLoader>::value) {
    // dense rows: unit column stride and 16-byte aligned rows for the float4 loads
    if (slice_vec_eligible(a) && ld.ld_col == 1 && (reinterpret_cast<uintptr_t>(ld.x) & 15) == 0 &&
        ld.ld_row % 4 == 0 && ld.ld_batch % 4 == 0 && a.cols % 4 == 0)
      return launch_slice_vec_path(ld, DenseRowSrc{ld.x, ld.ld_batch, ld.ld_row, static_cast<int>(a.cols)}, a,
                                   stream);
  } else {
    // convolution patches: one image in 32-bit indexing
    if (slice_vec_eligible(a) && ld.C * ld.H * ld.W < (int64_t{1} << 31) && ld.Wo > 0) {
      auto conv_src = [&](auto kh) {
        using Src = ConvRowSrc<decltype(kh)::value>;
        return Src{ld.x, static_cast<int>(ld.C), static_cast<int>(ld.H), static_cast<int>(ld.W),
                   static_cast<int>(ld.Wo), ld.kh, ld.kw, ld.sh, ld.sw, ld.ph, ld.pw, ld.dh, ld.dw,
                   static_cast<int>(a.cols)};
      };
      if (ld.kh == 3 && ld.kw == 3)
        return launch_slice_vec_path(ld, conv_src(std::integral_constant<int, 3>{}), a, stream);
      if (ld.kh == 1 && ld.kw == 1)
        return launch_slice_vec_path(ld, conv_src(std::integral_constant<int, 1>{}), a, stream);
      return launch_slice_vec_path(ld, conv_src(std::integral_constant<int, 0>{}), a, stream);
    }
  }
  if (!one_row) {
    block_absmax_kernel<<<grid_for(a.batch * a.nbr * a.nbc, 8), 256, 0, stream>>>(ld, a.batch, a.rows, a.cols, a.qg0,
                                                                                   a.qg1, a.nbr, a.nbc, a.block_max);
    count_launch();
  }
  const int grid = grid_for(a.batch * a.rows * a.nbc, 8);
  if (a.kind == MIB_OPERAND_E4M3)
    slice_rows_kernel<Loader, MIB_OPERAND_E4M3><<<grid, 256, 0, stream>>>(ld, a, !one_row);
  else
    slice_rows_kernel<Loader, MIB_OPERAND_FP16><<<grid, 256, 0, stream>>>(ld, a, !one_row);
  count_launch();
  if (!one_row && a.bfp && a.block_exp) launch_block_exp(a.block_max, a.block_exp, a.batch * a.nbr * a.nbc, stream);
  return cudaGetLastError();
}

__global__ void block_exp_kernel(const float* __restrict__ bmax, float* __restrict__ bexp, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    bexp[i] = static_cast<float>(bfp_exponent(bmax[i]));
}

void launch_block_exp(const float* bmax, float* bexp, int64_t n, cudaStream_t stream) {
  block_exp_kernel<<<grid_for(n, 256), 256, 0, stream>>>(bmax, bexp, n);
  count_launch();
}

cudaError_t slice_dense(const float* x, int64_t ld_batch, int64_t ld_row, SliceArgs a, cudaStream_t stream) {
  DenseLoader ld{x, ld_batch, ld_row, 1, a.rows, a.cols};
  return launch_slice(ld, a, stream);
}

// Fused producers: only the vector path (16-byte aligned rows, cols % 4 == 0, one-row quant blocks).
static bool fused_eligible(const void* x, int64_t ld_batch, int64_t ld_row, const SliceArgs& a) {
  return slice_vec_eligible(a) && a.qg0 == 1 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ld_row % 4 == 0 &&
         ld_batch % 4 == 0 && a.cols % 4 == 0;
}

cudaError_t slice_rmsnorm(const float* x, int64_t ld_batch, int64_t ld_row, const float* w, float eps, SliceArgs a,
                          cudaStream_t stream) {
  if (!fused_eligible(x, ld_batch, ld_row, a) || (reinterpret_cast<uintptr_t>(w) & 15) != 0)
    return cudaErrorNotSupported;
  DenseLoader ld{x, ld_batch, ld_row, 1, a.rows, a.cols};
  return launch_slice_vec_path(ld, RmsNormRowSrc{x, w, ld_batch, ld_row, static_cast<int>(a.cols), eps}, a, stream);
}

cudaError_t slice_swiglu(const float* x, int64_t ld_batch, int64_t ld_row, int64_t up_offset, SliceArgs a,
                         cudaStream_t stream) {
  if (!fused_eligible(x, ld_batch, ld_row, a) || up_offset % 4 != 0) return cudaErrorNotSupported;
  DenseLoader ld{x, ld_batch, ld_row, 1, a.rows, a.cols};
  return launch_slice_vec_path(ld, SwigluRowSrc{x, ld_batch, ld_row, up_offset, static_cast<int>(a.cols)}, a,
                               stream);
}

cudaError_t slice_conv(const float* x, int64_t C, int64_t H, int64_t W, int64_t Ho, int64_t Wo, int kh, int kw, int sh,
                       int sw, int ph, int pw, int dh, int dw, SliceArgs a, cudaStream_t stream) {
  ConvLoader ld{x, C, H, W, Ho, Wo, a.rows, a.cols, kh, kw, sh, sw, ph, pw, dh, dw};
  return launch_slice(ld, a, stream);
}

cudaError_t program_weight(const float* w, int64_t stride_k, int64_t stride_n, ProgramArgs a, cudaStream_t stream) {
  DenseLoader ld{w, 0, stride_k, stride_n, a.k, a.n};
  block_absmax_kernel<<<grid_for(a.nbr * a.nbc, 8), 256, 0, stream>>>(ld, 1, a.k, a.n, a.qg0, a.qg1, a.nbr, a.nbc,
                                                                      a.block_max);
  count_launch();
  if (a.bfp && a.block_exp) launch_block_exp(a.block_max, a.block_exp, a.nbr * a.nbc, stream);
  const int grid = grid_for(a.n * a.kt, 128);
  if (a.kind == MIB_OPERAND_E4M3)
    program_weight_kernel<MIB_OPERAND_E4M3><<<grid, 128, 0, stream>>>(ld, a);
  else
    program_weight_kernel<MIB_OPERAND_FP16><<<grid, 128, 0, stream>>>(ld, a);
  count_launch();
  return cudaGetLastError();
}

cudaError_t input_noise(const uint8_t* in, __half* out, int64_t n, float vnoise, uint64_t seed, uint64_t stream_id,
                        cudaStream_t stream) {
  const int64_t n8 = n / 8;
  input_noise_kernel<<<grid_for(n8, 256), 256, 0, stream>>>(in, out, n8, vnoise, seed, stream_id);
  count_launch();
  return cudaGetLastError();
}

cudaError_t read_noise(const uint8_t* levels, const float* gp, __half* out, __half* out_lo, int64_t n,
                       ReadNoiseArgs a, uint64_t seed, uint64_t stream_id, int background_blocks,
                       cudaStream_t stream) {
  const int64_t n4 = n / 4;
  const bool wide = (reinterpret_cast<uintptr_t>(levels) % 8 == 0) && (reinterpret_cast<uintptr_t>(gp) % 32 == 0) &&
                    (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (reinterpret_cast<uintptr_t>(out_lo) % 16 == 0);
  // background: at most `background_blocks` blocks of 128 threads stepping through the cells, small
  // enough (4 warps, at most 64 registers a thread, no shared memory) to run beside a crossbar MVM CTA
  const int threads = background_blocks > 0 ? 128 : 256;
  auto grid = [&](int64_t items) {
    const int g = grid_for(items, threads);
    return background_blocks > 0 && g > background_blocks ? background_blocks : g;
  };
  if (wide)
    read_noise_kernel<true><<<grid(n4 / 2 + 1), threads, 0, stream>>>(levels, gp, out, out_lo, n4, a, seed, stream_id);
  else
    read_noise_kernel<false><<<grid(n4), threads, 0, stream>>>(levels, gp, out, out_lo, n4, a, seed, stream_id);
  count_launch();
  return cudaGetLastError();
}

}  // namespace mib
