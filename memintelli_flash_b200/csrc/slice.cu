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
// ---------------------------------------------------------------------------
template <class Loader, int KIND>
__global__ void slice_rows_kernel(Loader ld, SliceArgs a, bool have_max) {
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
    const float scale = a.bfp ? pow2f(e + 2 - a.bits) : bm / static_cast<float>((1 << (a.bits - 1)) - 1);
    const int64_t tile0 = cb * tiles_per_block;
    const int64_t npos = static_cast<int64_t>(tiles_per_block) * a.pp;
    const int64_t plane_row = (b * a.rows + r) * a.row_pitch;
    for (int64_t pos = 4 * lane; pos < npos; pos += 128) {
      int q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t tp = pos + u;
        const int64_t tt = tp / a.pp;
        const int o = static_cast<int>(tp - tt * a.pp);
        const int64_t c = (tile0 + tt) * a.p + o;
        const float v = (o < a.p) ? ld(b, r, c) : 0.0f;
        q[u] = (o < a.p) ? quantize(v, bm, e, a.bits, a.bfp) : 0;
        if (o == 0) a.tile_scale[(tile0 + tt) * a.scale_ld + (b * a.rows + r)] = scale;
        if (a.packed && o < a.p) a.packed[(b * a.rows + r) * a.kp + c] = static_cast<uint8_t>(q[u]);
      }
      const int64_t dst = plane_row + tile0 * a.pp + pos;
      for (int t = 0; t < a.n_slices; ++t) {
        float lv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int code = (q[u] >> a.offs[t]) & a.maxes[t];
          lv[u] = static_cast<float>(level_map(code, a.maxes[t], a.lm1));
        }
        if constexpr (KIND == MIB_OPERAND_E4M3) {
          uchar4 o4 = make_uchar4(enc_e4m3(lv[0]), enc_e4m3(lv[1]), enc_e4m3(lv[2]), enc_e4m3(lv[3]));
          *reinterpret_cast<uchar4*>(static_cast<uint8_t*>(a.planes) + t * a.plane_stride + dst) = o4;
        } else {
          __half2 h01 = __floats2half2_rn(lv[0], lv[1]), h23 = __floats2half2_rn(lv[2], lv[3]);
          __half2* p2 = reinterpret_cast<__half2*>(static_cast<__half*>(a.planes) + t * a.plane_stride + dst);
          p2[0] = h01;
          p2[1] = h23;
        }
      }
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
        v[u] = v[u] * (1.0f + z0[u] * vnoise);
        v[4 + u] = v[4 + u] * (1.0f + z1[u] * vnoise);
      }
    }
    __half2 h[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) h[u] = __floats2half2_rn(v[2 * u], v[2 * u + 1]);
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(h);
  }
}

// 4 elements per thread: conductance from levels (or fp32 G planes), read
// variation G*exp(sigma*N), output (G' - LGS)/Q_G as FP16.
__global__ void read_noise_kernel(const uint8_t* __restrict__ levels, const float* __restrict__ gp,
                                  __half* __restrict__ out, int64_t n4, ReadNoiseArgs a, uint64_t seed,
                                  uint64_t stream) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float g[4];
    if (gp) {
      const float4 g4 = reinterpret_cast<const float4*>(gp)[i];
      g[0] = g4.x;
      g[1] = g4.y;
      g[2] = g4.z;
      g[3] = g4.w;
    } else {
      const uint32_t raw = reinterpret_cast<const uint32_t*>(levels)[i];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        g[u] = __fadd_rn(__fmul_rn(dec_e4m3(static_cast<uint8_t>(raw >> (8 * u))), a.qg_f), a.lgs_f);
    }
    if (a.any_sigma) {
      float z[4];
      normal4(seed, stream, static_cast<uint64_t>(i), z);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float sigma = a.sigma[0];
        if (a.per_level) {
          int lv = static_cast<int>(rintf((g[u] - a.lgs_f) / a.qg_f));
          lv = min(max(lv, 0), a.g_level - 1);
          sigma = a.sigma[lv];
        }
        g[u] = g[u] * expf(z[u] * sigma);
      }
    }
    __half2 h0 = __floats2half2_rn((g[0] - a.lgs_f) / a.qg_f, (g[1] - a.lgs_f) / a.qg_f);
    __half2 h1 = __floats2half2_rn((g[2] - a.lgs_f) / a.qg_f, (g[3] - a.lgs_f) / a.qg_f);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    reinterpret_cast<uint2*>(out)[i] = o;
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

template <class Loader>
static cudaError_t launch_slice(const Loader& ld, SliceArgs a, cudaStream_t stream) {
  const bool one_row = (a.qg0 == 1);
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

cudaError_t read_noise(const uint8_t* levels, const float* gp, __half* out, int64_t n, ReadNoiseArgs a, uint64_t seed,
                       uint64_t stream_id, cudaStream_t stream) {
  const int64_t n4 = n / 4;
  read_noise_kernel<<<grid_for(n4, 256), 256, 0, stream>>>(levels, gp, out, n4, a, seed, stream_id);
  count_launch();
  return cudaGetLastError();
}

}  // namespace mib
