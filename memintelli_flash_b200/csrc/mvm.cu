// Fused crossbar MVM on tcgen05 tensor cores.
//
// Computes, for one 128x128 output tile per CTA,
//   y[r,n] = sum_t  xs[t,r] * ws[t,n] * sum_{i,j} ADC_j( S_ij[r,t,n] ) * w_ij
// with S_ij[r,t,n] = sum_{k in tile t} A_i[r,k] * L_j[k,n] (exact crossbar sum),
// ADC_j(S) = round_half_even(S * (radc_j - 1) / D) and w_ij = m_i m_j c_i c_j * p/(radc-1),
// i.e. DPETensor._dot_inference (memmat_tensor.py:260-409) without ever writing
// the per slice-pair partial tensor to HBM.
//
// Warp roles (320 threads, one CTA per SM):
//   warps 0-7  epilogue: tcgen05.ld of each slice-pair accumulator, ADC,
//              shift-add, per-tile rescale, output store
//   warp 8     TMA producer (all slices of A and B for one K tile per stage)
//   warp 9     MMA issuer: one tcgen05.mma chain per (K tile, slice pair) into
//              one of 4 TMEM slots of 128 fp32 columns
#include "common.cuh"
#include "kernels.cuh"

namespace mib {

namespace {

constexpr int kEpiWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kSlots = 4;
constexpr int kTmemCols = 512;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: x + magic rounds x to an integer (half-even)
constexpr uint32_t kMagicBits = 0x4B400000u;

struct SmemCtl {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tfull[kSlots];
  uint64_t tempty[kSlots];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  const bool ok = mbar_wait(bar, parity, abort, code);
  return __all_sync(0xffffffffu, ok);
}

template <int KIND, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    mvm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ MvmArgs P) {
  constexpr bool kLut = (MODE & MODE_LUT) != 0;
  constexpr bool kFloatAcc = (MODE & MODE_FLOATACC) != 0;
  constexpr bool kDump = (MODE & MODE_DUMP) != 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [stages x stage_bytes] operand ring | [128 cols][128 rows] fp32 output tile | control | code table
  float* out_s = reinterpret_cast<float*>(smem + static_cast<size_t>(P.stages) * P.stage_bytes);
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(out_s + kMvmBM * kMvmBN);
  int32_t* lut_s = reinterpret_cast<int32_t*>(ctl + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kMvmBM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kMvmBN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&ctl->tfull[s], 1);
      mbar_init(&ctl->tempty[s], kEpiWarps);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if constexpr (kLut) {
    if (P.lut_smem)
      for (int i = threadIdx.x; i < P.Sy * P.lut_len; i += blockDim.x) lut_s[i] = P.lut[i];
  }
  if (warp == kProducerWarp) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int64_t issued = 0;
      for (int64_t t = 0; t < P.Kt; ++t) {
        const int s = static_cast<int>(t % P.stages);
        const uint32_t use = static_cast<uint32_t>(t / P.stages);
        if (t >= P.stages && !mbar_wait(&ctl->empty[s], (use - 1) & 1, abort, 11)) break;
        uint8_t* a_dst = smem + static_cast<size_t>(s) * P.stage_bytes;
        uint8_t* b_dst = a_dst + static_cast<size_t>(P.Sx) * P.a_slice_bytes;
        mbar_arrive_expect_tx(&ctl->full[s], P.stage_bytes);
        tma_load_3d(a_dst, &tma_a, &ctl->full[s], static_cast<int>(t * P.pp), static_cast<int>(m0), 0);
        tma_load_3d(b_dst, &tma_b, &ctl->full[s], static_cast<int>(t * P.pp), static_cast<int>(n0), 0);
        issued = t + 1;
      }
      // no TMA write may still be in flight when the CTA exits
      const int64_t first = issued > P.stages ? issued - P.stages : 0;
      for (int64_t t = first; t < issued; ++t)
        mbar_wait_drain(&ctl->full[t % P.stages], static_cast<uint32_t>(t / P.stages) & 1, 12);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc = instr_desc_m128(kMvmBN);
      const int ksteps = P.row_bytes / 32;
      int64_t g = 0;
      bool ok = true;
      for (int64_t t = 0; t < P.Kt && ok; ++t) {
        const int s = static_cast<int>(t % P.stages);
        if (!mbar_wait(&ctl->full[s], static_cast<uint32_t>(t / P.stages) & 1, abort, 21)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + static_cast<size_t>(s) * P.stage_bytes);
        const uint32_t b_base = a_base + P.Sx * P.a_slice_bytes;
        for (int i = 0; i < P.Sx && ok; ++i) {
          for (int j = 0; j < P.Sy; ++j, ++g) {
            const int slot = static_cast<int>(g % kSlots);
            if (g >= kSlots &&
                !mbar_wait(&ctl->tempty[slot], static_cast<uint32_t>(g / kSlots - 1) & 1, abort, 22)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + slot * kMvmBN;
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint64_t ad = smem_desc(a_base + i * P.a_slice_bytes + kk * 32, P.row_bytes);
              const uint64_t bd = smem_desc(b_base + j * P.b_slice_bytes + kk * 32, P.row_bytes);
              tc_mma<KIND>(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
            }
            tc_commit(&ctl->tfull[slot]);
          }
        }
        if (ok) tc_commit(&ctl->empty[s]);
      }
      // every issued MMA has completed before TMEM is released
      tc_commit(&ctl->drain);
      mbar_wait_drain(&ctl->drain, 0, 23);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int cb = (warp >> 2) * 64;  // 64-column half of the tile
    const int64_t row = m0 + q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + cb;
    // output accumulators live in shared memory, column-major, so lanes (rows) hit consecutive words
    float* out_col = out_s + static_cast<size_t>(cb) * kMvmBM + q * 32 + lane;
    uint32_t acc[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      acc[c] = 0u;
      out_col[c * kMvmBM] = 0.0f;
    }
    int64_t g = 0;
    int cnt = 0;
    bool ok = true;
    for (int64_t t = 0; t < P.Kt && ok; ++t) {
      for (int i = 0; i < P.Sx && ok; ++i) {
        for (int j = 0; j < P.Sy; ++j, ++g) {
          const int slot = static_cast<int>(g % kSlots);
          if (!warp_wait(&ctl->tfull[slot], static_cast<uint32_t>(g / kSlots) & 1, abort, 31)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float cj = P.cadc[j];
          const uint32_t wij = static_cast<uint32_t>(P.wpair[i * 8 + j]);
          const float wfij = P.wfpair[i * 8 + j];
          const int32_t* lut_j = (P.lut_smem ? lut_s : P.lut) + j * P.lut_len;
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            uint32_t r[32];
            tmem_ld32(lane_addr + slot * kMvmBN + ch * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float sv = __uint_as_float(r[c]);
              if constexpr (kLut) {
                const int idx = static_cast<int>(__float_as_uint(sv + kMagic) - kMagicBits);
                const int32_t code = lut_j[min(max(idx, 0), P.lut_len - 1)];
                if constexpr (kFloatAcc)
                  acc[ch * 32 + c] = __float_as_uint(fmaf(static_cast<float>(code), wfij, __uint_as_float(acc[ch * 32 + c])));
                else
                  acc[ch * 32 + c] += wij * static_cast<uint32_t>(code);
              } else {
                const float tq = fmaf(sv, cj, kMagic);
                if constexpr (kFloatAcc)
                  acc[ch * 32 + c] = __float_as_uint(fmaf(tq - kMagic, wfij, __uint_as_float(acc[ch * 32 + c])));
                else
                  acc[ch * 32 + c] += wij * __float_as_uint(tq);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->tempty[slot]);
        }
      }
      if (!ok) break;
      ++cnt;
      if (kDump || cnt == P.flush_tiles || t == P.Kt - 1) {
        const float xsv = row < P.M ? __ldg(P.xs + t * P.M + row) : 0.0f;
        const float rs = kFloatAcc ? xsv : xsv * P.out_scale;
        const uint32_t off = (kLut || kFloatAcc) ? 0u : static_cast<uint32_t>(cnt) * P.tile_offset;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int64_t n = n0 + cb + c;
          const float wsv = n < P.N ? __ldg(P.ws + t * P.N + n) : 0.0f;
          float v;
          if constexpr (kFloatAcc) {
            v = __uint_as_float(acc[c]);
          } else {
            const int32_t iv = static_cast<int32_t>(acc[c] - off);
            if constexpr (kDump) {
              if (row < P.M && n < P.N) P.acc_dump[(t * P.M + row) * P.N + n] = iv;
            }
            v = static_cast<float>(iv);
          }
          out_col[c * kMvmBM] = fmaf(v, rs * wsv, out_col[c * kMvmBM]);
          acc[c] = 0u;
        }
        cnt = 0;
      }
    }
    if (ok && row < P.M) {
      const int64_t grp = row / P.rows_per_group;
      const int64_t rr = row - grp * P.rows_per_group;
      float* yb = P.y + grp * P.group_stride + rr * P.row_stride;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int64_t n = n0 + cb + c;
        if (n < P.N) yb[n * P.col_stride] = out_col[c * kMvmBM] + (P.bias ? __ldg(P.bias + n) : 0.0f);
      }
    }
  }

  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int KIND, int MODE>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, size_t smem,
                       cudaStream_t stream) {
  auto fn = mvm_kernel<KIND, MODE>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid(static_cast<unsigned>((a.N + kMvmBN - 1) / kMvmBN), static_cast<unsigned>((a.M + kMvmBM - 1) / kMvmBM));
  fn<<<grid, kThreads, smem, stream>>>(ta, tb, a);
  count_launch();
  return cudaGetLastError();
}

template <int KIND>
cudaError_t launch_kind(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, int mode, size_t smem,
                        cudaStream_t stream) {
  switch (mode) {
    case 0: return launch_one<KIND, 0>(ta, tb, a, smem, stream);
    case MODE_LUT: return launch_one<KIND, MODE_LUT>(ta, tb, a, smem, stream);
    case MODE_FLOATACC: return launch_one<KIND, MODE_FLOATACC>(ta, tb, a, smem, stream);
    case MODE_LUT | MODE_FLOATACC: return launch_one<KIND, MODE_LUT | MODE_FLOATACC>(ta, tb, a, smem, stream);
    case MODE_DUMP: return launch_one<KIND, MODE_DUMP>(ta, tb, a, smem, stream);
    case MODE_DUMP | MODE_LUT: return launch_one<KIND, MODE_DUMP | MODE_LUT>(ta, tb, a, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t mvm_smem_bytes(const MvmArgs& a) {
  return 1024 + static_cast<size_t>(a.stages) * a.stage_bytes + sizeof(float) * kMvmBM * kMvmBN + sizeof(SmemCtl) +
         (a.lut_smem ? static_cast<size_t>(a.Sy) * a.lut_len * sizeof(int32_t) : 0);
}

cudaError_t launch_mvm(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, int kind, int mode,
                       cudaStream_t stream) {
  const size_t smem = mvm_smem_bytes(a);
  if (kind == MIB_OPERAND_E4M3) return launch_kind<MIB_OPERAND_E4M3>(ta, tb, a, mode, smem, stream);
  return launch_kind<MIB_OPERAND_FP16>(ta, tb, a, mode, smem, stream);
}

}  // namespace mib
