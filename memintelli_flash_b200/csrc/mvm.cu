// Fused crossbar MVM on tcgen05 tensor cores.
//
// For one 128 x BN output tile per CTA it computes
//   y[r,n] = sum_t  xs[t,r] * ws[t,n] * sum_{i,j} ADC_j( S_ij[r,t,n] ) * w_ij
// with S_ij[r,t,n] = sum_{k in tile t} A_i[r,k] * L_j[k,n] (exact crossbar sum),
// ADC_j(S) = round_half_even(S * (radc_j - 1) / D) and w_ij = m_i m_j c_i c_j * p/(radc-1),
// i.e. DPETensor._dot_inference (memmat_tensor.py:260-409), without writing the
// per slice-pair partial tensor anywhere.
//
// One tcgen05.mma chain per (K tile t, input slice i) covers every weight slice j
// at once: the Sy weight-slice tiles of a stage sit back to back in shared
// memory, so B is one K-major operand of Sy*BN rows and the accumulator is a
// 128 x (Sy*BN) fp32 block of tensor memory.  Two such slots alternate.
//
// Launches without split-K are persistent: 148 CTAs (one per SM) step through the output tiles.
//
// Warp roles (one CTA per SM):
//   warps 0 .. 4*CG-1  epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows) and
//                      columns 16*(w/4).. of every weight slice; ADC, shift-add,
//                      per-tile rescale, output store
//   warp 4*CG          TMA producer (all slices of A and B for one K tile per stage)
//   warp 4*CG+1        MMA issuer
#include "common.cuh"
#include "kernels.cuh"

#include <atomic>

namespace mib {

namespace {

constexpr int kSlots = 2;
constexpr int kTmemCols = 512;
constexpr int kSlotCols = 256;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: x + magic rounds x to an integer (half-even)
constexpr uint32_t kMagicBits = 0x4B400000u;

// Order in which a persistent launch steps through the output tiles: bands of `band` row tiles, each
// band column by column (row tiles fastest).  band = 1 is row by row.  With wider bands the SMs work on
// one band's rows at a time and every weight column tile is read from DRAM once per band, not once per
// row tile (MvmArgs::tile_band_rows says when the host widens them).
__host__ __device__ __forceinline__ void tile_coords(int64_t idx, int64_t n_tiles_m, int64_t n_tiles_n, int64_t band,
                                                     int64_t* tm, int64_t* tn) {
  const int64_t b = idx / (band * n_tiles_n);
  const int64_t first = b * band;
  const int64_t rows = n_tiles_m - first < band ? n_tiles_m - first : band;
  const int64_t local = idx - b * band * n_tiles_n;
  *tm = first + local % rows;
  *tn = local / rows;
}

struct SmemCtl {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tfull[kSlots];
  uint64_t tempty[kSlots];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code,
                                          long long limit) {
  const bool ok = mbar_wait(bar, parity, abort, code, limit);
  return __all_sync(0xffffffffu, ok);
}

// Two fp32 fused multiply-adds in one instruction (sm_100 f32x2): d = a * b + c on packed pairs.
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) {
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__host__ __device__ constexpr int column_groups(int sy) { return 16 / sy > 4 ? 4 : (16 / sy < 2 ? 2 : 16 / sy); }

// SXC > 0 fixes the input slice count at compile time (launched when it equals SY, the usual case of
// one slice method for inputs and weights): the epilogue's input-slice loop then unrolls and the
// slice-pair weights become immediate operands (5.6% faster at 4096^3 with 5 slices).  SXC == 0 reads
// it from the arguments.
template <int KIND, int MODE, int SY, bool SPLIT, int SXC>
__global__ void __launch_bounds__(32 * (4 * column_groups(SY) + 2), 1)
    mvm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ MvmArgs P) {
  constexpr int CG = column_groups(SY);
  constexpr bool kLut = (MODE & MODE_LUT) != 0;
  constexpr bool kFloatAcc = (MODE & MODE_FLOATACC) != 0;
  constexpr bool kDump = (MODE & MODE_DUMP) != 0;
  constexpr int kEpiWarps = 4 * CG;
  constexpr int kProducerWarp = kEpiWarps;
  constexpr int kMmaWarp = kEpiWarps + 1;
  constexpr int BN = 16 * CG;
  // Weight slices loaded from TMEM per wait.  Measured at 4096^3 (noise-free, E4M3): 2 for <= 4 slices
  // (the register budget of 16 epilogue warps), 3 for 5 and 8 slices, 4 for 6 (7 takes 6's value,
  // unmeasured); loading all of them at once was 1-4% slower.
  constexpr int kJChunk = CG >= 4 ? 2 : (SY == 6 || SY == 7 ? 4 : 3);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + static_cast<size_t>(P.stages) * P.stage_bytes);
  int32_t* lut_s = reinterpret_cast<int32_t*>(ctl + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Persistent (launches without split-K): CTA b processes output tiles b, b + grid, ... in the order of
  // tile_coords.  The stage ring, the TMEM slots and the barrier phases run on across tiles, so the next
  // tile's loads and MMAs proceed while this tile's outputs are stored.  The CTA's work is a list of
  // items: its whole tiles below dp_tiles, then at most one K range of a tail tile (see MvmArgs).
  constexpr bool kPersist = !SPLIT;
  const int64_t n_tiles_n = (P.N + BN - 1) / BN;
  const int64_t n_tiles_m = (P.M + kMvmBM - 1) / kMvmBM;
  const int64_t n_tiles = n_tiles_n * n_tiles_m;
  const int64_t bx = blockIdx.x;
  const int64_t my_dp = kPersist ? (P.dp_tiles > bx ? (P.dp_tiles - bx + gridDim.x - 1) / gridDim.x : 0) : 1;
  const int tail_s = kPersist ? P.tail_splits : 0;
  const bool has_tail = kPersist && tail_s > 1 && bx < (n_tiles - P.dp_tiles) * tail_s;
  const int n_items_tail = has_tail ? 1 : 0;
  const int64_t n_items = my_dp + n_items_tail;
  auto item_tile = [&](int64_t it) -> int64_t {   // linear output tile of item `it` (persistent)
    return it < my_dp ? bx + it * gridDim.x : P.dp_tiles + bx / (tail_s > 0 ? tail_s : 1);
  };
  auto tile_m0 = [&](int64_t it) -> int64_t {
    if (!kPersist) return static_cast<int64_t>(blockIdx.y) * kMvmBM;
    int64_t tm, tn;
    tile_coords(item_tile(it), n_tiles_m, n_tiles_n, P.tile_band_rows, &tm, &tn);
    return tm * kMvmBM;
  };
  auto tile_n0 = [&](int64_t it) -> int64_t {
    if (!kPersist) return static_cast<int64_t>(blockIdx.x) * BN;
    int64_t tm, tn;
    tile_coords(item_tile(it), n_tiles_m, n_tiles_n, P.tile_band_rows, &tm, &tn);
    return tn * BN;
  };
  constexpr int Sy = SY;
  const int Sx = SXC > 0 ? SXC : P.Sx;
  const int stages = P.stages;
  constexpr int kSxUnroll = SXC > 0 ? SXC : 1;
  // split-K: this CTA covers K tiles [t_begin, t_begin + Kt)
  const int t_begin = SPLIT ? static_cast<int>(blockIdx.z) * P.tiles_per_split : 0;
  const int Kt = SPLIT ? min(P.tiles_per_split, static_cast<int>(P.Kt) - t_begin) : static_cast<int>(P.Kt);
  // K tiles [item_lo, item_hi) of item `it`
  const int tail_lo = has_tail ? static_cast<int>(bx % tail_s) * P.tail_tiles_per_split : 0;
  const int tail_hi = has_tail ? min(Kt, tail_lo + P.tail_tiles_per_split) : 0;
  auto item_lo = [&](int64_t it) -> int { return it < my_dp ? 0 : tail_lo; };
  auto item_hi = [&](int64_t it) -> int { return it < my_dp ? Kt : tail_hi; };
  const int64_t steps = my_dp * Kt + (tail_hi - tail_lo);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
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
      for (int i = threadIdx.x; i < Sy * P.lut_len; i += blockDim.x) lut_s[i] = P.lut[i];
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
      int s = 0;
      uint32_t phase = 0;
      int64_t it = 0;   // item of this CTA and K tile inside it, stepped along with g (no division)
      int t = item_lo(0), hi = item_hi(0);
      int tm0 = static_cast<int>(tile_m0(0)), tn0 = static_cast<int>(tile_n0(0));
      for (int64_t g = 0; g < steps; ++g) {
        if (g >= stages && !mbar_wait(&ctl->empty[s], phase ^ 1u, abort, 11, P.wait_limit)) break;
        uint8_t* a_dst = smem + static_cast<size_t>(s) * P.stage_bytes;
        uint8_t* b_dst = a_dst + static_cast<size_t>(Sx) * P.a_slice_bytes;
        mbar_arrive_expect_tx(&ctl->full[s], P.stage_bytes);
        tma_load_3d(a_dst, &tma_a, &ctl->full[s], (t_begin + t) * P.pp, tm0, 0);
        tma_load_3d(b_dst, &tma_b, &ctl->full[s], (t_begin + t) * P.pp, tn0, 0);
        issued = g + 1;
        if (++s == stages) {
          s = 0;
          phase ^= 1u;
        }
        if (++t == hi && ++it < n_items) {
          t = item_lo(it);
          hi = item_hi(it);
          tm0 = static_cast<int>(tile_m0(it));
          tn0 = static_cast<int>(tile_n0(it));
        }
      }
      // no TMA write may still be in flight when the CTA exits
      const int64_t first = issued > stages ? issued - stages : 0;
      for (int64_t g = first; g < issued; ++g)
        mbar_wait_drain(&ctl->full[g % stages], static_cast<uint32_t>(g / stages) & 1u, 12);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc = instr_desc_m128(static_cast<uint32_t>(Sy * BN));
      const int ksteps = P.row_bytes / 32;
      int slot = 0, s = 0, uses = 0;
      uint32_t sphase = 0, tphase = 0;
      bool ok = P.hold_mma == 0;   // held (test hook): no MMA and no commit, the epilogue's wait runs out
      for (int64_t g = 0; g < steps && ok; ++g) {
        if (!mbar_wait(&ctl->full[s], sphase, abort, 21, P.wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + static_cast<size_t>(s) * P.stage_bytes);
        const uint32_t b_base = a_base + Sx * P.a_slice_bytes;
        for (int i = 0; i < Sx; ++i) {
          if (uses >= kSlots && !mbar_wait(&ctl->tempty[slot], tphase ^ 1u, abort, 22, P.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + slot * kSlotCols;
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint64_t ad = smem_desc(a_base + i * P.a_slice_bytes + kk * 32, P.row_bytes);
            const uint64_t bd = smem_desc(b_base + kk * 32, P.row_bytes);
            tc_mma<KIND>(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          if (P.b_split) {   // the FP16 residuals of the weight planes, into the same accumulator
            const uint32_t b_lo = b_base + static_cast<uint32_t>(Sy) * P.b_slice_bytes;
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint64_t ad = smem_desc(a_base + i * P.a_slice_bytes + kk * 32, P.row_bytes);
              const uint64_t bd = smem_desc(b_lo + kk * 32, P.row_bytes);
              tc_mma<KIND>(d, ad, bd, idesc, 1u);
            }
          }
          tc_commit(&ctl->tfull[slot]);
          ++uses;
          if (++slot == kSlots) {
            slot = 0;
            tphase ^= 1u;
          }
        }
        if (ok) tc_commit(&ctl->empty[s]);
        if (++s == stages) {
          s = 0;
          sphase ^= 1u;
        }
      }
      // every issued MMA has completed before TMEM is released
      tc_commit(&ctl->drain);
      mbar_wait_drain(&ctl->drain, 0, 23);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int cg = (warp >> 2) * 16;    // 16-column group inside each weight slice's BN columns
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + cg;
    // ADC constants (radc_j - 1) / D, duplicated into f32x2 pairs, and the rounding constant pair
    uint64_t cj2[SY];
#pragma unroll
    for (int j = 0; j < SY; ++j) cj2[j] = pack2(__float_as_uint(P.cadc[j]), __float_as_uint(P.cadc[j]));
    const uint64_t magic2 = pack2(kMagicBits, kMagicBits);
    uint32_t acc[16];
    float out[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      acc[c] = 0u;
      out[c] = 0.0f;
    }
    const int32_t* lut = kLut ? (P.lut_smem ? lut_s : P.lut) : nullptr;
    int slot = 0, cnt = 0;
    uint32_t tphase = 0;
    bool ok = true;
    int64_t m0 = tile_m0(0), n0 = tile_n0(0);
    int64_t row = m0 + q * 32 + lane;
    int64_t it = 0;                          // item of this CTA
    int t = item_lo(0), hi = item_hi(0);     // K tile inside it, and its end
    for (int64_t g = 0; g < steps && ok; ++g) {
#pragma unroll kSxUnroll
      for (int i = 0; i < Sx; ++i) {
        if (!warp_wait(&ctl->tfull[slot], tphase, abort, 31, P.wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = lane_addr + slot * kSlotCols;
        uint32_t wi[SY];
        float wfi[SY];
#pragma unroll
        for (int j = 0; j < SY; ++j) {
          wi[j] = static_cast<uint32_t>(P.wpair[i * 8 + j]);
          if constexpr (kFloatAcc) wfi[j] = P.wfpair[i * 8 + j];
        }
#pragma unroll
        for (int j0 = 0; j0 < SY; j0 += kJChunk) {
          uint32_t r[kJChunk][16];
#pragma unroll
          for (int jj = 0; jj < kJChunk; ++jj)
            if (j0 + jj < SY) tmem_ld16(base + (j0 + jj) * BN, r[jj]);
          tmem_wait_ld();
          if (j0 + kJChunk >= SY) {
            // every column of this slot is in registers: hand the slot back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->tempty[slot]);
          }
#pragma unroll
          for (int jj = 0; jj < kJChunk; ++jj) {
            const int j = j0 + jj;
            if (j < SY) {
              if constexpr (kLut) {
                const int32_t* lj = lut + j * P.lut_len;
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                  const int idx = static_cast<int>(__float_as_uint(__uint_as_float(r[jj][c]) + kMagic) - kMagicBits);
                  const int32_t code = lj[min(max(idx, 0), P.lut_len - 1)];
                  if constexpr (kFloatAcc)
                    acc[c] = __float_as_uint(fmaf(static_cast<float>(code), wfi[j], __uint_as_float(acc[c])));
                  else
                    acc[c] += wi[j] * static_cast<uint32_t>(code);
                }
              } else {
#pragma unroll
                for (int c = 0; c < 16; c += 2) {
                  const uint64_t tq = ffma2(pack2(r[jj][c], r[jj][c + 1]), cj2[j], magic2);
                  const uint32_t tx = static_cast<uint32_t>(tq), ty = static_cast<uint32_t>(tq >> 32);
                  if constexpr (kFloatAcc) {
                    acc[c] = __float_as_uint(fmaf(__uint_as_float(tx) - kMagic, wfi[j], __uint_as_float(acc[c])));
                    acc[c + 1] = __float_as_uint(fmaf(__uint_as_float(ty) - kMagic, wfi[j], __uint_as_float(acc[c + 1])));
                  } else {
                    acc[c] += wi[j] * tx;
                    acc[c + 1] += wi[j] * ty;
                  }
                }
              }
            }
          }
        }
        if (++slot == kSlots) {
          slot = 0;
          tphase ^= 1u;
        }
      }
      if (!ok) break;
      ++cnt;
      if (kDump || cnt == P.flush_tiles || t == hi - 1) {
        const int tg = t_begin + t;   // global K tile
        const float xsv = row < P.M ? __ldg(P.xs + static_cast<int64_t>(tg) * P.M + row) : 0.0f;
        const float rs = kFloatAcc ? xsv : xsv * P.out_scale;
        const uint32_t off = (kLut || kFloatAcc) ? 0u : static_cast<uint32_t>(cnt) * P.tile_offset;
        const float* wsr = P.ws + static_cast<int64_t>(tg) * P.N + n0 + cg;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const bool in = n0 + cg + c < P.N;
          const float wsv = in ? __ldg(wsr + c) : 0.0f;
          float v;
          if constexpr (kFloatAcc) {
            v = __uint_as_float(acc[c]);
          } else {
            const int32_t iv = static_cast<int32_t>(acc[c] - off);
            if constexpr (kDump) {
              if (row < P.M && in) P.acc_dump[(static_cast<int64_t>(tg) * P.M + row) * P.N + n0 + cg + c] = iv;
            }
            v = static_cast<float>(iv);
          }
          out[c] = fmaf(v, rs * wsv, out[c]);
          acc[c] = 0u;
        }
        cnt = 0;
      }
      if (kPersist && t == hi - 1) {
        if (it >= my_dp) {
          // a K range of a tail tile: the whole 128 x BN partial, summed by tail_reduce
          float* pt = P.tail_partial + (bx * kMvmBM + q * 32 + lane) * BN + cg;
#pragma unroll
          for (int c = 0; c < 16; ++c) pt[c] = out[c];
        } else if (row < P.M) {
          const int64_t grp = row / P.rows_per_group;
          const int64_t rr = row - grp * P.rows_per_group;
          float* yb = P.y + grp * P.group_stride + rr * P.row_stride;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int64_t n = n0 + cg + c;
            if (n < P.N) yb[n * P.col_stride] = out[c] + (P.bias ? __ldg(P.bias + n) : 0.0f);
          }
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) out[c] = 0.0f;
        if (++it < n_items) {
          t = item_lo(it);
          hi = item_hi(it);
          m0 = tile_m0(it);
          n0 = tile_n0(it);
          row = m0 + q * 32 + lane;
        }
      } else {
        ++t;
      }
    }
    if (kPersist) {
      // every tile was stored inside the loop
    } else if (SPLIT && ok && row < P.M) {
      float* pr = P.partial + (static_cast<int64_t>(blockIdx.z) * P.M + row) * P.N;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int64_t n = n0 + cg + c;
        if (n < P.N) pr[n] = out[c];
      }
    } else if (ok && row < P.M) {
      const int64_t grp = row / P.rows_per_group;
      const int64_t rr = row - grp * P.rows_per_group;
      float* yb = P.y + grp * P.group_stride + rr * P.row_stride;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int64_t n = n0 + cg + c;
        if (n < P.N) yb[n * P.col_stride] = out[c] + (P.bias ? __ldg(P.bias + n) : 0.0f);
      }
    }
  }

  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int KIND, int MODE, int SY, bool SPLIT, int SXC>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, size_t smem,
                       cudaStream_t stream) {
  auto fn = mvm_kernel<KIND, MODE, SY, SPLIT, SXC>;
  // The shared-memory cap is a per-device function attribute: raise it once on every device this
  // template instance runs on (one bit per device index, set after the attribute call succeeded).
  static std::atomic<uint64_t> configured[2] = {};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= 128) return cudaErrorInvalidDevice;
  const uint64_t bit = uint64_t(1) << (device & 63);
  if (!(configured[device >> 6].load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[device >> 6].fetch_or(bit, std::memory_order_release);
  }
  constexpr int CG = column_groups(SY);
  constexpr int BN = 16 * CG;
  const unsigned splits = SPLIT ? static_cast<unsigned>((a.Kt + a.tiles_per_split - 1) / a.tiles_per_split) : 1u;
  dim3 grid(static_cast<unsigned>((a.N + BN - 1) / BN), static_cast<unsigned>((a.M + kMvmBM - 1) / kMvmBM), splits);
  if (!SPLIT) {   // persistent: one CTA per SM (at most one fits, by shared memory)
    int sms = 0;
    e = device_sm_count(device, &sms);
    if (e != cudaSuccess) return e;
    const int64_t tiles = static_cast<int64_t>(grid.x) * grid.y;
    grid = dim3(static_cast<unsigned>(tiles < sms ? tiles : sms), 1, 1);
  }
  fn<<<grid, 32 * (4 * CG + 2), smem, stream>>>(ta, tb, a);
  count_launch();
  return cudaGetLastError();
}

template <int KIND, int MODE, int SY>
cudaError_t launch_split(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, size_t smem,
                         cudaStream_t stream) {
  if constexpr (MODE == 0 || MODE == MODE_FLOATACC) {
    if (a.Sx == SY) {
      if (a.partial) return launch_one<KIND, MODE, SY, true, SY>(ta, tb, a, smem, stream);
      return launch_one<KIND, MODE, SY, false, SY>(ta, tb, a, smem, stream);
    }
  }
  if (a.partial) return launch_one<KIND, MODE, SY, true, 0>(ta, tb, a, smem, stream);
  return launch_one<KIND, MODE, SY, false, 0>(ta, tb, a, smem, stream);
}

template <int KIND, int SY>
cudaError_t launch_sy(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, int mode, size_t smem,
                      cudaStream_t stream) {
  switch (mode) {
    case 0: return launch_split<KIND, 0, SY>(ta, tb, a, smem, stream);
    case MODE_LUT: return launch_split<KIND, MODE_LUT, SY>(ta, tb, a, smem, stream);
    case MODE_FLOATACC: return launch_split<KIND, MODE_FLOATACC, SY>(ta, tb, a, smem, stream);
    case MODE_LUT | MODE_FLOATACC: return launch_split<KIND, MODE_LUT | MODE_FLOATACC, SY>(ta, tb, a, smem, stream);
    case MODE_DUMP: return launch_split<KIND, MODE_DUMP, SY>(ta, tb, a, smem, stream);
    case MODE_DUMP | MODE_LUT: return launch_split<KIND, MODE_DUMP | MODE_LUT, SY>(ta, tb, a, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int KIND>
cudaError_t launch_kind(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, int mode, size_t smem,
                        cudaStream_t stream) {
  switch (a.Sy) {
    case 2: return launch_sy<KIND, 2>(ta, tb, a, mode, smem, stream);
    case 3: return launch_sy<KIND, 3>(ta, tb, a, mode, smem, stream);
    case 4: return launch_sy<KIND, 4>(ta, tb, a, mode, smem, stream);
    case 5: return launch_sy<KIND, 5>(ta, tb, a, mode, smem, stream);
    case 6: return launch_sy<KIND, 6>(ta, tb, a, mode, smem, stream);
    case 7: return launch_sy<KIND, 7>(ta, tb, a, mode, smem, stream);
    case 8: return launch_sy<KIND, 8>(ta, tb, a, mode, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

// Tail reduction of a persistent launch: every element of the tail tiles is the sum, in K order, of
// its tail_splits partials (tail_partial[tile * splits + s][row][col], tile-local), plus the bias.
__global__ void tail_reduce_kernel(const float* __restrict__ tail_partial, int splits, int64_t dp_tiles,
                                   int64_t tail_tiles, int bn, int64_t band, int64_t M, int64_t N,
                                   float* __restrict__ y,
                                   int64_t rows_per_group, int64_t group_stride, int64_t row_stride,
                                   int64_t col_stride, const float* __restrict__ bias) {
  const int64_t per_tile = static_cast<int64_t>(kMvmBM) * bn;
  const int64_t total = tail_tiles * per_tile;
  const int64_t n_tiles_n = (N + bn - 1) / bn, n_tiles_m = (M + kMvmBM - 1) / kMvmBM;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tl = e / per_tile, rem = e - tl * per_tile;
    const int64_t r = rem / bn, c = rem - r * bn;
    int64_t tm, tn;
    tile_coords(dp_tiles + tl, n_tiles_m, n_tiles_n, band, &tm, &tn);
    const int64_t m = tm * kMvmBM + r, n = tn * bn + c;
    if (m >= M || n >= N) continue;
    float v = 0.0f;
    for (int s = 0; s < splits; ++s) v += __ldg(tail_partial + (tl * splits + s) * per_tile + rem);
    if (bias) v += __ldg(bias + n);
    const int64_t grp = m / rows_per_group, rr = m - grp * rows_per_group;
    y[grp * group_stride + rr * row_stride + n * col_stride] = v;
  }
}

// Split-K reduction: y[layout(r, n)] = sum_s partial[s][r][n] + bias[n], splits added in order.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int64_t M, int64_t N,
                                     float* __restrict__ y, int64_t rows_per_group, int64_t group_stride,
                                     int64_t row_stride, int64_t col_stride, const float* __restrict__ bias) {
  const int64_t total = M * N;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / N, n = e - (e / N) * N;
    float v = 0.0f;
    for (int s = 0; s < splits; ++s) v += __ldg(partial + static_cast<int64_t>(s) * total + e);
    if (bias) v += __ldg(bias + n);
    const int64_t grp = r / rows_per_group, rr = r - grp * rows_per_group;
    y[grp * group_stride + rr * row_stride + n * col_stride] = v;
  }
}

}  // namespace

cudaError_t device_sm_count(int device, int* sms) {
  static std::atomic<int> sm_count[128] = {};
  if (device < 0 || device >= 128) return cudaErrorInvalidDevice;
  int v = sm_count[device].load(std::memory_order_relaxed);
  if (v == 0) {
    const cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return e;
    sm_count[device].store(v, std::memory_order_relaxed);
  }
  *sms = v;
  return cudaSuccess;
}

cudaError_t launch_tail_reduce(const float* tail_partial, int splits, int64_t dp_tiles, int64_t tail_tiles, int bn,
                               int64_t band, int64_t M, int64_t N, float* y, int64_t rows_per_group, int64_t group_stride,
                               int64_t row_stride, int64_t col_stride, const float* bias, cudaStream_t stream) {
  const int64_t total = tail_tiles * kMvmBM * bn;
  const int64_t blocks = (total + 255) / 256;
  tail_reduce_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0, stream>>>(
      tail_partial, splits, dp_tiles, tail_tiles, bn, band, M, N, y, rows_per_group, group_stride, row_stride, col_stride,
      bias);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_splitk_reduce(const float* partial, int splits, int64_t M, int64_t N, float* y,
                                 int64_t rows_per_group, int64_t group_stride, int64_t row_stride,
                                 int64_t col_stride, const float* bias, cudaStream_t stream) {
  const int64_t total = M * N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  splitk_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(partial, splits, M, N, y, rows_per_group,
                                                                          group_stride, row_stride, col_stride, bias);
  count_launch();
  return cudaGetLastError();
}

int mvm_column_groups(int sy) { return column_groups(sy); }  // Sy * 16 * CG <= 256 columns per TMEM slot

size_t mvm_smem_bytes(const MvmArgs& a) {
  return 1024 + static_cast<size_t>(a.stages) * a.stage_bytes + sizeof(SmemCtl) +
         (a.lut_smem ? static_cast<size_t>(a.Sy) * a.lut_len * sizeof(int32_t) : 0);
}

cudaError_t launch_mvm(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, int kind, int mode,
                       cudaStream_t stream) {
  const size_t smem = mvm_smem_bytes(a);
  if (kind == MIB_OPERAND_E4M3) return launch_kind<MIB_OPERAND_E4M3>(ta, tb, a, mode, smem, stream);
  return launch_kind<MIB_OPERAND_FP16>(ta, tb, a, mode, smem, stream);
}

}  // namespace mib
