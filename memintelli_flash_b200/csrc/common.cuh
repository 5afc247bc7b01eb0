// Shared device helpers: PTX wrappers for mbarrier / TMA / tcgen05 (sm_100a),
// bounded waits with an error flag, Philox4x32-10 and the numeric primitives
// that must reproduce the reference's fp32 quantisation arithmetic exactly.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "../../include/memintelli_b200.h"

namespace mib {

// ---------------------------------------------------------------------------
// device error flag (set by kernels whose bounded waits expire)
// ---------------------------------------------------------------------------
__device__ int g_device_error = 0;

// ~2 s at 1.9 GHz; no wait in a correct run comes near this.
constexpr long long kWaitTimeoutCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`.  Gives up when `abort` is raised by another
// thread or after `limit` cycles; on timeout it raises `abort` and records
// `code` in the device error flag.  Returns false when the wait did not complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code,
                                          long long limit = kWaitTimeoutCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > limit) {
      *abort = 1;
      atomicExch(&g_device_error, code);
      return false;
    }
  }
}

// Bounded wait used while draining in-flight asynchronous work before exit:
// ignores the abort flag, records `code` if it expires.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitTimeoutCycles) {
      atomicExch(&g_device_error, code);
      return;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this code base)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, one thread issues.  KIND selects the operand family.
template <int KIND>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (KIND == MIB_OPERAND_E4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile whose rows are
// `row_bytes` long (32/64/128, i.e. one swizzle atom wide) and packed densely
// (8-row core-matrix groups `8*row_bytes` apart).  Bit layout: start address
// [0,14), leading byte offset [16,30), stride byte offset [32,46), version=1
// at [46,48), swizzle mode [61,64) (6: 32B, 4: 64B, 2: 128B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t row_bytes) {
  const uint64_t swz = row_bytes == 32 ? 6ull : (row_bytes == 64 ? 4ull : 2ull);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>((8u * row_bytes) >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= swz << 61;
  return d;
}

// Instruction descriptor: f32 accumulate, A/B K-major, M=128, N=n.
// Format code 0 is E4M3 for kind::f8f6f4 and F16 for kind::f16.
__host__ __device__ constexpr uint32_t instr_desc_m128(uint32_t n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Philox4x32-10 counter-based generator (Salmon et al., "Parallel random
// numbers: as easy as 1, 2, 3", SC'11) and Box-Muller normals.
// ---------------------------------------------------------------------------
struct U4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ U4 philox4x32_10(U4 ctr, uint32_t k0, uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, ctr.x), lo0 = kM0 * ctr.x;
    const uint32_t hi1 = __umulhi(kM1, ctr.z), lo1 = kM1 * ctr.z;
    ctr = U4{hi1 ^ ctr.y ^ k0, lo1, hi0 ^ ctr.w ^ k1, lo0};
    k0 += kW0;
    k1 += kW1;
  }
  return ctr;
}
// uniform in (0, 1]
__device__ __forceinline__ float u01(uint32_t v) { return (static_cast<float>(v >> 8) + 1.0f) * (1.0f / 16777216.0f); }

// Four standard normals from one Philox block (two Box-Muller pairs: radius sqrt(-2 ln u1), angle
// 2 pi u2).  The radius uses the hardware log2 and reciprocal square root, the angle the hardware
// sine / cosine on [-pi, pi) (a uniform angle shifted by pi is still uniform); their absolute errors
// (about 1e-6) are far below the resolution of any noise statistic.
__device__ __forceinline__ void normal4(uint64_t seed, uint64_t stream, uint64_t index, float (&n)[4]) {
  U4 c{static_cast<uint32_t>(index), static_cast<uint32_t>(index >> 32), static_cast<uint32_t>(stream),
       static_cast<uint32_t>(stream >> 32)};
  U4 r = philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  const float two_pi = 6.283185307179586f, pi = 3.141592653589793f;
  const float m2ln2 = -1.3862943611198906f;  // -2 ln 2: -2 ln u = -2 ln 2 * log2 u
  const float a0 = m2ln2 * __log2f(u01(r.x)), a1 = m2ln2 * __log2f(u01(r.z));
  const float r0 = a0 * rsqrtf(fmaxf(a0, 1e-30f)), r1 = a1 * rsqrtf(fmaxf(a1, 1e-30f));
  float s0, c0, s1, c1;
  __sincosf(fmaf(two_pi, u01(r.y), -pi), &s0, &c0);
  __sincosf(fmaf(two_pi, u01(r.w), -pi), &s1, &c1);
  n[0] = r0 * c0;
  n[1] = r0 * s0;
  n[2] = r1 * c1;
  n[3] = r1 * s1;
}

// ---------------------------------------------------------------------------
// exact fp32 emulation of the reference's quantisation steps
// ---------------------------------------------------------------------------
// round(code / m * L) with the reference's two fp32 roundings, half-to-even.
__device__ __forceinline__ int level_map(int code, int m, int lm1) {
  return __float2int_rn(__fmul_rn(__fdiv_rn(static_cast<float>(code), static_cast<float>(m)), static_cast<float>(lm1)));
}

// floor(log2(bmax + 1e-10)) as torch evaluates it in fp32 (log2 correctly
// rounded to fp32): the log is taken in double and rounded to float.
__device__ __forceinline__ int bfp_exponent(float bmax) {
  const float b = __fadd_rn(bmax, 1e-10f);
  return static_cast<int>(floorf(__double2float_rn(log2(static_cast<double>(b)))));
}

// 2^e for e in the normal range.
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// Quantise one value to the two's complement code in [0, 2^bits).
//   INT: q = rne(v / bmax * (2^(bits-1)-1)); bmax == 0 gives q = 0.
//   BFP: q = clip(rne(v / 2^e * 2^(bits-2)), -2^(bits-1), 2^(bits-1)-1).
__device__ __forceinline__ int quantize(float v, float bmax, int e, int bits, bool bfp) {
  int q;
  if (bfp) {
    float t = __fmul_rn(__fdiv_rn(v, pow2f(e)), static_cast<float>(1 << (bits - 2)));
    float r = rintf(t);
    r = fminf(fmaxf(r, -static_cast<float>(1 << (bits - 1))), static_cast<float>((1 << (bits - 1)) - 1));
    q = static_cast<int>(r);
  } else {
    if (bmax == 0.0f) return 0;
    float t = __fmul_rn(__fdiv_rn(v, bmax), static_cast<float>((1 << (bits - 1)) - 1));
    q = static_cast<int>(rintf(t));
  }
  if (q < 0) q += (1 << bits);
  return q;
}

// Encode a small non-negative integer level as the MMA operand element.
__device__ __forceinline__ uint8_t enc_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float dec_e4m3(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

}  // namespace mib
