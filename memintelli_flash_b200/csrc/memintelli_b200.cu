// C ABI of the B200 CIM sliced matmul (declared in include/memintelli_b200.h).
//
// One translation unit: the kernel sources are included here so the device
// error flag and the kernels share a module.  This layer validates arguments
// with the reference's error semantics, derives the kernel parameter blocks,
// encodes the TMA tensor maps and launches.  It never allocates memory.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>

#include "slice.cu"
#include "mvm.cu"
#include "attn_prep.cu"
#include "row_lse.cu"

namespace {

thread_local std::string g_err;

// One-shot failure injection for tests (mib_test_inject_wait_expiry): the next mib_mvm launch on this
// thread holds its MMA warp and gives its abortable waits this many cycles.
thread_local long long g_inject_wait_limit = 0;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MIB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

struct SliceTab {
  int S = 0, bits = 0;
  int widths[8] = {}, offs[8] = {}, maxes[8] = {};
  long long coef[8] = {};  // shift weight c_t (LSB-first, sign slice negative)
};

// memintelli/pimpy/data_formats.py:45-46, 60-71
int make_tab(const mib_slice_spec* sp, SliceTab& t) {
  if (!sp) return fail(MIB_ERR_PARAM, "slice spec is NULL");
  if (sp->n_slices < 1 || sp->n_slices > MIB_MAX_SLICES)
    return fail(MIB_ERR_PARAM, "number of slices must be in [1, 8]");
  if (sp->slice_method[0] != 1) return fail(MIB_ERR_PARAM, "The first bit of the slice method should be 1");
  t.S = sp->n_slices;
  int off = 0;
  for (int i = 0; i < t.S; ++i) {
    const int w = sp->slice_method[t.S - 1 - i];
    if (w < 1 || w > 8) return fail(MIB_ERR_PARAM, "slice widths must be in [1, 8]");
    t.widths[i] = w;
    t.offs[i] = off;
    t.maxes[i] = (1 << w) - 1;
    t.coef[i] = 1ll << off;
    off += w;
  }
  t.coef[t.S - 1] = -t.coef[t.S - 1];
  t.bits = off;
  if (t.bits > 8) return fail(MIB_ERR_UNSUPPORTED, "total slice width above 8 bits is not supported");
  if (t.bits < 2) return fail(MIB_ERR_PARAM, "total slice width must be at least 2 bits");
  return MIB_OK;
}

int esize(int kind) { return kind == MIB_OPERAND_E4M3 ? 1 : 2; }

int check_kgeom(const mib_k_geom* kg, int kind) {
  if (!kg) return fail(MIB_ERR_PARAM, "k geometry is NULL");
  if (kg->p < 1) return fail(MIB_ERR_PARAM, "crossbar tile depth must be positive");
  if (kg->pp < kg->p || kg->pp % 4) return fail(MIB_ERR_PARAM, "padded tile depth must be >= p and a multiple of 4");
  const int rb = kg->pp * esize(kind);
  if (rb != 32 && rb != 64 && rb != 128)
    return fail(MIB_ERR_UNSUPPORTED, "padded tile row must be 32, 64 or 128 bytes");
  if (kg->kt * kg->p != kg->kp || kg->kp < kg->k)
    return fail(MIB_ERR_SHAPE, "inconsistent K geometry (kp != kt * p or kp < k)");
  return MIB_OK;
}

int max_level_for(int kind) { return kind == MIB_OPERAND_E4M3 ? 16 : 2048; }

void fill_slice_args(mib::SliceArgs& a, const SliceTab& t, const mib_slice_spec* sp, const mib_k_geom* kg,
                     int64_t batch, int64_t rows, int64_t cols, int32_t rdac, int32_t kind, void* planes,
                     float* tile_scale, float* block_max, float* block_exp, uint8_t* packed) {
  a.batch = batch;
  a.rows = rows;
  a.cols = cols;
  a.qg0 = sp->quant_gran[0];
  a.qg1 = sp->quant_gran[1];
  a.nbr = (rows + a.qg0 - 1) / a.qg0;
  a.nbc = (cols + a.qg1 - 1) / a.qg1;
  a.p = kg->p;
  a.pp = kg->pp;
  a.kt = kg->kt;
  a.kp = kg->kp;
  a.bits = t.bits;
  a.bfp = sp->bfp ? 1 : 0;
  a.n_slices = t.S;
  a.lm1 = rdac - 1;
  a.kind = kind;
  for (int i = 0; i < 8; ++i) {
    a.offs[i] = t.offs[i];
    a.maxes[i] = t.maxes[i] ? t.maxes[i] : 1;
  }
  a.planes = planes;
  a.row_pitch = kg->kt * kg->pp;
  a.plane_stride = batch * rows * a.row_pitch;
  a.tile_scale = tile_scale;
  a.scale_ld = batch * rows;
  a.block_max = block_max;
  a.block_exp = block_exp;
  a.packed = packed;
  a.vnoise = 0.0f;
  a.noise_seed = a.noise_stream = 0;
}

int check_input_geom(const SliceTab& t, const mib_slice_spec* sp, const mib_k_geom* kg, int64_t cols, int32_t rdac,
                     int32_t kind, const void* planes, const float* tile_scale, const float* block_max) {
  (void)t;
  if (!planes || !tile_scale || !block_max) return fail(MIB_ERR_PARAM, "output buffer is NULL");
  if (kind != MIB_OPERAND_E4M3 && kind != MIB_OPERAND_FP16) return fail(MIB_ERR_PARAM, "unknown operand kind");
  if (int r = check_kgeom(kg, kind)) return r;
  if (sp->paral[0] < 1 || sp->paral[1] < 1) return fail(MIB_ERR_PARAM, "paral_size must be positive");
  if (sp->paral[1] != kg->p) return fail(MIB_ERR_SHAPE, "input paral_size[1] must equal the crossbar tile depth");
  if (sp->quant_gran[0] < 1 || sp->quant_gran[1] < 1 || sp->quant_gran[0] % sp->paral[0] ||
      sp->quant_gran[1] % sp->paral[1])
    return fail(MIB_ERR_PARAM, "quant_gran must be a positive multiple of paral_size");
  const int64_t nbc = (cols + sp->quant_gran[1] - 1) / sp->quant_gran[1];
  if (nbc * sp->quant_gran[1] != kg->kp) return fail(MIB_ERR_SHAPE, "input K padding does not match the K geometry");
  if (rdac < 2) return fail(MIB_ERR_PARAM, "The resolution of the DAC should be larger than 1!");
  if (rdac - 1 > max_level_for(kind))
    return fail(MIB_ERR_UNSUPPORTED, "DAC levels do not fit the operand type (use FP16 operands)");
  return MIB_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over operand planes [S][rows][kt*pp]; box = one crossbar tile of `box_rows` rows, all slices.
int encode_planes(CUtensorMap* map, const void* base, int kind, int64_t rows, int64_t row_elems, int slices, int pp,
                  int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(MIB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int es = esize(kind);
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_elems), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(slices)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_elems * es), static_cast<cuuint64_t>(rows * row_elems * es)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(pp), static_cast<cuuint32_t>(box_rows),
                             static_cast<cuuint32_t>(slices)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const int rb = pp * es;
  const CUtensorMapSwizzle swz = rb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                          : (rb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMapDataType dt = kind == MIB_OPERAND_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) rows=%lld row_elems=%lld slices=%d pp=%d", int(r),
             static_cast<long long>(rows), static_cast<long long>(row_elems), slices, pp);
    return fail(MIB_ERR_CUDA, buf);
  }
  return MIB_OK;
}

// exact round_half_even(num / den) for num >= 0, den > 0
long long rne_div(long long num, long long den) {
  long long q = num / den, r = num % den;
  if (2 * r > den || (2 * r == den && (q & 1))) ++q;
  return q;
}

bool noise_free(const mib_device_spec* d) {
  if (d->vnoise != 0.0 || d->write_variation != 0.0) return false;
  for (int i = 0; i < std::max(1, d->n_read_sigma); ++i)
    if (d->read_sigma[i] != 0.0f) return false;
  return true;
}

// Largest factor by which per-call noise can raise a crossbar sum above its noise-free full scale.  The
// normals come from Box-Muller on 24-bit uniforms in (0, 1] (common.cuh normal4), so |z| <= sqrt(-2 ln 2^-24)
// = 5.77: read variation scales a cell by at most exp(5.8 sigma) (plus (LGS/Q_G)(e - 1) < 0.01 of a level
// here), voltage noise an input level by at most 1 + 5.8 vnoise.  Write variation is a torch.normal field
// without that bound, so it keeps a factor of 2.
double noisy_sum_factor(const mib_device_spec* d) {
  double smax = 0.0;
  for (int i = 0; i < std::max(1, d->n_read_sigma); ++i) smax = std::max(smax, static_cast<double>(d->read_sigma[i]));
  double f = std::exp(5.8 * smax) * 1.01;
  if (d->vnoise > 0.0) f *= 1.0 + 5.8 * d->vnoise;
  if (d->write_variation > 0.0) f *= 2.0;
  return f;
}

struct AdcPlan {
  int mode = 0;          // MODE_LUT / MODE_FLOATACC bits
  int lut_len = 0;       // entries per weight slice
  float cadc[8] = {};
  int flush = 1;
  long long R[8] = {};
  long long D = 0;
};

int radc_of(const mib_device_spec* d, int j, int Sy, long long* out) {
  if (d->n_radc == 1) {
    *out = d->radc[0];
  } else {
    if (d->n_radc != Sy) {
      char buf[128];
      snprintf(buf, sizeof(buf), "Length of radc array (%d) must match number of weight slices (%d)", d->n_radc, Sy);
      return fail(MIB_ERR_PARAM, buf);
    }
    *out = d->radc[j];
  }
  if (*out < 2) return fail(MIB_ERR_PARAM, "All ADC resolution values should be larger than 1!");
  return MIB_OK;
}

// Checks every quantity the ADC plan divides by or loops over, with the reference's messages
// (memmat_tensor.py:98-111, 284-285), so that every entry point reaching adc_plan (mib_mvm,
// mib_adc_plan, mib_mvm_workspace, mib_mvm_static_scratch) rejects them the same way.
int check_engine(const SliceTab& tw, const mib_k_geom* kg, const mib_device_spec* dev) {
  if (!kg || !dev) return fail(MIB_ERR_PARAM, "NULL argument");
  if (kg->p < 1) return fail(MIB_ERR_PARAM, "crossbar tile depth must be positive");
  if (kg->kt < 1) return fail(MIB_ERR_SHAPE, "K geometry has no crossbar tile");
  if (dev->rdac < 2) return fail(MIB_ERR_PARAM, "The resolution of the DAC should be larger than 1!");
  if (dev->g_level < 2) return fail(MIB_ERR_PARAM, "The number of the conductance levels should be larger than 1!");
  if (dev->n_radc < 1 || dev->n_radc > MIB_MAX_SLICES) return fail(MIB_ERR_PARAM, "radc list length must be in [1, 8]");
  if (dev->n_read_sigma < 0 || dev->n_read_sigma > MIB_MAX_LEVELS)
    return fail(MIB_ERR_PARAM, "read variation list length must be in [0, 256]");
  for (int j = 0; j < tw.S; ++j)
    if (tw.maxes[j] > dev->g_level - 1) return fail(MIB_ERR_PARAM, "The weight data is out of the range!");
  return MIB_OK;
}

// Chooses the ADC code source and the accumulation for one MVM configuration.
int adc_plan(const SliceTab& tx, const SliceTab& tw, const mib_slice_spec* xs, const mib_slice_spec* wsp,
             const mib_k_geom* kg, const mib_device_spec* dev, AdcPlan& pl) {
  if (int r = check_engine(tw, kg, dev)) return r;
  const long long D = static_cast<long long>(dev->rdac - 1) * (dev->g_level - 1) * kg->p;
  pl.D = D;
  bool uniform = true;
  for (int j = 0; j < tw.S; ++j) {
    if (int r = radc_of(dev, j, tw.S, &pl.R[j])) return r;
    pl.R[j] -= 1;
    pl.cadc[j] = static_cast<float>(static_cast<double>(pl.R[j]) / static_cast<double>(D));
    if (pl.R[j] != pl.R[0]) uniform = false;
  }
  const bool exact = noise_free(dev);
  bool need_lut = false;
  if (exact) {
    // magic-constant rounding must reproduce the exact half-even code for every reachable S in [0, D], both
    // as one fused multiply-add and as a rounded product followed by a rounded add, so that the result
    // does not depend on how the packed f32x2 instruction evaluates it
    for (int j = 0; j < tw.S && !need_lut; ++j) {
      for (long long S = 0; S <= D; ++S) {
        const float t = std::fma(static_cast<float>(S), pl.cadc[j], 12582912.0f) - 12582912.0f;
        volatile float prod = static_cast<float>(S) * pl.cadc[j];
        const float t2 = (prod + 12582912.0f) - 12582912.0f;
        if (static_cast<long long>(t) != rne_div(S * pl.R[j], D) || static_cast<long long>(t2) != rne_div(S * pl.R[j], D)) {
          need_lut = true;
          break;
        }
      }
    }
  }
  if (need_lut) {
    pl.mode |= mib::MODE_LUT;
    pl.lut_len = static_cast<int>(D + 1);
  }
  long long wsum = 0;
  for (int i = 0; i < tx.S; ++i)
    for (int j = 0; j < tw.S; ++j) wsum += std::llabs(tx.maxes[i] * tw.maxes[j] * tx.coef[i] * tw.coef[j]);
  long long qmax = 0;
  for (int j = 0; j < tw.S; ++j) qmax = std::max(qmax, pl.R[j]);
  if (!exact) qmax = static_cast<long long>(std::ceil(static_cast<double>(qmax) * noisy_sum_factor(dev))) + 2;
  const double limit = 0.98 * 2147483648.0;
  const double per_tile = static_cast<double>(wsum) * static_cast<double>(qmax);
  if (!uniform || per_tile >= limit) {
    pl.mode |= mib::MODE_FLOATACC;
    pl.flush = 1;
  } else {
    const long long fmax = static_cast<long long>(limit / per_tile);
    const long long kx = xs->quant_gran[1] / kg->p, kw = wsp->quant_gran[0] / kg->p;
    const long long kblk = std::gcd(kx, kw);
    long long f = 1;
    for (long long d = 1; d <= kblk; ++d)
      if (kblk % d == 0 && d <= fmax) f = d;
    pl.flush = static_cast<int>(f);
  }
  return MIB_OK;
}

// Split-K choice: when the output tiles fill less than ~3/4 of the 148 SMs, the K tiles are
// divided into `splits` contiguous ranges (multiples of the flush group, so no scale block is
// cut), each written as an fp32 partial and reduced afterwards.
struct SplitPlan {
  int splits = 1;
  int tiles_per_split = 0;
};

// Contiguous K ranges of whole flush groups; `want` ranges at most.
static SplitPlan split_ranges(int64_t kt, int flush, int64_t groups, int64_t want) {
  SplitPlan sp;
  sp.tiles_per_split = static_cast<int>(kt);
  if (want > groups) want = groups;
  if (want > 32) want = 32;
  if (want < 2) return sp;
  const int64_t per = (groups + want - 1) / want;           // flush groups per split
  sp.tiles_per_split = static_cast<int>(per * flush);
  sp.splits = static_cast<int>((kt + sp.tiles_per_split - 1) / sp.tiles_per_split);
  if (sp.splits < 2) sp = SplitPlan{1, static_cast<int>(kt)};
  return sp;
}

// Two cases split K:
//  * a grid under 3/4 of the 148 SMs: enough splits to fill them;
//  * with `balance`, a grid of up to 4 waves whose last wave is partly idle: the split
//    count (2..4) that minimises the wave-rounded time, if it saves at least 10%.  For
//    example, 352 output tiles take 3 waves unsplit and 5 half-length waves split in two.
SplitPlan split_plan(int64_t m, int64_t n, int64_t kt, int flush, int sy, bool balance) {
  const int64_t bn = 16 * mib::mvm_column_groups(sy);
  const int64_t ctas = ((n + bn - 1) / bn) * ((m + mib::kMvmBM - 1) / mib::kMvmBM);
  const int64_t groups = (kt + flush - 1) / flush;
  if (groups < 2) return split_ranges(kt, flush, groups, 1);
  if (ctas * 4 < 148 * 3) return split_ranges(kt, flush, groups, (148 + ctas - 1) / ctas);
  if (!balance || ctas >= 4 * 148) return split_ranges(kt, flush, groups, 1);
  SplitPlan best = split_ranges(kt, flush, groups, 1);
  double best_cost = static_cast<double>((ctas + 147) / 148);
  const double unsplit = best_cost;
  for (int64_t want = 2; want <= 4; ++want) {
    const SplitPlan sp = split_ranges(kt, flush, groups, want);
    if (sp.splits < 2) continue;
    const double cost = static_cast<double>((ctas * sp.splits + 147) / 148) / sp.splits;
    if (cost < best_cost) {
      best = sp;
      best_cost = cost;
    }
  }
  return best_cost <= 0.9 * unsplit ? best : split_ranges(kt, flush, groups, 1);
}

// Tail split of a persistent launch: when the last wave of output tiles fills at most half of the
// SMs, those tiles are cut into K ranges (whole flush groups) so that the wave's work is spread over
// all SMs; tail_reduce adds the ranges in K order.  For example 2816 tiles on 148 SMs take 20 waves,
// the last one 4 tiles; cut into 16 ranges each, they take 1/16 of a wave.
struct TailPlan {
  int64_t dp_tiles = 0;   // tiles stepped whole
  int splits = 1;         // K ranges per tail tile (1: no tail split)
  int tiles_per_split = 0;
  int64_t floats = 0;     // partial outputs: tail tiles x splits x 128 x BN
};

TailPlan tail_plan(int64_t m, int64_t n, int64_t kt, int flush, int sy, int sms) {
  TailPlan tp;
  const int64_t bn = 16 * mib::mvm_column_groups(sy);
  const int64_t tiles = ((n + bn - 1) / bn) * ((m + mib::kMvmBM - 1) / mib::kMvmBM);
  tp.dp_tiles = tiles;
  if (sms < 2 || tiles <= sms) return tp;
  const int64_t waves = (tiles + sms - 1) / sms;
  const int64_t rem = tiles - (waves - 1) * sms;
  const int64_t groups = (kt + flush - 1) / flush;
  if (2 * rem > sms || groups < 2) return tp;
  const SplitPlan sp = split_ranges(kt, flush, groups, sms / rem);
  if (sp.splits < 2) return tp;
  tp.dp_tiles = (waves - 1) * sms;
  tp.splits = sp.splits;
  tp.tiles_per_split = sp.tiles_per_split;
  tp.floats = rem * sp.splits * mib::kMvmBM * bn;
  return tp;
}

// Multiprocessor count of the current device.  A workspace query made where no CUDA device is
// visible (planning on a host without a GPU) plans for a B200's 148 SMs.
int current_sm_count(int* sms) {
  int device = 0, count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    *sms = 148;
    return MIB_OK;
  }
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = mib::device_sm_count(device, sms);
  if (e != cudaSuccess) return cuda_fail(e, "multiprocessor count");
  return MIB_OK;
}

}  // namespace

extern "C" {

const char* mib_last_error(void) { return g_err.c_str(); }

const char* mib_version(void) { return "memintelli_b200 0.1.0 (sm_100a)"; }

uint64_t mib_launch_count(void) { return mib::launch_count(); }

int mib_test_inject_wait_expiry(int64_t wait_limit_cycles) {
  if (wait_limit_cycles < 1 || wait_limit_cycles > mib::kWaitTimeoutCycles)
    return fail(MIB_ERR_PARAM, "wait limit must be in [1, 4e9] cycles");
  g_inject_wait_limit = wait_limit_cycles;
  return MIB_OK;
}

int mib_device_status(void) {
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "device synchronize");
  e = cudaMemcpyFromSymbol(&v, mib::g_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read device error flag");
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(mib::g_device_error, &zero, sizeof(int));
    char buf[96];
    snprintf(buf, sizeof(buf), "a bounded device wait expired (site %d)", v);
    return fail(MIB_ERR_TIMEOUT, buf);
  }
  return MIB_OK;
}

int mib_slice_input(const float* x, int64_t batch, int64_t rows, int64_t cols, int64_t ld_batch, int64_t ld_row,
                    const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, int32_t operand_kind,
                    void* planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                    cudaStream_t stream) {
  SliceTab t;
  if (int r = make_tab(spec, t)) return r;
  if (!x) return fail(MIB_ERR_PARAM, "input is NULL");
  if (batch < 1 || rows < 1 || cols < 1) return fail(MIB_ERR_SHAPE, "input must be non-empty");
  if (int r = check_input_geom(t, spec, kg, cols, rdac, operand_kind, planes, tile_scale, block_max)) return r;
  if (spec->bfp && !block_exp) return fail(MIB_ERR_PARAM, "block floating point needs the exponent buffer");
  mib::SliceArgs a;
  fill_slice_args(a, t, spec, kg, batch, rows, cols, rdac, operand_kind, planes, tile_scale, block_max, block_exp,
                  packed);
  cudaError_t e = mib::slice_dense(x, ld_batch, ld_row, a, stream);
  if (e != cudaSuccess) return cuda_fail(e, "slice_input launch");
  return MIB_OK;
}

// Shared checks of the fused producers; fills `a` on success.
static int fused_input_args(mib::SliceArgs& a, const float* x, int64_t batch, int64_t rows, int64_t cols,
                            const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, int32_t operand_kind,
                            void* planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed) {
  SliceTab t;
  if (int r = make_tab(spec, t)) return r;
  if (!x) return fail(MIB_ERR_PARAM, "input is NULL");
  if (batch < 1 || rows < 1 || cols < 1) return fail(MIB_ERR_SHAPE, "input must be non-empty");
  if (int r = check_input_geom(t, spec, kg, cols, rdac, operand_kind, planes, tile_scale, block_max)) return r;
  if (spec->bfp && !block_exp) return fail(MIB_ERR_PARAM, "block floating point needs the exponent buffer");
  fill_slice_args(a, t, spec, kg, batch, rows, cols, rdac, operand_kind, planes, tile_scale, block_max, block_exp,
                  packed);
  return MIB_OK;
}

int mib_slice_rmsnorm_input(const float* x, int64_t batch, int64_t rows, int64_t cols, int64_t ld_batch,
                            int64_t ld_row, const float* norm_weight, float eps, const mib_slice_spec* spec,
                            const mib_k_geom* kg, int32_t rdac, int32_t operand_kind, void* planes, float* tile_scale,
                            float* block_max, float* block_exp, uint8_t* packed, cudaStream_t stream) {
  mib::SliceArgs a;
  if (int r = fused_input_args(a, x, batch, rows, cols, spec, kg, rdac, operand_kind, planes, tile_scale, block_max,
                               block_exp, packed))
    return r;
  if (!norm_weight) return fail(MIB_ERR_PARAM, "norm weight is NULL");
  cudaError_t e = mib::slice_rmsnorm(x, ld_batch, ld_row, norm_weight, eps, a, stream);
  if (e == cudaErrorNotSupported) return fail(MIB_ERR_UNSUPPORTED, "layout not supported by the fused RMSNorm slicing");
  if (e != cudaSuccess) return cuda_fail(e, "slice_rmsnorm_input launch");
  return MIB_OK;
}

int mib_slice_swiglu_input(const float* gate_up, int64_t batch, int64_t rows, int64_t cols, int64_t ld_batch,
                           int64_t ld_row, int64_t up_offset, const mib_slice_spec* spec, const mib_k_geom* kg,
                           int32_t rdac, int32_t operand_kind, void* planes, float* tile_scale, float* block_max,
                           float* block_exp, uint8_t* packed, cudaStream_t stream) {
  mib::SliceArgs a;
  if (int r = fused_input_args(a, gate_up, batch, rows, cols, spec, kg, rdac, operand_kind, planes, tile_scale,
                               block_max, block_exp, packed))
    return r;
  if (up_offset < cols) return fail(MIB_ERR_SHAPE, "up columns overlap the gate columns");
  cudaError_t e = mib::slice_swiglu(gate_up, ld_batch, ld_row, up_offset, a, stream);
  if (e == cudaErrorNotSupported) return fail(MIB_ERR_UNSUPPORTED, "layout not supported by the fused SwiGLU slicing");
  if (e != cudaSuccess) return cuda_fail(e, "slice_swiglu_input launch");
  return MIB_OK;
}

int mib_qk_norm_rope_bf16(const float* qkv, int64_t tokens, int64_t ld_token, int32_t seq_len, int32_t q_heads,
                          int32_t kv_heads, int32_t head_dim, const float* q_norm, const float* k_norm, float eps,
                          const float* cos_table, const float* sin_table, void* q_out, void* k_out, void* v_out,
                          cudaStream_t stream) {
  if (!qkv || !q_norm || !k_norm || !cos_table || !sin_table || !q_out || !k_out || !v_out)
    return fail(MIB_ERR_PARAM, "NULL buffer");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return fail(MIB_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
  if (tokens < 1 || seq_len < 1 || q_heads < 1 || kv_heads < 1) return fail(MIB_ERR_SHAPE, "empty attention input");
  if (ld_token < static_cast<int64_t>(q_heads + 2 * kv_heads) * head_dim)
    return fail(MIB_ERR_SHAPE, "ld_token is shorter than the q/k/v heads");
  cudaError_t e = mib::qk_norm_rope(qkv, tokens, ld_token, seq_len, q_heads, kv_heads, head_dim, q_norm, k_norm, eps,
                                    cos_table, sin_table, q_out, k_out, v_out, stream);
  if (e != cudaSuccess) return cuda_fail(e, "qk_norm_rope launch");
  return MIB_OK;
}

static int slice_conv_impl(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int32_t kh, int32_t kw,
                           int32_t sh, int32_t sw, int32_t ph, int32_t pw, int32_t dh, int32_t dw,
                           const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, int32_t operand_kind,
                           void* planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                           double vnoise, uint64_t seed, uint64_t call, cudaStream_t stream) {
  SliceTab t;
  if (int r = make_tab(spec, t)) return r;
  if (!x) return fail(MIB_ERR_PARAM, "input is NULL");
  if (n < 1 || c < 1 || h < 1 || w < 1 || kh < 1 || kw < 1 || sh < 1 || sw < 1 || dh < 1 || dw < 1 || ph < 0 || pw < 0)
    return fail(MIB_ERR_SHAPE, "invalid convolution geometry");
  const int64_t ho = (h + 2 * ph - static_cast<int64_t>(dh) * (kh - 1) - 1) / sh + 1;
  const int64_t wo = (w + 2 * pw - static_cast<int64_t>(dw) * (kw - 1) - 1) / sw + 1;
  if (ho < 1 || wo < 1) return fail(MIB_ERR_SHAPE, "convolution output is empty");
  const int64_t cols = c * kh * kw;
  if (int r = check_input_geom(t, spec, kg, cols, rdac, operand_kind, planes, tile_scale, block_max)) return r;
  if (spec->bfp && !block_exp) return fail(MIB_ERR_PARAM, "block floating point needs the exponent buffer");
  mib::SliceArgs a;
  fill_slice_args(a, t, spec, kg, n, ho * wo, cols, rdac, operand_kind, planes, tile_scale, block_max, block_exp,
                  packed);
  if (vnoise != 0.0) {
    if (operand_kind != MIB_OPERAND_FP16) return fail(MIB_ERR_PARAM, "voltage noise needs FP16 planes");
    if (!(vnoise > 0.0)) return fail(MIB_ERR_PARAM, "voltage noise must be positive");
    a.vnoise = static_cast<float>(vnoise);
    a.noise_seed = seed;
    a.noise_stream = (call << 2) | 1u;   // the stream mib_input_noise draws for this call
  }
  cudaError_t e = mib::slice_conv(x, c, h, w, ho, wo, kh, kw, sh, sw, ph, pw, dh, dw, a, stream);
  if (e != cudaSuccess) return cuda_fail(e, "slice_conv_input launch");
  return MIB_OK;
}

int mib_row_logsumexp(const float* logits, int64_t rows, int64_t cols, int64_t ld, const int64_t* targets,
                      int64_t target_offset, float* row_max, float* row_sumexp, float* target_logit,
                      cudaStream_t stream) {
  if (!logits || !row_max || !row_sumexp || (target_logit && !targets)) return fail(MIB_ERR_PARAM, "NULL buffer");
  if (rows < 1 || cols < 1 || ld < cols) return fail(MIB_ERR_SHAPE, "invalid logit block");
  cudaError_t e = mib::row_lse(logits, rows, cols, ld, targets, target_offset, row_max, row_sumexp, target_logit,
                               stream);
  if (e != cudaSuccess) return cuda_fail(e, "row_logsumexp launch");
  return MIB_OK;
}

int mib_slice_conv_input(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int32_t kh, int32_t kw,
                         int32_t sh, int32_t sw, int32_t ph, int32_t pw, int32_t dh, int32_t dw,
                         const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, int32_t operand_kind,
                         void* planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                         cudaStream_t stream) {
  return slice_conv_impl(x, n, c, h, w, kh, kw, sh, sw, ph, pw, dh, dw, spec, kg, rdac, operand_kind, planes,
                         tile_scale, block_max, block_exp, packed, 0.0, 0, 0, stream);
}

int mib_slice_conv_input_noisy(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int32_t kh, int32_t kw,
                               int32_t sh, int32_t sw, int32_t ph, int32_t pw, int32_t dh, int32_t dw,
                               const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, void* planes_fp16,
                               float* tile_scale, float* block_max, float* block_exp, uint8_t* packed, double vnoise,
                               uint64_t seed, uint64_t call, cudaStream_t stream) {
  if (vnoise == 0.0) return fail(MIB_ERR_PARAM, "voltage noise must be positive");
  return slice_conv_impl(x, n, c, h, w, kh, kw, sh, sw, ph, pw, dh, dw, spec, kg, rdac, MIB_OPERAND_FP16, planes_fp16,
                         tile_scale, block_max, block_exp, packed, vnoise, seed, call, stream);
}

int mib_program_weight(const float* w, int64_t k, int64_t n, int64_t stride_k, int64_t stride_n,
                       const mib_slice_spec* spec, const mib_k_geom* kg, const mib_device_spec* dev,
                       const float* stuck_field, const float* write_field, int32_t operand_kind, void* planes,
                       float* g_planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                       cudaStream_t stream) {
  SliceTab t;
  if (int r = make_tab(spec, t)) return r;
  if (!w || !planes || !tile_scale || !block_max || !dev) return fail(MIB_ERR_PARAM, "NULL argument");
  if (k < 1 || n < 1) return fail(MIB_ERR_SHAPE, "weight must be non-empty");
  if (operand_kind != MIB_OPERAND_E4M3 && operand_kind != MIB_OPERAND_FP16)
    return fail(MIB_ERR_PARAM, "unknown operand kind");
  if (int r = check_kgeom(kg, operand_kind)) return r;
  if (spec->paral[0] != kg->p) return fail(MIB_ERR_SHAPE, "weight paral_size[0] must equal the crossbar tile depth");
  if (spec->paral[1] < 1) return fail(MIB_ERR_PARAM, "paral_size must be positive");
  if (spec->quant_gran[0] < 1 || spec->quant_gran[1] < 1 || spec->quant_gran[0] % spec->paral[0] ||
      spec->quant_gran[1] % spec->paral[1])
    return fail(MIB_ERR_PARAM, "quant_gran must be a positive multiple of paral_size");
  const int64_t nbr = (k + spec->quant_gran[0] - 1) / spec->quant_gran[0];
  const int64_t nbc = (n + spec->quant_gran[1] - 1) / spec->quant_gran[1];
  if (nbr * spec->quant_gran[0] != kg->kp) return fail(MIB_ERR_SHAPE, "weight K padding does not match the K geometry");
  if (dev->g_level < 2) return fail(MIB_ERR_PARAM, "The number of the conductance levels should be larger than 1!");
  if (dev->g_level - 1 > max_level_for(operand_kind))
    return fail(MIB_ERR_UNSUPPORTED, "conductance levels do not fit the operand type (use FP16 operands)");
  if (!(dev->lgs < dev->hgs))
    return fail(MIB_ERR_PARAM, "The low conductance state should be smaller than the high conductance state!");
  if (spec->bfp && !block_exp) return fail(MIB_ERR_PARAM, "block floating point needs the exponent buffer");
  if (write_field && !g_planes) return fail(MIB_ERR_PARAM, "write variation needs the conductance planes");
  mib::ProgramArgs a;
  a.k = k;
  a.n = n;
  a.kt = kg->kt;
  a.kp = kg->kp;
  a.p = kg->p;
  a.pp = kg->pp;
  a.qg0 = spec->quant_gran[0];
  a.qg1 = spec->quant_gran[1];
  a.nbr = nbr;
  a.nbc = nbc;
  a.bits = t.bits;
  a.bfp = spec->bfp ? 1 : 0;
  a.n_slices = t.S;
  a.g_level = dev->g_level;
  a.kind = operand_kind;
  for (int i = 0; i < 8; ++i) {
    a.offs[i] = t.offs[i];
    a.maxes[i] = t.maxes[i] ? t.maxes[i] : 1;
  }
  const double qg = (dev->hgs - dev->lgs) / (dev->g_level - 1);
  a.qg_f = static_cast<float>(qg);
  a.lgs_f = static_cast<float>(dev->lgs);
  a.hgs_f = static_cast<float>(dev->hgs);
  a.rate_h = static_cast<float>(dev->rate_stuck_hgs);
  a.rate_l = static_cast<float>(dev->rate_stuck_lgs);
  a.rate_hl = static_cast<float>(dev->rate_stuck_hgs + dev->rate_stuck_lgs);
  a.p0 = spec->paral[0];
  a.p1 = spec->paral[1];
  a.np_pad = nbc * spec->quant_gran[1];
  a.stuck_field = (dev->rate_stuck_hgs > 0 || dev->rate_stuck_lgs > 0) ? stuck_field : nullptr;
  a.write_field = dev->write_variation > 0 ? write_field : nullptr;
  a.planes = planes;
  a.g_planes = g_planes;
  a.row_pitch = kg->kt * kg->pp;
  a.tile_scale = tile_scale;
  a.block_max = block_max;
  a.block_exp = block_exp;
  a.packed = packed;
  cudaError_t e = mib::program_weight(w, stride_k, stride_n, a, stream);
  if (e != cudaSuccess) return cuda_fail(e, "program_weight launch");
  return MIB_OK;
}

int mib_input_noise(const uint8_t* planes_e4m3, __half* out_fp16, int64_t n_elems, double vnoise, uint64_t seed,
                    uint64_t call, cudaStream_t stream) {
  if (!planes_e4m3 || !out_fp16) return fail(MIB_ERR_PARAM, "NULL argument");
  if (n_elems % 8) return fail(MIB_ERR_SHAPE, "element count must be a multiple of 8");
  cudaError_t e = mib::input_noise(planes_e4m3, out_fp16, n_elems, static_cast<float>(vnoise), seed,
                                   (call << 2) | 1u, stream);
  if (e != cudaSuccess) return cuda_fail(e, "input_noise launch");
  return MIB_OK;
}

}  // extern "C"

namespace {

int weight_read_noise(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16, bool split,
                      int64_t n_elems, const mib_device_spec* dev, uint64_t seed, uint64_t call,
                      int background_blocks, cudaStream_t stream) {
  if (background_blocks < 0) return fail(MIB_ERR_PARAM, "background block count must be >= 0");
  if ((!planes_e4m3 && !g_planes) || !out_fp16 || !dev) return fail(MIB_ERR_PARAM, "NULL argument");
  if (n_elems % 4) return fail(MIB_ERR_SHAPE, "element count must be a multiple of 4");
  if (split && n_elems % 8) return fail(MIB_ERR_SHAPE, "element count must be a multiple of 8");
  mib::ReadNoiseArgs a;
  memset(&a, 0, sizeof(a));
  if (dev->g_level < 2 || !(dev->lgs < dev->hgs)) return fail(MIB_ERR_PARAM, "invalid conductance levels");
  const double qg = (dev->hgs - dev->lgs) / (dev->g_level - 1);
  a.qg_f = static_cast<float>(qg);
  a.lgs_f = static_cast<float>(dev->lgs);
  a.inv_qg = static_cast<float>(1.0 / qg);
  a.lgs_over_qg = static_cast<float>(dev->lgs / qg);
  a.g_level = dev->g_level;
  const int ns = std::max(1, dev->n_read_sigma);
  if (ns != 1 && ns != dev->g_level) return fail(MIB_ERR_PARAM, "read variation needs one value or one per level");
  bool any = false, same = true;
  for (int i = 0; i < ns; ++i) {
    a.sigma[i] = dev->read_sigma[i];
    any = any || dev->read_sigma[i] > 0.0f;
    same = same && dev->read_sigma[i] == dev->read_sigma[0];
  }
  // memmat_tensor.py:218-233: identical sigmas skip the level lookup
  a.any_sigma = any ? 1 : 0;
  a.per_level = (any && !same) ? 1 : 0;
  cudaError_t e = mib::read_noise(planes_e4m3, g_planes, out_fp16, split ? out_fp16 + n_elems : nullptr, n_elems, a,
                                  seed, (call << 2) | 2u, background_blocks, stream);
  if (e != cudaSuccess) return cuda_fail(e, "read_noise launch");
  return MIB_OK;
}

}  // namespace

extern "C" {

int mib_weight_read_noise(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16, int64_t n_elems,
                          const mib_device_spec* dev, uint64_t seed, uint64_t call, cudaStream_t stream) {
  return weight_read_noise(planes_e4m3, g_planes, out_fp16, false, n_elems, dev, seed, call, 0, stream);
}

int mib_weight_read_noise_split(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16,
                                int64_t n_elems, const mib_device_spec* dev, uint64_t seed, uint64_t call,
                                cudaStream_t stream) {
  return weight_read_noise(planes_e4m3, g_planes, out_fp16, true, n_elems, dev, seed, call, 0, stream);
}

int mib_weight_read_noise_background(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16,
                                     int64_t n_elems, const mib_device_spec* dev, uint64_t seed, uint64_t call,
                                     int32_t split, int32_t max_blocks, cudaStream_t stream) {
  if (max_blocks < 1) return fail(MIB_ERR_PARAM, "max_blocks must be positive");
  return weight_read_noise(planes_e4m3, g_planes, out_fp16, split != 0, n_elems, dev, seed, call, max_blocks,
                           stream);
}

int mib_adc_plan(const mib_slice_spec* x_spec, const mib_slice_spec* w_spec, const mib_k_geom* kg,
                 const mib_device_spec* dev, int32_t* mode_out, int32_t* table_len_out, int32_t* table_out) {
  SliceTab tx, tw;
  if (int r = make_tab(x_spec, tx)) return r;
  if (int r = make_tab(w_spec, tw)) return r;
  if (!kg || !dev) return fail(MIB_ERR_PARAM, "NULL argument");
  AdcPlan pl;
  if (int r = adc_plan(tx, tw, x_spec, w_spec, kg, dev, pl)) return r;
  if (mode_out) *mode_out = pl.mode;
  const int32_t len = (pl.mode & mib::MODE_LUT) ? tw.S * pl.lut_len : 0;
  if (table_len_out) *table_len_out = len;
  if (table_out && len) {
    for (int j = 0; j < tw.S; ++j)
      for (long long S = 0; S < pl.lut_len; ++S)
        table_out[j * pl.lut_len + S] = static_cast<int32_t>(rne_div(S * pl.R[j], pl.D));
  }
  return MIB_OK;
}

// Split-K scratch in floats for the plan with (mib_mvm) or without (built-in scratch) wave balancing.
static int split_workspace_floats(int64_t m, int64_t n, const mib_slice_spec* x_spec, const mib_slice_spec* w_spec,
                            const mib_k_geom* kg, const mib_device_spec* dev, bool balance, int64_t* floats_out) {
  SliceTab tx, tw;
  if (int r = make_tab(x_spec, tx)) return r;
  if (int r = make_tab(w_spec, tw)) return r;
  if (!kg || !dev || !floats_out) return fail(MIB_ERR_PARAM, "NULL argument");
  AdcPlan pl;
  if (int r = adc_plan(tx, tw, x_spec, w_spec, kg, dev, pl)) return r;
  const SplitPlan sp = split_plan(m, n, kg->kt, pl.flush, tw.S, balance);
  *floats_out = sp.splits > 1 ? static_cast<int64_t>(sp.splits) * m * n : 0;
  if (balance && sp.splits == 1) {
    int sms = 0;
    if (int r = current_sm_count(&sms)) return r;
    *floats_out = tail_plan(m, n, kg->kt, pl.flush, tw.S, sms).floats;
  }
  return MIB_OK;
}

int mib_mvm_workspace(int64_t m, int64_t n, const mib_slice_spec* x_spec, const mib_slice_spec* w_spec,
                      const mib_k_geom* kg, const mib_device_spec* dev, int64_t* floats_out) {
  return split_workspace_floats(m, n, x_spec, w_spec, kg, dev, true, floats_out);
}

int mib_mvm(const void* a_planes, const float* a_scale, int64_t m, const mib_slice_spec* x_spec,
            const void* b_planes, const float* b_scale, int64_t n, const mib_slice_spec* w_spec,
            const mib_k_geom* kg, const mib_device_spec* dev, int32_t operand_kind, const int32_t* adc_table,
            int32_t adc_table_len, float* y, const mib_out_layout* layout, const float* bias, int32_t* acc_dump,
            float* workspace, int64_t workspace_floats, cudaStream_t stream) {
  SliceTab tx, tw;
  if (int r = make_tab(x_spec, tx)) return r;
  if (int r = make_tab(w_spec, tw)) return r;
  if (!a_planes || !a_scale || !b_planes || !b_scale || !y || !layout || !dev)
    return fail(MIB_ERR_PARAM, "NULL argument");
  if (operand_kind != MIB_OPERAND_E4M3 && operand_kind != MIB_OPERAND_FP16 && operand_kind != MIB_OPERAND_FP16_SPLIT)
    return fail(MIB_ERR_PARAM, "unknown operand kind");
  const bool b_split = operand_kind == MIB_OPERAND_FP16_SPLIT;
  const int kind = b_split ? MIB_OPERAND_FP16 : operand_kind;   // element type of both operands' planes
  if (int r = check_kgeom(kg, kind)) return r;
  if (m < 1 || n < 1) return fail(MIB_ERR_SHAPE, "empty matmul");
  if (m > 65535LL * mib::kMvmBM) return fail(MIB_ERR_UNSUPPORTED, "too many rows for one launch");
  if (x_spec->paral[1] != kg->p || w_spec->paral[0] != kg->p)
    return fail(MIB_ERR_SHAPE, "The input data mismatches the shape of weight data!");
  if ((x_spec->bfp != 0) != (w_spec->bfp != 0))
    return fail(MIB_ERR_PARAM, "input and weight must both be INT or both be block floating point");
  if (dev->rdac < 2) return fail(MIB_ERR_PARAM, "The resolution of the DAC should be larger than 1!");
  if (dev->g_level < 2) return fail(MIB_ERR_PARAM, "The number of the conductance levels should be larger than 1!");
  for (int j = 0; j < tw.S; ++j)
    if (tw.maxes[j] > dev->g_level - 1) return fail(MIB_ERR_PARAM, "The weight data is out of the range!");
  AdcPlan pl;
  if (int r = adc_plan(tx, tw, x_spec, w_spec, kg, dev, pl)) return r;
  if ((pl.mode & mib::MODE_LUT) && (!adc_table || adc_table_len != tw.S * pl.lut_len))
    return fail(MIB_ERR_PARAM, "this ADC configuration needs the code table from mib_adc_plan");
  int mode = pl.mode;
  if (acc_dump) {
    if (pl.mode & mib::MODE_FLOATACC)
      return fail(MIB_ERR_UNSUPPORTED, "tile-sum dump needs a uniform ADC without int32 overflow");
    mode |= mib::MODE_DUMP;
  }
  mib::MvmArgs a;
  memset(&a, 0, sizeof(a));
  a.M = m;
  a.N = n;
  a.Kt = kg->kt;
  a.pp = kg->pp;
  a.Sx = tx.S;
  a.Sy = tw.S;
  a.row_bytes = kg->pp * esize(kind);
  const int bn = 16 * mib::mvm_column_groups(tw.S);
  const int b_planes_n = b_split ? 2 * tw.S : tw.S;
  a.a_slice_bytes = static_cast<uint32_t>(mib::kMvmBM * a.row_bytes);
  a.b_slice_bytes = static_cast<uint32_t>(bn * a.row_bytes);
  a.stage_bytes = static_cast<uint32_t>(tx.S) * a.a_slice_bytes + static_cast<uint32_t>(b_planes_n) * a.b_slice_bytes;
  a.b_split = b_split ? 1 : 0;
  a.lut_len = pl.lut_len;
  a.lut = adc_table;
  a.lut_smem = (pl.mode & mib::MODE_LUT) && static_cast<size_t>(tw.S) * pl.lut_len * 4 <= 48 * 1024 ? 1 : 0;
  const size_t budget = 225 * 1024;
  const size_t fixed = 1024 + sizeof(mib::SmemCtl) + (a.lut_smem ? static_cast<size_t>(tw.S) * pl.lut_len * 4 : 0);
  if (fixed + a.stage_bytes > budget) return fail(MIB_ERR_UNSUPPORTED, "one K tile of all slices exceeds shared memory");
  a.stages = static_cast<int32_t>(std::min<size_t>(8, (budget - fixed) / a.stage_bytes));
  a.flush_tiles = pl.flush;
  for (int j = 0; j < 8; ++j) a.cadc[j] = pl.cadc[j];
  uint32_t off = 0;
  for (int i = 0; i < tx.S; ++i)
    for (int j = 0; j < tw.S; ++j) {
      const long long wij = tx.maxes[i] * tw.maxes[j] * tx.coef[i] * tw.coef[j];
      a.wpair[i * 8 + j] = static_cast<int32_t>(wij);
      a.wfpair[i * 8 + j] = static_cast<float>(static_cast<double>(wij) * kg->p / static_cast<double>(pl.R[j]));
      off += static_cast<uint32_t>(wij) * mib::kMagicBits;
    }
  a.tile_offset = off;

  a.out_scale = static_cast<float>(static_cast<double>(kg->p) / static_cast<double>(pl.R[0]));
  a.xs = a_scale;
  a.ws = b_scale;
  a.y = y;
  a.rows_per_group = layout->rows_per_group > 0 ? layout->rows_per_group : m;
  a.group_stride = layout->group_stride;
  a.row_stride = layout->row_stride;
  a.col_stride = layout->col_stride;
  a.bias = bias;
  a.acc_dump = acc_dump;
  SplitPlan sp = split_plan(m, n, kg->kt, pl.flush, tw.S, true);
  if (sp.splits > 1 && (!workspace || workspace_floats < static_cast<int64_t>(sp.splits) * m * n))
    sp = SplitPlan{1, static_cast<int>(kg->kt)};
  a.tiles_per_split = sp.tiles_per_split;
  a.partial = sp.splits > 1 ? workspace : nullptr;
  TailPlan tl = tail_plan(m, n, kg->kt, pl.flush, tw.S, 0);   // no tail split: dp_tiles = every tile
  if (sp.splits == 1 && workspace) {
    int sms = 0;
    if (int r = current_sm_count(&sms)) return r;
    const TailPlan t2 = tail_plan(m, n, kg->kt, pl.flush, tw.S, sms);
    if (t2.splits > 1 && workspace_floats >= t2.floats) tl = t2;
  }
  a.dp_tiles = tl.dp_tiles;
  {
    // a weight operand within 48 MB stays in L2 across row tiles; a larger one is streamed once per band
    // of row tiles whose input planes (about 24 MB) stay in L2 instead
    const double es = esize(kind);
    const double b_bytes = static_cast<double>(n) * kg->kt * kg->pp * es * b_planes_n;
    const double a_tile_bytes = static_cast<double>(mib::kMvmBM) * kg->kt * kg->pp * es * tx.S;
    int64_t band = 1;
    if (b_bytes > 48e6) band = std::max<int64_t>(1, std::min<int64_t>(16, static_cast<int64_t>(24e6 / a_tile_bytes)));
    a.tile_band_rows = band;
  }
  a.tail_splits = tl.splits;
  a.tail_tiles_per_split = tl.tiles_per_split;
  a.tail_partial = tl.splits > 1 ? workspace : nullptr;
  a.wait_limit = mib::kWaitTimeoutCycles;
  if (g_inject_wait_limit > 0) {
    a.wait_limit = g_inject_wait_limit;
    a.hold_mma = 1;
    g_inject_wait_limit = 0;
  }
  CUtensorMap ta, tb;
  if (int r = encode_planes(&ta, a_planes, kind, m, kg->kt * kg->pp, tx.S, kg->pp, mib::kMvmBM)) return r;
  if (int r = encode_planes(&tb, b_planes, kind, n, kg->kt * kg->pp, b_planes_n, kg->pp, bn)) return r;
  cudaError_t e = mib::launch_mvm(ta, tb, a, kind, mode, stream);
  if (e != cudaSuccess) return cuda_fail(e, "mvm launch");
  if (a.partial) {
    e = mib::launch_splitk_reduce(a.partial, sp.splits, m, n, y, a.rows_per_group, a.group_stride, a.row_stride,
                                  a.col_stride, bias, stream);
    if (e != cudaSuccess) return cuda_fail(e, "split-K reduce launch");
  }
  if (a.tail_partial) {
    const int64_t tiles = ((n + bn - 1) / bn) * ((m + mib::kMvmBM - 1) / mib::kMvmBM);
    e = mib::launch_tail_reduce(a.tail_partial, tl.splits, tl.dp_tiles, tiles - tl.dp_tiles, bn, a.tile_band_rows, m,
                                n, y,
                                a.rows_per_group, a.group_stride, a.row_stride, a.col_stride, bias, stream);
    if (e != cudaSuccess) return cuda_fail(e, "tail reduce launch");
  }
  return MIB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// mib_mvm_static_scratch: the fused MVM for callers that cannot allocate device memory
// (an allocator-less runtime, a host without the CUDA allocator at hand, or a caller
// that must not grow its memory footprint while running).  The split-K partial
// outputs live in a fixed array compiled into this library instead of a
// caller-provided workspace.
// ---------------------------------------------------------------------------
namespace {

// Split-K scratch: 2^20 floats (4 MiB).  Every GPU that loads this library holds
// this array until the process exits.
constexpr int64_t kStaticScratchFloats = int64_t(1) << 20;
static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];

// Device address of g_static_scratch per device, resolved on the first call on that
// device (with it current).  Host code must not pass the symbol itself to a kernel.
std::mutex g_static_scratch_mu;
float* g_static_scratch_ptr[128] = {};

int static_scratch_address(float** out) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device < 0 || device >= 128) return fail(MIB_ERR_CUDA, "device index out of range for the static scratch");
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (!g_static_scratch_ptr[device]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static split-K scratch)");
    g_static_scratch_ptr[device] = static_cast<float*>(p);
  }
  *out = g_static_scratch_ptr[device];
  return MIB_OK;
}

}  // namespace

extern "C" int mib_mvm_static_scratch(const void* a_planes, const float* a_scale, int64_t m,
                                      const mib_slice_spec* x_spec, const void* b_planes, const float* b_scale,
                                      int64_t n, const mib_slice_spec* w_spec, const mib_k_geom* kg,
                                      const mib_device_spec* dev, int32_t operand_kind, const int32_t* adc_table,
                                      int32_t adc_table_len, float* y, const mib_out_layout* layout,
                                      const float* bias, cudaStream_t stream) {
  // Scratch is needed only where the grid underfills the GPU; the optional wave-balancing split
  // of mib_mvm is skipped here (mib_mvm runs unsplit when handed no or too little workspace).
  int64_t need = 0;
  if (int r = split_workspace_floats(m, n, x_spec, w_spec, kg, dev, false, &need)) return r;
  if (need > kStaticScratchFloats) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "this MVM needs %lld floats of split-K scratch but the built-in scratch holds %lld; "
             "use mib_mvm with a caller-provided workspace",
             static_cast<long long>(need), static_cast<long long>(kStaticScratchFloats));
    return fail(MIB_ERR_UNSUPPORTED, buf);
  }
  float* scratch = nullptr;
  if (need > 0) {
    if (int r = static_scratch_address(&scratch)) return r;
  }
  return mib_mvm(a_planes, a_scale, m, x_spec, b_planes, b_scale, n, w_spec, kg, dev, operand_kind, adc_table,
                 adc_table_len, y, layout, bias, nullptr, scratch, need > 0 ? kStaticScratchFloats : 0, stream);
}
