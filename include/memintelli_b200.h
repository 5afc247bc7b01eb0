/*
 * memintelli_b200.h -- C ABI of the B200 (sm_100a) compute-in-memory sliced matmul.
 *
 * The reference (zhuizhou/memintelli_flash) is pure Python/PyTorch; each entry
 * point below replaces a torch op chain of its hot path and names it.  All
 * pointers are device pointers (except the spec structs, which are host
 * memory read during the call); sizes are elements unless stated; every call
 * is asynchronous on `stream` and allocates nothing -- the caller owns every
 * buffer.  Return value: MIB_OK or one of the MIB_ERR_* codes, with a message
 * available from mib_last_error().
 *
 * Data layout in HBM (all row-major, last index fastest):
 *   operand planes  [S][rows][Kt * pp]   one plane per bit slice, LSB-first;
 *                    K is split into Kt crossbar tiles of p rows each, every
 *                    tile padded to pp = round_up(p, 32 bytes / element size)
 *                    elements with zeros.  Element = the DAC level (inputs) or
 *                    conductance level (weights) encoded as E4M3 (exact for
 *                    levels <= 16) or FP16 (exact integers; noisy values).
 *   tile scales     [Kt][rows] fp32      dequantisation factor of the quant
 *                    block that holds (row, tile): bmax/(2^(bits-1)-1) for INT,
 *                    2^(e+2-bits) for block floating point.
 *   packed codes    [rows][Kp] uint8     two's complement quantised value
 *                    (all slices of one element), K padded to Kp.
 *   block max / exp [batch][nbr][nbc] fp32 (SlicedData.max_data / e_bias).
 */
#ifndef MEMINTELLI_B200_H
#define MEMINTELLI_B200_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MIB_OK 0
#define MIB_ERR_PARAM 1       /* invalid parameter value  (reference: ValueError)          */
#define MIB_ERR_SHAPE 2       /* shape / layout mismatch  (reference: ValueError)          */
#define MIB_ERR_UNSUPPORTED 3 /* configuration not implemented (reference: NotImplementedError) */
#define MIB_ERR_CUDA 4        /* CUDA runtime or driver error                               */
#define MIB_ERR_TIMEOUT 5     /* a bounded device-side wait expired (reported by mib_device_status) */

#define MIB_OPERAND_E4M3 0
#define MIB_OPERAND_FP16 1
/* FP16 input planes; weight planes as FP16 hi planes followed by FP16 lo planes ([2*S][N][Kt*pp], from
 * mib_weight_read_noise_split): each crossbar MMA is followed by one on the lo planes into the same fp32
 * accumulator, so non-integer conductances enter at 22 significand bits. */
#define MIB_OPERAND_FP16_SPLIT 2

#define MIB_MAX_SLICES 8
#define MIB_MAX_LEVELS 256

/* Bit-slicing and quantisation of one operand (memintelli/pimpy/data_formats.py:21-58, 116-207). */
typedef struct mib_slice_spec {
  int32_t n_slices;                       /* S, 1..8                                        */
  int32_t slice_method[MIB_MAX_SLICES];   /* MSB-first widths, slice_method[0] == 1          */
  int32_t bfp;                            /* 0: INT (utils.py:44-83), 1: BFP (utils.py:86-128) */
  int32_t paral[2];                       /* paral_size (rows, cols)                          */
  int32_t quant_gran[2];                  /* decoded quant_gran, already rounded up to paral  */
} mib_slice_spec;

/* Crossbar device model (memintelli/pimpy/memmat_tensor.py:30-115). */
typedef struct mib_device_spec {
  double hgs, lgs;              /* high / low conductance state                               */
  int32_t g_level;              /* conductance levels                                         */
  int32_t rdac;                 /* DAC resolution                                             */
  int32_t n_radc;               /* 1: uniform ADC; else one entry per weight slice             */
  int32_t radc[MIB_MAX_SLICES]; /* ADC resolution, LSB-first weight-slice order (list flipped) */
  double vread;                 /* read voltage                                               */
  double vnoise;                /* relative voltage noise std                                 */
  double write_variation;       /* relative write variation std                               */
  double rate_stuck_hgs, rate_stuck_lgs;
  int32_t n_read_sigma;         /* 1: uniform read variation; g_level: per level              */
  float read_sigma[MIB_MAX_LEVELS];
} mib_device_spec;

/* Output placement: y[(r / rows_per_group) * group_stride + (r % rows_per_group) * row_stride
 *                     + n * col_stride] for matmul row r and output column n.
 * Linear (M,N) / (B,T,N): rows_per_group = rows, row_stride = N, col_stride = 1.
 * Conv NCHW:  rows_per_group = Ho*Wo, group_stride = Cout*Ho*Wo, row_stride = 1, col_stride = Ho*Wo. */
typedef struct mib_out_layout {
  int64_t rows_per_group;
  int64_t group_stride;
  int64_t row_stride;
  int64_t col_stride;
} mib_out_layout;

/* Geometry of the K dimension shared by both operands. */
typedef struct mib_k_geom {
  int64_t k;        /* true reduction length                           */
  int64_t kp;       /* padded length (multiple of both quant blocks)   */
  int32_t p;        /* crossbar tile depth (input paral[1] == weight paral[0]) */
  int32_t pp;       /* tile depth padded to the MMA K step             */
  int64_t kt;       /* number of tiles, kp / p                         */
} mib_k_geom;

/* Quantise + bit-slice an input matrix (batch, rows, cols) into DAC-level planes.
 * Replaces SlicedData.slice_data_imp for inputs: data_formats.py:95-114,116-207 with
 * quant_map_tensor / bfp_map_tensor (utils.py:44-128) and the DAC step of
 * DPETensor._dot_inference (memmat_tensor.py:295-297 / 358-360).
 * x[b*ld_batch + r*ld_row + c] (c contiguous).  `packed` may be NULL. */
int mib_slice_input(const float* x, int64_t batch, int64_t rows, int64_t cols, int64_t ld_batch, int64_t ld_row,
                    const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, int32_t operand_kind,
                    void* planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                    cudaStream_t stream);

/* Same for a convolution input (N,C,H,W) lowered without im2col: matmul row
 * r = n*Ho*Wo + oh*Wo + ow, column c*kh*kw + i*kw + j, the order of F.unfold
 * used by Conv2dMem (memintelli/NN_layers/convolution.py:105-121). */
int mib_slice_conv_input(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int32_t kh, int32_t kw,
                         int32_t sh, int32_t sw, int32_t ph, int32_t pw, int32_t dh, int32_t dw,
                         const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, int32_t operand_kind,
                         void* planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                         cudaStream_t stream);

/* mib_slice_conv_input with the call's voltage noise applied while the planes are written
 * (memmat_tensor.py:297-299: V * (1 + vnoise * N(0,1)) per input element and slice, shared by all output
 * columns).  The planes are FP16; the normals are the ones mib_input_noise(seed, call) would draw for the
 * same plane elements, so this equals mib_slice_conv_input to E4M3 followed by mib_input_noise, bit for
 * bit, in one pass.  For a layer that slices its input once per multiply (Conv2dMem). */
int mib_slice_conv_input_noisy(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int32_t kh, int32_t kw,
                               int32_t sh, int32_t sw, int32_t ph, int32_t pw, int32_t dh, int32_t dw,
                               const mib_slice_spec* spec, const mib_k_geom* kg, int32_t rdac, void* planes_fp16,
                               float* tile_scale, float* block_max, float* block_exp, uint8_t* packed, double vnoise,
                               uint64_t seed, uint64_t call, cudaStream_t stream);

/* Fused producers of an input (no reference counterpart).  Each slices a row transform of x with
 * the same arguments and buffers as mib_slice_input, without materialising the transformed matrix;
 * in the reference they are a torch pass followed by SlicedData.slice_data_imp.  Both need one-row
 * input quant blocks (quant_gran[0] == 1), unpadded power-of-two tiles, power-of-two quant blocks
 * of at most 128 columns, cols % 4 == 0 and 16-byte aligned rows; otherwise they return
 * MIB_ERR_UNSUPPORTED and the caller runs the transform and mib_slice_input.
 *
 * mib_slice_rmsnorm_input: row-wise RMSNorm, y = x * rsqrt(mean(x^2) + eps) * norm_weight
 * (norm_weight: cols floats, 16-byte aligned).  The sum of squares is a warp reduction, so y can
 * differ from torch's in the last fp32 bit. */
int mib_slice_rmsnorm_input(const float* x, int64_t batch, int64_t rows, int64_t cols, int64_t ld_batch,
                            int64_t ld_row, const float* norm_weight, float eps, const mib_slice_spec* spec,
                            const mib_k_geom* kg, int32_t rdac, int32_t operand_kind, void* planes, float* tile_scale,
                            float* block_max, float* block_exp, uint8_t* packed, cudaStream_t stream);

/* mib_slice_swiglu_input: SwiGLU of a fused gate/up activation, y[c] = silu(x[c]) * x[up_offset + c]
 * for c < cols (silu(g) = g / (1 + exp(-g))); up_offset % 4 == 0. */
int mib_slice_swiglu_input(const float* gate_up, int64_t batch, int64_t rows, int64_t cols, int64_t ld_batch,
                           int64_t ld_row, int64_t up_offset, const mib_slice_spec* spec, const mib_k_geom* kg,
                           int32_t rdac, int32_t operand_kind, void* planes, float* tile_scale, float* block_max,
                           float* block_exp, uint8_t* packed, cudaStream_t stream);

/* Quantise, slice and program a weight matrix W (K, N) into conductance-level planes.
 * Replaces SlicedData.slice_data_imp for weights + DPETensor._num2G (memmat_tensor.py:160-202):
 * level = round(code/m*(g-1)); stuck-at faults from `stuck_field` (torch.rand with the
 * reference's fixed seed 123, reference G layout (Kp/p0, Np/p1, S, p0, p1)); when
 * `write_field` (fixed seed 42 draw of N(0, wv), same layout) is given the fp32
 * conductance planes `g_planes` ([S][N][Kt*pp], siemens, as DPETensor keeps G) are written.
 * W element (k, n) at w[k*stride_k + n*stride_n]. */
int mib_program_weight(const float* w, int64_t k, int64_t n, int64_t stride_k, int64_t stride_n,
                       const mib_slice_spec* spec, const mib_k_geom* kg, const mib_device_spec* dev,
                       const float* stuck_field, const float* write_field, int32_t operand_kind, void* planes,
                       float* g_planes, float* tile_scale, float* block_max, float* block_exp, uint8_t* packed,
                       cudaStream_t stream);

/* Per-call input voltage noise (memmat_tensor.py:297-299): out = level * (1 + vnoise * N(0,1)),
 * E4M3 level planes in, FP16 planes out; vnoise == 0 converts only.  Counter-based
 * Philox normals keyed by (seed, call). */
int mib_input_noise(const uint8_t* planes_e4m3, __half* out_fp16, int64_t n_elems, double vnoise, uint64_t seed,
                    uint64_t call, cudaStream_t stream);

/* Per-call read variation (memmat_tensor.py:204-236): G' = G * exp(sigma(level) * N(0,1)),
 * out = (G' - LGS) / Q_G as FP16.  G comes from `g_planes` when non-NULL (write variation
 * present), else from the E4M3 level planes as level*Q_G + LGS. */
int mib_weight_read_noise(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16, int64_t n_elems,
                          const mib_device_spec* dev, uint64_t seed, uint64_t call, cudaStream_t stream);

/* mib_weight_read_noise for the split weight operand (MIB_OPERAND_FP16_SPLIT): `out_fp16` holds
 * 2 * n_elems halves, the FP16 rounding of every value followed by the FP16 rounding of its residual,
 * so that hi + lo carries 22 significand bits.  Used for conductances with write variation, whose
 * fixed-seed draw the reference evaluates in fp32 (memmat_tensor.py:175-180, 260-409).  n_elems must be
 * a multiple of 8. */
int mib_weight_read_noise_split(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16,
                                int64_t n_elems, const mib_device_spec* dev, uint64_t seed, uint64_t call,
                                cudaStream_t stream);

/* mib_weight_read_noise (split != 0: mib_weight_read_noise_split) as a background pass: at most
 * `max_blocks` blocks of 128 threads, each small enough to run on an SM beside a crossbar MVM CTA, so
 * that a pass launched on a second stream ahead of its multiply overlaps the crossbar work running
 * before it.  Same draws and outputs as the foreground entry points. */
int mib_weight_read_noise_background(const uint8_t* planes_e4m3, const float* g_planes, __half* out_fp16,
                                     int64_t n_elems, const mib_device_spec* dev, uint64_t seed, uint64_t call,
                                     int32_t split, int32_t max_blocks, cudaStream_t stream);

/* ADC plan for one MVM configuration.  In the noise-free mode the ADC code
 * round_half_even(S * (radc_j - 1) / D) must be exact for every reachable
 * crossbar sum S in [0, D]; when a single fp32 multiply-add cannot guarantee
 * that (a non-dyadic ratio with half-way ties) the MVM needs a code table of
 * *table_len_out int32 entries, filled into `table_out` (host memory, may be
 * NULL) and passed to mib_mvm in device memory.  *mode_out receives the
 * epilogue variant (bit 0: code table, bit 1: fp32 accumulation).
 * Mirrors the checks of DPETensor.__init__ / _validate_radc_with_slices
 * (memmat_tensor.py:98-127). */
int mib_adc_plan(const mib_slice_spec* x_spec, const mib_slice_spec* w_spec, const mib_k_geom* kg,
                 const mib_device_spec* dev, int32_t* mode_out, int32_t* table_len_out, int32_t* table_out);

/* Fused crossbar MVM: for every K tile and slice pair, tile partial sums on tcgen05
 * tensor cores (accumulators in TMEM), ADC round(S * (radc_j-1) / D) with
 * D = (rdac-1)(g_level-1)p, shift-add over slice pairs, block rescale, K-tile sum
 * and crop.  Replaces DPETensor.__call__ / MapReduceDot -> _dot_inference / _dot
 * (memmat_tensor.py:129-158, 260-495; utils.py:11-29).  a_planes [Sx][M][Kt*pp],
 * a_scale [Kt][M]; b_planes [Sy][N][Kt*pp], b_scale [Kt][N]; both E4M3 or both FP16.
 * `adc_table` as returned by mib_adc_plan (NULL when none is needed).  `bias` (N)
 * may be NULL.  `acc_dump`, when non-NULL, receives the exact int32 slice-pair
 * sums acc[t][r][n] = sum_ij code_ij * m_i m_j c_i c_j of every tile t (test hook).
 * `workspace` / `workspace_floats`: split-K scratch sized by mib_mvm_workspace (may be NULL). */
int mib_mvm(const void* a_planes, const float* a_scale, int64_t m, const mib_slice_spec* x_spec,
            const void* b_planes, const float* b_scale, int64_t n, const mib_slice_spec* w_spec,
            const mib_k_geom* kg, const mib_device_spec* dev, int32_t operand_kind, const int32_t* adc_table,
            int32_t adc_table_len, float* y, const mib_out_layout* layout, const float* bias, int32_t* acc_dump,
            float* workspace, int64_t workspace_floats, cudaStream_t stream);

/* Split-K workspace for mib_mvm, in floats (0 when the output tiles already fill the GPU).
 * mib_mvm divides the K tiles into contiguous ranges in two cases:
 *   - fewer than ~3/4 of the 148 SMs would get an output tile;
 *   - the grid spans up to 4 waves and the last wave is partly idle.  It then uses the 2-4
 *     ranges that cut the wave-rounded time by at least 10% (e.g. 2048 x 1024 outputs).
 * It writes one fp32 partial output per range into `workspace` ([splits][M][N]) and adds them
 * in a fixed order (deterministic).  A NULL or smaller workspace runs the MVM without
 * splitting. */
int mib_mvm_workspace(int64_t m, int64_t n, const mib_slice_spec* x_spec, const mib_slice_spec* w_spec,
                      const mib_k_geom* kg, const mib_device_spec* dev, int64_t* floats_out);

/* mib_mvm for callers that cannot allocate device memory: no counterpart in the reference
 * (whose torch path allocates freely).  It is meant for runtimes without a CUDA allocator
 * at hand and for callers that must not allocate while they run.  Same arguments and
 * result as mib_mvm without the workspace (and without the acc_dump test hook).  When
 * the output tiles fill less of the GPU than split-K needs, the split-K partials go to
 * a scratch array built into this library: 2^20 floats (4 MiB), held on every GPU that
 * loads the library until the process exits.  Problems whose underfilled-grid split needs
 * more than 2^20 floats are rejected with MIB_ERR_UNSUPPORTED.  The wave-balancing split
 * of mib_mvm is not used here; those problems run unsplit.
 * The first call on a device resolves the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture.  The array is shared by every call
 * and keeps the last call's contents (every split overwrites all of its partials before
 * they are read, so nothing needs clearing); calls that overlap on the GPU, e.g. on two
 * streams, race on it. */
int mib_mvm_static_scratch(const void* a_planes, const float* a_scale, int64_t m, const mib_slice_spec* x_spec,
                           const void* b_planes, const float* b_scale, int64_t n, const mib_slice_spec* w_spec,
                           const mib_k_geom* kg, const mib_device_spec* dev, int32_t operand_kind,
                           const int32_t* adc_table, int32_t adc_table_len, float* y, const mib_out_layout* layout,
                           const float* bias, cudaStream_t stream);

/* Attention input preparation for the Qwen3 prefill driver (outside the reference's CIM path, no
 * reference counterpart).  From the fused q/k/v crossbar output (tokens rows of ld_token floats: q heads,
 * then k heads, then v heads, head_dim each; token i is position i % seq_len) it writes bf16
 * q (tokens, q_heads, head_dim), k and v (tokens, kv_heads, head_dim):
 *   q = rope(rms_norm(q) * q_norm), k = rope(rms_norm(k) * k_norm), v = v,
 * rms_norm(x) = x * rsqrt(mean(x^2) + eps) and rope(x) = x * cos + rotate_half(x) * sin with
 * rotate_half(x) = cat(-x[D/2:], x[:D/2]); cos and sin are (seq_len, head_dim) fp32.
 * head_dim is 64, 128 or 256. */
int mib_qk_norm_rope_bf16(const float* qkv, int64_t tokens, int64_t ld_token, int32_t seq_len, int32_t q_heads,
                          int32_t kv_heads, int32_t head_dim, const float* q_norm, const float* k_norm, float eps,
                          const float* cos_table, const float* sin_table, void* q_out, void* k_out, void* v_out,
                          cudaStream_t stream);

/* Row log-sum-exp of a logit block for the Qwen3 prefill driver's loss (outside the reference's CIM path, no
 * reference counterpart; the reference's HF model computes the loss in torch).  For each row r of the
 * (rows, cols) block at logits[r * ld + c]: row_max[r] = max_c, row_sumexp[r] = sum_c exp(logit - row_max[r]),
 * and, when target_logit is non-NULL, target_logit[r] = the logit at column targets[r] - target_offset if
 * that column is inside the block, else 0.  Vocabulary shards combine as M = max over shards,
 * S = sum of row_sumexp * exp(row_max - M), loss = log S + M - target. */
int mib_row_logsumexp(const float* logits, int64_t rows, int64_t cols, int64_t ld, const int64_t* targets,
                      int64_t target_offset, float* row_max, float* row_sumexp, float* target_logit,
                      cudaStream_t stream);

/* Reads and clears the device-side error flag of the current device (synchronises it).
 * Returns MIB_OK, or MIB_ERR_TIMEOUT when a kernel gave up a bounded wait. */
int mib_device_status(void);

/* Test hook for the failure path of the bounded device waits (no reference counterpart; the reference
 * has no device-side waits).  Arms a one-shot flag on the calling thread: the next mib_mvm launched
 * from it runs with its MMA warp held (it issues and commits nothing, so no accumulator ever becomes
 * ready) and with `wait_limit_cycles` (1 .. 4e9) as the limit of its abortable mbarrier waits.  The
 * epilogue's first wait then runs out; the kernel raises its abort flag, drains its in-flight copies,
 * frees its tensor memory and returns, leaving that call's output undefined, and the next
 * mib_device_status() returns MIB_ERR_TIMEOUT.  Later launches are unaffected. */
int mib_test_inject_wait_expiry(int64_t wait_limit_cycles);

/* Message of the last error returned on this thread. */
const char* mib_last_error(void);

/* Library version string. */
const char* mib_version(void);

/* Number of CUDA kernels this library has launched in the process (all devices). */
uint64_t mib_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* MEMINTELLI_B200_H */
