// Kernel argument blocks and launcher declarations shared by the CUDA sources
// and the C-ABI layer.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace mib {

struct SliceArgs {
  int64_t batch, rows, cols;      // matmul view of the input
  int64_t nbr, nbc;               // quant blocks per batch along rows / cols
  int32_t qg0, qg1;               // quant block (rounded to paral)
  int32_t p, pp;                  // crossbar tile depth and padded depth
  int64_t kt, kp;                 // tiles, padded K
  int32_t bits, bfp, n_slices, lm1, kind;
  int32_t offs[8], maxes[8];      // LSB-first bit offset and max code per slice
  void* planes;                   // [S][batch*rows][kt*pp]
  int64_t plane_stride;           // batch*rows*kt*pp
  int64_t row_pitch;              // kt*pp
  float* tile_scale;              // [kt][scale_ld]
  int64_t scale_ld;               // batch*rows
  float* block_max;               // [batch][nbr][nbc]
  float* block_exp;               // same or null
  uint8_t* packed;                // [batch*rows][kp] or null
  float vnoise;                   // FP16 planes only: per-call voltage noise applied while storing (0: none)
  uint64_t noise_seed, noise_stream;
};

struct ProgramArgs {
  int64_t k, n, kt, kp;
  int32_t p, pp, qg0, qg1;
  int64_t nbr, nbc;
  int32_t bits, bfp, n_slices, g_level, kind;
  int32_t offs[8], maxes[8];
  float qg_f, lgs_f, hgs_f, rate_h, rate_l, rate_hl;  // rate_hl = fp32(rate_h + rate_l)
  int32_t p0, p1;                 // weight paral (reference G tile)
  int64_t np_pad;                 // reference padded N (G layout)
  const float* stuck_field;
  const float* write_field;
  void* planes;                   // [S][n][kt*pp]
  float* g_planes;                // [S][n][kt*pp] conductance (siemens) or null
  int64_t row_pitch;              // kt*pp
  float* tile_scale;              // [kt][n]
  float* block_max;               // [nbr][nbc]
  float* block_exp;
  uint8_t* packed;                // [n][kp] or null
};

struct ReadNoiseArgs {
  float qg_f, lgs_f;
  float inv_qg, lgs_over_qg;      // 1 / Q_G and LGS / Q_G
  int32_t any_sigma, per_level, g_level;
  float sigma[256];
};

// MVM epilogue variants.  The ADC code of a crossbar sum S is taken either
// from one fused multiply-add with a magic constant (rne(S*c_j), exact when
// verified on the host for every reachable S) or from a per-slice code table
// (exact for any ADC ratio).  Codes are accumulated over slice pairs either in
// exact modular int32 (uniform ADC) or in fp32 (per-slice ADC resolution, or
// when int32 could overflow).
enum MvmMode : int {
  MODE_LUT = 1,       // bit 0: code table instead of the magic-constant rounding
  MODE_FLOATACC = 2,  // bit 1: fp32 accumulation
  MODE_DUMP = 4,      // bit 2: write the exact int32 tile sums (test hook)
};

constexpr int kMvmBM = 128;
constexpr int kMaxLut = 4096;

struct MvmArgs {
  int64_t M, N, Kt;
  int32_t pp, Sx, Sy, stages, row_bytes;
  uint32_t a_slice_bytes, b_slice_bytes, stage_bytes;
  int32_t flush_tiles;
  float cadc[8];            // per weight slice: (radc_j - 1) / D
  int32_t wpair[64];        // [i*8+j] exact shift-add weight m_i m_j c_i c_j
  float wfpair[64];         // [i*8+j] w_ij * p / R_j  (ACC_FLOAT)
  uint32_t tile_offset;     // sum_ij w_ij * bits(magic), mod 2^32 (ACC_INT)
  float out_scale;          // p / R (ACC_INT, ACC_LUT)
  int32_t lut_len;          // entries per weight slice in the code table
  int32_t lut_smem;         // 1: copy the table to shared memory; 0: read it from global memory
  const int32_t* lut;       // [Sy][lut_len] ADC codes (MODE_LUT)
  const float* xs;          // [Kt][M]
  const float* ws;          // [Kt][N]
  float* y;
  int64_t rows_per_group, group_stride, row_stride, col_stride;
  const float* bias;
  int32_t* acc_dump;        // [Kt][M][N] or null
  int32_t tiles_per_split;  // K tiles per CTA along grid z (== Kt without split-K)
  float* partial;           // split-K: [splits][M][N] fp32 partial outputs, or null
  // Persistent launches (no split-K): output tiles [0, dp_tiles) are stepped whole, CTA b taking tiles
  // b, b + grid, ...  With tail_splits > 1 the remaining tiles (a partly idle last wave) are cut into
  // tail_splits K ranges of tail_tiles_per_split K tiles; CTA b takes range b % tail_splits of tile
  // dp_tiles + b / tail_splits and writes it to tail_partial[b][128][BN], summed by tail_reduce.
  int64_t dp_tiles;
  // Tile order of a persistent launch: bands of tile_band_rows row tiles, each band column by column.
  // 1 (row by row) keeps each row tile's input planes in L2 while all weight columns pass; a weight
  // operand too large for L2 (a wide lm_head) gets bands whose input planes fit, so that the weights
  // stream from DRAM once per band instead of once per row tile.
  int64_t tile_band_rows;
  int32_t tail_splits;
  int32_t tail_tiles_per_split;
  float* tail_partial;
  int64_t wait_limit;       // cycles after which an abortable mbarrier wait gives up (about 2 s normally)
  int32_t hold_mma;         // test hook: the MMA warp issues nothing, so the epilogue's first wait runs out
  int32_t b_split;          // 1: the weight planes are FP16 hi planes followed by lo planes ([2*Sy][N][K]);
                            // every (K tile, input slice) MMA is followed by one on the lo planes
};

cudaError_t slice_dense(const float* x, int64_t ld_batch, int64_t ld_row, SliceArgs a, cudaStream_t stream);
cudaError_t slice_rmsnorm(const float* x, int64_t ld_batch, int64_t ld_row, const float* w, float eps, SliceArgs a,
                          cudaStream_t stream);
cudaError_t slice_swiglu(const float* x, int64_t ld_batch, int64_t ld_row, int64_t up_offset, SliceArgs a,
                         cudaStream_t stream);
cudaError_t slice_conv(const float* x, int64_t C, int64_t H, int64_t W, int64_t Ho, int64_t Wo, int kh, int kw, int sh,
                       int sw, int ph, int pw, int dh, int dw, SliceArgs a, cudaStream_t stream);
cudaError_t program_weight(const float* w, int64_t stride_k, int64_t stride_n, ProgramArgs a, cudaStream_t stream);
cudaError_t input_noise(const uint8_t* in, __half* out, int64_t n, float vnoise, uint64_t seed, uint64_t stream_id,
                        cudaStream_t stream);
cudaError_t read_noise(const uint8_t* levels, const float* gp, __half* out, __half* out_lo, int64_t n,
                       ReadNoiseArgs a, uint64_t seed, uint64_t stream_id, int background_blocks,
                       cudaStream_t stream);
void launch_block_exp(const float* bmax, float* bexp, int64_t n, cudaStream_t stream);
cudaError_t qk_norm_rope(const float* qkv, int64_t tokens, int64_t ld_token, int seq_len, int q_heads, int kv_heads,
                         int head_dim, const float* q_norm, const float* k_norm, float eps, const float* cos_t,
                         const float* sin_t, void* q_out, void* k_out, void* v_out, cudaStream_t stream);
cudaError_t row_lse(const float* x, int64_t rows, int64_t cols, int64_t ld, const int64_t* targets,
                    int64_t target_offset, float* row_max, float* row_sumexp, float* target_logit,
                    cudaStream_t stream);
void count_launch(int n = 1);
size_t mvm_smem_bytes(const MvmArgs& a);
cudaError_t launch_splitk_reduce(const float* partial, int splits, int64_t M, int64_t N, float* y,
                                 int64_t rows_per_group, int64_t group_stride, int64_t row_stride,
                                 int64_t col_stride, const float* bias, cudaStream_t stream);
int mvm_column_groups(int sy);   // output tile width BN = 16 * mvm_column_groups(Sy)
cudaError_t launch_tail_reduce(const float* tail_partial, int splits, int64_t dp_tiles, int64_t tail_tiles, int bn,
                               int64_t band, int64_t M, int64_t N, float* y, int64_t rows_per_group, int64_t group_stride,
                               int64_t row_stride, int64_t col_stride, const float* bias, cudaStream_t stream);
// Multiprocessor count of `device`, cached per device.
cudaError_t device_sm_count(int device, int* sms);
cudaError_t launch_mvm(const CUtensorMap& ta, const CUtensorMap& tb, const MvmArgs& a, int kind, int acc_mode,
                       cudaStream_t stream);

}  // namespace mib
