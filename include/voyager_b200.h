/*
 * voyager_b200 -- C ABI of the B200 (sm_100a) quantization numerics library.
 *
 * Each entry point replaces one op of the reference's `quantized_ops`
 * torch.library (Joejoedesu/voyager-compiler,
 * src/voyager_compiler/ops/quantized.py) on CUDA tensors.  The reference binds
 * these ops from Python; the matching ctypes binding lives in
 * voyager_b200/_lib.py and the torch.library registration that makes exported
 * graphs dispatch here in voyager_b200/ops.py.
 *
 * Conventions
 *   - Tensors are dense, row-major (C-contiguous) device buffers described by
 *     vq_tensor; the caller allocates every output.  Entry points that launch
 *     work never allocate, never synchronise the host and are ordered on the
 *     `stream` argument (a cudaStream_t; NULL = the legacy default stream).
 *   - bfloat16 values are carried as their 16-bit patterns.
 *   - Every function returns a vq_status; nothing traps on the device.
 *     vq_status_string() names a status.  Invalid shapes, dtypes and sizes are
 *     rejected before any launch.
 *   - Rounding is bit-exact with the reference's eager CPU ops: binary ops are
 *     evaluated in float32 and rounded once to the result dtype (a 0-d scale
 *     keeps its float32 value and does not promote the result), and the
 *     element rounding is the reference's 65,536-entry bf16-indexed table,
 *     which vq_rounder_from_table() turns into a rounder the kernels evaluate.
 */
#ifndef VOYAGER_B200_H_
#define VOYAGER_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum vq_status {
  VQ_OK = 0,
  VQ_ERR_INVALID = 1,      /* bad argument value (sizes, block size, axes) */
  VQ_ERR_UNSUPPORTED = 2,  /* dtype / layout combination not provided      */
  VQ_ERR_ALIGNMENT = 3,    /* pointer or extent alignment not met          */
  VQ_ERR_CUDA = 4,         /* a CUDA runtime call failed                   */
  VQ_ERR_SHAPE = 5,        /* shapes do not broadcast as the op requires   */
  VQ_ERR_NULL = 6,         /* required pointer is NULL                     */
  VQ_ERR_TIMEOUT = 7,      /* a bounded device wait gave up                */
  VQ_ERR_TOO_LARGE = 8     /* problem exceeds a fixed-size scratch area    */
} vq_status;

typedef enum vq_dtype {
  VQ_BF16 = 0,
  VQ_F32 = 1,
  VQ_F16 = 2,
  VQ_I64 = 3,
  VQ_U8 = 4,
  VQ_I32 = 5
} vq_dtype;

#define VQ_MAX_DIMS 8

/* A dense row-major device tensor.  ndim == 0 is a 0-d (scalar) tensor. */
typedef struct vq_tensor {
  void* data;
  int32_t dtype; /* vq_dtype */
  int32_t ndim;
  int64_t shape[VQ_MAX_DIMS];
} vq_tensor;

/* How a bfloat16 bit pattern maps to its table entry (bf16 bits).
 *
 * vq_rounder_from_table() classifies a 65,536-entry table into the cheapest
 * exact form and verifies it against every entry:
 *   IDENTITY   entry == input bits
 *   MINIFLOAT  round-half-even to a minifloat with saturation
 *              (src/voyager_compiler/quantization/dtypes/fp8.py:69-133)
 *   INT        clamp(round-half-even(x), qmin, qmax)
 *              (src/voyager_compiler/quantization/fake_quantize.py:67-68)
 *   POSIT      posit<nbits,es> rounding (dtypes/posit.py:8-73)
 *   STEP       a step function of the sortable key with <= 64 breakpoints
 *              (NormalFloat / codebook index tables)
 *   TABLE      anything else: a gather from the device copy in `table`.   */
typedef enum vq_rounder_kind {
  VQ_R_IDENTITY = 0,
  VQ_R_MINIFLOAT = 1,
  VQ_R_INT = 2,
  VQ_R_POSIT = 3,
  VQ_R_STEP = 4,
  VQ_R_TABLE = 5
} vq_rounder_kind;

#define VQ_STEP_MAX 64

typedef struct vq_rounder {
  int32_t kind;
  /* MINIFLOAT */
  int32_t ebits, mbits, is_signed, min_exp;
  float max_norm;
  /* INT */
  float qmin, qmax;
  /* POSIT */
  int32_t nbits, es;
  /* NaN output pattern (MINIFLOAT / INT / POSIT) */
  uint32_t nan_bits;
  /* STEP: keys ascending; output step_vals[j] for keys in
   * [step_keys[j-1], step_keys[j]) with step_keys[-1] = 0, and
   * step_vals[nsteps] for keys >= step_keys[nsteps-1]. */
  int32_t nsteps;
  uint16_t step_keys[VQ_STEP_MAX];
  uint16_t step_vals[VQ_STEP_MAX + 1];
  uint16_t pad_;
  /* TABLE: device pointer to 65,536 bf16 entries (caller-owned). */
  const uint16_t* table;
  /* MINIFLOAT only: a hardware conversion that reproduces this rounder
   * (VQ_HW_*), set by vq_rounder_from_table() as a candidate and kept only
   * after vq_rounder_check_hw() has compared it with the table on the
   * device; 0 = evaluate analytically. */
  int32_t hw;
  int32_t pad2_;
  /* TABLE (and the POSIT / STEP kinds the kernels evaluate as a table):
   * optional byte-coded copy of a table with at most 256 distinct patterns,
   * table8[i] indexing palette[256] (device, caller-owned, 16-byte aligned);
   * the kernels then stage 64.5 KB of shared memory instead of 128 KB, which
   * lets two 1024-thread CTAs share an SM.  NULL: use `table`. */
  const uint8_t* table8;
  const uint16_t* palette;
} vq_rounder;

enum { VQ_HW_NONE = 0, VQ_HW_E4M3 = 1, VQ_HW_E5M2 = 2, VQ_HW_E2M1 = 3 };

/* Name of a status code (static string). */
const char* vq_status_string(int status);

/* Library version string. */
const char* vq_version(void);

/* Classify a 65,536-entry bf16 table held in HOST memory (host-only, no
 * CUDA).  On return `out` evaluates exactly like the table for all inputs.
 * For VQ_R_TABLE the caller sets out->table to a device copy of the table.
 * Replaces the reference's per-call gather `qmap[bits & 0xFFFF]`
 * (src/voyager_compiler/ops/quantized.py:174-203). */
int vq_rounder_from_table(const uint16_t* host_table, vq_rounder* out);

/* Evaluate a rounder on the host for one bf16 pattern (test hook; the
 * device code runs the same function). */
uint16_t vq_rounder_eval_host(const vq_rounder* r, uint16_t bits);

/* Host evaluation of the power-of-two block scale for one block amax
 * (test hook for calculate_mx_qparam(force_scale_power_of_two=True),
 * src/voyager_compiler/ops/quantized.py:823-840,850).  `amax_bits` is a bf16
 * pattern when dtype == VQ_BF16, else float32 bits.  Returns the scale's bits
 * in the same dtype. */
uint32_t vq_pow2_scale_host(uint32_t amax_bits, int32_t dtype, int32_t floor_log2_qmax);

/* quantized_ops::quantize (src/voyager_compiler/ops/quantized.py:340-397):
 *   out = table[bf16(input / scale [+ zero_point])]
 * `scale` / `zero_point` broadcast as the op does: with block_size > 0 a dim
 * whose size differs from the input's repeats block_size times (expand(),
 * quantized.py:158-171); otherwise ordinary broadcasting.  `zero_point` may
 * be NULL.  `out` has the promoted dtype and the input's shape. */
int vq_quantize(const vq_tensor* input, const vq_tensor* scale,
                const vq_tensor* zero_point, int64_t block_size,
                const vq_rounder* qmap, vq_tensor* out, void* stream);

/* quantized_ops::dequantize (quantized.py:400-452):
 *   out = output_qmap[(input_qmap[input] [- zero_point]) * scale]
 * Either rounder may be NULL. */
int vq_dequantize(const vq_tensor* input, const vq_tensor* scale,
                  const vq_tensor* zero_point, int64_t block_size,
                  const vq_rounder* input_qmap, const vq_rounder* output_qmap,
                  vq_tensor* out, void* stream);

/* quantized_ops::calculate_mx_qparam (quantized.py:787-851): one scale per
 * block of `block_size` elements along each axis in `axes`.  `scale_qmap`
 * may be NULL.  `floor_log2_qmax` = floor(log2(quant_max)) as the reference
 * computes it (math.floor(math.log2(quant_max))).  `out` has the input's
 * dtype and the blocked shape. */
int vq_calculate_mx_qparam(const vq_tensor* input, const int64_t* axes, int32_t naxes,
                           int64_t block_size, float quant_max, int32_t pow2,
                           int32_t floor_log2_qmax, const vq_rounder* scale_qmap,
                           vq_tensor* scale_out, void* stream);

/* quantized_ops::quantize_mx (quantized.py:854-881): calculate_mx_qparam
 * then quantize, fused into one pass over the input when the blocks run
 * along the last dim.  Writes `scale_out` (blocked shape) and `codes_out`
 * (input shape), both in the input dtype. */
int vq_quantize_mx(const vq_tensor* input, const vq_rounder* qmap, const int64_t* axes,
                   int32_t naxes, int64_t block_size, float quant_max, int32_t pow2,
                   int32_t floor_log2_qmax, const vq_rounder* scale_qmap,
                   vq_tensor* scale_out, vq_tensor* codes_out, void* stream);

/* Count, on the device, the bf16 patterns whose hardware-conversion rounding
 * (r->hw) differs from r->table (65,536 entries, device).  Writes the count
 * to *d_mismatches (device int32, zeroed by the call).  Used once per table
 * before r->hw is trusted. */
int vq_rounder_check_hw(const vq_rounder* r, int32_t* d_mismatches, void* stream);

/* ---- MXFP8 block-scaled GEMM (tcgen05) -------------------------------------
 * linear_mx / matmul_mx (src/voyager_compiler/ops/quantized.py:455-472,
 * 522-648) for E4M3 codes with power-of-two block-32 scales along K on both
 * operands: out = (A codes x 2^sA) @ (B codes x 2^sB)^T (+ bias), fp32
 * accumulation, bf16 out.  Operands are packed first. */

/* Bytes of a packed operand of `rows` x `k` codes: E4M3 bytes [rows padded to
 * row_multiple (128 for A, 256 for B)][k padded to 128] and UE8M0 scale atoms
 * [k/128][rows/128][512]. */
int vq_mx_pack_sizes(int64_t rows, int64_t k, int32_t row_multiple, int64_t* codes_bytes,
                     int64_t* sf_bytes, int64_t* ld_bytes);

/* Pack bf16 codes [R, K] and bf16 scales [R, ceil(K/32)] (block_size 32).
 * *d_inexact (device, may be NULL) counts codes that are not E4M3 values and
 * scales that are not normal powers of two; a caller that cannot vouch for
 * its operands checks it is 0 before using the GEMM. */
int vq_mx_pack(const vq_tensor* codes, const vq_tensor* scale, int64_t block_size,
               int32_t row_multiple, void* packed_codes, void* packed_sf, int32_t* d_inexact,
               void* stream);

/* quantize_mx for MXFP8 activations (E4M3 table, power-of-two scales,
 * block 32 along the last dim of a bf16 [R, C] input, C a multiple of 128)
 * that also writes the GEMM operand in the same pass: E4M3 bytes [R, C]
 * (rows beyond R of a 128-row tile are not written; the GEMM discards
 * their products) and UE8M0 scale atoms as vq_mx_pack lays them out. */
int vq_quantize_mx_packed(const vq_tensor* input, const vq_rounder* qmap, int32_t floor_log2_qmax,
                          vq_tensor* scale_out, vq_tensor* codes_out, void* packed_codes,
                          void* packed_sf, void* stream);

/* out[M, N] (bf16, row stride ldo) = A[M, K] . B[N, K]^T (+ bias[N], bf16),
 * from packed operands (A with row_multiple 128, B with 256).  N and ldo must
 * be multiples of 8.  *d_err (device) is zeroed, and set non-zero if a
 * bounded wait in the kernel gave up. */
int vq_gemm_mxf8(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t M,
                 int64_t N, int64_t K, const void* bias, void* out, int64_t ldo, int32_t* d_err,
                 void* stream);

/* vq_gemm_mxf8 with two epilogue options.
 * residual (or NULL): the graph's residual add after the linear,
 *   out = bf16(bf16(A . B^T (+ bias)) + residual), residual bf16 [M, ldr]
 *   (ldr >= N, a multiple of 8); out may be the residual buffer itself (each
 *   element is read before it is written, by the same thread).
 * out_multicast: `out` is an NVLS multicast address of a symmetric buffer
 *   (tensor parallel over N: every rank's copy of the full output receives
 *   this rank's columns from one store); not with a residual. */
int vq_gemm_mxf8_ex(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t M,
                    int64_t N, int64_t K, const void* bias, const void* residual, int64_t ldr,
                    void* out, int64_t ldo, int32_t out_multicast, int32_t* d_err,
                    void* stream);

/* quantized_ops::matmul_mx (src/voyager_compiler/ops/quantized.py:589-648)
 * for MXFP8 operands with leading (batch) dims: vq_mx_pack of `batch`
 * matrices at once.  codes bf16 [batch, R, K] with scale [batch, R, K/32]
 * (k_axis 2: blocks along the last dim), or codes [batch, K, R] with scale
 * [batch, K/32, R] (k_axis 1: blocks along dim -2, the right operand of a
 * matmul stored [.., K, N]).  Output: with RTb = round_up(R, row_multiple)
 * / 128 row tiles per batch, codes [batch * RTb * 128, Kp] bytes and scale
 * atoms [Kp / 128][batch * RTb][512] (batch b's tiles at b * RTb); sizes
 * batch * RTb * 128 * Kp and (Kp / 128) * batch * RTb * 512 bytes. */
int vq_mx_pack_batched(const vq_tensor* codes, const vq_tensor* scale, int64_t block_size,
                       int32_t row_multiple, int32_t k_axis, void* packed_codes, void* packed_sf,
                       int32_t* d_inexact, void* stream);

/* `batch` MXFP8 GEMMs in one launch: out[b] = A[b] . B[b]^T from operands
 * packed by vq_mx_pack_batched (A with a_rows_per_batch packed rows per
 * batch -- a multiple of 128, at least M; B with row_multiple 256), or one
 * B for every batch (b_shared: packed by vq_mx_pack, row_multiple 256).
 * out[b] = out + b * out_batch_stride elements, rows ldo apart. */
int vq_gemm_mxf8_batched(const void* a, const void* a_sf, const void* b, const void* b_sf,
                         int64_t batch, int64_t a_rows_per_batch, int64_t M, int64_t N, int64_t K,
                         int32_t b_shared, const void* bias, void* out, int64_t ldo,
                         int64_t out_batch_stride, int32_t* d_err, void* stream);

/* ---- bf16 tcgen05 GEMM with the weight dequantized in shared memory --------
 * quantized_ops::linear_mx / matmul_mx (src/voyager_compiler/ops/
 * quantized.py:455-472, 522-648) for every operand format but MXFP8 x
 * MXFP8: the weight read back as bf16(decode(code) * scale) -- the
 * reference's _dequantize_mx, one bf16 rounding of the exact product --
 * inside the kernel, times bf16 activations, float32 sums, bf16 out:
 *   out[b][m, n] = sum_k A[b][m, k] W[b][n, k] (+ bias[n]).
 * a    bf16 [batch * M, K] row-major (K a multiple of 8, 16-byte aligned)
 * mode 0 (TMA): w is a bf16 weight [wb * N, K] (the library's plain bf16 GEMM);
 *      1 (LUT4) / 2 (LUT8): w holds palette indices as vq_dq_pack writes
 *      them, palette bf16 [16 | 256], w_scale4 the quarter-step scales of
 *      vq_dq_pack_scales (or NULL: no scale); all 16-byte aligned.
 * wb = 1 when w_shared (one weight for every batch), else batch.
 * out bf16 [batch][M, ldo] at out + b * out_batch_stride; N, ldo multiples of 8.
 * *d_err (device) is zeroed and set non-zero (11-14) if a bounded wait gave up. */
int vq_gemm_dq(const void* a, int64_t batch, int64_t M, int64_t K, int32_t mode, const void* w,
               int32_t w_shared, int64_t N, const void* w_scale4, const void* palette,
               const void* bias, void* out, int64_t ldo, int64_t out_batch_stride, int32_t* d_err,
               void* stream);
/* vq_gemm_dq with each output tile's K steps split over `splits` CTA pairs
 * (the same op, quantized.py:455-472, 522-648, for few output tiles: small M
 * times small N).  splits == 1 is vq_gemm_dq.  splits > 1: batch 1, the K
 * steps (ceil(K / 64)) a multiple of splits, workspace float32
 * [splits, M, N] (16-byte aligned, no initial value needed): each slice
 * stores its float32 sums there, then a second launch adds the slices in
 * order, adds the bias and rounds once to bf16. */
int vq_gemm_dq_ex(const void* a, int64_t batch, int64_t M, int64_t K, int32_t mode, const void* w,
                  int32_t w_shared, int64_t N, const void* w_scale4, const void* palette,
                  const void* bias, void* out, int64_t ldo, int64_t out_batch_stride,
                  int32_t splits, float* workspace, int32_t* d_err, void* stream);
/* Measurement aid, no counterpart in the reference: one launch that reads
 * read_bytes from src and writes write_bytes to dst (both multiples of 16,
 * 16-byte aligned) and does nothing else -- the least time any one launch
 * moving those bytes can take on this device (launch, ramp-up and drain
 * included).  bench.py reports small kernels against it. */
int vq_stream_probe(const void* src, int64_t read_bytes, void* dst, int64_t write_bytes,
                    void* stream);
/* The split count vq_gemm_dq_ex uses best for these sizes on this device (1:
 * no split). */
int32_t vq_gemm_dq_splits(int64_t batch, int64_t M, int64_t N, int64_t K);
/* Bytes of the packed indices and quarter-step scales of wbatch weights
 * [N, K] (mode 1: 4-bit, 2: 8-bit): with KS = ceil(K / 64) and Npad = N
 * rounded up to 256, wbatch * KS * Npad * (32 | 64) and wbatch * KS * Npad * 8. */
int vq_dq_pack_sizes(int64_t wbatch, int64_t N, int64_t K, int32_t mode, int64_t* codes_bytes,
                     int64_t* scale_bytes);
/* Weight codes bf16 [wbatch * N, K] -> palette indices, step-major:
 * [wbatch][KS][Npad][32 | 64 bytes] (element k of a row in step k / 64, LUT4
 * nibbles low first; rows N..Npad zero).  index_mode 1: each code is the
 * index itself (a codebook's stored indices, quantized.py:323-337; npal =
 * the palette size); 0: the code's bf16 bit pattern is looked up in
 * keys[npal] (ascending bit patterns) and stored as key_index[i] (a palette
 * position, below 16 / 256).  *d_missing (device, may be NULL) counts codes
 * with no entry. */
int vq_dq_pack(const vq_tensor* codes, int64_t wbatch, int32_t mode, int32_t index_mode,
               const void* keys, const void* key_index, int32_t npal, void* out,
               int32_t* d_missing, void* stream);
/* Block scales bf16 [wbatch * N, nkb] (blocks of block_size, a power of two
 * >= 16, along K; nkb == 1: one per row) -> the scale of every 16-element
 * quarter of each 64-element step, [wbatch][KS][Npad][4] bf16. */
int vq_dq_pack_scales(const void* scale, int64_t wbatch, int64_t N, int64_t K, int64_t nkb,
                      int64_t block_size, void* out, void* stream);
/* present[bits] = 1 for every bf16 bit pattern in codes (65,536 bytes, zeroed here). */
int vq_dq_patterns(const vq_tensor* codes, void* present, void* stream);
/* The GEMM's weight decode alone: out bf16 [N, K] (16-byte aligned) = the
 * dequantized weight (the first of the packed batches), the same values the
 * GEMM decodes in shared memory.  linear_mx decodes a packed weight this way
 * once per call from 4096 activation rows on and multiplies it in TMA mode
 * (quantized.py:455-472: _dequantize_mx of the weight, done once). */
int vq_dq_decode(const void* w, int64_t N, int64_t K, int32_t mode, const void* w_scale4,
                 const void* palette, void* out, void* stream);
/* dst[b][c][r] = src[b][r][c], bf16 [batch][rows, cols]. */
int vq_transpose_bf16(const void* src, int64_t batch, int64_t rows, int64_t cols, void* dst,
                      void* stream);

/* ---- NVFP4 x NVFP4 linear (tcgen05 kind::mxf4nvf4, scale_vec::4X) ---------
 * quantized_ops::linear_mx (src/voyager_compiler/ops/quantized.py:522-586)
 * with both operands E2M1 codes (bf16 values) and E4M3-valued bf16 scales
 * per 16 along K (block_size 16): the tensor cores multiply code x scale
 * exactly and sum in float32.
 * vq_nvf4_pack: codes [R, K] -> packed E2M1 [RT * 128][ceil(K/256) * 128 bytes]
 * (element 2i in the low nibble of byte i), scales [R, ceil(K/16)] -> UE4M3
 * atoms [ceil(K/256)][RT][4][512] (RT: rows rounded up to row_multiple, in
 * 128-row chunks; A with 128, B with 256); *d_inexact counts codes that are
 * not E2M1 values and scales that are not positive E4M3 values.
 * vq_gemm_nvf4: out bf16 [M, ldo] = A . B^T (+ bias); N, ldo multiples of 8;
 * *d_err as for vq_gemm_mxf8. */
int vq_nvf4_pack_sizes(int64_t rows, int64_t k, int32_t row_multiple, int64_t* codes_bytes,
                       int64_t* sf_bytes);
int vq_nvf4_pack(const vq_tensor* codes, const vq_tensor* scale, int32_t row_multiple,
                 void* packed_codes, void* packed_sf, int32_t* d_inexact, void* stream);
int vq_gemm_nvf4(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t M,
                 int64_t N, int64_t K, const void* bias, void* out, int64_t ldo, int32_t* d_err,
                 void* stream);

/* MXFP8 linear that allocates nothing: for callers that cannot call
 * cudaMalloc -- an allocator-free runtime, code running under a caller-owned
 * memory budget, or a library hook invoked where allocating is not allowed.
 * This entry point has no counterpart in the reference; it is the
 * vq_mx_pack + vq_gemm_mxf8 pair with the packed activations and the
 * kernel's error word kept in a fixed device array inside the library
 * (VQ_NOALLOC_SCRATCH_BYTES per GPU, held from first use until exit).
 *   a_codes  bf16 [M, K] E4M3 codes, a_scale bf16 [M, ceil(K/32)] powers of two
 *   w_packed / w_sf_packed  the weight as vq_mx_pack wrote it (row_multiple
 *            256) into caller memory; N its rows
 *   out      bf16 [M, ldo], caller memory
 * Rejects with VQ_ERR_TOO_LARGE, before launching anything, when the packed
 * activations do not fit: with Mp = round_up(M, 128) and Kp = round_up(K, 128),
 * 256 + round_up(Mp * Kp, 256) + (Mp / 128) * (Kp / 128) * 512 bytes must be
 * at most VQ_NOALLOC_SCRATCH_BYTES (16 MiB: e.g. M = 2048 rows at K = 4096,
 * or M = 8192 at K = 1920).  The operand
 * exactness check of vq_mx_pack is not run: the codes must be E4M3 values
 * and the scales normal powers of two.  The first call on a device looks up
 * the array's device address (make it before any stream capture).  Every
 * call reuses the one array: calls that overlap on the GPU race. */
#define VQ_NOALLOC_SCRATCH_BYTES (16u << 20)
int vq_linear_mxf8_noalloc(const vq_tensor* a_codes, const vq_tensor* a_scale,
                           const void* w_packed, const void* w_sf_packed, int64_t N,
                           const void* bias, void* out, int64_t ldo, void* stream);
/* The error word of the last vq_linear_mxf8_noalloc call on this device
 * (kept in the same fixed array): 0, or the code of a bounded wait in the
 * kernel that gave up (the output is then incomplete).  Ordered on `stream`
 * after the calls queued there; copies the word to *code (host memory) and
 * synchronises the stream.  Allocates nothing. */
int vq_linear_mxf8_noalloc_status(int32_t* code, void* stream);

/* Sticky wait-timeout status of this library's tcgen05 and barrier kernels
 * on the current device: *code (host) = 0, or the first code any launch
 * recorded since the last clear -- GEMM 1-4, bf16 GEMM 11-14, W4A8 21-23,
 * tensor-parallel barrier
 * 100 + rank, attention 200 + its code.  The per-call error words report to
 * one caller; this one lets the host ask, after a batch of work, whether any
 * launch gave up.  clear != 0 resets the word.  Synchronises `stream`.  The
 * reference raises on the host and has no device waits; this has no
 * counterpart there. */
int vq_device_errors(int32_t* code, int32_t clear, void* stream);

/* ---- Fused MXFP8 attention (tcgen05) ---------------------------------------
 * quantized_ops::sdpa_mx (src/voyager_compiler/ops/quantized.py:651-784)
 * without residual operands, for E4M3 codes with power-of-two block-32
 * scales (query / key along head_dim, value along the keys) and the
 * probabilities quantized to E4M3 with power-of-two block-32 scales along
 * the keys (probs_qmap = E4M3, force_scale_power_of_two):
 *   out[b,h,i,:] = bf16( sum_j P[i,j] V[j,:] ),
 *   P = dequantized quantize_mx(bf16(softmax(bf16(bf16(Q K^T) * scale)
 *       masked)), E4M3, [-1], 32, 2^floor_log2_qmax .. )
 * Operands packed as vq_mx_pack (row_multiple 128) lays them out:
 *   q  [batch*heads*sq, 128] codes, k [batch*kv_heads*skv, 128] codes,
 *   vt [batch*kv_heads*128, skv] codes (the value transposed: keys
 *   contiguous) with their scale atoms.  head_dim must be 128, sq and skv
 *   multiples of 128, heads a multiple of kv_heads (grouped-query heads).
 * causal: keys past the query's position (top-left aligned) are masked.
 * out: bf16 [b, h, i, d] at element strides (out_stride_b, _h, _s), d
 * contiguous; strides multiples of 8.  *d_err (device) is zeroed and set
 * non-zero if a bounded wait in the kernel gave up. */
int vq_attn_mxf8(const void* q, const void* q_sf, const void* k, const void* k_sf, const void* vt,
                 const void* vt_sf, int64_t batch, int64_t heads, int64_t kv_heads, int64_t sq,
                 int64_t skv, int64_t head_dim, float scale, int32_t causal,
                 int32_t floor_log2_qmax, void* out, int64_t out_stride_b, int64_t out_stride_h,
                 int64_t out_stride_s, int32_t* d_err, void* stream);

/* ---- Decoder-graph fusions feeding quantize_mx -------------------------------
 * In a converted LLaMA layer, the bf16 graph ops in front of each MXFP8
 * quantize_mx (quantized.py:854-881 with an E4M3 qmap, block 32 along the
 * last dim, force_scale_power_of_two) computed and quantized in one pass.
 * Each writes quantize_mx's two outputs (bf16 codes, bf16 scales) and the
 * tcgen05 operand as vq_mx_pack lays it out (row_multiple 128; rows past the
 * last are not written), and accepts only an E4M3 rounder with hw set.
 * These entry points have no single counterpart in the reference: each
 * replaces a chain of its graph's aten ops and one quantize_mx.
 *
 * RMSNorm (x * rsqrt(mean(x^2) + eps) in float32, to bf16, times weight)
 * of x [rows, cols]; cols a multiple of 32.  Output [rows, cols]. */
int vq_rmsnorm_quantize_mx(const void* x, const void* weight, int64_t rows, int64_t cols, float eps,
                           const vq_rounder* qmap, int32_t floor_log2_qmax, void* codes,
                           void* scale, void* packed, void* packed_sf, void* stream);
/* Rotate-half RoPE (x * cos + cat(-x2, x1) * sin, each op rounded to bf16)
 * of the q and k heads of a fused projection qkv [batch*seq, ld] (q heads of
 * 128 at column q_off, k heads at k_off), cos / sin bf16 [seq, 128];
 * outputs head-major [batch, heads, seq, 128] (blocks along head_dim). */
int vq_rope_quantize_qk(const void* qkv, int64_t ld, int64_t q_off, int64_t k_off,
                        const void* cos, const void* sin, int64_t batch, int64_t seq,
                        int64_t heads, const vq_rounder* qmap, int32_t floor_log2_qmax,
                        void* q_codes, void* q_scale, void* q_packed, void* q_sf, void* k_codes,
                        void* k_scale, void* k_packed, void* k_sf, void* stream);
/* The v heads of qkv (column v_off) quantized along the tokens (blocks of
 * 32 tokens, seq a multiple of 128), written transposed: codes
 * [batch, heads, 128, seq], scales [batch, heads, 128, seq / 32]: the
 * value operand vq_attn_mxf8 takes. */
int vq_quantize_vt(const void* qkv, int64_t ld, int64_t v_off, int64_t batch, int64_t seq,
                   int64_t heads, const vq_rounder* qmap, int32_t floor_log2_qmax, void* codes,
                   void* scale, void* packed, void* packed_sf, void* stream);
/* bf16(silu(gate)) * up of gate_up [rows, ld] (gate at columns [0, cols),
 * up at [up_off, up_off + cols)); silu = g / (1 + expf(-g)).  Output
 * [rows, cols], cols a multiple of 32; the packed operand pads cols to 128
 * with zero codes. */
int vq_swiglu_quantize_mx(const void* gate_up, int64_t ld, int64_t up_off, int64_t rows,
                          int64_t cols, const vq_rounder* qmap, int32_t floor_log2_qmax,
                          void* codes, void* scale, void* packed, void* packed_sf, void* stream);

/* ---- Tensor-parallel decoder collectives (NVLink / NVSwitch) ---------------
 * No reference counterpart: the reference runs on one device.  These serve
 * the column-parallel decoder (every linear split by output features, the
 * residual stream split by hidden columns): a rank quantizes its column
 * shard and writes the MXFP8 operand (E4M3 bytes at packed + row * ld +
 * col_off, UE8M0 words in the [K/128][row_tiles][512] atom layout) through
 * a multicast address, so every rank's copy of the full-width operand is
 * filled by one store.  *_mc pointers are NVLS multicast addresses of
 * symmetric buffers; col_off and the shard width are multiples of 128.
 *
 * Barrier over the ranks: thread j stores `epoch` into rank j's flag
 * array at [rank] (peer_flag_ptrs: device array of the ranks' flag array
 * addresses) and waits until my_flags[j] >= epoch; a wait longer than 2 s
 * sets *d_err = 100 + j and returns. */
int vq_tp_barrier(const void* peer_flag_ptrs, void* my_flags, int32_t rank, int32_t world,
                  uint32_t epoch, int32_t* d_err, void* stream);
/* vq_tp_barrier with the wait limit given: timeout_ns of %globaltimer time
 * per flag (1 us .. 10 s), after which *d_err = 100 + j and the kernel ends. */
int vq_tp_barrier_ex(const void* peer_flag_ptrs, void* my_flags, int32_t rank, int32_t world,
                     uint32_t epoch, uint64_t timeout_ns, int32_t* d_err, void* stream);
/* vq_tp_barrier with the epoch kept on the device: the kernel takes
 * *d_counter + 1 (0 skipped) as the epoch and stores it back.  Every rank
 * makes the same sequence of barrier calls, so the counters (zero at the
 * start, like the flags) stay equal across the ranks, whether the launches
 * are issued one by one or replayed from a captured CUDA graph.  Do not mix
 * it with host-epoch calls on the same flags. */
int vq_tp_barrier_dev(const void* peer_flag_ptrs, void* my_flags, int32_t rank, int32_t world,
                      uint32_t* d_counter, uint64_t timeout_ns, int32_t* d_err, void* stream);
/* rows x row_bytes from src (row stride src_ld bytes) into every rank's copy
 * of a symmetric buffer through its multicast address (row stride dst_ld
 * bytes); all sizes and addresses 16-byte aligned. */
int vq_tp_copy_multicast(const void* src, int64_t src_ld, int64_t rows, int64_t row_bytes,
                         void* dst_mc, int64_t dst_ld, void* stream);
/* stats_mc[rank][row] = sum of squares of this rank's columns of x [rows, cols]. */
int vq_tp_sumsq(const void* x, int64_t rows, int64_t cols, void* stats_mc, int32_t rank,
                void* stream);
/* RMSNorm of this rank's columns (statistic: the ranks' partial sums added in
 * rank order, divided by full_cols) times its weight slice, quantized to
 * MXFP8 (quantize_mx with an E4M3 table, power-of-two scales, block 32). */
int vq_tp_norm_quantize(const void* x, int64_t rows, int64_t cols, const void* stats,
                        int32_t world, int64_t full_cols, const void* weight, float eps,
                        const vq_rounder* qmap, int32_t floor_log2_qmax, void* packed_mc,
                        void* atoms_mc, int64_t ld, int64_t col_off, int64_t row_tiles,
                        void* stream);
/* MXFP8 quantization of bf16 x [rows, cols] (row stride ldx). */
int vq_tp_quantize(const void* x, int64_t ldx, int64_t rows, int64_t cols, const vq_rounder* qmap,
                   int32_t floor_log2_qmax, void* packed_mc, void* atoms_mc, int64_t ld,
                   int64_t col_off, int64_t row_tiles, void* stream);
/* bf16(silu(gate)) * up (gate at columns [0, cols), up at [up_off,
 * up_off + cols) of gate_up) quantized to MXFP8; the shard's operand width is
 * cols rounded up to 128, the extra columns zero codes with scale 1. */
int vq_tp_swiglu_quantize(const void* gate_up, int64_t ld_in, int64_t up_off, int64_t rows,
                          int64_t cols, const vq_rounder* qmap, int32_t floor_log2_qmax,
                          void* packed_mc, void* atoms_mc, int64_t ld, int64_t col_off,
                          int64_t row_tiles, void* stream);

/* ---- W4A8 (NVFP4 weights x MXFP8 activations) for few tokens --------------
 * The reference has no single op for this pair; its result is aten.linear of
 * the operands dequantized with their own block sizes
 * (src/voyager_compiler/ops/quantized.py:455-472, 522-586). */

/* Bytes of the packed form of an NVFP4 weight [N, K] (K % 128 == 0): tiles
 * of 256 rows x 128 K, 18432 bytes each, in (row block, K chunk) order; -1
 * for shapes the packing does not take. */
int64_t vq_w4_packed_bytes(int64_t N, int64_t K);

/* Pack bf16 E2M1 codes [N, K] and bf16 E4M3 scales [N, K/16] into
 * vq_w4_packed_bytes(N, K) bytes at `packed` (16-byte aligned): per tile,
 * 256 rows of 64 nibble bytes (even k in the low nibble; within a row's 64
 * bytes, byte 16b + 4i + t stored at 16t + 4b + i, the order
 * vq_w4a8_linear_small reads), then the rows' 8 scale bytes; rows past N
 * zero.  *d_inexact (device, may be NULL) counts entries that are not such
 * values. */
int vq_w4_pack_weights(const vq_tensor* codes, const vq_tensor* scales, void* packed,
                       int32_t* d_inexact, void* stream);

/* Bytes of the float32 workspace vq_w4a8_linear_small needs for a weight
 * [N, K]: the sums of row blocks split between CTAs, [ceil(N/256) * 256]
 * rows x 16 tokens; -1 for shapes it does not take. */
int64_t vq_w4a8_workspace_bytes(int64_t N, int64_t K);

/* out[M, N] bf16 = A . W^T (+ bias) for M <= 16 tokens in one launch from
 * MXFP8 tokens (bf16 E4M3 codes [M, K], bf16 power-of-two scales [M, K/32],
 * K % 128 == 0) and the packed weights, streamed once.  `workspace`
 * (vq_w4a8_workspace_bytes(N, K) bytes, or more) and `counters` (int32,
 * >= ceil(N / 256)) must be zero before the first call and every call
 * leaves them zero, so calls that never overlap on the GPU (one stream) can
 * share one pair sized for the largest weight; overlapping calls with the
 * same pair race.  *d_err (device, may be NULL) receives the code of the
 * first bounded wait that gave up (21-24; the result is then not valid).
 * The kernel is launched with programmatic stream serialization: it may
 * start while the previous kernel on the stream finishes and reads the
 * packed weights before waiting for it (everything else after), so the
 * packed weights must not be written by a kernel that is the one just
 * before it on the stream and that triggers its dependents early
 * (vq_w4_pack_weights does not). */
int vq_w4a8_linear_small(const vq_tensor* a_codes, const vq_tensor* a_scales, const void* packed,
                         int64_t N, const void* bias, float* workspace, int32_t* counters,
                         int32_t* d_err, void* out, void* stream);

/* The per-block parameters of quantized_ops::quantize_affine
 * (quantized.py:884-948): for blocks of `block_size` elements along the one
 * axis in `axes` (zero-padded when ragged),
 *   scale = (max - min) / (quant_max - quant_min), 1 where not > 0,
 *   optionally rounded through scale_qmap (and 1 where not > 0 again),
 *   zero_point = -min / scale + quant_min, optionally through scale_qmap.
 * The codes are then vq_quantize(input, scale, zero_point, block_size). */
int vq_quantize_affine_qparams(const vq_tensor* input, const int64_t* axes, int32_t naxes,
                               int64_t block_size, float quant_min, float quant_max,
                               const vq_rounder* scale_qmap, vq_tensor* scale_out,
                               vq_tensor* zero_point_out, void* stream);

/* The observer step of per-tensor / per-channel symmetric fake quantization,
 * FusedAmaxObsFakeQuantize._update_amax_scale
 * (src/voyager_compiler/quantization/fake_quantize.py:494-527), on the
 * device.  input: bf16 or float32, at least one element.  C = 1 (per-tensor)
 * or input->shape[ch_axis] (per_channel; ch_axis already reduced to
 * 0 .. ndim - 1).  amax_history: float32 [history_len, C]; scale: float32
 * [C]; workspace: float32 [C] scratch.  With reset != 0 the history is first
 * set to zero and the scale to one (the reference's lazy sizing).  Then
 *   amax     = max over the history rows as they were (NaN propagates),
 *   history  = roll(history, -1, 0) with row 0 = amax of |input| (over every
 *              axis, or every axis but ch_axis),
 *   scale    = amax / quant_max where amax > 0 and finite, else unchanged,
 *              then 2^ceil(log2(scale)) when power_of_two.
 * Bit-exact with the reference on float32.  Two launches and one memset of
 * the workspace. */
int vq_amax_observe(const vq_tensor* input, int32_t per_channel, int32_t ch_axis,
                    float* amax_history, int64_t history_len, float* scale, float quant_max,
                    int32_t power_of_two, int32_t reset, float* workspace, void* stream);

/* ---------------------------------------------------------------------------
 * Outlier CSR side-stream (quantized.py:958-1327)
 * ------------------------------------------------------------------------- */

/* The compare |x| > threshold of filter_outlier (quantized.py:1007) as a
 * bit test: the double is rounded to float32 and, for VQ_BF16, to bfloat16
 * (as torch converts a Python scalar to the tensor's dtype); the result lo1
 * satisfies |x| > threshold <=> lo1 <= (bits of |x|) <= (bits of +inf). */
uint32_t vq_outlier_threshold_bits(double threshold, int32_t dtype);

/* Bytes of device scratch vq_filter_outlier needs for `input`. */
size_t vq_filter_outlier_workspace_bytes(const vq_tensor* input);

/* quantized_ops::filter_outlier (quantized.py:995-1045) on input [..., R, C]
 * (bf16 or float32, R * C < 2^31):
 *   data    [nb, max_nnz] input dtype   outlier values in row-major order
 *   indices [nb, max_nnz] int32         their columns
 *   indptr  [nb, R + 1]   int32         row pointers (+ indptr_offset,
 *                                       quantize_mx_outlier's argument)
 *   inliers [..., R, C]   (may be NULL) the input with outliers set to +0
 * Outliers are |x| > threshold (see vq_outlier_threshold_bits) and x != 0;
 * nb is the product of the batch dims.  Past max_nnz entries are dropped and
 * row pointers clamped to max_nnz; unused slots hold 0 / -1 (_pad_csr,
 * quantized.py:964-990).  Three launches (count per tile, scan, scatter),
 * no waits between CTAs.  `workspace` holds
 * vq_filter_outlier_workspace_bytes bytes; d_err is not used (may be NULL). */
int vq_filter_outlier(const vq_tensor* input, double threshold, int64_t max_nnz,
                      int32_t indptr_offset, void* data, int32_t* indices, int32_t* indptr,
                      void* inliers, void* workspace, size_t workspace_bytes, int32_t* d_err,
                      void* stream);

/* quantize_mx along the last dim of the input with its outliers (as
 * vq_filter_outlier defines them) quantized as +0: the quantize_mx half of
 * quantized_ops::quantize_mx_outlier (quantized.py:1078-1130) without
 * materialising the inliers.  Optionally also writes the MXFP8 GEMM operand
 * (as vq_quantize_mx_packed; both pointers or neither).  Returns
 * VQ_ERR_UNSUPPORTED for layouts the fused kernel does not take. */
int vq_quantize_mx_masked(const vq_tensor* input, const vq_rounder* qmap, int64_t block_size,
                          float quant_max, int32_t pow2, int32_t floor_log2_qmax,
                          const vq_rounder* scale_qmap, double threshold, vq_tensor* scale_out,
                          vq_tensor* codes_out, void* packed_codes, void* packed_sf,
                          void* stream);

/* quantized_ops::spmm_csr (quantized.py:1245-1311) after B is decoded,
 * scaled and laid out [K, N]: out[b, r, :] = sum over the row's entries j of
 * data[b, j] * B[(b,) indices[b, j], :], float32 fused multiply-adds in CSR
 * order, rounded to B's dtype.  data [nb, L] (bf16 / float32), indices and
 * indptr [nb, rows + 1] int32, B [K, N] or [nb, K, N], out [nb, rows, N].
 * Row bounds are cummax(clamp(indptr - indptr[0], 0, L)) and columns are
 * clamped to [0, K - 1], as the reference rebases them.  `workspace`: int32
 * [nb, rows + 1]. */
int vq_spmm_csr(const vq_tensor* data, const int32_t* indices, const int32_t* indptr,
                int64_t rows, const vq_tensor* b, vq_tensor* out, int32_t* workspace,
                void* stream);

/* quantized_ops::slice_csr_tensor (quantized.py:1173-1216) of a CSR matrix
 * with `rows` rows (data / indices [L], indptr [rows + 1], int32):
 *   dim 0: rows [start, end) -> new_indptr [end - start + 1]
 *   dim 1: columns [start, end) -> new_indptr [rows + 1], columns - start
 * into max_out slots (0 / -1 past the entries; clamped row pointers when
 * they do not fit).  workspace: int32 [2 * rows + 1] (dim 1 only). */
int vq_slice_csr(const vq_tensor* data, const int32_t* indices, const int32_t* indptr,
                 int64_t rows, int32_t dim, int64_t start, int64_t end, int64_t max_out,
                 void* new_data, int32_t* new_indices, int32_t* new_indptr, int32_t* workspace,
                 void* stream);

/* Codebook lookup per region (encode / decode of quantized.py:211-337 with a
 * codebook [*counts, k]): counts[d] (ncounts == ndim) splits dim d of the
 * input into equal regions, numbered row-major over the counts;
 * out[i] = tables[region(i) * 65536 + bf16 pattern of input[i]], the tables
 * (device, nregions x 65,536 entries) holding the output dtype (bf16 or
 * float32).  A float32 input is rounded to bf16 for the pattern, as
 * encode's `input.bfloat16()`; decode's tables map the patterns of the
 * integers 0..k-1. */
int vq_codebook_lookup(const vq_tensor* input, const int64_t* counts, int32_t ncounts,
                       const void* tables, int64_t nregions, vq_tensor* out, void* stream);

/* dst [..., C, R] = src [..., R, C] transposed (2- or 4-byte elements). */
int vq_transpose(const vq_tensor* src, vq_tensor* dst, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VOYAGER_B200_H_ */
