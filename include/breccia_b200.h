/*
 * breccia_b200 -- C ABI of the B200 (sm_100a) backend for breccia's hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream). Calls are
 * stream-ordered and asynchronous: they validate arguments on the host,
 * enqueue kernels and return. The library allocates nothing and frees
 * nothing: the caller owns every output and workspace buffer.
 *
 * Return value: BRC_OK (0) or a negative BRC_ERR_* status. On BRC_ERR_CUDA,
 * brc_last_cuda_error() gives the cudaError_t of the failing call on this
 * thread.
 *
 * Numerics follow the NumPy path of jvoltci/breccia v0.1.3 bit for bit
 * (codes and scales): round-to-nearest with ties toward zero for FP8/FP4
 * codes, IEEE float32 division by the scale, NumPy's float32 log2 for E8M0
 * scales, NumPy half-to-even rounding for INT4.
 *
 * "Reference:" lines name the function of jvoltci/breccia (path within that
 * project) that each entry point replaces for CUDA tensors.
 */
#ifndef BRECCIA_B200_H
#define BRECCIA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------- enums */
enum { BRC_DTYPE_F32 = 0, BRC_DTYPE_BF16 = 1, BRC_DTYPE_F16 = 2 };
enum { BRC_FP8_E4M3 = 0, BRC_FP8_E5M2 = 1 };
enum { BRC_SCALE_F16 = 0, BRC_SCALE_F32 = 1 };

enum {
  BRC_OK = 0,
  BRC_ERR_NULL = -1,        /* a required pointer is NULL */
  BRC_ERR_SHAPE = -2,       /* sizes inconsistent (e.g. cols % block != 0) */
  BRC_ERR_ALIGN = -3,       /* a pointer is not 16-byte aligned */
  BRC_ERR_DTYPE = -4,       /* unknown dtype / format enum */
  BRC_ERR_UNSUPPORTED = -5, /* valid request this build does not handle */
  BRC_ERR_CUDA = -6,        /* a CUDA runtime call or launch failed */
  BRC_ERR_TIMEOUT = -7,     /* a device-side bounded wait gave up */
  BRC_ERR_RANGE = -8        /* a size exceeds a documented limit */
};

/* Human-readable name of a status code (static string). */
const char* brc_status_string(int status);
/* cudaError_t of the last BRC_ERR_CUDA on the calling thread (0 if none). */
int brc_last_cuda_error(void);
/* ABI version: major * 10000 + minor * 100 + patch. */
int brc_version(void);

/* ======================================================= casts: per-tensor
 * DelayedScaling / Float8CurrentScaling.
 * Reference: src/breccia/kernels/reference/cast.py:364-373 (_cast_per_tensor_fp8)
 *            and src/breccia/kernels/reference/_utils.py:34-37 (tensor_amax).
 *
 * The global amax lives in a caller-provided device word `amax_bits` holding
 * the float32 bit pattern of max|x| (positive floats order like unsigned
 * integers; NaN orders above +inf, so NaN propagates).
 *   brc_amax_reset       : *amax_bits = 0
 *   brc_amax_accumulate  : *amax_bits = max(*amax_bits, bits(max|x|)) (atomic)
 *   brc_cast_pertensor_fp8_apply : scale = float32(max(amax, 1e-10) / fmt_max)
 *       computed as the reference does (float64 floor), codes = encode(x / scale),
 *       *scale_out = scale.
 * Sharded use: accumulate on each rank's shard, all-reduce(MAX) the word as an
 * unsigned 32-bit integer, then apply.
 */
int brc_amax_reset(uint32_t* amax_bits, void* stream);
int brc_amax_accumulate(const void* x, int x_dtype, int64_t n, uint32_t* amax_bits,
                        void* stream);
int brc_cast_pertensor_fp8_apply(const void* x, int x_dtype, int64_t n, int fmt,
                                 const uint32_t* amax_bits, uint8_t* codes,
                                 float* scale_out, void* stream);
/* reset + accumulate + apply in one call; `workspace` is one device word. */
int brc_cast_pertensor_fp8(const void* x, int x_dtype, int64_t n, int fmt, uint8_t* codes,
                           float* scale_out, uint32_t* workspace, void* stream);

/* Per-tensor FP8 cast that allocates nothing and takes no workspace, for
 * callers that cannot allocate device memory (a host runtime that hands over
 * only its input and output buffers, an op slot with no workspace argument,
 * code running where cudaMalloc is not allowed). No counterpart in the
 * reference; results equal brc_cast_pertensor_fp8 bit for bit.
 * The global amax goes through a scratch array inside the library
 * (16384 partial maxima + one word, 65,792 bytes per GPU that loads the
 * library, held until exit), so n is limited to 536,870,912 elements
 * (16384 chunks of 32768); larger inputs return BRC_ERR_RANGE. The first call
 * on a device looks up the scratch address on the current device; make that
 * first call before any stream capture. The address is kept for the life of
 * the process, so resetting that device (cudaDeviceReset) after the first
 * call is not supported: later calls would hand the kernels a stale address.
 * All calls on a device share the
 * scratch: calls whose kernels overlap on the GPU race and must be
 * serialised by the caller. Each call rewrites every scratch slot it reads. */
int brc_cast_pertensor_fp8_noalloc(const void* x, int x_dtype, int64_t n, int fmt,
                                   uint8_t* codes, float* scale_out, void* stream);

/* DelayedScaling with an amax history (extension: the reference's recipe
 * carries amax_history_len and margin, src/breccia/recipes.py:43-77, but its
 * cast uses the current amax, cast.py:364-373). `history` is a caller-owned
 * float32 ring of `history_len` amaxes on the device, most recent first.
 * use_history = 0: the current-amax cast (brc_cast_pertensor_fp8, bit for bit
 *   with the reference), then its amax is pushed into the ring.
 * use_history = 1: the scale is taken from the ring before the tensor is read,
 *   s = float32(max(max(history), 1e-10) / fmt_max) * 2^margin (a float32
 *   multiply), and the cast is ONE pass: each element is read once, clipped
 *   and encoded with s, while the tensor's amax is reduced; that amax is then
 *   pushed into the ring. Values beyond fmt_max * s saturate as the encoder
 *   clips them. margin in [-126, 127], else BRC_ERR_RANGE.
 * scale_out receives the scale used; workspace: one uint32 of device scratch. */
int brc_cast_pertensor_fp8_delayed(const void* x, int x_dtype, int64_t n, int fmt,
                                   float* history, int history_len, int margin, int use_history,
                                   uint8_t* codes, float* scale_out, uint32_t* workspace,
                                   void* stream);

/* ======================================================= casts: block FP8
 * Float8BlockScaling: one float32 scale per `block_k` run of the last axis.
 * Reference: src/breccia/kernels/reference/cast.py:384-404 (_cast_block_fp8),
 *            src/breccia/kernels/reference/_utils.py:11-31 (block_amax).
 * x is (rows, cols) row-major; codes (rows, cols); scales (rows, cols/block_k).
 */
int brc_cast_block_fp8(const void* x, int x_dtype, int64_t rows, int64_t cols, int block_k,
                       int fmt, uint8_t* codes, float* scales, void* stream);

/* block_m x block_k tiles (the 128x128 DeepSeek-v3 weight layout, which the
 * reference type system can describe as PerBlockMN(block_m, block_k) but the
 * reference cannot produce): the same arithmetic as _cast_block_fp8 over 2-D
 * tiles. scales is (rows/block_m, cols/block_k). */
int brc_cast_block_fp8_2d(const void* x, int x_dtype, int64_t rows, int64_t cols,
                          int block_m, int block_k, int fmt, uint8_t* codes, float* scales,
                          void* stream);

/* ======================================================= casts: MXFP8
 * MXFP8BlockScaling: 1x32 blocks, E8M0 scale.
 * Reference: src/breccia/kernels/reference/cast.py:420-446 (_cast_mxfp8),
 *            src/breccia/kernels/reference/_utils.py:40-56 (E8M0 helpers).
 * scales: (rows, cols/32) uint8, the reference layout.
 * scales_mma (optional, may be NULL): the same scales in the tcgen05
 * block-scale layout: 512-byte atoms of 128 rows x 4 scale columns, atom
 * (r/128, c/4) at ((r/128) * (ceil(cols/32/4)) + c/4) * 512, byte
 * (r%32)*16 + ((r/32)%4)*4 + c%4 within it; rows padded to 128 and scale
 * columns to 4 (padding is not written; callers zero it once).
 */
int brc_cast_mxfp8(const void* x, int x_dtype, int64_t rows, int64_t cols, int fmt,
                   uint8_t* codes, uint8_t* scales, uint8_t* scales_mma, void* stream);

/* ======================================================= casts: NVFP4
 * NVFP4BlockScaling: 1x16 blocks, E4M3 scale (division uses max(scale, 2^-9)).
 * Reference: src/breccia/kernels/reference/cast.py:468-496 (_cast_nvfp4).
 * codes (optional): one E2M1 code per byte (low nibble), the reference layout.
 * packed (optional): two codes per byte, element 2i in the LOW nibble (the
 *   tcgen05 / cuBLAS operand order; note breccia's pack_nibbles puts element
 *   2i in the HIGH nibble).
 * scales: (rows, cols/16) uint8 E4M3 codes. scales_mma: as for MXFP8.
 */
int brc_cast_nvfp4(const void* x, int x_dtype, int64_t rows, int64_t cols, uint8_t* codes,
                   uint8_t* packed, uint8_t* scales, uint8_t* scales_mma, void* stream);

/* ======================================================= casts: INT4
 * INT4Scaling, symmetric (signed or unsigned) or asymmetric (zero point).
 * Reference: src/breccia/kernels/reference/cast.py:516-571 (_cast_int4).
 * scales / zero_points: (rows, cols/group) in scale_dtype (BRC_SCALE_F16 for
 * "fp16"; BRC_SCALE_F32 for "fp32" and for "bf16", which the reference
 * stores as float32). zero_points is required iff !symmetric.
 * codes (optional): one code per byte (low nibble). packed (optional): two
 * per byte, element 2i in the LOW nibble.
 * packed_tiles / scale_tiles / zp_tiles (optional; group == 128 and
 * rows % 16 == 0): the layout brc_gemm_int4 streams. Tile T = (r/16) *
 * (cols/128) + g covers rows r/16*16 .. +15 and group g: 1024 bytes at
 * T * 1024, row r%16 at +64*(r%16); in each run of 8 elements 8j .. 8j+7 of
 * the row's group, byte 4j + i holds element 8j + i in the low nibble and
 * element 8j + i + 4 in the high nibble (i < 4). scale_tiles holds the
 * stored scale as float32 and zp_tiles (asymmetric only, else ignored)
 * 128 + the stored zero point as float32, both at T * 16 + 2 * (r%8) +
 * (r%16)/8.
 */
int brc_cast_int4(const void* x, int x_dtype, int64_t rows, int64_t cols, int group,
                  int is_signed, int symmetric, int scale_dtype, uint8_t* codes,
                  uint8_t* packed, void* scales, void* zero_points, uint8_t* packed_tiles,
                  float* scale_tiles, float* zp_tiles, void* stream);

/* ======================================================= stored 4-bit data, GEMM operands
 * breccia's on-disk nibble order puts element 2i in the HIGH nibble of byte i
 * (src/breccia/_formats.py:227-243 pack_nibbles, 246-260 unpack_nibbles); the
 * tensor cores read element 2i from the LOW nibble. Codes are one per byte in
 * the low nibble (the reference's ScaledTensor.data for NVFP4 and INT4).
 * n: number of codes, even. codes 16-byte aligned; packed buffers 8-byte
 * aligned (16-byte for brc_unpack_nibbles_hi).
 * brc_pack_nibbles_hi:   packed[i] = codes[2i] << 4 | codes[2i+1] (pack_nibbles).
 * brc_unpack_nibbles_hi: codes[2i] = packed[i] >> 4, codes[2i+1] = packed[i]
 *                        & 15 (unpack_nibbles), and/or the same pairs in the
 *                        tensor-core order into packed_lo (either may be NULL).
 * brc_pack_codes_lo:     packed_lo[i] = codes[2i] | codes[2i+1] << 4 (the
 *                        "packed" operand brc_cast_nvfp4 writes). */
int brc_pack_nibbles_hi(const uint8_t* codes, int64_t n, uint8_t* packed, void* stream);
int brc_unpack_nibbles_hi(const uint8_t* packed, int64_t n, uint8_t* codes, uint8_t* packed_lo,
                          void* stream);
int brc_pack_codes_lo(const uint8_t* codes, int64_t n, uint8_t* packed_lo, void* stream);
/* The tcgen05 scale-factor atoms (the sf_mma layout brc_cast_mxfp8 /
 * brc_cast_nvfp4 write) from stored one-byte scales (rows, scale_cols): MXFP8
 * E8M0 or NVFP4 E4M3 codes (cast.py:420-446, 468-496). atoms holds
 * ceil(rows/128) * ceil(scale_cols/4) * 512 bytes, every one written (padding
 * zero), 4-byte aligned. BRC_ERR_RANGE past 2^32 atoms. */
int brc_scale_atoms(const uint8_t* scales, int64_t rows, int64_t scale_cols, uint8_t* atoms,
                    void* stream);
/* The INT4 skinny-GEMM tiles brc_cast_int4 writes (packed_tiles, scale_tiles,
 * zp_tiles; layout in brc_cast_int4's comment) from a stored INT4 tensor of
 * group 128: codes (rows, cols) one per byte, scales and zero_points (rows,
 * cols/128) in scale_dtype (zero_points and zp_tiles both NULL when
 * symmetric) (cast.py:516-571). rows % 16 == 0, cols % 128 == 0;
 * BRC_ERR_RANGE when rows * cols / 16 exceeds 2^32. */
int brc_int4_tiles(const uint8_t* codes, int64_t rows, int64_t cols, const void* scales,
                   const void* zero_points, int scale_dtype, uint8_t* tiles, float* scale_tiles,
                   float* zp_tiles, void* stream);

/* ======================================================= cast_ste (fused)
 * The forward value of breccia.autograd.cast_ste / cast_ste_clipped for one
 * recipe in a single pass: out = x + (dequantize(cast(x, recipe)) - x) in
 * float32, per element, with the codes and stored scales the cast would
 * produce (src/breccia/autograd.py:84-87, 179-190; cast.py:364-586). No codes
 * or scales are written. out: float32, same element count as x, 16-byte
 * aligned.
 * brc_cast_ste_pertensor_fp8: Float8CurrentScaling / DelayedScaling;
 * amax_word: one uint32 of device scratch.
 * brc_cast_ste_block: kind BRC_STE_BLOCK_FP8 (block = block_k), BRC_STE_MXFP8
 * (block 32), BRC_STE_NVFP4 (block 16, fmt ignored), BRC_STE_INT4 (block =
 * group; is_signed, symmetric, scale_dtype as brc_cast_int4). Block sizes
 * 16/32/64/128/256; others return BRC_ERR_UNSUPPORTED. */
#define BRC_STE_BLOCK_FP8 0
#define BRC_STE_MXFP8 1
#define BRC_STE_NVFP4 2
#define BRC_STE_INT4 3
#define BRC_KIND_PERTENSOR_FP8 4
int brc_cast_ste_pertensor_fp8(const void* x, int x_dtype, int64_t n, int fmt,
                               uint32_t* amax_word, float* out, void* stream);
int brc_cast_ste_block(const void* x, int x_dtype, int64_t rows, int64_t cols, int kind,
                       int block, int fmt, int is_signed, int symmetric, int scale_dtype,
                       float* out, void* stream);

/* ======================================================= dequantize
 * out = decode(code) * scale (asymmetric INT4: (code - zp) * scale), written as
 * float32 (the reference's dtype) or, as an extension, bf16/f16.
 * Reference: src/breccia/kernels/reference/cast.py:376-378, 407-414, 449-459,
 *            499-506, 574-586.
 */
int brc_dequant_pertensor_fp8(const uint8_t* codes, int64_t n, int fmt, const float* scale,
                              void* out, int out_dtype, void* stream);
/* block_m = 1 for the 1 x block_k layout; scales (rows/block_m, cols/block_k). */
int brc_dequant_block_fp8(const uint8_t* codes, int64_t rows, int64_t cols, int block_m,
                          int block_k, int fmt, const float* scales, void* out,
                          int out_dtype, void* stream);
int brc_dequant_mxfp8(const uint8_t* codes, int64_t rows, int64_t cols, int fmt,
                      const uint8_t* scales, void* out, int out_dtype, void* stream);
int brc_dequant_nvfp4(const uint8_t* codes, int64_t rows, int64_t cols,
                      const uint8_t* scales, void* out, int out_dtype, void* stream);
int brc_dequant_int4(const uint8_t* codes, int64_t rows, int64_t cols, int group,
                     int is_signed, int scale_dtype, const void* scales,
                     const void* zero_points, void* out, int out_dtype, void* stream);

/* ======================================================= requantize
 * NVFP4 -> MXFP8 in one pass (no float32 round trip through memory); equal to
 * cast(dequantize(st), MXFP8BlockScaling(fmt)).
 * Reference: src/breccia/kernels/reference/cast.py:339-346 (requantize).
 */
int brc_requant_nvfp4_to_mxfp8(const uint8_t* codes, const uint8_t* scales, int64_t rows,
                               int64_t cols, int fmt, uint8_t* codes_out,
                               uint8_t* scales_out, uint8_t* scales_mma_out, void* stream);

/* ======================================================= scaled GEMMs
 * D[M, N] = A[M, K] * B[N, K]^T on the tcgen05 tensor cores with float32
 * accumulation; both operands K-major (B is the weight in nn.Linear
 * orientation, i.e. the cast of W^T for a (K, N) weight W). D is row-major
 * (ldd = N) in BRC_DTYPE_F32 / BF16 / F16. N % 16 == 0.
 * Reference: src/breccia/kernels/reference/matmul.py:42-133 (dequantize both
 * operands, float32 matmul) and, for the per-tensor kind,
 * src/breccia/kernels/triton/scaled_matmul.py:152-257 (scaled_matmul_triton).
 */
/* Per-tensor FP8 (DelayedScaling / Float8CurrentScaling): codes E4M3 / E5M2,
 * D = (A_codes @ B_codes^T) * a_scale * b_scale with the scales read from
 * device memory (0-d tensors). K % 128 == 0. */
int brc_gemm_fp8_pertensor(const uint8_t* a, const uint8_t* b, int M, int N, int K, int a_fmt,
                           int b_fmt, const float* a_scale, const float* b_scale, void* d,
                           int d_dtype, void* stream);
/* Fused activation cast + per-tensor FP8 GEMM (extension: the reference
 * casts, then multiplies -- cast.py:364-373 then matmul.py:42-133).
 * x (M, K) float32 / bfloat16 / float16 is cast to a_fmt codes and
 *   D = (A_codes @ B_codes^T) * a_scale * b_scale
 * in one GEMM launch whose extra warps encode A while the tensor cores run;
 * only the first tile group's rows (prologue_rows, < 0 = 4096) are encoded
 * before it. Outputs equal brc_cast_pertensor_fp8 (history == NULL, or
 * use_history == 0) or brc_cast_pertensor_fp8_delayed (history, use_history)
 * followed by brc_gemm_fp8_pertensor, bit for bit: a_codes / a_scale_out are
 * the cast's, d the GEMM's; with a history its ring receives x's amax.
 * amax_in (no history): the float32 bit pattern of the amax to scale with,
 * already reduced by the caller (the whole tensor's amax when x is one of
 * several ranks' copies or shards): brc_cast_pertensor_fp8_apply with that
 * word, then the GEMM; no amax pass here.
 * workspace: device scratch of brc_cast_gemm_workspace_bytes(M, K) bytes
 * (zeroed here). K % 128 == 0, N % 16 == 0, 16-byte aligned pointers. */
int64_t brc_cast_gemm_workspace_bytes(int M, int K);
int brc_cast_gemm_pertensor_fp8(const void* x, int x_dtype, int a_fmt, const uint8_t* b,
                                int b_fmt, const float* b_scale, int M, int N, int K,
                                float* history, int history_len, int margin, int use_history,
                                const uint32_t* amax_in, uint8_t* a_codes, float* a_scale_out,
                                void* d, int d_dtype, void* workspace, int64_t workspace_bytes,
                                int prologue_rows, void* stream);
/* MXFP8: scales in the tcgen05 layout written by brc_cast_mxfp8 (scales_mma)
 * for A (M rows) and B (N rows). K % 128 == 0. */
int brc_gemm_mxfp8(const uint8_t* a, const uint8_t* b, int M, int N, int K, int a_fmt,
                   int b_fmt, const uint8_t* a_sf_mma, const uint8_t* b_sf_mma, void* d,
                   int d_dtype, void* stream);
/* NVFP4: packed E2M1 codes (element 2i in the low nibble, as brc_cast_nvfp4
 * writes them; K/2 bytes per row) and E4M3 scales in the tcgen05 layout.
 * K % 256 == 0. */
int brc_gemm_nvfp4(const uint8_t* a_packed, const uint8_t* b_packed, int M, int N, int K,
                   const uint8_t* a_sf_mma, const uint8_t* b_sf_mma, void* d, int d_dtype,
                   void* stream);
/* Float8BlockScaling (DeepSeek-v3 layout): A codes with float32 scales
 * a_scales (M, K/128) (1 x 128 blocks), B codes with float32 scales
 * b_scales (ceil(N/128), K/128) (128 x 128 blocks of the (N, K) weight).
 * Each 128-K block is multiplied on the tensor cores and promoted into float32
 * accumulators with its two scales. K % 128 == 0.
 * Reference: matmul.py:42-133 on ScaledTensors from cast.py:384-404;
 * triton/scaled_matmul.py:263-407 (block_scaled_matmul_triton). */
int brc_gemm_block_fp8(const uint8_t* a, const uint8_t* b, int M, int N, int K, int a_fmt,
                       int b_fmt, const float* a_scales, const float* b_scales, void* d,
                       int d_dtype, void* stream);
/* INT4 weight-only skinny GEMM (decode shapes): D[M, N] = A[M, K] * W^T with
 * A bfloat16 (M <= 16) and W^T an (N, K) weight cast by brc_cast_int4 with
 * group 128, given in its tile layout (packed_tiles, scale_tiles, zp_tiles;
 * zp_tiles NULL for symmetric recipes). Per 128-element group the tensor
 * cores form sum A * (q - zp) and the group scale is applied in float32.
 * K % 1024 == 0, N % 16 == 0.
 * Reference: matmul.py:42-133 (raw activations x dequantized INT4 weight,
 * cast.py:574-586). */
int brc_gemm_int4(const void* a_bf16, int M, int K, const uint8_t* w_tiles, int N, int is_signed,
                  int symmetric, const float* scale_tiles, const float* zp_tiles, void* d,
                  int d_dtype, void* stream);
/* Dense bf16 GEMM on the tensor cores (tcgen05 kind::f16, float32 accumulate):
 * d[M, N] = a[M, K] * b[N, K]^T, both bf16 and K-major, K % 8 == 0 (a partial
 * last 64-element K step reads zeros), N % 16 == 0, 16-byte aligned.
 * This is the reference's matmul for operand pairs without a block-scaled
 * tensor-core kind: matmul.py:123-133 dequantizes both operands to float32
 * and multiplies. Operands that dequantize exactly into bf16 (MXFP8:
 * E4M3/E5M2 x 2^k; NVFP4: E2M1 x E4M3, at most 6 significant bits) give the
 * reference's products exactly, with float32 accumulation; block FP8,
 * per-tensor FP8 and INT4 values are rounded once to bf16 (relative error
 * <= 2^-9 per element). */
int brc_gemm_bf16(const void* a, const void* b, int M, int N, int K, void* d, int d_dtype,
                  void* stream);

/* ======================================================= layout
 * breccia's matmul takes b as (K, N) with scale blocks along N
 * (src/breccia/kernels/reference/matmul.py:123-133; cast.py blocks the last
 * axis); the tensor-core GEMMs take operands K-major (N, K). */
/* decode(code) * scale of a (rows, cols) tensor, written transposed as
 * (cols, rows) in out_dtype (float32 / bf16 / f16): the reference's float32
 * dequantize (cast.py:376-586) rounded once to the output type. kind:
 * BRC_STE_BLOCK_FP8 (float32 scales (rows, cols / block)), BRC_STE_MXFP8
 * (E8M0 bytes, block 32), BRC_STE_NVFP4 (E4M3 bytes, block 16; fmt ignored),
 * BRC_STE_INT4 (scale_dtype BRC_SCALE_F16 / F32, zero_points optional, block
 * = group, is_signed), BRC_KIND_PERTENSOR_FP8 (scales -> one float32).
 * rows % 8 == 0, cols % 16 == 0, block % 16 == 0. */
int brc_dequant_transposed(const uint8_t* codes, int64_t rows, int64_t cols, int kind, int fmt,
                           int block, int is_signed, int scale_dtype, const void* scales,
                           const void* zero_points, void* out, int out_dtype, void* stream);
/* (rows, cols) bytes -> (cols, rows), rows % 16 == 0, cols % 16 == 0: per-tensor
 * FP8 codes in breccia's (K, N) orientation into the GEMM's (N, K). */
int brc_transpose_u8(const uint8_t* in, int64_t rows, int64_t cols, uint8_t* out, void* stream);

/* Sticky device status of the GEMM kernels on the current device (bit 0: a
 * bounded wait timed out and the kernel returned early). Synchronous. The
 * status word's address is looked up once per device and kept for the life
 * of the process (a device reset after the first GEMM is not supported). */
int brc_gemm_status(int reset);
/* Failure-path self-test (no counterpart in the reference; the reference has
 * no device code). Runs the GEMMs' bounded-wait and tear-down code in one CTA
 * against a barrier nothing arrives at: one role waits with a `limit_us`
 * bound (1 .. 1,000,000 us, else BRC_ERR_RANGE), a second role waits with
 * the GEMMs' normal 2 s bound and must leave on the first role's abort flag;
 * TMEM is allocated and freed as in the GEMMs. No fault, trap or unbounded
 * wait is involved. Synchronous on `stream`. Returns BRC_ERR_TIMEOUT when the
 * timeout was recorded in the GEMM status word (the expected outcome; the
 * bit stays set until brc_gemm_status(1)); `roles_out` (optional) receives a
 * bit per role that left its wait without the barrier completing (3 = both). */
int brc_selftest_wait_timeout(int limit_us, int* roles_out, void* stream);

/* ======================================================= diagnostics
 * Writes, for each i, the float32 quotient x[i] / s[i] as the cast kernels
 * compute it (correctly rounded reciprocal refined by one FMA residual step)
 * and as IEEE division computes it, for self-tests. No reference counterpart.
 */
int brc_selftest_division(const float* x, const float* s, int64_t n, float* q_fast,
                          float* q_ieee, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* BRECCIA_B200_H */
