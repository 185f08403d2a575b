/*
 * qgemv_b200.h -- C ABI of libqgemv_b200.so, the sm_100a (B200) q8_0 / q4_0
 * quantized GEMV library.
 *
 * Rules for every entry point:
 *   - Pointers are device pointers owned by the caller (for example
 *     torch.Tensor.data_ptr() of CUDA tensors); nothing is allocated on the
 *     GEMV path.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); work is
 *     enqueued on it and the call returns without synchronising.
 *   - The return value is a qgemv_status; 0 means the work was enqueued.
 *     The library never exits or aborts.  qgemv_last_error() returns a
 *     message for the last failure on the calling thread.
 *   - Arguments are validated before anything is launched: K % 32 == 0,
 *     M, K >= 0, row counts and K below 2^31, alignment (quant planes, AoS
 *     blocks and roof buffers 16 bytes; scale planes 2 bytes; x and y 4
 *     bytes), ldx >= K and ldy >= M.
 *
 * Layouts (ggml, byte-identical; the reference declares them at
 * src/qgemv_kernels.cuh:16-26):
 *   q8_0 block: fp16 d (little endian) + 32 x int8              = 34 bytes
 *   q4_0 block: fp16 d (little endian) + 16 bytes, byte i = q[i] | q[i+16] << 4
 *                                                               = 18 bytes
 *   SoA planes: quants [M][K] int8 (q8_0) or [M][K/2] uint8 (q4_0), scales
 *   [M][K/32] fp16 (passed as uint16_t bits).  AoS: [M][K/32] blocks.
 *   Activations X: `ncols` vectors of K fp32, vector n at x + n * ldx.
 *   Outputs Y: `ncols` vectors of M fp32, vector n at y + n * ldy.
 *   Y[n][r] = sum_k dequant(W)[r][k] * X[n][k].
 */
#ifndef QGEMV_B200_H_
#define QGEMV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QGEMV_API __attribute__((visibility("default")))

typedef enum qgemv_status {
  QGEMV_OK = 0,
  QGEMV_ERR_NULL = 1,        /* a required pointer is NULL                    */
  QGEMV_ERR_SHAPE = 2,       /* negative size, K % 32 != 0, ld too small, ... */
  QGEMV_ERR_ALIGN = 3,       /* a pointer is not aligned as required          */
  QGEMV_ERR_CUDA = 4,        /* a CUDA runtime call or launch failed          */
  QGEMV_ERR_UNSUPPORTED = 5, /* shape beyond what this build handles          */
  QGEMV_ERR_TIMEOUT = 6,     /* a bounded device-side wait ran out            */
  QGEMV_ERR_ARG = 7          /* another invalid argument (format, flag, ...)  */
} qgemv_status;

typedef enum qgemv_format { QGEMV_Q8_0 = 8, QGEMV_Q4_0 = 4 } qgemv_format;

/* Ranks (one GPU each) of the multi-GPU entry points. */
#define QGEMV_MAX_RANKS 8

typedef struct qgemv_device_info {
  char name[256];
  int device;
  int cc_major, cc_minor;
  int sms;
  int l2_bytes;
  int mem_clock_khz;
  int bus_width_bits;
  int sm_clock_khz;
  int smem_per_block_optin;
  double datasheet_gbps; /* 2 * mem_clock * bus_width / 8, as src/bench.cu:267-271 */
} qgemv_device_info;

/* Library version, e.g. 100 for 1.0.0. */
QGEMV_API int qgemv_version(void);

/* Message for the last failed call on this thread ("" if none). */
QGEMV_API const char* qgemv_last_error(void);

/* Constant name of a status code. */
QGEMV_API const char* qgemv_status_string(int status);

/* Properties of `device`, the fields the reference prints in its device JSON
 * line (src/bench.cu:261-272). */
QGEMV_API int qgemv_device_info_get(int device, qgemv_device_info* out);

/* ---------------------------------------------------------------- GEMV --- */

/* q8_0 SoA GEMV.  Replaces qgemv_q8_v5_soa_smem (best) and the SoA ladder
 * qgemv_q8_v3_soa_vec / qgemv_q8_v4_split<2,4>
 * (src/qgemv_kernels.cuh:110-175, 264-291; launches src/bench.cu:403-419),
 * whose signature was (Q, D, x, y, M, K) for one column.  q: int8 [M][K],
 * d: fp16 bits [M][K/32].  ncols in [0, 1<<20]: more than 16 columns are done
 * 16 at a time. */
QGEMV_API int qgemv_q8_0_soa(const void* q, const void* d, const float* x, float* y,
                             int64_t M, int64_t K, int32_t ncols, int64_t ldx, int64_t ldy,
                             void* stream);

/* q4_0 SoA GEMV.  Replaces qgemv_q4_v5_soa_smem (best), qgemv_q4_v3_soa_vec and
 * qgemv_q4_v6_fastunpack (src/qgemv_kernels.cuh:228-254, 323-352, 373-414;
 * launches src/bench.cu:430-440).  The v6 kernel also took per-block sums of
 * x (src/bench.cu:341-349); no such input is needed here.  q: uint8 [M][K/2].
 *
 * Single-column calls on matrices that the kernel runs with two CTAs per SM
 * share the rows out at run time through a tile counter (a fixed device array
 * inside the library, no allocation): one counter per stream, keyed by the
 * stream's unique id, and a fresh one for each call made under stream capture.
 * Calls on one stream are ordered and calls on different streams use
 * different counters; launches of one executable graph are ordered by CUDA,
 * but two executable graphs instantiated from the same capture share its
 * counters: replay those one at a time.
 * The first call on a device looks up the array's address; make it outside
 * stream capture (a call captured before that streams contiguous row ranges,
 * with the same results).  The pool holds 16384 counters per device; counters
 * are never returned (a stream keeps its counter, a captured call keeps its
 * counter for the life of the process), so a process that captures many
 * graphs can use them all: later calls then stream contiguous row ranges,
 * with the same results and 2-5 % slower.  qgemv_tile_counters_used() reports
 * how many are taken.  qgemv_check_device_error(clear = 1) zeroes the
 * counters after a timeout. */
QGEMV_API int qgemv_q4_0_soa(const void* q, const void* d, const float* x, float* y,
                             int64_t M, int64_t K, int32_t ncols, int64_t ldx, int64_t ldy,
                             void* stream);

/* Two columns (ncols == 2) of q4_0 SoA planes, or of GGUF blocks of either
 * format (qgemv_q8_0_aos / qgemv_q4_0_aos), with K % 256 == 0,
 * 256 <= K <= 16384, x 16-byte aligned and ldx a multiple of 4, run on the
 * single-column TMA kernel in its two-column form: the weights stream once
 * for both columns, no workspace is used (a workspace passed in is left
 * untouched), and each column is bit-identical to a one-column call on it
 * whenever every 32-element block of both columns is finite with its largest
 * magnitude between 2^-74 and 2^100 (otherwise within the same 1e-5 bound).
 * Other batched SoA calls (ncols >= 2) run on the tensor cores when K % 256 == 0,
 * K <= 2^20 and q, d are 16-byte aligned; they need a workspace (the
 * activations re-laid as fp16 hi/lo pairs, about 4 * K * min(ncols, 16)
 * bytes).  qgemv_q8_0_soa / qgemv_q4_0_soa keep one per (device, stream),
 * allocated by the first such call on the stream and grown when a later
 * call needs more; that call must not be inside stream capture
 * (QGEMV_ERR_UNSUPPORTED).  qgemv_soa_ws takes the workspace from the caller
 * instead and allocates nothing.  Calls that share a workspace must be
 * ordered (one stream, or events between them).  The reference had no
 * batched kernel. */

/* Opt-in q8_1 activations (one column): x is quantized to int8 per 32-element
 * block inside the kernel (amax = max|x|, q = rint(x * (127 / amax)), scale
 * amax / 127, all fp32), the activation format of ggml's q8_1 route that the
 * reference's README names as the production alternative (README.md:208-210,
 * 286-292; no kernel for it in the reference).  Each 32-weight block is then
 * one dp4a set instead of three.  This CHANGES THE NUMERICS: y carries the
 * rounding of x to 8 bits per block (up to amax / 254 per element), which the
 * 1e-5 bound of the exact entry points does not cover.  Shapes: K % 256 == 0,
 * 256 <= K <= 16384, x 16-byte aligned (else QGEMV_ERR_UNSUPPORTED).
 * qgemv_soa_q8_1 takes SoA planes (q, d as qgemv_q8_0_soa / qgemv_q4_0_soa),
 * qgemv_aos_q8_1 ggml blocks (as qgemv_q8_0_aos / qgemv_q4_0_aos). */
QGEMV_API int qgemv_soa_q8_1(int format, const void* q, const void* d, const float* x, float* y,
                             int64_t M, int64_t K, void* stream);
QGEMV_API int qgemv_aos_q8_1(int format, const void* blocks, const float* x, float* y,
                             int64_t M, int64_t K, void* stream);

/* Workspace bytes of a batched SoA call on the current device (0 when the
 * call needs none).  With 2..16 columns and K % 256 == 0 the call runs the
 * tcgen05 batch kernel, whose workspace grows with M (per-row-tile counters)
 * and the SM count; a smaller workspace is refused. */
QGEMV_API size_t qgemv_soa_workspace_bytes(int format, int64_t M, int64_t K, int32_t ncols);

/* qgemv_q8_0_soa / qgemv_q4_0_soa (format QGEMV_Q8_0 or QGEMV_Q4_0) with a
 * caller-owned device workspace of at least qgemv_soa_workspace_bytes()
 * bytes, 16-byte aligned (unused, and may be NULL, when that is 0). */
QGEMV_API int qgemv_soa_ws(int format, const void* q, const void* d, const float* x, float* y,
                           int64_t M, int64_t K, int32_t ncols, int64_t ldx, int64_t ldy,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Frees the per-stream workspaces (synchronises their devices). */
QGEMV_API int qgemv_release_workspaces(void);

/* qgemv_soa_ws with the workspace taken from a 2 MiB array compiled into the
 * library (one per device) instead of from the caller or from cudaMalloc:
 * neither this call nor its first-call set-up allocates device memory.  For
 * callers that must not allocate on the call path and have no device buffer
 * of their own to lend, e.g. a plugin host that forbids device allocation
 * after its initialisation, or a foreign-language binding that cannot own
 * CUDA memory.  Kernel: the tcgen05 batch kernel when its workspace fits
 * the array (at 7B-layer shapes up to 8 columns; it grows with M, the column
 * count and the SM count), otherwise the mma.sync batch kernel, whose
 * workspace depends on K and the column count only.  Limit: calls needing
 * more than 2 MiB of mma.sync workspace (above K = 32256 at 16 columns) fail
 * with QGEMV_ERR_UNSUPPORTED before anything is launched.  The first call on
 * a device looks up the array's address
 * (cudaGetSymbolAddress) and caches it; make that call before any stream
 * capture.  The cached address assumes the device's primary context lives
 * as long as the process: after cudaDeviceReset the array moves, so a caller
 * that resets a device must not call this entry point on it again.  Nothing
 * in the array needs to start at zero.  The array is shared: calls that
 * overlap in time on one device (two streams or two threads) race on it;
 * calls on one stream are ordered and safe.  No counterpart in the
 * reference. */
QGEMV_API int qgemv_soa_static_ws(int format, const void* q, const void* d, const float* x,
                                  float* y, int64_t M, int64_t K, int32_t ncols, int64_t ldx,
                                  int64_t ldy, void* stream);

/* ------------------------------------------------ persistent decode stack --- */

/* A sequence of single-column SoA GEMVs run by one cooperative launch per
 * call of qgemv_stack_run (the 4 x n_layers GEMVs of a decode token): GEMV j
 * reads the first K outputs of GEMV j-1 as its x.  One CTA per SM keeps a row
 * slice of every matrix and streams the next matrices' weights while the
 * current GEMV waits for its input, so the per-launch completion and
 * pipeline fill are paid once per token instead of once per GEMV.
 *
 * Outputs are 8-byte slots: slot r holds the fp32 bits of y[r] in its low 32
 * bits and a tag in its high 32 bits (one 64-bit store).  A reader waits
 * (bounded) until a slot carries the tag of the current token and GEMV, so
 * no fence, flag or collective separates the GEMVs, on one GPU or across
 * ranks; the call completes once every slot of the last GEMV's output on this
 * rank holds this token's value.  Read y[r] as the low word of slot r.
 *
 * qgemv_stack_create: one GPU (r0 = 0, M = M_total).
 * qgemv_stack_create_ranks: P ranks, one process and one GPU each, all
 * running the same sequence.  Rank k holds rows [r0, r0 + M) of every matrix
 * and stores them into its own slots and into every other rank's (peer_y,
 * e.g. symmetric memory mapped over NVLink): the all-gather of every y is
 * done by the kernel's own stores (no NCCL call, no qgemv_soa_fused).
 *
 * Each GEMV needs 256 <= K <= 16384, K % 256 == 0, K <= M_total of the GEMV
 * before it, an even M_total, q, d and y (and x of GEMV 0) 16-byte aligned.
 * The launch uses at most min(SMs, smallest M) CTAs.  The pointers are fixed
 * at creation (copy a new input into GEMV 0's x before a run); creation
 * allocates the handle's small device state (not on the GEMV path).  Output
 * slots start zeroed.  All waits are bounded (QGEMV_ERR_TIMEOUT in
 * qgemv_check_device_error; then clear it, zero the slots on every rank and
 * call qgemv_stack_reset before the next run).  No reference counterpart (the
 * reference timed one GEMV at a time). */
typedef struct qgemv_stack_gemv {
  const void* q;   /* quant plane of this rank's rows */
  const void* d;   /* scale plane */
  const float* x;  /* GEMV 0: its K input floats; the others read GEMV j-1's slots */
  uint64_t* y;     /* this GEMV's M_total output slots on this rank */
  int64_t r0, M;   /* this rank's rows [r0, r0 + M) */
  int64_t M_total; /* rows of the whole matrix */
  int64_t K;
} qgemv_stack_gemv;
typedef struct qgemv_stack_ranks {
  int32_t nranks;           /* 1..QGEMV_MAX_RANKS */
  int32_t rank;             /* this rank */
  uint64_t* const* peer_y;  /* n x (nranks - 1): GEMV j's output slots on the other ranks,
                               rank order without this rank */
} qgemv_stack_ranks;
QGEMV_API int qgemv_stack_create(int format, const qgemv_stack_gemv* gemvs, int32_t n,
                                 void** handle);
QGEMV_API int qgemv_stack_create_ranks(int format, const qgemv_stack_gemv* gemvs, int32_t n,
                                       const qgemv_stack_ranks* ranks, void** handle);
QGEMV_API int qgemv_stack_run(void* handle, void* stream);
/* Token count back to zero (after a timeout, once the slots are zeroed). */
QGEMV_API int qgemv_stack_reset(void* handle, void* stream);
QGEMV_API int qgemv_stack_destroy(void* handle);

/* -------------------------------------------- fused all-gather (P GPUs) --- */

/* Single-column SoA GEMV of this rank's rows whose y is all-gathered by the
 * kernel itself: besides y (this rank's rows, usually inside its own full-y
 * buffer) it stores the rows into every other rank's full-y buffer through
 * peer pointers (NVLink), and the CTA that finishes last adds 1 to every
 * rank's counter sig_out[k].  With sig_in set, the kernel first waits until
 * the counter of the call that produced x reaches (*tok + 1) * nranks, i.e.
 * until every rank has delivered its part of x for the current token.  All
 * waits are bounded (~1 s; QGEMV_ERR_TIMEOUT in qgemv_check_device_error).
 * Buffers and counters must be mapped on every rank (e.g. symmetric memory);
 * counters start at zero; cta_count is a zeroed local counter per call site.
 * A call that times out (or any call while this device's error word is set)
 * sends no signal, so the other ranks time out in their own waits instead of
 * reading an incomplete slice; to recover, clear the error word on every rank
 * (qgemv_check_device_error(1, ...)) and zero every counter, cta_count and
 * tok before the next token.
 * Replaces the NCCL all-gather after a GEMV (the reference was single-GPU). */
typedef struct qgemv_fuse {
  float* peer_y[QGEMV_MAX_RANKS];     /* other ranks' buffers, at this rank's first row */
  unsigned* sig_out[QGEMV_MAX_RANKS]; /* every rank's counter for this call (this rank's too) */
  unsigned* cta_count;                /* local, zeroed, one per call site */
  const unsigned* sig_in;             /* local counter of the call that produced x, or NULL */
  const unsigned* tok;                /* local token count (qgemv_token_fence) */
  int32_t npeer;                      /* entries of peer_y */
  int32_t nranks;                     /* entries of sig_out */
} qgemv_fuse;
QGEMV_API int qgemv_soa_fused(int format, const void* q, const void* d, const float* x, float* y,
                              int64_t M, int64_t K, const qgemv_fuse* fuse, void* stream);

/* End of a token of fused calls: adds 1 to every rank's done[k], waits
 * (bounded) until done_local reaches (*tok + 1) * nranks -- every rank has
 * finished the token, so buffers may be rewritten -- and advances *tok. */
QGEMV_API int qgemv_token_fence(unsigned* const* done, int32_t nranks, const unsigned* done_local,
                                unsigned* tok, void* stream);

/* Batch tiles: the same quantized weights re-laid for the tensor-core batch
 * kernel, one contiguous block per 16 rows x 512 columns (quants in the
 * order the kernel reads them -- q8_0 bytes as w + 128, the sign bit flipped
 * -- then that block's fp16 scales; rows beyond M and columns beyond K hold
 * zero weights).  A block is then a single bulk copy; the SoA
 * planes, whose 16 rows lie K bytes apart, need 16 copies per block and
 * stream at a fraction of the HBM rate on this path.  Made once per weight
 * matrix (qgemv_tile_weights), from SoA planes (layout 0: q, d) or from
 * ggml blocks (layout 1: q = blocks, d unused).  No reference counterpart:
 * the reference had no batched kernel. */
QGEMV_API size_t qgemv_tiled_bytes(int format, int64_t M, int64_t K);
QGEMV_API int qgemv_tile_weights(int format, int layout, const void* q, const void* d, int64_t M,
                                 int64_t K, void* tiled, void* stream);

/* Y = X W^T from batch tiles, any ncols >= 0 (16 per launch), K % 32 == 0,
 * K <= 2^20.  workspace: qgemv_tiled_workspace_bytes(K, ncols) bytes,
 * 16-byte aligned, or NULL for the per-stream workspace described above. */
QGEMV_API size_t qgemv_tiled_workspace_bytes(int64_t K, int32_t ncols);
QGEMV_API int qgemv_tiled_gemv(int format, const void* tiled, int64_t M, int64_t K,
                               const float* x, float* y, int32_t ncols, int64_t ldx, int64_t ldy,
                               void* workspace, size_t workspace_bytes, void* stream);

/* tc tiles: the weights re-laid for the tcgen05 (5th-generation tensor core)
 * batch kernel, one contiguous tile per 128 rows x 256 columns; tile (row
 * tile t, K tile k) at (t * ceil(K / 256) + k) * tile bytes.
 *   q8_0 (34816 bytes): the int8 quants in the 128-byte-swizzled K-major
 *     layout the tensor core reads from shared memory (2 boxes of
 *     [128 rows][128 bytes]; 16-byte chunk c of row r at chunk position
 *     c ^ (r % 8); rows in groups of 8 at 1024 bytes), then the
 *     [128 rows][8 blocks] fp16 scales;
 *   q4_0 (18432 bytes): the blocks' 16 nibble bytes as [8 blocks][128 rows]
 *     (widened to int8 in shared memory by the kernel), then the scales.
 * Rows beyond M and columns beyond K hold zero quants and zero scales.  Made
 * once per weight matrix from SoA planes (layout 0: q, d) or ggml blocks
 * (layout 1: q = blocks).  No reference counterpart: the reference had no
 * batched kernel. */
QGEMV_API size_t qgemv_tc_bytes(int format, int64_t M, int64_t K);
QGEMV_API int qgemv_tc_tile(int format, int layout, const void* q, const void* d, int64_t M,
                            int64_t K, void* tiles, void* stream);

/* Y = X W^T from tc tiles on the tcgen05 tensor cores, any ncols >= 0 (16 per
 * launch), K % 32 == 0, K <= 2^20.  Each 32-weight block is one integer MMA
 * (kind::i8) against x in 22-bit block fixed point (three signed byte
 * digits); rows are within 1e-5 ||w_row|| ||x|| of the exact dot, a column
 * holding a NaN or an infinity gives NaN in every row.  workspace:
 * qgemv_tc_workspace_bytes(M, K) bytes on the current device (both formats,
 * any ncols), 16-byte aligned, or NULL for the per-stream workspace.  Calls
 * that share a workspace must not overlap in time.  The kernel's waits are
 * bounded by qgemv_set_wait_limit; a timeout is reported by
 * qgemv_check_device_error. */
QGEMV_API size_t qgemv_tc_workspace_bytes(int64_t M, int64_t K);
QGEMV_API int qgemv_tc_gemv(int format, const void* tiles, int64_t M, int64_t K, const float* x,
                            float* y, int32_t ncols, int64_t ldx, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream);

/* The same for q8_0 (format QGEMV_Q8_0 implied). */
QGEMV_API size_t qgemv_q8_0_tc_bytes(int64_t M, int64_t K);
QGEMV_API int qgemv_q8_0_tc_tile(int layout, const void* q, const void* d, int64_t M, int64_t K,
                                 void* tiles, void* stream);
QGEMV_API size_t qgemv_q8_0_tc_workspace_bytes(int64_t M, int64_t K);
QGEMV_API int qgemv_q8_0_tc(const void* tiles, int64_t M, int64_t K, const float* x, float* y,
                            int32_t ncols, int64_t ldx, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream);

/* GEMV straight from ggml/GGUF blocks (no repack).  Replaces the AoS kernels
 * qgemv_q8_v0_naive / v1_warp / v2_smem_x and qgemv_q4_v0 / v1 / v2
 * (src/qgemv_kernels.cuh:39-104, 180-224, 294-320; launches
 * src/bench.cu:393-402, 420-429), signature (W, x, y, M, K).  blocks:
 * [M][K/32] blocks of 34 (q8_0) or 18 (q4_0) bytes, 16-byte aligned base. */
QGEMV_API int qgemv_q8_0_aos(const void* blocks, const float* x, float* y, int64_t M,
                             int64_t K, int32_t ncols, int64_t ldx, int64_t ldy, void* stream);
QGEMV_API int qgemv_q4_0_aos(const void* blocks, const float* x, float* y, int64_t M,
                             int64_t K, int32_t ncols, int64_t ldx, int64_t ldy, void* stream);

/* Kernel ladder (the reference's --only selection of one of its 13 kernel
 * configurations, src/bench.cu:256,358): single-column SoA GEMV with
 * configuration `variant` in [0, qgemv_soa_variant_count()), named by
 * qgemv_soa_variant_name().  grid > 0 forces the number of CTAs (0 = the
 * persistent default).  Same arguments and result as qgemv_q8_0_soa /
 * qgemv_q4_0_soa with ncols = 1. */
QGEMV_API int qgemv_soa_variant_count(void);
QGEMV_API const char* qgemv_soa_variant_name(int variant);
QGEMV_API int qgemv_soa_variant(int format, int variant, int32_t grid, const void* q,
                                const void* d, const float* x, float* y, int64_t M, int64_t K,
                                void* stream);

/* Device-side error word of the current device: kernels whose waits are
 * bounded (the TMA-fed and tensor-core GEMVs, the fused all-gather, the
 * persistent stack and the token fence, which give up after the wait limit)
 * record QGEMV_ERR_TIMEOUT there instead of hanging.  Returns QGEMV_OK when
 * it is clear, else the recorded status; clear = 1 resets it and the tile
 * counters, after waiting until the whole device is idle (no other thread may
 * launch work on the device meanwhile).  Synchronises `stream`.  The
 * reference had no device-side error path: its harness exits on any CUDA
 * error (src/bench.cu:19-27). */
QGEMV_API int qgemv_check_device_error(int clear, void* stream);

/* Limit of every bounded device-side wait on the current device, in
 * microseconds at the device's maximum SM clock (converted to clock64
 * cycles, so a wait at a lower clock lasts longer); <= 0 restores the
 * default of about 1 s.  Takes effect for kernels launched afterwards.
 * Synchronous; call it outside stream capture. */
QGEMV_API int qgemv_set_wait_limit(int64_t microseconds);

/* Tile counters (see qgemv_q4_0_soa) handed out on `device` so far, and the
 * size of the pool; -1 for a device index out of range. */
QGEMV_API int32_t qgemv_tile_counters_used(int device);
QGEMV_API int32_t qgemv_tile_counters_capacity(void);

/* ------------------------------------------------------- quantize / repack --- */

/* GPU quantizer, byte-identical to quantize_q8_0 / quantize_q4_0 of the
 * reference's python/qformats.py:17-40 (and src/bench.cu:32-69).  w: fp32
 * [M][ldw] (ldw >= K).  Writes the SoA planes q (q8_0: int8 [M][K], q4_0:
 * uint8 [M][K/2]) and d (fp16 bits [M][K/32]). */
QGEMV_API int qgemv_quantize_soa(int format, const float* w, int64_t M, int64_t K, int64_t ldw,
                                 void* q, void* d, void* stream);

/* Same quantizer, writing ggml blocks [M][K/32] (34 or 18 bytes each). */
QGEMV_API int qgemv_quantize_aos(int format, const float* w, int64_t M, int64_t K,
                                 int64_t ldw, void* blocks, void* stream);

/* fp32 dequantization of SoA planes, as dequant_q8_0 / dequant_q4_0 of
 * python/qformats.py:43-56.  w: fp32 [M][K]. */
QGEMV_API int qgemv_dequant_soa(int format, const void* q, const void* d, float* w, int64_t M,
                                int64_t K, void* stream);

/* AoS <-> SoA repack (src/bench.cu:300-314).  to_soa = 1: blocks -> (q, d);
 * to_soa = 0: (q, d) -> blocks. */
QGEMV_API int qgemv_repack(int format, int to_soa, void* blocks, void* q, void* d, int64_t M,
                           int64_t K, void* stream);

/* --------------------------------------------------------------- roof --- */

/* Streaming-read roof probe: reads `bytes` (multiple of 16) with 128-bit
 * loads, grid = SMs x blocks_per_sm CTAs of 256 threads.  Replaces
 * stream_read / run_ceiling (src/bench.cu:162-191).  sink: >= 2 uint32 of
 * device memory, written only on a data-dependent branch. */
QGEMV_API int qgemv_roof_stream_read(const void* buf, size_t bytes, uint32_t* sink,
                                     int32_t blocks_per_sm, void* stream);

/* The same read with 1-D TMA bulk copies into a shared-memory ring (one CTA
 * per SM).  status: one device int, set to QGEMV_ERR_TIMEOUT if a bounded
 * mbarrier wait ran out (the caller zeroes it before the call). */
QGEMV_API int qgemv_roof_bulk_read(const void* buf, size_t bytes, uint32_t* sink, int* status,
                                   void* stream);

/* Device-to-device copy roof (src/bench.cu:193-202): cudaMemcpyAsync. */
QGEMV_API int qgemv_roof_d2d(void* dst, const void* src, size_t bytes, void* stream);

/* ------------------------------------------------------------- timing --- */

/* One GEMV of a timed step, over `ncopies` copies of the same-shaped weights
 * (copy i % ncopies is used in step i, so the working set can exceed L2). */
typedef struct qgemv_call_desc {
  int32_t format;        /* QGEMV_Q8_0 or QGEMV_Q4_0                     */
  int32_t layout;        /* 0 = SoA planes (q, d), 1 = AoS blocks (q);
                            2 / 3 = the same with q8_1 activations
                            (qgemv_soa_q8_1 / qgemv_aos_q8_1, ncols 1)   */
  int32_t ncopies;       /* entries in q (and d)                         */
  int32_t ncols;         /* activation vectors                           */
  int64_t M, K, ldx, ldy;
  const void* const* q;  /* quant planes, or AoS block buffers           */
  const void* const* d;  /* scale planes (SoA), else NULL                */
  const float* x;
  float* y;
} qgemv_call_desc;

/* Timing harness (replaces time_kernel, src/bench.cu:134-156): issues
 * `warmup` untimed steps, then `steps` timed steps on `stream`; a step runs
 * every call of `calls` once (call j on copy step % ncopies).
 * grouped = 0: steps in order, a CUDA event before the first step and after
 *              every call; ms_out[1 + j] = summed device time of call j.
 * grouped = 1: all `steps` launches of call 0 back to back, then of call 1,
 *              ...; events only between groups; ms_out[1 + j] = device time
 *              of group j.
 * ms_out[0] = total device time (ncalls + 1 floats).  Synchronises `stream`
 * before returning. */
QGEMV_API int qgemv_time_steps(const qgemv_call_desc* calls, int32_t ncalls, int32_t warmup,
                               int32_t steps, int32_t grouped, void* stream, float* ms_out);

/* ---- Multi-GPU handle: one process drives several GPUs ----------------------
 * A q8_0 / q4_0 matrix sharded by rows over the handle's P devices (rows
 * [g*M/P, (g+1)*M/P) on devices[g], copied there by qgemv_mg_shard), one GEMV
 * per device on that device's stream, and, when asked, an all-gather of y so
 * that every device holds all M rows: each device pushes its rows of every
 * column into every other device's y with one 2-D peer copy (NVLink through
 * NVSwitch where the devices can address each other; peer access is enabled
 * by qgemv_mg_init).  For hosts that run one process per GPU instead, the
 * Python ShardedQGemv shards the same way and all-gathers with NCCL.  No
 * counterpart in the reference, which runs on one GPU. */

/* devices: ndev (1..QGEMV_MAX_RANKS) distinct device ordinals; *handle
 * receives the handle (streams and events per device). */
QGEMV_API int qgemv_mg_init(int32_t ndev, const int32_t* devices, void** handle);

/* Copies the matrix's row shards onto the devices (synchronous; replaces a
 * matrix the handle held before).  layout 0: SoA planes q [M][K] int8 (q8_0)
 * or [M][K/2] uint8 (q4_0) and d [M][K/32] fp16; layout 1: ggml blocks in q,
 * d unused.  q and d may live in host memory or on any device. */
QGEMV_API int qgemv_mg_shard(void* handle, int format, int layout, const void* q, const void* d,
                             int64_t M, int64_t K);

/* The first row and the row count of shard `index` (the index-th device). */
QGEMV_API int qgemv_mg_rows(void* handle, int32_t index, int64_t* r0, int64_t* rows);

/* Y = X W^T for ncols columns: x[g] is devices[g]'s copy of X ([ncols][K]
 * floats, ldx = K), y[g] devices[g]'s Y ([ncols][M] floats, ldy = M); device
 * g writes its rows of y[g] and, with allgather != 0, every other device's
 * rows arrive in y[g] as well.  streams[g]: the stream of devices[g] (NULL,
 * or a NULL entry: the handle's own stream).  Asynchronous: work queued
 * afterwards on streams[g] sees y[g] complete; the copies into y[g] start
 * only after what was queued on streams[g] before the call. */
QGEMV_API int qgemv_mg_gemv(void* handle, const float* const* x, float* const* y, int32_t ncols,
                            int32_t allgather, void* const* streams);

/* Waits for the handle's own streams. */
QGEMV_API int qgemv_mg_synchronize(void* handle);

/* Waits for the handle's own streams, then frees the shards, streams and
 * events (NULL: no-op). */
QGEMV_API int qgemv_mg_destroy(void* handle);

#ifdef __cplusplus
}
#endif

#endif /* QGEMV_B200_H_ */
