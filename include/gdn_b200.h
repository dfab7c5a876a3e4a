/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Gated Delta Network kernels.
 *
 * Two destination-passing entry points replace the two reference plugins of
 * romitjain/kachua-mlsys:
 *
 *   gdn_decode_launch   replaces gdn_decode_qk4_v8_d128_k_last/solution/cuda/kernel.cu:982-1064
 *                       (launch_gdn, bound to Python at kernel.cu:1066-1068 and
 *                       loaded by solution/cuda/binding.py:20-51)
 *   gdn_prefill_launch  replaces gdn_prefill_qk4_v8_d128_k_last/solution/triton/kernel.py:56-262
 *                       (launch_gdn, registered as "flashinfer.kernel")
 *
 * Problem constants are those of both definitions: 4 q/k heads, 8 v heads,
 * head dim 128, k-last fp32 state [.., 8, 128 (V), 128 (K)].
 *
 * Conventions
 *   - Every pointer is a device pointer of the current CUDA device, except
 *     the argument structs themselves (host memory).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Launches are asynchronous; nothing here synchronises.
 *   - The caller owns every buffer and must fully pre-allocate `output` and
 *     `new_state` (destination-passing style, as the reference harness does).
 *   - `scale == 0` selects 1/sqrt(128), as the reference's `scale is None or
 *     scale == 0.0` (decode reference_torch_impl.py:32-33).
 *   - Functions return a gdn_status_t; nothing is launched unless GDN_OK.
 *     Kernels that detect bad device-side data (cu_seqlens out of range, a
 *     bounded wait that gave up) record it in a per-device status word read
 *     by gdn_read_device_status().
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_NUM_QK_HEADS 4
#define GDN_NUM_V_HEADS 8
#define GDN_HEAD_DIM 128

typedef enum gdn_status_t {
    GDN_OK = 0,
    GDN_ERR_NULL_POINTER = 1,      /* a required pointer is NULL */
    GDN_ERR_BAD_SIZE = 2,          /* negative or inconsistent sizes */
    GDN_ERR_MISALIGNED = 3,        /* a pointer violates its alignment rule */
    GDN_ERR_WORKSPACE = 4,         /* workspace missing or too small */
    GDN_ERR_CUDA = 5,              /* a CUDA runtime call failed */
    GDN_ERR_BAD_DTYPE = 6,         /* unsupported cu_seqlens dtype code */
    GDN_ERR_NO_DEVICE = 7,         /* no usable sm_100 device is current */
    GDN_ERR_DEVICE_BAD_SEQLENS = 16,  /* device status bit: cu_seqlens not monotone / out of range */
    GDN_ERR_DEVICE_TIMEOUT = 32       /* device status bit: a bounded wait expired */
} gdn_status_t;

/* ---------------------------------------------------------------- decode -- */

/* One decode step (one token per sequence).  Shapes (row-major, contiguous):
 *   q, k      bf16 [B, 1, 4, 128]     (8-byte aligned)
 *   v         bf16 [B, 1, 8, 128]
 *   state     fp32 [B, 8, 128, 128]   k-last, 16-byte aligned; may alias new_state
 *   A_log     fp32 [8]
 *   a, b      bf16 [B, 1, 8]
 *   dt_bias   fp32 [8]
 *   output    bf16 [B, 8, 128]        (identical bytes to [B, 1, 8, 128])
 *   new_state fp32 [B, 8, 128, 128]   16-byte aligned
 * Reference: gdn_decode_qk4_v8_d128_k_last/solution/cuda/kernel.cu:982-994. */
typedef struct GdnDecodeArgs {
    const void* q;
    const void* k;
    const void* v;
    const float* state;
    const float* A_log;
    const void* a;
    const float* dt_bias;
    const void* b;
    void* output;
    float* new_state;
    int64_t batch;
    float scale;
} GdnDecodeArgs;

int gdn_decode_launch(const GdnDecodeArgs* args, void* stream);

/* Decode of `tokens` >= 1 tokens per sequence in one call (speculative or
 * multi-token decode; the decode definition's seq_len axis,
 * flashinfer/trace/templates/gdn.py:104-110): q, k bf16 [B, T, 4, 128],
 * v bf16 [B, T, 8, 128], a, b bf16 [B, T, 8], output bf16 [B, T, 8, 128];
 * state / new_state as for gdn_decode_launch (may be the same buffer), the
 * state after all T tokens.  Alignment rules as gdn_decode_launch.  The
 * state is read and written once per call.  T = 1 is gdn_decode_launch. */
int gdn_decode_launch_tokens(const GdnDecodeArgs* args, int64_t tokens, void* stream);

/* gdn_decode_launch with the state stored in bf16: args->state and
 * args->new_state point to bf16 [B, 8, 128, 128] arrays (8-byte aligned; they
 * may be the same array).  The update is computed in fp32 and the new state
 * rounded to bf16 once per step, so the state stream (the whole cost of a
 * large-batch step) is half that of the fp32 state.  The reference keeps
 * the state in fp32 (kernel.cu:982-994); this variant trades its precision
 * (about 3 significant digits per element) for bandwidth. */
int gdn_decode_launch_bf16_state(const GdnDecodeArgs* args, void* stream);

/* Head counts other than 4 q/k and 8 v heads (head dim 128; num_v_heads a
 * multiple of num_qk_heads, v head h reading q/k head h / (num_v_heads /
 * num_qk_heads), the reference's repeat_interleave grouping,
 * reference_torch_impl.py:46-47; e.g. 16 / 32, the contest's other shape).
 * Every tensor's head axis has the given count; otherwise as
 * gdn_decode_launch_tokens (tokens >= 1, fp32 state) or, with bf16_state != 0,
 * gdn_decode_launch_bf16_state (tokens = 1). */
int gdn_decode_launch_heads(const GdnDecodeArgs* args, int32_t num_qk_heads, int32_t num_v_heads, int64_t tokens,
                            int32_t bf16_state, void* stream);

/* One decode step for a caller that keeps the state in HOST memory (state
 * offloaded between steps).  `host` holds host pointers to every input and
 * to output / new_state (pinned memory, or the copies do not overlap); `dev`
 * holds device buffers of the same batch that receive the inputs (q, k, v,
 * A_log, a, dt_bias, b), the output, and the state in place (dev->new_state;
 * dev->state must be NULL or equal to it).  The state is cut into `slices`
 * (1..64) whose host->device copy, kernel and device->host copy overlap on
 * three streams this library creates once per device; the call orders
 * itself after the work already on `stream`, and `stream` waits for all of
 * it.  Calls on one device are enqueued one at a time (they share those
 * streams).  No reference counterpart: the reference plugin took device
 * tensors only (kernel.cu:982-994). */
int gdn_decode_launch_host_staged(const GdnDecodeArgs* host, const GdnDecodeArgs* dev, int slices, void* stream);

/* --------------------------------------------------------------- prefill -- */

#define GDN_SEQLENS_INT32 0
#define GDN_SEQLENS_INT64 1

/* Prefill algorithm selector (GdnPrefillArgs.path).  AUTO sends batches of
 * short sequences (mean length <= 24) to the token-recurrent kernel and the
 * rest to the chunked tensor-core kernels.  No reference counterpart: the
 * reference's host dispatch chose among its Triton paths internally
 * (triton/kernel.py:93-129). */
#define GDN_PREFILL_PATH_AUTO 0
#define GDN_PREFILL_PATH_RECURRENT 1
#define GDN_PREFILL_PATH_CHUNKED 2
#define GDN_PREFILL_PATH_SEGMENTED 3  /* chunked, inter-chunk carry split into 4 composed segments per
                                         sequence (fewer for num_seqs > 3; used automatically, with as
                                         many segments as fit the SMs, when few long sequences leave
                                         SMs idle; needs the full workspace and num_seqs <= 4, else
                                         falls back to CHUNKED) */

/* Variable-length prefill over packed sequences.  Shapes:
 *   q, k       bf16 [T, 4, 128]        16-byte aligned
 *   v          bf16 [T, 8, 128]        16-byte aligned
 *   state      fp32 [N, 8, 128, 128]   or NULL (zero initial state)
 *   A_log      fp32 [8];  dt_bias fp32 [8]
 *   a, b       bf16 [T, 8]
 *   cu_seqlens int32 or int64 [N + 1], non-decreasing, cu[0] = 0, cu[N] <= T
 *   output     bf16 [T, 8, 128]        16-byte aligned
 *   new_state  fp32 [N, 8, 128, 128]   16-byte aligned; must not alias state
 * Empty sequences get a zero new_state row, as the reference oracle
 * (prefill reference_torch_impl.py:53-55).  Output rows of tokens that belong
 * to no sequence are written as zeros.
 * Reference: gdn_prefill_qk4_v8_d128_k_last/solution/triton/kernel.py:56-57. */
typedef struct GdnPrefillArgs {
    const void* q;
    const void* k;
    const void* v;
    const float* state;
    const float* A_log;
    const void* a;
    const float* dt_bias;
    const void* b;
    const void* cu_seqlens;
    int32_t cu_seqlens_dtype;
    int32_t path;            /* GDN_PREFILL_PATH_*; 0 = automatic choice */
    int64_t total_tokens;
    int64_t num_seqs;
    float scale;
    void* output;
    float* new_state;
} GdnPrefillArgs;

/* Bytes of device workspace for gdn_prefill_launch at these sizes (256-byte
 * aligned base).  Includes, for num_seqs <= 4, room for the segmented carry;
 * a smaller workspace that still holds the per-chunk operand images (about
 * 768 KiB per 64 tokens) is accepted and runs the single-pass carry.
 * Replaces the torch.empty scratch tensors the reference allocates per call
 * (triton/kernel.py:136-168, :196-218). */
size_t gdn_prefill_workspace_size(int64_t total_tokens, int64_t num_seqs);

int gdn_prefill_launch(const GdnPrefillArgs* args, void* workspace, size_t workspace_bytes,
                       void* stream);

/* gdn_prefill_launch for other head counts (rules as gdn_decode_launch_heads;
 * e.g. the contest's 16 q/k / 32 v heads): every tensor's head axis has the
 * given count, new_state is [N, num_v_heads, 128, 128].  args->path selects
 * the algorithm as for gdn_prefill_launch -- the chunked tensor-core kernels
 * take the head counts at run time -- and the workspace rules are the same
 * with gdn_prefill_workspace_size_heads(T, N, num_v_heads) in place of
 * gdn_prefill_workspace_size (a smaller workspace that holds the operand
 * records, (ceil(T / 64) + N) x num_v_heads x 96 KiB plus tables, runs the
 * single-pass carry; the token-recurrent path needs none and accepts NULL).
 * Reference: the reference kernels are fixed at 4 / 8 heads
 * (triton/kernel.py:30-33); its definition's head axes (FAQ.md:109-111). */
size_t gdn_prefill_workspace_size_heads(int64_t total_tokens, int64_t num_seqs, int32_t num_v_heads);
int gdn_prefill_launch_heads(const GdnPrefillArgs* args, int32_t num_qk_heads, int32_t num_v_heads,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Context parallelism: one batch of long sequences split by token range over
 * `world` GPUs (one process each).  Rank r holds the r-th consecutive range
 * of every sequence, every range at least one token (ranges of whole 64-token
 * chunks keep every chunk full); `args` describes the rank's local tokens
 * (local cu_seqlens).  args->state (the initial state) is read on rank 0 only.
 * Each rank cuts its range into up to 8 segments (the same count on every
 * rank, a function of num_seqs).
 *   1. gdn_prefill_cp_launch(args, ws, bytes, rank, world, 0, stream) on every
 *      rank: its chunk records, the carry summaries of its segments and their
 *      composition, the rank's summary (rank 0: the state after its range);
 *   2. all-gather world blocks of num_seqs x 8 x 98304 bytes at
 *      ws + gdn_prefill_cp_summary_offset(local_tokens, num_seqs), rank r
 *      contributing block r (e.g. an in-place NCCL all-gather on `stream`);
 *   3. gdn_prefill_cp_launch(..., 1, stream) on every rank: each segment
 *      composes the rank summaries before it and the rank's own segments
 *      before it into its start state and writes its outputs; new_state is
 *      the state after the rank's range (the last rank's is the batch's final
 *      state).
 * No reference counterpart (the reference prefill runs on one GPU,
 * triton/kernel.py:56-57); it lets one long sequence use several GPUs. */
size_t gdn_prefill_cp_workspace_size(int64_t local_tokens, int64_t num_seqs, int32_t world);
size_t gdn_prefill_cp_summary_offset(int64_t local_tokens, int64_t num_seqs);
int gdn_prefill_cp_launch(const GdnPrefillArgs* args, void* workspace, size_t workspace_bytes, int32_t rank,
                          int32_t world, int32_t phase, void* stream);

/* Size of the fixed scratch array behind gdn_prefill_launch_noalloc. */
#define GDN_NOALLOC_SCRATCH_BYTES (32u << 20)

/* gdn_prefill_launch for callers that cannot allocate device memory -- a
 * plugin host or server that owns all device memory and gives extensions no
 * allocator, or a step where cudaMalloc is not allowed (it may synchronise the
 * device and is illegal during stream capture).  No counterpart in the
 * reference, whose plugin allocated its scratch with torch.empty on every call.
 *
 * Same arguments and results as gdn_prefill_launch, but the scratch is a
 * fixed array of GDN_NOALLOC_SCRATCH_BYTES inside this library, held on every
 * GPU that loads the library until the process exits; nothing is allocated.
 * Limit: problems that run on the token-recurrent kernel (args->path
 * GDN_PREFILL_PATH_RECURRENT, or AUTO with total_tokens / num_seqs <= 24)
 * need no scratch and are always accepted.  Every other problem needs the
 * chunked kernels' per-chunk operand records in the array -- the minimum
 * workspace that gdn_prefill_launch also accepts, (ceil(T / 64) + N) x
 * 768 KiB plus small tables -- and is rejected with GDN_ERR_WORKSPACE before
 * anything runs when that exceeds GDN_NOALLOC_SCRATCH_BYTES (about 2,600
 * tokens of one sequence).  The segmented carry for few long sequences also
 * needs its summaries and runs only when the whole
 * gdn_prefill_workspace_size(T, N) fits; otherwise the single-pass carry
 * gives the same results more slowly.  The first call on each device
 * looks up the array's device address; make it before any stream capture.
 * All calls on a device share the array: calls whose kernels overlap on the
 * GPU (different streams or host threads) race and must be serialised. */
int gdn_prefill_launch_noalloc(const GdnPrefillArgs* args, void* stream);

/* ---------------------------------------------------------------- status -- */

/* Human-readable name of a gdn_status_t (static string). */
const char* gdn_status_string(int status);

/* Synchronises `stream`, then stores the current device's status word (OR of
 * GDN_ERR_DEVICE_* bits recorded by kernels since the last clear) in *out.
 * When `clear` is non-zero the word is reset to 0.  No reference counterpart:
 * the reference performs no error checking (kernel.cu:982-1064). */
int gdn_read_device_status(int* out, int clear, void* stream);

/* ABI version of this header (bumped on any struct or signature change, or a new entry point). */
int gdn_abi_version(void);

/* ------------------------------------------------------------ diagnostics -- */

#define GDN_MMA_KIND_BF16 1
#define GDN_MMA_KIND_TF32 2
#define GDN_MMA_KIND_F16 3

#define GDN_MMA_A_MN_MAJOR 1  /* A operand image stored MN-major */
#define GDN_MMA_B_MN_MAJOR 2  /* B operand image stored MN-major */
#define GDN_MMA_D_LANE16 4    /* accumulator at TMEM lane 16 (M = 64 only) */
#define GDN_MMA_A_TMEM 8      /* A operand read from TMEM (16-bit kinds, M = 128, K-major) */
#define GDN_MMA_NO_COMPLETION 16  /* diagnostic: issue no MMA and never signal its completion barrier, so the
                                     kernel's bounded wait expires: it records GDN_ERR_DEVICE_TIMEOUT in the
                                     device status word, releases its TMEM and returns; D is not written */

/* D[M x N] = A[M x K] . B[N x K]^T on one CTA through the same shared-memory
 * operand images, tcgen05 descriptors and TMEM read-back the prefill kernels
 * use; `flags` selects the operand majors and accumulator placement.  A, B
 * row-major in global memory (bf16 for BF16, fp16 for F16, fp32 for TF32 --
 * rounded to tf32); D fp32 row-major.  M in {64, 128}; N a multiple of 16 in [16, 256];
 * K in {64, 128}; an MN-major operand's M (or N) must fill whole 128-byte
 * rows (multiples of 64 bf16 / 32 tf32).  With GDN_MMA_NO_COMPLETION the call
 * exercises the device-side timeout instead (about 10 ms of GPU time).  No
 * reference counterpart: a self-test of the tensor-core layer. */
int gdn_mma_selftest(int kind, int flags, int M, int N, int K, const void* A, const void* B, float* D,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
