/*
 * wohper_b200.h -- C ABI of the B200 (sm_100a) dequant-matmul hot path of
 * Wohper (engine/zc_infer_core).  Every entry point here replaces one Rust
 * function of the reference's kernel layer; the comment above each cites the
 * reference interface it stands in for (path:line inside the reference
 * project).  A Rust FFI crate binds these symbols one to one.
 *
 * Conventions
 *  - All data pointers are DEVICE pointers owned by the caller (weights are
 *    uploaded once and stay resident in HBM); sizes are element counts unless
 *    a name says bytes.  Host-side descriptor structs (wh_fp4_matvec_spec,
 *    wh_fp4_expert, wh_moe_desc) hold device pointers.
 *  - Calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 *    stream).  Argument errors are detected on the host before anything is
 *    launched and returned immediately.  Errors that only the device can see
 *    (a non-finite output, a timed-out wait) are recorded in the context and
 *    returned by wh_ctx_sync(), which mirrors the reference's synchronous
 *    Result<(), Error>: call it after a call to get the reference's behaviour.
 *  - Status codes 1..8 are DeepSeekV4KernelError
 *    (engine/zc_infer_core/src/deepseek_v4.rs:398-408) in declaration order.
 *  - One wh_ctx per device and per calling thread at a time; calls on one ctx
 *    are not re-entrant (the reference serves one request at a time behind a
 *    mutex, src/server/api.rs:301).
 */
#ifndef WOHPER_B200_H
#define WOHPER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* wh_stream_t; /* == cudaStream_t */

typedef enum wh_status {
  WH_OK = 0,
  WH_ERR_EMPTY_SHAPE = 1,
  WH_ERR_INVALID_SHAPE = 2,
  WH_ERR_PACKED_WEIGHT_TOO_SMALL = 3,
  WH_ERR_SCALE_TOO_SMALL = 4,
  WH_ERR_INPUT_TOO_SMALL = 5,
  WH_ERR_OUTPUT_TOO_SMALL = 6,
  WH_ERR_SCRATCH_TOO_SMALL = 7,
  WH_ERR_NON_FINITE_OUTPUT = 8,
  WH_ERR_INVALID_POINTER = 9, /* ComputeError::InvalidPointer (src/compute.rs:337) */
  WH_ERR_UNSUPPORTED = 10,    /* ComputeError::UnsupportedQuantFormat / InvalidQuantBlock */
  WH_ERR_CUDA = 20,           /* a CUDA runtime call failed (detail: wh_last_error_detail) */
  WH_ERR_NCCL = 21,           /* a collective failed (expert parallelism) */
  WH_ERR_TIMEOUT = 22,        /* a bounded device-side wait expired */
  WH_ERR_DEVICE_ARG = 23,     /* a device-side index check failed (e.g. expert id) */
  /* ZCBLK01 blocks: ComputeError variants (src/compute.rs:329-343); the detail
   * string (wh_last_error_detail) is the variant's &'static str. */
  WH_ERR_BLOCK_MAGIC = 30,     /* InvalidQuantBlockMagic */
  WH_ERR_BLOCK_VERSION = 31,   /* UnsupportedQuantBlockVersion */
  WH_ERR_BLOCK_TRUNCATED = 32, /* TruncatedQuantBlock(field) */
  WH_ERR_BLOCK_INVALID = 33,   /* InvalidQuantBlock(reason) */
  WH_ERR_TENSOR_INDEX = 34,    /* TensorIndexOutOfRange */
  /* ZCINF01 model files: ModelFormatError variants (src/model_format.rs:31-55)
   * and SchedulerError::InvalidExpert (src/scheduler.rs:14). */
  WH_ERR_IO = 40,              /* Io */
  WH_ERR_MODEL_MAGIC = 41,     /* InvalidMagic */
  WH_ERR_MODEL_VERSION = 42,   /* UnsupportedVersion */
  WH_ERR_UNALIGNED = 43,       /* Unaligned { field } (detail = the field name) */
  WH_ERR_TRUNCATED_MANIFEST = 44, /* TruncatedManifest */
  WH_ERR_LAYER_COUNT = 45,     /* LayerCountMismatch */
  WH_ERR_EXPERT_TABLE = 46,    /* InvalidExpertTable */
  WH_ERR_SHARD_MAP = 47,       /* ShardMap (shard map or experts pack index) */
  WH_ERR_INVALID_EXPERT = 48   /* the layer has no expert with that id */
} wh_status;

/* ------------------------------------------------------------------------ */
/* Context                                                                   */
/* ------------------------------------------------------------------------ */
typedef struct wh_ctx wh_ctx;

/* Library ABI version (major*10000 + minor*100 + patch). */
int wh_version(void);

/* Creates a context on `device` (cudaSetDevice is called).  Allocates the
 * device status word and uploads the act-quant rounding table, which is
 * measured from the host's libm log2f so ceil(log2f(.)) matches the
 * reference bit for bit (src/compute.rs:2516).  The first context of a process
 * also measures the host libm's expf table (about 3 s of host time; every exp
 * of the kernels -- SiLU, the router, the MLA softmax -- then equals the
 * reference's f32::exp bit for bit), and each device gets its copy once (5.5 MB,
 * held until exit). */
wh_status wh_ctx_create(int device, wh_ctx** out);
void wh_ctx_destroy(wh_ctx* ctx);

/* Synchronises `stream` and returns the first device-side error recorded since
 * the previous wh_ctx_sync (WH_ERR_NON_FINITE_OUTPUT, WH_ERR_TIMEOUT,
 * WH_ERR_DEVICE_ARG), then clears it. */
wh_status wh_ctx_sync(wh_ctx* ctx, wh_stream_t stream);

/* Human-readable detail of the last error returned on this thread. */
const char* wh_last_error_detail(void);

/* Per-phase timing, the counterpart of the reference's ZC_PROF pass timers
 * (src/server/generation.rs:2344-2351).  While profiling is on, multi-kernel
 * entry points (wh_moe_ffn, wh_fp4_expert_forward) record a CUDA event before
 * and after each kernel and launch without programmatic dependent launch;
 * wh_ctx_phase_times synchronises and writes the last call's per-kernel
 * milliseconds (in launch order) to ms[0..n), returning the phase count. */
wh_status wh_ctx_set_profiling(wh_ctx* ctx, int on);
int wh_ctx_phase_times(wh_ctx* ctx, float* ms, int max_phases);

/* ------------------------------------------------------------------------ */
/* FP8 E4M3 x UE8M0 block-scaled GEMV                                        */
/* ------------------------------------------------------------------------ */
/* Replaces gemv_fp8_e4m3_ue8m0_tensorwise (src/compute.rs:6174-6239),
 * gemv_fp8_e4m3_ue8m0_rows (src/compute.rs:6244-6321) and
 * gemv_fp8_e4m3_ue8m0_rows_multi (src/compute.rs:6384-6577).
 *   weight [rows][cols] E4M3 bytes; scale [scale_rows][scale_cols] UE8M0
 *   bytes (rows % scale_rows == 0, cols % scale_cols == 0); computes output
 *   rows [row_start, row_end) for `batch` inputs x[b*ldx + c] into
 *   y[b*ldy + (r - row_start)].  Every output equals the reference's AVX2 row
 *   kernel bit for bit, for any batch.  act_quant_block > 0 first applies the
 *   reference's FP8 activation quant-dequant (block size act_quant_block) to
 *   a copy of each input, as its call sites do before every FP8 GEMV
 *   (src/compute.rs:4001). */
wh_status wh_fp8_gemv(wh_ctx* ctx, const uint8_t* weight, const uint8_t* scale, int rows, int cols,
                      int scale_rows, int scale_cols, int row_start, int row_end, const float* x,
                      int batch, int ldx, float* y, int ldy, int act_quant_block,
                      wh_stream_t stream);

/* Replaces fp8_act_quant_dequant_in_place (src/compute.rs:2504-2545): per
 * block, power-of-two scale from the block amax, nearest E4M3 value with ties
 * to the lower entry, in place. */
wh_status wh_act_quant_fp8(wh_ctx* ctx, float* values, size_t n, int block_size,
                           wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* FP4 E2M1 x UE8M0(per 32) matvec and expert forward                         */
/* ------------------------------------------------------------------------ */
/* Mirrors Fp4Matvec (src/deepseek_v4.rs:410-417); lengths are in bytes. */
typedef struct wh_fp4_matvec_spec {
  const uint8_t* packed_weight; /* [rows][(cols+1)/2], low nibble = even column */
  size_t packed_len;
  const uint8_t* ue8m0_scales; /* [rows][scale_cols] */
  size_t scales_len;
  size_t rows, cols, scale_cols;
} wh_fp4_matvec_spec;

/* Mirrors DeepSeekV4Fp4Expert (src/deepseek_v4.rs:419-428). */
typedef struct wh_fp4_expert {
  wh_fp4_matvec_spec w1, w3, w2;
} wh_fp4_expert;

/* Replaces fp4_e2m1_ue8m0_matvec_scalar (src/deepseek_v4.rs:464-549);
 * same validation order and errors as validate_fp4_matvec
 * (src/deepseek_v4.rs:434-462). */
wh_status wh_fp4_matvec(wh_ctx* ctx, const wh_fp4_matvec_spec* spec, const float* input,
                        size_t input_len, float* output, size_t output_len, wh_stream_t stream);

/* Replaces deepseek_v4_fp4_expert_scratch_len (src/deepseek_v4.rs:430-432). */
size_t wh_fp4_expert_scratch_len(size_t intermediate);

/* Replaces deepseek_v4_fp4_expert_forward_scalar (src/deepseek_v4.rs:561-601):
 * act quant(x) -> w1, w3 -> SwiGLU with the reference clamps -> act quant ->
 * w2.  `scratch` is a device buffer of scratch_len floats, at least
 * wh_fp4_expert_scratch_len(w1.rows). */
wh_status wh_fp4_expert_forward(wh_ctx* ctx, const wh_fp4_expert* expert, const float* input,
                                size_t input_len, float* output, size_t output_len,
                                float* scratch, size_t scratch_len, wh_stream_t stream);

/* wh_fp4_expert_forward without caller scratch and without any device
 * allocation: no reference counterpart (the reference's callers always pass
 * scratch).  For callers that cannot allocate device memory on the call path
 * -- a server whose arena owns all of HBM, or a decode loop that must not take
 * cudaMalloc/cudaFree's implicit synchronisation -- and cannot lend scratch.
 * Scratch is a fixed 65536-float device array inside the library; experts
 * with hidden + 2 * intermediate > 65536 return WH_ERR_SCRATCH_TOO_SMALL.
 * Nothing in it needs to start at zero.  The first call on each device looks
 * the array up (cudaGetSymbolAddress) and should happen before any stream
 * capture; after cudaDeviceReset the next call is a first call again (the
 * array is looked up anew in the new context).  The array is shared by every caller on a device: calls that
 * overlap in time there (other streams, threads or contexts) race; calls in
 * order on one stream are safe.  Computes the reference-order exact path;
 * device-side errors are reported by wh_ctx_sync like every other call. */
wh_status wh_fp4_expert_forward_noalloc(wh_ctx* ctx, const wh_fp4_expert* expert,
                                        const float* input, size_t input_len, float* output,
                                        size_t output_len, wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* FP8 E4M3 x UE8M0(128x128) expert (DeepSeek-V4's shared expert)             */
/* ------------------------------------------------------------------------ */
typedef struct wh_fp8_matrix {
  const uint8_t* weight; /* [rows][cols] E4M3 */
  const uint8_t* scale;  /* [scale_rows][scale_cols] UE8M0 */
  int rows, cols, scale_rows, scale_cols;
} wh_fp8_matrix;
typedef struct wh_fp8_expert {
  wh_fp8_matrix w1, w3, w2;
} wh_fp8_expert;

/* Floats of scratch wh_fp8_expert_forward needs (hidden + 2 * intermediate). */
size_t wh_fp8_expert_scratch_len(size_t hidden, size_t intermediate);
/* Replaces compute_deepseek_fp8_shared_expert_into_hidden
 * (src/compute.rs:5545-5614): act quant (block 64) of the input -> w1, w3 (FP8
 * GEMV, bit-exact) -> SwiGLU with the reference clamps -> act quant (64) -> w2,
 * written to output[0..w2.rows).  Shape errors in the reference's order. */
wh_status wh_fp8_expert_forward(wh_ctx* ctx, const wh_fp8_expert* expert, const float* input,
                                size_t input_len, float* output, size_t output_len,
                                float* scratch, size_t scratch_len, wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Router                                                                    */
/* ------------------------------------------------------------------------ */
#define WH_ROUTER_RAW_LOGITS 0     /* RouterMath::RawLogits + legacy softmax */
#define WH_ROUTER_SQRT_SOFTPLUS 1  /* RouterMath::DeepSeekV4SqrtSoftplus */

/* Replaces route_experts_from_dense_block (src/compute.rs:2129-2236) with
 * finalize_route_weights (src/compute.rs:2253-2268) and, in raw-logit mode,
 * normalize_route_weights_legacy (src/server/generation.rs:3152-3180).
 *   gate [experts][hidden] bf16 (uint16 bits); x [tokens][hidden];
 *   ids/weights [tokens][topk]; hash_ids (nullable, [tokens][topk]) is the
 *   tid2eid row of each token for hash layers (sqrt-softplus mode).  Expert
 *   ids are bit-exact with the reference.  logits (nullable,
 *   [tokens][experts]) receives the raw gate logits.  experts <= 1024,
 *   topk <= 32. */
wh_status wh_router_topk(wh_ctx* ctx, const uint16_t* gate, int experts, int hidden,
                         const float* x, int tokens, int topk, int mode, const float* bias,
                         float route_scale, const int32_t* hash_ids, int32_t* ids,
                         float* weights, float* logits, wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* MoE FFN layer (router + routed FP4 experts + shared expert + combine)      */
/* ------------------------------------------------------------------------ */
typedef struct wh_moe_desc {
  int num_experts;              /* routed experts (256 in DeepSeek-V4-Flash) */
  int hidden;                   /* 4096 */
  int inter;                    /* 2048 */
  const wh_fp4_expert* experts; /* host array [num_experts] of device-pointer specs */
  const wh_fp4_expert* shared;  /* nullable: always-on shared expert */
  const uint16_t* gate;         /* [num_experts][hidden] bf16 router weight */
  const float* gate_bias;       /* nullable selection bias (sqrt-softplus mode) */
  int topk;                     /* 6 */
  int router_mode;              /* WH_ROUTER_* */
  float route_scale;            /* 1.5 in DeepSeek-V4-Flash */
  int max_tokens;               /* largest `tokens` wh_moe_ffn will be given */
  int exact;                    /* 1: the bit-exact CUDA-core kernels for every call.
                                   0: calls of 32 or more tokens run on the tensor cores
                                   (grouped GEMMs, results within tolerance), smaller
                                   ones on the bit-exact kernels.  2: the tensor cores
                                   for every call.  The tensor-core path needs hidden
                                   and inter multiples of 512 and no UE8M0 scale byte 0
                                   or 255; otherwise the bit-exact kernels run. */
  const wh_fp8_expert* shared_fp8; /* nullable: an FP8 shared expert instead of `shared`
                                      (DeepSeek-V4's layout); y = shared(x) + routed, as
                                      compute_active_and_shared_experts adds them */
} wh_moe_desc;

typedef struct wh_moe_plan wh_moe_plan;

/* Validates every expert (as validate_fp4_matvec) and builds the device-side
 * descriptors (TMA tensor maps) once; allocates them on the device. */
wh_status wh_moe_plan_create(wh_ctx* ctx, const wh_moe_desc* desc, wh_moe_plan** out);
void wh_moe_plan_destroy(wh_moe_plan* plan);

/* Device scratch bytes wh_moe_ffn needs for `tokens` tokens. */
size_t wh_moe_scratch_bytes(const wh_moe_plan* plan, int tokens);

/* Where one intermediate array of the tensor-core (grouped) path lies inside
 * the scratch of a wh_moe_ffn call of `tokens` tokens: byte offset from the
 * scratch pointer and size.  For tests and debugging (the act-quantised SwiGLU
 * hidden of every routed row is WH_MOE_FIELD_HQ / _HSF); it has no
 * counterpart in the reference.  Rows of an expert are contiguous from
 * offsets[e]; the row of (token t, route k) is offsets[ids[t][k]] +
 * slot[t][k], the shared expert's row of token t is offsets[num_experts] + t.
 * Calls that do not take the grouped path return WH_ERR_UNSUPPORTED. */
#define WH_MOE_FIELD_SLOT 1      /* int32 [tokens][topk] */
#define WH_MOE_FIELD_OFFSETS 2   /* int32 [experts (+1 shared) + 1] */
#define WH_MOE_FIELD_COMBINE_W 3 /* f32 [tokens][topk]: w / sum(w) */
#define WH_MOE_FIELD_XQ 4        /* u8 [rows][hidden]: E4M3 act-quantised token */
#define WH_MOE_FIELD_XSF 5       /* u8 [rows][hidden/32]: UE8M0 */
#define WH_MOE_FIELD_HQ 6        /* u8 [rows][inter]: E4M3 act-quantised hidden */
#define WH_MOE_FIELD_HSF 7       /* u8 [rows][inter/32]: UE8M0 */
#define WH_MOE_FIELD_YROWS 8     /* f32 [rows][hidden]: each row's expert output */
wh_status wh_moe_scratch_field(const wh_moe_plan* plan, int tokens, int field, size_t* offset,
                               size_t* bytes);

/* One MoE FFN step for `tokens` tokens (x, y: [tokens][hidden] f32).
 * Replaces, per token, routing (see wh_router_topk) followed by
 * compute_active_and_shared_experts (src/compute.rs:1872-1946):
 * y = shared(x) + sum_k expert_k(x) * w_k/sum(w), summed in route order.
 * ids_out/weights_out (nullable, [tokens][topk]) receive the routes.
 * x and y may be device memory or pinned host memory that the device maps at
 * the same address (cudaHostAlloc / cudaHostRegister): the kernels then read x
 * and write y over the bus, with no copy-engine transfer; pageable host memory
 * returns WH_ERR_INVALID_POINTER.  The host-memory result is complete once the
 * stream has been synchronised. */
wh_status wh_moe_ffn(wh_ctx* ctx, const wh_moe_plan* plan, const float* x, int tokens,
                     const int32_t* hash_ids, float* y, int32_t* ids_out, float* weights_out,
                     void* scratch, size_t scratch_bytes, wh_stream_t stream);
/* on = 1: one-token calls of wh_moe_ffn run as one persistent kernel (router,
 * w1/w3, w2 and the combine; one cooperative CTA per SM) when the shapes allow
 * it: experts <= 2 x SM count, hidden % 512 == 0, inter % 256 == 0, hidden and
 * inter <= 4096, topk + shared <= 8.  The arithmetic is the same bit for bit.
 * The default (0) runs the router, moe_up and moe_down kernels, which are
 * faster on B200 today. */
wh_status wh_moe_plan_set_fused_decode(wh_moe_plan* plan, int on);

/* ------------------------------------------------------------------------ */
/* Expert parallelism: the routed experts sharded contiguously over `world`   */
/* ranks (rank r owns [r*E_l, (r+1)*E_l), E_l = plan's num_experts), the      */
/* shared expert replicated.  The reference runs on one host and has no       */
/* counterpart; these calls split its batched MoE (accumulate_expert_for_     */
/* positions + finish, src/compute.rs:1779-1870) across ranks.  The caller     */
/* moves data between them with its collectives (NCCL all-to-all):            */
/*   wh_ep_dispatch -> all-to-all(send_counts), all-to-all(send rows) ->        */
/*   wh_ep_expert_ffn -> all-to-all(result rows back) -> wh_ep_combine.         */
/* The plan's gate may be NULL; ids and weights come from the caller's router. */
/* ------------------------------------------------------------------------ */
/* Bytes of one dispatched row: hidden E4M3 bytes + hidden/32 UE8M0 bytes,
 * rounded up to 16. */
size_t wh_ep_row_bytes(int hidden);
/* Scratch for wh_ep_dispatch / wh_ep_expert_ffn with `tokens` own tokens and at
 * most `max_recv_rows` received rows. */
size_t wh_ep_scratch_bytes(const wh_moe_plan* plan, int world, int tokens, int max_recv_rows);
/* Act quant of the rank's tokens x [tokens][hidden] and one row per route in
 * send [tokens*topk][row_bytes], ordered by global expert id (so by destination
 * rank).  send_counts [world*E_l] (device) receives the routes per (rank, local
 * expert); pos [tokens*topk] the send row of each route (-1 for an invalid id,
 * which also sets WH_ERR_DEVICE_ARG). */
wh_status wh_ep_dispatch(wh_ctx* ctx, const wh_moe_plan* plan, int world, const float* x,
                         int tokens, const int32_t* ids, uint8_t* send, int32_t* send_counts,
                         int32_t* pos, void* scratch, size_t scratch_bytes, wh_stream_t stream);
/* The local experts over the received rows recv [recv_rows][row_bytes]
 * (source-major, counts recv_counts [world][E_l] on the device) and the shared
 * expert over the own tokens x_local.  y_rows [recv_rows + tokens][hidden]:
 * row i < recv_rows is the result of received row i, row recv_rows + t the
 * shared expert's output for own token t. */
wh_status wh_ep_expert_ffn(wh_ctx* ctx, const wh_moe_plan* plan, int world, const uint8_t* recv,
                           const int32_t* recv_counts, int recv_rows, const float* x_local,
                           int tokens, float* y_rows, void* scratch, size_t scratch_bytes,
                           wh_stream_t stream);
/* y[t] = y_shared[t] + sum over t's routes in ascending expert id of
 * y_back[pos] * w/sum(w) (uniform when the weights are not finite and
 * positive): y_back [tokens*topk][hidden] holds the result rows returned in
 * send order. */
wh_status wh_ep_combine(wh_ctx* ctx, const wh_moe_plan* plan, const int32_t* ids,
                        const float* weights, const int32_t* pos, int tokens, const float* y_back,
                        const float* y_shared, float* y, wh_stream_t stream);

/* Expert parallelism over peer memory: the same step without NCCL and without */
/* a host synchronisation.  Each rank creates a window (device memory the      */
/* other ranks store into over NVLink), exports its CUDA IPC handle, and       */
/* connects to every rank's handle (the caller moves the handles, e.g. with an */
/* all-gather).  Per step, on every rank and in this order:                    */
/*   wh_ep_p2p_dispatch -> wh_ep_p2p_expert_ffn -> wh_ep_p2p_combine          */
/* The kernels wait on the other ranks' arrival flags with a bounded wait     */
/* (WH_ERR_TIMEOUT at the next wh_ctx_sync when a rank never arrives).  All    */
/* ranks run the same number of steps; before wh_ep_window_destroy every rank  */
/* finishes its last step (device synchronised, then a host barrier), so that  */
/* no rank still stores into a window being freed.                             */
/* ------------------------------------------------------------------------ */
#define WH_EP_IPC_HANDLE_BYTES 64
typedef struct wh_ep_window wh_ep_window;
/* Bytes of one rank's exported window for at most max_tokens tokens per rank
 * (rows are laid out with room for max_tokens * topk rows from every source). */
size_t wh_ep_window_bytes(const wh_moe_plan* plan, int world, int max_tokens);
/* Allocates the window of `rank` and writes its IPC handle (64 bytes). */
wh_status wh_ep_window_create(wh_ctx* ctx, const wh_moe_plan* plan, int world, int rank,
                              int max_tokens, wh_ep_window** out, uint8_t* ipc_handle);
/* handles: [world][64], rank r's handle at r * 64 (this rank's own is ignored). */
wh_status wh_ep_window_connect(wh_ep_window* window, const uint8_t* handles);
void wh_ep_window_destroy(wh_ep_window* window);
/* Act quant of x [tokens][hidden] and one row per route stored into the
 * destination rank's window; pos [tokens*topk] receives the row of each route's
 * result in this rank's window (-1 for an invalid id, WH_ERR_DEVICE_ARG). */
wh_status wh_ep_p2p_dispatch(wh_ctx* ctx, wh_ep_window* window, const float* x, int tokens,
                             const int32_t* ids, int32_t* pos, wh_stream_t stream);
/* Waits for every source's rows, runs the local experts over them and the
 * shared expert over x_local (y_shared [tokens][hidden]); each result row is
 * stored into the window of the rank that owns its token. */
wh_status wh_ep_p2p_expert_ffn(wh_ctx* ctx, wh_ep_window* window, const float* x_local,
                               int tokens, float* y_shared, wh_stream_t stream);
/* Waits for every destination's results, then y as wh_ep_combine. */
wh_status wh_ep_p2p_combine(wh_ctx* ctx, wh_ep_window* window, const int32_t* ids,
                            const float* weights, const int32_t* pos, int tokens,
                            const float* y_shared, float* y, wh_stream_t stream);
/* The whole expert-parallel MoE layer on a connected window in one call:
 * wh_ep_p2p_dispatch -> wh_ep_p2p_expert_ffn -> wh_ep_p2p_combine, with the
 * route positions and the shared expert's output kept in the window's
 * rank-private memory.  x, y: [tokens][hidden] f32 of this rank's tokens
 * (tokens <= the window's max_tokens); ids, weights: [tokens][topk] routes
 * (global expert ids).  Every rank calls it once per step, in the same order;
 * the step splits the reference's batched MoE (accumulate_expert_for_positions
 * + finish, src/compute.rs:1779-1870) over the ranks, which the reference,
 * running on one host, has no counterpart for. */
wh_status wh_ep_moe_layer(wh_ctx* ctx, wh_ep_window* window, const float* x, int tokens,
                          const int32_t* ids, const float* weights, float* y,
                          wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* MLA attention (DeepSeek-V4 decode)                                          */
/* ------------------------------------------------------------------------ */
/* Replaces rope_inv_freqs (src/compute.rs:2591-2621) on the host: inv_freqs
 * [rope_dim/2].  yarn_factor <= 0 or original_seq_len == 0: plain RoPE. */
void wh_rope_inv_freqs(int rope_dim, float theta, float yarn_factor, float yarn_beta_fast,
                       float yarn_beta_slow, uint64_t yarn_original_seq_len, float* inv_freqs);
/* The attention core of compute_deepseek_v4_mla_attention (src/compute.rs:4080-4185),
 * bit-exact: scores q.k * head_dim^-0.5 over the sliding window
 * [max(0, token_pos + 1 - window), token_pos] of the layer's key cache and over
 * the compressed rows, softmax with the optional sink, the in-order weighted
 * sum of the keys (the values are the keys), division by the denominator and
 * the inverse RoPE of the rope part [nope_dim, head_dim).
 *   q [heads][head_dim]; keys: cache rows 0..token_pos, row stride key_stride;
 *   compressed [compressed_count][head_dim] (nullable when 0); sink [heads]
 *   (nullable); inv_freqs: HOST array [(head_dim - nope_dim)/2], the layer's
 *   rope_inv_freqs; out [heads][head_dim].  Device pointers otherwise.
 * The cos/sin of token_pos * inv_freq are computed on the host with the C
 * library, like the reference's f32::sin_cos; exp is the host C library's expf,
 * reproduced on the device through the table that wh_ctx_create installs.  The
 * scores live in a context-owned workspace: calls on one context are serialised
 * by the caller (one stream at a time).
 * Errors: InvalidShape (nope_dim > head_dim, odd rope part, key_stride <
 * head_dim, window < 1), Unsupported (rope part > 128, odd nope_dim, or
 * head_dim / visible rows beyond shared memory). */
wh_status wh_mla_attention(wh_ctx* ctx, const float* q, int heads, int head_dim, int nope_dim,
                           const float* keys, int key_stride, int token_pos, int window,
                           const float* compressed, int compressed_count, const float* sink,
                           const float* inv_freqs, float* out, wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* DeepSeek-V4 attention block: norm and the MLA projection path               */
/* ------------------------------------------------------------------------ */
/* Replaces apply_weighted_rms_norm (src/compute.rs:3077-3115) or, with
 * weight_bf16 NULL, rms_norm_in_place (src/compute.rs:7110-7122) for
 * `segments` vectors of n floats each (n <= 4096; in and out may be the same):
 * mean of squares summed in index order, inv = 1/sqrt(ms + 1e-6),
 * out = (x * inv) * weight.  Bit-exact. */
wh_status wh_rms_norm(wh_ctx* ctx, const float* in, float* out, int segments, int n,
                      const uint16_t* weight_bf16, wh_stream_t stream);

/* The reference's grouped low-rank projection wo_a (src/compute.rs:4244-4258:
 * gemv_fp8_e4m3_ue8m0_rows per group): row r of [row_start, row_end) reads
 * the input x + (r / group_rows) * group_offset (+ b * ldx for input b), with
 * the optional fused act quant applied to each group's input alone.  Bit-exact
 * as wh_fp8_gemv; y[b * ldy + r - row_start]. */
wh_status wh_fp8_gemv_grouped(wh_ctx* ctx, const uint8_t* weight, const uint8_t* scale, int rows,
                              int cols, int scale_rows, int scale_cols, int row_start,
                              int row_end, const float* x, int batch, int ldx, int group_rows,
                              long long group_offset, float* y, int ldy, int act_quant_block,
                              wh_stream_t stream);

/* One layer's MLA attention weights (DeepSeek-V4-Flash: hidden 4096, 64 heads
 * of 512 = 448 nope + 64 rope, q_lora_rank 1024, 8 output groups of rank 1024,
 * sliding window 128).  FP8 E4M3 matrices with UE8M0 128x128 scales. */
typedef struct wh_v4_attn {
  int hidden, heads, head_dim, nope_dim, q_lora_rank, o_groups, o_lora_rank, window;
  wh_fp8_matrix wq_a;   /* [q_lora_rank][hidden] */
  wh_fp8_matrix wq_b;   /* [heads * head_dim][q_lora_rank] */
  wh_fp8_matrix wkv;    /* [head_dim][hidden] */
  wh_fp8_matrix wo_a;   /* [o_groups * o_lora_rank][heads * head_dim / o_groups] */
  wh_fp8_matrix wo_b;   /* [hidden][o_groups * o_lora_rank] */
  const uint16_t* q_norm;  /* bf16 [q_lora_rank] (q_a_layernorm), NULL: unweighted */
  const uint16_t* kv_norm; /* bf16 [head_dim] (kv_a_layernorm), NULL: unweighted */
  const float* sink;       /* [heads] attention sink, nullable */
} wh_v4_attn;
/* Floats of scratch wh_v4_attention needs for `tokens` tokens. */
size_t wh_v4_attention_scratch_len(const wh_v4_attn* layer, int tokens);
/* Replaces compute_deepseek_v4_mla_attention (src/compute.rs:3924-4293) for
 * `tokens` decode tokens (1..32, each of its own sequence), bit-exact per
 * token: hidden [tokens][hidden] holds the normed attention inputs on entry
 * and the attention outputs on return.  q path wq_a -> q_norm -> act quant ->
 * wq_b -> per-head RMS -> RoPE; kv path wkv -> kv_norm -> RoPE of the rope
 * dims -> act quant of the nope dims, stored into row token_pos[t] of token
 * t's KV cache kv_caches[t] (row stride kv_stride); the attention core of
 * wh_mla_attention over the window and the compressed rows compressed[t]
 * [compressed_count[t]][head_dim] (produced by the caller's compressor; both
 * arrays nullable when there are none); act quant -> grouped wo_a -> act
 * quant -> wo_b.  The projections run once over all tokens (their weights
 * are read once, as in the reference's batched pass, src/compute.rs:4307).
 * token_pos, kv_caches, compressed, compressed_count and inv_freqs (the
 * layer's rope_inv_freqs) are HOST arrays; the pointers in them are device
 * pointers.  The MLA workspace is context-owned: calls on one context are
 * serialised by the caller. */
wh_status wh_v4_attention(wh_ctx* ctx, const wh_v4_attn* layer, int tokens, const int* token_pos,
                          float* hidden, float* const* kv_caches, int kv_stride,
                          const float* const* compressed, const int* compressed_count,
                          const float* inv_freqs, float* scratch, size_t scratch_len,
                          wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* mHC hyper-connections (DeepSeek-V4)                                         */
/* ------------------------------------------------------------------------ */
/* The residual stream of a layer is hc copies of the hidden vector: x is
 * [tokens][hc][hidden] f32 (hc_dim = hc * hidden per token).  All pointers are
 * device pointers; every result is bit-exact to the reference (sums in index
 * order without fused multiply-adds, exp = the host C library's expf).
 * wh_hc_pre and wh_hc_head keep their chain results in a context-owned
 * workspace: calls on one context are serialised by the caller.
 * Errors: InvalidShape (tokens, hc or hidden < 1, negative sinkhorn_iters),
 * Unsupported (hc > 8), InvalidPointer. */

/* Replaces hc_pre_into + hc_split_sinkhorn_scalar (src/compute.rs:4945-5053)
 * for each token: fn [(2 + hc) * hc][hc_dim], scale [3], base [(2 + hc) * hc];
 * outputs y [tokens][hidden] (the sub-block input), post [tokens][hc] and
 * comb [tokens][hc][hc] for the matching wh_hc_post. */
wh_status wh_hc_pre(wh_ctx* ctx, const float* fn, const float* scale, const float* base,
                    const float* x, int tokens, int hc, int hidden, int sinkhorn_iters,
                    float eps, float* y, float* post, float* comb, wh_stream_t stream);
/* Replaces hc_post_into (src/compute.rs:5055-5089): out[t][k] = post[t][k] y[t] +
 * sum_i comb[t][k][i] residual[t][i]; out [tokens][hc][hidden]. */
wh_status wh_hc_post(wh_ctx* ctx, const float* y, const float* residual, const float* post,
                     const float* comb, int tokens, int hc, int hidden, float* out,
                     wh_stream_t stream);
/* Replaces hc_head_pool (src/compute.rs:5091-5132): fn [hc][hc_dim], base [hc],
 * the scalar scale; pooled [tokens][hidden]. */
wh_status wh_hc_head(wh_ctx* ctx, const float* fn, float scale, const float* base, const float* x,
                     int tokens, int hc, int hidden, float eps, float* pooled,
                     wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* BF16 lm_head top-k                                                         */
/* ------------------------------------------------------------------------ */
/* Device scratch bytes wh_lm_head_topk needs. */
size_t wh_lm_head_scratch_bytes(long long rows, int top_k);
/* Replaces score_bf16_lm_head_topk (src/compute.rs:2867-2913) and
 * RowIndex::topk_bf16_lm_head (src/row_index.rs:208-300): every row's logit is
 * dot_bf16_row (src/compute.rs:6116-6136) of weight [rows][cols] (bf16 bits)
 * with x, bit-exact; the rows kept are those push_topk_candidate keeps
 * (src/compute.rs:2948-2962), ties and NaNs included, written sorted
 * descending by total_cmp: out_tokens / out_logits [min(top_k, rows)]
 * (device), token = row_base + row.  top_k < 1 means 1 (top_k.max(1)).
 * logits (nullable, [rows], device) also receives every row's logit.  Needs
 * cols % 8 == 0 and a 16-byte aligned weight; top_k <= 511; cols <= 16384. */
wh_status wh_lm_head_topk(wh_ctx* ctx, const uint16_t* weight, long long rows, int cols,
                          uint32_t row_base, const float* x, size_t x_len, int top_k,
                          uint32_t* out_tokens, float* out_logits, float* logits, void* scratch,
                          size_t scratch_bytes, wh_stream_t stream);
/* Device scratch bytes wh_lm_head_topk_batch needs for `tokens` inputs. */
size_t wh_lm_head_batch_scratch_bytes(long long rows, int top_k, int tokens);
/* wh_lm_head_topk for `tokens` inputs at once, as the reference's batched
 * decode scores each position (score_bf16_lm_head_topk per token of
 * run_positions_batch, src/server/generation.rs:2330): input t is
 * x + t * ldx; its result goes to out_tokens / out_logits + t * top_k and, when
 * logits is given, its logits to logits + t * rows.  Each token's result equals
 * wh_lm_head_topk's bit for bit; the weight is streamed once per tile of up to
 * 8 tokens instead of once per token.  Same limits as wh_lm_head_topk, and
 * 1 <= tokens <= 65535, ldx >= cols. */
wh_status wh_lm_head_topk_batch(wh_ctx* ctx, const uint16_t* weight, long long rows, int cols,
                                uint32_t row_base, const float* x, int tokens, int ldx,
                                int top_k, uint32_t* out_tokens, float* out_logits,
                                float* logits, void* scratch, size_t scratch_bytes,
                                wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* ZCBLK01 tensor blocks (host memory; no device work)                        */
/* ------------------------------------------------------------------------ */
/* A block is [header 40 B][records 52 B each][names][data][shapes]; all
 * positions below are byte offsets from the start of the block. */
typedef struct wh_zcblk_header {
  uint32_t tensor_count, quant_format, flags, reserved;
  uint64_t record_table_offset, names_offset;
} wh_zcblk_header;

typedef struct wh_zcblk_tensor {
  uint16_t dtype_original, quant_format;
  uint32_t rank, flags; /* role = flags & 0xffff (TensorRole, src/compute.rs:455-499) */
  uint64_t name_pos, name_len;
  uint64_t shape_pos;   /* the [rank:u32][dims:u64 x rank] blob */
  uint64_t data_pos, data_len;
  float scale, zero_point;
  uint32_t reserved;
} wh_zcblk_tensor;

/* Replaces parse_quant_block (src/compute.rs:1099-1147). */
wh_status wh_zcblk_parse(const uint8_t* block, size_t len, wh_zcblk_header* out);
/* Replaces QuantBlockLayout::tensor (src/compute.rs:545-595). */
wh_status wh_zcblk_tensor_at(const uint8_t* block, size_t len, uint32_t index,
                             wh_zcblk_tensor* out);
/* Replaces ShapeLayout::dim (src/compute.rs:514-520). */
wh_status wh_zcblk_tensor_dim(const uint8_t* block, size_t len, const wh_zcblk_tensor* tensor,
                              uint32_t index, uint64_t* out);
/* Replaces find_tensor_by_suffix (src/compute.rs:1149-1169): the one tensor
 * whose name ends with `suffix` (NUL-terminated). */
wh_status wh_zcblk_find_suffix(const uint8_t* block, size_t len, const char* suffix,
                               wh_zcblk_tensor* out);

typedef struct wh_zcblk_fp4_view {
  uint64_t weight_pos, weight_len, scale_pos, scale_len;
  uint64_t rows, cols, scale_cols;
} wh_zcblk_fp4_view;
typedef struct wh_zcblk_fp4_expert_view {
  wh_zcblk_fp4_view w1, w3, w2;
} wh_zcblk_fp4_expert_view;
/* Replaces parse_quant_block + deepseek_v4_fp4_expert_from_quant_block
 * (src/compute.rs:1199-1267): w1/w3/w2 found by the .wN.weight / .wN.scale
 * name suffixes, checked as FP4 E2M1 packed + UE8M0, shapes cross-checked. */
wh_status wh_zcblk_fp4_expert(const uint8_t* block, size_t len, wh_zcblk_fp4_expert_view* out);

/* Device bytes one expert block of `payload_bytes` needs once its six tensors
 * are placed at 256-byte boundaries (w1 weight, w1 scale, w3 weight, w3 scale,
 * w2 weight, w2 scale). */
size_t wh_fp4_expert_device_bytes(uint64_t payload_bytes);
/* Parses one FP4 expert block held in host memory and copies its six tensors
 * to `dst` (device, 256-byte aligned, at least wh_fp4_expert_device_bytes);
 * `out` receives device specs for wh_fp4_expert_forward / wh_moe_desc.  The
 * copies are asynchronous on `stream`; keep `block` alive until they finish. */
wh_status wh_fp4_expert_upload(wh_ctx* ctx, const uint8_t* block, size_t len, void* dst,
                               size_t dst_bytes, wh_fp4_expert* out, wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* ZCINF01 model manifest, shard map and experts pack                        */
/* ------------------------------------------------------------------------ */
/* EngineHeader (src/model_format.rs:57-81), 128 bytes. */
typedef struct wh_engine_header {
  uint8_t magic[8];
  uint32_t version, endian;
  uint64_t file_size, manifest_offset, manifest_size, tokenizer_offset, tokenizer_size;
  uint64_t router_metadata_offset, router_metadata_size;
  uint32_t model_family, architecture, num_layers, hidden_size, num_attention_heads;
  uint32_t num_kv_heads, experts_per_layer, active_experts_per_token, block_alignment;
  uint32_t disk_quant_format;
  uint64_t manifest_checksum, file_checksum;
} wh_engine_header;

/* MoELayerBlockDesc (src/model_format.rs:141-150); block type = flags & 0xff
 * (0 compute, 1 global auxiliary). */
typedef struct wh_model_layer {
  uint32_t layer_id, flags;
  uint64_t dense_offset, dense_disk_bytes, dense_payload_bytes, dense_dequant_bytes;
  uint32_t num_experts, reserved;
} wh_model_layer;

/* ExpertBlockDescDisk (src/model_format.rs:113-125), 56 bytes. */
typedef struct wh_model_expert {
  uint32_t layer_id, expert_id;
  uint64_t disk_offset, disk_bytes, payload_bytes, dequant_bytes;
  uint32_t quant_format, route_rank_hint;
  uint64_t checksum;
} wh_model_expert;

#define WH_SOURCE_MODEL 0 /* the model file at the manifest's disk_offset */
#define WH_SOURCE_SHARD 1 /* an expert shard file named by MODEL.shards.json */
#define WH_SOURCE_PACK 2  /* the experts pack named by MODEL.experts_pack.index.json */
typedef struct wh_expert_source {
  const char* path; /* owned by the model handle */
  uint64_t offset, disk_bytes, payload_bytes;
  int kind;         /* WH_SOURCE_* */
  int reserved;
} wh_expert_source;

typedef struct wh_model wh_model;
/* Replaces ModelManifest::load (src/model_format.rs:193-263): header,
 * manifest, layer and expert tables with their validation, then the optional
 * MODEL.shards.json (load_optional_shard_map, :339-436; merge_sidecar_experts
 * = the reference's ZC_SIDECAR_EXPERTS=all) and the optional
 * MODEL.experts_pack.index.json (load_optional_expert_pack, :463-505). */
wh_status wh_model_open(const char* path, int merge_sidecar_experts, wh_model** out);
void wh_model_close(wh_model* model);
wh_status wh_model_get_header(const wh_model* model, wh_engine_header* out);
int wh_model_layer_count(const wh_model* model);
/* `layer_index` is the position in the manifest's layer table (a global
 * auxiliary block may share layer_id 0 with the first compute layer). */
wh_status wh_model_get_layer(const wh_model* model, int layer_index, wh_model_layer* out);
wh_status wh_model_get_expert(const wh_model* model, int layer_index, int expert_index,
                              wh_model_expert* out);
/* Where an expert's block is read from, as MoEIoScheduler::enqueue_expert_read
 * (src/scheduler.rs:148-193): the experts pack when it has the expert, else
 * the manifest's block in its shard file (if the shard map names one) or in
 * the model file. */
wh_status wh_model_expert_source(const wh_model* model, int layer_index, uint32_t expert_id,
                                 wh_expert_source* out);

/* ------------------------------------------------------------------------ */
/* Expert loader: FP4 expert blocks from disk into HBM                        */
/* ------------------------------------------------------------------------ */
/* Reader threads pread each expert's block into pinned staging buffers (two
 * per thread) and the copy engines move its six tensors into a caller-owned
 * device arena at 256-byte boundaries while the next block is read.  No
 * reference counterpart: the reference reads blocks into host RAM
 * (src/direct_io.rs) and computes from there; here the experts live in HBM.
 * threads <= 0 picks 8; direct_io != 0 opens files with O_DIRECT where the
 * file system allows it. */
typedef struct wh_expert_loader wh_expert_loader;
wh_status wh_expert_loader_create(wh_ctx* ctx, const wh_model* model, int threads, int direct_io,
                                  wh_expert_loader** out);
void wh_expert_loader_destroy(wh_expert_loader* loader);
/* Arena bytes wh_expert_loader_load needs for these experts of a layer. */
wh_status wh_expert_arena_bytes(const wh_model* model, int layer_index,
                                const uint32_t* expert_ids, int n, size_t* out);
/* Loads experts expert_ids[0..n) of the layer into `arena` (device memory,
 * 256-byte aligned, at least wh_expert_arena_bytes); out[i] receives the
 * device specs of expert_ids[i].  Returns once every block has been read and
 * its copies queued; work queued on `stream` afterwards sees the weights. */
wh_status wh_expert_loader_load(wh_expert_loader* loader, int layer_index,
                                const uint32_t* expert_ids, int n, void* arena,
                                size_t arena_bytes, wh_fp4_expert* out, wh_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Test hooks (host-only, no device work): expose the host-side pieces the   */
/* kernels rely on so CPU tests can pin them.                                */
/* ------------------------------------------------------------------------ */
/* The act-quant ceil(log2f) threshold table: out[E] for biased exponent E. */
void wh_debug_act_quant_table(uint32_t out[256]);
/* The E4M3 nearest-with-ties-to-lower rounding the kernels use (|t| <= 448). */
float wh_debug_e4m3_round(float t);
void wh_debug_e4m3_round_n(const float* in, float* out, size_t n); /* host arrays */
/* The table that makes the device's exp equal the host C library's expf: the
 * first wh_ctx_create of a process builds it by scanning expf over (-104, 89)
 * (about 3 s of host time on 8 threads) and installs it on each device.
 * Returns the number of entries, negated if some difference fell outside the
 * device's midpoint gate (wh_ctx_create then fails with Unsupported). */
int wh_debug_expf_table(const uint32_t** keys, const float** vals);
/* The band the device's exp looks inputs up in: a result within this relative
 * distance of a float rounding midpoint is looked up in the table above.  It is
 * measured with the table: the smallest power of two at least twice the
 * farthest distance of any host difference, in [2^-44, 2^-30]. */
double wh_debug_expf_near(void);
/* y[i] = the host libm's expf(x[i]), evaluated on the device (device arrays). */
wh_status wh_debug_ref_expf(wh_ctx* ctx, const float* x, float* y, size_t n,
                            wh_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* WOHPER_B200_H */
