/*
 * C ABI of the B200-native fused FP8 block-scale MoE layer with DeepSeek-V3
 * routing (definition moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048).
 *
 * Plain pointers and sizes only: no torch, no CUDA types in the signatures.
 * Device pointers are CUDA global-memory addresses on the current device;
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Every entry point returns a moe_status (0 = success) and never aborts the
 * process.  Work is enqueued on `stream` without any host synchronisation,
 * except in moe_fp8_ds_read_device_error, which synchronises the stream.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   moe_fp8_ds_run            <- kernel(...) solution/python/kernel.py:95-120,
 *                                which calls run(...) solution/python/main.cpp:66-266
 *                                (pybind11 binding main.cpp:268-270); same
 *                                arguments, same destination-passing output.
 *   moe_fp8_ds_run_routed     <- the post-routing half of run(...):
 *                                main.cpp:95-265 given topk_idx/topk_w
 *                                (the reference has no separate entry; this one
 *                                serves expert-parallel dispatch).
 *   moe_fp8_ds_workspace_size <- the per-call torch::empty allocations of
 *                                main.cpp:87-89,110-112,122-127,141-144,169-170,
 *                                181-182,200-201,217-218 and
 *                                moe_grouped_gemm_fp8.cu:841-852, which become
 *                                one caller-owned workspace.
 *   moe_fp8_ds_read_device_error <- CUDA_CHECK in solution/python/kernel.h:28-34
 *                                (which only prints); here device-side faults
 *                                such as a timed-out wait are reported as a status.
 */
#ifndef MOE_FP8_DS_H_
#define MOE_FP8_DS_H_

#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum moe_status {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARGUMENT = 1,   /* null pointer, bad shape or scalar */
  MOE_ERR_MISALIGNED = 2,         /* a pointer is not 16-byte aligned */
  MOE_ERR_WORKSPACE_TOO_SMALL = 3,
  MOE_ERR_CUDA = 4,               /* a CUDA runtime call failed (launch, attribute) */
  MOE_ERR_NO_DEVICE = 5,          /* not an sm_100 device, or no driver entry point */
  MOE_ERR_DEVICE_TIMEOUT = 6,     /* a bounded device-side wait gave up */
  MOE_ERR_DEVICE_FAULT = 7,       /* another device-side check failed */
  MOE_ERR_TOO_LARGE = 8,          /* a size exceeds a fixed limit of the entry point */
} moe_status;

/* Arguments of one layer call.  Shapes follow the reference signature
 * (solution/python/kernel.py:95-107); E_l = num_local_experts.            */
typedef struct moe_fp8_ds_args {
  const float* routing_logits;        /* fp32 [T, 256]                                 */
  const void* routing_bias;           /* bf16 [256]                                    */
  const void* hidden_states;          /* e4m3 [T, 7168]                                */
  const float* hidden_states_scale;   /* fp32 [56, T]                                  */
  const void* gemm1_weights;          /* e4m3 [E_l, 4096, 7168]                        */
  const float* gemm1_weights_scale;   /* fp32 [E_l, 32, 56]                            */
  const void* gemm2_weights;          /* e4m3 [E_l, 7168, 2048]                        */
  const float* gemm2_weights_scale;   /* fp32 [E_l, 56, 16]                            */
  void* output;                       /* bf16 [T, 7168], fully overwritten (DPS)       */
  int32_t num_tokens;                 /* T >= 0                                        */
  int32_t num_local_experts;          /* E_l in [1, 256]                               */
  int32_t local_expert_offset;        /* global id of local expert 0                   */
  float routed_scaling_factor;
  /* Only for moe_fp8_ds_run_routed: the routing decision, global expert ids
   * (ascending per token) and their weights.  Ignored by moe_fp8_ds_run.   */
  const int32_t* topk_ids;            /* int32 [T, 8]                                  */
  const float* topk_weights;          /* fp32 [T, 8]                                   */
  /* Optional fp32 [T, 7168] destination.  When non-null the layer result is
   * written here in fp32 instead of bf16 to `output` (used by the
   * expert-parallel combine, which sums partial results of several ranks). */
  float* output_f32;
} moe_fp8_ds_args;

/* Byte offsets (from the workspace base) of the intermediate buffers, for
 * tests and debugging.  All offsets are 256-byte aligned.                  */
typedef struct moe_fp8_ds_layout {
  uint64_t total_bytes;
  uint64_t error_word;      /* int32 [4]                                          */
  uint64_t topk_ids;        /* int32 [T, 8]   global ids, ascending per token      */
  uint64_t topk_weights;    /* fp32  [T, 8]                                       */
  uint64_t inv_row;         /* int32 [T, 8]   permuted row of (t,k) or -1         */
  uint64_t seg_offsets;     /* int32 [E_l+1]  rows of local expert e              */
  uint64_t row_token;       /* int32 [R_cap]  source token of each permuted row   */
  uint64_t block_masks;     /* uint8 [E_l, 4*ceil(T/32)] bit w: token 8g+w picked e */
  uint64_t block_bases;     /* int32 [ceil(T/32), E_l] first row of block b in expert e */
  uint64_t inter;           /* e4m3  SwiGLU output in two terms: weights-on-M GEMMs
                               [R_cap][2][2048] rows (hi, lo), lo on scale/16;
                               tokens-on-M GEMMs [2][R_cap][2048] planes (hi, lo)
                               on one scale                                      */
  uint64_t inter_scale;     /* fp32  [16, R_cap]  1x128 scales of the SwiGLU output */
  uint64_t down;            /* fp32  [R_cap, 7168] GEMM2 output per permuted row  */
  uint64_t act;             /* e4m3  [R_cap, 7168] permuted hidden rows (e4m3 GEMM1 input) */
  uint64_t act_scale;       /* fp32  [56, R_cap]  their 1x128 scales              */
  int32_t row_capacity;     /* R_cap = T * min(8, E_l) rounded up to 16           */
  int32_t reserved;
} moe_fp8_ds_layout;

/* Workspace bytes needed for T tokens and E_l local experts. */
MOE_API int moe_fp8_ds_workspace_size(int32_t num_tokens, int32_t num_local_experts, uint64_t* bytes);

/* Offsets of the intermediate buffers inside the workspace. */
MOE_API int moe_fp8_ds_workspace_layout(int32_t num_tokens, int32_t num_local_experts,
                                moe_fp8_ds_layout* layout);

/* Full layer: routing, permutation, GEMM1 + SwiGLU, GEMM2, weighted combine.
 * `workspace` is a device buffer of at least moe_fp8_ds_workspace_size bytes,
 * 256-byte aligned, and zero-filled once before its first use (only the
 * 16-byte error word at offset 0 must start at zero; every other byte is
 * rewritten by each call).  A device-side error stays in the error word
 * until moe_fp8_ds_read_device_error clears it.  One workspace must not be
 * shared by calls that run concurrently.                                   */
MOE_API int moe_fp8_ds_run(const moe_fp8_ds_args* args, void* workspace, uint64_t workspace_bytes,
                   void* stream);

/* Same as moe_fp8_ds_run but with the routing supplied in args->topk_ids /
 * args->topk_weights (routing_logits and routing_bias are not read).       */
MOE_API int moe_fp8_ds_run_routed(const moe_fp8_ds_args* args, void* workspace,
                          uint64_t workspace_bytes, void* stream);

/* Allocation-free layer call, for callers that cannot allocate device
 * memory where they call the layer (an external memory manager owns all
 * allocations, or cudaMalloc is not allowed on the serving path).  No
 * counterpart in the reference.  Same arguments and result as
 * moe_fp8_ds_run (bit for bit: the same kernels on the same plan), but the
 * workspace is a 16 MiB array inside this library that every GPU loading the
 * library keeps until the process exits; T is limited to 16 tokens
 * (MOE_ERR_TOO_LARGE beyond).  The first call on a device (and context) looks
 * up that array's device address and zeroes its error block, so make it
 * before any stream capture.  All calls on a device share the array: calls
 * that overlap on the GPU (different streams, or threads) race and must be
 * serialised by the caller.  A device-side error of any call stays recorded
 * until moe_fp8_ds_noalloc_read_device_error reads it.                     */
MOE_API int moe_fp8_ds_run_noalloc(const moe_fp8_ds_args* args, void* stream);

/* Synchronises `stream`, reads and clears the device error word of the
 * allocation-free entry point's built-in workspace (as
 * moe_fp8_ds_read_device_error does for a caller's workspace).  No
 * counterpart in the reference.                                            */
MOE_API int moe_fp8_ds_noalloc_read_device_error(void* stream, int32_t* device_error);

/* Routing only: writes ids (ascending per token) and weights.              */
MOE_API int moe_fp8_ds_route(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                     float routed_scaling_factor, int32_t* topk_ids, float* topk_weights,
                     void* stream);

/* Synchronises `stream`, reads and clears the workspace's device error word.
 * *device_error receives the raw code (0 = none); the return value maps it
 * to a moe_status.                                                         */
MOE_API int moe_fp8_ds_read_device_error(void* workspace, void* stream, int32_t* device_error);

/* Failure-detection self test (no counterpart in the reference): enqueue a
 * one-thread kernel that waits, with the layer's bounded device-side wait
 * (about one second), on a workspace counter nothing increments.  The wait
 * gives up, records a timeout in the workspace error word and returns; the
 * next moe_fp8_ds_read_device_error reports MOE_ERR_DEVICE_TIMEOUT and the
 * context stays usable.  Uses 16 bytes at the workspace base.              */
MOE_API int moe_fp8_ds_selftest_wait_timeout(void* workspace, void* stream);

/* Description of the CUDA runtime error behind the calling thread's last
 * MOE_ERR_CUDA from a layer call (a launch or attribute failure); "no error"
 * if there was none.  No counterpart in the reference.                     */
MOE_API const char* moe_fp8_ds_last_cuda_error_string(void);

/* Static description of a status code. */
MOE_API const char* moe_fp8_ds_status_string(int status);

/* Tuning knob: force the token-tile cap (a multiple of 16, at most 256) of
 * GEMM1 and GEMM2 for calls on this process; 0 restores the automatic choice
 * from T.  The weights-on-M GEMMs take 16, 32, 64 or 128 and use the
 * automatic choice for other values; the tokens-on-M GEMMs take the GEMM1
 * value (at most 128) for both.  Takes effect for the next call (workspace
 * size included). */
MOE_API int moe_fp8_ds_set_tile_override(int32_t bn_gemm1, int32_t bn_gemm2);

/* Tuning knob: 0 = automatic GEMM family (e4m3 GEMMs with weights on the
 * MMA's M side for T < 1280, e4m3 GEMMs with tokens on M from 1280 tokens),
 * 1 = always weights-on-M, 2 = always tokens-on-M.  Takes effect for the next
 * call (workspace size included). */
MOE_API int moe_fp8_ds_set_path_override(int32_t mode);

/* Profiling hook: when `count` is 7, later calls on this process record
 * events[0..6] (cudaEvent_t handles) on the call's stream around the stages
 * route | scan | scatter | GEMM1 | GEMM2 | combine (for T <= 256 the first
 * three share one launch, timed by events 0..1; events 1 and 2 are then
 * recorded back to back),
 * so a caller can time every kernel;
 * count 0 turns it off.  The events must outlive the calls that use them. */
MOE_API int moe_fp8_ds_set_stage_events(void* const* events, int32_t count);

/* Number of kernel launches one moe_fp8_ds_run call with T tokens enqueues
 * (4 for T <= 256, where routing, row assignment and the activation gather
 * share one launch; 6 above; moe_fp8_ds_run_routed always enqueues 6). */
MOE_API int moe_fp8_ds_launches_per_call(int32_t num_tokens);

/* ---------------------------------------------------------------------------
 * Expert-parallel plumbing (no counterpart in the reference, whose only
 * multi-GPU hook is local_expert_offset, solution/python/kernel.py:104).
 * Rank r of `world` owns global experts [r*E_r, (r+1)*E_r), E_r*world = 256.
 * A dispatch row is hidden e4m3 [7168] | scales fp32 [56] | ids int32 [8] |
 * weights fp32 [8] = 7456 bytes; rows go to ranks in (rank, token) order.
 * ------------------------------------------------------------------------- */
#define MOE_EP_ROW_BYTES 7456

/* From the routing (topk_ids [T,8]): rows per destination rank (counts, int64
 * [world]), the send row of each (token, rank) pair or -1 (slot, int32
 * [T, world]) and the source token of each send row (src_token, int32, at
 * least T*world entries; the first sum(counts) are written).  world <= 8.   */
MOE_API int moe_fp8_ds_ep_plan(const int32_t* topk_ids, int32_t num_tokens, int32_t world,
                               int32_t experts_per_rank, int64_t* counts, int32_t* slot,
                               int32_t* src_token, void* stream);

/* Build `rows` dispatch rows (send, [rows, 7456] bytes) from src_token.     */
MOE_API int moe_fp8_ds_ep_pack(const int32_t* topk_ids, const float* topk_weights, const void* hidden_states,
                               const float* hidden_states_scale, int32_t num_tokens, const int32_t* src_token,
                               int32_t rows, void* send, void* stream);

/* Fixed-capacity form of the two calls above (world >= 2, capacity >= T):
 * rank r's send rows are [r*capacity, (r+1)*capacity), its real rows first
 * (token order), then padding rows (src_token = -1).  Every peer then gets
 * exactly `capacity` rows, so the all-to-alls need no counts on the host and
 * a step runs without a device-to-host synchronisation.  A padding row is
 * zero except its 8 expert ids, all equal to the first expert of rank r+1
 * (mod world): valid, but not owned by the receiver, whose layer gives the
 * row no work and a zero partial.  slot[t][r] points into this layout;
 * send holds world*capacity rows.                                            */
MOE_API int moe_fp8_ds_ep_plan_capacity(const int32_t* topk_ids, int32_t num_tokens, int32_t world,
                                        int32_t experts_per_rank, int32_t capacity, int64_t* counts,
                                        int32_t* slot, int32_t* src_token, void* stream);
MOE_API int moe_fp8_ds_ep_pack_capacity(const int32_t* topk_ids, const float* topk_weights,
                                        const void* hidden_states, const float* hidden_states_scale,
                                        int32_t num_tokens, const int32_t* src_token, int32_t world,
                                        int32_t experts_per_rank, int32_t capacity, void* send, void* stream);

/* Split received rows into the layer's argument layout: hidden e4m3
 * [rows, 7168], scales fp32 [56, rows], ids int32 [rows, 8], weights fp32
 * [rows, 8] (the inputs of moe_fp8_ds_run_routed).                          */
MOE_API int moe_fp8_ds_ep_unpack(const void* recv, int32_t rows, void* hidden_states, float* hidden_states_scale,
                                 int32_t* topk_ids, float* topk_weights, void* stream);

/* output[t] = bf16(sum over ranks r ascending with slot[t][r] >= 0 of
 * partials[slot[t][r]]), the sum in fp32 from +0; partials fp32 [S, 7168]
 * in send-row order (each rank's unrounded sum over its own experts), output
 * bf16 [T, 7168].                                                           */
MOE_API int moe_fp8_ds_ep_combine(const void* partials, const int32_t* slot, int32_t num_tokens, int32_t world,
                                  void* output, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_FP8_DS_H_ */
