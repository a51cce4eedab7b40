/*
 * murm.h — C ABI of the B200 (sm_100a) slot_murmurate library.
 *
 * One operation, forward and backward:
 *
 *   slot_murmurate(q, slots_k, slots_v, rounds, top_k=7, causal)
 *       -> (out, indices, weights)
 *
 * For R rounds every token (row of q) selects its 7 highest-scoring slots by
 * q . slots_k (top-7, ties to the lowest slot index), attends over them with a
 * softmax of the scaled scores, then the slots take an EMA step towards the
 * weighted mean of the tokens that selected them and a 3-point Laplace
 * diffusion along the slot axis. out = sum of the R attend outputs; indices
 * and weights are those of the last round. Token keys and token values are q.
 *
 * Reference interface this replaces (beaglabs/murmurative-attention):
 *   - torch-ext/torch_binding.cpp:6-33   TORCH_LIBRARY(murmurative_attention)
 *     op schemas slot_select_attend / slot_update / slot_diffusion /
 *     slot_update_diffuse and their _backward ops, which the Python round
 *     loop src/murmurative/ops.py:330-422 (slot_murmurate) calls once per
 *     phase per round;
 *   - torch-ext/cuda_ops.h:6-68          the per-phase launcher signatures;
 *   - src/murmurative/reference.py:138-191 the semantics (round loop).
 * Here the whole round loop is one call; the per-phase ops are not exported.
 *
 * Conventions
 *   - All tensors are device pointers on the current CUDA device. The caller
 *     allocates everything: outputs, the `saved` block (written by forward,
 *     read by backward, must stay untouched in between) and scratch
 *     workspaces. Sizes come from murm_slot_murmurate_sizes(). Pointers must
 *     be 16-byte aligned; `saved` and workspaces 256-byte aligned.
 *   - Strides are in elements, {batch, head, row}; the innermost (head_dim)
 *     stride is 1. A batch stride of 0 for slots_k / slots_v broadcasts one
 *     slot table to every batch element.
 *   - `stream` is a cudaStream_t. Calls only enqueue work; they never
 *     synchronise the device and never allocate.
 *   - Results are deterministic: the same inputs give bitwise-identical
 *     outputs (no floating-point atomics anywhere).
 *   - Errors come back as murm_status; murm_last_error_message() gives the
 *     detail of the calling thread's last failure.
 */
#ifndef MURM_H_
#define MURM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MURM_API __attribute__((visibility("default")))
#else
#define MURM_API
#endif

#define MURM_ABI_VERSION 1
#define MURM_TOP_K 7

typedef enum murm_status {
  MURM_OK = 0,
  MURM_ERR_INVALID_ARGUMENT = 1, /* shape, pointer, stride or size not valid   */
  MURM_ERR_UNSUPPORTED = 2,      /* valid but not provided (top_k != 7, ...)    */
  MURM_ERR_DTYPE = 3,            /* element type not fp32 / fp16 / bf16         */
  MURM_ERR_WORKSPACE = 4,        /* saved / workspace block too small/unaligned */
  MURM_ERR_CUDA = 5,             /* a CUDA runtime call or launch failed        */
  MURM_ERR_DEVICE = 6            /* a kernel reported an error on the device    */
} murm_status;

typedef enum murm_dtype { MURM_F32 = 0, MURM_F16 = 1, MURM_BF16 = 2 } murm_dtype;

typedef struct murm_shape {
  int32_t batch;     /* B */
  int32_t heads;     /* H */
  int32_t tokens;    /* N, >= 1 */
  int32_t slots;     /* M, 7 <= M <= 256 */
  int32_t head_dim;  /* d, one of 16, 32, 64 */
  int32_t rounds;    /* R, >= 0 */
  int32_t top_k;     /* must be 7 */
  int32_t causal;    /* nonzero: token n sees slots m <= n only */
  double alpha;      /* EMA keep factor (reference default 0.9)   */
  double gamma;      /* diffusion step (reference default 0.15)   */
  double scale;      /* score scale; <= 0 means 1/sqrt(head_dim)  */
  int32_t dtype;     /* murm_dtype of q, slots, out and gradients */
} murm_shape;

typedef struct murm_fwd_args {
  murm_shape shape;
  const void* q;       int64_t q_stride[3];   /* [B,H,N,d] */
  const void* slots_k; int64_t sk_stride[3];  /* [B,H,M,d] */
  const void* slots_v; int64_t sv_stride[3];  /* [B,H,M,d] */
  void* out;           int64_t out_stride[3]; /* [B,H,N,d] */
  int64_t* indices;    /* [B,H,N,7] contiguous int64, or NULL */
  float* weights;      /* [B,H,N,7] contiguous fp32,  or NULL */
  void* saved;         size_t saved_bytes;     /* kept for backward */
  void* workspace;     size_t workspace_bytes; /* scratch */
} murm_fwd_args;

typedef struct murm_bwd_args {
  murm_shape shape;                            /* same as the forward call */
  const void* q;        int64_t q_stride[3];
  const void* grad_out; int64_t go_stride[3];  /* dL/d out, [B,H,N,d] */
  const float* grad_weights;                   /* dL/d weights [B,H,N,7] contiguous, or NULL */
  const void* saved;    size_t saved_bytes;    /* written by the forward call */
  void* grad_q;         int64_t gq_stride[3];
  void* grad_slots_k;   int64_t gsk_stride[3]; /* [B,H,M,d]; batch stride must be nonzero */
  void* grad_slots_v;   int64_t gsv_stride[3];
  void* workspace;      size_t workspace_bytes;
} murm_bwd_args;

/* Bytes of the saved block and of the forward / backward scratch workspaces.
 * Any output pointer may be NULL. */
MURM_API murm_status murm_slot_murmurate_sizes(const murm_shape* shape, size_t* saved_bytes,
                                      size_t* fwd_workspace_bytes,
                                      size_t* bwd_workspace_bytes);

/* Forward. Replaces the per-round ops.py:376-419 loop of
 * slot_select_attend (torch_binding.cpp:7-10) + slot_update_diffuse
 * (torch_binding.cpp:29-32). */
MURM_API murm_status murm_slot_murmurate_fwd(const murm_fwd_args* args, void* stream);

/* Backward. Replaces slot_select_attend_backward (torch_binding.cpp:11-14),
 * slot_update_backward (19-22) and slot_diffusion_backward (26-28) chained by
 * autograd through ops.py:75-92 and 188-208. */
MURM_API murm_status murm_slot_murmurate_bwd(const murm_bwd_args* args, void* stream);

/* Forward from an fp32 slot state: identical to murm_slot_murmurate_fwd except
 * that slots_k and slots_v are fp32 tables (strides in fp32 elements) whatever
 * shape.dtype says for q, out and the arithmetic. The round loop keeps its slot
 * state in fp32 between rounds (as the reference's fp32 update does,
 * reference.py:86-115), so this call runs rounds r..R-1 of a longer loop from
 * the state entering round r exactly as the full loop would: the state a
 * reference run recorded (teacher-forced parity checks), or fp32 master slot
 * tables kept by a caller whose tokens are 16-bit. No counterpart in the
 * reference, whose op schemas take slots in the token dtype
 * (torch_binding.cpp:7-10). Forward only; saved/workspace as for
 * murm_slot_murmurate_fwd. */
MURM_API murm_status murm_slot_murmurate_fwd_f32_slots(const murm_fwd_args* args, void* stream);

/* Forward that needs no caller-provided scratch. No counterpart in the
 * reference. For callers that cannot allocate device memory: a serving plugin
 * that is handed only its input and output buffers under a memory budget fixed
 * at start-up, or a foreign-language host with no binding to the CUDA
 * allocator. The round records and partial sums live in one file-scope device
 * array of MURM_NOSCRATCH_BYTES (64 MiB) that every GPU loading this library
 * holds until the process exits; this call allocates nothing. `saved` and
 * `workspace` in args must be NULL / 0; the caller still passes q, slots and
 * the outputs. A problem whose scratch exceeds the array is rejected with
 * MURM_ERR_WORKSPACE. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and keeps it for the life of that device's
 * primary context (after cudaDeviceReset the process must not call this entry
 * again); make that first call before any stream capture. All calls share the
 * array: calls that overlap on the GPU (different streams, or other host
 * threads) race on it; serialise them. Output only — there is no backward for
 * this entry point. */
#define MURM_NOSCRATCH_BYTES (64u << 20)
MURM_API murm_status murm_slot_murmurate_fwd_noscratch(const murm_fwd_args* args, void* stream);

/* Forward and backward over HOST buffers: the drop-in for a caller whose tensors
 * live in host memory — the reference's CPU path (src/murmurative/reference.py:
 * 138-191 called on CPU tensors, then its autograd backward with grad_out).
 * All tensors are contiguous: q, grad_out, out, grad_q [B,H,N,d]; slots_k,
 * slots_v, grad_slots_k, grad_slots_v [B,H,M,d]; indices int64 and weights
 * fp32 [B,H,N,7] (either may be NULL). The (batch, head) pairs are split into
 * `groups` (0: automatic — groups of at least 4 pairs, 2 to 8 groups)
 * that go through a three-stage pipeline — copy in on one
 * stream, murm_slot_murmurate_fwd + _bwd on `stream`, copy out on another —
 * so the host<->device copies overlap the kernels and each other. Host
 * buffers should be page-locked (cudaHostAlloc / pinned) for the copies to
 * overlap. `workspace` is one device block of murm_host_step_sizes() bytes,
 * 256-byte aligned. The call is asynchronous: the results are in the host
 * buffers once `stream` has completed. Calls are serialised internally. */
typedef struct murm_host_step_args {
  murm_shape shape;
  const void* q;
  const void* slots_k;
  const void* slots_v;
  const void* grad_out;
  void* out;
  int64_t* indices;
  float* weights;
  void* grad_q;
  void* grad_slots_k;
  void* grad_slots_v;
  int32_t groups;
  void* workspace;   size_t workspace_bytes;
} murm_host_step_args;

MURM_API murm_status murm_host_step_sizes(const murm_shape* shape, int32_t groups, size_t* workspace_bytes);
MURM_API murm_status murm_slot_murmurate_host_step(const murm_host_step_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Per-phase operations: the reference's op surface one round at a time
 * (torch-ext/torch_binding.cpp:6-33 slot_select_attend, slot_update,
 * slot_diffusion and their _backward ops; src/murmurative/ops.py:219-327),
 * general CUDA-core kernels with everything the fused call leaves out: a
 * selection mask, a position bias, effective (dynamic) M, separate token keys
 * and values, any head_dim that is a multiple of 8 up to 128, and M up to
 * 1024 (M x head_dim x 4 bytes at most 200 KiB). Slot sums are deterministic
 * (slot-major: each slot's entries in four fixed contiguous parts, each summed
 * in token order, the parts added in order). Conventions as above; grads are written in the
 * tensors' dtype, weights fp32, indices int64 [B,H,N,7] contiguous.
 * ------------------------------------------------------------------------ */
typedef struct murm_phase_shape {
  int32_t batch, heads, tokens, slots, head_dim;
  int32_t dtype; /* murm_dtype of every non-index, non-weight tensor */
} murm_phase_shape;

/* Replaces slot_select_attend (torch_binding.cpp:8, cuda_ops.h:6-19;
 * semantics reference.py:6-68): scores q.k (+ position_bias) with masked,
 * causal (slot m > token n) and tail (m >= effective_m) slots at -inf, top-7
 * (ties to the lowest slot), softmax of scale * q.k over the 7 picks (the mask
 * and bias do not enter the attend, reference.py:61-63), weighted sum of their
 * values. With `indices_in` set the selection is skipped and those indices are
 * attended (slot_attend, reference.py:42-68; out-of-range values clamped). */
typedef struct murm_select_attend_args {
  murm_phase_shape shape;
  int32_t causal;
  int32_t effective_m;         /* <= 0 or >= M: every slot */
  double scale;                /* <= 0: 1/sqrt(head_dim) */
  const void* q; int64_t q_stride[3];
  const void* slot_keys; int64_t sk_stride[3];
  const void* slot_values; int64_t sv_stride[3];
  const uint8_t* mask; int64_t mask_stride[4];     /* optional; 0 = masked; element strides b,h,n,m (0 broadcasts) */
  const void* position_bias; int64_t bias_stride[4]; /* optional, dtype of q */
  const int64_t* indices_in;   /* optional [B,H,N,7]: attend only */
  void* out; int64_t out_stride[3];
  int64_t* indices;            /* [B,H,N,7]; may equal indices_in */
  float* weights;              /* [B,H,N,7] */
} murm_select_attend_args;
MURM_API murm_status murm_select_attend_fwd(const murm_select_attend_args* args, void* stream);

/* Replaces slot_select_attend_backward (torch_binding.cpp:9): gradients of q,
 * slot_keys and slot_values from grad_out and (optional) grad_weights. The
 * slot gradients are per batch element ([B,H,M,d]) even when the forward
 * broadcast the slots. */
typedef struct murm_select_attend_bwd_args {
  murm_phase_shape shape;
  double scale;
  const void* q; int64_t q_stride[3];
  const void* slot_keys; int64_t sk_stride[3];
  const void* slot_values; int64_t sv_stride[3];
  const int64_t* indices; const float* weights;    /* the forward's outputs */
  const void* grad_out; int64_t go_stride[3];
  const float* grad_weights;                        /* optional [B,H,N,7] */
  void* grad_q; int64_t gq_stride[3];
  void* grad_slot_keys; int64_t gsk_stride[3];
  void* grad_slot_values; int64_t gsv_stride[3];
  void* workspace; size_t workspace_bytes;         /* murm_phase_sizes */
} murm_select_attend_bwd_args;
MURM_API murm_status murm_select_attend_bwd(const murm_select_attend_bwd_args* args, void* stream);

/* Replaces slot_update (torch_binding.cpp:15-18; reference.py:71-115): per
 * slot, the weight-summed token keys/values of the (token, pick) pairs that
 * chose it, divided by (weight sum + 1e-8); slots with a positive weight sum
 * take alpha * old + (1 - alpha) * mean, the others keep their value. `saved`
 * keeps the means and weight sums for the backward. */
typedef struct murm_slot_update_args {
  murm_phase_shape shape;
  double alpha;
  const void* token_keys; int64_t tk_stride[3];
  const void* token_values; int64_t tv_stride[3];
  const void* slot_keys; int64_t sk_stride[3];
  const void* slot_values; int64_t sv_stride[3];
  const int64_t* indices; const float* weights;
  void* new_slot_keys; int64_t nsk_stride[3];
  void* new_slot_values; int64_t nsv_stride[3];
  void* saved; size_t saved_bytes;                 /* murm_phase_sizes */
  void* workspace; size_t workspace_bytes;
} murm_slot_update_args;
MURM_API murm_status murm_slot_update_fwd(const murm_slot_update_args* args, void* stream);

/* Replaces slot_update_backward (torch_binding.cpp:19-21). */
typedef struct murm_slot_update_bwd_args {
  murm_phase_shape shape;
  double alpha;
  const void* token_keys; int64_t tk_stride[3];
  const void* token_values; int64_t tv_stride[3];
  const int64_t* indices; const float* weights;
  const void* saved; size_t saved_bytes;           /* the forward's */
  const void* grad_new_keys; int64_t gnk_stride[3];
  const void* grad_new_values; int64_t gnv_stride[3];
  void* grad_token_keys; int64_t gtk_stride[3];
  void* grad_token_values; int64_t gtv_stride[3];
  void* grad_slot_keys; int64_t gsk_stride[3];
  void* grad_slot_values; int64_t gsv_stride[3];
  float* grad_weights;                              /* [B,H,N,7] */
  void* workspace; size_t workspace_bytes;
} murm_slot_update_bwd_args;
MURM_API murm_status murm_slot_update_bwd(const murm_slot_update_bwd_args* args, void* stream);

/* The first half of slot_update alone: per slot, the weight-summed token keys
 * and values and the weight sum of the (token, pick) pairs that chose it
 * (reference.py:87-103), fp32, contiguous [B,H,M,d] / [B,H,M,d] / [B,H,M]. Sums
 * over token shards add up, so sequence-parallel callers all-reduce these and
 * finish the EMA on the totals. No counterpart in the reference's op schemas. */
typedef struct murm_slot_sums_args {
  murm_phase_shape shape;
  const void* token_keys; int64_t tk_stride[3];
  const void* token_values; int64_t tv_stride[3];
  const int64_t* indices; const float* weights;
  float* key_sums; float* value_sums; float* weight_sums;
  void* workspace; size_t workspace_bytes;
} murm_slot_sums_args;
MURM_API murm_status murm_slot_sums_fwd(const murm_slot_sums_args* args, void* stream);

/* Backward of murm_slot_sums_fwd: token-key/value and weight gradients from the
 * sums' gradients (fp32 contiguous, like the forward's outputs). */
typedef struct murm_slot_sums_bwd_args {
  murm_phase_shape shape;
  const void* token_keys; int64_t tk_stride[3];
  const void* token_values; int64_t tv_stride[3];
  const int64_t* indices; const float* weights;
  const float* grad_key_sums; const float* grad_value_sums; const float* grad_weight_sums;
  void* grad_token_keys; int64_t gtk_stride[3];
  void* grad_token_values; int64_t gtv_stride[3];
  float* grad_weights;
} murm_slot_sums_bwd_args;
MURM_API murm_status murm_slot_sums_bwd(const murm_slot_sums_bwd_args* args, void* stream);

/* Replaces slot_diffusion and its backward (torch_binding.cpp:22-27;
 * reference.py:118-135): out[m] = x[m] + gamma (x[m-1] + x[m+1] - 2 x[m]) on
 * the interior slots, boundaries unchanged; the backward applies the
 * transposed stencil to the output gradients. Keys and values alike; `tokens`
 * of the shape is ignored. */
typedef struct murm_slot_diffusion_args {
  murm_phase_shape shape;
  double gamma;
  const void* in_keys; int64_t ik_stride[3];
  const void* in_values; int64_t iv_stride[3];
  void* out_keys; int64_t ok_stride[3];
  void* out_values; int64_t ov_stride[3];
} murm_slot_diffusion_args;
MURM_API murm_status murm_slot_diffusion_fwd(const murm_slot_diffusion_args* args, void* stream);
MURM_API murm_status murm_slot_diffusion_bwd(const murm_slot_diffusion_args* args, void* stream);

/* Streaming decode step (the reference's decode plan,
 * docs/murmurative-attention-kernel-plan.md:154-173; no counterpart in its code):
 * one new token per (batch, head) against a resident slot pool that is updated
 * in place. Select (top-7 of q . slot_keys, slots above the token's absolute
 * position masked when causal), attend (softmax of scale * q.k over the picks),
 * out = x + attend, then update the picked slots with the token's key/value
 * (reference.py:71-115 with one token) and diffuse the whole pool
 * (reference.py:118-135). O(M * head_dim) per token and head; one launch.
 * Slots live in the pool's dtype between steps (as type_as does in the
 * reference). M * (head_dim + 1) * 8 bytes must fit in 200 KiB. */
typedef struct murm_decode_args {
  int32_t batch, heads, slots, head_dim, dtype;
  int32_t causal;
  const int64_t* positions;                  /* [batch] absolute positions; required when causal */
  double alpha, gamma, scale;                /* scale <= 0: 1/sqrt(head_dim) */
  const void* q; int64_t q_stride[2];        /* [B, H, d], strides {batch, head} */
  const void* k; int64_t k_stride[2];
  const void* v; int64_t v_stride[2];
  const void* x; int64_t x_stride[2];        /* optional residual; NULL = 0 */
  void* out; int64_t out_stride[2];
  void* slot_keys; int64_t sk_stride[3];     /* pool [B, H, M, d], read and written */
  void* slot_values; int64_t sv_stride[3];
  int64_t* indices; float* weights;          /* [B, H, 7], optional */
} murm_decode_args;
MURM_API murm_status murm_decode_step(const murm_decode_args* args, void* stream);

/* Byte sizes of slot_update's saved block and of the workspace every
 * per-phase call above takes (one size fits all of them). */
MURM_API murm_status murm_phase_sizes(const murm_phase_shape* shape, size_t* update_saved_bytes,
                                      size_t* workspace_bytes);

/* Launch accounting and per-kernel timing (host-side instrumentation; no
 * effect on results). murm_kernel_launches() counts every kernel this library
 * has launched in the process. Between murm_profile_begin() and
 * murm_profile_end() every launch is bracketed by CUDA events recorded on the
 * launch's own stream; murm_profile_end() waits for them and returns, per
 * kernel name, the launch count and summed device time. */
typedef struct murm_kernel_time {
  char name[48];
  int64_t launches;
  double total_ms;
} murm_kernel_time;

MURM_API uint64_t murm_kernel_launches(void);
MURM_API murm_status murm_profile_begin(void);
MURM_API murm_status murm_profile_end(murm_kernel_time* out, int32_t capacity, int32_t* count);

/* Synchronises `stream`, then reads and clears this device's error word, which
 * tensor-core kernels set when a bounded wait gives up (a copy or an MMA that
 * never completed, or, bit 32, another CTA of the forward's one-launch round
 * loop that never finished its part of a round) before they wind down cleanly.
 * Returns MURM_ERR_DEVICE when it was set. */
MURM_API murm_status murm_device_status(void* stream);

/* Failure-detection probe: launches one block that waits, bounded by limit_ns
 * (at most 10 s), on an mbarrier of its own with the same bounded wait the
 * tensor-core kernels use for their copies and MMAs. With `arrive` nonzero a
 * thread arrives first and the wait completes; with 0 nothing arrives, the
 * wait runs out, and the kernel sets the device error word (bit 16) and
 * returns normally, so murm_device_status then reports MURM_ERR_DEVICE and the
 * context stays usable. Lets a caller check its error handling without a
 * fault. No counterpart in the reference (its launchers never check device
 * errors, slot_select_attend.cu:474-490). */
MURM_API murm_status murm_wait_probe(int32_t arrive, uint64_t limit_ns, void* stream);

MURM_API const char* murm_status_string(murm_status status);
MURM_API const char* murm_last_error_message(void);
MURM_API int32_t murm_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MURM_H_ */
