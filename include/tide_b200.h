/*
 * tide_b200.h -- C ABI of the B200 (sm_100a) early-exit hot path.
 *
 * Everything here takes plain device pointers, sizes and a CUDA stream
 * handle; no framework types cross this boundary.  Every call enqueues work
 * on `stream` (NULL = legacy default stream) and returns without waiting.
 * Return value: TIDE_OK (0) or a TIDE_ERR_* code; tide_last_error() gives a
 * message for the calling thread.  Faults the kernels detect on the device
 * (an exit position outside the output buffer, a look-back wait that ran out)
 * are reported through the optional `error_word` (device int32, bit mask of
 * TIDE_DEVERR_*): the affected write is skipped, the kernel returns, and the
 * word is read back by the caller at its next synchronisation point.
 *
 * Reference interfaces replaced (RightNow-AI/TIDE v0.2.1):
 *   tide_fused_layernorm_route  <- torch.ops.tide.fused_layernorm_route
 *                                  csrc/extensions/torch_bindings.cpp:77-134,298-299
 *   tide_batch_compact          <- torch.ops.tide.batch_compact
 *                                  csrc/extensions/torch_bindings.cpp:136-198,300
 *   tide_exit_scatter           <- torch.ops.tide.exit_scatter
 *                                  csrc/extensions/torch_bindings.cpp:200-243,301-302
 *   tide_exit_projection        <- torch.ops.tide.exit_projection
 *                                  csrc/extensions/torch_bindings.cpp:245-293,303-304
 *   tide_checkpoint             <- one checkpoint of TIDERuntime.forward:
 *                                  python/TIDE/runtime.py:168-180 (score, strict
 *                                  '>' threshold, normed exit scatter) with the
 *                                  compaction of SkipScheduler.process_exits,
 *                                  python/TIDE/scheduler.py:63-102
 *   tide_norm_scatter           <- final norm + scatter of the rows that never
 *                                  exit: python/TIDE/runtime.py:183-187,
 *                                  python/TIDE/scheduler.py:111-116
 *   tide_router_fold            <- the per-call weight casts/transposes of
 *                                  torch_bindings.cpp:101-103 and the
 *                                  pre-transpose of runtime.py:85-87, done once
 */
#ifndef TIDE_B200_H
#define TIDE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *tide_stream_t; /* a cudaStream_t */

enum tide_dtype { TIDE_DTYPE_F32 = 0, TIDE_DTYPE_F16 = 1, TIDE_DTYPE_BF16 = 2 };
enum tide_norm { TIDE_NORM_RMS = 0, TIDE_NORM_LAYER = 1 };
/* TIDE_PATH_TC: the single-pass fused cluster kernel (bf16/fp16, router width
 * 128, hidden size with a resident weight slice); TIDE_PATH_TC_SPLIT: the
 * tensor-core router followed by the stable-partition kernel; TIDE_PATH_SIMT:
 * fp32 SIMT router + partition (any dtype and shape). */
enum tide_path { TIDE_PATH_AUTO = 0, TIDE_PATH_SIMT = 1, TIDE_PATH_TC = 2, TIDE_PATH_TC_SPLIT = 3 };

enum tide_status {
  TIDE_OK = 0,
  TIDE_ERR_INVALID = 1,     /* bad argument (null pointer, size, dtype)   */
  TIDE_ERR_UNSUPPORTED = 2, /* valid but not handled by the chosen path    */
  TIDE_ERR_CUDA = 3,        /* a CUDA runtime call failed                  */
  TIDE_ERR_WORKSPACE = 4,   /* workspace missing, too small or misaligned  */
  TIDE_ERR_ALIGNMENT = 5    /* pointer/stride not 16-byte aligned          */
};

/* device-side error bits written to error_word */
enum tide_device_error {
  TIDE_DEVERR_POSITION = 1, /* exit position outside [0, n_total): row skipped */
  TIDE_DEVERR_TIMEOUT = 2,  /* a bounded spin wait expired; results invalid  */
  TIDE_DEVERR_COUNT = 4     /* device row count above the row capacity       */
};

int tide_abi_version(void);
const char *tide_last_error(void);

/* ---- reference operator set ------------------------------------------- */

/* scores[i] = sigmoid(up . SiLU(down_t^T . (RMSNorm(input[i]) * norm_weight)))
 * input [n_tokens, hidden_dim] of `dtype`; norm_weight [hidden_dim] fp32;
 * down_weight_t [hidden_dim, bottleneck_dim] fp32 (the pre-transposed layout
 * of runtime.py:85-87); up_weight_t [bottleneck_dim] fp32; scores [n] fp32.
 * bottleneck_dim <= 256, as in fused_layernorm_route.cu:104-168. */
int tide_fused_layernorm_route(int dtype, const void *input, const float *norm_weight,
                               const float *down_weight_t, const float *up_weight_t,
                               float eps, float *scores, int64_t n_tokens,
                               int64_t hidden_dim, int64_t bottleneck_dim,
                               tide_stream_t stream);

/* Stable split of rows by exit_mask (non-zero = exit).  Rows with mask 0 go
 * to compacted[0..num_remaining) with their source index in
 * continue_indices; rows with mask != 0 go to exited[0..n-num_remaining)
 * with their index in exit_indices.  Both orders are ascending source order.
 * compacted/exited have room for n_tokens rows.  num_remaining: device int32. */
size_t tide_batch_compact_workspace_size(int64_t n_tokens);
int tide_batch_compact(int dtype, const void *input, const int32_t *exit_mask,
                       void *compacted, void *exited, int32_t *continue_indices,
                       int32_t *exit_indices, int32_t *num_remaining, int64_t n_tokens,
                       int64_t hidden_dim, void *workspace, size_t workspace_bytes,
                       int32_t *error_word, tide_stream_t stream);

/* tide_batch_compact for callers that cannot allocate device memory: the
 * same split, outputs and argument meaning, but no workspace argument.  For
 * hosts that only lend the library the tensors they pass in (an FFI host
 * whose GPU memory belongs to another runtime, code running where allocation
 * is forbidden).  It has no counterpart in the reference.
 * Its look-back scratch is a file-scope device array sized for at most
 * TIDE_NOALLOC_MAX_ROWS rows (65,792 bytes, held by every GPU that loads the
 * library until exit); larger n_tokens is rejected with TIDE_ERR_INVALID.  It
 * calls no allocator.  The first call on a device looks the array's address
 * up (make it before any stream capture) and keeps it for the life of the
 * process: after a cudaDeviceReset (or anything else that destroys and
 * recreates the device's primary context) the kept address is stale, so do
 * not call this entry point on that device again in the same process.  All
 * calls on a device share the array: calls whose kernels overlap on the GPU
 * race, so serialise them. */
#define TIDE_NOALLOC_MAX_ROWS 1048576
int tide_batch_compact_noalloc(int dtype, const void *input, const int32_t *exit_mask,
                               void *compacted, void *exited, int32_t *continue_indices,
                               int32_t *exit_indices, int32_t *num_remaining, int64_t n_tokens,
                               int64_t hidden_dim, int32_t *error_word, tide_stream_t stream);

/* output_buffer[exit_positions[i]] = exited_states[i]  (bit copy) */
int tide_exit_scatter(int dtype, const void *exited_states, const int32_t *exit_positions,
                      void *output_buffer, int64_t n_exited, int64_t hidden_dim,
                      int64_t n_total, int32_t *error_word, tide_stream_t stream);

/* output_buffer[exit_positions[i]] = RMSNorm(exited_states[i]) * norm_weight,
 * computed in fp32 and rounded to `dtype`. */
int tide_exit_projection(int dtype, const void *exited_states, const float *norm_weight,
                         const int32_t *exit_positions, void *output_buffer, float eps,
                         int64_t n_exited, int64_t hidden_dim, int64_t n_total,
                         int32_t *error_word, tide_stream_t stream);

/* output_buffer[positions[i]] = final_norm(rows[i]) rounded to `dtype`, the
 * final norm being RMSNorm (norm_bias ignored) or LayerNorm (norm_bias may be
 * NULL), statistics in fp32.  The remaining-token step of TIDERuntime.forward,
 * python/TIDE/runtime.py:183-187, and SkipScheduler.finalize,
 * python/TIDE/scheduler.py:111-116. */
int tide_norm_scatter(int dtype, int norm_type, const void *rows, const int64_t *positions,
                      void *output_buffer, const float *norm_weight, const float *norm_bias,
                      float eps, int64_t n_rows, int64_t hidden_dim, int64_t n_total,
                      int32_t *error_word, tide_stream_t stream);

/* Rows of a full tensor picked through an index, for a live row count kept
 * on the device (checkpoint k-1's counts_out), so that checkpoints chain
 * without a host read-back.  i runs over [0, *n_rows_dev) (clamped to
 * n_rows; [0, n_rows) when n_rows_dev is NULL); an index outside [0, n_src)
 * skips the row and sets TIDE_DEVERR_POSITION.
 * tide_gather_rows:       dst[i] = src[index[i]], src [n_src, H]: the still-
 *                         active rows of a later layer's hidden states, the
 *                         `hidden[~exited]` of python/TIDE/runtime.py:172-174
 *                         (and of scheduler.py:98 in the live loop).
 * tide_norm_at_positions: out[positions[i]] = final_norm(src[positions[i]]),
 *                         src and out [n_total, H]: the rows that never exit,
 *                         python/TIDE/runtime.py:183-187. */
int tide_gather_rows(int dtype, const void *src, int64_t n_src, const int64_t *index,
                     const int32_t *n_rows_dev, int64_t n_rows, int64_t hidden_dim, void *dst,
                     int32_t *error_word, tide_stream_t stream);
int tide_norm_at_positions(int dtype, int norm_type, const void *src, const int64_t *positions,
                           const int32_t *n_rows_dev, int64_t n_rows, int64_t hidden_dim,
                           int64_t n_total, void *output_buffer, const float *norm_weight,
                           const float *norm_bias, float eps, int32_t *error_word,
                           tide_stream_t stream);

/* Decode attention over a KV cache addressed by slot: for each of the n_rows
 * rows still active in a decode step (their slot ids as compacted by
 * tide_checkpoint's slots_out),
 *   out[i, h] = softmax_j(scale * q[i, h] . K[slots[i], h/G, j]) . V[slots[i], h/G, j],
 *   j in [0, length), G = n_q_heads / n_kv_heads (at most 8), head_dim 128.
 * q, out [n_rows, n_q_heads, 128]; K, V caches [n_slots, n_kv_heads, max_len, 128],
 * bf16 or fp16.  Positions a sequence skipped hold zeros and count like any
 * other (the "zero_pad" K/V policy of python/TIDE/runtime.py:194-221).  It
 * replaces, for the rows that have not exited, the attention of the HF model
 * call inside the reference's decode loop (runtime.py:266-273).  A slot
 * outside [0, n_slots) skips its row and sets TIDE_DEVERR_POSITION.
 * n_rows_dev (optional, device int32): only rows below it are computed (the
 * live count a checkpoint wrote).  length_dev (optional, device int32): the
 * length is read from the device, clamped to [1, length]; `length` then only
 * bounds it (shared memory is sized for it).  Both keep a decode step free of
 * host values, so it can be captured in a CUDA graph. */
int tide_decode_attention(int dtype, const void *q, const void *k_cache, const void *v_cache,
                          const int32_t *slots, void *out, int64_t n_rows,
                          const int32_t *n_rows_dev, int64_t n_q_heads, int64_t n_kv_heads,
                          int64_t head_dim, int64_t n_slots, int64_t max_len, int64_t length,
                          const int32_t *length_dev, float scale, int32_t *error_word,
                          tide_stream_t stream);

/* Append one decode position to a KV cache addressed by slot:
 *   K[slots[i], h, pos, :] = k_new[i, h, :],  V[...] = v_new[i, h, :]
 * for i below the live row count (*n_rows_dev clamped to [0, n_rows]; n_rows
 * when NULL) and pos = *position_dev when given, else `position`.  k_new,
 * v_new [n_rows, n_kv_heads, 128]; caches as tide_decode_attention's.  A
 * position outside [0, max_len) or a slot outside [0, n_slots) writes
 * nothing for the rows concerned and sets TIDE_DEVERR_POSITION.  With the
 * checkpoint's compacted slot ids it stores the keys and values of the rows
 * still active in a decode step; an exited row's entry at that position
 * keeps the zeros it was created with (the reference's "zero_pad",
 * python/TIDE/runtime.py:194-221). */
int tide_kv_append(int dtype, const void *k_new, const void *v_new, const int32_t *slots,
                   const int32_t *n_rows_dev, int64_t n_rows, int64_t n_kv_heads,
                   int64_t head_dim, void *k_cache, void *v_cache, int64_t n_slots,
                   int64_t max_len, int64_t position, const int32_t *position_dev,
                   int32_t *error_word, tide_stream_t stream);

/* tide_norm_scatter with the row count on the device:
 *   output_buffer[positions[i]] = final_norm(rows[i]),  i < *n_rows_dev
 * (clamped to [0, n_rows]; n_rows when NULL).  The finalize step
 * (python/TIDE/scheduler.py:102-120) for survivors whose count a checkpoint
 * left on the device.  A position outside [0, n_total) skips its row and
 * sets TIDE_DEVERR_POSITION. */
int tide_norm_scatter_rows(int dtype, int norm_type, const void *rows, const int64_t *positions,
                           const int32_t *n_rows_dev, int64_t n_rows, int64_t hidden_dim,
                           int64_t n_total, void *output_buffer, const float *norm_weight,
                           const float *norm_bias, float eps, int32_t *error_word,
                           tide_stream_t stream);

/* The elementwise work of a Llama-family decode layer for the live decoder,
 * each rounding where the HF module it replaces rounds (bf16 or fp16 rows,
 * weights in the rows' type), rows below the live count only (*n_rows_dev
 * clamped to [0, n_rows]; n_rows when NULL):
 * tide_rms_norm:      s = x, or s = to_T(x + delta) written to sum_out (when
 *                     given); out = to_T(w * to_T(s * rsqrt(mean(s^2) + eps)))
 *                     -- HF LlamaRMSNorm / Qwen3RMSNorm with an optional fused
 *                     residual add.  hidden_dim % 8 == 0, <= 8192.
 * tide_qk_norm_rope:  q [n, hq, 128], k, v [n, hkv, 128], rows q_row_stride
 *                     and kv_row_stride elements apart (0: packed; k and v
 *                     share a stride, so q, k and v may be column slices of
 *                     one fused projection's output): optional per-head
 *                     RMSNorm of q and k (Qwen3 q_norm / k_norm; NULL weight =
 *                     none), the rotary embedding q*cos + rotate_half(q)*sin
 *                     with cos/sin = to_T(cos/sin(pos * inv_freq[j]) *
 *                     attention_scaling), then q to q_out and k, v into the
 *                     slot-addressed caches at pos (*position_dev when given).
 *                     rope_positions (optional, int64 per row): each row's own
 *                     rotary position instead of pos, and q written to
 *                     q_out[slots[i]] instead of q_out[i] (a prefill, which
 *                     passes [tokens, heads, 1, 128] buffers as the caches,
 *                     its rows' token indices as the slots and pos 0, so
 *                     that q, k and v land at their tokens' places).  A slot
 *                     or position outside the cache writes nothing for that
 *                     row and sets TIDE_DEVERR_POSITION.
 * tide_silu_mul:      out = to_T(to_T(silu(gate)) * up), [n, width], width % 8
 *                     == 0 -- the gated MLP's act_fn(gate_proj(x)) * up_proj(x).
 * The reference runs the model's own modules for these inside its decode
 * loop (python/TIDE/runtime.py:266-273). */
int tide_rms_norm(int dtype, const void *x, const void *delta, void *sum_out, const void *weight,
                  void *out, int64_t n_rows, const int32_t *n_rows_dev, int64_t hidden_dim,
                  float eps, tide_stream_t stream);
int tide_qk_norm_rope(int dtype, const void *q, const void *k, const void *v,
                      int64_t q_row_stride, int64_t kv_row_stride,
                      const void *q_norm_weight, const void *k_norm_weight, float eps,
                      const float *inv_freq, float attention_scaling, int64_t position,
                      const int32_t *position_dev, const int64_t *rope_positions,
                      const int32_t *slots, const int32_t *n_rows_dev, int64_t n_rows,
                      int64_t n_q_heads,
                      int64_t n_kv_heads, int64_t head_dim, void *q_out, void *k_cache,
                      void *v_cache, int64_t n_slots, int64_t max_len, int32_t *error_word,
                      tide_stream_t stream);
int tide_silu_mul(int dtype, const void *gate, const void *up, void *out, int64_t n_rows,
                  const int32_t *n_rows_dev, int64_t width, tide_stream_t stream);

/* ---- router preparation (once per router) ------------------------------ */

/* From the router's down.weight [B, H] fp32 and the final norm's weight (and
 * bias, LayerNorm only) [H] fp32, build:
 *   down_t      [H, B] fp32             (SIMT path; may be NULL)
 *   folded      [B, H] in fold_dtype    folded[b,i] = down[b,i] * norm_weight[i]
 *                                       (tensor-core path; may be NULL)
 *   colsum      [B] fp32                sum_i float(folded[b,i])   (may be NULL)
 *   bias_proj   [B] fp32                sum_i norm_bias[i]*down[b,i] (may be NULL) */
int tide_router_fold(int fold_dtype, const float *down, const float *norm_weight,
                     const float *norm_bias, int64_t hidden_dim, int64_t bottleneck_dim,
                     float *down_t, void *folded, float *colsum, float *bias_proj,
                     tide_stream_t stream);

/* ---- one checkpoint of the early-exit path ----------------------------- */

typedef struct tide_checkpoint_args {
  int32_t dtype;          /* element type of x, out_buffer, compact_out        */
  int32_t norm_type;      /* TIDE_NORM_RMS or TIDE_NORM_LAYER                  */
  int32_t path;           /* TIDE_PATH_AUTO / _SIMT / _TC                        */
  int32_t reserved0;
  int64_t n_rows;         /* rows of x (capacity when n_rows_dev != NULL)      */
  int64_t hidden_dim;     /* H                                                   */
  int64_t bottleneck_dim; /* B (router width)                                    */
  int64_t n_total;        /* rows of out_buffer                                  */
  const void *x;          /* [n_rows, H] hidden states of the active tokens     */
  const int32_t *n_rows_dev; /* optional device count of valid rows (<= n_rows) */
  /* final norm */
  const float *norm_weight; /* [H] fp32                                          */
  const float *norm_bias;   /* [H] fp32, LayerNorm only, may be NULL             */
  float eps;
  /* router (from tide_router_fold) */
  float up_bias;          /* scalar added before the sigmoid (0 = reference)   */
  const float *down_t;    /* [H, B] fp32: SIMT path                            */
  const void *folded;     /* [B, H] dtype: tensor-core path                    */
  const float *colsum;    /* [B]: LayerNorm on the tensor-core path            */
  const float *bias_proj; /* [B]: LayerNorm with bias                          */
  const float *up;        /* [B] fp32 up.weight                                */
  float threshold;        /* exit iff score > threshold (strict)               */
  int32_t reserved1;
  /* token bookkeeping */
  const int64_t *positions_in; /* [n_rows] original token position; NULL = row index */
  const int32_t *slots_in;     /* [n_rows] KV slot id; may be NULL                  */
  /* outputs (each may be NULL except counts_out) */
  void *out_buffer;            /* [n_total, H]: exiting rows, final-normed       */
  void *compact_out;           /* [n_rows, H]: surviving rows, stable order      */
  int64_t *positions_out;      /* [n_rows]: surviving rows' positions            */
  int32_t *slots_out;          /* [n_rows]: surviving rows' slots                */
  int64_t *exit_positions_out; /* [n_rows]: exiting rows' positions, stable      */
  float *scores_out;           /* [n_rows]: router scores                        */
  int32_t *counts_out;         /* [2] device: {survivors, exits}                 */
  int32_t *error_word;         /* device int32 bit mask, may be NULL             */
  void *workspace;             /* from tide_checkpoint_workspace_size            */
  size_t workspace_bytes;
} tide_checkpoint_args;

size_t tide_checkpoint_workspace_size(const tide_checkpoint_args *args);
int tide_checkpoint(const tide_checkpoint_args *args, tide_stream_t stream);

/* Which path tide_checkpoint would take for these arguments (TIDE_PATH_SIMT,
 * TIDE_PATH_TC or TIDE_PATH_TC_SPLIT), or a negative TIDE_ERR_* code. */
int tide_checkpoint_select_path(const tide_checkpoint_args *args);

#ifdef __cplusplus
}
#endif

#endif /* TIDE_B200_H */
