/*
 * fa8.h — C ABI of the B200 (sm_100a) FP8 flash-attention forward.
 *
 * Plain C: pointers, sizes and status codes only. No torch or CUDA types
 * appear in any signature (streams are passed as `void*` holding a
 * cudaStream_t). Every entry point returns an fa8_status and never exits
 * the process or synchronises the device.
 *
 * Reference interface replaced (Lemon7-UP/ada_cute_fp8_flash_attention):
 *   fa8_fwd        <- flash_attn_fp8_forward(q, k, v)
 *                     csrc/flash_attention.cu:508-543 (host forward),
 *                     csrc/flash_attention.cu:462-485 (fill_params),
 *                     csrc/flash_attention.cu:487-506 (launcher),
 *                     csrc/flash.h:11-26 (Flash_fwd_params),
 *                     bound at csrc/attention_api.cpp:6-9.
 *   fa8_bwd        <- no counterpart in the reference (forward only); the
 *                     gradient of the same attention for training callers.
 *   fa8_lse_merge  <- no counterpart in the reference (which emits no LSE);
 *                     merges partial outputs of the context-parallel ring.
 *   fa8_quantize_e4m3 <- the torch casts that prepare the kernel inputs in
 *                     test.py:35-37 and the V transpose at test.py:51-52.
 */
#ifndef FA8_H_
#define FA8_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fa8_status {
  FA8_OK = 0,
  FA8_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad layout code  */
  FA8_ERR_UNSUPPORTED = 2,   /* head_dim not 64/128, heads % heads_kv != 0    */
  FA8_ERR_ALIGNMENT = 3,     /* TMA needs 16-byte aligned bases and strides   */
  FA8_ERR_CUDA = 4,          /* a CUDA runtime call failed (see message)      */
  FA8_ERR_DRIVER = 5,        /* driver entry point for tensor maps missing    */
  FA8_ERR_NO_DEVICE = 6      /* current device is not sm_100                  */
} fa8_status;

/* Layout of V. The reference takes V pre-transposed to (B, H_kv, D, S_kv)
 * (test.py:51-52, csrc/flash_attention.cu:145-148). */
enum { FA8_V_BHDS = 0, FA8_V_BHSD = 1 };

/* Output element type. fp16 is the north-star contract; e4m3 reproduces the
 * reference's `empty_like(q)` output (csrc/flash_attention.cu:526); fp32
 * keeps partial outputs unrounded for a later log-sum-exp merge (context
 * parallel). */
enum { FA8_OUT_F16 = 0, FA8_OUT_E4M3 = 1, FA8_OUT_F32 = 2 };

/* Bits the kernel ORs into *status (an optional device word) instead of
 * faulting or hanging: a bounded wait gave up (TIMEOUT), a varlen sequence
 * whose K/V start is not a multiple of 16 (VARLEN_ALIGN), or a varlen
 * sequence whose offsets leave the packed tensors or that is longer than
 * max_seqlen_q (VARLEN_RANGE). A refused sequence is left unwritten. */
enum { FA8_DEVERR_TIMEOUT = 1, FA8_DEVERR_VARLEN_ALIGN = 2, FA8_DEVERR_VARLEN_RANGE = 4 };

/*
 * All strides are in ELEMENTS. Tensors are indexed [b][h][s][d] for Q, K and
 * O, [b][h][d][s] for V in FA8_V_BHDS layout (the reference's pre-transposed
 * V) and [b][h][s][d] in FA8_V_BHSD layout (read in place: the PV product
 * takes the V tile as an MN-major operand). The innermost dimension (d for
 * Q/K/O/V-BHSD, s for V-BHDS) must have unit stride. Q/K/V are e4m3 (1 byte),
 * O is fp16, e4m3 or fp32, LSE is fp32 [b][h][s] (natural log), optional.
 */
typedef struct fa8_fwd_params {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;               /* may be NULL */
  int32_t* status;          /* optional device word; kernel ORs FA8_DEVERR_* */

  int64_t batch;
  int64_t heads;            /* query heads                                  */
  int64_t heads_kv;         /* key/value heads, divides heads (GQA)         */
  int64_t seqlen_q;
  int64_t seqlen_kv;
  int64_t head_dim;         /* 64 or 128                                    */

  int64_t q_stride_b, q_stride_h, q_stride_s;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  int64_t v_stride_b, v_stride_h, v_stride_r;  /* r = d (BHDS) or s (BHSD)  */
  int64_t o_stride_b, o_stride_h, o_stride_s;
  int64_t lse_stride_b, lse_stride_h;          /* s stride is 1             */

  float softmax_scale;      /* natural-log scale, usually 1/sqrt(head_dim)  */
  int32_t causal;           /* mask key_pos > query_pos                     */
  int32_t v_layout;         /* FA8_V_BHDS or FA8_V_BHSD                     */
  int32_t out_dtype;        /* FA8_OUT_F16, FA8_OUT_E4M3 or FA8_OUT_F32     */

  /* Global positions of row 0 of this Q block and of this K/V block. Only
   * the causal mask reads them (context-parallel chunks); 0 otherwise. */
  int64_t q_offset;
  int64_t kv_offset;

  /* P is requantised to e4m3 as hi + lo (two PV products) for query tiles
   * whose first row sees fewer than this many keys; -1 selects the default
   * (1024), 0 disables the split. */
  int32_t split_keys;
  /* SM budget: > 0 runs the kernel on at most this many SMs (rounded up to a
   * multiple of 8) through a green-context stream that the library creates
   * once per device and count, ordered after `stream` and before its later
   * work; it leaves the other SMs to concurrent kernels (e.g. the NCCL
   * transfers of a context-parallel exchange). 0 = the whole GPU. */
  int32_t sm_budget;

  /* Per-tensor dequantisation factors of e4m3 Q, K, V (real value = code x
   * factor); 1.0 = unscaled inputs. The kernel folds descale_q * descale_k
   * into the softmax scale and multiplies O by descale_v. */
  float descale_q;
  float descale_k;
  float descale_v;
  int32_t reserved0;

  /* Variable-length batches (optional). When cu_seqlens_q is non-NULL, Q/O
   * and K/V hold `batch` sequences packed along the sequence dimension: Q is
   * [total_q][heads][head_dim] (seqlen_q = total_q, q_stride_s = heads * D,
   * q_stride_h = D), K likewise, V^T is [heads_kv][D][total_kv]; sequence b
   * occupies rows cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 (device int32
   * prefix sums with batch + 1 entries, same for cu_seqlens_kv). LSE is
   * [heads][total_q]. Every cu_seqlens_kv[b] must be a multiple of 16 (V^T
   * tiles start on 16-byte boundaries). The offsets are read only on the
   * device (no host copy, no synchronisation): a sequence that breaks the
   * alignment rule, leaves the packed tensors or is longer than max_seqlen_q
   * (which sizes the grid) is left unwritten and FA8_DEVERR_VARLEN_ALIGN /
   * FA8_DEVERR_VARLEN_RANGE is ORed into *status. */
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_kv;
  int64_t max_seqlen_q;

  /* Failure detection. Every barrier wait inside the kernel gives up after
   * wait_timeout_cycles SM clocks (0 = default, about two seconds); the CTA
   * then ORs FA8_DEVERR_TIMEOUT into *status, frees its resources and exits,
   * leaving the context usable. debug_skip_kv_loads (tests only) makes the
   * kernel issue no K/V loads so that the waits run out. */
  int64_t wait_timeout_cycles;
  int32_t debug_skip_kv_loads;
  int32_t reserved1;

  /* Per-(batch, head) dequantisation factors (optional device float arrays,
   * NULL = 1), applied on top of the per-tensor factors: query head h of
   * batch b uses descale_q_bh[b * descale_q_stride_b + h * descale_q_stride_h];
   * K and V use their K/V head hk with the kv strides. A batch stride of 0
   * shares one row of factors across the batch. For varlen calls b is the
   * sequence index. */
  const float* descale_q_bh;
  const float* descale_k_bh;
  const float* descale_v_bh;
  int64_t descale_q_stride_b;
  int64_t descale_q_stride_h;
  int64_t descale_kv_stride_b;
  int64_t descale_kv_stride_h;

  /* Split-KV (no counterpart in the reference, which launches one CTA per
   * 64-row query block): when a call has fewer query tiles than the GPU has
   * SMs, each 128-row query tile's K/V range is cut into kv_splits shares run
   * by separate CTAs, and the last share to finish merges the partial
   * outputs by log-sum-exp inside the same launch. kv_splits: 0 = automatic
   * (split only when the grid would not fill the GPU and `workspace` is large
   * enough, see fa8_fwd_workspace_size), 1 = never, n > 1 = up to n shares
   * (FA8_ERR_INVALID_ARG if the workspace is too small). workspace: device
   * memory, 256-byte aligned, of workspace_bytes bytes; its first
   * 256 * ceil(4 * query_tiles / 256) bytes are counters that must be zero
   * before the first call (the kernel leaves them zero; after a call that
   * reported FA8_DEVERR_TIMEOUT, zero them again). Not used for varlen calls. */
  void* workspace;
  int64_t workspace_bytes;
  int32_t kv_splits;
  int32_t reserved3;
} fa8_fwd_params;

/* Fill *p with defaults: contiguous strides for the given shape, scale
 * 1/sqrt(head_dim), non-causal, BHDS V, fp16 out, default split, unit
 * dequantisation factors. */
void fa8_fwd_params_init(fa8_fwd_params* p, int64_t batch, int64_t heads,
                         int64_t heads_kv, int64_t seqlen_q, int64_t seqlen_kv,
                         int64_t head_dim);

/* Launch the forward on `stream` (a cudaStream_t, NULL = legacy default).
 * Asynchronous; returns after the launch is queued. */
int fa8_fwd(const fa8_fwd_params* p, void* stream);

/* Workspace bytes fa8_fwd would use for split-KV with these parameters
 * (kv_splits 0 or n > 1); 0 when the call does not split. Host-only, no
 * device access. No counterpart in the reference. */
int64_t fa8_fwd_workspace_size(const fa8_fwd_params* p);

/*
 * The forward for callers that cannot allocate device memory (no counterpart
 * in the reference). Split-KV needs scratch that fa8_fwd takes from the
 * caller's `workspace`; code that runs inside a framework owning the memory
 * pool, plugins forbidden to call cudaMalloc, or launch paths that must not
 * allocate cannot provide one. This entry point ignores `workspace` /
 * `workspace_bytes` and uses a scratch array compiled into the library
 * (fa8_static_scratch_bytes() = 8 MiB, resident on every GPU that loads the
 * library until the process exits). It allocates nothing: it rejects a call
 * whose split plan needs more than that with FA8_ERR_INVALID_ARG (use
 * kv_splits = 1, or fa8_fwd with a workspace), and otherwise clears the split
 * counters with an asynchronous memset on `stream` and calls fa8_fwd. The
 * first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture. All calls
 * share the one array: calls whose kernels overlap on the GPU (other streams,
 * other threads) race on it and must be serialised by the caller.
 */
int fa8_fwd_static_scratch(const fa8_fwd_params* p, void* stream);
int64_t fa8_static_scratch_bytes(void);

/*
 * Log-sum-exp merge of `n_parts` partial attention outputs of the same rows:
 *   lse = log(sum_i exp(lse_i)), o = sum_i exp(lse_i - lse) * o_i.
 * o_parts: n_parts pointers to fp32 [rows][head_dim] or fp16 (o_is_f16);
 * lse_parts: n_parts pointers to fp32 [rows]. Parts with lse = -inf are
 * ignored. Writes o_out (fp16 [rows][head_dim], row stride o_out_stride) and
 * lse_out (fp32, may be NULL). All pointers are device pointers; the two
 * pointer arrays are host arrays of at most 16 entries. o_parts[i] and o_out
 * must be 16-byte aligned (FA8_ERR_ALIGNMENT otherwise).
 */
int fa8_lse_merge(int n_parts, const void* const* o_parts, int o_is_f16,
                  const float* const* lse_parts, int64_t rows,
                  int64_t head_dim, void* o_out, int64_t o_out_stride,
                  float* lse_out, void* stream);

/*
 * Quantise fp16 or bf16 x to e4m3 with round-to-nearest-even and saturation
 * to +-448, multiplying by `scale` first. x holds `batch` contiguous matrices
 * of rows x cols elements each (no row padding; the row stride is cols). If
 * `transpose` is set, y is written as batch contiguous matrices of cols x rows
 * — the V transpose to BHDS — else y has x's layout. in_dtype: 0 = fp16,
 * 1 = bf16. Without transpose the element count must be a multiple of 16 and
 * both buffers 16-byte aligned; with transpose, rows % 16 == 0, cols % 8 == 0
 * and 16-byte aligned buffers take the vectorised kernel, other shapes a
 * slower per-element one.
 */
int fa8_quantize_e4m3(const void* x, int in_dtype, void* y, int64_t batch,
                      int64_t rows, int64_t cols, float scale, int transpose,
                      void* stream);

/* Human-readable text for an fa8_status, plus the last CUDA error seen by
 * this thread when the status is FA8_ERR_CUDA. */
/*
 * Backward pass: gradients of O = softmax(scale * Q K^T [causal]) V with
 * respect to the e4m3 Q, K and V that fa8_fwd consumed. No counterpart in
 * the reference, which has no backward. Inputs: q, k (contiguous
 * [b][h][s][d] / [b][h_kv][s][d] e4m3), v (contiguous, v_layout), o and d_o
 * (contiguous fp16 [b][h][s_q][d], o as fa8_fwd wrote it), lse (contiguous
 * fp32 [b][h][s_q], natural log, as fa8_fwd wrote it). Outputs (fp32,
 * contiguous): dq [b][h][s_q][d], dk and dv [b][h_kv][s_kv][d] (GQA heads
 * summed). Causal masking is key <= query (no offsets). The caller provides
 * fa8_bwd_workspace_size() bytes of device workspace, 256-byte aligned.
 */
typedef struct fa8_bwd_params {
  int64_t batch, heads, heads_kv, seqlen_q, seqlen_kv, head_dim;
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* d_o;
  const float* lse;
  float* dq;
  float* dk;
  float* dv;
  int causal;             /* default 1                                    */
  float softmax_scale;    /* <= 0: 1/sqrt(head_dim)                       */
  int v_layout;           /* FA8_V_BHDS (default) or FA8_V_BHSD           */
  int* status;            /* optional device word, FA8_DEVERR_* bits      */
  long long timeout_cycles; /* bound of every wait; <= 0: ~2 s            */
} fa8_bwd_params;

void fa8_bwd_params_init(fa8_bwd_params* p, int64_t batch, int64_t heads, int64_t heads_kv,
                         int64_t seqlen_q, int64_t seqlen_kv, int64_t head_dim);
int64_t fa8_bwd_workspace_size(const fa8_bwd_params* p);
int fa8_bwd(const fa8_bwd_params* p, void* workspace, int64_t workspace_bytes, void* stream);

const char* fa8_status_string(int status);
const char* fa8_last_error_message(void);

/* Number of kernel launches fa8_* entry points issued from this process. */
uint64_t fa8_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* FA8_H_ */
