/*
 * sbda_b200.h -- C ABI of the B200 (sm_100a) SBDA sparse gather-softmax
 * attention kernels.
 *
 * SBDA (Staged Binary-Local Diffusion Attention) layer l lets query i attend
 * to at most four exact causal sources i - o, o in O_l, with
 * O_l = (0, 2^(l-1)) for l <= 2 and (0, 1, 2, 2^(l-1)) for l >= 3.
 * Sources with i - o < 0 are masked; scale = head_dim^-0.5.
 *
 * These entry points replace the device work of the reference autograd op
 * `fused_sbda_key_backward(q, k, v, offsets)` and of its native-GQA twin
 * `fused_sbda_gqa_key_backward` (BiAttn/sbda_triton.py:1467-1493):
 *
 *   sbda_b200_forward   <- _FusedSBDAKeyBackward.forward      (sbda_triton.py:1294-1327)
 *                          _FusedSBDAGQAKeyBackward.forward   (sbda_triton.py:1366-1400)
 *   sbda_b200_backward  <- _FusedSBDAKeyBackward.backward     (sbda_triton.py:1330-1360)
 *                          _FusedSBDAGQAKeyBackward.backward  (sbda_triton.py:1402-1434)
 *
 * The forward saves a fp32 log-sum-exp per query row instead of the
 * reference's per-source weight table W[B,H,L,S]; the backward recomputes
 * the weights from it.  Both are deterministic and use no atomics.
 *
 * Conventions
 *  - Every tensor is a [B, H, L, D] view described by its data pointer and
 *    four element strides (batch, head, position, channel).  q/out/grad_out/
 *    grad_q have H heads; k/v/grad_k/grad_v have kv_heads heads
 *    (H % kv_heads == 0; query head h reads kv head h / (H / kv_heads)).
 *  - lse is a contiguous fp32 [B, H, L] buffer owned by the caller.
 *  - offsets is a HOST array of n_offsets (1..4) distinct non-negative ints.
 *    At most one offset may exceed the tile height (64); that one is the
 *    "far" (dyadic) source, the rest are the "near" window.
 *  - No entry point allocates device memory, synchronises, or keeps state
 *    between calls.  Work is enqueued on `stream` (a cudaStream_t; NULL is
 *    the legacy default stream).
 *  - The attention kernels are launched with programmatic stream
 *    serialization and let the next kernel on the stream start early.  A
 *    kernel that the caller launches right after a call with that same launch
 *    attribute must wait on its grid dependency (cudaGridDependencySynchronize)
 *    before it reads the call's outputs; ordinary launches, copies and events
 *    see the call complete as usual.
 *  - Return value: SBDA_OK or an error code; sbda_b200_status_string() names it.
 */
#ifndef SBDA_B200_H_
#define SBDA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SBDA_B200_ABI_VERSION 2

/* Element types (match the reference's accepted dtypes, sbda_triton.py:1302-1303). */
enum sbda_dtype {
  SBDA_DTYPE_F32 = 0,
  SBDA_DTYPE_F16 = 1,
  SBDA_DTYPE_BF16 = 2
};

/* Status codes.  The Python wrapper maps them onto the reference's exception
 * types (sbda_triton.py:1295-1303): INVALID -> ValueError, DTYPE -> TypeError,
 * UNSUPPORTED / CUDA / DEVICE -> RuntimeError. */
enum sbda_status {
  SBDA_OK = 0,
  SBDA_ERR_INVALID = 1,      /* bad shape, stride, offsets or null pointer */
  SBDA_ERR_DTYPE = 2,        /* unsupported element type */
  SBDA_ERR_UNSUPPORTED = 3,  /* valid but outside the kernel's envelope (head_dim > 128, two far offsets) */
  SBDA_ERR_CUDA = 4,         /* a CUDA runtime / driver call failed */
  SBDA_ERR_DEVICE = 5        /* a kernel reported a device-side fault (bounded wait expired) */
};

/* A [B, H, L, D] view: element (0,0,0,0) and element strides. */
typedef struct sbda_tensor {
  void* data;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_l;
  int64_t stride_d;
} sbda_tensor;

/* Problem shape shared by forward and backward. */
typedef struct sbda_shape {
  int64_t batch;
  int64_t heads;     /* query heads H */
  int64_t kv_heads;  /* key/value heads; == heads for MHA */
  int64_t length;    /* sequence positions L */
  int64_t head_dim;  /* D, 1..128 */
} sbda_shape;

/* Library ABI version (SBDA_B200_ABI_VERSION). */
int sbda_b200_abi_version(void);

/* Human-readable name of a status code (static string). */
const char* sbda_b200_status_string(int status);

/*
 * Forward.  out[b,h,i,:] = sum_s p_s v[b,h/G,i-o_s,:] with
 * p = softmax_s(scale * <q[b,h,i,:], k[b,h/G,i-o_s,:]>) over valid sources,
 * lse[b,h,i] = log sum_s exp(score_s) (natural log; -inf if no source is valid).
 * out has q's dtype; math is fp32.
 */
int sbda_b200_forward(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                      float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                      sbda_tensor out, float* lse, void* stream);

/*
 * Backward (gather form).  Given the forward inputs, lse and grad_out, writes
 * grad_q, grad_k, grad_v (each exactly once, in the input dtype).  grad_k and
 * grad_v sum over the H / kv_heads query heads that share a kv head.
 */
int sbda_b200_backward(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                       float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                       sbda_tensor grad_out, const float* lse,
                       sbda_tensor grad_q, sbda_tensor grad_k, sbda_tensor grad_v,
                       void* stream);

/*
 * Backward for grouped-query attention (kv_heads < heads) on the windowed
 * kernels.  Replaces _FusedSBDAGQAKeyBackward.backward (sbda_triton.py:1402-1434),
 * which sums dK/dV over each group with atomics.  Here every query head writes
 * its dK/dV contributions as fp32 partials to `workspace` (at least
 * sbda_b200_backward_grouped_workspace_floats(shape) floats, 16-byte aligned),
 * and a second kernel sums the partials of each kv head in head order and
 * rounds once: deterministic.  Calls the windowed kernels do not serve (and MHA
 * calls) run sbda_b200_backward, which ignores the workspace.
 */
int64_t sbda_b200_backward_grouped_workspace_floats(sbda_shape shape);
int sbda_b200_backward_grouped(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                               float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                               sbda_tensor grad_out, const float* lse, sbda_tensor grad_q,
                               sbda_tensor grad_k, sbda_tensor grad_v, float* workspace,
                               int64_t workspace_floats, void* stream);

/*
 * Contiguous sequence shards (no counterpart in the reference, which runs
 * one sequence on one GPU).  Rank r of `world` (<= 8) holds
 * positions [r*L, (r+1)*L) of one sequence, L = shape.length, the same on
 * every rank and a multiple of the tile height (64 for 16-bit D <= 64).  The
 * far offset, if any, must also be a tile multiple, or shorter than a tile
 * where the windowed kernels serve the offsets (near offsets within {0,1,2},
 * heads == kv_heads; the default kernel path).  k_ranks[i] / v_ranks[i]
 * (and in the backward q, grad_out, lse) describe rank i's buffers as
 * addresses valid on this GPU (peer memory mapped into this process, e.g.
 * CUDA IPC or symmetric memory); the kernels stage remote rows over NVLink
 * with non-multicast TMA, per tile, from the rank that owns them.  All peers'
 * inputs must be complete before the call (a cross-rank barrier) and must not
 * be overwritten until every rank's call has finished.  Outputs are this
 * rank's rows only.  Same results as the single-GPU call on the whole
 * sequence.
 */
int sbda_b200_forward_sharded(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                              float scale, int32_t rank, int32_t world, sbda_tensor q,
                              const sbda_tensor* k_ranks, const sbda_tensor* v_ranks, sbda_tensor out,
                              float* lse, void* stream);

int sbda_b200_backward_sharded(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                               float scale, int32_t rank, int32_t world, const sbda_tensor* q_ranks,
                               const sbda_tensor* k_ranks, const sbda_tensor* v_ranks,
                               const sbda_tensor* grad_out_ranks, const float* const* lse_ranks,
                               sbda_tensor grad_q, sbda_tensor grad_k, sbda_tensor grad_v, void* stream);

/*
 * Per-head RMSNorm + half-split RoPE of q or k, forward.  Replaces the eager
 * _HeadRMSNorm + _apply_rope of BiAttn/attention_common.py:13-76 as applied
 * at BiAttn/left_v2.py:237-239.  x and y are [B, H, L, D] views (heads =
 * shape.heads; kv_heads is ignored); weight is the fp32 [D] norm weight;
 * cos_table / sin_table are [rows, D/2] in x's dtype (fp32 angles
 * position * theta^(-2i/D) cast to the dtype, attention_common.py:13-22) and
 * table row table_offset + l serves position l.  Odd D: norm only (no RoPE,
 * tables may be NULL).  y may alias x.
 */
int sbda_b200_norm_rope_forward(int dtype, sbda_shape shape, sbda_tensor x, sbda_tensor y,
                                const float* weight, float eps, const void* cos_table,
                                const void* sin_table, int64_t table_offset, void* stream);

/* fp32 floats of workspace sbda_b200_norm_rope_backward needs for `shape`. */
int64_t sbda_b200_norm_rope_workspace_floats(sbda_shape shape);

/*
 * Backward of sbda_b200_norm_rope_forward: from x and grad_y writes grad_x
 * (x's dtype) and grad_weight (fp32 [D], overwritten with the sum over all
 * rows).  The caller provides `workspace` (>= the floats reported above) for
 * the per-CTA weight-gradient partials; the reduction order is fixed, so
 * results are bitwise reproducible.
 */
int sbda_b200_norm_rope_backward(int dtype, sbda_shape shape, sbda_tensor x, sbda_tensor grad_y,
                                 const float* weight, float eps, const void* cos_table,
                                 const void* sin_table, int64_t table_offset, sbda_tensor grad_x,
                                 float* grad_weight, float* workspace, int64_t workspace_floats,
                                 void* stream);

/*
 * Allocation-free variant of sbda_b200_norm_rope_backward.  It has no
 * counterpart in the reference.  It exists for callers that cannot allocate
 * device memory where the backward runs (a replayed graph with a fixed pool,
 * a runtime or plugin host that only hands out tensors it planned): instead
 * of a caller workspace it uses a 512 KiB static device array that every GPU
 * loading this library holds until exit.  Shapes whose partials would not
 * fit are rejected with SBDA_ERR_UNSUPPORTED (none of the shapes the
 * backward accepts do today).  The first call on each device resolves the
 * array's device address; make that first call before any stream capture.
 * All calls share the array, so calls that overlap on the GPU race: run them
 * one after another.  Results are identical to sbda_b200_norm_rope_backward.
 */
int sbda_b200_norm_rope_backward_noalloc(int dtype, sbda_shape shape, sbda_tensor x, sbda_tensor grad_y,
                                         const float* weight, float eps, const void* cos_table,
                                         const void* sin_table, int64_t table_offset,
                                         sbda_tensor grad_x, float* grad_weight, void* stream);

/*
 * Attention with the per-head RMSNorm + RoPE of q and k inside the kernels.
 * Replaces, on the reference's fused route, _HeadRMSNorm and _apply_rope
 * (BiAttn/attention_common.py:13-76, applied at BiAttn/left_v2.py:237-239)
 * followed by fused_sbda_key_backward (sbda_triton.py:1467-1474): one kernel
 * each way instead of five.  q_raw / k_raw are the projections before the
 * norm ([B, H, L, D] views, like q / k above).  Each row is normalised in
 * fp32 (r = rsqrt(mean(x^2) + eps), y = cast(x * r * w)) and rotated in the
 * element type (z = cast(cast(y * cos) + cast(rotate_half(y) * sin))), with
 * cos_table / sin_table the [rows, D / 2] tables of the element type and row
 * table_offset + l serving position l.  Weights are fp32 [D], 16-byte aligned.
 *
 * Served (sbda_b200_normed_supported() == 1): head_dim 64, heads == kv_heads,
 * fp32 / fp16 / bf16, near offsets within {0, 1, 2} with at most one far
 * offset in the SBDA family's sets {0,1}, {0,2}, {0,1,2,d}, and views the copy
 * engine can stage (16-byte aligned rows and strides); other calls return
 * SBDA_ERR_UNSUPPORTED and the caller runs norm_rope + attention separately.
 */
int sbda_b200_normed_supported(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets);

int sbda_b200_forward_normed(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                             float scale, sbda_tensor q_raw, sbda_tensor k_raw, sbda_tensor v,
                             const float* q_weight, float q_eps, const float* k_weight, float k_eps,
                             const void* cos_table, const void* sin_table, int64_t table_offset,
                             sbda_tensor out, float* lse, void* stream);

/* fp32 workspace floats of sbda_b200_backward_normed (per-CTA weight-gradient
 * partials and their first reduction level); -1 if the call is not served. */
int64_t sbda_b200_backward_normed_workspace_floats(int dtype, sbda_shape shape, const int32_t* offsets,
                                                   int32_t n_offsets);

/*
 * Backward of sbda_b200_forward_normed: writes grad_q / grad_k with respect to
 * q_raw / k_raw (the RoPE transpose and the RMSNorm Jacobian applied in the
 * kernel), grad_v, and the fp32 [D] norm-weight gradients grad_q_weight /
 * grad_k_weight (summed over every row in a fixed order: deterministic).
 */
int sbda_b200_backward_normed(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                              float scale, sbda_tensor q_raw, sbda_tensor k_raw, sbda_tensor v,
                              sbda_tensor grad_out, const float* lse, const float* q_weight, float q_eps,
                              const float* k_weight, float k_eps, const void* cos_table,
                              const void* sin_table, int64_t table_offset, sbda_tensor grad_q,
                              sbda_tensor grad_k, sbda_tensor grad_v, float* grad_q_weight,
                              float* grad_k_weight, float* workspace, int64_t workspace_floats,
                              void* stream);

/*
 * Forward / backward with a per-row source mask, for rows whose usable sources
 * depend on the data: padding holes and segment (seam) resets.
 * source_mask[b * length + i], bit s set: source s of row i may be used (on
 * top of i - offsets[s] >= 0).  A contiguous uint8 [batch, length] device
 * array shared by all heads.  A row with no usable source gives zero output
 * and zero gradients.  No counterpart in the reference: it builds the same
 * per-row source validity inside its eager path (BiAttn/left_v2.py:349-373)
 * and never calls its fused op there.  Runs on the uniform kernels.
 */
int sbda_b200_forward_masked(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                             float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                             const uint8_t* source_mask, sbda_tensor out, float* lse, void* stream);
int sbda_b200_backward_masked(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                              float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                              const uint8_t* source_mask, sbda_tensor grad_out, const float* lse,
                              sbda_tensor grad_q, sbda_tensor grad_k, sbda_tensor grad_v, void* stream);

/*
 * Attention over caller path tables (the reference's eager route for
 * path_indices/path_valid, BiAttn/left_v2.py:212-231, 323-396; no fused
 * counterpart there).  path_index: int32 [batch, length, n_sources] source
 * positions (n_sources <= 4; indices outside [0, length) are not sources);
 * source_mask: uint8 [batch, length], bit s = source s usable (the caller folds
 * path_valid, causality, padding and segment rules in).  Vector layouts only
 * (16-byte aligned rows, unit channel stride).
 */
int sbda_b200_forward_paths(int dtype, sbda_shape shape, int32_t n_sources, float scale,
                            sbda_tensor q, sbda_tensor k, sbda_tensor v, const int32_t* path_index,
                            const uint8_t* source_mask, sbda_tensor out, float* lse, void* stream);

/* fp32 workspace floats of the path-table backward: batch * heads * length * n_sources * 2. */
int64_t sbda_b200_paths_workspace_floats(sbda_shape shape, int32_t n_sources);

/*
 * Backward over path tables, deterministic (no atomics).  key_offsets: int32
 * [batch, length + 1] and key_entries: int32 [batch, length * n_sources] are
 * the inverse index per batch: entries key_offsets[b, j] .. key_offsets[b, j+1]
 * of key_entries[b] are the codes i * n_sources + s of the (row, source)
 * pairs that read key j, in a fixed order (the sum order).
 */
int sbda_b200_backward_paths(int dtype, sbda_shape shape, int32_t n_sources, float scale,
                             sbda_tensor q, sbda_tensor k, sbda_tensor v, const int32_t* path_index,
                             const uint8_t* source_mask, const int32_t* key_offsets,
                             const int32_t* key_entries, sbda_tensor grad_out, const float* lse,
                             float* workspace, int64_t workspace_floats, sbda_tensor grad_q,
                             sbda_tensor grad_k, sbda_tensor grad_v, void* stream);

/*
 * Block parts around the attention op (BiAttn/model.py:299-335).  No C
 * counterpart in the reference, which runs them as eager torch ops
 * (RMSNorm model.py:25-29, residual add model.py:325, SwiGLU gate
 * model.py:58-59, padding-row mask left_v2.py:404).  Rows are contiguous
 * [rows, dim] arrays in the dtype, 16-byte aligned; dim % 8 == 0, dim <= 2048.
 *
 * Residual + row mask + RMSNorm: x1 = x + m * residual_add (when residual_add
 * is non-null; m = row_mask[row] != 0, all rows if row_mask is null; x1 is
 * rounded to the dtype and written to x1_out), y = x1 * rsqrt(mean(x1^2) +
 * eps) * weight; rstd[row] = that rsqrt (fp32, saved for the backward).
 * weight is fp32 [dim].
 */
int sbda_b200_rms_norm_forward(int dtype, int64_t rows, int64_t dim, const void* x,
                               const void* residual_add, const uint8_t* row_mask,
                               const float* weight, float eps, void* x1_out, void* y,
                               float* rstd, void* stream);

/* fp32 workspace floats the norm backward needs for `rows` x `dim`. */
int64_t sbda_b200_rms_norm_workspace_floats(int64_t rows, int64_t dim);

/*
 * Backward of the above: grad_x = d/dx1 (norm part) + grad_x1 (a gradient that
 * reaches x1 from elsewhere, nullable), grad_residual = m * grad_x (nullable),
 * grad_weight = fp32 [dim], summed over rows in a fixed order (deterministic).
 */
int sbda_b200_rms_norm_backward(int dtype, int64_t rows, int64_t dim, const void* x1,
                                const float* rstd, const float* weight, const void* grad_y,
                                const void* grad_x1, const uint8_t* row_mask, void* grad_x,
                                void* grad_residual, float* grad_weight, float* workspace,
                                int64_t workspace_floats, void* stream);

/*
 * SwiGLU gate over n elements (n % 8 == 0): h = silu(gate) * up, each op rounded
 * to the dtype as eager torch runs them; backward writes grad_gate, grad_up.
 */
int sbda_b200_silu_mul_forward(int dtype, int64_t n, const void* gate, const void* up, void* h,
                               void* stream);
int sbda_b200_silu_mul_backward(int dtype, int64_t n, const void* gate, const void* up,
                                const void* grad_h, void* grad_gate, void* grad_up, void* stream);

/*
 * The same four calls with the kernel family chosen by the caller, for tests
 * and benchmarks that compare the families (no counterpart in the reference,
 * which has one Triton kernel set).  family: 0 = automatic (what the calls
 * above do: the windowed chain-walking kernels wherever they apply, else the
 * general ones, else the uniform ones), 1 = general kernels (uniform ones for
 * offset sets with several far offsets), 2 = uniform kernels (sharded calls:
 * treated as 1).  Any other value returns SBDA_ERR_INVALID.  All families
 * compute the same function; their fp32 rounding differs, so a backward
 * should use the family its forward used.  The choice is an argument: the
 * library keeps no process-wide kernel setting.
 */
int sbda_b200_forward_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                         float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v, sbda_tensor out, float* lse,
                         void* stream);
int sbda_b200_backward_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                          float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v, sbda_tensor grad_out,
                          const float* lse, sbda_tensor grad_q, sbda_tensor grad_k, sbda_tensor grad_v,
                          void* stream);
int sbda_b200_forward_sharded_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets,
                                 int32_t n_offsets, float scale, int32_t rank, int32_t world, sbda_tensor q,
                                 const sbda_tensor* k_ranks, const sbda_tensor* v_ranks, sbda_tensor out,
                                 float* lse, void* stream);
int sbda_b200_backward_sharded_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets,
                                  int32_t n_offsets, float scale, int32_t rank, int32_t world,
                                  const sbda_tensor* q_ranks, const sbda_tensor* k_ranks,
                                  const sbda_tensor* v_ranks, const sbda_tensor* grad_out_ranks,
                                  const float* const* lse_ranks, sbda_tensor grad_q, sbda_tensor grad_k,
                                  sbda_tensor grad_v, void* stream);

/*
 * Reads (and, if reset != 0, clears) the calling device's fault word that
 * kernels set instead of trapping (bit 0: a bounded wait on a tensor-copy
 * barrier expired).  Synchronous: waits for the device.  Not for hot paths.
 */
int sbda_b200_device_status(uint32_t* flags_out, int reset);

#ifdef __cplusplus
}
#endif

#endif /* SBDA_B200_H_ */
