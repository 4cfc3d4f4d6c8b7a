/*
 * rfdetr_b200 -- C ABI of the B200 (sm_100a) backend for RF-DETR-JAX's training hot path.
 *
 * Every entry point takes raw device pointers, explicit sizes, element-type codes and the
 * CUDA stream to run on (passed as void*, it is a cudaStream_t), and returns an int status
 * (RFDETR_OK = 0).  Calls are asynchronous on that stream, never synchronise the device and
 * allocate no memory: scratch space comes from the caller as an explicit workspace.  They
 * keep no state between calls, so one process may drive several devices from several threads
 * (the device is the one current on the calling thread).  There is no CPU fallback: a build
 * without a usable sm_100a device fails with RFDETR_ERR_CUDA.
 *
 * Layouts are the reference's own (row-major, innermost last).  Paths cited as file:line are
 * inside the reference project (JESUSROYETH/rf-detr-jax).
 */
#ifndef RFDETR_B200_H
#define RFDETR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. */
enum rfdetr_dtype { RFDETR_F32 = 0, RFDETR_BF16 = 1 };

/* Status codes. */
enum rfdetr_status {
    RFDETR_OK = 0,
    RFDETR_ERR_SHAPE = 1,     /* sizes inconsistent, negative or beyond a supported limit */
    RFDETR_ERR_DTYPE = 2,     /* element type not supported for this argument */
    RFDETR_ERR_ALIGN = 3,     /* a pointer is not aligned to its element type */
    RFDETR_ERR_WORKSPACE = 4, /* workspace missing or smaller than the size query returned */
    RFDETR_ERR_CUDA = 5,      /* a CUDA runtime call or kernel launch failed */
    RFDETR_ERR_LIMIT = 6,     /* a device loop reached its iteration cap (reported via status buffer) */
    RFDETR_ERR_CAPACITY = 7   /* problem larger than the no-alloc entry point's static scratch */
};

/* Human-readable text for a status code (static storage). */
const char *rfdetr_status_string(int status);

/* ABI version of this library; bumped on any signature change. */
int rfdetr_abi_version(void);

/* Sets a process-wide tuning knob.  Knobs exist for experiments and tests; every default is the
 * tuned production choice.  `name` is one of
 *   "RFDETR_MSDA_FWD", "RFDETR_MSDA_BWD", "RFDETR_MSDA_SLAB_FWD", "RFDETR_MSDA_BINS",
 *   "RFDETR_MSDA_OWN", "RFDETR_MSDA_TILES", "RFDETR_MSDA_CELL" (sampler kernel selection and
 *   launch shapes, "a,b,c,d,e"),
 *   "RFDETR_LSAP_STAGE_KB" (the assignment's shared-memory cost stage, KiB),
 *   "RFDETR_LSAP_STEP_CAP" (scan steps an augmenting path may take before the solve gives up with
 *   RFDETR_ERR_LIMIT; default: the block's column count, which finite costs never exceed),
 *   "RFDETR_TOPK_SORT", "RFDETR_TOPK_UNSTAGED" (any value: the one-CTA sort kernels; the radix
 *   select without its shared-memory key stage);
 * `value` is up to five comma-separated integers, or NULL / "" for the default.  Environment
 * variables of the same names are read once, before the first knob is read or set; after that
 * only this call changes a knob (launches read them from atomics, never from the environment).
 * A knob changed while another thread launches may be seen half-updated by that launch.
 * Returns RFDETR_ERR_SHAPE for an unknown name or a malformed value.  No reference counterpart:
 * the reference tunes through XLA flags (src/rfdetr_jax/utilities/gpu_flags.py:15). */
int rfdetr_set_tuning(const char *name, const char *value);

/* Reads and clears the device fault word.  Kernels that wait on hardware barriers (the TMA
 * tile loads of the sampler backward) bound every wait; a wait that gives up sets this word and
 * the kernel finishes with undefined outputs instead of hanging.  Synchronises `stream`.
 * Returns RFDETR_OK when no wait gave up since the last call, RFDETR_ERR_LIMIT when one did,
 * RFDETR_ERR_CUDA when the copy fails.  No reference counterpart: the reference's sampler runs
 * under XLA, which has no device-side waits. */
int rfdetr_take_device_fault(void *stream);

/* Self-test of the bounded device waits: one CTA arms a shared-memory barrier for 16 bytes that
 * no copy delivers and waits at most `polls` polls (1 .. 2^22).  The wait gives up, *result
 * (device int32) receives 0 (1 would mean the barrier completed), and the fault word is raised,
 * so the next rfdetr_take_device_fault() returns RFDETR_ERR_LIMIT.  Nothing is left in flight and
 * the context stays usable.  Asynchronous on `stream`.  No reference counterpart. */
int rfdetr_selftest_bounded_wait(void *stream, int polls, int32_t *result);

/* ---------------------------------------------------------------------------------------
 * Multi-scale deformable attention sampler.
 *
 * Replaces ms_deform_attn_core_rows(value, spatial_shapes, sampling_locations,
 * attention_weights, sampler)  -- src/rfdetr_jax/models/ops.py:208-292 -- as the new
 * sampler "cuda", and its JAX-autodiff backward (the gather path's scatter-add,
 * tests/test_ops.py:157-167; analytic formulas deform_pallas.py:97-120).
 *
 *   value               [B*H, Lv, D]        value_dtype (f32 | bf16), Lv = sum_l H_l*W_l
 *   spatial_shapes      host int64 [L][2]   (H_l, W_l) per level
 *   level_start_index   host int64 [L]      offsets of the levels in Lv, or NULL to derive
 *                                           them from spatial_shapes (ops.py:265-267)
 *   sampling_locations  [B, Lq, H, L, P, 2] f32, (x, y) in [0, 1] (ops.py:220)
 *   attention_weights   [B, Lq, H, L*P]     weight_dtype (f32 | bf16)
 *   output              [B, Lq, H*D]        bf16 if value and weights are both bf16, else f32
 *                                           (result_type(value, weights), ops.py:260)
 * Numerics: positions are computed in float32 in the reference's op order
 * (2*loc-1, ((g+1)*W-1)/2; ops.py:83-84,270); interpolation and accumulation in float32.
 * Limits: 1 <= L <= 16, D <= 256, all sizes < 2^31 elements per tensor.
 * ------------------------------------------------------------------------------------- */
int rfdetr_msda_forward(void *stream,
                        const void *value, int value_dtype,
                        const int64_t *spatial_shapes, const int64_t *level_start_index,
                        const float *sampling_locations,
                        const void *attention_weights, int weight_dtype,
                        void *output, int output_dtype,
                        int64_t batch, int64_t n_heads, int64_t head_dim, int64_t len_query,
                        int64_t n_levels, int64_t n_points);

/* Workspace bytes of rfdetr_msda_backward's float32-accumulator path (0 when value_dtype is f32).
 * A workspace of this size always suffices; rfdetr_msda_backward_workspace_bytes() gives the
 * size that also enables the position-tile kernels. */
size_t rfdetr_msda_backward_workspace_size(int value_dtype, int64_t batch, int64_t n_heads,
                                           int64_t head_dim, int64_t len_value);

/* Workspace bytes with which rfdetr_msda_backward can take every kernel it has for this geometry,
 * the position-tile kernels of multi-level shapes included (their per-corner dot products and
 * per-slab flags live there): the maximum over its paths.  0 for invalid arguments. */
size_t rfdetr_msda_backward_workspace_bytes(int value_dtype, int weight_dtype, const int64_t *spatial_shapes,
                                            int64_t batch, int64_t n_heads, int64_t head_dim,
                                            int64_t len_query, int64_t n_levels, int64_t n_points);

/*
 * Backward of rfdetr_msda_forward against grad_output ([B, Lq, H*D], the output's dtype):
 *   grad_value               [B*H, Lv, D]        value_dtype   (overwritten)
 *   grad_sampling_locations  [B, Lq, H, L, P, 2] f32           (overwritten)
 *   grad_attention_weights   [B, Lq, H, L*P]     weight_dtype  (overwritten)
 * grad_value is accumulated in float32 and rounded once.  Non-finite sampling locations
 * give NaN location/weight gradients and add nothing to grad_value.
 */
int rfdetr_msda_backward(void *stream,
                         const void *value, int value_dtype,
                         const int64_t *spatial_shapes, const int64_t *level_start_index,
                         const float *sampling_locations,
                         const void *attention_weights, int weight_dtype,
                         const void *grad_output, int grad_output_dtype,
                         void *grad_value, float *grad_sampling_locations,
                         void *grad_attention_weights,
                         void *workspace, size_t workspace_bytes,
                         int64_t batch, int64_t n_heads, int64_t head_dim, int64_t len_query,
                         int64_t n_levels, int64_t n_points);

/*
 * rfdetr_msda_backward without a workspace argument, for callers that cannot allocate device
 * memory at the point of the call: a host framework whose allocator owns all device memory and
 * hands its custom calls no scratch buffer (an XLA FFI handler registered without a scratch
 * allocator, for instance), or latency-critical code that must not allocate after start-up.
 * There is no counterpart in the reference (its backward is JAX autodiff).
 *
 * The bf16 path's float32 accumulator lives in a static device array of the library
 * (RFDETR_MSDA_NOALLOC_SCRATCH_BYTES, 8 MiB; every GPU that loads the library holds it until the
 * process exits), so a call that needs it must have batch * n_heads * Lv * head_dim <= 2,097,152
 * elements; a larger call that needs it returns RFDETR_ERR_CAPACITY without launching anything.
 * Shapes that the scratch-free bf16 kernels serve (D in {16, 32}, L*P in {1, 2, 4, 8}, small
 * enough slabs -- the Nano decoder's among them) never touch the array and have no extra limit;
 * nor do float32 values.  The entry point itself allocates nothing.
 *
 * Each call looks up the array's device address in the current context (cudaGetSymbolAddress, a
 * host-side query): nothing is cached, so a context that was reset or recreated is simply looked
 * up again.  The first lookup may load the library's device code; make one call before any stream
 * capture.  Every call on a device shares the one array: the call clears it before use, but calls
 * whose work overlaps on the GPU (different streams, or different host threads, on the same
 * device) race on it and must be serialised by the caller.  Arguments and results are those of
 * rfdetr_msda_backward.
 */
#define RFDETR_MSDA_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
int rfdetr_msda_backward_noalloc(void *stream,
                                 const void *value, int value_dtype,
                                 const int64_t *spatial_shapes, const int64_t *level_start_index,
                                 const float *sampling_locations,
                                 const void *attention_weights, int weight_dtype,
                                 const void *grad_output, int grad_output_dtype,
                                 void *grad_value, float *grad_sampling_locations,
                                 void *grad_attention_weights,
                                 int64_t batch, int64_t n_heads, int64_t head_dim, int64_t len_query,
                                 int64_t n_levels, int64_t n_points);

/* ---------------------------------------------------------------------------------------
 * Two-stage query selection.
 *
 * Replaces, per row r of logits [R, N, C] (R = groups*batch):
 *   proposal_scores = logits.max(-1)                         (transformer.py:695)
 *   values, indices = jax.lax.top_k(proposal_scores, k)      (transformer.py:696)
 * Descending IEEE totalOrder (NaN first), equal scores keep the lower index first.
 * C == 1 selects directly over a [R, N] score tensor.
 *   scores_out  [R, N] f32 or NULL;  values_out [R, k] f32 or NULL;  indices_out [R, k] int32.
 * Limits: 1 <= k <= N <= 16384; for C == 1 (a flat score row, as the inference post-process's
 * top-k over Q*C sigmoid scores, postprocess.py:37-41) N may reach 2^24 when k <= 4096.
 * ------------------------------------------------------------------------------------- */
int rfdetr_topk_select(void *stream, const float *logits, int64_t rows, int64_t positions,
                       int64_t classes, int64_t k, float *scores_out, float *values_out,
                       int32_t *indices_out);

/*
 * select_rows(values, indices) -- src/rfdetr_jax/models/layers.py:225-244:
 *   out[r, i, :] = values[r, indices[r, i], :]
 *   values [R, N, W] (element_bytes each), indices [R, K] int32, out [R, K, W].
 * An index outside [0, N) writes a zero row and sets *status_out (device int32, may be NULL)
 * to RFDETR_ERR_SHAPE.
 */
int rfdetr_select_rows(void *stream, const void *values, int64_t element_bytes, int64_t rows,
                       int64_t positions, int64_t width, const int32_t *indices, int64_t k,
                       void *out, int32_t *status_out);

/* ---------------------------------------------------------------------------------------
 * Matching cost -- build_cost_matrix for classes and boxes, src/rfdetr_jax/models/matcher.py:44-103,141
 * (focal cost :36-41, GIoU utilities/box_ops.py:27-75):
 *   cost[b,q,t] = cost_bbox * |pb - tb|_1 + cost_class * focal(logit[b,q,label[b,t]])
 *                 + cost_giou * (-GIoU(pb, tb)),   or 1e4 where target_mask[b,t] == 0.
 *   pred_logits [B, Q, C] (f32 | bf16), pred_boxes [B, Q, 4] (f32 | bf16, cxcywh),
 *   target_labels [B, T] int32, target_boxes [B, T, 4] f32, target_mask [B, T] uint8,
 *   cost [B, Q, T] f32.  The target's logit is read as the reference's one-hot contraction
 *   gives it: a label outside [0, C) reads 0, and a non-finite logit at any other class of the
 *   row makes the row's class costs NaN (x * 0 = NaN).
 * ------------------------------------------------------------------------------------- */
int rfdetr_match_cost(void *stream, const void *pred_logits, int logits_dtype,
                      const void *pred_boxes, int boxes_dtype, const int32_t *target_labels,
                      const float *target_boxes, const uint8_t *target_mask, float *cost,
                      int64_t batch, int64_t queries, int64_t classes, int64_t targets,
                      float cost_class, float cost_bbox, float cost_giou, float focal_alpha);

/*
 * Batched exact assignment -- hungarian_match / _solve_batch, matcher.py:144-208, i.e.
 * scipy.optimize.linear_sum_assignment on every block cost[n, g*Qg:(g+1)*Qg, :sizes[n]]
 * (Qg = queries / group_detr), with SciPy's tie-breaking, in float64.
 *   cost [N, Q, T] f32, sizes [N] int32 (device), outputs [N, G*T]:
 *   rows int32 (global query index), cols int32, valid uint8; slots g*T.. in ascending row
 *   order, unused slots 0/0/0.  Non-finite block entries are replaced by max(finite)+1
 *   (matcher.py:169-172).  *status_out (device int32, required) is set to RFDETR_ERR_LIMIT
 *   if a solve hits its iteration cap (never for finite costs) -- read it when convenient.
 * Limits: queries % group_detr == 0, T <= 1024, Qg <= 4096.
 */
int rfdetr_lsap_batched(void *stream, const float *cost, const int32_t *sizes, int64_t problems,
                        int64_t queries, int64_t max_targets, int64_t group_detr, int32_t *rows,
                        int32_t *cols, uint8_t *valid, int32_t *status_out);

/* ---------------------------------------------------------------------------------------
 * Prologue of multi-scale deformable attention: query -> (sampling locations, weights).
 *
 * Replaces MSDeformAttn.__call__'s sampling_offsets / attention_weights Linear layers, the
 * location arithmetic and the softmax (ops.py:381-404), writing the sampler's inputs:
 *   query [B, Lq, C] (f32 or bf16); weight [H*L*P*3, C] in the query dtype (rows 0..H*L*P*2-1:
 *   sampling_offsets.weight, then attention_weights.weight); bias [H*L*P*3] f32 (likewise);
 *   reference_points [B, Lq, L, ref_dim] f32 with ref_dim 2 (points) or 4 (boxes);
 *   spatial_shapes [L][2] = (H_l, W_l), host memory.
 *   sampling_locations [B, Lq, H, L, P, 2] f32 (8-byte aligned); attention_weights
 *   [B, Lq, H, L*P] in the query dtype; offsets_out (may be NULL) [B*Lq, H*L*P*2] f32, 8-byte
 *   aligned, receives the biased offsets (the projection's offsets part, as rounded) -- what the
 *   box form's backward needs.  The projection and bias are rounded to the query dtype as the
 *   reference's Linear does (layers.py:276-279); the softmax runs in f32.
 * Limits: L <= 8, C <= 4096, H*L*P <= 1024; bf16 needs C % 16 == 0 and H*L*P % 8 == 0.
 * ------------------------------------------------------------------------------------- */
int rfdetr_msda_prologue(void *stream, const void *query, int query_dtype, const void *weight,
                         const float *bias, const float *reference_points, int64_t ref_dim,
                         const int64_t *spatial_shapes, float *sampling_locations,
                         void *attention_weights, float *offsets_out, int64_t batch, int64_t len_query,
                         int64_t channels, int64_t n_heads, int64_t n_levels, int64_t n_points);

/* Backward of the prologue's elementwise part (the derivatives of the softmax and of the
 * location arithmetic, ops.py:388-404), for the autodiff of MSDeformAttn's query side:
 *   grad_locations [B, Lq, H, L, P, 2] f32, grad_weights and attention_weights [B, Lq, H, L*P]
 *   (weights_dtype, the forward's attention output), reference_points as in the forward,
 *   offsets [B*Lq, H*L*P*2] f32 (the forward's biased projection, offsets part; box form only,
 *   else may be NULL), spatial_shapes as in the forward.
 *   grad_projection [B*Lq, H*L*P*3] (grad_projection_dtype: f32, or bf16 -- the cotangent
 *   dtype of a bf16 query's projection in the reference's autodiff) receives the gradient of the
 *   projection (offsets part, then logits part), grad_reference_points [B, Lq, L, ref_dim] f32
 *   that of the reference points.  The query / weight gradients are then two GEMMs with
 *   grad_projection, the bias gradient its column sum. */
int rfdetr_msda_prologue_backward(void *stream, const float *grad_locations, const void *grad_weights,
                                  const void *attention_weights, int weights_dtype,
                                  const float *reference_points, int64_t ref_dim, const float *offsets,
                                  const int64_t *spatial_shapes, void *grad_projection,
                                  int grad_projection_dtype, float *grad_reference_points, int64_t batch,
                                  int64_t len_query, int64_t n_heads, int64_t n_levels, int64_t n_points);

/* ---------------------------------------------------------------------------------------
 * Matching cost and exact assignment of stacked layers in one call.
 *
 * Replaces the stacked layer_cost + single solve of compute_losses (criterion.py:402-413): the
 * cost of every layer (one rfdetr_match_cost launch over all layers and images) followed by one
 * rfdetr_lsap_batched over all (layer, image, group) blocks, on `stream`.
 *   pred_logits [L, B, Q, C] and pred_boxes [L, B, Q, 4] (f32 or bf16); target_labels [B, T]
 *   int32, target_boxes [B, T, 4] f32, target_mask [B, T] uint8 and sizes [B] int32 are shared
 *   by the layers.  cost [L, B, Q, T] f32 receives the cost (the solver's input); rows/cols
 *   [L, B, G*T] int32 and valid [L, B, G*T] uint8 the assignment; *status_out (device int32)
 *   as for rfdetr_lsap_batched.  Results are bit for bit those of the two separate calls.
 * Limits: those of both entry points, and L * B <= 65535.
 * ------------------------------------------------------------------------------------- */
int rfdetr_match_stacked(void *stream, const void *pred_logits, int logits_dtype, const void *pred_boxes,
                         int boxes_dtype, const int32_t *target_labels, const float *target_boxes,
                         const uint8_t *target_mask, const int32_t *sizes, int64_t layers, int64_t batch,
                         int64_t queries, int64_t classes, int64_t targets, int64_t group_detr,
                         float cost_class, float cost_bbox, float cost_giou, float focal_alpha, float *cost,
                         int32_t *rows, int32_t *cols, uint8_t *valid, int32_t *status_out);

/* ---------------------------------------------------------------------------------------
 * Set-prediction losses of every decoder layer, with gradients, in one launch.
 *
 * Replaces loss_labels (criterion.py:157-224) and loss_boxes (criterion.py:233-250), called by
 * the reference once per output layer; here layer l of `layers` is one slice of each [L, ...]
 * argument (the targets are shared):
 *   losses_out[l, 0], ia_bce != 0 (IA-BCE, criterion.py:188-208): sum over [B, Q, C] of
 *     (neg * x - log_sigmoid(x) * (pos + neg)) / num_boxes, pos/neg = (w, 1 - w) at the matched
 *     (image, query, class) entries, with the stop-gradient weight
 *     w = max(sigmoid(x)^alpha * iou^(1 - alpha), 0.01), and (0, sigmoid(x)^2) elsewhere;
 *   losses_out[l, 0], ia_bce == 0 (criterion.py:210-224): the sigmoid focal loss (gamma 2,
 *     alpha_t from focal_alpha, none when it is negative) of the one-hot matched targets,
 *     summed over [B, Q, C] and divided by num_boxes;
 *   losses_out[l, 1] = sum over valid matches of |box - target box|_1 / num_boxes;
 *   losses_out[l, 2] = sum over valid matches of (1 - GIoU) / num_boxes.
 * Also writes the gradients for unit cotangents: grad_logits [L, B, Q, C] = d losses_out[l, 0]
 * / d logits, grad_boxes_l1 / grad_boxes_giou [L, B, Q, 4] = d losses_out[l, 1] / d boxes and
 * d losses_out[l, 2] / d boxes (zero for unmatched queries).
 *   pred_logits [L, B, Q, C] f32, pred_boxes [L, B, Q, 4] f32 cxcywh, target_labels [B, T]
 *   int32, target_boxes [B, T, 4] f32, rows/cols [L, B, S] int32 and valid [L, B, S] uint8
 *   from rfdetr_lsap_batched (a query is matched at most once per layer), num_boxes: device f32
 *   scalar, losses_out: device f32 [L, 3] (cleared on `stream` first).  Box arrays must be
 *   16-byte aligned (RFDETR_ERR_ALIGN otherwise).
 * ------------------------------------------------------------------------------------- */
int rfdetr_set_losses(void *stream, const float *pred_logits, const float *pred_boxes,
                      const int32_t *target_labels, const float *target_boxes, const int32_t *rows,
                      const int32_t *cols, const uint8_t *valid, const float *num_boxes, int64_t layers,
                      int64_t batch, int64_t queries, int64_t classes, int64_t targets, int64_t slots,
                      float focal_alpha, int32_t ia_bce, float *losses_out, float *grad_logits,
                      float *grad_boxes_l1, float *grad_boxes_giou);

/* ---------------------------------------------------------------------------------------
 * Data-parallel gradient all-reduce over NVLink peer memory.
 *
 * Replaces the train step's gradient `psum` over the batch axis (trainer.py:462-469), which XLA
 * lowers to an NCCL all-reduce: one process per GPU on one node, each rank's float32 buffer
 * summed elementwise across ranks in place.  Setup, once per buffer: every rank allocates a
 * zeroed flag buffer of rfdetr_allreduce_flag_bytes(), exports it and its buffer with
 * rfdetr_ipc_get_handle (an rfdetr_ipc_handle_bytes()-byte handle of the allocation holding the
 * pointer, and the pointer's offset in it), the ranks exchange handles and offsets (any host
 * channel), and each rank maps its peers' allocations with rfdetr_ipc_open_handle (peer pointer =
 * mapped base + offset) and releases them with rfdetr_ipc_close_handle.
 *
 * rfdetr_allreduce_sum_f32: `buffers` and `flags` are host arrays of `world` device pointers in
 * rank order (this rank's own and the mapped peers'), 16- and 4-byte aligned; every rank calls it
 * with the same n, world and epoch, epoch starting at 1 and increasing by one per call, after the
 * work that writes its buffer on `stream`.  When every rank's launch has completed, every buffer
 * holds the sum, identical on all ranks (rank-order summation).  `ctas` CTAs per rank (<= 1024;
 * 0 = 64).  A bounded wait for a peer that runs out (about a second) sets the device int32
 * *status_out to RFDETR_ERR_LIMIT, which the caller reads when it chooses (the buffers are then
 * not reduced).  Limits: 1 <= world <= 8 (world 1 returns at once).
 * ------------------------------------------------------------------------------------- */
size_t rfdetr_ipc_handle_bytes(void);
size_t rfdetr_allreduce_flag_bytes(void);
int rfdetr_ipc_get_handle(const void *device_ptr, void *handle_out, size_t *offset_out);
int rfdetr_ipc_open_handle(const void *handle, void **base_out);
int rfdetr_ipc_close_handle(void *base);
int rfdetr_allreduce_sum_f32(void *stream, float *const *buffers, unsigned *const *flags, int rank, int world,
                             int64_t n, uint32_t epoch, int ctas, int32_t *status_out);

#ifdef __cplusplus
}
#endif

#endif /* RFDETR_B200_H */
