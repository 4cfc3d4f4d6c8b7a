// XLA FFI handlers binding librfdetr_b200.so into JAX: one handler per C entry point of
// include/rfdetr_b200.h, so the kernels run inside jit and shard_map on XLA's own stream.
//
// NOT COMPILED IN THIS REPOSITORY: JAX/jaxlib (which ship the XLA FFI headers) are absent from
// this image and from the GPU hosts.  Where jaxlib is installed, build with
//
//   g++ -O2 -std=c++17 -shared -fPIC -o librfdetr_ffi.so rfdetr_ffi.cc \
//       -I"$(python -c 'import jax.ffi; print(jax.ffi.include_dir())')" -I../../include \
//       -I/usr/local/cuda/include -L.. -lrfdetr_b200 -Wl,-rpath,'$ORIGIN/..'
//
// and register the symbols from Python (cuda_backend.py beside this file).
//
// Conventions:
// * every handler takes the stream as Ctx<PlatformStream<cudaStream_t>> and maps the library's
//   status to an ffi::Error (argument errors -> kInvalidArgument, RFDETR_ERR_CUDA -> kInternal);
// * geometry that the reference holds as Python ints (spatial_shapes, k, group_detr, cost
//   weights) arrives as static attributes; everything else is read from buffer dimensions;
// * scratch memory comes from XLA's ScratchAllocator (the sampler backward's bf16 accumulator),
//   or, for a handler registered where no scratch can be requested, from the library's static
//   array (RfdetrMsdaBwdNoAlloc);
// * device status words (the assignment's iteration cap) are int32[1] results, never read on
//   the host inside the step.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "rfdetr_b200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

int dtype_code(ffi::DataType t) {
    switch (t) {
        case ffi::DataType::F32: return RFDETR_F32;
        case ffi::DataType::BF16: return RFDETR_BF16;
        default: return -1;
    }
}

ffi::Error status_error(int status, const char *what) {
    if (status == RFDETR_OK) return ffi::Error::Success();
    const std::string msg = std::string(what) + ": " + rfdetr_status_string(status);
    return ffi::Error(status == RFDETR_ERR_CUDA ? ffi::ErrorCode::kInternal : ffi::ErrorCode::kInvalidArgument, msg);
}

// spatial_shapes arrive flattened: (H_0, W_0, H_1, W_1, ...).
int64_t levels_of(ffi::Span<const int64_t> shapes) { return static_cast<int64_t>(shapes.size() / 2); }

int64_t dim(const ffi::AnyBuffer &b, int i) { return b.dimensions()[i]; }
template <ffi::DataType T>
int64_t dim(const ffi::Buffer<T> &b, int i) {
    return b.dimensions()[i];
}

}  // namespace

// ---- sampler --------------------------------------------------------------------------------
// value [B*H, Lv, D], loc [B, Lq, H, L, P, 2] f32, weights [B, Lq, H, L*P] -> out [B, Lq, H*D].
// Replaces ms_deform_attn_core_rows (src/rfdetr_jax/models/ops.py:208-292).
static ffi::Error MsdaFwd(cudaStream_t stream, ffi::AnyBuffer value, ffi::Buffer<ffi::F32> loc,
                          ffi::AnyBuffer weights, ffi::Span<const int64_t> shapes, ffi::Result<ffi::AnyBuffer> out) {
    const int64_t B = dim(loc, 0), Lq = dim(loc, 1), H = dim(loc, 2), L = dim(loc, 3), P = dim(loc, 4);
    if (L != levels_of(shapes)) return status_error(RFDETR_ERR_SHAPE, "RfdetrMsdaFwd");
    return status_error(
        rfdetr_msda_forward(stream, value.untyped_data(), dtype_code(value.element_type()), shapes.begin(), nullptr,
                            loc.typed_data(), weights.untyped_data(), dtype_code(weights.element_type()),
                            out->untyped_data(), dtype_code(out->element_type()), B, H, dim(value, 2), Lq, L, P),
        "RfdetrMsdaFwd");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMsdaFwd, MsdaFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Attr<ffi::Span<const int64_t>>("spatial_shapes")
                                  .Ret<ffi::AnyBuffer>());

// Backward: (value, loc, weights, grad_out) -> (grad_value, grad_loc, grad_weights); the bf16
// accumulator from XLA's scratch allocator.  Replaces the JAX autodiff of the gather sampler.
static ffi::Error MsdaBwd(cudaStream_t stream, ffi::ScratchAllocator scratch, ffi::AnyBuffer value,
                          ffi::Buffer<ffi::F32> loc, ffi::AnyBuffer weights, ffi::AnyBuffer grad_out,
                          ffi::Span<const int64_t> shapes, ffi::Result<ffi::AnyBuffer> grad_value,
                          ffi::Result<ffi::Buffer<ffi::F32>> grad_loc, ffi::Result<ffi::AnyBuffer> grad_weights) {
    const int64_t B = dim(loc, 0), Lq = dim(loc, 1), H = dim(loc, 2), L = dim(loc, 3), P = dim(loc, 4);
    const int64_t Lv = dim(value, 1), D = dim(value, 2);
    if (L != levels_of(shapes)) return status_error(RFDETR_ERR_SHAPE, "RfdetrMsdaBwd");
    const int vd = dtype_code(value.element_type());
    (void)Lv;
    const size_t bytes = rfdetr_msda_backward_workspace_bytes(vd, dtype_code(weights.element_type()),
                                                              shapes.begin(), B, H, D, Lq, L, P);
    void *ws = nullptr;
    if (bytes) {
        auto block = scratch.Allocate(bytes, 256);
        if (!block.has_value()) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "RfdetrMsdaBwd: workspace");
        ws = *block;
    }
    return status_error(
        rfdetr_msda_backward(stream, value.untyped_data(), vd, shapes.begin(), nullptr, loc.typed_data(),
                             weights.untyped_data(), dtype_code(weights.element_type()), grad_out.untyped_data(),
                             dtype_code(grad_out.element_type()), grad_value->untyped_data(), grad_loc->typed_data(),
                             grad_weights->untyped_data(), ws, bytes, B, H, D, Lq, L, P),
        "RfdetrMsdaBwd");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMsdaBwd, MsdaBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Attr<ffi::Span<const int64_t>>("spatial_shapes")
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>());

// The same backward for a registration that cannot request scratch: the library's static array.
static ffi::Error MsdaBwdNoAlloc(cudaStream_t stream, ffi::AnyBuffer value, ffi::Buffer<ffi::F32> loc,
                                 ffi::AnyBuffer weights, ffi::AnyBuffer grad_out, ffi::Span<const int64_t> shapes,
                                 ffi::Result<ffi::AnyBuffer> grad_value, ffi::Result<ffi::Buffer<ffi::F32>> grad_loc,
                                 ffi::Result<ffi::AnyBuffer> grad_weights) {
    const int64_t B = dim(loc, 0), Lq = dim(loc, 1), H = dim(loc, 2), L = dim(loc, 3), P = dim(loc, 4);
    if (L != levels_of(shapes)) return status_error(RFDETR_ERR_SHAPE, "RfdetrMsdaBwdNoAlloc");
    return status_error(
        rfdetr_msda_backward_noalloc(stream, value.untyped_data(), dtype_code(value.element_type()), shapes.begin(),
                                     nullptr, loc.typed_data(), weights.untyped_data(),
                                     dtype_code(weights.element_type()), grad_out.untyped_data(),
                                     dtype_code(grad_out.element_type()), grad_value->untyped_data(),
                                     grad_loc->typed_data(), grad_weights->untyped_data(), B, H, dim(value, 2), Lq, L,
                                     P),
        "RfdetrMsdaBwdNoAlloc");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMsdaBwdNoAlloc, MsdaBwdNoAlloc,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Attr<ffi::Span<const int64_t>>("spatial_shapes")
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>());

// ---- sampler prologue --------------------------------------------------------------------------
// query [B, Lq, C], weight [H*L*P*3, C] (query dtype), bias [H*L*P*3] f32, reference points
// [B, Lq, L, 2|4] f32 -> loc [B, Lq, H, L, P, 2] f32, attn [B, Lq, H, L*P] (query dtype), and the
// biased offsets [B*Lq, H*L*P*2] f32 (the box form's backward residual).
// Replaces MSDeformAttn.__call__'s query side (ops.py:381-404).
static ffi::Error MsdaPrologue(cudaStream_t stream, ffi::AnyBuffer query, ffi::AnyBuffer weight,
                               ffi::Buffer<ffi::F32> bias, ffi::Buffer<ffi::F32> ref, ffi::Span<const int64_t> shapes,
                               int64_t n_heads, int64_t n_points, ffi::Result<ffi::Buffer<ffi::F32>> loc,
                               ffi::Result<ffi::AnyBuffer> attn, ffi::Result<ffi::Buffer<ffi::F32>> offsets) {
    const int64_t B = dim(query, 0), Lq = dim(query, 1), C = dim(query, 2), L = levels_of(shapes);
    return status_error(rfdetr_msda_prologue(stream, query.untyped_data(), dtype_code(query.element_type()),
                                             weight.untyped_data(), bias.typed_data(), ref.typed_data(), dim(ref, 3),
                                             shapes.begin(), loc->typed_data(), attn->untyped_data(),
                                             offsets->typed_data(), B, Lq, C, n_heads, L, n_points),
                        "RfdetrMsdaPrologue");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMsdaPrologue, MsdaPrologue,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<ffi::Span<const int64_t>>("spatial_shapes")
                                  .Attr<int64_t>("n_heads")
                                  .Attr<int64_t>("n_points")
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

// Elementwise part of the prologue's backward: (grad_loc, grad_attn, attn, ref, offsets) ->
// (grad_projection [B*Lq, H*L*P*3] in f32 or bf16 -- the result's own dtype, grad_ref).  offsets
// is the forward's third result for box references; pass an empty [0] buffer for point references.
static ffi::Error MsdaPrologueBwd(cudaStream_t stream, ffi::Buffer<ffi::F32> grad_loc, ffi::AnyBuffer grad_attn,
                                  ffi::AnyBuffer attn, ffi::Buffer<ffi::F32> ref, ffi::Buffer<ffi::F32> offsets,
                                  ffi::Span<const int64_t> shapes, ffi::Result<ffi::AnyBuffer> grad_proj,
                                  ffi::Result<ffi::Buffer<ffi::F32>> grad_ref) {
    const int64_t B = dim(grad_loc, 0), Lq = dim(grad_loc, 1), H = dim(grad_loc, 2), L = dim(grad_loc, 3),
                  P = dim(grad_loc, 4);
    if (grad_attn.element_type() != attn.element_type())
        return status_error(RFDETR_ERR_DTYPE, "RfdetrMsdaPrologueBwd");
    const float *off = offsets.element_count() ? offsets.typed_data() : nullptr;
    return status_error(rfdetr_msda_prologue_backward(stream, grad_loc.typed_data(), grad_attn.untyped_data(),
                                                      attn.untyped_data(), dtype_code(attn.element_type()),
                                                      ref.typed_data(), dim(ref, 3), off, shapes.begin(),
                                                      grad_proj->untyped_data(), dtype_code(grad_proj->element_type()),
                                                      grad_ref->typed_data(), B, Lq, H, L, P),
                        "RfdetrMsdaPrologueBwd");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMsdaPrologueBwd, MsdaPrologueBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<ffi::Span<const int64_t>>("spatial_shapes")
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

// ---- two-stage selection ----------------------------------------------------------------------
// logits [R, N, C] f32 -> scores [R, N], values [R, k], indices [R, k] int32 (C == 1: a flat
// score row).  Replaces logits.max(-1) + jax.lax.top_k (transformer.py:694-696) and the
// post-process top-k (postprocess.py:37-41).
static ffi::Error TopkSelect(cudaStream_t stream, ffi::Buffer<ffi::F32> logits, int64_t k,
                             ffi::Result<ffi::Buffer<ffi::F32>> scores, ffi::Result<ffi::Buffer<ffi::F32>> values,
                             ffi::Result<ffi::Buffer<ffi::S32>> indices) {
    return status_error(rfdetr_topk_select(stream, logits.typed_data(), dim(logits, 0), dim(logits, 1),
                                           dim(logits, 2), k, scores->typed_data(), values->typed_data(),
                                           indices->typed_data()),
                        "RfdetrTopkSelect");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrTopkSelect, TopkSelect,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<int64_t>("k")
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>());

// values [R, N, W], indices [R, K] int32 -> out [R, K, W], status int32[1].
// Replaces select_rows (layers.py:225-244).
static ffi::Error SelectRows(cudaStream_t stream, ffi::AnyBuffer values, ffi::Buffer<ffi::S32> indices,
                             ffi::Result<ffi::AnyBuffer> out, ffi::Result<ffi::Buffer<ffi::S32>> status) {
    const int64_t esize = static_cast<int64_t>(ffi::ByteWidth(values.element_type()));
    if (cudaMemsetAsync(status->typed_data(), 0, sizeof(int32_t), stream) != cudaSuccess)
        return status_error(RFDETR_ERR_CUDA, "RfdetrSelectRows");
    return status_error(rfdetr_select_rows(stream, values.untyped_data(), esize, dim(values, 0), dim(values, 1),
                                           dim(values, 2), indices.typed_data(), dim(indices, 1), out->untyped_data(),
                                           status->typed_data()),
                        "RfdetrSelectRows");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrSelectRows, SelectRows,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::S32>>());

// ---- matcher ------------------------------------------------------------------------------------
// Cost weights as attributes (CriterionConfig's set_cost_* and focal_alpha, criterion.py:37-71).
#define RFDETR_COST_ATTRS                        \
    .Attr<float>("cost_class")                   \
        .Attr<float>("cost_bbox")                \
        .Attr<float>("cost_giou")                \
        .Attr<float>("focal_alpha")

// logits [B, Q, C], boxes [B, Q, 4], labels [B, T] int32, tboxes [B, T, 4] f32, mask [B, T] u8
// -> cost [B, Q, T] f32.  Replaces build_cost_matrix (matcher.py:44-141).
static ffi::Error MatchCost(cudaStream_t stream, ffi::AnyBuffer logits, ffi::AnyBuffer boxes,
                            ffi::Buffer<ffi::S32> labels, ffi::Buffer<ffi::F32> tboxes, ffi::Buffer<ffi::U8> mask,
                            float cost_class, float cost_bbox, float cost_giou, float focal_alpha,
                            ffi::Result<ffi::Buffer<ffi::F32>> cost) {
    return status_error(rfdetr_match_cost(stream, logits.untyped_data(), dtype_code(logits.element_type()),
                                          boxes.untyped_data(), dtype_code(boxes.element_type()), labels.typed_data(),
                                          tboxes.typed_data(), mask.typed_data(), cost->typed_data(), dim(logits, 0),
                                          dim(logits, 1), dim(logits, 2), dim(labels, 1), cost_class, cost_bbox,
                                          cost_giou, focal_alpha),
                        "RfdetrMatchCost");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMatchCost, MatchCost,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>() RFDETR_COST_ATTRS.Ret<ffi::Buffer<ffi::F32>>());

// cost [N, Q, T] f32, sizes [N] int32 -> rows, cols [N, G*T] int32, valid [N, G*T] u8,
// status int32[1].  Replaces hungarian_match / _solve_batch (matcher.py:144-208) with no host
// callback, so it runs per shard inside shard_map.
static ffi::Error LsapBatched(cudaStream_t stream, ffi::Buffer<ffi::F32> cost, ffi::Buffer<ffi::S32> sizes,
                              int64_t group_detr, ffi::Result<ffi::Buffer<ffi::S32>> rows,
                              ffi::Result<ffi::Buffer<ffi::S32>> cols, ffi::Result<ffi::Buffer<ffi::U8>> valid,
                              ffi::Result<ffi::Buffer<ffi::S32>> status) {
    if (cudaMemsetAsync(status->typed_data(), 0, sizeof(int32_t), stream) != cudaSuccess)
        return status_error(RFDETR_ERR_CUDA, "RfdetrLsapBatched");
    return status_error(rfdetr_lsap_batched(stream, cost.typed_data(), sizes.typed_data(), dim(cost, 0),
                                            dim(cost, 1), dim(cost, 2), group_detr, rows->typed_data(),
                                            cols->typed_data(), valid->typed_data(), status->typed_data()),
                        "RfdetrLsapBatched");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrLsapBatched, LsapBatched,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Attr<int64_t>("group_detr")
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::S32>>());

// Stacked layers: logits [L, B, Q, C], boxes [L, B, Q, 4], targets as MatchCost, sizes [B] ->
// cost [L, B, Q, T], rows/cols [L, B, G*T] int32, valid u8, status int32[1].  Replaces the
// stacked layer_cost + solve of compute_losses (criterion.py:402-413).
static ffi::Error MatchStacked(cudaStream_t stream, ffi::AnyBuffer logits, ffi::AnyBuffer boxes,
                               ffi::Buffer<ffi::S32> labels, ffi::Buffer<ffi::F32> tboxes, ffi::Buffer<ffi::U8> mask,
                               ffi::Buffer<ffi::S32> sizes, int64_t group_detr, float cost_class, float cost_bbox,
                               float cost_giou, float focal_alpha, ffi::Result<ffi::Buffer<ffi::F32>> cost,
                               ffi::Result<ffi::Buffer<ffi::S32>> rows, ffi::Result<ffi::Buffer<ffi::S32>> cols,
                               ffi::Result<ffi::Buffer<ffi::U8>> valid, ffi::Result<ffi::Buffer<ffi::S32>> status) {
    if (cudaMemsetAsync(status->typed_data(), 0, sizeof(int32_t), stream) != cudaSuccess)
        return status_error(RFDETR_ERR_CUDA, "RfdetrMatchStacked");
    return status_error(
        rfdetr_match_stacked(stream, logits.untyped_data(), dtype_code(logits.element_type()), boxes.untyped_data(),
                             dtype_code(boxes.element_type()), labels.typed_data(), tboxes.typed_data(),
                             mask.typed_data(), sizes.typed_data(), dim(logits, 0), dim(logits, 1), dim(logits, 2),
                             dim(logits, 3), dim(labels, 1), group_detr, cost_class, cost_bbox, cost_giou,
                             focal_alpha, cost->typed_data(), rows->typed_data(), cols->typed_data(),
                             valid->typed_data(), status->typed_data()),
        "RfdetrMatchStacked");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrMatchStacked, MatchStacked,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Attr<int64_t>("group_detr") RFDETR_COST_ATTRS.Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::S32>>());

// ---- set losses ---------------------------------------------------------------------------------
// logits [L, B, Q, C] f32, boxes [L, B, Q, 4] f32, labels [B, T], tboxes [B, T, 4], rows/cols
// [L, B, S] int32, valid [L, B, S] u8, num_boxes f32[1] -> losses [L, 3] f32, grad_logits
// [L, B, Q, C], grad_boxes_l1 / grad_boxes_giou [L, B, Q, 4].  Replaces loss_labels and
// loss_boxes (criterion.py:157-250).
static ffi::Error SetLosses(cudaStream_t stream, ffi::Buffer<ffi::F32> logits, ffi::Buffer<ffi::F32> boxes,
                            ffi::Buffer<ffi::S32> labels, ffi::Buffer<ffi::F32> tboxes, ffi::Buffer<ffi::S32> rows,
                            ffi::Buffer<ffi::S32> cols, ffi::Buffer<ffi::U8> valid, ffi::Buffer<ffi::F32> num_boxes,
                            float focal_alpha, int32_t ia_bce, ffi::Result<ffi::Buffer<ffi::F32>> losses,
                            ffi::Result<ffi::Buffer<ffi::F32>> grad_logits,
                            ffi::Result<ffi::Buffer<ffi::F32>> grad_boxes_l1,
                            ffi::Result<ffi::Buffer<ffi::F32>> grad_boxes_giou) {
    return status_error(
        rfdetr_set_losses(stream, logits.typed_data(), boxes.typed_data(), labels.typed_data(), tboxes.typed_data(),
                          rows.typed_data(), cols.typed_data(), valid.typed_data(), num_boxes.typed_data(),
                          dim(logits, 0), dim(logits, 1), dim(logits, 2), dim(logits, 3), dim(labels, 1),
                          dim(rows, 2), focal_alpha, ia_bce, losses->typed_data(), grad_logits->typed_data(),
                          grad_boxes_l1->typed_data(), grad_boxes_giou->typed_data()),
        "RfdetrSetLosses");
}
XLA_FFI_DEFINE_HANDLER_SYMBOL(RfdetrSetLosses, SetLosses,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Attr<float>("focal_alpha")
                                  .Attr<int32_t>("ia_bce")
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());
