// planner.cpp -- score_mod / runtime plan descriptors of the C++ API.
//
// make_score_mod_plan, make_block_mask_plan, make_causal_mask_tile_descriptor,
// make_runtime_plan and make_runtime_plan_cache_key return the same decisions and
// strings as the reference planner (src/onednn_flash/score_mod_plan.cpp:115-182,
// runtime_plan.cpp:72-199), so existing logs and plan caches keep their keys; the
// stage-1 planner accepts F32 only and routes every non-SameShapeTile bias to the
// epilogue, exactly as there.  make_sm100_* describe what the B200 kernel runs.
#include <limits>
#include <sstream>
#include <string>

#include "onednn_flash/runtime_plan.hpp"
#include "onednn_flash/score_mod_plan.hpp"

namespace onednn_flash {

namespace {

template <typename E, std::size_t N>
const char* name_of(E value, const char* const (&names)[N]) {
    const auto i = static_cast<std::size_t>(value);
    return i < N ? names[i] : "unknown";
}

constexpr const char* kDataTypeNames[] = {"f32", "bf16", "unsupported"};
constexpr const char* kScoreModNames[] = {"none", "scale", "additive_bias", "scale_additive_bias", "unsupported"};
constexpr const char* kBiasNames[] = {"none", "same_shape_tile", "broadcast_row", "broadcast_col",
                                      "alibi_generated", "unsupported"};
constexpr const char* kLoweringNames[] = {"lowered_to_onednn_post_ops", "partially_lowered", "onednn_flash_epilogue",
                                          "reference_fallback", "unsupported"};
constexpr const char* kFallbackNames[] = {"none",
                                          "onednn_disabled",
                                          "onednn_unavailable",
                                          "unsupported_dtype",
                                          "unsupported_shape",
                                          "unsupported_score_mod",
                                          "unsupported_block_mask",
                                          "unsupported_post_op",
                                          "unsupported_bias_layout",
                                          "unsupported_broadcast",
                                          "unsupported_edge_tile",
                                          "numerical_safety_fallback",
                                          "debug_forced_reference"};
constexpr const char* kBlockMaskNames[] = {"none", "causal", "unsupported"};
constexpr const char* kQkBackendNames[] = {"reference", "onednn_matmul", "onednn_brgemm_baseline", "sm100_tcgen05"};
constexpr const char* kQkLayoutNames[] = {"row_major_k_strided", "copied_transposed_k",
                                          "brgemm_transformed_k_baseline"};

std::string unsupported_signature(FallbackReason reason) {
    return std::string("unsupported:") + to_string(reason);
}

std::string score_mod_signature(ScoreModKind kind, BiasKind bias, DataType dtype, FallbackReason reason) {
    switch (kind) {
        case ScoreModKind::None: return "none";
        case ScoreModKind::Scale: return std::string("scale:") + to_string(dtype);
        case ScoreModKind::AdditiveBias:
            return std::string("additive_bias:") + to_string(bias) + ':' + to_string(dtype);
        case ScoreModKind::ScaleAdditiveBias:
            return std::string("scale_additive_bias:") + to_string(bias) + ':' + to_string(dtype);
        case ScoreModKind::Unsupported: return unsupported_signature(reason);
    }
    return "none";
}

bool shape_ok(const RuntimePlanInput& in) {
    return in.batch > 0 && in.heads > 0 && in.query_length > 0 && in.key_length > 0 && in.head_dim > 0 &&
           in.value_dim > 0;
}

std::string shape_key(const RuntimePlanInput& in) {
    std::ostringstream os;
    os << 'b' << in.batch << 'h' << in.heads << 'm' << in.query_length << 'n' << in.key_length << 'd' << in.head_dim
       << "dv" << in.value_dim;
    return os.str();
}

std::string dtype_key(const RuntimePlanInput& in) {
    return std::string("q") + to_string(in.q_dtype) + 'k' + to_string(in.k_dtype) + 'v' + to_string(in.v_dtype) +
           'o' + to_string(in.out_dtype);
}

void finish_plan(RuntimePlan& plan) {
    plan.requires_mask_tile_generator = plan.block_mask_plan.requires_mask_tile_generator;
    plan.requires_onednn_flash_epilogue =
        plan.requires_mask_tile_generator || plan.score_mod_plan.lowering_status == LoweringStatus::OneDNNFlashEpilogue;
    plan.runtime_plan_signature = shape_key(plan.input) + '|' + dtype_key(plan.input) + '|' +
                                  plan.score_mod_plan.signature + '|' + plan.block_mask_plan.signature + '|' +
                                  to_string(plan.qk_backend) + '|' + to_string(plan.qk_layout);
    plan.debug_summary = std::string("RuntimePlan{backend=") + to_string(plan.qk_backend) +
                         ", layout=" + to_string(plan.qk_layout) + ", score_mod=" + plan.score_mod_plan.signature +
                         ", block_mask=" + plan.block_mask_plan.signature +
                         ", fallback=" + to_string(plan.fallback_reason) + '}';
}

}  // namespace

const char* to_string(DataType value) { return name_of(value, kDataTypeNames); }
const char* to_string(ScoreModKind value) { return name_of(value, kScoreModNames); }
const char* to_string(BiasKind value) { return name_of(value, kBiasNames); }
const char* to_string(LoweringStatus value) { return name_of(value, kLoweringNames); }
const char* to_string(FallbackReason value) { return name_of(value, kFallbackNames); }
const char* to_string(BlockMaskKind value) { return name_of(value, kBlockMaskNames); }
const char* to_string(QkBackendKind value) { return name_of(value, kQkBackendNames); }
const char* to_string(QkLayoutKind value) { return name_of(value, kQkLayoutNames); }

ScoreModPlan make_score_mod_plan(ScoreModKind requested_kind, DataType dtype, bool has_scale, float scale_value,
                                 BiasKind requested_bias_kind, bool one_dnn_post_ops_available) {
    ScoreModPlan plan;
    plan.kind = requested_kind;
    plan.dtype = dtype;
    plan.has_scale = has_scale;
    plan.scale_value = has_scale ? scale_value : 1.0f;
    plan.bias_kind = requested_bias_kind;
    plan.has_bias = requested_bias_kind != BiasKind::None;

    // Stage-1 planner: fp32 only, every rejection falls back to the reference.
    if (dtype != DataType::F32) {
        plan.kind = ScoreModKind::Unsupported;
        plan.lowering_status = LoweringStatus::ReferenceFallback;
        plan.fallback_reason = FallbackReason::UnsupportedDType;
        plan.signature = unsupported_signature(plan.fallback_reason);
        return plan;
    }
    if (requested_kind == ScoreModKind::Unsupported) {
        plan.lowering_status = LoweringStatus::ReferenceFallback;
        plan.fallback_reason = FallbackReason::UnsupportedScoreMod;
        plan.signature = unsupported_signature(plan.fallback_reason);
        return plan;
    }
    if (plan.has_bias && requested_bias_kind != BiasKind::SameShapeTile) {
        const bool broadcast =
            requested_bias_kind == BiasKind::BroadcastRow || requested_bias_kind == BiasKind::BroadcastCol;
        plan.lowering_status = LoweringStatus::OneDNNFlashEpilogue;
        plan.fallback_reason = broadcast ? FallbackReason::UnsupportedBroadcast : FallbackReason::UnsupportedBiasLayout;
        plan.signature = unsupported_signature(plan.fallback_reason);
        return plan;
    }
    const bool to_epilogue = !one_dnn_post_ops_available && requested_kind != ScoreModKind::None;
    plan.lowering_status = to_epilogue ? LoweringStatus::OneDNNFlashEpilogue : LoweringStatus::LoweredToOneDnnPostOps;
    plan.fallback_reason = to_epilogue ? FallbackReason::UnsupportedPostOp : FallbackReason::None;
    plan.signature = score_mod_signature(requested_kind, requested_bias_kind, dtype, plan.fallback_reason);
    return plan;
}

ScoreModPlan make_sm100_score_mod_plan(ScoreModKind requested_kind, DataType dtype, bool has_scale, float scale_value,
                                       BiasKind requested_bias_kind, float softcap) {
    ScoreModPlan plan;
    plan.kind = requested_kind;
    plan.dtype = dtype;
    plan.has_scale = has_scale;
    plan.scale_value = has_scale ? scale_value : 1.0f;
    plan.bias_kind = requested_bias_kind;
    plan.has_bias = requested_bias_kind != BiasKind::None;
    plan.lowering_status = LoweringStatus::OneDNNFlashEpilogue;  // the kernel's register epilogue
    if (dtype != DataType::F32 && dtype != DataType::BF16) {
        plan.kind = ScoreModKind::Unsupported;
        plan.lowering_status = LoweringStatus::Unsupported;
        plan.fallback_reason = FallbackReason::UnsupportedDType;
        plan.signature = unsupported_signature(plan.fallback_reason);
        return plan;
    }
    if (requested_kind == ScoreModKind::Unsupported || !(softcap >= 0.0f)) {
        plan.lowering_status = LoweringStatus::Unsupported;
        plan.fallback_reason = FallbackReason::UnsupportedScoreMod;
        plan.signature = unsupported_signature(plan.fallback_reason);
        return plan;
    }
    if (plan.has_bias && requested_bias_kind != BiasKind::AlibiGenerated &&
        requested_bias_kind != BiasKind::SameShapeTile) {
        // row/column broadcasts are SameShapeTile tensors with zero strides on this path
        const bool broadcast =
            requested_bias_kind == BiasKind::BroadcastRow || requested_bias_kind == BiasKind::BroadcastCol;
        plan.lowering_status = LoweringStatus::Unsupported;
        plan.fallback_reason = broadcast ? FallbackReason::UnsupportedBroadcast : FallbackReason::UnsupportedBiasLayout;
        plan.signature = unsupported_signature(plan.fallback_reason);
        return plan;
    }
    plan.fallback_reason = FallbackReason::None;
    plan.signature = score_mod_signature(requested_kind, requested_bias_kind, dtype, plan.fallback_reason);
    if (softcap > 0.0f) plan.signature += ":softcap";
    return plan;
}

BlockMaskPlan make_block_mask_plan(BlockMaskKind requested_kind, int query_length, int key_length) {
    BlockMaskPlan plan;
    plan.kind = requested_kind;
    switch (requested_kind) {
        case BlockMaskKind::None:
            plan.signature = "none";
            return plan;
        case BlockMaskKind::Causal:
            plan.has_boundary_tiles = true;
            plan.can_skip_tiles = key_length > query_length;
            plan.requires_mask_tile_generator = true;
            plan.signature = "causal";
            return plan;
        default:
            plan.kind = BlockMaskKind::Unsupported;
            plan.fallback_reason = FallbackReason::UnsupportedBlockMask;
            plan.signature = "unsupported:unsupported_block_mask";
            return plan;
    }
}

MaskTileDescriptor make_causal_mask_tile_descriptor(int q_start, int k_start, int q_size, int k_size) {
    MaskTileDescriptor d;
    d.required = true;
    d.q_start = q_start;
    d.k_start = k_start;
    d.q_size = q_size;
    d.k_size = k_size;
    d.masked_value = -std::numeric_limits<float>::infinity();
    // Some row of the tile sees no key at or before it only if the first key is
    // beyond the last query of the tile.
    d.all_masked_row_possible = k_start > q_start + q_size - 1;
    return d;
}

RuntimePlan make_runtime_plan(const RuntimePlanInput& input, bool one_dnn_available, bool one_dnn_post_ops_available) {
    RuntimePlan plan;
    plan.input = input;
    const bool valid_shape = shape_ok(input);
    const bool f32_only = input.q_dtype == DataType::F32 && input.k_dtype == DataType::F32 &&
                          input.v_dtype == DataType::F32 && input.out_dtype == DataType::F32;
    const bool use_onednn =
        input.enable_onednn && one_dnn_available && !input.force_reference && valid_shape && f32_only;

    plan.score_mod_plan = make_score_mod_plan(input.requested_score_mod, input.q_dtype, input.has_scale,
                                              input.scale_value, input.requested_bias_kind,
                                              use_onednn && one_dnn_post_ops_available);
    plan.block_mask_plan = make_block_mask_plan(input.requested_block_mask, input.query_length, input.key_length);

    // First failing condition wins, in the reference's order.
    if (!valid_shape) plan.fallback_reason = FallbackReason::UnsupportedShape;
    else if (!f32_only) plan.fallback_reason = FallbackReason::UnsupportedDType;
    else if (input.force_reference) plan.fallback_reason = FallbackReason::DebugForcedReference;
    else if (!input.enable_onednn) plan.fallback_reason = FallbackReason::OneDnnDisabled;
    else if (!one_dnn_available) plan.fallback_reason = FallbackReason::OneDnnUnavailable;
    else if (plan.score_mod_plan.fallback_reason != FallbackReason::None)
        plan.fallback_reason = plan.score_mod_plan.fallback_reason;
    else plan.fallback_reason = plan.block_mask_plan.fallback_reason;

    const bool lowered = use_onednn && plan.score_mod_plan.lowering_status == LoweringStatus::LoweredToOneDnnPostOps &&
                         plan.block_mask_plan.fallback_reason == FallbackReason::None;
    plan.qk_backend = lowered ? QkBackendKind::OneDnnMatmul : QkBackendKind::Reference;
    plan.qk_layout = QkLayoutKind::RowMajorKStrided;
    plan.qk_lowering_status = lowered ? LoweringStatus::LoweredToOneDnnPostOps : LoweringStatus::ReferenceFallback;
    plan.uses_onednn_post_ops = lowered && input.requested_score_mod != ScoreModKind::None;
    finish_plan(plan);
    return plan;
}

RuntimePlanCacheKey make_runtime_plan_cache_key(const RuntimePlan& plan) {
    RuntimePlanCacheKey key;
    key.semantic_shape = shape_key(plan.input);
    key.dtype_signature = dtype_key(plan.input);
    key.score_mod_signature = plan.score_mod_plan.signature;
    key.block_mask_signature = plan.block_mask_plan.signature;
    key.policy_signature = std::string("force_reference=") + (plan.input.force_reference ? "true" : "false") +
                           ";enable_onednn=" + (plan.input.enable_onednn ? "true" : "false") +
                           ";backend=" + to_string(plan.qk_backend) + ";layout=" + to_string(plan.qk_layout);
    return key;
}

RuntimePlan make_sm100_runtime_plan(const RuntimePlanInput& input, float softcap) {
    RuntimePlan plan;
    plan.input = input;
    const auto gpu_dtype = [](DataType t) { return t == DataType::F32 || t == DataType::BF16; };
    const bool valid_shape = shape_ok(input) && input.head_dim == input.value_dim &&
                             (input.head_dim == 64 || input.head_dim == 128);
    const bool dtypes_ok = gpu_dtype(input.q_dtype) && gpu_dtype(input.k_dtype) && gpu_dtype(input.v_dtype) &&
                           gpu_dtype(input.out_dtype);
    plan.score_mod_plan = make_sm100_score_mod_plan(input.requested_score_mod, input.q_dtype, input.has_scale,
                                                    input.scale_value, input.requested_bias_kind, softcap);
    plan.block_mask_plan = make_block_mask_plan(input.requested_block_mask, input.query_length, input.key_length);
    if (plan.block_mask_plan.kind == BlockMaskKind::Causal) {
        plan.block_mask_plan.can_skip_tiles = true;  // fully masked 128x128 tiles are never loaded
    }
    if (!valid_shape) plan.fallback_reason = FallbackReason::UnsupportedShape;
    else if (!dtypes_ok) plan.fallback_reason = FallbackReason::UnsupportedDType;
    else if (plan.score_mod_plan.fallback_reason != FallbackReason::None)
        plan.fallback_reason = plan.score_mod_plan.fallback_reason;
    else plan.fallback_reason = plan.block_mask_plan.fallback_reason;
    const bool runs = plan.fallback_reason == FallbackReason::None;
    plan.qk_backend = runs ? QkBackendKind::Sm100Tcgen05 : QkBackendKind::Reference;
    plan.qk_layout = QkLayoutKind::RowMajorKStrided;
    plan.qk_lowering_status = runs ? LoweringStatus::OneDNNFlashEpilogue : LoweringStatus::Unsupported;
    plan.uses_onednn_post_ops = false;
    finish_plan(plan);
    return plan;
}

}  // namespace onednn_flash
