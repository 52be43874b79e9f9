// onednn_flash/score_mod_plan.hpp -- score_mod descriptors and planner.
//
// Same enums, struct and planner as the reference's
// include/onednn_flash/score_mod_plan.hpp (lines 7-81), with identical values,
// strings and decisions (make_score_mod_plan follows score_mod_plan.cpp:115-182),
// so plan signatures and logs stay comparable.  The GPU epilogue itself is
// described by make_sm100_score_mod_plan, an addition.
#pragma once

#include <string>

namespace onednn_flash {

enum class DataType {
    F32,
    BF16,
    Unsupported,
};

enum class ScoreModKind {
    None,
    Scale,
    AdditiveBias,
    ScaleAdditiveBias,
    Unsupported,
};

enum class BiasKind {
    None,
    SameShapeTile,
    BroadcastRow,
    BroadcastCol,
    AlibiGenerated,
    Unsupported,
};

enum class LoweringStatus {
    LoweredToOneDnnPostOps,
    PartiallyLowered,
    OneDNNFlashEpilogue,
    ReferenceFallback,
    Unsupported,
};

enum class FallbackReason {
    None,
    OneDnnDisabled,
    OneDnnUnavailable,
    UnsupportedDType,
    UnsupportedShape,
    UnsupportedScoreMod,
    UnsupportedBlockMask,
    UnsupportedPostOp,
    UnsupportedBiasLayout,
    UnsupportedBroadcast,
    UnsupportedEdgeTile,
    NumericalSafetyFallback,
    DebugForcedReference,
};

struct ScoreModPlan {
    ScoreModKind kind{ScoreModKind::None};
    DataType dtype{DataType::F32};

    bool has_scale{false};
    float scale_value{1.0f};

    BiasKind bias_kind{BiasKind::None};
    bool has_bias{false};

    LoweringStatus lowering_status{LoweringStatus::LoweredToOneDnnPostOps};
    FallbackReason fallback_reason{FallbackReason::None};

    std::string signature{"none"};
};

const char* to_string(DataType value);
const char* to_string(ScoreModKind value);
const char* to_string(BiasKind value);
const char* to_string(LoweringStatus value);
const char* to_string(FallbackReason value);

ScoreModPlan make_score_mod_plan(ScoreModKind requested_kind,
                                 DataType dtype,
                                 bool has_scale,
                                 float scale_value,
                                 BiasKind requested_bias_kind,
                                 bool one_dnn_post_ops_available);

// GPU (sm_100a) plan of the register epilogue: accepts F32 and BF16, scale,
// BiasKind::None / AlibiGenerated / SameShapeTile (a strided fp32 bias tensor,
// whose zero strides also express row and column broadcasts), and an optional
// soft-cap.  BroadcastRow / BroadcastCol report FallbackReason::UnsupportedBroadcast
// (pass them as a SameShapeTile tensor with zero strides), every other bias layout
// FallbackReason::UnsupportedBiasLayout.  Signatures extend the reference's format
// with ":softcap" when a soft-cap is requested.
ScoreModPlan make_sm100_score_mod_plan(ScoreModKind requested_kind,
                                       DataType dtype,
                                       bool has_scale,
                                       float scale_value,
                                       BiasKind requested_bias_kind,
                                       float softcap);

}  // namespace onednn_flash
