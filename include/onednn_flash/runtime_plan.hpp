// onednn_flash/runtime_plan.hpp -- runtime plan descriptors and planner.
//
// Same types and functions as the reference's include/onednn_flash/runtime_plan.hpp
// (lines 9-113); make_runtime_plan, make_block_mask_plan,
// make_causal_mask_tile_descriptor and make_runtime_plan_cache_key give the same
// results and strings as runtime_plan.cpp:72-199.  Additions (existing values
// unchanged): QkBackendKind::Sm100Tcgen05 and make_sm100_runtime_plan, which
// describes the plan the B200 kernel runs.
#pragma once

#include <string>

#include "onednn_flash/score_mod_plan.hpp"

namespace onednn_flash {

enum class BlockMaskKind {
    None,
    Causal,
    Unsupported,
};

enum class QkBackendKind {
    Reference,
    OneDnnMatmul,
    OneDnnBrgemmBaseline,
    Sm100Tcgen05,  // added: the sm_100a tcgen05 forward kernel
};

enum class QkLayoutKind {
    RowMajorKStrided,
    CopiedTransposedK,
    BrgemmTransformedKBaseline,
};

struct BlockMaskPlan {
    BlockMaskKind kind{BlockMaskKind::None};
    bool has_boundary_tiles{false};
    bool can_skip_tiles{false};
    bool requires_mask_tile_generator{false};
    FallbackReason fallback_reason{FallbackReason::None};
    std::string signature{"none"};
};

struct MaskTileDescriptor {
    bool required{false};
    int q_start{0};
    int k_start{0};
    int q_size{0};
    int k_size{0};
    float masked_value{0.0f};
    bool all_masked_row_possible{false};
};

struct RuntimePlanInput {
    int batch{1};
    int heads{1};
    int query_length{0};
    int key_length{0};
    int head_dim{0};
    int value_dim{0};

    DataType q_dtype{DataType::F32};
    DataType k_dtype{DataType::F32};
    DataType v_dtype{DataType::F32};
    DataType out_dtype{DataType::F32};

    ScoreModKind requested_score_mod{ScoreModKind::None};
    bool has_scale{false};
    float scale_value{1.0f};
    BiasKind requested_bias_kind{BiasKind::None};

    BlockMaskKind requested_block_mask{BlockMaskKind::None};

    bool force_reference{false};
    bool enable_onednn{true};
    bool enable_debug{false};
};

struct RuntimePlanCacheKey {
    std::string semantic_shape;
    std::string dtype_signature;
    std::string score_mod_signature;
    std::string block_mask_signature;
    std::string policy_signature;
};

struct RuntimePlan {
    RuntimePlanInput input;

    ScoreModPlan score_mod_plan;
    BlockMaskPlan block_mask_plan;

    QkBackendKind qk_backend{QkBackendKind::Reference};
    QkLayoutKind qk_layout{QkLayoutKind::RowMajorKStrided};
    LoweringStatus qk_lowering_status{LoweringStatus::ReferenceFallback};

    bool uses_onednn_post_ops{false};
    bool requires_onednn_flash_epilogue{false};
    bool requires_mask_tile_generator{false};

    FallbackReason fallback_reason{FallbackReason::None};

    std::string runtime_plan_signature;
    std::string debug_summary;
};

const char* to_string(BlockMaskKind value);
const char* to_string(QkBackendKind value);
const char* to_string(QkLayoutKind value);

BlockMaskPlan make_block_mask_plan(BlockMaskKind requested_kind,
                                   int query_length,
                                   int key_length);
MaskTileDescriptor make_causal_mask_tile_descriptor(int q_start,
                                                    int k_start,
                                                    int q_size,
                                                    int k_size);
RuntimePlan make_runtime_plan(const RuntimePlanInput& input,
                              bool one_dnn_available,
                              bool one_dnn_post_ops_available);
RuntimePlanCacheKey make_runtime_plan_cache_key(const RuntimePlan& plan);

// Plan of the sm_100a kernel for `input` (+ soft-cap): qk_backend Sm100Tcgen05 when
// the shape, dtypes (F32 or BF16) and score_mod run on the GPU, else the fallback
// reason that stops it (UnsupportedShape for head_dim/value_dim outside {64,128} or
// head_dim != value_dim).  The signature uses the reference's format.
RuntimePlan make_sm100_runtime_plan(const RuntimePlanInput& input, float softcap = 0.0f);

}  // namespace onednn_flash
