// onednn_flash/attention_workspace.hpp -- caller-owned scratch of the workspace path.
//
// Keeps the members and resize() of the reference's AttentionWorkspace
// (include/onednn_flash/attention_workspace.hpp:16-47) so callers that size it
// keep compiling.  On the GPU the per-tile buffers live in shared and tensor
// memory inside the kernel; what the workspace still owns is the device staging
// a call with fp32 device pointers needs (bf16 copies of Q/K/V, the uploaded
// BlockMask, the block-mask tile lists), held in `device` and grown on demand.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

namespace onednn_flash {

struct DeviceStaging;  // defined by the library; freed with the workspace

struct AttentionWorkspace {
    // Tile buffers of the reference's CPU loop (kept for API compatibility).
    std::vector<float> q_tile;
    std::vector<float> k_tile_t;
    std::vector<float> v_tile;
    std::vector<float> score_tile;
    std::vector<float> p_tile;
    std::vector<float> pv_tile;

    // Per-query-row state of the reference's CPU loop (kept for API compatibility).
    std::vector<float> running_max;
    std::vector<float> running_sum;
    std::vector<float> acc;
    std::vector<float> old_scales;
    std::vector<float> new_maxes;
    std::vector<float> block_sums;
    std::vector<std::uint8_t> row_has_valid;

    // Device staging used by the GPU path (created on first use).
    std::shared_ptr<DeviceStaging> device;

    // Sizes the host tile buffers as the reference does (attention_workspace.cpp:5-20).
    void resize(std::size_t q_block_size, std::size_t k_block_size,
                std::size_t head_dim, std::size_t value_dim);
};

}  // namespace onednn_flash
