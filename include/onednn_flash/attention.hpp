// onednn_flash/attention.hpp -- attention entry points, GPU (sm_100a) implementation.
//
// Drop-in for the reference's include/onednn_flash/attention.hpp (lines 13-85):
// the same types, fields and functions, computed by the B200 forward kernel.
// Pointer arguments may be host or device memory (detected per call); vector
// arguments are host memory.  All calls are synchronous, like the reference's.
//
// Semantics are those of flash_attention_qk_pv_tile_ws (attention.cpp:486-695):
// s = q.k * scale + bias, causal masking is top-left aligned, BlockMask blocks
// outside the bitmap are disallowed, and rows with no allowed key produce 0.
// Q/K/V are rounded to bf16 on the device; accumulation and softmax are fp32.
//
// Additions, all defaulted so existing code is unchanged:
//   AttentionOptions::bias_kind / alibi_slopes / softcap / kv_heads / lse
// Limits of the GPU path (reported as exceptions, like the reference's
// unavailable backends): head_dim == value_dim in {64, 128}; a ScoreBiasFn
// functor cannot run on the device (use bias_kind = BiasKind::AlibiGenerated).
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <vector>

#include "onednn_flash/attention_workspace.hpp"
#include "onednn_flash/score_mod_plan.hpp"
#include "onednn_flash/tile_kernel.hpp"

namespace onednn_flash {

struct AttentionShape {
    std::size_t query_tokens;
    std::size_t key_tokens;
    std::size_t head_dim;
    std::size_t value_dim;
};

struct BlockMask {
    std::size_t query_block_size = 1;
    std::size_t key_block_size = 1;
    std::size_t query_blocks = 0;
    std::size_t key_blocks = 0;
    // Row-major [query_blocks, key_blocks]; non-zero = allowed.
    std::vector<std::uint8_t> allowed;

    bool allows(std::size_t query_index, std::size_t key_index) const;
};

using ScoreBiasFn = std::function<float(std::size_t query_index, std::size_t key_index)>;

enum class QkTileLayout {
    CopiedTransposed,
    StridedK,
    BrgemmTransformedK,
};

struct AttentionOptions {
    float scale = 1.0f;
    bool causal = false;
    std::size_t key_block_size = 64;     // validated (non-zero); the GPU tiles are 128x128
    std::size_t query_block_size = 1;    // validated (non-zero)
    TileKernelKind qk_tile_kernel = TileKernelKind::Reference;  // accepted, ignored on the GPU
    TileKernelKind pv_tile_kernel = TileKernelKind::Reference;  // accepted, ignored on the GPU
    QkTileLayout qk_tile_layout = QkTileLayout::StridedK;       // accepted, ignored on the GPU
    const BlockMask* block_mask = nullptr;
    ScoreBiasFn score_bias = nullptr;    // host functor: rejected by the GPU path

    // ---- additions for the GPU path ----
    // Structured bias evaluated in the kernel's epilogue: BiasKind::None,
    // BiasKind::SameShapeTile (the `bias` tensor below) or BiasKind::AlibiGenerated
    // (bias = slope[h] * (kj - qi)).
    BiasKind bias_kind = BiasKind::None;
    // BiasKind::SameShapeTile: fp32 tensor in the same memory kind as q/k/v; element
    // (b, h, qi, kj) at bias[b*s0 + h*s1 + qi*s2 + kj*s3] with bias_strides = {s0..s3};
    // all zero = contiguous [B, H, M, N] (one [M, N] matrix for the single-head calls);
    // otherwise zero strides broadcast.
    const float* bias = nullptr;
    std::int64_t bias_strides[4] = {0, 0, 0, 0};
    // Host array of per-head ALiBi slopes; nullptr = 2^(-8 (h+1) / heads).
    const float* alibi_slopes = nullptr;
    // > 0: s <- softcap * tanh(s / softcap) after scale and bias.
    float softcap = 0.0f;
    // Batched calls only: K/V heads (0 = same as query heads); heads % kv_heads == 0.
    std::size_t kv_heads = 0;
    // Optional per-row natural-log LSE output ([B, H, M] fp32, same memory kind as the
    // tensors); -inf for rows with no allowed key.
    float* lse = nullptr;
};

std::vector<float> standard_attention(const std::vector<float>& q,
                                      const std::vector<float>& k,
                                      const std::vector<float>& v,
                                      const AttentionShape& shape,
                                      const AttentionOptions& options);

std::vector<float> flash_attention_tiled(const std::vector<float>& q,
                                         const std::vector<float>& k,
                                         const std::vector<float>& v,
                                         const AttentionShape& shape,
                                         const AttentionOptions& options);

std::vector<float> flash_attention_q_tile(const std::vector<float>& q,
                                          const std::vector<float>& k,
                                          const std::vector<float>& v,
                                          const AttentionShape& shape,
                                          const AttentionOptions& options);

std::vector<float> flash_attention_qk_pv_tile(const std::vector<float>& q,
                                              const std::vector<float>& k,
                                              const std::vector<float>& v,
                                              const AttentionShape& shape,
                                              const AttentionOptions& options);

float max_abs_diff(const std::vector<float>& a, const std::vector<float>& b);

// Raw-pointer path with caller-owned output and workspace (host or device pointers).
void flash_attention_qk_pv_tile_ws(const float* q,
                                   const float* k,
                                   const float* v,
                                   float* output,
                                   const AttentionShape& shape,
                                   const AttentionOptions& options,
                                   AttentionWorkspace& ws);

}  // namespace onednn_flash
