// onednn_flash/backend.hpp -- backend selector of the reference API.
//
// Mirrors include/onednn_flash/backend.hpp (lines 7-19) of the reference: the
// standard (materialising) and flash-tiled entry points.  On the GPU both run the
// same tiled forward kernel; the names are kept so logs and callers are unchanged.
#pragma once

#include <vector>

#include "onednn_flash/attention.hpp"

namespace onednn_flash {

enum class AttentionBackendKind {
    StandardReference,
    FlashTiledReference,
};

// "standard_reference" / "flash_tiled_reference" (backend.cpp:5-14 of the reference).
const char* backend_name(AttentionBackendKind kind);

std::vector<float> run_attention(AttentionBackendKind kind,
                                 const std::vector<float>& q,
                                 const std::vector<float>& k,
                                 const std::vector<float>& v,
                                 const AttentionShape& shape,
                                 const AttentionOptions& options);

}  // namespace onednn_flash
