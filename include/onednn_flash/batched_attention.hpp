// onednn_flash/batched_attention.hpp -- batched entry point (the TensorFlow op's call).
//
// Mirrors include/onednn_flash/batched_attention.hpp (lines 9-31) of the reference.
// Flat row-major tensors:
//   Q: [B, H, M, D]   K: [B, Hkv, N, D]   V: [B, Hkv, N, Dv]   O: [B, H, M, Dv]
// with Hkv = options.kv_heads (0 = H, as in the reference).  Pointers may be host
// or device memory.  The reference loops over B*H serially; here all heads run in
// one kernel launch (host buffers are streamed through the GPU in chunks with the
// copies overlapped).  A thread-local workspace holds the device staging, so
// repeated calls do not allocate.
#pragma once

#include <cstddef>

#include "onednn_flash/attention.hpp"

namespace onednn_flash {

struct BatchedAttentionShape {
    std::size_t batch;
    std::size_t heads;
    std::size_t query_tokens;
    std::size_t key_tokens;
    std::size_t head_dim;
    std::size_t value_dim;
};

void flash_attention_batched_qk_pv_tile(const float* q,
                                        const float* k,
                                        const float* v,
                                        float* out,
                                        const BatchedAttentionShape& shape,
                                        const AttentionOptions& options);

}  // namespace onednn_flash
