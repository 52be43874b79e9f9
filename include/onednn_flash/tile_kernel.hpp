// onednn_flash/tile_kernel.hpp -- tile-GEMM descriptors of the reference API.
//
// Mirrors include/onednn_flash/tile_kernel.hpp of the reference (lines 12-34):
// the shape structs and the TileKernelKind selector stay so existing option
// structs compile unchanged.  On the GPU both tile GEMMs of the attention loop
// are tcgen05 MMAs inside the forward kernel, so the kind is accepted and
// ignored; the reference's standalone matmul_tile* CPU helpers are not part of
// this library.
#pragma once

#include <cstddef>

namespace onednn_flash {

struct MatmulShape {
    std::size_t m;
    std::size_t n;
    std::size_t k;
};

struct StridedMatmulShape {
    std::size_t m;
    std::size_t n;
    std::size_t k;
    std::size_t a_stride_m;
    std::size_t a_stride_k;
    std::size_t b_stride_k;
    std::size_t b_stride_n;
    std::size_t c_stride_m;
    std::size_t c_stride_n;
};

enum class TileKernelKind {
    Reference,
    OneDnn,
    OneDnnBrgemm,
};

// "reference", "onednn", "onednn_brgemm" (tile_kernel.cpp:19-29 of the reference).
const char* tile_kernel_name(TileKernelKind kind);

}  // namespace onednn_flash
