// onednn_flash_api.cpp -- the reference's C++ API (include/onednn_flash/*.hpp) on the GPU.
//
// Every attention entry point validates its arguments with the reference's checks
// and messages (src/onednn_flash/attention.cpp:18-38, 145-147, 229-234, 493-505;
// batched_attention.cpp:15-21), then runs the sm_100a forward through the C ABI
// (include/odf_sm100.h):
//   - host pointers / vectors -> odf_flash_fwd_host (fp32 in, streamed in chunks)
//   - device pointers         -> fp32->bf16 staging + odf_flash_fwd_sm100
// Errors surface as the reference's exception types: std::invalid_argument for bad
// arguments, std::runtime_error for anything the GPU path cannot run.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "odf_sm100.h"
#include "onednn_flash/attention.hpp"
#include "onednn_flash/attention_workspace.hpp"
#include "onednn_flash/backend.hpp"
#include "onednn_flash/batched_attention.hpp"
#include "onednn_flash/tile_kernel.hpp"

namespace onednn_flash {

// Device staging owned by an AttentionWorkspace: grown on demand, freed with it.
struct DeviceStaging {
    enum Slot { kQ, kK, kV, kMask, kLists, kCount };
    int device = -1;
    void* buf[kCount] = {};
    size_t cap[kCount] = {};

    ~DeviceStaging() {
        for (void* b : buf)
            if (b) cudaFree(b);
    }
    void* reserve(Slot slot, size_t bytes) {
        if (bytes == 0) return nullptr;
        if (cap[slot] < bytes) {
            if (buf[slot]) cudaFree(buf[slot]);
            buf[slot] = nullptr;
            cap[slot] = 0;
            if (cudaMalloc(&buf[slot], bytes) != cudaSuccess) {
                cudaGetLastError();
                throw std::runtime_error("GPU attention: cudaMalloc of device staging failed");
            }
            cap[slot] = bytes;
        }
        return buf[slot];
    }
};

// ---------------------------------------------------------------- small helpers
bool BlockMask::allows(std::size_t query_index, std::size_t key_index) const {
    if (query_block_size == 0 || key_block_size == 0) {
        throw std::invalid_argument("BlockMask block sizes must be non-zero");
    }
    if (query_blocks == 0 || key_blocks == 0) {
        throw std::invalid_argument("BlockMask dimensions must be non-zero");
    }
    if (allowed.size() != query_blocks * key_blocks) {
        throw std::invalid_argument("BlockMask allowed bitmap size does not match dimensions");
    }
    const std::size_t qb = query_index / query_block_size;
    const std::size_t kb = key_index / key_block_size;
    return qb < query_blocks && kb < key_blocks && allowed[qb * key_blocks + kb] != 0;
}

void AttentionWorkspace::resize(std::size_t q_block_size, std::size_t k_block_size, std::size_t head_dim,
                                std::size_t value_dim) {
    q_tile.resize(q_block_size * head_dim);
    k_tile_t.resize(head_dim * k_block_size);
    v_tile.resize(k_block_size * value_dim);
    score_tile.resize(q_block_size * k_block_size);
    p_tile.resize(q_block_size * k_block_size);
    pv_tile.resize(q_block_size * value_dim);
    for (auto* row : {&running_max, &running_sum, &old_scales, &new_maxes, &block_sums}) row->resize(q_block_size);
    acc.resize(q_block_size * value_dim);
    row_has_valid.resize(q_block_size);
}

const char* tile_kernel_name(TileKernelKind kind) {
    switch (kind) {
        case TileKernelKind::Reference: return "reference";
        case TileKernelKind::OneDnn: return "onednn";
        case TileKernelKind::OneDnnBrgemm: return "onednn_brgemm";
    }
    return "unknown";
}

const char* backend_name(AttentionBackendKind kind) {
    switch (kind) {
        case AttentionBackendKind::StandardReference: return "standard_reference";
        case AttentionBackendKind::FlashTiledReference: return "flash_tiled_reference";
    }
    return "unknown";
}

float max_abs_diff(const std::vector<float>& a, const std::vector<float>& b) {
    if (a.size() != b.size()) {
        throw std::invalid_argument("Cannot compare vectors with different sizes");
    }
    float diff = 0.0f;
    for (std::size_t i = 0; i < a.size(); ++i) diff = std::max(diff, std::fabs(a[i] - b[i]));
    return diff;
}

namespace {

[[noreturn]] void throw_status(int rc, const char* what) {
    const std::string msg = std::string(what) + ": " + odf_last_error();
    if (rc == ODF_ERR_INVALID_ARG) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string("GPU attention: ") + what + ": " + cudaGetErrorString(e));
    }
}

bool on_device(const void* p) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();  // unregistered host memory
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

void validate_vectors(const std::vector<float>& q, const std::vector<float>& k, const std::vector<float>& v,
                      const AttentionShape& shape) {
    if (q.size() != shape.query_tokens * shape.head_dim) throw std::invalid_argument("Q size does not match shape");
    if (k.size() != shape.key_tokens * shape.head_dim) throw std::invalid_argument("K size does not match shape");
    if (v.size() != shape.key_tokens * shape.value_dim) throw std::invalid_argument("V size does not match shape");
    if (shape.query_tokens == 0 || shape.key_tokens == 0 || shape.head_dim == 0 || shape.value_dim == 0) {
        throw std::invalid_argument("Attention dimensions must be non-zero");
    }
}

void validate_mask(const BlockMask* mask) {
    if (!mask) return;
    if (mask->query_block_size == 0 || mask->key_block_size == 0)
        throw std::invalid_argument("BlockMask block sizes must be non-zero");
    if (mask->query_blocks == 0 || mask->key_blocks == 0)
        throw std::invalid_argument("BlockMask dimensions must be non-zero");
    if (mask->allowed.size() != mask->query_blocks * mask->key_blocks)
        throw std::invalid_argument("BlockMask allowed bitmap size does not match dimensions");
}

struct Problem {
    std::size_t batch, heads, kv_heads, m, n, d, dv;
};

// One forward over [B, H, M, D] fp32 tensors (all host or all device memory).
void run_forward(const float* q, const float* k, const float* v, float* out, const Problem& pb,
                 const AttentionOptions& opt, AttentionWorkspace& ws) {
    if (opt.score_bias) {
        throw std::runtime_error(
            "GPU attention: AttentionOptions::score_bias is a host functor and cannot run on the device; "
            "use bias_kind = BiasKind::AlibiGenerated or BiasKind::SameShapeTile");
    }
    if (opt.bias_kind != BiasKind::None && opt.bias_kind != BiasKind::AlibiGenerated &&
        opt.bias_kind != BiasKind::SameShapeTile) {
        throw std::runtime_error(std::string("GPU attention: bias kind ") + to_string(opt.bias_kind) +
                                 " is not supported on the device");
    }
    validate_mask(opt.block_mask);
    const std::size_t kvh = pb.kv_heads ? pb.kv_heads : pb.heads;
    if (pb.heads % kvh != 0) throw std::invalid_argument("heads must be a multiple of kv_heads");

    odf_fwd_params p;
    std::memset(&p, 0, sizeof(p));
    p.o_dtype = ODF_DTYPE_F32;
    p.batch = static_cast<int64_t>(pb.batch);
    p.heads_q = static_cast<int64_t>(pb.heads);
    p.heads_kv = static_cast<int64_t>(kvh);
    p.seqlen_q = static_cast<int64_t>(pb.m);
    p.seqlen_k = static_cast<int64_t>(pb.n);
    p.head_dim = static_cast<int64_t>(pb.d);
    p.value_dim = static_cast<int64_t>(pb.dv);
    p.scale = opt.scale;
    p.causal = opt.causal ? 1 : 0;
    p.bias_kind = opt.bias_kind == BiasKind::AlibiGenerated ? ODF_BIAS_ALIBI
                  : opt.bias_kind == BiasKind::SameShapeTile ? ODF_BIAS_SAME_SHAPE
                                                             : ODF_BIAS_NONE;
    p.alibi_slopes = opt.alibi_slopes;
    if (opt.bias_kind == BiasKind::SameShapeTile) {
        if (opt.bias == nullptr) throw std::invalid_argument("BiasKind::SameShapeTile needs AttentionOptions::bias");
        p.bias = opt.bias;
        for (int i = 0; i < 4; ++i) p.bias_strides[i] = opt.bias_strides[i];
    }
    p.softcap = opt.softcap;
    p.lse = opt.lse;
    if (opt.block_mask) {
        p.mask_qbs = static_cast<int64_t>(opt.block_mask->query_block_size);
        p.mask_kbs = static_cast<int64_t>(opt.block_mask->key_block_size);
        p.mask_qblocks = static_cast<int64_t>(opt.block_mask->query_blocks);
        p.mask_kblocks = static_cast<int64_t>(opt.block_mask->key_blocks);
    }

    const bool dq = on_device(q), dk = on_device(k), dvp = on_device(v), dout = on_device(out);
    if (!(dq == dk && dk == dvp && dvp == dout)) {
        throw std::invalid_argument("q, k, v and output must all be host memory or all be device memory");
    }
    if (p.bias != nullptr && on_device(p.bias) != dq) {
        throw std::invalid_argument("the bias tensor must be in the same memory kind as q, k, v");
    }
    if (!dq) {
        // Host buffers: streamed through the device by the host entry.
        p.q = q;
        p.k = k;
        p.v = v;
        p.o = out;
        p.qkv_dtype = ODF_DTYPE_F32;
        p.block_mask = opt.block_mask ? opt.block_mask->allowed.data() : nullptr;
        const int rc = odf_flash_fwd_host(&p);
        if (rc != ODF_OK) throw_status(rc, "GPU attention");
        return;
    }

    // Device buffers: bf16 staging in the workspace, then the device entry.
    int device = 0;
    check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    if (!ws.device || ws.device->device != device) {
        ws.device = std::make_shared<DeviceStaging>();
        ws.device->device = device;
    }
    DeviceStaging& stg = *ws.device;
    cudaStream_t stream = cudaStreamPerThread;
    const std::size_t nq = pb.batch * pb.heads * pb.m * pb.d;
    const std::size_t nk = pb.batch * kvh * pb.n * pb.d;
    const std::size_t nv = pb.batch * kvh * pb.n * pb.dv;
    auto* qb = static_cast<uint16_t*>(stg.reserve(DeviceStaging::kQ, nq * 2));
    auto* kb = static_cast<uint16_t*>(stg.reserve(DeviceStaging::kK, nk * 2));
    auto* vb = static_cast<uint16_t*>(stg.reserve(DeviceStaging::kV, nv * 2));
    int rc = odf_convert_f32_to_bf16(q, qb, static_cast<int64_t>(nq), stream);
    if (rc == ODF_OK) rc = odf_convert_f32_to_bf16(k, kb, static_cast<int64_t>(nk), stream);
    if (rc == ODF_OK) rc = odf_convert_f32_to_bf16(v, vb, static_cast<int64_t>(nv), stream);
    if (rc != ODF_OK) throw_status(rc, "GPU attention: fp32 -> bf16 staging");
    p.q = qb;
    p.k = kb;
    p.v = vb;
    p.o = out;
    p.qkv_dtype = ODF_DTYPE_BF16;
    if (opt.block_mask) {
        const std::size_t mbytes = opt.block_mask->allowed.size();
        void* dmask = stg.reserve(DeviceStaging::kMask, mbytes);
        check_cuda(cudaMemcpyAsync(dmask, opt.block_mask->allowed.data(), mbytes, cudaMemcpyHostToDevice, stream),
                   "BlockMask upload");
        p.block_mask = static_cast<const uint8_t*>(dmask);
    }
    const size_t wbytes = odf_fwd_workspace_size(&p);
    p.workspace = stg.reserve(DeviceStaging::kLists, wbytes);
    p.workspace_bytes = wbytes;
    rc = odf_flash_fwd_sm100(&p, stream);
    if (rc != ODF_OK) throw_status(rc, "GPU attention");
    check_cuda(cudaStreamSynchronize(stream), "kernel execution");
}

std::vector<float> vector_forward(const std::vector<float>& q, const std::vector<float>& k,
                                  const std::vector<float>& v, const AttentionShape& shape,
                                  const AttentionOptions& options) {
    std::vector<float> out(shape.query_tokens * shape.value_dim, 0.0f);
    thread_local AttentionWorkspace ws;
    run_forward(q.data(), k.data(), v.data(), out.data(),
                Problem{1, 1, 1, shape.query_tokens, shape.key_tokens, shape.head_dim, shape.value_dim}, options, ws);
    return out;
}

}  // namespace

// ---------------------------------------------------------------- entry points
std::vector<float> standard_attention(const std::vector<float>& q, const std::vector<float>& k,
                                      const std::vector<float>& v, const AttentionShape& shape,
                                      const AttentionOptions& options) {
    validate_vectors(q, k, v, shape);
    return vector_forward(q, k, v, shape, options);
}

std::vector<float> flash_attention_tiled(const std::vector<float>& q, const std::vector<float>& k,
                                         const std::vector<float>& v, const AttentionShape& shape,
                                         const AttentionOptions& options) {
    validate_vectors(q, k, v, shape);
    if (options.key_block_size == 0) throw std::invalid_argument("key_block_size must be non-zero");
    return vector_forward(q, k, v, shape, options);
}

std::vector<float> flash_attention_q_tile(const std::vector<float>& q, const std::vector<float>& k,
                                          const std::vector<float>& v, const AttentionShape& shape,
                                          const AttentionOptions& options) {
    validate_vectors(q, k, v, shape);
    if (options.key_block_size == 0) throw std::invalid_argument("key_block_size must be non-zero");
    if (options.query_block_size == 0) throw std::invalid_argument("query_block_size must be non-zero");
    return vector_forward(q, k, v, shape, options);
}

std::vector<float> flash_attention_qk_pv_tile(const std::vector<float>& q, const std::vector<float>& k,
                                              const std::vector<float>& v, const AttentionShape& shape,
                                              const AttentionOptions& options) {
    validate_vectors(q, k, v, shape);
    if (options.key_block_size == 0) throw std::invalid_argument("key_block_size must be non-zero");
    if (options.query_block_size == 0) throw std::invalid_argument("query_block_size must be non-zero");
    return vector_forward(q, k, v, shape, options);
}

void flash_attention_qk_pv_tile_ws(const float* q, const float* k, const float* v, float* output,
                                   const AttentionShape& shape, const AttentionOptions& options,
                                   AttentionWorkspace& ws) {
    if (q == nullptr || k == nullptr || v == nullptr || output == nullptr) {
        throw std::invalid_argument("attention pointers must be non-null");
    }
    if (shape.query_tokens == 0 || shape.key_tokens == 0 || shape.head_dim == 0 || shape.value_dim == 0) {
        throw std::invalid_argument("Attention dimensions must be non-zero");
    }
    if (options.key_block_size == 0) throw std::invalid_argument("key_block_size must be non-zero");
    if (options.query_block_size == 0) throw std::invalid_argument("query_block_size must be non-zero");
    ws.resize(options.query_block_size, options.key_block_size, shape.head_dim, shape.value_dim);
    run_forward(q, k, v, output,
                Problem{1, 1, 1, shape.query_tokens, shape.key_tokens, shape.head_dim, shape.value_dim}, options, ws);
}

void flash_attention_batched_qk_pv_tile(const float* q, const float* k, const float* v, float* out,
                                        const BatchedAttentionShape& shape, const AttentionOptions& options) {
    if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) {
        throw std::invalid_argument("batched attention input/output pointers must be non-null");
    }
    if (shape.batch == 0 || shape.heads == 0 || shape.query_tokens == 0 || shape.key_tokens == 0 ||
        shape.head_dim == 0 || shape.value_dim == 0) {
        throw std::invalid_argument("batched attention dimensions must be non-zero");
    }
    thread_local AttentionWorkspace ws;
    run_forward(q, k, v, out,
                Problem{shape.batch, shape.heads, options.kv_heads, shape.query_tokens, shape.key_tokens,
                        shape.head_dim, shape.value_dim},
                options, ws);
}

std::vector<float> run_attention(AttentionBackendKind kind, const std::vector<float>& q, const std::vector<float>& k,
                                 const std::vector<float>& v, const AttentionShape& shape,
                                 const AttentionOptions& options) {
    switch (kind) {
        case AttentionBackendKind::StandardReference: return standard_attention(q, k, v, shape, options);
        case AttentionBackendKind::FlashTiledReference: return flash_attention_tiled(q, k, v, shape, options);
    }
    throw std::invalid_argument("Unknown attention backend kind");
}

}  // namespace onednn_flash
