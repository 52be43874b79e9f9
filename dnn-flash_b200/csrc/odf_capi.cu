// odf_capi.cu -- the extern "C" boundary (include/odf_sm100.h).
//
// Validation mirrors the reference's argument checks
// (src/onednn_flash/attention.cpp:493-505, batched_attention.cpp:15-21) but
// reports status codes instead of throwing; the message of the last failure on
// the calling thread is kept for odf_last_error().
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "odf_internal.h"

namespace {

thread_local std::string t_last_error;
// Test hooks (odf_debug_set_wait): limit of the in-kernel waits and an injected stall, applied
// to the launches this thread makes.
thread_local uint64_t t_wait_limit_ns = 0;  // 0 = the default (2 s)
thread_local int32_t t_stall_load = -1;      // -1 = off

int fail(int code, const std::string& msg) {
    t_last_error = msg;
    return code;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Fills contiguous [B, H, T, D] strides when all three are zero.
void resolve_strides(const int64_t in[3], int64_t heads, int64_t tokens, int64_t feat, int64_t out[3]) {
    if (in[0] == 0 && in[1] == 0 && in[2] == 0) {
        out[2] = feat;
        out[1] = tokens * feat;
        out[0] = heads * tokens * feat;
    } else {
        out[0] = in[0];
        out[1] = in[1];
        out[2] = in[2];
    }
}

struct Resolved {
    int64_t qs[3], ks[3], vs[3], os[3];
    int64_t bs[4];  // same-shape bias element strides (all-zero input = contiguous [B, Hq, M, N])
    int32_t n_qt, n_kt;
};

// Shared checks of the device and host entries.  `host` relaxes the Q/K/V dtype to F32|BF16.
int validate(const odf_fwd_params* p, bool host, Resolved* r) {
    if (p == nullptr) return fail(ODF_ERR_INVALID_ARG, "params must be non-null");
    if (p->q == nullptr || p->k == nullptr || p->v == nullptr || p->o == nullptr)
        return fail(ODF_ERR_INVALID_ARG, "attention input/output pointers must be non-null");
    if (p->batch <= 0 || p->heads_q <= 0 || p->heads_kv <= 0 || p->seqlen_q <= 0 || p->seqlen_k <= 0 ||
        p->head_dim <= 0 || p->value_dim <= 0)
        return fail(ODF_ERR_INVALID_ARG, "attention dimensions must be non-zero");
    if (p->heads_q % p->heads_kv != 0)
        return fail(ODF_ERR_INVALID_ARG, "heads_q must be a multiple of heads_kv");
    if (p->head_dim != p->value_dim || (p->head_dim != 64 && p->head_dim != 128))
        return fail(ODF_ERR_UNSUPPORTED, "the sm_100a kernel supports head_dim == value_dim in {64, 128}");
    if (host) {
        if (p->qkv_dtype != ODF_DTYPE_F32 && p->qkv_dtype != ODF_DTYPE_BF16)
            return fail(ODF_ERR_UNSUPPORTED, "q/k/v dtype must be f32 or bf16");
    } else if (p->qkv_dtype != ODF_DTYPE_BF16) {
        return fail(ODF_ERR_UNSUPPORTED, "device q/k/v must be bf16 (convert with odf_convert_f32_to_bf16)");
    }
    if (p->o_dtype != ODF_DTYPE_F32 && p->o_dtype != ODF_DTYPE_BF16)
        return fail(ODF_ERR_UNSUPPORTED, "output dtype must be f32 or bf16");
    const int64_t n_qt = (p->seqlen_q + odf::kTileQ - 1) / odf::kTileQ;
    const int64_t n_kt = (p->seqlen_k + odf::kTileK - 1) / odf::kTileK;
    if (n_qt > 65535 || n_kt > 65535 || p->batch * p->heads_q > 0x7fffffffLL || p->seqlen_q > 0x7fffffffLL ||
        p->seqlen_k > 0x7fffffffLL)
        return fail(ODF_ERR_UNSUPPORTED, "sequence length or batch*heads beyond the kernel's grid limits");
    if (!std::isfinite(p->scale)) return fail(ODF_ERR_INVALID_ARG, "scale must be finite");
    if (!(p->softcap >= 0.0f) || !std::isfinite(p->softcap))
        return fail(ODF_ERR_INVALID_ARG, "softcap must be finite and >= 0");
    if (p->bias_kind != ODF_BIAS_NONE && p->bias_kind != ODF_BIAS_ALIBI && p->bias_kind != ODF_BIAS_SAME_SHAPE)
        return fail(ODF_ERR_UNSUPPORTED,
                    "only BiasKind::None, SameShapeTile and AlibiGenerated run on the GPU");
    if (p->bias_kind == ODF_BIAS_SAME_SHAPE) {
        if (p->bias == nullptr) return fail(ODF_ERR_INVALID_ARG, "BiasKind::SameShapeTile needs a bias tensor");
        for (int i = 0; i < 4; ++i)
            if (p->bias_strides[i] < 0) return fail(ODF_ERR_INVALID_ARG, "bias strides must be >= 0");
        if (!aligned4(p->bias)) return fail(ODF_ERR_INVALID_ARG, "the bias tensor must be 4-byte aligned");
        const int64_t* s = p->bias_strides;
        if (s[0] == 0 && s[1] == 0 && s[2] == 0 && s[3] == 0) {
            r->bs[0] = p->heads_q * p->seqlen_q * p->seqlen_k;
            r->bs[1] = p->seqlen_q * p->seqlen_k;
            r->bs[2] = p->seqlen_k;
            r->bs[3] = 1;
        } else {
            for (int i = 0; i < 4; ++i) r->bs[i] = s[i];
        }
    } else {
        for (int i = 0; i < 4; ++i) r->bs[i] = 0;
    }
    if (p->bias_kind == ODF_BIAS_ALIBI && p->alibi_slopes != nullptr && p->heads_q > ODF_MAX_EXPLICIT_SLOPES)
        return fail(ODF_ERR_UNSUPPORTED, "explicit ALiBi slopes are limited to 256 heads (use generated slopes)");
    if (p->block_mask != nullptr &&
        (p->mask_qbs <= 0 || p->mask_kbs <= 0 || p->mask_qblocks <= 0 || p->mask_kblocks <= 0))
        return fail(ODF_ERR_INVALID_ARG, "BlockMask block sizes and dimensions must be non-zero");
    resolve_strides(p->q_strides, p->heads_q, p->seqlen_q, p->head_dim, r->qs);
    resolve_strides(p->k_strides, p->heads_kv, p->seqlen_k, p->head_dim, r->ks);
    resolve_strides(p->v_strides, p->heads_kv, p->seqlen_k, p->value_dim, r->vs);
    resolve_strides(p->o_strides, p->heads_q, p->seqlen_q, p->value_dim, r->os);
    for (int i = 0; i < 3; ++i) {
        if (r->qs[i] <= 0 || r->ks[i] <= 0 || r->vs[i] <= 0 || r->os[i] <= 0)
            return fail(ODF_ERR_INVALID_ARG, "strides must be positive (or all zero for contiguous)");
    }
    if (host) {
        const int64_t* all[4] = {p->q_strides, p->k_strides, p->v_strides, p->o_strides};
        for (auto s : all)
            if (s[0] || s[1] || s[2]) return fail(ODF_ERR_UNSUPPORTED, "host entry takes contiguous tensors only");
    } else {
        if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->o))
            return fail(ODF_ERR_INVALID_ARG, "device pointers must be 16-byte aligned");
        for (int i = 0; i < 3; ++i) {
            if (r->qs[i] % 8 || r->ks[i] % 8 || r->vs[i] % 8)
                return fail(ODF_ERR_INVALID_ARG, "q/k/v strides must be multiples of 8 elements (16 bytes)");
            if (r->os[i] % (p->o_dtype == ODF_DTYPE_BF16 ? 8 : 4))
                return fail(ODF_ERR_INVALID_ARG, "output strides must be multiples of 16 bytes");
        }
    }
    r->n_qt = static_cast<int32_t>(n_qt);
    r->n_kt = static_cast<int32_t>(n_kt);
    return ODF_OK;
}

// Required workspace plus the optional room of a launch of `batch` x `heads_q` query heads over
// `heads_kv` KV heads: for causal ALiBi at d = 128 (no block mask) its far-tile bound; for other
// launches without a block mask whose work items leave SMs idle, the partial results of KV splits.
size_t workspace_with_far_bound(const odf_fwd_params* p, int64_t batch, int64_t heads_q, int64_t heads_kv) {
    size_t bytes = odf::workspace_bytes_for(p->seqlen_q, p->seqlen_k, p->block_mask != nullptr);
    const bool alibi_walk = p->causal && p->bias_kind == ODF_BIAS_ALIBI && p->head_dim == 128;
    if (p->block_mask == nullptr && alibi_walk)
        bytes += odf::far_bound_bytes(batch, heads_q, heads_kv, p->seqlen_q, p->seqlen_k);
    if (p->block_mask == nullptr && !alibi_walk)
        bytes += odf::kv_split_bytes(batch, heads_q, p->seqlen_q, p->seqlen_k, p->head_dim, true);
    return bytes;
}

float generated_slope(int64_t h, int64_t heads) {
    return std::exp2(-8.0f * static_cast<float>(h + 1) / static_cast<float>(heads));
}

odf::FwdLaunch make_launch(const odf_fwd_params* p, const Resolved& r) {
    odf::FwdLaunch L;
    std::memset(&L, 0, sizeof(L));
    L.q = p->q;
    L.k = p->k;
    L.v = p->v;
    std::copy(r.qs, r.qs + 3, L.q_strides);
    std::copy(r.ks, r.ks + 3, L.k_strides);
    std::copy(r.vs, r.vs + 3, L.v_strides);
    L.head_dim = static_cast<int32_t>(p->head_dim);
    L.has_alibi = p->bias_kind == ODF_BIAS_ALIBI;
    L.has_softcap = p->softcap > 0.0f;
    L.has_bias = p->bias_kind == ODF_BIAS_SAME_SHAPE;
    L.workspace = p->workspace;
    L.workspace_bytes = p->workspace_bytes;
    L.allow_split = 1;
    odf::FwdArgs& a = L.args;
    a.o = p->o;
    a.lse = p->lse;
    a.o_stride_b = r.os[0];
    a.o_stride_h = r.os[1];
    a.o_stride_t = r.os[2];
    a.o_bf16 = p->o_dtype == ODF_DTYPE_BF16;
    a.batch = static_cast<int32_t>(p->batch);
    a.heads_q = static_cast<int32_t>(p->heads_q);
    a.heads_kv = static_cast<int32_t>(p->heads_kv);
    a.m = static_cast<int32_t>(p->seqlen_q);
    a.n = static_cast<int32_t>(p->seqlen_k);
    a.n_qt = r.n_qt;
    a.n_kt = r.n_kt;
    a.causal = p->causal != 0;
    a.mode = p->block_mask ? odf::kModeList : (p->causal ? odf::kModeCausal : odf::kModeDense);
    // causal ALiBi at d = 128: diagonal tile first, so far tiles meet a settled running max
    a.kv_reverse = a.mode == odf::kModeCausal && p->bias_kind == ODF_BIAS_ALIBI && p->head_dim == 128;
    a.scale = p->scale;
    a.scale_log2 = p->scale * 1.4426950408889634f;
    a.softcap = p->softcap;
    a.inv_softcap = p->softcap > 0.0f ? 1.0f / p->softcap : 0.0f;
    a.mask = p->block_mask;
    a.mask_qbs = static_cast<int32_t>(std::min<int64_t>(p->mask_qbs, 0x7fffffff));
    a.mask_kbs = static_cast<int32_t>(std::min<int64_t>(p->mask_kbs, 0x7fffffff));
    a.mask_qblocks = static_cast<int32_t>(std::min<int64_t>(p->mask_qblocks, 0x7fffffff));
    a.mask_kblocks = static_cast<int32_t>(std::min<int64_t>(p->mask_kblocks, 0x7fffffff));
    a.visits = p->tile_visits;
    a.wait_limit_ns = t_wait_limit_ns;
    a.stall_load = t_stall_load;
    if (p->bias_kind == ODF_BIAS_SAME_SHAPE) {
        a.bias = p->bias;
        a.bias_s0 = r.bs[0];
        a.bias_s1 = r.bs[1];
        a.bias_s2 = r.bs[2];
        a.bias_s3 = r.bs[3];
    }
    // Generated slopes are evaluated here on the host (for up to 256 heads) so that the
    // device entry and the chunked host entry use bit-identical values.
    a.alibi_generated = 0;
    if (p->bias_kind == ODF_BIAS_ALIBI) {
        if (p->alibi_slopes != nullptr) {
            for (int64_t h = 0; h < p->heads_q; ++h) a.alibi_slopes[h] = p->alibi_slopes[h];
        } else if (p->heads_q <= ODF_MAX_EXPLICIT_SLOPES) {
            for (int64_t h = 0; h < p->heads_q; ++h) a.alibi_slopes[h] = generated_slope(h, p->heads_q);
        } else {
            a.alibi_generated = 1;
        }
    }
    return L;
}

int run_device(const odf_fwd_params* p, const Resolved& r, cudaStream_t stream, bool allow_split = true,
               int forced_splits = 0) {
    const size_t need = odf::workspace_bytes_for(p->seqlen_q, p->seqlen_k, p->block_mask != nullptr);
    if (p->block_mask != nullptr && p->workspace == nullptr)
        return fail(ODF_ERR_INVALID_ARG, "a block mask needs a device workspace of odf_fwd_workspace_size() bytes");
    if (p->workspace != nullptr && p->workspace_bytes < need)
        return fail(ODF_ERR_INVALID_ARG, "the workspace is smaller than odf_fwd_workspace_size() bytes");
    if (p->workspace != nullptr && !aligned16(p->workspace))
        return fail(ODF_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
    odf::FwdLaunch L = make_launch(p, r);
    L.allow_split = allow_split ? 1 : 0;
    L.forced_splits = forced_splits;
    const char* err = "";
    const int rc = odf::launch_flash_fwd(L, stream, &err);
    if (rc != ODF_OK) return fail(rc, err);
    return ODF_OK;
}

// ------------------------------------------------------------------ host entry
// Device buffers of the host entry, per thread and device, grown on demand.
// Three stages run on their own streams -- copy in (and fp32 -> bf16), the kernel, copy out --
// over kHostSets rotating buffer sets, so chunk c's upload, chunk c-1's kernel and chunk c-2's
// download overlap.  Events order a stage after the previous stage of its chunk and a buffer
// set's reuse after the last stage that read it.  Kernels of consecutive chunks alternate
// between two compute streams, so the next chunk's CTAs take the SMs that the previous
// chunk's last items leave idle.
constexpr int kHostSets = 3;
struct HostPool {
    int device = -1;
    cudaStream_t streams[4] = {nullptr, nullptr, nullptr, nullptr};  // copy in, compute x2, copy out
    cudaEvent_t in_done[kHostSets] = {}, comp_done[kHostSets] = {}, out_done[kHostSets] = {};
    void* buf[kHostSets][8] = {};
    size_t cap[kHostSets][8] = {};
    void* mask = nullptr;
    size_t mask_cap = 0;
    // K and V of units split into query-head pieces (problems with fewer than four units):
    // uploaded once by the unit's first piece, read by all its pieces' kernels.
    static constexpr int kSplitUnits = 3;
    void* kvd[kSplitUnits][2] = {};
    size_t kvd_cap[kSplitUnits][2] = {};
    // A same-shape bias broadcast over batch and heads: one plane, uploaded once per call.
    void* shared_bias = nullptr;
    size_t shared_bias_cap = 0;
    ~HostPool() {
        // Process teardown may run after the CUDA context is gone; freeing is best-effort.
        for (auto& set : buf)
            for (void*& b : set)
                if (b) cudaFree(b);
        if (mask) cudaFree(mask);
        for (auto& pair : kvd)
            for (void*& b : pair)
                if (b) cudaFree(b);
        if (shared_bias) cudaFree(shared_bias);
        for (auto* evs : {in_done, comp_done, out_done})
            for (int i = 0; i < kHostSets; ++i)
                if (evs[i]) cudaEventDestroy(evs[i]);
        for (auto& s : streams)
            if (s) cudaStreamDestroy(s);
    }
    cudaError_t reserve_shared_bias(size_t bytes, void** out) {
        if (shared_bias_cap < bytes) {
            if (shared_bias) cudaFree(shared_bias);
            shared_bias = nullptr;
            shared_bias_cap = 0;
            cudaError_t e = cudaMalloc(&shared_bias, bytes);
            if (e != cudaSuccess) return e;
            shared_bias_cap = bytes;
        }
        *out = shared_bias;
        return cudaSuccess;
    }
    cudaError_t reserve_kv(int which, int idx, size_t bytes, void** out) {
        if (kvd_cap[which][idx] < bytes) {
            if (kvd[which][idx]) cudaFree(kvd[which][idx]);
            kvd[which][idx] = nullptr;
            kvd_cap[which][idx] = 0;
            cudaError_t e = cudaMalloc(&kvd[which][idx], bytes);
            if (e != cudaSuccess) return e;
            kvd_cap[which][idx] = bytes;
        }
        *out = kvd[which][idx];
        return cudaSuccess;
    }
    cudaError_t reserve(int slot, int idx, size_t bytes, void** out) {
        if (cap[slot][idx] < bytes) {
            if (buf[slot][idx]) cudaFree(buf[slot][idx]);
            buf[slot][idx] = nullptr;
            cap[slot][idx] = 0;
            cudaError_t e = cudaMalloc(&buf[slot][idx], bytes);
            if (e != cudaSuccess) return e;
            cap[slot][idx] = bytes;
        }
        *out = buf[slot][idx];
        return cudaSuccess;
    }
};
thread_local HostPool t_pool;

}  // namespace

extern "C" {

int odf_flash_fwd_sm100(const odf_fwd_params* p, void* stream) {
    Resolved r;
    const int rc = validate(p, false, &r);
    if (rc != ODF_OK) return rc;
    return run_device(p, r, static_cast<cudaStream_t>(stream));
}

size_t odf_fwd_workspace_size(const odf_fwd_params* p) {
    if (p == nullptr) return 0;
    return workspace_with_far_bound(p, p->batch, p->heads_q, p->heads_kv);
}

int odf_flash_fwd_host(const odf_fwd_params* p) {
    Resolved r;
    int rc = validate(p, true, &r);
    if (rc != ODF_OK) return rc;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(ODF_ERR_NO_DEVICE, "no CUDA device");
    const char* err = "";
    rc = odf::ensure_device_ready(device, &err);
    if (rc != ODF_OK) return fail(rc, err);
    HostPool& pool = t_pool;
    if (pool.device != device) {
        pool.~HostPool();
        new (&pool) HostPool();
        pool.device = device;
    }
    cudaError_t e = cudaSuccess;
    for (auto& s : pool.streams)
        if (!s && e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    for (auto* evs : {pool.in_done, pool.comp_done, pool.out_done})
        for (int i = 0; i < kHostSets; ++i)
            if (!evs[i] && e == cudaSuccess) e = cudaEventCreateWithFlags(&evs[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
    cudaStream_t s_in = pool.streams[0], s_out = pool.streams[3];

    // Work is chunked over (batch, kv-head) units; a unit's Q/O rows (its
    // heads_q/heads_kv query heads) and K/V rows are contiguous.
    const int64_t G = p->heads_q / p->heads_kv;
    const int64_t units = p->batch * p->heads_kv;
    const int64_t M = p->seqlen_q, N = p->seqlen_k, D = p->head_dim, DV = p->value_dim;
    const int64_t n_qt = r.n_qt;
    int64_t n_chunks = std::min<int64_t>(units, 8);
    while (n_chunks > 1 && (units / n_chunks) * G * n_qt < 2 * 148) --n_chunks;
    const int64_t per = (units + n_chunks - 1) / n_chunks;
    // A chunk is units [u0, u0 + cu) with all their query heads, or query heads [g0, g0 + ng)
    // of the single unit u0.  Only the first chunk's upload and the last chunk's download run
    // alone, so with a pipeline of four or more chunks the first and the last unit are split:
    // a quarter of their query heads (at least one) goes first / last, and the rest of the unit
    // is a chunk of its own (its K/V uploaded twice, under the other chunks' kernels).
    // With fewer than four units (one GPU's share of a GQA problem split over several GPUs, or a
    // single kv-head) whole units would make a pipeline of one to three chunks, so every unit is
    // cut into pieces of query heads (about eight pieces in all); a unit's pieces share one upload
    // of its K/V into a buffer of its own (kvbuf = the unit, kv_up on its first piece).
    struct Chunk { int64_t u0, cu, g0, ng; int kvbuf; bool kv_up; };
    std::vector<Chunk> plan;
    const int64_t gs = std::max<int64_t>(1, G / 4);
    // Query heads per piece: about eight pieces in all, but each with at least 148 query tiles
    // (a piece's kernel should fill the GPU), otherwise the units stay whole.
    int64_t ps = (G + std::min<int64_t>(G, (8 + units - 1) / units) - 1) / std::min<int64_t>(G, (8 + units - 1) / units);
    while (ps < G && ps * n_qt < 148) ps = std::min(G, 2 * ps);
    const bool pieces = units < 4 && ps < G && units <= HostPool::kSplitUnits;
    const bool split_ends = !pieces && n_chunks >= 4 && units >= 2 && G >= 2;
    if (pieces) {
        for (int64_t u = 0; u < units; ++u)
            for (int64_t g = 0; g < G; g += ps) plan.push_back({u, 1, g, std::min(ps, G - g), static_cast<int>(u), g == 0});
    } else {
        const int64_t mid0 = split_ends ? 1 : 0, mid1 = split_ends ? units - 1 : units;
        if (split_ends) {
            plan.push_back({0, 1, 0, gs, -1, true});
            plan.push_back({0, 1, gs, G - gs, -1, true});
        }
        for (int64_t u = mid0; u < mid1; u += per) plan.push_back({u, std::min(per, mid1 - u), 0, G, -1, true});
        if (split_ends) {
            plan.push_back({units - 1, 1, 0, G - gs, -1, true});
            plan.push_back({units - 1, 1, G - gs, gs, -1, true});
        }
    }
    const size_t in_es = p->qkv_dtype == ODF_DTYPE_F32 ? 4 : 2;
    const size_t out_es = p->o_dtype == ODF_DTYPE_F32 ? 4 : 2;
    const size_t kv_unit = static_cast<size_t>(N * D), v_unit = static_cast<size_t>(N * DV);

    const uint8_t* dmask = nullptr;
    if (p->block_mask) {
        const size_t mbytes = static_cast<size_t>(p->mask_qblocks * p->mask_kblocks);
        if (pool.mask_cap < mbytes) {
            if (pool.mask) cudaFree(pool.mask);
            pool.mask = nullptr;
            pool.mask_cap = 0;
            e = cudaMalloc(&pool.mask, mbytes);
            if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
            pool.mask_cap = mbytes;
        }
        e = cudaMemcpyAsync(pool.mask, p->block_mask, mbytes, cudaMemcpyHostToDevice, pool.streams[0]);
        if (e == cudaSuccess) e = cudaStreamSynchronize(pool.streams[0]);
        if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        dmask = static_cast<const uint8_t*>(pool.mask);
    }
    // a chunk launches batch 1 over at most all query heads and all units
    const size_t ws_bytes = workspace_with_far_bound(p, 1, p->batch * p->heads_q, units);
    // Every chunk splits the key range as one device launch of the whole problem would, so each
    // query tile is computed the same way (and the result equals odf_flash_fwd_sm100's bit for bit).
    int sm_count = 0;
    if ((e = cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
        return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
    const bool alibi_walk = p->causal && p->bias_kind == ODF_BIAS_ALIBI && p->head_dim == 128;
    const int whole_splits = odf::plan_kv_splits(p->batch, p->heads_q, p->seqlen_q, p->seqlen_k,
                                                 p->block_mask == nullptr && !alibi_walk, sm_count)
                                 .n_splits;

    for (int64_t c = 0; c < static_cast<int64_t>(plan.size()); ++c) {
        const int64_t u0 = plan[c].u0, cu = plan[c].cu, g0 = plan[c].g0, ng = plan[c].ng;
        const int64_t h0 = u0 * G + g0;  // first global (batch, q-head) index of the chunk
        const int64_t nh = cu * ng;      // its query heads
        const size_t q_head = static_cast<size_t>(M * D), o_head = static_cast<size_t>(M * DV);
        const int slot = static_cast<int>(c % kHostSets);
        cudaStream_t st = s_in;                        // this chunk's copies and conversions
        cudaStream_t s_comp = pool.streams[1 + (c & 1)];  // its kernel
        const int kvbuf = plan[c].kvbuf;
        const bool kv_up = plan[c].kv_up;
        void *dq, *dk, *dv, *dout, *dlse = nullptr, *dstage = nullptr, *dws = nullptr;
        if (kvbuf < 0) {
            e = pool.reserve(slot, 1, cu * kv_unit * 2, &dk);
            if (e == cudaSuccess) e = pool.reserve(slot, 2, cu * v_unit * 2, &dv);
        } else {
            e = pool.reserve_kv(kvbuf, 0, kv_unit * 2, &dk);
            if (e == cudaSuccess) e = pool.reserve_kv(kvbuf, 1, v_unit * 2, &dv);
        }
        if (e != cudaSuccess || (e = pool.reserve(slot, 0, nh * q_head * 2, &dq)) != cudaSuccess ||
            (e = pool.reserve(slot, 3, nh * o_head * out_es, &dout)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        if (p->lse && (e = pool.reserve(slot, 4, nh * M * sizeof(float), &dlse)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        if (in_es == 4 && (e = pool.reserve(slot, 5, std::max(nh * q_head, cu * std::max(kv_unit, v_unit)) * 4,
                                            &dstage)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        if (ws_bytes && (e = pool.reserve(slot, 6, ws_bytes, &dws)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        // the set's inputs are rewritten once the kernel of chunk c - kHostSets has read them
        if (c >= kHostSets && (e = cudaStreamWaitEvent(s_in, pool.comp_done[slot], 0)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        // Same-shape bias: the footprint of each (batch, q-head) plane of this chunk, copied to a
        // device staging buffer with the row/key strides kept.  A bias broadcast over batch and
        // heads is one plane for every chunk: it is uploaded once, by the first chunk.
        const float* dbias = nullptr;
        int64_t bias_plane = 0;
        if (p->bias_kind == ODF_BIAS_SAME_SHAPE) {
            const int64_t* bs = r.bs;
            const int64_t foot = (M - 1) * bs[2] + (N - 1) * bs[3] + 1;
            const bool shared = bs[0] == 0 && bs[1] == 0;
            const int64_t planes = shared ? (c == 0 ? 1 : 0) : nh;
            bias_plane = shared ? 0 : (foot + 3) / 4 * 4;
            void* db = nullptr;
            e = shared ? pool.reserve_shared_bias(static_cast<size_t>(foot) * sizeof(float), &db)
                       : pool.reserve(slot, 7, static_cast<size_t>(planes * bias_plane) * sizeof(float), &db);
            if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
            for (int64_t j = 0; j < planes && e == cudaSuccess; ++j) {
                const int64_t gh = h0 + j;  // global (batch, q-head) index of this plane
                const int64_t b = gh / p->heads_q, h = gh % p->heads_q;
                e = cudaMemcpyAsync(static_cast<float*>(db) + j * bias_plane, p->bias + b * bs[0] + h * bs[1],
                                    static_cast<size_t>(foot) * sizeof(float), cudaMemcpyHostToDevice, st);
            }
            if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
            dbias = static_cast<const float*>(db);
        }

        const char* hq = static_cast<const char*>(p->q) + h0 * q_head * in_es;
        const char* hk = static_cast<const char*>(p->k) + u0 * kv_unit * in_es;
        const char* hv = static_cast<const char*>(p->v) + u0 * v_unit * in_es;
        struct Part { const char* src; void* dst; size_t elems; } parts[3] = {
            {hq, dq, nh * q_head}, {hk, dk, cu * kv_unit}, {hv, dv, cu * v_unit}};
        for (int pi = 0; pi < (kv_up ? 3 : 1); ++pi) {  // a unit's later pieces reuse its K/V
            const Part& part = parts[pi];
            if (in_es == 2) {
                e = cudaMemcpyAsync(part.dst, part.src, part.elems * 2, cudaMemcpyHostToDevice, st);
            } else {
                e = cudaMemcpyAsync(dstage, part.src, part.elems * 4, cudaMemcpyHostToDevice, st);
                if (e == cudaSuccess &&
                    odf::launch_convert_f32_bf16(static_cast<const float*>(dstage), static_cast<uint16_t*>(part.dst),
                                                 static_cast<int64_t>(part.elems), st) != ODF_OK)
                    e = cudaErrorLaunchFailure;
            }
            if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        }
        if ((e = cudaEventRecord(pool.in_done[slot], s_in)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        odf_fwd_params sub = *p;
        sub.q = dq;
        sub.k = dk;
        sub.v = dv;
        sub.o = dout;
        sub.lse = static_cast<float*>(dlse);
        sub.qkv_dtype = ODF_DTYPE_BF16;
        sub.batch = 1;
        sub.heads_kv = cu;
        sub.heads_q = nh;
        sub.block_mask = dmask;
        sub.workspace = dws;
        sub.workspace_bytes = ws_bytes;
        sub.tile_visits = nullptr;
        if (dbias) {
            sub.bias = dbias;
            sub.bias_strides[0] = 0;  // the sub-launch has batch 1
            sub.bias_strides[1] = bias_plane;
            sub.bias_strides[2] = r.bs[2];
            sub.bias_strides[3] = r.bs[3];  // never all four zero: r.bs came from a non-zero or contiguous set
        }
        // ALiBi slopes are per q-head: shift to this chunk's heads (units never straddle a batch row
        // of heads when heads are re-based, so slopes are indexed by head within the batch).
        std::vector<float> slopes;
        if (p->bias_kind == ODF_BIAS_ALIBI) {
            slopes.resize(static_cast<size_t>(nh));
            for (int64_t j = 0; j < nh; ++j) {
                const int64_t h = (h0 + j) % p->heads_q;
                slopes[j] = p->alibi_slopes ? p->alibi_slopes[h] : generated_slope(h, p->heads_q);
            }
            sub.alibi_slopes = slopes.data();
            if (nh > ODF_MAX_EXPLICIT_SLOPES) return fail(ODF_ERR_UNSUPPORTED, "too many heads per chunk for ALiBi");
        }
        Resolved rs;
        rc = validate(&sub, false, &rs);
        if (rc != ODF_OK) return rc;
        // kernel: after this chunk's copies, and after chunk c - kHostSets's outputs left the set
        e = cudaStreamWaitEvent(s_comp, pool.in_done[slot], 0);
        if (e == cudaSuccess && c >= kHostSets) e = cudaStreamWaitEvent(s_comp, pool.out_done[slot], 0);
        if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        rc = run_device(&sub, rs, s_comp, true, whole_splits);
        if (rc != ODF_OK) return rc;
        if ((e = cudaEventRecord(pool.comp_done[slot], s_comp)) != cudaSuccess)
            return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
        // copy out after the kernel
        e = cudaStreamWaitEvent(s_out, pool.comp_done[slot], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<char*>(p->o) + h0 * o_head * out_es, dout, nh * o_head * out_es,
                                cudaMemcpyDeviceToHost, s_out);
        if (e == cudaSuccess && p->lse)
            e = cudaMemcpyAsync(p->lse + h0 * M, dlse, nh * M * sizeof(float), cudaMemcpyDeviceToHost, s_out);
        if (e == cudaSuccess) e = cudaEventRecord(pool.out_done[slot], s_out);
        if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
    }
    for (auto& s : pool.streams) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
    }
    return ODF_OK;
}

int odf_tile_map_sm100(int64_t seqlen_q, int64_t seqlen_k, int32_t causal, const uint8_t* block_mask,
                       int64_t mask_qbs, int64_t mask_kbs, int64_t mask_qblocks, int64_t mask_kblocks, uint8_t* out,
                       void* stream) {
    if (out == nullptr) return fail(ODF_ERR_INVALID_ARG, "output pointer must be non-null");
    if (seqlen_q <= 0 || seqlen_k <= 0) return fail(ODF_ERR_INVALID_ARG, "dimensions must be non-zero");
    if (seqlen_q > 0x7fffffffLL || seqlen_k > 0x7fffffffLL) return fail(ODF_ERR_UNSUPPORTED, "sequence too long");
    if (block_mask && (mask_qbs <= 0 || mask_kbs <= 0 || mask_qblocks <= 0 || mask_kblocks <= 0))
        return fail(ODF_ERR_INVALID_ARG, "BlockMask block sizes and dimensions must be non-zero");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(ODF_ERR_NO_DEVICE, "no CUDA device");
    const int rc = odf::launch_tile_map(static_cast<int32_t>(seqlen_q), static_cast<int32_t>(seqlen_k), causal,
                                        block_mask, static_cast<int32_t>(std::min<int64_t>(mask_qbs, 0x7fffffff)),
                                        static_cast<int32_t>(std::min<int64_t>(mask_kbs, 0x7fffffff)),
                                        static_cast<int32_t>(std::min<int64_t>(mask_qblocks, 0x7fffffff)),
                                        static_cast<int32_t>(std::min<int64_t>(mask_kblocks, 0x7fffffff)), out,
                                        static_cast<cudaStream_t>(stream));
    if (rc != ODF_OK) return fail(rc, "tile map kernel launch failed");
    return ODF_OK;
}

int odf_convert_f32_to_bf16(const float* in, uint16_t* out, int64_t count, void* stream) {
    if ((in == nullptr || out == nullptr) && count > 0) return fail(ODF_ERR_INVALID_ARG, "pointers must be non-null");
    if (count < 0) return fail(ODF_ERR_INVALID_ARG, "count must be >= 0");
    const int rc = odf::launch_convert_f32_bf16(in, out, count, static_cast<cudaStream_t>(stream));
    if (rc != ODF_OK) return fail(rc, "conversion kernel launch failed");
    return ODF_OK;
}

int odf_device_status(int32_t* status_out, int32_t clear) {
    if (status_out == nullptr) return fail(ODF_ERR_INVALID_ARG, "status_out must be non-null");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(ODF_ERR_NO_DEVICE, "no CUDA device");
    const char* err = "";
    int rc = odf::ensure_device_ready(device, &err);
    if (rc != ODF_OK) return fail(rc, err);
    int* ptr = odf::device_status_ptr(device);
    int value = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&value, ptr, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(ptr, 0, sizeof(int));
    if (e != cudaSuccess) return fail(ODF_ERR_CUDA, cudaGetErrorString(e));
    *status_out = value;
    return ODF_OK;
}

const char* odf_last_error(void) { return t_last_error.c_str(); }

int odf_debug_check_bits(uint32_t* bits_out) {
    if (bits_out == nullptr) return fail(ODF_ERR_INVALID_ARG, "bits_out must be non-null");
    const int rc = odf::read_check_bits(bits_out);
    if (rc == ODF_ERR_UNSUPPORTED) return fail(rc, "in-kernel checks exist only in the checked build");
    if (rc != ODF_OK) return fail(rc, "reading the check bits failed");
    return ODF_OK;
}

int odf_debug_set_wait(uint64_t limit_ns, int32_t stall_load) {
    if (limit_ns != 0 && (limit_ns < 1000000ull || limit_ns > 60000000000ull))
        return fail(ODF_ERR_INVALID_ARG, "wait limit must be 0 (default) or within [1 ms, 60 s]");
    if (stall_load < -1) return fail(ODF_ERR_INVALID_ARG, "stall_load must be -1 (off) or a load index >= 0");
    t_wait_limit_ns = limit_ns;
    t_stall_load = stall_load;
    return ODF_OK;
}

const char* odf_version(void) { return "dnn-flash-b200 0.1.0 (sm_100a tcgen05/TMA forward)"; }

}  // extern "C"

// ------------------------------------------------------------------ no-allocation entry
// Scratch for odf_flash_fwd_sm100_noalloc: a fixed-size array in the module's device
// memory, present on every GPU that loads this library until the process exits.
// Host code must not use the symbol itself as a pointer (on the host it only names a
// stand-in); its device address is looked up once per device below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[ODF_NOALLOC_SCRATCH_BYTES];

namespace {

struct NoAllocDevice {
    void* ctx = nullptr;      // the CUDA context the address below belongs to
    void* scratch = nullptr;
};
NoAllocDevice g_noalloc[64];
std::mutex g_noalloc_mutex;

// Device address of g_noalloc_scratch in the current device's current context.  A __device__
// array's address belongs to the context the module was loaded into, so it is looked up again
// whenever that context changes (cudaDeviceReset, a context the caller made current).
int noalloc_scratch_for_current_device(void** out) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(ODF_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= 64) return fail(ODF_ERR_NO_DEVICE, "device index out of range");
    // the same capability and set-up checks, and status codes, as odf_flash_fwd_sm100
    const char* err = "";
    const int rc = odf::ensure_device_ready(device, &err);
    if (rc != ODF_OK) return fail(rc, err);
    void* ctx = odf::current_context();
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocDevice& d = g_noalloc[device];
    if (d.scratch == nullptr || ctx == nullptr || d.ctx != ctx) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            return fail(ODF_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e));
        d.scratch = ptr;
        d.ctx = odf::current_context();
    }
    *out = d.scratch;
    return ODF_OK;
}

}  // namespace

extern "C" int odf_flash_fwd_sm100_noalloc(const odf_fwd_params* p, void* stream) {
    Resolved r;
    int rc = validate(p, false, &r);
    if (rc != ODF_OK) return rc;
    const size_t need = odf::workspace_bytes_for(p->seqlen_q, p->seqlen_k, p->block_mask != nullptr);
    if (need > ODF_NOALLOC_SCRATCH_BYTES)
        return fail(ODF_ERR_UNSUPPORTED, "block-mask tile lists need " + std::to_string(need) +
                                             " bytes of scratch; odf_flash_fwd_sm100_noalloc has " +
                                             std::to_string(ODF_NOALLOC_SCRATCH_BYTES) +
                                             " (use odf_flash_fwd_sm100 with a workspace)");
    odf_fwd_params q = *p;
    q.workspace = nullptr;
    q.workspace_bytes = 0;
    if (need > 0) {
        void* scratch = nullptr;
        rc = noalloc_scratch_for_current_device(&scratch);
        if (rc != ODF_OK) return rc;
        q.workspace = scratch;
        q.workspace_bytes = ODF_NOALLOC_SCRATCH_BYTES;
    }
    return run_device(&q, r, static_cast<cudaStream_t>(stream), false);  // the scratch keeps its layout: no KV splits
}
