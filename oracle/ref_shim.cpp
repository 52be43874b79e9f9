// ref_shim.cpp -- extern "C" shim over the UNMODIFIED reference sources
// (TEST INFRASTRUCTURE ONLY; built into oracle/_ref/ by oracle/Makefile).
//
// It is compiled together with the reference's own src/onednn_flash/*.cpp and
// calls the reference's public API exactly as a user would:
//   - flash_attention_qk_pv_tile_ws   (attention.cpp:486-695), per (batch, head)
//   - flash_attention_batched_qk_pv_tile (batched_attention.cpp:9-49), as shipped
//   - standard_attention / flash_attention_tiled / flash_attention_q_tile /
//     flash_attention_qk_pv_tile (attention.cpp:88-484)
//   - make_score_mod_plan / make_runtime_plan / make_block_mask_plan /
//     make_causal_mask_tile_descriptor (score_mod_plan.cpp, runtime_plan.cpp)
// The (batch x head) thread pool below is the harness the CPU baseline uses to
// put every host core on the reference's per-head function; the reference
// itself loops serially (batched_attention.cpp:39-48).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <exception>
#include <string>
#include <thread>
#include <vector>

#include "onednn_flash/attention.hpp"
#include "onednn_flash/backend.hpp"
#include "onednn_flash/batched_attention.hpp"
#include "onednn_flash/runtime_plan.hpp"
#include "onednn_flash/score_mod_plan.hpp"

#include "odf_oracle.h"

namespace of = onednn_flash;

namespace {

bool make_options(const odf_oracle_params* p, of::BlockMask* mask_storage, of::AttentionOptions* opt) {
    opt->scale = p->scale;
    opt->causal = p->causal != 0;
    opt->query_block_size = static_cast<std::size_t>(p->q_block);
    opt->key_block_size = static_cast<std::size_t>(p->k_block);
    opt->qk_tile_kernel = of::TileKernelKind::Reference;
    opt->pv_tile_kernel = of::TileKernelKind::Reference;
    opt->qk_tile_layout = of::QkTileLayout::StridedK;
    if (p->mask) {
        mask_storage->query_block_size = static_cast<std::size_t>(p->mask_qbs);
        mask_storage->key_block_size = static_cast<std::size_t>(p->mask_kbs);
        mask_storage->query_blocks = static_cast<std::size_t>(p->mask_qblocks);
        mask_storage->key_blocks = static_cast<std::size_t>(p->mask_kblocks);
        mask_storage->allowed.assign(p->mask, p->mask + p->mask_qblocks * p->mask_kblocks);
        opt->block_mask = mask_storage;
    }
    return p->softcap == 0.0f;  // soft-cap does not exist in the reference
}

// The structured biases of odf_oracle_params as the reference's ScoreBiasFn (attention.hpp:31)
// for one (batch, q-head): ALiBi slope[h] * (kj - qi), a strided bias tensor, or their sum.
of::ScoreBiasFn bias_fn(const odf_oracle_params* p, int64_t b, int64_t h) {
    if (!p->alibi_slopes && !p->bias) return nullptr;
    const float slope = p->alibi_slopes ? p->alibi_slopes[h] : 0.0f;
    const bool has_alibi = p->alibi_slopes != nullptr;
    const float* bias = p->bias ? p->bias + b * p->bias_strides[0] + h * p->bias_strides[1] : nullptr;
    const int64_t sm = p->bias_strides[2], sn = p->bias_strides[3];
    return [=](std::size_t qi, std::size_t kj) {
        float v = 0.0f;
        if (has_alibi) v = slope * static_cast<float>(static_cast<int64_t>(kj) - static_cast<int64_t>(qi));
        if (bias) v += bias[static_cast<int64_t>(qi) * sm + static_cast<int64_t>(kj) * sn];
        return v;
    };
}

enum class Variant { Ws, Standard, Tiled, QTile, QkPvTile };

int run(const odf_oracle_params* p, Variant variant) {
    if (!p || !p->q || !p->k || !p->v || !p->o || p->batch <= 0 || p->heads_q <= 0 ||
        p->heads_kv <= 0 || p->heads_q % p->heads_kv != 0) {
        return ODF_ORACLE_EINVAL;
    }
    of::BlockMask mask;
    of::AttentionOptions base;
    if (!make_options(p, &mask, &base)) return ODF_ORACLE_EUNSUPPORTED;
    if (p->lse) return ODF_ORACLE_EUNSUPPORTED;  // the reference produces no LSE
    const int64_t units = p->batch * p->heads_q;
    const int64_t group = p->heads_q / p->heads_kv;
    const of::AttentionShape shape{static_cast<std::size_t>(p->m), static_cast<std::size_t>(p->n),
                                   static_cast<std::size_t>(p->d), static_cast<std::size_t>(p->dv)};
    int nt = std::max(1, p->nthreads);
    nt = static_cast<int>(std::min<int64_t>(nt, units));
    std::vector<int> status(nt, ODF_ORACLE_OK);

    auto worker = [&](int t) {
        of::AttentionWorkspace ws;
        try {
            for (int64_t u = t; u < units; u += nt) {
                const int64_t b = u / p->heads_q, h = u % p->heads_q, hk = h / group;
                const float* q = p->q + (b * p->heads_q + h) * p->m * p->d;
                const float* k = p->k + (b * p->heads_kv + hk) * p->n * p->d;
                const float* v = p->v + (b * p->heads_kv + hk) * p->n * p->dv;
                float* o = p->o + (b * p->heads_q + h) * p->m * p->dv;
                of::AttentionOptions opt = base;
                opt.score_bias = bias_fn(p, b, h);
                if (variant == Variant::Ws) {
                    std::fill(o, o + p->m * p->dv, 0.0f);  // rows with l <= 0 stay as the caller left them
                    of::flash_attention_qk_pv_tile_ws(q, k, v, o, shape, opt, ws);
                    continue;
                }
                std::vector<float> qv(q, q + p->m * p->d), kv(k, k + p->n * p->d), vv(v, v + p->n * p->dv);
                std::vector<float> out;
                switch (variant) {
                    case Variant::Standard: out = of::standard_attention(qv, kv, vv, shape, opt); break;
                    case Variant::Tiled: out = of::flash_attention_tiled(qv, kv, vv, shape, opt); break;
                    case Variant::QTile: out = of::flash_attention_q_tile(qv, kv, vv, shape, opt); break;
                    default: out = of::flash_attention_qk_pv_tile(qv, kv, vv, shape, opt); break;
                }
                std::copy(out.begin(), out.end(), o);
            }
        } catch (const std::exception&) {
            status[t] = ODF_ORACLE_EREF;
        }
    };
    if (nt == 1) {
        worker(0);
    } else {
        std::vector<std::thread> pool;
        for (int t = 0; t < nt; ++t) pool.emplace_back(worker, t);
        for (auto& th : pool) th.join();
    }
    for (int s : status) if (s) return s;
    return ODF_ORACLE_OK;
}

int copy_string(const std::string& s, char* buf, int cap) {
    if (!buf || cap <= 0) return static_cast<int>(s.size());
    const int n = std::min<int>(cap - 1, static_cast<int>(s.size()));
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
    return static_cast<int>(s.size());
}

}  // namespace

extern "C" {

int odf_ref_flash_ws(const odf_oracle_params* p) { return run(p, Variant::Ws); }
int odf_ref_standard(const odf_oracle_params* p) { return run(p, Variant::Standard); }
int odf_ref_tiled(const odf_oracle_params* p) { return run(p, Variant::Tiled); }
int odf_ref_q_tile(const odf_oracle_params* p) { return run(p, Variant::QTile); }
int odf_ref_qk_pv_tile(const odf_oracle_params* p) { return run(p, Variant::QkPvTile); }

// flash_attention_batched_qk_pv_tile as shipped: serial, one thread_local workspace,
// heads of Q/K/V equal (no GQA), no bias functor.
int odf_ref_batched(const odf_oracle_params* p) {
    if (!p || p->heads_q != p->heads_kv || p->alibi_slopes || p->bias || p->lse) return ODF_ORACLE_EUNSUPPORTED;
    of::BlockMask mask;
    of::AttentionOptions opt;
    if (!make_options(p, &mask, &opt)) return ODF_ORACLE_EUNSUPPORTED;
    const of::BatchedAttentionShape shape{
        static_cast<std::size_t>(p->batch), static_cast<std::size_t>(p->heads_q),
        static_cast<std::size_t>(p->m), static_cast<std::size_t>(p->n),
        static_cast<std::size_t>(p->d), static_cast<std::size_t>(p->dv)};
    try {
        of::flash_attention_batched_qk_pv_tile(p->q, p->k, p->v, p->o, shape, opt);
    } catch (const std::exception&) {
        return ODF_ORACLE_EREF;
    }
    return ODF_ORACLE_OK;
}

// make_score_mod_plan (score_mod_plan.cpp:115-182) -> "kind|dtype|has_scale|scale|bias|has_bias|lowering|fallback|signature"
int odf_ref_score_mod_plan(int kind, int dtype, int has_scale, float scale, int bias_kind,
                           int post_ops_available, char* buf, int cap) {
    const auto plan = of::make_score_mod_plan(static_cast<of::ScoreModKind>(kind),
                                              static_cast<of::DataType>(dtype), has_scale != 0, scale,
                                              static_cast<of::BiasKind>(bias_kind), post_ops_available != 0);
    std::string s = std::string(of::to_string(plan.kind)) + "|" + of::to_string(plan.dtype) + "|" +
                    (plan.has_scale ? "1" : "0") + "|" + std::to_string(plan.scale_value) + "|" +
                    of::to_string(plan.bias_kind) + "|" + (plan.has_bias ? "1" : "0") + "|" +
                    of::to_string(plan.lowering_status) + "|" + of::to_string(plan.fallback_reason) + "|" +
                    plan.signature;
    return copy_string(s, buf, cap);
}

// make_runtime_plan (runtime_plan.cpp:112-183) + make_runtime_plan_cache_key (:185-199).
int odf_ref_runtime_plan(const int* ints, float scale, int one_dnn_available, int post_ops_available,
                         char* buf, int cap) {
    of::RuntimePlanInput in;
    in.batch = ints[0]; in.heads = ints[1]; in.query_length = ints[2]; in.key_length = ints[3];
    in.head_dim = ints[4]; in.value_dim = ints[5];
    in.q_dtype = static_cast<of::DataType>(ints[6]); in.k_dtype = static_cast<of::DataType>(ints[7]);
    in.v_dtype = static_cast<of::DataType>(ints[8]); in.out_dtype = static_cast<of::DataType>(ints[9]);
    in.requested_score_mod = static_cast<of::ScoreModKind>(ints[10]);
    in.has_scale = ints[11] != 0;
    in.scale_value = scale;
    in.requested_bias_kind = static_cast<of::BiasKind>(ints[12]);
    in.requested_block_mask = static_cast<of::BlockMaskKind>(ints[13]);
    in.force_reference = ints[14] != 0; in.enable_onednn = ints[15] != 0; in.enable_debug = ints[16] != 0;
    const auto plan = of::make_runtime_plan(in, one_dnn_available != 0, post_ops_available != 0);
    const auto key = of::make_runtime_plan_cache_key(plan);
    std::string s = plan.runtime_plan_signature + "\n" + plan.debug_summary + "\n" +
                    of::to_string(plan.qk_backend) + "|" + of::to_string(plan.qk_layout) + "|" +
                    of::to_string(plan.qk_lowering_status) + "|" + (plan.uses_onednn_post_ops ? "1" : "0") +
                    "|" + (plan.requires_onednn_flash_epilogue ? "1" : "0") + "|" +
                    (plan.requires_mask_tile_generator ? "1" : "0") + "|" + of::to_string(plan.fallback_reason) +
                    "\n" + key.semantic_shape + "|" + key.dtype_signature + "|" + key.score_mod_signature +
                    "|" + key.block_mask_signature + "|" + key.policy_signature;
    return copy_string(s, buf, cap);
}

// make_block_mask_plan (runtime_plan.cpp:72-95) and make_causal_mask_tile_descriptor (:97-110).
int odf_ref_block_mask_plan(int kind, int query_length, int key_length, char* buf, int cap) {
    const auto plan = of::make_block_mask_plan(static_cast<of::BlockMaskKind>(kind), query_length, key_length);
    std::string s = std::string(of::to_string(plan.kind)) + "|" + (plan.has_boundary_tiles ? "1" : "0") + "|" +
                    (plan.can_skip_tiles ? "1" : "0") + "|" + (plan.requires_mask_tile_generator ? "1" : "0") +
                    "|" + of::to_string(plan.fallback_reason) + "|" + plan.signature;
    return copy_string(s, buf, cap);
}

int odf_ref_causal_mask_tile(int q_start, int k_start, int q_size, int k_size, char* buf, int cap) {
    const auto d = of::make_causal_mask_tile_descriptor(q_start, k_start, q_size, k_size);
    std::string s = std::string(d.required ? "1" : "0") + "|" + std::to_string(d.q_start) + "|" +
                    std::to_string(d.k_start) + "|" + std::to_string(d.q_size) + "|" + std::to_string(d.k_size) +
                    "|" + std::to_string(d.masked_value) + "|" + (d.all_masked_row_possible ? "1" : "0");
    return copy_string(s, buf, cap);
}

const char* odf_ref_backend_name(int kind) { return of::backend_name(static_cast<of::AttentionBackendKind>(kind)); }
const char* odf_ref_tile_kernel_name(int kind) { return of::tile_kernel_name(static_cast<of::TileKernelKind>(kind)); }

}  // extern "C"
