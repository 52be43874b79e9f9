// cpp_api_check.cpp -- drives the C++ API (include/onednn_flash/*.hpp) for the pytest suite.
//
//   cpp_api_check planner                      -> planner results, one per line, in the
//                                                 format of oracle/ref_shim.cpp
//   cpp_api_check run <in.bin> <out.bin>       -> one attention call (see read_case)
//
// Built by tests/test_cpp_api.py (nvcc, for the CUDA runtime calls of the device-pointer
// cases) against dnn-flash_b200/lib/libodf_sm100.so.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <vector>

#include "onednn_flash/attention.hpp"
#include "onednn_flash/backend.hpp"
#include "onednn_flash/batched_attention.hpp"
#include "onednn_flash/runtime_plan.hpp"
#include "onednn_flash/score_mod_plan.hpp"

namespace of = onednn_flash;

namespace {

std::string fmt_float(float v) { return std::to_string(v); }

void planner() {
    // make_score_mod_plan over every enum combination
    for (int kind = 0; kind < 5; ++kind)
        for (int dtype = 0; dtype < 3; ++dtype)
            for (int has_scale = 0; has_scale < 2; ++has_scale)
                for (int bias = 0; bias < 6; ++bias)
                    for (int post = 0; post < 2; ++post) {
                        const auto p = of::make_score_mod_plan(static_cast<of::ScoreModKind>(kind),
                                                               static_cast<of::DataType>(dtype), has_scale != 0,
                                                               0.125f, static_cast<of::BiasKind>(bias), post != 0);
                        std::printf("SMP %d %d %d %d %d|%s|%s|%d|%s|%s|%d|%s|%s|%s\n", kind, dtype, has_scale, bias,
                                    post, of::to_string(p.kind), of::to_string(p.dtype), p.has_scale ? 1 : 0,
                                    fmt_float(p.scale_value).c_str(), of::to_string(p.bias_kind), p.has_bias ? 1 : 0,
                                    of::to_string(p.lowering_status), of::to_string(p.fallback_reason),
                                    p.signature.c_str());
                    }
    // make_block_mask_plan / make_causal_mask_tile_descriptor
    for (int kind = 0; kind < 3; ++kind)
        for (int ql : {0, 64, 128})
            for (int kl : {64, 128, 256}) {
                const auto p = of::make_block_mask_plan(static_cast<of::BlockMaskKind>(kind), ql, kl);
                std::printf("BMP %d %d %d|%s|%d|%d|%d|%s|%s\n", kind, ql, kl, of::to_string(p.kind),
                            p.has_boundary_tiles ? 1 : 0, p.can_skip_tiles ? 1 : 0,
                            p.requires_mask_tile_generator ? 1 : 0, of::to_string(p.fallback_reason),
                            p.signature.c_str());
            }
    for (int qs : {0, 16, 128})
        for (int ks : {0, 16, 200})
            for (int qz : {1, 16})
                for (int kz : {16, 64}) {
                    const auto d = of::make_causal_mask_tile_descriptor(qs, ks, qz, kz);
                    std::printf("CMT %d %d %d %d|%d|%d|%d|%d|%d|%s|%d\n", qs, ks, qz, kz, d.required ? 1 : 0,
                                d.q_start, d.k_start, d.q_size, d.k_size, fmt_float(d.masked_value).c_str(),
                                d.all_masked_row_possible ? 1 : 0);
                }
    // make_runtime_plan + cache key over a grid of inputs
    const int shapes[][6] = {{1, 4, 512, 512, 64, 64}, {2, 8, 128, 256, 32, 32}, {0, 4, 512, 512, 64, 64},
                             {1, 1, 1, 0, 64, 64}};
    for (const auto& sh : shapes)
        for (int qd = 0; qd < 2; ++qd)
            for (int od = 0; od < 2; ++od)
                for (int sm = 0; sm < 5; ++sm)
                    for (int bias : {0, 1, 2, 4})
                        for (int bm = 0; bm < 3; ++bm)
                            for (int flags = 0; flags < 8; ++flags)
                                for (int avail = 0; avail < 4; ++avail) {
                                    of::RuntimePlanInput in;
                                    in.batch = sh[0]; in.heads = sh[1]; in.query_length = sh[2];
                                    in.key_length = sh[3]; in.head_dim = sh[4]; in.value_dim = sh[5];
                                    in.q_dtype = in.k_dtype = in.v_dtype = static_cast<of::DataType>(qd);
                                    in.out_dtype = static_cast<of::DataType>(od);
                                    in.requested_score_mod = static_cast<of::ScoreModKind>(sm);
                                    in.has_scale = (sm == 1 || sm == 3);
                                    in.scale_value = 0.25f;
                                    in.requested_bias_kind = static_cast<of::BiasKind>(bias);
                                    in.requested_block_mask = static_cast<of::BlockMaskKind>(bm);
                                    in.force_reference = flags & 1; in.enable_onednn = (flags & 2) != 0;
                                    in.enable_debug = (flags & 4) != 0;
                                    const auto p = of::make_runtime_plan(in, avail & 1, (avail & 2) != 0);
                                    const auto k = of::make_runtime_plan_cache_key(p);
                                    std::printf(
                                        "RTP %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d %d|%s\\n%s\\n%s|%s|%s|%d|%d|%d|%s\\n%s|%s|%s|%s|%s\n",
                                        sh[0], sh[1], sh[2], sh[3], sh[4], sh[5], qd, qd, qd, od, sm, in.has_scale ? 1 : 0,
                                        bias, bm, in.force_reference ? 1 : 0, in.enable_onednn ? 1 : 0,
                                        in.enable_debug ? 1 : 0, avail & 1, (avail & 2) ? 1 : 0,
                                        p.runtime_plan_signature.c_str(), p.debug_summary.c_str(),
                                        of::to_string(p.qk_backend), of::to_string(p.qk_layout),
                                        of::to_string(p.qk_lowering_status), p.uses_onednn_post_ops ? 1 : 0,
                                        p.requires_onednn_flash_epilogue ? 1 : 0, p.requires_mask_tile_generator ? 1 : 0,
                                        of::to_string(p.fallback_reason), k.semantic_shape.c_str(),
                                        k.dtype_signature.c_str(), k.score_mod_signature.c_str(),
                                        k.block_mask_signature.c_str(), k.policy_signature.c_str());
                                }
    for (int kind = 0; kind < 2; ++kind) std::printf("BKN %d|%s\n", kind, of::backend_name(static_cast<of::AttentionBackendKind>(kind)));
    for (int kind = 0; kind < 3; ++kind) std::printf("TKN %d|%s\n", kind, of::tile_kernel_name(static_cast<of::TileKernelKind>(kind)));
    // GPU plan of the sm_100a kernel (addition)
    of::RuntimePlanInput g;
    g.batch = 1; g.heads = 64; g.query_length = 32768; g.key_length = 32768; g.head_dim = 128; g.value_dim = 128;
    g.q_dtype = g.k_dtype = g.v_dtype = g.out_dtype = of::DataType::BF16;
    g.requested_score_mod = of::ScoreModKind::ScaleAdditiveBias;
    g.has_scale = true;
    g.requested_bias_kind = of::BiasKind::AlibiGenerated;
    g.requested_block_mask = of::BlockMaskKind::Causal;
    const auto gp = of::make_sm100_runtime_plan(g, 50.0f);
    std::printf("GPU|%s|%s|%s\n", gp.runtime_plan_signature.c_str(), of::to_string(gp.fallback_reason),
                of::to_string(gp.qk_backend));
    g.head_dim = g.value_dim = 96;
    const auto gp2 = of::make_sm100_runtime_plan(g, 0.0f);
    std::printf("GPU96|%s|%s\n", of::to_string(gp2.fallback_reason), of::to_string(gp2.qk_backend));
}

// Case file (little endian): int32 header[16], float params[4], then q, k, v (fp32), then
// an optional u8 mask, then optional fp32 alibi slopes [H] (bias = 1) or an fp32 bias
// tensor [B, H, M, N] (bias = 2, BiasKind::SameShapeTile with contiguous strides).
//   header: api, B, H, Hkv, M, N, D, DV, causal, q_block, k_block, mask_qbs, mask_kbs,
//           mask_qblocks, mask_kblocks, bias
//   params: scale, softcap, want_lse, device_pointers
//   api: 0 standard_attention, 1 flash_attention_tiled, 2 flash_attention_q_tile,
//        3 flash_attention_qk_pv_tile, 4 flash_attention_qk_pv_tile_ws,
//        5 flash_attention_batched_qk_pv_tile, 6 run_attention(Standard), 7 run_attention(FlashTiled)
// Output file: int32 status (0 ok, 1 invalid_argument, 2 runtime_error), then O (fp32) and LSE.
int run_case(const char* in_path, const char* out_path) {
    FILE* f = std::fopen(in_path, "rb");
    if (!f) return 3;
    int32_t hd[16];
    float pr[4];
    if (std::fread(hd, 4, 16, f) != 16 || std::fread(pr, 4, 4, f) != 4) return 3;
    const int api = hd[0], B = hd[1], H = hd[2], Hkv = hd[3], M = hd[4], N = hd[5], D = hd[6], DV = hd[7];
    std::vector<float> q(static_cast<size_t>(B) * H * M * D), k(static_cast<size_t>(B) * Hkv * N * D),
        v(static_cast<size_t>(B) * Hkv * N * DV);
    if (std::fread(q.data(), 4, q.size(), f) != q.size() || std::fread(k.data(), 4, k.size(), f) != k.size() ||
        std::fread(v.data(), 4, v.size(), f) != v.size())
        return 3;
    of::BlockMask mask;
    const bool has_mask = hd[13] > 0;
    if (has_mask) {
        mask.query_block_size = hd[11];
        mask.key_block_size = hd[12];
        mask.query_blocks = hd[13];
        mask.key_blocks = hd[14];
        mask.allowed.resize(static_cast<size_t>(hd[13]) * hd[14]);
        if (std::fread(mask.allowed.data(), 1, mask.allowed.size(), f) != mask.allowed.size()) return 3;
    }
    std::vector<float> slopes, bias;
    if (hd[15] == 1) {
        slopes.resize(H);
        if (std::fread(slopes.data(), 4, H, f) != static_cast<size_t>(H)) return 3;
    } else if (hd[15] == 2) {
        bias.resize(static_cast<size_t>(B) * H * M * N);
        if (std::fread(bias.data(), 4, bias.size(), f) != bias.size()) return 3;
    }
    std::fclose(f);

    of::AttentionOptions opt;
    opt.scale = pr[0];
    opt.causal = hd[8] != 0;
    opt.query_block_size = static_cast<size_t>(hd[9]);
    opt.key_block_size = static_cast<size_t>(hd[10]);
    opt.block_mask = has_mask ? &mask : nullptr;
    opt.softcap = pr[1];
    if (hd[15] == 1) {
        opt.bias_kind = of::BiasKind::AlibiGenerated;
        opt.alibi_slopes = slopes.data();
    } else if (hd[15] == 2) {
        opt.bias_kind = of::BiasKind::SameShapeTile;
        opt.bias = bias.data();  // all-zero strides: contiguous [B, H, M, N]
    }
    opt.kv_heads = static_cast<size_t>(Hkv);
    std::vector<float> lse(static_cast<size_t>(B) * H * M, 0.0f);
    if (pr[2] != 0.0f) opt.lse = lse.data();
    std::vector<float> out(static_cast<size_t>(B) * H * M * DV, 0.0f);
    int32_t status = 0;
    try {
        const of::AttentionShape shape{static_cast<size_t>(M), static_cast<size_t>(N), static_cast<size_t>(D),
                                       static_cast<size_t>(DV)};
        if (api <= 3 || api >= 6) {
            std::vector<float> r;
            switch (api) {
                case 0: r = of::standard_attention(q, k, v, shape, opt); break;
                case 1: r = of::flash_attention_tiled(q, k, v, shape, opt); break;
                case 2: r = of::flash_attention_q_tile(q, k, v, shape, opt); break;
                case 3: r = of::flash_attention_qk_pv_tile(q, k, v, shape, opt); break;
                case 6: r = of::run_attention(of::AttentionBackendKind::StandardReference, q, k, v, shape, opt); break;
                default: r = of::run_attention(of::AttentionBackendKind::FlashTiledReference, q, k, v, shape, opt); break;
            }
            std::memcpy(out.data(), r.data(), std::min(r.size(), out.size()) * 4);
        } else {
            // Raw-pointer entry points, on host buffers or (params[3] != 0) on device buffers.
            const bool on_device = pr[3] != 0.0f;
            const float *pq = q.data(), *pk = k.data(), *pv = v.data();
            float* po = out.data();
            float *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr, *dlse = nullptr, *dbias = nullptr;
            if (on_device) {
                if (cudaMalloc(&dq, q.size() * 4) || cudaMalloc(&dk, k.size() * 4) || cudaMalloc(&dv, v.size() * 4) ||
                    cudaMalloc(&dout, out.size() * 4) || cudaMalloc(&dlse, lse.size() * 4))
                    throw std::runtime_error("test driver: cudaMalloc failed");
                cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
                cudaMemcpy(dk, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
                cudaMemcpy(dv, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
                pq = dq; pk = dk; pv = dv; po = dout;
                if (opt.lse) opt.lse = dlse;
                if (!bias.empty()) {
                    if (cudaMalloc(&dbias, bias.size() * 4)) throw std::runtime_error("test driver: cudaMalloc failed");
                    cudaMemcpy(dbias, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice);
                    opt.bias = dbias;
                }
            }
            if (api == 4) {
                of::AttentionWorkspace ws;
                of::flash_attention_qk_pv_tile_ws(pq, pk, pv, po, shape, opt, ws);
                of::flash_attention_qk_pv_tile_ws(pq, pk, pv, po, shape, opt, ws);  // reuses the workspace
            } else {
                const of::BatchedAttentionShape bs{static_cast<size_t>(B), static_cast<size_t>(H),
                                                   static_cast<size_t>(M), static_cast<size_t>(N),
                                                   static_cast<size_t>(D), static_cast<size_t>(DV)};
                of::flash_attention_batched_qk_pv_tile(pq, pk, pv, po, bs, opt);
            }
            if (on_device) {
                cudaMemcpy(out.data(), dout, out.size() * 4, cudaMemcpyDeviceToHost);
                cudaMemcpy(lse.data(), dlse, lse.size() * 4, cudaMemcpyDeviceToHost);
                cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dout); cudaFree(dlse);
                if (dbias) cudaFree(dbias);
            }
        }
    } catch (const std::invalid_argument& e) {
        std::fprintf(stderr, "invalid_argument: %s\n", e.what());
        status = 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "runtime_error: %s\n", e.what());
        status = 2;
    }
    FILE* o = std::fopen(out_path, "wb");
    if (!o) return 3;
    std::fwrite(&status, 4, 1, o);
    std::fwrite(out.data(), 4, out.size(), o);
    std::fwrite(lse.data(), 4, lse.size(), o);
    std::fclose(o);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "planner") == 0) {
        planner();
        return 0;
    }
    if (argc >= 4 && std::strcmp(argv[1], "run") == 0) return run_case(argv[2], argv[3]);
    std::fprintf(stderr, "usage: cpp_api_check planner | run <in> <out>\n");
    return 2;
}
