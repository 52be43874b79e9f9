// flash_fwd_sm100.cu -- tiled attention forward for B200 (sm_100a).
//
// One CTA computes one 128-row query tile of one (batch, q-head) and walks the
// KV tiles the tiling does not skip.  It replaces the query-block and key-block
// loops of the reference's flash_attention_qk_pv_tile_ws
// (src/onednn_flash/attention.cpp:513-688): the two scalar tile GEMMs
// (tile_kernel.cpp:57-85) become tcgen05 MMAs with operands staged in shared
// memory by TMA and accumulators in tensor memory, and the per-row online
// softmax (attention.cpp:602-674) runs in registers, one thread per query row.
//
// Warp roles (192 threads):
//   warps 0-3  softmax + correction + epilogue; thread t owns query row t,
//              which is TMEM lane t, so row max / row sum need no shuffles.
//   warp  4    TMA producer: Q once, then K and V of each KV tile into a
//              STAGES-deep ring.
//   warp  5    MMA issuer (one thread): S = Q K^T into a double-buffered TMEM
//              S region, then O += P V once the softmax has published P.
// The MMA of S(j+1) runs while the softmax works on S(j), and the P V MMA of
// tile j runs while the softmax computes the exponentials of tile j+1.
//
// TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+D).
// Shared memory (1024-byte aligned 128B-swizzled tiles):
//   Q [128 x D] | K ring [STAGES][128 x D] | V ring [STAGES][128 x D] | P [128 x 128] | barriers
// Every wait is bounded (2 s); on timeout the CTA records ODF_ERR_DEVICE_TIMEOUT
// in the device status word, every role leaves its loop, and the TMEM columns
// are freed before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <math.h>
#include <mutex>

#include "odf_internal.h"
#include "sm100_ptx.cuh"

namespace odf {

namespace {

constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kChunkBytes = 128 * 128;  // 128 rows x 128 bytes (64 bf16)
constexpr uint32_t kPBytes = 128 * 128 * 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum ModFlags { kModAlibi = 1, kModSoftcap = 2 };

template <int D>
struct Config {
    static constexpr int kStages = (D == 64) ? 3 : 2;
    static constexpr int kChunks = D / 64;
    static constexpr uint32_t kQBytes = 128 * D * 2;
    static constexpr uint32_t kKVBytes = 128 * D * 2;
    static constexpr uint32_t kOffK = kQBytes;
    static constexpr uint32_t kOffV = kOffK + kStages * kKVBytes;
    static constexpr uint32_t kOffP = kOffV + kStages * kKVBytes;
    static constexpr uint32_t kOffBar = kOffP + kPBytes;
    static constexpr int kNumBars = 1 + 3 * kStages + 2 + 2 + 1 + 1 + 1;
    static constexpr uint32_t kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
};

struct Bars {
    uint64_t* q_full;
    uint64_t* k_full;
    uint64_t* v_full;
    uint64_t* kv_empty;
    uint64_t* s_full;
    uint64_t* s_free;
    uint64_t* p_full;
    uint64_t* pv_done;
    uint64_t* drain;
};

__device__ __forceinline__ int tile_kt(const FwdArgs& a, int qt, int i, uint32_t* flags) {
    if (a.mode == kModeList) {
        const uint32_t e = a.tile_list[static_cast<int64_t>(qt) * a.n_kt + i];
        *flags = e & 0xFFFF0000u;
        return static_cast<int>(e & 0xFFFFu);
    }
    *flags = 0;
    return i;
}

__device__ __forceinline__ bool mask_allows(const FwdArgs& a, int qi, int kj) {
    const int qb = qi / a.mask_qbs;
    const int kb = kj / a.mask_kbs;
    if (qb >= a.mask_qblocks || kb >= a.mask_kblocks) return false;
    return __ldg(a.mask + static_cast<int64_t>(qb) * a.mask_kblocks + kb) != 0;
}

// Accurate tanh from the identity tanh(t) = 1 - 2 / (1 + e^(2t)); absolute error
// a few fp32 ulps of 1, which keeps softcap * tanh within ~1e-5 of the fp32 value.
__device__ __forceinline__ float tanh_acc(float t) {
    const float e = ptx::ex2(t * (2.0f * kLog2e));
    return 1.0f - 2.0f * ptx::rcp(1.0f + e);
}

template <int D, int MOD>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ FwdArgs args) {
    using Cfg = Config<D>;
    constexpr int kStages = Cfg::kStages;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = ptx::smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* sQ = smem;
    uint8_t* sK = smem + Cfg::kOffK;
    uint8_t* sV = smem + Cfg::kOffV;
    uint8_t* sP = smem + Cfg::kOffP;
    uint64_t* bar_base = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    Bars bars;
    bars.q_full = bar_base;
    bars.k_full = bar_base + 1;
    bars.v_full = bars.k_full + kStages;
    bars.kv_empty = bars.v_full + kStages;
    bars.s_full = bars.kv_empty + kStages;
    bars.s_free = bars.s_full + 2;
    bars.p_full = bars.s_free + 2;
    bars.pv_done = bars.p_full + 1;
    bars.drain = bars.pv_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars.drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bh = blockIdx.x;
    const int qt = args.n_qt - 1 - static_cast<int>(blockIdx.y);  // longest causal rows first
    const int b = bh / args.heads_q;
    const int h = bh - b * args.heads_q;
    const int hk = h / (args.heads_q / args.heads_kv);
    const int q0 = qt * kTileQ;
    const int q_end = min(args.m, q0 + kTileQ);

    int n_tiles;
    if (args.mode == kModeList) {
        n_tiles = args.tile_count[qt];
    } else if (args.mode == kModeCausal) {
        n_tiles = min(args.n_kt, (q_end + kTileK - 1) / kTileK);
    } else {
        n_tiles = args.n_kt;
    }

    if (threadIdx.x == 0) {
        ptx::mbar_init(bars.q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            ptx::mbar_init(&bars.k_full[s], 1);
            ptx::mbar_init(&bars.v_full[s], 1);
            ptx::mbar_init(&bars.kv_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            ptx::mbar_init(&bars.s_full[s], 1);
            ptx::mbar_init(&bars.s_free[s], 128);
        }
        ptx::mbar_init(bars.p_full, 128);
        ptx::mbar_init(bars.pv_done, 1);
        ptx::mbar_init(bars.drain, 1);
        *abort_flag = 0;
        ptx::fence_barrier_init();
        ptx::fence_proxy_async_smem();
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_slot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0 && n_tiles > 0) {
            ptx::prefetch_tmap(&tmQ);
            ptx::prefetch_tmap(&tmK);
            ptx::prefetch_tmap(&tmV);
            ptx::mbar_arrive_expect_tx(bars.q_full, Cfg::kQBytes);
            for (int c = 0; c < Cfg::kChunks; ++c) {
                ptx::tma_load_4d(sQ + c * kChunkBytes, &tmQ, bars.q_full, c * 64, q0, h, b);
            }
            int issued = 0;
            for (int i = 0; i < n_tiles; ++i) {
                const int s = i % kStages;
                uint32_t fl;
                const int kt = tile_kt(args, qt, i, &fl);
                if (i >= kStages) {
                    if (!ptx::mbar_wait(&bars.kv_empty[s], ((i / kStages) - 1) & 1, abort_flag, args.status,
                                        ODF_ERR_DEVICE_TIMEOUT, kWaitLimitNs))
                        break;
                }
                uint8_t* dk = sK + s * Cfg::kKVBytes;
                uint8_t* dv = sV + s * Cfg::kKVBytes;
                ptx::mbar_arrive_expect_tx(&bars.k_full[s], Cfg::kKVBytes);
                for (int c = 0; c < Cfg::kChunks; ++c) {
                    ptx::tma_load_4d(dk + c * kChunkBytes, &tmK, &bars.k_full[s], c * 64, kt * kTileK, hk, b);
                }
                ptx::mbar_arrive_expect_tx(&bars.v_full[s], Cfg::kKVBytes);
                for (int c = 0; c < Cfg::kChunks; ++c) {
                    ptx::tma_load_4d(dv + c * kChunkBytes, &tmV, &bars.v_full[s], c * 64, kt * kTileK, hk, b);
                }
                ++issued;
            }
            if (*abort_flag) {
                // Let copies already issued land before the CTA's shared memory is released.
                volatile int no_abort = 0;
                const int first = issued > kStages ? issued - kStages : 0;
                for (int i = first; i < issued; ++i) {
                    ptx::mbar_wait(&bars.k_full[i % kStages], (i / kStages) & 1, &no_abort, nullptr, 0, kWaitLimitNs);
                    ptx::mbar_wait(&bars.v_full[i % kStages], (i / kStages) & 1, &no_abort, nullptr, 0, kWaitLimitNs);
                }
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0 && n_tiles > 0) {
            constexpr uint32_t kIdescQK = ptx::make_idesc_bf16(128, 128, false);
            constexpr uint32_t kIdescPV = ptx::make_idesc_bf16(128, D, true);
            const uint32_t aQ = ptx::smem_u32(sQ);
            const uint32_t aK = ptx::smem_u32(sK);
            const uint32_t aV = ptx::smem_u32(sV);
            const uint32_t aP = ptx::smem_u32(sP);

            auto issue_pv = [&](int j) -> bool {
                const int s = j % kStages;
                if (!ptx::mbar_wait(&bars.v_full[s], (j / kStages) & 1, abort_flag, args.status,
                                    ODF_ERR_DEVICE_TIMEOUT, kWaitLimitNs))
                    return false;
                if (!ptx::mbar_wait(bars.p_full, j & 1, abort_flag, args.status, ODF_ERR_DEVICE_TIMEOUT,
                                    kWaitLimitNs))
                    return false;
                ptx::tc_fence_after();
                const uint32_t vbase = aV + s * Cfg::kKVBytes;
#pragma unroll
                for (int kk = 0; kk < kTileK / 16; ++kk) {
                    const uint64_t pdesc =
                        ptx::make_sdesc_sw128(aP + (kk >> 2) * kChunkBytes + (kk & 3) * 32, 16, 1024);
                    const uint64_t vdesc = ptx::make_sdesc_sw128(vbase + kk * 2048, kChunkBytes, 1024);
                    ptx::mma_bf16_ss(tmem + kTmemO, pdesc, vdesc, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
                }
                ptx::tc_commit(&bars.kv_empty[s]);
                ptx::tc_commit(bars.pv_done);
                return true;
            };

            bool ok = ptx::mbar_wait(bars.q_full, 0, abort_flag, args.status, ODF_ERR_DEVICE_TIMEOUT,
                                     kWaitLimitNs);
            for (int i = 0; ok && i < n_tiles; ++i) {
                const int s = i % kStages;
                const int sb = i & 1;
                if (!ptx::mbar_wait(&bars.k_full[s], (i / kStages) & 1, abort_flag, args.status,
                                    ODF_ERR_DEVICE_TIMEOUT, kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                if (i >= 2 && !ptx::mbar_wait(&bars.s_free[sb], ((i >> 1) - 1) & 1, abort_flag, args.status,
                                              ODF_ERR_DEVICE_TIMEOUT, kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t kbase = aK + s * Cfg::kKVBytes;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
                    const uint64_t qdesc = ptx::make_sdesc_sw128(aQ + off, 16, 1024);
                    const uint64_t kdesc = ptx::make_sdesc_sw128(kbase + off, 16, 1024);
                    ptx::mma_bf16_ss(tmem + sb * 128, qdesc, kdesc, kIdescQK, kk > 0 ? 1u : 0u);
                }
                ptx::tc_commit(&bars.s_full[sb]);
                if (i >= 1 && !issue_pv(i - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok) ok = issue_pv(n_tiles - 1);
            if (!ok) {
                // Drain the MMAs already issued before the TMEM columns are freed.
                volatile int no_abort = 0;
                ptx::tc_commit(bars.drain);
                ptx::mbar_wait(bars.drain, 0, &no_abort, nullptr, 0, kWaitLimitNs);
            }
        }
    } else {
        // ------------------------------------------------------------ softmax warps 0-3
        const int row = threadIdx.x;  // 0..127 == TMEM lane
        const int qi = q0 + row;
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        float m_run = -INFINITY;  // running max, log2 units
        float l_run = 0.0f;       // running sum relative to m_run
        float slope = 0.0f;
        if (MOD & kModAlibi) {
            slope = args.alibi_generated ? exp2f(-8.0f * static_cast<float>(h + 1) / static_cast<float>(args.heads_q))
                                         : args.alibi_slopes[h];
        }
        const float slope_log2 = slope * kLog2e;
        bool ok = true;
        const uint32_t p_row = ptx::smem_u32(sP) + row * 128;
        const uint32_t swz = static_cast<uint32_t>(row & 7);

        for (int i = 0; i < n_tiles; ++i) {
            uint32_t fl;
            const int kt = tile_kt(args, qt, i, &fl);
            const int k0 = kt * kTileK;
            const int sb = i & 1;
            // Waits are per thread; the warp re-converges (and agrees) before the
            // .sync.aligned TMEM accesses that follow.
            const bool got_s = ptx::mbar_wait(&bars.s_full[sb], (i >> 1) & 1, abort_flag, args.status,
                                              ODF_ERR_DEVICE_TIMEOUT, kWaitLimitNs);
            if (!__all_sync(0xffffffffu, got_s)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            float s[128];
#pragma unroll
            for (int c = 0; c < 4; ++c) ptx::tmem_ld32(tmem + lane_off + sb * 128 + c * 32, &s[c * 32]);
            ptx::tc_fence_before();
            ptx::mbar_arrive(&bars.s_free[sb]);
            if (row == 0 && args.visits) {
                args.visits[(static_cast<int64_t>(bh) * args.n_qt + qt) * args.n_kt + kt] = 1;
            }

            // score_mod: s*scale (+ ALiBi) (-> soft-cap), in log2 units (attention.cpp:619)
            if (MOD & kModSoftcap) {
                const float base = static_cast<float>(k0 - qi);
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    float x = s[c] * args.scale;
                    if (MOD & kModAlibi) x = fmaf(slope, base + static_cast<float>(c), x);
                    x = args.softcap * tanh_acc(x * args.inv_softcap);
                    s[c] = x * kLog2e;
                }
            } else if (MOD & kModAlibi) {
                const float base = static_cast<float>(k0 - qi);
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    s[c] = fmaf(s[c], args.scale_log2, slope_log2 * (base + static_cast<float>(c)));
                }
            } else {
#pragma unroll
                for (int c = 0; c < 128; ++c) s[c] *= args.scale_log2;
            }

            // element mask on boundary tiles (attention.cpp:54-62, 608-617)
            const bool ragged = (k0 + kTileK > args.n);
            const bool diag = args.causal && (min(args.n, k0 + kTileK) - 1 > q0);
            const bool bitmap = (fl & kListBitmapPartial) != 0;
            if (ragged || diag || bitmap) {
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    const int kj = k0 + c;
                    bool masked = kj >= args.n;
                    if (args.causal) masked = masked || (kj > qi);
                    if (bitmap) masked = masked || !mask_allows(args, qi, kj);
                    if (masked) s[c] = -INFINITY;
                }
            }

            // online softmax (attention.cpp:628-644, 662-674)
            float mx = m_run;
#pragma unroll
            for (int c = 0; c < 128; ++c) mx = fmaxf(mx, s[c]);
            const float m_use = (mx == -INFINITY) ? 0.0f : mx;
            const float alpha = ptx::ex2(m_run - m_use);
            float sum = 0.0f;
#pragma unroll
            for (int c = 0; c < 128; ++c) {
                s[c] = ptx::ex2(s[c] - m_use);
                sum += s[c];
            }
            l_run = l_run * alpha + sum;
            m_run = mx;

            if (i > 0) {
                // P buffer and O are owned by the P V MMA of the previous tile until it completes.
                const bool got_pv = ptx::mbar_wait(bars.pv_done, (i - 1) & 1, abort_flag, args.status,
                                                   ODF_ERR_DEVICE_TIMEOUT, kWaitLimitNs);
                if (!__all_sync(0xffffffffu, got_pv)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
            }
            // P (bf16) into the 128B-swizzled K-major layout the P V MMA reads.
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const uint32_t addr = p_row + (u >> 3) * kChunkBytes + ((((u & 7) ^ swz)) << 4);
                ptx::st_shared_v4(addr, ptx::pack_bf16x2(s[8 * u + 0], s[8 * u + 1]),
                                  ptx::pack_bf16x2(s[8 * u + 2], s[8 * u + 3]),
                                  ptx::pack_bf16x2(s[8 * u + 4], s[8 * u + 5]),
                                  ptx::pack_bf16x2(s[8 * u + 6], s[8 * u + 7]));
            }
            // correction: O *= alpha when the running max moved
            if (i > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    float o[32];
                    ptx::tmem_ld32(tmem + lane_off + kTmemO + c * 32, o);
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] *= alpha;
                    ptx::tmem_st32(tmem + lane_off + kTmemO + c * 32, o);
                }
            }
            ptx::fence_proxy_async_smem();
            ptx::tc_fence_before();
            ptx::mbar_arrive(bars.p_full);
        }

        // ------------------------------------------------------------ epilogue
        if (ok && n_tiles > 0) {
            ok = ptx::mbar_wait(bars.pv_done, (n_tiles - 1) & 1, abort_flag, args.status, ODF_ERR_DEVICE_TIMEOUT,
                                kWaitLimitNs);
            ptx::tc_fence_after();
        }
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            const bool valid_row = qi < args.m;
            const float inv_l = (l_run > 0.0f) ? (1.0f / l_run) : 0.0f;
            const int64_t orow = static_cast<int64_t>(b) * args.o_stride_b + static_cast<int64_t>(h) * args.o_stride_h +
                                 static_cast<int64_t>(qi) * args.o_stride_t;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                float o[32];
                if (n_tiles > 0) {
                    ptx::tmem_ld32(tmem + lane_off + kTmemO + c * 32, o);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = 0.0f;
                }
                if (valid_row) {
                    if (args.o_bf16) {
                        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.o) + orow + c * 32);
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint4 w;
                            w.x = ptx::pack_bf16x2(o[8 * v + 0] * inv_l, o[8 * v + 1] * inv_l);
                            w.y = ptx::pack_bf16x2(o[8 * v + 2] * inv_l, o[8 * v + 3] * inv_l);
                            w.z = ptx::pack_bf16x2(o[8 * v + 4] * inv_l, o[8 * v + 5] * inv_l);
                            w.w = ptx::pack_bf16x2(o[8 * v + 6] * inv_l, o[8 * v + 7] * inv_l);
                            dst[v] = w;
                        }
                    } else {
                        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(args.o) + orow + c * 32);
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            dst[v] = make_float4(o[4 * v + 0] * inv_l, o[4 * v + 1] * inv_l, o[4 * v + 2] * inv_l,
                                                 o[4 * v + 3] * inv_l);
                        }
                    }
                }
            }
            if (valid_row && args.lse) {
                const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
                args.lse[static_cast<int64_t>(bh) * args.m + qi] =
                    (l_run > 0.0f) ? (m_use + log2f(l_run)) * kLn2 : -INFINITY;
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

// Tile classification / compaction: one warp per query tile, in increasing kv order.
__global__ void tile_map_kernel(int32_t m, int32_t n, int32_t n_qt, int32_t n_kt, int32_t causal,
                                const uint8_t* __restrict__ mask, int32_t mqbs, int32_t mkbs, int32_t mqblocks,
                                int32_t mkblocks, uint32_t* __restrict__ list, int32_t* __restrict__ count,
                                uint8_t* __restrict__ cls_out) {
    const int qt = blockIdx.x;
    const int lane = threadIdx.x;
    if (qt >= n_qt) return;
    const int q0 = qt * kTileQ;
    const int q1 = min(m, q0 + kTileQ);
    int base = 0;
    for (int kt0 = 0; kt0 < n_kt; kt0 += 32) {
        const int kt = kt0 + lane;
        uint32_t cls = 0, flags = 0;
        if (kt < n_kt) {
            const int k0 = kt * kTileK;
            const int k1 = min(n, k0 + kTileK);
            cls = 1;
            if (causal && k0 >= q1) {
                cls = 0;
            } else {
                if (causal && k1 - 1 > q0) cls = 2;
                if (mask) {
                    bool any_allowed = false, any_denied = false;
                    for (int qb = q0 / mqbs; qb <= (q1 - 1) / mqbs; ++qb) {
                        for (int kb = k0 / mkbs; kb <= (k1 - 1) / mkbs; ++kb) {
                            const bool okb = qb < mqblocks && kb < mkblocks &&
                                             mask[static_cast<int64_t>(qb) * mkblocks + kb] != 0;
                            any_allowed |= okb;
                            any_denied |= !okb;
                        }
                    }
                    if (!any_allowed) {
                        cls = 0;
                    } else if (any_denied) {
                        cls = 2;
                        flags |= kListBitmapPartial;
                    }
                }
            }
            if (cls_out) cls_out[static_cast<int64_t>(qt) * n_kt + kt] = static_cast<uint8_t>(cls);
        }
        const unsigned ballot = __ballot_sync(0xffffffffu, cls != 0);
        if (cls != 0 && list) {
            const int pos = base + __popc(ballot & ((1u << lane) - 1u));
            list[static_cast<int64_t>(qt) * n_kt + pos] = static_cast<uint32_t>(kt) | flags;
        }
        base += __popc(ballot);
    }
    if (lane == 0 && count) count[qt] = base;
}

__global__ void convert_f32_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
    for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
        if (i + 3 < n && (reinterpret_cast<uintptr_t>(in + i) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(out + i) & 7) == 0) {
            const float4 f = *reinterpret_cast<const float4*>(in + i);
            __nv_bfloat162 lo = __floats2bfloat162_rn(f.x, f.y);
            __nv_bfloat162 hi = __floats2bfloat162_rn(f.z, f.w);
            uint2 w;
            w.x = *reinterpret_cast<uint32_t*>(&lo);
            w.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(out + i) = w;
        } else {
            for (int64_t j = i; j < i + 4 && j < n; ++j) out[j] = __float2bfloat16_rn(in[j]);
        }
    }
}

__device__ int g_device_status;

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

struct DeviceState {
    bool ready = false;
    int status_code = ODF_OK;
    int* status_ptr = nullptr;
};
constexpr int kMaxDevices = 64;
DeviceState g_devices[kMaxDevices];
std::mutex g_device_mutex;

template <int D, int MOD>
cudaError_t set_kernel_attrs() {
    return cudaFuncSetAttribute(flash_fwd_kernel<D, MOD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                Config<D>::kSmemBytes);
}

CUresult encode_bf16_4d(CUtensorMap* map, const void* ptr, int64_t feat, int64_t tokens, int64_t heads,
                        int64_t batch, const int64_t strides[3]) {
    // strides[] = {batch, head, token} in elements; TMA wants {token, head, batch} in bytes.
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(feat), static_cast<cuuint64_t>(tokens),
                          static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
    cuuint64_t byte_strides[3] = {static_cast<cuuint64_t>(strides[2]) * 2, static_cast<cuuint64_t>(strides[1]) * 2,
                                  static_cast<cuuint64_t>(strides[0]) * 2};
    cuuint32_t box[4] = {64, 128, 1, 1};
    cuuint32_t elem_strides[4] = {1, 1, 1, 1};
    return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, byte_strides, box,
                    elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int D>
cudaError_t launch_d(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FwdArgs& a,
                     int mod, dim3 grid, cudaStream_t stream) {
    const size_t smem = Config<D>::kSmemBytes;
    switch (mod) {
        case 0: flash_fwd_kernel<D, 0><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        case 1: flash_fwd_kernel<D, 1><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        case 2: flash_fwd_kernel<D, 2><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        default: flash_fwd_kernel<D, 3><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
    }
    return cudaGetLastError();
}

}  // namespace

size_t workspace_bytes_for(int64_t seqlen_q, int64_t seqlen_k, bool has_mask) {
    if (!has_mask) return 0;
    const int64_t n_qt = (seqlen_q + kTileQ - 1) / kTileQ;
    const int64_t n_kt = (seqlen_k + kTileK - 1) / kTileK;
    const size_t list = static_cast<size_t>(n_qt * n_kt) * sizeof(uint32_t);
    const size_t count = static_cast<size_t>(n_qt) * sizeof(int32_t);
    return ((list + 255) & ~static_cast<size_t>(255)) + ((count + 255) & ~static_cast<size_t>(255));
}

int ensure_device_ready(int device, const char** err) {
    if (device < 0 || device >= kMaxDevices) {
        *err = "device index out of range";
        return ODF_ERR_NO_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_device_mutex);
    DeviceState& st = g_devices[device];
    if (st.ready) return ODF_OK;
    if (st.status_code != ODF_OK) {
        *err = "device previously failed initialisation (needs an sm_100 GPU)";
        return st.status_code;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        *err = "cudaGetDeviceProperties failed";
        return ODF_ERR_CUDA;
    }
    if (prop.major != 10) {
        st.status_code = ODF_ERR_NO_DEVICE;
        *err = "the sm_100a kernels need a compute capability 10.x (B200-class) device";
        return ODF_ERR_NO_DEVICE;
    }
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
    });
    if (!g_encode) {
        *err = "cuTensorMapEncodeTiled is not available from the driver";
        return ODF_ERR_CUDA;
    }
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = set_kernel_attrs<64, 0>();
    if (e == cudaSuccess) e = set_kernel_attrs<64, 1>();
    if (e == cudaSuccess) e = set_kernel_attrs<64, 2>();
    if (e == cudaSuccess) e = set_kernel_attrs<64, 3>();
    if (e == cudaSuccess) e = set_kernel_attrs<128, 0>();
    if (e == cudaSuccess) e = set_kernel_attrs<128, 1>();
    if (e == cudaSuccess) e = set_kernel_attrs<128, 2>();
    if (e == cudaSuccess) e = set_kernel_attrs<128, 3>();
    void* sp = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&sp, g_device_status);
    if (e != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return ODF_ERR_CUDA;
    }
    st.status_ptr = static_cast<int*>(sp);
    st.ready = true;
    return ODF_OK;
}

int* device_status_ptr(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_device_mutex);
    return g_devices[device].status_ptr;
}

int launch_tile_map(int32_t m, int32_t n, int32_t causal, const uint8_t* mask, int32_t mqbs, int32_t mkbs,
                    int32_t mqblocks, int32_t mkblocks, uint32_t* list, int32_t* count, uint8_t* cls_out,
                    cudaStream_t stream) {
    const int n_qt = (m + kTileQ - 1) / kTileQ;
    const int n_kt = (n + kTileK - 1) / kTileK;
    tile_map_kernel<<<n_qt, 32, 0, stream>>>(m, n, n_qt, n_kt, causal, mask, mqbs, mkbs, mqblocks, mkblocks, list,
                                              count, cls_out);
    return cudaGetLastError() == cudaSuccess ? ODF_OK : ODF_ERR_CUDA;
}

int launch_convert_f32_bf16(const float* in, uint16_t* out, int64_t count, cudaStream_t stream) {
    if (count <= 0) return ODF_OK;
    int64_t blocks = (count / 4 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 148 * 16) blocks = 148 * 16;
    convert_f32_bf16_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        in, reinterpret_cast<__nv_bfloat16*>(out), count);
    return cudaGetLastError() == cudaSuccess ? ODF_OK : ODF_ERR_CUDA;
}

int launch_flash_fwd(FwdLaunch& L, cudaStream_t stream, const char** err) {
    FwdArgs& a = L.args;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        *err = "cudaGetDevice failed";
        return ODF_ERR_CUDA;
    }
    int rc = ensure_device_ready(device, err);
    if (rc != ODF_OK) return rc;
    a.status = device_status_ptr(device);

    CUtensorMap tq, tk, tv;
    if (encode_bf16_4d(&tq, L.q, L.head_dim, a.m, a.heads_q, a.batch, L.q_strides) != CUDA_SUCCESS ||
        encode_bf16_4d(&tk, L.k, L.head_dim, a.n, a.heads_kv, a.batch, L.k_strides) != CUDA_SUCCESS ||
        encode_bf16_4d(&tv, L.v, L.head_dim, a.n, a.heads_kv, a.batch, L.v_strides) != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled rejected a Q/K/V layout (pointers and strides must be 16-byte aligned)";
        return ODF_ERR_INVALID_ARG;
    }
    if (a.mode == kModeList) {
        uint8_t* ws = static_cast<uint8_t*>(L.workspace);
        const size_t list_bytes = static_cast<size_t>(a.n_qt) * a.n_kt * sizeof(uint32_t);
        uint32_t* list = reinterpret_cast<uint32_t*>(ws);
        int32_t* count = reinterpret_cast<int32_t*>(ws + ((list_bytes + 255) & ~static_cast<size_t>(255)));
        rc = launch_tile_map(a.m, a.n, a.causal, a.mask, a.mask_qbs, a.mask_kbs, a.mask_qblocks, a.mask_kblocks,
                             list, count, nullptr, stream);
        if (rc != ODF_OK) {
            *err = "tile-list kernel launch failed";
            return rc;
        }
        a.tile_list = list;
        a.tile_count = count;
    }
    const int mod = (L.has_alibi ? kModAlibi : 0) | (L.has_softcap ? kModSoftcap : 0);
    const dim3 grid(static_cast<unsigned>(a.batch * a.heads_q), static_cast<unsigned>(a.n_qt), 1);
    cudaError_t e = (L.head_dim == 64) ? launch_d<64>(tq, tk, tv, a, mod, grid, stream)
                                       : launch_d<128>(tq, tk, tv, a, mod, grid, stream);
    if (e != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return ODF_ERR_CUDA;
    }
    return ODF_OK;
}

}  // namespace odf
