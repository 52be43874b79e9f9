/*
 * odf_oracle.h -- CPU oracle for the tiled attention forward (TEST INFRASTRUCTURE ONLY).
 *
 * Nothing in the product path links, loads or calls this code.  Only tests/,
 * __graft_entry__.smoke() (as the checker) and bench.py's cpu_baseline /
 * --impl reference legs use it.
 *
 * The oracle restates, in plain C, the reference's workspace flash path
 * flash_attention_qk_pv_tile_ws (src/onednn_flash/attention.cpp:486-695) and
 * its materialising standard_attention (src/onednn_flash/attention.cpp:88-137),
 * looped over (batch, head) the way flash_attention_batched_qk_pv_tile does
 * (src/onednn_flash/batched_attention.cpp:9-49).  Features the reference lacks
 * are added at the places the reference would put them:
 *   - LSE output: m + ln(l) from the final running max / running sum
 *     (attention.cpp:672-673);
 *   - soft-cap: s <- cap * tanh(s / cap), right after the scale + bias step
 *     (attention.cpp:619);
 *   - GQA: kv_head = q_head / (heads_q / heads_kv);
 *   - ALiBi as a structured additive bias slope[h] * (kj - qi), and a strided
 *     additive bias tensor, which the reference can only express through its
 *     ScoreBiasFn (attention.hpp:31).
 * The same struct is used by the shim over the real reference sources
 * (oracle/ref_shim.cpp), so the two can be compared call for call.
 */
#ifndef ODF_ORACLE_H
#define ODF_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct odf_oracle_params {
    const float* q;         /* [B, Hq, M, D]  row-major                        */
    const float* k;         /* [B, Hkv, N, D]                                  */
    const float* v;         /* [B, Hkv, N, Dv]                                 */
    float* o;               /* [B, Hq, M, Dv]; fully masked rows get 0         */
    float* lse;             /* [B, Hq, M] natural-log LSE, -inf if masked; or NULL */
    int64_t batch, heads_q, heads_kv;
    int64_t m, n, d, dv;
    float scale;
    int causal;             /* top-left aligned: key kj > query qi is masked   */
    int64_t q_block, k_block;   /* the reference's tile sizes (AttentionOptions) */
    /* BlockMask (attention.hpp:20-29): row-major [mask_qblocks, mask_kblocks],
       non-zero = allowed, out-of-range block = disallowed.  NULL = no mask. */
    const uint8_t* mask;
    int64_t mask_qbs, mask_kbs, mask_qblocks, mask_kblocks;
    const float* alibi_slopes;  /* [Hq] or NULL: bias = slope[h] * (kj - qi) */
    float softcap;              /* 0 = off */
    int nthreads;               /* threads over (batch, head); <=0 = 1 */
    /* Additive bias tensor (BiasKind::SameShapeTile, qk_score_tile.cpp:28-47), element
       (b, h, qi, kj) at bias[b*s0 + h*s1 + qi*s2 + kj*s3] with bias_strides = {s0..s3};
       zero strides broadcast.  NULL = none.  Added after the scale, like score_bias. */
    const float* bias;
    int64_t bias_strides[4];
} odf_oracle_params;

/* Status codes shared by the oracle and the reference shim. */
#define ODF_ORACLE_OK 0
#define ODF_ORACLE_EINVAL 1
#define ODF_ORACLE_EUNSUPPORTED 2
#define ODF_ORACLE_EREF 3

/* Flash tiled forward (restates attention.cpp:486-695). */
int odf_oracle_flash_fwd(const odf_oracle_params* p);

/* Materialising forward (restates attention.cpp:88-137); LSE is also produced. */
int odf_oracle_standard_fwd(const odf_oracle_params* p);

/*
 * Tile map for tile sizes (bq, bk) over an M x N score matrix:
 * out[qt * nkt + kt] = 0 skipped, 1 processed with every element allowed,
 * 2 processed with at least one masked element.  A tile is skipped iff
 * causal and kt*bk >= min(M, (qt+1)*bq) (the reference's causal break,
 * attention.cpp:537-539), or every mask block it covers is disallowed.
 */
int odf_oracle_tile_map(int64_t m, int64_t n, int64_t bq, int64_t bk, int causal,
                        const uint8_t* mask, int64_t mask_qbs, int64_t mask_kbs,
                        int64_t mask_qblocks, int64_t mask_kblocks, uint8_t* out);

/* Round-to-nearest-even fp32 -> bf16 -> fp32, for building bf16-exact inputs. */
void odf_oracle_round_bf16(const float* in, float* out, int64_t count);

#ifdef __cplusplus
}
#endif

#endif /* ODF_ORACLE_H */
