/*
 * odf_oracle.c -- CPU oracle for the tiled attention forward.
 *
 * TEST INFRASTRUCTURE ONLY: the product path never links or calls this file.
 * It is the checker used by tests/, __graft_entry__.smoke() and the CPU
 * baseline legs of bench.py.
 *
 * Every loop below restates the reference's scalar fp32 code in the same
 * operation order, so that with features the reference has (scale, causal,
 * BlockMask, additive bias) the results equal the reference bit for bit when
 * both are built with the same compiler flags (checked by
 * tests/test_oracle_vs_reference.py against oracle/_ref, which is compiled
 * from the reference's own sources).
 */
#include "odf_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* std::max(a, b) for floats is (a < b) ? b : a. */
static inline float ref_max(float a, float b) { return (a < b) ? b : a; }

static inline int is_neg_inf(float x) { return isinf(x) && x < 0.0f; }

/* BlockMask::allows (attention.cpp:70-86): out-of-range block = disallowed. */
static inline int mask_allows(const odf_oracle_params* p, int64_t qi, int64_t kj) {
    const int64_t qb = qi / p->mask_qbs;
    const int64_t kb = kj / p->mask_kbs;
    if (qb >= p->mask_qblocks || kb >= p->mask_kblocks) return 0;
    return p->mask[qb * p->mask_kblocks + kb] != 0;
}

/* masked_out (attention.cpp:54-62): causal is top-left aligned. */
static inline int masked_out(const odf_oracle_params* p, int64_t qi, int64_t kj) {
    if (p->causal && kj > qi) return 1;
    if (p->mask != NULL && !mask_allows(p, qi, kj)) return 1;
    return 0;
}

/* score * scale + score_bias(qi, kj) (attention.cpp:619), then the soft-cap. */
static inline float score_mod(const odf_oracle_params* p, int64_t batch, int64_t head, float score,
                              int64_t qi, int64_t kj) {
    float bias = 0.0f;
    if (p->alibi_slopes != NULL) {
        bias = p->alibi_slopes[head] * (float)(kj - qi);
    }
    if (p->bias != NULL) {
        bias += p->bias[batch * p->bias_strides[0] + head * p->bias_strides[1] + qi * p->bias_strides[2] +
                        kj * p->bias_strides[3]];
    }
    float s = score * p->scale + bias;
    if (p->softcap > 0.0f) {
        s = p->softcap * tanhf(s / p->softcap);
    }
    return s;
}

typedef struct head_ctx {
    const odf_oracle_params* p;
    int64_t b, h;
} head_ctx;

/* Per-thread scratch, the AttentionWorkspace equivalent (attention_workspace.hpp:16-47). */
typedef struct workspace {
    float* score;      /* [q_bs, k_bs] */
    float* ptile;      /* [q_bs, k_bs] */
    float* pv;         /* [q_bs, dv]   */
    float* acc;        /* [q_bs, dv]   */
    float* running_max;
    float* running_sum;
    float* old_scales;
    float* new_maxes;
    float* block_sums;
    uint8_t* row_has_valid;
} workspace;

static int ws_alloc(workspace* ws, int64_t qbs, int64_t kbs, int64_t dv) {
    memset(ws, 0, sizeof(*ws));
    ws->score = (float*)calloc((size_t)(qbs * kbs), sizeof(float));
    ws->ptile = (float*)calloc((size_t)(qbs * kbs), sizeof(float));
    ws->pv = (float*)calloc((size_t)(qbs * dv), sizeof(float));
    ws->acc = (float*)calloc((size_t)(qbs * dv), sizeof(float));
    ws->running_max = (float*)calloc((size_t)qbs, sizeof(float));
    ws->running_sum = (float*)calloc((size_t)qbs, sizeof(float));
    ws->old_scales = (float*)calloc((size_t)qbs, sizeof(float));
    ws->new_maxes = (float*)calloc((size_t)qbs, sizeof(float));
    ws->block_sums = (float*)calloc((size_t)qbs, sizeof(float));
    ws->row_has_valid = (uint8_t*)calloc((size_t)qbs, 1);
    return ws->score && ws->ptile && ws->pv && ws->acc && ws->running_max && ws->running_sum &&
           ws->old_scales && ws->new_maxes && ws->block_sums && ws->row_has_valid;
}

static void ws_free(workspace* ws) {
    free(ws->score); free(ws->ptile); free(ws->pv); free(ws->acc);
    free(ws->running_max); free(ws->running_sum); free(ws->old_scales);
    free(ws->new_maxes); free(ws->block_sums); free(ws->row_has_valid);
}

/* One (batch, q-head): restates flash_attention_qk_pv_tile_ws (attention.cpp:486-695). */
static void flash_head(const odf_oracle_params* p, int64_t b, int64_t h, workspace* ws) {
    const int64_t M = p->m, N = p->n, D = p->d, DV = p->dv;
    const int64_t group = p->heads_q / p->heads_kv;
    const int64_t hk = h / group;
    const float* q = p->q + ((b * p->heads_q + h) * M) * D;
    const float* k = p->k + ((b * p->heads_kv + hk) * N) * D;
    const float* v = p->v + ((b * p->heads_kv + hk) * N) * DV;
    float* out = p->o + ((b * p->heads_q + h) * M) * DV;
    float* lse = p->lse ? p->lse + (b * p->heads_q + h) * M : NULL;
    const float neg_inf = -INFINITY;
    const int64_t q_bs = p->q_block, k_bs = p->k_block;

    for (int64_t i = 0; i < M * DV; ++i) out[i] = 0.0f;
    if (lse) for (int64_t i = 0; i < M; ++i) lse[i] = neg_inf;

    for (int64_t q_begin = 0; q_begin < M; q_begin += q_bs) {                 /* :513 */
        const int64_t q_end = (q_begin + q_bs < M) ? q_begin + q_bs : M;
        const int64_t q_rows = q_end - q_begin;
        const float* q_tile = q + q_begin * D;                                 /* :520 */
        for (int64_t i = 0; i < q_rows; ++i) {                                 /* :523-530 */
            ws->running_max[i] = neg_inf;
            ws->running_sum[i] = 0.0f;
            ws->row_has_valid[i] = 0;
        }
        for (int64_t i = 0; i < q_rows * DV; ++i) ws->acc[i] = 0.0f;

        for (int64_t k_begin = 0; k_begin < N; k_begin += k_bs) {             /* :532 */
            const int64_t k_end = (k_begin + k_bs < N) ? k_begin + k_bs : N;
            const int64_t k_cols = k_end - k_begin;
            if (p->causal && k_begin >= q_end) break;                          /* :537-539 */

            /* S = Q_tile * K_view^T, strided scalar GEMM (tile_kernel.cpp:76-85). */
            const float* kt = k + k_begin * D;
            for (int64_t i = 0; i < q_rows; ++i) {
                for (int64_t j = 0; j < k_cols; ++j) {
                    float sum = 0.0f;
                    for (int64_t kk = 0; kk < D; ++kk) sum += q_tile[i * D + kk] * kt[j * D + kk];
                    ws->score[i * k_cols + j] = sum;
                }
            }
            for (int64_t i = 0; i < q_rows; ++i) {                             /* :602-606 */
                ws->new_maxes[i] = ws->running_max[i];
                ws->block_sums[i] = 0.0f;
                ws->row_has_valid[i] = 0;
            }
            for (int64_t lk = 0; lk < q_rows; ++lk) {                          /* :608-645 */
                const int64_t qi = q_begin + lk;
                float block_max = neg_inf;
                for (int64_t kk = 0; kk < k_cols; ++kk) {
                    const int64_t kj = k_begin + kk;
                    float* score = &ws->score[lk * k_cols + kk];
                    if (masked_out(p, qi, kj)) { *score = neg_inf; continue; }
                    *score = score_mod(p, b, h, *score, qi, kj);
                    block_max = ref_max(block_max, *score);
                    ws->row_has_valid[lk] = 1;
                }
                if (!ws->row_has_valid[lk]) continue;
                const float new_max = ref_max(ws->running_max[lk], block_max);
                ws->new_maxes[lk] = new_max;
                ws->old_scales[lk] = is_neg_inf(ws->running_max[lk])
                                         ? 0.0f : expf(ws->running_max[lk] - new_max);
                for (int64_t kk = 0; kk < k_cols; ++kk) {
                    const float score = ws->score[lk * k_cols + kk];
                    if (is_neg_inf(score)) { ws->ptile[lk * k_cols + kk] = 0.0f; continue; }
                    const float weight = expf(score - new_max);
                    ws->ptile[lk * k_cols + kk] = weight;
                    ws->block_sums[lk] += weight;
                }
            }
            /* PV = P_tile * V_view, contiguous scalar GEMM (tile_kernel.cpp:57-65). */
            const float* vt = v + k_begin * DV;
            for (int64_t i = 0; i < q_rows; ++i) {
                for (int64_t j = 0; j < DV; ++j) {
                    float sum = 0.0f;
                    for (int64_t kk = 0; kk < k_cols; ++kk) sum += ws->ptile[i * k_cols + kk] * vt[kk * DV + j];
                    ws->pv[i * DV + j] = sum;
                }
            }
            for (int64_t lk = 0; lk < q_rows; ++lk) {                          /* :662-674 */
                if (!ws->row_has_valid[lk]) continue;
                const float old_scale = ws->old_scales[lk];
                for (int64_t vd = 0; vd < DV; ++vd) {
                    ws->acc[lk * DV + vd] = ws->acc[lk * DV + vd] * old_scale + ws->pv[lk * DV + vd];
                }
                ws->running_sum[lk] = ws->running_sum[lk] * old_scale + ws->block_sums[lk];
                ws->running_max[lk] = ws->new_maxes[lk];
            }
        }
        for (int64_t lk = 0; lk < q_rows; ++lk) {                              /* :678-687 */
            const int64_t qi = q_begin + lk;
            if (ws->running_sum[lk] <= 0.0f) continue;
            const float inv = 1.0f / ws->running_sum[lk];
            for (int64_t vd = 0; vd < DV; ++vd) out[qi * DV + vd] = ws->acc[lk * DV + vd] * inv;
            if (lse) lse[qi] = ws->running_max[lk] + logf(ws->running_sum[lk]);
        }
    }
}

/* One (batch, q-head): restates standard_attention (attention.cpp:88-137). */
static void standard_head(const odf_oracle_params* p, int64_t b, int64_t h, float* scores) {
    const int64_t M = p->m, N = p->n, D = p->d, DV = p->dv;
    const int64_t group = p->heads_q / p->heads_kv;
    const int64_t hk = h / group;
    const float* q = p->q + ((b * p->heads_q + h) * M) * D;
    const float* k = p->k + ((b * p->heads_kv + hk) * N) * D;
    const float* v = p->v + ((b * p->heads_kv + hk) * N) * DV;
    float* out = p->o + ((b * p->heads_q + h) * M) * DV;
    float* lse = p->lse ? p->lse + (b * p->heads_q + h) * M : NULL;

    for (int64_t i = 0; i < M * DV; ++i) out[i] = 0.0f;
    for (int64_t qi = 0; qi < M; ++qi) {
        if (lse) lse[qi] = -INFINITY;
        float row_max = -INFINITY;
        int has_valid = 0;
        for (int64_t kj = 0; kj < N; ++kj) {
            if (masked_out(p, qi, kj)) { scores[kj] = -INFINITY; continue; }
            float dot = 0.0f;
            for (int64_t d = 0; d < D; ++d) dot += q[qi * D + d] * k[kj * D + d];
            scores[kj] = score_mod(p, b, h, dot, qi, kj);
            row_max = ref_max(row_max, scores[kj]);
            has_valid = 1;
        }
        if (!has_valid) continue;
        float denom = 0.0f;
        for (int64_t kj = 0; kj < N; ++kj) {
            if (is_neg_inf(scores[kj])) continue;
            scores[kj] = expf(scores[kj] - row_max);
            denom += scores[kj];
        }
        for (int64_t vd = 0; vd < DV; ++vd) {
            float acc = 0.0f;
            for (int64_t kj = 0; kj < N; ++kj) {
                if (is_neg_inf(scores[kj])) continue;
                acc += scores[kj] * v[kj * DV + vd];
            }
            out[qi * DV + vd] = acc / denom;
        }
        if (lse) lse[qi] = row_max + logf(denom);
    }
}

typedef struct pool_arg {
    const odf_oracle_params* p;
    int standard;
    int64_t first, stride;
    int ok;
} pool_arg;

static void* pool_main(void* raw) {
    pool_arg* a = (pool_arg*)raw;
    const odf_oracle_params* p = a->p;
    const int64_t units = p->batch * p->heads_q;
    workspace ws;
    float* scores = NULL;
    a->ok = 1;
    if (a->standard) {
        scores = (float*)malloc((size_t)p->n * sizeof(float));
        if (!scores) { a->ok = 0; return NULL; }
    } else if (!ws_alloc(&ws, p->q_block, p->k_block, p->dv)) {
        ws_free(&ws);
        a->ok = 0;
        return NULL;
    }
    for (int64_t u = a->first; u < units; u += a->stride) {
        const int64_t b = u / p->heads_q, h = u % p->heads_q;
        if (a->standard) standard_head(p, b, h, scores);
        else flash_head(p, b, h, &ws);
    }
    if (a->standard) free(scores);
    else ws_free(&ws);
    return NULL;
}

static int validate(const odf_oracle_params* p, int flash) {
    if (!p || !p->q || !p->k || !p->v || !p->o) return ODF_ORACLE_EINVAL;
    if (p->batch <= 0 || p->heads_q <= 0 || p->heads_kv <= 0 || p->m <= 0 || p->n <= 0 ||
        p->d <= 0 || p->dv <= 0)
        return ODF_ORACLE_EINVAL;
    if (p->heads_q % p->heads_kv != 0) return ODF_ORACLE_EINVAL;
    if (flash && (p->q_block <= 0 || p->k_block <= 0)) return ODF_ORACLE_EINVAL;
    if (p->mask && (p->mask_qbs <= 0 || p->mask_kbs <= 0 || p->mask_qblocks <= 0 ||
                    p->mask_kblocks <= 0))
        return ODF_ORACLE_EINVAL;
    if (p->softcap < 0.0f) return ODF_ORACLE_EINVAL;
    return ODF_ORACLE_OK;
}

static int run_pool(const odf_oracle_params* p, int standard) {
    const int64_t units = p->batch * p->heads_q;
    int nt = p->nthreads > 0 ? p->nthreads : 1;
    if (nt > units) nt = (int)units;
    if (nt > 256) nt = 256;
    pthread_t th[256];
    pool_arg args[256];
    for (int t = 0; t < nt; ++t) {
        args[t].p = p; args[t].standard = standard; args[t].first = t; args[t].stride = nt; args[t].ok = 0;
    }
    if (nt == 1) {
        pool_main(&args[0]);
        return args[0].ok ? ODF_ORACLE_OK : ODF_ORACLE_EINVAL;
    }
    int started = 0;
    for (int t = 0; t < nt; ++t) {
        if (pthread_create(&th[t], NULL, pool_main, &args[t]) != 0) break;
        ++started;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    if (started != nt) {
        /* Run whatever did not start on this thread. */
        for (int t = started; t < nt; ++t) pool_main(&args[t]);
    }
    for (int t = 0; t < nt; ++t) if (!args[t].ok) return ODF_ORACLE_EINVAL;
    return ODF_ORACLE_OK;
}

int odf_oracle_flash_fwd(const odf_oracle_params* p) {
    const int rc = validate(p, 1);
    if (rc) return rc;
    return run_pool(p, 0);
}

int odf_oracle_standard_fwd(const odf_oracle_params* p) {
    const int rc = validate(p, 0);
    if (rc) return rc;
    return run_pool(p, 1);
}

int odf_oracle_tile_map(int64_t m, int64_t n, int64_t bq, int64_t bk, int causal,
                        const uint8_t* mask, int64_t mqbs, int64_t mkbs,
                        int64_t mqblocks, int64_t mkblocks, uint8_t* out) {
    if (m <= 0 || n <= 0 || bq <= 0 || bk <= 0 || !out) return ODF_ORACLE_EINVAL;
    if (mask && (mqbs <= 0 || mkbs <= 0 || mqblocks <= 0 || mkblocks <= 0)) return ODF_ORACLE_EINVAL;
    const int64_t nqt = (m + bq - 1) / bq, nkt = (n + bk - 1) / bk;
    for (int64_t qt = 0; qt < nqt; ++qt) {
        const int64_t q0 = qt * bq, q1 = (q0 + bq < m) ? q0 + bq : m;
        for (int64_t kt = 0; kt < nkt; ++kt) {
            const int64_t k0 = kt * bk, k1 = (k0 + bk < n) ? k0 + bk : n;
            uint8_t cls = 1;
            if (causal && k0 >= q1) {
                cls = 0;
            } else {
                if (causal && k1 - 1 > q0) cls = 2;
                if (mask) {
                    int any_allowed = 0, any_denied = 0;
                    for (int64_t qb = q0 / mqbs; qb <= (q1 - 1) / mqbs; ++qb) {
                        for (int64_t kb = k0 / mkbs; kb <= (k1 - 1) / mkbs; ++kb) {
                            const int ok = qb < mqblocks && kb < mkblocks && mask[qb * mkblocks + kb] != 0;
                            if (ok) any_allowed = 1; else any_denied = 1;
                        }
                    }
                    if (!any_allowed) cls = 0;
                    else if (any_denied) cls = 2;
                }
            }
            out[qt * nkt + kt] = cls;
        }
    }
    return ODF_ORACLE_OK;
}

void odf_oracle_round_bf16(const float* in, float* out, int64_t count) {
    for (int64_t i = 0; i < count; ++i) {
        uint32_t u;
        memcpy(&u, &in[i], 4);
        if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
            u |= 0x00400000u;  /* quiet NaN */
        } else {
            u += 0x7fffu + ((u >> 16) & 1u);
        }
        u &= 0xffff0000u;
        memcpy(&out[i], &u, 4);
    }
}
