/*
 * odf_sm100.h -- C ABI of the B200 (sm_100a) tiled attention forward.
 *
 * This is the thin boundary between host code (the C++ API in
 * include/onednn_flash/, the TensorFlow op, ctypes/cgo/JNI users) and the
 * CUDA kernels.  Plain pointers, sizes and status codes only; nothing here
 * throws.  Every entry point replaces one piece of the reference's
 * hot path, cited beside it.
 *
 * Semantics follow the reference's workspace flash path
 * flash_attention_qk_pv_tile_ws (src/onednn_flash/attention.cpp:486-695):
 *   s = q.k * scale + bias(qi, kj)          (attention.cpp:619)
 *   s = softcap * tanh(s / softcap)         (added; no reference counterpart)
 *   masked (causal kj > qi, top-left aligned, attention.cpp:54-62; BlockMask,
 *   attention.cpp:70-86) -> -inf, then the online softmax and P.V.
 * Differences from the reference, by design:
 *   - Q/K/V are bf16 on the device (the reference is fp32 only); accumulation
 *     and softmax are fp32.
 *   - Fully masked rows are written as 0 with LSE = -inf (the reference leaves
 *     such rows unwritten, attention.cpp:680-682).
 *   - The per-row log-sum-exp (natural log) is an optional extra output.
 *   - GQA: heads_q may be a multiple of heads_kv (kv_head = q_head / group).
 */
#ifndef ODF_SM100_H
#define ODF_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (0 = success). */
#define ODF_OK 0
#define ODF_ERR_INVALID_ARG 1      /* null pointer, zero/negative size, bad stride, ... */
#define ODF_ERR_UNSUPPORTED 2      /* shape/dtype/score_mod the sm_100a kernel does not implement */
#define ODF_ERR_CUDA 3             /* a CUDA runtime/driver call failed */
#define ODF_ERR_DEVICE_TIMEOUT 4   /* a bounded in-kernel wait gave up (see odf_device_status) */
#define ODF_ERR_NO_DEVICE 5        /* no sm_100 device current */
#define ODF_ERR_DEVICE_CHECK 6     /* checked build only: an in-kernel invariant failed (odf_debug_check_bits) */

/* Element types; values equal onednn_flash::DataType (score_mod_plan.hpp:7-11). */
#define ODF_DTYPE_F32 0
#define ODF_DTYPE_BF16 1

/* Bias kinds; values equal onednn_flash::BiasKind (score_mod_plan.hpp:21-28). */
#define ODF_BIAS_NONE 0
#define ODF_BIAS_SAME_SHAPE 1      /* BiasKind::SameShapeTile: fp32 tensor, see odf_fwd_params::bias */
#define ODF_BIAS_ALIBI 4           /* BiasKind::AlibiGenerated: bias = slope[h] * (kj - qi) */

#define ODF_MAX_EXPLICIT_SLOPES 256

typedef struct odf_fwd_params {
    /* Tensors.  Device pointers for odf_flash_fwd_sm100, host pointers for
       odf_flash_fwd_host.  Layout [B, H, T, D] with the element strides below. */
    const void* q;              /* [B, heads_q,  seqlen_q, head_dim]  */
    const void* k;              /* [B, heads_kv, seqlen_k, head_dim]  */
    const void* v;              /* [B, heads_kv, seqlen_k, value_dim] */
    void* o;                    /* [B, heads_q,  seqlen_q, value_dim] */
    float* lse;                 /* [B, heads_q, seqlen_q] contiguous, natural log; NULL = not wanted */
    int32_t qkv_dtype;          /* ODF_DTYPE_BF16 (device); host entry also takes ODF_DTYPE_F32 */
    int32_t o_dtype;            /* ODF_DTYPE_F32 or ODF_DTYPE_BF16 */
    int64_t batch, heads_q, heads_kv, seqlen_q, seqlen_k, head_dim, value_dim;
    /* Element strides {batch, head, token}; all zero = contiguous.  The
       innermost (feature) stride is always 1. */
    int64_t q_strides[3], k_strides[3], v_strides[3], o_strides[3];
    float scale;                /* softmax scale (AttentionOptions::scale) */
    int32_t causal;             /* AttentionOptions::causal */
    /* BlockMask (attention.hpp:20-29): u8 row-major [mask_qblocks, mask_kblocks]
       on the device, non-zero = allowed; NULL = no block mask.  Needs a workspace. */
    const uint8_t* block_mask;
    int64_t mask_qbs, mask_kbs, mask_qblocks, mask_kblocks;
    int32_t bias_kind;          /* ODF_BIAS_NONE, ODF_BIAS_SAME_SHAPE or ODF_BIAS_ALIBI */
    /* ALiBi slopes, HOST array [heads_q] (copied into the launch); NULL with
       ODF_BIAS_ALIBI = generated slopes 2^(-8 (h+1) / heads_q). */
    const float* alibi_slopes;
    float softcap;              /* > 0: s = softcap * tanh(s / softcap); 0 = off */
    void* workspace;            /* device scratch of odf_fwd_workspace_size() bytes (16-byte aligned): its first
                                   256 bytes let the kernel hand work to SMs greedily, in L2-sized blocks
                                   of heads (faster for long sequences); NULL = a fixed order, allowed
                                   without a block mask */
    size_t workspace_bytes;
    /* Optional diagnostics (device, may be NULL): u8 [B*heads_q, q_tiles, kv_tiles],
       set to 1 for every 128x128 tile the kernel processes (never cleared by it). */
    uint8_t* tile_visits;
    /* ODF_BIAS_SAME_SHAPE (BiasKind::SameShapeTile, qk_score_tile.cpp:28-47 and 227-232):
       s = q.k * scale + bias[b*s0 + h*s1 + qi*s2 + kj*s3] (then the soft-cap), fp32, with
       the element strides bias_strides = {s0, s1, s2, s3} >= 0 over {batch, q-head, query,
       key}; all zero = contiguous [B, heads_q, M, N]; otherwise zero strides broadcast
       ({0,0,N,1}: one [M,N] matrix for every head; {0,0,0,1}: one bias per key).  Device pointer for odf_flash_fwd_sm100 (key-contiguous rows with
       16-byte aligned starts take the vector path), host pointer for odf_flash_fwd_host.
       Every element with qi < M and kj < N must be addressable; columns beyond N are not read. */
    const float* bias;
    int64_t bias_strides[4];
} odf_fwd_params;

/*
 * Forward pass on device buffers, asynchronous on `stream` (a cudaStream_t;
 * NULL = legacy default stream).  Replaces the (batch x head) loop of
 * flash_attention_batched_qk_pv_tile (src/onednn_flash/batched_attention.cpp:9-49)
 * and the tile loops of flash_attention_qk_pv_tile_ws (attention.cpp:486-695).
 */
int odf_flash_fwd_sm100(const odf_fwd_params* p, void* stream);

/* Device scratch bytes for these params: 256 (the work-item counter, optional) plus,
   with a block mask, the per-query-tile-pair KV lists (required), or, for causal ALiBi at
   head_dim 128, room for the far-tile bound (tile norms and per-pair first KV tiles;
   optional: a smaller workspace runs without the bound), or, for other launches whose work
   items would leave more than half of the GPU's SMs idle (few heads or query tiles over a
   long key range), room for the fp32 partial O and LSE of KV splits (optional: a smaller
   workspace splits less or not at all).  Plays the role of AttentionWorkspace::resize
   (src/onednn_flash/attention_workspace.cpp:5-20). */
size_t odf_fwd_workspace_size(const odf_fwd_params* p);

/* Capacity of the library-owned scratch used by odf_flash_fwd_sm100_noalloc. */
#define ODF_NOALLOC_SCRATCH_BYTES (1u << 20)

/*
 * Same forward pass as odf_flash_fwd_sm100, for callers that cannot allocate
 * device memory: code that runs where cudaMalloc is not allowed or not wanted
 * (a serving loop with a fixed memory budget where an allocation would
 * synchronise the device or fail, a plugin whose host framework owns the
 * allocator, a foreign-language binding with no allocator of its own).  The
 * caller still passes Q/K/V, O and LSE; p->workspace is ignored.
 *
 * Instead of a caller workspace, a fixed array of ODF_NOALLOC_SCRATCH_BYTES in
 * this library's device memory (held by every GPU that loads the library until
 * the process exits) holds the work-item counter (256 bytes), the block-mask
 * tile lists and, when it fits, causal ALiBi's far-tile bound (left out
 * otherwise).  Limit: the lists take about ceil(seqlen_q/256) *
 * ceil(seqlen_k/128) * 4 bytes; larger problems are rejected with
 * ODF_ERR_UNSUPPORTED.  The first call on a device looks up the array's device
 * address (a one-time, non-allocating runtime call, repeated only if the
 * device's CUDA context changes); make that first call before any stream
 * capture.  All calls share the one array, which keeps what the last call left
 * there.  A launch that hands out work through the counter (long plain d = 128
 * problems, causal ALiBi at d = 128) clears it first, a block-mask launch rewrites
 * the lists and a causal ALiBi launch the bound before reading them; the other
 * launches read nothing from the array.  So nothing
 * needs to start at zero, but calls that overlap on the GPU, on different
 * streams, race on the array: serialise them.
 * No counterpart in the reference (its workspace is always caller-owned).
 */
int odf_flash_fwd_sm100_noalloc(const odf_fwd_params* p, void* stream);

/*
 * Forward pass on HOST buffers (pageable or pinned) through the current
 * device; blocks until the result is in `p->o` / `p->lse`.  Q/K/V may be
 * ODF_DTYPE_F32 (converted to bf16 on the device) or ODF_DTYPE_BF16.  Host to
 * device copies, kernels and device to host copies are pipelined over chunks
 * of (batch, kv-head).  This is the call the reference's fp32 host API
 * flash_attention_batched_qk_pv_tile (batched_attention.hpp:26-31) and the
 * TensorFlow op (tensorflow_ops/onednn_flash_attention_op.cc:126-131) make.
 * The block mask and ALiBi slopes are host arrays here.
 */
int odf_flash_fwd_host(const odf_fwd_params* p);

/*
 * Tile map of the 128x128 tiling (the skip set): out[qt * kv_tiles + kt] =
 * 0 skipped, 1 processed with no masked element, 2 processed with an element
 * mask.  Skipped iff causal and kt*128 >= min(seqlen_q, (qt+1)*128) (the
 * reference's causal break, attention.cpp:537-539) or every BlockMask block
 * the tile covers is disallowed.  Device pointers; asynchronous on `stream`.
 */
int odf_tile_map_sm100(int64_t seqlen_q, int64_t seqlen_k, int32_t causal, const uint8_t* block_mask,
                       int64_t mask_qbs, int64_t mask_kbs, int64_t mask_qblocks, int64_t mask_kblocks,
                       uint8_t* out, void* stream);

/* Convert fp32 -> bf16 (round to nearest even) on the device, asynchronous. */
int odf_convert_f32_to_bf16(const float* in, uint16_t* out, int64_t count, void* stream);

/* Reads (and, if `clear`, resets) the device-side status word of the current
   device that bounded in-kernel waits set on timeout.  Synchronises the device. */
int odf_device_status(int32_t* status_out, int32_t clear);

/*
 * Test hook for the bounded in-kernel waits (no counterpart in the reference).
 * Applies to the forward launches this host thread makes from now on:
 *   limit_ns    limit of every in-kernel wait; 0 restores the default (2 s),
 *               otherwise within [1 ms, 60 s];
 *   stall_load  -1 = off; n >= 0 makes CTA 0 leave out its n-th K/V tile load,
 *               so a wait for it runs out: the kernel then records
 *               ODF_ERR_DEVICE_TIMEOUT in the status word (odf_device_status),
 *               drains its copies and MMAs, frees its tensor memory and returns,
 *               and the context stays usable.  That launch's output is undefined.
 * Failure drills and tests use it; a production caller never needs it.
 */
int odf_debug_set_wait(uint64_t limit_ns, int32_t stall_load);

/*
 * Test hook of the checked build (the same sources compiled with -DODF_CHECKED into
 * libodf_sm100_checked.so; no counterpart in the reference).  Synchronises the device, writes
 * the in-kernel invariant bits that failed since the last call to *bits_out (0 = none) and
 * clears them; a failure also sets ODF_ERR_DEVICE_CHECK in the status word if it was clean.
 * Bits: 0 work-item decode, 1 KV entry, 2 tensor-memory base, 3 ring loads issued vs waited,
 * 4 P.V count vs softmax tiles, 5 causal ALiBi bound.  The shipped library returns
 * ODF_ERR_UNSUPPORTED.
 */
int odf_debug_check_bits(uint32_t* bits_out);

/* Message for the last non-zero status returned on this host thread. */
const char* odf_last_error(void);

/* Library version string. */
const char* odf_version(void);

/* Tile geometry of the kernel (for sizing tile_visits and tile maps). */
#define ODF_TILE_Q 128
#define ODF_TILE_K 128

#ifdef __cplusplus
}
#endif

#endif /* ODF_SM100_H */
