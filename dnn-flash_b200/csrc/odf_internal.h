// odf_internal.h -- launch-side structures shared by the kernel file and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "odf_sm100.h"

namespace odf {

constexpr int kTileQ = ODF_TILE_Q;
constexpr int kTileK = ODF_TILE_K;

// How the kernel enumerates the KV tiles of a query tile.
enum TileMode : int32_t {
    kModeDense = 0,   // every KV tile
    kModeCausal = 1,  // KV tiles with kt*128 < min(M, (qt+1)*128)
    kModeList = 2,    // compacted per-query-tile list built from the block mask
};

// A KV-list entry of a query-tile pair: kv tile index in the low 16 bits, then
// which of the pair's two query tiles need the KV tile and which of them must test
// the BlockMask bitmap per element (a covered mask block is disallowed).
constexpr uint32_t kNeed0 = 1u << 16;
constexpr uint32_t kNeed1 = 1u << 17;
constexpr uint32_t kBitmap0 = 1u << 18;
constexpr uint32_t kBitmap1 = 1u << 19;

// Division of 32-bit values by a divisor fixed for a launch, as one multiply-high, a subtract, an
// add and two shifts (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, the round-up method of their section 4): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, every 32-bit x gives x / d = (t + ((x - t) >> 1)) >> (l - 1),
// t = mulhi(x, m).  d = 1 takes m = 0 and shifts of 0.  The kernels decode a work item with these
// instead of 64-bit divisions, which cost several hundred cycles each on the roles' critical paths.
struct FastDiv {
    uint32_t d, m, sh1, sh2;
};

inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0u, 0u, 0u};
    if (d <= 1) return f;
    uint32_t l = 0;
    while ((uint64_t{1} << l) < d) ++l;
    f.m = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1);
    f.sh1 = 1;
    f.sh2 = l - 1;
    return f;
}

__host__ __device__ __forceinline__ uint32_t fast_div(uint32_t x, const FastDiv& f) {
#ifdef __CUDA_ARCH__
    const uint32_t t = __umulhi(x, f.m);
#else
    const uint32_t t = static_cast<uint32_t>((static_cast<uint64_t>(x) * f.m) >> 32);
#endif
    return (t + ((x - t) >> f.sh1)) >> f.sh2;
}

// Everything the forward kernel needs besides the three tensor maps.
struct FwdArgs {
    void* o;
    float* lse;
    int64_t o_stride_b, o_stride_h, o_stride_t;  // elements
    int32_t o_bf16;
    int32_t batch, heads_q, heads_kv, m, n;
    int32_t n_qt, n_kt, n_pairs;
    // Few-item problems (every query tile fits on its own SM): an item is one query tile (its Q1
    // half left empty) instead of a pair, so twice as many SMs share the work.
    int32_t single_tile;
    int32_t mode;
    int32_t causal;
    // Causal mode only: an item walks its KV tiles from the diagonal down to tile 0 (set for
    // ALiBi at d = 128, whose nearest keys carry the row's largest scores).
    int32_t kv_reverse;
    // With kv_reverse, optional [batch * heads_q, n_pairs]: the pair's KV tiles below this index
    // are far for both of its query tiles by the norm bound (far_lo_kernel) and are not visited.
    const int32_t* kv_lo;
    float scale;        // natural-units softmax scale
    float scale_log2;   // scale * log2(e)
    float softcap;      // 0 = off
    float inv_softcap;
    const uint8_t* mask;
    int32_t mask_qbs, mask_kbs, mask_qblocks, mask_kblocks;
    const uint32_t* tile_list;  // [n_pairs, n_kt]
    const int32_t* tile_count;  // [n_pairs]
    uint8_t* visits;
    int* status;
    int32_t alibi_generated;    // slopes = 2^(-8 (h+1) / heads_q)
    float alibi_slopes[ODF_MAX_EXPLICIT_SLOPES];
    const float* bias;          // same-shape additive bias, element strides below (0 = broadcast)
    int64_t bias_s0, bias_s1, bias_s2, bias_s3;
    // Work items: blocks of units_per_block (batch, kv-head) units, the query-tile pairs of a
    // block longest first.  sched != NULL: a zeroed 64-bit counter in the caller's workspace that
    // hands items to CTAs as they become free; NULL: a fixed snake order (units_per_block is then
    // every unit).
    unsigned long long* sched;
    int32_t units_per_block;
    // Item decode in 32-bit arithmetic (set when every item index fits in 31 bits): dividers by
    // batch * heads_q, heads_q, heads_q / heads_kv, heads_kv, the items of a full block of units,
    // and the items per query-tile pair of a full and of the last (partial) block.
    int32_t fast_decode;
    FastDiv fd_bh, fd_hq, fd_gq, fd_hkv, fd_block, fd_row, fd_row_last;
    // KV splits (n_splits > 1; dense and causal modes without the ALiBi far-tile walk): every
    // query-tile pair becomes n_splits items over consecutive kv_per_split KV tiles each, whose
    // normalised O (fp32) and LSE go to per-split planes o_split / lse_split elements apart (o and
    // lse then point at workspace partials), merged afterwards by split_combine_kernel.
    int32_t n_splits, kv_per_split;
    FastDiv fd_split;
    int64_t o_split, lse_split;
    // Limit of every bounded in-kernel wait (ns); the host fills in the default of 2 s unless a
    // caller lowered it through odf_debug_set_wait.
    uint64_t wait_limit_ns;
    // Failure injection for tests (-1 = off): the producer warp of CTA 0 leaves out its ring load
    // number stall_load (neither the bytes nor the copy), so the MMA warp's wait for that slot runs
    // out and the abort path runs: status word set, roles leave, copies and MMAs drained.
    int32_t stall_load;
};

constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;

// The first kSchedBytes of a workspace hold the item counter; block-mask tile lists follow.
constexpr size_t kSchedBytes = 256;

// Validated, resolved launch request (device pointers only).
struct FwdLaunch {
    const void* q;
    const void* k;
    const void* v;
    int64_t q_strides[3], k_strides[3], v_strides[3];  // elements {b, h, t}
    int32_t head_dim;
    int32_t has_alibi;
    int32_t has_softcap;
    int32_t has_bias;
    FwdArgs args;
    void* workspace;
    size_t workspace_bytes;
    int32_t allow_split;    // KV splits may use the workspace (0: the layout of a workspace without them)
    int32_t forced_splits;  // > 0: this many KV splits (1: none) instead of the launch's own plan
};

// Launch the tile-list builder (block-mask mode) and the forward kernel on `stream`.
// Returns ODF_OK or an ODF_ERR_* code; `err` receives a message on failure.
int launch_flash_fwd(FwdLaunch& L, cudaStream_t stream, const char** err);

// Per-query-tile classification kernel for odf_tile_map_sm100.
int launch_tile_map(int32_t m, int32_t n, int32_t causal, const uint8_t* mask, int32_t mqbs, int32_t mkbs,
                    int32_t mqblocks, int32_t mkblocks, uint8_t* cls_out, cudaStream_t stream);

// fp32 -> bf16 conversion kernel.
int launch_convert_f32_bf16(const float* in, uint16_t* out, int64_t count, cudaStream_t stream);

// Per-device setup (capability check, kernel attributes, status word), redone when the device's
// current CUDA context changes (after cudaDeviceReset, or another context made current).
int ensure_device_ready(int device, const char** err);

// Checked build: the failed in-kernel invariant bits since the last call (read and cleared;
// synchronises the device).  ODF_ERR_UNSUPPORTED in the shipped library.
int read_check_bits(uint32_t* out);

// The calling thread's current CUDA context (driver handle, NULL if none), fetched through the
// runtime's driver entry point so the library needs no -lcuda.
void* current_context();

// Device address of the status word bounded waits write to (current device).
int* device_status_ptr(int device);

size_t workspace_bytes_for(int64_t seqlen_q, int64_t seqlen_k, bool has_mask);

// KV splits: when a launch's work items (query-tile pairs, or single query tiles) would leave more
// than half of `sm_count` SMs idle, each item's key range is cut into n_splits consecutive parts of
// kv_per_split (at least 4) KV tiles, one item each, and the parts are merged afterwards
// (n_splits = 1: none).
// Not for block-mask lists or the causal ALiBi walk at d = 128 (`eligible` false).
struct SplitPlan {
    int32_t n_splits, kv_per_split;
};
SplitPlan plan_kv_splits(int64_t batch, int64_t heads_q, int64_t seqlen_q, int64_t seqlen_k, bool eligible,
                         int64_t sm_count);
// Optional workspace bytes after kSchedBytes for the fp32 partial O and LSE of that plan (0 without
// splits), sized for a GPU of kSplitSizingSms SMs.
constexpr int64_t kSplitSizingSms = 148;
size_t kv_split_bytes(int64_t batch, int64_t heads_q, int64_t seqlen_q, int64_t seqlen_k, int64_t head_dim,
                      bool eligible);

// Optional workspace bytes after workspace_bytes_for(..., false) that causal ALiBi at d = 128
// uses for its far-tile bound (tile norms and the per-pair first visited KV tile).
size_t far_bound_bytes(int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seqlen_q, int64_t seqlen_k);

}  // namespace odf
