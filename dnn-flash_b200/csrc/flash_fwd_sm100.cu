// flash_fwd_sm100.cu -- tiled attention forward for B200 (sm_100a).
//
// Persistent kernel: one CTA per SM works through a sequence of work items (given out by a
// counter in the workspace, or a fixed snake order without one).
// An item is a PAIR of 128-row query tiles (Q0, Q1) of one (batch, q-head); the CTA
// walks the KV tiles the tiling does not skip, loading each K/V tile once for both
// query tiles.  The K/V ring, the barriers' phases and the TMEM allocation carry over
// from item to item, so the next item's Q load and first S MMAs overlap the current
// item's last P.V and its epilogue.  It replaces the query-block and key-block loops of the
// reference's flash_attention_qk_pv_tile_ws (src/onednn_flash/attention.cpp:513-688):
// the scalar tile GEMMs (tile_kernel.cpp:57-85) become tcgen05 MMAs fed by TMA and
// accumulating in tensor memory, and the per-row online softmax
// (attention.cpp:602-674) runs in registers, one thread per query row.
//
// Warp roles (384 threads, three warpgroups):
//   warps 0-3  softmax of Q0 (+ its epilogue); thread t owns row t = TMEM lane t
//   warps 4-7  softmax of Q1 (+ its epilogue)
//   warp  8    TMA producer (Q0/Q1 per item, K_j, V_j through a ring of slots);
//              it also owns the TMEM allocation
//   warp  9    MMA issuer (one thread)
//   warps 10-11 idle
// setmaxnreg moves registers from warpgroup 2 (168 -> 104) to the softmax warpgroups
// (168 -> 200), which hold a whole 128-column S row per thread.  The roles never meet in
// common code after the split (each ends with its own CTA barrier), so ptxas allocates
// each under its own budget.
// Tensor memory (512 columns):
//   S0 [0,128)  S1 [128,256)  O0 [256,256+D)  O1 [256+D,256+2D)
//   P_i (bf16, two per column) is the A operand of the P.V MMA read straight from tensor
//   memory.  D = 128: P_i is written over the first 64 columns of S_i.  D = 64: P_i has its
//   own columns [384 + 64 i, 448 + 64 i), so S_i(j+1) is issued once the softmax has read
//   S_i(j) (barrier s_free) and the softmax waits for P.V(j-1) (barrier pv_done) before it
//   overwrites P_i or rescales O_i.
// MMA issue order per KV tile j (in-order execution on the tensor core):
//   D = 128: PV0(j), S0(j+1), PV1(j), S1(j+1);  D = 64: S0(j+1), S1(j+1), PV0(j), PV1(j)
// and at an item's last tile PV0, PV1 (committed to o_done[0/1]) then S0, S1 of the next item
// so while the softmax of one query tile runs, the tensor core works on the other
// tile's P.V and S MMAs.  S_i(j+1) overwrites S_i/P_i only after PV_i(j) was issued.
// The softmax raises its running max only when a tile's max exceeds it by more than
// 2^8; the O rescale this needs is done by the softmax thread itself (PV_i(j-1) has
// completed once S_i(j) has, since a tcgen05 commit tracks all earlier MMAs).
// Every wait is bounded (args.wait_limit_ns, 2 s unless a test lowers it); on timeout the
// CTA records ODF_ERR_DEVICE_TIMEOUT in the device status word, all roles leave their loops,
// in-flight copies and MMAs are drained, and the TMEM columns are freed before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <math.h>
#include <mutex>

#include "odf_internal.h"
#include "sm100_ptx.cuh"
#include "softmax_math.cuh"

namespace odf {

namespace {

constexpr int kThreads = 384;  // three warpgroups
constexpr int kWarpProducer = 8;
constexpr int kWarpMma = 9;    // warps 10 and 11 only give their registers away
// Register split: the kernel is compiled for kLaunchRegs per thread (three warps share an
// SMSP); warpgroup 2 drops to RegSplit::kCtrl and the two softmax warpgroups rise to
// RegSplit::kSoftmax, which must not exceed what the block was launched with.  The host checks
// the compiled register count before the first launch.
constexpr int kLaunchRegs = 168;
// The split is per score-mod variant: the bias-tensor variants, with the larger control code,
// need 112 registers there; the others keep 200 for the softmax.
template <int MOD>
struct RegSplit {
    static constexpr int kCtrl = (MOD & 7) >= 4 ? 112 : 104;
    static constexpr int kSoftmax = (MOD & 7) >= 4 ? 192 : 200;
    static_assert(128 * kCtrl + 256 * kSoftmax <= kThreads * kLaunchRegs, "register split exceeds the launch");
    static_assert(kCtrl % 8 == 0 && kSoftmax % 8 == 0 && kSoftmax <= 256, "setmaxnreg operands");
};
constexpr uint32_t kTmemCols = 512;
constexpr int kItemQueue = 4;  // entries of the shared-memory queue of work items
constexpr uint32_t kChunkBytes = 128 * 128;  // 128 rows x 128 bytes (64 bf16)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// The running max is only raised when a tile's max exceeds it by more than this
// (log2 units), so P stays below 2^8 and O is rescaled rarely.
constexpr float kRescaleLog2 = 8.0f;
// ALiBi far tiles: a tile whose every score is below the running max by more than this (log2
// units) contributes P < 2^-48 per element, i.e. less than n * 2^-48 of l (l >= 1) over a row of
// n keys, far below fp32 resolution: its P is written as zeros without the exponentials.
constexpr float kFarLog2 = 48.0f;

// Checked build (compiled with -DODF_CHECKED; test infrastructure, never the shipped library):
// in-kernel invariants whose failure sets a bit in g_check_bits and, if the status word is clean,
// ODF_ERR_DEVICE_CHECK in it.  A failed check only records (it neither traps nor stops the
// kernel); the accesses it describes stay inside their buffers either way (TMA zero-fills rows past
// a tensor's end, and the epilogue writes no row at or past M).
//   bit 0  a work item decodes to a pair, (batch, head), kv-head and entry count inside the problem
//   bit 1  a KV entry names a tile inside K/V, needed by a query tile that has rows
//   bit 2  the tensor-memory allocation starts at lane 0, column 0
//   bit 3  the MMA warp waited for every ring load the producer issued, and for no other
//   bit 4  per query tile, the MMA warp's P.V count equals the tiles the softmax warps finished
//   bit 5  the causal ALiBi bound leaves each pair at least its diagonal tile
#ifdef ODF_CHECKED
__device__ unsigned int g_check_bits;
__device__ __noinline__ void check_failed(int bit, int* status) {
    atomicOr(&g_check_bits, 1u << bit);
    if (status) atomicCAS(status, 0, ODF_ERR_DEVICE_CHECK);
}
#define ODF_CHECK(cond, bit)                                        \
    do {                                                            \
        if (!(cond)) check_failed((bit), args.status);              \
    } while (0)
#define ODF_COUNT(x) (++(x))
#else
#define ODF_CHECK(cond, bit) \
    do {                     \
    } while (0)
#define ODF_COUNT(x) \
    do {             \
    } while (0)
#endif

// Score-mod variants: ALiBi and the same-shape bias are exclusive (one BiasKind per call).
// kModSkipMax marks the plain-score variant for long KV ranges whose unmasked tiles skip the
// row-max pass (the low three bits select the score mods).
enum ModFlags { kModAlibi = 1, kModSoftcap = 2, kModBias = 4, kModSkipMax = 8 };

template <int D>
struct Config {
    static constexpr int kSlots = (D == 64) ? 8 : 4;
    static constexpr int kChunks = D / 64;
    static constexpr uint32_t kTileBytes = 128 * D * 2;
    static constexpr uint32_t kOffSlots = 2 * kTileBytes;
    static constexpr uint32_t kOffBar = kOffSlots + kSlots * kTileBytes;
    static constexpr int kNumBars = 2 + 2 * kSlots + 2 + 2 + 2 + 2 + 2 + 2 * kItemQueue + 1;
    static constexpr uint32_t kOffRows = kOffBar + kNumBars * 8 + 16;  // after the barriers, TMEM slot, abort flag
    static constexpr uint32_t kOffQueue = kOffRows + 8 * 48;             // item queue (int64 x kItemQueue)
    // same-shape bias: 2 KB per softmax warp to transpose coalesced row reads (32 rows x 16 keys)
    static constexpr uint32_t kOffBias = (kOffQueue + 8 * kItemQueue + 127) & ~127u;  // float4 stores
    static_assert(kOffBias % 16 == 0 && kOffRows % 8 == 0 && kOffQueue % 8 == 0, "shared-memory alignment");
    static constexpr uint32_t kSmemBytes = kOffBias + 8 * 32 * 16 * 4 + 1024;  // + alignment slack
    static_assert(kSmemBytes <= 232448, "shared memory per block");
    static constexpr uint32_t kTmemO = 256;
    // D = 64 leaves 128 TMEM columns free: P_i gets its own 64 columns at kTmemP + 64 i, so that
    // S_i(j+1) can be computed as soon as the softmax has loaded S_i(j) (instead of after
    // P.V(j) has read P_i(j) out of S_i's columns).
    static constexpr bool kSepP = (D == 64);
    static constexpr uint32_t kTmemP = 384;
};

struct Bars {
    uint64_t* q_full;
    uint64_t* q_empty;
    uint64_t* slot_full;
    uint64_t* slot_empty;
    uint64_t* s_full;   // [2]
    uint64_t* p_full;   // [2]
    uint64_t* o_done;   // [2]
    uint64_t* s_free;   // [2] separate-P layout: the softmax has read S_i into registers
    uint64_t* pv_done;  // [2] separate-P layout: P_i.V has completed (P_i may be overwritten)
    uint64_t* item_full;   // [kItemQueue] the producer wrote the queue entry
    uint64_t* item_empty;  // [kItemQueue] the MMA thread and the 8 softmax warps read it
    uint64_t* drain;
};

// The current item as one softmax warp sees it, kept in shared memory (one record per
// warp, written by lane 0) and read where needed, so that no registers stay tied up
// across the softmax loop.
struct RowItem {
    int n_entries;  // KV tiles of the pair (reversed walk: up to and including the diagonal)
    int pair;
    int q0;         // first row of this warp's query tile
    int n_iter;     // list mode: n_entries; dense/causal: the KV tiles this query tile needs (0..n_iter-1)
    int bh, b, h;
    float slope;       // ALiBi slope of head h
    int64_t bias_off;  // same-shape bias: element offset of this (batch, head)'s plane
    int kv0;           // first KV tile of the item's split of the key range
    int split;         // which split (0 without KV splits)
};
static_assert(sizeof(RowItem) == 48, "RowItem layout");

// KV tile j of this query-tile pair: kv index in the low 16 bits, kNeed*/kBitmap* flags above.
// With KV splits, entry j of an item is KV tile kv0 + j of its split (dense and causal modes).
__device__ __forceinline__ uint32_t kv_entry(const FwdArgs& a, int pair, int j, bool valid1, int qend0, int qend1,
                                             int kv0) {
    if (a.mode == kModeList) return __ldg(a.tile_list + static_cast<int64_t>(pair) * a.n_kt + j);
    uint32_t e = static_cast<uint32_t>(kv0 + j);
    if (a.mode == kModeCausal) {
        // the pair's tiles 0 .. n_e - 1, in reverse with kv_reverse (diagonal first)
        const int kt = a.kv_reverse ? min(a.n_kt, (qend1 + kTileK - 1) / kTileK) - 1 - j : kv0 + j;
        e = static_cast<uint32_t>(kt);
        if (kt * kTileK < qend0) e |= kNeed0;
        if (valid1 && kt * kTileK < qend1) e |= kNeed1;
    } else {
        e |= kNeed0;
        if (valid1) e |= kNeed1;
    }
    return e;
}

// One work item: a pair of 128-row query tiles (Q0, Q1) of one (batch, q-head).
struct Item {
    int bh, b, h, hk, pair;
    int q00, q01;      // first rows of Q0 and Q1
    int qend0, qend1;  // their row ends (clipped to M)
    int n_entries;     // KV tiles visited by the pair (entries 0 .. n_entries - 1 of kv_entry)
    bool valid1;       // Q1 has rows
    int split, kv0;    // KV split of the item and its first KV tile (0, 0 without splits)
};

// Items come in blocks of units_per_block (batch, kv-head) units: inside a block, item i is
// query-tile pair n_pairs-1-i/(U G) (longest causal rows first) of q-head i mod (U G) of the
// block (G = q-heads per kv-head).  A block's K/V fits in L2 while its CTAs stream through it.
// With one block holding every unit this is plain pair-major order over all heads.  With KV
// splits, the n_splits splits of a pair's key range are consecutive items.
__device__ __forceinline__ Item decode_item(const FwdArgs& a, int64_t k) {
    Item I;
    I.split = 0;
    if (a.n_splits > 1) {
        if (a.fast_decode) {
            const uint32_t q = fast_div(static_cast<uint32_t>(k), a.fd_split);
            I.split = static_cast<int>(static_cast<uint32_t>(k) - q * a.fd_split.d);
            k = q;
        } else {
            I.split = static_cast<int>(k % a.n_splits);
            k /= a.n_splits;
        }
    }
    I.kv0 = I.split * a.kv_per_split;
    const int64_t n_bh = static_cast<int64_t>(a.batch) * a.heads_q;
    const int64_t n_units = static_cast<int64_t>(a.batch) * a.heads_kv;
    if (a.fast_decode) {  // the same decode in 32-bit arithmetic with the launch's dividers
        const uint32_t x = static_cast<uint32_t>(k);
        if (a.units_per_block >= n_units) {
            const uint32_t round = fast_div(x, a.fd_bh);
            I.bh = static_cast<int>(x - round * a.fd_bh.d);
            I.pair = a.n_pairs - 1 - static_cast<int>(round);
            I.b = static_cast<int>(fast_div(static_cast<uint32_t>(I.bh), a.fd_hq));
            I.h = I.bh - I.b * a.heads_q;
            I.hk = static_cast<int>(fast_div(static_cast<uint32_t>(I.h), a.fd_gq));
        } else {
            const uint32_t gq = a.fd_gq.d;
            const uint32_t blk = fast_div(x, a.fd_block);
            const uint32_t u0 = blk * static_cast<uint32_t>(a.units_per_block);
            const uint32_t i = x - blk * a.fd_block.d;
            const bool part = static_cast<int64_t>(u0) + a.units_per_block > n_units;  // the last, partial block
            const FastDiv& fr = part ? a.fd_row_last : a.fd_row;                   // items per pair
            const uint32_t pr = fast_div(i, fr);
            const uint32_t j = i - pr * fr.d;
            const uint32_t jq = fast_div(j, a.fd_gq);
            const uint32_t unit = u0 + jq;
            I.pair = a.n_pairs - 1 - static_cast<int>(pr);
            I.b = static_cast<int>(fast_div(unit, a.fd_hkv));
            I.hk = static_cast<int>(unit - static_cast<uint32_t>(I.b) * static_cast<uint32_t>(a.heads_kv));
            I.h = I.hk * static_cast<int>(gq) + static_cast<int>(j - jq * gq);
            I.bh = I.b * a.heads_q + I.h;
        }
    } else if (a.units_per_block >= n_units) {  // one block: pair-major over all heads
        const int64_t round = k / n_bh;
        I.bh = static_cast<int>(k - round * n_bh);
        I.pair = a.n_pairs - 1 - static_cast<int>(round);
        I.b = I.bh / a.heads_q;
        I.h = I.bh - I.b * a.heads_q;
        I.hk = I.h / (a.heads_q / a.heads_kv);
    } else {
        const int64_t gq = a.heads_q / a.heads_kv;
        const int64_t per_block = static_cast<int64_t>(a.units_per_block) * gq * a.n_pairs;
        const int64_t blk = k / per_block;
        const int64_t u0 = blk * a.units_per_block;
        const int64_t row = min(static_cast<int64_t>(a.units_per_block), n_units - u0) * gq;  // items per pair
        const int64_t i = k - blk * per_block;
        const int64_t pr = i / row;
        const int64_t j = i - pr * row;
        const int64_t unit = u0 + j / gq;
        I.pair = a.n_pairs - 1 - static_cast<int>(pr);
        I.b = static_cast<int>(unit / a.heads_kv);
        I.hk = static_cast<int>(unit - static_cast<int64_t>(I.b) * a.heads_kv);
        I.h = I.hk * static_cast<int>(gq) + static_cast<int>(j - (j / gq) * gq);
        I.bh = I.b * a.heads_q + I.h;
    }
    I.q00 = I.pair * (a.single_tile ? 1 : 2) * kTileQ;
    I.q01 = a.single_tile ? a.m : I.q00 + kTileQ;  // at M: Q1 has no rows, its epilogue writes none
    I.valid1 = I.q01 < a.m;
    I.qend0 = min(a.m, I.q00 + kTileQ);
    I.qend1 = I.valid1 ? min(a.m, I.q01 + kTileQ) : I.qend0;
    if (a.mode == kModeList) {
        I.n_entries = a.tile_count[I.pair];
    } else if (a.mode == kModeCausal) {
        I.n_entries = min(a.n_kt, (I.qend1 + kTileK - 1) / kTileK);
        // reversed walk: the tiles below kv_lo (far by the norm bound) are left out at its end
        if (a.kv_lo != nullptr) I.n_entries -= __ldg(a.kv_lo + static_cast<int64_t>(I.bh) * a.n_pairs + I.pair);
    } else {
        I.n_entries = a.n_kt;
    }
    if (a.n_splits > 1) I.n_entries = max(0, min(a.kv_per_split, I.n_entries - I.kv0));  // this split's part
    return I;
}

__device__ __forceinline__ uint32_t kv_entry(const FwdArgs& a, const Item& I, int j) {
    return kv_entry(a, I.pair, j, I.valid1, I.qend0, I.qend1, I.kv0);
}

// Item assignment.  With a counter (args.sched) the producer warp of a CTA takes the next
// item index whenever it starts a new item, so CTAs that finish early take more (greedy), and
// publishes it through a small queue in shared memory that the MMA and softmax warps read.
// Without one, CTA c takes one item per round of the grid, the c-th of round r when r is even
// and the (G-1-c)-th when r is odd (items sorted by decreasing causal work: long and short
// items even out), and every role computes that sequence itself.
__device__ __forceinline__ int64_t static_item(int64_t n_items, int it) {
    const int64_t g = gridDim.x;
    const int64_t c = (it & 1) ? (g - 1 - blockIdx.x) : blockIdx.x;
    const int64_t k = static_cast<int64_t>(it) * g + c;
    return k < n_items ? k : -1;
}

// P = 0 over a far tile's 128 keys (64 columns of bf16 pairs), ready for the P.V MMA once the
// caller arrives on p_full.
__device__ __forceinline__ void store_zero_p(uint32_t p_addr) {
    ptx::tmem_st64_zero_nowait(p_addr);
    ptx::tmem_st_wait();
    ptx::tc_fence_before();
}

// Bits of the 128 columns [k0, k0+128) that the BlockMask allows for query row qi
// (attention.cpp:70-86; blocks outside the bitmap are disallowed).  Walks the few mask
// blocks the tile spans instead of testing every column.
__device__ __forceinline__ uint4 row_allow_bits(const FwdArgs& a, int qi, int k0) {
    uint4 allow = make_uint4(0u, 0u, 0u, 0u);
    const int qb = qi / a.mask_qbs;
    if (qb >= a.mask_qblocks) return allow;
    const uint8_t* mrow = a.mask + static_cast<int64_t>(qb) * a.mask_kblocks;
#pragma unroll 1
    for (int kb = k0 / a.mask_kbs; kb < a.mask_kblocks; ++kb) {
        const int c0 = max(kb * a.mask_kbs - k0, 0);
        if (c0 >= kTileK) break;
        const int c1 = min((kb + 1) * a.mask_kbs - k0, kTileK);  // exclusive
        if (__ldg(mrow + kb) == 0) continue;
#pragma unroll
        for (int w = 0; w < 4; ++w) {  // the block's columns [c0, c1) within word w
            const int lo = min(max(c0 - 32 * w, 0), 32);
            const int hi = min(max(c1 - 32 * w, 0), 32);
            const uint32_t upto = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
            const uint32_t from = lo >= 32 ? 0u : ~((1u << lo) - 1u);
            const uint32_t bits = upto & from;
            if (w == 0) allow.x |= bits;
            if (w == 1) allow.y |= bits;
            if (w == 2) allow.z |= bits;
            if (w == 3) allow.w |= bits;
        }
    }
    return allow;
}

// Column pairs (index c/2 mod 8) whose exponentials use exp2_poly2, per head dim and score mod:
// where the MUFU unit is the binding limit (d = 64, and the soft-capped variants, which spend a
// second MUFU operation per score on tanh).
#ifndef ODF_POLY_MASK_D64
#define ODF_POLY_MASK_D64 0x80  // one pair in eight: the best of 0, 1/8, 1/4, 3/8, 1/2 measured at d = 64
#endif
#ifndef ODF_POLY_MASK_SOFTCAP
#define ODF_POLY_MASK_SOFTCAP 0x80  // one pair in eight: best of 0, 1/8, 1/4, 3/8, 1/2 on c3 and soft-cap-only 8K
#endif
template <int D, int MOD>
__host__ __device__ constexpr uint32_t poly_exp2_mask() {
    return D == 64 ? ODF_POLY_MASK_D64 : ((MOD & kModSoftcap) ? ODF_POLY_MASK_SOFTCAP : 0u);
}

template <int D, int MOD>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ FwdArgs args) {
    using Cfg = Config<D>;
    constexpr int kSlots = Cfg::kSlots;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = ptx::smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* sQ = smem;                        // [2][tile]
    uint8_t* sSlots = smem + Cfg::kOffSlots;   // [kSlots][tile]
    uint64_t* bar_base = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    Bars bars;
    bars.q_full = bar_base;
    bars.q_empty = bars.q_full + 1;
    bars.slot_full = bars.q_empty + 1;
    bars.slot_empty = bars.slot_full + kSlots;
    bars.s_full = bars.slot_empty + kSlots;
    bars.p_full = bars.s_full + 2;
    bars.o_done = bars.p_full + 2;
    bars.s_free = bars.o_done + 2;
    bars.pv_done = bars.s_free + 2;
    bars.item_full = bars.pv_done + 2;
    bars.item_empty = bars.item_full + kItemQueue;
    bars.drain = bars.item_empty + kItemQueue;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars.drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // [2][4] bytes: softmax warp w of query tile i wrote its last P as zeros (an ALiBi far tile);
    // when all four did, the MMA warp leaves out that tile's P.V
    volatile uint8_t* far_flags = reinterpret_cast<volatile uint8_t*>(tmem_slot + 2);
    constexpr bool kFarSkip = (MOD & kModAlibi) != 0 && !Cfg::kSepP;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t n_items = static_cast<int64_t>(args.batch) * args.heads_q * args.n_pairs * args.n_splits;
    // Greedy item assignment is compiled into the plain d = 128 kernel (the shapes whose K/V
    // outgrows L2 and whose speed depends on it) and the ALiBi d = 128 kernels (whose items'
    // lengths vary by head once far tiles are left out); the other variants keep the fixed order.
    constexpr bool kDyn = D == 128 && ((MOD & 7) == 0 || (MOD & (kModAlibi | kModBias)) == kModAlibi);
    volatile int64_t* item_q = reinterpret_cast<volatile int64_t*>(smem + Cfg::kOffQueue);

    if (threadIdx.x == 0) {
        ptx::mbar_init(bars.q_full, 1);
        ptx::mbar_init(bars.q_empty, 1);
        for (int s = 0; s < kSlots; ++s) {
            ptx::mbar_init(&bars.slot_full[s], 1);
            ptx::mbar_init(&bars.slot_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&bars.s_full[i], 1);
            ptx::mbar_init(&bars.p_full[i], 128);
            ptx::mbar_init(&bars.o_done[i], 1);
            ptx::mbar_init(&bars.s_free[i], 128);
            ptx::mbar_init(&bars.pv_done[i], 1);
        }
        for (int i = 0; i < kItemQueue; ++i) {
            ptx::mbar_init(&bars.item_full[i], 1);
            ptx::mbar_init(&bars.item_empty[i], 9);
        }
        ptx::mbar_init(bars.drain, 1);
        *abort_flag = 0;
        for (int i = 0; i < 8; ++i) far_flags[i] = 0;
        ptx::fence_barrier_init();
        ptx::fence_proxy_async_smem();
    }
    if (warp == kWarpProducer) {
        ptx::tmem_alloc(tmem_slot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
#ifdef ODF_CHECKED
    // ring loads issued / waited for, P.V count of Q0 and Q1, tiles finished by Q0's and Q1's softmax
    __shared__ int chk_counts[6];
    if (threadIdx.x == 0) ODF_CHECK(tmem == 0u, 2);
#endif

    if (warp >= kWarpProducer) {
        // Warpgroup 2 (producer, MMA issuer, two idle warps) hands registers to the
        // softmax warpgroups; all four of its warps execute this one instruction.
        ptx::setmaxnreg_dec<RegSplit<MOD>::kCtrl>();
        if (warp == kWarpProducer) {
            // ------------------------------------------------------------ TMA producer
            if (lane == 0) {
                ptx::prefetch_tmap(&tmQ);
                ptx::prefetch_tmap(&tmK);
                ptx::prefetch_tmap(&tmV);
                int issued = 0;  // ring uses so far, over all items (K and V tiles alternate)
                int q_loads = 0;
                bool ok = true;
                for (int it = 0; ok && !*abort_flag; ++it) {
                    int64_t k;
                    if (kDyn && args.sched) {
                        // take the next item and publish it to the MMA and softmax warps (-1: none left)
                        k = static_cast<int64_t>(atomicAdd(args.sched, 1ull));
                        if (k >= n_items) k = -1;
                        const int qs = it % kItemQueue;
                        if (it >= kItemQueue &&
                            !(ok = ptx::mbar_wait(&bars.item_empty[qs], ((it / kItemQueue) - 1) & 1, abort_flag,
                                                  args.status, ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns)))
                            break;
                        item_q[qs] = k;
                        ptx::mbar_arrive(&bars.item_full[qs]);
                    } else {
                        k = static_item(n_items, it);  // every role computes the same sequence
                    }
                    if (k < 0) break;
                    const Item I = decode_item(args, k);
                    ODF_CHECK(I.pair >= 0 && I.pair < args.n_pairs && I.bh >= 0 &&
                                  I.bh < args.batch * args.heads_q && I.hk >= 0 && I.hk < args.heads_kv &&
                                  I.n_entries >= 0 && I.n_entries <= args.n_kt,
                              0);
                    ODF_CHECK(args.kv_lo == nullptr || I.n_entries >= 1, 5);
                    if (I.n_entries == 0) continue;
                    // Q of this item replaces the previous item's once its last S MMAs have read it.
                    if (q_loads > 0 && !(ok = ptx::mbar_wait(bars.q_empty, (q_loads - 1) & 1, abort_flag, args.status,
                                                             ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns)))
                        break;
                    ptx::mbar_arrive_expect_tx(bars.q_full, (I.valid1 ? 2 : 1) * Cfg::kTileBytes);
                    for (int c = 0; c < Cfg::kChunks; ++c) {
                        ptx::tma_load_4d(sQ + c * kChunkBytes, &tmQ, bars.q_full, c * 64, I.q00, I.h, I.b);
                    }
                    if (I.valid1) {
                        for (int c = 0; c < Cfg::kChunks; ++c) {
                            ptx::tma_load_4d(sQ + Cfg::kTileBytes + c * kChunkBytes, &tmQ, bars.q_full, c * 64, I.q01,
                                             I.h, I.b);
                        }
                    }
                    ++q_loads;
                    for (int j = 0; ok && j < I.n_entries; ++j) {
                        const int kt = static_cast<int>(kv_entry(args, I, j) & 0xFFFFu);
#ifdef ODF_CHECKED
                        {
                            const uint32_t e_chk = kv_entry(args, I, j);
                            ODF_CHECK(kt < args.n_kt && kt * kTileK < args.n && (e_chk & (kNeed0 | kNeed1)) != 0 &&
                                          (I.valid1 || !(e_chk & kNeed1)),
                                      1);
                        }
#endif
                        for (int half = 0; half < 2; ++half) {
                            const int t = issued;
                            const int s = t % kSlots;
                            const int use = t / kSlots;
                            if (use >= 1 && !(ok = ptx::mbar_wait(&bars.slot_empty[s], (use - 1) & 1, abort_flag,
                                                                  args.status, ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns)))
                                break;
                            uint8_t* dst = sSlots + s * Cfg::kTileBytes;
                            if (!(t == args.stall_load && blockIdx.x == 0)) {  // test-only injected stall
                                ptx::mbar_arrive_expect_tx(&bars.slot_full[s], Cfg::kTileBytes);
                                const void* map =
                                    half == 0 ? static_cast<const void*>(&tmK) : static_cast<const void*>(&tmV);
                                for (int c = 0; c < Cfg::kChunks; ++c) {
                                    ptx::tma_load_4d(dst + c * kChunkBytes, map, &bars.slot_full[s], c * 64,
                                                     kt * kTileK, I.hk, I.b);
                                }
                            }
                            ++issued;
                        }
                    }
                }
                {
                    // Let copies already issued land before the CTA's shared memory is released (on
                    // the normal path the MMA warp has waited for them already; after an abort some
                    // were never consumed).  Older loads landed before their slot was reused.
                    volatile int no_abort = 0;
                    const int first = issued > kSlots ? issued - kSlots : 0;
                    for (int t = first; t < issued; ++t) {
                        if (t == args.stall_load && blockIdx.x == 0) continue;  // never issued
                        ptx::mbar_wait(&bars.slot_full[t % kSlots], (t / kSlots) & 1, &no_abort, nullptr, 0,
                                       args.wait_limit_ns);
                    }
                    if (q_loads > 0) ptx::mbar_wait(bars.q_full, (q_loads - 1) & 1, &no_abort, nullptr, 0, args.wait_limit_ns);
                }
#ifdef ODF_CHECKED
                chk_counts[0] = issued;
#endif
            }
        } else if (warp == kWarpMma) {
            // ------------------------------------------------------------ MMA issuer
            if (lane == 0) {
                constexpr uint32_t kIdescQK = ptx::make_idesc_bf16(128, 128, false);
                constexpr uint32_t kIdescPV = ptx::make_idesc_bf16(128, D, true);
                constexpr uint32_t kDescHi = ptx::sdesc_sw128_hi(1024);
                const uint32_t q_lo0 = ptx::sdesc_sw128_lo(ptx::smem_u32(sQ), 16);
                const uint32_t q_lo1 = ptx::sdesc_sw128_lo(ptx::smem_u32(sQ + Cfg::kTileBytes), 16);
                const uint32_t k_lo0 = ptx::sdesc_sw128_lo(ptx::smem_u32(sSlots), 16);
                const uint32_t v_lo0 = ptx::sdesc_sw128_lo(ptx::smem_u32(sSlots), kChunkBytes);
                constexpr uint32_t kSlotStep = Cfg::kTileBytes >> 4;  // descriptor units per ring slot
                int pv_count[2] = {0, 0};     // P.V MMAs so far (parity of p_full)
                int s_count[2] = {0, 0};      // S MMAs so far (separate-P layout: parity of s_free)
                bool acc[2] = {false, false};  // O_i already holds a P.V of the current item
                int q_loads = 0;
                bool ok = true;
#ifdef ODF_CHECKED
                int ring_waits = 0;
#endif

                // S_i = Q_i K^T (SS, M=128, N=128, K=D) into TMEM columns [128 i, 128 i + 128).
                // Separate-P layout: S_i is overwritten once the softmax has read the previous one.
                auto issue_s = [&](int i, int slot) -> bool {
                    if (Cfg::kSepP && s_count[i] > 0) {
                        if (!ptx::mbar_wait(&bars.s_free[i], (s_count[i] - 1) & 1, abort_flag, args.status,
                                            ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns))
                            return false;
                        ptx::tc_fence_after();
                    }
                    ++s_count[i];
                    const uint32_t qd = i == 0 ? q_lo0 : q_lo1;
                    const uint32_t kd = k_lo0 + static_cast<uint32_t>(slot) * kSlotStep;
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint32_t off = static_cast<uint32_t>(((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4);
                        ptx::mma_bf16_ss_lo(tmem + i * 128, qd + off, kd + off, kDescHi, kIdescQK, kk > 0 ? 1u : 0u);
                    }
                    ptx::tc_commit(&bars.s_full[i]);
                    return true;
                };
                // O_i += P_i V (TS: P_i from TMEM, V MN-major from shared memory; M=128, N=D, K=128).
                auto issue_pv = [&](int i, int slot) -> bool {
                    if (!ptx::mbar_wait(&bars.p_full[i], pv_count[i] & 1, abort_flag, args.status,
                                        ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns))
                        return false;
                    ptx::tc_fence_after();
                    if (kFarSkip && acc[i] &&
                        *reinterpret_cast<volatile const uint32_t*>(far_flags + 4 * i) == 0x01010101u) {
                        ++pv_count[i];  // P_i is zero in all 128 rows: O_i stays as it is
                        return true;
                    }
                    const uint32_t vd = v_lo0 + static_cast<uint32_t>(slot) * kSlotStep;
                    const uint32_t first = acc[i] ? 1u : 0u;
#pragma unroll
                    for (int kk = 0; kk < kTileK / 16; ++kk) {
                        ptx::mma_bf16_ts_lo(tmem + Cfg::kTmemO + i * D,
                                            tmem + (Cfg::kSepP ? Cfg::kTmemP + i * 64 : i * 128) + kk * 8,
                                            vd + static_cast<uint32_t>(kk * (2048 >> 4)), kDescHi, kIdescPV,
                                            (first | kk) ? 1u : 0u);
                    }
                    if (Cfg::kSepP) ptx::tc_commit(&bars.pv_done[i]);
                    acc[i] = true;
                    ++pv_count[i];
                    return true;
                };
                auto wait_full = [&](int t) -> bool {
#ifdef ODF_CHECKED
                    ++ring_waits;
#endif
                    return ptx::mbar_wait(&bars.slot_full[t % kSlots], (t / kSlots) & 1, abort_flag, args.status,
                                          ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns);
                };
                // Q of the next item, then S_0/S_1 of its first KV tile (ring index tk).
                auto start_item = [&](const Item& In, uint32_t en, int tk) -> bool {
                    if (!ptx::mbar_wait(bars.q_full, q_loads & 1, abort_flag, args.status, ODF_ERR_DEVICE_TIMEOUT,
                                        args.wait_limit_ns))
                        return false;
                    ++q_loads;
                    if (!wait_full(tk)) return false;
                    ptx::tc_fence_after();
                    if ((en & kNeed0) && !issue_s(0, tk % kSlots)) return false;
                    if ((en & kNeed1) && !issue_s(1, tk % kSlots)) return false;
                    ptx::tc_commit(&bars.slot_empty[tk % kSlots]);
                    if (In.n_entries == 1) ptx::tc_commit(bars.q_empty);
                    return true;
                };

                // Advances `it` to the next item that visits a KV tile; false at the end of the
                // sequence (or on a timeout, with ok cleared).
                auto next_nonempty = [&](int& it, Item& In) -> bool {
                    for (;;) {
                        ++it;
                        int64_t k;
                        if (kDyn && args.sched) {
                            const int qs = it % kItemQueue;
                            if (!ptx::mbar_wait(&bars.item_full[qs], (it / kItemQueue) & 1, abort_flag, args.status,
                                                ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns)) {
                                ok = false;
                                return false;
                            }
                            k = item_q[qs];
                            ptx::mbar_arrive(&bars.item_empty[qs]);
                        } else {
                            k = static_item(n_items, it);
                        }
                        if (k < 0) return false;
                        In = decode_item(args, k);
                        if (In.n_entries > 0) return true;
                    }
                };

                int it = -1;
                Item I;
                const bool have = next_nonempty(it, I);
                uint32_t e = have ? kv_entry(args, I, 0) : 0u;
                if (have) ok = start_item(I, e, 0);
                for (int j = 0, g = 0; have && ok; ++g) {
                    const int tv = 2 * g + 1;  // V of the current entry
                    const int tk = 2 * g + 2;  // K of the next entry
                    const bool last = j + 1 == I.n_entries;
                    if (!(ok = wait_full(tv))) break;
                    ptx::tc_fence_after();
                    if (!last && Cfg::kSepP) {
                        // separate P: the next S MMAs go first (they only wait for the softmax to
                        // have read S), then this tile's P.V MMAs as each P_i arrives
                        const uint32_t en = kv_entry(args, I, j + 1);
                        if (!(ok = wait_full(tk))) break;
                        ptx::tc_fence_after();
                        if ((en & kNeed0) && !(ok = issue_s(0, tk % kSlots))) break;
                        if ((en & kNeed1) && !(ok = issue_s(1, tk % kSlots))) break;
                        ptx::tc_commit(&bars.slot_empty[tk % kSlots]);
                        if (j + 2 == I.n_entries) ptx::tc_commit(bars.q_empty);  // last S MMAs of the item issued
                        if ((e & kNeed0) && !(ok = issue_pv(0, tv % kSlots))) break;
                        if ((e & kNeed1) && !(ok = issue_pv(1, tv % kSlots))) break;
                        ptx::tc_commit(&bars.slot_empty[tv % kSlots]);
                        e = en;
                        ++j;
                    } else if (!last) {
                        const uint32_t en = kv_entry(args, I, j + 1);
                        if ((e & kNeed0) && !(ok = issue_pv(0, tv % kSlots))) break;
                        if (!(ok = wait_full(tk))) break;
                        ptx::tc_fence_after();
                        if ((en & kNeed0) && !(ok = issue_s(0, tk % kSlots))) break;
                        if ((e & kNeed1) && !(ok = issue_pv(1, tv % kSlots))) break;
                        ptx::tc_commit(&bars.slot_empty[tv % kSlots]);
                        if ((en & kNeed1) && !(ok = issue_s(1, tk % kSlots))) break;
                        ptx::tc_commit(&bars.slot_empty[tk % kSlots]);
                        if (j + 2 == I.n_entries) ptx::tc_commit(bars.q_empty);  // last S MMAs of the item issued
                        e = en;
                        ++j;
                    } else {
                        // last KV tile of the item: finish O_0 and O_1, then open the next item
                        if ((e & kNeed0) && !(ok = issue_pv(0, tv % kSlots))) break;
                        if (acc[0]) ptx::tc_commit(&bars.o_done[0]);
                        if ((e & kNeed1) && !(ok = issue_pv(1, tv % kSlots))) break;
                        ptx::tc_commit(&bars.slot_empty[tv % kSlots]);
                        if (acc[1]) ptx::tc_commit(&bars.o_done[1]);
                        acc[0] = acc[1] = false;
                        if (!next_nonempty(it, I)) break;
                        e = kv_entry(args, I, 0);
                        j = 0;
                        if (!(ok = start_item(I, e, tk))) break;
                    }
                }
                if (!ok) {
                    // Drain the MMAs already issued before the TMEM columns are freed.
                    volatile int no_abort = 0;
                    ptx::tc_commit(bars.drain);
                    ptx::mbar_wait(bars.drain, 0, &no_abort, nullptr, 0, args.wait_limit_ns);
                }
#ifdef ODF_CHECKED
                chk_counts[1] = ring_waits;
                chk_counts[2] = pv_count[0];
                chk_counts[3] = pv_count[1];
#endif
            }
        }
        // ------------------------------------------------------------ teardown (control side)
        ptx::tc_fence_before();
        ptx::cta_barrier();
        if (warp == kWarpProducer) {
            ptx::tc_fence_after();
            ptx::tmem_dealloc(tmem, kTmemCols);
#ifdef ODF_CHECKED
            if (lane == 0 && !*abort_flag) {
                ODF_CHECK(chk_counts[0] == chk_counts[1], 3);
                ODF_CHECK(chk_counts[2] == chk_counts[4] && chk_counts[3] == chk_counts[5], 4);
            }
#endif
        }
    } else {
        // ------------------------------------------------------------ softmax warps
        ptx::setmaxnreg_inc<RegSplit<MOD>::kSoftmax>();
        const int qtile = warp >> 2;         // 0: Q0, 1: Q1
        const int wq = warp & 3;             // TMEM lane quarter
        const int row = wq * 32 + lane;      // 0..127 == TMEM lane
        const uint32_t need_bit = qtile == 0 ? kNeed0 : kNeed1;
        const uint32_t bitmap_bit = qtile == 0 ? kBitmap0 : kBitmap1;
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t s_addr = tmem + lane_off + qtile * 128;
        const uint32_t o_addr = tmem + lane_off + Cfg::kTmemO + qtile * D;
        const uint32_t p_addr = tmem + lane_off + (Cfg::kSepP ? Cfg::kTmemP + qtile * 64 : qtile * 128);
        // bit 0: parity of the next s_full wait, bit 1: of the next o_done wait,
        // bit 2: the current item has fed O_i (at least one S_i tile processed),
        // bit 3: parity of the next pv_done wait, bit 4: a P_i was stored before (separate-P layout)
        uint32_t phases = 0;
        bool ok = true;
#ifdef ODF_CHECKED
        int tiles_done = 0;  // P_i handed to the MMA warp (p_full arrivals of this thread)
#endif

        RowItem* rec_w = reinterpret_cast<RowItem*>(smem + Cfg::kOffRows) + warp;
        const volatile RowItem* rec = rec_w;

        for (int it = 0; ok; ++it) {
            int64_t item;
            if (kDyn && args.sched) {
                item = -1;
                if (lane == 0) {  // one reader per warp takes the item from the queue
                    const int qs = it % kItemQueue;
                    if (ptx::mbar_wait(&bars.item_full[qs], (it / kItemQueue) & 1, abort_flag, args.status,
                                       ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns)) {
                        item = item_q[qs];
                        ptx::mbar_arrive(&bars.item_empty[qs]);
                    } else {
                        item = -2;
                    }
                }
                item = __shfl_sync(0xffffffffu, item, 0);
                if (item == -2) {
                    ok = false;
                    break;
                }
            } else {
                item = static_item(n_items, it);
            }
            if (item < 0) break;
            __syncwarp();  // every lane is done with the previous record
            if (lane == 0) {
                const Item I = decode_item(args, item);
                RowItem r;
                // reversed walk: entry j is KV tile n_entries - 1 - j, counted from the top tile
                r.n_entries = args.kv_reverse ? min(args.n_kt, (I.qend1 + kTileK - 1) / kTileK) : I.n_entries;
                r.pair = I.pair;
                r.q0 = qtile == 0 ? I.q00 : I.q01;
                const bool valid = qtile == 0 || I.valid1;
                if (args.mode == kModeList) {
                    r.n_iter = I.n_entries;
                } else if (!valid) {
                    r.n_iter = 0;
                } else if (args.mode == kModeCausal && !args.kv_reverse) {  // tiles j with j * 128 < row end
                    r.n_iter = max(0, min(I.n_entries, ((qtile == 0 ? I.qend0 : I.qend1) + kTileK - 1) / kTileK - I.kv0));
                } else {
                    r.n_iter = I.n_entries;
                }
                r.bh = I.bh;
                r.b = I.b;
                r.h = I.h;
                r.kv0 = I.kv0;
                r.split = I.split;
                r.slope = 0.0f;
                r.bias_off = (MOD & kModBias) ? static_cast<int64_t>(I.b) * args.bias_s0 +
                                                    static_cast<int64_t>(I.h) * args.bias_s1
                                              : 0;
                if (MOD & kModAlibi) {
                    r.slope = args.alibi_generated
                                  ? exp2f(-8.0f * static_cast<float>(I.h + 1) / static_cast<float>(args.heads_q))
                                  : args.alibi_slopes[I.h];
                }
                *rec_w = r;
            }
            __syncwarp();
            float m_run = -INFINITY;  // running (reference) max, log2 units
            float l_run = 0.0f;       // running sum relative to m_run
            phases &= ~4u;

            const int n_iter = rec->n_iter;
            for (int j = 0; j < n_iter; ++j) {
                uint32_t e = static_cast<uint32_t>(rec->kv0 + j) | need_bit;
                if (args.kv_reverse) {  // causal, diagonal first: entry j is tile n_entries - 1 - j
                    const int kt_r = rec->n_entries - 1 - j;
                    if (kt_r * kTileK >= min(args.m, rec->q0 + kTileQ)) continue;  // beyond this tile's rows
                    e = static_cast<uint32_t>(kt_r) | need_bit;
                }
                if (args.mode == kModeList) {
                    e = __ldg(args.tile_list + static_cast<int64_t>(rec->pair) * args.n_kt + j);
                    if (!(e & need_bit)) continue;
                }
                const int kt = static_cast<int>(e & 0xFFFFu);
                const int k0 = kt * kTileK;
                const int q0 = rec->q0;  // loaded ahead of the wait, which hides its latency
                // Waits are per thread; the warp re-converges (and agrees) before the
                // .sync.aligned TMEM accesses that follow.
                const bool got = ptx::mbar_wait(&bars.s_full[qtile], phases & 1u, abort_flag, args.status,
                                                ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const int qi = q0 + row;
                float slope = 0.0f, slope_log2 = 0.0f;
                if (MOD & kModAlibi) {
                    slope = rec->slope;
                    slope_log2 = slope * kLog2e;
                }
                float s[128];
                ptx::tmem_ld128(s_addr, s);
                if constexpr ((MOD & kModSkipMax) != 0 && !Cfg::kSepP) {
                    // Unmasked tile, every row with a running max: the exponentials are taken against
                    // that max straight away and the row's sum of P is checked afterwards.  The max
                    // moves only past 2^8, which a sum of at most 2^8 rules out; otherwise S is read
                    // again and the general path below runs (with the same P where the max stays), so
                    // the result is the same as with the max pass first.
                    const bool interior = k0 + kTileK <= args.n && !(e & bitmap_bit) &&
                                          !(args.causal && k0 + kTileK - 1 > q0);
                    if (args.scale_log2 > 0.0f && interior && __all_sync(0xffffffffu, m_run != -INFINITY)) {
                        const uint64_t mul2 = ptx::f32x2(args.scale_log2);
                        const uint64_t neg2 = ptx::f32x2(-m_run);
                        uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int c = 0; c < 128; c += 2) {
                            const uint64_t x = ptx::ffma2(ptx::f32x2(s[c], s[c + 1]), mul2, neg2);
                            const float p0 = ptx::ex2(ptx::lo_f32(x));
                            const float p1 = ptx::ex2(ptx::hi_f32(x));
                            sum2[(c >> 1) & 3] = ptx::fadd2(sum2[(c >> 1) & 3], ptx::f32x2(p0, p1));
                            s[c >> 1] = __uint_as_float(ptx::pack_bf16x2(p0, p1));
                        }
                        const uint64_t sum4 = ptx::fadd2(ptx::fadd2(sum2[0], sum2[1]), ptx::fadd2(sum2[2], sum2[3]));
                        const float tile_sum = ptx::lo_f32(sum4) + ptx::hi_f32(sum4);
                        // every P is positive, so a row sum of at most 2^8 bounds each P by 2^8 (no
                        // separate max needed); a larger sum (rare) takes the exact path below
                        if (!__any_sync(0xffffffffu, !(tile_sum <= 256.0f))) {
                            l_run += tile_sum;
                            ptx::tmem_st64_nowait(p_addr, reinterpret_cast<const uint32_t*>(s));
                            ptx::tmem_st_wait();
                            ptx::tc_fence_before();
                            ptx::mbar_arrive(&bars.p_full[qtile]);
                            ODF_COUNT(tiles_done);
                            phases = (phases ^ 1u) | 4u;
                            if (row == 0 && args.visits) {
                                args.visits[(static_cast<int64_t>(rec->bh) * args.n_qt + (q0 / kTileQ)) * args.n_kt +
                                            kt] = 1;
                            }
                            continue;
                        }
                        ptx::tmem_ld128(s_addr, s);  // a row's sum passed 2^8: the general path, from S again
                    }
                }
                if (Cfg::kSepP) {  // S_i is in registers: the next S_i may be computed now
                    ptx::tc_fence_before();
                    ptx::mbar_arrive(&bars.s_free[qtile]);
                }
                if (row == 0 && args.visits) {
                    args.visits[(static_cast<int64_t>(rec->bh) * args.n_qt + (q0 / kTileQ)) * args.n_kt + kt] = 1;
                }

                // score_mod: s*scale (+ ALiBi or bias tensor) (-> soft-cap), in log2 units
                // (attention.cpp:619).  Without a score_mod the scale is folded into the exponent
                // below (raw scores); with a soft-cap, s[] holds tanh(t) and softcap * log2(e) is.
                const bool raw = ((MOD & 7) == 0) && (args.scale_log2 > 0.0f);
                const float fold = (MOD & kModSoftcap) ? args.softcap * kLog2e : (raw ? args.scale_log2 : 1.0f);
                if (MOD & kModBias) {
                    // same-shape additive bias (qk_score_tile.cpp:28-47): s*scale + bias(qi, kj) in
                    // the units of the next step (natural before a soft-cap, log2 otherwise).
                    // Columns at or beyond N, and rows beyond M, are not read (masked or unused).
                    const float mul = (MOD & kModSoftcap) ? args.scale : args.scale_log2;
                    const float bmul = (MOD & kModSoftcap) ? 1.0f : kLog2e;
                    const int ncols = (qi < args.m) ? min(kTileK, args.n - k0) : 0;
                    const float* brow = args.bias + rec->bias_off + static_cast<int64_t>(qi) * args.bias_s2 +
                                        static_cast<int64_t>(k0) * args.bias_s3;
                    const bool vec_row =
                        ncols == kTileK && args.bias_s3 == 1 && (reinterpret_cast<uintptr_t>(brow) & 15u) == 0;
                    if (__all_sync(0xffffffffu, vec_row)) {
                        // The warp's 32 rows are whole, key-contiguous and aligned: each load reads 8
                        // rows x 64 bytes (a thread owning a row would touch 32 lines per load); the
                        // rows are turned around, 16 keys at a time, through 2 KB of the warp's shared
                        // memory, whose 16-byte units are XOR-swizzled by row so the row reads are
                        // conflict-free.
                        float* stage = reinterpret_cast<float*>(smem + Cfg::kOffBias) + warp * (32 * 16);
                        const float* wrow0 = brow - static_cast<int64_t>(lane) * args.bias_s2;  // warp's row 0
#pragma unroll
                        for (int ch = 0; ch < kTileK / 16; ++ch) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int r = 8 * i + (lane >> 2);
                                const float4 v = __ldg(reinterpret_cast<const float4*>(
                                                           wrow0 + static_cast<int64_t>(r) * args.bias_s2 + ch * 16) +
                                                       (lane & 3));
                                reinterpret_cast<float4*>(stage + r * 16)[(lane & 3) ^ ((r >> 1) & 3)] = v;
                            }
                            __syncwarp();
#pragma unroll
                            for (int c4 = 0; c4 < 4; ++c4) {
                                const float4 bv =
                                    reinterpret_cast<const float4*>(stage + lane * 16)[c4 ^ ((lane >> 1) & 3)];
                                const int c = ch * 16 + 4 * c4;
                                s[c + 0] = fmaf(s[c + 0], mul, bv.x * bmul);
                                s[c + 1] = fmaf(s[c + 1], mul, bv.y * bmul);
                                s[c + 2] = fmaf(s[c + 2], mul, bv.z * bmul);
                                s[c + 3] = fmaf(s[c + 3], mul, bv.w * bmul);
                            }
                            __syncwarp();
                        }
                    } else if (vec_row) {
                        const float4* b4 = reinterpret_cast<const float4*>(brow);
#pragma unroll
                        for (int c4 = 0; c4 < kTileK / 4; ++c4) {
                            const float4 bv = __ldg(b4 + c4);
                            s[4 * c4 + 0] = fmaf(s[4 * c4 + 0], mul, bv.x * bmul);
                            s[4 * c4 + 1] = fmaf(s[4 * c4 + 1], mul, bv.y * bmul);
                            s[4 * c4 + 2] = fmaf(s[4 * c4 + 2], mul, bv.z * bmul);
                            s[4 * c4 + 3] = fmaf(s[4 * c4 + 3], mul, bv.w * bmul);
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < kTileK; ++c) {
                            const float bv = c < ncols ? __ldg(brow + static_cast<int64_t>(c) * args.bias_s3) : 0.0f;
                            s[c] = fmaf(s[c], mul, bv * bmul);
                        }
                    }
                    // start bringing this row's next tile into L2 while the rest of the tile runs
                    if (ncols == kTileK && args.bias_s3 == 1 && k0 + 2 * kTileK <= args.n) {
#pragma unroll
                        for (int l = 0; l < 4; ++l) ptx::prefetch_l2(brow + kTileK + 32 * l);
                    }
                }
                if (MOD & kModSoftcap) {
                    // t = (s * scale + ALiBi) / softcap, with 1/softcap folded into the FMAs that form
                    // it; s[] keeps tanh(t) and the exponent below multiplies by softcap * log2(e)
                    const float base = static_cast<float>(k0 - qi);
                    const uint64_t scale2 = ptx::f32x2(args.scale * args.inv_softcap);
                    const uint64_t slope2 = ptx::f32x2(slope * args.inv_softcap);
                    const uint64_t sb2 = ptx::f32x2(slope * base * args.inv_softcap);
                    // column indices (c, c + 1) as floats, stepped in four exact chains instead of
                    // materialising 64 constant pairs
                    uint64_t cidx[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) cidx[k] = ptx::f32x2(2.0f * k, 2.0f * k + 1.0f);
                    if constexpr ((MOD & kModAlibi) != 0 && !Cfg::kSepP) {
                        // t first, with its row max: tanh is monotone, so softcap * log2(e) * tanh(max t)
                        // bounds the row's scores (masked and ragged columns only raise it), and a
                        // far tile (every row below its running max by kFarLog2) skips tanh and ex2
                        float tmax4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                        for (int c = 0; c < 128; c += 2) {
                            uint64_t& ci = cidx[(c >> 1) & 3];
                            const uint64_t bias = ptx::ffma2(ci, slope2, sb2);
                            ci = ptx::fadd2(ci, ptx::f32x2(8.0f));
                            const uint64_t x = ptx::ffma2(ptx::f32x2(s[c], s[c + 1]), scale2, bias);
                            s[c] = ptx::lo_f32(x);
                            s[c + 1] = ptx::hi_f32(x);
                            tmax4[(c >> 1) & 3] = ptx::fmax3(tmax4[(c >> 1) & 3], s[c], s[c + 1]);
                        }
                        const float bound =
                            fold * ptx::tanh_approx(fmaxf(fmaxf(tmax4[0], tmax4[1]), fmaxf(tmax4[2], tmax4[3])));
                        if (__all_sync(0xffffffffu, m_run != -INFINITY && bound < m_run - kFarLog2)) {
                            store_zero_p(p_addr);
                            if (lane == 0) far_flags[qtile * 4 + wq] = 1;
                            ptx::mbar_arrive(&bars.p_full[qtile]);
                            ODF_COUNT(tiles_done);
                            phases = (phases ^ 1u) | 4u;
                            continue;
                        }
#pragma unroll
                        for (int c = 0; c < 128; c += 2) {
                            const uint64_t y = tanh2(ptx::f32x2(s[c], s[c + 1]));
                            s[c] = ptx::lo_f32(y);
                            s[c + 1] = ptx::hi_f32(y);
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < 128; c += 2) {
                            uint64_t x = ptx::f32x2(s[c], s[c + 1]);
                            if (MOD & kModAlibi) {
                                uint64_t& ci = cidx[(c >> 1) & 3];
                                const uint64_t bias = ptx::ffma2(ci, slope2, sb2);
                                ci = ptx::fadd2(ci, ptx::f32x2(8.0f));
                                x = ptx::ffma2(x, scale2, bias);
                            } else if (MOD & kModBias) {  // the bias pass left s * scale + bias
                                x = ptx::fmul2(x, ptx::f32x2(args.inv_softcap));
                            } else {
                                x = ptx::fmul2(x, scale2);
                            }
                            const uint64_t y = tanh2(x);
                            s[c] = ptx::lo_f32(y);
                            s[c + 1] = ptx::hi_f32(y);
                        }
                    }
                } else if (MOD & kModAlibi) {
                    // s * scale * log2(e) + slope * log2(e) * (base + c) on pairs: base + c (exact for the
                    // integer-valued columns) is stepped in four chains, then one multiply and one FMA
                    const float base = static_cast<float>(k0 - qi);
                    const uint64_t scale2 = ptx::f32x2(args.scale_log2);
                    const uint64_t slope2 = ptx::f32x2(slope_log2);
                    uint64_t col[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) col[k] = ptx::f32x2(base + 2.0f * k, base + 2.0f * k + 1.0f);
#pragma unroll
                    for (int c = 0; c < 128; c += 2) {
                        uint64_t& ck = col[(c >> 1) & 3];
                        const uint64_t y = ptx::ffma2(ptx::f32x2(s[c], s[c + 1]), scale2, ptx::fmul2(slope2, ck));
                        ck = ptx::fadd2(ck, ptx::f32x2(8.0f));
                        s[c] = ptx::lo_f32(y);
                        s[c + 1] = ptx::hi_f32(y);
                    }
                } else if (!raw && !(MOD & kModBias)) {
#pragma unroll
                    for (int c = 0; c < 128; ++c) s[c] *= args.scale_log2;
                }

                // element mask on boundary tiles (attention.cpp:54-62, 608-617): column c of the
                // tile survives iff c <= limit (causal kj <= qi, ragged kj < N) and, on tiles that
                // cover a disallowed BlockMask block, its bit in the row's 128-bit allow mask.
                const bool ragged = (k0 + kTileK > args.n);
                const bool diag = args.causal && (min(args.n, k0 + kTileK) - 1 > q0);
                const bool bitmap = (e & bitmap_bit) != 0;
                if (ragged || diag || bitmap) {
                    int limit = args.n - 1 - k0;
                    if (args.causal) limit = min(limit, qi - k0);
                    if (!bitmap) {  // the tile's entry is the same for the whole warp
#pragma unroll
                        for (int c = 0; c < 128; ++c) s[c] = (c <= limit) ? s[c] : -INFINITY;
                    } else {
                        const uint4 allow = row_allow_bits(args, qi, k0);
#pragma unroll
                        for (int c = 0; c < 128; ++c) {
                            const uint32_t word = (c < 32) ? allow.x : (c < 64) ? allow.y : (c < 96) ? allow.z : allow.w;
                            const bool keep = (c <= limit) && ((word >> (c & 31)) & 1u);
                            s[c] = keep ? s[c] : -INFINITY;
                        }
                    }
                }

                // online softmax (attention.cpp:628-644, 662-674) with tree reductions
                float mx8[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) mx8[t] = s[t];
#pragma unroll
                for (int c = 8; c < 128; c += 2) mx8[(c >> 1) & 7] = ptx::fmax3(mx8[(c >> 1) & 7], s[c], s[c + 1]);
                float tile_max = ptx::fmax3(ptx::fmax3(mx8[0], mx8[1], mx8[2]), ptx::fmax3(mx8[3], mx8[4], mx8[5]),
                                            fmaxf(mx8[6], mx8[7]));
                if (raw || (MOD & kModSoftcap)) tile_max *= fold;
                if constexpr ((MOD & kModAlibi) != 0 && (MOD & kModSoftcap) == 0 && !Cfg::kSepP) {
                    // ALiBi far tile: every row's max below its running max by kFarLog2
                    if (__all_sync(0xffffffffu, m_run != -INFINITY && tile_max < m_run - kFarLog2)) {
                        store_zero_p(p_addr);
                        if (lane == 0) far_flags[qtile * 4 + wq] = 1;
                        ptx::mbar_arrive(&bars.p_full[qtile]);
                        ODF_COUNT(tiles_done);
                        phases = (phases ^ 1u) | 4u;
                        continue;
                    }
                }
                float alpha = 1.0f;
                if (m_run == -INFINITY) {
                    m_run = tile_max;  // first valid tile of this row: O holds zeros so far
                } else if (tile_max > m_run + kRescaleLog2) {
                    alpha = ptx::ex2(m_run - tile_max);
                    m_run = tile_max;
                }
                const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
                // P = 2^(x - m) on fp32 pairs; the bf16 pairs are packed in place into s[0..63]
                // (element c/2 is written only after s[c] and s[c+1] were consumed).
                uint64_t sum2[4] = {0, 0, 0, 0};
                {
                    const uint64_t mul2 = ptx::f32x2(fold);
                    const uint64_t neg2 = ptx::f32x2(-m_use);
#pragma unroll
                    for (int c = 0; c < 128; c += 2) {
                        const uint64_t x = ptx::ffma2(ptx::f32x2(s[c], s[c + 1]), mul2, neg2);
                        float p0, p1;
                        if ((poly_exp2_mask<D, MOD>() >> ((c >> 1) & 7)) & 1u) {
                            const uint64_t p = exp2_poly2(x);
                            p0 = ptx::lo_f32(p);
                            p1 = ptx::hi_f32(p);
                        } else {
                            p0 = ptx::ex2(ptx::lo_f32(x));
                            p1 = ptx::ex2(ptx::hi_f32(x));
                        }
                        sum2[(c >> 1) & 3] = ptx::fadd2(sum2[(c >> 1) & 3], ptx::f32x2(p0, p1));
                        s[c >> 1] = __uint_as_float(ptx::pack_bf16x2(p0, p1));
                    }
                }
                const uint64_t sum_all = ptx::fadd2(ptx::fadd2(sum2[0], sum2[1]), ptx::fadd2(sum2[2], sum2[3]));
                l_run = l_run * alpha + (ptx::lo_f32(sum_all) + ptx::hi_f32(sum_all));

                // Separate-P layout: the previous P_i.V must have completed before P_i is overwritten
                // and before O_i is rescaled (S_i(j) can complete ahead of it there).
                if (Cfg::kSepP && (phases & 16u)) {
                    const bool done = ptx::mbar_wait(&bars.pv_done[qtile], (phases >> 3) & 1u, abort_flag,
                                                     args.status, ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns);
                    phases ^= 8u;
                    if (!__all_sync(0xffffffffu, done)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                }
                phases |= 16u;
                // correction: O_i *= alpha when the reference max moved (PV_i of the previous
                // tile is complete: the commit that released S_i(j) covers every earlier MMA, and
                // the separate-P layout waited for it above)
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                    for (int c = 0; c < D / 32; ++c) {
                        float o[32];
                        ptx::tmem_ld32(o_addr + c * 32, o);
#pragma unroll
                        for (int t = 0; t < 32; ++t) o[t] *= alpha;
                        ptx::tmem_st32_nowait(o_addr + c * 32, reinterpret_cast<const uint32_t*>(o));
                    }
                }
                // P_i (over the first 64 columns of S_i, or its own columns for D = 64), the A
                // operand of PV_i
                ptx::tmem_st64_nowait(p_addr, reinterpret_cast<const uint32_t*>(s));
                ptx::tmem_st_wait();
                ptx::tc_fence_before();
                if (kFarSkip && lane == 0) far_flags[qtile * 4 + wq] = 0;
                ptx::mbar_arrive(&bars.p_full[qtile]);
                ODF_COUNT(tiles_done);
                phases = (phases ^ 1u) | 4u;
            }
            if (!ok) break;

            // ---------------------------------------------------------- epilogue
            // O_i is final once the item's last P.V has completed; the next item's first P.V
            // (which overwrites O_i) waits for this thread's next p_full arrival.
            const bool fed = (phases & 4u) != 0;
            if (fed) {
                ok = ptx::mbar_wait(&bars.o_done[qtile], (phases >> 1) & 1u, abort_flag, args.status,
                                    ODF_ERR_DEVICE_TIMEOUT, args.wait_limit_ns);
                phases ^= 2u;
                ptx::tc_fence_after();
            }
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
                const int b = rec->b;
                const int h = rec->h;
                const int qi = rec->q0 + row;
                const bool valid_row = qi < args.m;
                const float inv_l = (l_run > 0.0f) ? (1.0f / l_run) : 0.0f;
                // O leaves through the warp's 2 KB of shared memory (16-byte units XOR-swizzled by
                // row, conflict-free both ways): a thread owning a row would write 32 rows x 16 B
                // per store; read back, each store writes 8 rows x 64 contiguous bytes.
                const int qw = rec->q0 + wq * 32;  // the warp's first row
                const int64_t obase = static_cast<int64_t>(rec->split) * args.o_split +
                                      static_cast<int64_t>(b) * args.o_stride_b +
                                      static_cast<int64_t>(h) * args.o_stride_h +
                                      static_cast<int64_t>(qw) * args.o_stride_t;
                uint4* srow = reinterpret_cast<uint4*>(smem + Cfg::kOffBias) + warp * (32 * 4) + lane * 4;
                const uint4* sbase = reinterpret_cast<const uint4*>(smem + Cfg::kOffBias) + warp * (32 * 4);
                const int wsw = (lane >> 1) & 3;  // swizzle of this thread's staging row
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    float o[32];
                    if (fed) {
                        ptx::tmem_ld32(o_addr + c * 32, o);
                    } else {
#pragma unroll
                        for (int t = 0; t < 32; ++t) o[t] = 0.0f;
                    }
                    // bf16: the 32 columns are one 64-byte piece per row; fp32: two 16-column pieces
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        if (args.o_bf16 && hf == 1) break;
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint4 w;
                            if (args.o_bf16) {
                                w.x = ptx::pack_bf16x2(o[8 * v + 0] * inv_l, o[8 * v + 1] * inv_l);
                                w.y = ptx::pack_bf16x2(o[8 * v + 2] * inv_l, o[8 * v + 3] * inv_l);
                                w.z = ptx::pack_bf16x2(o[8 * v + 4] * inv_l, o[8 * v + 5] * inv_l);
                                w.w = ptx::pack_bf16x2(o[8 * v + 6] * inv_l, o[8 * v + 7] * inv_l);
                            } else {
                                const int t = 16 * hf + 4 * v;
                                w = make_uint4(__float_as_uint(o[t + 0] * inv_l), __float_as_uint(o[t + 1] * inv_l),
                                               __float_as_uint(o[t + 2] * inv_l), __float_as_uint(o[t + 3] * inv_l));
                            }
                            srow[v ^ wsw] = w;
                        }
                        __syncwarp();
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int r = 8 * i + (lane >> 2);
                            const int u = lane & 3;
                            const uint4 w = sbase[r * 4 + (u ^ ((r >> 1) & 3))];
                            if (qw + r < args.m) {
                                const int64_t off = obase + static_cast<int64_t>(r) * args.o_stride_t;
                                if (args.o_bf16) {
                                    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.o) + off + c * 32 +
                                                              u * 8) = w;
                                } else {
                                    *reinterpret_cast<uint4*>(static_cast<float*>(args.o) + off + c * 32 + hf * 16 +
                                                              u * 4) = w;
                                }
                            }
                        }
                        __syncwarp();
                    }
                }
                if (valid_row && args.lse) {
                    const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
                    args.lse[static_cast<int64_t>(rec->split) * args.lse_split + static_cast<int64_t>(rec->bh) * args.m + qi] =
                        (l_run > 0.0f) ? (m_use + log2f(l_run)) * kLn2 : -INFINITY;
                }
            }
        }

        // ------------------------------------------------------------ teardown (softmax side)
        // Each role ends with its own copy of the CTA barrier, so the two register budgets
        // never meet in common code.
#ifdef ODF_CHECKED
        if (row == 0) chk_counts[4 + qtile] = tiles_done;
#endif
        ptx::tc_fence_before();
        ptx::cta_barrier();
    }
}

// Classification of one 128x128 tile: 0 skipped, 1 full, 2 element-masked; *bitmap_partial
// is set when a covered BlockMask block is disallowed (the kernel then tests the bitmap
// per element).  Skip rule: the reference's causal break (attention.cpp:537-539) or no
// allowed BlockMask block covered (attention.cpp:70-86).
__device__ uint32_t classify_tile(int32_t m, int32_t n, int qt, int kt, int32_t causal, const uint8_t* mask,
                                  int32_t mqbs, int32_t mkbs, int32_t mqblocks, int32_t mkblocks,
                                  bool* bitmap_partial) {
    *bitmap_partial = false;
    const int q0 = qt * kTileQ;
    const int q1 = min(m, q0 + kTileQ);
    const int k0 = kt * kTileK;
    const int k1 = min(n, k0 + kTileK);
    if (q0 >= m) return 0;
    if (causal && k0 >= q1) return 0;
    uint32_t cls = (causal && k1 - 1 > q0) ? 2u : 1u;
    if (mask) {
        bool any_allowed = false, any_denied = false;
        for (int qb = q0 / mqbs; qb <= (q1 - 1) / mqbs; ++qb) {
            for (int kb = k0 / mkbs; kb <= (k1 - 1) / mkbs; ++kb) {
                const bool okb = qb < mqblocks && kb < mkblocks && mask[static_cast<int64_t>(qb) * mkblocks + kb] != 0;
                any_allowed |= okb;
                any_denied |= !okb;
            }
        }
        if (!any_allowed) return 0;
        if (any_denied) {
            cls = 2;
            *bitmap_partial = true;
        }
    }
    return cls;
}

// Per-query-tile classes (odf_tile_map_sm100): one thread per tile.
__global__ void tile_class_kernel(int32_t m, int32_t n, int32_t n_qt, int32_t n_kt, int32_t causal,
                                  const uint8_t* __restrict__ mask, int32_t mqbs, int32_t mkbs, int32_t mqblocks,
                                  int32_t mkblocks, uint8_t* __restrict__ cls_out) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(n_qt) * n_kt) return;
    const int qt = static_cast<int>(idx / n_kt);
    const int kt = static_cast<int>(idx - static_cast<int64_t>(qt) * n_kt);
    bool bp;
    cls_out[idx] = static_cast<uint8_t>(classify_tile(m, n, qt, kt, causal, mask, mqbs, mkbs, mqblocks, mkblocks, &bp));
}

// Per-pair KV lists (block-mask mode): one warp per query-tile pair, increasing kv order.
__global__ void pair_list_kernel(int32_t m, int32_t n, int32_t n_pairs, int32_t n_kt, int32_t causal,
                                 const uint8_t* __restrict__ mask, int32_t mqbs, int32_t mkbs, int32_t mqblocks,
                                 int32_t mkblocks, uint32_t* __restrict__ list, int32_t* __restrict__ count) {
    const int pair = blockIdx.x;
    const int lane = threadIdx.x;
    if (pair >= n_pairs) return;
    int base = 0;
    for (int kt0 = 0; kt0 < n_kt; kt0 += 32) {
        const int kt = kt0 + lane;
        uint32_t entry = 0;
        if (kt < n_kt) {
            bool bp0, bp1;
            const uint32_t c0 = classify_tile(m, n, 2 * pair, kt, causal, mask, mqbs, mkbs, mqblocks, mkblocks, &bp0);
            const uint32_t c1 = classify_tile(m, n, 2 * pair + 1, kt, causal, mask, mqbs, mkbs, mqblocks, mkblocks, &bp1);
            if (c0 | c1) {
                entry = static_cast<uint32_t>(kt) | (c0 ? kNeed0 : 0u) | (c1 ? kNeed1 : 0u) | (bp0 ? kBitmap0 : 0u) |
                        (bp1 ? kBitmap1 : 0u);
            }
        }
        const unsigned ballot = __ballot_sync(0xffffffffu, entry != 0);
        if (entry != 0) list[static_cast<int64_t>(pair) * n_kt + base + __popc(ballot & ((1u << lane) - 1u))] = entry;
        base += __popc(ballot);
    }
    if (lane == 0) count[pair] = base;
}

// One bf16 [batch, heads, rows, 128] tensor for tile_norm_kernel (element strides {b, h, t},
// rows 16-byte aligned) and its output, one float per (batch, head, 128-row tile).
struct NormSrc {
    const __nv_bfloat16* x;
    int64_t sb, sh, st;
    int32_t heads, rows, n_tiles;
    int64_t n_blocks;  // batch * heads * n_tiles
    float* out;
};

// Largest row norm ||x_r||_2 of each 128-row tile of Q (the first blocks) and of K (the rest):
// one block of 128 threads per (batch, head, tile), 16 lanes reading a row's 256 bytes.  Rows
// at or beyond `rows` count 0.
__global__ void __launch_bounds__(128) tile_norm_kernel(const NormSrc src0, const NormSrc src1) {
    const bool first = blockIdx.x < src0.n_blocks;
    const NormSrc& S = first ? src0 : src1;
    const __nv_bfloat16* __restrict__ x = S.x;
    const int64_t sb = S.sb, sh = S.sh, st = S.st;
    const int32_t heads = S.heads, rows = S.rows, n_tiles = S.n_tiles;
    float* __restrict__ out = S.out;
    const int64_t idx = first ? static_cast<int64_t>(blockIdx.x) : static_cast<int64_t>(blockIdx.x) - src0.n_blocks;
    const int tile = static_cast<int>(idx % n_tiles);
    const int64_t bh = idx / n_tiles;
    const int64_t b = bh / heads;
    const int64_t h = bh - b * heads;
    const __nv_bfloat16* base = x + b * sb + h * sh;
    const int sub = threadIdx.x & 15;
    // all 16 of the thread's loads are issued before any is used (256 bytes in flight per thread)
    uint4 u[kTileQ / 8];
#pragma unroll
    for (int i = 0; i < kTileQ / 8; ++i) {
        const int row = tile * kTileQ + (threadIdx.x >> 4) + 8 * i;
        u[i] = row < rows ? __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(row) * st) + sub)
                          : make_uint4(0u, 0u, 0u, 0u);
    }
    float best = 0.0f;
#pragma unroll
    for (int i = 0; i < kTileQ / 8; ++i) {
        const uint32_t w[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
        float ss = 0.0f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float lo = __uint_as_float(w[t] << 16);
            const float hi = __uint_as_float(w[t] & 0xFFFF0000u);
            ss = fmaf(lo, lo, fmaf(hi, hi, ss));
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        best = fmaxf(best, ss);
    }
    best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 16));
    __shared__ float warp_best[4];
    if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0)
        out[idx] = sqrtf(fmaxf(fmaxf(warp_best[0], warp_best[1]), fmaxf(warp_best[2], warp_best[3])));
}

// Far KV tiles of causal ALiBi, from norms alone (one warp per (batch, q-head, pair), its lanes
// testing 32 KV tiles at a time): for row qi and key kj of KV tile kt,
// |s scale| <= |scale| |q_i| |k_j| (Cauchy-Schwarz) bounds the score from above by
//   U = c Kmax(kt) + slope (kt*128 + 127 - q0),   c = |scale| Qmax(qt) (1 + 2^-7)
// and every row's max from below by its diagonal key (kj = qi, ALiBi term 0), L = -c Kmax(qt).
// With f the soft-cap (or the identity), f(U) < f(L) - 48 ln 2 gives P < 2^-48 of the row's
// largest term on the whole tile.  kv_lo[pair] is the first KV tile that is not far for both
// query tiles of the pair (tiles below it are all far); the first KV tile not far stops the scan.
// A query tile with rows at or beyond N (no diagonal key), a non-positive or non-finite slope,
// or non-finite norms keeps every tile.
__global__ void far_lo_kernel(const FwdArgs a, const float* __restrict__ qn, const float* __restrict__ kn,
                              int32_t* __restrict__ kv_lo) {
    const int64_t idx = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t n_bh = static_cast<int64_t>(a.batch) * a.heads_q;
    if (idx >= n_bh * a.n_pairs) return;  // whole warps leave together
    const int64_t bh = idx / a.n_pairs;
    const int pair = static_cast<int>(idx - bh * a.n_pairs);
    const int b = static_cast<int>(bh / a.heads_q);
    const int h = static_cast<int>(bh - static_cast<int64_t>(b) * a.heads_q);
    const int hk = h / (a.heads_q / a.heads_kv);
    const float slope = a.alibi_generated ? exp2f(-8.0f * static_cast<float>(h + 1) / static_cast<float>(a.heads_q))
                                          : a.alibi_slopes[h];
    const float* kn_u = kn + (static_cast<int64_t>(b) * a.heads_kv + hk) * a.n_kt;
    const float thr = 48.0f * kLn2;
    int lo = 0x7fffffff;
    for (int qt = 2 * pair; qt <= 2 * pair + 1 && qt < a.n_qt; ++qt) {
        const int q0 = qt * kTileQ;
        const int qe = min(a.m, q0 + kTileQ);
        int lo_q = 0;
        const float c = fabsf(a.scale) * qn[bh * a.n_qt + qt] * (1.0f + 0.0078125f);
        if (qe - 1 < a.n && slope > 0.0f && isfinite(slope) && isfinite(c)) {
            const float L = -c * kn_u[qt];
            const float fL = a.softcap > 0.0f ? a.softcap * tanhf(L / a.softcap) : L;
            for (int kt0 = 0; kt0 < qt; kt0 += 32) {
                const int kt = kt0 + lane;
                bool far = false;
                if (kt < qt) {
                    const float U = c * kn_u[kt] + slope * static_cast<float>(kt * kTileK + kTileK - 1 - q0);
                    const float fU = a.softcap > 0.0f ? a.softcap * tanhf(U / a.softcap) : U;
                    far = fU < fL - thr;  // NaN keeps the tile
                }
                const unsigned near = ~__ballot_sync(0xffffffffu, far) & (qt - kt0 >= 32 ? 0xffffffffu : ((1u << (qt - kt0)) - 1u));
                if (near != 0u) {  // the first tile from 0 that is not far ends the scan
                    lo_q = kt0 + __ffs(near) - 1;
                    break;
                }
                lo_q = min(qt, kt0 + 32);
            }
        }
        lo = min(lo, lo_q);
    }
    if (lane == 0) kv_lo[idx] = lo;
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
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
std::once_flag g_encode_once;

// Per device: set up once per CUDA context.  Kernel attributes and the status word's address
// belong to the context the module was loaded into, so a new context on the device (after
// cudaDeviceReset, or a context the caller made current) repeats the set-up.
struct DeviceState {
    bool ready = false;
    void* ctx = nullptr;
    int status_code = ODF_OK;
    int* status_ptr = nullptr;
    int sm_count = 0;
};
constexpr int kMaxDevices = 64;
DeviceState g_devices[kMaxDevices];
std::mutex g_device_mutex;

// Sets the shared-memory limit and checks that the kernel was compiled with the register
// count the setmaxnreg split assumes: with fewer registers at launch the softmax warps'
// increase could never be granted, so such a build is refused instead of launched.
template <int D, int MOD>
cudaError_t set_kernel_attrs(bool* regs_ok) {
    cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<D, MOD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Config<D>::kSmemBytes);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, flash_fwd_kernel<D, MOD>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegs || fa.maxThreadsPerBlock < kThreads) *regs_ok = false;
    return cudaSuccess;
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
    if constexpr (D == 128) {
        if (mod == kModSkipMax) {
            flash_fwd_kernel<128, kModSkipMax><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a);
            return cudaGetLastError();
        }
    }
    switch (mod) {
        case 0: flash_fwd_kernel<D, 0><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        case 1: flash_fwd_kernel<D, 1><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        case 2: flash_fwd_kernel<D, 2><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        case 3: flash_fwd_kernel<D, 3><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        case 4: flash_fwd_kernel<D, 4><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
        default: flash_fwd_kernel<D, 6><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a); break;
    }
    return cudaGetLastError();
}

// Merge of the KV splits' partial results, one warp per (batch, q-head, query row): with the
// splits' natural-log LSE_s and normalised O_s, LSE = log sum_s exp(LSE_s) and
// O = sum_s exp(LSE_s - LSE) O_s (splits with LSE_s = -inf, no key of the row in them, weigh 0;
// a row with no key at all gets O = 0 and LSE = -inf, as without splits).
template <int D>
__global__ void __launch_bounds__(256) split_combine_kernel(const float* __restrict__ po, const float* __restrict__ pl,
                                                            int n_splits, int64_t o_split, int64_t l_split,
                                                            int64_t rows, int m, int heads_q, void* o, int o_bf16,
                                                            int64_t osb, int64_t osh, int64_t ost, float* lse) {
    constexpr int V = D / 32;  // columns per lane
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;  // whole warps leave together
    // the splits' LSEs, lane l holding splits l, l + 32, ...: the row's max, then its weight sum
    float mx = -INFINITY;
    for (int sp = lane; sp < n_splits; sp += 32) mx = fmaxf(mx, __ldg(pl + sp * l_split + row));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.0f;
    float sum = 0.0f;
    if (mx != -INFINITY) {
        for (int base = 0; base < n_splits; base += 32) {
            const int sp_l = base + lane;
            const float l = sp_l < n_splits ? __ldg(pl + sp_l * l_split + row) : -INFINITY;
            const float w_l = l == -INFINITY ? 0.0f : expf(l - mx);
            sum += w_l;
            const int cnt = min(32, n_splits - base);
            // split t's O row, its weight broadcast from lane t; the loads are independent, so
            // several are in flight at once
#pragma unroll 8
            for (int t = 0; t < cnt; ++t) {
                const float w = __shfl_sync(0xffffffffu, w_l, t);
                const float* src = po + (base + t) * o_split + row * D + lane * V;
                if constexpr (V == 4) {
                    const float4 x = __ldg(reinterpret_cast<const float4*>(src));
                    acc[0] = fmaf(w, x.x, acc[0]);
                    acc[1] = fmaf(w, x.y, acc[1]);
                    acc[2] = fmaf(w, x.z, acc[2]);
                    acc[3] = fmaf(w, x.w, acc[3]);
                } else {
                    const float2 x = __ldg(reinterpret_cast<const float2*>(src));
                    acc[0] = fmaf(w, x.x, acc[0]);
                    acc[1] = fmaf(w, x.y, acc[1]);
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    const int64_t bh = row / m;
    const int64_t qi = row - bh * m;
    const int64_t b = bh / heads_q;
    const int64_t h = bh - b * heads_q;
    const int64_t off = b * osb + h * osh + qi * ost + lane * V;
    if (o_bf16) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(o) + off;
        if constexpr (V == 4) {
            *reinterpret_cast<uint2*>(dst) = make_uint2(ptx::pack_bf16x2(acc[0] * inv, acc[1] * inv),
                                                        ptx::pack_bf16x2(acc[2] * inv, acc[3] * inv));
        } else {
            *reinterpret_cast<uint32_t*>(dst) = ptx::pack_bf16x2(acc[0] * inv, acc[1] * inv);
        }
    } else {
        float* dst = static_cast<float*>(o) + off;
        if constexpr (V == 4) {
            *reinterpret_cast<float4*>(dst) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
        } else {
            *reinterpret_cast<float2*>(dst) = make_float2(acc[0] * inv, acc[1] * inv);
        }
    }
    if (lse != nullptr && lane == 0) lse[row] = mx == -INFINITY ? -INFINITY : mx + logf(sum);
}

// Bytes of the partial O (fp32) and LSE of `n_splits` KV splits, each plane 256-byte aligned.
size_t split_partial_bytes(int64_t n_bh, int64_t m, int64_t d, int64_t n_splits) {
    auto up = [](int64_t bytes) { return static_cast<size_t>((bytes + 255) & ~int64_t{255}); };
    return up(n_splits * n_bh * m * d * 4) + up(n_splits * n_bh * m * 4);
}

}  // namespace

SplitPlan plan_kv_splits(int64_t batch, int64_t heads_q, int64_t seqlen_q, int64_t seqlen_k, bool eligible,
                         int64_t sm_count) {
    const int64_t n_qt = (seqlen_q + kTileQ - 1) / kTileQ;
    const int64_t n_kt = (seqlen_k + kTileK - 1) / kTileK;
    SplitPlan sp{1, static_cast<int32_t>(n_kt)};
    if (!eligible || n_kt < 2 || sm_count <= 0) return sp;
    // the same item rule as the launch: single query tiles when each fits on its own SM
    const bool single = n_qt > 1 && batch * heads_q * n_qt <= sm_count;
    const int64_t items = batch * heads_q * (single ? n_qt : (n_qt + 1) / 2);
    if (items <= 0 || 2 * items > sm_count) return sp;
    // at least kMinSplitTiles KV tiles per split: an item's fixed costs (Q load, epilogue) and the
    // merge launch outweigh fewer (c1, 4 KV tiles per query tile, measured 15.2 -> 18.0 us split in 4)
    constexpr int64_t kMinSplitTiles = 4;
    int64_t splits = sm_count / items < n_kt / kMinSplitTiles ? sm_count / items : n_kt / kMinSplitTiles;
    if (splits < 2) return sp;
    const int64_t per = (n_kt + splits - 1) / splits;
    splits = (n_kt + per - 1) / per;
    if (splits < 2) return sp;
    sp.n_splits = static_cast<int32_t>(splits);
    sp.kv_per_split = static_cast<int32_t>(per);
    return sp;
}

size_t kv_split_bytes(int64_t batch, int64_t heads_q, int64_t seqlen_q, int64_t seqlen_k, int64_t head_dim,
                      bool eligible) {
    const SplitPlan sp = plan_kv_splits(batch, heads_q, seqlen_q, seqlen_k, eligible, kSplitSizingSms);
    return sp.n_splits > 1 ? split_partial_bytes(batch * heads_q, seqlen_q, head_dim, sp.n_splits) : 0;
}

size_t workspace_bytes_for(int64_t seqlen_q, int64_t seqlen_k, bool has_mask) {
    if (!has_mask) return kSchedBytes;
    const int64_t n_qt = (seqlen_q + kTileQ - 1) / kTileQ;
    const int64_t n_pairs = (n_qt + 1) / 2;
    const int64_t n_kt = (seqlen_k + kTileK - 1) / kTileK;
    const size_t list = static_cast<size_t>(n_pairs * n_kt) * sizeof(uint32_t);
    const size_t count = static_cast<size_t>(n_pairs) * sizeof(int32_t);
    return kSchedBytes + ((list + 255) & ~static_cast<size_t>(255)) + ((count + 255) & ~static_cast<size_t>(255));
}

size_t far_bound_bytes(int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seqlen_q, int64_t seqlen_k) {
    const int64_t n_qt = (seqlen_q + kTileQ - 1) / kTileQ;
    const int64_t n_pairs = (n_qt + 1) / 2;
    const int64_t n_kt = (seqlen_k + kTileK - 1) / kTileK;
    auto up = [](int64_t bytes) { return static_cast<size_t>((bytes + 255) & ~int64_t{255}); };
    return up(batch * heads_q * n_qt * 4) + up(batch * heads_kv * n_kt * 4) + up(batch * heads_q * n_pairs * 4);
}

int read_check_bits(uint32_t* out) {
#ifdef ODF_CHECKED
    unsigned int bits = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&bits, g_check_bits, sizeof(bits));
    const unsigned int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_check_bits, &zero, sizeof(zero));
    if (e != cudaSuccess) return ODF_ERR_CUDA;
    *out = bits;
    return ODF_OK;
#else
    (void)out;
    return ODF_ERR_UNSUPPORTED;
#endif
}

void* current_context() {
    static CtxGetCurrentFn fn_ptr = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn_ptr = reinterpret_cast<CtxGetCurrentFn>(fn);
        }
    });
    CUcontext ctx = nullptr;
    if (fn_ptr == nullptr || fn_ptr(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

namespace {

int setup_device_locked(int device, DeviceState& st, const char** err) {
    st.ready = false;
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
    bool regs_ok = true;
    if (e == cudaSuccess) e = set_kernel_attrs<64, 0>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<64, 1>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<64, 2>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<64, 3>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<64, 4>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<64, 6>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, 0>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, 1>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, 2>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, 3>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, 4>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, 6>(&regs_ok);
    if (e == cudaSuccess) e = set_kernel_attrs<128, kModSkipMax>(&regs_ok);
    if (e == cudaSuccess && !regs_ok) {
        st.status_code = ODF_ERR_UNSUPPORTED;
        *err = "flash kernel built with an unexpected register count (the warp register split needs 168)";
        return ODF_ERR_UNSUPPORTED;
    }
    void* sp = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&sp, g_device_status);
    if (e != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return ODF_ERR_CUDA;
    }
    st.status_ptr = static_cast<int*>(sp);
    st.sm_count = prop.multiProcessorCount;
    st.ctx = current_context();  // the runtime calls above made the device's context current
    st.ready = true;
    return ODF_OK;
}

}  // namespace

int ensure_device_ready(int device, const char** err) {
    if (device < 0 || device >= kMaxDevices) {
        *err = "device index out of range";
        return ODF_ERR_NO_DEVICE;
    }
    void* ctx = current_context();
    std::lock_guard<std::mutex> lock(g_device_mutex);
    DeviceState& st = g_devices[device];
    if (st.ready && ctx != nullptr && st.ctx == ctx) return ODF_OK;
    return setup_device_locked(device, st, err);
}

int* device_status_ptr(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_device_mutex);
    return g_devices[device].status_ptr;
}

int launch_tile_map(int32_t m, int32_t n, int32_t causal, const uint8_t* mask, int32_t mqbs, int32_t mkbs,
                    int32_t mqblocks, int32_t mkblocks, uint8_t* cls_out, cudaStream_t stream) {
    const int n_qt = (m + kTileQ - 1) / kTileQ;
    const int n_kt = (n + kTileK - 1) / kTileK;
    const int64_t total = static_cast<int64_t>(n_qt) * n_kt;
    const int blocks = static_cast<int>((total + 255) / 256);
    tile_class_kernel<<<blocks, 256, 0, stream>>>(m, n, n_qt, n_kt, causal, mask, mqbs, mkbs, mqblocks, mkblocks,
                                                   cls_out);
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
    int sm_count = 0;
    {
        std::lock_guard<std::mutex> lock(g_device_mutex);
        sm_count = g_devices[device].sm_count;
    }
    // one query tile per item when even that leaves SMs idle (not for block-mask lists or the
    // causal ALiBi bound, which are built per pair)
    a.single_tile = a.mode != kModeList && !a.kv_reverse && a.n_qt > 1 &&
                    static_cast<int64_t>(a.batch) * a.heads_q * a.n_qt <= sm_count;
    a.n_pairs = a.single_tile ? a.n_qt : (a.n_qt + 1) / 2;
    if (a.wait_limit_ns == 0) a.wait_limit_ns = kDefaultWaitLimitNs;

    // KV splits when the items leave SMs idle and the workspace has room for the partial results
    // (as many splits as fit, down to none): O and LSE go to fp32 partials after the counter, and
    // split_combine_kernel writes the caller's O and LSE after the forward kernel.
    a.n_splits = 1;
    a.kv_per_split = a.n_kt;
    a.fd_split = make_fastdiv(1);
    a.o_split = 0;
    a.lse_split = 0;
    void* const out_o = a.o;
    float* const out_lse = a.lse;
    const int32_t out_bf16 = a.o_bf16;
    const int64_t out_sb = a.o_stride_b, out_sh = a.o_stride_h, out_st = a.o_stride_t;
    const int64_t n_bh = static_cast<int64_t>(a.batch) * a.heads_q;
    {
        const bool eligible = L.allow_split && a.mode != kModeList && !a.kv_reverse && L.workspace != nullptr;
        SplitPlan sp = plan_kv_splits(a.batch, a.heads_q, a.m, a.n, eligible, sm_count);
        if (L.forced_splits > 0) sp.n_splits = eligible ? L.forced_splits : 1;
        const size_t room = L.workspace_bytes > kSchedBytes ? L.workspace_bytes - kSchedBytes : 0;
        int64_t splits = sp.n_splits;
        while (splits > 1 && split_partial_bytes(n_bh, a.m, L.head_dim, splits) > room) --splits;
        if (splits > 1) {
            const int64_t per = (a.n_kt + splits - 1) / splits;
            splits = (a.n_kt + per - 1) / per;
        }
        if (splits > 1) {
            const int64_t per = (a.n_kt + splits - 1) / splits;
            uint8_t* ws = static_cast<uint8_t*>(L.workspace) + kSchedBytes;
            const int64_t o_plane = n_bh * a.m * L.head_dim;
            a.n_splits = static_cast<int32_t>(splits);
            a.kv_per_split = static_cast<int32_t>(per);
            a.fd_split = make_fastdiv(static_cast<uint32_t>(splits));
            a.o = ws;
            a.o_bf16 = 0;
            a.o_stride_b = static_cast<int64_t>(a.heads_q) * a.m * L.head_dim;
            a.o_stride_h = static_cast<int64_t>(a.m) * L.head_dim;
            a.o_stride_t = L.head_dim;
            a.o_split = o_plane;
            a.lse = reinterpret_cast<float*>(ws + ((splits * o_plane * 4 + 255) & ~int64_t{255}));
            a.lse_split = n_bh * a.m;
        }
    }

    CUtensorMap tq, tk, tv;
    if (encode_bf16_4d(&tq, L.q, L.head_dim, a.m, a.heads_q, a.batch, L.q_strides) != CUDA_SUCCESS ||
        encode_bf16_4d(&tk, L.k, L.head_dim, a.n, a.heads_kv, a.batch, L.k_strides) != CUDA_SUCCESS ||
        encode_bf16_4d(&tv, L.v, L.head_dim, a.n, a.heads_kv, a.batch, L.v_strides) != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled rejected a Q/K/V layout (pointers and strides must be 16-byte aligned)";
        return ODF_ERR_INVALID_ARG;
    }
    // Item assignment.  When the K/V of all (batch, kv-head) units exceeds what L2 keeps (about
    // 32 MB of bf16 K and V per block) and a workspace is given, items come in blocks of units
    // whose K/V fit, handed out greedily by a counter at the workspace's start (zeroed here), so
    // the CTAs working at the same time share their K/V tiles in L2.  Otherwise (small K/V,
    // block-mask lists whose uneven items want the global longest-first order, or no workspace)
    // the fixed pair-major snake order, which needs no counter.
    const int64_t n_units = static_cast<int64_t>(a.batch) * a.heads_kv;
    a.sched = nullptr;
    a.units_per_block = static_cast<int32_t>(n_units);
    {
        const int64_t kv_unit_bytes = 4 * static_cast<int64_t>(a.n) * L.head_dim;
        int64_t per_block = (int64_t{32} << 20) / (kv_unit_bytes > 0 ? kv_unit_bytes : 1);
        if (per_block < 1) per_block = 1;
        if (per_block < n_units && a.n_splits == 1 && a.mode != kModeList && L.workspace != nullptr &&
            L.workspace_bytes >= kSchedBytes && L.head_dim == 128 && !L.has_alibi && !L.has_softcap &&
            !L.has_bias) {  // the instantiation with greedy assignment compiled in
            a.sched = static_cast<unsigned long long*>(L.workspace);
            a.units_per_block = static_cast<int32_t>(per_block);
        } else if (a.kv_reverse && a.n_splits == 1 && L.workspace != nullptr && L.workspace_bytes >= kSchedBytes) {
            // causal ALiBi: greedy over one block (pair-major over all heads), so that CTAs whose
            // items lost their far tiles take more items
            a.sched = static_cast<unsigned long long*>(L.workspace);
        }
        if (a.sched != nullptr && cudaMemsetAsync(L.workspace, 0, sizeof(unsigned long long), stream) != cudaSuccess) {
            *err = "clearing the work-item counter failed";
            return ODF_ERR_CUDA;
        }
    }
    if (a.mode == kModeList) {
        uint8_t* ws = static_cast<uint8_t*>(L.workspace) + kSchedBytes;
        const size_t list_bytes = static_cast<size_t>(a.n_pairs) * a.n_kt * sizeof(uint32_t);
        uint32_t* list = reinterpret_cast<uint32_t*>(ws);
        int32_t* count = reinterpret_cast<int32_t*>(ws + ((list_bytes + 255) & ~static_cast<size_t>(255)));
        pair_list_kernel<<<a.n_pairs, 32, 0, stream>>>(a.m, a.n, a.n_pairs, a.n_kt, a.causal, a.mask, a.mask_qbs,
                                                        a.mask_kbs, a.mask_qblocks, a.mask_kblocks, list, count);
        if (cudaGetLastError() != cudaSuccess) {
            *err = "tile-list kernel launch failed";
            return ODF_ERR_CUDA;
        }
        a.tile_list = list;
        a.tile_count = count;
    }
    // 32-bit item decode when every item index (and so every quantity the decode forms) fits
    {
        const int64_t items = static_cast<int64_t>(a.batch) * a.heads_q * a.n_pairs * a.n_splits;
        a.fast_decode = items <= INT32_MAX ? 1 : 0;
        if (a.fast_decode) {
            const uint32_t gq = static_cast<uint32_t>(a.heads_q / a.heads_kv);
            const uint32_t upb = static_cast<uint32_t>(a.units_per_block);
            const uint32_t last = static_cast<uint32_t>(n_units - (n_units - 1) / upb * upb);  // units of the last block
            a.fd_bh = make_fastdiv(static_cast<uint32_t>(a.batch) * static_cast<uint32_t>(a.heads_q));
            a.fd_hq = make_fastdiv(static_cast<uint32_t>(a.heads_q));
            a.fd_gq = make_fastdiv(gq);
            a.fd_hkv = make_fastdiv(static_cast<uint32_t>(a.heads_kv));
            a.fd_block = make_fastdiv(upb * gq * static_cast<uint32_t>(a.n_pairs));
            a.fd_row = make_fastdiv(upb * gq);
            a.fd_row_last = make_fastdiv((last < upb ? last : upb) * gq);
        }
    }
    // causal ALiBi: the norm bound over whole KV tiles, when the workspace has room for it
    a.kv_lo = nullptr;
    if (a.kv_reverse && L.workspace != nullptr &&
        L.workspace_bytes >= kSchedBytes + far_bound_bytes(a.batch, a.heads_q, a.heads_kv, a.m, a.n)) {
        uint8_t* ws = static_cast<uint8_t*>(L.workspace) + kSchedBytes;
        const int64_t nq = static_cast<int64_t>(a.batch) * a.heads_q * a.n_qt;
        const int64_t nk = static_cast<int64_t>(a.batch) * a.heads_kv * a.n_kt;
        float* qn = reinterpret_cast<float*>(ws);
        float* kn = reinterpret_cast<float*>(ws + ((nq * 4 + 255) & ~int64_t{255}));
        int32_t* lo = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(kn) + ((nk * 4 + 255) & ~int64_t{255}));
        const NormSrc sq{static_cast<const __nv_bfloat16*>(L.q), L.q_strides[0], L.q_strides[1], L.q_strides[2],
                         a.heads_q, a.m, a.n_qt, nq, qn};
        const NormSrc sk{static_cast<const __nv_bfloat16*>(L.k), L.k_strides[0], L.k_strides[1], L.k_strides[2],
                         a.heads_kv, a.n, a.n_kt, nk, kn};
        tile_norm_kernel<<<static_cast<unsigned>(nq + nk), 128, 0, stream>>>(sq, sk);
        const int64_t n_lo = static_cast<int64_t>(a.batch) * a.heads_q * a.n_pairs;  // one warp each
        far_lo_kernel<<<static_cast<unsigned>((n_lo + 3) / 4), 128, 0, stream>>>(a, qn, kn, lo);
        if (cudaGetLastError() != cudaSuccess) {
            *err = "far-tile bound kernel launch failed";
            return ODF_ERR_CUDA;
        }
        a.kv_lo = lo;
    }
    int mod = (L.has_alibi ? kModAlibi : 0) | (L.has_softcap ? kModSoftcap : 0) | (L.has_bias ? kModBias : 0);
    // KV ranges of 16 or more tiles with a plain score: the variant whose unmasked tiles skip the
    // row-max pass (with the row-sum check, N = 4096 measured +2-5%, N = 2048 level; block-masked
    // problems, with few unmasked tiles per row, keep the general variant)
    if (mod == 0 && L.head_dim == 128 && a.mode != kModeList && a.n_kt >= 16) mod = kModSkipMax;
    // persistent grid: one CTA per SM (the kernel's shared memory allows one), at most one per item
    const int64_t n_items = static_cast<int64_t>(a.batch) * a.heads_q * a.n_pairs * a.n_splits;
    const dim3 grid(static_cast<unsigned>(n_items < sm_count ? n_items : sm_count), 1, 1);
    cudaError_t e = (L.head_dim == 64) ? launch_d<64>(tq, tk, tv, a, mod, grid, stream)
                                       : launch_d<128>(tq, tk, tv, a, mod, grid, stream);
    if (e == cudaSuccess && a.n_splits > 1) {
        const int64_t rows = n_bh * a.m;
        const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
        const float* po = static_cast<const float*>(a.o);
        if (L.head_dim == 64) {
            split_combine_kernel<64><<<blocks, 256, 0, stream>>>(po, a.lse, a.n_splits, a.o_split, a.lse_split, rows, a.m,
                                                                 a.heads_q, out_o, out_bf16, out_sb, out_sh, out_st,
                                                                 out_lse);
        } else {
            split_combine_kernel<128><<<blocks, 256, 0, stream>>>(po, a.lse, a.n_splits, a.o_split, a.lse_split, rows,
                                                                  a.m, a.heads_q, out_o, out_bf16, out_sb, out_sh,
                                                                  out_st, out_lse);
        }
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return ODF_ERR_CUDA;
    }
    return ODF_OK;
}

}  // namespace odf
