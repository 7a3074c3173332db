// FlashAttention-2 forward for B200 (sm_100a): TMA + mbarrier ring, tcgen05.mma into tensor
// memory, online base-2 softmax in warpgroups that own one TMEM lane (= one query row) per
// thread, TMA epilogue.
//
//   O = softmax(Q K^T * scale) V        Q, K, V, O: [B, H, N, D] fp16 (or bf16), D in {64, 128}
//
// It replaces the reference's mma.sync kernel (csrc/kernels/flash_fwd.cu:154-561) and its
// launcher (:563-652) behind the same parameters; the algorithm (FA2 online softmax with the
// scale folded into a base-2 exponent, causal tiles above the diagonal skipped, masking only
// on diagonal / ragged tiles, lazy rescaling for the "opt" variant, per-tile fp16 partials for
// "fp16acc") is the reference's, the machine mapping is new:
//
// Element types (FwdCfg's BF16 / FP8 flags, extensions of the reference): bf16 runs the same
// pipeline with bf16 operands; e4m3 (d = 128) reads Q and K as 128-byte rows, V transposed (a
// separate kernel writes V^T so that both MMAs read K-major operands), issues kind::f8f6f4 MMAs
// of K = 32 and stores P as e4m3, with fp32 scores and accumulators and a float16 O.
//
// Work item = one (b,h) head x NQ consecutive 128-row query tiles (NQ = 2; 1 for fp16acc, d = 128)
// x one key range (split-KV). Each CTA runs one item, or, for short rows (N <= 2048), a
// persistent grid of one CTA per SM walks the items: every role loops over the same items
// and the barrier phases run on across them, so an item's Q load and first S overlap the
// previous item's last tiles and epilogue. O leaves through a TMA store, staged in the tile's
// Q buffer (one item per CTA) or in a staging tile after the K/V ring that the query tiles
// take in turns (persistent grid).
// Warp roles (warp-specialised, one CTA per SM, whole warpgroups):
//   warpgroup t < NQ    softmax for query tile t; thread i of the warpgroup owns TMEM lane i
//                       = query row i of the tile, so row max and row sum need no shuffles.
//                       It also rescales O in TMEM when its running max moves, and runs the
//                       epilogue of its tile.
//   warpgroup NQ        warp 0: TMA producer (Q tiles once, then K_0, V_0, K_1, V_1, ...
//                       through a STAGES-deep ring of 128 x D tiles, 128-byte swizzle);
//                       warp 1: MMA issuer (one thread) and TMEM allocation; warp 2: the
//                       issuer of query tile 1 where tiles have their own issuers (d = 64);
//                       the remaining warps idle.
//   Tuning knobs (compile-time, defaults measured fastest on B200): the software-2^x share and
//   polynomial degree, the MMA issuer count, the d = 64 ring depth and the register split
//   between the softmax warpgroups and the producer/MMA warpgroup (setmaxnreg).
//
// Tensor memory (512 columns x 128 lanes, fp32 cells):
//   S_t  columns [128 t, 128 t + 128)   scores of tile t, fp32 (fp16acc at d = 128, NQ = 1: two
//        S buffers, columns [0, 128) and [128, 256), for alternate key tiles)
//   O_t  columns [128 NQ kSBufs + D t, +D)  fp32 output accumulator of tile t
//   P_t  (d = 128) columns [128 t, +64) over S_t once S_t has been read (e4m3 inputs: four P
//        values per column, [128 t, +32)): S_t(j+1) is issued after PV_t(j), and tcgen05.mma
//        operations of one thread execute in issue order;
//        (d = 64) its own columns [128 NQ + D NQ + 64 t, +64), so that S_t(j+1) can run while
//        the softmax of tile j is still computing P_t(j).
//   T_t  (fp16acc) the D columns after the O_t: fp16 partial of P.V over the current K/V tile,
//        one value per column; P_t lies over S_t as at d = 128.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>

#include "fa_internal.h"
#include "sm100_ptx.cuh"
#include "softmax_common.cuh"
#include "tma_host.h"

// Software-exp2 share (how many of every 8 column pairs of a 128-key tile take exp2_poly2
// instead of ex2.approx); compile-time tuning knobs.
#ifndef FA_EMU_PER8_D128
#define FA_EMU_PER8_D128 1
#endif
#ifndef FA_EMU_PER8_D64
#define FA_EMU_PER8_D64 2
#endif
#ifndef FA_EMU_PER8_FP8
#define FA_EMU_PER8_FP8 1  // e4m3 inputs (d = 128)
#endif
#ifndef FA_EMU_PER8_ACC16_D64
#define FA_EMU_PER8_ACC16_D64 1  // fp16acc at d = 64 (its fold adds FMA-pipe work): 1/8 measured fastest
#endif
// Register split between the softmax warpgroups and the producer/MMA warpgroup (NQ = 2):
// 0 keeps every warp at the launch allocation (168); otherwise softmax warps go to this many
// and the other warpgroup gives up the difference.
#ifndef FA_REGS_SOFTMAX
#define FA_REGS_SOFTMAX 184  // softmax warps' registers with two query tiles (setmaxnreg; 0 = none)
#endif
// Degree of the software 2^x polynomial per head dim (3: the reference's degree, 4: ours, 2.9e-6).
#ifndef FA_EXP_POLY_DEG_D128
#define FA_EXP_POLY_DEG_D128 3
#endif
#ifndef FA_EXP_POLY_DEG_D64
#define FA_EXP_POLY_DEG_D64 3
#endif
// MMA issuing threads per head dim (fp32 variants, NQ = 2): 2 gives each query tile its own
// issuer warp, so the tensor pipe can interleave the two tiles' P.V / S MMAs. Measured on
// B200: +5% at d = 64; at d = 128 the two tiles then fall into step (both softmaxes at once,
// then both tiles' MMAs) and lose a quarter, so d = 128 keeps the single issuer, whose issue
// order keeps the tiles alternating.
#ifndef FA_MMA_ISSUERS_D64
#define FA_MMA_ISSUERS_D64 2
#endif
#ifndef FA_MMA_ISSUERS_D128
#define FA_MMA_ISSUERS_D128 1
#endif
#ifndef FA_MMA_ISSUERS_ACC16
#define FA_MMA_ISSUERS_ACC16 1
#endif
// TMEM columns per tcgen05.ld of the softmax's S readout (32, 64 or 128): one 128-column load
// per tile measured +1% at d = 64 (fewer instructions through the sub-partition's MIO queue,
// which the MMA issuers share), neutral at d = 128.
#ifndef FA_S_LD_COLS
#define FA_S_LD_COLS 128
#endif
#ifndef FA_STAGES_D64
#define FA_STAGES_D64 8  // K/V ring slots at d = 64 (16 KB each)
#endif
#ifndef FA_REGS_SOFTMAX_D64
#define FA_REGS_SOFTMAX_D64 184  // d = 64: softmax warps' registers (setmaxnreg; 0 = none)
#endif

namespace fa_sm100 {

constexpr int kBM = 128;             // query rows per tile (= TMEM lanes = MMA M)
constexpr int kBN = 128;             // keys per K/V tile (= MMA N of Q K^T)
constexpr int kBoxBytes = 128 * 128; // one TMA box: 128 rows x 128 B (64 fp16 or 128 e4m3; one swizzle span)
constexpr int kPersistentMaxN = 2048; // persistent grid (one CTA per SM walks the items) up to this N
constexpr int kPersistentMaxNFull = 8192;  // ... and up to this N without the causal mask

template <int D_, bool CAUSAL_, int VARIANT_, bool BF16_ = false, bool FP8_ = false>
struct FwdCfg {
    static constexpr int D = D_;
    static constexpr bool CAUSAL = CAUSAL_;
    static constexpr int VARIANT = VARIANT_;
    // Element type of Q, K, V, O and of P (the P.V operand): bfloat16 when BF16, else float16.
    // The MMAs accumulate in fp32 either way; bf16 operands have no fp16 accumulator, so the
    // fp16acc variant is float16 only.
    static constexpr bool BF16 = BF16_;
    static_assert(!(BF16_ && VARIANT_ == kVariantFp16Acc), "fp16acc needs float16 operands");
    // e4m3 Q, K, V (per-tensor descales applied on the host side of the scores and in the
    // epilogue), P rounded to e4m3 in TMEM, kind::f8f6f4 MMAs with fp32 accumulation, fp16 O.
    // V arrives transposed ([B*H][D][N], keys contiguous), so that both MMAs read K-major
    // operands. d = 128 and the fp32-accumulating variants only.
    static constexpr bool FP8 = FP8_;
    static_assert(!FP8_ || (D_ == 128 && VARIANT_ != kVariantFp16Acc && !BF16_), "fp8: d = 128, fp32 accumulation");
    // fp16acc (reference ACC16, flash_fwd.cu:439-470): P.V of each 128-key tile accumulated in
    // fp16 into a fresh partial T_t, which the softmax folds into the fp32 O_t. Exact max (no
    // lazy rescale), so p <= 1. P is stored as p * 2^-kAccShift, which bounds |T_t| by
    // (128 >> kAccShift) * max|V|: the reference's per-tile bound (its tiles hold BC = 32 keys
    // at d = 64 and 64 at d = 128), so the partial overflows fp16 for no input the reference
    // accepts. O_t and the row sum carry the same power-of-two factor, which O / l cancels.
    static constexpr bool ACC16 = (VARIANT_ == kVariantFp16Acc);
    static constexpr int kAccShift = ACC16 ? (D == 64 ? 2 : 1) : 0;
    // Lazy rescale (reference LAZY, flash_fwd.cu:365-376): keep a stale row max until the
    // tile max exceeds it by more than 2^8. Threshold 0 = exact running max.
    // fp8: P is stored as p * 2^(8 - threshold) so that, with p <= 2^threshold under the lazy
    // rule, the stored value stays within e4m3's range (448) and small p keep more bits; the
    // lazy threshold is 4 there (p * 2^4 <= 256).
    static constexpr float kRescaleThreshold =
        (VARIANT_ == kVariantOpt) ? (FP8_ ? 4.0f : 8.0f) : 0.0f;
    static constexpr float kPLog2Scale = FP8_ ? 8.0f - kRescaleThreshold : 0.0f;
    // Query tiles per CTA. fp16acc at d = 128 needs S + O + T = 384 columns for one tile; it
    // spends the remaining 128 on a second S buffer (kSBufs): S(j+1) is computed while the
    // softmax works on tile j, and the fold of T(j) waits until the end of tile j+1, so no
    // tile waits for the previous tile's P.V.
    static constexpr int NQ = (ACC16 && D == 128) ? 1 : 2;
    static constexpr int kSBufs = (ACC16 && NQ == 1) ? 2 : 1;
    static constexpr bool SEP_P = !ACC16 && D == 64;
    static constexpr int kEmuPer8 =
        FP8 ? FA_EMU_PER8_FP8 : ((D == 128) ? FA_EMU_PER8_D128 : (ACC16 ? FA_EMU_PER8_ACC16_D64 : FA_EMU_PER8_D64));
    static constexpr int kPolyDeg = (D == 128) ? FA_EXP_POLY_DEG_D128 : FA_EXP_POLY_DEG_D64;
    static constexpr int kElemBytes = FP8 ? 1 : 2;
    static constexpr int kTileBytes = kBM * D * kElemBytes;  // one Q, K or V tile (BM == BN)
    static constexpr int kOutTileBytes = kBM * D * 2;        // one O tile (fp16 / bf16)
    // A Q buffer also stages its tile's O for the TMA store.
    static constexpr int kQTileBytes = kTileBytes > kOutTileBytes ? kTileBytes : kOutTileBytes;
    static constexpr int kBoxes = D * kElemBytes / 128;       // TMA boxes per Q, K or V tile
    static constexpr int kBoxElems = 128 / kElemBytes;        // elements per box row
    static constexpr int kOutBoxes = D / 64;                  // TMA boxes per O tile
    static constexpr int kKSteps = D * kElemBytes / 32;       // MMA K steps of Q K^T (32 B each)
    static constexpr int kPvSteps = kBN * kElemBytes / 32;    // MMA K steps of P V
    static constexpr int STAGES = FP8 ? 8 : ((D == 128) ? 4 : FA_STAGES_D64);
    static_assert(STAGES <= 16, "K/V ring barriers");
    // Shared memory (offsets from a 1024-byte aligned base).
    static constexpr int kSmemQ = 0;
    static constexpr int kSmemKV = NQ * kQTileBytes;
    // O staging tile of the persistent grid's epilogue (the Q buffers hold the next item's Q).
    static constexpr int kSmemStage = kSmemKV + STAGES * kTileBytes;
    static constexpr int kSmemBytes = kSmemStage + kOutTileBytes;
    static constexpr int kSmemAlloc = kSmemBytes + 1024;
    // Tensor memory columns.
    static constexpr int kTmemS = 0;
    static constexpr int kTmemO = NQ * kSBufs * kBN;
    static constexpr int kTmemExtra = kTmemO + NQ * D;  // P_t (SEP_P) or T_t (ACC16)
    static constexpr int kTmemUsed = kTmemExtra + (ACC16 ? NQ * D : (SEP_P ? NQ * 64 : 0));
    // fp16acc partial of tile t (fp16 cells, one value per column).
    static constexpr int tmem_t(int t) { return kTmemExtra + D * t; }
    static constexpr int kTmemCols = 512;
    static_assert(kTmemUsed <= kTmemCols, "tensor memory budget");
    // Warps: NQ softmax warpgroups + one producer/MMA warpgroup.
    static constexpr int kSoftmaxWarps = 4 * NQ;
    static constexpr int kIssuers =  // MMA issuer warps kMmaWarp and kIssuerWarp1
        (NQ == 2 && (ACC16 ? FA_MMA_ISSUERS_ACC16 : (D == 64 ? FA_MMA_ISSUERS_D64 : FA_MMA_ISSUERS_D128)) == 2)
            ? 2
            : 1;
    static constexpr int kProducerWarp = kSoftmaxWarps;
    static constexpr int kMmaWarp = kSoftmaxWarps + 1;
    static constexpr int kIssuerWarp1 = kMmaWarp + 1;
    static constexpr int kThreads = 32 * (kSoftmaxWarps + 4);
    // Register split: every warp is launched with kRegsLaunch (65536 / threads, a multiple of
    // 8); with FA_REGS_SOFTMAX != 0 the softmax warpgroups go to that many and the
    // producer/MMA warpgroup gives up the difference.
    static constexpr int kRegsLaunch = ((65536 / kThreads) / 8 * 8) > 255 ? 248 : (65536 / kThreads) / 8 * 8;
    // fp16acc at d = 64 (exponentials, then the fold of its fp16 partial) takes 200.
    static constexpr int kRegsSoftmax = (D == 64) ? (ACC16 ? 200 : FA_REGS_SOFTMAX_D64) : FA_REGS_SOFTMAX;
    static constexpr int kRegsOther =
        kRegsSoftmax == 0
            ? kRegsLaunch
            : ((kThreads * kRegsLaunch - 32 * kSoftmaxWarps * kRegsSoftmax) / 128) / 8 * 8;
    static_assert(kRegsSoftmax == 0 || NQ != 2 ||
                      (32 * kSoftmaxWarps * kRegsSoftmax + 128 * kRegsOther <= kThreads * kRegsLaunch &&
                       kRegsOther >= 24 && kRegsSoftmax % 8 == 0 && kRegsSoftmax <= 256),
                  "register split exceeds the launch allocation");
    static_assert(D == 64 || D == 128, "head dim");
    static_assert(kSmemAlloc <= 227 * 1024, "shared memory budget");
    static_assert(kSmemAlloc > 114 * 1024, "one CTA per SM (it owns all 512 TMEM columns)");
};

constexpr int kMaxStages = 16;
struct SharedBarriers {
    uint64_t q_full[2];
    uint64_t kv_full[kMaxStages];
    uint64_t kv_empty[kMaxStages];
    uint64_t s_full[2];
    uint64_t s_free[2];
    uint64_t p_full[2];
    uint64_t o_done[2];
    uint64_t q_empty[2];
    uint64_t epi[2];
    uint64_t stg_free;  // persistent grid: the staging tile's turns, tile 0 then tile 1 per item
    uint64_t mma_idle;
    uint32_t tmem_base;
    int abort;
};

// fp16 accumulator cells hold one value per 32-bit column, in the low half.
__device__ __forceinline__ float f16cell_to_float(uint32_t cell) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(cell & 0xFFFFu)));
}

// MMA issue helpers. The issuing thread shares its SM sub-partition with busy softmax warps,
// so descriptors are derived from precomputed bases with one add each (a descriptor's start
// address is its low 14 bits in 16-byte units; shared memory stays below 256 KB, so adding an
// offset never carries out of the field). `qd` / `kd` / `vd` = the descriptor of the Q / K / V
// tile's first byte.
template <class Cfg>
__device__ __forceinline__ void issue_s_mma(uint32_t tmem_s, uint64_t qd, uint64_t kd) {
    // kind::f8f6f4 with e4m3 A and B (format code 0) has the bit layout of kind::f16 with f16.
    constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, /*d_f32=*/true, /*b_mn_major=*/false, Cfg::BF16);
#pragma unroll
    for (int kk = 0; kk < Cfg::kKSteps; ++kk) {
        const uint64_t off = static_cast<uint64_t>(((kk / 4) * kBoxBytes + (kk % 4) * 32) >> 4);
        if constexpr (Cfg::FP8) {
            umma_ss_f8(tmem_s, qd + off, kd + off, idesc, kk > 0 ? 1u : 0u);
        } else {
            umma_ss(tmem_s, qd + off, kd + off, idesc, kk > 0 ? 1u : 0u);
        }
    }
}

// O (fp32) += P V over the 128 keys of one tile; `first` starts the accumulator.
template <class Cfg>
__device__ __forceinline__ void issue_pv_mma_f32(uint32_t tmem_o, uint32_t tmem_p, uint64_t vd,
                                                 bool first) {
    if constexpr (Cfg::FP8) {
        // fp8: V^T tile K-major (keys contiguous, like a K tile), P four e4m3 per column.
        constexpr uint32_t idesc8 = make_idesc_f16(kBM, Cfg::D, /*d_f32=*/true, /*b_mn_major=*/false);
#pragma unroll
        for (int kk = 0; kk < Cfg::kPvSteps; ++kk) {
            umma_ts_f8(tmem_o, tmem_p + kk * 8, vd + static_cast<uint64_t>((kk * 32) >> 4), idesc8,
                       (first && kk == 0) ? 0u : 1u);
        }
        return;
    }
    constexpr uint32_t idesc = make_idesc_f16(kBM, Cfg::D, /*d_f32=*/true, /*b_mn_major=*/true, Cfg::BF16);
#pragma unroll
    for (int kk = 0; kk < kBN / 16; ++kk) {
        umma_ts(tmem_o, tmem_p + kk * 8, vd + static_cast<uint64_t>(kk * (2048 >> 4)), idesc,
                (first && kk == 0) ? 0u : 1u);
    }
}

// fp16acc: T = P V over the 128 keys of one tile, accumulated in fp16, fresh per tile.
template <class Cfg>
__device__ __forceinline__ void issue_pv_mma_f16(uint32_t tmem_t, uint32_t tmem_p, uint64_t vd) {
    constexpr uint32_t idesc = make_idesc_f16(kBM, Cfg::D, /*d_f32=*/false, /*b_mn_major=*/true);
#pragma unroll
    for (int kk = 0; kk < kBN / 16; ++kk) {
        umma_ts(tmem_t, tmem_p + kk * 8, vd + static_cast<uint64_t>(kk * (2048 >> 4)), idesc,
                kk == 0 ? 0u : 1u);
    }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_o, const FwdArgs args) {
    constexpr int D = Cfg::D;
    constexpr int NQ = Cfg::NQ;
    constexpr int STAGES = Cfg::STAGES;

    extern __shared__ uint8_t smem_raw[];
    __shared__ SharedBarriers sb;

    const int warp = static_cast<int>(threadIdx.x) / 32;
    const int lane = static_cast<int>(threadIdx.x) % 32;

    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t smem_base = smem_u32(smem);

    // Work items: (row block, head, key range). A CTA takes items blockIdx.x, then, round by
    // round, one item of every run of gridDim.x consecutive items, in serpentine order (so that
    // under the causal schedule's longest-first order each CTA gets a long and a short item in
    // alternate rounds). With gridDim.x == num_items each CTA runs one item.
    const int n = args.seqlen;
    const int nb = (n + NQ * kBM - 1) / (NQ * kBM);  // row blocks per head
    const int per_split = nb * args.num_bh;           // items per key range
    const int grid_n = static_cast<int>(gridDim.x);
    const int cta = static_cast<int>(blockIdx.x);
    auto item_index = [&](int r) -> int {
        const long long idx = static_cast<long long>(r) * grid_n + ((r & 1) ? (grid_n - 1 - cta) : cta);
        return idx < static_cast<long long>(args.num_items) ? static_cast<int>(idx) : -1;
    };
    struct Item {
        int bh;
        int q_row0;
        int kv0;       // first key tile of the item's key range
        int n_kv[NQ];  // key tiles query tile t processes, from kv0
        int n_max;
        bool split;    // the rows' partials go to split records (merged by the combine kernel)
        long long rec0;  // split record of the item's first row (row 0 of query tile 0)
    };
    auto decode = [&](int idx, Item& it) {
        // Row block `lin` in item order, key range z of `nsplit`, and its split records.
        int lin, z, nsplit, p = 0;
        if (idx >= args.tail_from) {
            // Tail split: the last tail_blocks row blocks, tail_splits consecutive items each.
            const int j = idx - args.tail_from;
            p = args.div_tail.div(j);
            z = j - p * args.tail_splits;
            lin = args.tail_from + p;
            nsplit = args.tail_splits;
        } else {
            z = args.div_per_split.div(idx);
            lin = idx - z * per_split;
            nsplit = args.num_splits;
        }
        int m_block;
        if constexpr (Cfg::CAUSAL) {
            // A causal row block covers more key tiles the later its rows are. Items run in
            // index order, so the index is mapped to (row block, head) longest first across a
            // group of args.head_group heads (whose K/V stay resident in L2 together): the short
            // blocks of every group then fill the gaps the long ones leave, instead of a head's
            // long block starting last and running alone.
            const int group = args.div_group_items.div(lin);
            const int head0 = group * args.head_group;
            const int within = lin - group * nb * args.head_group;
            const bool last = args.num_bh - head0 < args.head_group;
            const int heads = last ? args.num_bh - head0 : args.head_group;
            const int rank = last ? args.div_last_group.div(within) : args.div_group.div(within);
            it.bh = head0 + within - rank * heads;
            m_block = nb - 1 - rank;
        } else {
            it.bh = args.div_nb.div(lin);
            m_block = lin - it.bh * nb;
        }
        it.q_row0 = m_block * NQ * kBM;
        const int n_tiles_all = (n + kBN - 1) / kBN;
        it.n_max = 0;
#pragma unroll
        for (int t = 0; t < NQ; ++t) {
            const int q0 = it.q_row0 + t * kBM;
            it.n_kv[t] = (q0 >= n) ? 0 : (Cfg::CAUSAL ? (q0 / kBN + 1) : n_tiles_all);
            it.n_max = max(it.n_max, it.n_kv[t]);
        }
        it.kv0 = 0;
        it.split = nsplit > 1;
        it.rec0 = 0;
        if (it.split) {
            // The block's key tiles [0, n_max) in nsplit contiguous ranges; range z here.
            const int per = (it.n_max + nsplit - 1) / nsplit;
            it.kv0 = z * per;
#pragma unroll
            for (int t = 0; t < NQ; ++t) {
                it.n_kv[t] = max(0, min(it.n_kv[t] - it.kv0, per));
            }
            it.n_max = max(0, min(it.n_max - it.kv0, per));
            // Split records: [num_splits][num_bh][rows_pad] (split-KV) or
            // [tail_splits][tail_blocks][NQ * 128] (tail split).
            it.rec0 = idx >= args.tail_from
                          ? (static_cast<long long>(z) * args.tail_blocks + p) * (NQ * kBM)
                          : (static_cast<long long>(z) * args.num_bh + it.bh) * args.rows_pad + it.q_row0;
        }
    };

    const WaitCtx wctx{&sb.abort, &args.status->code, &args.status->epoch_aborted, args.epoch};
    // O leaves through the Q buffer and a TMA store when each CTA runs one item (the buffer is
    // free once the item's last S MMA has completed); a persistent CTA reloads Q for its next
    // item meanwhile, so there each thread stores its row directly.
    const bool tma_store_o = grid_n >= args.num_items;

    if (threadIdx.x == 0) {
        sb.abort = 0;
        for (int t = 0; t < NQ; ++t) {
            mbar_init(smem_u32(&sb.q_full[t]), 1);
            mbar_init(smem_u32(&sb.q_empty[t]), 1);
            mbar_init(smem_u32(&sb.s_full[t]), 1);
            // Softmax-side barriers take one arrival per warp (after __syncwarp), not one per
            // thread: 128 arrivals on one barrier word serialise in the shared-memory atomics.
            mbar_init(smem_u32(&sb.s_free[t]), 4);
            mbar_init(smem_u32(&sb.p_full[t]), 4);
            if (Cfg::kSBufs == 2) {
                mbar_init(smem_u32(&sb.s_full[1]), 1);  // second S buffer (NQ = 1)
            }
            mbar_init(smem_u32(&sb.o_done[t]), 1);
            mbar_init(smem_u32(&sb.epi[t]), 4);
        }
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&sb.kv_full[s]), 1);
            mbar_init(smem_u32(&sb.kv_empty[s]), Cfg::kIssuers);
        }
        mbar_init(smem_u32(&sb.mma_idle), Cfg::kIssuers);
        mbar_init(smem_u32(&sb.stg_free), 1);
        mbar_fence_init();
    }
    if (warp == Cfg::kMmaWarp) {
        tmem_alloc(smem_u32(&sb.tmem_base), Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == Cfg::kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        if (tma_store_o) {
            tma_prefetch_desc(&tm_o);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sb.tmem_base;

    if constexpr (NQ == 2 && Cfg::kRegsSoftmax != 0) {
        if (warp < Cfg::kSoftmaxWarps) {
            asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Cfg::kRegsSoftmax));
        } else {
            asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::kRegsOther));
        }
    }

    // Barrier phases run on across items: every per-tile barrier completes once per S, P or P.V
    // of its tile, so the waits take their parity from running counts kept by each role.
    if (warp < Cfg::kSoftmaxWarps) {
        // ================================ softmax warpgroups ================================
        constexpr int NC = kBN;                         // S columns of this thread
        const int t = warp / 4;                         // query tile
        const int row = (warp % 4) * 32 + lane;         // TMEM lane == query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>((warp % 4) * 32) << 16;
        const uint32_t t_s = tmem + lane_off + Cfg::kTmemS + t * kBN;
        const uint32_t t_o = tmem + lane_off + Cfg::kTmemO + t * D;
        const uint32_t t_p = Cfg::SEP_P ? (tmem + lane_off + Cfg::kTmemExtra + t * 64)
                                        : (tmem + lane_off + Cfg::kTmemS + t * kBN);
        const uint32_t t_t = tmem + lane_off + Cfg::tmem_t(t);
        const uint32_t bar_s = smem_u32(&sb.s_full[t]);
        const uint32_t bar_sf = smem_u32(&sb.s_free[t]);
        const uint32_t bar_p = smem_u32(&sb.p_full[t]);
        const uint32_t bar_o = smem_u32(&sb.o_done[t]);
        const float scale_log2 = args.scale_log2;
        // With P in its own columns the wait for the previous P.V is deferred to the first P
        // store, so the exponentials of the first chunk overlap that P.V.
        constexpr bool kLateWait = Cfg::SEP_P;
        // fp16acc: O_t = a * O_t + T_t (or O_t = T_t for a tile's first key tile), one
        // 32-column chunk at a time (two 32-register loads in flight).
        auto fold_t = [&](float a, bool first) {
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t tv[32];
                uint32_t o[32];
                tmem_ld32(t_t + c * 32, tv);
                if (!first) {
                    tmem_ld32(t_o + c * 32, o);
                }
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float v = f16cell_to_float(tv[e]);
                    o[e] = f2u(first ? v : fmaf(u2f(o[e]), a, v));
                }
                tmem_st32(t_o + c * 32, o);
            }
            tmem_wait_st();
        };

        int g0 = 0;  // S / P / P.V count of this tile before the current item
        int stg_items = 0;  // persistent grid: items whose epilogue took a staging turn
        bool ok = true;

        // A warp that gave up on a wait keeps walking its items and key tiles without touching
        // TMEM (every later wait returns at once), so that all roles leave their loops.
        for (int r = 0;; ++r) {
            const int idx = item_index(r);
            if (idx < 0) {
                break;
            }
            // Only what the key-tile loop needs stays live through it; the epilogue decodes the
            // item again for its head and key range.
            int q0, nt, kv0;
            {
                Item it;
                decode(idx, it);
                q0 = it.q_row0 + t * kBM;
                nt = (t == 0) ? it.n_kv[0] : it.n_kv[NQ - 1];  // a select keeps `it` in registers
                kv0 = it.kv0;
            }
            const int grow = q0 + row;  // global query row
            // Last key index this row may see: keys > lim are masked (ragged N, causal).
            const int lim = Cfg::CAUSAL ? min(n - 1, grow) : (n - 1);

            float row_max = -INFINITY;  // running max of the scaled scores (log2 units)
            float row_sum = 0.0f;       // running sum of this thread's fp16-rounded probabilities
            float alpha_prev = 1.0f;    // two S buffers: the rescale of the fold still pending

            for (int j = 0; j < nt; ++j) {
                const int gj = g0 + j;  // running index of S_t(j), P_t(j) and P.V_t(j)
                // Two S buffers (kSBufs): S(j) in buffer gj & 1, whose barrier completes every
                // other S.
                const uint32_t s_off = (Cfg::kSBufs == 2) ? static_cast<uint32_t>((gj & 1) * kBN) : 0u;
                ok = ok && __all_sync(0xffffffffu,
                                      (Cfg::kSBufs == 2)
                                          ? mbar_wait(smem_u32(&sb.s_full[gj & 1]), (gj >> 1) & 1, wctx,
                                                      kStatusTimeoutSoftmax)
                                          : mbar_wait(bar_s, gj & 1, wctx, kStatusTimeoutSoftmax));
                if (!ok) {
                    continue;
                }
                tc_fence_after();
                uint32_t sr[NC];
                if constexpr (FA_S_LD_COLS == 128) {
                    tmem_ld128(t_s + s_off, sr);
                } else {
#pragma unroll
                    for (int c = 0; c < NC / FA_S_LD_COLS; ++c) {
                        if constexpr (FA_S_LD_COLS == 64) {
                            tmem_ld64(t_s + s_off + c * 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[c * 64]));
                        } else {
                            tmem_ld32(t_s + s_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
                        }
                    }
                }
                tmem_wait_ld();
                if constexpr (Cfg::SEP_P) {
                    // S_t is in registers: the MMA warp may overwrite it with the next S_t.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(bar_sf);
                    }
                }

                const int kbase = (kv0 + j) * kBN;
                // Only the last key tile can hold keys >= N, and for causal rows only the
                // diagonal tile (key tile q0 / 128) holds keys after the row: every other tile
                // is unmasked.
                const bool masked = (kbase + kBN > n) || (Cfg::CAUSAL && kbase == q0);
                float tile_max;
                float mul;
                if (masked) {
                    // Scale first, then mask, so masked scores are -inf whatever the scale's sign.
                    const int cmax = lim - kbase;
#pragma unroll
                    for (int c = 0; c < NC; ++c) {
                        sr[c] = f2u((c > cmax) ? -INFINITY : u2f(sr[c]) * scale_log2);
                    }
                    tile_max = row_extreme<true, NC>(sr);
                    mul = 1.0f;
                } else {
                    // max(s * scale) is max(s) * scale, or min(s) * scale for a negative scale.
                    tile_max = (scale_log2 >= 0.0f ? row_extreme<true, NC>(sr)
                                                   : row_extreme<false, NC>(sr)) *
                               scale_log2;
                    mul = scale_log2;
                }
                // Running max update (lazy for "opt": keep the old max unless it grew by > 2^8).
                const float new_max = (tile_max > row_max + Cfg::kRescaleThreshold) ? tile_max : row_max;
                const float max_used = (new_max == -INFINITY) ? 0.0f : new_max;
                const bool grew = (new_max != row_max);
                const float alpha = grew ? ex2_approx(row_max - max_used) : 1.0f;  // 0 on tile 0
                row_max = new_max;

                // P_t(j-1) (d = 64: in its own columns) must have been consumed before P_t(j) is
                // written; O must hold P.V up to tile j-1 before it is rescaled.
                const bool need_rescale = (!Cfg::ACC16) && j > 0 && (__any_sync(0xffffffffu, grew) != 0);
                if (!kLateWait && ((Cfg::SEP_P && j > 0) || need_rescale)) {
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(bar_o, (gj - 1) & 1, wctx, kStatusTimeoutSoftmax));
                    if (!ok) {
                        continue;
                    }
                    tc_fence_after();
                }

                // Probabilities, packed fp16 pairs, into P_t.
                const float2 mul2 = make_float2(mul, mul);
                // fp16acc stores p * 2^-kAccShift, fp8 p * 2^kPLog2Scale: the shift joins the max
                // in the exponent.
                const float neg = Cfg::FP8 ? Cfg::kPLog2Scale - max_used
                                           : ((Cfg::kAccShift != 0) ? -max_used - static_cast<float>(Cfg::kAccShift)
                                                                    : -max_used);
                const float2 neg2 = make_float2(neg, neg);
                float2 sum2[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    sum2[i] = make_float2(0.0f, 0.0f);
                }
#pragma unroll
                for (int chunk = 0; chunk < NC / 64 && Cfg::FP8; ++chunk) {
                    // fp8: the 64 keys of the chunk become 16 columns of four e4m3 each (key
                    // 4w + b in byte b of column w); the row sum adds the rounded values.
                    uint32_t pk8[16];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int c = chunk * 64 + 2 * i;
                        const float2 x2 = __ffma2_rn(make_float2(u2f(sr[c]), u2f(sr[c + 1])), mul2, neg2);
                        const float2 e = ((i % 8) < Cfg::kEmuPer8)
                                             ? (Cfg::kPolyDeg == 3 ? exp2_poly2_deg3(x2) : exp2_poly2(x2))
                                             : make_float2(ex2_approx(x2.x), ex2_approx(x2.y));
                        const uint32_t b = pack_e4m3x2(e.x, e.y);
                        pk8[i / 2] = (i & 1) ? (pk8[i / 2] | (b << 16)) : b;
                        add_x2_to_f32<false>(sum2[i % 4].x, sum2[i % 4].y, e4m3x2_to_half2(b));
                    }
                    tmem_st16(t_p + s_off + chunk * 16, pk8);
                }
#pragma unroll
                for (int chunk = 0; chunk < NC / 64 && !Cfg::FP8; ++chunk) {
                    uint32_t pk[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int c = chunk * 64 + 2 * i;
                        const float2 x2 = __ffma2_rn(make_float2(u2f(sr[c]), u2f(sr[c + 1])), mul2, neg2);
                        const float2 e = ((i % 8) < Cfg::kEmuPer8)
                                             ? (Cfg::kPolyDeg == 3 ? exp2_poly2_deg3(x2) : exp2_poly2(x2))
                                             : make_float2(ex2_approx(x2.x), ex2_approx(x2.y));
                        const uint32_t h = pack2<Cfg::BF16>(e.x, e.y);
                        // The row sum adds the fp16-rounded values the MMA consumes, so that O
                        // is normalised by the weights it was accumulated with. (The reference
                        // sums the fp32 values, csrc/kernels/flash_fwd.cu:403-417; measured here
                        // that adds error: cfg4's outlier rows exceed 2e-3.)
                        // fp32 += fp16 with the mixed-precision add (no separate conversion).
                        add_x2_to_f32<Cfg::BF16>(sum2[i % 4].x, sum2[i % 4].y, h);
                        pk[i] = h;
                    }
                    if (kLateWait && chunk == 0 && j > 0) {
                        // P_t(j-1) consumed and O up to date (needed by the rescale below too).
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait(bar_o, (gj - 1) & 1, wctx, kStatusTimeoutSoftmax));
                        if (ok) {
                            tc_fence_after();
                        }
                    }
                    if (ok) {
                        tmem_st32(t_p + s_off + chunk * 32, pk);
                    }
                }
                if (!ok) {
                    continue;
                }
                const float2 s01 = __fadd2_rn(sum2[0], sum2[1]);
                const float2 s23 = __fadd2_rn(sum2[2], sum2[3]);
                const float2 s4 = __fadd2_rn(s01, s23);
                row_sum = fmaf(row_sum, alpha, s4.x + s4.y);

                if constexpr (!Cfg::ACC16) {
                    if (need_rescale) {
                        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
                        for (int c = 0; c < D / 32; ++c) {
                            uint32_t o[32];
                            tmem_ld32(t_o + c * 32, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; e += 2) {
                                const float2 v = __fmul2_rn(make_float2(u2f(o[e]), u2f(o[e + 1])), a2);
                                o[e] = f2u(v.x);
                                o[e + 1] = f2u(v.y);
                            }
                            tmem_st32(t_o + c * 32, o);
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(bar_p);
                    }
                } else if constexpr (Cfg::kSBufs == 2) {
                    // Fold the previous tile's partial now, while S(j+1) is ready in the other
                    // buffer: P.V(j) overwrites T only after this tile's P arrival below.
                    if (j > 0) {
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait(bar_o, (gj - 1) & 1, wctx, kStatusTimeoutSoftmax));
                        if (!ok) {
                            continue;
                        }
                        tc_fence_after();
                        fold_t(alpha_prev, j == 1);
                    }
                    alpha_prev = alpha;
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(bar_p);
                    }
                } else {
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(bar_p);
                    }
                    // Fold this tile's fp16 partial into the fp32 accumulator: O = alpha * O + T.
                    // T lies in its own columns, so the next S_t (issued right after this P.V)
                    // runs meanwhile; the next P.V overwrites T only after this warp's next P
                    // arrival, which follows the fold.
                    ok = __all_sync(0xffffffffu, mbar_wait(bar_o, gj & 1, wctx, kStatusTimeoutSoftmax));
                    if (!ok) {
                        continue;
                    }
                    tc_fence_after();
                    fold_t(alpha, j == 0);
                }
            }
            if constexpr (Cfg::kSBufs == 2) {
                // The last tile's partial.
                if (ok && nt > 0) {
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(bar_o, (g0 + nt - 1) & 1, wctx, kStatusTimeoutSoftmax));
                    if (ok) {
                        tc_fence_after();
                        fold_t(alpha_prev, nt == 1);
                    }
                }
            }

            // --------------------------------- epilogue ---------------------------------
            // O_t is read out of TMEM here, before this warp's next P arrival: the MMA warp
            // overwrites O_t (next item's first P.V) only after that arrival.
            if (ok && nt > 0) {
                if constexpr (!Cfg::ACC16) {
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(bar_o, (g0 + nt - 1) & 1, wctx, kStatusTimeoutSoftmax));
                    tc_fence_after();
                }
            }
            Item it;
            decode(idx, it);
            if (it.split) {
                // Split-KV: the row's unnormalised O over this item's key range and its (m, l) go
                // to the workspace; a range with no keys for this tile records l = 0, which the
                // combine skips. Every record of a row that exists (q0 < N) is written, so the
                // workspace needs no initialisation.
                if (q0 < n && (ok || nt == 0)) {
                    const size_t rec = static_cast<size_t>(it.rec0 + t * kBM + row);
                    float4* dst = reinterpret_cast<float4*>(args.ws_o + rec * D);
                    if (nt > 0) {
#pragma unroll
                        for (int c = 0; c < D / 32; ++c) {
                            uint32_t o[32];
                            tmem_ld32(t_o + c * 32, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                dst[c * 8 + i] = make_float4(u2f(o[4 * i]), u2f(o[4 * i + 1]),
                                                             u2f(o[4 * i + 2]), u2f(o[4 * i + 3]));
                            }
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < D / 4; ++i) {
                            dst[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        }
                    }
                    reinterpret_cast<float2*>(args.ws_ml)[rec] =
                        make_float2(nt > 0 ? row_max : -INFINITY, nt > 0 ? row_sum : 0.0f);
                }
            } else if (tma_store_o && ok && nt > 0) {
                float inv_sum = (row_sum > 0.0f) ? (1.0f / row_sum) : 0.0f;
                if constexpr (Cfg::FP8) {
                    inv_sum *= args.out_scale;  // V's descale
                }
                // Stage O (fp16) in this tile's Q buffer, in the swizzled layout of the TMA box.
                // Every MMA that read Q_t has completed (its S was consumed above).
                uint8_t* out = smem + Cfg::kSmemQ + t * Cfg::kQTileBytes;
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(t_o + c * 32, o);
                    tmem_wait_ld();
                    uint32_t h[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        h[e] = pack2<Cfg::BF16>(u2f(o[2 * e]) * inv_sum, u2f(o[2 * e + 1]) * inv_sum);
                    }
                    const int col = c * 32;  // first O column of this chunk
                    const int box = col / 64;
                    const int chunk0 = (col % 64) / 8;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int cc = chunk0 + i;
                        uint4* dst = reinterpret_cast<uint4*>(out + box * kBoxBytes + row * 128 +
                                                              ((cc ^ (row & 7)) << 4));
                        *dst = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(&sb.epi[t]));
                }
                if (row == 0) {
                    if (mbar_wait(smem_u32(&sb.epi[t]), 0, wctx, kStatusTimeoutEpilogue)) {
#pragma unroll
                        for (int b = 0; b < Cfg::kOutBoxes; ++b) {
                            tma_store_3d(&tm_o, smem_u32(out) + b * kBoxBytes, b * 64, q0, it.bh);
                        }
                        tma_store_commit();
                        tma_store_wait_read();
                    }
                }
                __syncwarp();
            } else if (!tma_store_o) {
                // Persistent grid (the Q buffers already hold the next item's Q): O goes through
                // the staging tile, which the query tiles take in turns, tile 0 then tile 1 of
                // each item; the turn passes once the TMA store has read the tile. A tile with
                // nothing to store still takes and passes its turn.
                const int use = NQ * stg_items + t;
                bool turn = ok;
                if (turn && use > 0) {
                    turn = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sb.stg_free), (use - 1) & 1, wctx,
                                                             kStatusTimeoutEpilogue));
                }
                uint8_t* out = smem + Cfg::kSmemStage;
                if (turn && nt > 0) {
                    float inv_sum = (row_sum > 0.0f) ? (1.0f / row_sum) : 0.0f;
                    if constexpr (Cfg::FP8) {
                        inv_sum *= args.out_scale;
                    }
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(t_o + c * 32, o);
                        tmem_wait_ld();
                        uint32_t h[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            h[e] = pack2<Cfg::BF16>(u2f(o[2 * e]) * inv_sum, u2f(o[2 * e + 1]) * inv_sum);
                        }
                        const int col = c * 32;
                        const int box = col / 64;
                        const int chunk0 = (col % 64) / 8;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int cc = chunk0 + i;
                            uint4* dst = reinterpret_cast<uint4*>(out + box * kBoxBytes + row * 128 +
                                                                  ((cc ^ (row & 7)) << 4));
                            *dst = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
                        }
                    }
                    fence_proxy_async_smem();
                }
                __syncwarp();
                if (ok && lane == 0) {
                    mbar_arrive(smem_u32(&sb.epi[t]));
                }
                if (ok && row == 0) {
                    // The store clips rows >= N (the tensor map's bound).
                    if (mbar_wait(smem_u32(&sb.epi[t]), stg_items & 1, wctx, kStatusTimeoutEpilogue) && turn &&
                        nt > 0) {
#pragma unroll
                        for (int b = 0; b < Cfg::kOutBoxes; ++b) {
                            tma_store_3d(&tm_o, smem_u32(out) + b * kBoxBytes, b * 64, q0, it.bh);
                        }
                        tma_store_commit();
                        tma_store_wait_read();
                    }
                    mbar_arrive(smem_u32(&sb.stg_free));
                }
                __syncwarp();
                ++stg_items;
            }
            g0 += nt;
        }
    } else if (warp == Cfg::kProducerWarp) {
        // ================================== TMA producer ===================================
        if (lane == 0) {
            int last_parity[STAGES];
            bool loaded[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) {
                loaded[s] = false;
                last_parity[s] = 0;
            }
            int q_loads[NQ];  // Q_t loads so far
#pragma unroll
            for (int t = 0; t < NQ; ++t) {
                q_loads[t] = 0;
            }
            bool ok = true;
            int ring = 0;
            for (int r = 0; ok; ++r) {
                const int idx = item_index(r);
                if (idx < 0) {
                    break;
                }
                Item it;
                decode(idx, it);
#pragma unroll
                for (int t = 0; t < NQ; ++t) {
                    if (ok && it.n_kv[t] > 0) {
                        // Q_t is free once the previous item's last S_t MMA has completed.
                        if (q_loads[t] > 0) {
                            ok = mbar_wait(smem_u32(&sb.q_empty[t]), (q_loads[t] - 1) & 1, wctx,
                                           kStatusTimeoutProducer);
                        }
                        if (ok) {
                            const uint32_t bar = smem_u32(&sb.q_full[t]);
                            mbar_arrive_expect_tx(bar, Cfg::kTileBytes);
#pragma unroll
                            for (int b = 0; b < Cfg::kBoxes; ++b) {
                                tma_load_3d(smem_base + Cfg::kSmemQ + t * Cfg::kQTileBytes + b * kBoxBytes,
                                            &tm_q, bar, b * Cfg::kBoxElems, it.q_row0 + t * kBM, it.bh);
                            }
                            ++q_loads[t];
                        }
                    }
                }
                for (int j = 0; j < it.n_max && ok; ++j) {
#pragma unroll
                    for (int kind = 0; kind < 2; ++kind) {
                        const int stage = ring % STAGES;
                        const int phase = (ring / STAGES) & 1;
                        if (!mbar_wait(smem_u32(&sb.kv_empty[stage]), phase ^ 1, wctx,
                                       kStatusTimeoutProducer)) {
                            ok = false;
                            break;
                        }
                        const uint32_t bar = smem_u32(&sb.kv_full[stage]);
                        mbar_arrive_expect_tx(bar, Cfg::kTileBytes);
                        const CUtensorMap* map = (kind == 0) ? &tm_k : &tm_v;
                        if (Cfg::FP8 && kind == 1) {
                            // V^T: [B*H][D][keys], one box of 128 keys x D rows.
                            tma_load_3d(smem_base + Cfg::kSmemKV + stage * Cfg::kTileBytes, map, bar,
                                        (it.kv0 + j) * kBN, 0, it.bh);
                        } else {
#pragma unroll
                            for (int b = 0; b < Cfg::kBoxes; ++b) {
                                tma_load_3d(smem_base + Cfg::kSmemKV + stage * Cfg::kTileBytes + b * kBoxBytes,
                                            map, bar, b * Cfg::kBoxElems, (it.kv0 + j) * kBN, it.bh);
                            }
                        }
                        loaded[stage] = true;
                        last_parity[stage] = phase;
                        ++ring;
                    }
                }
            }
            if (!ok) {
                // Let every copy still in flight land before the CTA releases its memory.
                for (int s = 0; s < STAGES; ++s) {
                    if (loaded[s]) {
                        mbar_wait_drain(smem_u32(&sb.kv_full[s]), last_parity[s], wctx,
                                        kStatusTimeoutTeardown);
                    }
                }
                for (int t = 0; t < NQ; ++t) {
                    if (q_loads[t] > 0) {
                        mbar_wait_drain(smem_u32(&sb.q_full[t]), (q_loads[t] - 1) & 1, wctx,
                                        kStatusTimeoutTeardown);
                    }
                }
            }
        }
        __syncwarp();
    } else if (Cfg::kIssuers == 2 && (warp == Cfg::kMmaWarp || warp == Cfg::kIssuerWarp1)) {
        // =========================== MMA issuers, one per query tile ===========================
        // Issuer t walks the whole K/V ring (so that each slot's release takes one arrival per
        // issuer) and issues only tile t's MMAs. It waits for every slot to land before it
        // releases it, even one its tile does not read, so it can never release a later use
        // of a slot before the producer has filled the current one.
        if (lane == 0) {
            const int t = (warp == Cfg::kMmaWarp) ? 0 : 1;
            bool ok = true;
            const uint32_t kv_addr0 = smem_base + Cfg::kSmemKV;
            const uint64_t qd = make_desc_kmajor_sw128(smem_base + Cfg::kSmemQ + t * Cfg::kQTileBytes);
            const uint64_t kd0 = make_desc_kmajor_sw128(kv_addr0);
            const uint64_t vd0 = make_desc_mnmajor_sw128(kv_addr0, kBoxBytes);
            auto stage_off = [](int stage) -> uint64_t {
                return static_cast<uint64_t>(stage * (Cfg::kTileBytes >> 4));
            };
            const uint32_t s_addr = tmem + Cfg::kTmemS + t * kBN;
            const uint32_t o_addr = tmem + Cfg::kTmemO + t * Cfg::D;
            const uint32_t p_addr = Cfg::SEP_P ? (tmem + Cfg::kTmemExtra + t * 64) : s_addr;
            int ring = 0;
            int q_uses = 0;  // Q_t loads consumed
            int s_cnt = 0;   // S_t MMAs issued
            int pv_cnt = 0;  // P_t consumed (P.V_t issued)
            for (int r = 0; ok; ++r) {
                const int idx = item_index(r);
                if (idx < 0) {
                    break;
                }
                Item it;
                decode(idx, it);
                const int n_t = (t == 0) ? it.n_kv[0] : it.n_kv[NQ - 1];
                const int n_max = it.n_max;
                if (n_t > 0) {
                    ok = mbar_wait(smem_u32(&sb.q_full[t]), q_uses & 1, wctx, kStatusTimeoutMma);
                    ++q_uses;
                }
                if (ok && n_max > 0) {
                    const int k_slot = ring++;
                    ok = mbar_wait(smem_u32(&sb.kv_full[k_slot % STAGES]), (k_slot / STAGES) & 1, wctx,
                                   kStatusTimeoutMma);
                    if (ok && n_t > 0) {
                        if constexpr (Cfg::SEP_P) {
                            // The softmax has the previous item's last S_t in registers.
                            if (s_cnt > 0) {
                                ok = mbar_wait(smem_u32(&sb.s_free[t]), (s_cnt - 1) & 1, wctx,
                                               kStatusTimeoutMma);
                            }
                        }
                        if (ok) {
                            tc_fence_after();
                            issue_s_mma<Cfg>(s_addr, qd, kd0 + stage_off(k_slot % STAGES));
                            umma_commit(smem_u32(&sb.s_full[t]));
                            if (n_t == 1) {
                                umma_commit(smem_u32(&sb.q_empty[t]));  // Q_t read for the last time
                            }
                            ++s_cnt;
                        }
                    }
                    if (ok) {
                        umma_commit(smem_u32(&sb.kv_empty[k_slot % STAGES]));
                    }
                }
                for (int j = 0; ok && j < n_max; ++j) {
                    const int v_slot = ring++;
                    const int vs = v_slot % STAGES;
                    const bool has_next = (j + 1 < n_max);
                    const int k_slot = has_next ? ring++ : 0;
                    const int ks = k_slot % STAGES;
                    const bool active = (j < n_t);
                    const bool next_s = (j + 1 < n_t);
                    bool k_ready = false;
                    if (active) {
                        if constexpr (Cfg::SEP_P) {
                            // S_t(j+1) as soon as the softmax has S_t(j) in registers.
                            if (next_s) {
                                ok = mbar_wait(smem_u32(&sb.s_free[t]), (s_cnt - 1) & 1, wctx, kStatusTimeoutMma);
                                ok = ok && mbar_wait(smem_u32(&sb.kv_full[ks]), (k_slot / STAGES) & 1, wctx,
                                                     kStatusTimeoutMma);
                                if (!ok) {
                                    break;
                                }
                                k_ready = true;
                                tc_fence_after();
                                issue_s_mma<Cfg>(s_addr, qd, kd0 + stage_off(ks));
                                umma_commit(smem_u32(&sb.s_full[t]));
                                if (j + 2 == n_t) {
                                    umma_commit(smem_u32(&sb.q_empty[t]));
                                }
                                ++s_cnt;
                            }
                        }
                        ok = mbar_wait(smem_u32(&sb.p_full[t]), pv_cnt & 1, wctx, kStatusTimeoutMma);
                        ok = ok && mbar_wait(smem_u32(&sb.kv_full[vs]), (v_slot / STAGES) & 1, wctx,
                                             kStatusTimeoutMma);
                        if (!ok) {
                            break;
                        }
                        tc_fence_after();
                        if constexpr (Cfg::ACC16) {
                            issue_pv_mma_f16<Cfg>(tmem + Cfg::tmem_t(t), p_addr, vd0 + stage_off(vs));
                        } else {
                            issue_pv_mma_f32<Cfg>(o_addr, p_addr, vd0 + stage_off(vs), j == 0);
                        }
                        umma_commit(smem_u32(&sb.o_done[t]));
                        ++pv_cnt;
                        if constexpr (!Cfg::SEP_P) {
                            // S_t(j+1) reuses the columns P_t(j) was read from by the MMAs above
                            // (tcgen05.mma operations of one thread execute in issue order).
                            if (next_s) {
                                ok = mbar_wait(smem_u32(&sb.kv_full[ks]), (k_slot / STAGES) & 1, wctx,
                                                     kStatusTimeoutMma);
                                if (!ok) {
                                    break;
                                }
                                k_ready = true;
                                tc_fence_after();
                                issue_s_mma<Cfg>(s_addr, qd, kd0 + stage_off(ks));
                                umma_commit(smem_u32(&sb.s_full[t]));
                                if (j + 2 == n_t) {
                                    umma_commit(smem_u32(&sb.q_empty[t]));
                                }
                                ++s_cnt;
                            }
                        }
                    } else {
                        ok = mbar_wait(smem_u32(&sb.kv_full[vs]), (v_slot / STAGES) & 1, wctx,
                                       kStatusTimeoutMma);
                    }
                    if (ok && has_next && !k_ready) {
                        ok = mbar_wait(smem_u32(&sb.kv_full[ks]), (k_slot / STAGES) & 1, wctx,
                                       kStatusTimeoutMma);
                    }
                    if (!ok) {
                        break;
                    }
                    umma_commit(smem_u32(&sb.kv_empty[vs]));
                    if (has_next) {
                        umma_commit(smem_u32(&sb.kv_empty[ks]));
                    }
                }
            }
            // Every MMA issued above must be complete before tensor memory is released.
            umma_commit(smem_u32(&sb.mma_idle));
            mbar_wait_drain(smem_u32(&sb.mma_idle), 0, wctx, kStatusTimeoutTeardown);
        }
        __syncwarp();
    } else if (Cfg::kSBufs == 2 && warp == Cfg::kMmaWarp) {
        // ================= MMA issuer: one query tile, two S buffers (fp16acc) =================
        // S(i) goes to buffer (running S count) & 1. Per item S(0) and S(1) are issued at
        // once; after P.V(j) (which reads P(j) from S(j)'s buffer) comes S(j+2) into that same
        // buffer, in issue order. K_i and V_i are loads 2i and 2i+1 of the item's share of the
        // producer's sequence; each slot is released after its MMA (slots alternate K / V,
        // so every slot's releases follow its loads in order).
        if (lane == 0) {
            bool ok = true;
            const uint32_t kv_addr0 = smem_base + Cfg::kSmemKV;
            const uint64_t qd = make_desc_kmajor_sw128(smem_base + Cfg::kSmemQ);
            const uint64_t kd0 = make_desc_kmajor_sw128(kv_addr0);
            const uint64_t vd0 = make_desc_mnmajor_sw128(kv_addr0, kBoxBytes);
            auto stage_off = [](int stage) -> uint64_t {
                return static_cast<uint64_t>(stage * (Cfg::kTileBytes >> 4));
            };
            auto wait_load = [&](int load) -> bool {
                return mbar_wait(smem_u32(&sb.kv_full[load % STAGES]), (load / STAGES) & 1, wctx,
                                 kStatusTimeoutMma);
            };
            int ring = 0;    // producer loads of the items before the current one
            int q_uses = 0;  // Q loads consumed
            int s_cnt = 0;   // S MMAs issued
            int pv_cnt = 0;  // P consumed (P.V issued)
            auto issue_s = [&](int load, bool last_of_item) {
                const int buf = s_cnt & 1;
                tc_fence_after();
                issue_s_mma<Cfg>(tmem + Cfg::kTmemS + buf * kBN, qd, kd0 + stage_off(load % STAGES));
                umma_commit(smem_u32(&sb.s_full[buf]));
                umma_commit(smem_u32(&sb.kv_empty[load % STAGES]));
                if (last_of_item) {
                    umma_commit(smem_u32(&sb.q_empty[0]));  // Q read for the last time
                }
                ++s_cnt;
            };
            for (int r = 0; ok; ++r) {
                const int idx = item_index(r);
                if (idx < 0) {
                    break;
                }
                Item it;
                decode(idx, it);
                const int nk = it.n_kv[0];  // == it.n_max with one query tile
                const int base = ring;
                ring += 2 * it.n_max;
                if (nk == 0) {
                    continue;
                }
                ok = mbar_wait(smem_u32(&sb.q_full[0]), q_uses & 1, wctx, kStatusTimeoutMma);
                ++q_uses;
                for (int i = 0; ok && i < min(nk, 2); ++i) {
                    ok = wait_load(base + 2 * i);
                    if (ok) {
                        issue_s(base + 2 * i, i == nk - 1);
                    }
                }
                for (int j = 0; ok && j < nk; ++j) {
                    const int v_load = base + 2 * j + 1;
                    ok = mbar_wait(smem_u32(&sb.p_full[0]), pv_cnt & 1, wctx, kStatusTimeoutMma) &&
                         wait_load(v_load);
                    if (!ok) {
                        break;
                    }
                    tc_fence_after();
                    issue_pv_mma_f16<Cfg>(tmem + Cfg::tmem_t(0), tmem + Cfg::kTmemS + (pv_cnt & 1) * kBN,
                                          vd0 + stage_off(v_load % STAGES));
                    umma_commit(smem_u32(&sb.o_done[0]));
                    umma_commit(smem_u32(&sb.kv_empty[v_load % STAGES]));
                    ++pv_cnt;
                    if (j + 2 < nk) {
                        ok = wait_load(base + 2 * (j + 2));
                        if (ok) {
                            issue_s(base + 2 * (j + 2), j + 2 == nk - 1);
                        }
                    }
                }
            }
            // Every MMA issued above must be complete before tensor memory is released.
            umma_commit(smem_u32(&sb.mma_idle));
            mbar_wait_drain(smem_u32(&sb.mma_idle), 0, wctx, kStatusTimeoutTeardown);
        }
        __syncwarp();
    } else if (Cfg::kIssuers == 1 && Cfg::kSBufs == 1 && warp == Cfg::kMmaWarp) {
        // ================================== MMA issuer ====================================
        if (lane == 0) {
            bool ok = true;
            const uint32_t q_addr0 = smem_base + Cfg::kSmemQ;
            const uint32_t kv_addr0 = smem_base + Cfg::kSmemKV;
            const uint64_t qd0 = make_desc_kmajor_sw128(q_addr0);
            auto q_desc = [qd0](int t) -> uint64_t {
                return qd0 + static_cast<uint64_t>(t * (Cfg::kQTileBytes >> 4));
            };
            const uint64_t kd0 = make_desc_kmajor_sw128(kv_addr0);
            const uint64_t vd0 = Cfg::FP8 ? make_desc_kmajor_sw128(kv_addr0) : make_desc_mnmajor_sw128(kv_addr0, kBoxBytes);
            auto stage_off = [](int stage) -> uint64_t {
                return static_cast<uint64_t>(stage * (Cfg::kTileBytes >> 4));
            };
            int ring = 0;
            int q_uses[NQ];  // Q_t loads consumed
            int s_cnt[NQ];   // S_t MMAs issued
            int pv_cnt[NQ];  // P_t consumed (P.V_t issued)
#pragma unroll
            for (int t = 0; t < NQ; ++t) {
                q_uses[t] = 0;
                s_cnt[t] = 0;
                pv_cnt[t] = 0;
            }
            // Issues the next S_t (K tile in ring slot ks) once its columns are free.
            auto issue_s = [&](int t, int ks, bool last_of_item) -> bool {
                if constexpr (Cfg::SEP_P) {
                    if (s_cnt[t] > 0 &&
                        !mbar_wait(smem_u32(&sb.s_free[t]), (s_cnt[t] - 1) & 1, wctx, kStatusTimeoutMma)) {
                        return false;
                    }
                }
                tc_fence_after();
                issue_s_mma<Cfg>(tmem + Cfg::kTmemS + t * kBN, q_desc(t), kd0 + stage_off(ks));
                umma_commit(smem_u32(&sb.s_full[t]));
                if (last_of_item) {
                    umma_commit(smem_u32(&sb.q_empty[t]));  // Q_t read for the last time
                }
                ++s_cnt[t];
                return true;
            };
            for (int r = 0; ok; ++r) {
                const int idx = item_index(r);
                if (idx < 0) {
                    break;
                }
                Item it;
                decode(idx, it);
                const int n_max = it.n_max;
#pragma unroll
                for (int t = 0; t < NQ; ++t) {
                    if (ok && it.n_kv[t] > 0) {
                        ok = mbar_wait(smem_u32(&sb.q_full[t]), q_uses[t] & 1, wctx, kStatusTimeoutMma);
                        ++q_uses[t];
                    }
                }
                if (ok && n_max > 0) {
                    // S_t(0) of every tile of the item: each follows the previous item's last
                    // P.V_t in issue order (P_t of that tile lay in S_t's columns).
                    const int k_slot = ring++;
                    ok = mbar_wait(smem_u32(&sb.kv_full[k_slot % STAGES]), (k_slot / STAGES) & 1, wctx,
                                   kStatusTimeoutMma);
#pragma unroll
                    for (int t = 0; t < NQ; ++t) {
                        if (ok && it.n_kv[t] > 0) {
                            ok = issue_s(t, k_slot % STAGES, it.n_kv[t] == 1);
                        }
                    }
                    if (ok) {
                        umma_commit(smem_u32(&sb.kv_empty[k_slot % STAGES]));
                    }
                }
                for (int j = 0; ok && j < n_max; ++j) {
                    const int v_slot = ring++;
                    const int vs = v_slot % STAGES;
                    const bool has_next = (j + 1 < n_max);
                    const int k_slot = has_next ? ring++ : 0;
                    const int ks = k_slot % STAGES;
                    bool k_ready = false;
                    bool v_ready = false;
#pragma unroll
                    for (int t = 0; t < NQ; ++t) {
                        if (!ok || j >= it.n_kv[t]) {
                            continue;
                        }
                        const bool next_s = (j + 1 < it.n_kv[t]);
                        const uint32_t s_addr = tmem + Cfg::kTmemS + t * kBN;
                        if constexpr (Cfg::SEP_P) {
                            // S_t(j+1) as soon as the softmax has S_t(j) in registers.
                            if (next_s) {
                                if (!k_ready) {
                                    ok = mbar_wait(smem_u32(&sb.kv_full[ks]), (k_slot / STAGES) & 1,
                                                   wctx, kStatusTimeoutMma);
                                    k_ready = true;
                                }
                                ok = ok && issue_s(t, ks, j + 2 == it.n_kv[t]);
                                if (!ok) {
                                    break;
                                }
                            }
                        }
                        ok = mbar_wait(smem_u32(&sb.p_full[t]), pv_cnt[t] & 1, wctx, kStatusTimeoutMma);
                        if (ok && !v_ready) {
                            ok = mbar_wait(smem_u32(&sb.kv_full[vs]), (v_slot / STAGES) & 1, wctx,
                                           kStatusTimeoutMma);
                            v_ready = true;
                        }
                        if (!ok) {
                            break;
                        }
                        tc_fence_after();
                        const uint64_t vd = vd0 + stage_off(vs);
                        if constexpr (Cfg::ACC16) {
                            issue_pv_mma_f16<Cfg>(tmem + Cfg::tmem_t(t), s_addr, vd);
                        } else if constexpr (Cfg::SEP_P) {
                            issue_pv_mma_f32<Cfg>(tmem + Cfg::kTmemO + t * Cfg::D,
                                                  tmem + Cfg::kTmemExtra + t * 64, vd, j == 0);
                        } else {
                            issue_pv_mma_f32<Cfg>(tmem + Cfg::kTmemO + t * Cfg::D, s_addr, vd, j == 0);
                        }
                        umma_commit(smem_u32(&sb.o_done[t]));
                        ++pv_cnt[t];
                        if constexpr (!Cfg::SEP_P) {
                            // S_t(j+1) reuses the columns P_t(j) was read from by the MMAs above.
                            if (next_s) {
                                if (!k_ready) {
                                    ok = mbar_wait(smem_u32(&sb.kv_full[ks]), (k_slot / STAGES) & 1,
                                                   wctx, kStatusTimeoutMma);
                                    k_ready = true;
                                }
                                ok = ok && issue_s(t, ks, j + 2 == it.n_kv[t]);
                                if (!ok) {
                                    break;
                                }
                            }
                        }
                    }
                    if (!ok) {
                        break;
                    }
                    umma_commit(smem_u32(&sb.kv_empty[vs]));
                    if (has_next) {
                        umma_commit(smem_u32(&sb.kv_empty[ks]));
                    }
                }
            }
            // Every MMA issued above must be complete before tensor memory is released.
            umma_commit(smem_u32(&sb.mma_idle));
            mbar_wait_drain(smem_u32(&sb.mma_idle), 0, wctx, kStatusTimeoutTeardown);
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == Cfg::kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// Split-KV combine (reference: none; Flash-Decoding's merge of per-range softmax partials).
// One warp per output row, lanes over the head dim, ranges merged in index order (so the result
// is deterministic): M = max m_s over the ranges with l_s > 0, then
// O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, rounded to fp16 (BF16: bfloat16).
// Rows: with split-KV (tail_blocks == 0) every row of every head, row r of head bh at record
// bh * rows_pad + r; with a tail split the rows of the tail blocks, row r of tail block p at
// record p * rows_per_block + r, the block being row block tail_from + p of the non-causal item
// order (head lin / nb, block lin % nb). Range s adds s * split_stride records.
struct CombineArgs {
    const float* ws_o;
    const float2* ws_ml;
    void* o;                 // [B*H][N][D] fp16 or bf16
    int n;
    int num_splits;
    long long split_stride;  // records per key range
    long long rows;          // output rows of this launch
    int tail_blocks;         // 0: split-KV layout
    int tail_from;
    int nb;                  // row blocks per head
    int rows_per_block;
    int rows_pad;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(256) splitkv_combine_kernel(const CombineArgs a) {
    constexpr int PER = D / 32;  // columns per lane
    const long long item = static_cast<long long>(blockIdx.x) * 8 + threadIdx.x / 32;
    const int lane = static_cast<int>(threadIdx.x) % 32;
    if (item >= a.rows) {
        return;
    }
    long long rec0, out_row;
    if (a.tail_blocks == 0) {
        const long long bh = item / a.n;
        rec0 = bh * a.rows_pad + (item - bh * a.n);
        out_row = item;
    } else {
        const long long p = item / a.rows_per_block;
        const long long lin = a.tail_from + p;
        const long long bh = lin / a.nb;
        const long long grow = (lin - bh * a.nb) * a.rows_per_block + (item - p * a.rows_per_block);
        if (grow >= a.n) {
            return;
        }
        rec0 = item;
        out_row = bh * a.n + grow;
    }
    float m_max = -INFINITY;
    for (int sp = 0; sp < a.num_splits; ++sp) {
        const float2 ml = a.ws_ml[rec0 + sp * a.split_stride];
        if (ml.y > 0.0f) {
            m_max = fmaxf(m_max, ml.x);
        }
    }
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        acc[i] = 0.0f;
    }
    float l = 0.0f;
    for (int sp = 0; sp < a.num_splits; ++sp) {
        const long long rec = rec0 + sp * a.split_stride;
        const float2 ml = a.ws_ml[rec];
        if (!(ml.y > 0.0f)) {
            continue;
        }
        const float w = exp2f(ml.x - m_max);
        l = fmaf(ml.y, w, l);
        const float* src = a.ws_o + rec * D + lane * PER;
        if constexpr (PER == 4) {
            const float4 v = *reinterpret_cast<const float4*>(src);
            acc[0] = fmaf(v.x, w, acc[0]);
            acc[1] = fmaf(v.y, w, acc[1]);
            acc[2] = fmaf(v.z, w, acc[2]);
            acc[3] = fmaf(v.w, w, acc[3]);
        } else {
            const float2 v = *reinterpret_cast<const float2*>(src);
            acc[0] = fmaf(v.x, w, acc[0]);
            acc[1] = fmaf(v.y, w, acc[1]);
        }
    }
    const float inv = (l > 0.0f) ? (1.0f / l) : 0.0f;
    uint16_t* dst = static_cast<uint16_t*>(a.o) + out_row * D + lane * PER;
    if constexpr (PER == 4) {
        *reinterpret_cast<uint2*>(dst) =
            make_uint2(pack2<BF16>(acc[0] * inv, acc[1] * inv), pack2<BF16>(acc[2] * inv, acc[3] * inv));
    } else {
        *reinterpret_cast<uint32_t*>(dst) = pack2<BF16>(acc[0] * inv, acc[1] * inv);
    }
}

// fp8 V transpose: V [B*H][N][128] e4m3 -> V^T [B*H][128][vt_cols] (keys contiguous, zeros for
// keys >= N), so that P.V reads V^T K-major like Q K^T reads K. One CTA per 64 keys of a head:
// 64 rows of 128 bytes in through shared memory, 128 rows of 64 bytes out, 16-byte accesses.
__global__ void __launch_bounds__(256) fp8_transpose_v_kernel(const uint8_t* __restrict__ v,
                                                               uint8_t* __restrict__ vt, int n, int vt_cols) {
    __shared__ __align__(16) uint8_t tile[64][128 + 16];
    const long long bh = blockIdx.y;
    const int k0 = static_cast<int>(blockIdx.x) * 64;
    const uint8_t* src = v + bh * n * 128ll;
    for (int i = static_cast<int>(threadIdx.x); i < 64 * 8; i += 256) {
        const int r = i / 8;
        const int c = i % 8;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (k0 + r < n) {
            val = *reinterpret_cast<const uint4*>(src + static_cast<long long>(k0 + r) * 128 + c * 16);
        }
        *reinterpret_cast<uint4*>(&tile[r][c * 16]) = val;
    }
    __syncthreads();
    uint8_t* dst = vt + bh * 128ll * vt_cols;
    for (int i = static_cast<int>(threadIdx.x); i < 128 * 4; i += 256) {
        const int dd = i / 4;
        const int g = i % 4;
        const int kk = k0 + g * 16;
        if (kk >= vt_cols) {
            continue;
        }
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t x = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                x |= static_cast<uint32_t>(tile[g * 16 + q * 4 + b][dd]) << (8 * b);
            }
            w[q] = x;
        }
        *reinterpret_cast<uint4*>(dst + static_cast<long long>(dd) * vt_cols + kk) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

cudaError_t launch_fp8_transpose_v(const void* v, void* vt, int num_bh, int seqlen, cudaStream_t stream) {
    const int vt_cols = (seqlen + 15) / 16 * 16;
    const dim3 grid(static_cast<unsigned>((vt_cols + 63) / 64), static_cast<unsigned>(num_bh));
    fp8_transpose_v_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(v), static_cast<uint8_t*>(vt),
                                                     seqlen, vt_cols);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Host-side dispatch
// ------------------------------------------------------------------------------------------
int device_sm_count() {
    static int counts[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        return 148;
    }
    int c = __atomic_load_n(&counts[dev], __ATOMIC_RELAXED);
    if (c == 0) {
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) {
            return 148;
        }
        __atomic_store_n(&counts[dev], c, __ATOMIC_RELAXED);
    }
    return c;
}

// A positive number from the environment, or `fallback`.
static double env_double(const char* name, double fallback) {
    const char* v = std::getenv(name);
    if (v == nullptr) {
        return fallback;
    }
    const double x = std::atof(v);
    return x > 0.0 ? x : fallback;
}

Plan make_plan(int num_bh, int seqlen, int head_dim, bool causal, int variant, int num_splits,
               bool allow_tail, int sm_count) {
    Plan p{};
    sm_count = std::max(1, sm_count);
    p.rows_per_item = kernel_rows_per_cta(head_dim, variant);
    const long long nb = (seqlen + p.rows_per_item - 1) / p.rows_per_item;
    const long long row_blocks = nb * num_bh;
    p.row_blocks = static_cast<int>(std::min<long long>(row_blocks, 0x7fffffffLL));
    const int key_tiles = (seqlen + kBN - 1) / kBN;
    // Short rows run on a persistent grid, so that each item's Q load and first S overlap the
    // previous item's tail (measured: B16 H16 N1000 d128 causal 496 -> 554 TFLOPS); longer rows
    // one CTA per item (cfg1 N4096 causal: 911 vs 862 persistent, its items differ in length).
    // Without the mask every item costs the same and the static assignment stays balanced: N3000
    // d128 937 -> 983, d64 581 -> 631, N4096 d128 963 -> 1001; N8192 and 16384 unchanged.
    p.persistent = seqlen <= kPersistentMaxN || (!causal && seqlen <= kPersistentMaxNFull);
    // Split-KV when the row blocks leave SMs idle (few heads x long rows): about SMs / row
    // blocks ranges, at least two key tiles each, at most 16.
    int splits = num_splits;
    if (splits <= 0) {
        splits = 1;
        if (row_blocks < sm_count) {
            splits = static_cast<int>(sm_count / row_blocks);
            splits = std::min(splits, std::max(1, key_tiles / 2));
            splits = std::max(1, std::min(splits, 16));
        }
    }
    p.num_splits = splits;
    // Tail split (non-causal, whose row blocks all cost the same): when the grid's last wave is
    // partial and the waves are few, cut the last wave's row blocks into k key ranges so that it
    // takes about 1/k of a full item. In units of one item: the tail costs
    // ceil(T k / SMs) waves of pieces of 1/k + 2 / key_tiles (a piece's fixed part, its pipeline
    // fill and drain and its epilogue, is about two key tiles); k = 1 costs one wave.
    if (allow_tail && num_splits <= 0 && splits == 1 && !causal) {
        const long long waves = row_blocks / sm_count;
        const long long tail = row_blocks % sm_count;
        if (tail > 0 && waves < 8) {
            double best = 1.0;
            int best_k = 1;
            for (int k = 2; k <= 4 && key_tiles / k >= 8; ++k) {
                const double piece = 1.0 / k + 2.0 / key_tiles;
                const double cost = static_cast<double>((tail * k + sm_count - 1) / sm_count) * piece;
                if (cost < best - 0.05) {
                    best = cost;
                    best_k = k;
                }
            }
            if (best_k > 1) {
                p.tail_blocks = static_cast<int>(tail);
                p.tail_splits = best_k;
            }
        }
    }
    // Causal head groups: ceil(heads / G) heads per group with G the number of groups that keep
    // each group's K and V (4 N d bytes per head) within about 64 MiB of the 126 MB L2; a single
    // group when all of it fits in 96 MiB, so that few heads (a GPU's shard of a sharded
    // problem) get one longest-first sweep.
    p.head_groups = 1;
    if (causal) {
        // Tuning knobs (MiB): FA_L2_GROUP_MIB, the K/V budget of a group; FA_L2_SINGLE_MIB, the
        // K/V total up to which all heads form one group.
        static const double group_mib = env_double("FA_L2_GROUP_MIB", 64.0);
        static const double single_mib = env_double("FA_L2_SINGLE_MIB", 96.0);
        const double kv = 4.0 * seqlen * head_dim * static_cast<double>(num_bh);
        const double mib = 1048576.0;
        if (kv > single_mib * mib) {
            const int groups = static_cast<int>(std::min<double>(num_bh, std::ceil(kv / (group_mib * mib))));
            // ceil(heads / groups) heads per group: equal groups whenever they divide evenly
            const int per_group = (num_bh + groups - 1) / groups;
            p.head_groups = (num_bh + per_group - 1) / per_group;
        }
    }
    const long long items = p.tail_blocks > 0 ? row_blocks + static_cast<long long>(p.tail_blocks) * (p.tail_splits - 1)
                                              : row_blocks * splits;
    p.items = static_cast<int>(std::min<long long>(items, 0x7fffffffLL));
    p.ctas = p.persistent ? static_cast<int>(std::min<long long>(items, sm_count)) : p.items;
    const unsigned long long rec_bytes = static_cast<unsigned long long>(head_dim + 2) * 4ull;
    if (p.tail_blocks > 0) {
        p.workspace_bytes = static_cast<unsigned long long>(p.tail_blocks) * p.tail_splits * p.rows_per_item * rec_bytes;
    } else if (splits > 1) {
        p.workspace_bytes = splitkv_workspace_bytes(num_bh, seqlen, head_dim, splits);
    }
    return p;
}

template <int D, bool CAUSAL, int VARIANT, bool BF16 = false, bool FP8 = false>
cudaError_t launch_cfg(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                       const CUtensorMap& tm_o, const FwdArgs& args, const Plan& plan, cudaStream_t stream) {
    using Cfg = FwdCfg<D, CAUSAL, VARIANT, BF16, FP8>;
    auto* kernel = fa_fwd_sm100_kernel<Cfg>;
    cudaError_t err = ensure_smem_limit<fa_fwd_sm100_kernel<Cfg>>(Cfg::kSmemAlloc);
    if (err != cudaSuccess) {
        return err;
    }
    if (plan.items <= 0 || plan.ctas <= 0 || plan.rows_per_item != Cfg::NQ * kBM) {
        return cudaErrorInvalidValue;
    }
    kernel<<<dim3(static_cast<unsigned>(plan.ctas)), Cfg::kThreads, Cfg::kSmemAlloc, stream>>>(tm_q, tm_k, tm_v,
                                                                                              tm_o, args);
    return cudaGetLastError();
}

template <bool CAUSAL>
cudaError_t launch_variant_fp8(int variant, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                               const CUtensorMap& tm_v, const CUtensorMap& tm_o, const FwdArgs& args,
                               const Plan& plan, cudaStream_t stream) {
    switch (variant) {
        case kVariantBaseline:
            return launch_cfg<128, CAUSAL, kVariantBaseline, false, true>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
        case kVariantOpt:
            return launch_cfg<128, CAUSAL, kVariantOpt, false, true>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

template <int D, bool CAUSAL>
cudaError_t launch_variant(int variant, bool bf16, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                           const CUtensorMap& tm_v, const CUtensorMap& tm_o, const FwdArgs& args,
                           const Plan& plan, cudaStream_t stream) {
    if (bf16) {
        // bfloat16 inputs: the fp32-accumulating variants only (validated by the C ABI).
        switch (variant) {
            case kVariantBaseline:
                return launch_cfg<D, CAUSAL, kVariantBaseline, true>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
            case kVariantOpt:
                return launch_cfg<D, CAUSAL, kVariantOpt, true>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
            default:
                return cudaErrorInvalidValue;
        }
    }
    switch (variant) {
        case kVariantBaseline:
            return launch_cfg<D, CAUSAL, kVariantBaseline>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
        case kVariantOpt:
            return launch_cfg<D, CAUSAL, kVariantOpt>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
        case kVariantFp16Acc:
            return launch_cfg<D, CAUSAL, kVariantFp16Acc>(tm_q, tm_k, tm_v, tm_o, args, plan, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t launch_forward(const FwdProblem& prob, const FwdArgs& args, const Plan& plan,
                           cudaStream_t stream) {
    // This kernel: 128-row boxes for Q, K, V and O.
    CUtensorMap maps[4];
    if (prob.fp8) {
        // e4m3 Q and K with 128-byte rows, V^T (128 keys x 128 rows per box), fp16 O.
        if (prob.head_dim != 128 || prob.vt == nullptr ||
            encode_u8_map(&maps[0], prob.q, 128, prob.seqlen, prob.num_bh, 128, kBM) != CUDA_SUCCESS ||
            encode_u8_map(&maps[1], prob.k, 128, prob.seqlen, prob.num_bh, 128, kBN) != CUDA_SUCCESS ||
            encode_u8_map(&maps[2], prob.vt, prob.vt_cols, 128, prob.num_bh, kBN, 128) != CUDA_SUCCESS ||
            encode_bhnd_map(&maps[3], prob.o, prob.num_bh, prob.seqlen, 128, kBM, false) != CUDA_SUCCESS) {
            return cudaErrorInvalidValue;
        }
    } else {
        const void* ptrs[4] = {prob.q, prob.k, prob.v, prob.o};
        for (int i = 0; i < 4; ++i) {
            if (encode_bhnd_map(&maps[i], ptrs[i], prob.num_bh, prob.seqlen, prob.head_dim, kBM, prob.bf16) !=
                CUDA_SUCCESS) {
                return cudaErrorInvalidValue;
            }
        }
    }
    FwdArgs a = args;
    a.o = prob.o;
    a.num_items = plan.items;
    a.num_splits = plan.num_splits;
    a.head_group = (prob.num_bh + std::max(1, plan.head_groups) - 1) / std::max(1, plan.head_groups);
    const int nb = (prob.seqlen + plan.rows_per_item - 1) / plan.rows_per_item;
    a.div_nb = FastDiv(nb);
    a.div_per_split = FastDiv(nb * prob.num_bh);
    a.div_group_items = FastDiv(nb * a.head_group);
    a.div_group = FastDiv(a.head_group);
    const int last = prob.num_bh % a.head_group;
    a.div_last_group = FastDiv(last == 0 ? a.head_group : last);
    a.tail_blocks = plan.tail_blocks;
    a.tail_splits = plan.tail_blocks > 0 ? plan.tail_splits : 1;
    a.div_tail = FastDiv(a.tail_splits);
    a.tail_from = plan.tail_blocks > 0 ? plan.row_blocks - plan.tail_blocks : plan.items;
    const int variant = prob.variant;
    const bool bf16 = prob.bf16;
    if (prob.fp8) {
        return prob.causal ? launch_variant_fp8<true>(variant, maps[0], maps[1], maps[2], maps[3], a, plan, stream)
                           : launch_variant_fp8<false>(variant, maps[0], maps[1], maps[2], maps[3], a, plan, stream);
    }
    if (prob.head_dim == 64) {
        return prob.causal
                   ? launch_variant<64, true>(variant, bf16, maps[0], maps[1], maps[2], maps[3], a, plan, stream)
                   : launch_variant<64, false>(variant, bf16, maps[0], maps[1], maps[2], maps[3], a, plan, stream);
    }
    if (prob.head_dim == 128) {
        return prob.causal
                   ? launch_variant<128, true>(variant, bf16, maps[0], maps[1], maps[2], maps[3], a, plan, stream)
                   : launch_variant<128, false>(variant, bf16, maps[0], maps[1], maps[2], maps[3], a, plan, stream);
    }
    return cudaErrorInvalidValue;
}

template <int D>
int smem_for(int variant) {
    switch (variant) {
        case kVariantBaseline:
            return FwdCfg<D, false, kVariantBaseline>::kSmemAlloc;
        case kVariantOpt:
            return FwdCfg<D, false, kVariantOpt>::kSmemAlloc;
        default:
            return FwdCfg<D, false, kVariantFp16Acc>::kSmemAlloc;
    }
}

template <int D>
int threads_for(int variant) {
    switch (variant) {
        case kVariantBaseline:
            return FwdCfg<D, false, kVariantBaseline>::kThreads;
        case kVariantOpt:
            return FwdCfg<D, false, kVariantOpt>::kThreads;
        default:
            return FwdCfg<D, false, kVariantFp16Acc>::kThreads;
    }
}

cudaError_t launch_splitkv_combine(const FwdProblem& prob, const FwdArgs& args, const Plan& plan,
                                   cudaStream_t stream) {
    CombineArgs a{};
    a.ws_o = args.ws_o;
    a.ws_ml = reinterpret_cast<const float2*>(args.ws_ml);
    a.o = prob.o;
    a.n = prob.seqlen;
    a.nb = (prob.seqlen + plan.rows_per_item - 1) / plan.rows_per_item;
    a.rows_per_block = plan.rows_per_item;
    a.rows_pad = args.rows_pad;
    if (plan.tail_blocks > 0) {
        a.num_splits = plan.tail_splits;
        a.tail_blocks = plan.tail_blocks;
        a.tail_from = plan.row_blocks - plan.tail_blocks;
        a.rows = static_cast<long long>(plan.tail_blocks) * plan.rows_per_item;
        a.split_stride = a.rows;
    } else {
        a.num_splits = plan.num_splits;
        a.rows = static_cast<long long>(prob.num_bh) * prob.seqlen;
        a.split_stride = static_cast<long long>(prob.num_bh) * args.rows_pad;
    }
    const dim3 grid(static_cast<unsigned>((a.rows + 7) / 8));
    if (prob.head_dim == 64) {
        if (prob.bf16) {
            splitkv_combine_kernel<64, true><<<grid, 256, 0, stream>>>(a);
        } else {
            splitkv_combine_kernel<64, false><<<grid, 256, 0, stream>>>(a);
        }
    } else {
        if (prob.bf16) {
            splitkv_combine_kernel<128, true><<<grid, 256, 0, stream>>>(a);
        } else {
            splitkv_combine_kernel<128, false><<<grid, 256, 0, stream>>>(a);
        }
    }
    return cudaGetLastError();
}

int kernel_smem_bytes(int head_dim, bool /*causal*/, int variant) {
    return head_dim == 64 ? smem_for<64>(variant) : smem_for<128>(variant);
}

int kernel_threads(int head_dim, bool /*causal*/, int variant) {
    return head_dim == 64 ? threads_for<64>(variant) : threads_for<128>(variant);
}

int kernel_rows_per_cta(int head_dim, int variant) {
    const bool acc16 = variant == kVariantFp16Acc;
    return kBM * (head_dim == 64 ? FwdCfg<64, false, kVariantOpt>::NQ
                                 : (acc16 ? FwdCfg<128, false, kVariantFp16Acc>::NQ
                                          : FwdCfg<128, false, kVariantOpt>::NQ));
}


}  // namespace fa_sm100

