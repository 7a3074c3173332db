// FlashAttention-2 forward for B200 (sm_100a), head_dim 128, fp32 accumulation ("baseline" and
// "opt"), on CTA pairs: a cluster of two CTAs on two SMs shares each tcgen05.mma
// (cta_group::2, M = 256). Same algorithm and contract as the one-CTA kernel in
// flash_fwd_sm100.cu (which keeps head_dim 64, fp16acc and split-KV); replaces the reference's
// mma.sync kernel (csrc/kernels/flash_fwd.cu:154-561) for d = 128.
//
// Why pairs. With two 128-row query tiles per SM, TMEM (512 columns) holds exactly S and O for
// both tiles, so P has to overwrite S and the next S of a tile cannot be computed before that
// tile's softmax and P.V are done: every tile alternates softmax and MMA and the SM idles in
// between. With one query tile per SM and the key/value tiles split between the two SMs of a
// pair (each SM loads half, the pair MMA reads both halves), TMEM holds two S buffers, two P
// buffers and O, so S(j+1) is computed while the softmax works on S(j): the softmax runs tile
// after tile without waiting, and the per-SM shared-memory and L2 traffic stays that of two
// query tiles per SM.
//
// CTA r of pair (m, bh) owns query rows [256 m + 128 r, +128) of head bh.
//   warps 0-7   softmax: warp w owns rows 32 (w % 4) .. +31 (its TMEM lanes) and S columns
//               [64 h, 64 h + 64) with h = w / 4; the two warps of a row exchange row max and
//               row sum through shared memory over a 64-thread named barrier.
//   warp 8      TMA producer (both CTAs): this CTA's Q rows once; then the key/value ring in
//               consumption order K0, K1, V0, K2, V1, K3, ...: a K slot holds this CTA's 64 keys
//               (all 128 columns), a V slot this CTA's 64 columns (all 128 keys). Every load
//               counts its bytes on the leader's barrier.
//   warp 9      TMEM allocation (both CTAs, pair allocation) and, in the leader (r = 0), the
//               MMA issuer: S(0), S(1), then per key tile j: P.V(j) interleaved four-and-four
//               with S(j+2) (they touch disjoint TMEM, and runs of at most four SS / TS MMAs keep
//               the tensor pipe at full rate, measured).
//   warps 10-11 idle (whole warpgroups).
// Tensor memory (same columns in both CTAs): S_0 [0,128), S_1 [128,256), P_0 [256,320),
// P_1 [320,384) (fp16 pairs), O [384,512).
//
// Ordering (every wait bounded): S(j+2) reuses S buffer j % 2 after the leader has seen
// P-ready(j) from all 16 softmax warps of the pair (they read S(j) before writing P(j)).
// P(j) reuses P buffer j % 2 after P.V(j-2) completed (o_done[j % 2]); O is rescaled after
// P.V(j-1) completed. Barriers that receive arrivals from the other CTA are waited on with
// cluster-scope acquire.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "fa_internal.h"
#include "sm100_ptx.cuh"
#include "softmax_common.cuh"
#include "tma_host.h"

#ifndef FA_PAIR_RUN
#define FA_PAIR_RUN 1  // P.V / S interleave granularity: 1 = one by one, else runs of four
#endif
#ifndef FA_PAIR_STAGES
#define FA_PAIR_STAGES 10
#endif

namespace fa_sm100 {
namespace pair {

constexpr int D = 128;
constexpr int kRows = 128;                 // query rows per CTA
constexpr int kKeys = 128;                 // keys per key/value tile
constexpr int kQBytes = kRows * D * 2;     // this CTA's Q tile: 32 KB (two 64-column boxes)
constexpr int kQBox = kRows * 128;         // one box of Q / O: 128 rows x 128 B
constexpr int kSlotBytes = 16 * 1024;      // half a K tile (64 keys x 128) or of a V tile (128 x 64)
constexpr int kKBox = 64 * 128;            // one box of a K half: 64 rows x 128 B
constexpr int STAGES = FA_PAIR_STAGES;
constexpr int kSmemQ = 0;
constexpr int kSmemKV = kQBytes;
constexpr int kSmemBytes = kSmemKV + STAGES * kSlotBytes;
constexpr int kSmemAlloc = kSmemBytes + 1024;
constexpr int kThreads = 384;
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kTmemS = 0;    // + 128 b
constexpr int kTmemP = 256;  // + 64 b
constexpr int kTmemO = 384;
static_assert(kSmemAlloc + 4096 <= 227 * 1024, "shared memory budget (dynamic + static)");

struct Barriers {
    uint64_t q_full;        // leader: both CTAs' Q rows landed
    uint64_t kv_full[16];   // leader: both halves of ring slot s landed
    uint64_t kv_empty[16];  // both: the pair MMAs finished with slot s
    uint64_t p_full[2];     // leader: 16 softmax warps wrote P(j) into P buffer j % 2
    uint64_t s_full[2];     // both: S(j) is in S buffer j % 2
    uint64_t o_done[2];     // both: every MMA up to P.V(j) completed (j % 2)
    uint64_t epi;           // this CTA: the 8 softmax warps staged O
    uint64_t mma_idle;      // both: teardown
    uint32_t tmem_base;
    int abort;
};
static_assert(STAGES <= 16, "ring barrier arrays");

// Optional event trace of one CTA pair (build with -DFA_TRACE; off in the product build): SM
// clock stamps, read back with fa_pair_trace_read(). Per CTA rank r, base 2048 r:
// [0, 4 * 128): softmax (warp 0) key tile j: {S ready, S loaded, row max exchanged, P arrived};
// [512, +32 * 16): softmax warp w, key tile j < 16: the same four events at 32 j + 4 w;
// [1024, +4 * 128): leader MMA thread, tile j: {P ready seen, K/V ready, MMAs issued, -}.
#ifdef FA_TRACE
__device__ unsigned long long g_pair_trace[4096];
#define PAIR_TRACE(traced, idx)                     \
    do {                                            \
        if (traced) {                               \
            g_pair_trace[(idx)] = clock64();        \
        }                                           \
    } while (0)
#else
#define PAIR_TRACE(traced, idx) \
    do {                        \
    } while (0)
#endif

struct RowStats {
    float red_max[2][2][kRows];  // [tile parity][column half][row]
    float red_sum[2][kRows];
};

// Bounded wait with cluster-scope acquire (barriers the other CTA arrives on). Same policy as
// mbar_wait: shared-memory polling, the global abort epoch read only after 2^20 cycles.
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                             unsigned code) {
    if (mbar_try_wait_cluster(bar, parity)) {
        return true;
    }
    const long long t0 = clock64();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) {
            return true;
        }
        if ((++spins & 31u) == 0) {
            if (*w.cta_abort != 0) {
                return false;
            }
            const long long waited = clock64() - t0;
            if (waited > (1ll << 20)) {
                if (*w.epoch_word == w.epoch) {
                    *w.cta_abort = 1;
                    return false;
                }
                if (waited > (1ll << 31)) {
                    atomicOr(w.code_word, code);
                    *w.epoch_word = w.epoch;
                    *w.cta_abort = 1;
                    return false;
                }
            }
        }
    }
}

template <bool CAUSAL, int VARIANT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    fa_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o, const FwdArgs args) {
    // Lazy rescale (reference LAZY, flash_fwd.cu:365-376) for "opt"; exact max otherwise.
    constexpr float kRescaleThreshold = (VARIANT == kVariantOpt) ? 8.0f : 0.0f;
    extern __shared__ uint8_t smem_raw[];
    __shared__ Barriers sb;
    __shared__ RowStats rs;

    const int warp = static_cast<int>(threadIdx.x) / 32;
    const int lane = static_cast<int>(threadIdx.x) % 32;
    const uint32_t rank = cluster_ctarank();
    const bool leader = (rank == 0);

    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t smem_base = smem_u32(smem);

    const int n = args.seqlen;
    const int nbp = static_cast<int>(gridDim.x) / 2;  // pairs per head
    const int pb = static_cast<int>(blockIdx.x) / 2;
    int bh = static_cast<int>(blockIdx.y);
    int m_pair = pb;
    if constexpr (CAUSAL) {
        // Longest row blocks first across a group of args.head_group heads (see the one-CTA
        // kernel): the linear pair id maps to (row block, head).
        const int lin = pb + nbp * static_cast<int>(blockIdx.y);
        const int group = lin / (nbp * args.head_group);
        const int head0 = group * args.head_group;
        const int heads = min(args.head_group, args.num_bh - head0);
        const int within = lin - group * nbp * args.head_group;
        bh = head0 + within % heads;
        m_pair = nbp - 1 - within / heads;
    }
    const int q0 = m_pair * 2 * kRows + static_cast<int>(rank) * kRows;  // this CTA's first row
    const int n_tiles_all = (n + kKeys - 1) / kKeys;
    // Key tiles the pair processes: up to the diagonal of the pair's last rows (causal).
    const int nt = CAUSAL ? min(n_tiles_all, 2 * m_pair + 2) : n_tiles_all;

    const WaitCtx wctx{&sb.abort, &args.status->code, &args.status->epoch_aborted, args.epoch};
    const bool traced_pair = (pb == nbp / 2) && (blockIdx.y == 0);
    const int tbase = static_cast<int>(rank) * 2048;
    (void)traced_pair;
    (void)tbase;

    if (threadIdx.x == 0) {
        sb.abort = 0;
        mbar_init(smem_u32(&sb.q_full), 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&sb.kv_full[s]), 1);
            mbar_init(smem_u32(&sb.kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&sb.p_full[b]), 2 * kSoftmaxWarps);
            mbar_init(smem_u32(&sb.s_full[b]), 1);
            mbar_init(smem_u32(&sb.o_done[b]), 1);
        }
        mbar_init(smem_u32(&sb.epi), kSoftmaxWarps);
        mbar_init(smem_u32(&sb.mma_idle), 1);
        mbar_fence_init_cluster();
    }
    if (warp == kMmaWarp) {
        tmem_alloc_pair(smem_u32(&sb.tmem_base), 512);
        tmem_relinquish_pair();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        tma_prefetch_desc(&tm_o);
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem = sb.tmem_base;

    if (warp < kSoftmaxWarps) {
        // ================================ softmax (8 warps) ================================
        const int half = warp / 4;                      // S columns [64 half, +64)
        const int row = (warp % 4) * 32 + lane;         // TMEM lane == query row in this CTA
        const int grow = q0 + row;                      // global query row
        const int pair_id = 1 + (warp % 4);             // named barrier of the row's two warps
        const uint32_t lane_off = static_cast<uint32_t>((warp % 4) * 32) << 16;
        const uint32_t t_base = tmem + lane_off;
        const uint32_t t_o = t_base + kTmemO + half * 64;
        // P-ready goes to the leader's barrier (remote arrival from the other CTA).
        const uint32_t p_full_cl[2] = {mapa_shared(smem_u32(&sb.p_full[0]), 0),
                                       mapa_shared(smem_u32(&sb.p_full[1]), 0)};
        const float scale_log2 = args.scale_log2;
        const int lim = CAUSAL ? min(n - 1, grow) : (n - 1);  // last key this row may see

        float row_max = -INFINITY;
        float row_sum = 0.0f;
        bool ok = true;
        // A warp that gave up on a wait keeps iterating without touching TMEM, so that the two
        // warps of a row pass the same number of pair barriers.
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            ok = ok && __all_sync(0xffffffffu, mbar_wait(smem_u32(&sb.s_full[b]), (j >> 1) & 1,
                                                         wctx, kStatusTimeoutSoftmax));
            if (!ok) {
                pair_sync(pair_id);
                continue;
            }
            [[maybe_unused]] const bool tr = traced_pair && warp == 0 && lane == 0 && j < 128;
            [[maybe_unused]] const bool trw = traced_pair && lane == 0 && j < 16;
            [[maybe_unused]] const int wb = tbase + 512 + j * 32 + warp * 4;
            PAIR_TRACE(tr, tbase + j * 4 + 0);
            PAIR_TRACE(trw, wb + 0);
            tc_fence_after();
            uint32_t sr[64];
            tmem_ld32(t_base + kTmemS + b * 128 + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(t_base + kTmemS + b * 128 + half * 64 + 32,
                      *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_wait_ld();
            PAIR_TRACE(tr, tbase + j * 4 + 1);
            PAIR_TRACE(trw, wb + 1);

            const int kbase = j * kKeys + half * 64;  // key of this thread's first column
            // Masked: the last (ragged) tile, and for causal rows the tiles at or after the
            // row block's diagonal (for the leader's rows the pair's last tile is entirely
            // after the diagonal: all its scores are masked).
            const bool masked = (j * kKeys + kKeys > n) || (CAUSAL && j * kKeys + kKeys - 1 > q0);
            float tile_max;
            float mul;
            if (masked) {
                // Scale first, then mask, so masked scores are -inf whatever the scale's sign.
                const int cmax = lim - kbase;
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sr[c] = f2u((c > cmax) ? -INFINITY : u2f(sr[c]) * scale_log2);
                }
                tile_max = row_extreme<true, 64>(sr);
                mul = 1.0f;
            } else {
                tile_max = (scale_log2 >= 0.0f ? row_extreme<true, 64>(sr)
                                               : row_extreme<false, 64>(sr)) *
                           scale_log2;
                mul = scale_log2;
            }
            // Row max over both column halves (one buffer per tile parity).
            rs.red_max[b][half][row] = tile_max;
            pair_sync(pair_id);
            tile_max = fmaxf(tile_max, rs.red_max[b][half ^ 1][row]);
            PAIR_TRACE(tr, tbase + j * 4 + 2);
            PAIR_TRACE(trw, wb + 2);

            const float new_max = (tile_max > row_max + kRescaleThreshold) ? tile_max : row_max;
            const float max_used = (new_max == -INFINITY) ? 0.0f : new_max;
            const bool grew = (new_max != row_max);
            const float alpha = grew ? ex2_approx(row_max - max_used) : 1.0f;  // 0 on tile 0
            row_max = new_max;
            const bool need_rescale = j > 0 && (__any_sync(0xffffffffu, grew) != 0);

            if (need_rescale) {
                // O must hold P.V up to tile j-1 before it is rescaled.
                ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sb.o_done[(j - 1) & 1]),
                                                       ((j - 1) >> 1) & 1, wctx, kStatusTimeoutSoftmax));
                if (!ok) {
                    continue;
                }
                tc_fence_after();
                const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
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
            if (j >= 2) {
                // P buffer b was last read by P.V(j-2).
                ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sb.o_done[b]), ((j - 2) >> 1) & 1,
                                                       wctx, kStatusTimeoutSoftmax));
                if (!ok) {
                    continue;
                }
                tc_fence_after();
            }

            // Probabilities 2^(s * mul - max_used), packed fp16 pairs, into P buffer b. The row
            // sum adds the fp16-rounded values the MMA consumes.
            const float2 mul2 = make_float2(mul, mul);
            const float2 neg2 = make_float2(-max_used, -max_used);
            float2 sum2[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                sum2[i] = make_float2(0.0f, 0.0f);
            }
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float2 x2 =
                    __ffma2_rn(make_float2(u2f(sr[2 * i]), u2f(sr[2 * i + 1])), mul2, neg2);
                const uint32_t h = pack_half2(ex2_approx(x2.x), ex2_approx(x2.y));
                sum2[i % 4] = __fadd2_rn(sum2[i % 4], unpack_half2(h));
                pk[i] = h;
            }
            tmem_st32(t_base + kTmemP + b * 64 + half * 32, pk);
            const float2 s01 = __fadd2_rn(sum2[0], sum2[1]);
            const float2 s23 = __fadd2_rn(sum2[2], sum2[3]);
            const float2 s4 = __fadd2_rn(s01, s23);
            row_sum = fmaf(row_sum, alpha, s4.x + s4.y);

            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_cluster(p_full_cl[b]);
                PAIR_TRACE(trw, wb + 3);
            }
            PAIR_TRACE(tr, tbase + j * 4 + 3);
        }

        // ----------------------------------- epilogue -----------------------------------
        if (ok && nt > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sb.o_done[(nt - 1) & 1]),
                                                   ((nt - 1) >> 1) & 1, wctx, kStatusTimeoutSoftmax));
            tc_fence_after();
        }
        // Row sum over both column halves (both warps of the pair reach this barrier).
        rs.red_sum[half][row] = row_sum;
        pair_sync(pair_id);
        row_sum += rs.red_sum[half ^ 1][row];
        if (ok && nt > 0 && q0 < n) {
            const float inv_sum = (row_sum > 0.0f) ? (1.0f / row_sum) : 0.0f;
            // Stage O (fp16) in this CTA's Q buffer (every MMA that read it has completed),
            // in the swizzled layout of the TMA box; column half = box.
            uint8_t* out = smem + kSmemQ;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t o[32];
                tmem_ld32(t_o + c * 32, o);
                tmem_wait_ld();
                uint32_t h[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    h[e] = pack_half2(u2f(o[2 * e]) * inv_sum, u2f(o[2 * e + 1]) * inv_sum);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int cc = c * 4 + i;  // 16-byte chunk within the 128-byte box row
                    uint4* dst = reinterpret_cast<uint4*>(out + half * kQBox + row * 128 +
                                                          ((cc ^ (row & 7)) << 4));
                    *dst = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(&sb.epi));
            }
            if (warp == 0 && lane == 0) {
                if (mbar_wait(smem_u32(&sb.epi), 0, wctx, kStatusTimeoutEpilogue)) {
                    tma_store_3d(&tm_o, smem_u32(out), 0, q0, bh);
                    tma_store_3d(&tm_o, smem_u32(out) + kQBox, 64, q0, bh);
                    tma_store_commit();
                    tma_store_wait_read();
                }
            }
            __syncwarp();
        }
    } else if (warp == kProducerWarp) {
        // ================================== TMA producer ===================================
        if (lane == 0) {
            int last_parity[STAGES];
            bool loaded[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) {
                loaded[s] = false;
                last_parity[s] = 0;
            }
            bool ok = true;
            if (nt > 0) {
                const uint32_t bar = smem_u32(&sb.q_full);
                if (leader) {
                    mbar_arrive_expect_tx(bar, 2 * kQBytes);
                }
                tma_load_3d_pair(smem_base + kSmemQ, &tm_q, bar, 0, q0, bh);
                tma_load_3d_pair(smem_base + kSmemQ + kQBox, &tm_q, bar, 64, q0, bh);
            }
            // Ring order = the MMA's consumption order: K0, K1, then V(j) and K(j+2) for
            // j = 0, 1, ... (K(j+2) only while j + 2 < nt).
            int item = 0;
            auto load = [&](bool is_k, int tile) -> bool {
                const int stage = item % STAGES;
                const int phase = (item / STAGES) & 1;
                ++item;
                if (!mbar_wait(smem_u32(&sb.kv_empty[stage]), phase ^ 1, wctx, kStatusTimeoutProducer)) {
                    return false;
                }
                const uint32_t bar = smem_u32(&sb.kv_full[stage]);
                if (leader) {
                    mbar_arrive_expect_tx(bar, 2 * kSlotBytes);
                }
                const uint32_t dst = smem_base + kSmemKV + stage * kSlotBytes;
                if (is_k) {
                    const int key0 = tile * kKeys + static_cast<int>(rank) * 64;
                    tma_load_3d_pair(dst, &tm_k, bar, 0, key0, bh);
                    tma_load_3d_pair(dst + kKBox, &tm_k, bar, 64, key0, bh);
                } else {
                    tma_load_3d_pair(dst, &tm_v, bar, static_cast<int>(rank) * 64, tile * kKeys, bh);
                }
                loaded[stage] = true;
                last_parity[stage] = phase;
                return true;
            };
            for (int t = 0; ok && t < min(nt, 2); ++t) {
                ok = load(true, t);
            }
            for (int j = 0; ok && j < nt; ++j) {
                ok = load(false, j);
                if (ok && j + 2 < nt) {
                    ok = load(true, j + 2);
                }
            }
            if (!ok) {
                // Let every copy this CTA issued land before the pair releases its memory: the
                // bytes count on the leader's barrier, so the wait is the leader's.
                if (leader) {
                    for (int s = 0; s < STAGES; ++s) {
                        if (loaded[s]) {
                            mbar_wait_drain(smem_u32(&sb.kv_full[s]), last_parity[s], wctx,
                                            kStatusTimeoutTeardown);
                        }
                    }
                    if (nt > 0) {
                        mbar_wait_drain(smem_u32(&sb.q_full), 0, wctx, kStatusTimeoutTeardown);
                    }
                } else {
                    // This CTA cannot see its copies land (their bytes count on the leader's
                    // barrier); each is one 16 KB tile, so a grace of 2^16 cycles (~33 us)
                    // covers them before the final cluster barrier lets the CTA go.
                    const long long t0 = clock64();
                    while (clock64() - t0 < (1ll << 16)) {
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp && leader) {
        // ============================ MMA issuer (pair leader) =============================
        if (lane == 0) {
            bool ok = nt > 0;
            const uint32_t peer = 1;
            auto both = [&](uint64_t* bar) {
                umma_commit_pair(smem_u32(bar));
                umma_commit_pair(mapa_shared(smem_u32(bar), peer));
            };
            if (ok) {
                ok = mbar_wait(smem_u32(&sb.q_full), 0, wctx, kStatusTimeoutMma);
            }
            const uint64_t qd = make_desc_kmajor_sw128(smem_base + kSmemQ);
            const uint64_t kv0 = make_desc_kmajor_sw128(smem_base + kSmemKV);
            const uint64_t vv0 = make_desc_mnmajor_sw128(smem_base + kSmemKV, kQBox);
            auto slot_off = [](int stage) -> uint64_t {
                return static_cast<uint64_t>(stage * (kSlotBytes >> 4));
            };
            constexpr uint32_t idesc_s = make_idesc_f16(256, kKeys, /*d_f32=*/true, /*b_mn_major=*/false);
            constexpr uint32_t idesc_o = make_idesc_f16(256, D, /*d_f32=*/true, /*b_mn_major=*/true);
            auto s_step = [&](int b, int stage, int kk) {
                const uint64_t offq = static_cast<uint64_t>(((kk / 4) * kQBox + (kk % 4) * 32) >> 4);
                const uint64_t offk = static_cast<uint64_t>(((kk / 4) * kKBox + (kk % 4) * 32) >> 4);
                umma_ss_pair(tmem + kTmemS + b * 128, qd + offq, kv0 + slot_off(stage) + offk, idesc_s,
                             kk > 0 ? 1u : 0u);
            };
            auto pv_step = [&](int b, int stage, int kk, bool first) {
                umma_ts_pair(tmem + kTmemO, tmem + kTmemP + b * 64 + kk * 8,
                             vv0 + slot_off(stage) + static_cast<uint64_t>(kk * (2048 >> 4)), idesc_o,
                             (first && kk == 0) ? 0u : 1u);
            };
            int ring = 0;
            // S(0) and S(1)
            for (int j = 0; ok && j < min(nt, 2); ++j) {
                const int stage = ring % STAGES;
                ok = mbar_wait(smem_u32(&sb.kv_full[stage]), (ring / STAGES) & 1, wctx, kStatusTimeoutMma);
                if (!ok) {
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    s_step(j, stage, kk);
                }
                both(&sb.s_full[j]);
                both(&sb.kv_empty[stage]);
                ++ring;
            }
            for (int j = 0; ok && j < nt; ++j) {
                const int b = j & 1;
                const int v_item = ring++;
                const bool next2 = (j + 2 < nt);
                const int k_item = next2 ? ring++ : 0;
                const int vs = v_item % STAGES;
                const int ks = k_item % STAGES;
                [[maybe_unused]] const bool tr = traced_pair && j < 128;
                ok = mbar_wait_cl(smem_u32(&sb.p_full[b]), (j >> 1) & 1, wctx, kStatusTimeoutMma);
                PAIR_TRACE(tr, 1024 + j * 4 + 0);
                ok = ok && mbar_wait(smem_u32(&sb.kv_full[vs]), (v_item / STAGES) & 1, wctx,
                                     kStatusTimeoutMma);
                if (ok && next2) {
                    ok = mbar_wait(smem_u32(&sb.kv_full[ks]), (k_item / STAGES) & 1, wctx,
                                   kStatusTimeoutMma);
                }
                PAIR_TRACE(tr, 1024 + j * 4 + 1);
                if (!ok) {
                    break;
                }
                tc_fence_after();
                if (next2) {
                    // P.V(j) and S(j+2) interleaved (they touch disjoint TMEM: O and P_b / S_b).
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
#if FA_PAIR_RUN == 1
                        pv_step(b, vs, kk, j == 0);
                        s_step(b, ks, kk);
#else
                        if (kk % 4 == 0) {
#pragma unroll
                            for (int q = kk; q < kk + 4; ++q) {
                                pv_step(b, vs, q, j == 0);
                            }
#pragma unroll
                            for (int q = kk; q < kk + 4; ++q) {
                                s_step(b, ks, q);
                            }
                        }
#endif
                    }
                } else {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        pv_step(b, vs, kk, j == 0);
                    }
                }
                both(&sb.o_done[b]);
                both(&sb.kv_empty[vs]);
                if (next2) {
                    both(&sb.s_full[b]);
                    both(&sb.kv_empty[ks]);
                }
                PAIR_TRACE(tr, 1024 + j * 4 + 2);
            }
            // Every MMA issued above must be complete before tensor memory is released.
            both(&sb.mma_idle);
            mbar_wait_drain(smem_u32(&sb.mma_idle), 0, wctx, kStatusTimeoutTeardown);
        }
        __syncwarp();
    }

    if (!leader && warp == kMmaWarp && lane == 0) {
        // The leader's last commit also arrives here: no MMA may still touch this CTA's
        // memory when it is released.
        mbar_wait_drain(smem_u32(&sb.mma_idle), 0, wctx, kStatusTimeoutTeardown);
    }
    tc_fence_before();
    cluster_sync();  // no CTA leaves while the other may still arrive on its barriers
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

template <bool CAUSAL, int VARIANT>
cudaError_t launch(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                   const CUtensorMap& tm_o, const FwdArgs& args, cudaStream_t stream) {
    auto* kernel = fa_fwd_pair_kernel<CAUSAL, VARIANT>;
    cudaError_t err = ensure_smem_limit<fa_fwd_pair_kernel<CAUSAL, VARIANT>>(kSmemAlloc);
    if (err != cudaSuccess) {
        return err;
    }
    FwdArgs launch_args = args;
    const double kv_bytes = 4.0 * static_cast<double>(args.seqlen) * D;
    launch_args.head_group =
        static_cast<int>(std::min<double>(args.num_bh, std::max(1.0, (48.0 * 1048576.0) / kv_bytes)));
    const int pairs = (args.seqlen + 2 * kRows - 1) / (2 * kRows);
    const dim3 grid(static_cast<unsigned>(2 * pairs), static_cast<unsigned>(args.num_bh));
    kernel<<<grid, kThreads, kSmemAlloc, stream>>>(tm_q, tm_k, tm_v, tm_o, launch_args);
    return cudaGetLastError();
}

}  // namespace pair

#ifdef FA_TRACE
extern "C" __attribute__((visibility("default"))) int fa_pair_trace_read(unsigned long long* out, int n) {
    n = n < 4096 ? n : 4096;
    return cudaMemcpyFromSymbol(out, pair::g_pair_trace, sizeof(unsigned long long) * n) == cudaSuccess ? n : -1;
}
extern "C" __attribute__((visibility("default"))) int fa_pair_trace_clear(void) {
    static unsigned long long zero[4096] = {};
    return cudaMemcpyToSymbol(pair::g_pair_trace, zero, sizeof(zero)) == cudaSuccess ? 0 : -1;
}
#endif

bool pair_kernel_supports(const FwdProblem& prob, const FwdArgs& args) {
    return prob.head_dim == 128 && prob.variant != kVariantFp16Acc && args.num_splits <= 1;
}

cudaError_t launch_forward_pair(const FwdProblem& prob, const FwdArgs& args, cudaStream_t stream) {
    CUtensorMap tm_q, tm_k, tm_v, tm_o;
    if (encode_bhnd_map(&tm_q, prob.q, prob.num_bh, prob.seqlen, 128, pair::kRows) != CUDA_SUCCESS ||
        encode_bhnd_map(&tm_k, prob.k, prob.num_bh, prob.seqlen, 128, 64) != CUDA_SUCCESS ||
        encode_bhnd_map(&tm_v, prob.v, prob.num_bh, prob.seqlen, 128, pair::kKeys) != CUDA_SUCCESS ||
        encode_bhnd_map(&tm_o, prob.o, prob.num_bh, prob.seqlen, 128, pair::kRows) != CUDA_SUCCESS) {
        return cudaErrorInvalidValue;
    }
    if (prob.variant == kVariantOpt) {
        return prob.causal ? pair::launch<true, kVariantOpt>(tm_q, tm_k, tm_v, tm_o, args, stream)
                           : pair::launch<false, kVariantOpt>(tm_q, tm_k, tm_v, tm_o, args, stream);
    }
    return prob.causal ? pair::launch<true, kVariantBaseline>(tm_q, tm_k, tm_v, tm_o, args, stream)
                       : pair::launch<false, kVariantBaseline>(tm_q, tm_k, tm_v, tm_o, args, stream);
}

}  // namespace fa_sm100
