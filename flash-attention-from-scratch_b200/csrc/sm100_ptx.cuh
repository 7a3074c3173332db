#pragma once
// Inline-PTX building blocks for sm_100a (B200): mbarriers with bounded waits, TMA tensor
// loads/stores, tcgen05 MMA with TMEM accumulators, TMEM load/store, and the shared-memory /
// instruction descriptors those MMAs take.
//
// This header replaces the sm_80 helper set of the reference (csrc/common.cuh:57-142:
// cp.async, ldmatrix, mma.sync, ex2.f16x2). Nothing here is a translation of it: the data
// movement is TMA + mbarrier, the contraction is tcgen05.mma, and the accumulators live in
// tensor memory instead of registers.
//
// Descriptor bit layouts follow the PTX ISA (tcgen05 "shared memory descriptor" and
// "instruction descriptor" tables); the canonical 128-byte-swizzle layouts are the ones TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace fa_sm100 {

// ------------------------------------------------------------------------------------------
// Error codes written to the device status word when a bounded wait gives up.
// ------------------------------------------------------------------------------------------
enum : unsigned {
    kStatusOk = 0,
    kStatusTimeoutProducer = 1u << 0,  // TMA producer waited too long for a free ring slot
    kStatusTimeoutMma = 1u << 1,       // MMA issuer waited too long for data / P
    kStatusTimeoutSoftmax = 1u << 2,   // softmax warps waited too long for S / O
    kStatusTimeoutEpilogue = 1u << 3,  // epilogue store waited too long for its rows
    kStatusTimeoutTeardown = 1u << 4,  // teardown waited too long for in-flight async work
};

// The teardown wait (mbar_wait_drain) gives up after this many nanoseconds of %globaltimer;
// mbar_wait bounds its waits by 2^31 SM cycles (about as long). Every legitimate wait in the
// kernel is a few microseconds; a second only trips on a real deadlock.
constexpr unsigned long long kWaitTimeoutNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Where a bounded wait reports that it gave up.
struct WaitCtx {
    volatile int* cta_abort;           // shared flag: some thread of this CTA gave up
    unsigned* code_word;               // global sticky error bits (host reads and clears)
    volatile unsigned* epoch_word;     // global: epoch of the last launch that gave up
    unsigned epoch;                    // this launch's epoch (never 0)
};

// Bounded wait for the phase with the given parity. Returns false when the wait ran out of
// time (after setting `code` in the global status, the CTA abort flag and the launch's abort
// epoch), or when another thread of this CTA or another CTA of this launch has given up.
// The result is per thread; callers that go on to warp-collective instructions vote on it.
// The hot path polls shared memory only: the SM cycle counter bounds the wait (2^31 cycles,
// about 1.1 s at the 1965 MHz boost clock and longer at lower clocks), and the global abort
// epoch written by other CTAs is read only once a wait has lasted 2^20 cycles (~0.5 ms),
// far beyond any wait of a healthy launch, so that a global load never delays a wake-up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                          unsigned code) {
    if (mbar_try_wait(bar, parity)) {
        return true;
    }
    const long long t0 = clock64();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) {
            return true;
        }
        // The abort flag and the clock are checked every 32 polls only: a polling warp shares
        // its SM sub-partition's issue slots with the warps doing the work.
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

// Bounded wait used on the way out after an abort: it ignores the abort flags (the point is to
// let in-flight asynchronous copies / MMAs land before shared or tensor memory is released)
// and only gives up on time.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                                unsigned code) {
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicOr(w.code_word, code);
            *w.epoch_word = w.epoch;
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), 3-D tiled, no multicast.
// Coordinates are {x = element along the contiguous head dim, y = row, z = head}; x is always
// a multiple of 64 (128 bytes), so every copy starts on a 16-byte boundary.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y,
                                             int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until the bulk stores of this thread have finished READING shared memory.
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Generic-proxy writes to shared memory become visible to the async proxy (TMA store).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// Tensor memory (TMEM). Addresses: bits 31..16 = lane, bits 15..0 = 32-bit column.
// A warp may only touch lanes [32 * (warp % 4), 32 * (warp % 4) + 32).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base + i),
// register c = column (col + c).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// 32 lanes x 64 consecutive 32-bit columns in one instruction (register c = column col + c).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
}

// 32 lanes x 128 consecutive 32-bit columns in one instruction (register c = column col + c).
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05.mma, kind::f16 (fp16 x fp16, fp32 or fp16 accumulate), one CTA.
// ------------------------------------------------------------------------------------------
// A and B both from shared memory (descriptors).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// A from tensor memory (16-bit elements packed two per column, K-major), B from shared memory.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// kind::f8f6f4 (8-bit operands, here e4m3 x e4m3, fp32 accumulate): the same forms with K = 32
// per instruction, i.e. the same 32 bytes of each operand row as a kind::f16 step of K = 16.
__device__ __forceinline__ void umma_ss_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// A from tensor memory (8-bit elements packed four per column, K-major), B from shared memory.
__device__ __forceinline__ void umma_ts_f8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The mbarrier gets one arrival once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// ------------------------------------------------------------------------------------------
// Descriptors
// ------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor (64 bit):
//   [0,14)  start address >> 4        [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) version = 1 (tcgen05)     [49,52) base offset = 0 (atoms are 1024-byte aligned)
//   [61,64) layout: 2 = 128-byte swizzle
constexpr uint64_t kDescSwizzle128 = 2;

__host__ __device__ constexpr uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                                      uint32_t sbo_bytes) {
    return (static_cast<uint64_t>((saddr >> 4) & 0x3FFFu)) |
           (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (kDescSwizzle128 << 61);
}

// Operand stored K-major with 128-byte swizzle: rows of 64 fp16 (128 B), 8-row atoms of
// 1024 B stacked along M/N. LBO is unused for swizzled K-major layouts (encoded as 16 B);
// SBO = 1024 B between 8-row groups. Stepping K by 16 elements inside an atom adds 32 B to
// the start address.
__host__ __device__ constexpr uint64_t make_desc_kmajor_sw128(uint32_t saddr) {
    return make_smem_desc(saddr, 16, 1024);
}

// Operand stored MN-major with 128-byte swizzle (V as the B operand of P.V: N = head dim is
// contiguous). A row of the smem tile is one key (K index) holding 64 head-dim values;
// SBO = 1024 B between groups of 8 keys, LBO = byte distance between 64-wide head-dim blocks.
__host__ __device__ constexpr uint64_t make_desc_mnmajor_sw128(uint32_t saddr,
                                                               uint32_t mn_block_bytes) {
    return make_smem_desc(saddr, mn_block_bytes, 1024);
}

// Instruction descriptor for kind::f16 (32 bit):
//   [4,6) D format (0 = f16, 1 = f32)   [7,10) A format (0 = f16, 1 = bf16)
//   [10,13) B format (0 = f16, 1 = bf16)   [15] A major (0 = K)   [16] B major (0 = K, 1 = MN)
//   [17,23) N >> 3   [24,29) M >> 4
// A and B always get the same format (bf16 operands accumulate into an f32 D only).
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n, bool d_f32, bool b_mn_major,
                                                      bool ab_bf16 = false) {
    return (static_cast<uint32_t>(d_f32 ? 1 : 0) << 4) |
           (static_cast<uint32_t>(ab_bf16 ? 1 : 0) << 7) | (static_cast<uint32_t>(ab_bf16 ? 1 : 0) << 10) |
           (static_cast<uint32_t>(b_mn_major ? 1 : 0) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// ------------------------------------------------------------------------------------------
// Arithmetic helpers
// ------------------------------------------------------------------------------------------
// 2^x on the special-function unit (flush-to-zero; 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA pipe for two values (a software alternative to the special-function unit,
// whose 16 results / clock / SM equal the tensor cores' rate on a 128 x 128 x 128 tile).
// 2^x = 2^j * 2^f with j = round(x) taken from the low mantissa bits of x + 1.5 * 2^23 and
// f = x - j in [-1/2, 1/2]; 2^f by a degree-4 polynomial fitted for minimax relative error
// with Lawson's algorithm (csrc/fit_exp2_poly.py: max relative error 2.9e-6 in float32, far
// below the 4.9e-4 of the fp16 rounding that follows); 2^j is added into the exponent field.
// Inputs below -126 are clamped (their 2^x rounds to 0 in fp16 anyway); -inf gives 2^-126.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    x.x = fmaxf(x.x, -126.0f);
    x.y = fmaxf(x.y, -126.0f);
    const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
    const float2 r = __fadd2_rn(t, make_float2(-kRound, -kRound));
    const float2 f = __ffma2_rn(r, make_float2(-1.0f, -1.0f), x);
    float2 p = __ffma2_rn(make_float2(0.009582852944731712f, 0.009582852944731712f), f,
                          make_float2(0.055906426161527634f, 0.055906426161527634f));
    p = __ffma2_rn(p, f, make_float2(0.24024099111557007f, 0.24024099111557007f));
    p = __ffma2_rn(p, f, make_float2(0.6931241750717163f, 0.6931241750717163f));
    p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
    // t's bits are 0x4B400000 + j; shifted left by 23 only j survives (mod 2^9), which adds j to
    // the exponent of p in [2^-1/2, 2^1/2].
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// Cheaper variant of exp2_poly2: degree-3 polynomial (fit_exp2_poly.py 3: max relative error
// 1.0e-4 in float32, below the 2.4e-4 worst relative rounding of the fp16 value it feeds).
__device__ __forceinline__ float2 exp2_poly2_deg3(float2 x) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    x.x = fmaxf(x.x, -126.0f);
    x.y = fmaxf(x.y, -126.0f);
    const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
    const float2 r = __fadd2_rn(t, make_float2(-kRound, -kRound));
    const float2 f = __ffma2_rn(r, make_float2(-1.0f, -1.0f), x);
    float2 p = __ffma2_rn(make_float2(0.05500892922282219f, 0.05500892922282219f), f,
                          make_float2(0.24221095442771912f, 0.24221095442771912f));
    p = __ffma2_rn(p, f, make_float2(0.6932829022407532f, 0.6932829022407532f));
    p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// Row-max helper: three-input max.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float fmin3(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// lo_acc += low half of h, hi_acc += high half of h (fp16 -> fp32 exactly, then an fp32 add).
__device__ __forceinline__ void add_f16x2_to_f32(float& lo_acc, float& hi_acc, uint32_t h) {
    asm("{\n\t.reg .b16 l, u;\n\tmov.b32 {l, u}, %2;\n\t"
        "add.rn.f32.f16 %0, l, %0;\n\tadd.rn.f32.f16 %1, u, %1;\n\t}"
        : "+f"(lo_acc), "+f"(hi_acc)
        : "r"(h));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// bfloat16 counterparts: lo_acc += low half of b, hi_acc += high half (bf16 -> fp32 exactly,
// then an fp32 add), and two floats rounded to nearest-even bfloat16, lo in the low half.
__device__ __forceinline__ void add_bf16x2_to_f32(float& lo_acc, float& hi_acc, uint32_t b) {
    asm("{\n\t.reg .b16 l, u;\n\tmov.b32 {l, u}, %2;\n\t"
        "add.rn.f32.bf16 %0, l, %0;\n\tadd.rn.f32.bf16 %1, u, %1;\n\t}"
        : "+f"(lo_acc), "+f"(hi_acc)
        : "r"(b));
}

__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Two floats rounded to nearest-even e4m3 (saturating to +-448), lo in the low byte of the
// returned 16 bits; and two e4m3 values (low byte first) widened exactly to an f16x2 pair.
__device__ __forceinline__ uint32_t pack_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint32_t e4m3x2_to_half2(uint32_t b) {
    uint32_t r;
    asm("{\n\t.reg .b16 l;\n\tcvt.u16.u32 l, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\t}" : "=r"(r) : "r"(b));
    return r;
}

// The element type's pair helpers, chosen at compile time (BF16: bfloat16, else float16).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (BF16) {
        return pack_bf162(lo, hi);
    } else {
        return pack_half2(lo, hi);
    }
}

template <bool BF16>
__device__ __forceinline__ void add_x2_to_f32(float& lo_acc, float& hi_acc, uint32_t h) {
    if constexpr (BF16) {
        add_bf16x2_to_f32(lo_acc, hi_acc, h);
    } else {
        add_f16x2_to_f32(lo_acc, hi_acc, h);
    }
}

__device__ __forceinline__ float2 unpack_half2(uint32_t r) {
    return __half22float2(*reinterpret_cast<const __half2*>(&r));
}

}  // namespace fa_sm100
