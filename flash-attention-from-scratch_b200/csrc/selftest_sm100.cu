// Building-block checks for the sm_100a primitives the forward kernel relies on, in the
// spirit of the reference's exact-equality layout tests (tests/cpp/test_ptx.cu:93-336), but
// for the Blackwell data path: TMA 3-D loads into 128-byte-swizzled smem, the K-major and
// MN-major shared-memory descriptors, tcgen05.mma SS (S = Q K^T) and TS (O = P V with P in
// tensor memory), the fp16-accumulator cell layout in TMEM, tcgen05.ld/st, and the swizzled
// TMA store used by the epilogue.
//
// One CTA of 128 threads (4 warps, warp w owns TMEM lanes 32w..32w+31):
//   TMEM columns: S [0,128)  O32 [128,128+D)  O16 [256,256+D)  P [384,448)
// Inputs are small integers (exact in fp16 and fp32), so every output is exact.
// Built into libfa_selftest.so, which only the tests load.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>

#include "fa_internal.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace fa_sm100 {
namespace {

constexpr int kTile = 128 * 128 * 2;  // bytes of a 128 x 128 fp16 tile (max D)
constexpr int kBox = 128 * 128;

struct ProbeShared {
    uint64_t tma_bar;
    uint64_t mma_bar;
    uint32_t tmem_base;
    int abort;
};

__device__ DeviceStatus g_probe_status;

template <int D>
__global__ void __launch_bounds__(128, 1)
    umma_probe_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_out, const __half* __restrict__ p,
                      float* __restrict__ s_out, float* __restrict__ o_out,
                      uint32_t* __restrict__ o16_raw, int* __restrict__ flags) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ ProbeShared sh;
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t base = smem_u32(smem);
    const uint32_t sq = base;
    const uint32_t sk = base + kTile;
    const uint32_t sv = base + 2 * kTile;
    const int warp = threadIdx.x / 32;
    const int row = threadIdx.x;
    const WaitCtx w{&sh.abort, &g_probe_status.code, &g_probe_status.epoch_aborted, 1u};

    if (threadIdx.x == 0) {
        sh.abort = 0;
        mbar_init(smem_u32(&sh.tma_bar), 1);
        mbar_init(smem_u32(&sh.mma_bar), 1);
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&sh.tmem_base), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;

    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(smem_u32(&sh.tma_bar), 3 * 128 * D * 2);
        for (int b = 0; b < D / 64; ++b) {
            tma_load_3d(sq + b * kBox, &tm_q, smem_u32(&sh.tma_bar), b * 64, 0, 0);
            tma_load_3d(sk + b * kBox, &tm_k, smem_u32(&sh.tma_bar), b * 64, 0, 0);
            tma_load_3d(sv + b * kBox, &tm_v, smem_u32(&sh.tma_bar), b * 64, 0, 0);
        }
    }
    // P row -> TMEM columns [384, 448), fp16 packed two per column.
    {
        uint32_t pk[32];
        const uint32_t* prow = reinterpret_cast<const uint32_t*>(p + row * 128);
        for (int half = 0; half < 2; ++half) {
            for (int i = 0; i < 32; ++i) {
                pk[i] = prow[half * 32 + i];
            }
            tmem_st32(tmem + lane_off + 384 + half * 32, pk);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (threadIdx.x == 0) {
        bool ok = mbar_wait(smem_u32(&sh.tma_bar), 0, w, 1u);
        if (ok) {
            tc_fence_after();
            // S = Q K^T
            constexpr uint32_t idesc_s = make_idesc_f16(128, 128, true, false);
            for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t off = (kk / 4) * kBox + (kk % 4) * 32;
                umma_ss(tmem + 0, make_desc_kmajor_sw128(sq + off), make_desc_kmajor_sw128(sk + off),
                        idesc_s, kk > 0);
            }
            // O32 = P V (fp32 accumulate), O16 = P V (fp16 accumulate)
            constexpr uint32_t idesc_o32 = make_idesc_f16(128, D, true, true);
            constexpr uint32_t idesc_o16 = make_idesc_f16(128, D, false, true);
            for (int kk = 0; kk < 8; ++kk) {
                const uint64_t bdesc = make_desc_mnmajor_sw128(sv + kk * 2048, kBox);
                umma_ts(tmem + 128, tmem + 384 + kk * 8, bdesc, idesc_o32, kk > 0);
                umma_ts(tmem + 256, tmem + 384 + kk * 8, bdesc, idesc_o16, kk > 0);
            }
            umma_commit(smem_u32(&sh.mma_bar));
        }
        flags[0] = ok ? 1 : 0;
    }
    __syncwarp();
    const bool done = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.mma_bar), 0, w, 2u));
    if (done) {
        tc_fence_after();
        uint32_t r[32];
        for (int c = 0; c < 4; ++c) {
            tmem_ld32(tmem + lane_off + c * 32, r);
            tmem_wait_ld();
            for (int e = 0; e < 32; ++e) {
                s_out[row * 128 + c * 32 + e] = __uint_as_float(r[e]);
            }
        }
        for (int c = 0; c < D / 32; ++c) {
            tmem_ld32(tmem + lane_off + 128 + c * 32, r);
            tmem_wait_ld();
            for (int e = 0; e < 32; ++e) {
                o_out[row * D + c * 32 + e] = __uint_as_float(r[e]);
            }
            // Stage O32 as fp16 in the Q buffer (swizzled like the TMA box) for the store test.
            for (int i = 0; i < 4; ++i) {
                const int col = c * 32 + i * 8;
                const int box = col / 64;
                const int cc = (col % 64) / 8;
                uint4 v;
                v.x = pack_half2(__uint_as_float(r[i * 8 + 0]), __uint_as_float(r[i * 8 + 1]));
                v.y = pack_half2(__uint_as_float(r[i * 8 + 2]), __uint_as_float(r[i * 8 + 3]));
                v.z = pack_half2(__uint_as_float(r[i * 8 + 4]), __uint_as_float(r[i * 8 + 5]));
                v.w = pack_half2(__uint_as_float(r[i * 8 + 6]), __uint_as_float(r[i * 8 + 7]));
                *reinterpret_cast<uint4*>(smem + box * kBox + row * 128 + ((cc ^ (row & 7)) << 4)) = v;
            }
            tmem_ld32(tmem + lane_off + 256 + c * 32, r);
            tmem_wait_ld();
            for (int e = 0; e < 32; ++e) {
                o16_raw[row * D + c * 32 + e] = r[e];
            }
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        if (done) {
            for (int b = 0; b < D / 64; ++b) {
                tma_store_3d(&tm_out, sq + b * kBox, b * 64, 0, 0);
            }
            tma_store_commit();
            tma_store_wait_read();
        }
        flags[1] = done ? 1 : 0;
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Software exp2 (exp2_poly2, two lanes at a time) and the SFU ex2.approx on the same inputs.
__global__ void exp2_probe_kernel(const float* __restrict__ x, float* __restrict__ poly,
                                  float* __restrict__ sfu, int n) {
    const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i + 1 < n) {
        const float2 e = exp2_poly2(make_float2(x[i], x[i + 1]));
        poly[i] = e.x;
        poly[i + 1] = e.y;
        sfu[i] = ex2_approx(x[i]);
        sfu[i + 1] = ex2_approx(x[i + 1]);
    }
}

__global__ void exp2_deg3_probe_kernel(const float* __restrict__ x, float* __restrict__ poly, int n) {
    const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i + 1 < n) {
        const float2 e = exp2_poly2_deg3(make_float2(x[i], x[i + 1]));
        poly[i] = e.x;
        poly[i + 1] = e.y;
    }
}

// Watchdog probe: waits with the kernels' bounded wait (mbar_wait) on an mbarrier that no
// thread ever arrives on. The wait must give up after 2^31 SM cycles, record its code in the
// status word and let the kernel return; flags[0] = 1 if the wait reported failure, flags[1]
// = 1 once the kernel reached its end.
__global__ void watchdog_probe_kernel(int* flags) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(smem_u32(&bar), 1);
        mbar_fence_init();
    }
    __syncthreads();
    const WaitCtx w{&abort_flag, &g_probe_status.code, &g_probe_status.epoch_aborted, 7u};
    const bool ok = mbar_wait(smem_u32(&bar), 0, w, kStatusTimeoutSoftmax);
    const bool all_failed = __all_sync(0xffffffffu, !ok);
    __syncthreads();
    if (threadIdx.x == 0) {
        flags[0] = all_failed ? 1 : 0;
        flags[1] = 1;
    }
}

thread_local std::string g_err;

}  // namespace
}  // namespace fa_sm100

extern "C" {

// Runs the probe on the current device: q, k, v are [128][d] fp16, p is [128][128] fp16
// (device pointers); outputs: s_out [128][128] f32, o_out [128][d] f32, o16_raw [128][d] raw
// 32-bit TMEM cells of the fp16 accumulator, o_half [128][d] fp16 written by TMA store,
// flags [2] int. Synchronises. Returns 0 on success, else a message in fa_selftest_error().
__attribute__((visibility("default"))) int fa_selftest_umma(const void* q, const void* k, const void* v, const void* p, float* s_out,
                     float* o_out, uint32_t* o16_raw, void* o_half, int* flags, int d) {
    using namespace fa_sm100;
    if (d != 64 && d != 128) {
        g_err = "d must be 64 or 128";
        return 1;
    }
    CUtensorMap maps[4];
    const void* ptrs[4] = {q, k, v, o_half};
    for (int i = 0; i < 4; ++i) {
        if (encode_bhnd_map(&maps[i], ptrs[i], 1, 128, d, 128) != CUDA_SUCCESS) {
            g_err = "tensor map encoding failed";
            return 2;
        }
    }
    const int smem = 3 * kTile + 1024;
    cudaError_t err;
    if (d == 64) {
        err = cudaFuncSetAttribute(umma_probe_kernel<64>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err == cudaSuccess) {
            umma_probe_kernel<64><<<1, 128, smem>>>(maps[0], maps[1], maps[2], maps[3],
                                                    static_cast<const __half*>(p), s_out, o_out,
                                                    o16_raw, flags);
        }
    } else {
        err = cudaFuncSetAttribute(umma_probe_kernel<128>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err == cudaSuccess) {
            umma_probe_kernel<128><<<1, 128, smem>>>(maps[0], maps[1], maps[2], maps[3],
                                                     static_cast<const __half*>(p), s_out, o_out,
                                                     o16_raw, flags);
        }
    }
    if (err == cudaSuccess) {
        err = cudaGetLastError();
    }
    if (err == cudaSuccess) {
        err = cudaDeviceSynchronize();
    }
    if (err != cudaSuccess) {
        g_err = std::string("CUDA error: ") + cudaGetErrorString(err);
        return 3;
    }
    return 0;
}

// Evaluates the kernel's two exp2 implementations on n (even) device floats. Synchronises.
__attribute__((visibility("default"))) int fa_selftest_exp2(const float* x, float* poly, float* sfu,
                                                            int n) {
    using namespace fa_sm100;
    if (n <= 0 || (n & 1) != 0) {
        g_err = "n must be positive and even";
        return 1;
    }
    const int pairs = n / 2;
    exp2_probe_kernel<<<(pairs + 255) / 256, 256>>>(x, poly, sfu, n);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) {
        err = cudaDeviceSynchronize();
    }
    if (err != cudaSuccess) {
        g_err = std::string("CUDA error: ") + cudaGetErrorString(err);
        return 3;
    }
    return 0;
}

// exp2_poly2_deg3 (the degree-3 software 2^x) on n (even) device floats; synchronises.
__attribute__((visibility("default"))) int fa_selftest_exp2_deg3(const float* x, float* poly, int n) {
    using namespace fa_sm100;
    if (n <= 0 || (n & 1) != 0) {
        g_err = "n must be positive and even";
        return 1;
    }
    exp2_deg3_probe_kernel<<<(n / 2 + 255) / 256, 256>>>(x, poly, n);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) {
        err = cudaDeviceSynchronize();
    }
    if (err != cudaSuccess) {
        g_err = std::string("CUDA error: ") + cudaGetErrorString(err);
        return 3;
    }
    return 0;
}

// Runs the watchdog probe on the current device (one CTA of 64 threads) and synchronises.
// Writes the probe's status word (then clears it) to *code_out. Returns 0 on success.
__attribute__((visibility("default"))) int fa_selftest_watchdog(int* flags, unsigned* code_out) {
    using namespace fa_sm100;
    watchdog_probe_kernel<<<1, 64>>>(flags);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) {
        err = cudaDeviceSynchronize();
    }
    DeviceStatus st{};
    if (err == cudaSuccess) {
        err = cudaMemcpyFromSymbol(&st, g_probe_status, sizeof(st));
    }
    if (err == cudaSuccess) {
        const DeviceStatus zero{};
        err = cudaMemcpyToSymbol(g_probe_status, &zero, sizeof(zero));
    }
    if (err != cudaSuccess) {
        g_err = std::string("CUDA error: ") + cudaGetErrorString(err);
        return 3;
    }
    *code_out = st.code;
    return 0;
}

__attribute__((visibility("default"))) const char* fa_selftest_error(void) { return fa_sm100::g_err.c_str(); }

}  // extern "C"
